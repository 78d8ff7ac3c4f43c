"""Generate the golden fixtures from the reference's own functions.

    python tests/golden/make_golden.py /path/to/cache-eviction

Imports tonghuikang/cache-eviction's code/cache_eviction/sglang_evict_runtime.py
and core.py from a read-only checkout (the path argument) and runs them on
CPU tensors; torch.cuda.synchronize is replaced by a no-op in this process only.
Inputs come from tests/golden/scenarios.py (numpy, fixed seeds), so only the
reference's outputs are stored.  The checkout is needed only to regenerate;
tests read the .npz files.
"""
from __future__ import annotations

import hashlib
import importlib.util
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from golden import scenarios as sc  # noqa: E402


def load_reference(root: Path):
    torch.cuda.synchronize = lambda *a, **k: None  # CPU run: the reference syncs at boundaries
    spec = importlib.util.spec_from_file_location(
        "ref_gstar_evict", root / "code/cache_eviction/sglang_evict_runtime.py")
    rt = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rt)
    sys.path.insert(0, str(root / "code"))
    from cache_eviction import core
    return rt, core


def bf16_tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.int16).numpy().tobytes()
                          if t.dtype == torch.bfloat16 else t.contiguous().numpy().tobytes()).hexdigest()


def gen_choose(rt):
    out = {}
    for i, c in enumerate(sc.choose_cases()):
        pos = torch.from_numpy(c["pos"])
        L, G, N = pos.shape
        if c["name"] == "random_reservoir_2048":
            score = rt.reservoir_scores(c["seed"], pos, torch.arange(L), torch.arange(G))
        elif c["name"] == "h2o_global_2048":
            score = torch.from_numpy(c["global_key"])
        elif c["score"] is None:
            score = torch.zeros(pos.shape, dtype=torch.float64)
        else:
            score = torch.from_numpy(c["score"])
        name = "head_sum_2048" if c["name"] == "h2o_global_2048" else c["name"]
        try:
            keep, count = rt.choose(name, pos, c["n"], c["budget"], c["prefix"], c["recent"], score,
                                    c["cursor"])
            if keep is None:
                status, kept = 2, np.zeros((L, G, 0), np.int32)
            else:
                status, kept = 0, np.sort(keep.numpy(), -1).astype(np.int32)
        except RuntimeError:
            status, kept, count = 3, np.zeros((L, G, 0), np.int32), -1
        out[f"case{i}_status"] = np.int32(status)
        out[f"case{i}_count"] = np.int32(count)
        out[f"case{i}_kept"] = kept
    np.savez_compressed(HERE / "choose.npz", **out)
    return out


def gen_reservoir(rt, core):
    pos = torch.arange(1000).expand(2, 8, -1)
    vals = {}
    for seed in (7, 3, (1 << 63) + 5, -3):
        s = rt.reservoir_scores(seed, pos, torch.arange(2), torch.arange(8))
        vals[f"seed_{seed & ((1 << 64) - 1)}"] = (s[:, :, :128] * float(1 << 53)).numpy().astype(np.uint64)
    vals["kat_7_1_5_321"] = np.float64(core.reservoir_score(7, 1, 5, 321))
    vals["kat_runtime_7_1_5_321"] = np.float64(
        rt.reservoir_scores(7, pos, torch.arange(2), torch.arange(8))[1, 5, 321])
    np.savez_compressed(HERE / "reservoir.npz", **vals)


def make_backend(setup):
    keys = {l: bf16_tensor(setup["keys"][l]).clone() for l in range(4)}
    values = {l: bf16_tensor(setup["values"][l]).clone() for l in range(4)}
    pool = SimpleNamespace(layers_mapping={l: (l, l not in sc.FULL) for l in range(4)},
                           get_key_buffer=keys.__getitem__, get_value_buffer=values.__getitem__)
    return SimpleNamespace(token_to_kv_pool=pool, max_kv_splits=8,
                           req_to_token_pool=SimpleNamespace(req_to_token=torch.zeros(
                               (setup["rows"], setup["width"]), dtype=torch.int32)),
                           kv_indptr=torch.zeros(setup["rows"] + 1, dtype=torch.int32)), keys, values


def gen_boundaries(rt, core):
    out = {}
    setup = sc.boundary_setup()
    n = setup["n"]
    orig_scores = rt._scores

    def scores_with_global(st, entry, name, pos, slots, nn):
        if name == "h2o_global_2048":
            s = st.scores[:, :, slots]
            acc = torch.zeros(s.shape[0], s.shape[2], dtype=torch.float32)
            for g in range(s.shape[1]):
                acc = acc + s[:, g]
            return acc[:, None, :].expand(-1, s.shape[1], -1).double()
        return orig_scores(st, entry, name, pos, slots, nn)

    rt._scores = scores_with_global
    for name, kind in sc.BOUNDARY_NAMES:
        rt.STATE = None
        b, keys, values = make_backend(setup)
        st = rt.state(b)
        slot_of = torch.from_numpy(setup["slot_of"])
        st.req_to_token[1, :n] = slot_of.int()
        st.scores[:, :, slot_of] = torch.from_numpy(setup["score"])
        cfg = sc.boundary_cfg(name)
        if name == "h2o_global_2048":
            entry = {"kind": kind, "key": "r", "cfg": dict(cfg, record=False), "mode": 1, "events": [],
                     "error": None, "frontier": 0, "count": 0, "last_boundary": 0,
                     "peak_full_entries": 0, "layer_error": []}
        else:
            entry = rt._live_entry(SimpleNamespace(rid="r", session=None), dict(cfg, record=False), kind)
        freed = []
        alloc = SimpleNamespace(free_full=lambda s: freed.append(s.clone()),
                                full_to_swa_index_mapping=torch.zeros(setup["slots"], dtype=torch.int64))
        policies = {(l, g): core.Policy(name if name != "h2o_global_2048" else "head_sum_2048",
                                        cfg["budget"], cfg["prefix"], cfg["recent"], seed=4, stream=(l, g))
                    for l in range(2) for g in range(8)}
        key = f"{name}_{kind}"
        for k, boundary in enumerate((2048, 4096)):
            cursor = boundary - 200
            if kind == "replay":
                rt._boundary(st, 1, entry, boundary)
            else:
                rt._boundary(st, 1, entry, boundary, cursor, alloc)
            cnt = entry["count"]
            out[f"{key}_b{k}_table"] = st.table[1, :cnt].numpy().copy()
            out[f"{key}_b{k}_pos"] = entry["pos"].numpy().astype(np.int32).copy()
            out[f"{key}_b{k}_frontier"] = np.int32(int(st.frontier[1]))
            out[f"{key}_b{k}_r2u"] = st.req_to_token[1, :n].numpy().copy()
            out[f"{key}_b{k}_freed"] = (torch.cat(freed).numpy().astype(np.int32) if freed
                                        else np.zeros(0, np.int32))
            # the reference test's own check: kept sets equal core.Policy's
            if name not in ("random_2048", "h2o_global_2048"):
                for p in policies.values():
                    for t in range(p.next_position, boundary):
                        p.append(t)
                for (l, g), p in policies.items():
                    p.scores = {t: float(setup["score"][l, g, t]) for t in p.resident}
                    p.finish()
                for (l, g), p in policies.items():
                    assert set(entry["pos"][l, g].tolist()) == p.resident, (name, boundary, l, g)
        out[f"{key}_keys_sha"] = np.array([sha(keys[l]) for l in sc.FULL])
        out[f"{key}_values_sha"] = np.array([sha(values[l]) for l in sc.FULL])
        out[f"{key}_scores_sha"] = np.array([sha(st.scores)])
    rt._scores = orig_scores
    np.savez_compressed(HERE / "boundary.npz", **out)


RECORD_NAMES = ("head_sum_2048", "random_reservoir_2048", "random_2048", "prefix_sliding_2048")


def gen_records(rt, core):
    """Retention records (runtime:465-467, 500-507) of the check_boundaries
    scenario with record=True, captured from the reference's write_payload."""
    import base64
    out = {}
    setup = sc.boundary_setup()
    n = setup["n"]
    captured = []
    orig_write = rt.write_payload
    rt.write_payload = lambda key, obj: captured.append((key, obj))
    for name in RECORD_NAMES:
        rt.STATE = None
        b, keys, values = make_backend(setup)
        st = rt.state(b)
        slot_of = torch.from_numpy(setup["slot_of"])
        st.req_to_token[1, :n] = slot_of.int()
        st.scores[:, :, slot_of] = torch.from_numpy(setup["score"])
        cfg = dict(sc.boundary_cfg(name), record=True)
        entry = rt._live_entry(SimpleNamespace(rid="r", session=None), cfg, "live")
        alloc = SimpleNamespace(free_full=lambda s_: None,
                                full_to_swa_index_mapping=torch.zeros(setup["slots"], dtype=torch.int64))
        captured.clear()
        for k, boundary in enumerate((2048, 4096)):
            rt._boundary(st, 1, entry, boundary, boundary - 200, alloc)
        assert [key for key, _ in captured] == ["r-b2048", "r-b4096"], captured
        for k, (_, obj) in enumerate(captured):
            assert obj["kind"] == "retention" and obj["kv_heads"] == 8 and obj["layers"] == list(sc.FULL)
            for field, dt in (("evicted_delta", np.uint32), ("evicted_counts", np.int32)):
                a = obj[field]
                assert a["dtype"] == np.dtype(dt).name
                out[f"{name}_b{k}_{field}"] = np.frombuffer(base64.b64decode(a["data"]), dt).copy()
    rt.write_payload = orig_write
    np.savez_compressed(HERE / "records.npz", **out)


def gen_diagnostic(rt):
    """Lost mass, score tables and resident masks of the reference's regret
    diagnostic (_diagnose / _diagnostic_boundary, runtime:549-613)."""
    d = sc.diagnostic_setup()
    keys, q = bf16_tensor(d["keys"]), bf16_tensor(d["q"])
    sinks = torch.from_numpy(d["sinks"])
    st = SimpleNamespace(first_full=1, full_layers=[1])
    layer = SimpleNamespace(layer_id=1, tp_q_head_num=sc.DIAG_H, tp_k_head_num=sc.DIAG_G, scaling=d["scale"])
    req = SimpleNamespace(rid="r", session=None, origin_input_ids=[0] * sc.DIAG_LEN)
    e = rt._diagnostic_entry(req, {"seed": d["seed"], "policies": d["policies"]}, "cpu", 1, sc.DIAG_G)
    for lo, hi in sc.DIAG_CHUNKS:
        rt._diagnose(st, e, 0, layer, q[lo:hi], keys, sinks, torch.arange(1, hi + 1), lo)
    np.savez_compressed(HERE / "diagnostic.npz", lost=e["lost"].numpy(), score_sum=e["score_sum"].numpy(),
                        score_max=e["score_max"].numpy(), resident=e["resident"].numpy())


def gen_replay(rt):
    """Per-token layer error of the reference's static replay
    (_replay_layer_difference, runtime:520-546) for three chunks: one before
    any eviction (count 0: everything visible) and two after the boundary."""
    d = sc.replay_setup()
    layer = SimpleNamespace(tp_q_head_num=sc.REPLAY_H, tp_k_head_num=sc.REPLAY_G, scaling=d["scale"])
    sinks = torch.from_numpy(d["sinks"])
    q = bf16_tensor(d["q"])
    out = {}
    for i, (lo, hi, evicted) in enumerate(sc.REPLAY_CHUNKS):
        entry = {"shadow_k": bf16_tensor(d["keys"]), "shadow_v": bf16_tensor(d["values"]), "layer_error": [],
                 "count": sc.REPLAY_KEEP if evicted else 0, "frontier": sc.REPLAY_FRONTIER if evicted else 0,
                 "pos": torch.from_numpy(d["pos"])[None]}
        rt._replay_layer_difference(None, entry, q[lo:hi], layer, sinks, lo)
        out[f"chunk{i}"] = torch.cat(entry["layer_error"]).numpy()
    np.savez_compressed(HERE / "replay.npz", **out)


def gen_decode(rt):
    d = sc.decode_setup()
    keys = bf16_tensor(d["keys"]).float()
    values = bf16_tensor(d["values"]).float()
    q = bf16_tensor(d["q"]).float()
    sinks = bf16_tensor(d["sinks"]).float()
    out = {}
    for i, length in enumerate(sc.DECODE_LENGTHS):
        slots = torch.from_numpy(d["perm"][d["indptr"][i]:d["indptr"][i + 1]]).long()
        k = keys[slots]
        p = rt._probabilities(q[i:i + 1], k, sinks, d["scale"], sc.G, torch.tensor([length - 1]),
                              torch.arange(length))  # [G, group, 1, len]
        out[f"seq{i}_sum"] = p.sum(1)[:, 0].numpy().astype(np.float32)
        out[f"seq{i}_max"] = p.amax(1)[:, 0].numpy().astype(np.float32)
        o = torch.einsum("gjk,kgd->gjd", p[:, :, 0].double(), values[slots].double())
        out[f"seq{i}_out"] = o.reshape(sc.H, sc.D).numpy().astype(np.float32)
    np.savez_compressed(HERE / "decode.npz", **out)


def gen_prefill(rt):
    """_prefill_scores (runtime:327-340) on each entry of the prefill scenario,
    from zero scores, for head_sum (mode 1) and head_max (mode 2)."""
    d = sc.prefill_setup()
    keys = bf16_tensor(d["keys"])
    q = bf16_tensor(d["q"])
    sinks = bf16_tensor(d["sinks"])
    layer = SimpleNamespace(tp_q_head_num=sc.H, tp_k_head_num=sc.G, scaling=d["scale"])
    out = {}
    for mode in (1, 2):
        for i, (prefix, nq) in enumerate(sc.PREFILL_ENTRIES):
            st = SimpleNamespace(scores=torch.zeros((1, sc.G, d["slots"]), dtype=torch.float32))
            lst = torch.from_numpy(d["lists"][i]).long()
            chunk = q[d["qo_indptr"][i]:d["qo_indptr"][i + 1]]
            rt._prefill_scores(st, 0, mode, layer, chunk, keys, sinks, lst[:prefix], lst[prefix:])
            out[f"mode{mode}_entry{i}"] = st.scores[0][:, lst].numpy()  # [G, prefix + nq]
    np.savez_compressed(HERE / "prefill.npz", **out)


def main():
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py /path/to/cache-eviction")
    root = Path(sys.argv[1])
    rt, core = load_reference(root)
    gen_choose(rt)
    gen_reservoir(rt, core)
    gen_boundaries(rt, core)
    gen_records(rt, core)
    gen_diagnostic(rt)
    gen_replay(rt)
    gen_decode(rt)
    gen_prefill(rt)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
