"""KV-head tensor parallelism on 2, 4 and 8 GPUs (NCCL): a head-sharded run
must reproduce the single-GPU run on every rank.

Each rank builds the same 8-head state, runs it whole (tp = 1) on its GPU,
then runs its own 8 / tp heads (head offset rank * 8 / tp) and compares:
decode outputs and scores of its heads (test tolerance), and boundary
results, tables, freed units, positions, scores and K/V pools bit for bit,
for H2O global (per-head scores all-gathered over NCCL), random (slice of the
shared draw) and reservoir (global head index) rows.  Each world size is
skipped when the box has fewer GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

G, H, D, P, L = 8, 64, 64, 16, 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _bf16(rng, shape):
    x = rng.standard_normal(shape, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((x + 0x7FFF + ((x >> 16) & 1)) >> 16).astype(np.uint16)


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    from cache_eviction_b200 import kernels, tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    errs = []
    try:
        gl = G // world
        h0, q0 = rank * gl, rank * gl * 8
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        t16 = lambda a: t(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
        rng = np.random.default_rng(123)
        # ---------------- decode: sharded heads vs the whole layer ----------------
        lengths = [33, 700, 1600, 4097]
        pages = [-(-n // P) for n in lengths]
        units = sum(pages) + 3
        kp, vp = _bf16(rng, (units, G, P, D)), _bf16(rng, (units, G, P, D))
        qq = _bf16(rng, (len(lengths), H, D))
        sinks = rng.standard_normal(H).astype(np.float32)
        idx = ((rng.permutation(units - 1) + 1)[:sum(pages)]).astype(np.int32)
        indptr = np.concatenate([[0], np.cumsum(pages)]).astype(np.int32)
        toks = np.array(lengths, np.int32)
        modes = np.array([1, 2, 1, 0], np.int32)
        sc0 = rng.random((G, units), dtype=np.float32)
        s_full = t(sc0)
        o_full = kernels.decode_attn_score(t16(qq), t16(kp), t16(vp), t(indptr), t(idx), t(toks), 0.125, P,
                                           sinks=t(sinks), mode_of_row=t(modes), scores=s_full, out_f32=True)
        s_loc = t(sc0[h0:h0 + gl])
        o_loc = kernels.decode_attn_score(t16(qq[:, q0:q0 + 8 * gl]), t16(kp[:, h0:h0 + gl]),
                                          t16(vp[:, h0:h0 + gl]), t(indptr), t(idx), t(toks), 0.125, P,
                                          sinks=t(sinks[q0:q0 + 8 * gl]), mode_of_row=t(modes),
                                          scores=s_loc, out_f32=True)
        torch.cuda.synchronize()
        ref = o_full[:, q0:q0 + 8 * gl]
        rel = float((o_loc - ref).norm() / ref.norm())
        if rel > 1e-3:
            errs.append(f"decode output rel {rel:.2e}")
        if not torch.allclose(s_loc, s_full[h0:h0 + gl], rtol=1e-3, atol=1e-6):
            errs.append("decode scores differ")
        # ---------------- boundary: three rows, one policy each ----------------
        rows, units, width, cap = 3, 1600, 512, 256
        kl = [_bf16(rng, (units, G, P, D)) for _ in range(L)]
        vl = [_bf16(rng, (units, G, P, D)) for _ in range(L)]
        r2u = np.zeros((rows, width), np.int32)
        perm = rng.permutation(units - 1) + 1
        for r in range(rows):
            r2u[r, :400] = perm[r * 400:(r + 1) * 400]
        scores = rng.lognormal(0, 2, (L, G, units)).astype(np.float32)
        names = ["h2o_global_2048", "random_2048", "random_reservoir_2048"]
        n = 384
        params = [dict(n=n, budget=96, prefix=24, recent=24, cursor=n - 11, policy=names[r], seed=50 + r)
                  for r in range(rows)]
        max_cols = n
        draw = rng.random((rows, L, G, max_cols))

        def run(heads, off, group):
            sl = slice(heads[0], heads[1])
            st = {"table": t(np.zeros((rows, width), np.int32)), "r2u": t(r2u),
                  "frontier": t(np.zeros(rows, np.int32)), "count": t(np.zeros(rows, np.int32)),
                  "pos": t(np.zeros((rows, L, heads[1] - heads[0], cap), np.int32)),
                  "scores": t(scores[:, sl])}
            k = [t16(a[:, sl]) for a in kl]
            v = [t16(a[:, sl]) for a in vl]
            rows_t = torch.arange(rows, dtype=torch.int32, device=dev)
            prm = kernels.row_params(params, dev)
            gsc = None
            if group is not None:
                local = kernels.gather_row_scores(st["table"], st["r2u"], st["frontier"], st["count"],
                                                  st["scores"], rows_t, prm, max_cols)
                gsc = tp.all_gather_heads(local, group)
            res, fr = kernels.boundary(st["table"], st["r2u"], st["frontier"], st["count"], st["pos"],
                                       st["scores"], kernels.layer_pointers(k, dev),
                                       kernels.layer_pointers(v, dev), heads[1] - heads[0], P, rows_t, prm,
                                       max_cols, n + 1, True, marks=torch.zeros(units, dtype=torch.int32, device=dev),
                                       epoch=1, uniforms=t(draw[:, :, sl]), global_scores=gsc, head_offset=off)
            torch.cuda.synchronize()
            return res.cpu(), fr.cpu(), {kk: vv.cpu() for kk, vv in st.items()}, [a.cpu() for a in k], [a.cpu() for a in v]

        res_f, fr_f, st_f, k_f, v_f = run((0, G), 0, None)
        res_l, fr_l, st_l, k_l, v_l = run((h0, h0 + gl), h0, dist.group.WORLD)
        if not torch.equal(res_f, res_l):
            errs.append(f"boundary results differ {res_f.tolist()} vs {res_l.tolist()}")
        for r in range(rows):
            nf = int(res_f[r, 3])
            if not torch.equal(fr_f[r, :nf], fr_l[r, :nf]):
                errs.append(f"freed units differ for row {r}")
        for key in ("table", "r2u", "frontier", "count"):
            if not torch.equal(st_f[key], st_l[key]):
                errs.append(f"{key} differs")
        if not torch.equal(st_f["pos"][:, :, h0:h0 + gl], st_l["pos"]):
            errs.append("pos slice differs")
        if not torch.equal(st_f["scores"][:, h0:h0 + gl], st_l["scores"]):
            errs.append("scores slice differs")
        for a, b in zip(k_f + v_f, k_l + v_l):
            if not torch.equal(a[:, h0:h0 + gl].view(torch.int16), b.view(torch.int16)):
                errs.append("pool slice differs")
                break
        # every rank freed the same units
        mine = torch.cat([fr_l[r, :int(res_l[r, 3])] for r in range(rows)]).to(dev)
        others = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(others, mine)
        if not all(torch.equal(o, mine) for o in others):
            errs.append("ranks freed different units")
    except Exception as e:  # report instead of hanging the peer
        errs.append(repr(e))
    finally:
        q.put((rank, errs))
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_sharding_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for rank in range(world):
        assert out[rank] == [], (rank, out[rank])
    assert all(p.exitcode == 0 for p in procs)
