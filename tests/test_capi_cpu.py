"""The C-ABI library loads without a GPU and exports every entry point that
the headers in include/ declare (no compute calls here)."""
import ctypes as C
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def header_text():
    """Every header under include/, comments removed."""
    text = "\n".join(h.read_text() for h in sorted((ROOT / "include").glob("*.h")))
    return re.sub(r"/\*.*?\*/", "", text, flags=re.S)


def declared_functions():
    return sorted(set(re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(ce_\w+)\s*\(", header_text(), flags=re.M)))


def test_library_exports_every_declared_symbol():
    from cache_eviction_b200 import capi
    lib = capi.load()
    names = declared_functions()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(capi.SIGNATURES), set(names) ^ set(capi.SIGNATURES)


def test_binding_argument_counts_match_header():
    from cache_eviction_b200 import capi
    text = header_text()
    for name, (_, args) in capi.SIGNATURES.items():
        m = re.search(r"\b" + name + r"\s*\(([^)]*)\)\s*;", text)
        assert m, name
        params = [a for a in m.group(1).split(",") if a.strip() and a.strip() != "void"]
        assert len(params) == len(args), (name, len(params), len(args))


def test_version_and_status_strings_without_gpu():
    from cache_eviction_b200 import capi
    lib = capi.load()
    assert b"sm_100a" in lib.ce_version()
    assert lib.ce_status_string(capi.CE_ERR_WORKSPACE) == b"workspace too small"


def test_workspace_queries_are_host_only():
    from cache_eviction_b200 import capi
    lib = capi.load()
    assert lib.ce_choose_workspace_bytes(2, 16, 100) > 0
    assert lib.ce_prefill_workspace_bytes(2048, 64) >= 2048 * 64 * 4
    assert lib.ce_prefill_workspace_bytes(-1, 64) == -1
    # the relocation scratch scales with the widest middle set, not the column count
    wide = lib.ce_boundary_workspace_bytes(32, 1, 8, 64, 16, 4096, 0, 0, 0)
    narrow = lib.ce_boundary_workspace_bytes(32, 1, 8, 64, 16, 4096, 256, 0, 0)
    assert narrow < wide
    assert lib.ce_boundary_workspace_bytes(1, 2, 8, 64, 16, 100, 0, 0, 0) > 0
    assert lib.ce_boundary_workspace_bytes(1, 2, 8, 32, 16, 100, 0, 0, 0) == -1  # head_dim 64 only


def test_row_params_layout_matches_header():
    from cache_eviction_b200 import capi, kernels
    assert C.sizeof(capi.RowParams) == 32 and kernels.ROW_DTYPE.itemsize == 32


def test_live_boundary_needs_a_positive_epoch():
    """ce_boundary tags real slots with epoch and freed units with -epoch in
    the caller's zero-initialised marks, so a live call with epoch 0 is
    refused on the host, before any device work (the pointers below are never
    dereferenced)."""
    from cache_eviction_b200 import capi
    lib = capi.load()
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "ce_api.h").read_text(), flags=re.S)
    params = re.search(r"\bce_boundary\s*\(([^)]*)\)\s*;", text).group(1).split(",")
    names = [re.findall(r"\w+", p)[-1] for p in params]
    ints = {"table_width": 16, "r2u_width": 16, "pos_cap": 16, "pool_units": 64, "layers": 1,
            "kv_heads": 8, "head_dim": 64, "page_size": 1, "num_rows": 1, "live": 1, "max_cols": 16,
            "max_n": 16, "epoch": 0}
    args = []
    for name, p in zip(names, params):
        if "*" in p:
            null = name in ("swa_mapping", "uniforms", "global_scores", "record_delta", "record_counts",
                            "err", "stream")
            args.append(None if null else C.c_void_p(4096))
        else:
            args.append(ints.get(name, 16 if "stride" in name else 0))
    args[names.index("workspace_bytes")] = 1 << 40
    args[names.index("hazard_bytes")] = 1 << 20
    assert lib.ce_boundary(*args) == capi.CE_ERR_ARG
    assert b"epoch" in lib.ce_last_error()


def test_static_decode_refuses_deferred_scores():
    """ce_decode_attn_score_static has no caller workspace for
    ce_decode_scores to read, so CE_SCORE_DEFER is refused on the host before
    any device work (the pointers below are never dereferenced)."""
    from cache_eviction_b200 import capi
    lib = capi.load()
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "ce_api.h").read_text(), flags=re.S)
    params = re.search(r"\bce_decode_attn_score_static\s*\(([^)]*)\)\s*;", text).group(1).split(",")
    names = [re.findall(r"\w+", p)[-1] for p in params]
    ints = {"bs": 1, "num_q_heads": 64, "num_kv_heads": 8, "head_dim": 64, "page_size": 16,
            "score_flags": 3 | capi.CE_SCORE_DEFER, "pool_units": 4, "kv_capacity": 4}
    args = []
    for name, p in zip(names, params):
        if "*" in p:
            args.append(None if name in ("err", "stream", "lse_out", "sinks", "rows") else C.c_void_p(4096))
        elif "float" in p:
            args.append(0.125)
        else:
            args.append(ints.get(name, 0))
    assert lib.ce_decode_attn_score_static(*args) == capi.CE_ERR_ARG
    assert b"caller workspace" in lib.ce_last_error()


def test_deferred_scores_check_shapes_on_the_host():
    """ce_decode_scores validates its sizes before any device work: an
    unsupported head layout or page size is an error status, and a call with
    nothing to score (no mode table) is a no-op (pointers never dereferenced)."""
    from cache_eviction_b200 import capi
    lib = capi.load()
    dummy = C.c_void_p(4096)

    def call(H, G, page, modes=dummy):
        return lib.ce_decode_scores(dummy, dummy, dummy, 16, 16, modes, None, 2, H, G, page, dummy, 16, 1, 3,
                                    dummy, 1 << 20, None, None)
    assert call(63, 8, 16) == capi.CE_ERR_UNSUPPORTED
    assert call(64, 8, 8) == capi.CE_ERR_UNSUPPORTED
    assert call(32, 4, 1) == capi.CE_ERR_UNSUPPORTED        # page size 1 needs 8 KV heads
    assert call(64, 8, 16, modes=None) == capi.CE_OK
