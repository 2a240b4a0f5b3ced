"""C ABI checks that need no GPU: the library loads, exports every symbol include/rmoe.h
declares, and host-side validation rejects bad descriptions with the documented status
codes before any device call (the reference panics or returns EngineError there)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from rusty_engine_b200 import _lib, build, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "rmoe.h")).read()
    return sorted(set(re.findall(r"RMOE_API\s+[\w\s\*]+?\b(rmoe_\w+)\s*\(", src)))


def test_library_builds_and_loads():
    path = build.build()
    assert os.path.exists(path)
    _lib.load()


def test_exports_every_declared_symbol():
    syms = header_symbols()
    assert len(syms) >= 12
    L = _lib.load()
    for s in syms:
        assert hasattr(L, s), f"librmoe.so does not export {s}"
    assert set(syms) == set(_lib.EXPORTS)


def test_build_info_names_arch():
    assert b"sm_100a" in _lib.load().rmoe_build_info()


def _desc(lw, **over):
    d = _lib.LayerDesc()
    d.hidden, d.inter, d.n_experts, d.top_k, d.gate = lw.H, lw.I, lw.E, lw.k, lw.gate
    keep = np.ascontiguousarray(lw.router_w)
    d.router_w = keep.ctypes.data
    from rusty_engine_b200.moe import _tensor

    d.gate_exps, d.up_exps, d.down_exps = _tensor(lw.gate_exps), _tensor(lw.up_exps), _tensor(lw.down_exps)
    for k, v in over.items():
        setattr(d, k, v)
    return d, keep


def _create(d):
    h = C.c_void_p()
    st = _lib.load().rmoe_layer_create(C.byref(d) if d is not None else None, C.byref(h))
    return st, _lib.load().rmoe_last_error().decode()


@pytest.fixture(scope="module")
def tiny():
    return synth.make_layer(256, 256, 4, 2, gate_t=2, up_t=2, down_t=2, dlo=0.005, dhi=0.02, seed=5)


def test_null_desc_is_invalid():
    st, msg = _create(None)
    assert st == _lib.RMOE_ERR_INVALID and "null" in msg


def test_zero_top_k_is_invalid(tiny):
    d, _k = _desc(tiny, top_k=0)
    st, msg = _create(d)
    assert st == _lib.RMOE_ERR_INVALID and "top_k" in msg


def test_bad_gate_is_invalid(tiny):
    d, _k = _desc(tiny, gate=7)
    st, _ = _create(d)
    assert st == _lib.RMOE_ERR_INVALID


def test_too_many_experts_unsupported(tiny):
    d, _k = _desc(tiny, n_experts=4096)
    st, _ = _create(d)
    assert st == _lib.RMOE_ERR_UNSUPPORTED


def test_width_not_multiple_of_256_unsupported(tiny):
    d, _k = _desc(tiny, hidden=96)
    st, msg = _create(d)
    assert st == _lib.RMOE_ERR_UNSUPPORTED and "256" in msg


def test_dims_mismatch_invalid(tiny):
    d, _k = _desc(tiny)
    d.down_exps.dims[0] = 512
    st, msg = _create(d)
    assert st == _lib.RMOE_ERR_INVALID and "ffn_down_exps" in msg


def test_null_router_invalid(tiny):
    d, _k = _desc(tiny)
    d.router_w = None
    st, msg = _create(d)
    assert st == _lib.RMOE_ERR_INVALID and "router" in msg


def test_dequant_errors_match_reference_messages():
    L = _lib.load()
    assert L.rmoe_dequant(99, None, 8, None, None) == _lib.RMOE_ERR_UNSUPPORTED
    assert "no scalar dequant for ggml type 99" in L.rmoe_last_error().decode()
    assert L.rmoe_dequant(2, None, 17, None, None) == _lib.RMOE_ERR_INVALID
    assert L.rmoe_last_error().decode() == "Q4_0 data len 17 not a multiple of 18"
    assert L.rmoe_dequant(30, None, 3, None, None) == _lib.RMOE_ERR_INVALID
    assert L.rmoe_last_error().decode() == "BF16 data len 3 not a multiple of 2"


def test_forward_null_layer_invalid():
    L = _lib.load()
    assert L.rmoe_layer_forward(None, None, 1, None, None, 0) == _lib.RMOE_ERR_INVALID


def test_route_rejects_large_k():
    L = _lib.load()
    assert L.rmoe_route(None, 1, 64, 40, 0, None, None, None) == _lib.RMOE_ERR_UNSUPPORTED


def test_route_grouped_host_validation():
    """rmoe_route_grouped rejects unsupported shapes on the host, before any device call."""
    L = _lib.load()
    ids = np.zeros(64, np.uint32)
    w = np.zeros(64, np.float32)
    lg = np.zeros(64, np.float32)
    cases = [
        (dict(E=1024, k=8, ng=8, nbias=0), _lib.RMOE_ERR_UNSUPPORTED),  # E > 512
        (dict(E=64, k=0, ng=8, nbias=0), _lib.RMOE_ERR_UNSUPPORTED),  # k = 0
        (dict(E=64, k=33, ng=8, nbias=0), _lib.RMOE_ERR_UNSUPPORTED),  # k > 32
        (dict(E=512, k=8, ng=65, nbias=0), _lib.RMOE_ERR_UNSUPPORTED),  # more than 64 groups
        (dict(E=64, k=8, ng=8, nbias=4), _lib.RMOE_ERR_INVALID),  # a bias length with no bias
    ]
    for c, want in cases:
        st = L.rmoe_route_grouped(lg.ctypes.data, None, c["nbias"], 1, c["E"], c["k"], c["ng"], 4, 1,
                                  ids.ctypes.data, w.ctypes.data, None)
        assert st == want, (c, L.rmoe_last_error())
    # n_groups is clamped to E (n_groups.max(1).min(n), src/moe.rs:211): 65 groups of 32 experts is legal
    assert L.rmoe_route_grouped(lg.ctypes.data, None, 0, 0, 32, 8, 65, 4, 1, ids.ctypes.data, w.ctypes.data,
                                None) == _lib.RMOE_OK  # T = 0: nothing to do


def test_qmat_host_validation():
    L = _lib.load()
    h = C.c_void_p()
    raw = np.zeros(18 * 32, np.uint8)
    st = L.rmoe_qmat_create(2, raw.ctypes.data, raw.nbytes, 32, 1024, 0, C.byref(h))
    assert st == _lib.RMOE_ERR_UNSUPPORTED and b"multiple of 64" in L.rmoe_last_error()
    assert L.rmoe_qmat_create(2, raw.ctypes.data, raw.nbytes, 64, 256, 0, None) == _lib.RMOE_ERR_INVALID
    assert L.rmoe_qmat_forward(None, None, 4, None, None) == _lib.RMOE_ERR_INVALID
    assert L.rmoe_qmat_status(None) == _lib.RMOE_ERR_INVALID
    L.rmoe_qmat_destroy(None)  # a null handle is ignored


def test_ep_placement_host_validation(tiny):
    """rmoe_ep_layer_create_placed checks the placement table before touching a device: every
    entry a rank of the world, every rank holding at least one expert."""
    d, keep = _desc(tiny)
    uid = (C.c_uint8 * 128)()
    L = _lib.load()

    def create(pl, rank=0, world=2):
        h = C.c_void_p()
        arr = np.ascontiguousarray(pl, dtype=np.int32)
        st = L.rmoe_ep_layer_create_placed(C.byref(d), rank, world, uid, arr.ctypes.data, C.byref(h))
        return st, L.rmoe_last_error().decode()

    st, msg = create([0, 1, 2, 0])
    assert st == _lib.RMOE_ERR_INVALID and "expert_rank[2] = 2" in msg, msg
    st, msg = create([0, 0, 0, 0])
    assert st == _lib.RMOE_ERR_INVALID and "rank 1 holds no expert" in msg, msg
    st, msg = create([-1, 0, 1, 1])
    assert st == _lib.RMOE_ERR_INVALID and "expert_rank[0] = -1" in msg, msg
    h = C.c_void_p()
    st = L.rmoe_ep_layer_create(C.byref(d), 0, 3, uid, C.byref(h))
    assert st == _lib.RMOE_ERR_INVALID and "split evenly" in L.rmoe_last_error().decode()
