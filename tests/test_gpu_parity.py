"""GPU parity: the CUDA path through the C ABI against the CPU oracle on identical seeded
inputs.

Contract:
* top-k expert ids bit-exact against the oracle's (moe::matvec + top_k), with only near-ties
  under a 1e-6 float64 logit gap allowed to differ (reported).  With RMOE_FLAG_EXACT_ROUTER the
  logits themselves are bit-exact; the default (fast) router rescores near-ties with the
  sequential sums, so its ids are bit-exact too (routing_check.py);
* routing weights within 2 ulp-scale (CUDA's and glibc's expf differ by <= 2 ulp) for exact
  logits, 1e-5 relative for fast ones;
* layer outputs: relative L2 <= 5e-3 and max-abs <= 2e-2 * max(1, RMS) (oracle.max_abs_bound).
"""
import numpy as np
import pytest

from oracle import oracle as O
from routing_check import check_logit_margin, check_routing
from rusty_engine_b200 import _lib, synth

pytestmark = pytest.mark.gpu

REL_L2 = O.REL_L2
MAX_ABS = O.MAX_ABS


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b.astype(np.float64)), 1e-30))


def assert_layer_close(got, want, what=""):
    r, mx, rms = O.layer_errors(got, want)
    bound = O.max_abs_bound(rms)
    print(f"{what}: rel-L2 {r:.2e}, max-abs {mx:.3e}, rms {rms:.3e}, max-abs/rms {mx / max(rms, 1e-30):.2e} "
          f"(bar {bound:.3e})")
    assert r <= REL_L2, f"{what}: rel-L2 {r:.3e} > {REL_L2}"
    assert mx <= bound, f"{what}: max-abs {mx:.3e} > {bound:.3e} (rms {rms:.3e})"


@pytest.fixture(scope="module")
def torch_cuda(gpu):
    import torch

    return torch


def run_layer(torch, lw, x, flags=0, routing=True):
    from rusty_engine_b200.moe import MoELayer

    layer = MoELayer(lw, device=0)
    xd = torch.from_numpy(x).cuda()
    out = layer.forward(xd, flags=flags | (_lib.FLAG_ROUTING_OUT if routing else 0))
    torch.cuda.synchronize()
    res = {"out": out.cpu().numpy(), "refined": layer.router_refined()}
    if routing:
        res["ids"], res["w"] = layer.routing(x.shape[0])
        res["logits"] = layer.logits(x.shape[0])
    layer.close()
    return res


# ---- stand-alone operators -------------------------------------------------------------------
@pytest.mark.parametrize("t", [2, 6, 8, 12, 13, 14, 0, 1, 30])
def test_dequant_bit_exact(torch_cuda, t):
    from rusty_engine_b200.moe import dequant

    rng = np.random.default_rng(t)
    el, _ = synth.BLOCK[t]
    raw = synth.gen_blocks(rng, t, 64 if el > 1 else 4096, 0.001, 0.05)
    got = dequant(t, raw)
    want = O.dequant(t, raw.tobytes())
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_dequant_errors(torch_cuda):
    from rusty_engine_b200.moe import EngineError, dequant

    with pytest.raises(EngineError, match="Q4_0 data len 17 not a multiple of 18"):
        dequant(2, bytes(17))


def test_route_reference_kats(torch_cuda):
    from rusty_engine_b200.moe import Gate, RouterConfig, route, top_k, top_k_sigmoid

    s = top_k([0.1, 0.9, 0.2, 0.8], 2)  # src/moe.rs:632-641
    assert [e.id for e in s] == [1, 3] and abs(sum(e.weight for e in s) - 1) < 1e-5
    assert len(top_k([0.5, 0.4], 8)) == 2  # src/moe.rs:643-646
    s = top_k_sigmoid([1.0, 5.0, 2.0, 4.0], 2)  # src/moe.rs:656-663
    assert [e.id for e in s] == [1, 3] and abs(sum(e.weight for e in s) - 1) < 1e-5
    assert [e.id for e in route([0.0, 3.0, 1.0, 2.0], RouterConfig(Gate.Sigmoid, 2))] == [1, 3]
    assert route([], RouterConfig()) == []


def test_route_grouped_reference_kats(torch_cuda):
    """The reference's group-routing tests (src/moe.rs:666-710) through rmoe_route_grouped."""
    from rusty_engine_b200.moe import route_group, route_noaux_tc

    logits = [5.0, 2.0, -9.0, -9.0, 0.0, 0.0, 0.0, 0.0]
    s = route_noaux_tc(logits, [], 2, 1, 1)  # the dominant pair's group wins
    assert s[0].id == 0 and abs(s[0].weight - 1.0) < 1e-5
    assert 4 <= route_group(logits, [], 2, 1, 1)[0].id <= 7  # the all-sum version: the other group
    s = route_noaux_tc(logits, [], 2, 2, 1)
    assert [e.id for e in s] == [0, 1] and abs(sum(e.weight for e in s) - 1.0) < 1e-5
    assert route_noaux_tc([], [], 2, 1, 1) == []


@pytest.mark.parametrize("E,ng,tkg,k,noaux", [(256, 8, 4, 8, True), (256, 8, 4, 8, False), (96, 7, None, 6, True),
                                              (128, 1, 1, 8, True), (16, 8, 1, 4, True)])
def test_route_grouped_vs_oracle(torch_cuda, E, ng, tkg, k, noaux):
    """rmoe_route_grouped against the oracle's restatement on random logits and bias: ids equal
    (a difference only where the two experts' sigmoid scores are within a few ulp: CUDA's and
    glibc's expf may differ by an ulp), weights within 1e-5 relative; picks beyond the eligible
    experts are empty (id 0xFFFFFFFF, weight 0)."""
    from rusty_engine_b200.moe import route_grouped_batch

    rng = np.random.default_rng(E * 31 + ng)
    T = 300
    logits = rng.standard_normal((T, E), dtype=np.float32)
    bias = (rng.standard_normal(E, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    ids, w = route_grouped_batch(logits, bias, ng, k, tkg, noaux)
    sig = (1.0 / (1.0 + np.exp(-(logits + bias).astype(np.float64)))).astype(np.float32)
    for t in range(T):
        ref = O.route_grouped(logits[t], bias, ng, k, tkg, noaux)
        rid = np.array([i for i, _ in ref], dtype=np.int64)
        rw = np.array([x for _, x in ref], dtype=np.float32)
        n = len(ref)
        assert (ids[t, n:] == 0xFFFFFFFF).all() and (w[t, n:] == 0).all()
        got = ids[t, :n].astype(np.int64)
        for j in np.nonzero(got != rid)[0]:
            a, b = sig[t, got[j]], sig[t, rid[j]]
            assert abs(float(a) - float(b)) <= 4 * np.spacing(np.float32(max(a, b))), (t, j, got[j], rid[j])
        if (got == rid).all():
            np.testing.assert_allclose(w[t, :n], rw, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("gate", [0, 1])
def test_route_random_with_ties_bit_exact(torch_cuda, gate):
    from rusty_engine_b200.moe import Gate, RouterConfig, route_batch

    rng = np.random.default_rng(11 + gate)
    T, E, k = 257, 128, 8
    lg = rng.standard_normal((T, E)).astype(np.float32)
    lg[:, 5] = lg[:, 9]  # exact ties: the lower index must win
    lg[::3, 100:110] = 1.5
    ids, w = route_batch(lg, RouterConfig(Gate(gate), k))
    wids, ww = O.route_batch(lg, gate, k)
    assert np.array_equal(ids.astype(np.uint32), wids)
    assert np.allclose(w, ww, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("t", [2, 6, 8, 12, 13, 14, 0])
def test_qmat_matmul_parity(torch_cuda, t):
    from rusty_engine_b200.moe import QMat

    rng = np.random.default_rng(100 + t)
    m, n, rows = 128, 512, 37
    el, _ = synth.BLOCK[t]
    raw = synth.gen_blocks(rng, t, m * n // el, 0.001, 0.01)
    x = rng.standard_normal((rows, n)).astype(np.float32)
    got = QMat.from_bytes(t, raw, m, n).matmul(x, rows)
    deq = O.dequant(t, raw.tobytes()).reshape(m, n)
    want = np.stack([O.matvec(deq, m, n, x[r]) for r in range(rows)])
    assert rel_l2(got, want) <= REL_L2


@pytest.mark.parametrize("t", [12, 14, 2, 8, 0])
def test_qmat_matmul_many_rows_tensor_cores(torch_cuda, t):
    """QMat::matmul at prefill row counts (the tcgen05 path: rows >= 128, m % 128 == 0,
    n % 256 == 0), ragged last tile, against the dequantized sequential-f32 matvec per row."""
    from rusty_engine_b200.moe import QMat

    rng = np.random.default_rng(200 + t)
    m, n, rows = 256, 1024, 600
    el, _ = synth.BLOCK[t]
    raw = synth.gen_blocks(rng, t, m * n // el, 0.001, 0.01)
    x = rng.standard_normal((rows, n)).astype(np.float32)
    got = QMat.from_bytes(t, raw, m, n).matmul(x, rows)
    deq = O.dequant(t, raw.tobytes()).reshape(m, n)
    want = np.stack([O.matvec(deq, m, n, x[r]) for r in range(rows)])
    assert rel_l2(got, want) <= REL_L2


def test_qmat_resident_handle_reuse(torch_cuda):
    """One resident QMat (rmoe_qmat_create) driven with growing and shrinking row counts,
    across both kernels: every product equals a fresh handle's, bit for bit."""
    from rusty_engine_b200.moe import QMat

    rng = np.random.default_rng(7)
    m, n = 256, 1024
    raw = synth.gen_blocks(rng, 12, m * n // 256, 0.001, 0.01)
    q = QMat.from_bytes(12, raw, m, n)
    for rows in (5, 300, 130, 1, 700, 64):
        x = rng.standard_normal((rows, n)).astype(np.float32)
        a = q.matmul(x, rows)
        b = QMat.from_bytes(12, raw, m, n).matmul(x, rows)
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("rows", [37, 300])
def test_qmat_x_beyond_fp16_range(torch_cuda, rows):
    """QMat::matmul is f32 throughout: rows with |x| far beyond 65504 are carried as fp16 x 2^e
    (the product scaled back exactly), so the result stays finite and matches the dequantized
    sequential matvec on both kernels; a non-finite x is reported by rmoe_qmat_status."""
    import ctypes as C

    from rusty_engine_b200.moe import QMat

    rng = np.random.default_rng(300 + rows)
    m, n = 256, 1024
    raw = synth.gen_blocks(rng, 12, m * n // 256, 0.001, 0.01)
    x = rng.standard_normal((rows, n)).astype(np.float32)
    x[1] *= np.float32(1e6)
    x[rows // 2, 17] = np.float32(3.0e5)
    q = QMat.from_bytes(12, raw, m, n)
    got = q.matmul(x, rows)
    deq = O.dequant(12, raw.tobytes()).reshape(m, n)
    want = np.stack([O.matvec(deq, m, n, x[r]) for r in range(rows)])
    assert np.isfinite(got).all()
    for r in (0, 1, rows // 2):
        assert rel_l2(got[r], want[r]) <= REL_L2, f"row {r}"
    L = _lib.load()
    assert L.rmoe_qmat_status(q._handle()) == _lib.RMOE_OK
    x[3, 5] = np.inf
    q.matmul_device(torch_cuda.from_numpy(x).cuda())
    torch_cuda.cuda.synchronize()
    assert L.rmoe_qmat_status(q._handle()) == _lib.RMOE_ERR_DEVICE
    assert L.rmoe_qmat_status(q._handle()) == _lib.RMOE_OK
    # Out is written with 16-B vector stores: a misaligned view is refused on the host
    xd = torch_cuda.from_numpy(x[:, :]).cuda()
    buf = torch_cuda.empty(rows * m + 4, dtype=torch_cuda.float32, device="cuda")
    st = L.rmoe_qmat_forward(q._handle(), xd.data_ptr(), rows, buf[1:].data_ptr(),
                             C.c_void_p(torch_cuda.cuda.current_stream().cuda_stream))
    assert st == _lib.RMOE_ERR_INVALID and "16-byte aligned" in L.rmoe_last_error().decode()


# ---- the layer --------------------------------------------------------------------------------
def check_layer(got, lw, x, out, ids, w, what):
    """Fast-router contract: ids bit-exact up to reported sub-1e-6 near-ties, outputs on the
    tokens routed alike (all of them unless a near-tie differed)."""
    same = check_routing(got["ids"], got["w"], ids, w, x, lw.router_w, lw.E, what)
    print(f"{what}: {got.get('refined', 0)} token(s) refined with the sequential sums")
    assert_layer_close(got["out"][same], out[same], what)


def test_c1_layer_parity(torch_cuda):
    """H 1024, E 16, top-4, I 512, Q4_0, 128 tokens, seed 0."""
    lw = synth.config_c1()
    x = synth.activations(128, lw.H)
    out, ids, w, logits = O.moe_layer_q_exact(x, lw)
    got = run_layer(torch_cuda, lw, x, flags=_lib.FLAG_EXACT_ROUTER)
    assert np.array_equal(got["logits"].view(np.uint32), logits.view(np.uint32)), "router logits not bit-exact"
    assert np.array_equal(got["ids"], ids), "top-k ids not bit-exact"
    assert np.allclose(got["w"], w, rtol=2e-6, atol=1e-7)
    assert_layer_close(got["out"], out, "c1 exact router")
    got = run_layer(torch_cuda, lw, x)
    check_logit_margin(got["logits"], logits, x, lw.router_w, "c1")
    check_layer(got, lw, x, out, ids, w, "c1")


def test_c1_deterministic_mode_reproducible(torch_cuda):
    lw = synth.config_c1()
    x = synth.activations(128, lw.H)
    a = run_layer(torch_cuda, lw, x, flags=_lib.FLAG_DETERMINISTIC, routing=False)["out"]
    b = run_layer(torch_cuda, lw, x, flags=_lib.FLAG_DETERMINISTIC, routing=False)["out"]
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    want = O.moe_layer_q_exact(x, lw)[0]
    assert_layer_close(a, want, "c1 deterministic")


def test_c2_layer_parity(torch_cuda):
    """BASELINE config 2 (Qwen3-30B-A3B layer, Q4_K gate/up, Q6_K down), 4096 tokens, every
    token against the exact oracle: with the exact router, logits and ids bit-exact; with the
    default (timed) router, ids bit-exact up to sub-1e-6 near-ties; outputs on all tokens."""
    lw = synth.config_c2()
    x = synth.activations(4096, lw.H)
    out, ids, w, logits = O.moe_layer_q_exact(x, lw)
    got = run_layer(torch_cuda, lw, x, flags=_lib.FLAG_EXACT_ROUTER)
    assert np.array_equal(got["logits"].view(np.uint32), logits.view(np.uint32)), "router logits not bit-exact"
    assert np.array_equal(got["ids"], ids)
    assert np.allclose(got["w"], w, rtol=2e-6, atol=1e-7)
    assert_layer_close(got["out"], out, "c2 exact router")
    got = run_layer(torch_cuda, lw, x)
    check_logit_margin(got["logits"], logits, x, lw.router_w, "c2")
    check_layer(got, lw, x, out, ids, w, "c2")


@pytest.fixture(scope="module")
def c5_workload():
    """BASELINE config 5 layer (H 4096, E 128, top-8, I 1536, Q4_K gate/up, Q6_K down) with the
    Zipf(1.1) expert load realised in the router, 1024 tokens."""
    lw, x = synth.zipf_workload(synth.config_c5(), 1024, seed=1)
    return lw, x


def test_c5_layer_parity(torch_cuda, c5_workload):
    """Config 5 shapes (K = 1536 Q6_K down rows of 1260 B; skewed per-expert tile lists) on the
    tensor-core path, every token against the exact oracle, default router."""
    lw, x = c5_workload
    out, ids, w, logits = O.moe_layer_q_exact(x, lw)
    got = run_layer(torch_cuda, lw, x)
    load = np.bincount(ids.ravel().astype(np.int64), minlength=lw.E)
    print(f"c5: busiest expert {load.max()} rows, idlest {load.min()} rows")
    check_logit_margin(got["logits"], logits, x, lw.router_w, "c5")
    check_layer(got, lw, x, out, ids, w, "c5")
    got = run_layer(torch_cuda, lw, x[:48], routing=True)  # the decode kernels on the same layer
    check_layer(got, lw, x[:48], out[:48], ids[:48], w[:48], "c5 48 tokens")


@pytest.mark.parametrize("gate", [0, 1])
@pytest.mark.parametrize("T", [12, 40, 300, 1500])
def test_router_near_ties_refined(torch_cuda, gate, T):
    """Router rows built to tie: rows 9 and 10 equal row 5 up to one element perturbed by a
    few ulp (float64 logit gaps ~1e-8 to 1e-6), rows 20 and 21 exactly equal.  The fast
    router's sums cannot order such picks by themselves; the refinement must reproduce the
    sequential sums' order (ids bit-exact) through each router path: the one-launch layer
    (T <= 16), the one-launch router (T <= 64), the warp-per-expert logits (T < 1024) and the
    tensor-core logits."""
    lw = synth.make_layer(2048, 256, 128, 8, gate_t=12, up_t=12, down_t=14, dlo=0.001, dhi=0.004, seed=21 + gate,
                          gate=gate)
    rw = lw.router_w
    rw *= np.float32(3.0)  # bring the tied rows into the top picks more often
    rw[9] = rw[5]
    rw[9, 7] = np.nextafter(rw[5, 7], np.float32(1), dtype=np.float32)
    rw[10] = rw[5]
    rw[10, 1000] = np.nextafter(np.nextafter(rw[5, 1000], np.float32(-1), dtype=np.float32), np.float32(-1),
                                dtype=np.float32)
    rw[21] = rw[20]
    x = synth.activations(T, lw.H, seed=50 + T)
    logits = O.router_logits(x, lw.router_w, lw.E)
    ids, w = O.route_batch(logits, gate, lw.k)
    got = run_layer(torch_cuda, lw, x)
    same = check_routing(got["ids"], got["w"], ids, w, x, lw.router_w, lw.E, f"near-ties gate={gate} T={T}")
    if gate == 0:  # (sigmoid scores also carry expf's last-ulp differences between CUDA and glibc)
        assert same.all(), "a near-tie was ordered differently from the sequential sums"
    tied = (np.isin(ids, [5, 9, 10]).sum(axis=1) >= 2) | (np.isin(ids, [20, 21]).sum(axis=1) >= 1)
    print(f"near-ties gate={gate} T={T}: {int(tied.sum())} tokens pick a tied row; {got['refined']} refined")
    assert got["refined"] >= (1 if tied.any() else 0)


@pytest.mark.parametrize("E,T", [(256, 1100), (96, 1100), (64, 1030), (16, 1024), (128, 2053)])
def test_large_batch_router_logits(torch_cuda, E, T):
    """The fast router at >= 1024 tokens (tensor-core product of split fp32 operands for up to
    128 experts, the FFMA product above; K-split partial sums added in split order): logits
    well inside the refinement window of the sequential sums, ids bit-exact, for expert counts
    16..256 and token counts off the 128-token tile grid."""
    lw = synth.make_layer(1024, 256, E, 8, gate_t=synth.GGML_Q4_0, up_t=synth.GGML_Q4_0,
                          down_t=synth.GGML_Q4_0, dlo=0.005, dhi=0.02, seed=E)
    x = synth.activations(T, lw.H, seed=T)
    logits = O.router_logits(x, lw.router_w, lw.E)
    ids, w = O.route_batch(logits, 0, lw.k)
    got = run_layer(torch_cuda, lw, x)
    check_logit_margin(got["logits"], logits, x, lw.router_w, f"E={E} T={T}")
    same = check_routing(got["ids"], got["w"], ids, w, x, lw.router_w, lw.E, f"E={E} T={T}")
    assert same.all()


@pytest.fixture(scope="module")
def c2_weights():
    return synth.config_c2()


@pytest.mark.parametrize("T", [1, 5, 8, 16, 32, 64])
def test_c3_decode_parity(torch_cuda, c2_weights, T):
    """the C2 layer at decode batch sizes, through the decode GEMV kernels
    (Q4_K gate/up, Q6_K down): up to 16 tokens the whole layer in one launch (atomic combine),
    else the routing and expert kernels; the deterministic combine always takes the latter."""
    lw = c2_weights
    x = synth.activations(T, lw.H, seed=100 + T)
    out, ids, w, _ = O.moe_layer_q_exact(x, lw)
    for det in (0, _lib.FLAG_DETERMINISTIC):
        got = run_layer(torch_cuda, lw, x, flags=det)
        check_layer(got, lw, x, out, ids, w, f"c3 b={T} det={det}")


@pytest.mark.parametrize("T", [1, 5, 8, 16])
def test_one_launch_decode_layer(torch_cuda, c2_weights, T, monkeypatch):
    """The whole decode layer as one cooperative launch (RMOE_SMALL_LAYER=1): the C2 layer at
    up to 16 tokens, and a sigmoid-gate layer with a shared expert, against the oracle."""
    monkeypatch.setenv("RMOE_SMALL_LAYER", "1")
    lw = c2_weights
    x = synth.activations(T, lw.H, seed=200 + T)
    out, ids, w, _ = O.moe_layer_q_exact(x, lw)
    got = run_layer(torch_cuda, lw, x)
    check_layer(got, lw, x, out, ids, w, f"one-launch b={T}")
    ls = synth.make_layer(512, 256, 16, 4, gate_t=12, up_t=12, down_t=14, dlo=0.001, dhi=0.01, seed=9, gate=1,
                          shared=True)
    xs = synth.activations(T, ls.H, seed=9)
    out, ids, w, _ = O.moe_layer_q_exact(xs, ls)
    got = run_layer(torch_cuda, ls, xs)
    check_layer(got, ls, xs, out, ids, w, f"one-launch sigmoid+shared b={T}")


@pytest.mark.parametrize("T", [1, 3, 127])
def test_ragged_token_counts(torch_cuda, T):
    lw = synth.config_c1()
    x = synth.activations(T, lw.H, seed=T)
    got = run_layer(torch_cuda, lw, x)
    out, ids, w, _ = O.moe_layer_q_exact(x, lw)
    check_layer(got, lw, x, out, ids, w, f"T={T}")


PATHS = {"mma_sync": _lib.FLAG_FORCE_SMALL, "tcgen05": _lib.FLAG_FORCE_LARGE}


@pytest.mark.parametrize("path", sorted(PATHS))
@pytest.mark.parametrize("gt,dt", [(2, 2), (6, 6), (8, 8), (12, 14), (13, 13), (14, 14), (12, 12), (0, 0)])
def test_formats_small_layer(torch_cuda, gt, dt, path):
    lw = synth.make_layer(512, 256, 8, 2, gate_t=gt, up_t=gt, down_t=dt, dlo=0.002, dhi=0.02, seed=gt * 16 + dt)
    x = synth.activations(40, lw.H, seed=7)
    got = run_layer(torch_cuda, lw, x, flags=PATHS[path])
    out, ids, w, _ = O.moe_layer_q_exact(x, lw)
    check_layer(got, lw, x, out, ids, w, f"types {gt}/{dt} {path}")


@pytest.mark.parametrize("path", sorted(PATHS))
def test_c1_both_paths(torch_cuda, path):
    """Config 1 through each expert-product path, atomic and deterministic combine."""
    lw = synth.config_c1()
    x = synth.activations(128, lw.H)
    want = O.moe_layer_q_exact(x, lw)[0]
    for det in (0, _lib.FLAG_DETERMINISTIC):
        got = run_layer(torch_cuda, lw, x, flags=PATHS[path] | det, routing=False)["out"]
        assert_layer_close(got, want, f"c1 {path} det={det}")


@pytest.mark.parametrize("T", [6, 33])
def test_sigmoid_gate_and_shared_expert(torch_cuda, T):
    lw = synth.make_layer(512, 256, 16, 4, gate_t=12, up_t=12, down_t=14, dlo=0.001, dhi=0.01, seed=9, gate=1,
                          shared=True)
    x = synth.activations(T, lw.H, seed=9)
    for flags in (0, _lib.FLAG_DETERMINISTIC):
        got = run_layer(torch_cuda, lw, x, flags=flags)
        out, ids, w, _ = O.moe_layer_q_exact(x, lw)
        check_layer(got, lw, x, out, ids, w, "sigmoid+shared")
        got = run_layer(torch_cuda, lw, x, flags=flags | _lib.FLAG_EXACT_ROUTER)
        assert np.array_equal(got["ids"], ids)
        assert np.allclose(got["w"], w, rtol=2e-6, atol=1e-7)
        assert_layer_close(got["out"], out, "sigmoid+shared exact router")


def test_host_io_matches_device_path(torch_cuda):
    from rusty_engine_b200.moe import MoELayer

    lw = synth.config_c1()
    x = synth.activations(64, lw.H, seed=3)
    layer = MoELayer(lw, device=0)
    a = layer.forward_host(x, flags=_lib.FLAG_DETERMINISTIC)
    b = layer.forward(torch_cuda.from_numpy(x).cuda(), flags=_lib.FLAG_DETERMINISTIC).cpu().numpy()
    layer.close()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("T", [2048, 3000])
def test_host_io_chunked_pipeline(torch_cuda, T):
    """Large host-buffer forwards are split into token chunks whose copies overlap the compute
    (four and five chunks of the C1 layer here, each at least 128 routed rows per expert):
    outputs match the one-shot device-buffer forward (deterministic combine, so both sum each
    token's experts in the same order) and the oracle."""
    from rusty_engine_b200.moe import MoELayer

    lw = synth.config_c1()
    x = synth.activations(T, lw.H, seed=T)
    layer = MoELayer(lw, device=0)
    a = layer.forward_host(x, flags=_lib.FLAG_DETERMINISTIC)
    b = layer.forward(torch_cuda.from_numpy(x).cuda(), flags=_lib.FLAG_DETERMINISTIC).cpu().numpy()
    layer.close()
    # a chunk of fewer than 1024 tokens takes the FFMA router logits instead of the tensor-core
    # ones, so the routing weights (not the ids) may differ in the last bits
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-5)
    assert_layer_close(a, O.moe_layer_q_exact(x, lw)[0], f"host-IO chunked T={T}")


def test_reference_layer_kats_f32_experts(torch_cuda):
    """moe_layer_routes_to_best_expert / moe_layer_adds_shared_expert (src/moe.rs:773-801)
    through the f32-ExpertWeights signature (zero-padded to the kernel widths)."""
    from rusty_engine_b200.moe import ExpertWeights, Gate, RouterConfig, moe_layer_forward

    silu1 = O.silu(1.0)
    ide = lambda s: ExpertWeights(np.array([1.0, 0, 0, 1.0]), np.array([1.0, 0, 0, 1.0]), np.array([s, 0, 0, s]))
    out = moe_layer_forward([1.0, 0.0], [0.0, 0.0, 10.0, 0.0], 2, [ide(1.0), ide(2.0)], None, 2,
                            RouterConfig(Gate.Softmax, 1))
    assert abs(out[0] - 2 * silu1) <= MAX_ABS and abs(out[1]) <= MAX_ABS
    out = moe_layer_forward([1.0, 0.0], [10.0, 0.0, 0.0, 0.0], 2, [ide(1.0), ide(1.0)], ide(1.0), 2,
                            RouterConfig(Gate.Sigmoid, 1))
    assert abs(out[0] - 2 * silu1) <= MAX_ABS and abs(out[1]) <= MAX_ABS
