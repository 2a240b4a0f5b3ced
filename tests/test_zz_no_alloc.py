"""rmoe_layer_forward_noalloc (static device scratch, no cudaMalloc) against rmoe_layer_forward.

Both are called through the C ABI on the same resident layer and the same device inputs; the
no-allocation forward must agree with the allocating one within the layer tolerance used by
the parity tests (relative L2 <= 5e-3; max-abs <= 2e-2, or 2e-2 x RMS for outputs whose RMS
is >= 50), on two calls in a row with different batches, so that what the first call leaves
in the shared scratch cannot leak into the second.
"""
import ctypes as C

import numpy as np
import pytest

from rusty_engine_b200 import _lib, synth

pytestmark = pytest.mark.gpu

REL_L2 = 5e-3
MAX_ABS = 2e-2


def assert_close(got, want, what):
    got = got.astype(np.float64)
    want = want.astype(np.float64)
    rel = float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))
    rms = float(np.sqrt(np.mean(want**2)))
    bound = MAX_ABS if rms < 1.0 / MAX_ABS else MAX_ABS * rms
    assert rel <= REL_L2, f"{what}: rel-L2 {rel:.3e}"
    assert np.abs(got - want).max() <= bound, f"{what}: max-abs {np.abs(got - want).max():.3e} (rms {rms:.3e})"


@pytest.fixture(scope="module")
def layer(gpu):
    import torch

    from rusty_engine_b200.moe import MoELayer

    torch.cuda.set_device(0)
    lw = synth.config_c2()
    m = MoELayer(lw, device=0)
    yield torch, m
    m.close()


def _pair(torch, m, T, seed):
    """(allocating forward, no-allocation forward) of the same x, both on the current stream."""
    L = _lib.load()
    x = torch.from_numpy(synth.activations(T, m.H, seed=seed)).cuda()
    ref = torch.empty_like(x)
    got = torch.full_like(x, float("nan"))  # the call must write every element
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(L.rmoe_layer_forward(m._h, x.data_ptr(), T, ref.data_ptr(), s, 0))
    _lib.check(L.rmoe_layer_forward_noalloc(m._h, x.data_ptr(), T, got.data_ptr(), s))
    torch.cuda.synchronize()
    return ref.cpu().numpy(), got.cpu().numpy()


def test_noalloc_matches_forward_two_calls(layer):
    torch, m = layer
    ref1, got1 = _pair(torch, m, 64, seed=11)
    ref2, got2 = _pair(torch, m, 5, seed=12)
    assert np.isfinite(got1).all() and np.isfinite(got2).all()
    assert_close(got1, ref1, "noalloc call 1 (64 tokens)")
    assert_close(got2, ref2, "noalloc call 2 (5 tokens)")


def test_noalloc_rejects_batches_beyond_scratch(layer):
    torch, m = layer
    L = _lib.load()
    T = 4096  # needs far more than the static scratch for this layer
    x = torch.zeros((T, m.H), dtype=torch.float32, device="cuda")
    out = torch.zeros_like(x)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = L.rmoe_layer_forward_noalloc(m._h, x.data_ptr(), T, out.data_ptr(), s)
    assert st == _lib.RMOE_ERR_INVALID
    msg = L.rmoe_last_error().decode()
    assert "bytes of scratch" in msg and str(_lib.NOALLOC_SCRATCH_BYTES) in msg, msg
