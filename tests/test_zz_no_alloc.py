"""rmoe_layer_forward_noalloc (static device scratch, no cudaMalloc) against rmoe_layer_forward.

Both are called through the C ABI on the same resident layer and the same device inputs; the
no-allocation forward must agree with the allocating one within the layer tolerance used by
the parity tests (relative L2 <= 5e-3; max-abs <= 2e-2 x max(1, RMS): oracle.max_abs_bound),
on calls in a row with different batches, so that what one
call leaves in the shared scratch cannot leak into the next.  The third batch (150 tokens) is
past the one-launch small-batch router, so the multi-kernel dispatch also runs on the static
scratch; it is checked against the CPU oracle as well.  Device errors of a call are read back
with rmoe_noalloc_status.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from rusty_engine_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def assert_close(got, want, what):
    rel, mx, rms = O.layer_errors(got, want)
    assert rel <= O.REL_L2, f"{what}: rel-L2 {rel:.3e}"
    assert mx <= O.max_abs_bound(rms), f"{what}: max-abs {mx:.3e} (rms {rms:.3e})"


@pytest.fixture(scope="module")
def layer(gpu):
    import torch

    from rusty_engine_b200.moe import MoELayer

    torch.cuda.set_device(0)
    lw = synth.config_c2()
    m = MoELayer(lw, device=0)
    m.lw = lw
    yield torch, m
    m.close()


def _pair(torch, m, T, seed, x_np=None):
    """(allocating forward, no-allocation forward) of the same x, both on the current stream."""
    L = _lib.load()
    x = torch.from_numpy(synth.activations(T, m.H, seed=seed) if x_np is None else x_np).cuda()
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
    assert _lib.load().rmoe_noalloc_status(0) == _lib.RMOE_OK


def test_noalloc_multi_kernel_dispatch_matches_oracle(layer):
    """150 tokens: logits, top-k with counts, count scan and row scatter as separate kernels,
    all on the static scratch; against the allocating forward and the exact CPU oracle."""
    torch, m = layer
    x = synth.activations(150, m.H, seed=13)
    ref, got = _pair(torch, m, 150, seed=13, x_np=x)
    assert np.isfinite(got).all()
    assert _lib.load().rmoe_noalloc_status(0) == _lib.RMOE_OK
    assert_close(got, ref, "noalloc 150 tokens vs forward")
    assert_close(got, O.moe_layer_q_exact(x, m.lw)[0], "noalloc 150 tokens vs oracle")


def test_noalloc_status_reports_fp16_range(layer):
    """An x value beyond the fp16 MMA operand range is reported by rmoe_noalloc_status (not
    silently turned into inf), and the read clears the word."""
    torch, m = layer
    L = _lib.load()
    x = synth.activations(4, m.H, seed=14)
    x[2, 100] = 1.0e6
    _pair(torch, m, 4, seed=14, x_np=x)
    assert L.rmoe_noalloc_status(0) == _lib.RMOE_ERR_DEVICE
    assert "fp16 range" in L.rmoe_last_error().decode()
    assert L.rmoe_noalloc_status(0) == _lib.RMOE_OK


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
