"""Failure handling on the GPU without a fault: a bounded wait that runs out.

rmoe_selftest_bounded_wait makes one CTA wait on an mbarrier that nothing arrives at, with a
100 us limit instead of the product kernels' 1 s; the kernel must record DERR_TIMEOUT, free its
tensor memory and return, the call must report RMOE_ERR_DEVICE, and the context must stay
usable: a layer forward afterwards still matches the oracle."""
import numpy as np
import pytest

from oracle import oracle as O
from rusty_engine_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_context_survives(gpu):
    import torch

    from rusty_engine_b200.moe import MoELayer

    L = _lib.load()
    st = L.rmoe_selftest_bounded_wait(0, 100)
    assert st == _lib.RMOE_ERR_DEVICE, L.rmoe_last_error().decode()
    msg = L.rmoe_last_error().decode()
    assert "DERR_TIMEOUT" in msg and "100 us" in msg, msg
    assert L.rmoe_selftest_bounded_wait(0, 0) == _lib.RMOE_ERR_INVALID
    lw = synth.config_c1()
    x = synth.activations(128, lw.H, seed=4)
    layer = MoELayer(lw, device=0)
    got = layer.forward(torch.from_numpy(x).cuda(), flags=_lib.FLAG_FORCE_LARGE).cpu().numpy()
    layer.close()
    rel, mx, rms = O.layer_errors(got, O.moe_layer_q_exact(x, lw)[0])
    assert rel <= O.REL_L2 and mx <= O.max_abs_bound(rms)
