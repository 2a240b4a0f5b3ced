"""Layer golden fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py from the
oracle's exact-f32 layer on seeded inputs).  CPU: the oracle still reproduces them bit for bit
(a change to the oracle or to the synthetic generator shows up here first).  GPU: the CUDA
path matches them -- with the exact router, routing ids and logits exactly; with the default
FFMA router, ids up to reported near-ties -- and outputs within the layer tolerance
(relative L2 <= 5e-3; max-abs <= 2e-2, or 2e-2 x RMS for outputs whose RMS is >= 50)."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, HERE)
import make_golden as G  # noqa: E402

CASES = sorted(G.CASES)


def _load(name):
    return np.load(os.path.join(HERE, name + ".npz"))


@pytest.mark.parametrize("name", CASES)
def test_oracle_reproduces_golden(name):
    f = _load(name)
    _, _, out, ids, w, logits = G.compute(name)
    assert np.array_equal(out, f["out"]) and np.array_equal(ids, f["ids"])
    assert np.array_equal(w, f["w"]) and np.array_equal(logits, f["logits"])


def _close_to_golden(out, want):
    from oracle import oracle as O

    rel, mx, rms = O.layer_errors(out, want)
    assert rel <= O.REL_L2, f"rel-L2 {rel:.3e}"
    assert mx <= O.max_abs_bound(rms), f"max-abs {mx:.3e} (rms {rms:.3e})"


@pytest.mark.gpu
@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("name", CASES)
def test_gpu_matches_golden(name, exact, gpu):
    import torch

    from routing_check import check_routing
    from rusty_engine_b200 import _lib, synth
    from rusty_engine_b200.moe import MoELayer

    build, T, seed = G.CASES[name]
    lw = build()
    x = synth.activations(T, lw.H, seed=seed)
    f = _load(name)
    layer = MoELayer(lw, device=0)
    flags = _lib.FLAG_ROUTING_OUT | (_lib.FLAG_EXACT_ROUTER if exact else 0)
    out = layer.forward(torch.from_numpy(x).cuda(), flags=flags).cpu().numpy()
    ids, w = layer.routing(T)
    logits = layer.logits(T)
    layer.close()
    if exact:
        assert np.array_equal(logits, f["logits"]), "router logits differ"
        assert np.array_equal(ids, f["ids"]), "top-k ids differ"
        np.testing.assert_allclose(w, f["w"], rtol=3e-7, atol=0)
        _close_to_golden(out, f["out"])
    else:
        same = check_routing(ids, w, f["ids"], f["w"], x, lw.router_w, lw.E, name)
        _close_to_golden(out[same], f["out"][same])
