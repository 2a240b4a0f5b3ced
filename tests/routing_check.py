"""Routing comparison under the parity contract: top-k expert ids are
bit-exact against the oracle except at near-ties -- a pick whose expert and the oracle's
expert have float64 logits within 1e-6 of each other -- which are reported, not failed.

The fast router sums the logits with fused multiply-adds (a few ulp from moe::matvec's
sequential sums), so an id can differ only where two logits are that close.  Tokens whose
routing differs are left out of the output comparison (the oracle routed them elsewhere)."""
import numpy as np

from oracle import oracle as O

NEAR_TIE = 1e-6


def check_routing(got_ids, got_w, ref_ids, ref_w, x, router_w, E, what=""):
    """Assert the contract; return the mask of tokens whose ids match exactly (their weights
    are checked against the oracle's too)."""
    got_ids = np.asarray(got_ids).astype(np.int64)
    ref_ids = np.asarray(ref_ids).astype(np.int64)
    same = (got_ids == ref_ids).all(axis=1)
    bad = np.nonzero(~same)[0]
    if bad.size:
        l64 = O.router_logits_f64(np.asarray(x)[bad], router_w, E)
        for r, t in enumerate(bad):
            for j in np.nonzero(got_ids[t] != ref_ids[t])[0]:
                gap = abs(l64[r, got_ids[t, j]] - l64[r, ref_ids[t, j]])
                assert gap < NEAR_TIE, (f"{what}: token {t} slot {j}: expert {got_ids[t, j]} vs oracle "
                                        f"{ref_ids[t, j]}, float64 logit gap {gap:.3e}")
        print(f"{what}: near-tie routing differences reported for tokens {bad.tolist()}")
    np.testing.assert_allclose(np.asarray(got_w)[same], np.asarray(ref_w)[same], rtol=1e-5, atol=1e-7)
    return same
