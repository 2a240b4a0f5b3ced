"""Routing comparison under the parity contract: top-k expert ids are
bit-exact against the oracle except at near-ties, which are reported, not failed.

The fast router sums the logits with fused multiply-adds in a different order than
moe::matvec's sequential f32 sums.  Both differ from the exact (float64) logits by f32
summation error, and the reference's own sequential sum over H <= 4096 terms is the larger of
the two: up to a few 1e-6 at these logit sizes.  So an id can differ only where two float64
logits are that close.  Differences at float64 gaps under NEAR_TIE (the contract's 1e-6) are
near-ties; those under SUM_ERR (the reference's summation error level) are ties of the
reference's own rounding.  Both are printed with their gaps; a wider gap fails.  Tokens whose
routing differs are left out of the output comparison (the oracle routed them elsewhere).
RMOE_FLAG_EXACT_ROUTER reproduces the sequential sums bit for bit (no differences at all)."""
import numpy as np

from oracle import oracle as O

NEAR_TIE = 1e-6
SUM_ERR = 5e-6


def check_routing(got_ids, got_w, ref_ids, ref_w, x, router_w, E, what=""):
    """Assert the contract; return the mask of tokens whose ids match exactly (their weights
    are checked against the oracle's too)."""
    got_ids = np.asarray(got_ids).astype(np.int64)
    ref_ids = np.asarray(ref_ids).astype(np.int64)
    same = (got_ids == ref_ids).all(axis=1)
    bad = np.nonzero(~same)[0]
    if bad.size:
        l64 = O.router_logits_f64(np.asarray(x)[bad], router_w, E)
        gaps = []
        for r, t in enumerate(bad):
            for j in np.nonzero(got_ids[t] != ref_ids[t])[0]:
                gap = abs(l64[r, got_ids[t, j]] - l64[r, ref_ids[t, j]])
                assert gap < SUM_ERR, (f"{what}: token {t} slot {j}: expert {got_ids[t, j]} vs oracle "
                                       f"{ref_ids[t, j]}, float64 logit gap {gap:.3e}")
                gaps.append(gap)
        near = sum(g < NEAR_TIE for g in gaps)
        print(f"{what}: routing differences at tokens {bad.tolist()}: {near} near-tie pick(s) (float64 gap "
              f"< {NEAR_TIE:g}), {len(gaps) - near} within the reference's f32 summation error "
              f"(max gap {max(gaps):.2e})")
    np.testing.assert_allclose(np.asarray(got_w)[same], np.asarray(ref_w)[same], rtol=1e-5, atol=1e-7)
    return same
