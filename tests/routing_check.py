"""Routing comparison under the parity contract: top-k expert ids are
bit-exact against the oracle, except at near-ties within 1e-6 (float64 logit gap), which are
reported.

The fast router sums the logits in another order than moe::matvec's sequential f32 chain, so
its logits differ from the reference's by f32 summation error.  For every token whose k + 1
best scores hold two within REFINE_UNITS * u * ||w||max * ||x_t|| of each other (u = 2^-24),
the router rescores the experts around the k-th pick with the sequential chain
(``warp_topk_refined_n`` in route.cu) before choosing, so the ids it returns are the
reference's on every token.  ``check_routing`` therefore allows a difference only under the
contract's 1e-6 window, and ``check_logit_margin`` checks that the fast sums stay well inside
the window the refinement relies on.
"""
import numpy as np

from oracle import oracle as O

NEAR_TIE = 1e-6
REFINE_UNITS = 64.0  # the router's near-tie window, in units of u * ||w||max * ||x_t|| (route.cu)
U = 2.0 ** -24


def check_routing(got_ids, got_w, ref_ids, ref_w, x, router_w, E, what=""):
    """Assert the contract; return the mask of tokens whose ids match exactly (their weights
    are checked against the oracle's too).  Prints the count of differing tokens (0 expected)."""
    got_ids = np.asarray(got_ids).astype(np.int64)
    ref_ids = np.asarray(ref_ids).astype(np.int64)
    same = (got_ids == ref_ids).all(axis=1)
    bad = np.nonzero(~same)[0]
    gaps = []
    if bad.size:
        l64 = O.router_logits_f64(np.asarray(x)[bad], router_w, E)
        for r, t in enumerate(bad):
            for j in np.nonzero(got_ids[t] != ref_ids[t])[0]:
                gap = abs(l64[r, got_ids[t, j]] - l64[r, ref_ids[t, j]])
                assert gap < NEAR_TIE, (f"{what}: token {t} slot {j}: expert {got_ids[t, j]} vs oracle "
                                        f"{ref_ids[t, j]}, float64 logit gap {gap:.3e} >= {NEAR_TIE:g}")
                gaps.append(gap)
    print(f"{what}: top-k ids bit-exact on {int(same.sum())} of {len(same)} tokens; "
          f"{len(gaps)} near-tie pick difference(s) under {NEAR_TIE:g}"
          + (f" (max float64 gap {max(gaps):.2e})" if gaps else ""))
    # a softmax weight moves by at most twice the largest logit difference (a few 1e-5 for the
    # fast sums at these sizes; 0 for refined or exact logits)
    np.testing.assert_allclose(np.asarray(got_w)[same], np.asarray(ref_w)[same], rtol=1e-4, atol=1e-7)
    return same


def logit_units(x, router_w):
    """Per-token unit of the router's near-tie window: u * max_e ||w_e|| * ||x_t||."""
    wmax = float(np.sqrt((np.asarray(router_w, dtype=np.float64) ** 2).sum(axis=1)).max())
    xn = np.sqrt((np.asarray(x, dtype=np.float64) ** 2).sum(axis=1))
    return U * wmax * xn


def check_logit_margin(got, seq, x, router_w, what=""):
    """Fast-router logits against the sequential f32 sums, in window units: the refinement
    needs every distance below REFINE_UNITS / 2; the bar here is a third of the window, so the
    router keeps half as much again in hand.  Returns the largest distance in units."""
    unit = logit_units(x, router_w)[:, None]
    d = np.abs(np.asarray(got, dtype=np.float64) - np.asarray(seq, dtype=np.float64)) / unit
    m = float(d.max())
    print(f"{what}: max |fast - sequential| logit = {m:.2f} units of u*||w||*||x|| "
          f"(window {REFINE_UNITS:g}; bar {REFINE_UNITS / 3:.1f})")
    assert m <= REFINE_UNITS / 3, f"{what}: fast logits {m:.2f} units from the sequential sums"
    return m
