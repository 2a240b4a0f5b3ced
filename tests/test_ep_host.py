"""Expert-parallel exchange on CPU: two gloo ranks run the host restatement of ep.cu's plan /
pack / local experts / return / combine (tests/ep_sim.py) and must reproduce the whole-layer
oracle on their own tokens (only the f32 summation order over a token's experts differs).
Ragged shards, a rank without tokens and picks that all land on one rank are covered."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from rusty_engine_b200 import synth
from rusty_engine_b200.synth import GGML_Q4_K, GGML_Q6_K, row_bytes

REL = 2e-6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _experts_f32(lw):
    from oracle import oracle as O

    out = []
    for e in range(lw.E):
        def part(qt, rows, K):
            nb = rows * row_bytes(qt.ggml_type, K)
            return O.dequant(qt.ggml_type, qt.data[e * nb:(e + 1) * nb]).reshape(rows, K)
        out.append((part(lw.gate_exps, lw.I, lw.H), part(lw.up_exps, lw.I, lw.H), part(lw.down_exps, lw.H, lw.I)))
    return out


def _rank(rank, world, port, tokens, seed, bias_to, shared=False, placement=None):
    import torch.distributed as dist

    from oracle import oracle as O
    from tests import ep_sim

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        lw = synth.make_layer(256, 256, 8, 3, gate_t=GGML_Q4_K, up_t=GGML_Q4_K, down_t=GGML_Q6_K, dlo=0.001,
                              dhi=0.01, seed=seed, name="ep-sim", shared=shared)
        if bias_to is not None:  # every token's picks on one rank's experts (e % 2 == bias_to)
            lw.router_w[bias_to::2] += np.float32(0.5)
        ex = _experts_f32(lw)
        x = synth.activations(tokens[rank], lw.H, seed=100 + rank) if tokens[rank] else np.zeros((0, lw.H), np.float32)
        sh = None
        if shared:
            sh = tuple(O.dequant(q.ggml_type, q.data).reshape(r, c)
                       for q, r, c in zip(lw.shared, (lw.I, lw.I, lw.H), (lw.H, lw.H, lw.I)))
        got = ep_sim.ep_forward(x, lw, ex, rank, world, sh, placement)
        if tokens[rank]:
            want = O.moe_layer_q_exact(x, lw)[0]
            rel = np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want)
            assert rel <= REL, f"rank {rank}: rel-L2 {rel:.3e}"
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens,bias_to", [((5, 3), None), ((4, 0), None), ((3, 6), 1)])
def test_ep_exchange_matches_whole_layer(tokens, bias_to):
    mp.start_processes(_rank, args=(2, _free_port(), tokens, 7, bias_to), nprocs=2, start_method="spawn", join=True)


@pytest.mark.parametrize("tokens", [(5, 3), (4, 0)])
def test_ep_exchange_with_shared_expert(tokens):
    """The shared expert replicated on both ranks: every token is also sent to its own rank,
    which adds the shared expert's output to that row's partial sum (src/moe.rs:381-386)."""
    mp.start_processes(_rank, args=(2, _free_port(), tokens, 9, None, True), nprocs=2, start_method="spawn",
                       join=True)


@pytest.mark.parametrize("placement", [[1, 1, 1, 1, 1, 1, 1, 0], [0, 0, 1, 0, 1, 1, 0, 1]])
def test_ep_exchange_with_placement(placement):
    """A caller-given expert placement (rmoe_ep_layer_create_placed): uneven expert counts per
    rank, local ids in ascending global order, the empty id = the destination's expert count."""
    mp.start_processes(_rank, args=(2, _free_port(), (5, 4), 11, None, False, placement), nprocs=2,
                       start_method="spawn", join=True)


def test_balanced_placement_spreads_load():
    """ep_balanced_placement: largest-first fill to the least-loaded rank; every rank holds an
    expert even when most loads are zero; the busiest rank stays near the mean on a Zipf load."""
    from rusty_engine_b200.moe import EngineError, ep_balanced_placement

    p = ep_balanced_placement([0, 0, 0, 0, 0, 9, 0, 0], 4)
    assert sorted(set(p.tolist())) == [0, 1, 2, 3] and p[5] == 0
    load = 1.0 / np.arange(1, 129) ** 1.1
    for G in (2, 4, 8):
        p = ep_balanced_placement(load, G)
        per = np.bincount(p, weights=load, minlength=G)
        rr = np.array([load[r::G].sum() for r in range(G)])
        assert per.max() <= rr.max() + 1e-12
        assert per.max() <= max(per.mean() * 1.02, load.max())
    with pytest.raises(EngineError):
        ep_balanced_placement([1.0, 2.0], 4)


def test_bench_expert_placement_on_a_zipf_layer():
    """The expert-parallel bench's placement (bench.ep_placement: pick counts of a calibration
    batch of another seed, routed on the host, spread largest-first) gives every rank an expert
    and keeps the busiest rank of the timed batch no busier than the round-robin deal does."""
    import bench

    lw0 = synth.make_layer(256, 256, 16, 4, gate_t=GGML_Q4_K, up_t=GGML_Q4_K, down_t=GGML_Q6_K, dlo=0.001,
                           dhi=0.01, seed=3, name="zipf-small")
    lw, x = synth.zipf_workload(lw0, 1024, seed=1)
    rows_e = bench.host_expert_rows(lw, x)
    assert rows_e.sum() == 1024 * lw.k
    for G in (2, 4):
        pl = bench.ep_placement(lw, G, T_cal=1024)
        assert pl.shape == (lw.E,) and sorted(set(pl.tolist())) == list(range(G))
        busiest = np.bincount(pl, weights=rows_e, minlength=G).max()
        rr = np.bincount(np.arange(lw.E) % G, weights=rows_e, minlength=G).max()
        assert busiest <= rr, (G, busiest, rr)
