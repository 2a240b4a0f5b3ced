"""Expert-parallel layer over NCCL on two GPUs: each rank's outputs for its own tokens match the
oracle's whole layer (routing ids bit-exact up to sub-1e-6 near-ties) within the layer
tolerance (relative L2 <= 5e-3; max-abs <= 2e-2 x max(1, RMS)), on the small-batch and the
tensor-core local paths.  Skipped where fewer than two GPUs are visible."""
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from rusty_engine_b200 import synth

pytestmark = pytest.mark.gpu

def _check(got, want, what):
    from oracle import oracle as O

    rel, mx, rms = O.layer_errors(got, want)
    assert rel <= O.REL_L2, f"{what}: rel-L2 {rel:.3e}"
    assert mx <= O.max_abs_bound(rms), f"{what}: max-abs {mx:.3e} (rms {rms:.3e})"


def _rank(rank, world, uid, tokens, shared=False, placement=None):
    import torch

    from oracle import oracle as O
    from routing_check import check_routing
    from rusty_engine_b200.moe import MoELayer

    torch.cuda.set_device(rank)
    lw = synth.config_c1() if not shared else synth.make_layer(
        1024, 512, 16, 4, gate_t=12, up_t=12, down_t=14, dlo=0.001, dhi=0.004, seed=3, shared=True)
    layer = MoELayer.expert_parallel(lw, rank, world, uid, device=rank, placement=placement)
    for T in tokens:
        x = synth.activations(T, lw.H, seed=10 * rank + T)
        out = layer.forward(torch.from_numpy(x).cuda())
        torch.cuda.synchronize()
        want, ids, w, _ = O.moe_layer_q_exact(x, lw)
        got_ids, got_w = layer.routing(T)
        same = check_routing(got_ids, got_w, ids, w, x, lw.router_w, lw.E, f"rank {rank} T {T}")
        _check(out.cpu().numpy()[same], want[same], f"rank {rank} T {T}")
    layer.close()


def _run(world, tokens, timeout_s=300, shared=False, placement=None):
    from rusty_engine_b200.moe import ep_unique_id

    uid = ep_unique_id()
    ctx = mp.start_processes(_rank, args=(world, uid, tokens, shared, placement), nprocs=world, start_method="spawn",
                             join=False)
    deadline = time.time() + timeout_s
    while not ctx.join(timeout=5):
        if time.time() > deadline:
            for p in ctx.processes:
                if p.is_alive():
                    p.kill()
            pytest.fail(f"expert-parallel ranks did not finish in {timeout_s} s")


def test_ep_two_gpus_matches_oracle(gpu):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    # 3 and 16 tokens: small-batch local path; 512: tensor-core local path
    _run(2, (3, 16, 512))


def test_ep_two_gpus_shared_expert(gpu):
    """A layer with a shared expert (replicated on both ranks, applied by each rank to its own
    tokens) against the oracle's whole layer, small-batch and tensor-core local paths."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run(2, (5, 300), shared=True)


def test_ep_two_gpus_placed(gpu):
    """A caller-given placement (rmoe_ep_layer_create_placed): rank 0 holds 3 of the 16
    experts, rank 1 the other 13, on the small-batch and the tensor-core local paths."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    placement = [1] * 16
    for e in (2, 7, 11):
        placement[e] = 0
    _run(2, (6, 512), placement=placement)


def _create_alone(q):
    """Rank 0 of a two-rank layer whose other rank never calls in (child process)."""
    import os
    import time

    os.environ["RMOE_EP_TIMEOUT_MS"] = "3000"
    from rusty_engine_b200.moe import MoELayer, ep_unique_id

    t0 = time.time()
    try:
        MoELayer.expert_parallel(synth.config_c1(), 0, 2, ep_unique_id(), device=0)
        q.put((0, "created", time.time() - t0))
    except Exception as e:  # RmoeError: "rmoe NCCL: <message>"
        q.put((-1, f"{type(e).__name__}: {e}", time.time() - t0))


def test_ep_create_times_out_when_a_rank_never_joins(gpu):
    """Failure made on the host: rank 0 of a two-rank expert-parallel layer is created while
    rank 1 never calls in.  The non-blocking NCCL communicator init gives up after
    RMOE_EP_TIMEOUT_MS (3 s here), aborts, and the create fails with RMOE_ERR_NCCL instead of
    blocking for good.  Runs in a child process, itself bounded by a timeout."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_create_alone, args=(q,))
    p.start()
    p.join(120)
    if p.is_alive():
        p.kill()
        pytest.fail("the create did not return within 120 s")
    code, msg, dt = q.get(timeout=10)
    assert code != 0, msg
    assert "NCCL" in msg and "no progress" in msg, msg
    assert dt < 60, dt


def _leave_rank(rank, world, uid, q, left):
    """Both ranks run one forward; then rank 1 closes its layer and leaves (between steps,
    nothing in flight) while rank 0 runs a second forward, which must fail within the
    communicator timeout instead of waiting for good."""
    import os
    import time

    os.environ["RMOE_EP_TIMEOUT_MS"] = "5000"
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    from rusty_engine_b200.moe import MoELayer

    torch.cuda.set_device(rank)
    lw = synth.config_c1()
    layer = MoELayer.expert_parallel(lw, rank, world, uid, device=rank)
    x = torch.from_numpy(synth.activations(8, lw.H, seed=rank)).cuda()
    layer.forward(x)
    torch.cuda.synchronize()
    if rank == 1:
        layer.close()
        left.set()
        return
    left.wait(60)
    t0 = time.time()
    try:
        layer.forward(x)
        torch.cuda.synchronize()
        q.put((0, "forward returned", time.time() - t0))
    except Exception as e:
        q.put((-1, f"{type(e).__name__}: {e}", time.time() - t0))
    layer.close()


def test_ep_peer_leaves_forward_fails_within_timeout(gpu):
    """Failure made on the host, on two GPUs: a rank leaves between steps; the other rank's next
    forward ends with RMOE_ERR_NCCL (an NCCL error, or no progress for RMOE_EP_TIMEOUT_MS, then
    the communicator is aborted) instead of hanging.  NVLS off, as for every such test."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from rusty_engine_b200.moe import ep_unique_id

    ctx = mp.get_context("spawn")
    q, left = ctx.Queue(), ctx.Event()
    uid = ep_unique_id()
    procs = [ctx.Process(target=_leave_rank, args=(r, 2, uid, q, left)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish within 180 s"
    code, msg, dt = q.get(timeout=10)
    assert code != 0 and "NCCL" in msg, msg
    assert dt < 60, dt
