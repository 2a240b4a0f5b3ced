"""MoE-layer throughput on B200: tokens/s of rusty-engine's moe_layer_forward hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c1|c3b1|c3b8|c3b32|c3b64|c5]
                    [--impl ours|reference] [--no-cpu-baseline] [--no-sub]

One step = one forward of the whole MoE layer (router, dispatch, gate/up+SwiGLU, down,
combine) over one batch of synthetic tokens already resident in HBM; the timed region is
bracketed by a barrier + synchronize, each step by CUDA events on the forward's stream, and
L2 is flushed between steps outside the events (a 256 MiB write).  ``e2e`` is the same metric
through the public host-buffer entry point (pinned host x in, host out, copies inside).

N = 1 (no torchrun): the headline is config 2 (4096-token prefill); the same line carries
``sub`` results for config 3 (decode batches 1, 8, 32, 64) and config 5 (the 235B-shaped layer,
8192 tokens, Zipf(1.1) expert load), each with its roofline fraction.
Launched by torchrun (the scaling run) at N = 1: config 5 on one GPU (the plain layer), the
base of the scaling curve.
N > 1 (torchrun, one rank per GPU): config 5 as an expert-parallel layer, strong scaling: the
8192 tokens are split evenly over the ranks (8192 / N each), experts placed by the pick counts
of a separate calibration batch (largest load first to the least-loaded rank), tokens exchanged
with NCCL; value = 8192 / (max over ranks of the step time).

``--impl reference`` times the CPU restatement of rusty-engine's pooled path (oracle/, all host
threads) on the same config: the whole 4096-token batch per step for config 2.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

C5_TOKENS = 8192

CONFIGS = {
    # name: (builder, tokens, workload label)
    "c1": ("config_c1", 128, "c1 moe_layer_forward H1024 E16 k4 I512 Q4_0, 128 tokens"),
    "c2": ("config_c2", 4096, "c2 Qwen3-30B-A3B MoE layer prefill H2048 E128 k8 I768 Q4_K/Q6_K, 4096 tokens"),
    "c3b1": ("config_c2", 1, "c3 Qwen3-30B-A3B MoE layer decode batch 1"),
    "c3b8": ("config_c2", 8, "c3 Qwen3-30B-A3B MoE layer decode batch 8"),
    "c3b32": ("config_c2", 32, "c3 Qwen3-30B-A3B MoE layer decode batch 32"),
    "c3b64": ("config_c2", 64, "c3 Qwen3-30B-A3B MoE layer decode batch 64"),
    "c5": ("config_c5", C5_TOKENS, "c5 Qwen3-235B-A22B MoE layer H4096 E128 k8 I1536 Q4_K/Q6_K, 8192 tokens, "
                                   "Zipf(1.1) expert load"),
    "c4": (None, 2048, "c4 random-init 48-layer Qwen3-30B-A3B-shaped stack (GQA 32/4, head_dim 128, RMSNorm, "
                       "RoPE 1e6, vocab 151936, Q4_K_M mix), 2048-token prompt, MoE layers timed"),
}
# reference-arm tokens per step: the whole batch, except config 5 (about 20 s of CPU per pass)
REF_SAMPLE = {"c5": 1024}


def kernels_per_forward(lw, T, world=1, rows_local=None):
    """Kernels of this library one forward launches.  Whole layer: routing (one kernel up to 64
    tokens; else logits, top-k, count scan, row scatter), gate/up (+SwiGLU), down (+atomic
    weighted combine); the tensor-core path (T*k >= 32*E) adds the expert-sorted x gather and
    the h rescale.  Expert-parallel: logits + top-k (one kernel up to 64 tokens), plan, pack,
    unpack, the local layer over the received rows (given routing: top-k-free dispatch, one
    kernel up to 64 rows, else count, scan, scatter) and the combine."""
    def experts(rows, E):
        return (2 if rows * lw.k >= 32 * E else 0) + 2
    if world == 1:
        return (1 if T <= 64 else 4) + experts(T, lw.E)
    router = 1 if T <= 64 else 2
    return router + 3 + (1 if rows_local <= 64 else 3) + experts(rows_local, lw.E // world) + 1


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the dominant kernels,
# from one ncu --set full capture each of the same bench command on a B200
NCU_TRAFFIC = {
    ("c2", "gateup"): 386.080e6 + 42.816e6,
    ("c2", "down"): 268.007e6 + 30.732e6,
    ("c3b64", "gateup"): 246.296e6 + 4.087e6,
    ("c3b64", "down"): 164.055e6 + 3.826e6,
    ("c3b1", "gateup"): 15.762e6,
    ("c3b1", "down"): 10.372e6,
}
STAGES = ["route_dispatch", "gateup", "down", "combine"]


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU, read through NVML every 2 ms while
    the timed region runs (read-only queries; nothing is set).  The GPU is found by UUID so the
    NVML index need not match the CUDA index."""

    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, cuda_index: int):
        self.h, self.samples, self.reasons, self.err = None, [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml as N
            import torch

            N.nvmlInit()
            self.N = N
            uuid = str(torch.cuda.get_device_properties(cuda_index).uuid)
            try:
                self.h = N.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                pr = torch.cuda.get_device_properties(cuda_index)
                self.h = N.nvmlDeviceGetHandleByPciBusId(
                    f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0")
            self.smax = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: reported, not fatal
            self.err = f"nvml unavailable: {type(e).__name__}"

    def _sample(self):
        N = self.N
        self.samples.append(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM))
        r = N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        for name, bit in self.REASONS.items():
            if r & bit:
                self.reasons.add(name)

    def _loop(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                pass
            time.sleep(0.002)

    def start(self):
        if self.h is None:
            return
        self._sample()
        self.t = threading.Thread(target=self._loop, daemon=True)
        self.t.start()

    def stop(self):
        if self.h is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "nvml unavailable"]}
        self._stop.set()
        self.t.join(timeout=1)
        self._sample()
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.smax,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "src": "nvml, 2 ms poll"}


def workload(cfg_name):
    """(layer weights, the config's whole token batch) -- seeded synthetic data of the shapes
    and distributions the config names."""
    from rusty_engine_b200 import synth

    builder, T, label = CONFIGS[cfg_name]
    lw = getattr(synth, builder)()
    if cfg_name == "c5":
        lw, x = synth.zipf_workload(lw, T, seed=1)
    else:
        x = synth.activations(T, lw.H, seed=1)
    return lw, x, label


def host_expert_rows(lw, x):
    """Rows per expert of a batch (its top-k picks, routed on the host in float64)."""
    logits = x.astype(np.float64) @ np.asarray(lw.router_w, dtype=np.float64).reshape(lw.E, lw.H).T
    ids = np.argpartition(-logits, lw.k - 1, axis=1)[:, :lw.k]
    return np.bincount(ids.ravel(), minlength=lw.E)


def ep_placement(lw, world, T_cal=2048):
    """Expert placement for the expert-parallel step: the per-expert pick counts of a separate
    calibration batch of the config's distribution (another seed; routed on the host in
    float64), spread over the ranks largest-first (ep_balanced_placement).  The same on every
    rank, with no exchange."""
    from rusty_engine_b200 import synth
    from rusty_engine_b200.moe import ep_balanced_placement

    x = synth.activations(T_cal, lw.H, seed=7) + np.float32(1.0)  # zipf_workload's activations
    return ep_balanced_placement(host_expert_rows(lw, x), world)


def cpu_baseline(cfg_name, lw, x, budget_s=15.0):
    """The oracle's pooled restatement of rusty-engine's CPU path on all host threads."""
    from oracle import oracle as O

    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    O.pool_init(threads)
    T = x.shape[0]
    probe = min(T, 256)
    t0 = time.perf_counter()
    O.moe_layer_pooled(x[:probe], lw)
    dt = time.perf_counter() - t0
    n = probe
    if T > probe and dt * T / probe < budget_s:
        t0 = time.perf_counter()
        O.moe_layer_pooled(x, lw)
        dt, n = time.perf_counter() - t0, T
    return {"value": n / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} of {T} tokens of the {cfg_name} layer, one pooled pass ({dt:.2f} s)"}


def algorithmic(lw, T, ids=None):
    """FLOPs of the expert products and the bytes a layer must read (weights of distinct
    experts touched + router + activations in/out)."""
    from rusty_engine_b200.synth import row_bytes

    H, I, E, k = lw.H, lw.I, lw.E, lw.k
    flops_gateup = 4.0 * T * k * H * I
    flops_down = 2.0 * T * k * H * I
    per_expert = 2 * I * row_bytes(lw.gate_exps.ggml_type, H) + H * row_bytes(lw.down_exps.ggml_type, I)
    touched = E if ids is None else len(np.unique(ids))
    bytes_total = touched * per_expert + E * H * 4 + 2 * T * H * 4
    gu_bytes = touched * 2 * I * row_bytes(lw.gate_exps.ggml_type, H)
    return flops_gateup, flops_down, bytes_total, gu_bytes, touched


def arm_config(args, world):
    """The workload of this run: config 5 (the expert-parallel layer of the scaling curve) at
    every N launched by torchrun, including N = 1, where it is the plain one-GPU layer, the base
    of that curve; the --config choice (config 2, the headline, by default) otherwise."""
    return "c5" if world > 1 or "TORCHELASTIC_RUN_ID" in os.environ else args.config


def reference_arm(args, rank, world):
    """rusty-engine's pooled CPU path (C restatement, all host threads) on our arm's config:
    rank 0 only; the whole batch per step (config 5: a 1024-token sample)."""
    if rank != 0:
        return
    from oracle import oracle as O

    cfg = arm_config(args, world)
    if cfg == "c4":
        # per-layer work of the stack: one MoE layer of its shape over the 2048-token prompt
        from rusty_engine_b200 import synth

        lw = synth.config_c2(seed=100)
        x = synth.activations(CONFIGS["c4"][1], lw.H, seed=1)
        label = CONFIGS["c4"][2] + " (CPU: one MoE layer of the stack's shape per step)"
    else:
        lw, x, label = workload(cfg)
    T = x.shape[0]
    sample = min(T, REF_SAMPLE.get(cfg, T))
    xs = np.ascontiguousarray(x[:sample])
    threads = len(os.sched_getaffinity(0))
    O.pool_init(threads)
    for _ in range(args.warmup):
        O.moe_layer_pooled(xs, lw)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.moe_layer_pooled(xs, lw)
        times.append(time.perf_counter() - t0)
    ms = statistics.mean(times) * 1e3
    val = sample / (ms / 1e3)
    what = "all" if sample == T else f"a {sample}-token sample of the"
    print(json.dumps({
        "impl": "reference", "metric": "moe_layer_tokens_per_s", "value": val, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "min_ms_per_step": min(times) * 1e3,
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": label, "tokens": T, "sample_tokens": sample},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{what} {T} tokens per step (C restatement of the pooled AVX2 path)"},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


class Bench:
    """Timing helpers on one rank's GPU."""

    def __init__(self, torch, dist):
        self.torch, self.dist = torch, dist
        self.flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
        self.stream = torch.cuda.current_stream()

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, v):
        if self.dist is None:
            return v
        t = self.torch.tensor([v], device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def steps(self, layer, x, out, steps, warmup, sampler=None):
        """Mean ms of `steps` forwards (CUDA events on the stream, L2 flushed in between)."""
        torch = self.torch
        for _ in range(warmup):
            layer.forward(x, out)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        self.barrier()
        if sampler:
            sampler.start()
        for i in range(steps):
            self.flush.fill_(float(i))
            starts[i].record(self.stream)
            layer.forward(x, out)
            ends[i].record(self.stream)
        self.barrier()
        clocks = sampler.stop() if sampler else None
        ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
        return ms, clocks

    def stages(self, layer, x, out, n):
        """Per-stage ms from separate forwards (the events between stages serialise kernels
        that otherwise overlap their launch through programmatic dependent launch)."""
        from rusty_engine_b200 import _lib

        stage = np.zeros(4)
        for i in range(n):
            self.flush.fill_(float(i))
            layer.forward(x, out, flags=_lib.FLAG_STAGE_TIMING)
            stage += np.array(layer.stage_ms())
        return stage / n

    def e2e(self, layer, x_np, n):
        """Mean s of `n` host-buffer forwards (pinned x in, host out, copies inside the call)."""
        import ctypes as C

        from rusty_engine_b200 import _lib

        torch = self.torch
        xh = torch.from_numpy(x_np).pin_memory()
        oh = torch.empty_like(xh).pin_memory()
        L = _lib.load()
        sptr = C.c_void_p(self.stream.cuda_stream)
        T = x_np.shape[0]
        for _ in range(2):
            _lib.check(L.rmoe_layer_forward(layer._h, xh.data_ptr(), T, oh.data_ptr(), sptr, _lib.FLAG_HOST_IO))
        self.barrier()
        times = []
        for _ in range(n):
            self.flush.fill_(0.0)
            torch.cuda.synchronize()
            s0 = time.perf_counter()
            _lib.check(L.rmoe_layer_forward(layer._h, xh.data_ptr(), T, oh.data_ptr(), sptr, _lib.FLAG_HOST_IO))
            times.append(time.perf_counter() - s0)
        return statistics.mean(times)


def roofline_single(lw, T, ids, stage, peaks, cfg):
    """Roofline of the dominant kernel (by stage time): tensor FLOPs for prefill (T >= 256),
    HBM bytes for decode."""
    fg, fd, nbytes, gu_bytes, touched = algorithmic(lw, T, ids)
    dom = int(np.argmax(stage))
    if T >= 256:
        work = {1: fg, 2: fd}.get(dom, fg)
        ach = work / (stage[dom] / 1e3) / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": ach / peaks["bf16_tflops"], "traffic": NCU_TRAFFIC.get((cfg, STAGES[dom])),
                "traffic_unit": "bytes per launch (ncu)", "kernel": STAGES[dom],
                "peak_src": peaks["src"] + " burst bf16"}, touched
    gb = (gu_bytes if dom == 1 else nbytes - gu_bytes) / (stage[dom] / 1e3) / 1e9
    return {"bound": "hbm", "achieved": gb, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": gb / peaks["hbm_gbs"], "traffic": NCU_TRAFFIC.get((cfg, STAGES[dom])),
            "traffic_unit": "bytes per launch (ncu)", "kernel": STAGES[dom],
            "peak_src": peaks["src"] + " copy"}, touched


def sub_result(B, lw, x_np, cfg, steps, warmup, peaks):
    """One config's numbers on this GPU (N = 1 line's ``sub``)."""
    from rusty_engine_b200 import _lib
    from rusty_engine_b200.moe import MoELayer

    torch = B.torch
    T = x_np.shape[0]
    layer = MoELayer(lw, device=torch.cuda.current_device())
    x = torch.from_numpy(x_np).cuda()
    out = torch.empty_like(x)
    ms, _ = B.steps(layer, x, out, steps, warmup)
    layer.forward(x, out, flags=_lib.FLAG_ROUTING_OUT)
    torch.cuda.synchronize()
    ids, _ = layer.routing(T)
    stage = B.stages(layer, x, out, max(3, min(steps, 10)))
    roof, touched = roofline_single(lw, T, ids, stage, peaks, cfg)
    layer.close()
    fg, fd, nbytes, _, _ = algorithmic(lw, T, ids)
    res = {"workload": CONFIGS[cfg][2], "tokens": T, "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3),
           "experts_touched": int(touched), "stage_ms": {n: float(v) for n, v in zip(STAGES, stage)},
           "roofline": roof, "steps": steps, "warmup": warmup}
    if T >= 256:
        res["layer_tensor_frac"] = (fg + fd) / (ms / 1e3) / 1e12 / peaks["bf16_tflops"]
    else:
        res["layer_hbm_frac"] = nbytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]
    return res


def bench_c4(args):
    """Config 4: a 48-block stack (rusty_engine_b200.stack) over a 2048-token prompt of uniform
    random ids; one step = one whole forward; only the MoE layers are timed (CUDA events around
    each of the 48 MoE forwards, summed).  Layers are built and uploaded one at a time."""
    import torch

    from rusty_engine_b200 import synth
    from rusty_engine_b200.stack import QWEN3_30B_A3B, QWEN3_30B_A3B_LAYERS, MoEStack, make_block

    g = QWEN3_30B_A3B
    T = CONFIGS["c4"][1]
    torch.cuda.set_device(0)
    base = synth.config_c2(seed=100)
    stack = MoEStack(g, [make_block(g, 0, base_moe=base)], device=0)
    for i in range(1, QWEN3_30B_A3B_LAYERS):
        stack.add_layer(make_block(g, i, base_moe=base))
    gen = torch.Generator(device="cuda").manual_seed(0)
    embed = torch.randn((g.vocab, g.d_model), generator=gen, device="cuda", dtype=torch.float32)
    ids = torch.randint(0, g.vocab, (T,), generator=gen, device="cuda")
    x = embed[ids].contiguous()
    del embed
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    for _ in range(args.warmup):
        stack.forward(x)
    moe, whole = [], []
    sampler = ClockSampler(0)
    sampler.start()
    for i in range(args.steps):
        flush.fill_(float(i))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        stack.forward(x)
        e1.record()
        torch.cuda.synchronize()
        moe.append(sum(stack.moe_ms))
        whole.append(e0.elapsed_time(e1))
    clocks = sampler.stop()
    per_layer = [m for m in stack.moe_ms]
    stack.close()
    moe_ms = statistics.mean(moe)
    nl = QWEN3_30B_A3B_LAYERS
    peaks = load_peaks()
    flops = 6.0 * T * g.top_k * g.d_model * g.inter * nl
    print(json.dumps({
        "metric": "moe_layer_tokens_per_s", "value": T * nl / (moe_ms / 1e3), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": moe_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16-mma/f32-acc/f32-router", "data": "synthetic",
        "config": {"workload": CONFIGS["c4"][2], "tokens": T, "layers": nl,
                   "timed": "the 48 MoE layers of each forward (CUDA events around each MoE forward, summed); "
                            "value = tokens x layers / that time",
                   "l2": "flushed between steps (256 MiB write); every layer reads its own expert weights"},
        "moe_ms_per_forward": moe_ms, "moe_ms_per_layer_mean": moe_ms / nl,
        "moe_ms_per_layer_last_step": per_layer, "whole_forward_ms": statistics.mean(whole),
        "roofline": {"bound": "tensor", "achieved": flops / (moe_ms / 1e3) / 1e12, "peak": peaks["bf16_tflops_sustained"],
                     "unit": "TFLOP/s", "frac": flops / (moe_ms / 1e3) / 1e12 / peaks["bf16_tflops_sustained"],
                     "kernel": "all 48 MoE layers of a forward", "peak_src": peaks["src"] + " sustained bf16"},
        "clocks": clocks,
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="N = 1: skip the config 3 / config 5 sub-results")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        reference_arm(args, rank, world)
        return
    if args.config == "c4":
        if args.impl == "ours" and world == 1:
            bench_c4(args)
        return

    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist_mod

        dist = dist_mod
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    from rusty_engine_b200 import _lib
    from rusty_engine_b200.moe import MoELayer

    cfg = arm_config(args, world)
    lw, x_all, label = workload(cfg)
    if world > 1:
        # strong scaling: this rank's share of the config's whole batch
        T_all = x_all.shape[0]
        per = (T_all + world - 1) // world
        x_np = np.ascontiguousarray(x_all[rank * per:min(T_all, (rank + 1) * per)])
        from rusty_engine_b200.moe import ep_unique_id

        box = [ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        placement = ep_placement(lw, world)
        layer = MoELayer.expert_parallel(lw, rank, world, box[0], device=local, placement=placement)
    else:
        T_all = x_all.shape[0]
        x_np = x_all
        layer = MoELayer(lw, device=local)
    T = x_np.shape[0]
    B = Bench(torch, dist)
    x = torch.from_numpy(x_np).cuda()
    out = torch.empty_like(x)
    layer.forward(x, out, flags=_lib.FLAG_ROUTING_OUT)
    torch.cuda.synchronize()
    ids, _ = layer.routing(T)

    sampler = ClockSampler(local)
    layer.router_refined()  # resets the device counter: the timed forwards' count is read below
    ms, clocks = B.steps(layer, x, out, args.steps, args.warmup, sampler)
    refined = layer.router_refined() / float(args.steps + args.warmup)  # near-tie tokens per forward
    stage = B.stages(layer, x, out, max(3, min(args.steps, 10))) if world == 1 else None
    B.barrier()
    ms = B.max_over_ranks(ms)
    e2e_s = B.max_over_ranks(B.e2e(layer, x_np, max(3, min(args.steps, 10))))
    layer.close()

    peaks = load_peaks()
    subs = {}
    if world == 1 and not args.no_sub and cfg == "c2":
        for b in (1, 8, 32, 64):
            subs[f"c3b{b}"] = sub_result(B, lw, x_all[:b].copy(), f"c3b{b}", args.steps, args.warmup, peaks)
        lw5, x5, _ = workload("c5")
        subs["c5"] = sub_result(B, lw5, x5, "c5", args.steps, args.warmup, peaks)
        del lw5, x5

    if rank == 0:
        lwr = lw
        fg, fd, nbytes, gu_bytes, touched = algorithmic(lwr, T_all if world > 1 else T, None if world > 1 else ids)
        value = T_all / (ms / 1e3)
        if world > 1:
            # the whole job: expert products of all 8192 tokens over the step, per GPU
            ach = (fg + fd) / (ms / 1e3) / 1e12 / world
            roof = {"bound": "tensor", "achieved": ach, "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                    "frac": ach / peaks["bf16_tflops_sustained"], "traffic": None,
                    "kernel": "whole expert-parallel step per GPU (router, exchanges, experts, combine)",
                    "peak_src": peaks["src"] + " sustained bf16"}
        else:
            roof, touched = roofline_single(lwr, T, ids, stage, peaks, cfg)
        line = {
            "metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if cfg == "c5" else "weak", "vs_baseline": None,
            "dtype": "fp16-mma/f32-acc/f32-router", "data": "synthetic",
            "config": {"workload": label, "tokens_total": T_all, "tokens_per_gpu": T,
                       "experts_touched": int(touched),
                       "l2": "flushed between steps (256 MiB write outside the events)",
                       "parallelism": f"ep{world}" if world > 1 else "single"},
            **({"placement": "experts placed by the pick counts of a 2048-token calibration batch "
                             "(another seed), largest load first to the least-loaded rank"} if world > 1 else {}),
            "roofline": roof,
            "e2e": {"value": T_all / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": T * lwr.H * 4,
                    "d2h_bytes_per_step": T * lwr.H * 4},
            "gpu_launches": kernels_per_forward(lwr, T, world, T) * args.steps,
            "router_refined_tokens_per_forward": refined,
            "clocks": clocks,
        }
        if stage is not None:
            line["stage_ms"] = {n: float(v) for n, v in zip(STAGES, stage)}
        if world > 1:
            # per-GPU load of the timed batch: expert rows each rank computes (host routing)
            rows = np.bincount(placement, weights=host_expert_rows(lw, x_all), minlength=world)
            line["ep_expert_rows_per_rank"] = [int(r) for r in rows]
            line["ep_busiest_over_mean"] = float(rows.max() / rows.mean())
        if subs:
            line["sub"] = subs
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, lwr, x_np)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
