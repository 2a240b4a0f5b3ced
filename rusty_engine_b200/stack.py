"""MoE transformer stack around the layer: the BASELINE config-4 harness.

rusty-engine has no batched MoE prefill block (its moe_block_forward, src/moe.rs:443-469, is a
one-token decode step over the KV cache); this module composes the prefill block the same way
block_forward_prefill_cached does (src/forward.rs:532-571) with the dense SwiGLU FFN replaced by
the MoE layer, as moe_block_forward does for one token:

    x_norm = rmsnorm(x, attn_norm)                                   (src/infer.rs:72-81)
    q, k, v = QMat products of x_norm (+ biases)                     (src/forward.rs:548-553)
    RoPE, NeoX rotate-half, angle = pos * base^(-2i/d)               (src/infer.rs:90-145)
    ctx = causal GQA attention, scores * 1/sqrt(head_dim), softmax   (src/forward.rs:218-283)
    y = x + o(ctx)                                                   (src/forward.rs:557-558)
    out = y + moe_layer_forward(rmsnorm(y, ffn_norm))                (src/moe.rs:462-468)

Only the MoE layers are this library's hot path and only they are timed (CUDA events around
each MoE forward).  The rest runs on the GPU as plumbing: the q/k/v/o projections on this
library's resident QMat products, norms, RoPE and the attention core as torch f32 operations.
Weights are random (seeded); the expert stacks of the layers are generated quickly as
variants of one base stack (the quant bytes xor-ed with a per-layer random mask, the block
scales kept), so every layer reads its own 392 MB of expert weights.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import numpy as np

from . import synth

try:
    import torch
except Exception:  # pragma: no cover - torch is part of the image
    torch = None


@dataclass
class Geometry:
    """src/forward.rs:17-27 Geometry, with the MoE shape of the block."""

    d_model: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    n_experts: int
    top_k: int
    inter: int
    rope_freq_base: float = 1e6
    rms_eps: float = 1e-6
    vocab: int = 151936


# Qwen3-30B-A3B: 48 layers, GQA 32 q / 4 kv heads of 128, 128 experts top-8 of width 768
QWEN3_30B_A3B = Geometry(d_model=2048, n_heads=32, n_kv_heads=4, head_dim=128, n_experts=128, top_k=8, inter=768)
QWEN3_30B_A3B_LAYERS = 48


@dataclass
class BlockWeights:
    """One MoE block (src/forward.rs:58-78 BlockWeights with the FFN replaced by the MoE layer)."""

    attn_norm: np.ndarray
    q: synth.QTensor
    k: synth.QTensor
    v: synth.QTensor
    o: synth.QTensor
    ffn_norm: np.ndarray
    moe: synth.LayerWeights


def _qt(rng, t, rows, cols, dlo, dhi):
    nb = rows * cols // synth.BLOCK[t][0]
    data = synth.gen_q4k_centered(rng, nb, dlo, dhi) if t == synth.GGML_Q4_K else synth.gen_blocks(rng, t, nb, dlo, dhi)
    return synth.QTensor(t, data, (cols, rows))


def _variant(base: synth.QTensor, rng) -> synth.QTensor:
    """Another tensor of the same type and scales: quant bytes xor-ed with random bytes (the
    fp16 scale fields and Q4_K / Q6_K sub-scales kept), so it decodes to other weights of the
    same distribution."""
    t = base.ggml_type
    el, by = synth.BLOCK[t]
    blk = base.data.reshape(-1, by)
    mask = np.frombuffer(rng.bytes(blk.size), dtype=np.uint8).reshape(blk.shape).copy()
    if t in (synth.GGML_Q4_K, synth.GGML_Q5_K):
        mask[:, 0:16] = 0
    elif t == synth.GGML_Q6_K:
        mask[:, 192:210] = 0
    elif t in (synth.GGML_Q4_0, synth.GGML_Q5_0, synth.GGML_Q8_0):
        mask[:, 0:2] = 0
    else:
        raise ValueError("variant: quantized types only")
    return synth.QTensor(t, (blk ^ mask).reshape(-1), base.dims)


def make_block(g: Geometry, seed: int, base_moe: Optional[synth.LayerWeights] = None,
               dlo: float = 0.001, dhi: float = 0.01, attn_dlo: float = 0.0002, attn_dhi: float = 0.001,
               attn_types=(synth.GGML_Q4_K, synth.GGML_Q4_K, synth.GGML_Q6_K, synth.GGML_Q4_K)) -> BlockWeights:
    """Random block in the Q4_K_M mix: q / k / o Q4_K, v Q6_K (zero-mean draws with small
    scales, so attention scores stay O(1)), experts as config 2 (Q4_K gate/up and Q6_K down,
    scales U(dlo, dhi)); norms around 1; router N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    qd, kvd = g.n_heads * g.head_dim, g.n_kv_heads * g.head_dim
    tq, tk, tv, to = attn_types
    q = _qt(rng, tq, qd, g.d_model, attn_dlo, attn_dhi)
    k = _qt(rng, tk, kvd, g.d_model, attn_dlo, attn_dhi)
    v = _qt(rng, tv, kvd, g.d_model, attn_dlo, attn_dhi)
    o = _qt(rng, to, g.d_model, qd, attn_dlo, attn_dhi)
    norm = lambda: (1.0 + 0.1 * rng.standard_normal(g.d_model)).astype(np.float32)
    attn_norm, ffn_norm = norm(), norm()
    if base_moe is None:
        moe = synth.make_layer(g.d_model, g.inter, g.n_experts, g.top_k, gate_t=synth.GGML_Q4_K,
                               up_t=synth.GGML_Q4_K, down_t=synth.GGML_Q6_K, dlo=dlo, dhi=dhi, seed=seed + 1)
    else:
        router = (rng.standard_normal((g.n_experts, g.d_model), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        moe = synth.LayerWeights(g.d_model, g.inter, g.n_experts, g.top_k, 0, router,
                                 _variant(base_moe.gate_exps, rng), _variant(base_moe.up_exps, rng),
                                 _variant(base_moe.down_exps, rng), name=f"stack-layer-{seed}")
    return BlockWeights(attn_norm, q, k, v, o, ffn_norm, moe)


def rope_tables(g: Geometry, seq: int, pos_start: int = 0):
    """(cos, sin) of angle = pos * base^(-2i/d) for every position and pair, in f32 as
    rope_table computes them (src/infer.rs:90-96, 115-127)."""
    d = g.head_dim
    i = np.arange(d // 2, dtype=np.float32)
    freqs = (np.float32(1.0) / np.power(np.float32(g.rope_freq_base), (2 * i) / np.float32(d))).astype(np.float32)
    pos = np.arange(pos_start, pos_start + seq, dtype=np.float32)
    ang = (pos[:, None] * freqs[None, :]).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


class MoEStack:
    """A resident stack of MoE blocks on one GPU.  forward(x) runs every block over a prompt
    and returns the hidden states; moe_ms holds the CUDA-event time of each MoE layer."""

    def __init__(self, g: Geometry, blocks: List[BlockWeights], device: Optional[int] = None):
        from .moe import MoELayer, QMat

        self.g = g
        self.device = torch.cuda.current_device() if device is None else device
        dev = torch.device("cuda", self.device)
        self.layers = []
        for b in blocks:
            L = {
                "attn_norm": torch.from_numpy(b.attn_norm).to(dev),
                "ffn_norm": torch.from_numpy(b.ffn_norm).to(dev),
                "q": QMat(b.q.ggml_type, b.q.data, g.n_heads * g.head_dim, g.d_model),
                "k": QMat(b.k.ggml_type, b.k.data, g.n_kv_heads * g.head_dim, g.d_model),
                "v": QMat(b.v.ggml_type, b.v.data, g.n_kv_heads * g.head_dim, g.d_model),
                "o": QMat(b.o.ggml_type, b.o.data, g.d_model, g.n_heads * g.head_dim),
                "moe": MoELayer(b.moe, device=self.device),
            }
            for n in ("q", "k", "v", "o"):
                L[n]._handle()  # upload now
            self.layers.append(L)
        self.moe_ms: List[float] = []

    def add_layer(self, b: BlockWeights):
        self.layers.extend(MoEStack(self.g, [b], self.device).layers)

    def _rmsnorm(self, x, w):
        # x * (1 / sqrt(mean(x^2) + eps)) * w, per row (src/infer.rs:72-81)
        ms = (x * x).sum(dim=1, keepdim=True) / x.shape[1]
        return x * (1.0 / torch.sqrt(ms + self.g.rms_eps)) * w

    def _rope(self, t, heads, cos, sin):
        # NeoX rotate-half per head: (x0, x1) -> (x0 c - x1 s, x1 c + x0 s)  (src/infer.rs:131-139)
        T, hd = t.shape[0], self.g.head_dim
        h = t.view(T, heads, hd)
        x0, x1 = h[..., : hd // 2], h[..., hd // 2:]
        c, s = cos[:, None, :], sin[:, None, :]
        return torch.cat((x0 * c - x1 * s, x1 * c + x0 * s), dim=-1).reshape(T, heads * hd)

    def _attention(self, q, k, v):
        # causal GQA attention, scores * 1/sqrt(hd), softmax over 0..=i (src/forward.rs:218-283)
        g = self.g
        T = q.shape[0]
        rep = g.n_heads // g.n_kv_heads
        qh = q.view(T, g.n_heads, g.head_dim).transpose(0, 1)
        kh = k.view(T, g.n_kv_heads, g.head_dim).transpose(0, 1).repeat_interleave(rep, dim=0)
        vh = v.view(T, g.n_kv_heads, g.head_dim).transpose(0, 1).repeat_interleave(rep, dim=0)
        scores = torch.matmul(qh, kh.transpose(1, 2)) * (1.0 / math.sqrt(g.head_dim))
        mask = torch.ones(T, T, dtype=torch.bool, device=q.device).triu(1)
        scores = scores.masked_fill(mask, float("-inf"))
        p = torch.softmax(scores, dim=-1)
        return torch.matmul(p, vh).transpose(0, 1).reshape(T, g.n_heads * g.head_dim)

    def forward(self, x, pos_start: int = 0, time_moe: bool = True, collect: bool = False):
        """x: [T, d_model] f32 cuda tensor -> [T, d_model]; self.moe_ms gets the MoE layers'
        times (ms, CUDA events on the current stream).  collect: also keep every block's input
        in self.block_inputs and every block's attention residual (before the MoE FFN) in
        self.block_mids (for per-part checks)."""
        g = self.g
        T = x.shape[0]
        cos, sin = (torch.from_numpy(a).to(x.device) for a in rope_tables(g, T, pos_start))
        stream = torch.cuda.current_stream()
        events = []
        self.block_inputs, self.block_mids = [], []
        for L in self.layers:
            if collect:
                self.block_inputs.append(x.clone())
            xn = self._rmsnorm(x, L["attn_norm"])
            q = L["q"].matmul_device(xn)
            k = L["k"].matmul_device(xn)
            v = L["v"].matmul_device(xn)
            q = self._rope(q, g.n_heads, cos, sin)
            k = self._rope(k, g.n_kv_heads, cos, sin)
            ctx = self._attention(q, k, v).contiguous()
            y = x + L["o"].matmul_device(ctx)
            if collect:
                self.block_mids.append(y.clone())
            yn = self._rmsnorm(y, L["ffn_norm"]).contiguous()
            if time_moe:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            m = L["moe"].forward(yn)
            if time_moe:
                e1.record(stream)
                events.append((e0, e1))
            x = y + m
        if time_moe:
            torch.cuda.synchronize()
            self.moe_ms = [a.elapsed_time(b) for a, b in events]
        return x

    def close(self):
        for L in self.layers:
            L["moe"].close()
        self.layers = []
