"""TEST INFRASTRUCTURE ONLY: CPU restatement of rusty-engine's prefill block with the MoE FFN,
the checker for ``rusty_engine_b200.stack``.  Only ``tests/`` may import it.

Per block (block_forward_prefill_cached, src/forward.rs:532-571, with moe_block_forward's MoE
FFN, src/moe.rs:443-469):
  rmsnorm per row: x * (1 / sqrt(sum(x^2) / n + eps)) * w         (src/infer.rs:72-81)
  q / k / v = QMat products of the normed rows (dequantized weights, quant::dequant)
  RoPE NeoX rotate-half, angle = pos * (1 / base^(2i/d)) in f32,    (src/infer.rs:90-145,
  (x0, x1) -> (x0 c - x1 s, x1 c + x0 s)                             src/forward.rs:188-206)
  causal GQA attention, kv head = h * n_kv / n_heads, scores * 1/sqrt(d), softmax over
  positions 0..=i, context = sum p_j v_j                            (src/forward.rs:218-283)
  y = x + o(ctx); out = y + moe_layer_forward(rmsnorm(y, ffn_norm)) (src/moe.rs:461-468)
The projections and attention sums are float64 here (the reference sums in f32 in its own
orders); the MoE layer is the oracle's exact-f32 restatement.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O


def rmsnorm(x, w, eps):
    x = x.astype(np.float32)
    ms = (x.astype(np.float64) ** 2).sum(axis=1, keepdims=True) / x.shape[1]
    inv = 1.0 / np.sqrt(ms + eps)
    return (x * inv * w).astype(np.float32)


def rope(t, heads, hd, cos, sin):
    T = t.shape[0]
    h = t.reshape(T, heads, hd).astype(np.float64)
    x0, x1 = h[..., : hd // 2], h[..., hd // 2:]
    c, s = cos[:, None, :].astype(np.float64), sin[:, None, :].astype(np.float64)
    return np.concatenate((x0 * c - x1 * s, x1 * c + x0 * s), axis=-1).reshape(T, heads * hd)


def proj(qt, rows, cols, x):
    w = O.dequant(qt.ggml_type, qt.data.tobytes()).reshape(rows, cols).astype(np.float64)
    return x.astype(np.float64) @ w.T


def attention(q, k, v, g):
    T = q.shape[0]
    hd = g.head_dim
    ctx = np.zeros((T, g.n_heads * hd))
    scale = 1.0 / np.sqrt(hd)
    mask = np.triu(np.ones((T, T), dtype=bool), 1)
    for h in range(g.n_heads):
        kvh = h * g.n_kv_heads // g.n_heads
        qh = q[:, h * hd:(h + 1) * hd]
        kh = k[:, kvh * hd:(kvh + 1) * hd]
        vh = v[:, kvh * hd:(kvh + 1) * hd]
        sc = (qh @ kh.T) * scale
        sc[mask] = -np.inf
        sc -= sc.max(axis=1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(axis=1, keepdims=True)
        ctx[:, h * hd:(h + 1) * hd] = p @ vh
    return ctx


def attention_residual(g, b, x, cos, sin):
    """y = x + o(attention(rmsnorm(x))): the block before its MoE FFN, float64 inside."""
    qd, kvd = g.n_heads * g.head_dim, g.n_kv_heads * g.head_dim
    x = x.astype(np.float32)
    xn = rmsnorm(x, b.attn_norm, g.rms_eps)
    q = rope(proj(b.q, qd, g.d_model, xn), g.n_heads, g.head_dim, cos, sin)
    k = rope(proj(b.k, kvd, g.d_model, xn), g.n_kv_heads, g.head_dim, cos, sin)
    v = proj(b.v, kvd, g.d_model, xn)
    ctx = attention(q, k, v, g)
    return (x.astype(np.float64) + proj(b.o, g.d_model, qd, ctx)).astype(np.float32)


def moe_residual(g, b, y):
    """The MoE FFN of a block on its attention residual y: moe_layer_forward(rmsnorm(y))."""
    return O.moe_layer_q_exact(rmsnorm(y, b.ffn_norm, g.rms_eps), b.moe)[0]


def stack_forward(g, blocks, x, cos, sin):
    """Hidden states after every block, [T, d_model] f32 each (last one = the output)."""
    outs = []
    x = x.astype(np.float32)
    qd, kvd = g.n_heads * g.head_dim, g.n_kv_heads * g.head_dim
    for b in blocks:
        xn = rmsnorm(x, b.attn_norm, g.rms_eps)
        q = rope(proj(b.q, qd, g.d_model, xn), g.n_heads, g.head_dim, cos, sin)
        k = rope(proj(b.k, kvd, g.d_model, xn), g.n_kv_heads, g.head_dim, cos, sin)
        v = proj(b.v, kvd, g.d_model, xn)
        ctx = attention(q, k, v, g)
        y = (x.astype(np.float64) + proj(b.o, g.d_model, qd, ctx)).astype(np.float32)
        yn = rmsnorm(y, b.ffn_norm, g.rms_eps)
        m = O.moe_layer_q_exact(yn, b.moe)[0]
        x = (y + m).astype(np.float32)
        outs.append(x)
    return outs
