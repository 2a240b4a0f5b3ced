"""Seeded synthetic MoE layers in GGUF layout (no dataset or checkpoint is involved).

Tensors follow the GGUF expert layout rusty-engine reads (src/model.rs:366-391):
``ffn_gate_inp`` [H, E] (E rows of H f32), ``ffn_{gate,up}_exps`` [H, I, E] (expert e = I
rows of row_bytes(H) at byte offset e*I*row_bytes(H)), ``ffn_down_exps`` [I, H, E].
Block bytes follow the ggml superblock formats that src/quant.rs:75-357 decodes.

Value distributions are the ones the benchmark configurations name: f16 scales uniform in a
range, nibbles / 6-bit codes uniform, Q6_K int8 sub-scales uniform in [-32, 31], router
weights N(0, 0.02), activations N(0, 1).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q5_0, GGML_Q8_0 = 0, 1, 2, 6, 8
GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_BF16 = 12, 13, 14, 30

# (elements per block, bytes per block): src/quant.rs:75-88
BLOCK = {
    GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_BF16: (1, 2),
    GGML_Q4_0: (32, 18), GGML_Q5_0: (32, 22), GGML_Q8_0: (32, 34),
    GGML_Q4_K: (256, 144), GGML_Q5_K: (256, 176), GGML_Q6_K: (256, 210),
}
TYPE_NAMES = {0: "F32", 1: "F16", 2: "Q4_0", 6: "Q5_0", 8: "Q8_0", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K", 30: "BF16"}


def row_bytes(t: int, n: int) -> int:
    e, b = BLOCK[t]
    assert n % e == 0, f"row of {n} elements is not whole {TYPE_NAMES[t]} blocks"
    return n // e * b


@dataclass
class QTensor:
    """One GGUF tensor: ggml type, raw bytes, GGUF dims (innermost first)."""

    ggml_type: int
    data: np.ndarray  # uint8
    dims: tuple

    @property
    def nbytes(self) -> int:
        return int(self.data.nbytes)


@dataclass
class LayerWeights:
    H: int
    I: int
    E: int
    k: int
    gate: int  # 0 softmax, 1 sigmoid (moe.rs Gate)
    router_w: np.ndarray  # [E, H] f32
    gate_exps: QTensor
    up_exps: QTensor
    down_exps: QTensor
    shared: Optional[tuple] = None  # (gate, up, down) QTensors, dims [H, I] / [I, H]
    name: str = ""
    meta: dict = field(default_factory=dict)


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint8).reshape(-1, 2)


def pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """The 12 packed bytes of eight 6-bit (scale, min) pairs: the inverse of get_scale_min_k4
    (src/quant.rs:250-258)."""
    q = np.zeros((sc.shape[0], 12), dtype=np.uint8)
    q[:, 0:4] = sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)
    q[:, 4:8] = mn[:, 0:4] | ((mn[:, 4:8] >> 4) << 6)
    q[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
    return q


def gen_q4k_centered(rng: np.random.Generator, nblocks: int, dlo: float, dhi: float) -> np.ndarray:
    """Q4_K superblocks whose weights have mean ~0 (dmin = d, min = 7.5 * scale rounded, scales
    in 0..8), for projections where the uniform-scale draw's positive mean would make every
    output the same large common mode."""
    out = gen_blocks(rng, GGML_Q4_K, nblocks, dlo, dhi).reshape(nblocks, 144)
    out[:, 2:4] = out[:, 0:2]
    sc = rng.integers(0, 9, (nblocks, 8), dtype=np.uint8)
    mn = np.rint(7.5 * sc).astype(np.uint8)
    out[:, 4:16] = pack_scale_min_k4(sc, mn)
    return out.reshape(-1)


def gen_blocks(rng: np.random.Generator, t: int, nblocks: int, dlo: float, dhi: float) -> np.ndarray:
    """Random superblocks of type ``t`` (uint8 array of nblocks * block_bytes)."""
    e, b = BLOCK[t]
    if t == GGML_F32:
        return rng.standard_normal(nblocks, dtype=np.float32).view(np.uint8)
    out = np.frombuffer(rng.bytes(nblocks * b), dtype=np.uint8).reshape(nblocks, b).copy()
    d = rng.uniform(dlo, dhi, nblocks)
    if t in (GGML_Q4_0, GGML_Q5_0, GGML_Q8_0):
        out[:, 0:2] = _f16_bytes(d)
    elif t in (GGML_Q4_K, GGML_Q5_K):
        out[:, 0:2] = _f16_bytes(d)
        out[:, 2:4] = _f16_bytes(rng.uniform(dlo, dhi, nblocks))
        sc = rng.integers(0, 64, (nblocks, 8), dtype=np.uint8)
        mn = rng.integers(0, 64, (nblocks, 8), dtype=np.uint8)
        out[:, 4:16] = pack_scale_min_k4(sc, mn)
    elif t == GGML_Q6_K:
        out[:, 192:208] = rng.integers(-32, 32, (nblocks, 16), dtype=np.int8).view(np.uint8)
        out[:, 208:210] = _f16_bytes(d)
    elif t in (GGML_F16, GGML_BF16):
        v = rng.standard_normal(nblocks).astype(np.float32) * 0.05
        if t == GGML_F16:
            return v.astype(np.float16).view(np.uint8).copy()
        return (v.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).copy()
    return out.reshape(-1)


def make_layer(
    H: int, I: int, E: int, k: int, *, gate_t: int, up_t: int, down_t: int,
    dlo: float, dhi: float, seed: int = 0, gate: int = 0, shared: bool = False, name: str = "",
) -> LayerWeights:
    rng = np.random.default_rng(seed)
    router_w = (rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.02)).astype(np.float32)

    def qt(t, n_in, n_out, experts):
        nel = n_in * n_out * experts
        e, _ = BLOCK[t]
        data = gen_blocks(rng, t, nel // e, dlo, dhi)
        dims = (n_in, n_out, experts) if experts > 1 or not shared else (n_in, n_out)
        return QTensor(t, data, dims)

    g = qt(gate_t, H, I, E)
    u = qt(up_t, H, I, E)
    d = qt(down_t, I, H, E)
    sh = None
    if shared:
        sh = (QTensor(gate_t, gen_blocks(rng, gate_t, H * I // BLOCK[gate_t][0], dlo, dhi), (H, I)),
              QTensor(up_t, gen_blocks(rng, up_t, H * I // BLOCK[up_t][0], dlo, dhi), (H, I)),
              QTensor(down_t, gen_blocks(rng, down_t, H * I // BLOCK[down_t][0], dlo, dhi), (I, H)))
    return LayerWeights(H, I, E, k, gate, router_w, g, u, d, sh, name=name)


def activations(T: int, H: int, seed: int = 1) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((T, H), dtype=np.float32)


# ---- the benchmark configurations ------------------------------------------------------
def config_c1(seed: int = 0) -> LayerWeights:
    """hidden 1024, 16 experts, top-4 softmax, inter 512, Q4_0 gate/up/down, d ~ U(0.005, 0.02)."""
    return make_layer(1024, 512, 16, 4, gate_t=GGML_Q4_0, up_t=GGML_Q4_0, down_t=GGML_Q4_0,
                      dlo=0.005, dhi=0.02, seed=seed, name="c1-h1024-e16-k4-i512-q4_0")


def config_c2(seed: int = 0) -> LayerWeights:
    """Qwen3-30B-A3B-shaped: hidden 2048, 128 experts, top-8, inter 768, Q4_K gate/up, Q6_K down."""
    return make_layer(2048, 768, 128, 8, gate_t=GGML_Q4_K, up_t=GGML_Q4_K, down_t=GGML_Q6_K,
                      dlo=0.001, dhi=0.01, seed=seed, name="c2-qwen3-30b-a3b-h2048-e128-k8-i768-q4k-q6k")


def config_c5(seed: int = 0) -> LayerWeights:
    """Qwen3-235B-A22B-shaped: hidden 4096, 128 experts, top-8, inter 1536, Q4_K / Q6_K."""
    return make_layer(4096, 1536, 128, 8, gate_t=GGML_Q4_K, up_t=GGML_Q4_K, down_t=GGML_Q6_K,
                      dlo=0.001, dhi=0.01, seed=seed, name="c5-qwen3-235b-a22b-h4096-e128-k8-i1536-q4k-q6k")


def zipf_router_bias(layer: LayerWeights, x: np.ndarray, s: float = 1.1, iters: int = 200,
                     sample: int = 2048, seed: int = 3) -> np.ndarray:
    """Per-expert logit bias so that top-k load over ``x`` follows Zipf(s) by expert rank.

    Damped log-ratio updates on a sample (loads floored at a quarter pick so unloaded experts
    do not blow the step up, mean removed each round).  A token picks an expert at most once,
    so no expert can carry more than 1/k of the picks: the head of the distribution saturates
    there.  The bias is realised inside the router by ``zipf_workload``.
    """
    rng = np.random.default_rng(seed)
    xs = x[rng.choice(x.shape[0], min(sample, x.shape[0]), replace=False)]
    logits = xs.astype(np.float64) @ layer.router_w.T.astype(np.float64)
    E, k = layer.E, layer.k
    target = 1.0 / np.arange(1, E + 1) ** s
    target = target / target.sum()
    b = np.zeros(E)
    for _ in range(iters):
        top = np.argpartition(-(logits + b), k, axis=1)[:, :k]
        load = np.bincount(top.ravel(), minlength=E) / top.size
        b += 0.2 * (np.log(target) - np.log(np.maximum(load, 0.25 / top.size)))
        b -= b.mean()
    return b.astype(np.float32)


def zipf_workload(layer: LayerWeights, T: int, s: float = 1.1, seed: int = 1, mean: float = 1.0):
    """Activations with a common mean mu (every element `mean`) and the layer with the Zipf(s)
    per-expert bias folded into its router: row e gains b_e * mu / |mu|^2, so W.x = W.x_0 +
    b_e (1 + mu.z / |mu|^2) ~ W.x_0 + b_e.  Returns (layer with the folded router, x)."""
    x = activations(T, layer.H, seed=seed) + np.float32(mean)
    b = zipf_router_bias(layer, x, s=s)
    mu = np.full(layer.H, mean, dtype=np.float64)
    rw = (layer.router_w.astype(np.float64) + np.outer(b, mu / (mu @ mu))).astype(np.float32)
    lw = LayerWeights(layer.H, layer.I, layer.E, layer.k, layer.gate, rw, layer.gate_exps, layer.up_exps,
                      layer.down_exps, layer.shared, name=layer.name + f"-zipf{s}")
    return lw, x

