"""The config-4 harness (rusty_engine_b200.stack): MoE transformer blocks around the layer,
against the CPU restatement of rusty-engine's prefill block with the MoE FFN
(oracle/stack_ref.py: src/forward.rs:532-571 with src/moe.rs:443-469), on a two-block stack of
small shapes, through both expert-product paths (40 tokens: decode kernels; 300 tokens:
tcgen05 kernels).  Hidden states after every block within relative L2 5e-3."""
import numpy as np
import pytest

from rusty_engine_b200 import synth


def small_geometry():
    from rusty_engine_b200.stack import Geometry

    return Geometry(d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, n_experts=8, top_k=2, inter=256,
                    rope_freq_base=1e6, rms_eps=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [40, 300])
def test_stack_matches_reference_block(gpu, T):
    """Each part of each block against the CPU restatement on the GPU's own input to that part,
    so that the check is the part's error, not errors carried in from earlier parts: the
    attention residual y = x + o(attention(rmsnorm(x))) (the QMat products' fp16 operands) and
    the MoE FFN on rmsnorm(y) (the layer contract); relative L2 <= 5e-3 each."""
    import torch

    from oracle import stack_ref
    from rusty_engine_b200.stack import MoEStack, make_block, rope_tables

    g = small_geometry()
    blocks = [make_block(g, seed=10 + i, dlo=0.001, dhi=0.004, attn_dlo=0.002, attn_dhi=0.01) for i in range(2)]
    x = synth.activations(T, g.d_model, seed=T)
    stack = MoEStack(g, blocks, device=0)
    out = stack.forward(torch.from_numpy(x).cuda(), collect=True).cpu().numpy()
    ins = [t.cpu().numpy() for t in stack.block_inputs]
    mids = [t.cpu().numpy() for t in stack.block_mids]
    assert len(stack.moe_ms) == 2 and all(ms > 0 for ms in stack.moe_ms)
    stack.close()
    assert np.isfinite(out).all()
    cos, sin = rope_tables(g, T)
    outs = ins[1:] + [out]
    rel = lambda a, b: float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b))
    for i, b in enumerate(blocks):
        ra = rel(mids[i], stack_ref.attention_residual(g, b, ins[i], cos, sin))
        rm = rel(outs[i] - mids[i], stack_ref.moe_residual(g, b, mids[i]))
        print(f"stack T={T} block {i}: attention residual rel-L2 {ra:.2e}, MoE FFN rel-L2 {rm:.2e}")
        assert ra <= 5e-3 and rm <= 5e-3, (i, ra, rm)


def test_rope_tables_match_reference_formula():
    """cos / sin of pos * base^(-2i/d) in f32 (src/infer.rs:90-96, 115-127)."""
    from rusty_engine_b200.stack import rope_tables

    g = small_geometry()
    c, s = rope_tables(g, 5, pos_start=3)
    d = g.head_dim
    for pos in (3, 7):
        for i in (0, 1, 63):
            f = np.float32(1.0) / np.power(np.float32(g.rope_freq_base), np.float32(2 * i) / np.float32(d))
            ang = np.float32(pos) * np.float32(f)
            assert c[pos - 3, i] == np.float32(np.cos(ang)) and s[pos - 3, i] == np.float32(np.sin(ang))
