"""GGUF expert binding (rmoe_gguf_*; MmapModel::open / tensor_bytes, src/loader.rs:33-102; the
MoE tensors of a block, src/model.rs:366-391).  The CPU tests parse files written by
tests/gguf_writer.py through the library (host code) and check every field and error path; the
GPU test runs a layer bound straight from the file against the same weights passed in memory
and against the oracle."""
import numpy as np
import pytest

from gguf_writer import ARR, F32, I32, STR, U32, U64, U8, gguf_bytes, moe_block_tensors
from rusty_engine_b200 import synth
from rusty_engine_b200.gguf import MmapModel
from rusty_engine_b200.moe import EngineError


def small_layer(seed, gt=synth.GGML_Q4_K, dt=synth.GGML_Q6_K, shared=False, E=8, k=2):
    return synth.make_layer(512, 256, E, k, gate_t=gt, up_t=gt, down_t=dt, dlo=0.001, dhi=0.02, seed=seed,
                            shared=shared)


def meta(arch="qwen3moe", E=8, k=2, extra=()):
    m = [("general.architecture", STR, arch), ("general.alignment", U32, 32),
         ("tokenizer.ggml.tokens", ARR, (STR, ["a", "bb", "ccc"])),
         ("nested", ARR, (ARR, [(U8, [1, 2]), (U8, [])])),
         ("rope.freq_base", F32, 1e6)]
    if E is not None:
        m.append((f"{arch}.expert_count", U32, E))
    if k is not None:
        m.append((f"{arch}.expert_used_count", U32, k))
    return m + list(extra)


@pytest.fixture(scope="module")
def model_file(tmp_path_factory):
    l0 = small_layer(1)
    l1 = small_layer(2, gt=synth.GGML_Q4_0, dt=synth.GGML_Q8_0, shared=True)
    ts = moe_block_tensors(0, l0) + moe_block_tensors(1, l1, router_type=1)
    ts.append(("token_embd.weight", [512, 4], 0, np.zeros((4, 512), np.float32).tobytes()))
    p = tmp_path_factory.mktemp("gguf") / "moe.gguf"
    p.write_bytes(gguf_bytes(meta(), ts))
    return str(p), l0, l1


def write(tmp_path, data, name="m.gguf"):
    p = tmp_path / name
    p.write_bytes(data)
    return str(p)


def test_block_desc_and_bytes(model_file):
    path, l0, l1 = model_file
    with MmapModel(path) as m:
        assert m.meta_uint("qwen3moe.expert_count") == 8 and m.meta_uint("general.alignment") == 32
        assert m.meta_uint("missing.key") is None
        d = m.moe_layer_desc(0)
        assert (d.hidden, d.inter, d.n_experts, d.top_k, d.gate, d.has_shared) == (512, 256, 8, 2, 0, 0)
        assert tuple(d.gate_exps.dims) == (512, 256, 8) and tuple(d.down_exps.dims) == (256, 512, 8)
        lw = m.moe_layer_weights(0)
        np.testing.assert_array_equal(lw.router_w, l0.router_w)
        for a, b in ((lw.gate_exps, l0.gate_exps), (lw.up_exps, l0.up_exps), (lw.down_exps, l0.down_exps)):
            assert a.ggml_type == b.ggml_type and a.dims == tuple(b.dims)
            np.testing.assert_array_equal(a.data, b.data)
        # block 1: F16 router widened exactly, shared expert present
        lw1 = m.moe_layer_weights(1)
        assert lw1.shared is not None and lw1.gate_exps.ggml_type == synth.GGML_Q4_0
        np.testing.assert_array_equal(lw1.router_w, l1.router_w.astype(np.float16).astype(np.float32))
        for a, b in zip(lw1.shared, l1.shared):
            np.testing.assert_array_equal(a.data, b.data)
            assert a.dims == tuple(b.dims)
        # tensor_bytes: a read-only view of the mapping, None when absent
        tb = m.tensor_bytes("blk.0.ffn_up_exps.weight")
        np.testing.assert_array_equal(tb, l0.up_exps.data)
        assert not tb.flags.writeable
        assert m.tensor_bytes("blk.9.ffn_up_exps.weight") is None
        t = m.tensor("token_embd.weight")
        assert t.ggml_type == 0 and t.dims == (512, 4) and t.nbytes == 512 * 4 * 4
        with pytest.raises(EngineError, match="missing required tensor 'blk.2.ffn_gate_exps.weight'"):
            m.moe_layer_desc(2)


def test_bf16_router_sigmoid_gate_and_general_keys(tmp_path):
    lw = small_layer(3)
    extra = [("qwen3moe.expert_gating_func", U32, 2), ("general.expert_used_count", U64, 3)]
    p = write(tmp_path, gguf_bytes(meta(k=None, extra=extra), moe_block_tensors(0, lw, router_type=2)))
    with MmapModel(p) as m:
        d = m.moe_layer_desc(0)
        assert d.gate == 1 and d.top_k == 3
        got = m.moe_layer_weights(0).router_w
        want = (lw.router_w.view(np.uint32) & 0xffff0000).view(np.float32)
        np.testing.assert_array_equal(got, want)


def test_version2_and_alignment(tmp_path):
    lw = small_layer(4)
    m2 = [x for x in meta() if x[0] != "general.alignment"] + [("general.alignment", U32, 64)]
    p = write(tmp_path, gguf_bytes(m2, moe_block_tensors(0, lw), version=2, alignment=64))
    with MmapModel(p) as m:
        np.testing.assert_array_equal(m.moe_layer_weights(0).down_exps.data, lw.down_exps.data)


@pytest.mark.parametrize("mutate,match", [
    (lambda b: b"GGUX" + b[4:], "gguf parse error at 0: missing GGUF magic"),
    (lambda b: b[:4] + (4).to_bytes(4, "little") + b[8:], "unsupported GGUF version 4 \\(need 2 or 3\\)"),
    (lambda b: b[:300], "gguf parse error at \\d+: unexpected EOF"),
])
def test_parse_errors(tmp_path, mutate, match):
    lw = small_layer(5)
    p = write(tmp_path, mutate(gguf_bytes(meta(), moe_block_tensors(0, lw))))
    with pytest.raises(EngineError, match=match):
        MmapModel(p)


def test_shape_and_metadata_errors(tmp_path):
    lw = small_layer(6)
    ts = moe_block_tensors(0, lw)
    bad = [(n, [256, 512, 8] if "up_exps" in n else d, t, b) for n, d, t, b in ts]
    with MmapModel(write(tmp_path, gguf_bytes(meta(), bad), "a.gguf")) as m:
        with pytest.raises(EngineError, match=r"blk.0.ffn_up_exps.weight: dims \[256, 512, 8\] != expected \[512, 256, 8\]"):
            m.moe_layer_desc(0)
    with MmapModel(write(tmp_path, gguf_bytes(meta(E=16), ts), "b.gguf")) as m:
        with pytest.raises(EngineError, match="holds 8 experts, qwen3moe.expert_count is 16"):
            m.moe_layer_desc(0)
    with MmapModel(write(tmp_path, gguf_bytes(meta(k=None), ts), "c.gguf")) as m:
        with pytest.raises(EngineError, match="missing required key 'qwen3moe.expert_used_count'"):
            m.moe_layer_desc(0)
    with MmapModel(write(tmp_path, gguf_bytes(meta(extra=[("qwen3moe.expert_gating_func", I32, 3)]), ts), "d.gguf")) as m:
        with pytest.raises(EngineError, match="expert_gating_func 3"):
            m.moe_layer_desc(0)
    part = ts + [("blk.0.ffn_gate_shexp.weight", [512, 256], lw.gate_exps.ggml_type,
                  lw.gate_exps.data[: lw.gate_exps.nbytes // 8].tobytes())]
    with MmapModel(write(tmp_path, gguf_bytes(meta(), part), "e.gguf")) as m:
        with pytest.raises(EngineError, match="1 of the 3 shared-expert tensors present"):
            m.moe_layer_desc(0)


def test_tensor_out_of_bounds(tmp_path):
    lw = small_layer(7)
    data = gguf_bytes(meta(), moe_block_tensors(0, lw))
    p = write(tmp_path, data[: len(data) - 100])  # the last tensor's bytes run past the end
    with MmapModel(p) as m:
        assert m.tensor_bytes("blk.0.ffn_down_exps.weight") is None
        with pytest.raises(EngineError, match="bytes out of bounds"):
            m.moe_layer_desc(0)


@pytest.mark.gpu
def test_layer_from_gguf_matches_in_memory_layer(gpu, model_file):
    """A layer bound straight from the mapping (no host copy) computes the same outputs, bit
    for bit, as the same weights passed from memory, and passes the oracle parity bars."""
    import torch

    from oracle import oracle as O
    from rusty_engine_b200 import _lib
    from rusty_engine_b200.moe import MoELayer
    from test_gpu_parity import assert_layer_close

    path, l0, l1 = model_file
    x = synth.activations(37, 512, seed=11)
    xd = torch.from_numpy(x).cuda()
    for block, lw in ((0, l0), (1, l1)):
        with MmapModel(path) as m:
            a = m.moe_layer(block)
            lw_file = m.moe_layer_weights(block)
        b = MoELayer(lw_file)
        flags = _lib.FLAG_DETERMINISTIC | _lib.FLAG_EXACT_ROUTER
        ya = a.forward(xd, flags=flags).cpu().numpy()
        yb = b.forward(xd, flags=flags).cpu().numpy()
        np.testing.assert_array_equal(ya, yb)
        assert_layer_close(ya, O.moe_layer_q_exact(x, lw_file)[0], f"gguf block {block}")
        a.close()
        b.close()
