"""A small GGUF (version 2 / 3) writer for the binding tests: typed metadata, tensor-info table,
aligned tensor data.  It writes the format the reference's parser reads (src/gguf.rs:307-392)
so the tests can build model files with MoE blocks; it is test infrastructure only."""
import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q",
        I64: "<q", F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(kind: int, v) -> bytes:
    if kind == STR:
        return _str(v)
    if kind == ARR:
        ek, items = v
        return struct.pack("<IQ", ek, len(items)) + b"".join(_value(ek, x) for x in items)
    return struct.pack(_FMT[kind], v)


def gguf_bytes(meta, tensors, version=3, alignment=32, magic=b"GGUF"):
    """meta: [(key, kind, value)]; tensors: [(name, dims, ggml_type, bytes)].  Tensor data is
    laid out in order, each at an offset aligned to `alignment`."""
    out = [magic, struct.pack("<I", version)]
    cnt = "<QQ" if version >= 3 else "<II"
    out.append(struct.pack(cnt, len(tensors), len(meta)))
    for k, kind, v in meta:
        out.append(_str(k) + struct.pack("<I", kind) + _value(kind, v))
    off = 0
    offsets = []
    for name, dims, t, data in tensors:
        offsets.append(off)
        out.append(_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) +
                   struct.pack("<IQ", t, off))
        off += (len(data) + alignment - 1) // alignment * alignment
    head = b"".join(out)
    head += b"\0" * ((-len(head)) % alignment)
    body = bytearray(off)
    for (name, dims, t, data), o in zip(tensors, offsets):
        body[o:o + len(data)] = bytes(data)
    return head + bytes(body)


def moe_block_tensors(block, lw, router_type=0):
    """The tensors of one MoE block (src/model.rs:366-391) from synth LayerWeights."""
    p = f"blk.{block}."
    if router_type == 0:
        router = np.ascontiguousarray(lw.router_w, dtype=np.float32).tobytes()
    elif router_type == 1:
        router = lw.router_w.astype(np.float16).tobytes()
    else:  # bf16: the high halves
        router = (lw.router_w.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
    ts = [
        (p + "ffn_gate_inp.weight", [lw.H, lw.E], router_type if router_type < 2 else 30, router),
        (p + "ffn_gate_exps.weight", list(lw.gate_exps.dims), lw.gate_exps.ggml_type, lw.gate_exps.data.tobytes()),
        (p + "ffn_up_exps.weight", list(lw.up_exps.dims), lw.up_exps.ggml_type, lw.up_exps.data.tobytes()),
        (p + "ffn_down_exps.weight", list(lw.down_exps.dims), lw.down_exps.ggml_type, lw.down_exps.data.tobytes()),
    ]
    if lw.shared is not None:
        for nm, q in zip(("gate", "up", "down"), lw.shared):
            ts.append((p + f"ffn_{nm}_shexp.weight", list(q.dims), q.ggml_type, q.data.tobytes()))
    return ts
