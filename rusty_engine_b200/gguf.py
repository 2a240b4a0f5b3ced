"""GGUF expert binding: the reference's ``MmapModel`` (src/loader.rs:23-132) over the C ABI's
``rmoe_gguf_*`` entry points, and the MoE block of a model file (src/model.rs:366-391) as a
``LayerWeights`` or straight as a resident ``MoELayer``.

The parsing and the bounds checks happen in librmoe.so (host code, no GPU needed); this module
marshals pointers.  Like the reference, a missing tensor is ``None`` from ``tensor_bytes`` and an
error (``EngineError`` with the library's message) everywhere a tensor is required.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from . import _lib
from .synth import LayerWeights, QTensor


def _err(status: int) -> Exception:
    from .moe import EngineError

    return EngineError(_lib.load().rmoe_last_error().decode(errors="replace"))


class MmapModel:
    """A GGUF file mapped read-only with its parsed header (rmoe_gguf_open)."""

    def __init__(self, path: str):
        L = _lib.load()
        h = C.c_void_p()
        st = L.rmoe_gguf_open(str(path).encode(), C.byref(h))
        if st != _lib.RMOE_OK:
            raise _err(st)
        self._h = h
        self.path = str(path)

    @classmethod
    def open(cls, path: str) -> "MmapModel":
        return cls(path)

    def _tensor(self, name: str):
        t = _lib.Tensor()
        st = _lib.load().rmoe_gguf_tensor(self._h, name.encode(), C.byref(t))
        return st, t

    def tensor_bytes(self, name: str) -> Optional[np.ndarray]:
        """The tensor's bytes inside the mapping (a read-only view), or None when the tensor is
        absent, unsized or out of bounds (MmapModel::tensor_bytes, src/loader.rs:97-102)."""
        st, t = self._tensor(name)
        if st != _lib.RMOE_OK:
            return None
        buf = (C.c_uint8 * t.nbytes).from_address(t.data)
        a = np.frombuffer(buf, dtype=np.uint8)
        a.flags.writeable = False
        return a

    def tensor(self, name: str) -> QTensor:
        """A copy of the named tensor (type, bytes, GGUF dims); raises when it is missing."""
        st, t = self._tensor(name)
        if st != _lib.RMOE_OK:
            raise _err(st)
        data = np.frombuffer(C.string_at(t.data, t.nbytes), dtype=np.uint8).copy()
        dims = tuple(int(d) for d in t.dims)
        while len(dims) > 1 and dims[-1] == 1:
            dims = dims[:-1]
        return QTensor(int(t.ggml_type), data, dims)

    def meta_uint(self, key: str) -> Optional[int]:
        v = C.c_uint64()
        st = _lib.load().rmoe_gguf_meta_uint(self._h, key.encode(), C.byref(v))
        return int(v.value) if st == _lib.RMOE_OK else None

    def moe_layer_desc(self, block: int) -> _lib.LayerDesc:
        """Block `block`'s layer description, pointing into the mapping (valid until close)."""
        d = _lib.LayerDesc()
        st = _lib.load().rmoe_gguf_moe_layer_desc(self._h, block, C.byref(d))
        if st != _lib.RMOE_OK:
            raise _err(st)
        return d

    def moe_layer_weights(self, block: int) -> LayerWeights:
        """Copies of block `block`'s MoE tensors (router widened to f32)."""
        d = self.moe_layer_desc(block)

        def q(t: _lib.Tensor, nd: int) -> QTensor:
            data = np.frombuffer(C.string_at(t.data, t.nbytes), dtype=np.uint8).copy()
            return QTensor(int(t.ggml_type), data, tuple(int(x) for x in t.dims[:nd]))

        router = np.frombuffer(C.string_at(d.router_w, 4 * d.n_experts * d.hidden), dtype=np.float32)
        shared = None
        if d.has_shared:
            shared = (q(d.gate_shexp, 2), q(d.up_shexp, 2), q(d.down_shexp, 2))
        return LayerWeights(d.hidden, d.inter, d.n_experts, d.top_k, d.gate,
                            router.reshape(d.n_experts, d.hidden).copy(),
                            q(d.gate_exps, 3), q(d.up_exps, 3), q(d.down_exps, 3), shared,
                            name=f"{self.path}:blk.{block}")

    def moe_layer(self, block: int, device: Optional[int] = None):
        """Block `block` as a resident MoELayer on `device`: the expert bytes go from the
        mapping to HBM without a host copy."""
        from .moe import MoELayer

        return MoELayer.from_desc(self.moe_layer_desc(block), device)

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            _lib.load().rmoe_gguf_close(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
