"""Host-side mirror of rusty-engine's MoE-layer interface, backed by librmoe.so on a B200.

Names, argument meaning and error behaviour follow the Rust API so callers (and the parity
tests) read like the reference's own:

* ``Gate``, ``RouterConfig``, ``ExpertScore``, ``ExpertWeights``  -- src/moe.rs:11-41, 348-353
* ``route(logits, cfg)``                                          -- src/moe.rs:120-125
* ``route_noaux_tc`` / ``route_group`` (+ ``route_grouped_batch``) -- src/moe.rs:127-268
* ``moe_layer_forward(hidden, router_w, n_experts, experts, shared, inter, cfg)``
                                                                   -- src/moe.rs:360-388
* ``QMat.from_bytes(...).matvec/.matmul``                         -- src/qmat.rs:51-182
* ``dequant(ggml_type, data)``                                    -- src/quant.rs:363-453
* ``MoELayer``: a resident layer over GGUF expert tensors (the B200 handle that
  ``moe_layer_forward`` drives when the experts come from ``ffn_*_exps``); ``gguf.MmapModel``
  binds a model file's ``blk.N.ffn_*_exps`` to it (src/loader.rs:97-102, src/model.rs:366-391).

Shape errors raise ``ValueError`` where the Rust code asserts (panics); recoverable errors
raise ``EngineError`` (src/core.rs:56-68).  Every computation runs on the GPU through the C
ABI; there is no CPU path in this module.
"""
from __future__ import annotations

import ctypes as C
import enum
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

from . import _lib
from .synth import BLOCK, LayerWeights, QTensor

try:  # torch provides device memory and streams (plumbing only)
    import torch
except Exception:  # pragma: no cover
    torch = None


class EngineError(Exception):
    """rusty-engine's EngineError{message} (src/core.rs:56-68)."""

    def __init__(self, message: str):
        super().__init__(message)
        self.message = message


class Gate(enum.IntEnum):
    Softmax = 0
    Sigmoid = 1


@dataclass(frozen=True)
class RouterConfig:
    gate: Gate = Gate.Softmax
    top_k: int = 2


@dataclass(frozen=True)
class ExpertScore:
    id: int
    weight: float


@dataclass
class ExpertWeights:
    """f32 row-major: gate/up are inter x hidden, down is hidden x inter (src/moe.rs:348-353)."""

    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray


def _require_cuda():
    if torch is None or not torch.cuda.is_available():
        raise RuntimeError("rusty_engine_b200 needs a CUDA device (B200); there is no CPU fallback")


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _call(status):
    try:
        _lib.check(status)
    except _lib.RmoeError as e:
        if e.status in (_lib.RMOE_ERR_INVALID,):
            raise EngineError(e.message) from None
        raise


def _dev_f32(a) -> "torch.Tensor":
    if torch.is_tensor(a):
        return a.to(device="cuda", dtype=torch.float32).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


# ---- route ----------------------------------------------------------------------------
def route_batch(logits, cfg: RouterConfig):
    """route() over a [T, E] batch of logits on the GPU -> (ids [T,k] int32, weights [T,k])."""
    _require_cuda()
    lg = _dev_f32(logits)
    if lg.dim() == 1:
        lg = lg[None]
    T, E = lg.shape
    k = min(cfg.top_k, E)
    if T == 0 or E == 0:
        return np.zeros((T, 0), np.int32), np.zeros((T, 0), np.float32)
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    _call(_lib.load().rmoe_route(lg.data_ptr(), T, E, k, int(cfg.gate), ids.data_ptr(), w.data_ptr(), _stream()))
    torch.cuda.synchronize()
    return ids.cpu().numpy(), w.cpu().numpy()


def route(logits: Sequence[float], cfg: RouterConfig) -> List[ExpertScore]:
    """route (src/moe.rs:120-125): top-k experts with their normalised weights."""
    if len(logits) == 0:
        return []
    ids, w = route_batch(np.asarray(logits, dtype=np.float32)[None], cfg)
    return [ExpertScore(int(i), float(x)) for i, x in zip(ids[0], w[0])]


def top_k(scores: Sequence[float], k: int) -> List[ExpertScore]:
    return route(scores, RouterConfig(Gate.Softmax, k))


def top_k_sigmoid(scores: Sequence[float], k: int) -> List[ExpertScore]:
    return route(scores, RouterConfig(Gate.Sigmoid, k))


def route_grouped_batch(logits, bias, n_groups: int, top_k: int, top_k_group: Optional[int], noaux: bool = True):
    """Group routing of a [T, E] batch on the GPU (rmoe_route_grouped) -> (ids [T, k] uint32,
    weights [T, k]); picks beyond the eligible experts have id 0xFFFFFFFF and weight 0."""
    _require_cuda()
    lg = _dev_f32(logits)
    if lg.dim() == 1:
        lg = lg[None]
    T, E = lg.shape
    if T == 0 or E == 0 or top_k == 0:
        return np.zeros((T, 0), np.uint32), np.zeros((T, 0), np.float32)
    b = _dev_f32(bias) if bias is not None and len(bias) else None
    ids = torch.empty((T, top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, top_k), dtype=torch.float32, device="cuda")
    _call(_lib.load().rmoe_route_grouped(lg.data_ptr(), b.data_ptr() if b is not None else None,
                                         0 if b is None else b.numel(), T, E, top_k, n_groups,
                                         -1 if top_k_group is None else top_k_group, 1 if noaux else 0,
                                         ids.data_ptr(), w.data_ptr(), _stream()))
    torch.cuda.synchronize()
    return ids.cpu().numpy().view(np.uint32), w.cpu().numpy()


def _grouped(logits, bias, n_groups, top_k, top_k_group, noaux) -> List[ExpertScore]:
    if len(logits) == 0:
        return []
    ids, w = route_grouped_batch(np.asarray(logits, dtype=np.float32)[None], bias, n_groups, top_k, top_k_group,
                                 noaux)
    return [ExpertScore(int(i), float(x)) for i, x in zip(ids[0], w[0]) if i != 0xFFFFFFFF]


def route_noaux_tc(logits, bias, n_groups: int, top_k: int, top_k_group: Optional[int]) -> List[ExpertScore]:
    """route_noaux_tc (src/moe.rs:192-268): sigmoid(logit + bias) scores, groups ranked by the
    sum of their top-2 scores, the top_k_group best eligible, top_k experts renormalised."""
    return _grouped(logits, bias, n_groups, top_k, top_k_group, True)


def route_group(logits, bias, n_groups: int, top_k: int, top_k_group: Optional[int]) -> List[ExpertScore]:
    """route_group (src/moe.rs:127-190): as route_noaux_tc with groups ranked by their summed score."""
    return _grouped(logits, bias, n_groups, top_k, top_k_group, False)


# ---- dequant / QMat -------------------------------------------------------------------
def dequant(ggml_type: int, data) -> np.ndarray:
    """quant::dequant on the GPU; raises EngineError with the reference's message."""
    _require_cuda()
    raw = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else data.view(np.uint8)
    if ggml_type not in BLOCK:
        _call(_lib.load().rmoe_dequant(ggml_type, None, len(raw), None, _stream()))
    el, by = BLOCK[ggml_type]
    n = (len(raw) // by) * el if len(raw) % by == 0 else 0
    src = torch.from_numpy(raw.copy()).cuda() if len(raw) else torch.empty(16, dtype=torch.uint8, device="cuda")
    dst = torch.empty(max(n, 1), dtype=torch.float32, device="cuda")
    _call(_lib.load().rmoe_dequant(ggml_type, src.data_ptr(), len(raw), dst.data_ptr(), _stream()))
    torch.cuda.synchronize()
    return dst[:n].cpu().numpy()


class QMat:
    """Quantized m x n weight matrix (src/qmat.rs:30-42); products run on the GPU."""

    def __init__(self, ggml_type: int, data: np.ndarray, m: int, n: int):
        self.ggml_type, self.bytes, self.m, self.n = ggml_type, np.ascontiguousarray(data, dtype=np.uint8), m, n

    @classmethod
    def from_bytes(cls, ggml_type: int, data, m: int, n: int) -> "QMat":
        return cls(ggml_type, np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else data, m, n)

    @classmethod
    def from_f32(cls, data, m: int, n: int) -> "QMat":
        a = np.ascontiguousarray(data, dtype=np.float32)
        if a.size != m * n:
            raise ValueError("QMat::from_f32: shape mismatch")
        return cls(0, a.view(np.uint8).reshape(-1), m, n)

    def rows(self) -> int:
        return self.m

    def cols(self) -> int:
        return self.n

    def _handle(self):
        """The resident device copy (rmoe_qmat_create), made on first use."""
        h = getattr(self, "_h", None)
        if h is None:
            _require_cuda()
            h = C.c_void_p()
            b = self.bytes
            _call(_lib.load().rmoe_qmat_create(self.ggml_type, b.ctypes.data, b.nbytes, self.m, self.n,
                                               torch.cuda.current_device(), C.byref(h)))
            self._h = h
        return h

    def matmul_device(self, x, out=None, *, stream=None):
        """X [rows, n] f32 cuda tensor -> [rows, m] on the device (rmoe_qmat_forward: resident
        weights, stream-ordered, no synchronisation)."""
        rows = x.shape[0]
        if x.shape[1] != self.n:
            raise ValueError("matmul: X rows x n")
        if out is None:
            out = torch.empty((rows, self.m), dtype=torch.float32, device=x.device)
        s = C.c_void_p(stream.cuda_stream) if stream is not None else _stream()
        _call(_lib.load().rmoe_qmat_forward(self._handle(), x.data_ptr(), rows, out.data_ptr(), s))
        return out

    def matmul(self, x, rows: int) -> np.ndarray:
        """W[m x n] . X[rows x n] -> [rows x m] (QMat::matmul, src/qmat.rs:169-182)."""
        _require_cuda()
        xd = _dev_f32(x).reshape(-1)
        if xd.numel() != rows * self.n:
            raise ValueError("matmul: X rows x n")
        if rows == 0:
            return np.zeros((0, self.m), np.float32)
        out = self.matmul_device(xd.reshape(rows, self.n))
        torch.cuda.synchronize()
        _call(_lib.load().rmoe_qmat_status(self._handle()))
        return out.cpu().numpy()

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.load().rmoe_qmat_destroy(h)
            except Exception:
                pass

    def matvec(self, x) -> np.ndarray:
        return self.matmul(x, 1)[0]


# ---- the layer --------------------------------------------------------------------------
def _tensor(q: Optional[QTensor]) -> _lib.Tensor:
    t = _lib.Tensor()
    if q is None:
        return t
    t.ggml_type = q.ggml_type
    t.data = q.data.ctypes.data
    t.nbytes = q.nbytes
    dims = list(q.dims) + [0] * (3 - len(q.dims))
    for i in range(3):
        t.dims[i] = dims[i]
    return t


def ep_unique_id() -> bytes:
    """A fresh NCCL unique id (rmoe_ep_unique_id) for the ranks of one expert-parallel layer."""
    buf = (C.c_uint8 * 128)()
    _call(_lib.load().rmoe_ep_unique_id(buf))
    return bytes(buf)


def ep_balanced_placement(load: Sequence[float], world: int) -> np.ndarray:
    """An expert placement for rmoe_ep_layer_create_placed from per-expert loads (e.g. the pick
    counts of a calibration batch, summed over the ranks): largest load first, each expert to
    the rank with the least load so far (then the fewest experts, then the lowest rank), so
    every rank gets at least one expert when there are at least `world` experts.  Returns
    placement[e] = rank."""
    load = np.asarray(load, dtype=np.float64)
    E = load.shape[0]
    if world < 1 or E < world:
        raise EngineError(f"{E} experts cannot be placed on {world} ranks (each rank needs one)")
    acc = np.zeros(world)
    n = np.zeros(world, dtype=np.int64)
    out = np.empty(E, dtype=np.int32)
    for e in sorted(range(E), key=lambda i: (-load[i], i)):
        r = min(range(world), key=lambda q: (acc[q], n[q], q))
        out[e] = r
        acc[r] += load[e]
        n[r] += 1
    return out


class MoELayer:
    """A resident MoE layer on one GPU (rmoe_layer_create / rmoe_layer_forward)."""

    @classmethod
    def expert_parallel(cls, lw: LayerWeights, rank: int, world: int, uid: bytes, device: Optional[int] = None,
                        placement=None):
        """This rank's shard of an expert-parallel layer on `device`; every rank calls it with
        the same uid (and the same placement).  placement[e] is the rank holding expert e
        (rmoe_ep_layer_create_placed, e.g. from ep_balanced_placement); None deals the experts
        round-robin (rmoe_ep_layer_create: rank r holds r, r + world, ...).  forward() then
        takes this rank's tokens and returns their full layer outputs."""
        return cls(lw, device, _ep=(rank, world, uid, placement))

    def __init__(self, lw: LayerWeights, device: Optional[int] = None, *, _ep=None):
        _require_cuda()
        self.lw = lw
        self.H, self.I, self.E, self.k = lw.H, lw.I, lw.E, min(lw.k, lw.E)
        dev = torch.cuda.current_device() if device is None else device
        self.device = dev
        self._router = np.ascontiguousarray(lw.router_w, dtype=np.float32)
        d = _lib.LayerDesc()
        d.hidden, d.inter, d.n_experts, d.top_k, d.gate = lw.H, lw.I, lw.E, lw.k, int(lw.gate)
        d.router_w = self._router.ctypes.data
        d.gate_exps, d.up_exps, d.down_exps = _tensor(lw.gate_exps), _tensor(lw.up_exps), _tensor(lw.down_exps)
        d.has_shared = 1 if lw.shared is not None else 0
        if lw.shared is not None:
            d.gate_shexp, d.up_shexp, d.down_shexp = (_tensor(t) for t in lw.shared)
        d.device = dev
        h = C.c_void_p()
        L = _lib.load()
        if _ep is None:
            _call(L.rmoe_layer_create(C.byref(d), C.byref(h)))
        else:
            rank, world, uid, placement = _ep
            idbuf = (C.c_uint8 * 128).from_buffer_copy(bytes(uid))
            if placement is None:
                _call(L.rmoe_ep_layer_create(C.byref(d), rank, world, idbuf, C.byref(h)))
            else:
                pl = np.ascontiguousarray(placement, dtype=np.int32)
                if pl.shape != (lw.E,):
                    raise EngineError(f"placement has {pl.size} entries for {lw.E} experts")
                _call(L.rmoe_ep_layer_create_placed(C.byref(d), rank, world, idbuf, pl.ctypes.data, C.byref(h)))
        self._h = h

    @classmethod
    def from_desc(cls, d: _lib.LayerDesc, device: Optional[int] = None) -> "MoELayer":
        """A layer from a filled rmoe_layer_desc (e.g. gguf.MmapModel.moe_layer_desc): the
        bytes it points to are copied to HBM inside the call."""
        _require_cuda()
        self = cls.__new__(cls)
        self.lw = None
        self.H, self.I, self.E, self.k = d.hidden, d.inter, d.n_experts, min(d.top_k, d.n_experts)
        self.device = torch.cuda.current_device() if device is None else device
        self._router = None
        d.device = self.device
        h = C.c_void_p()
        _call(_lib.load().rmoe_layer_create(C.byref(d), C.byref(h)))
        self._h = h
        return self

    def forward(self, x, out=None, *, flags: int = 0, stream=None):
        """x: [T, H] f32 cuda tensor -> out [T, H] f32 (stream-ordered, no sync)."""
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, self.H), dtype=torch.float32, device=x.device)
        s = C.c_void_p(stream.cuda_stream) if stream is not None else _stream()
        _call(_lib.load().rmoe_layer_forward(self._h, x.data_ptr(), T, out.data_ptr(), s, flags))
        return out

    def forward_host(self, x: np.ndarray, *, flags: int = 0) -> np.ndarray:
        """Host in, host out (copies inside the call): the end-to-end entry point."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        _call(_lib.load().rmoe_layer_forward(self._h, x.ctypes.data, x.shape[0], out.ctypes.data, _stream(),
                                             flags | _lib.FLAG_HOST_IO))
        return out

    def routing(self, T: int):
        ids = np.zeros((T, self.k), dtype=np.uint32)
        w = np.zeros((T, self.k), dtype=np.float32)
        _call(_lib.load().rmoe_layer_routing(self._h, T, ids.ctypes.data, w.ctypes.data))
        return ids, w

    def logits(self, T: int) -> np.ndarray:
        lg = np.zeros((T, self.E), dtype=np.float32)
        _call(_lib.load().rmoe_layer_logits(self._h, T, lg.ctypes.data))
        return lg

    def router_refined(self) -> int:
        """Tokens whose fast-router top-k met a near-tie (and were rescored with the
        sequential sums) since the last call; reads and resets the count."""
        n = C.c_uint32()
        _call(_lib.load().rmoe_layer_router_refined(self._h, C.byref(n)))
        return int(n.value)

    def stage_ms(self):
        """[route, gate/up, down, combine] ms of the last forward with FLAG_STAGE_TIMING."""
        ms = (C.c_float * 4)()
        _call(_lib.load().rmoe_layer_stage_ms(self._h, ms))
        return list(ms)

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            _lib.load().rmoe_layer_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _pad_to(a: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.zeros((rows, cols), dtype=np.float32)
    out[: a.shape[0], : a.shape[1]] = a
    return out


def moe_layer_forward(hidden, router_w, n_experts: int, experts: Sequence[ExpertWeights],
                      shared: Optional[ExpertWeights], inter: int, cfg: RouterConfig) -> np.ndarray:
    """moe_layer_forward (src/moe.rs:360-388) with f32 ExpertWeights, on the GPU.

    ``hidden`` may be one token [H] (the reference signature) or a batch [T, H].  Widths are
    zero-padded to the kernels' 256-multiples: zero rows/columns add exact zeros to every
    router sum and expert product, so the padded layer computes the same function.  Missing
    experts (``len(experts) < n_experts``) contribute nothing, as ``experts.get(e.id)`` skips
    them in the reference (src/moe.rs:374).
    """
    x = np.asarray(hidden, dtype=np.float32)
    single = x.ndim == 1
    x = x.reshape(1, -1) if single else x
    T, H = x.shape
    rw = np.asarray(router_w, dtype=np.float32).reshape(-1)
    if rw.size != n_experts * H:
        raise ValueError("matvec: weight size mismatch")
    Hp, Ip = -(-H // 256) * 256, -(-inter // 256) * 256
    E = n_experts
    g = np.zeros((E, Ip, Hp), np.float32)
    u = np.zeros((E, Ip, Hp), np.float32)
    d = np.zeros((E, Hp, Ip), np.float32)
    for e, ew in enumerate(list(experts)[:E]):
        g[e] = _pad_to(np.asarray(ew.gate, np.float32).reshape(inter, H), Ip, Hp)
        u[e] = _pad_to(np.asarray(ew.up, np.float32).reshape(inter, H), Ip, Hp)
        d[e] = _pad_to(np.asarray(ew.down, np.float32).reshape(H, inter), Hp, Ip)
    qt = lambda a, dims: QTensor(0, a.reshape(-1).view(np.uint8), dims)
    sh = None
    if shared is not None:
        sh = (qt(_pad_to(np.asarray(shared.gate, np.float32).reshape(inter, H), Ip, Hp), (Hp, Ip)),
              qt(_pad_to(np.asarray(shared.up, np.float32).reshape(inter, H), Ip, Hp), (Hp, Ip)),
              qt(_pad_to(np.asarray(shared.down, np.float32).reshape(H, inter), Hp, Ip), (Ip, Hp)))
    lw = LayerWeights(Hp, Ip, E, cfg.top_k, int(cfg.gate), _pad_to(rw.reshape(E, H), E, Hp),
                      qt(g, (Hp, Ip, E)), qt(u, (Hp, Ip, E)), qt(d, (Ip, Hp, E)), sh)
    layer = MoELayer(lw)
    try:
        out = layer.forward_host(_pad_to(x, T, Hp), flags=_lib.FLAG_DETERMINISTIC)[:, :H]
    finally:
        layer.close()
    return out[0] if single else out
