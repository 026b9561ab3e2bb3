"""kore_b200 — B200 attention path for kore (BJZR/kore), behind a C ABI.

The product is ``kore_b200/libkore_cuda.so`` (sources in ``kore_b200/csrc``,
ABI in ``include/kore_cuda.h``). This module binds it with ctypes and mirrors
kore's per-layer attention call: ``decode`` replaces kore.cpp:1424-1455 and
``prefill`` kore.cpp:1527-1563, with kore's host buffers (numpy arrays here);
the ``*_dev`` forms take device tensors and stay on the context's stream.
``set_attn_weights`` + ``attn_block_decode`` run a decode step's whole
attention block (kore.cpp:1418-1457), its Q4_K / Q6_K projections included.

There is no fallback: if the library is missing, importing this module works
but creating a context raises, naming the build command.
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

from .build import LIB, INCLUDE

__all__ = ["KoreCuda", "KoreCudaError", "KvView", "Server", "load_library", "declared_symbols", "STATUS"]

STATUS = {
    0: "KORE_CUDA_OK", -1: "KORE_CUDA_EINVAL", -2: "KORE_CUDA_ERANGE", -3: "KORE_CUDA_ENOMEM",
    -4: "KORE_CUDA_ECUDA", -5: "KORE_CUDA_ESTATE", -6: "KORE_CUDA_EDEVICE", -7: "KORE_CUDA_ENCCL",
}


class KoreCudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


class _Cfg(ctypes.Structure):
    _fields_ = [
        ("n_layer", ctypes.c_int), ("n_head", ctypes.c_int), ("n_head_kv", ctypes.c_int),
        ("head_dim", ctypes.c_int), ("ctx_max", ctypes.c_int), ("max_seqs", ctypes.c_int),
        ("page_tokens", ctypes.c_int), ("n_pages", ctypes.c_int), ("rope_base", ctypes.c_float),
        ("inv_freq", ctypes.POINTER(ctypes.c_float)), ("device", ctypes.c_int),
        ("shard_rank", ctypes.c_int), ("shard_count", ctypes.c_int),
    ]


class KvView(ctypes.Structure):
    """kore_cuda_kv_view: a caller-owned paged KV cache for the no-allocation
    decode entry point (all pointers are device addresses)."""
    _fields_ = [
        ("k_pages", ctypes.c_void_p), ("v_pages", ctypes.c_void_p), ("page_table", ctypes.c_void_p),
        ("n_table", ctypes.c_int), ("n_pages", ctypes.c_int), ("page_tokens", ctypes.c_int),
        ("n_head", ctypes.c_int), ("n_head_kv", ctypes.c_int), ("head_dim", ctypes.c_int),
        ("rope_cs", ctypes.c_void_p), ("n_rope", ctypes.c_int),
    ]


class _QMat(ctypes.Structure):
    """kore_cuda_qmat: one quantised weight matrix in host memory."""
    _fields_ = [("type", ctypes.c_int), ("rows", ctypes.c_int), ("cols", ctypes.c_int), ("data", ctypes.c_void_p)]


class _LayerW(ctypes.Structure):
    """kore_cuda_layer_weights."""
    _fields_ = ([(n, _QMat) for n in ("wq", "wk", "wv", "wo")]
                + [(n, ctypes.c_void_p) for n in ("bq", "bk", "bv", "attn_norm", "ffn_norm")]
                + [(n, _QMat) for n in ("w_gate", "w_up", "w_down")])


class _Model(ctypes.Structure):
    """kore_cuda_model."""
    _fields_ = [("n_ff", ctypes.c_int), ("n_vocab", ctypes.c_int), ("rms_eps", ctypes.c_float),
                ("tok_embd", _QMat), ("out_norm", ctypes.c_void_p), ("out_w", _QMat),
                ("layers", ctypes.POINTER(_LayerW))]


class _Event(ctypes.Structure):
    """kore_cuda_event."""
    _fields_ = [("session", ctypes.c_int), ("token", ctypes.c_int), ("status", ctypes.c_int)]


EV_TOKEN, EV_END, EV_FULL, EV_LIMIT = 0, 1, 2, 3


def _addr(a) -> int | None:
    """Host address of an array argument: an int is taken as an address, None as NULL."""
    if a is None or isinstance(a, int):
        return a
    if not (isinstance(a, np.ndarray) and a.flags.c_contiguous):
        raise ValueError("expected a C-contiguous numpy array or an address")
    return a.ctypes.data


def _qm(m) -> _QMat:
    """kore_cuda_qmat of a matrix with .type, .rows, .cols and .data (array) or .addr (address)."""
    addr = getattr(m, "addr", None)
    return _QMat(m.type, m.rows, m.cols, addr if addr is not None else _addr(m.data))


_lib = None
_vp = ctypes.c_void_p
_ip = ctypes.POINTER(ctypes.c_int)
_i = ctypes.c_int


def declared_symbols() -> list[str]:
    """Entry points declared in include/*.h (the ABI the library must export)."""
    names: list[str] = []
    for fn in sorted(os.listdir(INCLUDE)):
        if fn.endswith(".h"):
            src = open(os.path.join(INCLUDE, fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"\b(kore_cuda_\w+)\s*\(", src)
    return sorted(set(names))


def load_library(path: str | None = None):
    """Loads the C-ABI library once: `path`, else $KORE_CUDA_LIB (a build of
    the same sources with other compile-time shapes), else the in-tree build."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("KORE_CUDA_LIB") or LIB
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m kore_b200.build`")
    L = ctypes.CDLL(path)
    L.kore_cuda_cfg_default.argtypes = [ctypes.POINTER(_Cfg)] + [_i] * 5
    L.kore_cuda_cfg_default.restype = None
    L.kore_cuda_create.argtypes = [ctypes.POINTER(_vp), ctypes.POINTER(_Cfg)]
    L.kore_cuda_destroy.argtypes = [_vp]
    L.kore_cuda_destroy.restype = None
    L.kore_cuda_last_error.argtypes = [_vp]
    L.kore_cuda_last_error.restype = ctypes.c_char_p
    L.kore_cuda_seq_reset.argtypes = [_vp, _i]
    L.kore_cuda_seq_len.argtypes = [_vp, _i, _i]
    for n in ("kore_cuda_kv_append", "kore_cuda_kv_append_dev"):
        getattr(L, n).argtypes = [_vp, _i, _i, _i, _i, _vp, _vp]
    for n in ("kore_cuda_attn_prefill", "kore_cuda_attn_prefill_dev"):
        getattr(L, n).argtypes = [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp]
    for n in ("kore_cuda_attn_decode", "kore_cuda_attn_decode_dev"):
        getattr(L, n).argtypes = [_vp, _i, _i, _i, _vp, _vp, _vp, _vp]
    for n in ("kore_cuda_attn_decode_batch", "kore_cuda_attn_decode_batch_dev"):
        getattr(L, n).argtypes = [_vp, _i, _i, _ip, _ip, _vp, _vp, _vp, _vp]
    L.kore_cuda_attn_decode_partial_dev.argtypes = [_vp, _i, _i, _i, _vp, _vp, _vp, _vp]
    L.kore_cuda_lse_merge_dev.argtypes = [_vp, _i, _vp, _vp]
    L.kore_cuda_attn_prefill_partial_dev.argtypes = [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp]
    L.kore_cuda_lse_merge_batch_dev.argtypes = [_vp, _i, _i, _vp, _vp]
    L.kore_cuda_peer_handle.argtypes = [_vp, ctypes.c_char_p]
    L.kore_cuda_peer_open.argtypes = [_vp, ctypes.c_char_p]
    L.kore_cuda_attn_decode_sharded_dev.argtypes = [_vp, _i, _i, _i, _vp, _vp, _vp, _vp]
    L.kore_cuda_attn_decode_sharded.argtypes = [_vp, _i, _i, _i, _vp, _vp, _vp, _vp]
    L.kore_cuda_kv_read.argtypes = [_vp, _i, _i, _i, _i, _vp, _vp]
    L.kore_cuda_attn_decode_noalloc.argtypes = [ctypes.POINTER(KvView), _i, _vp, _vp, _vp, _vp, _vp, _vp]
    L.kore_cuda_set_attn_weights.argtypes = [_vp, _i] + [ctypes.POINTER(_QMat)] * 4 + [_vp] * 3
    L.kore_cuda_qmatvec.argtypes = [_vp, _i, _i, _vp, _vp]
    for n in ("kore_cuda_attn_block_decode", "kore_cuda_attn_block_decode_dev"):
        getattr(L, n).argtypes = [_vp, _i, _i, _i, _vp, _vp]
    L.kore_cuda_set_model.argtypes = [_vp, ctypes.POINTER(_Model)]
    L.kore_cuda_decode_step.argtypes = [_vp, _i, _i, _i, _ip, _vp]
    L.kore_cuda_decode_step_dev.argtypes = [_vp, _i, _vp, _i, _vp, _vp]
    L.kore_cuda_prefill.argtypes = [_vp, _i, _ip, _i, _i, _ip, _vp]
    L.kore_cuda_matmul_batch.argtypes = [_vp, _i, _i, _i, _vp, _vp]
    L.kore_cuda_seq_truncate.argtypes = [_vp, _i, _i]
    L.kore_cuda_server_create.argtypes = [ctypes.POINTER(_vp), _vp, _i, _i]
    L.kore_cuda_server_destroy.argtypes = [_vp]
    L.kore_cuda_server_destroy.restype = None
    L.kore_cuda_server_last_error.argtypes = [_vp]
    L.kore_cuda_server_last_error.restype = ctypes.c_char_p
    L.kore_cuda_server_open.argtypes = [_vp, _ip]
    L.kore_cuda_server_close.argtypes = [_vp, _i]
    L.kore_cuda_server_submit.argtypes = [_vp, _i, _ip, _i, _i]
    L.kore_cuda_server_step.argtypes = [_vp, ctypes.POINTER(_Event), _i, _ip]
    L.kore_cuda_server_condense.argtypes = [_vp, _i, _ip, _i]
    L.kore_cuda_server_history.argtypes = [_vp, _i, _ip, _i]
    L.kore_cuda_sync.argtypes = [_vp]
    L.kore_cuda_set_wait_limit.argtypes = [_vp, ctypes.c_ulonglong]
    L.kore_cuda_stream.argtypes = [_vp]
    L.kore_cuda_stream.restype = _vp
    L.kore_cuda_set_stream.argtypes = [_vp, _vp]
    _lib = L
    return L


def _host(a, n: int) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    if a.size != n:
        raise ValueError(f"expected {n} floats, got {a.size}")
    return a


def _dptr(t) -> int:
    """Device address of a contiguous fp32 CUDA tensor."""
    if not (t.is_cuda and t.dtype.__str__() == "torch.float32" and t.is_contiguous()):
        raise ValueError("expected a contiguous float32 CUDA tensor")
    return t.data_ptr()


class KoreCuda:
    """One attention context: the paged KV cache of every layer of a model,
    for up to ``max_seqs`` sequences, on one GPU (or one shard of the KV
    positions when ``shard_count`` > 1)."""

    def __init__(self, n_layer: int, n_head: int, n_head_kv: int, head_dim: int, ctx_max: int, *,
                 max_seqs: int = 1, page_tokens: int = 256, n_pages: int = 0, rope_base: float = 1e6,
                 inv_freq=None, device: int = 0, shard_rank: int = 0, shard_count: int = 1):
        L = load_library()
        cfg = _Cfg()
        L.kore_cuda_cfg_default(ctypes.byref(cfg), n_layer, n_head, n_head_kv, head_dim, ctx_max)
        cfg.max_seqs, cfg.page_tokens, cfg.n_pages = max_seqs, page_tokens, n_pages
        cfg.rope_base, cfg.device = rope_base, device
        cfg.shard_rank, cfg.shard_count = shard_rank, shard_count
        self._inv = None
        if inv_freq is not None:
            self._inv = np.ascontiguousarray(inv_freq, np.float32)
            cfg.inv_freq = self._inv.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        h = _vp()
        rc = L.kore_cuda_create(ctypes.byref(h), ctypes.byref(cfg))
        if rc:
            raise KoreCudaError(rc, L.kore_cuda_last_error(None).decode())
        self._h = h
        self._L = L
        self.n_layer, self.H, self.G, self.d, self.ctx_max = n_layer, n_head, n_head_kv, head_dim, ctx_max
        self.kvd = n_head_kv * head_dim

    # ---------------------------------------------------------------- plumbing
    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.kore_cuda_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _ck(self, rc: int) -> None:
        if rc:
            raise KoreCudaError(rc, self._L.kore_cuda_last_error(self._h).decode())

    def c_call(self, name: str):
        """The C-ABI entry point `name` bound to this context: f(*args) calls
        name(ctx, *args) with the arguments as given (raw host or device
        addresses as ints, as kore passes its own buffers) and raises
        KoreCudaError on a non-zero return. No numpy conversion or allocation
        per call: the caller owns every buffer."""
        fn, h, ck = getattr(self._L, name), self._h, self._ck

        def call(*args):
            rc = fn(h, *args)
            if rc:
                ck(rc)
        return call

    @property
    def handle(self) -> int:
        return self._h.value

    @property
    def stream(self) -> int:
        return self._L.kore_cuda_stream(self._h) or 0

    def set_stream(self, stream: int) -> None:
        self._ck(self._L.kore_cuda_set_stream(self._h, stream))

    def sync(self) -> None:
        self._ck(self._L.kore_cuda_sync(self._h))

    def set_wait_limit(self, seconds: float) -> None:
        """Limit of the decode and exchange kernels' bounded waits (0: the 2 s default)."""
        self._ck(self._L.kore_cuda_set_wait_limit(self._h, int(seconds * 1e9)))

    def seq_reset(self, seq: int) -> None:
        self._ck(self._L.kore_cuda_seq_reset(self._h, seq))

    def seq_truncate(self, seq: int, n: int) -> None:
        self._ck(self._L.kore_cuda_seq_truncate(self._h, seq, n))

    def seq_len(self, seq: int, layer: int) -> int:
        r = self._L.kore_cuda_seq_len(self._h, seq, layer)
        if r < 0:
            raise KoreCudaError(r, "seq/layer out of range")
        return r

    # ---------------------------------------------------------------- host buffers (kore's path)
    def append(self, seq: int, layer: int, pos0: int, k, v) -> None:
        k = np.ascontiguousarray(k, np.float32).reshape(-1, self.kvd)
        n = k.shape[0]
        v = _host(v, n * self.kvd)
        self._ck(self._L.kore_cuda_kv_append(self._h, seq, layer, pos0, n, k.ctypes.data, v.ctypes.data))

    def decode(self, seq: int, layer: int, pos: int, q, k, v) -> np.ndarray:
        q = _host(q, self.H * self.d)
        k = _host(k, self.kvd)
        v = _host(v, self.kvd)
        out = np.empty(self.H * self.d, np.float32)
        self._ck(self._L.kore_cuda_attn_decode(self._h, seq, layer, pos, q.ctypes.data, k.ctypes.data,
                                               v.ctypes.data, out.ctypes.data))
        return out.reshape(self.H, self.d)

    def decode_batch(self, layer: int, seqs, pos, q, k, v) -> np.ndarray:
        seqs = np.ascontiguousarray(seqs, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        n = seqs.size
        q = _host(q, n * self.H * self.d)
        k = _host(k, n * self.kvd)
        v = _host(v, n * self.kvd)
        out = np.empty(n * self.H * self.d, np.float32)
        self._ck(self._L.kore_cuda_attn_decode_batch(self._h, layer, n, seqs.ctypes.data_as(_ip),
                                                     pos.ctypes.data_as(_ip), q.ctypes.data, k.ctypes.data,
                                                     v.ctypes.data, out.ctypes.data))
        return out.reshape(n, self.H, self.d)

    def prefill(self, seq: int, layer: int, pos0: int, q, k, v) -> np.ndarray:
        q = np.ascontiguousarray(q, np.float32).reshape(-1, self.H * self.d)
        n = q.shape[0]
        k = _host(k, n * self.kvd)
        v = _host(v, n * self.kvd)
        out = np.empty((n, self.H * self.d), np.float32)
        self._ck(self._L.kore_cuda_attn_prefill(self._h, seq, layer, pos0, n, q.ctypes.data, k.ctypes.data,
                                                v.ctypes.data, out.ctypes.data))
        return out.reshape(n, self.H, self.d)

    def kv_read(self, seq: int, layer: int, pos0: int, n: int):
        k = np.zeros((n, self.kvd), np.float32)
        v = np.zeros((n, self.kvd), np.float32)
        self._ck(self._L.kore_cuda_kv_read(self._h, seq, layer, pos0, n, k.ctypes.data, v.ctypes.data))
        return k, v

    # ---------------------------------------------------------------- device tensors (stream-ordered)
    def append_dev(self, seq: int, layer: int, pos0: int, n: int, k, v) -> None:
        self._ck(self._L.kore_cuda_kv_append_dev(self._h, seq, layer, pos0, n, _dptr(k), _dptr(v)))

    def decode_dev(self, seq: int, layer: int, pos: int, q, k, v, out) -> None:
        self._ck(self._L.kore_cuda_attn_decode_dev(self._h, seq, layer, pos, _dptr(q), _dptr(k), _dptr(v),
                                                   _dptr(out)))

    def decode_batch_dev(self, layer: int, seqs, pos, q, k, v, out) -> None:
        seqs = np.ascontiguousarray(seqs, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        self._ck(self._L.kore_cuda_attn_decode_batch_dev(self._h, layer, seqs.size, seqs.ctypes.data_as(_ip),
                                                         pos.ctypes.data_as(_ip), _dptr(q), _dptr(k), _dptr(v),
                                                         _dptr(out)))

    def decode_partial_dev(self, seq: int, layer: int, pos: int, q, k, v, part) -> None:
        """KV-sharded decode: packed partial [H*d outputs][H log2-LSE] of this shard."""
        self._ck(self._L.kore_cuda_attn_decode_partial_dev(self._h, seq, layer, pos, _dptr(q), _dptr(k), _dptr(v),
                                                           _dptr(part)))

    def lse_merge_dev(self, n_parts: int, parts, out) -> None:
        self._ck(self._L.kore_cuda_lse_merge_dev(self._h, n_parts, _dptr(parts), _dptr(out)))

    def prefill_partial_dev(self, seq: int, layer: int, pos0: int, n: int, q, k, v, part) -> None:
        """KV-sharded prefill chunk: this shard's partial, outputs [n][H*d] then LSEs [n][H]."""
        self._ck(self._L.kore_cuda_attn_prefill_partial_dev(self._h, seq, layer, pos0, n, _dptr(q), _dptr(k), _dptr(v),
                                                            _dptr(part)))

    def lse_merge_batch_dev(self, n_parts: int, n_q: int, parts, out) -> None:
        self._ck(self._L.kore_cuda_lse_merge_batch_dev(self._h, n_parts, n_q, _dptr(parts), _dptr(out)))

    PEER_HANDLE_BYTES = 64

    def peer_handle(self) -> bytes:
        """This rank's exchange-buffer handle, to be given to every rank's peer_open."""
        buf = ctypes.create_string_buffer(self.PEER_HANDLE_BYTES)
        self._ck(self._L.kore_cuda_peer_handle(self._h, buf))
        return buf.raw

    def peer_open(self, handles: list[bytes]) -> None:
        blob = b"".join(handles)
        self._ck(self._L.kore_cuda_peer_open(self._h, ctypes.c_char_p(blob)))

    def decode_sharded_dev(self, seq: int, layer: int, pos: int, q, k, v, out) -> None:
        """KV-sharded decode with the exchange over peer memory: full output on every rank."""
        self._ck(self._L.kore_cuda_attn_decode_sharded_dev(self._h, seq, layer, pos, _dptr(q), _dptr(k),
                                                           _dptr(v), _dptr(out)))

    def decode_sharded(self, seq: int, layer: int, pos: int, q, k, v) -> np.ndarray:
        """KV-sharded decode with kore's host buffers: the merged output on every rank."""
        q = _host(q, self.H * self.d)
        k = _host(k, self.kvd)
        v = _host(v, self.kvd)
        out = np.empty(self.H * self.d, np.float32)
        self._ck(self._L.kore_cuda_attn_decode_sharded(self._h, seq, layer, pos, q.ctypes.data, k.ctypes.data,
                                                       v.ctypes.data, out.ctypes.data))
        return out.reshape(self.H, self.d)

    @property
    def part_floats(self) -> int:
        return self.H * self.d + self.H

    def prefill_dev(self, seq: int, layer: int, pos0: int, n: int, q, k, v, out) -> None:
        self._ck(self._L.kore_cuda_attn_prefill_dev(self._h, seq, layer, pos0, n, _dptr(q), _dptr(k), _dptr(v),
                                                    _dptr(out)))

    # ---------------------------------------------------------------- attention block with its projections
    def set_attn_weights(self, layer: int, wq, wk, wv, wo, bq=None, bk=None, bv=None) -> None:
        """Uploads one layer's Wq, Wk, Wv, Wo (``qweights.QMat``) and biases."""
        mats = [_QMat(m.type, m.rows, m.cols, m.data.ctypes.data) for m in (wq, wk, wv, wo)]
        keep = [m.data for m in (wq, wk, wv, wo)]
        if bq is None:
            b = [None, None, None]
        else:
            b = [_host(bq, self.H * self.d), _host(bk, self.kvd), _host(bv, self.kvd)]
        ptrs = [x.ctypes.data if x is not None else None for x in b]
        self._ck(self._L.kore_cuda_set_attn_weights(self._h, layer, *[ctypes.byref(m) for m in mats], *ptrs))
        del keep

    def qmatvec(self, layer: int, which: int, x) -> np.ndarray:
        """kore's mv() + quant() with an uploaded matrix (0 wq, 1 wk, 2 wv, 3 wo)."""
        rows = self.H * self.d if which in (0, 3) else self.kvd
        x = _host(x, self.H * self.d)
        out = np.empty(rows, np.float32)
        self._ck(self._L.kore_cuda_qmatvec(self._h, layer, which, x.ctypes.data, out.ctypes.data))
        return out

    def attn_block_decode(self, seq: int, layer: int, pos: int, xb) -> np.ndarray:
        """kore.cpp:1419-1457 for one token: xb [n_embd] -> Wo*att [n_embd]."""
        xb = _host(xb, self.H * self.d)
        o = np.empty(self.H * self.d, np.float32)
        self._ck(self._L.kore_cuda_attn_block_decode(self._h, seq, layer, pos, xb.ctypes.data, o.ctypes.data))
        return o

    # ---------------------------------------------------------------- the whole decode step
    def set_model(self, n_ff: int, n_vocab: int, rms_eps: float, tok_embd, out_norm, out_w, layers) -> None:
        """Uploads the whole model. tok_embd/out_w and the layers' matrices have
        .type/.rows/.cols and .data (uint8 array) or .addr; out_norm and each
        layer's attn_norm, ffn_norm, bq, bk, bv are float32 arrays or addresses.
        layers: one dict per layer with keys wq wk wv wo w_gate w_up w_down
        bq bk bv attn_norm ffn_norm."""
        arr = (_LayerW * len(layers))()
        keep = []
        for i, Lw in enumerate(layers):
            vals = {k: Lw[k] for k in Lw}
            keep.append(vals)
            arr[i] = _LayerW(*[_qm(vals[n]) for n in ("wq", "wk", "wv", "wo")],
                             *[_addr(vals.get(n)) for n in ("bq", "bk", "bv", "attn_norm", "ffn_norm")],
                             *[_qm(vals[n]) for n in ("w_gate", "w_up", "w_down")])
        m = _Model(n_ff, n_vocab, rms_eps, _qm(tok_embd), _addr(out_norm), _qm(out_w), arr)
        self._ck(self._L.kore_cuda_set_model(self._h, ctypes.byref(m)))
        self.n_vocab = n_vocab
        del keep

    def decode_step(self, seq: int, token: int, pos: int, want_logits: bool = False):
        """kore's forward() + greedy sample_token for one token: (next token, logits or None)."""
        nxt = ctypes.c_int(-1)
        logits = np.empty(self.n_vocab, np.float32) if want_logits else None
        self._ck(self._L.kore_cuda_decode_step(self._h, seq, token, pos, ctypes.byref(nxt),
                                               logits.ctypes.data if want_logits else None))
        return nxt.value, logits

    def prefill_tokens(self, seq: int, tokens, pos0: int, want_logits: bool = False):
        """kore's forward_batch() of prompt tokens at pos0.. on the device: (next token, logits or None)."""
        toks = np.ascontiguousarray(tokens, np.int32)
        nxt = ctypes.c_int(-1)
        logits = np.empty(self.n_vocab, np.float32) if want_logits else None
        self._ck(self._L.kore_cuda_prefill(self._h, seq, toks.ctypes.data_as(_ip), toks.size, pos0, ctypes.byref(nxt),
                                           logits.ctypes.data if want_logits else None))
        return nxt.value, logits

    def matmul_batch(self, layer: int, which: int, x, rows: int) -> np.ndarray:
        """kore's matmul_batch_float of rows x [B][cols] with an uploaded matrix: [B][rows]."""
        x = np.ascontiguousarray(x, np.float32)
        B = x.shape[0]
        out = np.empty((B, rows), np.float32)
        self._ck(self._L.kore_cuda_matmul_batch(self._h, layer, which, B, x.ctypes.data, out.ctypes.data))
        return out

    def decode_step_dev(self, seq: int, token, pos: int, next_token, logits=None) -> None:
        """Stream-ordered step: token / next_token are int32 CUDA tensors of one element."""
        for t in (token, next_token):
            if not (t.is_cuda and str(t.dtype) == "torch.int32"):
                raise ValueError("token and next_token must be int32 CUDA tensors")
        self._ck(self._L.kore_cuda_decode_step_dev(self._h, seq, token.data_ptr(), pos, next_token.data_ptr(),
                                                   _dptr(logits) if logits is not None else None))

    def attn_block_decode_dev(self, seq: int, layer: int, pos: int, xb, o) -> None:
        self._ck(self._L.kore_cuda_attn_block_decode_dev(self._h, seq, layer, pos, _dptr(xb), _dptr(o)))


class Server:
    """Many chat sessions over one KoreCuda context with its model uploaded
    (kore_cuda_server_*): kore's ChatSession / prefill() / gen_step() /
    condense() with every session a sequence of the shared page pool."""

    def __init__(self, ctx: KoreCuda, eos: int = -1, bos: int = -1):
        self._L = ctx._L
        self.ctx = ctx
        h = _vp()
        rc = self._L.kore_cuda_server_create(ctypes.byref(h), ctx._h, eos, bos)
        if rc:
            raise KoreCudaError(rc, self._L.kore_cuda_server_last_error(None).decode())
        self._h = h
        self._ev = (_Event * 4096)()

    def _ck(self, rc: int) -> None:
        if rc:
            raise KoreCudaError(rc, self._L.kore_cuda_server_last_error(self._h).decode())

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.kore_cuda_server_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def open(self) -> int:
        s = ctypes.c_int(-1)
        self._ck(self._L.kore_cuda_server_open(self._h, ctypes.byref(s)))
        return s.value

    def close_session(self, session: int) -> None:
        self._ck(self._L.kore_cuda_server_close(self._h, session))

    def submit(self, session: int, ids, max_new: int = 0) -> None:
        ids = np.ascontiguousarray(ids, np.int32)
        self._ck(self._L.kore_cuda_server_submit(self._h, session, ids.ctypes.data_as(_ip), ids.size, max_new))

    def step(self) -> list[tuple[int, int, int]]:
        """One round: [(session, token, status)] for every session that was generating."""
        n = ctypes.c_int(0)
        self._ck(self._L.kore_cuda_server_step(self._h, self._ev, len(self._ev), ctypes.byref(n)))
        return [(self._ev[i].session, self._ev[i].token, self._ev[i].status) for i in range(n.value)]

    def condense(self, session: int, ids) -> None:
        ids = np.ascontiguousarray(ids, np.int32)
        self._ck(self._L.kore_cuda_server_condense(self._h, session, ids.ctypes.data_as(_ip), ids.size))

    def history(self, session: int) -> list[int]:
        n = self._L.kore_cuda_server_history(self._h, session, None, 0)
        if n < 0:
            raise KoreCudaError(n, "session not open")
        buf = np.zeros(max(n, 1), np.int32)
        self._L.kore_cuda_server_history(self._h, session, buf.ctypes.data_as(_ip), n)
        return buf[:n].tolist()
