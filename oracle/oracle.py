"""ctypes access to the checkers — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module. It loads

* ``oracle/_build/libkore_oracle.so`` — the C restatements of kore's attention
  (kore_attn_oracle.c) and of its Q8_K / Q4_K / Q6_K projections
  (kore_proj_oracle.c), and
* ``oracle/_ref/libkore_ref.so`` — the reference engine itself (kore.cpp,
  compiled in place by oracle/Makefile) driven through ref_harness.cpp, and
* ``oracle/_ref/libkore_engine.so`` — the reference engine with
  engine_harness.cpp: greedy decoding on a random-init model, by kore and by
  kore with its attention regions on the CUDA library.

Both are built by ``make -C oracle``; the reference library is optional (it
needs the reference sources at build time) and ``ref_available()`` says
whether it is present.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libkore_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libkore_ref.so")
ENGINE_SO = os.path.join(HERE, "_ref", "libkore_engine.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_oracle = None
_ref = None


def build(ref_dir: str | None = None) -> None:
    """Compile the restatement and, when a reference checkout is named (the
    argument, else the KORE_REF_DIR environment variable) and holds kore.cpp,
    the reference harness. Without one the prebuilt oracle/_ref libraries, if
    any, stay as they are."""
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
    ref_dir = ref_dir or os.environ.get("KORE_REF_DIR")
    if not ref_dir:
        print("oracle: KORE_REF_DIR is not set; the reference harness (oracle/_ref) is not rebuilt")
        return
    if not os.path.exists(os.path.join(ref_dir, "kore.cpp")):
        raise FileNotFoundError(f"KORE_REF_DIR={ref_dir} holds no kore.cpp")
    subprocess.run(["make", "-s", "-C", HERE, "ref", f"KORE_REF_DIR={ref_dir}"], check=True)


class KorcQW(ctypes.Structure):
    """korc_qw (kore_step_oracle.h)."""
    _fields_ = [("type", ctypes.c_int), ("rows", ctypes.c_int), ("cols", ctypes.c_int), ("data", ctypes.c_void_p)]


class KorcLayer(ctypes.Structure):
    """korc_layer (kore_step_oracle.h)."""
    _fields_ = [("attn_norm", ctypes.c_void_p), ("ffn_norm", ctypes.c_void_p), ("bq", ctypes.c_void_p),
                ("bk", ctypes.c_void_p), ("bv", ctypes.c_void_p)] + \
               [(n, KorcQW) for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")]


class KorcModel(ctypes.Structure):
    """korc_model (kore_step_oracle.h)."""
    _fields_ = [("n_layer", ctypes.c_int), ("n_embd", ctypes.c_int), ("n_ff", ctypes.c_int),
                ("n_head", ctypes.c_int), ("n_head_kv", ctypes.c_int), ("n_vocab", ctypes.c_int),
                ("rms_eps", ctypes.c_float), ("tok_embd", ctypes.c_void_p), ("out_norm", ctypes.c_void_p),
                ("out_w", KorcQW), ("layers", ctypes.POINTER(KorcLayer)), ("inv_freq", ctypes.c_void_p)]


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def lib():
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        L.korc_inv_freq.argtypes = [ctypes.c_float, ctypes.c_int, _f32p]
        L.korc_rope_angles.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p, _f32p]
        L.korc_rope_key.argtypes = [ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int, _f32p, _f32p]
        L.korc_cpu_has_avx2.restype = ctypes.c_int
        L.korc_hd_dot.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.korc_hd_dot.restype = ctypes.c_float
        L.korc_attn_decode.argtypes = [ctypes.c_int] * 3 + [_f32p, ctypes.c_int] + [_f32p] * 7
        L.korc_attn_prefill.argtypes = ([ctypes.c_int] * 3 + [_f32p, ctypes.c_int, ctypes.c_int]
                                        + [_f32p] * 7 + [ctypes.c_int])
        L.korc_argmax.argtypes = [_f32p, ctypes.c_int]
        vp = ctypes.c_void_p
        L.korc_q8k_quantize.argtypes = [vp, ctypes.c_int, vp, vp, vp]
        for n in ("korc_dot_q4k", "korc_dot_q6k"):
            getattr(L, n).argtypes = [ctypes.c_int, vp, vp, vp, vp, ctypes.c_int]
            getattr(L, n).restype = ctypes.c_float
        L.korc_qmatvec.argtypes = [ctypes.c_int] * 3 + [vp] * 4 + [ctypes.c_int]
        L.korc_decode_step.argtypes = [ctypes.POINTER(KorcModel), vp, vp, ctypes.c_int, ctypes.c_int, vp, ctypes.c_int]
        _oracle = L
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib():
    global _ref
    if _ref is None:
        L = ctypes.CDLL(REF_SO)
        L.kref_create.argtypes = [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_int]
        L.kref_create.restype = ctypes.c_void_p
        L.kref_destroy.argtypes = [ctypes.c_void_p]
        L.kref_avx2.argtypes = [ctypes.c_void_p]
        L.kref_ctx.argtypes = [ctypes.c_void_p]
        L.kref_inv_freq.argtypes = [ctypes.c_void_p]
        L.kref_inv_freq.restype = _f32p
        L.kref_kcache.argtypes = [ctypes.c_void_p]
        L.kref_kcache.restype = _f32p
        L.kref_vcache.argtypes = [ctypes.c_void_p]
        L.kref_vcache.restype = _f32p
        L.kref_fill.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _f32p, _f32p]
        L.kref_decode.argtypes = [ctypes.c_void_p, ctypes.c_int, _f32p, _f32p, _f32p, _f32p]
        L.kref_prefill.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _f32p, _f32p, _f32p, _f32p]
        L.kref_argmax.argtypes = [_f32p, ctypes.c_int]
        L.kref_now_ms.restype = ctypes.c_double
        vp = ctypes.c_void_p
        L.kref_q8k_quantize.argtypes = [vp, ctypes.c_int, vp, vp, vp]
        L.kref_qdot.argtypes = [ctypes.c_int, ctypes.c_int, vp, vp, vp, vp, ctypes.c_int]
        L.kref_qdot.restype = ctypes.c_float
        L.kref_qmatvec_ms.argtypes = [ctypes.c_int] * 3 + [vp] * 3 + [ctypes.c_int] * 2
        L.kref_qmatvec_ms.restype = ctypes.c_double
        _ref = L
    return _ref


# ----------------------------------------------------------------- projections (kore_proj_oracle.c)

def _q8k_call(fn, x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    n = x.size
    d = np.zeros(n // 256, np.float32)
    qs = np.zeros(n, np.int8)
    bs = np.zeros(n // 16, np.int16)
    fn(x.ctypes.data, n, d.ctypes.data, qs.ctypes.data, bs.ctypes.data)
    return d, qs, bs


def q8k_quantize(x: np.ndarray):
    """kore.cpp:422-447 restated: (d [n/256], qs [n] int8, bsums [n/16] int16)."""
    return _q8k_call(lib().korc_q8k_quantize, x)


def ref_q8k_quantize(x: np.ndarray):
    """The reference's own quantize_row_q8_K."""
    return _q8k_call(ref_lib().kref_q8k_quantize, x)


def qdot(qtype: int, wrow: np.ndarray, xq, avx2: bool = True) -> np.float32:
    """One row (uint8 blocks) against Q8_K xq, restated (AVX2 lane order or scalar)."""
    d, qs, bs = xq
    fn = lib().korc_dot_q4k if qtype == 12 else lib().korc_dot_q6k
    return np.float32(fn(qs.size, wrow.ctypes.data, d.ctypes.data, qs.ctypes.data, bs.ctypes.data, int(avx2)))


def ref_qdot(qtype: int, wrow: np.ndarray, xq, avx2: bool = True) -> np.float32:
    """The reference's own dot_q4_K_q8_K / dot_q6_K_q8_K (its AVX2 kernel if avx2 and the CPU has it)."""
    d, qs, bs = xq
    return np.float32(ref_lib().kref_qdot(qtype, qs.size, wrow.ctypes.data, d.ctypes.data, qs.ctypes.data,
                                          bs.ctypes.data, int(avx2)))


def ref_qmatvec_ms(m, x: np.ndarray, threads: int = 1, reps: int = 3):
    """kore's own quantize + matvec_mt of m with x: (best ms, output)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    out = np.empty(m.rows, np.float32)
    ms = ref_lib().kref_qmatvec_ms(m.type, m.rows, m.cols, m.data.ctypes.data, x.ctypes.data, out.ctypes.data,
                                   threads, reps)
    return ms, out


def qmatvec(m, x: np.ndarray, bias=None, avx2: bool = True) -> np.ndarray:
    """kore's mv() + quant() (+ bias) restated: m has .type, .rows, .cols, .data (uint8)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    assert x.size == m.cols
    out = np.empty(m.rows, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    rc = lib().korc_qmatvec(m.type, m.rows, m.cols, m.data.ctypes.data, x.ctypes.data,
                            None if b is None else b.ctypes.data, out.ctypes.data, int(avx2))
    assert rc == 0
    return out


# ----------------------------------------------------------------- restatement

def inv_freq(rope_base: float, head_dim: int) -> np.ndarray:
    out = np.empty(head_dim // 2, np.float32)
    lib().korc_inv_freq(rope_base, head_dim, _fp(out))
    return out


def rope_angles(inv: np.ndarray, pos: int):
    half = inv.shape[0]
    c = np.empty(half, np.float32)
    s = np.empty(half, np.float32)
    lib().korc_rope_angles(_fp(inv), half, pos, _fp(c), _fp(s))
    return c, s


def rope_keys(G: int, d: int, inv: np.ndarray, pos0: int, k_pre: np.ndarray) -> np.ndarray:
    """Post-RoPE key rows as kore stores them, for positions pos0.. ."""
    k_pre = np.ascontiguousarray(k_pre, np.float32).reshape(-1, G * d)
    out = np.empty_like(k_pre)
    for z in range(k_pre.shape[0]):
        lib().korc_rope_key(G, d, _fp(inv), pos0 + z, _fp(k_pre[z]), _fp(out[z]))
    return out


def cpu_has_avx2() -> bool:
    return bool(lib().korc_cpu_has_avx2())


class OracleLayer:
    """One layer's fp32 KV cache, [ctx][G*d] rows, in kore's layout
    (kore.cpp:1260, :1344-1345), driven by the restated decode/prefill."""

    def __init__(self, H: int, G: int, d: int, ctx: int, rope_base: float = 1e6):
        self.H, self.G, self.d, self.ctx = H, G, d, ctx
        self.inv = inv_freq(rope_base, d)
        self.kc = np.zeros((ctx, G * d), np.float32)
        self.vc = np.zeros((ctx, G * d), np.float32)

    def fill(self, pos0: int, k_pre: np.ndarray, v: np.ndarray) -> None:
        n = k_pre.shape[0]
        self.kc[pos0:pos0 + n] = rope_keys(self.G, self.d, self.inv, pos0, k_pre)
        self.vc[pos0:pos0 + n] = v.reshape(n, -1)

    def decode(self, pos: int, q, k, v) -> np.ndarray:
        q = np.ascontiguousarray(q, np.float32).reshape(-1)
        k = np.ascontiguousarray(k, np.float32).reshape(-1)
        v = np.ascontiguousarray(v, np.float32).reshape(-1)
        out = np.empty(self.H * self.d, np.float32)
        scores = np.empty(pos + 1, np.float32)
        rc = lib().korc_attn_decode(self.H, self.G, self.d, _fp(self.inv), pos, _fp(q), _fp(k), _fp(v),
                                    _fp(self.kc), _fp(self.vc), _fp(out), _fp(scores))
        if rc:
            raise ValueError("korc_attn_decode: bad arguments")
        return out.reshape(self.H, self.d)

    def prefill(self, pos0: int, q, k, v, avx2: bool | None = None) -> np.ndarray:
        n = q.shape[0]
        q = np.ascontiguousarray(q, np.float32).reshape(n, -1)
        k = np.ascontiguousarray(k, np.float32).reshape(n, -1)
        v = np.ascontiguousarray(v, np.float32).reshape(n, -1)
        out = np.empty((n, self.H * self.d), np.float32)
        scratch = np.empty(pos0 + n + n * self.H * self.d, np.float32)
        if avx2 is None:
            avx2 = cpu_has_avx2()
        rc = lib().korc_attn_prefill(self.H, self.G, self.d, _fp(self.inv), pos0, n, _fp(q), _fp(k), _fp(v),
                                     _fp(self.kc), _fp(self.vc), _fp(out), _fp(scratch), int(avx2))
        if rc:
            raise ValueError("korc_attn_prefill: bad arguments")
        return out.reshape(n, self.H, self.d)


class RefLayer:
    """The same, but running the reference engine's own forward()/forward_batch()
    (oracle/_ref/libkore_ref.so)."""

    def __init__(self, H: int, G: int, d: int, ctx: int, rope_base: float = 1e6, threads: int = 1):
        self.H, self.G, self.d, self.ctx = H, G, d, ctx
        self.h = ref_lib().kref_create(H, G, d, ctx, rope_base, threads)
        if not self.h:
            raise RuntimeError("kore engine_init refused the shape")
        kvd = G * d
        self.kc = np.ctypeslib.as_array(ref_lib().kref_kcache(self.h), shape=(ctx, kvd))
        self.vc = np.ctypeslib.as_array(ref_lib().kref_vcache(self.h), shape=(ctx, kvd))

    def __del__(self):
        h = getattr(self, "h", None)
        if h:
            ref_lib().kref_destroy(h)
            self.h = None

    @property
    def avx2(self) -> bool:
        return bool(ref_lib().kref_avx2(self.h))

    def fill(self, pos0: int, k_pre: np.ndarray, v: np.ndarray) -> None:
        k_pre = np.ascontiguousarray(k_pre, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        if ref_lib().kref_fill(self.h, pos0, k_pre.shape[0], _fp(k_pre), _fp(v)):
            raise ValueError("kref_fill: out of range")

    def decode(self, pos: int, q, k, v) -> np.ndarray:
        q = np.ascontiguousarray(q, np.float32).reshape(-1)
        k = np.ascontiguousarray(k, np.float32).reshape(-1)
        v = np.ascontiguousarray(v, np.float32).reshape(-1)
        out = np.empty(self.H * self.d, np.float32)
        if ref_lib().kref_decode(self.h, pos, _fp(q), _fp(k), _fp(v), _fp(out)):
            raise ValueError("kore forward() returned false")
        return out.reshape(self.H, self.d)

    def prefill(self, pos0: int, q, k, v) -> np.ndarray:
        n = q.shape[0]
        q = np.ascontiguousarray(q, np.float32).reshape(n, -1)
        k = np.ascontiguousarray(k, np.float32).reshape(n, -1)
        v = np.ascontiguousarray(v, np.float32).reshape(n, -1)
        out = np.empty((n, self.H * self.d), np.float32)
        if ref_lib().kref_prefill(self.h, pos0, n, _fp(q), _fp(k), _fp(v), _fp(out)):
            raise ValueError("kore forward_batch() returned false")
        return out.reshape(n, self.H, self.d)


def seeded_inputs(seed: int, *shapes):
    """N(0,1) fp32 arrays from one numpy Generator (PCG64) seeded with `seed`."""
    g = np.random.default_rng(seed)
    return [g.standard_normal(s, dtype=np.float32) for s in shapes]


_engine = None


def engine_available() -> bool:
    return os.path.exists(ENGINE_SO)


def engine_lib():
    global _engine
    if _engine is None:
        L = ctypes.CDLL(ENGINE_SO)
        vp, ip, fp = ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_float)
        L.keng_create.restype = vp
        L.keng_create.argtypes = [ctypes.c_int] * 7 + [ctypes.c_ulonglong, ctypes.c_int]
        L.keng_destroy.argtypes = [vp]
        L.keng_error.restype = ctypes.c_char_p
        L.keng_error.argtypes = [vp]
        L.keng_ctx.argtypes = [vp]
        L.keng_chunk.argtypes = [vp]
        L.keng_generate_ref.argtypes = [vp, ip, ctypes.c_int, ctypes.c_int, ip, fp]
        L.keng_attach_cuda.argtypes = [vp, ctypes.c_char_p, ctypes.c_int]
        L.keng_generate_cuda.argtypes = [vp, ip, ctypes.c_int, ctypes.c_int, ip]
        L.keng_generate_cuda_block.argtypes = [vp, ip, ctypes.c_int, ctypes.c_int, ip]
        L.keng_generate_cuda_step.argtypes = [vp, ip, ctypes.c_int, ctypes.c_int, ip]
        L.keng_get_row.argtypes = [ctypes.c_int] * 3 + [vp, ctypes.c_int, fp]
        L.keng_forward_batch.argtypes = [vp, ip, ctypes.c_int, ctypes.c_int, fp]
        L.keng_turn_ref.argtypes = [vp, ip, ctypes.c_int, ctypes.c_int, ctypes.c_int, ip]
        L.keng_forward_cuda.argtypes = [vp, ctypes.c_int, ctypes.c_int, fp]
        L.keng_forward_batch_cuda.argtypes = [vp, ip, ctypes.c_int, ctypes.c_int, fp]
        L.keng_matmul_batch.argtypes = [vp] + [ctypes.c_int] * 3 + [vp, fp, ctypes.c_int, fp]
        L.keng_forward.argtypes = [vp, ctypes.c_int, ctypes.c_int, fp]
        L.keng_tensor.argtypes = [vp, ctypes.c_char_p, ip, ip, ip]
        L.keng_tensor.restype = vp
        L.keng_inv_freq.argtypes = [vp]
        L.keng_inv_freq.restype = vp
        L.keng_avx2.argtypes = [vp]
        L.keng_rms_eps.argtypes = [vp]
        L.keng_rms_eps.restype = ctypes.c_float
        _engine = L
    return _engine


class GreedyEngine:
    """A seeded random-init Qwen2-style model inside the reference engine, with
    greedy generation by kore itself (``generate_ref``), by kore with its
    attention on the CUDA library (``generate_cuda``, after ``attach_cuda``)
    and by kore with each decode step's whole attention block, projections
    included, on the CUDA library (``generate_cuda_block``)."""

    def __init__(self, n_layer: int, n_embd: int, n_head: int, n_head_kv: int, n_ff: int, n_vocab: int,
                 ctx: int, seed: int = 12345, threads: int = 0):
        threads = threads or os.cpu_count() or 1
        self.n_vocab = n_vocab
        self.h = engine_lib().keng_create(n_layer, n_embd, n_head, n_head_kv, n_ff, n_vocab, ctx, seed, threads)
        if not self.h:
            raise RuntimeError("kore engine_init refused the model")

    def __del__(self):
        h = getattr(self, "h", None)
        if h:
            engine_lib().keng_destroy(h)
            self.h = None

    @property
    def chunk(self) -> int:
        return engine_lib().keng_chunk(self.h)

    def _err(self) -> str:
        return engine_lib().keng_error(self.h).decode()

    def generate_ref(self, prompt, n_gen: int):
        p = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(n_gen, np.int32)
        margins = np.zeros(n_gen, np.float32)
        ip = ctypes.POINTER(ctypes.c_int)
        if engine_lib().keng_generate_ref(self.h, p.ctypes.data_as(ip), len(p), n_gen, ids.ctypes.data_as(ip),
                                          _fp(margins)) != n_gen:
            raise RuntimeError(self._err())
        return ids, margins

    def attach_cuda(self, lib_path: str, device: int = 0) -> None:
        if engine_lib().keng_attach_cuda(self.h, lib_path.encode(), device):
            raise RuntimeError(self._err())

    def generate_cuda(self, prompt, n_gen: int):
        p = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(n_gen, np.int32)
        ip = ctypes.POINTER(ctypes.c_int)
        if engine_lib().keng_generate_cuda(self.h, p.ctypes.data_as(ip), len(p), n_gen, ids.ctypes.data_as(ip)) != n_gen:
            raise RuntimeError(self._err())
        return ids

    def generate_cuda_block(self, prompt, n_gen: int):
        p = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(n_gen, np.int32)
        ip = ctypes.POINTER(ctypes.c_int)
        if engine_lib().keng_generate_cuda_block(self.h, p.ctypes.data_as(ip), len(p), n_gen,
                                                 ids.ctypes.data_as(ip)) != n_gen:
            raise RuntimeError(self._err())
        return ids

    def generate_cuda_step(self, prompt, n_gen: int):
        """Greedy IDs with the prompt through the CUDA attention path and every
        decode step wholly on the GPU (kore_cuda_decode_step)."""
        p = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(n_gen, np.int32)
        ip = ctypes.POINTER(ctypes.c_int)
        if engine_lib().keng_generate_cuda_step(self.h, p.ctypes.data_as(ip), len(p), n_gen,
                                                ids.ctypes.data_as(ip)) != n_gen:
            raise RuntimeError(self._err())
        return ids

    # ---- the reference's own decode step and model, for pinning the step restatement
    def forward_ref(self, token: int, pos: int) -> np.ndarray:
        """kore's forward() of one token at pos (positions in order from 0): its logits."""
        out = np.empty(self.n_vocab, np.float32)
        if engine_lib().keng_forward(self.h, token, pos, _fp(out)):
            raise RuntimeError("kore forward() refused the token or position")
        return out

    def forward_batch_ref(self, tokens, pos0: int) -> np.ndarray:
        """kore's forward_batch() of up to e.bsz tokens at pos0: the last token's logits."""
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(self.n_vocab, np.float32)
        if engine_lib().keng_forward_batch(self.h, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), t.size, pos0,
                                           _fp(out)):
            raise RuntimeError("kore forward_batch() refused the tokens or positions")
        return out

    def forward_cuda(self, token: int, pos: int) -> np.ndarray:
        """kore's forward() with its attention on the attached CUDA context: the logits."""
        out = np.empty(self.n_vocab, np.float32)
        if engine_lib().keng_forward_cuda(self.h, token, pos, _fp(out)):
            raise RuntimeError(self._err() or "kore forward() with CUDA attention failed")
        return out

    def forward_batch_cuda(self, tokens, pos0: int) -> np.ndarray:
        """kore's forward_batch() with its attention on the attached CUDA context: the last logits."""
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(self.n_vocab, np.float32)
        if engine_lib().keng_forward_batch_cuda(self.h, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), t.size, pos0,
                                                _fp(out)):
            raise RuntimeError(self._err() or "kore forward_batch() with CUDA attention failed")
        return out

    def turn_ref(self, ids, base: int, n_gen: int) -> list[int]:
        """kore's prefill() of ids at base, then n_gen greedy gen_step()s: the generated ids."""
        t = np.ascontiguousarray(ids, np.int32)
        out = np.zeros(max(n_gen, 1), np.int32)
        ip = ctypes.POINTER(ctypes.c_int)
        if engine_lib().keng_turn_ref(self.h, t.ctypes.data_as(ip), t.size, base, n_gen, out.ctypes.data_as(ip)) != n_gen:
            raise RuntimeError("kore refused the turn")
        return out[:n_gen].tolist()

    def matmul_batch_ref(self, m, x: np.ndarray) -> np.ndarray:
        """kore's matmul_batch_float of rows x [B][cols] with matrix m (.type .rows .cols, .data or .addr)."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty((x.shape[0], m.rows), np.float32)
        addr = getattr(m, "addr", None)
        addr = addr if addr is not None else m.data.ctypes.data
        # kore's kernel takes at most KORE_BMAX = 64 rows at a time (kore.cpp:690); every
        # output row depends on its own input row only
        for b0 in range(0, x.shape[0], 64):
            xs = np.ascontiguousarray(x[b0:b0 + 64])
            os_ = np.empty((xs.shape[0], m.rows), np.float32)
            engine_lib().keng_matmul_batch(self.h, m.type, m.rows, m.cols, addr, _fp(xs), xs.shape[0], _fp(os_))
            out[b0:b0 + xs.shape[0]] = os_
        return out

    def tensor(self, name: str):
        """(type, rows, cols, data address) of one of the model's tensors."""
        t, r, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        p = engine_lib().keng_tensor(self.h, name.encode(), ctypes.byref(t), ctypes.byref(r), ctypes.byref(c))
        if not p:
            raise KeyError(name)
        return t.value, r.value, c.value, p


def ref_get_row(qtype: int, rows: int, cols: int, data, row: int) -> np.ndarray:
    """kore's own get_row (kore.cpp:384-407) of a table (uint8 array or address)."""
    out = np.empty(cols, np.float32)
    addr = data if isinstance(data, int) else np.ascontiguousarray(data).ctypes.data
    if engine_lib().keng_get_row(qtype, rows, cols, addr, row, _fp(out)):
        raise ValueError("kore's get_row refused the table or row")
    return out


class StepOracle:
    """The step restatement (korc_decode_step) over a GreedyEngine's own
    weights, with its own per-layer KV cache."""

    def __init__(self, eng: GreedyEngine, n_layer: int, n_embd: int, n_head: int, n_head_kv: int, n_ff: int,
                 n_vocab: int, ctx: int):
        L = engine_lib()
        kvd = n_head_kv * (n_embd // n_head)

        def qw(name):
            t, r, c, p = eng.tensor(name)
            return KorcQW(t, r, c, p)

        def f32(name):
            return eng.tensor(name)[3]

        self.layers = (KorcLayer * n_layer)()
        for l in range(n_layer):
            b = f"blk.{l}."
            self.layers[l] = KorcLayer(f32(b + "attn_norm.weight"), f32(b + "ffn_norm.weight"),
                                       f32(b + "attn_q.bias"), f32(b + "attn_k.bias"), f32(b + "attn_v.bias"),
                                       *[qw(b + n + ".weight") for n in ("attn_q", "attn_k", "attn_v", "attn_output",
                                                                           "ffn_gate", "ffn_up", "ffn_down")])
        self.model = KorcModel(n_layer, n_embd, n_ff, n_head, n_head_kv, n_vocab, L.keng_rms_eps(eng.h),
                               f32("token_embd.weight"), f32("output_norm.weight"), qw("output.weight"),
                               self.layers, L.keng_inv_freq(eng.h))
        self.avx2 = L.keng_avx2(eng.h)
        self.kc = [np.zeros((ctx, kvd), np.float32) for _ in range(n_layer)]
        self.vc = [np.zeros((ctx, kvd), np.float32) for _ in range(n_layer)]
        self._kp = (ctypes.c_void_p * n_layer)(*[a.ctypes.data for a in self.kc])
        self._vp = (ctypes.c_void_p * n_layer)(*[a.ctypes.data for a in self.vc])
        self.n_vocab = n_vocab
        self.eng = eng   # keeps the weights alive

    def step(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.n_vocab, np.float32)
        if lib().korc_decode_step(ctypes.byref(self.model), self._kp, self._vp, token, pos, out.ctypes.data,
                                  self.avx2):
            raise RuntimeError("korc_decode_step refused its arguments")
        return out
