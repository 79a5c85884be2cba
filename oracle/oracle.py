"""ctypes wrapper of the CPU oracle (liboracle.so).

Test infrastructure only: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, always as the checker or the
CPU baseline, never as the thing the GPU path calls.
"""
import ctypes as C
import os

import numpy as np

from . import build as _build

_lib = None

F32, Q4_0, Q8_0, BF16 = 0, 2, 8, 30
BLOCK_BYTES = {Q8_0: 34, Q4_0: 18, BF16: 64}

_fp = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_u32p = C.POINTER(C.c_uint32)


class Config(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_blocks", "embed_dim", "ffn_dim", "n_heads", "n_kv_heads",
                                       "head_dim", "vocab_size", "context_length")] + [
        ("rope_base", C.c_float), ("rms_eps", C.c_float),
        ("bos_token_id", C.c_uint32), ("eos_token_id", C.c_uint32), ("weight_type", C.c_int)]


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = C.CDLL(path)
        sig = {
            "or_f16_to_f32": (C.c_float, [C.c_uint16]),
            "or_f32_to_f16": (C.c_uint16, [C.c_float]),
            "or_dequantize": (None, [C.c_int, _u8p, C.c_size_t, _fp]),
            "or_quantize_row_q8_0": (None, [_fp, C.c_size_t, _u8p]),
            "or_dot_f32_q8_0": (C.c_float, [_fp, _u8p, C.c_size_t]),
            "or_dot_f32_q4_0": (C.c_float, [_fp, _u8p, C.c_size_t]),
            "or_dot_f32_bf16": (C.c_float, [_fp, _u8p, C.c_size_t]),
            "or_dot_q8_0_q8_0": (C.c_float, [_u8p, _u8p, C.c_size_t]),
            "or_dot_q8_0_q4_0": (C.c_float, [_u8p, _u8p, C.c_size_t]),
            "or_dot_f32_f32": (C.c_float, [_fp, _fp, C.c_size_t]),
            "or_linear": (C.c_int, [_fp, C.c_int, C.c_int, _u8p, C.c_int, C.c_int, _fp, C.c_int, C.c_int]),
            "or_rms_norm": (C.c_int, [_fp, _fp, _fp, C.c_int, C.c_int, C.c_float]),
            "or_rms_norm_inplace": (C.c_int, [_fp, _fp, C.c_int, C.c_int, C.c_float]),
            "or_rope_rows": (C.c_int, [_fp, C.c_int, C.c_int, C.c_int, _fp, C.c_int]),
            "or_softmax": (C.c_int, [_fp, _fp, C.c_int]),
            "or_sdpa": (C.c_int, [_fp, _fp, _fp, _fp] + [C.c_int] * 6),
            "or_sigmoid": (C.c_float, [C.c_float]),
            "or_silu": (None, [_fp, C.c_int]),
            "or_mul": (C.c_int, [_fp, _fp, _fp, C.c_int]),
            "or_add_inplace": (C.c_int, [_fp, _fp, C.c_int]),
            "or_greedy": (C.c_int64, [_fp, C.c_size_t]),
            "or_embed": (C.c_int, [_u32p, C.c_int, _u8p, C.c_int, C.c_int, C.c_int, _fp]),
            "or_rope_inv_freq": (None, [C.c_int, C.c_float, C.c_float, C.c_float, C.c_float, C.c_float, _fp]),
            "or_model_load": (C.c_void_p, [C.c_char_p, C.c_int, C.POINTER(C.c_int)]),
            "or_model_free": (None, [C.c_void_p]),
            "or_model_config": (None, [C.c_void_p, C.POINTER(Config)]),
            "or_model_inv_freq": (_fp, [C.c_void_p]),
            "or_ctx_new": (C.c_void_p, [C.c_void_p]),
            "or_ctx_free": (None, [C.c_void_p]),
            "or_ctx_reset": (None, [C.c_void_p]),
            "or_ctx_seq_len": (C.c_int, [C.c_void_p]),
            "or_forward": (C.c_int, [C.c_void_p, C.c_void_p, _u32p, C.c_int, C.c_int]),
            "or_ctx_logits": (_fp, [C.c_void_p]),
            "or_generate": (C.c_int, [C.c_void_p, _u32p, C.c_int, C.c_int, C.c_int, _u32p,
                                      C.POINTER(C.c_double), _fp, C.c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _f(a):
    return a.ctypes.data_as(_fp)


def _u8(a):
    return a.ctypes.data_as(_u8p)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def nthreads_default():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def f32_to_f16(x: float) -> int:
    return lib().or_f32_to_f16(x)


def f16_to_f32(h: int) -> float:
    return lib().or_f16_to_f32(h)


def dequantize(wtype: int, blocks: np.ndarray) -> np.ndarray:
    blocks = _c(blocks, np.uint8)
    nb = blocks.size // BLOCK_BYTES[wtype]
    out = np.empty(nb * 32, np.float32)
    lib().or_dequantize(wtype, _u8(blocks), nb, _f(out))
    return out


def quantize_row_q8_0(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32).ravel()
    out = np.empty(x.size // 32 * 34, np.uint8)
    lib().or_quantize_row_q8_0(_f(x), x.size, _u8(out))
    return out


def dot(kind: str, a: np.ndarray, b: np.ndarray) -> float:
    L = lib()
    if kind == "f32_f32":
        a, b = _c(a, np.float32), _c(b, np.float32)
        return L.or_dot_f32_f32(_f(a), _f(b), a.size)
    b = _c(b, np.uint8)
    if kind in ("q8_0_q8_0", "q8_0_q4_0"):
        a = _c(a, np.uint8)
        nb = a.size // 34
        return getattr(L, "or_dot_" + kind)(_u8(a), _u8(b), nb)
    a = _c(a, np.float32)
    return getattr(L, "or_dot_" + kind)(_f(a), _u8(b), a.size // 32)


def linear(x: np.ndarray, w: np.ndarray, wtype: int, out_dim: int, acts_q8: bool = False,
           nthreads: int = 0) -> np.ndarray:
    x = _c(x, np.float32)
    m, in_dim = x.shape
    w = _c(w, np.uint8)
    out = np.empty((m, out_dim), np.float32)
    st = lib().or_linear(_f(x), m, in_dim, _u8(w), wtype, out_dim, _f(out), int(acts_q8),
                         nthreads or nthreads_default())
    if st:
        raise ValueError(f"oracle linear status {st}")
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x, w = _c(x, np.float32), _c(w, np.float32)
    rows, dim = x.reshape(-1, x.shape[-1]).shape
    out = np.empty_like(x)
    lib().or_rms_norm(_f(x), _f(w), _f(out), rows, dim, eps)
    return out


def rope_rows(x: np.ndarray, base_pos: int, inv_freq: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32).copy()
    inv_freq = _c(inv_freq, np.float32)
    seq, row_dim = x.shape
    st = lib().or_rope_rows(_f(x), seq, row_dim, base_pos, _f(inv_freq), inv_freq.size)
    if st:
        raise ValueError(f"oracle rope status {st}")
    return x


def softmax(a: np.ndarray) -> np.ndarray:
    a = _c(a, np.float32)
    out = np.empty_like(a)
    st = lib().or_softmax(_f(a), _f(out), a.size)
    if st:
        raise ValueError(f"oracle softmax status {st}")
    return out


def sdpa(q, k, v, seq_q, seq_k, n_heads, n_kv_heads, head_dim, nthreads=0):
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    out = np.empty(seq_q * n_heads * head_dim, np.float32)
    st = lib().or_sdpa(_f(q), _f(k), _f(v), _f(out), seq_q, seq_k, n_heads, n_kv_heads, head_dim,
                       nthreads or nthreads_default())
    if st:
        raise ValueError(f"oracle sdpa status {st}")
    return out


def silu(x):
    x = _c(x, np.float32).copy()
    lib().or_silu(_f(x), x.size)
    return x


def sigmoid(x: float) -> float:
    return lib().or_sigmoid(x)


def greedy(logits) -> int:
    logits = _c(logits, np.float32)
    return int(lib().or_greedy(_f(logits), logits.size))


def embed(tokens, w, wtype, embed_dim, vocab):
    tokens = _c(tokens, np.uint32)
    w = _c(w, np.uint8)
    out = np.empty((tokens.size, embed_dim), np.float32)
    st = lib().or_embed(tokens.ctypes.data_as(_u32p), tokens.size, _u8(w), wtype, embed_dim, vocab, _f(out))
    if st:
        raise ValueError(f"oracle embed status {st}")
    return out


def rope_inv_freq(head_dim, base, factor=32.0, low=1.0, high=4.0, orig_ctx=8192.0):
    out = np.empty(head_dim // 2, np.float32)
    lib().or_rope_inv_freq(head_dim, base, factor, low, high, orig_ctx, _f(out))
    return out


class Model:
    """Llama3_2 + ModelContext restated on the CPU (one context)."""

    def __init__(self, path: str, acts_q8: bool = False):
        L = lib()
        st = C.c_int(0)
        self._m = L.or_model_load(path.encode(), int(acts_q8), C.byref(st))
        if not self._m:
            raise ValueError(f"oracle could not load {path}: status {st.value}")
        cfg = Config()
        L.or_model_config(self._m, C.byref(cfg))
        self.config = cfg
        self._ctx = L.or_ctx_new(self._m)

    def close(self):
        L = lib()
        if self._ctx:
            L.or_ctx_free(self._ctx)
            self._ctx = None
        if self._m:
            L.or_model_free(self._m)
            self._m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def inv_freq(self):
        p = lib().or_model_inv_freq(self._m)
        return np.ctypeslib.as_array(p, (self.config.head_dim // 2,)).copy()

    def reset(self):
        lib().or_ctx_reset(self._ctx)

    @property
    def seq_len(self):
        return lib().or_ctx_seq_len(self._ctx)

    def forward(self, ids, nthreads=0) -> np.ndarray:
        ids = _c(ids, np.uint32)
        st = lib().or_forward(self._m, self._ctx, ids.ctypes.data_as(_u32p), ids.size,
                              nthreads or nthreads_default())
        if st:
            raise ValueError(f"oracle forward status {st}")
        p = lib().or_ctx_logits(self._ctx)
        return np.ctypeslib.as_array(p, (self.config.vocab_size,)).copy()

    def generate(self, prompt, max_tokens, ignore_eos=True, want_logits=False, nthreads=0):
        prompt = _c(prompt, np.uint32)
        out = np.zeros(max_tokens, np.uint32)
        ms = np.zeros(max_tokens, np.float64)
        logits = np.zeros((max_tokens, self.config.vocab_size), np.float32) if want_logits else None
        n = lib().or_generate(self._m, prompt.ctypes.data_as(_u32p), prompt.size, max_tokens,
                              int(ignore_eos), out.ctypes.data_as(_u32p),
                              ms.ctypes.data_as(C.POINTER(C.c_double)),
                              _f(logits) if logits is not None else None,
                              nthreads or nthreads_default())
        if n < 0:
            raise ValueError(f"oracle generate status {-n}")
        return out[:n], ms[:n], (logits[:n] if logits is not None else None)
