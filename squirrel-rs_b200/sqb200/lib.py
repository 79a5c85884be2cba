"""Python mirror of squirrel-rs's op and model interfaces over the C ABI
(include/squirrel_cuda.h). Device memory comes from torch CUDA tensors; every
call goes through libsquirrel_cuda.so — there is no other implementation, so a
missing or unloadable library is an error.

Op names follow the reference's `src/ops` (linear, linear_shared, embed,
rms_norm, rms_norm_inplace, rope_rows, sdpa_cached, silu, elementwise_mul,
elementwise_add) and `src/kernels` (quantize_row_q8_0, dequantize); errors
raise KernelError carrying the reference's error kind.
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "lib", "libsquirrel_cuda.so")

F32, Q4_0, Q8_0, BF16 = 0, 2, 8, 30
ACTS_F32, ACTS_Q8 = 0, 1
BLOCK_BYTES = {Q8_0: 34, Q4_0: 18, BF16: 64}
STATUS = {0: "Ok", 1: "ShapeMismatch", 2: "InvalidType", 3: "EmptyInput", 4: "TensorAlignmentError",
          5: "InvalidArgument", 6: "Io", 7: "InvalidConfig", 16: "Cuda", 17: "Nccl", 18: "Timeout",
          19: "CacheFull"}

_lib = None


class KernelError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code
        self.kind = STATUS.get(code, str(code))


class LlamaConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_blocks", "embed_dim", "ffn_dim", "n_heads", "n_kv_heads",
                                       "head_dim", "vocab_size", "context_length")] + [
        ("rope_base", C.c_float), ("rms_eps", C.c_float),
        ("bos_token_id", C.c_uint32), ("eos_token_id", C.c_uint32), ("weight_type", C.c_int),
        ("rope_factor", C.c_float), ("rope_low_freq", C.c_float), ("rope_high_freq", C.c_float),
        ("rope_orig_ctx", C.c_float)]


_vp, _i, _sz, _f = C.c_void_p, C.c_int, C.c_size_t, C.c_float
SIGNATURES = {
    "sq_last_error": (C.c_char_p, []),
    "sq_version": (C.c_char_p, []),
    "sq_wait_status": (_i, [_i]),
    "sq_linear": (_i, [_vp, _vp, _i, _i, _vp, _i, _i, _vp, _i]),
    "sq_linear_shared": (_i, [_vp, _vp, _i, _i, _i, C.POINTER(_vp), C.POINTER(_i), _i, C.POINTER(_vp), _i, _vp]),
    "sq_embed": (_i, [_vp, _vp, _i, _vp, _i, _i, _i, _vp]),
    "sq_rms_norm": (_i, [_vp, _vp, _vp, _vp, _i, _i, _f]),
    "sq_rms_norm_inplace": (_i, [_vp, _vp, _vp, _i, _i, _f]),
    "sq_rope_rows": (_i, [_vp, _vp, _i, _i, _i, _vp, _i]),
    "sq_sdpa_cached": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i]),
    "sq_silu": (_i, [_vp, _vp, _sz]),
    "sq_elementwise_mul": (_i, [_vp, _vp, _vp, _vp, _sz]),
    "sq_elementwise_add": (_i, [_vp, _vp, _vp, _sz]),
    "sq_silu_mul": (_i, [_vp, _vp, _vp, _vp, _sz]),
    "sq_quantize_row_q8_0": (_i, [_vp, _vp, _sz, _vp]),
    "sq_dequantize": (_i, [_vp, _vp, _i, _sz, _vp]),
    "sq_argmax": (_i, [_vp, _vp, _sz, _vp]),
    "sq_argmax_noalloc": (_i, [_vp, _vp, _sz, _vp]),
    "sq_model_create": (_i, [C.POINTER(LlamaConfig), _i, _i, C.POINTER(_vp)]),
    "sq_model_upload_tensor": (_i, [_vp, C.c_char_p, _i, C.POINTER(C.c_uint64), _i, _vp, _sz]),
    "sq_model_finalize": (_i, [_vp]),
    "sq_model_load_gguf": (_i, [C.c_char_p, _i, _i, C.POINTER(_vp)]),
    "sq_model_config": (_i, [_vp, C.POINTER(LlamaConfig)]),
    "sq_model_free": (None, [_vp]),
    "sq_ctx_create": (_i, [_vp, _i, C.POINTER(_vp)]),
    "sq_ctx_free": (None, [_vp]),
    "sq_ctx_reset": (_i, [_vp]),
    "sq_ctx_seq_len": (_i, [_vp, C.POINTER(_i)]),
    "sq_forward": (_i, [_vp, C.POINTER(C.c_uint32), _sz, C.POINTER(C.c_uint32)]),
    "sq_ctx_logits": (_i, [_vp, C.POINTER(_f), _sz]),
    "sq_generate": (_i, [_vp, C.POINTER(C.c_uint32), _sz, _i, _i, C.POINTER(C.c_uint32), C.POINTER(_f),
                         C.POINTER(_i)]),
    "sq_decode_steps": (_i, [_vp, _i, C.POINTER(C.c_uint32)]),
    "sq_ctx_stream": (_vp, [_vp]),
    "sq_ctx_launches_per_token": (_i, [_vp, C.POINTER(_i)]),
    "sq_nccl_unique_id": (_i, [_vp, _sz]),
    "sq_tp_recover": (_i, [_vp]),
    "sq_model_create_tp": (_i, [C.POINTER(LlamaConfig), _i, _i, _i, _i, _vp, C.POINTER(_vp)]),
    "sq_model_load_gguf_tp": (_i, [C.c_char_p, _i, _i, _i, _i, _vp, C.POINTER(_vp)]),
    "sq_tp_shard_tensor": (_i, [C.c_char_p, _i, C.POINTER(C.c_uint64), _i, _i, _i, _vp, _sz, _vp, _sz,
                                C.POINTER(C.c_uint64), C.POINTER(_sz)]),
}


def load(build_if_missing: bool = True):
    """Load libsquirrel_cuda.so (building it in-tree first if it is absent)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH) and build_if_missing:
        sys.path.insert(0, PKG)
        import build as _b  # squirrel-rs_b200/build.py
        _b.build()
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"libsquirrel_cuda.so not found at {LIB_PATH}; run squirrel-rs_b200/build.py")
    L = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _check(code):
    if code != 0:
        raise KernelError(code, load().sq_last_error().decode())


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def wait_status(clear=True):
    """sq_wait_status: raise KernelError (Timeout) if a bounded device-side wait of an
    op-level call expired on the current device (call after synchronizing)."""
    _check(load().sq_wait_status(int(clear)))


# ---- op level (torch CUDA tensors) ------------------------------------------------

def linear(x, w, wtype, out_dim, acts=ACTS_F32, out=None):
    import torch
    m, in_dim = x.shape
    out = out if out is not None else torch.empty((m, out_dim), dtype=torch.float32, device=x.device)
    _check(load().sq_linear(_stream(), _p(x), m, in_dim, _p(w), wtype, out_dim, _p(out), acts))
    return out


def linear_shared(x, weights, wtype, out_dims, acts=ACTS_F32, act_scratch=None):
    import torch
    m, in_dim = x.shape
    outs = [torch.empty((m, d), dtype=torch.float32, device=x.device) for d in out_dims]
    n = len(weights)
    wp = (C.c_void_p * n)(*[w.data_ptr() for w in weights])
    op = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
    dims = (C.c_int * n)(*out_dims)
    _check(load().sq_linear_shared(_stream(), _p(x), m, in_dim, n, wp, dims, wtype, op, acts, _p(act_scratch)))
    return outs


def embed(tokens, w, wtype, embed_dim, vocab):
    import torch
    out = torch.empty((tokens.numel(), embed_dim), dtype=torch.float32, device=tokens.device)
    _check(load().sq_embed(_stream(), _p(tokens), tokens.numel(), _p(w), wtype, embed_dim, vocab, _p(out)))
    return out


def rms_norm(x, w, eps):
    import torch
    out = torch.empty_like(x)
    _check(load().sq_rms_norm(_stream(), _p(x), _p(w), _p(out), x.numel() // x.shape[-1], x.shape[-1], eps))
    return out


def rms_norm_inplace(x, w, eps):
    _check(load().sq_rms_norm_inplace(_stream(), _p(x), _p(w), x.numel() // x.shape[-1], x.shape[-1], eps))
    return x


def rope_rows(x, base_pos, inv_freq):
    seq, row_dim = x.shape
    _check(load().sq_rope_rows(_stream(), _p(x), seq, row_dim, base_pos, _p(inv_freq), inv_freq.numel()))
    return x


def sdpa_cached(q, k, v, seq_q, seq_k, n_heads, n_kv_heads, head_dim):
    import torch
    out = torch.empty_like(q)
    _check(load().sq_sdpa_cached(_stream(), _p(q), _p(k), _p(v), _p(out), seq_q, seq_k, n_heads, n_kv_heads,
                                 head_dim))
    return out


def silu(x):
    _check(load().sq_silu(_stream(), _p(x), x.numel()))
    return x


def elementwise_mul(a, b):
    import torch
    out = torch.empty_like(a)
    _check(load().sq_elementwise_mul(_stream(), _p(a), _p(b), _p(out), a.numel()))
    return out


def elementwise_add(a, b):
    _check(load().sq_elementwise_add(_stream(), _p(a), _p(b), a.numel()))
    return a


def silu_mul(g, u):
    import torch
    out = torch.empty_like(g)
    _check(load().sq_silu_mul(_stream(), _p(g), _p(u), _p(out), g.numel()))
    return out


def quantize_row_q8_0(x):
    import torch
    out = torch.empty(x.numel() // 32 * 34, dtype=torch.uint8, device=x.device)
    _check(load().sq_quantize_row_q8_0(_stream(), _p(x), x.numel(), _p(out)))
    return out


def dequantize(blocks, wtype, n_elems):
    import torch
    out = torch.empty(n_elems, dtype=torch.float32, device=blocks.device)
    _check(load().sq_dequantize(_stream(), _p(blocks), wtype, n_elems, _p(out)))
    return out


def argmax(logits):
    import torch
    out = torch.empty(1, dtype=torch.int64, device=logits.device)
    _check(load().sq_argmax(_stream(), _p(logits), logits.numel(), _p(out)))
    return out


ARGMAX_NOALLOC_MAX_N = 1 << 24


def argmax_noalloc(logits, out=None):
    """sq_argmax_noalloc: the argmax without device allocation inside the call
    (n <= ARGMAX_NOALLOC_MAX_N); `out` may be a caller-owned int64 device tensor."""
    import torch
    if out is None:
        out = torch.empty(1, dtype=torch.int64, device=logits.device)
    _check(load().sq_argmax_noalloc(_stream(), _p(logits), logits.numel(), _p(out)))
    return out


# ---- model level --------------------------------------------------------------------

NCCL_ID_BYTES = 128


def nccl_unique_id() -> bytes:
    """ncclGetUniqueId (rank 0 makes it; every rank of the group uses the same bytes)."""
    buf = C.create_string_buffer(NCCL_ID_BYTES)
    _check(load().sq_nccl_unique_id(buf, NCCL_ID_BYTES))
    return buf.raw


def tp_shard_tensor(name, ggml_type, dims, data, tp_rank, tp_size):
    """The shard of one GGUF tensor that rank tp_rank holds (host bytes, no GPU):
    returns (dims, bytes)."""
    L = load()
    data = np.ascontiguousarray(data)
    d = (C.c_uint64 * len(dims))(*dims)
    od = (C.c_uint64 * len(dims))()
    nb = C.c_size_t()
    _check(L.sq_tp_shard_tensor(name.encode(), ggml_type, d, len(dims), tp_rank, tp_size, None, 0, None, 0, od,
                                C.byref(nb)))
    out = np.empty(nb.value, np.uint8)
    _check(L.sq_tp_shard_tensor(name.encode(), ggml_type, d, len(dims), tp_rank, tp_size,
                                data.ctypes.data_as(C.c_void_p), data.nbytes, out.ctypes.data_as(C.c_void_p),
                                out.nbytes, od, C.byref(nb)))
    return [int(v) for v in od], out


class Model:
    """Llama3_2 on one GPU (models/llama/model.rs), loaded from a GGUF file."""

    def __init__(self, path=None, device=0, acts=ACTS_F32, _handle=None, tp_rank=0, tp_size=1, nccl_id=None):
        """tp_size > 1: this process is rank tp_rank of a tensor-parallel group; every
        rank passes the same nccl_id (bytes from nccl_unique_id() on rank 0)."""
        L = load()
        h = C.c_void_p()
        if _handle is not None:
            h = _handle
        elif tp_size > 1:
            buf = C.create_string_buffer(bytes(nccl_id), NCCL_ID_BYTES)
            _check(L.sq_model_load_gguf_tp(path.encode(), device, acts, tp_rank, tp_size, buf, C.byref(h)))
        else:
            _check(L.sq_model_load_gguf(path.encode(), device, acts, C.byref(h)))
        self._h = h
        cfg = LlamaConfig()
        _check(L.sq_model_config(h, C.byref(cfg)))
        self.config = cfg

    @classmethod
    def from_tensors(cls, cfg: LlamaConfig, tensors, device=0, acts=ACTS_F32):
        """The reference-side upload path: create, upload each tensor, finalize."""
        L = load()
        h = C.c_void_p()
        _check(L.sq_model_create(C.byref(cfg), device, acts, C.byref(h)))
        try:
            for name, ttype, dims, data in tensors:
                data = np.ascontiguousarray(data)
                d = (C.c_uint64 * len(dims))(*dims)
                _check(L.sq_model_upload_tensor(h, name.encode(), ttype, d, len(dims),
                                                data.ctypes.data_as(C.c_void_p), data.nbytes))
            _check(L.sq_model_finalize(h))
        except Exception:
            L.sq_model_free(h)
            raise
        return cls(_handle=h)

    def close(self):
        if self._h:
            load().sq_model_free(self._h)
            self._h = None

    def new_context(self, max_ctx=0):
        return Context(self, max_ctx)

    def tp_recover(self):
        """sq_tp_recover: collective re-synchronization of a tensor-parallel group's
        all-reduce after a timeout (every rank calls it; then reset the contexts)."""
        _check(load().sq_tp_recover(self._h))


class Context:
    """ModelContext on the device: KV cache + workspace + one CUDA stream."""

    def __init__(self, model: Model, max_ctx=0):
        self.model = model
        h = C.c_void_p()
        _check(load().sq_ctx_create(model._h, max_ctx, C.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            load().sq_ctx_free(self._h)
            self._h = None

    def reset(self):
        _check(load().sq_ctx_reset(self._h))

    @property
    def seq_len(self):
        v = C.c_int()
        _check(load().sq_ctx_seq_len(self._h, C.byref(v)))
        return v.value

    @property
    def stream(self):
        return load().sq_ctx_stream(self._h)

    @property
    def launches_per_token(self):
        v = C.c_int()
        _check(load().sq_ctx_launches_per_token(self._h, C.byref(v)))
        return v.value

    def forward(self, ids):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = C.c_uint32()
        _check(load().sq_forward(self._h, ids.ctypes.data_as(C.POINTER(C.c_uint32)), ids.size, C.byref(out)))
        return out.value

    def logits(self):
        v = np.empty(self.model.config.vocab_size, np.float32)
        _check(load().sq_ctx_logits(self._h, v.ctypes.data_as(C.POINTER(C.c_float)), v.size))
        return v

    def generate(self, prompt, max_tokens, ignore_eos=True):
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max(max_tokens, 1), np.uint32)
        ms = np.zeros(max(max_tokens, 1), np.float32)
        n = C.c_int()
        _check(load().sq_generate(self._h, prompt.ctypes.data_as(C.POINTER(C.c_uint32)), prompt.size, max_tokens,
                                  int(ignore_eos), out.ctypes.data_as(C.POINTER(C.c_uint32)),
                                  ms.ctypes.data_as(C.POINTER(C.c_float)), C.byref(n)))
        return out[:n.value], ms[:n.value]

    def decode_steps(self, n_steps):
        out = np.zeros(max(n_steps, 1), np.uint32)
        _check(load().sq_decode_steps(self._h, n_steps, out.ctypes.data_as(C.POINTER(C.c_uint32))))
        return out[:n_steps]
