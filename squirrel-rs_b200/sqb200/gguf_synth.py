"""Seeded random-init Llama GGUF files (the stand-in for the reference's real
Llama-3.2 GGUFs, which are not available here).

Writes GGUF v3 with exactly the metadata keys and types the reference's
`LlamaConfig::from_gguf` reads (models/llama/config.rs:29-73: U32 / F32 only)
and the tensor names of `LlamaWeights::from_gguf` (models/llama/weights.rs:50-97),
with tensor data aligned to 32 bytes (file_parser/gguf_file.rs:10,45-46).

Weights: N(0, 0.02) float32 from a per-tensor PCG64 stream, then quantized:
  Q8_0  d = amax/127 (f16), q = rint(x / d)                     (34-byte blocks)
  Q4_0  d = m / -8 with m the signed value of largest magnitude, q = min(15, trunc(x/d + 8.5))
        packed low nibble = element j, high nibble = element j+16 (18-byte blocks)
  BF16  round-to-nearest-even of the float32 bits              (64 bytes / 32 elements)
Norm weights are 1.0 float32 (N(0, 0.02) norms would shrink logits below the
1e-2 comparison tolerance). The exact weight rounding does not affect parity:
the CPU oracle and the GPU read the same bytes.
"""
import hashlib
import json
import os
import struct

import numpy as np

F32, Q4_0, Q8_0, BF16 = 0, 2, 8, 30
TYPE_NAMES = {"q8_0": Q8_0, "q4_0": Q4_0, "bf16": BF16}
BLOCK_BYTES = {Q8_0: 34, Q4_0: 18, BF16: 64}

SPECS = {
    # Llama-3.2-1B architecture
    "1b": dict(hidden=2048, layers=16, heads=32, kv_heads=8, head_dim=64, ffn=8192,
               vocab=128256, tied=True, ctx=131072),
    # Llama-3-8B architecture
    "8b": dict(hidden=4096, layers=32, heads=32, kv_heads=8, head_dim=128, ffn=14336,
               vocab=128256, tied=False, ctx=131072),
    # small shapes for fast parity tests (all dims multiples of 256)
    "tiny": dict(hidden=256, layers=2, heads=8, kv_heads=2, head_dim=32, ffn=512,
                 vocab=1024, tied=False, ctx=4096),
    "small": dict(hidden=512, layers=3, heads=8, kv_heads=2, head_dim=64, ffn=1536,
                  vocab=4096, tied=False, ctx=4096),
}

ROPE_BASE = 500000.0
RMS_EPS = 1e-5
BOS, EOS = 128000, 128009


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    b = x.reshape(-1, 32).astype(np.float32)
    amax = np.abs(b).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d > 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = np.clip(np.rint(b * inv[:, None]), -127, 127).astype(np.int8)
    out = np.empty((b.shape[0], 34), np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    b = x.reshape(-1, 32).astype(np.float32)
    idx = np.abs(b).argmax(axis=1)
    mx = b[np.arange(b.shape[0]), idx]
    d = (mx / np.float32(-8.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = np.minimum(15, np.trunc(b * inv[:, None] + np.float32(8.5))).astype(np.uint8)
    out = np.empty((b.shape[0], 18), np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def to_bf16(x: np.ndarray) -> np.ndarray:
    u = x.astype(np.float32).reshape(-1).view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)
    return r.view(np.uint8)


def quantize(x: np.ndarray, wtype: int) -> np.ndarray:
    if wtype == Q8_0:
        return quantize_q8_0(x)
    if wtype == Q4_0:
        return quantize_q4_0(x)
    if wtype == BF16:
        return to_bf16(x)
    raise ValueError(wtype)


def tensor_nbytes(numel: int, ttype: int) -> int:
    if ttype == F32:
        return numel * 4
    return numel // 32 * BLOCK_BYTES[ttype]


def tensor_list(spec: dict, wtype: int):
    """(name, dims as GGUF ne[] = [in_dim, out_dim], type) in file order."""
    H, F, hd = spec["hidden"], spec["ffn"], spec["head_dim"]
    Q, KV = spec["heads"] * hd, spec["kv_heads"] * hd
    out = [("token_embd.weight", [H, spec["vocab"]], wtype)]
    for i in range(spec["layers"]):
        out += [
            (f"blk.{i}.attn_norm.weight", [H], F32),
            (f"blk.{i}.attn_q.weight", [H, Q], wtype),
            (f"blk.{i}.attn_k.weight", [H, KV], wtype),
            (f"blk.{i}.attn_v.weight", [H, KV], wtype),
            (f"blk.{i}.attn_output.weight", [Q, H], wtype),
            (f"blk.{i}.ffn_norm.weight", [H], F32),
            (f"blk.{i}.ffn_gate.weight", [H, F], wtype),
            (f"blk.{i}.ffn_up.weight", [H, F], wtype),
            (f"blk.{i}.ffn_down.weight", [F, H], wtype),
        ]
    out.append(("output_norm.weight", [H], F32))
    if not spec["tied"]:
        out.append(("output.weight", [H, spec["vocab"]], wtype))
    return out


def _kv(key: str, vtype: int, payload: bytes) -> bytes:
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<I", vtype) + payload


def _u32(key, v):
    return _kv(key, 4, struct.pack("<I", v))


def _f32(key, v):
    return _kv(key, 6, struct.pack("<f", v))


def _str(key, s):
    b = s.encode()
    return _kv(key, 8, struct.pack("<Q", len(b)) + b)


def write_gguf(path: str, spec_name: str, wtype: int, seed: int = 0, rope_scaling_keys: bool = False):
    spec = SPECS[spec_name]
    H = spec["hidden"]
    meta = [
        _str("general.architecture", "llama"),
        _str("general.name", f"squirrel-b200 synthetic {spec_name}"),
        _u32("general.alignment", 32),
        _u32("llama.block_count", spec["layers"]),
        _u32("llama.context_length", spec["ctx"]),
        _u32("llama.embedding_length", H),
        _u32("llama.feed_forward_length", spec["ffn"]),
        _u32("llama.attention.head_count", spec["heads"]),
        _u32("llama.attention.head_count_kv", spec["kv_heads"]),
        _u32("llama.rope.dimension_count", spec["head_dim"]),
        _f32("llama.rope.freq_base", ROPE_BASE),
        _f32("llama.attention.layer_norm_rms_epsilon", RMS_EPS),
        _u32("llama.vocab_size", spec["vocab"]),
        _u32("tokenizer.ggml.bos_token_id", BOS),
        _u32("tokenizer.ggml.eos_token_id", EOS),
    ]
    if rope_scaling_keys:
        meta += [_f32("llama.rope.scaling.factor", 32.0),
                 _f32("llama.rope.scaling.low_freq_factor", 1.0),
                 _f32("llama.rope.scaling.high_freq_factor", 4.0),
                 _u32("llama.rope.scaling.original_context_length", 8192)]
    tensors = tensor_list(spec, wtype)
    infos, offset, offsets = [], 0, []
    for name, dims, ttype in tensors:
        numel = int(np.prod(dims))
        nb = name.encode()
        infos.append(struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims)) +
                     b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", ttype, offset))
        offsets.append(offset)
        offset += tensor_nbytes(numel, ttype)
        offset = (offset + 255) // 256 * 256  # 256-aligned tensor starts (valid: multiples of 32)
    header = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta)) + b"".join(meta) + b"".join(infos)
    pad = (-len(header)) % 32
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(header + b"\0" * pad)
        base = f.tell()
        f.truncate(base + offset)
    jobs = [(tmp, base + off, ti, dims, ttype, seed) for ti, ((name, dims, ttype), off) in enumerate(zip(tensors, offsets))]
    big = sum(int(np.prod(d)) for _, d, t in tensors if t != F32) > (1 << 28)
    workers = min(16, os.cpu_count() or 1) if big else 1
    workers = int(os.environ.get("SQB200_GEN_WORKERS", workers))
    import sys
    main_file = getattr(sys.modules.get("__main__"), "__file__", None)
    if workers > 1 and not (main_file and os.path.exists(main_file)):
        workers = 1  # spawned workers re-import __main__: impossible for stdin or interactive programs
    if workers > 1:  # every tensor has its own RNG stream and byte range: same bytes in any order
        import concurrent.futures as cf
        import multiprocessing as mp
        with cf.ProcessPoolExecutor(workers, mp_context=mp.get_context("spawn")) as ex:
            for _ in ex.map(_fill_tensor, jobs, chunksize=1):
                pass
    else:
        for j in jobs:
            _fill_tensor(j)
    os.replace(tmp, path)
    return path


def _fill_tensor(job):
    """Write one tensor's bytes at its file offset (its own PCG64 stream [seed, index])."""
    tmp, at, ti, dims, ttype, seed = job
    fd = os.open(tmp, os.O_WRONLY)
    try:
        if ttype == F32:
            os.pwrite(fd, np.ones(int(np.prod(dims)), np.float32).tobytes(), at)
            return
        rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, ti])))
        rows, in_dim = dims[1], dims[0]
        chunk = max(1, (1 << 20) // in_dim)  # small chunks: cache-resident temporaries
        for r0 in range(0, rows, chunk):
            n = min(chunk, rows - r0)
            x = rng.standard_normal(n * in_dim, dtype=np.float32) * np.float32(0.02)
            b = quantize(x, ttype).tobytes()
            os.pwrite(fd, b, at)
            at += len(b)
    finally:
        os.close(fd)


def default_cache_dir() -> str:
    return os.environ.get("SQB200_MODEL_DIR", "/tmp/sqb200_models")


def ensure_gguf(spec_name: str, wtype_name: str = "q8_0", seed: int = 0, cache_dir: str = None,
                rope_scaling_keys: bool = False) -> str:
    """Path of the seeded GGUF, written on first use (deterministic bytes)."""
    cache_dir = cache_dir or default_cache_dir()
    os.makedirs(cache_dir, exist_ok=True)
    tag = f"{spec_name}_{wtype_name}_s{seed}{'_rs' if rope_scaling_keys else ''}"
    path = os.path.join(cache_dir, tag + ".gguf")
    if not os.path.exists(path):
        write_gguf(path, spec_name, TYPE_NAMES[wtype_name], seed, rope_scaling_keys)
    return path


def file_digest(path: str, limit: int = 1 << 62) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(1 << 24)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


def prompt_ids(n: int, seed: int = 1234, high: int = 128000) -> np.ndarray:
    """Uniform random token ids in [0, high) from their own seed."""
    return np.random.default_rng(seed).integers(0, high, size=n, dtype=np.int64).astype(np.uint32)
