"""Op-level parity: every C-ABI op on the B200 against the CPU oracle on the same
seeded inputs. Integer / byte work (dequant, quantizer, embed, argmax) is
bit-exact; float reductions use the tolerances stated per test."""
import math

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def rand_blocks(wtype, nblocks, rng):
    """Random block bytes with finite f16 scales (every nibble / int8 value reachable)."""
    if wtype == O.BF16:
        x = rng.standard_normal(nblocks * 32).astype(np.float32)
        return (x.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
    bb = O.BLOCK_BYTES[wtype]
    raw = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    scales = (rng.standard_normal(nblocks) * 0.01).astype(np.float16)
    raw[:, :2] = scales.view(np.uint8).reshape(-1, 2)
    return raw.reshape(-1)


def quant_weights(wtype, rows, cols, rng):
    from sqb200 import gguf_synth as g
    x = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    return g.quantize(x, wtype)


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0, O.BF16])
def test_dequantize_bit_exact(gpu_lib, wtype):
    from sqb200 import lib
    rng = np.random.default_rng(1)
    nb = 4099
    blocks = rand_blocks(wtype, nb, rng)
    if wtype != O.BF16:  # include every finite f16 scale class: subnormal, normal, zero
        blocks.reshape(nb, -1)[:3, :2] = np.array([[1, 0], [0, 0], [0xff, 0x7b]], np.uint8)
    got = host(lib.dequantize(dev(blocks), wtype, nb * 32))
    want = O.dequantize(wtype, blocks)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_quantize_row_q8_0_bit_exact(gpu_lib):
    from sqb200 import lib
    src = np.float32([math.sin(i * 0.37) * 4.0 - 0.5 for i in range(32 * 6)])  # dot_prod.rs:629-654
    src[32:64] = 0.0
    src[64] = -100.0
    src[96] = 0.5
    src[97] = -0.5
    src[128] = np.finfo(np.float32).max / 2
    rng = np.random.default_rng(2)
    more = (rng.standard_normal(32 * 4096) * rng.choice([1e-6, 1e-2, 1, 300], 32 * 4096)).astype(np.float32)
    ties = (np.arange(32 * 64, dtype=np.float32) - 1024) / 2  # x*inv lands on .5 for many values
    for x in (src, more, ties):
        got = host(lib.quantize_row_q8_0(dev(x)))
        assert np.array_equal(got, O.quantize_row_q8_0(x))


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0, O.BF16])
def test_embed_bit_exact(gpu_lib, wtype):
    from sqb200 import lib
    rng = np.random.default_rng(3)
    vocab, dim = 1000, 256
    w = rand_blocks(wtype, vocab * dim // 32, rng)
    toks = np.array([0, 999, 5, 5, 123, 777], np.uint32)
    got = host(lib.embed(dev(toks), dev(w), wtype, dim, vocab))
    want = O.embed(toks, w, wtype, dim, vocab)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def term_magnitude(x, w, wtype, out_dim):
    """Sum of |a_i * w_i| per output, the scale float summation error grows with."""
    deq = O.dequantize(wtype, w).reshape(out_dim, -1).astype(np.float64)
    return np.abs(x.astype(np.float64)) @ np.abs(deq).T


SHAPES = [(1, 64, 7), (3, 96, 9), (1, 2048, 2048), (1, 2048, 512), (1, 8192, 2048), (5, 2048, 300), (32, 256, 64)]


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0, O.BF16])
@pytest.mark.parametrize("shape", SHAPES)
def test_linear_f32_acts(gpu_lib, wtype, shape):
    """W8A32/W4A32/BF16 (x86 path). Tolerance: |gpu - oracle| <= 1e-5 * sum|a_i w_i| + 1e-6."""
    from sqb200 import lib
    m, k, n = shape
    rng = np.random.default_rng(hash(shape) % 1000 + wtype)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = quant_weights(wtype, n, k, rng)
    got = host(lib.linear(dev(x), dev(w), wtype, n))
    want = O.linear(x, w, wtype, n)
    mag = term_magnitude(x, w, wtype, n)
    assert np.all(np.abs(got - want) <= 1e-5 * mag + 1e-6)


# The m = 1 streaming matvec: 7 input segments (8B ffn_down width), a partial segment,
# short rows (64-row tiles), two segments; output counts not a multiple of anything.
MV_SHAPES = [(1, 14336, 300), (1, 1536, 1000), (1, 256, 5000), (1, 4096, 4097)]


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0, O.BF16])
@pytest.mark.parametrize("shape", MV_SHAPES)
def test_matvec_shapes(gpu_lib, wtype, shape):
    """Same tolerance as test_linear_f32_acts; the segment partial sums are added in
    segment order, so two calls give identical bits."""
    from sqb200 import lib
    m, k, n = shape
    rng = np.random.default_rng(k + n + wtype)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = quant_weights(wtype, n, k, rng)
    xd, wd = dev(x), dev(w)
    got = host(lib.linear(xd, wd, wtype, n))
    again = host(lib.linear(xd, wd, wtype, n))
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
    want = O.linear(x, w, wtype, n)
    mag = term_magnitude(x, w, wtype, n)
    assert np.all(np.abs(got - want) <= 1e-5 * mag + 1e-6)


# Tensor-core GEMM (bf16 weights, m >= 2): ragged rows and outputs, K not a multiple
# of the 64-element stage, and shapes small enough in tiles that K is split.
TC_SHAPES = [(2, 64, 128), (3, 96, 9), (129, 160, 130), (100, 2048, 512), (256, 2048, 2048),
             (16, 8192, 512), (300, 1024, 384), (64, 4096, 1000)]


@pytest.mark.parametrize("shape", TC_SHAPES)
def test_linear_bf16_tensor_cores(gpu_lib, shape):
    """Activations split into three bf16 terms (exact), bf16 x bf16 products (exact),
    f32 accumulation on the tensor cores. Same tolerance as the CUDA-core path:
    |gpu - oracle| <= 1e-5 * sum|a_i w_i| + 1e-6."""
    from sqb200 import lib
    m, k, n = shape
    rng = np.random.default_rng(m * 7 + k * 3 + n)
    x = (rng.standard_normal((m, k)) * rng.choice([1e-3, 1.0, 40.0], (m, 1))).astype(np.float32)
    w = quant_weights(O.BF16, n, k, rng)
    got = host(lib.linear(dev(x), dev(w), O.BF16, n))
    want = O.linear(x, w, O.BF16, n)
    mag = term_magnitude(x, w, O.BF16, n)
    err = np.abs(got - want)
    assert np.all(err <= 1e-5 * mag + 1e-6), float((err / (mag + 1e-6)).max())


# Quantized rows on the tensor cores: K a multiple of the 256-element raw chunk;
# ragged rows and outputs, 1..16 K splits, every BN (32, 64, 128).
TCQ_SHAPES = [(2, 256, 128), (33, 512, 130), (64, 2048, 512), (129, 1024, 300), (256, 2048, 2048),
              (16, 8192, 512), (300, 768, 384), (32, 2048, 8192)]


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("shape", TCQ_SHAPES)
def test_linear_quantized_tensor_cores(gpu_lib, wtype, shape):
    """Quants as exact bf16, activations as three exact bf16 terms, one f32 block sum
    per 32-element block scaled by its f16 scale and accumulated in block order (the
    W8A32 / W4A32 scheme). |gpu - oracle| <= 1e-5 * sum|a_i w_i| + 1e-6."""
    from sqb200 import lib
    m, k, n = shape
    rng = np.random.default_rng(m * 5 + k + n * 3 + wtype)
    x = (rng.standard_normal((m, k)) * rng.choice([1e-3, 1.0, 40.0], (m, 1))).astype(np.float32)
    w = rand_blocks(wtype, n * k // 32, rng)  # every int8 / nibble value reachable
    got = host(lib.linear(dev(x), dev(w), wtype, n))
    want = O.linear(x, w, wtype, n)
    mag = term_magnitude(x, w, wtype, n)
    err = np.abs(got - want)
    assert np.all(err <= 1e-5 * mag + 1e-6), float((err / (mag + 1e-6)).max())


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("shape", SHAPES)
def test_linear_q8_acts(gpu_lib, wtype, shape):
    """W8A8/W4A8 (aarch64 scheme): exact integer block sums; float accumulation order
    free. Same tolerance as the f32 path."""
    from sqb200 import lib
    m, k, n = shape
    rng = np.random.default_rng(hash(shape) % 997 + wtype)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = quant_weights(wtype, n, k, rng)
    got = host(lib.linear(dev(x), dev(w), wtype, n, acts=lib.ACTS_Q8))
    want = O.linear(x, w, wtype, n, acts_q8=True)
    mag = term_magnitude(x, w, wtype, n)
    assert np.all(np.abs(got - want) <= 1e-5 * mag + 1e-6)


def test_linear_lm_head_shape(gpu_lib):
    from sqb200 import lib
    rng = np.random.default_rng(9)
    k, n = 2048, 128256
    x = rng.standard_normal((1, k)).astype(np.float32)
    w = quant_weights(O.Q8_0, n, k, rng)
    got = host(lib.linear(dev(x), dev(w), O.Q8_0, n))
    want = O.linear(x, w, O.Q8_0, n)
    assert np.max(np.abs(got - want)) <= 1e-3
    assert int(np.argmax(got)) == int(np.argmax(want))


@pytest.mark.parametrize("acts", [0, 1])
def test_linear_shared_equals_separate(gpu_lib, acts):  # matmul.rs:257-279: bit-identical
    from sqb200 import lib
    rng = np.random.default_rng(4)
    x = dev(rng.standard_normal((3, 256)).astype(np.float32))
    ws = [dev(quant_weights(O.Q8_0, n, 256, rng)) for n in (4, 6, 5)]
    scratch = torch.empty(3 * 8 * 34, dtype=torch.uint8, device="cuda")
    fused = lib.linear_shared(x, ws, O.Q8_0, [4, 6, 5], acts=acts, act_scratch=scratch)
    for w, n, f in zip(ws, (4, 6, 5), fused):
        sep = lib.linear(x, w, O.Q8_0, n, acts=acts)
        assert torch.equal(sep, f)


def test_linear_errors(gpu_lib):
    from sqb200 import lib
    x = torch.zeros((1, 40), device="cuda")
    w = torch.zeros(64, dtype=torch.uint8, device="cuda")
    with pytest.raises(lib.KernelError) as e:
        lib.linear(x, w, O.Q8_0, 2)
    assert e.value.kind == "ShapeMismatch"
    with pytest.raises(lib.KernelError) as e:
        lib.linear(torch.zeros((1, 64), device="cuda"), w, 1, 2)  # F16 weights
    assert e.value.kind == "InvalidType"


def test_rms_norm(gpu_lib):
    from sqb200 import lib
    got = host(lib.rms_norm(dev(np.float32([[1, 2, 3, 4]])), dev(np.ones(4, np.float32)), 0.0))[0]
    rms = math.sqrt(7.5)  # rms_norm.rs:86-98
    assert np.allclose(got, np.arange(1, 5) / rms, atol=1e-6)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((7, 2048)).astype(np.float32) * 3
    w = rng.standard_normal(2048).astype(np.float32)
    got = host(lib.rms_norm(dev(x), dev(w), 1e-5))
    want = O.rms_norm(x, w, 1e-5)
    assert np.all(np.abs(got - want) <= 2e-6 * np.abs(want) + 1e-7)
    z = host(lib.rms_norm(dev(np.zeros((1, 4), np.float32)), dev(np.ones(4, np.float32)), 1e-5))
    assert np.isfinite(z).all() and np.abs(z).max() == 0  # rms_norm.rs:100-108
    xi = dev(x.copy())
    lib.rms_norm_inplace(xi, dev(w), 1e-5)
    assert np.array_equal(host(xi), got)


def test_rope_rows(gpu_lib):
    """Double-precision sin/cos rounded once: within 2 ulp of the C library's sinf/cosf."""
    from sqb200 import lib
    inv = O.rope_inv_freq(64, 500000.0)
    rng = np.random.default_rng(6)
    x = rng.standard_normal((5, 2048)).astype(np.float32)
    for base in (0, 17, 4000):
        got = host(lib.rope_rows(dev(x.copy()), base, dev(inv)))
        want = O.rope_rows(x, base, inv)
        assert np.all(np.abs(got - want) <= 4e-7 * (np.abs(x.reshape(5, -1, 2)).sum(-1).repeat(2, -1)) + 1e-30)


@pytest.mark.parametrize("cfg", [(1, 1, 1, 1, 4), (2, 2, 1, 1, 2), (1, 1, 4, 2, 32), (1, 2049, 32, 8, 64),
                                 (1, 2304, 32, 8, 64), (37, 37, 8, 2, 64), (16, 80, 32, 8, 128),
                                 (1, 130, 32, 8, 128),
                                 # seq_q >= 64, head_dim 64: the tensor-core kernel (ragged query
                                 # blocks, keys before the chunk, GQA groups 1..8)
                                 (64, 64, 8, 2, 64), (200, 333, 32, 8, 64), (300, 300, 4, 4, 64),
                                 (129, 1000, 8, 1, 64)])
def test_sdpa_cached(gpu_lib, cfg):
    """Tolerance |gpu - oracle| <= 2e-5 * max|v| (softmax-weighted average of V rows)."""
    from sqb200 import lib
    seq_q, seq_k, H, KVH, hd = cfg
    if hd % 32:
        pytest.skip("head_dim must be a multiple of 32 on the GPU path")
    rng = np.random.default_rng(seq_k + H)
    q = rng.standard_normal(seq_q * H * hd).astype(np.float32)
    k = rng.standard_normal(seq_k * KVH * hd).astype(np.float32)
    v = rng.standard_normal(seq_k * KVH * hd).astype(np.float32)
    got = host(lib.sdpa_cached(dev(q), dev(k), dev(v), seq_q, seq_k, H, KVH, hd))
    want = O.sdpa(q, k, v, seq_q, seq_k, H, KVH, hd)
    assert np.max(np.abs(got - want)) <= 2e-5 * np.abs(v).max()


def test_sdpa_reference_identities(gpu_lib):  # attention.rs:84-171 (head_dim 32 variants)
    from sqb200 import lib
    rng = np.random.default_rng(7)
    q = rng.standard_normal(32).astype(np.float32)
    v = rng.standard_normal(32).astype(np.float32)
    out = host(lib.sdpa_cached(dev(q), dev(q), dev(v), 1, 1, 1, 1, 32))
    assert np.allclose(out, v, atol=1e-6)  # single token returns v
    k = rng.standard_normal(64).astype(np.float32)
    va, vb = rng.standard_normal(64).astype(np.float32), rng.standard_normal(64).astype(np.float32)
    vb[:32] = va[:32]
    q2 = rng.standard_normal(64).astype(np.float32)
    a = host(lib.sdpa_cached(dev(q2), dev(k), dev(va), 2, 2, 1, 1, 32))
    b = host(lib.sdpa_cached(dev(q2), dev(k), dev(vb), 2, 2, 1, 1, 32))
    assert np.array_equal(a[:32], b[:32]) and np.allclose(a[:32], va[:32], atol=1e-6)  # causal mask
    with pytest.raises(lib.KernelError):
        lib.sdpa_cached(dev(np.zeros(96, np.float32)), dev(np.zeros(64, np.float32)),
                        dev(np.zeros(64, np.float32)), 1, 1, 3, 2, 32)


def test_silu_mul_add(gpu_lib):
    from sqb200 import lib
    rng = np.random.default_rng(8)
    g = (rng.standard_normal(100003) * 6).astype(np.float32)
    u = rng.standard_normal(100003).astype(np.float32)
    s = host(lib.silu(dev(g.copy())))
    want = O.silu(g)
    assert np.all(np.abs(s - want) <= 3e-7 * np.abs(want) + 1e-30)  # expf within 2 ulp
    assert np.array_equal(host(lib.elementwise_mul(dev(g), dev(u))), g * u)
    a = dev(g.copy())
    lib.elementwise_add(a, dev(u))
    assert np.array_equal(host(a), g + u)
    sm = host(lib.silu_mul(dev(g), dev(u)))  # silu's 2 ulp plus one rounding of the product
    assert np.all(np.abs(sm - want * u) <= 5e-7 * np.abs(want * u) + 1e-30)


@pytest.mark.parametrize("case", ["known", "nan", "ties", "random", "vocab", "all_nan_tail"])
def test_argmax_semantics(gpu_lib, case):
    from sqb200 import lib
    rng = np.random.default_rng(10)
    if case == "known":
        x = np.float32([0.1, -2.3, 5.7, 4.0])  # greedy.rs:21-24
    elif case == "nan":
        x = np.float32([1.0, np.nan, 3.0, 2.0])  # greedy.rs:27-31
    elif case == "ties":
        x = np.zeros(50000, np.float32)
        x[[7, 4097, 30000]] = 5.0
    elif case == "random":
        x = rng.standard_normal(1 << 20).astype(np.float32)
        x[rng.integers(0, 1 << 20, 50)] = np.nan
    elif case == "vocab":
        x = rng.standard_normal(128256).astype(np.float32)
        x[[100, 90000]] = x.max() + 1
    else:
        x = rng.standard_normal(10000).astype(np.float32)
        x[-1] = np.nan
    got = int(host(lib.argmax(dev(x)))[0])
    assert got == O.greedy(x)
