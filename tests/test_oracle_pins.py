"""Pins the CPU oracle to the reference's own known-answer unit tests.

Every case restates a #[test] of squirrel-rs (file:line given per test); the
aarch64-gated ones (dot_prod.rs:551) are restated against the scalar twins the
oracle implements. These run without a GPU.
"""
import math
import struct

import numpy as np
import pytest

from oracle import oracle as O


def q8_block(scale, qs):
    return np.frombuffer(struct.pack("<H", O.f32_to_f16(scale)) + bytes(np.int8(qs).view(np.uint8)), np.uint8)


def q4_block(scale, qs):
    return np.frombuffer(struct.pack("<H", O.f32_to_f16(scale)) + bytes(np.uint8(qs)), np.uint8)


def bf16_bits(x):
    u = np.float32(x).view(np.uint32)
    return np.uint16((int(u) + 0x7FFF + ((int(u) >> 16) & 1)) >> 16)


def test_f16_rne_matches_numpy():
    # half::f16::from_f32 is IEEE RNE; numpy's float16 cast is too.
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 1e-3,
        rng.standard_normal(20000).astype(np.float32) * 100,
        np.float32([0.0, -0.0, 65504, 65519.99, 65520, 1e-8, 2 ** -25, 2 ** -24, 3 * 2 ** -26,
                    6.1e-5, -6.1e-5, np.inf, -np.inf, 1.0 / 127, 100.0 / 127]),
        (np.arange(1, 1 << 16, dtype=np.uint32) << 13).view(np.float32)[:30000],
    ])
    for v in vals:
        want = int(np.float32(v).astype(np.float16).view(np.uint16))
        assert O.f32_to_f16(float(v)) == want, v
    for h in range(0, 1 << 16, 7):
        x = np.uint16(h).view(np.float16)
        if np.isnan(x):
            continue
        assert O.f16_to_f32(h) == float(np.float32(x))


def test_softmax_known_values():  # softmax.rs:50-57
    out = O.softmax(np.float32([1, 2, 3]))
    for got, want in zip(out, [0.09003057, 0.24472847, 0.66524096]):
        assert abs(got - want) < 1e-6
    assert abs(out.sum() - 1) < 1e-6


def test_softmax_large_values_and_empty():  # softmax.rs:59-91
    out = O.softmax(np.float32([100.0, 101.0]))
    assert np.isfinite(out).all() and out[1] > out[0] and abs(out.sum() - 1) < 1e-6
    with pytest.raises(ValueError):
        O.softmax(np.float32([]))


def test_rms_norm_hand_computed():  # rms_norm.rs:86-98
    rms = np.float32(math.sqrt(7.5))
    out = O.rms_norm(np.float32([[1, 2, 3, 4]]), np.float32([1, 1, 1, 1]), 0.0)[0]
    for i, v in enumerate(out):
        assert abs(v - (i + 1) / rms) < 1e-5


def test_rms_norm_zero_and_weight():  # rms_norm.rs:100-122
    out = O.rms_norm(np.zeros((1, 4), np.float32), np.ones(4, np.float32), 1e-5)
    assert np.isfinite(out).all() and np.abs(out).max() < 1e-5
    x = np.float32([[1, 2, 3, 4]])
    unit = O.rms_norm(x, np.ones(4, np.float32), 0.0)
    scaled = O.rms_norm(x, np.full(4, 2, np.float32), 0.0)
    assert np.allclose(scaled, 2 * unit, atol=1e-5)


def test_attention_identities():  # attention.rs:84-160
    q = np.float32([0.5, -1.0, 2.0, 0.25])
    v = np.float32([7, 8, 9, 10])
    assert np.allclose(O.sdpa(q, q, v, 1, 1, 1, 1, 4), v, atol=1e-5)
    # causal mask hides the future
    q = np.float32([1, 0, 0.5, 0.5]); k = np.float32([1, 0, 0, 1])
    a = O.sdpa(q, k, np.float32([3, 4, 99, -99]), 2, 2, 1, 1, 2)
    b = O.sdpa(q, k, np.float32([3, 4, -42, 1234]), 2, 2, 1, 1, 2)
    assert np.allclose(a[:2], b[:2]) and np.allclose(a[:2], [3, 4], atol=1e-5)
    # GQA heads sharing a kv head
    out = O.sdpa(np.float32([1, 0, 1, 0, 0, 1, 0, 1]), np.float32([1, 1, 0.5, -0.5]),
                 np.float32([10, 20, 30, 40]), 1, 1, 4, 2, 2)
    assert np.allclose(out[0:2], out[2:4]) and np.allclose(out[4:6], out[6:8])
    # decode against one cached token returns v
    out = O.sdpa(np.float32([0.1, 0.2, 0.3, 0.4]), np.float32([1, 0, -1, 2]), np.float32([5, 6, 7, 8]),
                 1, 1, 2, 2, 2)
    assert np.allclose(out, [5, 6, 7, 8], atol=1e-5)
    with pytest.raises(ValueError):  # attention.rs:162-171
        O.sdpa(np.zeros(6, np.float32), np.zeros(6, np.float32), np.zeros(6, np.float32), 1, 1, 3, 2, 2)


def test_greedy_picks_max_and_nan():  # greedy.rs:21-31
    assert O.greedy(np.float32([0.1, -2.3, 5.7, 4.0])) == 2
    assert O.greedy(np.float32([1.0, np.nan, 3.0, 2.0])) == 2
    # ties resolve to the later index (Iterator::max_by)
    assert O.greedy(np.float32([1.0, 3.0, 3.0, 2.0])) == 2


def _test_q8_acts(n):  # dot_prod.rs:657-671
    blocks = []
    for blk in range(n):
        qs = [((i * 11 + blk * 17) % 251) - 125 for i in range(32)]
        blocks.append(q8_block(0.002 * (blk + 1), qs))
    return np.concatenate(blocks)


def _test_q4_blocks(n):  # dot_prod.rs:705-720
    blocks = []
    for blk in range(n):
        qs = [(((i * 7 + blk * 5) % 16) << 4) | ((i + blk * 3) % 16) for i in range(16)]
        blocks.append(q4_block(0.003 * (blk + 1), qs))
    return np.concatenate(blocks)


def test_q4_dequant_matches_dot():  # dot_prod.rs:722-742
    blocks = _test_q4_blocks(2)
    deq = O.dequantize(O.Q4_0, blocks)
    for pos in [0, 1, 15, 16, 17, 31, 32, 63]:
        oh = np.zeros(64, np.float32); oh[pos] = 1
        assert abs(O.dot("f32_q4_0", oh, blocks) - deq[pos]) < 1e-6


def test_q4_int_dot_exact_on_integers():  # dot_prod.rs:774-803
    qs = [((i % 16) << 4) | (15 - i % 16) for i in range(16)]
    w = q4_block(1.0, qs)
    a_qs = [i - 16 for i in range(32)]
    a = q8_block(1.0, a_qs)
    expected = sum(a_qs[j] * ((qs[j] & 15) - 8) + a_qs[j + 16] * ((qs[j] >> 4) - 8) for j in range(16))
    assert O.dot("q8_0_q4_0", a, w) == float(expected)


def test_int_dots_close_to_f32():  # dot_prod.rs:588-627, 747-772
    blocks = np.concatenate([q8_block(0.002 * (blk + 1), [((i * 5 + blk * 11) % 251) - 125 for i in range(32)])
                             for blk in range(8)])
    a = np.float32([math.cos(i * 0.017) * 2.5 for i in range(256)])
    ref = O.dot("f32_q8_0", a, blocks)
    got = O.dot("q8_0_q8_0", O.quantize_row_q8_0(a), blocks)
    assert abs(got - ref) <= 1e-2 * max(abs(ref), 1.0)
    w4 = _test_q4_blocks(8)
    a = np.float32([math.sin(i * 0.019) * 2.0 + 0.3 for i in range(256)])
    ref = O.dot("f32_q4_0", a, w4)
    got = O.dot("q8_0_q4_0", O.quantize_row_q8_0(a), w4)
    assert abs(got - ref) <= 1e-2 * max(abs(ref), 1.0)


def test_q8_scalar_int_dot_is_exact_sum():  # dot_prod.rs:673-686 (scalar twin)
    acts, w = _test_q8_acts(4), _test_q8_acts(4)
    total = np.float32(0)
    for k in range(4):
        qa = acts[k * 34 + 2:(k + 1) * 34].view(np.int8).astype(np.int32)
        isum = int((qa * qa).sum())
        s = np.float32(O.f16_to_f32(int(acts[k * 34:k * 34 + 2].view(np.uint16)[0])))
        total = np.float32(total + np.float32(np.float32(isum) * s) * s)
    assert O.dot("q8_0_q8_0", acts, w) == total


def test_quantizer_edge_cases():  # dot_prod.rs:629-654 (scalar semantics pinned directly)
    src = np.float32([math.sin(i * 0.37) * 4.0 - 0.5 for i in range(32 * 6)])
    src[32:64] = 0.0
    src[64] = -100.0
    src[96] = 0.5
    src[97] = -0.5
    src[128] = np.finfo(np.float32).max / 2
    q = O.quantize_row_q8_0(src).reshape(6, 34)
    for b in range(6):
        chunk = src[b * 32:(b + 1) * 32]
        amax = np.float32(np.abs(chunk).max())
        scale = np.float32(amax / np.float32(127))
        inv = np.float32(1) / scale if scale > 0 else np.float32(0)
        assert int(q[b, :2].view(np.uint16)[0]) == int(np.float32(scale).astype(np.float16).view(np.uint16))
        with np.errstate(over="ignore", invalid="ignore"):
            prod = (chunk * inv).astype(np.float32)
        want = np.clip(np.where(np.isnan(prod), 0, np.sign(prod) * np.floor(np.abs(prod) + 0.5)), -127, 127)
        assert (q[b, 2:].view(np.int8) == want.astype(np.int8)).all(), b
    assert (q[1, 2:] == 0).all() and q[1, 0] == 0 and q[1, 1] == 0
    assert q[2, 2:].view(np.int8)[0] == -127


def test_bf16_dequant_matches_dot():  # dot_prod.rs:836-856
    v = [bf16_bits(math.sin(i * 0.11 + blk) * 2.5) for blk in range(2) for i in range(32)]
    blocks = np.array(v, np.uint16).view(np.uint8)
    deq = O.dequantize(O.BF16, blocks)
    for pos in [0, 1, 15, 16, 31, 32, 63]:
        oh = np.zeros(64, np.float32); oh[pos] = 1
        assert abs(O.dot("f32_bf16", oh, blocks) - deq[pos]) < 1e-6


def _bf16_weights(b_cols, a_cols):  # matmul.rs:186-197
    vals = []
    for blk in range(b_cols * (a_cols // 32)):
        vals += [bf16_bits(math.cos((blk * 32 + i) * 0.011) * 0.4) for i in range(32)]
    return np.array(vals, np.uint16).view(np.uint8)


def _acts(rows, cols):  # matmul.rs:180-184
    return np.float32([math.sin(i * 0.037) * 2.0 - 0.5 for i in range(rows * cols)]).reshape(rows, cols)


@pytest.mark.parametrize("shape", [(1, 128, 7), (5, 96, 9)])
def test_linear_matches_naive(shape):  # matmul.rs:236-255
    m, k, n = shape
    a, w = _acts(m, k), _bf16_weights(n, k)
    wf = O.dequantize(O.BF16, w).reshape(n, k).astype(np.float64)
    got = O.linear(a, w, O.BF16, n)
    want = a.astype(np.float64) @ wf.T
    assert np.all(np.abs(got - want) <= 1e-4 * np.maximum(np.abs(want), 1))


def test_fused_equals_separate():  # matmul.rs:257-279: one input, projections computed singly
    a = _acts(3, 64)
    outs = [O.linear(a, _bf16_weights(c, 64), O.BF16, c) for c in (4, 6, 5)]
    again = [O.linear(a, _bf16_weights(c, 64), O.BF16, c, nthreads=3) for c in (4, 6, 5)]
    for x, y in zip(outs, again):
        assert (x == y).all()


def test_linear_rejects_non_block_cols():  # matmul.rs:351-361
    with pytest.raises(ValueError):
        O.linear(_acts(1, 40), _bf16_weights(2, 64), O.BF16, 2)


def test_rope_inv_freq_llama3_defaults():  # config.rs:83-127
    f = O.rope_inv_freq(64, 500000.0)
    base = np.float32([np.float32(500000.0) ** np.float32(-2.0 * j / 64) for j in range(32)])
    assert f[0] == 1.0
    assert abs(f[-1] / base[-1] - 1 / 32) < 1e-6  # lowest frequencies divided by the factor
    assert np.all(np.diff(f) < 0)
