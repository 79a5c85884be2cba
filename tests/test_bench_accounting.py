"""The roofline accounting of bench.py against the per-token byte and FLOP figures
of the hot-path scope (1B Llama-3.2 shape): weights 1,312,980,992 B (Q8_0),
695,107,584 B (Q4_0), 2,471,493,632 B (BF16); norms 270,336 B; K/V 65,536 B a
position; the embedding row; 513,024 B of logits; prefill GEMM 1.946 GFLOP a
token. No GPU."""
import importlib.util
import os
import sys
from types import SimpleNamespace

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    argv = sys.argv
    try:
        sys.argv = ["bench.py"]
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    return mod


CFG_1B = SimpleNamespace(embed_dim=2048, ffn_dim=8192, n_heads=32, n_kv_heads=8, head_dim=64, n_blocks=16,
                         vocab_size=128256)


@pytest.mark.parametrize("wtype,weights", [(8, 1_312_980_992), (2, 695_107_584), (30, 2_471_493_632)])
def test_decode_bytes(bench, wtype, weights):
    bb = {8: 34, 2: 18, 30: 64}[wtype]
    kv_len = 96
    got = bench.bytes_per_step(CFG_1B, wtype, kv_len)
    want = weights + 270_336 + 65_536 * (kv_len + 1) + 2048 // 32 * bb + 513_024
    assert got == want


def test_prefill_flops(bench):
    per_row, _ = bench.prefill_flops(CFG_1B, 1)
    attn_1 = 16 * 32 * 4 * 64 * 1  # one row attends one key
    assert per_row - attn_1 - 2 * 2048 * 128256 == 2 * 973_078_528
