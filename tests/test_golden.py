"""End-to-end golden fixtures (tests/golden/, made by tests/golden/make_golden.py):
the oracle must still reproduce them bit for bit (CPU), and the CUDA path must give
the same greedy ids with logits within tolerance (GPU), through the persistent
decode kernel and through the op-level step."""
import os

import numpy as np
import pytest

from golden import make_golden as MG  # tests/golden/make_golden.py

ABS_TOL, REL_TOL = 1e-2, 1e-3  # logits (max-abs, and max-abs relative to the largest logit)


def load(spec, wt):
    z = np.load(MG.fixture_path(spec, wt))
    return {k: z[k] for k in z.files}


def assert_logits_close(got, want):
    err = float(np.max(np.abs(got - want)))
    assert err <= ABS_TOL, err
    assert err / float(np.max(np.abs(want))) <= REL_TOL, err


@pytest.mark.parametrize("spec,wt", MG.CASES)
def test_oracle_reproduces_golden(spec, wt):
    from oracle import build as oracle_build
    from sqb200 import gguf_synth as G
    oracle_build.build()
    g = load(spec, wt)
    assert MG.sha256(G.ensure_gguf(spec, wt)) == str(g["gguf_sha256"])  # the GGUF writer is unchanged
    got = MG.compute(spec, wt)
    assert np.array_equal(got["prompt"], g["prompt"])
    assert np.array_equal(got["ids"], g["ids"])
    assert np.array_equal(got["logits_first"], g["logits_first"])  # bit for bit
    assert np.array_equal(got["logits_last"], g["logits_last"])


@pytest.mark.parametrize("spec,wt", MG.CASES_A8)
def test_oracle_reproduces_golden_q8_acts(spec, wt):
    from oracle import build as oracle_build
    oracle_build.build()
    z = np.load(MG.fixture_path(spec, wt, True))
    got = MG.compute(spec, wt, True)
    for k in ("prompt", "ids", "logits_first", "logits_last"):
        assert np.array_equal(got[k], z[k]), k


@pytest.mark.gpu
@pytest.mark.parametrize("op_level", [False, True])
@pytest.mark.parametrize("spec,wt", MG.CASES)
def test_cuda_matches_golden(gpu_lib, monkeypatch, spec, wt, op_level):
    from sqb200 import gguf_synth as G
    from sqb200 import lib
    if op_level:
        monkeypatch.setenv("SQ_DISABLE_DECODE_KERNEL", "1")  # read when the context is created
    g = load(spec, wt)
    m = lib.Model(G.ensure_gguf(spec, wt), device=0)
    ctx = m.new_context(64)
    assert int(ctx.forward(g["prompt"])) == int(g["ids"][0])
    assert_logits_close(ctx.logits(), g["logits_first"])
    rest = ctx.decode_steps(len(g["ids"]) - 1)
    assert np.array_equal(rest, g["ids"][1:])
    assert_logits_close(ctx.logits(), g["logits_last"])
    ctx.close()
    m.close()


def test_oracle_reproduces_config1_golden():
    """The 1B Q8_0 fixture of config 1 (tests/golden/cfg1_1b_q8_0.npz: the bench's GGUF
    seed and 32-token prompt, 33 greedy ids, logits after the prompt and after the last
    step) is the oracle's output bit for bit; the GPU tests and the bench check their
    ids against it."""
    from oracle import build as oracle_build
    from sqb200 import gguf_synth as G
    oracle_build.build()
    z = np.load(MG.config_fixture_path("cfg1_1b_q8_0"))
    assert MG.sha256(G.ensure_gguf("1b", "q8_0")) == str(z["gguf_sha256"])
    got = MG.compute_config("cfg1_1b_q8_0")
    for k in ("prompt", "ids", "logits_first", "logits_last"):
        assert np.array_equal(got[k], z[k]), k
