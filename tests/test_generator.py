"""The generation loop of text_generator.rs (sqb200.generator): with the KV cache,
without it (SQUIRREL_NO_KV_CACHE: reset and feed the whole sequence each step),
EOS handling and the stderr progress lines. CPU: driven by the oracle, where the
cached and uncached loops must give the same ids as the oracle's own generate.
GPU: the same through the C ABI."""
import io
import re

import numpy as np
import pytest

from oracle import oracle as O
from sqb200 import generator as GEN
from sqb200 import gguf_synth as G

STEPS = 8


def oracle_loop(m):
    return (lambda ids: O.greedy(m.forward(ids))), m.reset


@pytest.mark.parametrize("no_kv_cache", [False, True])
def test_oracle_loop_matches_oracle_generate(no_kv_cache):
    from oracle import build as oracle_build
    oracle_build.build()
    path = G.ensure_gguf("tiny", "q8_0")
    prompt = G.prompt_ids(6, seed=3, high=G.SPECS["tiny"]["vocab"])
    m = O.Model(path)
    want, _, _ = m.generate(prompt, STEPS)
    m.reset()
    fwd, reset = oracle_loop(m)
    log = io.StringIO()
    got = GEN.generate_ids(fwd, reset, prompt, STEPS, eos_id=-1, no_kv_cache=no_kv_cache, log=log)
    m.close()
    assert np.array_equal(got, want)
    lines = log.getvalue().splitlines()
    assert lines[0] == "[prompt: 6 tokens]"
    assert len(lines) == 1 + STEPS and all(re.fullmatch(r"\[step +\d+: +\d+\.\dms\]  \d+", l) for l in lines[1:])


def test_eos_stops_unless_ignored(monkeypatch):
    from oracle import build as oracle_build
    oracle_build.build()
    path = G.ensure_gguf("tiny", "q8_0")
    prompt = G.prompt_ids(6, seed=3, high=G.SPECS["tiny"]["vocab"])
    m = O.Model(path)
    first = O.greedy(m.forward(prompt))
    m.reset()
    fwd, reset = oracle_loop(m)
    log = io.StringIO()
    assert GEN.generate_ids(fwd, reset, prompt, STEPS, eos_id=first, log=log) == []  # EOS at step 1
    assert log.getvalue().splitlines()[-1].endswith("<eos>")
    m.reset()
    monkeypatch.setenv("SQUIRREL_IGNORE_EOS", "1")
    assert len(GEN.generate_ids(fwd, reset, prompt, 3, eos_id=first, log=None)) == 3
    m.close()


@pytest.mark.gpu
@pytest.mark.parametrize("no_kv_cache", [False, True])
def test_cuda_loop_matches_oracle(gpu_lib, no_kv_cache):
    from sqb200 import lib
    path = G.ensure_gguf("small", "q8_0")
    prompt = G.prompt_ids(8, seed=13, high=G.SPECS["small"]["vocab"])
    om = O.Model(path)
    want, _, _ = om.generate(prompt, STEPS)
    om.close()
    m = lib.Model(path, device=0)
    ctx = m.new_context(64)
    got = GEN.generate(ctx, prompt, STEPS, eos_id=-1, no_kv_cache=no_kv_cache, log=None)
    ctx.close()
    m.close()
    assert np.array_equal(got, want)
