"""The BASELINE configurations' own shapes on the B200, against the oracle's pinned
output (tests/golden/cfg*.npz, made by tests/golden/make_golden.py --configs on the
same seeded GGUF and prompt; the GGUF's sha256 is checked first):

  cfg1_1b_q8_0  config 1: 1B Q8_0 with its tied LM head (token_embd, weights.rs:89)
                and 128256-row vocabulary, 32-token prompt, 32 greedy steps through
                the persistent decode kernel
  cfg3_1b_q4_0  config 3: 1B Q4_0, 2048-token prompt, 16 steps at KV 2048-2064
                (split-KV attention inside the decode kernel)
  cfg4_1b_bf16  config 4: an 8192-token BF16 prefill (tensor-core GEMMs and
                attention), the next id and its logits
  cfg5_8b_q8_0  config 5's model on one GPU: head_dim 128, FFN 14336 (the down
                projection's input in two parts), untied LM head, 16-token prompt,
                8 greedy steps through the persistent decode kernel

Bar (north star): identical greedy ids; logits within max-abs 1e-2 and max-abs /
max|logit| <= 1e-3 after the prompt and after the last step."""
import numpy as np
import pytest

from golden import make_golden as MG  # tests/golden/make_golden.py

pytestmark = pytest.mark.gpu

ABS_TOL, REL_TOL = 1e-2, 1e-3


def assert_logits_close(got, want):
    err = float(np.max(np.abs(got - want)))
    assert err <= ABS_TOL, err
    assert err / float(np.max(np.abs(want))) <= REL_TOL, err


@pytest.mark.parametrize("name", list(MG.CONFIG_CASES))
def test_config_shape_matches_oracle(gpu_lib, name):
    from sqb200 import gguf_synth as G
    from sqb200 import lib
    c = MG.CONFIG_CASES[name]
    z = np.load(MG.config_fixture_path(name))
    path = G.ensure_gguf(c["spec"], c["wt"])
    assert MG.sha256(path) == str(z["gguf_sha256"])  # the same weights the oracle read
    prompt, ids = z["prompt"], z["ids"]
    assert np.array_equal(prompt, G.prompt_ids(c["prompt"], seed=MG.CONFIG_PROMPT_SEED))
    m = lib.Model(path, device=0)
    ctx = m.new_context(len(prompt) + len(ids) + 8)
    try:
        assert int(ctx.forward(prompt)) == int(ids[0])
        assert_logits_close(ctx.logits(), z["logits_first"])
        if len(ids) > 1:
            assert ctx.launches_per_token == 1  # the persistent decode kernel serves both shapes
            rest = ctx.decode_steps(len(ids) - 1)
            assert np.array_equal(rest, ids[1:])
            assert_logits_close(ctx.logits(), z["logits_last"])
        lib.wait_status()
    finally:
        ctx.close()
        m.close()
