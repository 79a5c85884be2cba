"""Teacher-forced perplexity (bin/perplexity.rs:61-114) through sqb200.perplexity.
CPU: on the oracle, the windowed, cached, teacher-forced scoring equals scoring
every position from a fresh prefill of its prefix (exact in the oracle), and
log_softmax_at matches a direct f64 formula. GPU: the CUDA path's NLL per token
stays within tolerance of the oracle's."""
import numpy as np
import pytest

from oracle import oracle as O
from sqb200 import gguf_synth as G
from sqb200 import perplexity as PPL

N_CTX = 8


def ids_for(spec, n, seed=5):
    return G.prompt_ids(n, seed=seed, high=G.SPECS[spec]["vocab"])


def bos_for(cfg):
    """The model's BOS id, or 1 where the synthetic model's vocabulary is smaller
    than Llama's BOS (128000)."""
    return int(cfg.bos_token_id) if cfg.bos_token_id < cfg.vocab_size else 1


def test_log_softmax_at():
    rng = np.random.default_rng(0)
    l = (rng.standard_normal(1000) * 3).astype(np.float32)
    want = float(l[17]) - np.log(np.sum(np.exp(l.astype(np.float64))))
    assert abs(PPL.log_softmax_at(l, 17) - want) < 1e-9


def test_oracle_cached_scoring_equals_fresh_prefixes():
    from oracle import build as oracle_build
    oracle_build.build()
    path = G.ensure_gguf("tiny", "q8_0")
    ids = ids_for("tiny", 2 * (N_CTX - 1) + 3)  # two windows, a ragged tail that is dropped
    m = O.Model(path)
    bos = bos_for(m.config)
    state = {}

    def fwd(x):
        state["logits"] = m.forward(x)

    got = PPL.perplexity(fwd, lambda: state["logits"], m.reset, ids, bos, n_ctx=N_CTX, log=None)
    # independent: every scored position from a fresh prefill of its whole prefix
    nll, scored = 0.0, 0
    for w in range(2):
        window = np.concatenate([[bos], ids[w * (N_CTX - 1):(w + 1) * (N_CTX - 1)]]).astype(np.uint32)
        for i in range(N_CTX // 2, len(window)):
            m.reset()
            nll -= PPL.log_softmax_at(m.forward(window[:i]), int(window[i]))
            scored += 1
    m.close()
    assert got["windows"] == 2 and got["scored_tokens"] == scored == 2 * (N_CTX - N_CTX // 2)
    assert got["nll_per_token"] == nll / scored
    assert got["ppl"] == pytest.approx(np.exp(nll / scored), rel=1e-12)


def test_rejects_tiny_context():
    with pytest.raises(ValueError):
        PPL.perplexity(None, None, None, [1, 2, 3], 0, n_ctx=3)


@pytest.mark.gpu
def test_cuda_perplexity_matches_oracle(gpu_lib):
    from sqb200 import lib
    path = G.ensure_gguf("small", "q8_0")
    ids = ids_for("small", 3 * 15)
    om = O.Model(path)
    bos = bos_for(om.config)
    state = {}

    def fwd(x):
        state["logits"] = om.forward(x)

    want = PPL.perplexity(fwd, lambda: state["logits"], om.reset, ids, bos, n_ctx=16, log=None)
    om.close()
    m = lib.Model(path, device=0)
    ctx = m.new_context(64)
    got = PPL.context_perplexity(ctx, ids, bos, n_ctx=16, log=None)
    ctx.close()
    m.close()
    assert got["scored_tokens"] == want["scored_tokens"]
    assert abs(got["nll_per_token"] - want["nll_per_token"]) <= 1e-3
