"""Teacher-forced perplexity over token ids (bin/perplexity.rs:61-114), driving a
context through the C ABI.

The ids are cut into windows of n_ctx - 1 tokens, each led by BOS. Per window the
cache starts empty, the first n_ctx / 2 tokens are prefilled in one pass (burn-in),
and from there every position is scored with log-softmax of the current logits at
the actual next token, then that token is fed (teacher forcing). Returns the mean
negative log-likelihood per scored token and its exponential. The corpus
(wikitext-2) and the tokenizer the reference binary reads are not part of this
library; any id sequence works.
"""
import sys

import numpy as np


def log_softmax_at(logits, idx: int) -> float:
    """log p(idx) under softmax(logits) in f64 with the max subtracted
    (perplexity.rs:110-114; the f64 sum is numpy's pairwise sum)."""
    l = np.asarray(logits, dtype=np.float32)
    mx = float(np.max(l))
    s = float(np.sum(np.exp(l.astype(np.float64) - mx)))
    return float(l[idx]) - mx - float(np.log(s))


def perplexity(forward, logits, reset, ids, bos: int, n_ctx: int = 512, max_windows: int = 0, log=sys.stderr):
    """forward(ids) runs Model::forward on the context; logits() returns the last
    row's logits; reset() gives the window a fresh cache."""
    if n_ctx < 4:
        raise ValueError("n_ctx must be at least 4")
    ids = np.asarray(ids, dtype=np.uint32)
    per_window = n_ctx - 1  # one slot for BOS
    total = len(ids) // per_window
    n_windows = total if max_windows == 0 else min(max_windows, total)
    burn = n_ctx // 2
    nll, scored = 0.0, 0
    for w in range(n_windows):
        window = np.concatenate([np.array([bos], np.uint32), ids[w * per_window:(w + 1) * per_window]])
        reset()
        forward(window[:burn])
        for i in range(burn, len(window)):
            nll -= log_softmax_at(logits(), int(window[i]))
            scored += 1
            if i + 1 < len(window):
                forward(window[i:i + 1])
        if log:
            print(f"[window {w + 1:>4}/{n_windows}] ppl so far: {np.exp(nll / scored):.4f}", file=log)
    if scored == 0:
        raise ValueError("no window fits the ids")
    return {"nll_per_token": nll / scored, "ppl": float(np.exp(nll / scored)), "scored_tokens": scored,
            "windows": n_windows}


def context_perplexity(ctx, ids, bos: int, **kw):
    """perplexity() on a sqb200.lib context."""
    return perplexity(ctx.forward, ctx.logits, ctx.reset, ids, bos, **kw)
