"""The reference's generation loop over token ids (TextTokenGenerator::generate,
text_generator.rs:38-101), driving a context through the C ABI.

The first forward prefills the prompt; each later step feeds only the new token
against the KV cache, or — with SQUIRREL_NO_KV_CACHE set to anything but "0" —
resets the cache and feeds the whole sequence again (text_generator.rs:10-13,
76-79). Generation stops at the model's EOS id unless SQUIRREL_IGNORE_EOS is set
(:16-19, 67-73). Progress goes to stderr in the reference's format
(`[prompt: N tokens]`, `[step   N:     X.Xms]`, :50, 67-93), with the new token id
where the reference prints the decoded text (the tokenizer is not part of this
library).
"""
import os
import sys
import time

import numpy as np


def env_flag(name: str) -> bool:
    v = os.environ.get(name)
    return v is not None and v != "0"


def generate_ids(forward, reset, prompt, max_tokens: int, eos_id: int, no_kv_cache=None, ignore_eos=None,
                 log=sys.stderr):
    """forward(ids) -> next greedy id (one Model::forward plus GreedySampler::sample);
    reset() empties the KV cache. Returns the generated ids (EOS excluded)."""
    no_kv_cache = env_flag("SQUIRREL_NO_KV_CACHE") if no_kv_cache is None else no_kv_cache
    ignore_eos = env_flag("SQUIRREL_IGNORE_EOS") if ignore_eos is None else ignore_eos
    tokens = [int(t) for t in prompt]
    if log:
        print(f"[prompt: {len(tokens)} tokens]", file=log)
    inp = list(tokens)
    out = []
    for step in range(1, max_tokens + 1):
        t0 = time.perf_counter()
        nxt = int(forward(np.asarray(inp, dtype=np.uint32)))
        ms = (time.perf_counter() - t0) * 1e3
        if nxt == eos_id and not ignore_eos:
            if log:
                print(f"[step {step:>3}: {ms:>7.1f}ms]  <eos>", file=log)
            break
        tokens.append(nxt)
        out.append(nxt)
        if no_kv_cache:
            reset()
            inp = list(tokens)
        else:
            inp = [nxt]
        if log:
            print(f"[step {step:>3}: {ms:>7.1f}ms]  {nxt}", file=log)
    return out


def generate(ctx, prompt, max_tokens: int, eos_id: int, **kw):
    """generate_ids on a sqb200.lib context (its forward returns the device argmax)."""
    return generate_ids(ctx.forward, ctx.reset, prompt, max_tokens, eos_id, **kw)
