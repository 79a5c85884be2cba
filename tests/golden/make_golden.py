"""Generate the end-to-end golden fixtures (tests/golden/e2e_*.npz).

The reference pins no end-to-end output (its tests are op-level), so these files
pin the oracle's: for each small seeded model (the synthetic GGUF writer with seed
0) and weight type, the prompt, the oracle's greedy ids for 16 steps (EOS ignored,
text_generator.rs:58-97) and its full logits after the prompt and after the last
step, plus the GGUF's sha256 so a change of the writer is caught too. The CPU tests
check that the oracle still reproduces them bit for bit; the GPU tests check the
CUDA path against them (identical ids, logits within tolerance).

    python tests/golden/make_golden.py              # tiny / small models (seconds)
    python tests/golden/make_golden.py --configs    # BASELINE-shape cases (CONFIG_CASES)
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, os.path.join(ROOT, "squirrel-rs_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

CASES = [(spec, wt) for spec in ("tiny", "small") for wt in ("q8_0", "q4_0", "bf16")]
# the aarch64 scheme (Q8_0 activations, W8A8 / W4A8 integer block dots): oracle pins only
CASES_A8 = [(spec, wt) for spec in ("tiny", "small") for wt in ("q8_0", "q4_0")]
PROMPT_LEN, STEPS, PROMPT_SEED = 8, 16, 21

# The BASELINE configurations' own shapes (the 1B model with its tied LM head and
# 128256-row vocabulary; the 8B model with head_dim 128 and an untied LM head). The
# oracle takes minutes on these, too long inside a GPU test, so their greedy ids
# and the logits after the prompt and after the last step are pinned here. Prompts
# are the bench's: uniform ids in [0, 128000) from seed 1234.
CONFIG_CASES = {
    # config 1: 32-token prompt, then greedy decode (the bench's headline workload)
    "cfg1_1b_q8_0": dict(spec="1b", wt="q8_0", prompt=32, steps=33),
    # config 3: 2048-token prompt, then decode at KV 2048-2064 (split-KV attention)
    "cfg3_1b_q4_0": dict(spec="1b", wt="q4_0", prompt=2048, steps=17),
    # config 4: an 8192-token BF16 prefill (the next id and its logits)
    "cfg4_1b_bf16": dict(spec="1b", wt="bf16", prompt=8192, steps=1),
    # config 5's shape on one GPU: 16-token prompt, then greedy decode
    "cfg5_8b_q8_0": dict(spec="8b", wt="q8_0", prompt=16, steps=9),
    # config 1's model under the aarch64 scheme (Q8_0 activations, integer block dots);
    # the top-2 logit margin of every step is pinned too (the GPU test, teacher-forced,
    # compares ids only at steps whose margin exceeds the scheme's last-bit noise)
    "cfg1_1b_q8_0_a8": dict(spec="1b", wt="q8_0", prompt=32, steps=17, acts_q8=True),
}
CONFIG_PROMPT_SEED = 1234


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def fixture_path(spec, wt, acts_q8=False):
    return os.path.join(HERE, f"e2e_{spec}_{wt}{'_a8' if acts_q8 else ''}.npz")


def config_fixture_path(name):
    return os.path.join(HERE, f"{name}.npz")


def compute_config(name):
    from oracle import oracle as O
    from sqb200 import gguf_synth as G
    c = CONFIG_CASES[name]
    path = G.ensure_gguf(c["spec"], c["wt"])
    prompt = G.prompt_ids(c["prompt"], seed=CONFIG_PROMPT_SEED)
    m = O.Model(path, acts_q8=c.get("acts_q8", False))
    ids, _, logits = m.generate(prompt, c["steps"], want_logits=True)
    m.close()
    margins = [float(np.diff(np.sort(lg)[-2:])[0]) for lg in logits]
    return dict(prompt=np.asarray(prompt, np.uint32), ids=np.asarray(ids, np.uint32),
                logits_first=np.asarray(logits[0], np.float32), logits_last=np.asarray(logits[-1], np.float32),
                margins=np.asarray(margins, np.float32), gguf_sha256=np.array(sha256(path)))


def compute(spec, wt, acts_q8=False):
    from oracle import oracle as O
    from sqb200 import gguf_synth as G
    path = G.ensure_gguf(spec, wt)
    prompt = G.prompt_ids(PROMPT_LEN, seed=PROMPT_SEED, high=G.SPECS[spec]["vocab"])
    m = O.Model(path, acts_q8=acts_q8)
    ids, _, logits = m.generate(prompt, STEPS, want_logits=True)
    m.close()
    return dict(prompt=np.asarray(prompt, np.uint32), ids=np.asarray(ids, np.uint32),
                logits_first=np.asarray(logits[0], np.float32), logits_last=np.asarray(logits[-1], np.float32),
                gguf_sha256=np.array(sha256(path)))


def main():
    from oracle import build as oracle_build
    oracle_build.build()
    if len(sys.argv) > 1 and sys.argv[1] == "--configs":  # the BASELINE-shape cases (minutes each)
        for name in sys.argv[2:] or list(CONFIG_CASES):
            np.savez_compressed(config_fixture_path(name), **compute_config(name))
            print("wrote", config_fixture_path(name), flush=True)
        return
    for spec, wt in CASES:
        np.savez_compressed(fixture_path(spec, wt), **compute(spec, wt))
        print("wrote", fixture_path(spec, wt))
    for spec, wt in CASES_A8:
        np.savez_compressed(fixture_path(spec, wt, True), **compute(spec, wt, True))
        print("wrote", fixture_path(spec, wt, True))


if __name__ == "__main__":
    main()
