"""Tensor parallel on two GPUs (one process per GPU, NCCL): the sharded model's
greedy ids equal the single-GPU model's and the CPU oracle's, and its gathered
logits stay within the model tests' tolerance. Skipped with fewer than 2 GPUs."""
import os

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ABS_TOL, REL_TOL = 1e-2, 1e-3


def _tp_rank(rank, size, path, prompt, steps, qin, qout):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from sqb200 import lib
    try:
        if rank == 0:
            uid = lib.nccl_unique_id()
            for _ in range(size - 1):
                qin.put(uid)
        else:
            uid = qout.get(timeout=60)
        m = lib.Model(path, device=rank, tp_rank=rank, tp_size=size, nccl_id=uid)
        ctx = m.new_context(len(prompt) + steps + 4)
        first = ctx.forward(prompt)
        logits = ctx.logits()  # collective: every rank gathers the vocabulary shards
        ids = [int(first)] + [int(i) for i in ctx.decode_steps(steps)]
        ctx.close()
        m.close()
        qin.put(("ok", rank, ids, logits if rank == 0 else None))
    except Exception as e:  # report instead of hanging the parent
        qin.put(("err", rank, repr(e), None))


@pytest.mark.parametrize("wt", ["q8_0", "bf16"])
def test_tp2_matches_single_gpu_and_oracle(wt):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from sqb200 import gguf_synth as G
    from sqb200 import lib
    path = G.ensure_gguf("small", wt)
    prompt = G.prompt_ids(12, seed=5, high=4000)
    steps = 10
    single = lib.Model(path, device=0)
    sctx = single.new_context(len(prompt) + steps + 4)
    s_first = sctx.forward(prompt)
    s_logits = sctx.logits()
    s_ids = [int(s_first)] + [int(i) for i in sctx.decode_steps(steps)]
    sctx.close()
    single.close()
    om = O.Model(path)
    o_ids, _, _ = om.generate(prompt, steps + 1)
    om.close()

    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    qin, qout = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, path, prompt, steps, qin if r == 0 else qin, qout))
             for r in range(2)]
    for p in procs:
        p.start()
    # rank 0 puts the id for rank 1 on qin; relay it
    uid = qin.get(timeout=120)
    qout.put(uid)
    results = [qin.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    errs = [r for r in results if r[0] != "ok"]
    assert not errs, errs
    r0 = next(r for r in results if r[1] == 0)
    r1 = next(r for r in results if r[1] == 1)
    assert r0[2] == r1[2], "ranks disagree"
    assert r0[2] == s_ids, (r0[2], s_ids)
    assert r0[2] == [int(i) for i in o_ids], (r0[2], list(o_ids))
    diff = np.abs(r0[3] - s_logits)
    assert float(diff.max()) <= ABS_TOL, float(diff.max())
    assert float((diff / np.maximum(np.abs(s_logits), 1.0)).max()) <= REL_TOL
