"""Failure detection of the bounded device waits, without a GPU fault: the
persistent decode kernel (one GPU and tensor parallel), the peer all-reduce and the
streaming matvec.

Every cross-CTA wait of the decode kernel is bounded (about 2 s of SM clocks); when
one expires the kernel sets an error word, every other wait sees it and gives up at
once, the CTAs let their in-flight copies land and return, and the host reports
SQ_ERR_TIMEOUT and clears the kernel's counters. Here the wait runs out because a
word is never written: SQ_TEST_DROP_EXCHANGE=n (read when the context is created)
makes the n-th launch skip one residual word after layer 0's O projection, so the
gate/up stage polls a word that nothing sets. Nothing traps or hangs; the test then
checks that the same context decodes the oracle's ids again."""
import os
import time

import numpy as np
import pytest

from golden import make_golden as MG  # tests/golden/make_golden.py

pytestmark = pytest.mark.gpu


def test_decode_wait_expires_reports_timeout_and_context_recovers(gpu_lib, monkeypatch):
    from sqb200 import gguf_synth as G
    from sqb200 import lib
    z = np.load(MG.fixture_path("small", "q8_0"))
    prompt, ids = z["prompt"], z["ids"]
    monkeypatch.setenv("SQ_TEST_DROP_EXCHANGE", "3")  # the context's third decode launch
    m = lib.Model(G.ensure_gguf("small", "q8_0"), device=0)
    ctx = m.new_context(64)
    monkeypatch.delenv("SQ_TEST_DROP_EXCHANGE")
    try:
        assert ctx.launches_per_token == 1  # the persistent kernel serves this model
        assert ctx.forward(prompt) == ids[0]  # prefill: not a decode launch
        t0 = time.monotonic()
        with pytest.raises(lib.KernelError) as e:
            ctx.decode_steps(5)  # launches 1..5; the third one loses a word
        assert e.value.kind == "Timeout", e.value
        assert time.monotonic() - t0 < 60  # one expired wait (~2 s), then every wait gives up at once
        # the device and the context stay usable: a fresh prefill decodes the oracle's ids
        ctx.reset()
        assert ctx.forward(prompt) == ids[0]
        assert np.array_equal(ctx.decode_steps(len(ids) - 1), ids[1:])
        lib.wait_status()
    finally:
        ctx.close()
        m.close()


def _matvec_child(q):
    """A fresh process (the launch count starts at zero): its second k_matvec launch
    leaves its first tile uncopied (SQ_TEST_SKIP_MATVEC=2)."""
    os.environ["SQ_TEST_SKIP_MATVEC"] = "2"
    try:
        import torch
        from oracle import oracle as O
        from sqb200 import gguf_synth as G
        from sqb200 import lib
        rng = np.random.default_rng(7)
        k, n = 2048, 512
        x = torch.from_numpy(rng.standard_normal((1, k)).astype(np.float32)).cuda()
        w = torch.from_numpy(G.quantize((rng.standard_normal(n * k) * 0.02).astype(np.float32), O.Q8_0)).cuda()
        first = lib.linear(x, w, O.Q8_0, n)  # launch 1
        torch.cuda.synchronize()
        lib.wait_status()
        t0 = time.monotonic()
        lib.linear(x, w, O.Q8_0, n)  # launch 2: the consumers' wait for tile 0 runs out
        torch.cuda.synchronize()
        try:
            lib.wait_status()
            kind = "none"
        except lib.KernelError as e:
            kind = e.kind
        took = time.monotonic() - t0
        again = lib.linear(x, w, O.Q8_0, n)  # launch 3: a normal call after the error was cleared
        torch.cuda.synchronize()
        lib.wait_status()
        same = bool(torch.equal(first, again))
        q.put(("ok", kind, took, same))
    except Exception as e:  # report instead of hanging the parent
        q.put(("err", repr(e), 0.0, False))


def test_matvec_wait_expires_reports_timeout_and_next_call_is_correct():
    """The streaming matvec's bounded waits (k_matvec): a tile whose copy is never
    issued makes the consumers' wait expire (and the producer's wait for their
    release, and its drain of that slot); the kernel returns, sq_wait_status reports
    Timeout, and the next call on the same device gives the first call's bits."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_matvec_child, args=(q,))
    p.start()
    try:
        status, kind, took, same = q.get(timeout=300)
    finally:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert status == "ok", kind
    assert kind == "Timeout", kind
    assert took < 60, took  # three bounded waits of ~2 s
    assert same


def _fault_rank(rank, path, prompt, ids, mode, qin, qout):
    """Rank 1 leaves one exchange unwritten in its first decode steps: on the
    persistent kernel ("kernel") its partial of hidden row 0 after layer 0's O
    projection in its third launch (SQ_TEST_DROP_EXCHANGE=3), on the op-level step
    ("op") the flags of its third peer all-reduce (SQ_TEST_WITHHOLD_PARTIAL=3). A
    bounded wait on rank 0 expires and reports Timeout (rank 1's may too: it waits
    for its own word, or ran ahead while rank 0 waited); both ranks run the whole
    step, then re-synchronize (sq_tp_recover), reset their contexts and decode the
    oracle's ids again."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    if mode == "op":
        os.environ["SQB200_TP_DECODE"] = "op"
        if rank == 1:
            os.environ["SQ_TEST_WITHHOLD_PARTIAL"] = "3"
    from sqb200 import lib
    out = {"rank": rank}
    try:
        if rank == 0:
            uid = lib.nccl_unique_id()
            qin.put(("uid", uid))
        else:
            uid = qout.get(timeout=120)
        m = lib.Model(path, device=rank, tp_rank=rank, tp_size=2, nccl_id=uid)
        if mode == "kernel" and rank == 1:
            os.environ["SQ_TEST_DROP_EXCHANGE"] = "3"  # read when the context is created
        ctx = m.new_context(64)
        os.environ.pop("SQ_TEST_DROP_EXCHANGE", None)
        out["launches_per_token"] = ctx.launches_per_token
        out["first"] = int(ctx.forward(prompt))  # prefill: NCCL's all-reduces
        t0 = time.monotonic()
        try:
            ctx.decode_steps(4)  # decode rows
            out["fault"] = "none"
        except lib.KernelError as e:
            out["fault"] = e.kind
        out["fault_s"] = time.monotonic() - t0
        m.tp_recover()
        ctx.reset()
        out["ids"] = [int(ctx.forward(prompt))] + [int(i) for i in ctx.decode_steps(len(ids) - 1)]
        ctx.close()
        m.close()
        qin.put(("ok", out))
    except Exception as e:  # report instead of hanging the parent
        qin.put(("err", {"rank": rank, "error": repr(e)}))


@pytest.mark.parametrize("mode", ["kernel", "op"])
def test_tp_exchange_wait_expires_reports_timeout_and_group_recovers(mode):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from sqb200 import gguf_synth as G
    z = np.load(MG.fixture_path("small", "q8_0"))
    prompt, ids = z["prompt"], [int(i) for i in z["ids"]]
    path = G.ensure_gguf("small", "q8_0")
    ctx = mp.get_context("spawn")
    qin, qout = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_fault_rank, args=(r, path, prompt, ids, mode, qin, qout)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    try:
        while len(results) < 2:
            kind, val = qin.get(timeout=300)
            if kind == "uid":
                qout.put(val)  # rank 0's NCCL id, relayed to rank 1
            else:
                results.append((kind, val))
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    errs = [v for k, v in results if k != "ok"]
    assert not errs, errs
    by_rank = {v["rank"]: v for _, v in results}
    for v in by_rank.values():  # which decode path ran
        assert (v["launches_per_token"] == 1) == (mode == "kernel"), v
    assert by_rank[0]["fault"] == "Timeout", by_rank[0]  # waited for rank 1's missing word
    # rank 1 ran ahead while rank 0 waited, so its next wait may expire as well
    assert by_rank[1]["fault"] in ("none", "Timeout"), by_rank[1]
    assert by_rank[0]["fault_s"] < 60 and by_rank[1]["fault_s"] < 60
    for r in (0, 1):
        assert by_rank[r]["ids"] == ids, by_rank[r]
