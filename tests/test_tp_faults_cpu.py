"""Failure detection of a tensor-parallel group on the host (sqb200.tp), with gloo
ranks on the CPU: no GPU, no NCCL, nothing faults or hangs a device. A rank that
dies before the group forms, or leaves between steps, is named by the others
within the time limit instead of leaving them blocked; a slow rank inside the
limit is waited for."""
import os
import time

import pytest

torch = pytest.importorskip("torch")

TIMEOUT_S = 3.0


def _rank(rank, world, port, scenario, q):
    import datetime

    import torch.distributed as dist
    from sqb200 import tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    out = None
    try:
        grp = tp.Group.from_default_store(timeout_s=TIMEOUT_S)
        if scenario == "dead_before_init" and rank == world - 1:
            out = ("left",)
            return
        if scenario == "slow" and rank == 1:
            time.sleep(1.0)
        if scenario == "reuse":
            # a second share_id, a second group and a repeated tag must wait for fresh
            # keys: rank 0 publishes each new id late, and a rank that left after the
            # first "step" check-in must be missed at the second one
            ids = [grp.share_id(lambda: b"first" + bytes(123))]
            if rank == 0:
                time.sleep(0.5)
            ids.append(grp.share_id(lambda: b"second" + bytes(122)))
            grp2 = tp.Group.from_default_store(timeout_s=TIMEOUT_S)
            if rank == 0:
                time.sleep(0.5)
            ids.append(grp2.share_id(lambda: b"third" + bytes(123)))
            grp.check_in("step")
            if rank == 1:
                out = ("left",)
                return
            try:
                grp.check_in("step")
                out = ("ok", ids, None)
            except tp.GroupTimeout as e:
                out = ("ok", ids, sorted(e.missing))
            return
        t0 = time.monotonic()
        try:
            nid = grp.share_id(lambda: b"id-from-rank-0" + bytes(114))
        except tp.GroupTimeout as e:
            out = ("timeout", sorted(e.missing), time.monotonic() - t0)
            return
        if scenario == "leaves_between_steps":
            grp.check_in("step-1")
            if rank == 1:
                out = ("left",)
                return
            t0 = time.monotonic()
            try:
                grp.check_in("step-2")
            except tp.GroupTimeout as e:
                out = ("timeout", sorted(e.missing), time.monotonic() - t0)
                return
        out = ("ok", nid)
    finally:
        q.put((rank, out))
        if out and out[0] != "left":
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def run(scenario, world=3):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + (os.getpid() + hash(scenario)) % 800
    procs = [ctx.Process(target=_rank, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=90) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_every_rank_gets_rank0_id():
    res = run("healthy")
    ids = {r: v[1] for r, v in res.items()}
    assert all(v[0] == "ok" for v in res.values()), res
    assert len(set(ids.values())) == 1 and ids[0].startswith(b"id-from-rank-0")


def test_dead_rank_is_named_not_waited_for():
    res = run("dead_before_init")
    assert res[2] == ("left",)
    for r in (0, 1):
        kind, missing, waited = res[r]
        assert kind == "timeout" and missing == [2], res
        assert waited < TIMEOUT_S + 5.0  # ends near the limit: no hang


def test_slow_rank_within_limit_is_waited_for():
    res = run("slow")
    assert all(v[0] == "ok" for v in res.values()), res


def test_rank_leaving_between_steps_is_found_before_the_next_step():
    res = run("leaves_between_steps")
    assert res[1] == ("left",)
    for r in (0, 2):
        kind, missing, waited = res[r]
        assert kind == "timeout" and missing == [1], res
        assert waited < TIMEOUT_S + 5.0


def test_keys_are_not_reused_across_groups_ids_and_tags():
    """A second share_id, a second group and a repeated check-in tag wait for keys
    of their own instead of passing on keys an earlier phase left in the store."""
    res = run("reuse")
    assert res[1] == ("left",)
    for r in (0, 2):
        kind, ids, missing = res[r]
        assert kind == "ok", res
        assert [i[:6].rstrip(b"\0") for i in ids] == [b"first", b"second", b"third"], res
        assert missing == [1], res
