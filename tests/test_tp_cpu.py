"""Tensor-parallel sharding on the host (no GPU): sq_tp_shard_tensor's shards put
back together give the tensor again, and with world_size 2 (gloo ranks on CPU) the
shards' partial projections summed by an all-reduce give the unsharded projection
- the arithmetic the multi-GPU forward relies on (column-parallel Q/K/V/gate/up,
row-parallel O/down with an all-reduce)."""
import os

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")


def q8_rows(rows, in_dim, seed):
    """rows x in_dim/32 Q8_0 blocks of N(0, 0.02) weights, quantized by the oracle."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, in_dim)) * 0.02).astype(np.float32)
    return np.stack([O.quantize_row_q8_0(r) for r in w]), w


def shard(name, dims, data, rank, size):
    from sqb200 import lib
    return lib.tp_shard_tensor(name, O.Q8_0, dims, data, rank, size)


@pytest.mark.parametrize("size", [2, 4])
def test_row_shards_concatenate(size):
    blocks, _ = q8_rows(64, 256, 1)
    got = [shard("blk.3.attn_q.weight", [256, 64], blocks, r, size) for r in range(size)]
    assert all(d == [256, 64 // size] for d, _ in got)
    assert np.array_equal(np.concatenate([b for _, b in got]), blocks.reshape(-1).view(np.uint8))


@pytest.mark.parametrize("size", [2, 4])
def test_column_shards_concatenate_per_row(size):
    blocks, _ = q8_rows(16, 512, 2)  # ffn_down-like: rows of 16 blocks
    got = [shard("blk.0.ffn_down.weight", [512, 16], blocks, r, size) for r in range(size)]
    assert all(d == [512 // size, 16] for d, _ in got)
    per_row = blocks.reshape(16, -1)
    rebuilt = np.concatenate([b.reshape(16, -1) for _, b in got], axis=1)
    assert np.array_equal(rebuilt, per_row)


def test_replicated_and_errors():
    from sqb200 import lib
    norm = np.arange(256, dtype=np.float32)
    d, b = lib.tp_shard_tensor("blk.0.attn_norm.weight", O.F32, [256], norm, 1, 2)
    assert d == [256] and np.array_equal(b.view(np.float32), norm)
    blocks, _ = q8_rows(3, 256, 3)
    with pytest.raises(lib.KernelError) as e:  # 3 rows do not split in 2
        shard("output.weight", [256, 3], blocks, 0, 2)
    assert e.value.kind == "ShapeMismatch"
    blocks, _ = q8_rows(4, 96, 4)  # 3 blocks a row do not split in 2 whole-block runs
    with pytest.raises(lib.KernelError):
        shard("blk.0.attn_output.weight", [96, 4], blocks, 0, 2)


def _rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        E, F = 256, 512
        rng = np.random.default_rng(7)
        x = rng.standard_normal((1, E)).astype(np.float32)
        up, _ = q8_rows(F, E, 11)      # column-parallel: rows split
        down, _ = q8_rows(E, F, 12)    # row-parallel: each row's blocks split
        d_up, b_up = shard("blk.0.ffn_up.weight", [E, F], up, rank, world)
        d_dn, b_dn = shard("blk.0.ffn_down.weight", [F, E], down, rank, world)
        h = O.linear(x, b_up, O.Q8_0, d_up[1])                      # this rank's F/world rows
        part = O.linear(h, b_dn, O.Q8_0, d_dn[1])  # partial sums over its inputs
        t = torch.from_numpy(np.ascontiguousarray(part, dtype=np.float32))
        dist.all_reduce(t)
        full_h = O.linear(x, up.reshape(-1).view(np.uint8), O.Q8_0, F)
        full = O.linear(full_h, down.reshape(-1).view(np.uint8), O.Q8_0, E)
        q.put((rank, float(np.abs(t.numpy() - full).max()), float(np.abs(full).max())))
    finally:
        dist.destroy_process_group()


def test_two_rank_partial_projections_sum_to_full():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = []
    for _ in procs:
        out.append(q.get(timeout=90))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, scale in out:
        assert err <= 1e-5 * max(1.0, scale), (rank, err, scale)
