"""Multi-GPU host logic on CPU: the sequence partition, the whole-job
throughput aggregation and the gather of per-rank outputs, run as two gloo
ranks (one process each, like one process per GPU).  Each rank decodes its own
shard of sequences with the oracle (standing in for its GPU); rank 0 checks the
gathered result against an unsharded decode of all sequences."""
import os
import socket

import numpy as np
import pytest

from kvdata import R, SCALE, W

import sharding


def test_lpt_partition_covers_and_balances():
    rng = np.random.default_rng(7)
    lens = np.floor(np.exp(rng.uniform(np.log(128), np.log(65536), 512))).astype(np.int64)
    for k in (1, 2, 3, 4, 8):
        parts, loads = sharding.lpt_partition(lens, k)
        flat = sorted(s for p in parts for s in p)
        assert flat == list(range(lens.size))  # disjoint cover
        assert loads == [int(lens[p].sum()) for p in parts]
        assert max(loads) - min(loads) <= int(lens.max())  # LPT bound
        assert all(p == sorted(p) for p in parts)
    # deterministic, ties to the lower part
    assert sharding.lpt_partition([5, 5, 5, 5], 2) == ([[0, 2], [1, 3]], [10, 10])
    assert sharding.lpt_partition([], 3) == ([[], [], []], [0, 0, 0])
    with pytest.raises(ValueError):
        sharding.lpt_partition([1], 0)


def test_aggregate_single_process():
    assert sharding.aggregate_throughput(12, 3.0) == (12.0, 3.0)


BS, H, SEED = 16, 4, 21


def _lens():
    return np.random.default_rng(SEED).integers(0, 200, 9).astype(np.int64)


def _decode(kvoracle, seqs, lens, q):
    """Oracle decode of the given sequences on a pool holding only them (what one rank owns)."""
    lens = np.asarray([lens[s] for s in seqs], np.int64)
    nb = int(sum((L + BS - 1) // BS for L in lens)) + 1
    pool = kvoracle.Pool(1, nb, BS, R, 64, True)
    offs, tabs, k = [0], [], 0
    for i, s in enumerate(seqs):
        L = int(lens[i])
        need = (L + BS - 1) // BS
        tabs.extend(range(k, k + need))
        k += need
        offs.append(len(tabs))
        if L:
            rows = kvoracle.gen_rows(SEED, 0, np.full(L, s, np.uint32), np.arange(L, dtype=np.uint32), W,
                                     0.01, n_threads=1)
            t = np.arange(L)
            pool.put_rows(0, np.array(tabs[offs[i]:offs[i + 1]], np.uint32)[t // BS], t % BS, rows)
    return pool.attention_batch(0, np.array(offs, np.uint32), np.array(tabs or [0], np.uint32),
                                lens.astype(np.uint32), q[list(seqs)], SCALE, n_threads=1)


def _rank(rank, world, port, out_dir):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "oracle"), os.path.join(root, "mobile-moe.zig_b200")]
    import torch
    import torch.distributed as dist

    import kvoracle
    import sharding as sh

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lens = _lens()
        q = np.random.default_rng(SEED + 1).standard_normal((lens.size, H, W)).astype(np.float32)
        parts, loads = sh.lpt_partition(lens, world)
        mine = parts[rank]
        local = _decode(kvoracle, mine, lens, q) if mine else np.zeros((0, H, R), np.float32)
        full = sh.gather_to_root(torch.from_numpy(local), parts, dist)
        work, secs = sh.aggregate_throughput(int(lens[mine].sum()), 1.0 + rank, dist)
        if rank == 0:
            np.savez(os.path.join(out_dir, "rank0.npz"), full=full.numpy(), work=work, secs=secs,
                     loads=np.array(loads))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_shard_decode_and_gather(tmp_path, oracle):
    import torch.multiprocessing as mp

    world = 2
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    r = np.load(tmp_path / "rank0.npz")
    lens = _lens()
    q = np.random.default_rng(SEED + 1).standard_normal((lens.size, H, W)).astype(np.float32)
    want = _decode(oracle, list(range(lens.size)), lens, q)
    # sharding changes where a sequence lives, not its result
    assert np.array_equal(r["full"], want)
    assert float(r["work"]) == float(lens.sum())  # summed over ranks
    assert float(r["secs"]) == 2.0  # slowest rank
    assert int(r["loads"].sum()) == int(lens.sum())
