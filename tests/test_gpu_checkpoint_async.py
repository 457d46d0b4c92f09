"""Background checkpoint save while serving continues
(kvcache_save_to_file_v2_async, the asynchronous checkpoint I/O around
src/kv_cache.zig:453-591).

The file must hold the cache exactly as it was at the call, although the
test appends to every sequence, rewrites part of one sequence after a
truncate and resets another while the worker copies the pool: those writes go
to copies of the snapshot's blocks (copy-on-write), never to the blocks being
saved.  Afterwards every block is either free or held by a live sequence."""
import numpy as np
import pytest

from kvdata import W

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kv():
    import torch

    import kvcu

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    kvcu.init(0)
    return kvcu


def test_async_save_keeps_the_snapshot_while_serving(kv, tmp_path):
    import torch

    lens = [70, 300, 1500, 64, 900, 2000]
    nl, bs, n = 3, 64, len(lens)
    nb = sum((L + 200 + bs - 1) // bs for L in lens) + 40
    c = kv.KVCache.with_blocks(nl, 512, 64, nb, block_size=bs, quantized=True)
    for _ in range(n - 1):
        c.seq_create()
    ids = np.arange(n, dtype=np.uint32)
    for i in range(n):
        c.seq_ensure_capacity(i, lens[i] + 100)
    for layer in range(nl):
        c.prefill_synthetic(layer, ids, lens, 61, 0.01)
    torch.cuda.synchronize()
    snap = {(layer, s): c.gather(layer, s) for layer in range(nl) for s in range(n)}
    tables = [c.seq_block_table(s) for s in range(n)]
    path = tmp_path / "async.ckpt"
    job = c.saveToFileV2Async(path)
    rng = np.random.default_rng(61)
    # serving goes on: one token per sequence per layer, a few steps
    for step in range(4):
        pos = (np.array(lens) + step).astype(np.uint32)
        for layer in range(nl):
            c.appendBatch(layer, ids, pos, rng.standard_normal((n, W)).astype(np.float32))
    # rewrite the tail of sequence 2 inside the snapshot's range, reset sequence 5
    c.seq_truncate(2, 1000)
    for layer in range(nl):
        c.appendBatch(layer, np.array([2], np.uint32), np.array([1000], np.uint32),
                      rng.standard_normal((1, W)).astype(np.float32))
    c.seq_reset(5)
    job.wait()
    # blocks: every one either free or in a live table once per holder
    live = [b for s in range(n) for b in c.seq_block_table(s)]
    assert c.numFreeBlocks() + len(set(live)) == nb
    assert all(c.refcount(b) == live.count(b) for b in set(live))
    # the file is the snapshot
    d = kv.KVCache.with_blocks(nl, 512, 64, nb, block_size=bs, quantized=True)
    d.loadFromFileV2(path)
    assert d.num_seqs == n
    for s in range(n):
        assert d.seq_len(s) == lens[s]
        assert d.seq_block_table(s) == tables[s]
        for layer in range(nl):
            assert np.array_equal(d.gather(layer, s), snap[(layer, s)]), (layer, s)
    # the live cache kept its own writes: sequence 2 was truncated and extended
    assert c.seq_len(2) == 1001 and c.seq_len(5) == 0
    assert np.array_equal(c.gather(0, 2)[:1000], snap[(0, 2)][:1000])
    d.deinit()
    c.deinit()


def test_async_save_refuses_a_second_save_and_loads_while_running(kv, tmp_path):
    c = kv.KVCache.with_blocks(1, 512, 64, 64, block_size=64, quantized=True)
    c.seq_ensure_capacity(0, 3000)
    c.prefill_synthetic(0, [0], [3000], 62, 0.0)
    job = c.saveToFileV2Async(tmp_path / "a.ckpt")
    with pytest.raises(kv.KVCudaError):
        c.saveToFileV2Async(tmp_path / "b.ckpt")
    with pytest.raises(kv.KVCudaError):
        c.loadFromFileV2(tmp_path / "a.ckpt")
    job.wait()
    assert c.refcount(c.seq_block_table(0)[0]) == 1
    d = kv.KVCache.with_blocks(1, 512, 64, 64, block_size=64, quantized=True)
    d.loadFromFileV2(tmp_path / "a.ckpt")
    assert np.array_equal(d.gather(0, 0), c.gather(0, 0))
    d.deinit()
    c.deinit()
