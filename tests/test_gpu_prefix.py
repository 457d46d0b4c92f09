"""Prefix blocks shared between sequences of one pool (kvcache_seq_cache_block,
kvcache_find_prefix_blocks, kvcache_seq_reuse_prefix_blocks) and copy-on-write
when a sequence writes into a block it shares: decode reads the shared blocks,
and no write ever changes another owner's data."""
import numpy as np
import pytest

from kvdata import REL_TOL, SCALE, W, rel_err_rows

pytestmark = pytest.mark.gpu

R, P, BS, H = 512, 64, 16, 20


@pytest.fixture(scope="module")
def kv():
    import torch

    import kvcu

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    kvcu.init(0)
    return kvcu


def _shared_pair(kv, quant, layers=2, seed=71):
    """Sequence 0: 74 tokens with its 4 full blocks registered; sequence 1
    reuses the 3 blocks of the 48-token common prefix and appends 20 tokens."""
    rng = np.random.default_rng(seed)
    c = kv.KVCache.with_blocks(layers, R, P, 64, BS, quantized=quant)
    c.seq_create()
    t0 = rng.integers(0, 50000, 74).astype(np.uint32)
    t1 = np.concatenate([t0[:48], rng.integers(0, 50000, 20).astype(np.uint32)])
    c.seq_ensure_capacity(0, 74)
    rows0 = rng.standard_normal((layers, 74, W)).astype(np.float32)
    for layer in range(layers):
        c.appendBatch(layer, np.zeros(74, np.uint32), np.arange(74, dtype=np.uint32), rows0[layer])
    prefix = kv.NO_HASH
    for bi in range(4):
        c.seq_cache_block(0, bi, t0[bi * BS:(bi + 1) * BS], prefix)
        prefix = kv.KVCache.computeHash(t0[bi * BS:(bi + 1) * BS], prefix)
    assert c.findPrefixBlocks(t1) == 3
    c.seq_reuse_prefix_blocks(1, t1, 3)
    assert c.seq_len(1) == 48
    assert c.seq_block_table(1) == c.seq_block_table(0)[:3]
    assert all(c.refcount(b) == 2 for b in c.seq_block_table(0)[:3])
    c.seq_ensure_capacity(1, 68)
    rows1 = rng.standard_normal((layers, 20, W)).astype(np.float32)
    for layer in range(layers):
        c.appendBatch(layer, np.ones(20, np.uint32), np.arange(48, 68, dtype=np.uint32), rows1[layer])
    return c, rows0, rows1


@pytest.mark.parametrize("quant", [True, False])
def test_shared_prefix_decode_matches_oracle(kv, oracle, quant):
    c, rows0, rows1 = _shared_pair(kv, quant)
    assert c.seq_block_table(1)[:3] == c.seq_block_table(0)[:3]  # appends went to fresh blocks
    lens = [74, 68]
    nb = 64
    o = oracle.Pool(2, nb, BS, R, P, quant)
    offs, tabs = [0], []
    for s, L in enumerate(lens):
        tab = np.array(c.seq_block_table(s), np.uint32)
        data = rows0 if s == 0 else np.concatenate([rows0[:, :48], rows1], axis=1)
        t = np.arange(L)
        for layer in range(2):
            o.put_rows(layer, tab[t // BS], t % BS, data[layer])
        tabs.extend(tab.tolist())
        offs.append(len(tabs))
    q = np.random.default_rng(5).standard_normal((2, H, W)).astype(np.float32)
    for layer in range(2):
        got = c.mlaDecode(layer, q, np.arange(2, dtype=np.uint32), SCALE)
        want = o.attention_batch(layer, np.array(offs, np.uint32), np.array(tabs, np.uint32),
                                 np.array(lens, np.uint32), q, SCALE)
        assert rel_err_rows(got, want) <= REL_TOL
    # the shared prefix reads the same bytes through either sequence
    for layer in range(2):
        assert np.array_equal(c.gather(layer, 1)[:48], c.gather(layer, 0)[:48])


@pytest.mark.parametrize("quant", [True, False])
def test_write_into_shared_block_copies_it_first(kv, quant):
    c, rows0, rows1 = _shared_pair(kv, quant)
    before0 = [c.gather(layer, 0) for layer in range(2)]
    shared = c.seq_block_table(0)[2]
    # sequence 1 falls back into the shared third block and writes position 40
    c.seq_truncate(1, 40)
    assert c.seq_block_table(1)[2] == shared and c.refcount(shared) == 2
    x = np.random.default_rng(9).standard_normal((1, W)).astype(np.float32)
    c.appendBatch(0, np.ones(1, np.uint32), np.array([40], np.uint32), x)  # layer 0, sequence 1
    fresh = c.seq_block_table(1)[2]
    assert fresh != shared
    assert c.refcount(shared) == 1 and c.refcount(fresh) == 1
    # the other owner is untouched, in every layer
    for layer in range(2):
        assert np.array_equal(c.gather(layer, 0), before0[layer])
    # the copy holds the shared rows of every layer (layer 1 untouched by the
    # write, all 41 rows), then the new row on layer 0
    g1 = c.gather(1, 1)
    assert np.array_equal(g1, before0[1][:41])
    g0 = c.gather(0, 1)
    assert np.array_equal(g0[:40], before0[0][:40])
    assert g0.shape[0] == 41
    if not quant:
        assert np.array_equal(g0[40], x[0])
    else:
        assert np.allclose(g0[40], x[0], atol=np.abs(x).max() / 127 * 0.51)
    # a second write into the now private block needs no further copy
    c.appendBatch(0, np.ones(1, np.uint32), np.array([41], np.uint32), x)
    assert c.seq_block_table(1)[2] == fresh


def test_device_append_path_copies_shared_block(kv):
    import torch

    c, rows0, rows1 = _shared_pair(kv, True, layers=1)
    before = c.gather(0, 0)
    shared = c.seq_block_table(0)[1]
    c.seq_truncate(1, 20)
    x = torch.randn((1, W), device="cuda")
    ids, pos = np.ones(1, np.uint32), np.array([20], np.uint32)
    c.appendBatch_dev(0, ids, pos, torch.from_numpy(ids).cuda(), torch.from_numpy(pos).cuda(), x)
    torch.cuda.synchronize()
    assert c.seq_block_table(1)[1] != shared
    assert np.array_equal(c.gather(0, 0), before)
    assert np.array_equal(c.gather(0, 1)[:20], before[:20])
