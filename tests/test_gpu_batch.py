"""Continuous batching over one shared pool (kvcu_batch_*, BatchScheduler of
src/batch_queue.zig:75-232): the reference's three scheduler tests
(src/batch_queue.zig:234-389), then a serving loop where requests join and
leave between decode steps, each step's decode checked against the oracle."""
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


def _cache(kv, nb=64):
    return kv.KVCache.with_blocks(1, R, P, nb, BS, quantized=True)


def test_lifecycle(kv):
    # src/batch_queue.zig:234-280
    c = _cache(kv)
    s = kv.BatchScheduler(c, 4)
    id1, id2 = s.addRequest(32), s.addRequest(32)
    assert (id1, id2) == (1, 2)
    ids, seqs = s.collectBatch(0)
    assert len(ids) == 2
    s.markRunning(ids)
    assert s.runningCount() == 2
    s.markCompleted(id1)
    s.reapCompleted()
    assert len(s) == 1


def test_priority_ordering(kv):
    # src/batch_queue.zig:282-332: low, critical, normal with room for two -> critical, normal
    c = _cache(kv)
    s = kv.BatchScheduler(c, 2)
    s.addRequest(32, kv.PRIORITY_LOW)
    id_critical = s.addRequest(32, kv.PRIORITY_CRITICAL)
    id_normal = s.addRequest(32, kv.PRIORITY_NORMAL)
    ids, _ = s.collectBatch(0)
    assert list(ids) == [id_critical, id_normal]


def test_kv_block_reclaim(kv):
    # src/batch_queue.zig:334-389 (blocks come back to the shared pool)
    c = _cache(kv)
    s = kv.BatchScheduler(c, 4)
    id1 = s.addRequest(32)
    id2 = s.addRequest(32)
    c.seq_ensure_capacity(s.seq(id1), 32)
    c.seq_ensure_capacity(s.seq(id2), 32)
    ids, _ = s.collectBatch(0)
    s.markRunning(ids)
    s.markCompleted(id1)
    before = c.numFreeBlocks()
    assert s.reclaimBlocks() > 0
    assert c.numFreeBlocks() > before
    assert c.seq_len(s.seq(id2)) == 0 and len(c.seq_block_table(s.seq(id2))) == 2  # untouched


def test_finished_by_eos_and_max_tokens(kv):
    c = _cache(kv)
    s = kv.BatchScheduler(c, 4)
    a, b = s.addRequest(3), s.addRequest(10)
    for t in (5, 6, 7):
        s.pushToken(a, t)
    s.pushToken(b, 9)
    s.pushToken(b, 2)  # eos 2
    assert s.isFinished(a, 2) and s.isFinished(b, 2)
    ids, _ = s.collectBatch(2)
    assert len(ids) == 0
    assert not s.isFinished(b, 0)


def test_serving_loop_decodes_match_oracle(kv, oracle):
    c = _cache(kv, nb=96)
    s = kv.BatchScheduler(c, 2)
    rng = np.random.default_rng(11)
    rows = {}  # request id -> [len][W] rows written so far
    prompt = {}
    prompt[s.addRequest(3)] = 50
    prompt[s.addRequest(4)] = 20
    free0 = c.numFreeBlocks()
    step, batches, seq_of = 0, [], {}
    while len(s):
        if step == 1:
            prompt[s.addRequest(2, kv.PRIORITY_HIGH)] = 30
        if step == 3:  # after requests 1 and 3 have been reaped
            prompt[s.addRequest(1)] = 10
            assert s.seq(4) in (seq_of[1], seq_of[3])  # a freed pool sequence is reused
        ids, seqs = s.collectBatch(0)
        for rid, sq in zip(ids, seqs):
            seq_of.setdefault(int(rid), int(sq))
        assert len(ids) > 0
        batches.append(list(ids))
        s.markRunning(ids)
        for rid, sq in zip(ids, seqs):
            rid = int(rid)
            if rid not in rows:  # prefill the prompt
                new = rng.standard_normal((prompt[rid], W)).astype(np.float32)
                start = 0
                rows[rid] = new
            else:  # one generated token
                new = rng.standard_normal((1, W)).astype(np.float32)
                start = rows[rid].shape[0]
                rows[rid] = np.concatenate([rows[rid], new])
            L = rows[rid].shape[0]
            c.seq_ensure_capacity(int(sq), L)
            c.appendBatch(0, np.full(new.shape[0], sq, np.uint32), np.arange(start, L, dtype=np.uint32), new)
        q = rng.standard_normal((len(ids), H, W)).astype(np.float32)
        got = c.mlaDecode(0, q, seqs.astype(np.uint32), SCALE)
        o = oracle.Pool(1, 96, BS, R, P, True)
        offs, tabs, lens = [0], [], []
        for rid, sq in zip(ids, seqs):
            tab = np.array(c.seq_block_table(int(sq)), np.uint32)
            L = rows[int(rid)].shape[0]
            t = np.arange(L)
            o.put_rows(0, tab[t // BS], t % BS, rows[int(rid)])
            tabs.extend(tab.tolist())
            offs.append(len(tabs))
            lens.append(L)
        want = o.attention_batch(0, np.array(offs, np.uint32), np.array(tabs, np.uint32),
                                 np.array(lens, np.uint32), q, SCALE)
        assert rel_err_rows(got, want) <= REL_TOL, step
        for rid in ids:
            s.pushToken(int(rid), step + 1)
            if s.isFinished(int(rid), 0):
                s.markCompleted(int(rid))
        s.reapCompleted()
        step += 1
        assert step < 20
    # the high-priority request joins at step 1 and leads every batch it is in
    assert batches[1][0] == 3
    assert all(b[0] == 3 for b in batches if 3 in b)
    # every block is back; sequence 0 plus three pool sequences served four requests
    assert c.numFreeBlocks() == free0
    assert c.num_seqs == 4
