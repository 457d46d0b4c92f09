"""Causal multi-query (prefill) attention over the paged cache:
InferenceEngine.mlaAttentionBatch (src/inference.zig:670-883), whose loop
(:771-877) lets each new prompt position start_pos + i attend every cached
position <= itself.  The GPU runs all positions of a prompt in one call per
layer (kvcache_mla_attention_batch: one causal plan, one decode launch); each
checked position must match the oracle's attention over its own prefix,
max relative error per (position, head) row <= 1e-3."""
import numpy as np
import pytest

from kvdata import REL_TOL, SCALE, W, gen_seq_rows, oracle_pool_for, rel_err_rows

pytestmark = pytest.mark.gpu

SEED, OUTLIER_P = 31, 0.01


@pytest.fixture(scope="module")
def kv():
    import torch

    import kvcu

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    kvcu.init(0)
    return kvcu


def _oracle_per_position(oracle, rows, bs, quant, start_pos, idx, q):
    """Each sampled query idx[j] attends positions [0, start_pos + idx[j]]."""
    total = rows.shape[0]
    pool, offs, tabs = oracle_pool_for(oracle, [[rows]], [total], bs, quant)
    t = tabs[offs[0]:offs[1]]
    m = len(idx)
    offs_e = np.arange(m + 1, dtype=np.uint32) * t.size
    tabs_e = np.tile(t, m).astype(np.uint32)
    lens_e = (start_pos + np.asarray(idx) + 1).astype(np.uint32)
    return pool.attention_batch(0, offs_e, tabs_e, lens_e, q, SCALE, n_threads=16)


@pytest.mark.parametrize("quant,bs,H,start_pos,n_pos", [(True, 64, 20, 0, 2048), (True, 16, 20, 1000, 1500),
                                                        (False, 16, 8, 37, 300)])
def test_prefill_positions_against_oracle(kv, oracle, quant, bs, H, start_pos, n_pos):
    total = start_pos + n_pos
    nb = (total + bs - 1) // bs + 2
    c = kv.KVCache.with_blocks(1, 512, 64, nb, block_size=bs, quantized=quant)
    c.seq_ensure_capacity(0, total)
    c.prefill_synthetic(0, [0], [total], SEED, OUTLIER_P)  # the earlier turns and the new prompt rows
    rng = np.random.default_rng(SEED + n_pos)
    q = rng.standard_normal((n_pos, H, W)).astype(np.float32)
    out = c.mlaAttentionBatch(0, 0, start_pos, q, SCALE)
    rows = gen_seq_rows(oracle, SEED, 0, 0, total, OUTLIER_P)
    idx = sorted(set(list(range(0, min(n_pos, 12))) + list(range(n_pos - 6, n_pos)) +
                     rng.choice(n_pos, min(n_pos, 40), replace=False).tolist()))
    want = _oracle_per_position(oracle, rows, bs, quant, start_pos, idx, q[idx])
    assert rel_err_rows(out[idx], want) <= REL_TOL
    c.deinit()


def test_prefill_device_api_mixed_sequences_and_clipped_lengths(kv, oracle):
    """kvcu_decode_plan_causal directly: entries of two sequences, lengths 0,
    within range, and beyond the sequence (clipped to its length)."""
    import torch

    lens = [700, 2100]
    bs, H = 64, 20
    nb = sum((L + bs - 1) // bs for L in lens) + 2
    c = kv.KVCache.with_blocks(1, 512, 64, nb, block_size=bs, quantized=True)
    c.seq_create()
    for s, L in enumerate(lens):
        c.seq_ensure_capacity(s, L)
    c.prefill_synthetic(0, [0, 1], lens, SEED, OUTLIER_P)
    pool = c.pool()
    seq = np.array([0, 1, 1, 0, 1, 0], np.uint32)
    elen = np.array([1, 2100, 129, 0, 5000, 700], np.uint32)
    n = seq.size
    offs = np.zeros(3, np.uint32)
    tables = []
    for s in range(2):
        tables.extend(c.seq_block_table(s))
        offs[s + 1] = len(tables)
    dev = torch.device("cuda", 0)
    d_seq = torch.from_numpy(seq.astype(np.int32)).to(dev)
    d_el = torch.from_numpy(elen.astype(np.int32)).to(dev)
    d_lens = torch.tensor(lens, dtype=torch.int32, device=dev)
    d_toff = torch.from_numpy(offs.astype(np.int32)).to(dev)
    d_tab = torch.tensor(tables, dtype=torch.int32, device=dev)
    q = torch.randn((n, H, W), device=dev, generator=torch.Generator(device=dev).manual_seed(SEED))
    out = torch.full((n, H, 512), float("nan"), device=dev)
    ws = kv.DecodeWorkspace(0, n, H)
    rc = kv.lib().kvcu_decode_plan_causal(ws._h, pool.handle, n, d_seq.data_ptr(), 2, d_lens.data_ptr(),
                                          d_el.data_ptr(), None)
    assert rc == 0, kv.last_error()
    ws.decode(pool, 0, q, d_toff, d_tab, d_lens, SCALE, out, seq_ids=d_seq)
    torch.cuda.synchronize()
    assert pool.status() == 0
    got = out.cpu().numpy()
    qs = q.cpu().numpy()
    for s in range(2):
        rows = gen_seq_rows(oracle, SEED, 0, s, lens[s], OUTLIER_P)
        pick = [b for b in range(n) if seq[b] == s]
        eff = {b: min(int(elen[b]), lens[s]) for b in pick}
        live = [b for b in pick if eff[b] > 0]
        want = _oracle_per_position(oracle, rows, bs, True, 0, [eff[b] - 1 for b in live], qs[live])
        assert rel_err_rows(got[live], want) <= REL_TOL
        for b in pick:
            if eff[b] == 0:
                assert not np.any(got[b])  # an empty context attends nothing: zeros
    ws.close()
    c.deinit()


def test_prefill_rejects_positions_not_written(kv):
    c = kv.KVCache.with_blocks(1, 512, 64, 8, block_size=16, quantized=True)
    c.seq_ensure_capacity(0, 100)
    c.prefill_synthetic(0, [0], [50], SEED, 0.0)
    q = np.zeros((10, 4, W), np.float32)
    with pytest.raises(kv.KVCudaError) as e:
        c.mlaAttentionBatch(0, 0, 45, q, SCALE)  # positions 45..54, only 50 written
    assert e.value.name == "PositionNotWritten"
    c.deinit()
