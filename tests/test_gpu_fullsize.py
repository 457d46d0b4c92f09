"""Config 5 at its full size (512 sequences, log-uniform lengths in [128, 65536],
5.2 M context tokens, Q8_0, block size 64, 20 heads), one layer, checked by
properties that do not depend on the size:

- decode of a sample of sequences (the shortest, median ones and the longest,
  which the plan splits across many work items) against the oracle, <= 1e-3;
- permutation invariance: decoding the batch in another order permutes the
  outputs (<= 1e-3: the plan cuts the batch into per-CTA ranges in batch
  order, so a sequence may be split at other points);
- a sequence decoded alone matches its row of the full batch (<= 1e-3: the
  split points differ, so partial sums are combined in another order).
"""
import math

import numpy as np
import pytest

from kvdata import REL_TOL, SCALE, W, rel_err_rows

pytestmark = pytest.mark.gpu

N_SEQS, BS, H, SEED, OUTLIER_P = 512, 64, 20, 5, 0.01


def config5_lengths(n=N_SEQS, seed=SEED):
    # the benchmark's distribution: log-uniform in [128, 65536]
    rng = np.random.default_rng(seed)
    u = rng.uniform(math.log(128), math.log(65536), n)
    return np.minimum(np.floor(np.exp(u)).astype(np.int64), 65536)


@pytest.fixture(scope="module")
def full(oracle):
    import torch

    import kvcu

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    kvcu.init(0)
    lens = config5_lengths()
    nb = int(sum((int(L) + BS - 1) // BS for L in lens)) + 8
    cache = kvcu.KVCache.with_blocks(1, 512, 64, nb, BS, quantized=True)
    for _ in range(N_SEQS - 1):
        cache.seq_create()
    ids = np.arange(N_SEQS, dtype=np.uint32)
    for i in range(N_SEQS):
        cache.seq_ensure_capacity(i, int(lens[i]))
    cache.prefill_synthetic(0, ids, lens, SEED, OUTLIER_P)
    gen = torch.Generator(device="cuda").manual_seed(SEED)
    q = torch.randn((N_SEQS, H, W), device="cuda", generator=gen)
    out = torch.empty((N_SEQS, H, 512), device="cuda")
    cache.mlaDecode_dev(0, ids, q, SCALE, out)
    torch.cuda.synchronize()
    assert cache.pool().status() == 0
    yield kvcu, cache, lens, q, out
    cache.deinit()


def test_fullsize_sample_against_oracle(full, oracle):
    kvcu, cache, lens, q, out = full
    order = np.argsort(lens)
    sample = [int(s) for s in list(order[:4]) + list(order[254:256]) + [order[-1]]]
    L = [int(lens[s]) for s in sample]
    nb = sum((x + BS - 1) // BS for x in L) + 1
    pool = oracle.Pool(1, nb, BS, 512, 64, True)
    offs, tabs, k = [0], [], 0
    for i, s in enumerate(sample):
        need = (L[i] + BS - 1) // BS
        tabs.extend(range(k, k + need))
        k += need
        offs.append(len(tabs))
        rows = oracle.gen_rows(SEED, 0, np.full(L[i], s, np.uint32), np.arange(L[i], dtype=np.uint32), W,
                               OUTLIER_P)
        t = np.arange(L[i])
        pool.put_rows(0, np.array(tabs[offs[i]:offs[i + 1]], np.uint32)[t // BS], t % BS, rows)
    qs = q[sample].cpu().numpy()
    want = pool.attention_batch(0, np.array(offs, np.uint32), np.array(tabs, np.uint32),
                                np.array(L, np.uint32), qs, SCALE, n_threads=16)
    got = out[sample].cpu().numpy()
    assert rel_err_rows(got, want) <= REL_TOL


def test_fullsize_permutation_invariance(full):
    import torch

    kvcu, cache, lens, q, out = full
    perm = np.random.default_rng(11).permutation(N_SEQS).astype(np.uint32)
    out_p = torch.empty_like(out)
    cache.mlaDecode_dev(0, perm, q[torch.from_numpy(perm.astype(np.int64)).cuda()], SCALE, out_p)
    torch.cuda.synchronize()
    assert cache.pool().status() == 0
    want = out[torch.from_numpy(perm.astype(np.int64)).cuda()]
    assert rel_err_rows(out_p.cpu().numpy(), want.cpu().numpy()) <= REL_TOL


def test_fullsize_single_sequence_matches_batch_row(full):
    import torch

    kvcu, cache, lens, q, out = full
    s = int(np.argmax(lens))  # the longest: many work items in the batch plan, fewer alone
    one = torch.empty((1, H, 512), device="cuda")
    cache.mlaDecode_dev(0, np.array([s], np.uint32), q[s:s + 1].contiguous(), SCALE, one)
    torch.cuda.synchronize()
    assert cache.pool().status() == 0
    assert rel_err_rows(one.cpu().numpy(), out[s:s + 1].cpu().numpy()) <= REL_TOL
