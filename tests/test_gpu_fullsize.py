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


# ------------------------------------------------------------------ config 4
C4_SEQS, C4_LAYERS, C4_LO, C4_HI, C4_SEED = 64, 4, 8192, 32768, 4


def config4_lengths():
    # 64 sequences, context lengths uniform in [8192, 32768]
    return np.random.default_rng(C4_SEED).integers(C4_LO, C4_HI + 1, C4_SEQS).astype(np.int64)


def test_config4_full_shape_step_against_oracle(oracle):
    """Config 4 at its stated shape: 64 sequences of 8k-32k tokens, 4 layers,
    Q8_0, block size 64, 20 heads.  One step appends one token per sequence per
    layer, then decodes each layer; a sample (shortest, median, longest) of
    every layer is checked against the oracle, <= 1e-3."""
    import torch

    import kvcu

    kvcu.init(0)
    lens = config4_lengths()
    nb = int(sum((int(L) + 1 + BS - 1) // BS for L in lens)) + 8
    cache = kvcu.KVCache.with_blocks(C4_LAYERS, 512, 64, nb, BS, quantized=True)
    for _ in range(C4_SEQS - 1):
        cache.seq_create()
    ids = np.arange(C4_SEQS, dtype=np.uint32)
    for i in range(C4_SEQS):
        cache.seq_ensure_capacity(i, int(lens[i]) + 1)
    gen = torch.Generator(device="cuda").manual_seed(C4_SEED)
    outs = []
    for layer in range(C4_LAYERS):
        cache.prefill_synthetic(layer, ids, lens, C4_SEED, OUTLIER_P)
    for layer in range(C4_LAYERS):  # the step: append one token, then decode
        cache.prefill_synthetic(layer, ids, lens + 1, C4_SEED, OUTLIER_P, start=lens)
        q = torch.randn((C4_SEQS, H, W), device="cuda", generator=gen)
        out = torch.empty((C4_SEQS, H, 512), device="cuda")
        cache.mlaDecode_dev(layer, ids, q, SCALE, out)
        outs.append((q, out))
    torch.cuda.synchronize()
    assert cache.pool().status() == 0
    assert all(cache.seq_len(i) == int(lens[i]) + 1 for i in range(C4_SEQS))
    order = np.argsort(lens)
    sample = [int(order[0]), int(order[C4_SEQS // 2]), int(order[-1])]
    L = [int(lens[s]) + 1 for s in sample]
    for layer in range(C4_LAYERS):
        nbo = sum((x + BS - 1) // BS for x in L) + 1
        pool = oracle.Pool(1, nbo, BS, 512, 64, True)
        offs, tabs, k = [0], [], 0
        for i, s in enumerate(sample):
            need = (L[i] + BS - 1) // BS
            tabs.extend(range(k, k + need))
            k += need
            offs.append(len(tabs))
            rows = oracle.gen_rows(C4_SEED, layer, np.full(L[i], s, np.uint32), np.arange(L[i], dtype=np.uint32),
                                   W, OUTLIER_P)
            t = np.arange(L[i])
            pool.put_rows(0, np.array(tabs[offs[i]:offs[i + 1]], np.uint32)[t // BS], t % BS, rows)
        q, out = outs[layer]
        want = pool.attention_batch(0, np.array(offs, np.uint32), np.array(tabs, np.uint32), np.array(L, np.uint32),
                                    q[sample].cpu().numpy(), SCALE, n_threads=16)
        assert rel_err_rows(out[sample].cpu().numpy(), want) <= REL_TOL, layer
    cache.deinit()
