"""Shared helpers for the parity tests: seeded synthetic workloads in the shapes
of BASELINE.json's configs, block tables, and the comparison rule."""
from __future__ import annotations

import numpy as np

R, P, W = 512, 64, 576
SCALE = float(np.float32(1.0 / np.sqrt(192.0)))  # 1/sqrt(head_dim), head_dim = 64 + 128
REL_TOL = 1e-3  # north_star: attention within max relative error 1e-3


def seeded_tables(lens, block_size, num_blocks, seed):
    """Allocate ceil(len/BS) blocks per sequence in a seeded shuffled order."""
    rng = np.random.default_rng(seed)
    need = [(int(L) + block_size - 1) // block_size for L in lens]
    assert sum(need) <= num_blocks
    order = rng.permutation(num_blocks).astype(np.uint32)
    offs, flat, k = [0], [], 0
    for n in need:
        flat.extend(order[k:k + n].tolist())
        k += n
        offs.append(len(flat))
    return np.array(offs, np.uint32), np.array(flat if flat else [0], np.uint32)


def gen_seq_rows(oracle, seed, layer, seq, length, outlier_p):
    """Rows of one sequence: the same counter-based stream the device uses."""
    if length == 0:
        return np.zeros((0, W), np.float32)
    b = np.full(length, seq, np.uint32)
    c = np.arange(length, dtype=np.uint32)
    return oracle.gen_rows(seed, layer, b, c, W, outlier_p)


# The largest error any attention comparison of this test session returned
# (reported at the end of the run by conftest.py).
WORST = {"err": 0.0, "where": None}


def rel_err_rows(got, want):
    """max over rows of max|got-want| / max|want| (rows = last axis)."""
    got = np.asarray(got, np.float64).reshape(-1, got.shape[-1])
    want = np.asarray(want, np.float64).reshape(-1, want.shape[-1])
    den = np.abs(want).max(axis=1)
    num = np.abs(got - want).max(axis=1)
    err = np.where(den > 0, num / np.where(den > 0, den, 1), num)
    e = float(err.max()) if err.size else 0.0
    if e > WORST["err"]:
        import os

        WORST["err"], WORST["where"] = e, os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0]
    return e


def oracle_pool_for(oracle, layer_rows, lens, block_size, quantized, n_layers=1):
    """Oracle pool with contiguous tables holding the given sequences' rows.

    layer_rows[l][s] = rows of sequence s at layer l.  Returns (pool, offs, tables)."""
    need = [(int(L) + block_size - 1) // block_size for L in lens]
    nb = max(1, sum(need))
    pool = oracle.Pool(n_layers, nb, block_size, R, P, quantized)
    offs, flat, k = [0], [], 0
    for n in need:
        flat.extend(range(k, k + n))
        k += n
        offs.append(len(flat))
    offs = np.array(offs, np.uint32)
    tables = np.array(flat if flat else [0], np.uint32)
    for l in range(n_layers):
        for s, L in enumerate(lens):
            L = int(L)
            if L == 0:
                continue
            t = np.arange(L)
            pool.put_rows(l, tables[offs[s] + t // block_size], t % block_size, layer_rows[l][s][:L])
    return pool, offs, tables
