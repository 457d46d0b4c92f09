"""Generate the golden fixtures in tests/golden/ (run from the repo root).

The reference (Zig) cannot be built or run in this container, so these vectors
come from INDEPENDENT restatements of the reference's arithmetic that share no
code with oracle/kvoracle.c:

* f32 -> f16 bits: numpy's IEEE round-to-nearest-even cast.  It equals the
  reference's f32ToF16 (src/dequant.zig:50-95) on every normal, overflow and
  zero input; on the f16-subnormal range it is the documented correct-RNE
  replacement for the reference's mis-shifted branch (src/dequant.zig:76-77).
* Q8_0 blocks: numpy float32 arithmetic following src/kv_cache.zig:294-349
  (amax, d = amax/127 in f32, f16(d), q = round-half-away(x/d) clamped to
  +-127, tail zero-fill).
* Attention: float64 numpy softmax(q K^T * scale) V over the dequantized rows,
  the absorbed form of src/inference.zig:572-660.
* Prefix hashes: the python-xxhash package (XXH64, seed 0) over the byte
  stream of src/kv_cache.zig:596-609.

The oracle is pinned against these files by tests/test_oracle.py.
"""
from __future__ import annotations

import json
import os

import numpy as np
import xxhash

HERE = os.path.dirname(os.path.abspath(__file__))
NO_HASH = (1 << 64) - 1


def f16_bits(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def round_half_away(v: np.ndarray) -> np.ndarray:
    v64 = v.astype(np.float64)  # exact widening; the +0.5 below is then exact
    return (np.sign(v64) * np.floor(np.abs(v64) + 0.5)).astype(np.float64)


def q8_0_numpy(row: np.ndarray):
    """Quantize a 1-D float32 array into (d16 bits [nb], qs [nb, 32])."""
    n = row.size
    nb = (n + 31) // 32
    d16 = np.zeros(nb, np.uint16)
    qs = np.zeros((nb, 32), np.int8)
    for b in range(nb):
        x = row[b * 32: min(n, b * 32 + 32)].astype(np.float32)
        amax = np.float32(np.max(np.abs(x))) if x.size else np.float32(0)
        d = np.float32(amax / np.float32(127.0)) if amax > 0 else np.float32(0)
        d16[b] = f16_bits(np.array([d]))[0]
        if d > 0:
            quot = (x / d).astype(np.float32)
            q = np.clip(round_half_away(quot), -127, 127).astype(np.int8)
            qs[b, : x.size] = q
    return d16, qs


def f16_to_f32_numpy(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)


def dequant_numpy(d16, qs, n):
    vals = (f16_to_f32_numpy(d16)[:, None] * qs.astype(np.float32)).astype(np.float32)
    return vals.reshape(-1)[:n]


def compute_hash(tokens, prefix):
    data = b""
    if prefix != NO_HASH:
        data += int(prefix).to_bytes(8, "little")
    data += np.asarray(tokens, "<u4").tobytes()
    return xxhash.xxh64_intdigest(data, seed=0)


def main():
    rng = np.random.default_rng(20261201)

    # ---- f32 -> f16 -------------------------------------------------------
    mags = 10.0 ** rng.uniform(-9, 5.5, 4000)
    vals = (rng.standard_normal(4000) * mags).astype(np.float32)
    edge = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65519.99, 65520.0, 1e6, -1e6,
                     6.103515625e-05, 6.0975552e-05, 5.9604645e-08, 2.9802322e-08,
                     2.9802326e-08, 8.940697e-08, 1e-45, 3.4e38, np.inf, -np.inf,
                     1.00048828125, 1.0009765625, 1.00146484375, 0.0590551, 7.75e-3,
                     3.1e-5], np.float32)
    f32_in = np.concatenate([edge, vals]).astype(np.float32)
    f16_out = f16_bits(f32_in)

    # ---- Q8_0 rows ----------------------------------------------------------
    rows = []
    rows.append(np.zeros(576, np.float32))  # all-zero row -> d=0, qs=0
    rows.append((0.5 * np.arange(576)).astype(np.float32))
    tie = np.zeros(576, np.float32)
    tie[:32] = np.array([127.0] + [k + 0.5 for k in range(-15, 16)], np.float32)  # d = 1, ties
    rows.append(tie)
    tiny = (rng.standard_normal(576) * 1e-3).astype(np.float32)  # f16-subnormal scales
    rows.append(tiny)
    for _ in range(40):
        r = rng.standard_normal(576).astype(np.float32)
        mask = rng.random(576) < 0.01
        r[mask] *= np.float32(20.0)
        rows.append(r)
    q_rows = np.stack(rows).astype(np.float32)
    q_d16 = np.zeros((q_rows.shape[0], 18), np.uint16)
    q_qs = np.zeros((q_rows.shape[0], 18, 32), np.int8)
    for i, r in enumerate(q_rows):
        q_d16[i], q_qs[i] = q8_0_numpy(r)
    # partial blocks (reference test dims: kv_rank 16, rope 8; src/kv_cache.zig:615-641)
    small_kv = (0.5 * np.arange(16)).astype(np.float32)
    small_pe = (0.25 * np.arange(8)).astype(np.float32)
    s_kv_d, s_kv_q = q8_0_numpy(small_kv)
    s_pe_d, s_pe_q = q8_0_numpy(small_pe)

    # ---- attention (float64 numpy, absorbed MLA) ------------------------------
    R, P, H = 512, 64, 20
    scale = np.float32(1.0 / np.sqrt(192.0))
    att = {}
    for name, n_tok, quant in (("att_f32", 150, False), ("att_q8", 133, True), ("att_len1", 1, True)):
        kvrows = rng.standard_normal((n_tok, R + P)).astype(np.float32)
        if quant:
            deq = np.zeros_like(kvrows)
            for t in range(n_tok):
                d_kv, q_kv = q8_0_numpy(kvrows[t, :R])
                d_pe, q_pe = q8_0_numpy(kvrows[t, R:])
                deq[t, :R] = dequant_numpy(d_kv, q_kv, R)
                deq[t, R:] = dequant_numpy(d_pe, q_pe, P)
        else:
            deq = kvrows
        q = rng.standard_normal((H, R + P)).astype(np.float32)
        K = deq.astype(np.float64)
        s = (q.astype(np.float64) @ K.T) * float(scale)
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        out = (p @ K[:, :R]) / p.sum(axis=1, keepdims=True)
        att[name + "_rows"] = kvrows
        att[name + "_q"] = q
        att[name + "_out"] = out.astype(np.float64)

    np.savez_compressed(
        os.path.join(HERE, "golden.npz"),
        f32_in=f32_in, f16_out=f16_out,
        q_rows=q_rows, q_d16=q_d16, q_qs=q_qs,
        small_kv=small_kv, small_pe=small_pe,
        small_kv_d=s_kv_d, small_kv_q=s_kv_q, small_pe_d=s_pe_d, small_pe_q=s_pe_q,
        att_scale=np.array([scale], np.float32),
        **att,
    )

    # ---- prefix-hash chain -----------------------------------------------------
    tokens_a = list(range(1, 17))
    tokens_b = list(range(17, 33))
    h1 = compute_hash(tokens_a, NO_HASH)
    h2 = compute_hash(tokens_b, h1)
    h2_other = compute_hash(tokens_b, 0)
    chain = []
    prefix = NO_HASH
    toks = rng.integers(0, 150000, 16 * 6).tolist()
    for bi in range(6):
        prefix = compute_hash(toks[bi * 16:(bi + 1) * 16], prefix)
        chain.append(str(prefix))
    hashes = {
        "tokens_a": tokens_a, "tokens_b": tokens_b,
        "h1": str(h1), "h2": str(h2), "h2_other": str(h2_other),
        "chain_tokens": toks, "chain": chain,
        "xxh64_empty": str(xxhash.xxh64_intdigest(b"")),
        "xxh64_abc": str(xxhash.xxh64_intdigest(b"abc")),
        "xxh64_100": str(xxhash.xxh64_intdigest(bytes(range(100)))),
    }
    with open(os.path.join(HERE, "hashes.json"), "w") as f:
        json.dump(hashes, f, indent=1)
    print("wrote", os.path.join(HERE, "golden.npz"), "and hashes.json")


if __name__ == "__main__":
    main()
