"""Pins the CPU oracle (oracle/kvoracle.c) before it is trusted as the checker.

Each test restates a known-answer test from the reference's own test blocks
(file:line given) or compares against the independent fixtures in
tests/golden/ (see tests/golden/make_golden.py).
"""
import json
import math
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

R_TEST, P_TEST, L_TEST = 16, 8, 2  # src/kv_cache.zig:615-641 testHyperParams


# ------------------------------------------------------------------ f16 (src/dequant.zig:663-707)
def test_f16_to_f32_subnormal_precision(oracle):
    assert abs(oracle.f16_to_f32(0x0001) - 5.9604645e-8) < 1e-14
    assert abs(oracle.f16_to_f32(0x03FF) - 6.097555e-5) < 1e-8
    assert abs(oracle.f16_to_f32(0x0080) - 7.6293945e-6) < 1e-12


def test_f16_to_f32_comprehensive(oracle):
    assert oracle.f16_to_f32(0x0000) == 0.0
    assert math.copysign(1.0, oracle.f16_to_f32(0x8000)) == -1.0
    assert oracle.f16_to_f32(0x3C00) == 1.0
    assert oracle.f16_to_f32(0x4000) == 2.0
    assert oracle.f16_to_f32(0x3800) == 0.5
    assert oracle.f16_to_f32(0xBC00) == -1.0
    assert 0.0 < oracle.f16_to_f32(0x03FF) < 0.001
    assert math.isinf(oracle.f16_to_f32(0x7C00)) and math.isinf(oracle.f16_to_f32(0xFC00))
    assert math.isnan(oracle.f16_to_f32(0x7C01))


def test_f16_to_f32_exhaustive_matches_ieee(oracle):
    bits = np.arange(1 << 16, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(b)) for b in bits], np.float32)
    finite = np.isfinite(ref)
    assert np.array_equal(got[finite].view(np.uint32), ref[finite].view(np.uint32))
    assert np.all(np.isnan(got[np.isnan(ref)]))


def test_f32_to_f16_golden(oracle, golden):
    f32_in, f16_out = golden["f32_in"], golden["f16_out"]
    got = np.array([oracle.f32_to_f16(float(v)) for v in f32_in], np.uint16)
    assert np.array_equal(got, f16_out)


def test_f32_to_f16_reference_special_cases(oracle):
    # src/dequant.zig:58-66: f32 subnormals -> signed zero; NaN keeps its top mantissa bits
    assert oracle.f32_to_f16(1e-45) == 0
    assert oracle.f32_to_f16(-1e-45) == 0x8000
    qnan = np.array([0x7FC00000], np.uint32).view(np.float32)[0]
    assert oracle.f32_to_f16(float(qnan)) == 0x7E00
    assert oracle.f32_to_f16(float("inf")) == 0x7C00
    assert oracle.f32_to_f16(1e6) == 0x7C00  # exp16 >= 31 -> inf


# ------------------------------------------------------------------ Q8_0 (src/kv_cache.zig:294-349)
def test_q8_0_golden_rows(oracle, golden):
    rows, d16, qs = golden["q_rows"], golden["q_d16"], golden["q_qs"]
    for i in range(rows.shape[0]):
        blocks = oracle.quantize_q8_0(rows[i])
        assert np.array_equal(blocks["d"], d16[i]), i
        assert np.array_equal(blocks["qs"], qs[i]), i


def test_q8_0_partial_blocks_golden(oracle, golden):
    b = oracle.quantize_q8_0(golden["small_kv"])
    assert np.array_equal(b["d"], golden["small_kv_d"]) and np.array_equal(b["qs"], golden["small_kv_q"])
    b = oracle.quantize_q8_0(golden["small_pe"])
    assert np.array_equal(b["d"], golden["small_pe_d"]) and np.array_equal(b["qs"], golden["small_pe_q"])
    assert np.all(b["qs"][0, 8:] == 0)  # tail zero-fill, src/kv_cache.zig:346-348


def test_q8_0_ties_round_away_from_zero(oracle):
    x = np.zeros(32, np.float32)
    x[0] = 127.0  # d = 1.0 exactly
    x[1], x[2], x[3] = 2.5, -2.5, 0.5
    b = oracle.quantize_q8_0(x)
    assert oracle.f16_to_f32(int(b["d"][0])) == 1.0
    assert list(b["qs"][0, :4]) == [127, 3, -3, 1]


# ------------------------------------------------------------------ KVCache tests (src/kv_cache.zig:643-842)
def _cache(oracle):
    return oracle.KVCache(L_TEST, R_TEST, P_TEST, 64)


def test_kvcache_init_and_basic_operations(oracle):
    kv = _cache(oracle)
    assert kv.num_blocks == 4 and kv.numFreeBlocks() == 4 and kv.len == 0
    assert kv.ensureCapacity(20) == 0
    assert len(kv.block_table) == 2 and kv.numFreeBlocks() == 2


def test_kvcache_put_and_get(oracle):
    kv = _cache(oracle)
    assert kv.ensureCapacity(4) == 0
    kv_comp = np.arange(R_TEST, dtype=np.float32)
    k_pe = np.arange(P_TEST, dtype=np.float32) + 100
    assert kv.put(0, 0, kv_comp, k_pe) == 0
    assert kv.len == 1
    rc, got = kv.getKVCompressed(0, 0)
    assert rc == 0 and np.array_equal(got, kv_comp)
    rc, got = kv.getKPe(0, 0)
    assert rc == 0 and np.array_equal(got, k_pe)


def test_kvcache_quantization_roundtrip(oracle):
    kv = _cache(oracle)
    assert kv.enableQuantization() == 0 and kv.quantized
    assert kv.ensureCapacity(4) == 0
    kv_comp = 0.5 * np.arange(R_TEST, dtype=np.float32)
    k_pe = 0.25 * np.arange(P_TEST, dtype=np.float32)
    assert kv.put(0, 0, kv_comp, k_pe) == 0
    _, got_kv = kv.getKVCompressed(0, 0)
    _, got_pe = kv.getKPe(0, 0)
    assert np.all(np.abs(got_kv - kv_comp) < 0.05 * np.abs(kv_comp) + 1e-2)
    assert np.all(np.abs(got_pe - k_pe) < 0.05 * np.abs(k_pe) + 1e-2)


def test_kvcache_save_load_non_quantized(oracle, tmp_path):
    kv = _cache(oracle)
    kv.ensureCapacity(4)
    kv_comp = np.arange(R_TEST, dtype=np.float32)
    k_pe = np.arange(P_TEST, dtype=np.float32) + 100
    kv.put(0, 0, kv_comp, k_pe)
    kv.put(1, 1, kv_comp, k_pe)
    path = str(tmp_path / "test_kv_nonq.bin")
    assert kv.saveToFile(path) == 0
    kv2 = _cache(oracle)
    assert kv2.loadFromFile(path) == 0
    assert kv.len == kv2.len and kv.block_table == kv2.block_table
    assert np.array_equal(kv2.getKVCompressed(0, 0)[1], kv_comp)
    assert np.array_equal(kv2.getKPe(0, 0)[1], k_pe)
    # file layout: 40-byte header + table + f32 pools (kv then pe)
    data = open(path, "rb").read()
    assert data[:4] == b"KVCK" and int.from_bytes(data[4:8], "little") == 1
    assert data[13:16] == b"\0\0\0"
    assert len(data) == 40 + 4 * 1 + 2 * 4 * 16 * (R_TEST + P_TEST) * 4


def test_kvcache_save_load_quantized(oracle, tmp_path):
    kv = _cache(oracle)
    kv.enableQuantization()
    kv.ensureCapacity(4)
    kv_comp = 0.5 * np.arange(R_TEST, dtype=np.float32)
    k_pe = 0.25 * np.arange(P_TEST, dtype=np.float32)
    kv.put(0, 0, kv_comp, k_pe)
    kv.put(1, 1, kv_comp, k_pe)
    path = str(tmp_path / "test_kv_q.bin")
    assert kv.saveToFile(path) == 0
    kv2 = _cache(oracle)
    assert kv2.loadFromFile(path) == 0
    assert kv2.quantized and kv.len == kv2.len and kv.block_table == kv2.block_table
    # payload round trip (the reference test stops at metadata; we check the bytes too)
    path2 = str(tmp_path / "test_kv_q2.bin")
    assert kv2.saveToFile(path2) == 0
    assert open(path, "rb").read() == open(path2, "rb").read()
    assert np.array_equal(kv2.getKVCompressed(1, 1)[1], kv.getKVCompressed(1, 1)[1])


def test_kvcache_checkpoint_bad_magic(oracle, tmp_path):
    kv = _cache(oracle)
    path = tmp_path / "test_kv_bad.bin"
    hdr = bytearray(40)
    hdr[0:4] = b"BAD!"
    hdr[4:8] = (1).to_bytes(4, "little")
    for off, v in ((20, L_TEST), (24, 4), (28, 16), (32, R_TEST), (36, P_TEST)):
        hdr[off:off + 4] = v.to_bytes(4, "little")
    path.write_bytes(bytes(hdr))
    assert kv.loadFromFile(str(path)) == oracle.ERR_BAD_MAGIC


def test_kvcache_checkpoint_version_shape_eof(oracle, tmp_path):
    kv = _cache(oracle)
    kv.ensureCapacity(4)
    good = tmp_path / "good.bin"
    assert kv.saveToFile(str(good)) == 0
    data = bytearray(good.read_bytes())
    bad = tmp_path / "bad.bin"
    d = bytearray(data)
    d[4:8] = (2).to_bytes(4, "little")
    bad.write_bytes(bytes(d))
    assert kv.loadFromFile(str(bad)) == oracle.ERR_BAD_VERSION
    d = bytearray(data)
    d[32:36] = (32).to_bytes(4, "little")
    bad.write_bytes(bytes(d))
    assert kv.loadFromFile(str(bad)) == oracle.ERR_SHAPE_MISMATCH
    bad.write_bytes(bytes(data[:-7]))
    assert kv.loadFromFile(str(bad)) == oracle.ERR_EOF
    d = bytearray(data)
    d[40:44] = (99).to_bytes(4, "little")  # block id out of range
    bad.write_bytes(bytes(d))
    assert kv.loadFromFile(str(bad)) == oracle.ERR_BAD_BLOCK_ID


def test_kvcache_load_takes_blocks_off_free_list(oracle, tmp_path):
    kv = _cache(oracle)
    kv.ensureCapacity(35)  # blocks 0,1,2
    path = str(tmp_path / "c.bin")
    kv.saveToFile(path)
    kv2 = _cache(oracle)
    assert kv2.loadFromFile(path) == 0
    assert kv2.numFreeBlocks() == 1
    kv2.ensureCapacity(64)
    assert sorted(kv2.block_table) == [0, 1, 2, 3]


def test_kvcache_truncate_and_reset(oracle):
    kv = _cache(oracle)
    kv.ensureCapacity(35)
    assert len(kv.block_table) == 3
    kv.truncate(16)
    assert len(kv.block_table) == 1
    kv.reset()
    assert len(kv.block_table) == 0 and kv.len == 0 and kv.numFreeBlocks() == 4


def test_kvcache_errors(oracle):
    kv = _cache(oracle)
    kv.ensureCapacity(16)
    z = np.zeros(R_TEST, np.float32)
    zp = np.zeros(P_TEST, np.float32)
    assert kv.put(2, 0, z, zp) == oracle.ERR_LAYER_OOB
    assert kv.put(0, 16, z, zp) == oracle.ERR_POSITION_OOB
    assert kv.getKVCompressed(0, 0)[0] == oracle.ERR_POSITION_NOT_WRITTEN
    kv.put(0, 3, z, zp)
    assert kv.len == 4 and kv.getKVCompressed(0, 3)[0] == 0
    assert kv.getKVCompressed(5, 0)[0] == oracle.ERR_LAYER_OOB
    assert kv.ensureCapacity(16 * 5) == oracle.ERR_OUT_OF_BLOCKS


# ------------------------------------------------------------------ hashing (src/root.zig:298-315)
def test_block_hash_chain(oracle):
    g = json.load(open(os.path.join(ROOT, "tests", "golden", "hashes.json")))
    h1 = oracle.compute_hash(g["tokens_a"], oracle.NO_HASH)
    h2 = oracle.compute_hash(g["tokens_b"], h1)
    assert h2 == oracle.compute_hash(g["tokens_b"], h1)
    assert h2 != oracle.compute_hash(g["tokens_b"], 0)
    assert str(h1) == g["h1"] and str(h2) == g["h2"]
    assert str(oracle.compute_hash(g["tokens_b"], 0)) == g["h2_other"]
    prefix = oracle.NO_HASH
    toks = g["chain_tokens"]
    for bi, want in enumerate(g["chain"]):
        prefix = oracle.compute_hash(toks[bi * 16:(bi + 1) * 16], prefix)
        assert str(prefix) == want
    assert str(oracle.xxh64(b"")) == g["xxh64_empty"]
    assert str(oracle.xxh64(b"abc")) == g["xxh64_abc"]
    assert str(oracle.xxh64(bytes(range(100)))) == g["xxh64_100"]


def test_prefix_cache_find_and_reuse(oracle):
    kv = oracle.KVCache(1, R_TEST, P_TEST, 16 * 8)
    toks = list(range(100, 100 + 40))
    kv.ensureCapacity(len(toks))
    prefix = oracle.NO_HASH
    for bi in range(len(toks) // 16):
        kv.cacheBlock(bi, toks[bi * 16:(bi + 1) * 16], prefix)
        prefix = oracle.compute_hash(toks[bi * 16:(bi + 1) * 16], prefix)
    assert kv.findPrefixBlocks(toks) == 2
    assert kv.findPrefixBlocks(toks[:20]) == 1
    assert kv.findPrefixBlocks([1] + toks[1:]) == 0
    # re-sync onto its own cached blocks keeps them allocated (deviation 6)
    before = kv.numFreeBlocks()
    assert kv.reusePrefixBlocks(toks, 2) == 0
    assert kv.len == 32 and kv.numFreeBlocks() == before
    assert kv.refcount(kv.block_table[0]) == 1
    assert kv.reusePrefixBlocks([5] * 32, 1) == oracle.ERR_PREFIX_MISS


# ------------------------------------------------------------------ attention (src/inference.zig:572-660)
@pytest.mark.parametrize("name,quant", [("att_f32", False), ("att_q8", True), ("att_len1", True)])
def test_attention_matches_float64_golden(oracle, golden, name, quant):
    rows, q, want = golden[name + "_rows"], golden[name + "_q"], golden[name + "_out"]
    n = rows.shape[0]
    bs = 16
    nb = (n + bs - 1) // bs + 3
    pool = oracle.Pool(1, nb, bs, 512, 64, quant)
    rng = np.random.default_rng(7)
    table = rng.permutation(nb)[: (n + bs - 1) // bs].astype(np.uint32)
    for t in range(n):
        pool.put(0, int(table[t // bs]), t % bs, rows[t, :512], rows[t, 512:])
    out = pool.attention(0, table, n, q, float(golden["att_scale"][0]))
    err = np.abs(out - want).max(axis=1) / np.abs(want).max(axis=1)
    assert err.max() < 1e-5


def test_attention_empty_sequence_is_zero(oracle):
    pool = oracle.Pool(1, 2, 16, 512, 64, True)
    q = np.ones((3, 576), np.float32)
    out = pool.attention(0, np.array([0], np.uint32), 0, q, 0.07)
    assert np.all(out == 0)


def test_attention_threaded_matches_inline(oracle):
    rng = np.random.default_rng(3)
    B, H, bs, nb = 5, 4, 16, 64
    pool = oracle.Pool(1, nb, bs, 512, 64, True)
    lens = np.array([1, 17, 64, 100, 33], np.uint32)
    offs, tabs, nxt = [], [], 0
    for L in lens:
        k = (int(L) + bs - 1) // bs
        offs.append(len(tabs))
        tabs.extend(range(nxt, nxt + k))
        nxt += k
    offs.append(len(tabs))
    for b, L in enumerate(lens):
        for t in range(int(L)):
            r = rng.standard_normal(576).astype(np.float32)
            pool.put(0, tabs[offs[b] + t // bs], t % bs, r[:512], r[512:])
    q = rng.standard_normal((B, H, 576)).astype(np.float32)
    a = pool.attention_batch(0, offs, tabs, lens, q, 0.072, n_threads=1)
    b = pool.attention_batch(0, offs, tabs, lens, q, 0.072, n_threads=4)
    assert np.array_equal(a, b)


def test_absorbed_equals_expanded_mla(oracle):
    """score = (k_b^T q_nope).c + q_rope.k_pe; out = v_b (sum p c)/l (src/inference.zig:539-660)."""
    rng = np.random.default_rng(11)
    R, P, H, dn, dv, n = 512, 64, 4, 128, 128, 70
    k_b = (rng.standard_normal((H, dn, R)) / np.sqrt(R)).astype(np.float32)
    v_b = (rng.standard_normal((H, dv, R)) / np.sqrt(R)).astype(np.float32)
    c = rng.standard_normal((n, R)).astype(np.float32)
    pe = rng.standard_normal((n, P)).astype(np.float32)
    q_nope = rng.standard_normal((H, dn)).astype(np.float32)
    q_rope = rng.standard_normal((H, P)).astype(np.float32)
    scale = 1.0 / np.sqrt(192.0)
    # expanded (reference form), float64
    out_exp = np.zeros((H, dv))
    for h in range(H):
        k_nope = c.astype(np.float64) @ k_b[h].T.astype(np.float64)
        s = (k_nope @ q_nope[h] + pe @ q_rope[h]) * scale
        p = np.exp(s - s.max())
        v = c.astype(np.float64) @ v_b[h].T.astype(np.float64)
        out_exp[h] = p @ v / p.sum()
    # absorbed form through the oracle kernel
    pool = oracle.Pool(1, 8, 16, R, P, False)
    table = np.arange(8, dtype=np.uint32)
    for t in range(n):
        pool.put(0, t // 16, t % 16, c[t], pe[t])
    q_abs = np.concatenate([np.einsum("hdr,hd->hr", k_b, q_nope), q_rope], axis=1).astype(np.float32)
    lat = pool.attention(0, table, n, q_abs, scale)
    out_abs = np.einsum("hdr,hr->hd", v_b.astype(np.float64), lat.astype(np.float64))
    assert np.abs(out_abs - out_exp).max() / np.abs(out_exp).max() < 1e-4


# ------------------------------------------------------------------ generator
def test_generator_distribution(oracle):
    z = oracle.gen_rows(5, 1, np.arange(64), np.zeros(64), 576, 0.0)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01
    k = ((z - z.mean()) ** 4).mean() / z.var() ** 2
    assert abs(k - 3.0) < 0.1
    zo = oracle.gen_rows(5, 1, np.arange(64), np.zeros(64), 576, 0.01)
    frac = np.mean(zo != z)
    assert 0.006 < frac < 0.014
    assert np.allclose(zo[zo != z], 20 * z[zo != z])


def test_generator_is_counter_based(oracle):
    a = oracle.gen_rows(9, 3, [4, 5], [10, 11], 40)
    b = oracle.gen_rows(9, 3, [5], [11], 40, n_threads=1)
    assert np.array_equal(a[1], b[0])
    assert oracle.gen_normal(9, 3, 5, 11 * 1024 + 7) == a[1, 7]
