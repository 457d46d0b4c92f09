"""GPU parity tests: the CUDA path (through the C-ABI) against the CPU oracle.

Bit-exact: generator rows, appended Q8_0 payload + f16 scales (compared in the
reference's checkpoint byte order), gathered / dequantized rows, checkpoint
files.  Attention: max over (sequence, head) rows of
max|gpu - oracle| / max|oracle| <= 1e-3 (REL_TOL, the north_star bound).
"""
import numpy as np
import pytest

from kvdata import P, R, REL_TOL, SCALE, W, gen_seq_rows, oracle_pool_for, rel_err_rows, seeded_tables

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kv():
    import torch

    import kvcu

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    kvcu.init(0)
    return kvcu


@pytest.fixture(scope="module")
def torch_mod():
    import torch

    return torch


# ------------------------------------------------------------------ generator
def test_generator_bit_exact(kv, oracle, torch_mod):
    torch = torch_mod
    b = np.array([0, 3, 7, 511, 65535], np.uint32)
    c = np.array([0, 1, 4095, 32767, 65535], np.uint32)
    for p in (0.0, 0.01):
        want = oracle.gen_rows(77, 5, b, c, W, p)
        out = torch.empty((b.size, W), dtype=torch.float32, device="cuda")
        kv.synth_rows(77, 5, torch.from_numpy(b).cuda(), torch.from_numpy(c).cuda(), W, out, p)
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ------------------------------------------------------------------ reference KVCache tests on the GPU
R_T, P_T, L_T = 16, 8, 2  # src/kv_cache.zig:615-641


def test_kvcache_init_and_basic_operations(kv):
    c = kv.KVCache(L_T, R_T, P_T, 64)
    assert c.num_blocks == 4 and c.numFreeBlocks() == 4 and c.len == 0
    c.ensureCapacity(20)
    assert len(c.block_table) == 2 and c.numFreeBlocks() == 2


def test_kvcache_put_and_get(kv):
    c = kv.KVCache(L_T, R_T, P_T, 64)
    c.ensureCapacity(4)
    kvc = np.arange(R_T, dtype=np.float32)
    kpe = np.arange(P_T, dtype=np.float32) + 100
    c.put(0, 0, kvc, kpe)
    assert c.len == 1
    assert np.array_equal(c.getKVCompressed(0, 0), kvc)
    assert np.array_equal(c.getKPe(0, 0), kpe)


def test_kvcache_quantization_roundtrip_bit_exact(kv, oracle):
    c = kv.KVCache(L_T, R_T, P_T, 64)
    c.enableQuantization()
    assert c.quantized
    c.ensureCapacity(4)
    o = oracle.KVCache(L_T, R_T, P_T, 64)
    o.enableQuantization()
    o.ensureCapacity(4)
    kvc = 0.5 * np.arange(R_T, dtype=np.float32)
    kpe = 0.25 * np.arange(P_T, dtype=np.float32)
    c.put(0, 0, kvc, kpe)
    o.put(0, 0, kvc, kpe)
    got_kv, got_pe = c.getKVCompressed(0, 0), c.getKPe(0, 0)
    assert np.all(np.abs(got_kv - kvc) < 0.05 * np.abs(kvc) + 1e-2)
    assert np.all(np.abs(got_pe - kpe) < 0.05 * np.abs(kpe) + 1e-2)
    assert np.array_equal(got_kv, o.getKVCompressed(0, 0)[1])
    assert np.array_equal(got_pe, o.getKPe(0, 0)[1])


@pytest.mark.parametrize("quant", [False, True])
def test_kvcache_save_load_file_bytes_match_oracle(kv, oracle, tmp_path, quant):
    c = kv.KVCache(L_T, R_T, P_T, 64)
    o = oracle.KVCache(L_T, R_T, P_T, 64)
    if quant:
        c.enableQuantization()
        o.enableQuantization()
    for x in (c, o):
        x.ensureCapacity(4)
    kvc = np.arange(R_T, dtype=np.float32) * (0.5 if quant else 1.0)
    kpe = np.arange(P_T, dtype=np.float32) * (0.25 if quant else 1.0) + (0 if quant else 100)
    for x in (c, o):
        x.put(0, 0, kvc, kpe)
        x.put(1, 1, kvc, kpe)
    pg, po = tmp_path / "gpu.bin", tmp_path / "oracle.bin"
    c.saveToFile(pg)
    assert o.saveToFile(str(po)) == 0
    assert pg.read_bytes() == po.read_bytes()
    c2 = kv.KVCache(L_T, R_T, P_T, 64)
    c2.loadFromFile(pg)
    assert c2.quantized == quant and c2.len == c.len and c2.block_table == c.block_table
    assert np.array_equal(c2.getKVCompressed(1, 1), c.getKVCompressed(1, 1))
    assert np.array_equal(c2.getKPe(0, 0), c.getKPe(0, 0))
    # the oracle loads the GPU's file and vice versa
    o2 = oracle.KVCache(L_T, R_T, P_T, 64)
    assert o2.loadFromFile(str(pg)) == 0
    assert np.array_equal(o2.getKVCompressed(1, 1)[1], c.getKVCompressed(1, 1))


def test_kvcache_checkpoint_errors(kv, tmp_path):
    c = kv.KVCache(L_T, R_T, P_T, 64)
    c.ensureCapacity(4)
    good = tmp_path / "good.bin"
    c.saveToFile(good)
    data = bytearray(good.read_bytes())
    bad = tmp_path / "bad.bin"
    cases = [((0, b"BAD!"), "InvalidCheckpointMagic"), ((4, (2).to_bytes(4, "little")), "UnsupportedCheckpointVersion"),
             ((32, (32).to_bytes(4, "little")), "CheckpointShapeMismatch"),
             ((40, (99).to_bytes(4, "little")), "BadBlockId")]
    for (off, val), name in cases:
        d = bytearray(data)
        d[off:off + len(val)] = val
        bad.write_bytes(bytes(d))
        with pytest.raises(kv.KVCudaError) as e:
            c.loadFromFile(bad)
        assert e.value.name == name
    bad.write_bytes(bytes(data[:-5]))
    with pytest.raises(kv.KVCudaError) as e:
        c.loadFromFile(bad)
    assert e.value.name == "EndOfStream"


def test_v1_load_refuses_a_cache_with_other_live_sequences(kv, tmp_path):
    # A v1 file restores a single-sequence cache; loading it into a pool whose
    # other sequences hold blocks would overwrite their rows.
    c = kv.KVCache.with_blocks(L_T, R_T, P_T, 8, block_size=16)
    c.ensureCapacity(20)
    path = tmp_path / "v1.bin"
    c.saveToFile(path)
    s1 = c.seq_create()
    c.seq_ensure_capacity(s1, 5)
    free_before = c.numFreeBlocks()
    with pytest.raises(kv.KVCudaError) as e:
        c.loadFromFile(path)
    assert e.value.name == "InvalidArgument"
    assert c.numFreeBlocks() == free_before and len(c.block_table) == 2
    # an empty extra sequence is no obstacle
    c.seq_reset(s1)
    c.loadFromFile(path)
    assert len(c.block_table) == 2


def test_kvcache_truncate_reset_and_errors(kv):
    c = kv.KVCache(L_T, R_T, P_T, 64)
    c.ensureCapacity(35)
    assert len(c.block_table) == 3
    c.truncate(16)
    assert len(c.block_table) == 1
    c.reset()
    assert len(c.block_table) == 0 and c.len == 0 and c.numFreeBlocks() == 4
    c.ensureCapacity(16)
    z, zp = np.zeros(R_T, np.float32), np.zeros(P_T, np.float32)
    for args, name in (((2, 0), "LayerOutOfBounds"), ((0, 16), "PositionOutOfBounds")):
        with pytest.raises(kv.KVCudaError) as e:
            c.put(*args, z, zp)
        assert e.value.name == name
    with pytest.raises(kv.KVCudaError) as e:
        c.getKVCompressed(0, 0)
    assert e.value.name == "PositionNotWritten"
    with pytest.raises(kv.KVCudaError) as e:
        c.ensureCapacity(16 * 5)
    assert e.value.name == "OutOfKVCacheBlocks"


def test_prefix_cache_on_gpu_cache(kv, oracle):
    c = kv.KVCache(1, R_T, P_T, 16 * 8)
    toks = list(range(100, 140))
    c.ensureCapacity(len(toks))
    prefix = kv.NO_HASH
    for bi in range(len(toks) // 16):
        c.cacheBlock(bi, toks[bi * 16:(bi + 1) * 16], prefix)
        prefix = kv.KVCache.computeHash(toks[bi * 16:(bi + 1) * 16], prefix)
        assert prefix == oracle.compute_hash(toks[bi * 16:(bi + 1) * 16],
                                             oracle.NO_HASH if bi == 0 else prev)
        prev = prefix
    assert c.findPrefixBlocks(toks) == 2
    before = c.numFreeBlocks()
    c.reusePrefixBlocks(toks, 2)
    assert c.len == 32 and c.numFreeBlocks() == before


# ------------------------------------------------------------------ config 1: f32 append + gather
def test_config1_f32_append_one_at_a_time_gather_bit_exact(kv, oracle):
    rng = np.random.default_rng(1)
    perm = rng.permutation(64).astype(np.uint32)[:32]
    free = perm[::-1].copy()  # LIFO: pops hand out perm[0], perm[1], ...
    c = kv.KVCache(1, R, P, 64 * 16)
    o = oracle.KVCache(1, R, P, 64 * 16)
    c.set_free_list(free)
    o.set_free_list(free)
    c.ensureCapacity(512)
    o.ensureCapacity(512)
    assert c.block_table == [int(x) for x in perm] == o.block_table
    rows = gen_seq_rows(oracle, 11, 0, 0, 512, 0.0)
    for t in range(512):
        c.put(0, t, rows[t, :R], rows[t, R:])
        o.put(0, t, rows[t, :R], rows[t, R:])
    got = c.gather(0, 0)
    assert got.shape == (512, W)
    assert np.array_equal(got.view(np.uint32), rows.view(np.uint32))
    want = o.pool().gather(0, np.array(o.block_table, np.uint32), 512)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ------------------------------------------------------------------ config 2: Q8_0 append + dequant-gather
def _multi_seq_cache(kv, oracle, lens, bs, nb, seed, quant, outlier_p, n_layers=1):
    c = kv.KVCache.with_blocks(n_layers, R, P, nb, bs, quantized=quant)
    o = oracle.Pool(n_layers, nb, bs, R, P, quant)
    for _ in range(len(lens) - 1):
        c.seq_create()
    rng = np.random.default_rng(seed)
    free = rng.permutation(nb).astype(np.uint32)
    c.set_free_list(free)
    for s, L in enumerate(lens):
        c.seq_ensure_capacity(s, L)
    rows = {}
    for layer in range(n_layers):
        for s, L in enumerate(lens):
            r = gen_seq_rows(oracle, seed, layer, s, L, outlier_p)
            rows[(layer, s)] = r
            tab = np.array(c.seq_block_table(s), np.uint32)
            t = np.arange(L)
            if L:
                o.put_rows(layer, tab[t // bs], t % bs, r)
            # append in a shuffled order, in two batches
            order = rng.permutation(L)
            half = L // 2
            for part in (order[:half], order[half:]):
                if part.size:
                    c.appendBatch(layer, np.full(part.size, s, np.uint32), part.astype(np.uint32), r[part])
    return c, o, rows


def test_config2_q8_append_gather_bit_exact(kv, oracle):
    lens = [300, 1024, 77, 2048]
    c, o, rows = _multi_seq_cache(kv, oracle, lens, 16, 256, 2, True, 0.01)
    assert c.numFreeBlocks() == 256 - 216
    # payload + scales, in the reference's BlockQ8_0 byte order
    assert c.pool().read_checkpoint() == o.serialize()
    for s, L in enumerate(lens):
        got = c.gather(0, s)
        want = o.gather(0, np.array(c.seq_block_table(s), np.uint32), L)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert c.seq_len(s) == L


def test_q8_edge_values_bit_exact(kv, oracle):
    """Zero rows, f16-subnormal scales, huge outliers, exact ties, inf."""
    rows = np.zeros((6, W), np.float32)
    rows[1] = 1e-4 * np.random.default_rng(3).standard_normal(W)
    rows[2, :32] = np.array([127.0] + [k + 0.5 for k in range(-15, 16)], np.float32)
    rows[3] = np.random.default_rng(4).standard_normal(W) * 1e5
    rows[4, 5] = np.inf
    rows[4, 40] = -np.inf
    rows[5] = np.random.default_rng(5).standard_normal(W).astype(np.float32) * np.float32(3e-39)
    c = kv.KVCache.with_blocks(1, R, P, 1, 16, quantized=True)
    o = oracle.Pool(1, 1, 16, R, P, True)
    c.ensureCapacity(16)
    c.appendBatch(0, np.zeros(6, np.uint32), np.arange(6, dtype=np.uint32), rows)
    o.put_rows(0, np.zeros(6, np.uint32), np.arange(6), rows)
    assert c.pool().read_checkpoint() == o.serialize()


def test_q8_near_tie_quotients_bit_exact(kv, oracle):
    """Quotients x/d within a few ulps of half-integers, for many inexact
    scales: the append kernel's multiply-then-check rounding must agree with
    roundf(x / d) everywhere, including both sides of every tie."""
    rng = np.random.default_rng(77)
    n = 64
    rows = np.zeros((n, W), np.float32)
    for r in range(n):
        for b in range(W // 32):
            amax = np.float32(np.exp(rng.uniform(-8, 8)))
            d = np.float32(amax / np.float32(127.0))
            blk = np.empty(32, np.float32)
            blk[0] = amax if rng.random() < 0.5 else -amax
            k = rng.integers(-127, 127, 31).astype(np.float32)
            x = ((k + np.float32(0.5)) * d).astype(np.float32)
            step = rng.integers(-3, 4, 31)
            for i in range(31):
                v = x[i]
                for _ in range(abs(int(step[i]))):
                    v = np.nextafter(v, np.float32(np.inf) if step[i] > 0 else np.float32(-np.inf))
                x[i] = v
            blk[1:] = np.clip(x, -amax, amax)
            rows[r, 32 * b:32 * b + 32] = rng.permutation(blk)
    c = kv.KVCache.with_blocks(1, R, P, 4, 16, quantized=True)
    o = oracle.Pool(1, 4, 16, R, P, True)
    c.ensureCapacity(n)
    pos = np.arange(n, dtype=np.uint32)
    c.appendBatch(0, np.zeros(n, np.uint32), pos, rows)
    o.put_rows(0, np.array(c.seq_block_table(0), np.uint32)[pos // 16], pos % 16, rows)
    assert c.pool().read_checkpoint() == o.serialize()


# ------------------------------------------------------------------ decode parity
def _decode_case(kv, oracle, lens, bs, quant, n_heads, seed, outlier_p=0.0, n_layers=1, impl=None,
                 expect_impl=None):
    nb = sum((int(L) + bs - 1) // bs for L in lens) + 3
    c, o, rows = _multi_seq_cache(kv, oracle, lens, bs, nb, seed, quant, outlier_p, n_layers)
    if impl is not None:
        c.set_decode_impl(impl)
    rng = np.random.default_rng(seed + 100)
    offs = [0]
    tabs = []
    for s in range(len(lens)):
        tabs.extend(c.seq_block_table(s))
        offs.append(len(tabs))
    offs = np.array(offs, np.uint32)
    tabs = np.array(tabs if tabs else [0], np.uint32)
    for layer in range(n_layers):
        q = rng.standard_normal((len(lens), n_heads, W)).astype(np.float32)
        got = c.mlaDecode(layer, q, np.arange(len(lens), dtype=np.uint32), SCALE)  # checks the status word
        if expect_impl is not None:
            assert c.last_decode_impl == expect_impl
        want = o.attention_batch(layer, offs, tabs, np.array(lens, np.uint32), q, SCALE, n_threads=8)
        err = rel_err_rows(got, want)
        assert err <= REL_TOL, (layer, err)
        for s, L in enumerate(lens):
            if L == 0:
                assert np.all(got[s] == 0)
    return c


def test_config3_decode_f32(kv, oracle):
    lens = np.random.default_rng(3).integers(1, 4097, 16).tolist()
    _decode_case(kv, oracle, lens, 16, False, 20, 3, expect_impl=kv.DECODE_CUDA_CORE)


@pytest.mark.parametrize("impl", [1, 2])
def test_decode_q8_config4_shape_reduced(kv, oracle, impl):
    lens = np.random.default_rng(4).integers(1000, 9000, 6).tolist()
    _decode_case(kv, oracle, lens, 64, True, 20, 4, outlier_p=0.01, n_layers=2, impl=impl,
                 expect_impl=impl)


@pytest.mark.parametrize("bs", [16, 32, 64, 128, 256])
def test_decode_block_sizes_and_ragged_lengths(kv, oracle, bs):
    lens = [0, 1, 15, 16, 17, 63, 64, 65, 127, 129, 300, 1000]
    _decode_case(kv, oracle, lens, bs, True, 20, 10 + bs, expect_impl=kv.DECODE_TENSOR_CORE)


@pytest.mark.parametrize("n_heads", [1, 4, 7, 8, 9, 16, 17, 20, 21, 24, 25, 32])
def test_decode_head_counts(kv, oracle, n_heads):
    expect = kv.DECODE_TENSOR_CORE if n_heads <= 24 else kv.DECODE_CUDA_CORE
    _decode_case(kv, oracle, [5, 200, 1000], 16, True, n_heads, 50 + n_heads, expect_impl=expect)


def test_decode_tensor_core_vs_cuda_core_same_data(kv, oracle):
    lens = [1, 130, 4000, 9000]
    c = _decode_case(kv, oracle, lens, 64, True, 20, 77, outlier_p=0.01)
    q = np.random.default_rng(78).standard_normal((len(lens), 20, W)).astype(np.float32)
    ids = np.arange(len(lens), dtype=np.uint32)
    c.set_decode_impl(kv.DECODE_TENSOR_CORE)
    a = c.mlaDecode(0, q, ids, SCALE)
    assert c.last_decode_impl == kv.DECODE_TENSOR_CORE
    c.set_decode_impl(kv.DECODE_CUDA_CORE)
    b = c.mlaDecode(0, q, ids, SCALE)
    assert c.last_decode_impl == kv.DECODE_CUDA_CORE
    assert rel_err_rows(a, b) <= REL_TOL


def test_decode_layers_layered_plan_against_the_oracle(kv, oracle, torch_mod):
    """The multi-layer call of the kvcache mirror balances all (layer, entry)
    pairs of the call as one list (a layered plan); every layer's output must
    still match the oracle."""
    torch = torch_mod
    lens = [0, 1, 200, 1500, 4100, 9000, 130, 64]
    nl, H, bs = 3, 20, 64
    nb = sum((L + bs - 1) // bs for L in lens) + 3
    c, o, _ = _multi_seq_cache(kv, oracle, lens, bs, nb, 91, True, 0.01, nl)
    offs, tabs = [0], []
    for s in range(len(lens)):
        tabs.extend(c.seq_block_table(s))
        offs.append(len(tabs))
    offs, tabs = np.array(offs, np.uint32), np.array(tabs, np.uint32)
    q = np.random.default_rng(92).standard_normal((nl, len(lens), H, W)).astype(np.float32)
    ids = np.arange(len(lens), dtype=np.uint32)
    q_dev = torch.from_numpy(q).cuda()
    out_dev = torch.full((nl, len(lens), H, R), float("nan"), device="cuda")
    c.mlaDecodeLayers_dev(0, ids, q_dev, SCALE, out_dev)
    torch.cuda.synchronize()
    got = out_dev.cpu().numpy()
    assert c.pool().status() == 0
    for layer in range(nl):
        want = o.attention_batch(layer, offs, tabs, np.array(lens, np.uint32), q[layer], SCALE, n_threads=8)
        err = rel_err_rows(got[layer], want)
        assert err <= REL_TOL, (layer, err)
        assert np.all(got[layer][0] == 0)  # the empty entry


def test_decode_lazy_rescale_when_scores_jump(kv, oracle):
    """Scores that double from one 128-token tile to the next (a sawtooth of 4
    tiles, gains 1, 2, 4, 8) inside items of several tiles: the tensor-core
    kernel must rescale its TMEM accumulators whenever a head's max grows by
    more than 2^14 (here from the third tile of a run on, ~27 -> ~54 in log2
    units).  The batch (8 x 12,800 tokens, ~5 tiles per CTA) makes the plan give
    every CTA multi-tile items, so most CTAs cross a doubling inside an item.
    (The gains stop at 8: the query's two-digit encoding has an error relative
    to |q|, so the score error grows with |k|; at gains of 128, scores near
    1,000 log2 units, it reaches ~0.02 and the output error 6e-3.)"""
    n, L, bs = 8, 12800, 64
    nbs = (L + bs - 1) // bs
    c = kv.KVCache.with_blocks(1, R, P, n * nbs + 1, bs, quantized=True)
    o = oracle.Pool(1, n * nbs + 1, bs, R, P, True)
    for _ in range(n - 1):
        c.seq_create()
    t = np.arange(L)
    gain = np.float32(2.0) ** ((t // 128) % 4).astype(np.float32)
    offs, tabs = [0], []
    for s in range(n):
        c.seq_ensure_capacity(s, L)
        rows = gen_seq_rows(oracle, 91 + s, 0, s, L, 0.0) * gain[:, None]
        c.appendBatch(0, np.full(L, s, np.uint32), t.astype(np.uint32), rows)
        tab = np.array(c.seq_block_table(s), np.uint32)
        o.put_rows(0, tab[t // bs], t % bs, rows)
        tabs.extend(tab.tolist())
        offs.append(len(tabs))
    q = np.random.default_rng(92).standard_normal((n, 20, W)).astype(np.float32)
    got = c.mlaDecode(0, q, np.arange(n, dtype=np.uint32), SCALE)
    assert c.last_decode_impl == kv.DECODE_TENSOR_CORE
    want = o.attention_batch(0, np.array(offs, np.uint32), np.array(tabs, np.uint32),
                             np.full(n, L, np.uint32), q, SCALE, n_threads=8)
    assert rel_err_rows(got, want) <= REL_TOL


def test_tensor_core_forced_on_f32_pool_is_unsupported(kv):
    c = kv.KVCache.with_blocks(1, R, P, 4, 16, quantized=False)
    c.ensureCapacity(16)
    c.appendBatch(0, np.zeros(3, np.uint32), np.arange(3, dtype=np.uint32), np.ones((3, W), np.float32))
    c.set_decode_impl(kv.DECODE_TENSOR_CORE)
    with pytest.raises(kv.KVCudaError) as e:
        c.mlaDecode(0, np.ones((1, 20, W), np.float32), np.zeros(1, np.uint32), SCALE)
    assert e.value.name == "Unsupported"
    c.set_decode_impl(kv.DECODE_AUTO)
    out = c.mlaDecode(0, np.ones((1, 20, W), np.float32), np.zeros(1, np.uint32), SCALE)
    assert np.allclose(out, 1.0)


def test_decode_device_api_plan_reuse_with_growth(kv, oracle, torch_mod):
    """Append one token per step on the device and decode with the plan reused."""
    torch = torch_mod
    lens = [40, 700, 3000, 5]
    steps = 5
    bs = 16
    nb = sum((L + steps + bs - 1) // bs for L in lens) + 1
    c = kv.KVCache.with_blocks(1, R, P, nb, bs, quantized=True)
    for _ in range(len(lens) - 1):
        c.seq_create()
    for s, L in enumerate(lens):
        c.seq_ensure_capacity(s, L + steps)
        c.appendBatch(0, np.full(L, s, np.uint32), np.arange(L, dtype=np.uint32),
                      gen_seq_rows(oracle, 9, 0, s, L, 0.01))
    ids = np.arange(len(lens), dtype=np.uint32)
    rng = np.random.default_rng(9)
    q = rng.standard_normal((len(lens), 20, W)).astype(np.float32)
    qd = torch.from_numpy(q).cuda()
    out = torch.empty((len(lens), 20, R), dtype=torch.float32, device="cuda")
    cur = list(lens)
    for step in range(steps):
        newrows = np.stack([gen_seq_rows(oracle, 9, 0, s, cur[s] + 1, 0.01)[-1] for s in range(len(lens))])
        pos = np.array(cur, np.uint32)
        c.appendBatch_dev(0, ids, pos, torch.from_numpy(ids).cuda(), torch.from_numpy(pos).cuda(),
                          torch.from_numpy(newrows).cuda())
        cur = [x + 1 for x in cur]
        c.mlaDecode_dev(0, ids, qd, SCALE, out)
        torch.cuda.synchronize()
    want_rows = [[gen_seq_rows(oracle, 9, 0, s, cur[s], 0.01) for s in range(len(lens))]]
    pool, offs, tabs = oracle_pool_for(oracle, want_rows, cur, bs, True)
    want = pool.attention_batch(0, offs, tabs, np.array(cur, np.uint32), q, SCALE, n_threads=8)
    assert rel_err_rows(out.cpu().numpy(), want) <= REL_TOL
    assert [c.seq_len(s) for s in range(len(lens))] == cur


def test_decode_host_api_pinned_buffers_in_place(kv, oracle, torch_mod):
    """Pinned, mapped q / out are read and written in place by the kernels; the
    outputs equal the copy path's and the device API's bit for bit, and match
    the oracle."""
    torch = torch_mod
    lens = [1, 300, 2500, 70, 9000]
    bs, H = 64, 20
    nb = sum((L + bs - 1) // bs for L in lens) + 2
    c, o, _ = _multi_seq_cache(kv, oracle, lens, bs, nb, 41, True, 0.01)
    ids = np.arange(len(lens), dtype=np.uint32)
    q = np.random.default_rng(41).standard_normal((len(lens), H, W)).astype(np.float32)
    # pageable: copied
    out_copy = c.mlaDecode(0, q, ids, SCALE)
    assert not c.last_decode_mapped
    # pinned q and out: used in place
    q_pin = torch.from_numpy(q).pin_memory()
    out_pin = torch.full((len(lens), H, R), float("nan")).pin_memory()
    c.mlaDecode_ptr(0, len(lens), ids, q_pin.data_ptr(), H, SCALE, out_pin.data_ptr())
    assert c.last_decode_mapped
    # pinned q, pageable out: copied
    out_mixed = np.full((len(lens), H, R), np.nan, np.float32)
    c.mlaDecode_ptr(0, len(lens), ids, q_pin.data_ptr(), H, SCALE, out_mixed.ctypes.data)
    assert not c.last_decode_mapped
    out_dev = torch.empty((len(lens), H, R), device="cuda")
    c.mlaDecode_dev(0, ids, torch.from_numpy(q).cuda(), SCALE, out_dev)
    torch.cuda.synchronize()
    assert np.array_equal(out_pin.numpy(), out_copy)
    assert np.array_equal(out_mixed, out_copy)
    assert np.array_equal(out_dev.cpu().numpy(), out_copy)
    offs = [0]
    tabs = []
    for s in range(len(lens)):
        tabs.extend(c.seq_block_table(s))
        offs.append(len(tabs))
    want = o.attention_batch(0, np.array(offs, np.uint32), np.array(tabs, np.uint32),
                             np.array(lens, np.uint32), q, SCALE, n_threads=8)
    assert rel_err_rows(out_copy, want) <= REL_TOL


def test_decode_split_matches_unsplit(kv, oracle):
    """A long sequence decoded alone (split across CTAs) equals the same sequence
    decoded inside a batch of short ones (different split) to 2e-4: the
    tensor-core kernel rounds P to f16 against each item's running maximum, so
    other split points round other values (each side is within 1e-3 of the
    oracle)."""
    lens = [20000, 3, 3, 3]
    c = _decode_case(kv, oracle, lens, 64, True, 20, 21)
    q = np.random.default_rng(22).standard_normal((1, 20, W)).astype(np.float32)
    a = c.mlaDecode(0, q, np.array([0], np.uint32), SCALE)
    qq = np.concatenate([q, q, q], axis=0)
    b = c.mlaDecode(0, qq, np.array([1, 0, 2], np.uint32), SCALE)
    assert rel_err_rows(b[1:2], a) <= 2e-4


# ------------------------------------------------------------------ checkpoint v2
def test_checkpoint_v2_roundtrip(kv, oracle, tmp_path):
    lens = [300, 1024, 77]
    c, o, _ = _multi_seq_cache(kv, oracle, lens, 16, 128, 31, True, 0.01)
    path = tmp_path / "multi.kvck"
    c.saveToFileV2(path)
    d = kv.KVCache.with_blocks(1, R, P, 128, 16, quantized=True)
    d.loadFromFileV2(path)
    assert d.num_seqs == 3
    assert [d.seq_len(s) for s in range(3)] == lens
    assert [d.seq_block_table(s) for s in range(3)] == [c.seq_block_table(s) for s in range(3)]
    assert d.pool().read_checkpoint() == c.pool().read_checkpoint() == o.serialize()
    assert d.numFreeBlocks() == c.numFreeBlocks()
    q = np.random.default_rng(5).standard_normal((3, 20, W)).astype(np.float32)
    ids = np.arange(3, dtype=np.uint32)
    assert np.array_equal(c.mlaDecode(0, q, ids, SCALE), d.mlaDecode(0, q, ids, SCALE))


@pytest.mark.parametrize("quant,nb,bs,lens", [(True, 4096, 64, [60000, 70000, 50000]),
                                              (False, 2048, 16, [12000, 9000, 9000])])
def test_checkpoint_v2_roundtrip_multi_chunk(kv, tmp_path, quant, nb, bs, lens):
    """Pools larger than the 64 MB I/O chunk (160 MB Q8_0, 75 MB f32): the pipelined save
    and load give back the same bytes."""
    c = kv.KVCache.with_blocks(1, R, P, nb, bs, quantized=quant)
    for _ in range(len(lens) - 1):
        c.seq_create()
    ids = np.arange(len(lens), dtype=np.uint32)
    for s, L in enumerate(lens):
        c.seq_ensure_capacity(s, L)
    c.prefill_synthetic(0, ids, np.array(lens), 3, 0.01)
    path = tmp_path / "big.kvck"
    c.saveToFileV2(path)
    d = kv.KVCache.with_blocks(1, R, P, nb, bs, quantized=quant)
    d.loadFromFileV2(path)
    assert [d.seq_len(s) for s in range(len(lens))] == lens
    assert d.pool().read_checkpoint() == c.pool().read_checkpoint()
    assert np.array_equal(d.gather(0, 2), c.gather(0, 2))


# ------------------------------------------------------------------ bad indices set the status word
def test_bad_table_entries_set_status_without_fault(kv, torch_mod):
    torch = torch_mod
    pool = kv.DevicePool(0, 1, 4, 16, R, P, True)
    rows = torch.zeros((2, W), dtype=torch.float32, device="cuda")
    toff = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    tables = torch.tensor([1000], dtype=torch.int32, device="cuda")  # >= num_blocks
    seq = torch.zeros(2, dtype=torch.int32, device="cuda")
    pos = torch.tensor([0, 40], dtype=torch.int32, device="cuda")  # 40 -> beyond the table
    pool.append(0, rows, seq, pos, toff, tables)
    st = pool.status()
    assert st & 0x2 and st & 0x1
    assert pool.status() == 0  # read-and-clear
    out = torch.zeros((16, W), dtype=torch.float32, device="cuda")
    pool.gather(0, tables, 16, out)
    assert pool.status() & 0x2
    assert torch.count_nonzero(out).item() == 0
