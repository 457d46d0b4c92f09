"""The MLA decode step on the GPU (kvcache_mla_step_dev: kvcu_mla_prepare,
append, kvcu_mla_decode_lse over the history, kvcu_mla_finish) against the
reference's non-absorbed step restated on the CPU (oracle/mla_ref.py, one
oracle KVCache per sequence holding the same history), <= 1e-3 relative."""
import numpy as np
import pytest

from kvdata import REL_TOL, rel_err_rows

pytestmark = pytest.mark.gpu

R, P, H, QK_NOPE, V_DIM = 512, 64, 20, 128, 128
EPS, BASE = 1e-6, 10000.0
SCALE = float(np.float32(1.0 / np.sqrt(QK_NOPE + P)))


@pytest.fixture(scope="module")
def kv():
    import torch

    import kvcu

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    kvcu.init(0)
    return kvcu


def _run_step(kv, oracle, hist, bs, quant, seed, n_heads=H, layers=1, layer=0):
    import torch

    import mla_ref

    rng = np.random.default_rng(seed)
    n = len(hist)
    cap = [L + 1 for L in hist]
    nb = sum((c + bs - 1) // bs for c in cap) + 2
    cache = kv.KVCache.with_blocks(layers, R, P, nb, bs, quantized=quant)
    for _ in range(n - 1):
        cache.seq_create()
    refs = []
    for s, L in enumerate(hist):
        cache.seq_ensure_capacity(s, cap[s])
        oc = oracle.KVCache(layers, R, P, cap[s] + bs, bs)
        if quant:
            oc.enableQuantization()
        assert oc.ensureCapacity(cap[s]) == 0
        if L:
            rows = rng.standard_normal((L, R + P)).astype(np.float32)
            cache.appendBatch(layer, np.full(L, s, np.uint32), np.arange(L, dtype=np.uint32), rows)
            for p in range(L):
                assert oc.put(layer, p, rows[p, :R], rows[p, R:]) == 0
        refs.append(oc)
    q = rng.standard_normal((n, n_heads, QK_NOPE + P)).astype(np.float32)
    kv_a = rng.standard_normal((n, R + P)).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(R)).astype(np.float32)
    k_b = (rng.standard_normal((n_heads * QK_NOPE, R)) / np.sqrt(R)).astype(np.float32)
    v_b = (rng.standard_normal((n_heads * V_DIM, R)) / np.sqrt(R)).astype(np.float32)
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(a).to(dev)
    attn = torch.full((n, n_heads, V_DIM), float("nan"), device=dev)
    ids = np.arange(n, dtype=np.uint32)
    pos = np.array(hist, np.uint32)
    cache.mla_step_dev(layer, ids, pos, t(q), t(kv_a), t(w), EPS, BASE, t(k_b), t(v_b), QK_NOPE, V_DIM, SCALE,
                       attn)
    torch.cuda.synchronize()
    assert cache.pool().status() == 0
    got = attn.cpu().numpy()
    want = np.stack([mla_ref.mla_attention(refs[b], layer, hist[b], q[b], kv_a[b], w, EPS, BASE, k_b, v_b,
                                           QK_NOPE, P, V_DIM) for b in range(n)])
    return cache, refs, got, want


@pytest.mark.parametrize("quant", [True, False])
def test_mla_step_matches_reference(kv, oracle, quant):
    # empty history, one token, block edges, a long sequence that the plan splits
    hist = [0, 1, 63, 64, 65, 300, 1500]
    cache, refs, got, want = _run_step(kv, oracle, hist, 64, quant, 31)
    assert np.isfinite(got).all()
    assert rel_err_rows(got, want) <= REL_TOL
    assert [cache.seq_len(s) for s in range(len(hist))] == [L + 1 for L in hist]


def test_mla_step_appends_the_normalised_roped_row(kv, oracle):
    # the step's append stores RMSNorm(latent) and RoPE(k_pe) as the reference's put does (f32 cache)
    hist = [5, 130]
    cache, refs, got, want = _run_step(kv, oracle, hist, 16, False, 32)
    for s, L in enumerate(hist):
        row = cache.gather(0, s)[L]
        c_ref = refs[s].getKVCompressed(0, L)[1]
        k_ref = refs[s].getKPe(0, L)[1]
        assert np.allclose(row[:R], c_ref, rtol=1e-5, atol=1e-6)
        assert np.allclose(row[R:], k_ref, rtol=1e-5, atol=1e-5)


def test_mla_step_cuda_core_heads_and_large_positions(kv, oracle):
    # 28 heads take the CUDA-core decode; positions past 4096 exercise RoPE's large angles
    hist = [4100, 17, 0]
    cache, refs, got, want = _run_step(kv, oracle, hist, 16, True, 33, n_heads=28)
    assert cache.last_decode_impl == kv.DECODE_CUDA_CORE
    assert rel_err_rows(got, want) <= REL_TOL


def test_mla_step_rejects_repeated_sequence(kv):
    import torch

    cache = kv.KVCache.with_blocks(1, R, P, 8, 16, quantized=True)
    cache.seq_ensure_capacity(0, 4)
    dev = torch.device("cuda", 0)
    z = lambda *s: torch.zeros(s, device=dev)
    with pytest.raises(kv.KVCudaError):
        cache.mla_step_dev(0, [0, 0], [0, 1], z(2, H, QK_NOPE + P), z(2, R + P), z(R), EPS, BASE,
                           z(H * QK_NOPE, R), z(H * V_DIM, R), QK_NOPE, V_DIM, SCALE, z(2, H, V_DIM))


@pytest.mark.parametrize("between", [False, True])
def test_mla_step_layers_share_the_plan(kv, oracle, between):
    """Two layers of one step with the same positions: the second layer reuses
    the first layer's plan (one launch fewer), unless another decode planned on
    the workspace in between. Both layers match the reference either way."""
    import torch

    import mla_ref

    rng = np.random.default_rng(41)
    hist = [0, 63, 300, 1500]
    n, bs, layers = len(hist), 64, 2
    cap = [L + 1 for L in hist]
    nb = sum((c + bs - 1) // bs for c in cap) + 2
    cache = kv.KVCache.with_blocks(layers, R, P, nb, bs, quantized=True)
    for _ in range(n - 1):
        cache.seq_create()
    refs = []
    for s, L in enumerate(hist):
        cache.seq_ensure_capacity(s, cap[s])
        oc = oracle.KVCache(layers, R, P, cap[s] + bs, bs)
        oc.enableQuantization()
        assert oc.ensureCapacity(cap[s]) == 0
        for layer in range(layers):
            if L:
                rows = rng.standard_normal((L, R + P)).astype(np.float32)
                cache.appendBatch(layer, np.full(L, s, np.uint32), np.arange(L, dtype=np.uint32), rows)
                for p in range(L):
                    assert oc.put(layer, p, rows[p, :R], rows[p, R:]) == 0
        refs.append(oc)
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(a).to(dev)
    ids = np.arange(n, dtype=np.uint32)
    pos = np.array(hist, np.uint32)
    w = (1.0 + 0.1 * rng.standard_normal(R)).astype(np.float32)
    launches = []
    for layer in range(layers):
        q = rng.standard_normal((n, H, QK_NOPE + P)).astype(np.float32)
        kv_a = rng.standard_normal((n, R + P)).astype(np.float32)
        k_b = (rng.standard_normal((H * QK_NOPE, R)) / np.sqrt(R)).astype(np.float32)
        v_b = (rng.standard_normal((H * V_DIM, R)) / np.sqrt(R)).astype(np.float32)
        attn = torch.full((n, H, V_DIM), float("nan"), device=dev)
        cache.mla_step_dev(layer, ids, pos, t(q), t(kv_a), t(w), EPS, BASE, t(k_b), t(v_b), QK_NOPE, V_DIM,
                           SCALE, attn)
        launches.append(cache.last_launches)
        torch.cuda.synchronize()
        assert cache.pool().status() == 0
        got = attn.cpu().numpy()
        want = np.stack([mla_ref.mla_attention(refs[b], layer, hist[b], q[b], kv_a[b], w, EPS, BASE, k_b, v_b,
                                               QK_NOPE, P, V_DIM) for b in range(n)])
        assert rel_err_rows(got, want) <= REL_TOL, layer
        if between and layer == 0:
            # a plain decode of layer 0 over the full lengths plans on the same workspace
            cache.mlaDecode(0, rng.standard_normal((n, H, R + P)).astype(np.float32), ids, SCALE)
    assert launches[1] == launches[0] - (0 if between else 1)


def test_mla_finish_public_entry_matches_float64(kv):
    """kvcu_mla_finish (the C-ABI call a caller with its own scratch uses: the
    in-place merge, then the v_b product) against float64 on the same inputs:
    the newest token's score with its latent and k_pe (an f32 pool keeps k_pe
    as given), the log-sum-exp merge into the history output, and v_b. One entry
    has an empty history (lse = -inf), so its output is the newest token alone."""
    import torch

    n, v_dim = 6, V_DIM
    pool = kv.DevicePool(0, 1, 4, 16, R, P, False)
    try:
        g = torch.Generator(device="cuda").manual_seed(43)
        dev = torch.device("cuda", 0)
        q_abs = torch.randn((n, H, R + P), device=dev, generator=g) * 0.05
        rows = torch.randn((n, R + P), device=dev, generator=g)
        latent = torch.randn((n, H, R), device=dev, generator=g)
        lse = torch.randn((n, H), device=dev, generator=g) * 3.0
        lse[2] = float("-inf")
        v_b = torch.randn((H * v_dim, R), device=dev, generator=g) / R ** 0.5
        attn = torch.full((n, H, v_dim), float("nan"), device=dev)
        lat64, rows64, q64, lse64 = latent.double(), rows.double(), q_abs.double(), lse.double()
        s = (q64 * rows64[:, None, :]).sum(-1) * SCALE
        m = torch.maximum(lse64, s)
        wh = torch.where(torch.isinf(lse64), torch.zeros_like(m), torch.exp(lse64 - m))
        wc = torch.exp(s - m)
        merged = (lat64 * wh[..., None] + rows64[:, None, :R] * wc[..., None]) / (wh + wc)[..., None]
        want = torch.einsum("bhr,hjr->bhj", merged, v_b.double().view(H, v_dim, R))
        torch.cuda.synchronize()
        rc = kv.lib().kvcu_mla_finish(pool.handle, n, H, v_dim, q_abs.data_ptr(), rows.data_ptr(),
                                      latent.data_ptr(), lse.data_ptr(), SCALE, v_b.data_ptr(), attn.data_ptr(),
                                      None)
        torch.cuda.synchronize()
        assert rc == 0
        assert pool.status() == 0
        err = ((attn.double() - want).abs().amax() / want.abs().amax()).item()
        assert err <= 2e-5, err
    finally:
        pool.close()
