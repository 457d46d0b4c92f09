"""CPU checks of the MLA-step restatement (oracle/mla_ref.py) that the GPU
step is compared against: the reference's own rmsNorm test, RoPE's defining
properties, and the non-absorbed reference form against an independent
absorbed evaluation (the algebra the CUDA path relies on)."""
import numpy as np

import kvoracle
import mla_ref


def test_rms_norm_reference_kat():
    # src/math.zig:244-254: weight 1, x = 2 -> 2 * 1/sqrt(4 + 1e-5) ~ 1.0 (abs 1e-4)
    out = mla_ref.rms_norm(np.full(4, 2.0, np.float32), np.ones(4, np.float32), 1e-5)
    assert np.allclose(out, 1.0, atol=1e-4)


def test_rms_norm_formula():
    rng = np.random.default_rng(1)
    x = rng.standard_normal(512).astype(np.float32)
    w = rng.standard_normal(512).astype(np.float32)
    want = x / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-6) * w
    assert np.allclose(mla_ref.rms_norm(x, w, 1e-6), want, rtol=1e-5, atol=1e-6)


def test_rope_properties():
    rng = np.random.default_rng(2)
    v = rng.standard_normal(64).astype(np.float32)
    assert np.array_equal(mla_ref.rope_apply(v, 0, 64, 10000.0), v)  # cos 0 = 1, sin 0 = 0
    for pos in (1, 17, 4095, 65535):
        r = mla_ref.rope_apply(v, pos, 64, 10000.0)
        n0 = v[0::2] ** 2 + v[1::2] ** 2
        n1 = r[0::2].astype(np.float64) ** 2 + r[1::2].astype(np.float64) ** 2
        assert np.allclose(n0, n1, rtol=1e-5)
        # pair i turns by pos * base^(-2i/dim)
        i = np.arange(32)
        theta = pos * 10000.0 ** (-2.0 * i / 64)
        want0 = v[0::2] * np.cos(theta) - v[1::2] * np.sin(theta)
        assert np.allclose(r[0::2], want0, atol=2e-3 * max(1.0, pos / 4096))


def _case(rng, H, qk_nope, qk_rope, v_dim, R):
    q = rng.standard_normal((H, qk_nope + qk_rope)).astype(np.float32)
    kv_a = rng.standard_normal(R + qk_rope).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(R)).astype(np.float32)
    k_b = (rng.standard_normal((H * qk_nope, R)) / np.sqrt(R)).astype(np.float32)
    v_b = (rng.standard_normal((H * v_dim, R)) / np.sqrt(R)).astype(np.float32)
    return q, kv_a, w, k_b, v_b


def test_reference_form_matches_absorbed_form():
    R, P, H, qk_nope, v_dim = 64, 16, 3, 32, 16
    rng = np.random.default_rng(3)
    for quant in (False, True):
        for pos in (0, 1, 63, 64, 70):
            cache = kvoracle.KVCache(1, R, P, 128, 16)
            if quant:
                cache.enableQuantization()
            assert cache.ensureCapacity(pos + 1) == 0
            for p in range(pos):
                row = rng.standard_normal(R + P).astype(np.float32)
                assert cache.put(0, p, row[:R], row[R:]) == 0
            hist_c = np.array([cache.getKVCompressed(0, p)[1] for p in range(pos)]).reshape(-1, R)
            hist_kpe = np.array([cache.getKPe(0, p)[1] for p in range(pos)]).reshape(-1, P)
            q, kv_a, w, k_b, v_b = _case(rng, H, qk_nope, P, v_dim, R)
            got = mla_ref.mla_attention(cache, 0, pos, q, kv_a, w, 1e-6, 10000.0, k_b, v_b, qk_nope, P, v_dim)
            kpe_cur = cache.getKPe(0, pos)[1]  # the newest k_pe as cached
            want = mla_ref.mla_attention_absorbed(hist_c, hist_kpe, pos, q, kv_a, w, 1e-6, 10000.0, k_b, v_b,
                                                  qk_nope, P, v_dim, kpe_cur=kpe_cur)
            err = np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)
            assert err < 2e-5, (quant, pos, err)
