"""CPU restatement of the reference's MLA decode step around the KV cache.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA step (kvcu_mla_prepare,
kvcu_append, kvcu_mla_decode_lse, kvcu_mla_finish). Only tests/ may import it.

It follows the reference statement by statement in float32:
  rms_norm            src/math.zig:7-35
  RoPE table / apply  src/math.zig:197-240 (table built as RoPECache.init does)
  mat_vec             src/math.zig:79-99 (row-major w[out_dim][in_dim])
  mla_attention       src/inference.zig:492-513 (norm, RoPE, put) and 518-660
                      (k_b / v_b expansion per position, 64-position blocks of
                      online softmax, out = o / l, 0 when l <= 0)
The KV cache itself is the C oracle's KVCache (kvoracle.py), driven with the
reference's calls (put, getKVCompressed, getKPe).

Pinning: rms_norm reproduces the reference's own unit test (math.zig:244-254).
RoPE has no test in the reference; it is checked by its defining properties
(identity at position 0, pair norms preserved, the frequency formula). The
attention arithmetic has no golden vectors in the reference; it is checked
against an independent absorbed-form evaluation (mla_attention_absorbed).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def rms_norm(x, w, eps):
    """math.zig:7-35: x / sqrt(mean(x^2) + eps) * w, in f32."""
    x = np.asarray(x, F32)
    ss = F32(np.sum(x * x, dtype=F32))
    ss = F32(ss / F32(x.size) + F32(eps))
    inv = F32(F32(1.0) / np.sqrt(ss, dtype=F32))
    return (x * inv * np.asarray(w, F32)).astype(F32)


def rope_tables(pos, dim, base):
    """RoPECache.init (math.zig:205-222) for one position: cos/sin[i], i < dim."""
    i = np.arange(dim, dtype=np.int64)
    expo = (2 * i).astype(F32) / F32(dim)
    freq = F32(1.0) / np.power(F32(base), expo, dtype=F32)
    theta = F32(pos) * freq
    return np.cos(theta, dtype=F32), np.sin(theta, dtype=F32)


def rope_apply(v, pos, dim, base):
    """RoPECache.apply (math.zig:227-238): rotate pairs (2i, 2i+1), i < dim/2."""
    cs, sn = rope_tables(pos, dim, base)
    out = np.array(v, F32)
    for i in range(dim // 2):
        q0, q1 = out[2 * i], out[2 * i + 1]
        out[2 * i] = F32(q0 * cs[i] - q1 * sn[i])
        out[2 * i + 1] = F32(q0 * sn[i] + q1 * cs[i])
    return out


def mat_vec(w, x):
    """math.zig:79-99: out[row] = sum_j w[row][j] x[j] (f32)."""
    return (np.asarray(w, F32) @ np.asarray(x, F32)).astype(F32)


def prepare(kv_a, q, pos, norm_w, eps, rope_base, kv_rank, qk_nope, qk_rope):
    """inference.zig:492-513: the cached latent, k_pe and the roped query."""
    kv_comp = rms_norm(kv_a[:kv_rank], norm_w, eps)
    k_pe = rope_apply(kv_a[kv_rank:kv_rank + qk_rope], pos, qk_rope, rope_base)
    qr = np.array(q, F32)
    for h in range(qr.shape[0]):
        qr[h, qk_nope:qk_nope + qk_rope] = rope_apply(qr[h, qk_nope:qk_nope + qk_rope], pos, qk_rope, rope_base)
    return kv_comp, k_pe, qr


def mla_attention(cache, layer, pos, q, kv_a, norm_w, eps, rope_base, k_b, v_b, qk_nope, qk_rope, v_dim):
    """One decode step of inference.zig:518-660 for one sequence; returns attn_out [H][v_dim].

    `cache` is a kvoracle.KVCache already holding positions < pos of `layer`.
    """
    kv_rank = cache.kv_rank
    n_heads = q.shape[0]
    head_dim = qk_nope + qk_rope
    kv_comp, k_pe, qr = prepare(kv_a, q, pos, norm_w, eps, rope_base, kv_rank, qk_nope, qk_rope)
    rc = cache.put(layer, pos, kv_comp, k_pe)
    if rc:
        raise RuntimeError(f"put failed: {rc}")
    cur_k_nope = mat_vec(k_b, kv_comp)
    cur_v = mat_vec(v_b, kv_comp)
    hist_c = np.stack([cache.getKVCompressed(layer, p)[1] for p in range(pos)]) if pos else None
    kpe = np.stack([cache.getKPe(layer, p)[1] for p in range(pos + 1)])
    if pos:
        hist_k = (hist_c @ np.asarray(k_b, F32).T).astype(F32)  # [pos][H*qk_nope]
        hist_v = (hist_c @ np.asarray(v_b, F32).T).astype(F32)  # [pos][H*v_dim]
    out = np.zeros((n_heads, v_dim), F32)
    sq = np.sqrt(F32(head_dim), dtype=F32)
    BLOCK = 64
    for h in range(n_heads):
        q_nope = qr[h, :qk_nope]
        q_rope = qr[h, qk_nope:head_dim]
        m_vec, l_vec = F32(-np.inf), F32(0.0)
        o_vec = np.zeros(v_dim, F32)
        for b_start in range(0, pos + 1, BLOCK):
            b_end = min(b_start + BLOCK, pos + 1)
            scores = np.zeros(b_end - b_start, F32)
            for p in range(b_start, b_end):
                kn = cur_k_nope[h * qk_nope:(h + 1) * qk_nope] if p == pos else hist_k[p, h * qk_nope:(h + 1) * qk_nope]
                s = F32(np.dot(q_nope, kn)) + F32(np.dot(q_rope, kpe[p]))
                scores[p - b_start] = F32(s / sq)
            m_j = F32(scores.max())
            e = np.exp(scores - m_j, dtype=F32)
            l_j = F32(e.sum(dtype=F32))
            m_new = max(m_vec, m_j)
            scale_o = F32(np.exp(F32(m_vec - m_new))) if m_vec != -np.inf else F32(0.0)
            scale_s = F32(np.exp(F32(m_j - m_new)))
            o_vec = (o_vec * scale_o).astype(F32)
            for p in range(b_start, b_end):
                wgt = F32(e[p - b_start] * scale_s)
                vv = cur_v[h * v_dim:(h + 1) * v_dim] if p == pos else hist_v[p, h * v_dim:(h + 1) * v_dim]
                o_vec = (o_vec + wgt * vv).astype(F32)
            m_vec = m_new
            l_vec = F32(l_vec * scale_o + l_j * scale_s)
        out[h] = o_vec / l_vec if l_vec > 0 else 0.0
    return out


def mla_attention_absorbed(hist_c, hist_kpe, pos, q, kv_a, norm_w, eps, rope_base, k_b, v_b, qk_nope, qk_rope,
                           v_dim, kpe_cur=None):
    """The same step evaluated in absorbed form in float64 (an independent check
    of the algebra the GPU path uses): q_abs = [k_b_h^T q_nope, q_rope],
    out_h = v_b_h (softmax-weighted sum of latents). hist_c / hist_kpe are the
    cached latents / k_pe of positions < pos; the newest token uses its
    unquantized latent and `kpe_cur` (its k_pe as cached; default: unquantized)."""
    kv_rank = k_b.shape[1]
    n_heads = q.shape[0]
    head_dim = qk_nope + qk_rope
    kv_comp, k_pe, qr = prepare(kv_a, q, pos, norm_w, eps, rope_base, kv_rank, qk_nope, qk_rope)
    if kpe_cur is None:
        kpe_cur = k_pe
    C = np.concatenate([np.asarray(hist_c, np.float64).reshape(-1, kv_rank), kv_comp[None].astype(np.float64)])
    KP = np.concatenate([np.asarray(hist_kpe, np.float64).reshape(-1, qk_rope), kpe_cur[None].astype(np.float64)])
    out = np.zeros((n_heads, v_dim))
    for h in range(n_heads):
        kb = np.asarray(k_b, np.float64)[h * qk_nope:(h + 1) * qk_nope]
        vb = np.asarray(v_b, np.float64)[h * v_dim:(h + 1) * v_dim]
        q_abs = kb.T @ qr[h, :qk_nope].astype(np.float64)
        s = (C @ q_abs + KP @ qr[h, qk_nope:head_dim].astype(np.float64)) / np.sqrt(head_dim)
        w = np.exp(s - s.max())
        out[h] = vb @ (w @ C / w.sum())
    return out.astype(F32)
