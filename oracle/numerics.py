"""CPU oracle for the Enigma hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, and only as the checker or the timed CPU baseline.
The product path (enigma-dsl_b200/) never calls it.

Each function restates, in numpy, the reference's own numpy check for that
operator (the reference keeps its checks inline in its examples and tests;
there are no stored golden arrays).  Parity pins:
  * rmsnorm          examples/benchmark_rmsnorm.py:117-118 and
                     examples/qwen_megakernel.py:308-310
  * sdpa             examples/showcase_attention.py:150-153 (scaled, max-subtracted
                     softmax) and examples/benchmark_sdpa.py:198-208 (GQA head map
                     kvh = qh // QMUL).  The reference has no causal variant:
                     the causal mask here (key j > i + Sk - Sq masked) is
                     "parity unpinned" beyond the softmax formula.
  * gemm             tests/metal/test_gemm_matmul_runtime.py:136,166 (`a @ b`),
                     enigma/ops/gemm.py:144-167 (C += A @ B).
  * decode layer     examples/qwen_megakernel.py:320-342 (full_decode_np), at the
                     BASELINE shapes; standard theta RoPE replaces the example's
                     synthetic angles (the rotation itself is rope_np's half-split
                     form at :313-317).

Pinning: tests/golden/numerics.npz holds outputs of the reference's own numpy
code (extracted from the example scripts by tests/golden/make_numerics_golden.py
and run on seeded inputs); tests/test_numerics_golden.py checks every function
above against them.  Not pinned by any reference code: the causal mask and the
theta-RoPE angle table (the rotation given the angles is pinned).
"""
from __future__ import annotations

import numpy as np


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even), returned as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    # uint32 arithmetic: for every non-NaN pattern u + 0x8000 < 2^32, so nothing wraps;
    # NaNs are passed through below.
    r = (u >> 16) & np.uint32(1)
    r += np.uint32(0x7FFF)
    r += u
    r &= np.uint32(0xFFFF0000)
    out = r.view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = x[nan]
    return out


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# --------------------------------------------------------------------------- RMSNorm
def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """y = x / sqrt(mean(x^2) + eps) * w, per row (benchmark_rmsnorm.py:117-118).

    The mean is accumulated in fp64 so the oracle is more exact than any
    fp32 device reduction; the result is returned in fp32.
    """
    x64 = np.asarray(x, dtype=np.float64)
    ms = np.mean(x64 * x64, axis=-1, keepdims=True)
    y = x64 / np.sqrt(ms + eps) * np.asarray(w, dtype=np.float64)
    return y.astype(np.float32)


def rmsnorm_fp32(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """The reference's own check written as it is, in fp32 end to end
    (benchmark_rmsnorm.py:115-116: rms = sqrt(mean(X**2, axis=1) + EPS); (X / rms) * W).
    This is the form the CPU baseline times; `rmsnorm` above is the (fp64) checker."""
    x = np.asarray(x, dtype=np.float32)
    rms = np.sqrt(np.mean(x ** 2, axis=-1, keepdims=True) + np.float32(eps))
    return (x / rms) * np.asarray(w, dtype=np.float32)


# --------------------------------------------------------------------------- GEMM
def gemm(a: np.ndarray, b: np.ndarray, c: np.ndarray | None = None) -> np.ndarray:
    """C (+)= A @ B in fp32 (test_gemm_matmul_runtime.py:136,166; ops/gemm.py:144-167)."""
    out = np.asarray(a, dtype=np.float32) @ np.asarray(b, dtype=np.float32)
    if c is not None:
        out = out + np.asarray(c, dtype=np.float32)
    return out.astype(np.float32)


# --------------------------------------------------------------------------- SDPA
def sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, causal: bool = False,
         sinks: np.ndarray | None = None) -> np.ndarray:
    """softmax(scale * Q K^T [+ mask]) V for [B, Hq, Sq, D] / [B, Hkv, Sk, D] inputs.

    Max-subtracted softmax as in showcase_attention.py:150-153; q-head h reads
    kv-head h // (Hq // Hkv) as in benchmark_sdpa.py:198-208.  `sinks` [Hq] (optional)
    are attention-sink logits in the units of scale * q.k that join the denominator only
    (the running max starts at s[h] with l = 1: examples/metal/sdpa_handwritten.metal:39-42,
    benchmark_sdpa.py:64-72).  fp64 internally.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    bsz, hq, sq, d = q.shape
    hk, sk = k.shape[1], k.shape[2]
    g = hq // hk
    out = np.zeros((bsz, hq, sq, d), dtype=np.float64)
    mask = None
    if causal:
        i = np.arange(sq)[:, None]
        j = np.arange(sk)[None, :]
        mask = j > i + (sk - sq)
    for b in range(bsz):
        for h in range(hq):
            s = (q[b, h] @ k[b, h // g].T) * scale
            if mask is not None:
                s = np.where(mask, -np.inf, s)
            m = np.max(s, axis=-1, keepdims=True)
            if sinks is not None:
                m = np.maximum(m, float(sinks[h]))
            m = np.where(np.isfinite(m), m, 0.0)
            p = np.exp(s - m)
            den = p.sum(axis=-1, keepdims=True)
            if sinks is not None:
                den = den + np.exp(float(sinks[h]) - m)
            out[b, h] = np.where(den > 0, (p @ v[b, h // g]) / np.where(den > 0, den, 1.0), 0.0)
    return out.astype(np.float32)


def sdpa_rows(q, k, v, scale, causal, rows):
    """sdpa restricted to the listed (b, h) pairs: a bounded sample for large shapes."""
    q = np.asarray(q)
    hq, hk = q.shape[1], k.shape[1]
    g = hq // hk
    res = []
    for b, h in rows:
        res.append(sdpa(q[b:b + 1, h:h + 1], k[b:b + 1, h // g:h // g + 1],
                        v[b:b + 1, h // g:h // g + 1], scale, causal)[0, 0])
    return np.stack(res)


def sdpa_query_rows(q_rows, k, v, scale, causal, row_idx, sk_minus_sq=0):
    """Exact attention output for selected query rows of one (batch, head).

    q_rows [R, D] are the queries at absolute positions row_idx [R]; k / v [Sk, D] the
    head's keys and values.  Causal masking keeps key j for query i iff j <= i + (Sk - Sq),
    as `sdpa`; the same max-subtracted softmax in fp64.  For full-size checks, where the
    whole score matrix would not fit in host memory."""
    q = np.asarray(q_rows, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    s = (q @ k.T) * scale
    if causal:
        j = np.arange(k.shape[0])[None, :]
        s = np.where(j > np.asarray(row_idx)[:, None] + sk_minus_sq, -np.inf, s)
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    return ((p @ v) / p.sum(axis=1, keepdims=True)).astype(np.float32)


# --------------------------------------------------------------------------- error metrics
def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def rel_fro(a, b) -> float:
    """||a - b||_F / ||b||_F with b the reference."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


# --------------------------------------------------------------------------- decode layer
def rope(t, cos, sin):
    """Half-split rotary embedding over the last axis (rope_np,
    examples/qwen_megakernel.py:313-317): [lo, hi] -> [lo c - hi s, hi c + lo s] with the
    first half of cos / sin applied to lo and the second half to hi.  fp64."""
    t = np.asarray(t, np.float64)
    cos = np.asarray(cos, np.float64)
    sin = np.asarray(sin, np.float64)
    half = t.shape[-1] // 2
    lo, hi = t[..., :half], t[..., half:]
    return np.concatenate([lo * cos[:half] - hi * sin[:half],
                           hi * cos[half:] + lo * sin[half:]], axis=-1)


def decode_layer(x, w, k_cache, v_cache, cos, sin, position, heads_q, heads_kv, head_dim,
                 eps, q_norm=None, k_norm=None):
    """One decode step, restating full_decode_np (examples/qwen_megakernel.py:320-342)
    for a batch, bf16 weights given as fp32 arrays.

    x [B, H]; k_cache / v_cache [B, Hkv, cap, D] with `position` valid entries (the new
    k, v are placed at `position`, the caches are not modified); cos / sin [D].
    q_norm / k_norm [D] (optional) apply the Qwen3 per-head RMSNorm before RoPE
    (qwen_megakernel.py:325-326); the BASELINE layer omits it (None).
    Returns (out [B, H], q_rot, k_new, v_new).  fp64 internally.
    """
    x = np.asarray(x, np.float64)
    f = {k: np.asarray(v, np.float64) for k, v in w.items()}
    B, H = x.shape
    D, G = head_dim, heads_q // heads_kv

    def rms(v, wt):
        return v / np.sqrt(np.mean(v * v, axis=-1, keepdims=True) + eps) * wt

    def head_norm(t, wt):
        return t if wt is None else rms(t, np.asarray(wt, np.float64))

    xn = rms(x, f["w_in_norm"])
    qkv = xn @ f["w_qkv"]
    q = rope(head_norm(qkv[:, :heads_q * D].reshape(B, heads_q, D), q_norm), cos, sin)
    k = rope(head_norm(qkv[:, heads_q * D:(heads_q + heads_kv) * D].reshape(B, heads_kv, D),
                       k_norm), cos, sin)
    v = qkv[:, (heads_q + heads_kv) * D:].reshape(B, heads_kv, D)
    kc = np.asarray(k_cache[:, :, :position], np.float64)
    vc = np.asarray(v_cache[:, :, :position], np.float64)
    K = np.concatenate([kc, k[:, :, None]], axis=2)          # [B, Hkv, L, D]
    V = np.concatenate([vc, v[:, :, None]], axis=2)
    attn = np.empty((B, heads_q, D))
    for h in range(heads_q):
        s = np.einsum("bd,bld->bl", q[:, h], K[:, h // G]) / np.sqrt(D)
        p = np.exp(s - s.max(axis=1, keepdims=True))
        attn[:, h] = np.einsum("bl,bld->bd", p / p.sum(axis=1, keepdims=True), V[:, h // G])
    h1 = x + attn.reshape(B, heads_q * D) @ f["w_o"]
    gu = rms(h1, f["w_post_norm"]) @ f["w_gate_up"]
    inter = gu.shape[1] // 2
    g, u = gu[:, :inter], gu[:, inter:]
    out = h1 + (g / (1 + np.exp(-g)) * u) @ f["w_down"]
    return out.astype(np.float32), q.astype(np.float32), k.astype(np.float32), v.astype(np.float32)


def qwen_decode_f32(x, w_norm, Wq, Wk, Wv, w_q_norm, w_k_norm, cos_p, sin_p, k_cache, v_cache,
                    Wo, w_post, Wg, Wu, Wd, heads_q, heads_kv, eps):
    """full_decode_np of examples/qwen_megakernel.py:320-342 for caches that already
    hold the new k / v (the reference's host pre-fills them, :358-364).  fp64."""
    f = lambda a: np.asarray(a, np.float64)  # noqa: E731
    x, Wq, Wk, Wv, Wo, Wg, Wu, Wd = map(f, (x, Wq, Wk, Wv, Wo, Wg, Wu, Wd))
    D = f(w_q_norm).shape[0]
    half = D // 2

    def rms(v, w):
        return v / np.sqrt(np.mean(v * v, axis=-1, keepdims=True) + eps) * f(w)

    def rope(t):
        lo, hi = t[..., :half], t[..., half:]
        c, s = f(cos_p), f(sin_p)
        return np.concatenate([lo * c[:half] - hi * s[:half], hi * c[half:] + lo * s[half:]], -1)

    n1 = rms(x, w_norm)
    q = rope(rms((Wq @ n1).reshape(heads_q, D), w_q_norm))
    kc, vc = f(k_cache), f(v_cache)
    g = heads_q // heads_kv
    attn = np.empty((heads_q, D))
    for h in range(heads_q):
        sc = kc[h // g] @ q[h] / np.sqrt(D)
        p = np.exp(sc - sc.max())
        attn[h] = (p / p.sum()) @ vc[h // g]
    o = Wo @ attn.ravel() + x
    post = rms(o, w_post)
    gate, up = Wg @ post, Wu @ post
    return (Wd @ (gate / (1 + np.exp(-gate)) * up) + o).astype(np.float32)
