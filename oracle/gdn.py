"""Gated delta rule, restated in numpy. TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Layouts follow the reference's PyTorch core (pseudobrain/gated_deltanet.py:72-75):
q, k [B,T,H,K]; v [B,T,H,V]; g, beta [B,T,H] (g <= 0 is the log decay);
h0 [B,H,K,V]. Both functions return (o [B,T,H,V], final state [B,H,K,V]) in fp32
(fp64 when q is fp64), like the reference.

The reference's caller expands q and k from the key heads to the value heads with
``repeat_interleave`` (gated_deltanet.py:422-424): value head j reads key head
j // (Hv // Hk). ``expand_key_heads`` restates that map, so the oracle can be fed
the GQA-native tensors the CUDA kernels take.
"""
from __future__ import annotations

import numpy as np

CHUNK = 64  # pseudobrain/gated_deltanet.py:48


def _compute_dtype(x: np.ndarray):
    """fp32 arithmetic, fp64 for fp64 inputs (gated_deltanet.py:78-80)."""
    return np.float64 if x.dtype == np.float64 else np.float32


def expand_key_heads(x: np.ndarray, value_heads: int) -> np.ndarray:
    """[B,T,Hk,K] -> [B,T,Hv,K], value head j <- key head j // (Hv // Hk)
    (the repeat_interleave of gated_deltanet.py:422-424)."""
    hk = x.shape[2]
    if value_heads % hk:
        raise ValueError("value heads must be a multiple of key heads")
    return np.repeat(x, value_heads // hk, axis=2)


def delta_rule_sequential(q, k, v, g, beta, scale, h0):
    """Per-step recurrence, gated_deltanet.py:93-107.

    S <- exp(g_t) S;  u = (v_t - S^T k_t) beta_t;  S <- S + k_t u^T;  o_t = S^T (scale q_t).
    """
    dt = _compute_dtype(q)
    state = np.array(h0, dtype=dt, copy=True)
    q = q.astype(dt) * dt(scale)
    k, v = k.astype(dt), v.astype(dt)
    decay, beta = np.exp(g.astype(dt)), beta.astype(dt)
    batch, length, heads, _ = q.shape
    out = np.empty((batch, length, heads, v.shape[-1]), dtype=dt)
    for t in range(length):
        state *= decay[:, t, :, None, None]
        kt = k[:, t]
        u = (v[:, t] - np.einsum("bhkv,bhk->bhv", state, kt)) * beta[:, t, :, None]
        state += kt[..., None] * u[..., None, :]
        out[:, t] = np.einsum("bhkv,bhk->bhv", state, q[:, t])
    return out, state


def _unit_lower_inverse(a: np.ndarray) -> np.ndarray:
    """(I + A)^-1 for strictly lower-triangular A [..., C, C] by forward substitution.

    The reference uses torch.linalg.solve_triangular(I + A, I, unitriangular=True)
    (gated_deltanet.py:147-150); row i of the inverse is e_i - A[i, :i] @ T[:i, :].
    """
    size = a.shape[-1]
    t = np.zeros_like(a)
    idx = np.arange(size)
    t[..., idx, idx] = 1.0
    for i in range(1, size):
        t[..., i, :i] -= np.einsum("...j,...jc->...c", a[..., i, :i], t[..., :i, :i])
    return t


def delta_rule_chunked(q, k, v, g, beta, scale, h0, chunk: int | None = None):
    """Chunkwise WY gated delta rule, gated_deltanet.py:110-165.

    Per chunk of C steps with cumulative log decay c (gamma = exp(c)):
      D_ti = exp(c_t - c_i) for i <= t;  A = strict_lower(beta_t k_t.k_i D_ti);  T = (I + A)^-1
      W = T (K * beta gamma);  U' = T (V * beta);  then chunk by chunk
      U = U' - W S;  O = (Q gamma) S + (Q K^T * D) U;  S = gamma_C S + (exp(c_C - c_i) k_i)^T U.
    The time axis is padded to a multiple of C with identity steps (k = v = 0, g = 0,
    beta = 0), as the reference does (:126-136).
    """
    batch, length, heads, dk = q.shape
    dv = v.shape[-1]
    size = min(CHUNK if chunk is None else chunk, length)
    pad = (-length) % size
    dt = _compute_dtype(q)
    # [B,H,T,*] (gated_deltanet.py:129-133); q is scaled before chunking.
    qh = np.ascontiguousarray(q.astype(dt).transpose(0, 2, 1, 3)) * dt(scale)
    kh = np.ascontiguousarray(k.astype(dt).transpose(0, 2, 1, 3))
    vh = np.ascontiguousarray(v.astype(dt).transpose(0, 2, 1, 3))
    gh = np.ascontiguousarray(g.astype(dt).transpose(0, 2, 1))
    bh = np.ascontiguousarray(beta.astype(dt).transpose(0, 2, 1))
    if pad:
        qh, kh, vh = (np.pad(x, ((0, 0), (0, 0), (0, pad), (0, 0))) for x in (qh, kh, vh))
        gh, bh = (np.pad(x, ((0, 0), (0, 0), (0, pad))) for x in (gh, bh))
    count = (length + pad) // size
    qh = qh.reshape(batch, heads, count, size, dk)
    kh = kh.reshape(batch, heads, count, size, dk)
    vh = vh.reshape(batch, heads, count, size, dv)
    c = np.cumsum(gh.reshape(batch, heads, count, size), axis=-1, dtype=dt)
    bh = bh.reshape(batch, heads, count, size)
    inclusive = np.tril(np.ones((size, size), dtype=bool))
    strict = np.tril(inclusive, -1)
    with np.errstate(over="ignore"):
        diff = c[..., :, None] - c[..., None, :]
    decay = np.where(inclusive, np.exp(np.where(inclusive, diff, 0.0)), 0.0).astype(dt)
    kk = kh @ kh.swapaxes(-1, -2)
    a = np.where(strict, bh[..., :, None] * kk * decay, 0.0).astype(dt)
    solve = _unit_lower_inverse(a)
    gamma = np.exp(c)
    w = solve @ (kh * (bh * gamma)[..., None])
    u0 = solve @ (vh * bh[..., None])
    qk = (qh @ kh.swapaxes(-1, -2)) * decay
    qg = qh * gamma[..., None]
    tail = np.exp(c[..., -1:] - c)[..., None] * kh
    last = gamma[..., -1]
    state = np.array(h0, dtype=dt, copy=True)
    out = np.empty((batch, heads, count, size, dv), dtype=dt)
    for n in range(count):
        u = u0[:, :, n] - w[:, :, n] @ state
        out[:, :, n] = qg[:, :, n] @ state + qk[:, :, n] @ u
        state = state * last[:, :, n, None, None] + tail[:, :, n].swapaxes(-1, -2) @ u
    o = out.reshape(batch, heads, count * size, dv)[:, :, :length]
    return np.ascontiguousarray(o.transpose(0, 2, 1, 3)), state


def chunk_aux(k, g, beta, chunk: int = CHUNK):
    """The chunk quantities the reference's fla op returns beside (o, state)
    (pseudobrain::gated_delta_chunk, gated_deltanet.py:200-216): gc [B,T,H], the cumulative g
    within each chunk of ``chunk`` steps, and a [B,T,H,chunk], row t of its chunk's
    T = (I + A)^-1 with A_ti = beta_t k_t.k_i exp(c_t - c_i) (i < t) -- the reference's
    `solve` (gated_deltanet.py:141-150), chunks of the fixed fla size with identity padding."""
    batch, length, heads, dk = k.shape
    pad = (-length) % chunk
    dt = _compute_dtype(k)
    kh = np.ascontiguousarray(k.astype(dt).transpose(0, 2, 1, 3))
    gh = np.ascontiguousarray(g.astype(dt).transpose(0, 2, 1))
    bh = np.ascontiguousarray(beta.astype(dt).transpose(0, 2, 1))
    if pad:
        kh = np.pad(kh, ((0, 0), (0, 0), (0, pad), (0, 0)))
        gh, bh = (np.pad(x, ((0, 0), (0, 0), (0, pad))) for x in (gh, bh))
    count = (length + pad) // chunk
    kh = kh.reshape(batch, heads, count, chunk, dk)
    c = np.cumsum(gh.reshape(batch, heads, count, chunk), axis=-1, dtype=dt)
    bh = bh.reshape(batch, heads, count, chunk)
    strict = np.tril(np.ones((chunk, chunk), dtype=bool), -1)
    with np.errstate(over="ignore"):
        diff = np.where(strict, c[..., :, None] - c[..., None, :], 0.0)
    a = np.where(strict, bh[..., :, None] * (kh @ kh.swapaxes(-1, -2)) * np.exp(diff), 0.0).astype(dt)
    solve = _unit_lower_inverse(a)
    gc = c.reshape(batch, heads, count * chunk)[:, :, :length].transpose(0, 2, 1)
    ta = solve.reshape(batch, heads, count * chunk, chunk)[:, :, :length].transpose(0, 2, 1, 3)
    return np.ascontiguousarray(gc), np.ascontiguousarray(ta)


def rel_err(x: np.ndarray, ref: np.ndarray) -> float:
    """Norm-wise relative error ||x - ref|| / ||ref|| in fp64 (the parity metric)."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(x - ref) / (den if den > 0 else 1.0))


# ------------------------------------------------------------------------------------------
# The layer pieces around the recurrence (GatedDeltaNetLayer.forward, gated_deltanet.py:411-440)
# ------------------------------------------------------------------------------------------
L2_EPS = 1e-6    # gated_deltanet.py:55
NORM_EPS = 1e-5  # gated_deltanet.py:72


def short_convolution(x, tail, weight):
    """Causal depthwise convolution over time with a carried input tail, then SiLU
    (gated_deltanet.py:314-338). x [B,T,C]; tail [B,K-1,C]; weight [C,K] (weight[:, -1]
    multiplies the current input) or None. fp32. Returns (y [B,T,C], new tail [B,K-1,C])."""
    x = x.astype(np.float32)
    if weight is None:
        return x / (1.0 + np.exp(-x)), tail
    size = weight.shape[1]
    length = x.shape[1]
    ext = np.concatenate((tail.astype(np.float32), x), axis=1) if size > 1 else x
    new_tail = ext[:, ext.shape[1] - (size - 1):] if size > 1 else tail
    w = weight.astype(np.float32)
    y = ext[:, :length] * w[:, 0]
    for j in range(1, size):
        y = y + ext[:, j:j + length] * w[:, j]
    return (y / (1.0 + np.exp(-y))).astype(np.float32), new_tail


def l2_normalize(x, mode="max", eps=L2_EPS):
    """q/k normalisation over the last dim (gated_deltanet.py:59-70): 'max' is
    x / max(||x||, eps) (F.normalize), 'hf' is x * rsqrt(sum x^2 + eps), in fp32."""
    xf = x.astype(np.float32)
    ss = np.sum(xf * xf, axis=-1, keepdims=True)
    if mode == "max":
        return xf / np.maximum(np.sqrt(ss), eps)
    if mode == "hf":
        return xf / np.sqrt(ss + eps)
    raise ValueError(mode)


def gating(a, b, a_log, dt_bias):
    """g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) (gated_deltanet.py:427-429);
    softplus with F.softplus's threshold of 20. fp32."""
    x = a.astype(np.float32) + dt_bias.astype(np.float32)
    sp = np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))
    g = -np.exp(a_log.astype(np.float32)) * sp
    beta = 1.0 / (1.0 + np.exp(-b.astype(np.float32)))
    return g.astype(np.float32), beta.astype(np.float32)


def gated_out_norm(o, gate, weight, eps=NORM_EPS):
    """o * rsqrt(mean(o^2) + eps) * weight * SiLU(gate) over the value dim
    (gated_deltanet.py:439-440). o, gate [B,T,H,V]; weight [V]. fp32."""
    o = o.astype(np.float32)
    gt = gate.astype(np.float32)
    y = o / np.sqrt(np.mean(o * o, axis=-1, keepdims=True) + eps)
    return (y * weight.astype(np.float32) * (gt / (1.0 + np.exp(-gt)))).astype(np.float32)
