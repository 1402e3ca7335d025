"""vLLM's Gated DeltaNet decode ops, restated in numpy. TEST INFRASTRUCTURE ONLY (see
oracle/__init__.py).

The served PB-27 model's decode runs through vLLM's GDN layer; these restate the
three ops vLLM 0.22 calls for it, from their Triton sources (paths under
vllm/model_executor/layers/fla/ops/):

* ``packed_decode``  -- fused_recurrent_gated_delta_rule_packed_decode, fused_recurrent.py:256-336
  (q | k | v packed in one row per token, gating and the q/k norm in the kernel, the state
  pool updated in place; a null slot (index <= 0) writes a zero output);
* ``sigmoid_gating_update`` -- fused_sigmoid_gating_delta_rule_update, fused_sigmoid_gating.py:24-180
  (variable-length sequences, speculative decoding with 2-D state indices and
  num_accepted_tokens);
* ``recurrent`` -- fused_recurrent_gated_delta_rule, fused_recurrent.py:20-170 (g and beta given).

All three run the recurrence of pseudobrain/gated_deltanet.py:93-107 in the [V, K] pool
layout: h <- exp(g) h; v' = (v - h k) beta; h <- h + v' k^T; o = h q. Computed in float64 on
the given values. Pools are [slots, HV, V, K].
"""
from __future__ import annotations

import numpy as np


def _softplus(x, sb, thr):
    """fused_sigmoid_gating.py: log(1 + exp(sb x)) / sb while sb x <= threshold, else x."""
    return np.where(sb * x <= thr, np.log1p(np.exp(np.minimum(sb * x, thr))) / sb, x)


def gating(a, b, a_log, dt_bias, sb=1.0, thr=20.0, beta_round=None):
    """g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) (rounded by beta_round, a
    function, when given: the packed decode rounds it to b's dtype). a, b [..., HV]."""
    x = a.astype(np.float64) + dt_bias.astype(np.float64)
    g = -np.exp(a_log.astype(np.float64)) * _softplus(x, sb, thr)
    beta = 1.0 / (1.0 + np.exp(-b.astype(np.float64)))
    if beta_round is not None:
        beta = beta_round(beta.astype(np.float32)).astype(np.float64)
    return g, beta


def _norm(x, mode, eps=1e-6):
    if mode == 0:
        return x
    ss = (x * x).sum(-1, keepdims=True) + eps
    return x / np.sqrt(ss) if mode == 1 else x * (1.0 / np.sqrt(ss))


def _step(h, q, k, v, g, beta, scale, l2):
    """One token for all value heads of one sequence: h [HV, V, K], q/k [HV, K] (already
    expanded), v [HV, V]. Returns (o [HV, V], h)."""
    q = _norm(q, l2) * scale
    k = _norm(k, l2)
    h = h * np.exp(g)[:, None, None]
    u = (v - np.einsum("hvk,hk->hv", h, k)) * beta[:, None]
    h = h + u[:, :, None] * k[:, None, :]
    return np.einsum("hvk,hk->hv", h, q), h


def recurrent(q, k, v, g, beta, scale, pool, cu_seqlens=None, indices=None, num_accepted=None, l2=0,
              null_le_zero=True):
    """fused_recurrent_gated_delta_rule (inplace_final_state) and, with g and beta from
    ``gating``, fused_sigmoid_gating_delta_rule_update. q, k [B, T, H, K] (or [1, rows, ...]
    with cu_seqlens), v [.., HV, V], g, beta [.., HV]. indices [N] or [N, cols] (speculative:
    the initial state from column num_accepted - 1, the state after token t to column t).
    Returns (o [.., HV, V] with NaN rows for skipped sequences, new pool)."""
    pool = pool.astype(np.float64).copy()
    hv, h_ = v.shape[2], q.shape[2]
    rep = hv // h_
    qf, kf = np.repeat(q.astype(np.float64), rep, 2), np.repeat(k.astype(np.float64), rep, 2)
    vf, gf, bf = v.astype(np.float64), g.astype(np.float64), beta.astype(np.float64)
    o = np.full(v.shape, np.nan)
    if cu_seqlens is None:
        spans = [(n, 0, q.shape[1]) for n in range(q.shape[0])]
    else:
        spans = [(0, int(cu_seqlens[n]), int(cu_seqlens[n + 1]) - int(cu_seqlens[n])) for n in range(len(cu_seqlens) - 1)]
    null = (lambda s: s <= 0) if null_le_zero else (lambda s: s < 0)
    for n, (bsel, r0, tn) in enumerate(spans):
        if tn == 0:
            continue
        two_d = indices is not None and indices.ndim == 2
        if indices is None:
            slot = n
        elif two_d:
            slot = int(indices[n, (int(num_accepted[n]) - 1) if num_accepted is not None else 0])
        else:
            slot = int(indices[n])
        if indices is not None and null(slot):
            continue
        h = pool[slot].copy()
        for t in range(tn):
            r = r0 + t
            out, h = _step(h, qf[bsel, r], kf[bsel, r], vf[bsel, r], gf[bsel, r], bf[bsel, r], scale, l2)
            o[bsel, r] = out
            if two_d:
                st = int(indices[n, t])
                if not null(st):
                    pool[st] = h
        if not two_d:
            pool[slot] = h
    return o, pool


def packed_decode(mixed, a, b, a_log, dt_bias, scale, pool, indices, k_dim, hv, v_dim, l2=1, beta_round=None):
    """fused_recurrent_gated_delta_rule_packed_decode: mixed [N, 2 H K + HV V] (q | k | v),
    a, b [N, HV]; one token per row; indices [N] (<= 0: null, zero output). Returns
    (o [N, 1, HV, V], new pool)."""
    n_tok = mixed.shape[0]
    h_ = (mixed.shape[1] - hv * v_dim) // (2 * k_dim)
    q = mixed[:, : h_ * k_dim].reshape(n_tok, 1, h_, k_dim)
    k = mixed[:, h_ * k_dim: 2 * h_ * k_dim].reshape(n_tok, 1, h_, k_dim)
    v = mixed[:, 2 * h_ * k_dim:].reshape(n_tok, 1, hv, v_dim)
    g, beta = gating(a, b, a_log, dt_bias, beta_round=beta_round)
    o, pool = recurrent(q, k, v, g[:, None], beta[:, None], scale, pool, indices=indices, l2=l2)
    o = np.where(np.isnan(o), 0.0, o)
    return o, pool
