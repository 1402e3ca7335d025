"""Causal sliding-window attention with sinks, restated in numpy. TEST INFRASTRUCTURE ONLY.

Follows pseudobrain/transplant.py:417-436 (``causal_attention``) and its exact chunked
form :346-362 (``_chunked_window_attention``): q [B,H,T,hd], k/v [B,KV,T,hd] with
query head j reading key head j // (H // KV) (the repeat_interleave of :426-429);
query t sees key s when

    s <= t  and  (window is None  or  t - s < window  or  s < sinks),

softmax(q.k * hd**-0.5) over the visible keys (SDPA's default scale), times V.
Computed in float64 on the given values, in query chunks so memory stays
O(chunk * (window + chunk)).
"""
from __future__ import annotations

import numpy as np


def visible(qpos: np.ndarray, kpos: np.ndarray, window: int | None, sinks: int) -> np.ndarray:
    """[len(qpos), len(kpos)] mask of transplant.py:356-357 / :432-433."""
    qp, kp = qpos[:, None], kpos[None, :]
    m = kp <= qp
    if window is not None:
        m &= ((qp - kp) < window) | (kp < sinks)
    return m


def _rows(q64, k64, v64, rows, window, sinks):
    """[B,H,len(rows),hd] attention of the consecutive query positions `rows`."""
    h, g = q64.shape[1], q64.shape[1] // k64.shape[1]
    s, e = int(rows[0]), int(rows[-1]) + 1
    lo = 0 if window is None else max(0, s - window + 1)
    keys = np.concatenate((np.arange(min(sinks, lo)), np.arange(lo, e)))
    mask = visible(np.arange(s, e), keys, window, sinks)
    scale = q64.shape[-1] ** -0.5
    out = np.zeros((q64.shape[0], h, e - s, q64.shape[-1]), np.float64)
    for j in range(h):
        kk, vv = k64[:, j // g][:, keys], v64[:, j // g][:, keys]       # [B, S, d]
        sc = np.einsum("btd,bsd->bts", q64[:, j, s:e], kk) * scale
        sc = np.where(mask[None], sc, -np.inf)
        sc -= sc.max(-1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(-1, keepdims=True)
        out[:, j] = np.einsum("bts,bsd->btd", p, vv)
    return out


def causal_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, window: int | None = None, sinks: int = 0,
                     chunk: int = 256) -> np.ndarray:
    """[B,H,T,hd] float64 output of transplant.py:417-436."""
    q64, k64, v64 = (np.asarray(x, np.float64) for x in (q, k, v))
    out = np.zeros(q64.shape, np.float64)
    t = q64.shape[2]
    for s in range(0, t, chunk):
        out[:, :, s:s + chunk] = _rows(q64, k64, v64, np.arange(s, min(t, s + chunk)), window, sinks)
    return out


def causal_attention_at(q: np.ndarray, k: np.ndarray, v: np.ndarray, starts, length: int,
                        window: int | None = None, sinks: int = 0) -> dict:
    """Outputs of the query runs [s, s + length) for s in `starts` only (for long sequences
    whose full oracle would take too long): {s: [B,H,length,hd] float64}."""
    q64, k64, v64 = (np.asarray(x, np.float64) for x in (q, k, v))
    return {s: _rows(q64, k64, v64, np.arange(s, s + length), window, sinks) for s in starts}
