"""Quest page-bounded exact memory, restated in numpy. TEST INFRASTRUCTURE ONLY.

Follows pseudobrain/exact_memory.py (the flat mode in ``retrieve``; the two-level
super-block selection, the exact rerank, ``prompt_top`` and ``neighbors`` in
``retrieve_modes``) and the exact attention of its caller
pseudobrain/transplant.py:612-628. Layouts: keys/values [B,KV,N,D], page bounds
[B,KV,P,D], queries [B,H,T,D] with H = KV * groups (head h reads key head
h // groups).

Scores are computed the way the reference's CPU path computes them: q cast to
fp32, split into its positive and negative parts, two fp32 products against the
page maxima and minima, then the maximum over the G*T query rows that share a key
head (exact_memory.py:94-98,124-125). The ``canonical_*`` functions sum the same
exact products in a fixed order (dimension 0..127, fp32): the order every selection
kernel of this build selects on, so they pin its page indices bit for bit, where the
GEMM-order scores agree only up to near-ties. Page selection keeps the ``budget`` highest
scores with ties going to the lowest page index (the tie rule of this build; the
reference's ``torch.topk`` leaves it unspecified) and returns them in position
order (exact_memory.py:135,144).
"""
from __future__ import annotations

import numpy as np


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even) and return it as fp32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 values that are exact bf16 -> their uint16 bit patterns."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> fp32."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def page_bounds(keys: np.ndarray, page: int) -> tuple[np.ndarray, np.ndarray]:
    """Elementwise max and min of every page of ``page`` keys, exact_memory.py:43-50.

    A trailing partial page is padded with its own last key, so its bounds are those
    of the keys it holds."""
    b, h, n, d = keys.shape
    pad = (-n) % page
    if pad:
        keys = np.concatenate((keys, np.broadcast_to(keys[:, :, -1:], (b, h, pad, d))), axis=2)
    blocks = keys.reshape(b, h, -1, page, d)
    return blocks.max(axis=3), blocks.min(axis=3)


class Archive:
    """Evicted keys/values [B,KV,N,D] and per-page bounds [B,KV,P,D] (exact_memory.py:27-40)."""

    def __init__(self, keys, values, kmax, kmin):
        self.keys, self.values, self.kmax, self.kmin = keys, values, kmax, kmin

    @property
    def length(self) -> int:
        return self.keys.shape[2]


def archive_append(archive: Archive | None, keys, values, page: int) -> Archive | None:
    """Append evicted keys/values and redo the bounds from the first incomplete page on,
    exact_memory.py:66-85 (complete pages are final)."""
    if keys.shape[2] == 0:
        return archive
    if archive is None:
        kmax, kmin = page_bounds(keys, page)
        return Archive(keys, values, kmax, kmin)
    full = (archive.length // page) * page
    new_k = np.concatenate((archive.keys, keys), axis=2)
    new_v = np.concatenate((archive.values, values), axis=2)
    tmax, tmin = page_bounds(new_k[:, :, full:], page)
    kmax = np.concatenate((archive.kmax[:, :, : full // page], tmax), axis=2)
    kmin = np.concatenate((archive.kmin[:, :, : full // page], tmin), axis=2)
    return Archive(new_k, new_v, kmax, kmin)


def page_scores(q: np.ndarray, kmax: np.ndarray, kmin: np.ndarray, groups: int) -> np.ndarray:
    """Upper bound of every page's attention logit, max over the G*T query rows of a key
    head: sum_d max(q_d, 0) kmax_d + min(q_d, 0) kmin_d (exact_memory.py:94-98,124-125).

    q [B,H,T,D]; kmax, kmin [B,KV,P,D] (complete pages only) -> [B,KV,P] fp32."""
    b, h, t, d = q.shape
    kv = h // groups
    qg = q.astype(np.float32).reshape(b, kv, groups * t, d)
    pos, neg = np.maximum(qg, 0), np.minimum(qg, 0)
    bound = pos @ kmax.astype(np.float32).swapaxes(-1, -2) + neg @ kmin.astype(np.float32).swapaxes(-1, -2)
    return bound.max(axis=2).astype(np.float32)


def select_pages(score: np.ndarray, budget: int) -> np.ndarray:
    """The min(budget, P) highest-scoring pages of every row, ties to the lowest index,
    returned in ascending page order (exact_memory.py:135,144). [..., P] -> [..., k] int64."""
    p = score.shape[-1]
    k = min(budget, p)
    order = np.argsort(-score.astype(np.float64), axis=-1, kind="stable")[..., :k]
    return np.sort(order, axis=-1).astype(np.int64)


def retrieve(archive: Archive | None, q: np.ndarray, groups: int, page: int, budget: int):
    """Flat Quest retrieval, exact_memory.py:88-152 with superblock=0, rerank=0,
    neighbors=0: score complete pages, keep the top ``budget``, gather them in position
    order and append the partial tail. Returns (keys, values, pages) or None."""
    if archive is None or archive.length == 0:
        return None
    b, h, t, d = q.shape
    kv = h // groups
    full = archive.length // page
    tail = archive.length - full * page
    parts_k, parts_v = [], []
    top = np.zeros((b, kv, 0), dtype=np.int64)
    if full:
        score = page_scores(q, archive.kmax[:, :, :full], archive.kmin[:, :, :full], groups)
        top = select_pages(score, budget)
        idx = (top[..., None] * page + np.arange(page)).reshape(b, kv, -1)
        parts_k.append(np.take_along_axis(archive.keys, idx[..., None], axis=2))
        parts_v.append(np.take_along_axis(archive.values, idx[..., None], axis=2))
    if tail:
        parts_k.append(archive.keys[:, :, full * page:])
        parts_v.append(archive.values[:, :, full * page:])
    return np.concatenate(parts_k, axis=2), np.concatenate(parts_v, axis=2), top


def super_bounds(kmax: np.ndarray, kmin: np.ndarray, sblk: int) -> tuple[np.ndarray, np.ndarray]:
    """Super-block bounds, exact_memory.py:53-63: the max of ``sblk`` consecutive page
    maxima and the min of their minima; a trailing partial super-block is padded with its
    last page, so it takes the bounds of the pages it holds. [..., P, D] -> [..., ceil(P/sblk), D]."""
    p, d = kmax.shape[-2:]
    pad = (-p) % sblk
    if pad:
        kmax = np.concatenate((kmax, np.repeat(kmax[..., -1:, :], pad, axis=-2)), axis=-2)
        kmin = np.concatenate((kmin, np.repeat(kmin[..., -1:, :], pad, axis=-2)), axis=-2)
    shape = kmax.shape[:-2] + (-1, sblk, d)
    return kmax.reshape(shape).max(axis=-2), kmin.reshape(shape).min(axis=-2)


def _bound_scores(qg: np.ndarray, bmax: np.ndarray, bmin: np.ndarray) -> np.ndarray:
    """max over rows r of sum_d max(q_rd,0) bmax_pd + min(q_rd,0) bmin_pd: qg [..., R, D],
    bmax/bmin [..., P, D] -> [..., P] (fp64 sums of the exact fp32 products)."""
    q = qg.astype(np.float64)
    pos, neg = np.maximum(q, 0), np.minimum(q, 0)
    return (pos @ bmax.astype(np.float64).swapaxes(-1, -2) + neg @ bmin.astype(np.float64).swapaxes(-1, -2)).max(-2)


def canonical_bound_scores(qg: np.ndarray, bmax: np.ndarray, bmin: np.ndarray) -> np.ndarray:
    """The bound scores in this build's canonical order, bit for bit what every selection kernel
    selects on: for each query row, an fp32 sum over d = 0..127 in order of the exact fp32
    products t_d = q_d * (kmax_d if q_d > 0 else kmin_d), then the max over rows.

    The reference sums the same products in its GEMM's order (exact_memory.py:97-98,124-125),
    which no other implementation reproduces; near-ties may resolve either way there. Fixing
    the order makes the selection a function of the inputs alone. qg [..., R, D] query rows of
    each key head; bmax/bmin [..., P, D] -> [..., P] fp32."""
    q = np.asarray(qg, dtype=np.float32)
    bx = np.moveaxis(np.asarray(bmax, dtype=np.float32), -1, 0)  # [D, ..., P]
    bn = np.moveaxis(np.asarray(bmin, dtype=np.float32), -1, 0)
    acc = np.zeros(q.shape[:-1] + (bx.shape[-1],), np.float32)   # [..., R, P]
    for d in range(q.shape[-1]):
        qd = q[..., d][..., None]
        acc += qd * np.where(qd > 0, bx[d][..., None, :], bn[d][..., None, :])  # exact product, fp32 add
    return acc.max(axis=-2)


def canonical_page_scores(q: np.ndarray, kmax: np.ndarray, kmin: np.ndarray, groups: int) -> np.ndarray:
    """page_scores in the canonical order (canonical_bound_scores). q [B,H,T,D] -> [B,KV,P]."""
    b, h, t, d = q.shape
    return canonical_bound_scores(q.reshape(b, h // groups, groups * t, d), kmax, kmin)


def canonical_key_scores(qg: np.ndarray, ck: np.ndarray) -> np.ndarray:
    """The exact rerank score in the canonical order: for candidate c, the max over the head's
    query rows and the candidate's keys of an fp32 sum over d = 0..127 in order of q_d * k_d
    (each product exact). qg [..., R, D], ck [..., c, S, D] -> [..., c] fp32."""
    q = np.asarray(qg, dtype=np.float32)
    c, s_, d_ = ck.shape[-3:]
    kf = np.asarray(ck, dtype=np.float32).reshape(ck.shape[:-3] + (c * s_, d_))
    acc = np.zeros(q.shape[:-1] + (c * s_,), np.float32)
    for d in range(q.shape[-1]):
        acc += q[..., d][..., None] * kf[..., d][..., None, :]
    return acc.max(axis=-2).reshape(ck.shape[:-3] + (c, s_)).max(axis=-1)


def canonical_rerank_scores(qg: np.ndarray, keys: np.ndarray, cand: np.ndarray, page: int) -> np.ndarray:
    """canonical_key_scores of the candidate pages' keys. qg [..., R, D], keys [..., N, D],
    cand [..., c] -> [..., c] fp32."""
    idx = (cand[..., :, None] * page + np.arange(page)).reshape(cand.shape[:-1] + (-1,))
    ck = np.take_along_axis(np.asarray(keys, dtype=np.float32), idx[..., None], axis=-2)  # [..., c*page, D]
    return canonical_key_scores(qg, ck.reshape(cand.shape + (page, ck.shape[-1])))


def _topk_lowest(score: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest entries of each row (ties to the lowest index), ascending."""
    order = np.argsort(-score.astype(np.float64), axis=-1, kind="stable")[..., :k]
    return np.sort(order, axis=-1)


def select_two_level(qg: np.ndarray, kmax: np.ndarray, kmin: np.ndarray, smax: np.ndarray, smin: np.ndarray,
                     full: int, k: int, sblk: int, hole: tuple[int, int] = (0, 0), canonical: bool = False) -> np.ndarray:
    """Two-level Quest selection, exact_memory.py:107-122 (pb27_vllm/memory.py:802-836 with its
    archive hole): score the ceil(full/sblk) super-blocks on smax/smin, keep
    m_sb = min(max(16, ceil(2k/sblk)), n_sb) of them, score their pages (pages at or past
    ``full`` and pages in [hole) score -inf; indices clamp to full-1) and keep the best
    min(k, m_sb*sblk). qg [..., R, D] query rows of each key head; bounds [..., P, D].
    Ties go to the lowest index at both levels. Returns [..., k'] page indices, ascending.
    canonical: score in the canonical order (canonical_bound_scores) at both levels."""
    score_fn = canonical_bound_scores if canonical else _bound_scores
    n_sb = (full + sblk - 1) // sblk
    sb_score = score_fn(qg, smax[..., :n_sb, :], smin[..., :n_sb, :])
    m_sb = min(max(16, (2 * k + sblk - 1) // sblk), n_sb)
    top_sb = _topk_lowest(sb_score, m_sb)                                    # ascending
    raw = (top_sb[..., :, None] * sblk + np.arange(sblk)).reshape(top_sb.shape[:-1] + (m_sb * sblk,))
    idx = np.minimum(raw, full - 1)
    bmax = np.take_along_axis(kmax[..., :full, :], idx[..., None], axis=-2)
    bmin = np.take_along_axis(kmin[..., :full, :], idx[..., None], axis=-2)
    sub = score_fn(qg, bmax, bmin)
    invalid = (raw >= full) | ((idx >= hole[0]) & (idx < hole[1]))
    sub = np.where(invalid, -np.inf, sub)
    keep = _topk_lowest(sub, min(k, m_sb * sblk))
    return np.take_along_axis(idx, keep, axis=-1)


def rerank_pages(qg: np.ndarray, keys: np.ndarray, cand: np.ndarray, page: int, k: int,
                 canonical: bool = False) -> np.ndarray:
    """Exact rerank, exact_memory.py:126-133: candidate page c scores the max over the head's
    query rows and the page's tokens of q.k; keep the best k (ties to the lowest candidate
    position). qg [..., R, D], keys [..., N, D], cand [..., c] ascending -> [..., k] ascending.
    canonical: q.k summed in the canonical order (canonical_rerank_scores)."""
    if canonical:
        return np.take_along_axis(cand, _topk_lowest(canonical_rerank_scores(qg, keys, cand, page), k), axis=-1)
    idx = (cand[..., :, None] * page + np.arange(page)).reshape(cand.shape[:-1] + (-1,))
    ck = np.take_along_axis(keys, idx[..., None], axis=-2).astype(np.float64)
    exact = (qg.astype(np.float64) @ ck.swapaxes(-1, -2)).max(-2).reshape(cand.shape + (page,)).max(-1)
    return np.take_along_axis(cand, _topk_lowest(exact, k), axis=-1)


def retrieve_modes(keys, values, kmax, kmin, q, groups: int, page: int, budget: int, superblock: int = 0,
                   rerank: int = 0, neighbors: int = 0, prompt_top=None, canonical: bool = False):
    """retrieve, exact_memory.py:88-152, with its other modes: the two-level super-block
    selection for decode queries (t <= 64, rerank <= k, superblock > 1, full > 16 superblock;
    :107-122), the exact rerank of the best ``rerank`` pages (:126-133), a prompt selection
    prepended to a decode selection (:138-140) and ``neighbors`` following pages (:141-143).
    keys/values [B,KV,N,D], bounds [B,KV,P,D], q [B,H,T,D]. Returns (keys, values, top).
    canonical: every score in the canonical order (canonical_bound_scores)."""
    b, h, t, d = q.shape
    kv = h // groups
    n = keys.shape[2]
    full, tail = n // page, n % page
    qg = q.astype(np.float32).reshape(b, kv, groups * t, d)
    parts_k, parts_v = [], []
    top = np.zeros((b, kv, 0), dtype=np.int64)
    if full:
        k = min(budget, full)
        if t <= 64 and rerank <= k and superblock > 1 and full > superblock * 16:
            smax, smin = super_bounds(kmax, kmin, superblock)
            top = select_two_level(qg, kmax, kmin, smax, smin, full, k, superblock, canonical=canonical)
        else:
            score = (canonical_bound_scores if canonical else _bound_scores)(qg, kmax[:, :, :full], kmin[:, :, :full])
            if rerank > k:
                cand = _topk_lowest(score, min(rerank, full))
                top = rerank_pages(qg, keys, cand, page, k, canonical=canonical)
            else:
                top = _topk_lowest(score, k)
        if t <= 64 and prompt_top is not None:
            top = np.concatenate((np.minimum(prompt_top, full - 1), top), axis=-1)
        if neighbors:
            top = np.concatenate([top] + [np.minimum(top + j, full - 1) for j in range(1, neighbors + 1)], axis=-1)
        top = np.sort(top, axis=-1)
        idx = (top[..., None] * page + np.arange(page)).reshape(b, kv, -1)
        parts_k.append(np.take_along_axis(keys, idx[..., None], axis=2))
        parts_v.append(np.take_along_axis(values, idx[..., None], axis=2))
    if tail:
        parts_k.append(keys[:, :, full * page:])
        parts_v.append(values[:, :, full * page:])
    return np.concatenate(parts_k, axis=2), np.concatenate(parts_v, axis=2), top.astype(np.int64)


def window_mask(qpos: np.ndarray, kpos: np.ndarray, window: int, sinks: int) -> np.ndarray:
    """Causal sliding-window visibility of cached keys, transplant.py:621-622:
    kpos <= qpos and (qpos - kpos < window or kpos < sinks). -> [T, S] bool."""
    q_, k_ = qpos[:, None], kpos[None, :]
    return (k_ <= q_) & (((q_ - k_) < window) | (k_ < sinks))


def attend(q, rk, rv, wk, wv, qpos, kpos, window: int, sinks: int, groups: int) -> np.ndarray:
    """Exact softmax attention over [retrieved ; window] keys, transplant.py:619-628.

    q [B,H,T,D]; rk, rv [B,KV,R,D] (all visible); wk, wv [B,KV,S,D] with positions kpos [S];
    queries at positions qpos [T]. Scale 1/sqrt(D) (SDPA's default). Computed in fp64,
    returned as fp32 [B,H,T,D]."""
    b, h, t, d = q.shape
    mask = np.concatenate((np.ones((t, rk.shape[2]), dtype=bool),
                           window_mask(qpos, kpos, window, sinks)), axis=1)
    kk = np.concatenate((rk, wk), axis=2).astype(np.float64)
    vv = np.concatenate((rv, wv), axis=2).astype(np.float64)
    kk = np.repeat(kk, groups, axis=1)
    vv = np.repeat(vv, groups, axis=1)
    logits = (q.astype(np.float64) @ kk.swapaxes(-1, -2)) / np.sqrt(d)
    logits = np.where(mask, logits, -np.inf)
    logits -= logits.max(axis=-1, keepdims=True)
    p = np.exp(logits)
    p /= p.sum(axis=-1, keepdims=True)
    return (p @ vv).astype(np.float32)
