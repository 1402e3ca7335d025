"""The serving twins of the exact memory (pb27_vllm/memory.py), restated in numpy.
TEST INFRASTRUCTURE ONLY.

Follows serving/pb27_vllm/pb27_vllm/memory.py:
* ``retrieve_blocks`` (:760-878): bound scores of the full blocks of an
  archive [KV, cap, D] whose blocks start after ORIGIN sink positions (:764, :845-853),
  ``topk(k)`` (:877) or, with ``rerank``, the ``rerank_pool`` best blocks by bound
  rescored exactly (max over query rows and block tokens of q.k, :854-872), then sorted;
  the two-level super-block selection (:802-839), the archive hole (:769-777) and block
  neighbours (:873-875).
  Budget: decode_blocks when reranking, else blocks (:779-780); the SCALE thresholds
  (:781-787) only raise it for archives of more than 2048 blocks.
* ``piece_attention`` (:1311-1490), SDPA branch with own=None: keys are the sinks
  [0, ns), the retrieved blocks, the partial block [tail0, lo) and the window [lo, hi)
  with the causal sliding-window mask (:1433-1490); RoPE repositioning is a no-op while
  lo <= ROPE_HORIZON (:583, :628).
Ties in the top-k go to the lowest block index (torch.topk leaves them unspecified).
"""
from __future__ import annotations

import numpy as np

ORIGIN = 4        # memory.py:46 (FAITHFUL, SINKS = 4)
SINKS = 4         # memory.py:37
SCALE = [2048, 384, 4096, 512, 8192, 1024]  # memory.py:49


def _topk_sorted(score: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest entries of each row, ties to the lowest index, ascending."""
    order = np.lexsort((np.arange(score.shape[-1])[None].repeat(score.shape[0], 0), -score), axis=-1)
    return np.sort(order[:, :k], axis=-1)


def budget(memory: dict, full: int, rerank: bool, prompt_len: int, limit: int) -> int:
    """memory.py:779-787."""
    b = memory["decode_blocks"] if (rerank and memory["decode_blocks"]) else memory["blocks"]
    in_prompt_mid = not rerank and limit + memory["window"] < prompt_len
    if not in_prompt_mid:
        n_arch = max(full, (prompt_len - memory["window"] - ORIGIN) // memory["block_size"])
        for thresh, blocks in zip(SCALE[0::2], SCALE[1::2]):
            if n_arch > thresh:
                b = max(b, blocks)
    return b


def super_bounds(kmax, kmin, n_blk: int, sblk: int):
    """Archive._update_superbounds (memory.py:280-306) over blocks [0, n_blk): super-block s
    takes the max of the maxima and the min of the minima of blocks [s sblk, min(n_blk,
    (s+1) sblk))."""
    n_sb = (n_blk + sblk - 1) // sblk
    smax = np.stack([kmax[:, s * sblk:min(n_blk, (s + 1) * sblk)].max(1) for s in range(n_sb)], axis=1)
    smin = np.stack([kmin[:, s * sblk:min(n_blk, (s + 1) * sblk)].min(1) for s in range(n_sb)], axis=1)
    return smax, smin


def retrieve_blocks(keys, kmax, kmin, q, groups, limit, rerank, memory, prompt_len, smax=None, smin=None, sblk=0,
                    hole=(0, 0)):
    """keys [KV, cap, D]; kmax/kmin [KV, n_blk, D]; q [T, H, D] -> [KV, k] block indices or None.

    With smax/smin [KV, n_sb, D] and sblk > 1, a call without rerank over more than 16 sblk
    full blocks takes the two-level selection (memory.py:802-839). ``hole`` = (hole_lo,
    hole_hi) archive positions whose blocks score -inf (memory.py:769-777, 834-835, 852-853);
    memory["neighbors"] adds the following blocks (:873-875)."""
    from .quest import select_two_level
    block = memory["block_size"]
    full = (limit - ORIGIN) // block
    if full <= 0:
        return None
    t, h, d = q.shape
    kv = h // groups
    n_valid, hb0, hb1 = full, 0, 0
    if hole[1] > hole[0]:
        hb0 = max(0, hole[0] - ORIGIN) // block
        hb1 = min(full, (hole[1] - ORIGIN + block - 1) // block)
        if hb1 > hb0:
            n_valid = full - (hb1 - hb0)
        if n_valid <= 0:
            return None
    k = min(budget(memory, full, rerank, prompt_len, limit), n_valid)
    qg = np.asarray(q, np.float64).transpose(1, 0, 2).reshape(kv, groups * t, d)   # [KV, G*T, D]
    nb = memory.get("neighbors", 0)

    def with_neighbors(top):
        if nb:
            top = np.concatenate([top] + [np.minimum(top + j, full - 1) for j in range(1, nb + 1)], axis=-1)
        return np.sort(top, axis=-1)

    if not rerank and sblk > 1 and smax is not None and full > sblk * 16:
        return with_neighbors(select_two_level(qg, kmax, kmin, smax, smin, full, k, sblk, (hb0, hb1)))
    pos, neg = np.maximum(qg, 0), np.minimum(qg, 0)
    score = (np.einsum("grd,gnd->grn", pos, kmax[:, :full].astype(np.float64))
             + np.einsum("grd,gnd->grn", neg, kmin[:, :full].astype(np.float64))).max(1)      # [KV, full]
    score[:, hb0:hb1] = -np.inf
    pool = max(memory["rerank"], 2 * k) if memory["rerank"] > 0 else 0
    if rerank and pool > k:
        c = min(pool, n_valid)
        cand = _topk_sorted(score, c)                                                   # [KV, c] ascending
        blk = keys[:, ORIGIN:ORIGIN + full * block].reshape(kv, full, block, d).astype(np.float64)
        ck = np.take_along_axis(blk, cand[:, :, None, None], axis=1)                    # [KV, c, block, D]
        exact = np.einsum("grd,gcsd->grcs", qg, ck).max(axis=(1, 3))                   # [KV, c]
        keep = _topk_sorted(exact, k)
        return with_neighbors(np.take_along_axis(cand, keep, axis=1))
    return with_neighbors(_topk_sorted(score, k))


def piece_attention(keys, values, q, q_pos, top, groups, window, scale, block):
    """q [T, H, D] at positions q_pos -> [T, H, D] float64 (SDPA branch, own=None)."""
    t, h, d = q.shape
    kv = h // groups
    q_min, q_max = int(q_pos.min()), int(q_pos.max())
    lo, hi = max(0, q_min - window + 1), q_max + 1
    ns = min(SINKS, lo)
    tail0 = ORIGIN + ((lo - ORIGIN) // block) * block
    out = np.zeros((t, h, d))
    for g in range(kv):
        parts_k, parts_v, vis = [], [], []
        idx = list(range(ns))
        if top is not None:
            for b in top[g]:
                idx += list(range(ORIGIN + b * block, ORIGIN + (b + 1) * block))
            if lo > tail0:
                idx += list(range(tail0, lo))
        always = len(idx)
        idx += list(range(lo, hi))
        kk, vv = keys[g, idx].astype(np.float64), values[g, idx].astype(np.float64)
        wpos = np.arange(lo, hi)
        for j in range(groups):
            hq = g * groups + j
            sc = q[:, hq].astype(np.float64) @ kk.T * scale                              # [T, N]
            mask = np.ones_like(sc, dtype=bool)
            mask[:, always:] = (wpos[None, :] <= q_pos[:, None]) & (wpos[None, :] >= q_pos[:, None] - window + 1)
            sc = np.where(mask, sc, -np.inf)
            sc -= sc.max(-1, keepdims=True)
            p = np.exp(sc)
            p /= p.sum(-1, keepdims=True)
            out[:, hq] = p @ vv
    return out
