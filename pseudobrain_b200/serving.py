"""The serving twins of the exact memory on B200: drop-ins for pb27_vllm/memory.py's
``retrieve_blocks`` (:760-878) and ``piece_attention`` (:1311-1490).

The serving archive holds one request's keys/values ``[KV, cap, D]`` (no batch dim) with
blocks of ``MEMORY["block_size"]`` tokens starting after the ``ORIGIN`` sink positions
(memory.py:37-46), and per-block key bounds ``kmax``/``kmin`` ``[KV, cap // block, D]``.
Any object with those attributes (and ``prompt_len``, ``hole_lo``, ``hole_hi``, optional
``smax`` and ``dirty_lo``/``dirty_hi``) can be passed, the reference's ``Archive``
included; dirty bounds are refreshed with this package's bounds kernel.

Covered: flat block scoring, the two-level super-block selection (:802-839, super-block
bounds refreshed with the block bounds, :280-306), the archive hole (:769-777), block
neighbours (:873-875), the exact rerank of the ``rerank`` best candidates (:854-872), the
budget rules (:779-787), the query's RoPE-dims mask for scoring past ROPE_HORIZON
(:795-797), and the attention over [sinks ; retrieved blocks ; partial block before the
window ; masked window] (the SDPA branch, own=None; the reference's LSE-merge branch
computes the same softmax). Not covered (they raise NotImplementedError): the ORACLE
diagnostic, per-token selection and own-block masks, global landmarks, and the RoPE
repositioning of keys past ROPE_HORIZON (:574-711) in the rerank and the attention.

Kernels: pbk_quest_select (scores + top-k), pbk_quest_select_levels, pbk_quest_rerank,
pbk_quest_superbounds, pbk_quest_attend_sinks (libpbk.so, sm_100a); head dim 128.
"""
from __future__ import annotations

import torch

from . import _capi
from ._capi import LIB, check
from .exact_memory import (_attend_desc, _workspace, page_bounds_, rerank_pages, select_pages, select_pages_levels,
                           super_bounds_)

# memory.py:33-34 defaults (window: PB27_WINDOW, 16384)
MEMORY: dict = {"enabled": True, "blocks": 256, "block_size": 64, "decode_blocks": 256, "neighbors": 0,
                "rerank": 512, "chunk": 64, "window": 16384}
SINKS = 4                                   # memory.py:37
ORIGIN = SINKS                              # memory.py:46 (FAITHFUL)
SCALE = [2048, 384, 4096, 512, 8192, 1024]  # memory.py:49
ROPE_HORIZON = 262144                       # memory.py:50
SBLK = 64                                   # memory.py:79


def _refresh(arc, block: int) -> None:
    """Recompute the bounds of blocks [dirty_lo, dirty_hi] and of the super-blocks holding
    them (memory.py:280-306, 399-430)."""
    lo, hi = getattr(arc, "dirty_lo", 1 << 60), getattr(arc, "dirty_hi", -1)
    if hi < lo:
        return
    size = min(arc.keys.shape[1], getattr(arc, "size", arc.keys.shape[1]))
    # written keys after the sinks, up to the end of block dirty_hi and of the bounds array
    n = min(size - ORIGIN, (hi + 1) * block, arc.kmax.shape[1] * block)
    if n > 0 and lo * block < n:
        page_bounds_(arc.keys[:, ORIGIN:ORIGIN + n], block, arc.kmax, arc.kmin, first_page=lo)
    smax, smin = getattr(arc, "smax", None), getattr(arc, "smin", None)
    if smax is not None and smin is not None and size > ORIGIN:
        n_blk = min(arc.kmax.shape[1], (size - ORIGIN + block - 1) // block)
        sb0 = max(0, lo // SBLK)
        sb1 = min(smax.shape[1] - 1, min(hi, max(0, n_blk - 1)) // SBLK)
        if sb1 >= sb0:
            super_bounds_(arc.kmax, arc.kmin, n_blk, SBLK, smax, smin, sb0, sb1 + 1)
    arc.dirty_lo, arc.dirty_hi = 1 << 60, -1


def budget_for(full: int, rerank: bool, prompt_len: int, limit: int, budget: int = 0) -> int:
    """Blocks to keep (memory.py:779-787)."""
    if not budget:
        budget = MEMORY["decode_blocks"] if (rerank and MEMORY["decode_blocks"]) else MEMORY["blocks"]
    in_prompt_mid = not rerank and limit + MEMORY["window"] < prompt_len
    if not in_prompt_mid:
        n_arch = max(full, (prompt_len - MEMORY["window"] - ORIGIN) // MEMORY["block_size"])
        for thresh, blocks in zip(SCALE[0::2], SCALE[1::2]):
            if n_arch > thresh:
                budget = max(budget, blocks)
    return budget


def retrieve_blocks(arc, q: torch.Tensor, groups: int, limit: int, rerank: bool, budget: int = 0):
    """Top blocks among archived positions [ORIGIN, limit) for query piece q [T, H, D]:
    [KV, k] int64 block indices, ascending, or None (memory.py:760)."""
    block = MEMORY["block_size"]
    full = (limit - ORIGIN) // block
    if full <= 0:
        return None
    n_valid, hb0, hb1 = full, 0, 0
    hole_lo, hole_hi = getattr(arc, "hole_lo", 0), getattr(arc, "hole_hi", 0)
    if hole_hi > hole_lo:  # memory.py:769-777
        hb0 = max(0, hole_lo - ORIGIN) // block
        hb1 = min(full, (hole_hi - ORIGIN + block - 1) // block)
        if hb1 > hb0:
            n_valid = full - (hb1 - hb0)
        if n_valid <= 0:
            return None
    hole = (hb0, hb1) if hb1 > hb0 else (0, 0)
    t, h, d = q.shape
    k = min(budget_for(full, rerank, arc.prompt_len, limit, budget), n_valid)
    pool = max(MEMORY["rerank"], 2 * k) if MEMORY["rerank"] > 0 else 0
    if limit > ROPE_HORIZON and rerank and pool > k:
        raise NotImplementedError("RoPE repositioning of reranked keys past ROPE_HORIZON (memory.py:861-862)")
    _refresh(arc, block)
    qi = q.to(torch.bfloat16).unsqueeze(0)                        # [1, T, H, D]
    if limit > ROPE_HORIZON:  # memory.py:795-797: the RoPE'd dims do not score
        qi = qi.clone()
        qi[..., : d // 4] = 0
    kmax, kmin = arc.kmax[:, :full], arc.kmin[:, :full]
    smax, smin = getattr(arc, "smax", None), getattr(arc, "smin", None)

    def select(kk: int) -> torch.Tensor:
        if hole != (0, 0):
            return select_pages_levels(qi, kmax, kmin, full * block, block, kk, hole=hole)
        return select_pages(qi, kmax, kmin, full * block, block, kk)

    if not rerank and SBLK > 1 and smax is not None and smin is not None and full > SBLK * 16:
        pages = select_pages_levels(qi, kmax, kmin, full * block, block, k, smax, smin, SBLK, hole)
    elif rerank and pool > k:
        cand = select(min(pool, n_valid))                         # [1, KV, c] ascending
        pages = rerank_pages(qi, arc.keys[:, ORIGIN:], cand, block, k)
    else:
        pages = select(k)
    top = pages[0].long()
    if MEMORY["neighbors"]:  # memory.py:873-875
        top = torch.cat([top] + [(top + j).clamp(max=full - 1) for j in range(1, MEMORY["neighbors"] + 1)], dim=-1)
        top = top.sort(-1).values
    return top


def piece_attention(arc, q: torch.Tensor, q_pos: torch.Tensor, top: torch.Tensor | None, groups: int,
                    window: int, scale: float, own: torch.Tensor | None = None, q_min: int | None = None,
                    q_max: int | None = None) -> torch.Tensor:
    """Exact attention of piece q [T, H, D] at positions q_pos over its sinks, retrieved
    blocks `top` [KV, k], the partial block before its window and its causal sliding
    window, all read from the archive: [T, H, D] in q's dtype (memory.py:1311)."""
    if own is not None:
        raise NotImplementedError("per-token own-block masks (memory.py:1009-1294)")
    if getattr(arc, "is_global_agg", False):
        raise NotImplementedError("global super-block landmarks")
    block = MEMORY["block_size"]
    t, h, d = q.shape
    if q_min is None or q_max is None:
        q_min, q_max = int(q_pos.min()), int(q_pos.max())
    lo, hi = max(0, q_min - window + 1), q_max + 1
    if lo > ROPE_HORIZON:
        raise NotImplementedError("RoPE repositioning past ROPE_HORIZON (memory.py:574-711)")
    ns = min(SINKS, lo)
    qi = q.to(torch.bfloat16).unsqueeze(0)
    out = torch.empty(1, t, h, d, dtype=torch.float32, device=q.device)
    qpos = q_pos.to(device=q.device, dtype=torch.int32).view(1, t)
    kpos = torch.arange(lo, hi, dtype=torch.int32, device=q.device)
    win = (arc.keys[:, lo:hi], arc.values[:, lo:hi], kpos, window, 0, scale, out)
    if top is not None:  # retrieved blocks + the partial block before the window
        desc = _attend_desc(qi, qpos, arc.keys[:, ORIGIN:], arc.values[:, ORIGIN:], max(0, lo - ORIGIN), block,
                            top.to(torch.int32).unsqueeze(0).contiguous(), *win)
    else:  # sinks and window only: no archive part
        dummy = torch.zeros(1, h // groups, 1, dtype=torch.int32, device=q.device)
        desc = _attend_desc(qi, qpos, arc.keys, arc.values, block, block, dummy, *win)
        desc.n_arch, desc.budget = 0, 0
    ws = _workspace(LIB.pbk_quest_attend_sinks_workspace(desc, ns), q.device)
    with torch.cuda.device(q.device):
        check(LIB.pbk_quest_attend_sinks(desc, arc.keys.data_ptr(), arc.values.data_ptr(), ns, arc.keys.stride(0),
                                         arc.keys.stride(1), ws.data_ptr(), ws.numel(),
                                         torch.cuda.current_stream(q.device).cuda_stream),
              "pbk_quest_attend_sinks")
    return out[0].to(q.dtype)
