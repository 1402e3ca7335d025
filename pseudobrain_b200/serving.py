"""The serving twins of the exact memory on B200: drop-ins for pb27_vllm/memory.py's
``retrieve_blocks`` (:760-878) and ``piece_attention`` (:1311-1490).

The serving archive holds one request's keys/values ``[KV, cap, D]`` (no batch dim) with
blocks of ``MEMORY["block_size"]`` tokens starting after the ``ORIGIN`` sink positions
(memory.py:37-46), and per-block key bounds ``kmax``/``kmin`` ``[KV, cap // block, D]``.
Any object with those attributes (and ``prompt_len``, ``hole_lo``, ``hole_hi``, optional
``smax`` and ``dirty_lo``/``dirty_hi``) can be passed, the reference's ``Archive``
included; dirty bounds are refreshed with this package's bounds kernel.

Covered: flat block scoring, the exact rerank of the ``rerank`` best candidates
(memory.py:854-872), the budget rules (:779-787), and the attention over [sinks ;
retrieved blocks ; partial block before the window ; masked window] (the SDPA branch,
own=None; the reference's LSE-merge branch computes the same softmax). Not covered (they
raise NotImplementedError): super-block selection (:800-840), archive holes, block
neighbours, the ORACLE diagnostic, per-token selection and own-block masks, global
landmarks, and contexts past ROPE_HORIZON where RoPE repositioning applies (:574-711).

Kernels: pbk_quest_select (scores + top-k), pbk_quest_rerank, pbk_quest_attend_sinks
(libpbk.so, sm_100a); head dim 128.
"""
from __future__ import annotations

import torch

from . import _capi
from ._capi import LIB, check
from .exact_memory import _attend_desc, _desc, _workspace, page_bounds_, select_pages

# memory.py:33-34 defaults (window: PB27_WINDOW, 16384)
MEMORY: dict = {"enabled": True, "blocks": 256, "block_size": 64, "decode_blocks": 256, "neighbors": 0,
                "rerank": 512, "chunk": 64, "window": 16384}
SINKS = 4                                   # memory.py:37
ORIGIN = SINKS                              # memory.py:46 (FAITHFUL)
SCALE = [2048, 384, 4096, 512, 8192, 1024]  # memory.py:49
ROPE_HORIZON = 262144                       # memory.py:50
SBLK = 64                                   # memory.py:79


def _refresh(arc, block: int) -> None:
    """Recompute the bounds of blocks [dirty_lo, dirty_hi] (memory.py:399-430)."""
    lo, hi = getattr(arc, "dirty_lo", 1 << 60), getattr(arc, "dirty_hi", -1)
    if hi < lo:
        return
    # written keys after the sinks, up to the end of block dirty_hi and of the bounds array
    n = min(arc.keys.shape[1], getattr(arc, "size", arc.keys.shape[1])) - ORIGIN
    n = min(n, (hi + 1) * block, arc.kmax.shape[1] * block)
    if n > 0 and lo * block < n:
        page_bounds_(arc.keys[:, ORIGIN:ORIGIN + n], block, arc.kmax, arc.kmin, first_page=lo)
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
    if MEMORY["neighbors"]:
        raise NotImplementedError("block neighbours (memory.py:873-875)")
    if getattr(arc, "hole_hi", 0) > getattr(arc, "hole_lo", 0):
        raise NotImplementedError("archive holes (memory.py:769-777)")
    if limit > ROPE_HORIZON:
        raise NotImplementedError("RoPE repositioning past ROPE_HORIZON (memory.py:798-800, 861-862)")
    if not rerank and SBLK > 1 and getattr(arc, "smax", None) is not None and full > SBLK * 16:
        raise NotImplementedError("super-block selection (memory.py:802-840)")
    _refresh(arc, block)
    t, h, d = q.shape
    kv = h // groups
    k = min(budget_for(full, rerank, arc.prompt_len, limit, budget), full)
    qi = q.to(torch.bfloat16).unsqueeze(0)                        # [1, T, H, D]
    kmax, kmin = arc.kmax[:, :full], arc.kmin[:, :full]
    pool = max(MEMORY["rerank"], 2 * k) if MEMORY["rerank"] > 0 else 0
    if rerank and pool > k:
        c = min(pool, full)
        cand = select_pages(qi, kmax, kmin, full * block, block, c)   # [1, KV, c] ascending
        pages = torch.empty(1, kv, k, dtype=torch.int32, device=q.device)
        keys = arc.keys[:, ORIGIN:]
        desc = _desc(qi, block, full * block, k, keys=keys, values=arc.values[:, ORIGIN:], pages=pages)
        ws = _workspace(LIB.pbk_quest_rerank_workspace(desc, c), q.device)
        with torch.cuda.device(q.device):
            check(LIB.pbk_quest_rerank(desc, cand.data_ptr(), c, ws.data_ptr(), ws.numel(),
                                       torch.cuda.current_stream(q.device).cuda_stream), "pbk_quest_rerank")
    else:
        pages = select_pages(qi, kmax, kmin, full * block, block, k)
    return pages[0].long()


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
