"""The serving path's per-token selector on B200: pb27_vllm/memory.py's
``retrieve_blocks_per_token`` (:1009-1294), the block selection the served model runs by
default (PERTOKEN, :65), with the helpers it calls (_ranks :881, _dedup_priority :888,
_expand_successors_dedup :900, _second_hop_blocks :914, _detect_global_agg :963,
_stratified_superblock_peaks :981, _record_block_visits :995).

Every query token scores the blocks over its own query heads; the scores are standardised
per token (z-scores, raw and relative to the piece's mean), ranked, and combined into tier
keys; the candidates of each ranking are interleaved in priority order with first-occurrence
dedup; in the prefill branch the candidates are rescored exactly per token and ranked again,
and a key-to-key "second hop" adds blocks that resemble the best ones; successors follow
each kept block; a decode step merges its blocks with the prompt's and the previous step's.

Data-parallel parts on this package's kernels (libpbk.so, sm_100a):
  * per-token block scores over the block or super-block bounds, with the candidate lists,
    the archive hole and the RoPE-dims mask in the kernel (pbk_quest_token_scores);
  * the exact per-token rescoring of the candidates (pbk_quest_token_rerank);
  * every rank (pbk_quest_row_ranks: a bitonic sort per row in shared memory, ties in index
    order).
The bookkeeping around them (z-score arithmetic over [KV, T, blocks], tier keys, the
priority interleaving and dedup over [KV, <= 4c] index arrays, the second hop's two plain
GEMMs over the unrotated key dims) runs as tensor operations on the same device.

The reference's ranking uses torch's argsort/topk, whose order among exactly equal values is
unspecified; here ties go to the lower index. Scores are fp32 sums over the dims in order
(the reference's CPU path adds its two bound products after summing each).
"""
from __future__ import annotations

import ctypes
import os

import torch
import torch.nn.functional as F

from . import serving
from ._capi import LIB, PbkTokenDesc, check

# memory.py:65-85 (the same environment switches)
PERTOKEN_CAND = int(os.environ.get("PB27_MEMORY_PERTOKEN_CAND", "4") or 4)
DECODE_STRIDE = int(os.environ.get("PB27_MEMORY_DECODE_STRIDE", "64") or 64)
DECODE_BLOCKS = int(os.environ.get("PB27_MEMORY_DECODE_BLOCKS", "64") or 64)
DECODE_RERANK = os.environ.get("PB27_MEMORY_DECODE_RERANK", "0") == "1"
GLOBAL_AGG = os.environ.get("PB27_MEMORY_GLOBAL_AGG", "auto").strip().lower()
GLOBAL_DECODE_STRIDE = int(os.environ.get("PB27_MEMORY_GLOBAL_DECODE_STRIDE", "16") or 16)
NOVELTY_ALPHA = float(os.environ.get("PB27_MEMORY_NOVELTY_ALPHA", "0.75") or 0.75)


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("the per-token selector runs on CUDA tensors only (no CPU fallback)")


# ------------------------------------------------------------------ kernels
def token_scores(q: torch.Tensor, kmax: torch.Tensor, kmin: torch.Tensor, full: int, n_pool: int,
                 cand: torch.Tensor | None = None, hole: tuple[int, int] = (0, 0), rope_mask: bool = False,
                 kv: int | None = None) -> torch.Tensor:
    """[KV, T, n_pool] fp32: candidate j of key head h (block cand[h, j], or j) scored for
    each query token t of q [T, H, 128] as the max over the head's query heads of the bound
    score; -inf outside [0, full) and inside the hole (memory.py:1079-1098)."""
    _require_cuda(q, kmax, kmin)
    t, h, d = q.shape
    kv = kmax.shape[0] if kv is None else kv
    qb = q.to(torch.bfloat16)
    if qb.stride(-1) != 1:
        qb = qb.contiguous()
    out = torch.empty(kv, t, n_pool, dtype=torch.float32, device=q.device)
    if t == 0 or n_pool == 0:
        return out
    if kmax.dtype != torch.bfloat16 or kmin.dtype != torch.bfloat16:
        kmax, kmin = kmax.to(torch.bfloat16), kmin.to(torch.bfloat16)
    if cand is not None:
        cand = cand.to(torch.int32).contiguous()
    desc = PbkTokenDesc(t=t, h=h, kv=kv, d=d, n_pool=n_pool, full=full, hole_lo=hole[0], hole_hi=hole[1],
                        rope_mask=int(rope_mask), block=0, q=qb.data_ptr(), q_stride_t=qb.stride(0),
                        q_stride_h=qb.stride(1), kmax=kmax.data_ptr(), kmin=kmin.data_ptr(),
                        bnd_stride_kv=kmax.stride(0), bnd_stride_p=kmax.stride(1),
                        cand=cand.data_ptr() if cand is not None else None,
                        cand_stride_kv=cand.stride(0) if cand is not None else 0, out=out.data_ptr(),
                        out_stride_kv=out.stride(0), out_stride_t=out.stride(1))
    with torch.cuda.device(q.device):
        check(LIB.pbk_quest_token_scores(ctypes.byref(desc), _stream(q)), "pbk_quest_token_scores")
    return out


def token_rerank(q: torch.Tensor, keys: torch.Tensor, block: int, cand: torch.Tensor | None, n_pool: int,
                 kv: int | None = None) -> torch.Tensor:
    """[KV, T, n_pool] fp32: the exact score of candidate block cand[h, j] (or j) of keys
    [KV, rows, 128] for each query token: max over the head's query heads and the block's
    tokens of q . k (memory.py:1192-1202)."""
    _require_cuda(q, keys)
    t, h, d = q.shape
    kv = keys.shape[0] if kv is None else kv
    qb = q.to(torch.bfloat16)
    if qb.stride(-1) != 1:
        qb = qb.contiguous()
    out = torch.empty(kv, t, n_pool, dtype=torch.float32, device=q.device)
    if t == 0 or n_pool == 0:
        return out
    if cand is not None:
        cand = cand.to(torch.int32).contiguous()
    desc = PbkTokenDesc(t=t, h=h, kv=kv, d=d, n_pool=n_pool, full=0, block=block, q=qb.data_ptr(),
                        q_stride_t=qb.stride(0), q_stride_h=qb.stride(1), keys=keys.data_ptr(),
                        key_stride_kv=keys.stride(0), key_stride_n=keys.stride(1),
                        cand=cand.data_ptr() if cand is not None else None,
                        cand_stride_kv=cand.stride(0) if cand is not None else 0, out=out.data_ptr(),
                        out_stride_kv=out.stride(0), out_stride_t=out.stride(1))
    with torch.cuda.device(q.device):
        check(LIB.pbk_quest_token_rerank(ctypes.byref(desc), _stream(q)), "pbk_quest_token_rerank")
    return out


def ranks(x: torch.Tensor) -> torch.Tensor:
    """Rank (0 = largest) of every entry along the last axis, ties in index order
    (_ranks, memory.py:881-885): int64, x's shape."""
    _require_cuda(x)
    n = x.shape[-1]
    rows = x.reshape(-1, n).float().contiguous()
    out = torch.empty(rows.shape, dtype=torch.int32, device=x.device)
    if rows.numel():
        with torch.cuda.device(x.device):
            check(LIB.pbk_quest_row_ranks(rows.data_ptr(), rows.stride(0), rows.shape[0], n, out.data_ptr(),
                                          out.stride(0), _stream(x)), "pbk_quest_row_ranks")
    return out.view(x.shape).long()


# ------------------------------------------------------------------ selection bookkeeping
def first_k(r: torch.Tensor, k: int) -> torch.Tensor:
    """Indices of the k smallest keys of each row, smallest first (ties in index order)."""
    return torch.sort(r, dim=-1, stable=True).indices[..., :k]


def top_k(x: torch.Tensor, k: int) -> torch.Tensor:
    """Indices of the k largest values of each row, largest first (ties in index order)."""
    return torch.sort(x, dim=-1, descending=True, stable=True).indices[..., :k]


def dedup_priority(seq: torch.Tensor, u: int) -> torch.Tensor:
    """The first min(u, M) entries of each row of seq [KV, M] (block indices >= 0) in
    priority order after moving every repeat of an earlier value behind all first
    occurrences (_dedup_priority, memory.py:888-897)."""
    kv, m = seq.shape
    pos = torch.arange(m, device=seq.device)
    by_value = torch.argsort(seq.long() * m + pos, dim=-1)           # value-major, position-minor
    sv = seq.gather(-1, by_value)
    rep_sorted = torch.zeros_like(sv, dtype=torch.bool)
    rep_sorted[:, 1:] = sv[:, 1:] == sv[:, :-1]
    repeat = torch.empty_like(rep_sorted).scatter_(-1, by_value, rep_sorted)
    order = torch.argsort(pos + repeat.long() * m, dim=-1)[:, : min(u, m)]
    return seq.gather(-1, order)


def expand_successors_dedup(blk_ord: torch.Tensor, full: int, u: int, m_succ: int = 80):
    """Each of the first m_succ blocks followed by its successor (clamped to full - 1),
    then the rest; the first u unique (memory.py:900-911): (priority order, ascending)."""
    kv, m = blk_ord.shape
    ms = min(m_succ, m)
    head = blk_ord[:, :ms]
    pairs = torch.stack((head, (head + 1).clamp(max=full - 1)), dim=-1).view(kv, 2 * ms)
    seq = torch.cat((pairs, blk_ord[:, ms:]), dim=-1) if ms < m else pairs
    top = dedup_priority(seq, u)
    return top, top.sort(-1).values


def zscores(score: torch.Tensor):
    """(relative, raw) z-scores of per-token scores [KV, T, P] (memory.py:1084-1088): raw
    standardises each token's finite scores over the blocks; relative first subtracts each
    block's mean over the tokens (T > 1). -inf entries count as 0 in the statistics."""
    inf = torch.isinf(score)
    fin = score.masked_fill(inf, 0.0)
    rel = score - fin.mean(1, keepdim=True) if score.shape[1] > 1 else score
    rel_fin = rel.masked_fill(inf, 0.0)
    z_rel = (rel - rel_fin.mean(-1, keepdim=True)) / rel_fin.std(-1, keepdim=True).clamp(min=1e-6)
    z_raw = (score - fin.mean(-1, keepdim=True)) / fin.std(-1, keepdim=True).clamp(min=1e-6)
    return z_rel, z_raw


def gather_blocks(t: torch.Tensor, blocks: torch.Tensor, block: int) -> torch.Tensor:
    """Rows of blocks [KV, B] (block b = rows ORIGIN + b * block ..) of t [KV, cap, D] ->
    [KV, B * block, D] (memory.py:714-722)."""
    kv, cap, d = t.shape
    rows = serving.ORIGIN + blocks.long()[:, :, None] * block + torch.arange(block, device=blocks.device)
    return t.gather(1, rows.reshape(kv, -1, 1).expand(-1, -1, d))


def detect_global_agg(z_raw: torch.Tensor, full: int) -> bool:
    """Dense global aggregation: many blocks score moderately, none stands out
    (memory.py:963-978)."""
    if GLOBAL_AGG in ("0", "false", "off", "no"):
        return False
    if GLOBAL_AGG in ("1", "true", "on", "yes", "force"):
        return True
    if full < 128:
        return False
    z_tail = z_raw[:, -min(z_raw.shape[1], 16):].amax(1)
    z_1d = (z_tail - z_tail.mean(-1, keepdim=True)) / z_tail.std(-1, keepdim=True).clamp(min=1e-6)
    mass = (z_1d - 1.0).clamp(min=0.0)
    l1, l2 = mass.sum(-1), (mass * mass).sum(-1).clamp(min=1e-6)
    n_eff = float((l1 * l1 / l2).mean().item())
    return n_eff > max(64.0, 0.12 * float(full)) and float(z_1d.amax().item()) < 4.5


def stratified_peaks(score_1d: torch.Tensor, full: int, max_sb: int) -> torch.Tensor:
    """The best block of each of n_seg equal segments of [0, full) -> [KV, n_seg]
    (memory.py:981-992)."""
    sblk = serving.SBLK
    n_seg = min(max(1, max_sb), full // max(1, sblk))
    if n_seg <= 1:
        return score_1d.argmax(dim=-1, keepdim=True)
    seg = full // n_seg
    best = score_1d[:, : n_seg * seg].view(score_1d.shape[0], n_seg, seg).argmax(dim=-1)
    return torch.arange(n_seg, device=score_1d.device) * seg + best


def record_block_visits(arc, blk: torch.Tensor, full: int) -> None:
    """Per-block visit counts of the global-aggregation sweep (memory.py:995-1006)."""
    kv, cap_blk = blk.shape[0], arc.kmax.shape[1]
    vc = getattr(arc, "visit_counts", None)
    if vc is None or vc.shape[1] < cap_blk:
        grown = torch.zeros(kv, cap_blk, dtype=torch.int16, device=blk.device)
        if vc is not None:
            grown[:, : vc.shape[1]] = vc
        arc.visit_counts = vc = grown
    b = blk.clamp(min=0, max=cap_blk - 1)
    vc.scatter_add_(1, b, torch.ones_like(b, dtype=torch.int16))


def _interleave(first: torch.Tensor, second: torch.Tensor) -> torch.Tensor:
    """first[0], second[0], first[1], ... over their common length, then first's rest."""
    kv = first.shape[0]
    n = min(first.shape[1], second.shape[1])
    inter = torch.stack((first[:, :n], second[:, :n]), dim=-1).view(kv, 2 * n)
    return torch.cat((inter, first[:, n:]), dim=-1) if n < first.shape[1] else inter


def second_hop_blocks(arc, blk_ord: torch.Tensor, full: int, n_valid: int, block: int, k2: int = 64,
                      c2_cap: int = 512) -> torch.Tensor:
    """Blocks whose keys resemble the keys of the best blocks, over the unrotated dims
    d/4 .. (memory.py:914-960) -> [KV, <= k2]."""
    kv = blk_ord.shape[0]
    d = arc.keys.shape[2]
    d0 = d // 4
    m1 = min(6, blk_ord.shape[1])
    b1 = blk_ord[:, :m1]
    seeds = dedup_priority(torch.stack((b1, (b1 + 1).clamp(max=full - 1)), dim=-1).view(kv, 2 * m1), min(10, full))
    k_seed = gather_blocks(arc.keys, seeds, block).float()[..., d0:]
    kmax_u, kmin_u = arc.kmax[:, :full, d0:].float(), arc.kmin[:, :full, d0:].float()
    k_mean = 0.5 * (kmax_u + kmin_u).mean(1, keepdim=True)
    q2 = F.normalize(k_seed - k_mean, dim=-1)
    s2 = q2.clamp(min=0) @ (kmax_u - k_mean).transpose(-1, -2) + q2.clamp(max=0) @ (kmin_u - k_mean).transpose(-1, -2)
    hole_lo, hole_hi = getattr(arc, "hole_lo", 0), getattr(arc, "hole_hi", 0)
    if hole_hi > hole_lo:
        b0 = max(0, hole_lo - serving.ORIGIN) // block
        b_hi = min(full, (hole_hi - serving.ORIGIN + block - 1) // block)
        if b_hi > b0:
            s2[..., b0:b_hi] = float("-inf")
    inf = torch.isinf(s2)
    rel = s2 - s2.masked_fill(inf, 0.0).mean(1, keepdim=True)
    rel_fin = rel.masked_fill(inf, 0.0)
    z2 = (rel - rel_fin.mean(-1, keepdim=True)) / rel_fin.std(-1, keepdim=True).clamp(min=1e-6)
    c2 = min(c2_cap, n_valid)
    cand2 = top_k(z2.amax(1), c2)
    ck2 = F.normalize(gather_blocks(arc.keys, cand2, block).float()[..., d0:] - k_mean, dim=-1)
    n_q2 = min(128, q2.shape[1])
    q2_top = q2.gather(1, top_k(z2.amax(-1), n_q2).unsqueeze(-1).expand(-1, -1, q2.shape[-1]))
    ex2 = torch.bmm(q2_top, ck2.transpose(-1, -2)).view(kv, n_q2, c2, block).amax(-1)
    ex2_rel = ex2 - ex2.mean(1, keepdim=True)
    ze2 = (ex2_rel - ex2_rel.mean(-1, keepdim=True)) / ex2_rel.std(-1, keepdim=True).clamp(min=1e-6)
    e2_tier = ranks(ex2).amin(1) * c2 + ranks(ex2.amax(1))
    u2 = min(k2, c2)
    inter2 = torch.stack((first_k(ranks(ze2.amax(1)), u2), first_k(e2_tier, u2)), dim=-1).view(kv, 2 * u2)
    return cand2.gather(-1, dedup_priority(inter2, u2))


def _rank_lists(score: torch.Tensor, z_rel: torch.Tensor, z_raw: torch.Tensor, n: int, lead, tail_rule: str):
    """The ranked candidate lists of one stage (memory.py:1091-1108, 1178-1202, 1216-1240):
    tier = (min rank over tokens, rank of the best token's score); with many tokens also
    the last tokens' tier. tail_rule: "prefill" (min rank of the last <= 96 tokens, rank of
    their best score) or "decode" (min rank of the last 8, then of the last <= 16)."""
    t_ev = score.shape[1]
    rk = ranks(score)
    tier = rk.amin(1) * n + ranks(score.amax(1))
    if tail_rule == "prefill" and lead is not None and lead < 0 and t_ev > 36:
        tt = min(t_ev, 96)
        tail = rk[:, -tt:].amin(1) * n + ranks(score[:, -tt:].amax(1))
        return "prefill", tail, ranks(z_rel[:, -tt:].amax(1)), ranks(z_raw[:, -tt:].amax(1)), tier
    if lead == 0 and t_ev > 8:
        td = min(t_ev, 16)
        tail = rk[:, -8:].amin(1) * n + rk[:, -td:].amin(1)
        return "decode", tail, ranks(z_rel[:, -td:].amax(1)), ranks(z_raw[:, -td:].amax(1)), tier
    return "short", None, ranks(z_rel.amax(1)), ranks(z_raw.amax(1)), tier


def _novelty(arc, z_rel, z_raw, full):
    vc_pen = NOVELTY_ALPHA * torch.log1p(arc.visit_counts[:, :full].float()).unsqueeze(1)
    return z_rel - vc_pen, z_raw - vc_pen


def _reset_decode_state(arc) -> None:
    arc.decode_step = 0
    arc.last_hop_head = None
    arc.cached_top = arc.cached_rk = arc.cached_rv = None
    arc.cached_pre_k = arc.cached_pre_v = None
    arc.cached_ns = -1
    if getattr(arc, "visit_counts", None) is not None:
        arc.visit_counts.zero_()


def retrieve_blocks_per_token(arc, q: torch.Tensor, groups: int, limit: int, budget: int = 0,
                              lead: int | None = None, union: int = 0, q_hist: torch.Tensor | None = None):
    """Blocks for query piece q [T, H, D] among archived positions [ORIGIN, limit): (top
    [KV, k] int64 ascending, None) or None (memory.py:1009). lead: 0 a decode piece, < 0 a
    prompt piece (resets the decode state and keeps the prompt's blocks), None neither.
    q_hist: the recent decode queries [T', H, D] (the last row is replaced by q[:1])."""
    block = serving.MEMORY["block_size"]
    origin = serving.ORIGIN
    full = (limit - origin) // block
    if full <= 0:
        return None
    _require_cuda(q, arc.kmax)
    for name, default in (("decode_step", 0), ("cached_top", None), ("last_hop_head", None),
                          ("visit_counts", None), ("is_global_agg", False), ("decode_top", None),
                          ("prompt_top", None), ("last_prio_rank", None), ("last_top", None), ("last_rk", None)):
        if not hasattr(arc, name):
            setattr(arc, name, default)
    stride = GLOBAL_DECODE_STRIDE if arc.is_global_agg else DECODE_STRIDE
    if lead == 0 and q.shape[0] <= serving.MEMORY["chunk"]:
        arc.decode_step += 1
        if stride > 1 and arc.cached_top is not None and arc.decode_step % stride != 0:
            return arc.cached_top, None
    elif lead is not None and lead < 0:
        _reset_decode_state(arc)
    serving._refresh(arc, block)
    q_step = q[:1] if (lead == 0 and q.shape[0] > 1) else q
    q_eval = torch.cat((q_hist[:-1].to(q_step.dtype), q_step), 0) if (
        q_hist is not None and lead == 0 and q_hist.shape[0] > 1) else q_step
    t_ev, h, d = q_eval.shape
    kv = h // groups
    rope_mask = serving.ROPE_HORIZON > 0 and limit > serving.ROPE_HORIZON
    n_valid, hole = full, (0, 0)
    hole_lo, hole_hi = getattr(arc, "hole_lo", 0), getattr(arc, "hole_hi", 0)
    if hole_hi > hole_lo:
        b0 = max(0, hole_lo - origin) // block
        b1 = min(full, (hole_hi - origin + block - 1) // block)
        if b1 > b0:
            n_valid, hole = full - (b1 - b0), (b0, b1)
        if n_valid <= 0:
            return None
    qe = q_eval.to(device=arc.kmax.device)
    if lead == 0 and not DECODE_RERANK:
        return _decode_pick(arc, qe, full, n_valid, hole, rope_mask, kv, t_ev)
    return _prompt_pick(arc, qe, groups, limit, budget, lead, full, n_valid, hole, rope_mask, kv, t_ev, block)


def _decode_pick(arc, qe, full, n_valid, hole, rope_mask, kv, t_ev):
    """The decode branch (memory.py:1053-1140): bound scores only, one ranking stage."""
    mem = serving.MEMORY
    sblk = serving.SBLK
    k_dec = min(DECODE_BLOCKS if DECODE_BLOCKS > 0 else (mem["decode_blocks"] or mem["blocks"]), n_valid)
    smax, smin = getattr(arc, "smax", None), getattr(arc, "smin", None)
    fine = None
    if sblk > 1 and smax is not None and smin is not None and full > sblk * 16 and not arc.is_global_agg:
        n_sb = (full + sblk - 1) // sblk
        sb = token_scores(qe, smax, smin, n_sb, n_sb, rope_mask=rope_mask, kv=kv)
        m_sb = min(max(16, (2 * k_dec + sblk - 1) // sblk), n_sb)
        top_sb = top_k(sb.amax(1), m_sb)
        fine_raw = (top_sb.unsqueeze(-1) * sblk + torch.arange(sblk, device=qe.device)).reshape(kv, m_sb * sblk)
        score = token_scores(qe, arc.kmax, arc.kmin, full, m_sb * sblk, cand=fine_raw, hole=hole,
                             rope_mask=rope_mask, kv=kv)
        fine = fine_raw.clamp(max=full - 1)
    else:
        score = token_scores(qe, arc.kmax, arc.kmin, full, full, hole=hole, rope_mask=rope_mask, kv=kv)
    n_pool = score.shape[-1]
    k_sel = min(k_dec, n_pool)
    z_rel, z_raw = zscores(score)
    if arc.is_global_agg and arc.visit_counts is not None and fine is None:
        z_rel, z_raw = _novelty(arc, z_rel, z_raw, full)
    rule, tail, r_zrel, r_zraw, tier = _rank_lists(score, z_rel, z_raw, n_pool, 0, "decode")
    lists = ([tail] if rule == "decode" else []) + [r_zrel, r_zraw, tier]
    keep = dedup_priority(torch.stack([first_k(r, k_sel) for r in lists], dim=-1).view(kv, -1), k_sel)
    blk_ord = fine.gather(-1, keep) if fine is not None else keep
    if arc.is_global_agg and fine is None and full >= serving.SBLK * 2:
        strat = stratified_peaks(z_raw.amax(1), full, max(8, k_sel // 2))
        n_top = max(1, k_sel // 2)
        blk_ord = dedup_priority(torch.cat((blk_ord[:, :n_top], strat, blk_ord[:, n_top:]), dim=-1), k_sel)
    if arc.decode_top is not None and not arc.is_global_agg:
        blk_ord = dedup_priority(_interleave(blk_ord, arc.decode_top.clamp(max=full - 1)), k_sel)
    arc.decode_top = blk_ord
    if kv > 1:  # one block set for every key head, in the heads' interleaved priority
        blk_ord = dedup_priority(blk_ord.transpose(0, 1).reshape(1, -1), k_sel).expand(kv, -1).contiguous()
    dec_prio, dec_sorted = expand_successors_dedup(blk_ord, full, k_sel, m_succ=k_sel)
    if arc.prompt_top is not None:
        p_prev = arc.prompt_top.clamp(max=full - 1)
        k_out = min(p_prev.shape[1], n_valid)
        n_pin = (k_out // 2) if arc.is_global_agg else max(0, k_out - dec_prio.shape[1])
        top_prio = dedup_priority(torch.cat((p_prev[:, :n_pin], dec_prio, p_prev[:, n_pin:]), dim=-1), k_out)
        blk, arc.last_prio_rank = top_prio.sort(-1)
    else:
        _, arc.last_prio_rank = dec_prio.sort(-1)
        blk = dec_sorted
    if arc.is_global_agg:
        record_block_visits(arc, dec_prio, full)
    return blk, None


def _prompt_pick(arc, qe, groups, limit, budget, lead, full, n_valid, hole, rope_mask, kv, t_ev, block):
    """The prompt / rescoring branch (memory.py:1142-1294): bound scores pick c candidates,
    exact per-token scores pick k of them, then the second hop, the merges and the
    successors."""
    mem = serving.MEMORY
    score = token_scores(qe, arc.kmax, arc.kmin, full, full, hole=hole, rope_mask=rope_mask, kv=kv)
    if not budget:
        budget = mem["decode_blocks"] or mem["blocks"]
    n_arch = max(full, (arc.prompt_len - mem["window"] - serving.ORIGIN) // block)
    for thresh, blocks in zip(serving.SCALE[0::2], serving.SCALE[1::2]):
        if n_arch > thresh:
            budget = max(budget, blocks)
    floor_k = 1024 if n_arch > 8192 else (512 if n_arch > 4096 else (384 if n_arch > 2048 else budget))
    k = min(max(budget, floor_k), n_valid)
    pool = max(mem["rerank"], 2 * k) if mem["rerank"] > 0 else 0
    c0 = min(max(pool, k), n_valid)
    mult = max(PERTOKEN_CAND, 2) if (lead is not None or t_ev > 1) else max(PERTOKEN_CAND, 1)
    if lead == 0 and arc.decode_step > 2 and arc.prompt_top is not None:
        c = min(max(k, 768), n_valid)
    elif lead == 0 and arc.prompt_top is not None:
        c = min(max(k, 1536), n_valid)
    else:
        c_floor = ((16384 if (lead is not None and lead < 0) else 8192) if n_arch > 8192
                   else (4096 if n_arch > 4096 else (3072 if n_arch > 2048 else 1536)))
        c = min(max(c0 * mult, c_floor), n_valid)
    z_rel, z_raw = zscores(score)
    if lead is not None and lead < 0:
        arc.is_global_agg = detect_global_agg(z_raw, full)
    elif lead == 0 and arc.is_global_agg and arc.visit_counts is not None:
        z_rel, z_raw = _novelty(arc, z_rel, z_raw, full)
    rule, tail, r_zrel, r_zraw, tier = _rank_lists(score, z_rel, z_raw, full, lead, "prefill")
    lists = ([tail] if tail is not None else []) + [r_zrel, r_zraw, tier]
    cand = dedup_priority(torch.stack([first_k(r, c) for r in lists], dim=-1).view(kv, -1), c)
    arc.last_top = arc.last_rk = None
    if mem["rerank"]:
        if limit > serving.ROPE_HORIZON > 0:  # the candidates' keys moved in proportion (memory.py:1197-1198)
            ck, _ = serving.rope_gather(arc.keys, None, cand.to(torch.int32), block, serving.ORIGIN, cand.shape[1],
                                        "proportional", ref_pos=limit)
            exact = token_rerank(qe, ck, block, None, cand.shape[1], kv=kv)
        else:
            exact = token_rerank(qe, arc.keys[:, serving.ORIGIN:], block, cand, cand.shape[1], kv=kv)
    else:
        exact = score.gather(-1, cand.unsqueeze(1).expand(kv, t_ev, cand.shape[1]))
    n_c = cand.shape[1]
    ez_rel, ez_raw = zscores(exact)
    rule, e_tail, r_ezrel, r_ezraw, e_tier = _rank_lists(exact, ez_rel, ez_raw, n_c, lead, "prefill")
    if rule == "prefill":
        lists = [r_ezrel, r_ezraw, e_tail, e_tier]
    elif rule == "decode":
        lists = [e_tail, r_ezrel, r_ezraw, e_tier]
    else:
        lists = [r_ezrel, r_ezraw, e_tier]
    keep = dedup_priority(torch.stack([first_k(r, k) for r in lists], dim=-1).view(kv, -1), k)
    blk_ord = cand.gather(-1, keep)
    if arc.is_global_agg and full >= serving.SBLK * 2:
        strat = stratified_peaks(z_raw.amax(1), full, max(16, k // 4))
        n_keep = max(1, (3 * k) // 4)
        blk_ord = dedup_priority(torch.cat((blk_ord[:, :n_keep], strat, blk_ord[:, n_keep:]), dim=-1), k)
    if mem["rerank"] and n_valid > 16:
        head = blk_ord[:, : min(8, blk_ord.shape[1])]
        last = arc.last_hop_head
        if (lead is None or lead < 0 or arc.decode_step <= 2 or last is None or head.shape != last.shape
                or not torch.equal(head, last)):
            arc.last_hop_head = head
            c2_cap = 256 if (lead == 0 and arc.decode_step > 2) else (384 if lead == 0 else 512)
            hop2 = second_hop_blocks(arc, blk_ord, full, n_valid, block, k2=min(64, max(32, k // 4)), c2_cap=c2_cap)
            n_head = min(16, blk_ord.shape[1])
            blk_ord = dedup_priority(torch.cat((blk_ord[:, :n_head], hop2, blk_ord[:, n_head:]), dim=-1), k)
    if lead is not None and lead < 0:
        arc.decode_top = None
        merged = blk_ord
    elif arc.prompt_top is not None:
        if arc.decode_top is not None and not arc.is_global_agg:
            blk_ord = dedup_priority(_interleave(blk_ord, arc.decode_top.clamp(max=full - 1)), k)
        arc.decode_top = blk_ord
        merged = dedup_priority(_prompt_first(arc.prompt_top.clamp(max=full - 1), blk_ord), k)
    else:
        merged = blk_ord
    m_succ = min(640, k) if k > 1024 else k
    top_prio, _ = expand_successors_dedup(merged, full, k, m_succ=m_succ)
    blk, arc.last_prio_rank = top_prio.sort(-1)
    if lead is not None and lead < 0:
        arc.prompt_top = top_prio
    if arc.is_global_agg:
        record_block_visits(arc, top_prio, full)
    return blk, None


def _prompt_first(p_prev: torch.Tensor, blk_ord: torch.Tensor) -> torch.Tensor:
    """prompt[0], block[0], prompt[1], ... over the common length, then the blocks' rest
    (memory.py:1278-1281)."""
    kv = blk_ord.shape[0]
    n = min(p_prev.shape[1], blk_ord.shape[1])
    inter = torch.stack((p_prev[:, :n], blk_ord[:, :n]), dim=-1).view(kv, 2 * n)
    return torch.cat((inter, blk_ord[:, n:]), dim=-1) if n < blk_ord.shape[1] else inter
