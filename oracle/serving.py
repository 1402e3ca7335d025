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
  with the causal sliding-window mask (:1433-1490); past ROPE_HORIZON the sinks and the
  retrieved blocks' keys move to new RoPE positions (:574-677, :1402-1425).
Ties in the top-k go to the lowest block index (torch.topk leaves them unspecified).
"""
from __future__ import annotations

import numpy as np

ORIGIN = 4        # memory.py:46 (FAITHFUL, SINKS = 4)
SINKS = 4         # memory.py:37
SCALE = [2048, 384, 4096, 512, 8192, 1024]  # memory.py:49


ROPE_HORIZON = 262144  # memory.py:50
ROPE_ARC_SPAN = 98304  # memory.py:51
ROPE_THETA = 10000000.0  # memory.py:52


def inv_freq(d_rot: int, theta: float = ROPE_THETA) -> np.ndarray:
    """memory.py:563-571, in fp32."""
    return (np.float32(1.0) / (np.float32(theta) ** (np.arange(0, d_rot, 2, dtype=np.float32)
                                                     / np.float32(d_rot)))).astype(np.float32)


def _rotate(x: np.ndarray, delta: np.ndarray, theta: float, bf16: bool = True) -> np.ndarray:
    """Turn the first d/4 dims of x [..., D] in the pairs (i, i + d/8) by delta [...] * inv_freq,
    fp32 with each product and sum rounded, then to the keys' dtype: bf16, or fp32 when
    bf16=False (memory.py:598-606, 665-677)."""
    from .quest import bf16_round as _r
    bf16_round = _r if bf16 else (lambda v: v)
    d = x.shape[-1]
    half = d // 8
    ang = (delta[..., None].astype(np.float32) * inv_freq(d // 4, theta)).astype(np.float32)
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    x1, x2 = x[..., :half].astype(np.float32), x[..., half:2 * half].astype(np.float32)
    out = np.array(x, dtype=np.float32)
    out[..., :half] = bf16_round((x1 * c).astype(np.float32) - (x2 * s).astype(np.float32))
    out[..., half:2 * half] = bf16_round((x2 * c).astype(np.float32) + (x1 * s).astype(np.float32))
    return out


def block_shifts(blk_idx: np.ndarray, block: int, ref_pos: int, contiguous_runs: bool,
                 arc_span: int = ROPE_ARC_SPAN) -> np.ndarray:
    """Per-block RoPE position shift of _reposition_rope_blocks (memory.py:640-664), fp32:
    blk_idx [KV, n] -> [KV, n]."""
    f32 = np.float32
    idx = blk_idx.astype(np.int64)
    n = idx.shape[1]
    orig = (ORIGIN + idx * block).astype(f32)
    if not contiguous_runs:
        scale = f32(1.0 - min(1.0, float(arc_span) / float(max(1, ref_pos))))
        target = orig + np.rint(np.maximum(f32(ref_pos) - orig, f32(0)) * scale).astype(f32)
        return np.maximum(target - orig, f32(0))
    eff_span = max(arc_span, n * block)
    base_start = max(ORIGIN, ref_pos - eff_span)
    slack = f32(max(0, (ref_pos - base_start) - n * block))
    g_pre = np.maximum(orig[:, :1] - f32(ORIGIN), f32(0))
    if n > 1:
        g_mid = (np.maximum(idx[:, 1:] - idx[:, :-1] - 1, 0) * block).astype(f32)
        g_cum = np.concatenate((g_pre, g_pre + np.cumsum(g_mid, axis=1, dtype=f32)), axis=1)
        g_mid_sum = g_mid.sum(axis=1, keepdims=True, dtype=f32)
    else:
        g_cum, g_mid_sum = g_pre, np.zeros_like(g_pre)
    g_post = np.maximum(f32(ref_pos) - (orig[:, -1:] + f32(block)), f32(0))
    g_tot = np.maximum(g_pre + g_mid_sum + g_post, f32(1))
    j_steps = (np.arange(n, dtype=f32) * f32(block))[None]
    target = (f32(base_start) + j_steps) + np.rint(g_cum * (slack / g_tot)).astype(f32)
    return np.maximum(target - orig, f32(0))


def reposition_blocks(rk: np.ndarray, blk_idx: np.ndarray, block: int, ref_pos: int, contiguous_runs: bool,
                      horizon: int = ROPE_HORIZON, arc_span: int = ROPE_ARC_SPAN,
                      theta: float = ROPE_THETA, bf16: bool = True) -> np.ndarray:
    """_reposition_rope_blocks (memory.py:610-677): rk [KV, n*block, D] of blocks blk_idx [KV, n]."""
    if ref_pos <= horizon or rk.size == 0:
        return rk
    kv, total, d = rk.shape
    n = blk_idx.shape[1]
    delta = block_shifts(blk_idx, block, ref_pos, contiguous_runs, arc_span)
    return _rotate(rk.reshape(kv, n, block, d), np.repeat(delta[:, :, None], block, axis=2), theta,
                   bf16).reshape(kv, total, d)


def reposition_sinks(sk: np.ndarray, ref_pos: int, n_blk: int, block: int, horizon: int = ROPE_HORIZON,
                     arc_span: int = ROPE_ARC_SPAN, theta: float = ROPE_THETA, bf16: bool = True) -> np.ndarray:
    """_reposition_rope_sinks (memory.py:574-607): sk [KV, ns, D] moved to end before the first
    repositioned block."""
    if ref_pos <= horizon or sk.size == 0:
        return sk
    ns = sk.shape[1]
    base_start = max(ORIGIN, ref_pos - max(arc_span, n_blk * block))
    delta = max(0, base_start - ns)
    if delta <= 0:
        return sk
    return _rotate(sk, np.full(sk.shape[:2], delta, dtype=np.float32), theta, bf16)


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
                    hole=(0, 0), rope=(ROPE_HORIZON, ROPE_ARC_SPAN, ROPE_THETA), bf16_keys=True,
                    canonical=False):
    """keys [KV, cap, D]; kmax/kmin [KV, n_blk, D]; q [T, H, D] -> [KV, k] block indices or None.

    With smax/smin [KV, n_sb, D] and sblk > 1, a call without rerank over more than 16 sblk
    full blocks takes the two-level selection (memory.py:802-839). ``hole`` = (hole_lo,
    hole_hi) archive positions whose blocks score -inf (memory.py:769-777, 834-835, 852-853);
    memory["neighbors"] adds the following blocks (:873-875). Past the horizon (rope =
    (horizon, arc_span, theta)) the first d/4 query dims do not score the bounds (:795-797)
    and the rerank's candidate keys move in proportion (:861-862). canonical: every score in
    the canonical order of oracle.quest (the bit-exact pin of the kernels' selections)."""
    from .quest import canonical_bound_scores, canonical_key_scores, select_two_level
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
    qs = qg.copy()
    if limit > rope[0]:
        qs[..., : d // 4] = 0
    nb = memory.get("neighbors", 0)

    def with_neighbors(top):
        if nb:
            top = np.concatenate([top] + [np.minimum(top + j, full - 1) for j in range(1, nb + 1)], axis=-1)
        return np.sort(top, axis=-1)

    if not rerank and sblk > 1 and smax is not None and full > sblk * 16:
        return with_neighbors(select_two_level(qs, kmax, kmin, smax, smin, full, k, sblk, (hb0, hb1),
                                               canonical=canonical))
    if canonical:
        score = canonical_bound_scores(qs, kmax[:, :full], kmin[:, :full]).astype(np.float64)   # [KV, full]
    else:
        pos, neg = np.maximum(qs, 0), np.minimum(qs, 0)
        score = (np.einsum("grd,gnd->grn", pos, kmax[:, :full].astype(np.float64))
                 + np.einsum("grd,gnd->grn", neg, kmin[:, :full].astype(np.float64))).max(1)  # [KV, full]
    score[:, hb0:hb1] = -np.inf
    pool = max(memory["rerank"], 2 * k) if memory["rerank"] > 0 else 0
    if rerank and pool > k:
        c = min(pool, n_valid)
        cand = _topk_sorted(score, c)                                                   # [KV, c] ascending
        blk = keys[:, ORIGIN:ORIGIN + full * block].reshape(kv, full, block, d).astype(np.float64)
        ck = np.take_along_axis(blk, cand[:, :, None, None], axis=1)                    # [KV, c, block, D]
        if limit > rope[0]:
            ck = reposition_blocks(ck.reshape(kv, -1, d), cand, block, limit, False, *rope,
                                   bf16=bf16_keys).reshape(ck.shape)
        if canonical:
            exact = canonical_key_scores(qg, ck).astype(np.float64)                      # [KV, c]
        else:
            exact = np.einsum("grd,gcsd->grcs", qg, ck).max(axis=(1, 3))               # [KV, c]
        keep = _topk_sorted(exact, k)
        return with_neighbors(np.take_along_axis(cand, keep, axis=1))
    return with_neighbors(_topk_sorted(score, k))


def piece_attention(keys, values, q, q_pos, top, groups, window, scale, block,
                    rope=(ROPE_HORIZON, ROPE_ARC_SPAN, ROPE_THETA), bf16_keys=True):
    """q [T, H, D] at positions q_pos -> [T, H, D] float64 (SDPA branch, own=None). Past the
    horizon (lo > rope[0]) the sinks and the retrieved blocks' keys move (memory.py:1402-1425),
    rounded to bf16 (bf16_keys) or kept in fp32 as an fp32 archive keeps them."""
    t, h, d = q.shape
    kv = h // groups
    q_min, q_max = int(q_pos.min()), int(q_pos.max())
    lo, hi = max(0, q_min - window + 1), q_max + 1
    ns = min(SINKS, lo)
    tail0 = ORIGIN + ((lo - ORIGIN) // block) * block
    keys_sink = reposition_sinks(keys[:, :ns], lo, top.shape[1] if top is not None else 0, block, *rope,
                                 bf16=bf16_keys)
    keys_blk = None
    if top is not None:
        gathered = np.stack([np.concatenate([keys[g, ORIGIN + b * block:ORIGIN + (b + 1) * block] for b in top[g]])
                             for g in range(kv)]) if top.shape[1] else np.zeros((kv, 0, d), np.float32)
        keys_blk = reposition_blocks(gathered, top, block, lo, True, *rope, bf16=bf16_keys)
    out = np.zeros((t, h, d))
    for g in range(kv):
        idx = list(range(ns))
        kparts = [keys_sink[g]]
        if top is not None:
            for b in top[g]:
                idx += list(range(ORIGIN + b * block, ORIGIN + (b + 1) * block))
            kparts.append(keys_blk[g])
            if lo > tail0:
                idx += list(range(tail0, lo))
                kparts.append(keys[g, tail0:lo])
        always = len(idx)
        idx += list(range(lo, hi))
        kparts.append(keys[g, lo:hi])
        kk, vv = np.concatenate(kparts).astype(np.float64), values[g, idx].astype(np.float64)
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


class ArchiveState:
    """The serving archive's storage and block summaries, memory.py:120-431, restated: keys /
    values [KV, cap, D] (fp32 holding bf16 values), per-block kmax, kmin, bmean_k, bmean_v
    [KV, cap // block, D] and per-super-block smax, smin, smean_k, smean_v (fp32; the GPU
    keeps them in bf16). Blocks start after ORIGIN sink positions."""

    def __init__(self, kv: int, d: int, cap: int, block: int, sblk: int):
        n_blk = cap // block
        n_sb = (n_blk + sblk - 1) // sblk
        self.block, self.sblk, self.size = block, sblk, 0
        self.keys = np.zeros((kv, cap, d), np.float32)
        self.values = np.zeros((kv, cap, d), np.float32)
        for name, rows in (("kmax", n_blk), ("kmin", n_blk), ("bmean_k", n_blk), ("bmean_v", n_blk),
                           ("smax", n_sb), ("smin", n_sb), ("smean_k", n_sb), ("smean_v", n_sb)):
            setattr(self, name, np.zeros((kv, rows, d), np.float32))
        self.dirty_lo, self.dirty_hi = 1 << 60, -1

    def _refresh_range(self, lo_b: int, hi_b: int) -> None:
        """memory.py:399-421: the summaries of blocks lo_b .. hi_b over the rows written, a
        partial block padded with its last row."""
        block = self.block
        lo, hi = ORIGIN + lo_b * block, min(self.size, ORIGIN + (hi_b + 1) * block)
        if hi <= lo:
            return
        seg, seg_v = self.keys[:, lo:hi], self.values[:, lo:hi]
        pad = (-seg.shape[1]) % block
        if pad:
            seg = np.concatenate((seg, np.repeat(seg[:, -1:], pad, axis=1)), axis=1)
            seg_v = np.concatenate((seg_v, np.repeat(seg_v[:, -1:], pad, axis=1)), axis=1)
        kvh, _, d = seg.shape
        blocks, blocks_v = seg.reshape(kvh, -1, block, d), seg_v.reshape(kvh, -1, block, d)
        nb = blocks.shape[1]
        self.kmax[:, lo_b:lo_b + nb] = blocks.max(2)
        self.kmin[:, lo_b:lo_b + nb] = blocks.min(2)
        self.bmean_k[:, lo_b:lo_b + nb] = blocks.astype(np.float64).mean(2)
        self.bmean_v[:, lo_b:lo_b + nb] = blocks_v.astype(np.float64).mean(2)

    def _update_superbounds(self, lo_b: int, hi_b: int) -> None:
        """memory.py:280-306."""
        sblk = self.sblk
        if hi_b < lo_b or self.size <= ORIGIN:
            return
        n_blk = min(self.kmax.shape[1], (self.size - ORIGIN + self.block - 1) // self.block)
        sb0 = max(0, lo_b // sblk)
        sb1 = min(self.smax.shape[1] - 1, min(hi_b, max(0, n_blk - 1)) // sblk)
        for sb in range(sb0, sb1 + 1):
            b0, b1 = sb * sblk, min(n_blk, (sb + 1) * sblk)
            if b1 > b0:
                self.smax[:, sb] = self.kmax[:, b0:b1].max(1)
                self.smin[:, sb] = self.kmin[:, b0:b1].min(1)
                self.smean_k[:, sb] = self.bmean_k[:, b0:b1].astype(np.float64).mean(1)
                self.smean_v[:, sb] = self.bmean_v[:, b0:b1].astype(np.float64).mean(1)

    def write(self, pos: np.ndarray, k: np.ndarray, v: np.ndarray) -> None:
        """Archive.write (memory.py:310-395) for an archive that holds `pos`: k/v [N, KV, D]."""
        block = self.block
        hi, p0, n = int(pos.max()) + 1, int(pos.min()), pos.size
        contig = hi - p0 == n
        self.keys[:, pos] = k.transpose(1, 0, 2)
        self.values[:, pos] = v.transpose(1, 0, 2)
        fast, b_start, b_end = False, 0, 0
        if hi - 1 >= ORIGIN and contig and n >= block:
            b_start = max(0, (p0 - ORIGIN + block - 1) // block)
            b_end = max(b_start, (hi - ORIGIN) // block)
            if b_end > b_start:
                self.size = max(self.size, hi)
                self._refresh_range(b_start, b_end - 1)  # full blocks: the same summaries as the fast path
                fast = True
        self.size = max(self.size, hi)
        if hi - 1 < ORIGIN:
            return
        lo_b, hi_b = max(0, p0 - ORIGIN) // block, (hi - 1 - ORIGIN) // block
        if fast:
            if lo_b < b_start:
                self._refresh_range(lo_b, b_start - 1)
            if hi_b >= b_end:
                self._refresh_range(b_end, hi_b)
            self._update_superbounds(lo_b, hi_b)
            return
        self.dirty_lo, self.dirty_hi = min(self.dirty_lo, lo_b), max(self.dirty_hi, hi_b)

    def refresh_bounds(self) -> None:
        """memory.py:423-430."""
        if self.dirty_hi < self.dirty_lo:
            return
        self._refresh_range(self.dirty_lo, self.dirty_hi)
        self._update_superbounds(self.dirty_lo, self.dirty_hi)
        self.dirty_lo, self.dirty_hi = 1 << 60, -1
