"""Generate the golden fixtures in tests/golden/ by running the REFERENCE implementation.

Run once, in a container where defnotean/pseudobrain's source tree is available:

    python tests/golden/make_golden.py /path/to/pseudobrain-checkout

It imports the reference's own PyTorch functions (pseudobrain.gated_deltanet and
pseudobrain.exact_memory) from that checkout, feeds them seeded inputs and stores
inputs and outputs as .npz files next to this script. Nothing at test time imports
the reference: the tests only read these files. bf16 tensors are stored as their
uint16 bit patterns.

Fixtures:
  gdn_fp32.npz    delta_rule_chunked and delta_rule_sequential, fp32, ragged T=100
                  (one full chunk of 64 and a partial one), GQA 1 key head / 2 value
                  heads, nonzero initial state.
  gdn_bf16.npz    delta_rule_chunked on bf16 q/k/v/beta (fp32 g and state), B=2, T=80.
  gdn_decode.npz  delta_rule_sequential (the kernel select_kernel picks for T <= 4),
                  T=3 tokens, bf16 inputs, fp32 state ~ N(0, 0.02).
  swa.npz         causal_attention (pseudobrain/transplant.py:417-436) on bf16-valued
                  inputs (run in fp32), GQA 4 query / 2 key heads, d=128: a sliding window
                  of 100 with 4 sinks over T=260 through the reference's query-chunked path
                  (_chunked_window_attention, chunk forced to 128), and full causal T=200.
  serving.npz     the serving twins of pb27_vllm/memory.py: retrieve_blocks (flat bound scores,
                  exact rerank of the candidates, and the flat path without rerank) and
                  piece_attention (sinks + retrieved blocks + partial tail + masked window,
                  the SDPA branch) over an Archive of 2 key heads, 64-token blocks after the 4
                  sink positions, for a decode piece (T=1) and a 3-token piece.
  gdn_io.npz      the layer pieces around the recurrence: short_convolution with a carried
                  tail (width 4), l2_normalize in both modes, the gating and gated output
                  norm expressions of GatedDeltaNetLayer.forward.
  quest_levels.npz  retrieve's two-level super-block selection (page 16, super-blocks of 2
                  pages, 101 full pages), exact rerank, neighbours and a kept prompt selection;
                  the serving retrieve_blocks' super-block path, with and without an archive
                  hole, its flat path with a hole and its rerank path with a hole.
  rope.npz        RoPE repositioning past the horizon (lowered to 1500 tokens): the block moves
                  in both modes and the sink move called directly, and retrieve_blocks (rerank,
                  flat) + piece_attention on a 3000-token serving archive.
  pertoken.npz    the serving per-token selector retrieve_blocks_per_token: prompt, decode,
                  no-lead, global-aggregation and holed-archive steps with the selector state
                  before and after each.
  pertoken256.npz the same at PB-27's attention shape (4 key heads x 6 query heads, head dim 256).
  serving256.npz  the serving twins at PB-27's shape: archive summaries, retrieve_blocks (flat,
                  super-block, rerank, holed rerank, rerank past a lowered RoPE horizon) and
                  piece_attention.
  archive_write.npz  the serving Archive.write: a prefill write, short and scattered writes
                  and a long write across super-blocks into a CPU archive, then
                  refresh_bounds; its final storage, block and super-block summaries.
  quest.npz       archive_append + retrieve (flat mode, page 16, budget 4 pages) for a
                  decode query (T=1) and a 3-token query, plus the exact attention over
                  [retrieved ; window] as pseudobrain/transplant.py:619-628 computes it.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _bits(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _gdn_inputs(gen, batch, length, hk, hv, dk, dv, dtype, state_std):
    """Config-0 distributions: q,k ~ N(0,1) L2-normalised per head; v ~ N(0,1);
    beta = sigmoid(N(0,1)); g = logsigmoid(N(2,1))."""
    import torch
    import torch.nn.functional as F
    q = F.normalize(torch.randn(batch, length, hk, dk, generator=gen), dim=-1)
    k = F.normalize(torch.randn(batch, length, hk, dk, generator=gen), dim=-1)
    v = torch.randn(batch, length, hv, dv, generator=gen)
    beta = torch.sigmoid(torch.randn(batch, length, hv, generator=gen))
    g = F.logsigmoid(torch.randn(batch, length, hv, generator=gen) + 2.0)
    h0 = torch.randn(batch, hv, dk, dv, generator=gen) * state_std
    q, k, v, beta = (x.to(dtype) for x in (q, k, v, beta))
    return q, k, v, g, beta, h0


def _expand(x, hv):
    return x.repeat_interleave(hv // x.shape[2], dim=2)


def make_gdn(G):
    import torch
    dk = dv = 128
    scale = dk ** -0.5

    gen = torch.Generator().manual_seed(100)
    q, k, v, g, beta, h0 = _gdn_inputs(gen, 1, 100, 1, 2, dk, dv, torch.float32, 0.02)
    oc, sc = G.delta_rule_chunked(_expand(q, 2), _expand(k, 2), v, g, beta, scale, h0)
    os_, ss = G.delta_rule_sequential(_expand(q, 2), _expand(k, 2), v, g, beta, scale, h0)
    np.savez_compressed(os.path.join(HERE, "gdn_fp32.npz"), q=q.numpy(), k=k.numpy(), v=v.numpy(),
                        g=g.numpy(), beta=beta.numpy(), h0=h0.numpy(), scale=np.float64(scale),
                        o_chunked=oc.numpy(), s_chunked=sc.numpy(),
                        o_sequential=os_.numpy(), s_sequential=ss.numpy())

    gen = torch.Generator().manual_seed(101)
    q, k, v, g, beta, h0 = _gdn_inputs(gen, 2, 80, 1, 2, dk, dv, torch.bfloat16, 0.0)
    oc, sc = G.delta_rule_chunked(_expand(q, 2), _expand(k, 2), v, g, beta, scale, h0)
    np.savez_compressed(os.path.join(HERE, "gdn_bf16.npz"), q=_bits(q), k=_bits(k), v=_bits(v),
                        g=g.numpy(), beta=_bits(beta), h0=h0.numpy(), scale=np.float64(scale),
                        o_chunked=oc.numpy(), s_chunked=sc.numpy())

    gen = torch.Generator().manual_seed(102)
    q, k, v, g, beta, h0 = _gdn_inputs(gen, 2, 3, 1, 2, dk, dv, torch.bfloat16, 0.02)
    g = g.to(torch.bfloat16)
    assert G.select_kernel("reference", False, 3, h0) == "sequential"
    os_, ss = G.delta_rule_sequential(_expand(q, 2), _expand(k, 2), v, g, beta, scale, h0)
    np.savez_compressed(os.path.join(HERE, "gdn_decode.npz"), q=_bits(q), k=_bits(k), v=_bits(v),
                        g=_bits(g), beta=_bits(beta), h0=h0.numpy(), scale=np.float64(scale),
                        o_sequential=os_.numpy(), s_sequential=ss.numpy())


def make_quest(E):
    import torch
    import torch.nn.functional as F
    page, budget, kv, groups, d = 16, 4, 2, 4, 128
    E.EXACT_MEMORY.update(enabled=True, block_size=page, blocks=budget, decode_blocks=budget,
                          superblock=0, rerank=0, decode_rerank=0, neighbors=0, keys_like_values=False)
    gen = torch.Generator().manual_seed(103)
    n_arch, n_win, window = 16 * page + 8, 24, 24
    keys = torch.randn(1, kv, n_arch + n_win, d, generator=gen).to(torch.bfloat16)
    values = torch.randn(1, kv, n_arch + n_win, d, generator=gen).to(torch.bfloat16)
    # Two appends (the second completes the first's partial page), as eviction does.
    arc = E.archive_append(None, keys[:, :, :100], values[:, :, :100])
    arc = E.archive_append(arc, keys[:, :, 100:n_arch], values[:, :, 100:n_arch])
    out = dict(keys=_bits(keys), values=_bits(values), kmax=_bits(arc.kmax), kmin=_bits(arc.kmin),
               page=np.int64(page), budget=np.int64(budget), groups=np.int64(groups),
               n_arch=np.int64(n_arch), window=np.int64(window))
    wk, wv = keys[:, :, n_arch:], values[:, :, n_arch:]
    kpos = torch.arange(n_arch, n_arch + n_win)
    for name, t in (("t1", 1), ("t3", 3)):
        q = torch.randn(1, kv * groups, t, d, generator=gen).to(torch.bfloat16)
        arc.prompt_top = None
        rk, rv = E.retrieve(arc, q, groups)
        # Page indices: match each gathered page against the archive's pages.
        full = n_arch // page
        pages = arc.keys[:, :, : full * page].reshape(1, kv, full, page * d)
        got = rk[:, :, : budget * page].reshape(1, kv, budget, page * d)
        top = torch.stack([torch.stack([
            torch.tensor([int(torch.nonzero((pages[0, h] == got[0, h, j]).all(-1))[0]) for j in range(budget)])
            for h in range(kv)])])
        # transplant.py:619-628: mask, GQA repeat, SDPA (run here in fp32).
        qpos = torch.arange(n_arch + n_win - t, n_arch + n_win)
        mask = (kpos[None, :] <= qpos[:, None]) & ((qpos[:, None] - kpos[None, :]) < window)
        mask = torch.cat((torch.ones(t, rk.shape[2], dtype=torch.bool), mask), dim=1)
        kk = torch.cat((rk, wk), dim=2).float().repeat_interleave(groups, dim=1)
        vv = torch.cat((rv, wv), dim=2).float().repeat_interleave(groups, dim=1)
        a = F.scaled_dot_product_attention(q.float(), kk, vv, attn_mask=mask)
        out.update({f"{name}_q": _bits(q), f"{name}_top": top.numpy().astype(np.int64),
                    f"{name}_rk": _bits(rk), f"{name}_rv": _bits(rv), f"{name}_out": a.numpy(),
                    f"{name}_qpos": qpos.numpy().astype(np.int64)})
    out["kpos"] = kpos.numpy().astype(np.int64)
    np.savez_compressed(os.path.join(HERE, "quest.npz"), **out)


def _pages_of(arc_keys, rk, page, sel):
    """Page index of each of the first `sel` gathered pages, matched against the archive."""
    import torch
    kv, d = arc_keys.shape[1], arc_keys.shape[3]
    full = arc_keys.shape[2] // page
    pages = arc_keys[0, :, : full * page].reshape(kv, full, page * d)
    got = rk[0, :, : sel * page].reshape(kv, sel, page * d)
    return torch.stack([torch.tensor([int(torch.nonzero((pages[h] == got[h, j]).all(-1))[0]) for j in range(sel)])
                        for h in range(kv)]).unsqueeze(0)


def make_quest_levels(E, MEM):
    """retrieve's other modes (two-level super-blocks, exact rerank, neighbours, a prompt
    selection kept for decode) and the serving retrieve_blocks' super-block path with and
    without an archive hole, the flat path with a hole, and the rerank path with a hole."""
    import torch
    page, budget, kv, groups, d, sblk = 16, 8, 2, 4, 128, 2
    gen = torch.Generator().manual_seed(107)
    n_arch = 101 * page + 5
    keys = torch.randn(1, kv, n_arch, d, generator=gen).to(torch.bfloat16)
    values = torch.randn(1, kv, n_arch, d, generator=gen).to(torch.bfloat16)
    base = dict(enabled=True, block_size=page, blocks=budget, decode_blocks=budget, superblock=sblk, rerank=0,
                decode_rerank=0, neighbors=0, keys_like_values=False)
    E.EXACT_MEMORY.update(base)
    arc = E.archive_append(None, keys[:, :, :700], values[:, :, :700])
    arc = E.archive_append(arc, keys[:, :, 700:], values[:, :, 700:])
    out = dict(keys=_bits(keys), values=_bits(values), kmax=_bits(arc.kmax), kmin=_bits(arc.kmin),
               smax=_bits(arc.smax), smin=_bits(arc.smin), page=np.int64(page), budget=np.int64(budget),
               groups=np.int64(groups), sblk=np.int64(sblk))
    cases = (("sb_t1", 1, {}), ("sb_t3", 3, {}), ("rerank_t1", 1, {"decode_rerank": 24}),
             ("sb_nb_t1", 1, {"neighbors": 1}), ("prompt_t80", 80, {}), ("sb_after_prompt_t1", 1, {}))
    for name, t, extra in cases:
        E.EXACT_MEMORY.update(base)
        E.EXACT_MEMORY.update(extra)
        if name != "sb_after_prompt_t1":
            arc.prompt_top = None
        q = torch.randn(1, kv * groups, t, d, generator=gen).to(torch.bfloat16)
        rk, _ = E.retrieve(arc, q, groups)
        sel = (rk.shape[2] - n_arch % page) // page
        out.update({f"{name}_q": _bits(q), f"{name}_top": _pages_of(arc.keys, rk, page, sel).numpy().astype(np.int64),
                    f"{name}_extra": np.array(sorted(extra.items()), dtype=object).astype(str)})
    E.EXACT_MEMORY.update(base)
    # serving: an archive of 2 key heads, 16-token blocks after the sinks, super-blocks of 2
    MEM.SBLK = sblk
    MEM.MEMORY.update(blocks=8, decode_blocks=8, rerank=0, block_size=page, neighbors=0, window=64)
    cap = MEM.ORIGIN + 101 * page + 20
    skeys = torch.randn(kv, cap, d, generator=gen).to(torch.bfloat16).float()
    svalues = torch.randn(kv, cap, d, generator=gen).to(torch.bfloat16).float()
    n_blk = cap // page
    n_sb = (n_blk + sblk - 1) // sblk
    sarc = MEM.Archive(skeys, svalues, torch.empty(kv, n_blk, d), torch.empty(kv, n_blk, d))
    sarc.smax, sarc.smin = torch.empty(kv, n_sb, d), torch.empty(kv, n_sb, d)
    sarc.size = sarc.prompt_len = cap
    sarc.dirty_lo, sarc.dirty_hi = 0, n_blk - 1
    sarc.refresh_bounds(page)
    out.update(s_keys=_bits(skeys.to(torch.bfloat16)), s_kmax=_bits(sarc.kmax.to(torch.bfloat16)),
               s_kmin=_bits(sarc.kmin.to(torch.bfloat16)), s_smax=_bits(sarc.smax.to(torch.bfloat16)),
               s_smin=_bits(sarc.smin.to(torch.bfloat16)), s_origin=np.int64(MEM.ORIGIN), s_limit=np.int64(cap - 40))
    hole = (MEM.ORIGIN + 30 * page + 3, MEM.ORIGIN + 52 * page)  # positions: blocks 30 .. 51
    for name, t, rerank, hole_on, no_sb, extra in (("s_sb", 1, False, False, False, {}),
                                                 ("s_sb_hole", 2, False, True, False, {}),
                                                 ("s_sb_nb", 1, False, False, False, {"neighbors": 1}),
                                                 ("s_flat_hole", 1, False, True, True, {}),
                                                 ("s_rerank_hole", 1, True, True, False, {"rerank": 12})):
        MEM.MEMORY.update(rerank=0, neighbors=0)
        MEM.MEMORY.update(extra)
        sarc.hole_lo, sarc.hole_hi = hole if hole_on else (0, 0)
        saved = (sarc.smax, sarc.smin)
        if no_sb:
            sarc.smax = sarc.smin = None
        q = torch.randn(t, kv * groups, d, generator=gen).to(torch.bfloat16).float()
        top = MEM.retrieve_blocks(sarc, q, groups, cap - 40, rerank)
        sarc.smax, sarc.smin = saved
        out.update({f"{name}_q": _bits(q.to(torch.bfloat16)), f"{name}_top": top.numpy().astype(np.int64),
                    f"{name}_rerank": np.int64(rerank), f"{name}_hole": np.array(hole if hole_on else (0, 0)),
                    f"{name}_nosb": np.int64(no_sb), f"{name}_neighbors": np.int64(extra.get("neighbors", 0)),
                    f"{name}_pool": np.int64(extra.get("rerank", 0))})
    MEM.MEMORY.update(rerank=0, neighbors=0)
    np.savez_compressed(os.path.join(HERE, "quest_levels.npz"), **out)


def make_rope(MEM):
    """RoPE repositioning past the horizon (pb27_vllm/memory.py:574-677): the block and sink
    moves called directly, then retrieve_blocks (rerank and flat) and piece_attention on an
    archive whose window starts past the horizon. The horizon and arc span are lowered
    (ROPE_HORIZON 1500, ROPE_ARC_SPAN 600) so a 3000-token archive crosses them."""
    import torch
    MEM.ROPE_HORIZON, MEM.ROPE_ARC_SPAN = 1500, 600
    kv, groups, d, block = 2, 3, 128, 16
    gen = torch.Generator().manual_seed(109)
    out = dict(horizon=np.int64(1500), arc_span=np.int64(600), theta=np.float64(MEM.ROPE_THETA), block=np.int64(block))
    # direct: 9 blocks with runs and gaps, ref_pos 2900
    idx = torch.tensor([[3, 4, 5, 9, 20, 21, 40, 41, 42], [0, 7, 8, 9, 10, 60, 61, 70, 100]])
    rk = torch.randn(kv, 9 * block, d, generator=gen).to(torch.bfloat16)
    sk = torch.randn(kv, 4, d, generator=gen).to(torch.bfloat16)
    out.update(rk=_bits(rk), idx=idx.numpy().astype(np.int64), sk=_bits(sk), ref_pos=np.int64(2900),
               rk_runs=_bits(MEM._reposition_rope_blocks(rk, idx, block, 2900, contiguous_runs=True)),
               rk_prop=_bits(MEM._reposition_rope_blocks(rk, idx, block, 2900, contiguous_runs=False, span=0)),
               sk_moved=_bits(MEM._reposition_rope_sinks(sk, 2900, n_blk=9, block=block)))
    # end to end on an archive
    MEM.MEMORY.update(blocks=4, decode_blocks=4, rerank=12, block_size=block, neighbors=0, window=256)
    cap = MEM.ORIGIN + 190 * block + 9
    keys = torch.randn(kv, cap, d, generator=gen).to(torch.bfloat16).float()
    values = torch.randn(kv, cap, d, generator=gen).to(torch.bfloat16).float()
    n_blk = cap // block
    arc = MEM.Archive(keys, values, torch.empty(kv, n_blk, d), torch.empty(kv, n_blk, d))
    arc.size = arc.prompt_len = cap
    arc.dirty_lo, arc.dirty_hi = 0, n_blk - 1
    arc.refresh_bounds(block)
    out.update(keys=_bits(keys.to(torch.bfloat16)), values=_bits(values.to(torch.bfloat16)), window=np.int64(256),
               groups=np.int64(groups))
    for name, t, rerank in (("rr", 1, True), ("flat", 2, False)):
        q = torch.randn(t, kv * groups, d, generator=gen).to(torch.bfloat16).float()
        q_pos = torch.arange(cap - t, cap)
        q_min, q_max = int(q_pos[0]), int(q_pos[-1])
        limit = q_min - 256 + 1
        top = MEM.retrieve_blocks(arc, q, groups, limit, rerank)
        o = MEM.piece_attention(arc, q, q_pos, top, groups, 256, d ** -0.5, None, q_min=q_min, q_max=q_max)
        out.update({f"{name}_q": _bits(q.to(torch.bfloat16)), f"{name}_pos": q_pos.numpy().astype(np.int64),
                    f"{name}_limit": np.int64(limit), f"{name}_rerank": np.int64(rerank),
                    f"{name}_top": top.numpy().astype(np.int64), f"{name}_out": o.float().numpy()})
    MEM.ROPE_HORIZON, MEM.ROPE_ARC_SPAN = 262144, 98304
    np.savez_compressed(os.path.join(HERE, "rope.npz"), **out)


def make_archive_write(MEM):
    """Archive.write (pb27_vllm/memory.py:310-395) on a CPU archive (fp32 storage and
    summaries) with 16-token blocks and super-blocks of 2: a contiguous prefill write, two
    short contiguous writes, a scattered write, a long contiguous write across super-blocks,
    then refresh_bounds. The inputs and the final storage and summaries are kept."""
    import torch
    MEM.SBLK = 2
    kv, d, block, cap = 2, 128, 16, 640
    gen = torch.Generator().manual_seed(111)
    arc = MEM.Archive.new(kv, d, cap, block, torch.float32, torch.device("cpu"))
    writes = [np.arange(0, 41), np.arange(41, 44), np.arange(44, 45), np.array([10, 30, 50, 43]),
              np.arange(45, 300)]
    out = dict(block=np.int64(block), sblk=np.int64(2), cap=np.int64(cap), n_writes=np.int64(len(writes)))
    for i, pos in enumerate(writes):
        k = torch.randn(len(pos), kv, d, generator=gen).to(torch.bfloat16).float()
        v = torch.randn(len(pos), kv, d, generator=gen).to(torch.bfloat16).float()
        arc.write(torch.from_numpy(pos), k, v, block)
        out.update({f"w{i}_pos": pos.astype(np.int64), f"w{i}_k": _bits(k.to(torch.bfloat16)),
                    f"w{i}_v": _bits(v.to(torch.bfloat16))})
    arc.refresh_bounds(block)
    out.update(size=np.int64(arc.size), keys=_bits(arc.keys.to(torch.bfloat16)),
               values=_bits(arc.values.to(torch.bfloat16)))
    for name in ("kmax", "kmin", "bmean_k", "bmean_v", "smax", "smin", "smean_k", "smean_v"):
        out[name] = getattr(arc, name).float().numpy()
    MEM.SBLK = 64
    np.savez_compressed(os.path.join(HERE, "archive_write.npz"), **out)


def make_swa(TR):
    import torch
    out = {}
    gen = torch.Generator().manual_seed(104)
    for name, t, window, sinks, chunk in (("win", 260, 100, 4, 128), ("full", 200, None, 0, 4096)):
        q = torch.randn(1, 4, t, 128, generator=gen).to(torch.bfloat16)
        k = torch.randn(1, 2, t, 128, generator=gen).to(torch.bfloat16)
        v = torch.randn(1, 2, t, 128, generator=gen).to(torch.bfloat16)
        saved = dict(TR.WINDOW_CHUNK)
        TR.WINDOW_CHUNK["queries"] = chunk
        try:
            o = TR.causal_attention(q.float(), k.float(), v.float(), window=window, sinks=sinks)
        finally:
            TR.WINDOW_CHUNK.update(saved)
        out.update({f"{name}_q": _bits(q), f"{name}_k": _bits(k), f"{name}_v": _bits(v), f"{name}_o": o.numpy(),
                    f"{name}_window": np.int64(-1 if window is None else window), f"{name}_sinks": np.int64(sinks)})
    np.savez_compressed(os.path.join(HERE, "swa.npz"), **out)


def make_serving(MEM):
    import torch
    kv, groups, d, block = 2, 3, 128, 64
    MEM.MEMORY.update(blocks=4, decode_blocks=4, rerank=12, block_size=block, neighbors=0, window=256)
    cap = MEM.ORIGIN + 40 * block + 20
    gen = torch.Generator().manual_seed(105)
    keys = torch.randn(kv, cap, d, generator=gen).to(torch.bfloat16).float()
    values = torch.randn(kv, cap, d, generator=gen).to(torch.bfloat16).float()
    n_blk = cap // block
    arc = MEM.Archive(keys, values, torch.empty(kv, n_blk, d), torch.empty(kv, n_blk, d))
    arc.size = arc.prompt_len = cap
    arc.dirty_lo, arc.dirty_hi = 0, n_blk - 1
    arc.refresh_bounds(block)
    out = dict(keys=_bits(keys.to(torch.bfloat16)), values=_bits(values.to(torch.bfloat16)),
               kmax=_bits(arc.kmax.to(torch.bfloat16)), kmin=_bits(arc.kmin.to(torch.bfloat16)),
               origin=np.int64(MEM.ORIGIN), sinks=np.int64(MEM.SINKS), block=np.int64(block),
               window=np.int64(256), groups=np.int64(groups), budget=np.int64(4), rerank_pool=np.int64(12))
    for name, t, rerank in (("t1", 1, True), ("t3", 3, True), ("flat", 1, False)):
        q = torch.randn(t, kv * groups, d, generator=gen).to(torch.bfloat16).float()
        q_pos = torch.arange(cap - t, cap)
        q_min, q_max = int(q_pos[0]), int(q_pos[-1])
        window = 256
        limit = q_min - window + 1
        top = MEM.retrieve_blocks(arc, q, groups, limit, rerank)
        o = MEM.piece_attention(arc, q, q_pos, top, groups, window, d ** -0.5, None, q_min=q_min, q_max=q_max)
        out.update({f"{name}_q": _bits(q.to(torch.bfloat16)), f"{name}_pos": q_pos.numpy().astype(np.int64),
                    f"{name}_limit": np.int64(limit), f"{name}_rerank": np.int64(rerank),
                    f"{name}_top": top.numpy().astype(np.int64), f"{name}_out": o.float().numpy()})
    np.savez_compressed(os.path.join(HERE, "serving.npz"), **out)


def make_pertoken(MEM):
    """The per-token selector retrieve_blocks_per_token (pb27_vllm/memory.py:1009-1294) on a
    CPU archive of 2 key heads x 3 query heads, 16-token blocks, super-blocks of 2: a prompt
    piece (48 tokens: the prompt branch with exact rescoring and the second hop), two decode
    steps with a query history (the super-block path, the prompt and decode merges), a piece
    without a lead, the same with dense global aggregation forced (stratified peaks, visit
    counts, the novelty penalty on the next decode step) and a prompt piece over an archive
    hole. Each step records the selector's state before and after it. The reference's topk
    and argsort run with ties in index order (torch's CPU order among equal values, e.g. the
    tied integer tier keys, is implementation-defined), the tie rule this build uses."""
    import torch
    orig_sort = torch.Tensor.sort

    def topk(self, k, dim=-1, largest=True, sorted=True):
        idx = orig_sort(self, dim=dim, descending=largest, stable=True).indices.narrow(dim, 0, k)
        return torch.return_types.topk((self.gather(dim, idx), idx))

    def argsort(self, dim=-1, descending=False, stable=False):
        return orig_sort(self, dim=dim, descending=descending, stable=True).indices

    saved = (torch.Tensor.topk, torch.Tensor.argsort)
    torch.Tensor.topk, torch.Tensor.argsort = topk, argsort
    try:
        _make_pertoken(MEM, 2, 3, 128, 300, "pertoken.npz")
        _make_pertoken(MEM, 4, 6, 256, 120, "pertoken256.npz")  # PB-27's attention shape: 24 query / 4 key heads
    finally:
        torch.Tensor.topk, torch.Tensor.argsort = saved


def _make_pertoken(MEM, kv, groups, d, n_blocks, fname):
    import torch
    block = 16
    MEM.SBLK = 2
    MEM.MEMORY.update(blocks=8, decode_blocks=8, rerank=12, block_size=block, neighbors=0, window=64, chunk=64)
    cap = MEM.ORIGIN + n_blocks * block + 10
    gen = torch.Generator().manual_seed(207)
    keys = torch.randn(kv, cap, d, generator=gen).to(torch.bfloat16).float()
    values = torch.randn(kv, cap, d, generator=gen).to(torch.bfloat16).float()
    n_blk = cap // block
    n_sb = (n_blk + MEM.SBLK - 1) // MEM.SBLK
    arc = MEM.Archive(keys, values, torch.empty(kv, n_blk, d), torch.empty(kv, n_blk, d))
    arc.smax, arc.smin = torch.empty(kv, n_sb, d), torch.empty(kv, n_sb, d)
    arc.bmean_k, arc.bmean_v = torch.empty(kv, n_blk, d), torch.empty(kv, n_blk, d)
    arc.smean_k, arc.smean_v = torch.empty(kv, n_sb, d), torch.empty(kv, n_sb, d)
    arc.size = arc.prompt_len = cap
    arc.dirty_lo, arc.dirty_hi = 0, n_blk - 1
    arc.refresh_bounds(block)
    out = dict(keys=_bits(keys.to(torch.bfloat16)), values=_bits(values.to(torch.bfloat16)),
               kmax=_bits(arc.kmax.to(torch.bfloat16)), kmin=_bits(arc.kmin.to(torch.bfloat16)),
               smax=_bits(arc.smax.to(torch.bfloat16)), smin=_bits(arc.smin.to(torch.bfloat16)),
               smean_k=arc.smean_k.numpy(), smean_v=arc.smean_v.numpy(), origin=np.int64(MEM.ORIGIN),
               sblk=np.int64(MEM.SBLK), block=np.int64(block), groups=np.int64(groups), prompt_len=np.int64(cap),
               window=np.int64(64))
    limit = cap - 80  # a decode piece at limit + 63 keeps its 64-key window inside the archive
    hole = (MEM.ORIGIN + 120 * block + 5, MEM.ORIGIN + 150 * block)

    def state(prefix):
        st = {}
        for name in ("prompt_top", "decode_top", "last_hop_head", "visit_counts"):
            v = getattr(arc, name, None)
            st[f"{prefix}_{name}"] = np.zeros((0,), np.int64) if v is None else v.numpy().astype(np.int64)
        st[f"{prefix}_decode_step"] = np.int64(arc.decode_step)
        st[f"{prefix}_global"] = np.int64(bool(arc.is_global_agg))
        return st

    steps = (("prompt", 48, -1, False, "auto", False), ("dec1", 1, 0, True, "auto", False),
             ("dec2", 1, 0, True, "auto", False), ("nolead", 1, None, False, "auto", False),
             ("gprompt", 40, -1, False, "1", False), ("gdec", 1, 0, True, "1", False),
             ("hole", 44, -1, False, "auto", True))
    hist = torch.randn(24, kv * groups, d, generator=gen).to(torch.bfloat16).float()
    names = []
    for name, t, lead, with_hist, gagg, hole_on in steps:
        MEM.GLOBAL_AGG = gagg
        arc.hole_lo, arc.hole_hi = hole if hole_on else (0, 0)
        q = torch.randn(t, kv * groups, d, generator=gen).to(torch.bfloat16).float()
        q_hist = None
        if with_hist:
            hist = torch.cat((hist[1:], q[:1]), 0)
            q_hist = hist[-16:]
        out.update(state(f"{name}_before"))
        res = MEM.retrieve_blocks_per_token(arc, q, groups, limit, 0, lead, 0, q_hist)
        blk = res[0] if res is not None else torch.zeros(0, dtype=torch.int64)
        out.update(state(f"{name}_after"))
        if name in ("dec2", "gdec"):  # the piece's attention over sinks, landmarks, blocks, tail and window
            q_pos = torch.tensor([limit + 63])
            o = MEM.piece_attention(arc, q, q_pos, blk, groups, 64, d ** -0.5, None, q_min=limit + 63,
                                    q_max=limit + 63)
            out[f"{name}_attn"] = o.float().numpy()
        out.update({f"{name}_q": _bits(q.to(torch.bfloat16)), f"{name}_lead": np.int64(-9 if lead is None else lead),
                    f"{name}_hist": (_bits(q_hist.to(torch.bfloat16)) if q_hist is not None
                                     else np.zeros((0,), np.uint16)),
                    f"{name}_gagg": np.int64(gagg == "1"), f"{name}_hole": np.array(hole if hole_on else (0, 0)),
                    f"{name}_top": blk.numpy().astype(np.int64)})
        names.append(name)
    MEM.GLOBAL_AGG = "auto"
    out["steps"] = np.array(names)
    out["limit"] = np.int64(limit)
    np.savez_compressed(os.path.join(HERE, fname), **out)


def make_serving256(MEM):
    """The serving twins at PB-27's attention shape (24 query / 4 key heads, head dim 256):
    the archive summaries (block bounds and means, super-block bounds and means after the
    refresh), retrieve_blocks in its flat, super-block (super-blocks of 2), rerank and
    holed-rerank paths, and past a lowered RoPE horizon (1000) the rerank with moved
    candidates, each followed by piece_attention over sinks, blocks, tail and window."""
    import torch
    kv, groups, d, block = 4, 6, 256, 16
    MEM.SBLK = 2
    MEM.MEMORY.update(blocks=6, decode_blocks=6, rerank=12, block_size=block, neighbors=0, window=256)
    cap = MEM.ORIGIN + 100 * block + 9
    gen = torch.Generator().manual_seed(311)
    keys = torch.randn(kv, cap, d, generator=gen).to(torch.bfloat16).float()
    values = torch.randn(kv, cap, d, generator=gen).to(torch.bfloat16).float()
    n_blk = cap // block
    n_sb = (n_blk + MEM.SBLK - 1) // MEM.SBLK
    arc = MEM.Archive(keys, values, torch.empty(kv, n_blk, d), torch.empty(kv, n_blk, d))
    arc.smax, arc.smin = torch.empty(kv, n_sb, d), torch.empty(kv, n_sb, d)
    arc.bmean_k, arc.bmean_v = torch.empty(kv, n_blk, d), torch.empty(kv, n_blk, d)
    arc.smean_k, arc.smean_v = torch.empty(kv, n_sb, d), torch.empty(kv, n_sb, d)
    arc.size = arc.prompt_len = cap
    arc.dirty_lo, arc.dirty_hi = 0, n_blk - 1
    arc.refresh_bounds(block)
    out = dict(keys=_bits(keys.to(torch.bfloat16)), values=_bits(values.to(torch.bfloat16)),
               kmax=_bits(arc.kmax.to(torch.bfloat16)), kmin=_bits(arc.kmin.to(torch.bfloat16)),
               smax=_bits(arc.smax.to(torch.bfloat16)), smin=_bits(arc.smin.to(torch.bfloat16)),
               bmean_k=arc.bmean_k.numpy(), bmean_v=arc.bmean_v.numpy(), smean_k=arc.smean_k.numpy(),
               smean_v=arc.smean_v.numpy(), origin=np.int64(MEM.ORIGIN), sblk=np.int64(MEM.SBLK),
               block=np.int64(block), groups=np.int64(groups), window=np.int64(256), cap=np.int64(cap))
    hole = (MEM.ORIGIN + 40 * block + 3, MEM.ORIGIN + 70 * block)
    for name, t, rerank, use_sb, hole_on, horizon in (("flat", 1, False, False, False, 0),
                                                      ("sb", 1, False, True, False, 0),
                                                      ("rr", 1, True, False, False, 0),
                                                      ("hole_rr", 2, True, True, True, 0),
                                                      ("rope_rr", 1, True, False, False, 1000)):
        if horizon:
            MEM.ROPE_HORIZON = horizon
        arc.hole_lo, arc.hole_hi = hole if hole_on else (0, 0)
        saved = (arc.smax, arc.smin)
        if not use_sb:
            arc.smax = arc.smin = None
        q = torch.randn(t, kv * groups, d, generator=gen).to(torch.bfloat16).float()
        q_pos = torch.arange(cap - t, cap)
        q_min, q_max = int(q_pos[0]), int(q_pos[-1])
        limit = q_min - 256 + 1
        top = MEM.retrieve_blocks(arc, q, groups, limit, rerank)
        arc.smax, arc.smin = saved
        o = MEM.piece_attention(arc, q, q_pos, top, groups, 256, d ** -0.5, None, q_min=q_min, q_max=q_max)
        out.update({f"{name}_q": _bits(q.to(torch.bfloat16)), f"{name}_limit": np.int64(limit),
                    f"{name}_rerank": np.int64(rerank), f"{name}_sb": np.int64(use_sb),
                    f"{name}_hole": np.array(hole if hole_on else (0, 0)), f"{name}_horizon": np.int64(horizon),
                    f"{name}_top": top.numpy().astype(np.int64), f"{name}_out": o.float().numpy()})
        MEM.ROPE_HORIZON = 262144
    arc.hole_lo = arc.hole_hi = 0
    MEM.SBLK = 64
    out["cases"] = np.array(["flat", "sb", "rr", "hole_rr", "rope_rr"])
    np.savez_compressed(os.path.join(HERE, "serving256.npz"), **out)


def make_gdn_io(G):
    """The layer pieces around the recurrence: short_convolution (with a carried tail) and
    l2_normalize (both modes) are the reference's functions; gating and the gated output
    norm are GatedDeltaNetLayer.forward's expressions (gated_deltanet.py:427-429, 439-440),
    evaluated with the reference's torch ops."""
    import torch
    import torch.nn.functional as F
    gen = torch.Generator().manual_seed(77)
    b, t, hk, hv, d, width = 2, 70, 1, 2, 128, 4
    ch = (2 * hk + hv) * d
    x = torch.randn(b, t, ch, generator=gen)
    tail = torch.randn(b, width - 1, ch, generator=gen)
    weight = torch.randn(ch, width, generator=gen) * 0.5
    y, new_tail = G.short_convolution(x, tail, weight)
    q, k, v = y.split((hk * d, hk * d, hv * d), dim=-1)
    out = {"x": x.numpy(), "tail": tail.numpy(), "weight": weight.numpy(), "y": y.numpy(),
           "new_tail": new_tail.numpy()}
    for mode in ("max", "hf"):
        out[f"q_{mode}"] = G.l2_normalize(q.reshape(b, t, hk, d), mode).numpy()
        out[f"k_{mode}"] = G.l2_normalize(k.reshape(b, t, hk, d), mode).numpy()
    out["v"] = v.reshape(b, t, hv, d).numpy()
    small = torch.zeros(1, 1, d)
    small[..., 0] = 1e-4  # the modes differ for small vectors
    out["small_max"], out["small_hf"] = G.l2_normalize(small, "max").numpy(), G.l2_normalize(small, "hf").numpy()
    decay = torch.randn(b, t, 2 * hv, generator=gen) * 3.0
    decay[0, 0, 0] = 25.0  # past softplus's threshold
    a_log = torch.randn(hv, generator=gen)
    dt_bias = torch.randn(hv, generator=gen)
    a, bb = decay.chunk(2, dim=-1)
    g = -a_log.exp() * F.softplus(a + dt_bias)
    beta = torch.sigmoid(bb)
    out.update({"decay": decay.numpy(), "a_log": a_log.numpy(), "dt_bias": dt_bias.numpy(), "g": g.numpy(),
                "beta": beta.numpy()})
    o = torch.randn(b, t, hv, d, generator=gen)
    gate = torch.randn(b, t, hv * d, generator=gen)
    o_norm = torch.randn(d, generator=gen) * 0.3 + 1.0
    on = o * torch.rsqrt(o.square().mean(-1, keepdim=True) + G.NORM_EPS)
    on = on * o_norm * F.silu(gate.view(b, t, hv, d))
    out.update({"o": o.numpy(), "gate": gate.numpy(), "o_norm": o_norm.numpy(), "out": on.numpy()})
    np.savez_compressed(os.path.join(HERE, "gdn_io.npz"), **out)


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from pseudobrain import exact_memory as E
    from pseudobrain import gated_deltanet as G
    from pseudobrain import transplant as TR
    sys.path.insert(0, os.path.join(reference_root, "serving", "pb27_vllm"))
    os.environ.setdefault("PB27_MEMORY_OFFLOAD", "")
    import pb27_vllm.memory as MEM
    makers = {"gdn": lambda: make_gdn(G), "quest": lambda: make_quest(E), "swa": lambda: make_swa(TR),
              "serving": lambda: make_serving(MEM), "gdn_io": lambda: make_gdn_io(G),
              "quest_levels": lambda: make_quest_levels(E, MEM), "rope": lambda: make_rope(MEM),
              "archive_write": lambda: make_archive_write(MEM), "pertoken": lambda: make_pertoken(MEM),
              "serving256": lambda: make_serving256(MEM)}
    for name in (sys.argv[2:] if len(sys.argv) > 2 else makers):  # all, or only the named fixtures
        makers[name]()
    for name in sorted(os.listdir(HERE)):
        if name.endswith(".npz"):
            print(name, os.path.getsize(os.path.join(HERE, name)), "bytes")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <pseudobrain source checkout> [gdn|quest|swa ...]")
    main(sys.argv[1])
