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
computes the same softmax), with the super-block landmarks after the sinks under dense
global aggregation (:1332, 1411-1416). The per-token selector retrieve_blocks_per_token
(:1009-1294) is in pertoken.py. Not covered: the ORACLE diagnostic and per-query own-block
masks (NotImplementedError; the reference's selectors never produce them). Past
ROPE_HORIZON the reranked candidates' keys, the sinks and the retrieved blocks move to new
RoPE positions as the reference moves them (:574-677, 861-862, 1402-1425), gathered with
the move (pbk_quest_rope_gather).

``archive_write`` is Archive.write (:310-395) for an archive in HBM: the KV write fused
with the block summaries (max, min, key and value means) and the super-block refresh.

Kernels: pbk_quest_select (scores + top-k), pbk_quest_select_levels, pbk_quest_rerank,
pbk_quest_superbounds, pbk_quest_supermeans, pbk_quest_archive_write, pbk_quest_rope_gather,
pbk_quest_attend_sinks (libpbk.so, sm_100a); head dims 128 and 256 (PB-27's 24 query / 4 key
heads at 256 run on the SIMT score and attention kernels).
"""
from __future__ import annotations

import os
import types

import torch

from . import _capi
from ._capi import LIB, check
from .exact_memory import (_attend_desc, _workspace, rerank_pages, select_pages, select_pages_levels,
                           super_bounds_)

# memory.py:33-34 defaults (window: PB27_WINDOW, 16384)
MEMORY: dict = {"enabled": True, "blocks": 256, "block_size": 64, "decode_blocks": 256, "neighbors": 0,
                "rerank": 512, "chunk": 64, "window": 16384}
SINKS = 4                                   # memory.py:37
ORIGIN = SINKS                              # memory.py:46 (FAITHFUL)
SCALE = [2048, 384, 4096, 512, 8192, 1024]  # memory.py:49
ROPE_HORIZON = 262144                       # memory.py:50
ROPE_ARC_SPAN = 98304                       # memory.py:51
ROPE_THETA = float(os.environ.get("PB27_MEMORY_ROPE_THETA", "10000000.0") or 10000000.0)  # memory.py:52
SBLK = 64                                   # memory.py:79

_INV_FREQ: dict = {}


def _inv_freq(device: torch.device, d_rot: int) -> torch.Tensor:
    """The rotary inverse frequencies of the first d_rot dims, computed on the device by the
    reference's expression (memory.py:563-571), once per (device, d_rot, theta)."""
    key = (str(device), d_rot, ROPE_THETA)
    if key not in _INV_FREQ:
        _INV_FREQ[key] = 1.0 / (ROPE_THETA ** (torch.arange(0, d_rot, 2, device=device, dtype=torch.float32)
                                               / float(d_rot)))
    return _INV_FREQ[key]


ROPE_MODES = {"none": 0, "runs": 1, "proportional": 2, "constant": 3}


def rope_gather(keys: torch.Tensor, values: torch.Tensor | None, blocks: torch.Tensor | None, block: int,
                origin: int, n_blk: int, mode: str, ref_pos: int = 0, arc_span: int = 0, tail0: int = 0,
                tail_n: int = 0, const_delta: float = 0.0):
    """Gather blocks of an archive [KV, N, 128] with their keys moved to new RoPE positions
    (pbk_quest_rope_gather; memory.py:574-677): block j of key head h is archive rows origin +
    blocks[h][j] * block .. (blocks None: block j), followed by rows [tail0, tail0 + tail_n) as
    they are. mode 'runs' is _reposition_rope_blocks with contiguous_runs=True, 'proportional'
    with contiguous_runs=False, 'constant' turns every block by const_delta positions
    (_reposition_rope_sinks), 'none' only gathers. Returns (keys, values or None)
    [KV, n_blk * block + tail_n, 128] bf16."""
    kv, n_rows, d = keys.shape
    rows = n_blk * block + tail_n
    ok = torch.empty(kv, rows, d, dtype=keys.dtype, device=keys.device)
    ov = torch.empty_like(ok) if values is not None else None
    blk32 = blocks.to(torch.int32).contiguous() if blocks is not None else None
    delta = torch.empty(kv, max(n_blk, 1), dtype=torch.float32, device=keys.device)
    inv = _inv_freq(keys.device, d // 4)
    span = arc_span if arc_span > 0 else ROPE_ARC_SPAN
    desc = _capi.PbkRopeGatherDesc(
        kv=kv, d=d, block=block, n_blk=n_blk, origin=origin, n_rows=n_rows, ref_pos=ref_pos, arc_span=span,
        mode=ROPE_MODES[mode], tail0=tail0, tail_n=tail_n,
        scale=1.0 - min(1.0, float(span) / float(max(1, ref_pos))), const_delta=float(const_delta),
        blocks=blk32.data_ptr() if blk32 is not None else None, inv_freq=inv.data_ptr(), keys=keys.data_ptr(),
        values=values.data_ptr() if values is not None else None, stride_kv=keys.stride(0), stride_n=keys.stride(1),
        out_keys=ok.data_ptr(), out_values=ov.data_ptr() if ov is not None else None, delta=delta.data_ptr())
    if values is not None and (values.stride(0), values.stride(1)) != (keys.stride(0), keys.stride(1)):
        raise ValueError("keys and values must share strides")
    with torch.cuda.device(keys.device):
        check(LIB.pbk_quest_rope_gather(desc, torch.cuda.current_stream(keys.device).cuda_stream),
              "pbk_quest_rope_gather")
    return ok, ov


def sink_shift(ref_pos: int, ns: int, n_blk: int, block: int) -> int:
    """Positions the sink keys move by past ROPE_HORIZON (memory.py:585-596): to just before
    the first repositioned block."""
    if ref_pos <= ROPE_HORIZON or ns == 0:
        return 0
    base_start = max(ORIGIN, ref_pos - max(ROPE_ARC_SPAN, n_blk * block))
    return max(0, base_start - ns)


def _write(arc, block: int, size: int, blk_lo: int, blk_hi: int, k=None, v=None, p0: int = 0,
           pos: torch.Tensor | None = None, origin: int | None = None) -> None:
    """pbk_quest_archive_write: new rows k/v [N, KV, D] at p0.. (or at pos) into the archive,
    and the max, min and (when the archive keeps them) mean summaries of blocks
    [blk_lo, blk_hi] (block b at row origin + b block, origin ORIGIN by default) over the rows
    written so far. A host-resident archive (offload_archive) takes its new rows by a
    device-to-host copy, and the summarised blocks' rows are staged into HBM for the kernel."""
    if not arc.keys.is_cuda:
        _write_host(arc, block, size, blk_lo, blk_hi, k, v, p0, pos)
        return
    origin = ORIGIN if origin is None else origin
    kv, cap, d = arc.keys.shape
    bmean_k, bmean_v = getattr(arc, "bmean_k", None), getattr(arc, "bmean_v", None)
    if blk_hi >= blk_lo and blk_hi >= arc.kmax.shape[1]:
        raise ValueError(f"block {blk_hi} past the bounds array ({arc.kmax.shape[1]} blocks)")
    if (arc.values.stride(0), arc.values.stride(1)) != (arc.keys.stride(0), arc.keys.stride(1)):
        raise ValueError("archive keys and values must share strides")
    for t_ in (bmean_k, bmean_v):
        if t_ is not None and (t_.dtype != torch.bfloat16 or t_.stride() != arc.kmax.stride()):
            raise ValueError("block means must be bf16 in the bounds' layout")
    n = 0 if k is None else k.shape[0]
    pos32 = pos.to(device=arc.keys.device, dtype=torch.int32).contiguous() if pos is not None else None
    if k is not None:
        k, v = k.to(torch.bfloat16), v.to(torch.bfloat16)
        if k.stride(-1) != 1 or v.stride() != k.stride():
            raise ValueError("k and v must share strides with a contiguous last dim")
    desc = _capi.PbkArchiveWriteDesc(
        kv=kv, d=d, block=block, origin=origin, cap=cap, size=size, p0=p0, n=n, blk_lo=blk_lo, blk_hi=blk_hi,
        pos=pos32.data_ptr() if pos32 is not None else None, k=k.data_ptr() if k is not None else None,
        v=v.data_ptr() if v is not None else None, in_stride_n=k.stride(0) if k is not None else 0,
        in_stride_kv=k.stride(1) if k is not None else 0, keys=arc.keys.data_ptr(), values=arc.values.data_ptr(),
        arc_stride_kv=arc.keys.stride(0), arc_stride_n=arc.keys.stride(1), kmax=arc.kmax.data_ptr(),
        kmin=arc.kmin.data_ptr(), kmean=bmean_k.data_ptr() if bmean_k is not None else None,
        vmean=bmean_v.data_ptr() if bmean_v is not None else None, bnd_stride_kv=arc.kmax.stride(0),
        bnd_stride_p=arc.kmax.stride(1))
    with torch.cuda.device(arc.keys.device):
        check(LIB.pbk_quest_archive_write(desc, torch.cuda.current_stream(arc.keys.device).cuda_stream),
              "pbk_quest_archive_write")


def _host_rows(t: torch.Tensor, rows: torch.Tensor, dev: torch.device) -> torch.Tensor:
    """Rows `rows` [KV, n] (int64, host) of a host tensor t [KV, N, D], per key head, into HBM
    [KV, n, D] through pinned memory."""
    kv, n = rows.shape
    buf = torch.empty(kv, n, t.shape[2], dtype=t.dtype, pin_memory=True)
    for h in range(kv):
        torch.index_select(t[h], 0, rows[h], out=buf[h])
    return buf.to(dev, non_blocking=True)


def _host_range(t: torch.Tensor, lo: int, hi: int, dev: torch.device) -> torch.Tensor:
    """Rows [lo, hi) of a host tensor [KV, N, D] into HBM, through pinned memory."""
    buf = torch.empty(t.shape[0], hi - lo, t.shape[2], dtype=t.dtype, pin_memory=True)
    buf.copy_(t[:, lo:hi])
    return buf.to(dev, non_blocking=True)


def _write_host(arc, block, size, blk_lo, blk_hi, k, v, p0, pos) -> None:
    dev = arc.kmax.device
    if k is not None:  # the new rows into the mapped archive
        kt, vt = k.to(arc.keys.dtype).transpose(0, 1).cpu(), v.to(arc.values.dtype).transpose(0, 1).cpu()
        if pos is None:
            arc.keys[:, p0:p0 + k.shape[0]] = kt
            arc.values[:, p0:p0 + k.shape[0]] = vt
        else:
            idx = pos.to("cpu", torch.int64)
            arc.keys[:, idx] = kt
            arc.values[:, idx] = vt
    if blk_hi < blk_lo:
        return
    end = size if pos is not None or k is None else max(size, p0 + k.shape[0])
    r_lo = ORIGIN + blk_lo * block
    r_hi = min(end, ORIGIN + (blk_hi + 1) * block, arc.keys.shape[1])
    if r_hi <= r_lo:
        return
    bmean_k, bmean_v = getattr(arc, "bmean_k", None), getattr(arc, "bmean_v", None)
    staged = types.SimpleNamespace(
        keys=_host_range(arc.keys, r_lo, r_hi, dev), values=_host_range(arc.values, r_lo, r_hi, dev),
        kmax=arc.kmax[:, blk_lo:], kmin=arc.kmin[:, blk_lo:],
        bmean_k=bmean_k[:, blk_lo:] if bmean_k is not None else None,
        bmean_v=bmean_v[:, blk_lo:] if bmean_v is not None else None)
    # the staged rows begin with block blk_lo: origin 0 there, every row already in place
    _write(staged, block, r_hi - r_lo, 0, blk_hi - blk_lo, origin=0)


def offload_archive(kv: int, d: int, cap: int, block: int, device: torch.device, directory: str | None = None):
    """A serving archive whose keys and values live in host memory backed by unlinked sparse
    files (the reference's NVMe offload format, memory.py:457-469: one raw bf16 [KV, cap, D]
    array per file; only the pages touched use disk or page cache), with every block and
    super-block summary in HBM. archive_write, retrieve_blocks and piece_attention accept it:
    new rows go to the files by device-to-host copies, and the rows a call reads (the blocks
    being summarised, the rerank's candidates, the attention's sinks, blocks, tail and window)
    are gathered on the host into pinned memory and copied to HBM for the same kernels."""
    import mmap
    import tempfile

    def mapped():
        nbytes = kv * cap * d * 2
        fd, path = tempfile.mkstemp(dir=directory, prefix="pbk_arc_")
        try:
            os.unlink(path)
            os.ftruncate(fd, nbytes)
            mm = mmap.mmap(fd, nbytes)
        except Exception:
            os.close(fd)
            raise
        return torch.frombuffer(mm, dtype=torch.bfloat16).view(kv, cap, d), (fd, mm)

    (keys, fk), (values, fv) = mapped(), mapped()
    n_blk = cap // block
    n_sb = (n_blk + SBLK - 1) // SBLK
    z = lambda rows: torch.zeros(kv, rows, d, dtype=torch.bfloat16, device=device)  # noqa: E731
    return types.SimpleNamespace(keys=keys, values=values, kmax=z(n_blk), kmin=z(n_blk), bmean_k=z(n_blk),
                                 bmean_v=z(n_blk), smax=z(n_sb), smin=z(n_sb), smean_k=z(n_sb), smean_v=z(n_sb),
                                 size=0, prompt_len=0, hole_lo=0, hole_hi=0, dirty_lo=1 << 60, dirty_hi=-1,
                                 mapped_files=[fk, fv])


def _update_super(arc, lo_b: int, hi_b: int, block: int) -> None:
    """Super-block bounds and means over the blocks [lo_b, hi_b] touched (memory.py:280-306)."""
    smax, smin = getattr(arc, "smax", None), getattr(arc, "smin", None)
    size = min(arc.keys.shape[1], getattr(arc, "size", arc.keys.shape[1]))
    if smax is None or smin is None or hi_b < lo_b or size <= ORIGIN:
        return
    n_blk = min(arc.kmax.shape[1], (size - ORIGIN + block - 1) // block)
    sb0 = max(0, lo_b // SBLK)
    sb1 = min(smax.shape[1] - 1, min(hi_b, max(0, n_blk - 1)) // SBLK)
    if sb1 < sb0:
        return
    super_bounds_(arc.kmax, arc.kmin, n_blk, SBLK, smax, smin, sb0, sb1 + 1)
    for src, dst in (("bmean_k", "smean_k"), ("bmean_v", "smean_v")):
        bm, sm = getattr(arc, src, None), getattr(arc, dst, None)
        if bm is None or sm is None:
            continue
        with torch.cuda.device(bm.device):
            check(LIB.pbk_quest_supermeans(bm.data_ptr(), bm.shape[0], n_blk, bm.shape[2], SBLK, bm.stride(0),
                                           bm.stride(1), sm.data_ptr(), sm.stride(0), sm.stride(1), sb0, sb1 + 1,
                                           torch.cuda.current_stream(bm.device).cuda_stream), "pbk_quest_supermeans")


def _refresh(arc, block: int) -> None:
    """Recompute the summaries of blocks [dirty_lo, dirty_hi] (max, min and the means the
    archive keeps) and of the super-blocks holding them (memory.py:280-306, 399-430)."""
    lo, hi = getattr(arc, "dirty_lo", 1 << 60), getattr(arc, "dirty_hi", -1)
    if hi < lo:
        return
    size = min(arc.keys.shape[1], getattr(arc, "size", arc.keys.shape[1]))
    hi_c = min(hi, arc.kmax.shape[1] - 1)
    if size > ORIGIN and hi_c >= lo:
        _write(arc, block, size, lo, hi_c)
    _update_super(arc, lo, hi, block)
    arc.dirty_lo, arc.dirty_hi = 1 << 60, -1


def _grow(arc, need: int, block: int) -> None:
    """Archive.grow (memory.py:225-278) for an archive in HBM: capacity doubled until it holds
    `need` rows; block and super-block arrays extended with zeros."""
    cap = arc.keys.shape[1]
    if need <= cap:
        return
    if not arc.keys.is_cuda:
        raise RuntimeError(f"offloaded archive full: need {need} rows > {cap}")
    new_cap = max(cap, 1)
    while new_cap < need:
        new_cap *= 2
    kv, d = arc.keys.shape[0], arc.keys.shape[2]
    for name in ("keys", "values"):
        old = getattr(arc, name)
        buf = torch.empty(kv, new_cap, d, dtype=old.dtype, device=old.device)
        buf[:, :cap] = old
        setattr(arc, name, buf)
    n_blk, n_sb = new_cap // block, (new_cap // block + SBLK - 1) // SBLK
    for names, rows in ((("kmax", "kmin", "bmean_k", "bmean_v"), n_blk), (("smax", "smin", "smean_k", "smean_v"), n_sb)):
        for name in names:
            old = getattr(arc, name, None)
            if old is not None and old.shape[1] < rows:
                buf = torch.zeros(kv, rows, d, dtype=old.dtype, device=old.device)
                buf[:, : old.shape[1]] = old
                setattr(arc, name, buf)


def archive_write(arc, pos: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block: int, p0: int | None = None,
                  hi: int | None = None) -> None:
    """Archive.write (memory.py:310-395) for an archive in HBM: k/v [N, KV, D] stored at
    positions pos [N] (grown as needed). A contiguous write (pos = p0 .. hi - 1) summarises
    every block it touches as it writes them, one pass over the new rows
    (pbk_quest_archive_write), then the super-blocks holding them; the reference summarises
    full blocks at once and the partial ends at the next retrieval, which reads the same
    summaries. Other writes scatter the rows and leave their blocks dirty for the next
    refresh, as the reference does."""
    if p0 is None or hi is None:
        hi = int(pos.max()) + 1
        p0 = int(pos.min())
    n = int(pos.numel())
    contig = hi - p0 == n
    _grow(arc, hi, block)
    size = getattr(arc, "size", 0)
    lo_b, hi_b = max(0, p0 - ORIGIN) // block, (hi - 1 - ORIGIN) // block
    if contig:
        blk_hi = min(hi_b, arc.kmax.shape[1] - 1) if hi - 1 >= ORIGIN else -1
        _write(arc, block, size, lo_b, blk_hi, k, v, p0=p0)
        arc.size = max(size, hi)
        if hi - 1 >= ORIGIN:
            _update_super(arc, lo_b, hi_b, block)
        return
    _write(arc, block, size, 0, -1, k, v, pos=pos)
    arc.size = max(size, hi)
    if hi - 1 >= ORIGIN:
        arc.dirty_lo = min(getattr(arc, "dirty_lo", 1 << 60), lo_b)
        arc.dirty_hi = max(getattr(arc, "dirty_hi", -1), hi_b)


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
    _refresh(arc, block)
    qi = q.to(torch.bfloat16).unsqueeze(0)                        # [1, T, H, D]
    qs = qi
    if limit > ROPE_HORIZON:  # memory.py:795-797: the RoPE'd dims do not score the bounds
        qs = qi.clone()
        qs[..., : d // 4] = 0
    kmax, kmin = arc.kmax[:, :full], arc.kmin[:, :full]
    smax, smin = getattr(arc, "smax", None), getattr(arc, "smin", None)

    def select(kk: int) -> torch.Tensor:
        if hole != (0, 0):
            return select_pages_levels(qs, kmax, kmin, full * block, block, kk, hole=hole)
        return select_pages(qs, kmax, kmin, full * block, block, kk)

    if not rerank and SBLK > 1 and smax is not None and smin is not None and full > SBLK * 16:
        pages = select_pages_levels(qs, kmax, kmin, full * block, block, k, smax, smin, SBLK, hole)
    elif rerank and pool > k:
        cand = select(min(pool, n_valid))                         # [1, KV, c] ascending
        if not arc.keys.is_cuda:  # the candidates' blocks staged from the host archive
            if limit > ROPE_HORIZON:
                raise NotImplementedError("RoPE moves on an offloaded archive")
            c = cand.shape[-1]
            rows = (ORIGIN + cand[0].long().cpu()[:, :, None] * block + torch.arange(block)).reshape(cand.shape[1], -1)
            ck = _host_rows(arc.keys, rows, q.device)
            ident = torch.arange(c, dtype=torch.int32, device=q.device).expand(1, cand.shape[1], c).contiguous()
            pages = cand.gather(-1, rerank_pages(qi, ck, ident, block, k).long()).to(torch.int32)
        elif limit > ROPE_HORIZON:  # the candidates' keys moved in proportion (memory.py:861-862)
            c = cand.shape[-1]
            ck, _ = rope_gather(arc.keys, None, cand[0], block, ORIGIN, c, "proportional", ref_pos=limit)
            ident = torch.arange(c, dtype=torch.int32, device=q.device).expand(1, cand.shape[1], c).contiguous()
            pages = cand.gather(-1, rerank_pages(qi, ck, ident, block, k).long()).to(torch.int32)
        else:
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
    if own is not None:  # the reference's selectors return none (memory.py:1023, 1140, 1294)
        raise NotImplementedError("per-query own-block masks")
    block = MEMORY["block_size"]
    t, h, d = q.shape
    if q_min is None or q_max is None:
        q_min, q_max = int(q_pos.min()), int(q_pos.max())
    lo, hi = max(0, q_min - window + 1), q_max + 1
    ns = min(SINKS, lo)
    qi = q.to(torch.bfloat16).unsqueeze(0)
    out = torch.empty(1, t, h, d, dtype=torch.float32, device=q.device)
    qpos = q_pos.to(device=q.device, dtype=torch.int32).view(1, t)
    kpos = torch.arange(lo, hi, dtype=torch.int32, device=q.device)
    win = (arc.keys[:, lo:hi], arc.values[:, lo:hi], kpos, window, 0, scale, out)
    rope = lo > ROPE_HORIZON  # sinks and retrieved blocks move to new RoPE positions (memory.py:1402-1425)
    n_blk = top.shape[1] if top is not None else 0
    if not arc.keys.is_cuda:
        if rope:
            raise NotImplementedError("RoPE moves on an offloaded archive")
        return _piece_attention_host(arc, qi, qpos, kpos, top, groups, window, scale, lo, hi, ns, block, out, q.dtype)
    sink_k, sink_v = arc.keys, arc.values
    shift = sink_shift(lo, ns, n_blk, block) if rope else 0
    if shift > 0:
        sink_k, sink_v = rope_gather(arc.keys, arc.values, None, ns, 0, 1, "constant", const_delta=shift)
    n_land = _landmark_count(arc, lo, block)
    if n_land > 0:  # dense global aggregation: the super-block mean keys follow the sinks (memory.py:1332, 1411-1416)
        land_k = _move_landmarks(arc.smean_k[:, :n_land].to(torch.bfloat16), block, lo)
        sink_k = torch.cat((sink_k[:, :ns].to(torch.bfloat16), land_k), dim=1)
        sink_v = torch.cat((sink_v[:, :ns].to(torch.bfloat16), arc.smean_v[:, :n_land].to(torch.bfloat16)), dim=1)
        ns += n_land
    if top is not None:  # the reference's cache of the last retrieved set (memory.py:1427-1436)
        arc.cached_top = top if getattr(arc, "prompt_top", None) is not None else None
    if top is not None and rope:  # [moved blocks ; partial block before the window], gathered
        tail0 = ORIGIN + ((lo - ORIGIN) // block) * block
        tail_n = lo - tail0 if lo > tail0 else 0
        rk, rv = rope_gather(arc.keys, arc.values, top, block, ORIGIN, n_blk, "runs", ref_pos=lo, tail0=tail0,
                             tail_n=tail_n)
        ident = torch.arange(n_blk, dtype=torch.int32, device=q.device).expand(1, h // groups, n_blk).contiguous()
        desc = _attend_desc(qi, qpos, rk, rv, n_blk * block + tail_n, block, ident, *win)
    elif top is not None:  # retrieved blocks + the partial block before the window, in place
        desc = _attend_desc(qi, qpos, arc.keys[:, ORIGIN:], arc.values[:, ORIGIN:], max(0, lo - ORIGIN), block,
                            top.to(torch.int32).unsqueeze(0).contiguous(), *win)
    else:  # sinks and window only: no archive part
        dummy = torch.zeros(1, h // groups, 1, dtype=torch.int32, device=q.device)
        desc = _attend_desc(qi, qpos, arc.keys, arc.values, block, block, dummy, *win)
        desc.n_arch, desc.budget = 0, 0
    ws = _workspace(LIB.pbk_quest_attend_sinks_workspace(desc, ns), q.device)
    with torch.cuda.device(q.device):
        check(LIB.pbk_quest_attend_sinks(desc, sink_k.data_ptr(), sink_v.data_ptr(), ns, sink_k.stride(0),
                                         sink_k.stride(1), ws.data_ptr(), ws.numel(),
                                         torch.cuda.current_stream(q.device).cuda_stream),
              "pbk_quest_attend_sinks")
    return out[0].to(q.dtype)


def _landmark_count(arc, lo: int, block: int) -> int:
    """Super-block landmarks a piece sees under dense global aggregation: the super-blocks
    wholly before its window (memory.py:1332)."""
    if not getattr(arc, "is_global_agg", False):
        return 0
    if getattr(arc, "smean_k", None) is None or getattr(arc, "smean_v", None) is None:
        return 0
    return max(0, ((lo - ORIGIN) // block) // SBLK)


def _move_landmarks(smk: torch.Tensor, block: int, ref_pos: int) -> torch.Tensor:
    """Past ROPE_HORIZON, super-block landmark keys [KV, n, D] at their centres ORIGIN + (i +
    1/2) * SBLK * block move toward ref_pos in proportion (memory.py:680-711): the pairs (i,
    i + d/8) of the first d/4 dims turn by delta * inv_freq, in fp32."""
    if ROPE_HORIZON <= 0 or ref_pos <= ROPE_HORIZON or smk.numel() == 0:
        return smk
    kv, n_sb, d = smk.shape
    d_rot = d // 4
    half = d_rot // 2
    scale = 1.0 - min(1.0, float(ROPE_ARC_SPAN) / float(max(1, ref_pos)))
    orig = float(ORIGIN) + (torch.arange(n_sb, device=smk.device, dtype=torch.float32) + 0.5) * float(SBLK * block)
    delta = (orig + torch.round((float(ref_pos) - orig).clamp(min=0.0) * scale) - orig).clamp(min=0.0)
    ang = delta[None, :, None] * _inv_freq(smk.device, d_rot)
    cos, sin = ang.cos(), ang.sin()
    x1, x2 = smk[..., :half].float(), smk[..., half:d_rot].float()
    out = smk.clone()
    out[..., :half] = (x1 * cos - x2 * sin).to(smk.dtype)
    out[..., half:d_rot] = (x2 * cos + x1 * sin).to(smk.dtype)
    return out


def _piece_attention_host(arc, qi, qpos, kpos, top, groups, window, scale, lo, hi, ns, block, out, dtype):
    """piece_attention over an offloaded archive: the sinks, the retrieved blocks with the
    partial block before the window, and the window are gathered on the host and copied to
    HBM, then attended as an archive of the retrieved blocks in order (the same kernel and key
    order as the in-HBM archive)."""
    dev = qi.device
    kv = arc.keys.shape[0]
    h = qi.shape[2]
    wk, wv = _host_range(arc.keys, lo, hi, dev), _host_range(arc.values, lo, hi, dev)
    if ns > 0:
        sk, sv = _host_range(arc.keys, 0, ns, dev), _host_range(arc.values, 0, ns, dev)
    else:
        sk, sv = wk, wv
    n_land = _landmark_count(arc, lo, block)
    if n_land > 0:  # the super-block landmarks (in HBM) after the sinks
        sk = torch.cat((sk[:, :ns], arc.smean_k[:, :n_land].to(torch.bfloat16)), dim=1)
        sv = torch.cat((sv[:, :ns], arc.smean_v[:, :n_land].to(torch.bfloat16)), dim=1)
        ns += n_land
    win = (wk, wv, kpos, window, 0, scale, out)
    if top is not None:
        n_blk = top.shape[1]
        tail0 = ORIGIN + ((lo - ORIGIN) // block) * block
        tail = torch.arange(tail0, lo) if lo > tail0 else torch.zeros(0, dtype=torch.int64)
        blk_rows = (ORIGIN + top.long().cpu()[:, :, None] * block + torch.arange(block)).reshape(kv, -1)
        rows = torch.cat((blk_rows, tail[None].expand(kv, -1)), dim=1)
        rk, rv = _host_rows(arc.keys, rows, dev), _host_rows(arc.values, rows, dev)
        ident = torch.arange(n_blk, dtype=torch.int32, device=dev).expand(1, h // groups, n_blk).contiguous()
        desc = _attend_desc(qi, qpos, rk, rv, n_blk * block + tail.numel(), block, ident, *win)
    else:
        dummy = torch.zeros(1, h // groups, 1, dtype=torch.int32, device=dev)
        desc = _attend_desc(qi, qpos, wk, wv, block, block, dummy, *win)
        desc.n_arch, desc.budget = 0, 0
    ws = _workspace(LIB.pbk_quest_attend_sinks_workspace(desc, ns), dev)
    with torch.cuda.device(dev):
        check(LIB.pbk_quest_attend_sinks(desc, sk.data_ptr(), sv.data_ptr(), ns, sk.stride(0), sk.stride(1),
                                         ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream),
              "pbk_quest_attend_sinks")
    return out[0].to(dtype)
