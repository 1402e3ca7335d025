"""Quest page-bounded exact memory on B200: drop-in for pseudobrain/exact_memory.py.

Same names and meanings as the reference (pseudobrain/exact_memory.py:20-152):

    EXACT_MEMORY                                  configuration dict
    Archive(keys, values, kmax, kmin, ...)        evicted keys/values [B,KV,N,hd] + page bounds
    archive_append(archive, keys, values)        -> Archive
    retrieve(archive, q, groups)                 -> (keys, values) [B,KV,R,hd] or None

plus the fused path of this build, which never materialises the gathered keys:

    select_pages(...)         page scores + exact top-k   (pbk_quest_select)
    attend_pages(...)         split-key exact attention over pages + tail + window (pbk_quest_attend)
    select_attend_pages(...)  both, the window half overlapped with the top-k
                              (pbk_quest_select_parts, pbk_quest_attend_parts)
    retrieve_attend(...)      the same for one Archive, with the reference's mask
                              (pseudobrain/transplant.py:612-628)

``retrieve`` takes every selection mode of the reference: flat, the two-level
super-block selection of decode queries (pbk_quest_select_levels over the super-block
bounds that ``archive_append`` keeps), the exact ``rerank`` (pbk_quest_rerank), a kept
prompt selection and ``neighbors``. Keys are bf16 with head_dim 128 or 256 (256 on the SIMT
kernels: the tensor-core score and attention kernels are written for 128); every call runs CUDA
kernels from libpbk.so and there is no CPU path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _capi
from ._capi import LIB, PbkQuestDesc, PbkQuestLevels, check

EXACT_MEMORY = {"enabled": False, "blocks": 64, "block_size": 64, "decode_blocks": 64, "neighbors": 0, "rerank": 0,
                "decode_rerank": 0, "superblock": 64, "keys_like_values": False}


@dataclass
class Archive:
    """Evicted rotated keys/values [B,KV,N,hd] and per-page bounds [B,KV,pages,hd]
    (reference: exact_memory.py:27-40)."""
    keys: torch.Tensor
    values: torch.Tensor
    kmax: torch.Tensor
    kmin: torch.Tensor
    smax: torch.Tensor | None = None
    smin: torch.Tensor | None = None
    prompt_top: torch.Tensor | None = None

    @property
    def length(self) -> int:
        return self.keys.shape[2]


def _require(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what}: pseudobrain_b200 runs on CUDA only (no CPU fallback)")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{what}: bf16 expected, got {t.dtype}")
    if t.shape[-1] not in (128, 256) or t.stride(-1) != 1:
        raise ValueError(f"{what}: head_dim must be 128 or 256 and contiguous")


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def page_bounds_(keys: torch.Tensor, page: int, kmax: torch.Tensor, kmin: torch.Tensor, first_page: int = 0) -> None:
    """Write the bounds of pages first_page.. of keys [KV,N,hd] into kmax/kmin [KV,P,hd]
    (reference: _bounds, exact_memory.py:43-50)."""
    _require(keys, "keys")
    kv, n, d = keys.shape
    if kmax.shape != kmin.shape or kmax.shape[0] != kv or kmax.shape[1] < (n + page - 1) // page:
        raise ValueError(f"bounds {tuple(kmax.shape)} too small for {n} keys in pages of {page}")
    _require(kmax, "kmax")
    _require(kmin, "kmin")
    with torch.cuda.device(keys.device):
        check(LIB.pbk_quest_bounds(keys.data_ptr(), kv, n, d, page, keys.stride(0), keys.stride(1), kmax.data_ptr(),
                                   kmin.data_ptr(), kmax.stride(0), kmax.stride(1), first_page, _stream(keys)),
              "pbk_quest_bounds")


def page_bounds(keys: torch.Tensor, page: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(kmax, kmin) [B,KV,ceil(N/page),hd] of keys [B,KV,N,hd]."""
    b, kv, n, d = keys.shape
    p = (n + page - 1) // page
    kmax = torch.empty(b, kv, p, d, dtype=keys.dtype, device=keys.device)
    kmin = torch.empty_like(kmax)
    for i in range(b):
        page_bounds_(keys[i], page, kmax[i], kmin[i])
    return kmax, kmin


def super_bounds_(kmax: torch.Tensor, kmin: torch.Tensor, n_blk: int, sblk: int, smax: torch.Tensor,
                  smin: torch.Tensor, first_sb: int = 0, end_sb: int | None = None) -> None:
    """Write the bounds of super-blocks [first_sb, end_sb) (all from first_sb when None) of
    the pages [0, n_blk) of kmax/kmin [KV,P,hd] into smax/smin [KV,S,hd]: the max of sblk
    consecutive page maxima and the min of their minima, a trailing partial super-block over
    the pages it holds (reference: _superbounds, exact_memory.py:53-63;
    Archive._update_superbounds, pb27_vllm/memory.py:280-306)."""
    for t_, w in ((kmax, "kmax"), (kmin, "kmin"), (smax, "smax"), (smin, "smin")):
        _require(t_, w)
    kv, _, d = kmax.shape
    n_sb = (n_blk + sblk - 1) // sblk
    end = n_sb if end_sb is None else min(end_sb, n_sb)
    if smax.shape != smin.shape or smax.shape[0] != kv or smax.shape[1] < end:
        raise ValueError(f"super-block bounds {tuple(smax.shape)} too small for {end} super-blocks")
    with torch.cuda.device(kmax.device):
        check(LIB.pbk_quest_superbounds(kmax.data_ptr(), kmin.data_ptr(), kv, n_blk, d, sblk, kmax.stride(0),
                                        kmax.stride(1), smax.data_ptr(), smin.data_ptr(), smax.stride(0),
                                        smax.stride(1), first_sb, end, _stream(kmax)), "pbk_quest_superbounds")


def super_bounds(kmax: torch.Tensor, kmin: torch.Tensor, sblk: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(smax, smin) [B,KV,ceil(P/sblk),hd] of page bounds [B,KV,P,hd] (exact_memory.py:53-63)."""
    b, kv, p, d = kmax.shape
    smax = torch.empty(b, kv, (p + sblk - 1) // sblk, d, dtype=kmax.dtype, device=kmax.device)
    smin = torch.empty_like(smax)
    for i in range(b):
        super_bounds_(kmax[i], kmin[i], p, sblk, smax[i], smin[i])
    return smax, smin


def _superblock() -> int:
    return int(EXACT_MEMORY.get("superblock", 64) or 0)


def archive_append(archive: Archive | None, keys: torch.Tensor, values: torch.Tensor) -> Archive | None:
    """Append evicted keys/values and refresh the page bounds from the first incomplete page
    on, and the super-block bounds from the super-block holding it (reference:
    exact_memory.py:66-85; super-blocks of EXACT_MEMORY["superblock"] pages when > 1)."""
    if keys.shape[2] == 0:
        return archive
    page = EXACT_MEMORY["block_size"]
    sblk = _superblock()
    if EXACT_MEMORY["keys_like_values"]:
        keys = keys.to(values.dtype)
    if archive is None:
        kmax, kmin = page_bounds(keys, page)
        smax, smin = super_bounds(kmax, kmin, sblk) if sblk > 1 else (None, None)
        return Archive(keys, values, kmax, kmin, smax, smin)
    full = archive.length // page
    new_k = torch.cat((archive.keys, keys), dim=2)
    new_v = torch.cat((archive.values, values), dim=2)
    b, kv, n, d = new_k.shape
    p = (n + page - 1) // page
    kmax = torch.empty(b, kv, p, d, dtype=new_k.dtype, device=new_k.device)
    kmin = torch.empty_like(kmax)
    kmax[:, :, :full] = archive.kmax[:, :, :full]
    kmin[:, :, :full] = archive.kmin[:, :, :full]
    for i in range(b):
        page_bounds_(new_k[i], page, kmax[i], kmin[i], first_page=full)
    smax = smin = None
    if sblk > 1:
        first_sb = full // sblk  # earlier super-blocks hold complete pages only: final
        smax = torch.empty(b, kv, (p + sblk - 1) // sblk, d, dtype=kmax.dtype, device=kmax.device)
        smin = torch.empty_like(smax)
        if archive.smax is not None and archive.smin is not None and first_sb > 0:
            smax[:, :, :first_sb] = archive.smax[:, :, :first_sb]
            smin[:, :, :first_sb] = archive.smin[:, :, :first_sb]
        else:
            first_sb = 0
        for i in range(b):
            super_bounds_(kmax[i], kmin[i], p, sblk, smax[i], smin[i], first_sb)
    return Archive(new_k, new_v, kmax, kmin, smax, smin, archive.prompt_top)


def _desc(q: torch.Tensor, page: int, n_arch: int, budget: int, *, kmax=None, kmin=None, keys=None, values=None,
          pages=None, scores=None) -> PbkQuestDesc:
    """q [nq, t, h, 128] bf16 (any strides with a contiguous last dim)."""
    _require(q, "q")
    nq, t, h, d = q.shape
    kv = (kmax if kmax is not None else keys).shape[0]
    desc = PbkQuestDesc(nq=nq, t=t, h=h, kv=kv, d=d, page=page, n_arch=n_arch, budget=budget,
                        q=q.data_ptr(), q_stride_n=q.stride(0), q_stride_t=q.stride(1), q_stride_h=q.stride(2),
                        pages=_ptr(pages), scores=_ptr(scores))
    if kmax is not None:
        desc.kmax, desc.kmin = kmax.data_ptr(), kmin.data_ptr()
        desc.bnd_stride_kv, desc.bnd_stride_p = kmax.stride(0), kmax.stride(1)
    if keys is not None:
        desc.keys, desc.values = keys.data_ptr(), values.data_ptr()
        desc.arc_stride_kv, desc.arc_stride_n = keys.stride(0), keys.stride(1)
    return desc


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)


def select_pages(q: torch.Tensor, kmax: torch.Tensor, kmin: torch.Tensor, n_arch: int, page: int, budget: int,
                 scores: torch.Tensor | None = None) -> torch.Tensor:
    """Top pages per (query group, key head): q [nq,t,h,128]; kmax/kmin [KV,P,128] bf16 over
    the archive's n_arch tokens (complete pages n_arch // page are candidates). Returns int32
    [nq, KV, min(budget, n_arch // page)], ascending; ties go to the lowest page. ``scores``
    (fp32 [nq,KV,n_arch // page]) receives the page scores when given."""
    _require(kmax, "kmax")
    _require(kmin, "kmin")
    nq = q.shape[0]
    kv = kmax.shape[0]
    k = min(budget, n_arch // page)
    pages = torch.empty(nq, kv, k, dtype=torch.int32, device=q.device)
    desc = _desc(q, page, n_arch, budget, kmax=kmax, kmin=kmin, pages=pages, scores=scores)
    ws = _workspace(LIB.pbk_quest_select_workspace(desc), q.device)
    with torch.cuda.device(q.device):
        check(LIB.pbk_quest_select(desc, ws.data_ptr(), ws.numel(), _stream(q)), "pbk_quest_select")
    return pages


def m_superblocks(k: int, full: int, sblk: int) -> int:
    """Super-blocks the two-level selection keeps for k pages (exact_memory.py:116,
    pb27_vllm/memory.py:814): min(max(16, ceil(2k / sblk)), ceil(full / sblk))."""
    return min(max(16, (2 * k + sblk - 1) // sblk), (full + sblk - 1) // sblk)


def select_pages_levels(q: torch.Tensor, kmax: torch.Tensor, kmin: torch.Tensor, n_arch: int, page: int,
                        budget: int, smax: torch.Tensor | None = None, smin: torch.Tensor | None = None,
                        sblk: int = 0, hole: tuple[int, int] = (0, 0)) -> torch.Tensor:
    """select_pages with the reference's other scoring modes (pbk_quest_select_levels): with
    super-block bounds smax/smin [KV,S,128] and sblk > 1, the two-level selection
    (exact_memory.py:107-122, pb27_vllm/memory.py:802-836): the best m_superblocks(k) super-
    blocks, then the best min(k, m_sb * sblk) of their pages; pages [hole) score -inf
    (memory.py:834-835, 852-853). k = min(budget, n_arch // page): a caller whose hole leaves
    fewer pages passes the smaller budget. Returns int32 [nq, KV, k'] ascending."""
    _require(kmax, "kmax")
    _require(kmin, "kmin")
    nq = q.shape[0]
    kv = kmax.shape[0]
    full = n_arch // page
    k = min(budget, full)
    lv = PbkQuestLevels(hole_lo=int(hole[0]), hole_hi=int(hole[1]))
    if smax is not None:
        _require(smax, "smax")
        _require(smin, "smin")
        if sblk < 2:
            raise ValueError("two-level selection needs sblk >= 2")
        lv.smax, lv.smin = smax.data_ptr(), smin.data_ptr()
        lv.sb_stride_kv, lv.sb_stride_p = smax.stride(0), smax.stride(1)
        lv.sblk = sblk
        lv.m_sb = m_superblocks(k, full, sblk) if full else 0
        k = min(k, lv.m_sb * sblk)
    pages = torch.empty(nq, kv, k, dtype=torch.int32, device=q.device)
    desc = _desc(q, page, n_arch, budget, kmax=kmax, kmin=kmin, pages=pages)
    ws = _workspace(LIB.pbk_quest_select_levels_workspace(desc, lv), q.device)
    with torch.cuda.device(q.device):
        check(LIB.pbk_quest_select_levels(desc, lv, ws.data_ptr(), ws.numel(), _stream(q)), "pbk_quest_select_levels")
    return pages


def rerank_pages(q: torch.Tensor, keys: torch.Tensor, cand: torch.Tensor, page: int, k: int) -> torch.Tensor:
    """Exact rerank (exact_memory.py:126-133, pb27_vllm/memory.py:854-872): each candidate page
    of cand [nq,KV,c] int32 (ascending) scores the max over the head's query rows and the
    page's tokens of q.k (fp32 on bf16 keys [KV,N,128]); the best k (ties to the lowest) are
    returned as int32 [nq,KV,k] ascending (pbk_quest_rerank)."""
    _require(keys, "keys")
    nq, kv, c = cand.shape
    k = min(k, c)
    pages = torch.empty(nq, kv, k, dtype=torch.int32, device=q.device)
    cand = cand.to(torch.int32).contiguous()
    desc = _desc(q, page, keys.shape[1], k, keys=keys, values=keys, pages=pages)
    ws = _workspace(LIB.pbk_quest_rerank_workspace(desc, c), q.device)
    with torch.cuda.device(q.device):
        check(LIB.pbk_quest_rerank(desc, cand.data_ptr(), c, ws.data_ptr(), ws.numel(), _stream(q)), "pbk_quest_rerank")
    return pages


def _attend_desc(q, qpos, keys, values, n_arch, page, pages, win_keys, win_values, kpos, window, sinks, scale, out):
    """Descriptor of an attention call (see attend_pages); `out` [nq,t,h,128] receives it."""
    for t_, w in ((keys, "keys"), (values, "values"), (win_keys, "win_keys"), (win_values, "win_values")):
        _require(t_, w)
    nq, t, h, d = q.shape
    desc = _desc(q, page, n_arch, pages.shape[-1], keys=keys, values=values, pages=pages)
    desc.n_win, desc.window, desc.sinks = win_keys.shape[1], window, sinks
    desc.scale = float(d ** -0.5 if scale is None else scale)
    desc.qpos, desc.kpos = qpos.data_ptr(), kpos.data_ptr()
    desc.win_keys, desc.win_values = win_keys.data_ptr(), win_values.data_ptr()
    desc.win_stride_kv, desc.win_stride_n = win_keys.stride(0), win_keys.stride(1)
    desc.out = out.data_ptr()
    desc.out_stride_n, desc.out_stride_t, desc.out_stride_h = out.stride(0), out.stride(1), out.stride(2)
    desc.out_dtype = _capi.PBK_BF16 if out.dtype == torch.bfloat16 else _capi.PBK_F32
    if qpos.dtype != torch.int32 or kpos.dtype != torch.int32:
        raise TypeError("qpos and kpos must be int32")
    if pages.shape[:2] != (nq, keys.shape[0]) or pages.dtype != torch.int32 or not pages.is_contiguous():
        raise ValueError("pages must be contiguous int32 [nq, KV, k]")
    if pages.shape[-1] > n_arch // page:
        raise ValueError("more selected pages than complete archive pages")
    return desc


def attend_pages(q: torch.Tensor, qpos: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, n_arch: int,
                 page: int, pages: torch.Tensor, win_keys: torch.Tensor, win_values: torch.Tensor,
                 kpos: torch.Tensor, window: int, sinks: int = 0, scale: float | None = None,
                 out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Exact attention of q [nq,t,h,128] (positions qpos [nq,t] int32) over, per key head,
    the selected pages [nq,KV,k] of keys/values [KV,N,128], the archive's partial tail and
    the window keys win_keys/win_values [KV,S,128] at positions kpos [S] int32 under the
    reference's window mask. Returns [nq,t,h,128]."""
    nq, t, h, d = q.shape
    out = torch.empty(nq, t, h, d, dtype=out_dtype, device=q.device)
    desc = _attend_desc(q, qpos, keys, values, n_arch, page, pages, win_keys, win_values, kpos, window, sinks,
                        scale, out)
    ws = _workspace(LIB.pbk_quest_attend_workspace(desc), q.device)
    with torch.cuda.device(q.device):
        check(LIB.pbk_quest_attend(desc, ws.data_ptr(), ws.numel(), _stream(q)), "pbk_quest_attend")
    return out


_SIDE: dict[int, torch.cuda.Stream] = {}


def _side_stream(dev: torch.device) -> torch.cuda.Stream:
    """One auxiliary high-priority stream per device (made on the first call, outside any
    graph capture): the block scheduler dispatches its blocks before the default-priority
    stream's."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _SIDE:
        _SIDE[idx] = torch.cuda.Stream(dev, priority=-1)
    return _SIDE[idx]


def select_attend_pages(q: torch.Tensor, qpos: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                        kmax: torch.Tensor, kmin: torch.Tensor, n_arch: int, page: int, budget: int,
                        win_keys: torch.Tensor, win_values: torch.Tensor, kpos: torch.Tensor, window: int,
                        sinks: int = 0, scale: float | None = None, out_dtype: torch.dtype = torch.float32):
    """select_pages followed by attend_pages (same arguments and results: (pages, out)), with
    the window half of the attention overlapped with the top-k selection: the page scores
    first, then on a side stream the window keys' partials while the top-k runs, then the
    selected pages' partials and the combine (pbk_quest_select_parts, pbk_quest_attend_parts).
    The window half needs no selected page, and the top-k occupies one SM per (query, key head)
    row, leaving the others idle. Graph capturable (fork and join through the side stream)."""
    _require(kmax, "kmax")
    _require(kmin, "kmin")
    dev = q.device
    nq, t, h, d = q.shape
    kv = kmax.shape[0]
    k = min(budget, n_arch // page)
    pages = torch.empty(nq, kv, k, dtype=torch.int32, device=dev)
    out = torch.empty(nq, t, h, d, dtype=out_dtype, device=dev)
    sdesc = _desc(q, page, n_arch, budget, kmax=kmax, kmin=kmin, pages=pages)
    adesc = _attend_desc(q, qpos, keys, values, n_arch, page, pages, win_keys, win_values, kpos, window, sinks,
                         scale, out)
    sws = _workspace(LIB.pbk_quest_select_workspace(sdesc), dev)
    aws = _workspace(LIB.pbk_quest_attend_workspace(adesc), dev)
    side = _side_stream(dev)
    with torch.cuda.device(dev):
        cur = torch.cuda.current_stream(dev)
        check(LIB.pbk_quest_select_parts(sdesc, 1, sws.data_ptr(), sws.numel(), cur.cuda_stream),
              "pbk_quest_select_parts (scores)")
        # the top-k and the pages' attention on the high-priority side stream (the top-k's
        # blocks are dispatched first), the window's attention beside them on this stream
        side.wait_stream(cur)  # after the persistent score kernel, which holds every SM
        check(LIB.pbk_quest_select_parts(sdesc, 2, sws.data_ptr(), sws.numel(), side.cuda_stream),
              "pbk_quest_select_parts (top-k)")
        check(LIB.pbk_quest_attend_parts(adesc, None, None, 0, 0, 0, 1, aws.data_ptr(), aws.numel(), side.cuda_stream),
              "pbk_quest_attend_parts (pages)")
        check(LIB.pbk_quest_attend_parts(adesc, None, None, 0, 0, 0, 2, aws.data_ptr(), aws.numel(), cur.cuda_stream),
              "pbk_quest_attend_parts (window)")
        cur.wait_stream(side)
        check(LIB.pbk_quest_attend_parts(adesc, None, None, 0, 0, 0, 4, aws.data_ptr(), aws.numel(), cur.cuda_stream),
              "pbk_quest_attend_parts (combine)")
    # the current stream joined the side stream before the combine, so later work (and the
    # allocator's reuse of the workspaces and `pages`) on it is ordered after the side stream
    return pages, out


def gather_pages(keys: torch.Tensor, values: torch.Tensor, n_arch: int, page: int, pages: torch.Tensor,
                 q: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Keys/values of `pages` [nq,KV,sel] followed by the partial tail: [nq,KV,sel*page+tail,128]."""
    nq, kv, sel = pages.shape
    if pages.dtype != torch.int32 or not pages.is_contiguous() or q.shape[0] != nq:
        raise ValueError("pages must be contiguous int32 [nq, KV, sel] with nq query groups")
    rows = sel * page + n_arch % page
    ok = torch.empty(nq, kv, rows, keys.shape[-1], dtype=keys.dtype, device=keys.device)
    ov = torch.empty_like(ok)
    desc = _desc(q, page, n_arch, sel, keys=keys, values=values, pages=pages)
    with torch.cuda.device(keys.device):
        check(LIB.pbk_quest_gather(desc, sel, ok.data_ptr(), ov.data_ptr(), _stream(keys)), "pbk_quest_gather")
    return ok, ov


def _budget(t: int) -> tuple[int, bool]:
    is_decode = t <= 64
    budget = (EXACT_MEMORY["decode_blocks"] if (is_decode and EXACT_MEMORY["decode_blocks"])
              else EXACT_MEMORY["blocks"])
    return budget, is_decode


def _mode(archive: Archive, full: int, k: int, is_decode: bool) -> str:
    """Which selection retrieve makes (exact_memory.py:107, :126): 'levels', 'rerank' or 'flat'."""
    sblk = _superblock()
    rerank = int(EXACT_MEMORY.get("decode_rerank", 0) if is_decode else EXACT_MEMORY.get("rerank", 0))
    if (is_decode and rerank <= k and sblk > 1 and archive.smax is not None and archive.smin is not None
            and full > sblk * 16):
        return "levels"
    return "rerank" if rerank > k else "flat"


def _select(archive: Archive, i: int, qi: torch.Tensor, full: int, budget: int, is_decode: bool) -> torch.Tensor:
    """int32 [1, KV, k] pages of batch row i for the query group qi [1,T,H,128]."""
    k = min(budget, full)
    mode = _mode(archive, full, k, is_decode)
    page = EXACT_MEMORY["block_size"]
    if mode == "levels":
        return select_pages_levels(qi, archive.kmax[i], archive.kmin[i], archive.length, page, budget,
                                   archive.smax[i], archive.smin[i], _superblock())
    if mode == "rerank":
        c = int(EXACT_MEMORY.get("decode_rerank", 0) if is_decode else EXACT_MEMORY.get("rerank", 0))
        cand = select_pages(qi, archive.kmax[i], archive.kmin[i], archive.length, page, min(c, full))
        return rerank_pages(qi, archive.keys[i], cand, page, k)
    return select_pages(qi, archive.kmax[i], archive.kmin[i], archive.length, page, budget)


def retrieve(archive: Archive | None, q: torch.Tensor, groups: int) -> tuple[torch.Tensor, torch.Tensor] | None:
    """Top pages per key head for query chunk q [B,H,T,hd]: (keys, values) [B,KV,R,hd] or None
    (reference: exact_memory.py:88-152: the flat, two-level and rerank selections,
    ``prompt_top`` and ``neighbors`` behave as there)."""
    if archive is None or archive.length == 0:
        return None
    page = EXACT_MEMORY["block_size"]
    b, h, t, d = q.shape
    full = archive.length // page
    out_k, out_v = [], []
    budget, is_decode = _budget(t)
    qs = q.to(torch.bfloat16)
    tops = []
    for i in range(b):
        qi = qs[i].transpose(0, 1).unsqueeze(0)  # [1, T, H, hd] view
        top = (_select(archive, i, qi, full, budget, is_decode)[0]
               if full else torch.empty(h // groups, 0, dtype=torch.int32, device=q.device))
        tops.append(top)
    top = torch.stack(tops).long()
    if full:
        if not is_decode:
            archive.prompt_top = top
        elif archive.prompt_top is not None:
            top = torch.cat((archive.prompt_top.clamp(max=full - 1), top), dim=-1)
        if EXACT_MEMORY["neighbors"]:
            top = torch.cat([top] + [(top + j).clamp(max=full - 1) for j in range(1, EXACT_MEMORY["neighbors"] + 1)],
                            dim=-1)
        top = top.sort(-1).values
    top32 = top.to(torch.int32).contiguous()
    for i in range(b):
        qi = qs[i].transpose(0, 1).unsqueeze(0)
        ok, ov = gather_pages(archive.keys[i], archive.values[i], archive.length, page, top32[i:i + 1], qi)
        out_k.append(ok[0])
        out_v.append(ov[0])
    return torch.stack(out_k), torch.stack(out_v)


def retrieve_attend(archive: Archive, q: torch.Tensor, groups: int, win_keys: torch.Tensor,
                    win_values: torch.Tensor, qpos: torch.Tensor, kpos: torch.Tensor, window: int,
                    sinks: int = 0, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Fused retrieve + exact attention for one archive: q [1,H,T,hd] at positions qpos [T];
    window cache win_keys/win_values [1,KV,S,hd] at positions kpos [S]. Equals
    SDPA(q, [retrieve(archive, q) ; window], mask) of transplant.py:612-628 for the query's
    budget and selection mode (flat, two-level or rerank; without a kept prompt selection or
    neighbours). Returns [1,H,T,hd]."""
    page = EXACT_MEMORY["block_size"]
    b, h, t, d = q.shape
    if b != 1:
        raise ValueError("retrieve_attend takes one archive (B=1)")
    budget, is_decode = _budget(t)
    full = archive.length // page
    qi = q.to(torch.bfloat16)[0].transpose(0, 1).unsqueeze(0)
    qpos32, kpos32 = qpos.to(torch.int32).view(1, t), kpos.to(torch.int32)
    if full and _mode(archive, full, min(budget, full), is_decode) != "flat":
        pages = _select(archive, 0, qi, full, budget, is_decode)
        out = attend_pages(qi, qpos32, archive.keys[0], archive.values[0], archive.length, page, pages, win_keys[0],
                           win_values[0], kpos32, window, sinks, out_dtype=out_dtype)
    else:
        _, out = select_attend_pages(qi, qpos32, archive.keys[0], archive.values[0], archive.kmax[0],
                                     archive.kmin[0], archive.length, page, budget, win_keys[0], win_values[0],
                                     kpos32, window, sinks, out_dtype=out_dtype)
    return out[0].transpose(0, 1).unsqueeze(0)
