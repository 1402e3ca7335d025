"""Chunked gated delta rule (prefill) through pbk_gdn_prefill.

``gdn_prefill`` has the semantics of the reference's delta_rule_chunked
(pseudobrain/gated_deltanet.py:110-165): inputs [B,T,H,*], initial state h0
[B,Hv,K,V], returns (o [B,T,Hv,V], final state [B,Hv,K,V] fp32). ``gdn_prefill_``
is the in-place/out-parameter form the serving adapters use.
"""
from __future__ import annotations

import torch

from ._capi import LIB, check
from .gated_deltanet import _check_cuda, _desc, _stream


@torch.library.custom_op("pbk::gdn_chunked", mutates_args=("state", "o"))
def gdn_prefill_(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                 h0: torch.Tensor | None, state: torch.Tensor, o: torch.Tensor, scale: float,
                 state_indices: torch.Tensor | None = None, layout: int = 0) -> None:
    """Chunkwise recurrence over the T tokens of every sequence. Reads h0 (None: zeros;
    h0 may be ``state`` itself), writes the final state into ``state`` [slots,Hv,K,V]
    (layout 0) or [slots,Hv,V,K] (layout 1) and the outputs into o [B,T,Hv,V]."""
    dev = _check_cuda(q, k, v, g, beta, state, o)
    if state_indices is not None and state_indices.dtype != torch.int32:
        raise TypeError("state_indices must be int32")
    d = _desc(q, k, v, g, beta, o, h0, state, scale, state_indices, layout)
    with torch.cuda.device(dev):
        _run(d, dev, "pbk_gdn_prefill")


def _run(d, dev: torch.device, what: str) -> None:
    """pbk_gdn_prefill_ws with a stream-ordered workspace from the caching allocator (the
    chunk solve runs for all chunks at once first) where the tensor-core path takes the
    call; pbk_gdn_prefill otherwise."""
    n = LIB.pbk_gdn_prefill_workspace(d)
    if n == 0:
        check(LIB.pbk_gdn_prefill(d, _stream(dev)), what)
        return
    ws = torch.empty(n, dtype=torch.uint8, device=dev)
    check(LIB.pbk_gdn_prefill_ws(d, ws.data_ptr(), n, _stream(dev)), what)


@gdn_prefill_.register_fake
def _(q, k, v, g, beta, h0, state, o, scale, state_indices=None, layout=0):
    return None


def gdn_prefill(q, k, v, g, beta, scale, h0=None, out_dtype: torch.dtype = torch.float32):
    """(o [B,T,Hv,V] in out_dtype, final state [B,Hv,K,V] fp32) from h0 (None: zeros)."""
    _check_cuda(q, k, v, g, beta)
    b, t, _, dk = q.shape
    hv, dv = v.shape[2], v.shape[3]
    if h0 is not None:
        _check_cuda(q, h0)
        h0 = h0.float().contiguous()
    state = torch.empty(b, hv, dk, dv, dtype=torch.float32, device=q.device)
    o = torch.empty(b, t, hv, dv, dtype=out_dtype, device=q.device)
    gdn_prefill_(q, k, v, g, beta, h0, state, o, float(scale))
    return o, state


# ------------------------------------------------------------------------------------------
# Long sequences with few heads: split T into segments that run in parallel
# ------------------------------------------------------------------------------------------
@torch.library.custom_op("pbk::gdn_final_state", mutates_args=("state",))
def gdn_final_state_(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                     h0: torch.Tensor | None, state: torch.Tensor, scale: float) -> None:
    """The final state of the chunked recurrence only (no outputs written): bf16 q/k/v."""
    dev = _check_cuda(q, k, v, g, beta, state)
    d = _desc(q, k, v, g, beta, None, h0, state, scale, None, 0)
    with torch.cuda.device(dev):
        _run(d, dev, "pbk_gdn_prefill (state only)")


@gdn_final_state_.register_fake
def _(q, k, v, g, beta, h0, state, scale):
    return None


def segment_scan(b: torch.Tensor, m: torch.Tensor, h0: torch.Tensor | None, starts: torch.Tensor) -> None:
    """starts[:, 0] = h0 (None: 0), starts[:, p+1] = (m[:, p] - b[:, p]) starts[:, p] + b[:, p];
    b, m [B, nseg-1, Hv, 128, 128], starts [B, nseg, Hv, 128, 128], fp32 contiguous."""
    batch, nseg, hv = starts.shape[:3]
    for t in (b, m, h0, starts):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()):
            raise ValueError("segment scan: fp32 contiguous tensors expected")
    if b.shape != (batch, nseg - 1, hv, 128, 128) or m.shape != b.shape:
        raise ValueError("segment scan: b and m must be [B, nseg - 1, Hv, 128, 128]")
    dev = _check_cuda(b, m, starts)
    with torch.cuda.device(dev):
        check(LIB.pbk_gdn_segment_scan(b.data_ptr(), m.data_ptr(), None if h0 is None else h0.data_ptr(),
                                       starts.data_ptr(), batch, nseg, hv, _stream(dev)), "pbk_gdn_segment_scan")


def auto_segments(batch: int, hv: int, seqlen: int, sms: int | None = None) -> int:
    """Segments per sequence so that batch x heads x segments CTAs fill the SMs once
    (1 when the batch already does, or when segments would be under 16 chunks)."""
    if sms is None:
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    chunks = -(-seqlen // 64)
    want = sms // max(1, batch * hv)
    return max(1, min(want, chunks // 16))


def chunk_solve(q, k, v, g, beta, state, scale, ws: torch.Tensor | None = None) -> torch.Tensor:
    """pbk_gdn_chunk_solve of the (bf16) inputs into ws (a new workspace when None); `state`
    only shapes the call."""
    dev = q.device
    d = _desc(q, k, v, g, beta, None, None, state, scale, None, 0)
    n = LIB.pbk_gdn_prefill_workspace(d)
    if n == 0:
        raise ValueError("the chunk solve runs on the bf16 tensor-core path only")
    if ws is None:
        ws = torch.empty(n, dtype=torch.uint8, device=dev)
    elif ws.numel() < n:
        raise ValueError("workspace too small")
    check(LIB.pbk_gdn_chunk_solve(d, ws.data_ptr(), n, _stream(dev)), "pbk_gdn_chunk_solve")
    return ws


def prefill_solved(q, k, v, g, beta, h0, state, o, scale, ws: torch.Tensor, offset: int = 0) -> None:
    """pbk_gdn_prefill_solved from the solve slots starting `offset` bytes into ws."""
    dev = q.device
    d = _desc(q, k, v, g, beta, o, h0, state, scale, None, 0)
    need = LIB.pbk_gdn_prefill_workspace(d)
    if need == 0 or offset % 16 or offset + need > ws.numel():
        raise ValueError("workspace slice out of range")
    check(LIB.pbk_gdn_prefill_solved(d, ws.data_ptr() + offset, need, _stream(dev)), "pbk_gdn_prefill_solved")


def gdn_prefill_segmented(q, k, v, g, beta, scale, h0=None, segments: int | None = None,
                          out_dtype: torch.dtype = torch.float32, o: torch.Tensor | None = None):
    """delta_rule_chunked's (o, final state) with every sequence split into `segments`
    pieces of whole 64-token chunks that run in parallel (bf16 q/k/v):

    1. all full segments from zeros and from the identity (final states b and m only);
    2. pbk_gdn_segment_scan chains them into each segment's true initial state;
    3. all segments again from those states, writing the outputs and the final state.

    The chunk boundaries are those of the unsplit sequence, so this is the reference's
    arithmetic reassociated across segments (exact in real arithmetic)."""
    _check_cuda(q, k, v, g, beta)
    b, t, hk, dk = q.shape
    hv, dv = v.shape[2], v.shape[3]
    if segments is None:
        segments = auto_segments(b, hv, t)
    chunks = -(-t // 64)
    seg_len = -(-chunks // max(1, segments)) * 64
    nseg = -(-t // seg_len)
    if o is None:
        o = torch.empty(b, t, hv, dv, dtype=out_dtype, device=q.device)
    if h0 is not None:
        h0 = h0.float().contiguous()
    final = torch.empty(b, hv, dk, dv, dtype=torch.float32, device=q.device)
    if nseg == 1:
        gdn_prefill_(q, k, v, g, beta, h0, final, o, float(scale))
        return o, final
    full = nseg - 1
    cut = full * seg_len
    for i in range(b):  # one sequence at a time: its full segments form a batch (a view)
        def seg(x):
            return x[i, :cut].unflatten(0, (full, seg_len))

        # one chunk solve of the whole sequence serves all three runs: slot (segment p,
        # chunk c) of the segment batch is slot (0, p * seg_chunks + c) of the sequence
        ws = chunk_solve(q[i:i + 1], k[i:i + 1], v[i:i + 1], g[i:i + 1], beta[i:i + 1], final[i:i + 1],
                          float(scale))
        slot = ws.numel() // (chunks * hv)
        qs, ks, vs, gs, bs = (seg(x) for x in (q, k, v, g, beta))
        bst = torch.empty(full, hv, dk, dv, dtype=torch.float32, device=q.device)
        mst = torch.empty_like(bst)
        eye = torch.eye(dk, dtype=torch.float32, device=q.device).expand(full, hv, dk, dv).contiguous()
        prefill_solved(qs, ks, vs, gs, bs, None, bst, None, float(scale), ws, 0)
        prefill_solved(qs, ks, vs, gs, bs, eye, mst, None, float(scale), ws, 0)
        starts = torch.empty(1, nseg, hv, dk, dv, dtype=torch.float32, device=q.device)
        segment_scan(bst.unsqueeze(0), mst.unsqueeze(0), None if h0 is None else h0[i:i + 1], starts)
        # the last (shorter) segment runs beside the full ones on a side stream, so the
        # two launches share the SMs; `eye` receives the full segments' final states
        # (not needed afterwards)
        cur = torch.cuda.current_stream(q.device)
        side = torch.cuda.Stream(q.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            prefill_solved(q[i:i + 1, cut:], k[i:i + 1, cut:], v[i:i + 1, cut:], g[i:i + 1, cut:],
                            beta[i:i + 1, cut:], starts[:, full], final[i:i + 1], o[i:i + 1, cut:], float(scale),
                            ws, (cut // 64) * hv * slot)
        starts.record_stream(side)
        ws.record_stream(side)
        prefill_solved(qs, ks, vs, gs, bs, starts[0, :full], eye, seg(o), float(scale), ws, 0)
        cur.wait_stream(side)
    return o, final


# ------------------------------------------------------------------------------------------
# Packed varlen prefill (vLLM's chunked-prefill batch: cu_seqlens over [1, T, H, 128])
# ------------------------------------------------------------------------------------------
@torch.library.custom_op("pbk::gdn_prefill_varlen", mutates_args=("state", "o"))
def gdn_prefill_varlen_(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                        h0: torch.Tensor | None, state: torch.Tensor, o: torch.Tensor, scale: float,
                        cu_seqlens: torch.Tensor, state_indices: torch.Tensor | None = None,
                        layout: int = 0) -> None:
    """delta_rule_chunked on each packed sequence: q, k [1, T, Hk, 128], v [1, T, Hv, 128]
    bf16, g, beta [1, T, Hv]; sequence s is rows cu_seqlens[s] .. cu_seqlens[s+1] (int32 on
    the device). Reads h0 (None: zeros; h0 may be ``state``: in place) and writes the final
    state of sequence s into slot state_indices[s] (or s) of ``state`` ([slots, Hv, K, V],
    layout 0, or [slots, Hv, V, K], layout 1) and its outputs into its rows of o [1, T, Hv, 128]."""
    dev = _check_cuda(q, k, v, g, beta, state, o, cu_seqlens)
    if cu_seqlens.dtype != torch.int32 or cu_seqlens.dim() != 1 or not cu_seqlens.is_contiguous():
        raise TypeError("cu_seqlens must be a contiguous int32 vector")
    if state_indices is not None and state_indices.dtype != torch.int32:
        raise TypeError("state_indices must be int32")
    if q.shape[0] != 1:
        raise ValueError("packed inputs have batch 1")
    num_seqs = cu_seqlens.numel() - 1
    d = _desc(q, k, v, g, beta, o, h0, state, scale, state_indices, layout)
    with torch.cuda.device(dev):
        n = LIB.pbk_gdn_prefill_varlen_workspace(d, num_seqs)
        if n == 0:
            raise ValueError("varlen prefill runs on the bf16 tensor-core path (bf16 q/k/v, 16-byte strides)")
        ws = torch.empty(n, dtype=torch.uint8, device=dev)
        check(LIB.pbk_gdn_prefill_varlen(d, cu_seqlens.data_ptr(), num_seqs, ws.data_ptr(), n, _stream(dev)),
              "pbk_gdn_prefill_varlen")


@gdn_prefill_varlen_.register_fake
def _(q, k, v, g, beta, h0, state, o, scale, cu_seqlens, state_indices=None, layout=0):
    return None
