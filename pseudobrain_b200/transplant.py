"""Causal sliding-window attention (the hybrid layer's attention branch) on B200.

Drop-in for pseudobrain/transplant.py:417-436:

    causal_attention(q, k, v, window=None, sinks=0) -> o

q [B,H,T,hd] and k, v [B,KV,T,hd] (H a multiple of KV; query head j reads key head
j // (H // KV), the reference's repeat_interleave, never materialised); query t sees
key s when s <= t and (window is None or t - s < window or s < sinks), softmax at
SDPA's default scale hd**-0.5. Returns [B,H,T,hd] in q's dtype, like the reference's
SDPA. The reference evaluates long sequences in query chunks of 4096
(``_chunked_window_attention``, transplant.py:346-362); that is the same function.

``window_attention_`` is the out-variant custom op over any [B,T,H,hd]-strided views
(the reference layout [B,H,T,hd] is the same tensors with permuted strides), so a
model's [B,T,H*hd] projections can be used without a transpose copy.

The kernel is tcgen05 (libpbk.so, sm_100a): bf16 q/k/v, fp32 accumulation, bf16 or
fp32 output, hd == 128. There is no CPU path.
"""
from __future__ import annotations

import torch

from ._capi import LIB, PbkSwaDesc, check
from .gated_deltanet import _check_cuda, _stream, view4


@torch.library.custom_op("pbk::window_attention", mutates_args=("o",))
def window_attention_(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, window: int,
                      sinks: int, scale: float) -> None:
    """o[b,t,j] = softmax over visible keys of scale * q[b,t,j].k[b,s,j//G], times v.

    q, o [B,T,H,hd]; k, v [B,T,KV,hd] (views with a contiguous last dim); window <= 0
    means unbounded (full causal)."""
    dev = _check_cuda(q, k, v, o)
    b, t, h, d = q.shape
    kv = k.shape[2]
    if k.shape != (b, t, kv, d) or v.shape != k.shape or o.shape != q.shape:
        raise ValueError(f"window attention: inconsistent shapes q{tuple(q.shape)} k{tuple(k.shape)} "
                         f"v{tuple(v.shape)} o{tuple(o.shape)}")
    if h % kv:
        raise ValueError(f"{h} query heads do not split over {kv} key heads")
    desc = PbkSwaDesc(batch=b, seqlen=t, h=h, kv=kv, d=d, window=int(window), sinks=int(sinks), scale=float(scale),
                      q=view4(q, "q"), k=view4(k, "k"), v=view4(v, "v"), o=view4(o, "o"))
    with torch.cuda.device(dev):
        check(LIB.pbk_swa_prefill(desc, _stream(dev)), "pbk_swa_prefill")


@window_attention_.register_fake
def _(q, k, v, o, window, sinks, scale):
    return None


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window: int | None = None,
                     sinks: int = 0) -> torch.Tensor:
    """Reference signature (transplant.py:417): q [B,H,T,hd], k/v [B,KV,T,hd] -> [B,H,T,hd]
    in q's dtype. Inputs in another float dtype are rounded to bf16 for the tensor cores."""
    _check_cuda(q, k, v)
    if q.dim() != 4 or k.dim() != 4 or v.shape != k.shape:
        raise ValueError("causal_attention: q [B,H,T,hd] and k, v [B,KV,T,hd] expected")
    qb, kb, vb = (x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16) for x in (q, k, v))
    # [B,H,T,hd] -> [B,T,H,hd] views (strides only); last dim made contiguous if needed
    qt, kt, vt = (x.transpose(1, 2) if x.stride(-1) == 1 else x.contiguous().transpose(1, 2) for x in (qb, kb, vb))
    out_dtype = q.dtype if q.dtype in (torch.bfloat16, torch.float32) else torch.float32
    o = torch.empty(q.shape, dtype=out_dtype, device=q.device)
    window_attention_(qt, kt, vt, o.transpose(1, 2), 0 if window is None else int(window), int(sinks),
                      q.shape[-1] ** -0.5)
    return o if o.dtype == q.dtype else o.to(q.dtype)
