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
        check(LIB.pbk_gdn_prefill(d, _stream(dev)), "pbk_gdn_prefill")


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
