"""The Gated DeltaNet layer's pieces around the recurrence, on the GPU (pbk_gdn_conv_norm,
pbk_gdn_gating, pbk_gdn_out_norm), with the reference's names and argument meanings:

* ``short_convolution(x, tail, weight)`` (pseudobrain/gated_deltanet.py:314-338), here
  fused with the q/k ``l2_normalize`` (:59-70) of the split that follows it
  (``conv_qkv``);
* the decay and beta gating (:427-429): ``gdn_gating``;
* the output RMSNorm and SiLU gate (:439-440): ``gated_out_norm``;
* ``gated_deltanet_core``: GatedDeltaNetLayer.forward (:411-440) from the input projection's
  output to the gated, normed per-step output, the recurrence included (prefill on the
  tensor-core kernels, decode on the register kernel), as the vLLM adapter runs it;
* ``gated_deltanet_decode``: the same for a decode step (the few tokens select_kernel sends
  to the sequential recurrence, :291-294) as ONE kernel (pbk_gdn_decode_layer), the state
  and the conv tail updated in place, fp32 between the stages as in the reference;
* ``gated_deltanet_prefill``: the same for a prefill (pbk_gdn_prefill_layer), the conv, norm
  and gating fused into the chunk solve.
``gated_deltanet_core`` runs the pieces as separate kernels: at config-1 and config-2 shapes
they measured faster than the two fused entry points.
"""
from __future__ import annotations

import torch

from . import _capi
from ._capi import LIB, PbkConvDesc, PbkGatingDesc, PbkGdnLayerDesc, PbkOutNormDesc, PbkView, check
from .gated_deltanet import _check_cuda, _dtype_code, _stream, view3, view4

L2_MODES = {"max": 1, "hf": 2}
L2_EPS = 1e-6
NORM_EPS = 1e-5


def _none_view() -> PbkView:
    return PbkView(None, 0, 0, 0, _capi.PBK_F32, 0)


def conv_qkv(x: torch.Tensor, tail: torch.Tensor | None, weight: torch.Tensor | None, hk: int, hv: int,
             l2mode: str | None = "max", new_tail: torch.Tensor | None = None, out_dtype=torch.bfloat16,
             eps: float = L2_EPS):
    """short_convolution of x [B,T,(2hk+hv)*128] (tail [B,K-1,C], weight [C,K]; None: SiLU
    only), split into q, k [B,T,hk,128] (L2-normalised, mode 'max' or 'hf'; None: not) and v
    [B,T,hv,128] in out_dtype; the last K-1 inputs go to new_tail [B,K-1,C] when given (it
    must not be `tail`). Returns (q, k, v)."""
    dev = _check_cuda(x, *(t for t in (tail, weight, new_tail) if t is not None))
    b, t, c = x.shape
    if c != (2 * hk + hv) * 128:
        raise ValueError(f"x has {c} channels, expected (2*{hk}+{hv})*128")
    if weight is not None and (weight.dtype != torch.float32 or not weight.is_contiguous() or weight.shape[0] != c):
        raise ValueError("weight must be fp32 [C, K], contiguous")
    width = weight.shape[1] if weight is not None else 1
    if tail is not None and tail.shape != (b, width - 1, c):
        raise ValueError("tail must be [B, K-1, C]")
    q = torch.empty(b, t, hk, 128, device=dev, dtype=out_dtype)
    k = torch.empty_like(q)
    v = torch.empty(b, t, hv, 128, device=dev, dtype=out_dtype)
    d = PbkConvDesc(batch=b, seqlen=t, hk=hk, hv=hv, width=width, l2mode=L2_MODES[l2mode] if l2mode else 0,
                    eps=eps, pad_=0, x=view3(x, "x"), tail=view3(tail, "tail") if tail is not None else _none_view(),
                    new_tail=view3(new_tail, "new_tail") if new_tail is not None else _none_view(),
                    weight=weight.data_ptr() if weight is not None else None,
                    q=view4(q, "q"), k=view4(k, "k"), v=view4(v, "v"))
    with torch.cuda.device(dev):
        check(LIB.pbk_gdn_conv_norm(d, _stream(dev)), "pbk_gdn_conv_norm")
    return q, k, v


def gdn_gating(decay: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor, beta_dtype=torch.float32):
    """g = -exp(A_log) softplus(a + dt_bias) (fp32), beta = sigmoid(b) for decay = [a | b]
    [B,T,2Hv]. Returns (g, beta) [B,T,Hv]."""
    dev = _check_cuda(decay, a_log, dt_bias)
    b, t, two_hv = decay.shape
    hv = two_hv // 2
    if a_log.dtype != torch.float32 or dt_bias.dtype != torch.float32 or a_log.numel() != hv or dt_bias.numel() != hv:
        raise ValueError("A_log and dt_bias must be fp32 [Hv]")
    a_log, dt_bias = a_log.contiguous(), dt_bias.contiguous()
    g = torch.empty(b, t, hv, device=dev, dtype=torch.float32)
    beta = torch.empty(b, t, hv, device=dev, dtype=beta_dtype)
    d = PbkGatingDesc(batch=b, seqlen=t, hv=hv, pad_=0, decay=view3(decay, "decay"), a_log=a_log.data_ptr(),
                      dt_bias=dt_bias.data_ptr(), g=view3(g, "g"), beta=view3(beta, "beta"))
    with torch.cuda.device(dev):
        check(LIB.pbk_gdn_gating(d, _stream(dev)), "pbk_gdn_gating")
    return g, beta


def gated_out_norm(o: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, eps: float = NORM_EPS,
                   out_dtype=None) -> torch.Tensor:
    """o * rsqrt(mean(o^2) + eps) * weight * SiLU(gate) per 128-wide head row; o [B,T,Hv,128],
    gate [B,T,Hv*128] or [B,T,Hv,128], weight [128]. Returns [B,T,Hv,128] in out_dtype (o's)."""
    dev = _check_cuda(o, gate, weight)
    b, t, hv, dv = o.shape
    if dv != 128 or weight.numel() != 128:
        raise ValueError("the value dim is 128")
    gate4 = gate.view(b, t, hv, dv) if gate.dim() == 3 else gate
    weight = weight.contiguous()
    out = torch.empty(b, t, hv, dv, device=dev, dtype=out_dtype or o.dtype)
    d = PbkOutNormDesc(batch=b, seqlen=t, hv=hv, weight_dtype=_dtype_code(weight, "weight"), eps=eps, pad_=0,
                       o=view4(o, "o"), gate=view4(gate4, "gate"), out=view4(out, "out"), weight=weight.data_ptr())
    with torch.cuda.device(dev):
        check(LIB.pbk_gdn_out_norm(d, _stream(dev)), "pbk_gdn_out_norm")
    return out


def gated_deltanet_core(qkv: torch.Tensor, gate: torch.Tensor, decay: torch.Tensor, conv_tail: torch.Tensor,
                        conv_weight: torch.Tensor | None, a_log: torch.Tensor, dt_bias: torch.Tensor,
                        o_norm: torch.Tensor, state: torch.Tensor, hk: int, hv: int, l2mode: str = "max",
                        norm_eps: float = NORM_EPS):
    """GatedDeltaNetLayer.forward (gated_deltanet.py:411-440) from the projection's output
    (qkv [B,T,C], gate [B,T,Hv*128], decay [B,T,2Hv]) to the gated, normed output [B,T,Hv,128]
    (fp32), with the conv tail [B,K-1,C] and the fp32 state [B,Hv,128,128] carried.
    Returns (out, new state, new tail)."""
    from .gated_deltanet import gated_delta_rule
    b, t, _ = qkv.shape
    new_tail = torch.empty_like(conv_tail)
    q, k, v = conv_qkv(qkv, conv_tail, conv_weight, hk, hv, l2mode, new_tail)
    g, beta = gdn_gating(decay, a_log, dt_bias, beta_dtype=torch.bfloat16)
    o, new_state = gated_delta_rule(q, k, v, g, beta, 128 ** -0.5, state, "sequential" if t <= 4 else "chunked")
    out = gated_out_norm(o, gate, o_norm, norm_eps, torch.float32)
    return out, new_state, new_tail


def gated_deltanet_decode(qkv: torch.Tensor, gate: torch.Tensor, decay: torch.Tensor, conv_tail: torch.Tensor | None,
                          conv_weight: torch.Tensor | None, a_log: torch.Tensor, dt_bias: torch.Tensor,
                          o_norm: torch.Tensor, state: torch.Tensor, hk: int, hv: int, l2mode: str | None = "max",
                          norm_eps: float = NORM_EPS, *, state_layout: str = "kv", state_indices=None,
                          out_dtype=torch.float32, l2_eps: float = L2_EPS) -> torch.Tensor:
    """GatedDeltaNetLayer.forward's decode step (gated_deltanet.py:411-440 with the sequential
    recurrence, :93-107) in one kernel: qkv [B,T,(2hk+hv)*128], gate [B,T,hv*128] and decay
    [B,T,2hv] from the input projection; conv_tail [B,K-1,C] (updated in place to the last K-1
    inputs; None with conv_weight None: SiLU only); conv_weight [C,K] fp32; state
    [slots,hv,128,128] fp32 ("kv": [K,V] per head, "vk": [V,K]) updated in place, slot
    state_indices[b] (int32 [B], negative: skipped) or b. Returns the gated, normed output
    [B,T,hv,128] in out_dtype; q, k, v, g and beta stay in the kernel's registers."""
    dev = _check_cuda(qkv, gate, decay, a_log, dt_bias, o_norm, state,
                      *(x for x in (conv_tail, conv_weight, state_indices) if x is not None))
    b, t, c = qkv.shape
    if c != (2 * hk + hv) * 128:
        raise ValueError(f"qkv has {c} channels, expected (2*{hk}+{hv})*128")
    if conv_weight is not None:
        if conv_weight.dtype != torch.float32 or not conv_weight.is_contiguous() or conv_weight.shape[0] != c:
            raise ValueError("conv_weight must be fp32 [C, K], contiguous")
        width = conv_weight.shape[1]
        if width > 1 and (conv_tail is None or conv_tail.shape != (b, width - 1, c)):
            raise ValueError("conv_tail must be [B, K-1, C]")
    else:
        width = 1
    if state.dtype != torch.float32 or state.dim() != 4 or state.shape[1:] != (hv, 128, 128) or state.stride(-1) != 1:
        raise ValueError("state must be fp32 [slots, hv, 128, 128] with rows contiguous")
    if a_log.dtype != torch.float32 or dt_bias.dtype != torch.float32 or a_log.numel() != hv or dt_bias.numel() != hv:
        raise ValueError("A_log and dt_bias must be fp32 [hv]")
    if o_norm.numel() != 128:
        raise ValueError("o_norm must have 128 entries")
    if state_indices is not None and (state_indices.dtype != torch.int32 or state_indices.numel() != b):
        raise ValueError("state_indices must be int32 [B]")
    a_log, dt_bias, o_norm = a_log.contiguous(), dt_bias.contiguous(), o_norm.contiguous()
    out = torch.empty(b, t, hv, 128, device=dev, dtype=out_dtype)
    tail_view = view3(conv_tail, "conv_tail") if (conv_tail is not None and width > 1) else _none_view()
    d = PbkGdnLayerDesc(batch=b, seqlen=t, hk=hk, hv=hv, width=width, l2mode=L2_MODES[l2mode] if l2mode else 0,
                        l2_eps=l2_eps, norm_eps=norm_eps, scale=128 ** -0.5,
                        state_layout=_capi.PBK_STATE_KV if state_layout == "kv" else _capi.PBK_STATE_VK,
                        qkv=view3(qkv, "qkv"), tail=tail_view, new_tail=tail_view,
                        conv_weight=conv_weight.data_ptr() if conv_weight is not None else None,
                        decay=view3(decay, "decay"), a_log=a_log.data_ptr(), dt_bias=dt_bias.data_ptr(),
                        gate=view3(gate, "gate"), o_norm=o_norm.data_ptr(), o_norm_dtype=_dtype_code(o_norm, "o_norm"),
                        pad_=0, out=view4(out, "out"), state=state.data_ptr(), state_slot_stride=state.stride(0),
                        state_indices=state_indices.data_ptr() if state_indices is not None else None)
    with torch.cuda.device(dev):
        check(LIB.pbk_gdn_decode_layer(d, _stream(dev)), "pbk_gdn_decode_layer")
    return out


def gated_deltanet_prefill(qkv: torch.Tensor, gate: torch.Tensor, decay: torch.Tensor, conv_tail: torch.Tensor | None,
                           conv_weight: torch.Tensor | None, a_log: torch.Tensor, dt_bias: torch.Tensor,
                           o_norm: torch.Tensor, state: torch.Tensor, hk: int, hv: int, l2mode: str | None = "max",
                           norm_eps: float = NORM_EPS, *, new_tail: torch.Tensor | None = None,
                           state_layout: str = "kv", state_indices=None, out_dtype=torch.float32,
                           l2_eps: float = L2_EPS) -> torch.Tensor:
    """GatedDeltaNetLayer.forward over a prefill (gated_deltanet.py:411-440 with the chunked
    recurrence, :110-165) as pbk_gdn_prefill_layer: the chunk solve with the conv, SiLU, q/k
    norm and gating fused in, the tensor-core recurrence, the gated output norm. qkv
    [B,T,(2hk+hv)*128] bf16 (channels contiguous), gate [B,T,hv*128], decay [B,T,2hv];
    conv_tail [B,K-1,C] is read and new_tail (a different tensor, or None) receives the last
    K-1 inputs; state [slots,hv,128,128] fp32 is the initial state and receives the final one
    (slot state_indices[b] or b). Returns the gated, normed output [B,T,hv,128] in out_dtype."""
    dev = _check_cuda(qkv, gate, decay, a_log, dt_bias, o_norm, state,
                      *(x for x in (conv_tail, conv_weight, new_tail, state_indices) if x is not None))
    b, t, c = qkv.shape
    if c != (2 * hk + hv) * 128:
        raise ValueError(f"qkv has {c} channels, expected (2*{hk}+{hv})*128")
    if qkv.dtype != torch.bfloat16 or qkv.stride(-1) != 1 or gate.stride(-1) != 1:
        raise ValueError("qkv must be bf16 and qkv / gate channels contiguous")
    width = 1
    if conv_weight is not None:
        if conv_weight.dtype != torch.float32 or not conv_weight.is_contiguous() or conv_weight.shape[0] != c:
            raise ValueError("conv_weight must be fp32 [C, K], contiguous")
        width = conv_weight.shape[1]
        for x, what in ((conv_tail, "conv_tail"), (new_tail, "new_tail")):
            if x is not None and x.shape != (b, width - 1, c):
                raise ValueError(f"{what} must be [B, K-1, C]")
    if new_tail is not None and conv_tail is not None and new_tail.data_ptr() == conv_tail.data_ptr():
        raise ValueError("new_tail must not be conv_tail")
    if state.dtype != torch.float32 or state.dim() != 4 or state.shape[1:] != (hv, 128, 128) or state.stride(-1) != 1:
        raise ValueError("state must be fp32 [slots, hv, 128, 128] with rows contiguous")
    if a_log.dtype != torch.float32 or dt_bias.dtype != torch.float32 or a_log.numel() != hv or dt_bias.numel() != hv:
        raise ValueError("A_log and dt_bias must be fp32 [hv]")
    a_log, dt_bias, o_norm = a_log.contiguous(), dt_bias.contiguous(), o_norm.contiguous()
    out = torch.empty(b, t, hv, 128, device=dev, dtype=out_dtype)
    conv = width > 1
    d = PbkGdnLayerDesc(batch=b, seqlen=t, hk=hk, hv=hv, width=width, l2mode=L2_MODES[l2mode] if l2mode else 0,
                        l2_eps=l2_eps, norm_eps=norm_eps, scale=128 ** -0.5,
                        state_layout=_capi.PBK_STATE_KV if state_layout == "kv" else _capi.PBK_STATE_VK,
                        qkv=view3(qkv, "qkv"),
                        tail=view3(conv_tail, "conv_tail") if (conv and conv_tail is not None) else _none_view(),
                        new_tail=view3(new_tail, "new_tail") if (conv and new_tail is not None) else _none_view(),
                        conv_weight=conv_weight.data_ptr() if conv_weight is not None else None,
                        decay=view3(decay, "decay"), a_log=a_log.data_ptr(), dt_bias=dt_bias.data_ptr(),
                        gate=view3(gate, "gate"), o_norm=o_norm.data_ptr(), o_norm_dtype=_dtype_code(o_norm, "o_norm"),
                        pad_=0, out=view4(out, "out"), state=state.data_ptr(), state_slot_stride=state.stride(0),
                        state_indices=state_indices.data_ptr() if state_indices is not None else None)
    nbytes = LIB.pbk_gdn_prefill_layer_workspace(d)
    if nbytes == 0 and t > 0:
        raise ValueError("pbk_gdn_prefill_layer: unsupported problem")
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(LIB.pbk_gdn_prefill_layer(d, ws.data_ptr(), nbytes, _stream(dev)), "pbk_gdn_prefill_layer")
    return out
