"""Gated DeltaNet recurrence on B200: drop-in for pseudobrain/gated_deltanet.py's kernels.

Same names, argument meanings and return values as the reference's PyTorch core
(pseudobrain/gated_deltanet.py:72-308):

    gated_delta_rule(q, k, v, g, beta, scale, h0, kernel="chunked") -> (o, S)
    delta_rule_sequential(q, k, v, g, beta, scale, h0)               -> (o, S)
    delta_rule_chunked(q, k, v, g, beta, scale, h0, chunk=None)      -> (o, S)
    select_kernel(backend, serial, length, *tensors)                  -> kernel name

q, k [B,T,Hk,K]; v [B,T,Hv,V]; g, beta [B,T,Hv]; h0 [B,Hv,K,V]; o [B,T,Hv,V] and
S [B,Hv,K,V] come back in fp32. The reference's caller repeats q and k up to the
value heads first (gated_deltanet.py:422-424); these functions accept either that
expanded form (Hk == Hv) or the GQA-native one (Hv a multiple of Hk, value head j
reading key head j // (Hv // Hk)), which never materialises the repeat.

Every kernel is CUDA (libpbk.so, sm_100a). There is no CPU path: CPU tensors raise.
"""
from __future__ import annotations

import torch

from . import _capi
from ._capi import LIB, PbkGdnDesc, PbkView, check

CHUNK = 64           # pseudobrain/gated_deltanet.py:48
SEQUENTIAL_MAX = 4   # pseudobrain/gated_deltanet.py:54
KERNELS = ("sequential", "chunked")
_DTYPES = {torch.float32: _capi.PBK_F32, torch.bfloat16: _capi.PBK_BF16}


def _dtype_code(t: torch.Tensor, what: str) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"{what}: dtype {t.dtype} is not supported (float32 or bfloat16)") from None


def view4(t: torch.Tensor, what: str) -> PbkView:
    """[B,T,H,D] with a contiguous last dimension."""
    if t.dim() != 4 or t.stride(-1) != 1:
        raise ValueError(f"{what}: expected [B,T,H,D] with a contiguous last dim, got {tuple(t.shape)}")
    return PbkView(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2), _dtype_code(t, what), 0)


def view3(t: torch.Tensor, what: str) -> PbkView:
    """[B,T,H]."""
    if t.dim() != 3:
        raise ValueError(f"{what}: expected [B,T,H], got {tuple(t.shape)}")
    return PbkView(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2), _dtype_code(t, what), 0)


def _check_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if t is not None and (not t.is_cuda or t.device != dev):
            raise RuntimeError("pseudobrain_b200 runs on CUDA only: every tensor must be on the same GPU "
                               "(there is no CPU fallback)")
    return dev


def _desc(q, k, v, g, beta, o, h0, state, scale, state_indices, layout) -> PbkGdnDesc:
    b, t, hk, dk = q.shape
    hv, dv = v.shape[2], v.shape[3]
    if k.shape != q.shape or v.shape[:2] != (b, t) or g.shape != (b, t, hv) or beta.shape != (b, t, hv):
        raise ValueError("gated delta rule: inconsistent shapes "
                         f"q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)} g{tuple(g.shape)} beta{tuple(beta.shape)}")
    if state.dtype != torch.float32 or state.stride(-1) != 1:
        raise ValueError("state must be fp32 with a contiguous last dim")
    if h0 is not None and (h0.dtype != torch.float32 or h0.shape[1:] != state.shape[1:]
                           or h0.stride()[1:] != state.stride()[1:]
                           or (h0.shape[0] > 1 and h0.stride(0) != state.stride(0))):
        raise ValueError("h0 must be fp32 with the state's strides")  # the kernels index both alike
    return PbkGdnDesc(
        batch=b, seqlen=t, hk=hk, hv=hv, dk=dk, dv=dv,
        q=view4(q, "q"), k=view4(k, "k"), v=view4(v, "v"), g=view3(g, "g"), beta=view3(beta, "beta"),
        o=(view4(o, "o") if o is not None else PbkView(None, 0, 0, 0, _capi.PBK_BF16, 0)),
        h0=(h0.data_ptr() if h0 is not None else None), state=state.data_ptr(),
        state_slot_stride=state.stride(0), state_layout=layout, pad_=0,
        state_indices=(state_indices.data_ptr() if state_indices is not None else None),
        scale=float(scale), pad2_=0)


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


@torch.library.custom_op("pbk::gdn_recurrent", mutates_args=("state", "o"))
def gdn_recurrent_(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                   h0: torch.Tensor | None, state: torch.Tensor, o: torch.Tensor, scale: float,
                   state_indices: torch.Tensor | None = None, layout: int = 0) -> None:
    """Register-resident recurrence over the T tokens of each sequence (decode and T <= 4).

    Reads h0 (or, when h0 is None, ``state`` itself: in place), writes the final state
    into ``state`` and the outputs into ``o`` [B,T,Hv,V] (fp32 or bf16). ``state`` is
    [slots,Hv,K,V] (layout 0) or [slots,Hv,V,K] (layout 1, vLLM's pool); state_indices
    [B] int32 picks each sequence's slot (negative: skip)."""
    dev = _check_cuda(q, k, v, g, beta, state, o)
    if state_indices is not None and state_indices.dtype != torch.int32:
        raise TypeError("state_indices must be int32")
    d = _desc(q, k, v, g, beta, o, h0, state, scale, state_indices, layout)
    with torch.cuda.device(dev):
        check(LIB.pbk_gdn_decode(d, _stream(dev)), "pbk_gdn_decode")


@gdn_recurrent_.register_fake
def _(q, k, v, g, beta, h0, state, o, scale, state_indices=None, layout=0):
    return None


def delta_rule_sequential(q, k, v, g, beta, scale, h0):
    """Per-step recurrence (reference: gated_deltanet.py:93-107) as one CUDA launch with the
    state in registers. Returns (o [B,T,Hv,V] fp32, new state [B,Hv,K,V] fp32); h0 is not
    modified."""
    _check_cuda(q, k, v, g, beta, h0)
    b, t, _, _ = q.shape
    hv, dv = v.shape[2], v.shape[3]
    h0 = h0.float().contiguous()
    state = torch.empty_like(h0)
    o = torch.empty(b, t, hv, dv, dtype=torch.float32, device=q.device)
    gdn_recurrent_(q, k, v, g, beta, h0, state, o, float(scale))
    return o, state


def select_kernel(backend: str, serial: bool, length: int, *tensors: torch.Tensor) -> str:
    """Kernel for one call (reference: gated_deltanet.py:291-297): the per-step kernel for
    serial calls and sequences of at most SEQUENTIAL_MAX tokens, the chunked one otherwise."""
    if serial or length <= SEQUENTIAL_MAX:
        return "sequential"
    return "chunked"


def gated_delta_rule(q, k, v, g, beta, scale, h0, kernel: str = "chunked"):
    """The recurrence with the given kernel (reference: gated_deltanet.py:300-308). The
    reference's 'fla' name maps to the chunked CUDA kernel."""
    if kernel == "sequential":
        return delta_rule_sequential(q, k, v, g, beta, scale, h0)
    if kernel in ("chunked", "fla"):
        return delta_rule_chunked(q, k, v, g, beta, scale, h0)
    raise ValueError(f"gated delta rule kernel must be one of {KERNELS}")


def delta_rule_chunked(q, k, v, g, beta, scale, h0, chunk: int | None = None):
    """Chunkwise WY recurrence (reference: gated_deltanet.py:110-165) on CUDA.

    When the (sequence x value head) chains are too few to fill the GPU and the sequences
    are long (bf16 inputs, at least 4 segments of 16+ chunks per sequence), the sequences
    are split along T (gdn_prefill_segmented): three passes over the tokens, spread over
    all SMs instead of one pass on a few."""
    from .gdn_prefill import auto_segments, gdn_prefill, gdn_prefill_segmented
    if chunk not in (None, CHUNK):
        raise ValueError(f"the CUDA chunked kernel uses chunk={CHUNK}")
    if q.dtype == torch.bfloat16 and q.is_cuda:
        segs = auto_segments(q.shape[0], v.shape[2], q.shape[1])
        if segs >= 4:
            return gdn_prefill_segmented(q, k, v, g, beta, scale, h0, segments=segs)
    return gdn_prefill(q, k, v, g, beta, scale, h0)
