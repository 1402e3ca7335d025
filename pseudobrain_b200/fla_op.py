"""The reference's GPU prefill op, ``pseudobrain::gated_delta_chunk``, on this package's kernels.

The reference registers (pseudobrain/gated_deltanet.py:200-227)

    pseudobrain::gated_delta_chunk(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta,
                                   Tensor h0, float scale) -> (Tensor, Tensor, Tensor, Tensor)

returning (o [B,T,H,V] in q's dtype, final state [B,H,K,V] fp32, the chunk-local cumulative
g [B,T,H] fp32, the WY inverse A [B,T,H,64] in k's dtype), and routes select_kernel's "fla"
kernel to it (:280-285, :291-297). Its body calls flash-linear-attention's Triton kernels; here
the same op runs pbk_gdn_prefill_aux (the tensor-core prefill for bf16 inputs, the exact fp32
kernel otherwise). q and k come already expanded to the value heads, as the reference's caller
passes them.

Importing this module makes the op available either way:
* if the reference's module has already registered it, this module registers a CUDA kernel for
  it (torch.library.register_kernel), so the reference's own calls on CUDA tensors run here;
* otherwise it defines the op with the same schema and a fake (meta) implementation, as the
  reference does, so torch.ops.pseudobrain.gated_delta_chunk works on its own.
CPU tensors raise: there is no CPU path.
"""
from __future__ import annotations

import ctypes

import torch

from ._capi import LIB, PbkView, check
from .gated_deltanet import _check_cuda, _desc, _dtype_code, _stream

OP = "pseudobrain::gated_delta_chunk"
SCHEMA = ("(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, Tensor h0, float scale) "
          "-> (Tensor, Tensor, Tensor, Tensor)")
CHUNK = 64  # fla's chunk (gated_deltanet.py:50, FLA_CHUNK)


def gated_delta_chunk_cuda(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                           h0: torch.Tensor, scale: float):
    """(o in q's dtype, final fp32, gc fp32, A in k's dtype) of the chunked gated delta rule."""
    dev = _check_cuda(q, k, v, g, beta, h0)
    b, t, h, kd = q.shape
    vd = v.shape[-1]
    o = torch.empty(b, t, h, vd, dtype=q.dtype, device=dev)
    final = torch.empty(b, h, kd, vd, dtype=torch.float32, device=dev)
    gc = torch.empty(b, t, h, dtype=torch.float32, device=dev)
    a = torch.empty(b, t, h, CHUNK, dtype=k.dtype, device=dev)
    h0f = h0.float().contiguous()
    d = _desc(q, k, v, g, beta, o, h0f, final, scale, None, 0)
    gcv = PbkView(gc.data_ptr(), gc.stride(0), gc.stride(1), gc.stride(2), _dtype_code(gc, "gc"), 0)
    av = PbkView(a.data_ptr(), a.stride(0), a.stride(1), a.stride(2), _dtype_code(a, "A"), 0)
    with torch.cuda.device(dev):
        n = LIB.pbk_gdn_prefill_workspace(d)
        ws = torch.empty(max(n, 16), dtype=torch.uint8, device=dev)
        check(LIB.pbk_gdn_prefill_aux(d, ctypes.byref(gcv), ctypes.byref(av), ws.data_ptr(), n, _stream(dev)),
              "pbk_gdn_prefill_aux")
    return o, final, gc, a


def _fake(q, k, v, g, beta, h0, scale):
    batch, length, heads, dk = q.shape
    return (q.new_empty(batch, length, heads, v.shape[-1]),
            h0.new_empty(batch, heads, dk, v.shape[-1], dtype=torch.float32),
            g.new_empty(batch, length, heads, dtype=torch.float32),
            k.new_empty(batch, length, heads, CHUNK))


def _registered() -> bool:
    try:
        torch._C._dispatch_find_schema_or_throw(OP, "")
        return True
    except RuntimeError:
        return False


if _registered():
    # the reference's op exists in this process: serve its CUDA calls
    torch.library.register_kernel(OP, "cuda", gated_delta_chunk_cuda)
    DEFINED_HERE = False
else:
    @torch.library.custom_op(OP, mutates_args=(), schema=SCHEMA)
    def _gated_delta_chunk(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                           h0: torch.Tensor, scale: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor,
                                                                    torch.Tensor]:
        return gated_delta_chunk_cuda(q, k, v, g, beta, h0, scale)

    _gated_delta_chunk.register_fake(_fake)
    DEFINED_HERE = True


def delta_rule_fla(q, k, v, g, beta, scale, h0):
    """The reference's fla path (gated_deltanet.py:280-285) through the op: q/k/v at q's
    precision, fp32 state and decay; returns (o fp32, final state fp32)."""
    o, final, _, _ = torch.ops.pseudobrain.gated_delta_chunk(q, k, v.to(q.dtype), g.float(), beta.to(q.dtype),
                                                             h0.float(), float(scale))
    return o.float(), final
