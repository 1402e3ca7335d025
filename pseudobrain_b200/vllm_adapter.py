"""Drop-ins for vLLM's Gated DeltaNet ops, on this package's kernels:

    ChunkGatedDeltaRule()(q, k, v, g, beta, initial_state, output_final_state, cu_seqlens,
                          chunk_indices, chunk_offsets, use_qk_l2norm_in_kernel,
                          core_attn_out) -> (o, final_state)
        vllm/model_executor/layers/mamba/gdn/qwen_gdn_linear_attn.py:291-417 (the prefill
        op of Qwen3-Next's linear attention; vllm/model_executor/layers/fla/ops/chunk.py)
    fused_recurrent_gated_delta_rule(q, k, v, g, beta, scale, initial_state,
                                     inplace_final_state, cu_seqlens, ssm_state_indices,
                                     num_accepted_tokens, use_qk_l2norm_in_kernel)
        vllm/model_executor/layers/fla/ops/fused_recurrent.py:516-611 (the decode op)

Same argument meanings and layouts as vLLM: packed q, k [1, T, H, K] and v [1, T, HV, V]
(or a dense batch [B, T, ...] without cu_seqlens), g the log decay [.., HV] (fp32), beta
[.., HV], states [N, HV, V, K] fp32 (vLLM's pool layout), scale K**-0.5 by default, and the
in-kernel q/k normalisation x * rsqrt(sum x^2 + 1e-6). The prefill runs the split tensor-core
path (pbk_gdn_prefill_varlen / pbk_gdn_prefill_ws), the decode the register kernel
(pbk_gdn_decode) on the pool in place through ssm_state_indices; the q/k norm is
pbk_l2norm. chunk_indices and chunk_offsets are accepted and not needed (the kernels derive
the chunks from cu_seqlens). Not covered (NotImplementedError): speculative decoding
(num_accepted_tokens, 2-D ssm_state_indices) and non-uniform token counts in the decode op.
"""
from __future__ import annotations

import torch

from ._capi import LIB, check
from .gated_deltanet import _check_cuda, _stream, gdn_recurrent_, view4
from .gdn_prefill import gdn_prefill_, gdn_prefill_varlen_

STATE_VK = 1  # [N, HV, V, K]
L2_EPS = 1e-6


def l2norm(x: torch.Tensor, eps: float = L2_EPS, mode: str = "rsqrt") -> torch.Tensor:
    """Rows of 128 of x [B, T, H, 128] normalised (pbk_l2norm): 'rsqrt' x * rsqrt(sum x^2 +
    eps) (vLLM's in-kernel norm), 'max' x / max(|x|, eps) (F.normalize). Same dtype."""
    dev = _check_cuda(x)
    out = torch.empty_like(x)
    b, t, h, d = x.shape
    if d != 128:
        raise ValueError("rows of 128")
    with torch.cuda.device(dev):
        check(LIB.pbk_l2norm(view4(x, "x"), view4(out, "out"), b, t, h, 2 if mode == "rsqrt" else 1, eps,
                             _stream(dev)), "pbk_l2norm")
    return out


def _state_for(initial_state: torch.Tensor | None, n: int, hv: int, v: int, k: int, dev) -> torch.Tensor:
    if initial_state is not None:
        if initial_state.dtype != torch.float32 or tuple(initial_state.shape[1:]) != (hv, v, k):
            raise ValueError(f"initial_state must be fp32 [N, {hv}, {v}, {k}]")
    return torch.empty(n, hv, v, k, dtype=torch.float32, device=dev)


class ChunkGatedDeltaRule:
    """vLLM's ChunkGatedDeltaRule (qwen_gdn_linear_attn.py:291-417) on the tensor-core
    prefill. Call it (or .forward / .forward_cuda / .forward_native) with vLLM's arguments."""

    def __call__(self, *args, **kwargs):
        return self.forward(*args, **kwargs)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                initial_state: torch.Tensor | None, output_final_state: bool, cu_seqlens: torch.Tensor | None = None,
                chunk_indices: torch.Tensor | None = None, chunk_offsets: torch.Tensor | None = None,
                use_qk_l2norm_in_kernel: bool = True, core_attn_out: torch.Tensor | None = None):
        dev = _check_cuda(q, k, v, g, beta)
        if use_qk_l2norm_in_kernel:
            q, k = l2norm(q), l2norm(k)
        b, t, hv, vd = v.shape
        kd = q.shape[-1]
        n = cu_seqlens.numel() - 1 if cu_seqlens is not None else b
        final = _state_for(initial_state, n, hv, vd, kd, dev)
        o = torch.empty(b, t, hv, vd, dtype=q.dtype, device=dev)
        scale = kd ** -0.5
        if cu_seqlens is not None:
            if b != 1:
                raise ValueError("packed (cu_seqlens) inputs have batch 1")
            gdn_prefill_varlen_(q, k, v, g, beta, initial_state, final, o, scale, cu_seqlens.to(torch.int32), None,
                                STATE_VK)
        else:
            gdn_prefill_(q, k, v, g, beta, initial_state, final, o, scale, None, STATE_VK)
        if core_attn_out is not None:  # vLLM's output buffer, filled from the front
            flat = o.reshape(-1)
            core_attn_out.reshape(-1)[: flat.numel()].copy_(flat)
        return o, (final if output_final_state else None)

    forward_cuda = forward
    forward_native = forward


def fused_recurrent_gated_delta_rule(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                                     beta: torch.Tensor | None = None, scale: float | None = None,
                                     initial_state: torch.Tensor | None = None, inplace_final_state: bool = True,
                                     cu_seqlens: torch.Tensor | None = None,
                                     ssm_state_indices: torch.Tensor | None = None,
                                     num_accepted_tokens: torch.Tensor | None = None,
                                     use_qk_l2norm_in_kernel: bool = False):
    """vLLM's decode op (fused_recurrent.py:516-611) on the register-resident recurrence:
    with inplace_final_state the pool initial_state [slots, HV, V, K] is updated in place at
    ssm_state_indices (negative: padding, skipped) and returned as final_state."""
    if num_accepted_tokens is not None or (ssm_state_indices is not None and ssm_state_indices.dim() != 1):
        raise NotImplementedError("speculative decoding (num_accepted_tokens) is not built")
    dev = _check_cuda(q, k, v, g)
    if scale is None:
        scale = k.shape[-1] ** -0.5
    if beta is None:
        beta = torch.ones_like(q[..., 0])
    if use_qk_l2norm_in_kernel:
        q, k = l2norm(q), l2norm(k)
    if cu_seqlens is not None:  # packed sequences of equal length: a batch view, no copy
        if q.shape[0] != 1:
            raise ValueError("The batch size is expected to be 1 when using cu_seqlens")
        n = cu_seqlens.numel() - 1
        lens = torch.diff(cu_seqlens).cpu()
        if n == 0 or not bool((lens == lens[0]).all()) or int(lens[0]) * n != q.shape[1]:
            raise NotImplementedError("decode sequences of different lengths")
        t = int(lens[0])

        def per_seq(x):
            return x.reshape((n, t) + tuple(x.shape[2:]))

        q, k, v, g, beta = (per_seq(x) for x in (q, k, v, g, beta))
    b, t, hv, vd = v.shape
    o = torch.empty(b, t, hv, vd, dtype=q.dtype, device=dev)
    idx = ssm_state_indices.to(torch.int32).contiguous() if ssm_state_indices is not None else None
    if initial_state is None:
        raise ValueError("initial_state is required")
    if inplace_final_state:
        gdn_recurrent_(q, k, v, g, beta, None, initial_state, o, scale, idx, STATE_VK)
        final = initial_state
    else:
        if idx is not None:
            raise NotImplementedError("ssm_state_indices with inplace_final_state=False")
        final = initial_state[:b].clone()  # the decode kernel updates its state in place
        gdn_recurrent_(q, k, v, g, beta, None, final, o, scale, None, STATE_VK)
    if cu_seqlens is not None:
        o = o.reshape((1, b * t) + tuple(o.shape[2:]))
    return o, final
