"""Drop-ins for vLLM's Gated DeltaNet ops, on this package's kernels:

    ChunkGatedDeltaRule()(q, k, v, g, beta, initial_state, output_final_state, cu_seqlens,
                          chunk_indices, chunk_offsets, use_qk_l2norm_in_kernel,
                          core_attn_out) -> (o, final_state)
        vllm/model_executor/layers/mamba/gdn/qwen_gdn_linear_attn.py:291-417 (the prefill
        op of Qwen3-Next's linear attention; vllm/model_executor/layers/fla/ops/chunk.py)
    fused_recurrent_gated_delta_rule_packed_decode(mixed_qkv, a, b, A_log, dt_bias, scale,
                                                   initial_state, out, ssm_state_indices,
                                                   use_qk_l2norm_in_kernel)
        vllm/model_executor/layers/fla/ops/fused_recurrent.py:339 (the non-speculative decode
        fast path, qwen_gdn_linear_attn.py:1592-1645)
    fused_sigmoid_gating_delta_rule_update(A_log, a, b, dt_bias, q, k, v, beta, threshold,
                                           scale, initial_state, inplace_final_state,
                                           cu_seqlens, ssm_state_indices, num_accepted_tokens,
                                           use_qk_l2norm_in_kernel, is_kda)
        vllm/model_executor/layers/fla/ops/fused_sigmoid_gating.py:181 (the decode and
        speculative-decode path, qwen_gdn_linear_attn.py:1438-1460, 1488-1510)
    fused_recurrent_gated_delta_rule(q, k, v, g, beta, scale, initial_state,
                                     inplace_final_state, cu_seqlens, ssm_state_indices,
                                     num_accepted_tokens, use_qk_l2norm_in_kernel)
        vllm/model_executor/layers/fla/ops/fused_recurrent.py:516-611

Same argument meanings and layouts as vLLM: packed q, k [1, T, H, K] and v [1, T, HV, V]
(or a dense batch [B, T, ...] without cu_seqlens), g the log decay [.., HV] (fp32), beta
[.., HV], states [N, HV, V, K] fp32 (vLLM's pool layout), scale K**-0.5 by default. The
prefill runs the split tensor-core path (pbk_gdn_prefill_varlen / pbk_gdn_prefill_ws, the
q/k norm x * rsqrt(sum x^2 + 1e-6) by pbk_l2norm); the three decode ops run the
register-resident recurrence with vLLM's semantics (pbk_gdn_decode_ext): the gating
g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) and each op's q/k norm inside the
kernel, sequences of any length, vLLM's null state slot (index <= 0: skipped), and
speculative decoding (2-D ssm_state_indices with num_accepted_tokens: the initial state from
column num_accepted - 1, the state after token t into column t). chunk_indices and
chunk_offsets are accepted and not needed (the kernels derive the chunks from cu_seqlens).
Not covered (NotImplementedError): KDA (per-key-dim decay), head-wise vector beta, and
inplace_final_state=False with more than one token per sequence.
"""
from __future__ import annotations

import torch

import ctypes

from . import _capi
from ._capi import LIB, PbkDecodeExt, PbkView, check
from .gated_deltanet import _check_cuda, _desc, _dtype_code, _stream, view3, view4
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




def _ext(gating=None, l2=0, null_slot=True, zero_skipped=False, cu_seqlens=None, indices=None,
         num_accepted=None) -> PbkDecodeExt:
    """The pbk_decode_ext of one call. gating: (a, b, A_log, dt_bias, softplus_beta,
    threshold, beta_round) with a, b [B, T, HV] views."""
    e = PbkDecodeExt()
    empty = PbkView(None, 0, 0, 0, _capi.PBK_F32, 0)
    e.a = e.b = empty
    if gating is not None:
        a, b, a_log, dt_bias, sb, thr, rnd = gating
        e.gating, e.beta_round, e.softplus_beta, e.softplus_threshold = 1, int(rnd), float(sb), float(thr)
        e.a, e.b = view3(a, "a"), view3(b, "b")
        e.a_log, e.dt_bias = a_log.data_ptr(), dt_bias.data_ptr()
        e.a_log_dtype, e.dt_bias_dtype = _dtype_code(a_log, "A_log"), _dtype_code(dt_bias, "dt_bias")
    e.l2norm, e.eps = l2, 1e-6
    e.null_slot, e.zero_skipped = int(null_slot), int(zero_skipped)
    e.cu_seqlens = cu_seqlens.data_ptr() if cu_seqlens is not None else None
    e.index_stride = indices.stride(0) if (indices is not None and indices.dim() == 2) else 0
    e.num_accepted = num_accepted.data_ptr() if num_accepted is not None else None
    return e


def _decode_ext(q, k, v, g, beta, o, pool, scale, indices, ext, dense_batch) -> None:
    """One pbk_gdn_decode_ext call over [B, T, ...] views (B = 1 with cu_seqlens, the batch of
    the descriptor then being the sequence count)."""
    dev = _check_cuda(q, k, v, o, pool)
    desc = _desc(q, k, v, g, beta, o, None, pool, scale, indices, STATE_VK)
    desc.batch = dense_batch
    with torch.cuda.device(dev):
        check(LIB.pbk_gdn_decode_ext(ctypes.byref(desc), ctypes.byref(ext), _stream(dev)), "pbk_gdn_decode_ext")


def _int32(x: torch.Tensor | None) -> torch.Tensor | None:
    return None if x is None else x.to(torch.int32).contiguous()


def _seq_count(q, cu_seqlens) -> int:
    if cu_seqlens is None:
        return q.shape[0]
    if q.shape[0] != 1:
        raise ValueError("The batch size is expected to be 1 when using cu_seqlens")
    return cu_seqlens.numel() - 1


def fused_recurrent_gated_delta_rule_packed_decode(mixed_qkv: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                                                   A_log: torch.Tensor, dt_bias: torch.Tensor, scale: float,
                                                   initial_state: torch.Tensor, out: torch.Tensor,
                                                   ssm_state_indices: torch.Tensor,
                                                   use_qk_l2norm_in_kernel: bool = False):
    """vLLM's packed decode (fused_recurrent.py:339): one token per row, mixed_qkv [N, 2 H K +
    HV V] holding q | k | v, a, b [N, HV] the raw gate inputs, the state pool initial_state
    [slots, HV, V, K] updated in place at ssm_state_indices [N] (an index <= 0 is vLLM's null
    block: its output row is written as zeros), out [N, 1, HV, V] written. The gating
    (beta = sigmoid(b) rounded to b's dtype, as vLLM does), the q/k norm x / sqrt(sum x^2 +
    1e-6) and the query scale all run inside the decode kernel. Returns (out, initial_state)."""
    if mixed_qkv.ndim != 2 or mixed_qkv.stride(-1) != 1:
        raise ValueError("`mixed_qkv` must be a 2D tensor contiguous in the last dim")
    if a.ndim != 2 or b.ndim != 2 or a.stride(-1) != 1 or b.stride(-1) != 1:
        raise ValueError("`a` and `b` must be 2D tensors contiguous in the last dim")
    if A_log.ndim != 1 or dt_bias.ndim != 1:
        raise ValueError("`A_log`/`dt_bias` must be 1D tensors")
    if ssm_state_indices.ndim != 1:
        raise ValueError("`ssm_state_indices` must be 1D for packed decode")
    if not out.is_contiguous():
        raise ValueError("`out` must be contiguous")
    n = mixed_qkv.shape[0]
    if initial_state.ndim != 4 or initial_state.stride(-1) != 1:
        raise ValueError("`initial_state` must be a 4D tensor contiguous in the last dim")
    hv, vd, kd = initial_state.shape[-3:]
    if a.shape != (n, hv) or b.shape != (n, hv) or A_log.numel() != hv or dt_bias.numel() != hv:
        raise ValueError(f"`a`/`b` must be [{n}, {hv}] and `A_log`/`dt_bias` [{hv}]")
    if out.shape != (n, 1, hv, vd):
        raise ValueError(f"`out` must have shape {(n, 1, hv, vd)}")
    qk_dim = mixed_qkv.shape[1] - hv * vd
    if qk_dim <= 0 or qk_dim % 2 or (qk_dim // 2) % kd:
        raise ValueError(f"Invalid packed `mixed_qkv` last dim={mixed_qkv.shape[1]} for HV={hv}, V={vd}")
    h = qk_dim // 2 // kd
    if hv % h:
        raise ValueError(f"Invalid head config inferred from mixed_qkv: H={h}, HV={hv}")
    row = mixed_qkv.stride(0)
    q = mixed_qkv[:, : h * kd].as_strided((n, 1, h, kd), (row, row, kd, 1))
    k = mixed_qkv[:, h * kd: 2 * h * kd].as_strided((n, 1, h, kd), (row, row, kd, 1))
    v = mixed_qkv[:, 2 * h * kd:].as_strided((n, 1, hv, vd), (row, row, vd, 1))
    a3, b3 = a.unsqueeze(1), b.unsqueeze(1)
    ext = _ext(gating=(a3, b3, A_log, dt_bias, 1.0, 20.0, True), l2=1 if use_qk_l2norm_in_kernel else 0,
               zero_skipped=True)
    _decode_ext(q, k, v, a3, b3, out, initial_state, scale, _int32(ssm_state_indices), ext, n)
    return out, initial_state


def fused_sigmoid_gating_delta_rule_update(A_log: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                                           dt_bias: torch.Tensor, q: torch.Tensor, k: torch.Tensor,
                                           v: torch.Tensor, beta: float = 1.0, threshold: float = 20.0,
                                           scale: float | None = None, initial_state: torch.Tensor | None = None,
                                           inplace_final_state: bool = True,
                                           cu_seqlens: torch.Tensor | None = None,
                                           ssm_state_indices: torch.Tensor | None = None,
                                           num_accepted_tokens: torch.Tensor | None = None,
                                           use_qk_l2norm_in_kernel: bool = False, is_kda: bool = False):
    """vLLM's fused_sigmoid_gating_delta_rule_update (fused_sigmoid_gating.py:181): g =
    -exp(A_log) softplus_beta(a + dt_bias) (softplus with vLLM's `beta` and `threshold`),
    gate = sigmoid(b), the q/k norm x * rsqrt(sum x^2 + 1e-6), then the recurrence over each
    sequence's tokens with the pool [slots, HV, V, K] updated in place at ssm_state_indices
    ([N], or [N, cols] with num_accepted_tokens for speculative decoding). a, b [.., HV] per
    token. Returns (o [B, T, HV, V] in q's dtype, initial_state)."""
    if is_kda:
        raise NotImplementedError("KDA (per-key-dim decay) is not built")
    if not inplace_final_state:
        raise NotImplementedError("inplace_final_state=False is not built for this op")
    if initial_state is None:
        raise ValueError("initial_state is required")
    if scale is None:
        scale = k.shape[-1] ** -0.5
    nseq = _seq_count(q, cu_seqlens)
    bsz, t, hv, vd = v.shape
    a3 = a.reshape(bsz, t, hv)
    b3 = b.reshape(bsz, t, hv)
    o = torch.empty(bsz, t, hv, vd, dtype=q.dtype, device=q.device)
    idx = _int32(ssm_state_indices)
    ext = _ext(gating=(a3, b3, A_log, dt_bias, beta, threshold, False), l2=2 if use_qk_l2norm_in_kernel else 0,
               cu_seqlens=_int32(cu_seqlens), indices=idx, num_accepted=_int32(num_accepted_tokens))
    _decode_ext(q, k, v, a3, b3, o, initial_state, scale, idx, ext, nseq)
    return o, initial_state


def fused_recurrent_gated_delta_rule(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                                     beta: torch.Tensor | None = None, scale: float | None = None,
                                     initial_state: torch.Tensor | None = None, inplace_final_state: bool = True,
                                     cu_seqlens: torch.Tensor | None = None,
                                     ssm_state_indices: torch.Tensor | None = None,
                                     num_accepted_tokens: torch.Tensor | None = None,
                                     use_qk_l2norm_in_kernel: bool = False):
    """vLLM's decode op (fused_recurrent.py:516-611) on the register-resident recurrence:
    with inplace_final_state the pool initial_state [slots, HV, V, K] is updated in place at
    ssm_state_indices ([N]; [N, cols] with num_accepted_tokens for speculative decoding; an
    index <= 0 is vLLM's null block, skipped) and returned as final_state; the q/k norm is x /
    sqrt(sum x^2 + 1e-6) inside the kernel. Without inplace_final_state (one token per
    sequence), final_state[n] receives the state after sequence n's token and the pool is not
    modified."""
    dev = _check_cuda(q, k, v, g)
    if initial_state is None:
        raise ValueError("initial_state is required")
    if scale is None:
        scale = k.shape[-1] ** -0.5
    if beta is None:
        beta = torch.ones_like(q[..., 0])
    if beta.dim() == v.dim():
        raise NotImplementedError("head-wise vector beta is not built")
    nseq = _seq_count(q, cu_seqlens)
    bsz, t, hv, vd = v.shape
    o = torch.empty(bsz, t, hv, vd, dtype=q.dtype, device=dev)
    l2 = 1 if use_qk_l2norm_in_kernel else 0
    idx = _int32(ssm_state_indices)
    if inplace_final_state:
        ext = _ext(l2=l2, cu_seqlens=_int32(cu_seqlens), indices=idx, num_accepted=_int32(num_accepted_tokens))
        _decode_ext(q, k, v, g, beta, o, initial_state, scale, idx, ext, nseq)
        return o, initial_state
    if idx is not None or num_accepted_tokens is not None:
        raise NotImplementedError("ssm_state_indices with inplace_final_state=False")
    rows = q.shape[1] if cu_seqlens is not None else bsz * t
    if rows != nseq:
        raise NotImplementedError("inplace_final_state=False with more than one token per sequence")
    final = initial_state[:nseq].clone()  # vLLM's per-token states: one token per sequence here
    ext = _ext(l2=l2, cu_seqlens=_int32(cu_seqlens))
    _decode_ext(q, k, v, g, beta, o, final, scale, None, ext, nseq)
    return o, final
