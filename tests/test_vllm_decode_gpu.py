"""GPU parity of the vLLM decode drop-ins on pbk_gdn_decode_ext against oracle/vllm_decode.py
(a numpy restatement of vLLM's three decode ops): the packed decode with fused gating and the
in-kernel q/k norm, fused_sigmoid_gating_delta_rule_update over sequences of different lengths
and under speculative decoding (2-D state indices, num_accepted_tokens), and
fused_recurrent_gated_delta_rule with vLLM's null slot. Outputs bf16 (2e-2, the bar for bf16
inputs), pool states fp32 (1e-4); untouched slots must stay bit-identical."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from oracle import vllm_decode as ovd
from oracle.quest import bf16_round

pytestmark = pytest.mark.gpu
TOL_O, TOL_S = 2e-2, 1e-4


def _d(x, dev, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev, dtype)


def _pool(rng, slots, hv):
    return (rng.standard_normal((slots, hv, 128, 128)) * 0.05).astype(np.float32)


def _check_pool(got, want, before, touched):
    for s in range(got.shape[0]):
        if s in touched:
            assert ogdn.rel_err(got[s], want[s]) < TOL_S, s
        else:
            assert np.array_equal(got[s], before[s]), s


def test_packed_decode_matches_vllm_semantics(cuda_device):
    from pseudobrain_b200.vllm_adapter import fused_recurrent_gated_delta_rule_packed_decode
    rng = np.random.default_rng(1)
    n, h, hv, slots = 7, 2, 4, 9
    mixed = bf16_round(rng.standard_normal((n, 2 * h * 128 + hv * 128)).astype(np.float32))
    a = bf16_round(rng.standard_normal((n, hv)).astype(np.float32) * 3)
    a[0, 0] = 30.0  # past the softplus threshold
    b = bf16_round(rng.standard_normal((n, hv)).astype(np.float32))
    a_log = rng.standard_normal(hv).astype(np.float32) * 0.5
    dt_bias = rng.standard_normal(hv).astype(np.float32)
    pool = _pool(rng, slots, hv)
    idx = np.array([3, 0, 5, -1, 8, 1, 2], dtype=np.int32)  # 0 and -1: vLLM's null block
    dpool = _d(pool, cuda_device, torch.float32)
    out = torch.full((n, 1, hv, 128), 7.0, dtype=torch.bfloat16, device=cuda_device)
    o, st = fused_recurrent_gated_delta_rule_packed_decode(
        _d(mixed, cuda_device), _d(a, cuda_device), _d(b, cuda_device), _d(a_log, cuda_device, torch.float32),
        _d(dt_bias, cuda_device, torch.float32), 128 ** -0.5, dpool, out, torch.from_numpy(idx).to(cuda_device),
        use_qk_l2norm_in_kernel=True)
    assert o is out and st is dpool
    ro, rpool = ovd.packed_decode(mixed, a, b, a_log, dt_bias, 128 ** -0.5, pool, idx, 128, hv, 128, l2=1,
                                  beta_round=bf16_round)
    got = out.float().cpu().numpy()
    for t in range(n):
        if idx[t] <= 0:
            assert np.all(got[t] == 0), t  # the null slot writes zeros
        else:
            assert ogdn.rel_err(got[t], ro[t]) < TOL_O, t
    _check_pool(dpool.cpu().numpy(), rpool, pool, {int(s) for s in idx if s > 0})


@pytest.mark.parametrize("l2", [True, False])
def test_sigmoid_gating_update_variable_lengths(cuda_device, l2):
    """Non-speculative decode and short prefill pieces: 1-D indices, cu_seqlens of different
    lengths, softplus with vLLM's beta 1 / threshold 20."""
    from pseudobrain_b200.vllm_adapter import fused_sigmoid_gating_delta_rule_update
    rng = np.random.default_rng(2 + l2)
    lens, h, hv, slots = [3, 1, 0, 4, 2], 2, 4, 8
    t = sum(lens)
    q = bf16_round(rng.standard_normal((1, t, h, 128)).astype(np.float32))
    k = bf16_round(rng.standard_normal((1, t, h, 128)).astype(np.float32))
    v = bf16_round(rng.standard_normal((1, t, hv, 128)).astype(np.float32))
    if not l2:
        q, k = bf16_round(ogdn.l2_normalize(q, "max")), bf16_round(ogdn.l2_normalize(k, "max"))
    a = bf16_round(rng.standard_normal((t, hv)).astype(np.float32) * 2)
    b = bf16_round(rng.standard_normal((t, hv)).astype(np.float32))
    a_log = rng.standard_normal(hv).astype(np.float32) * 0.5
    dt_bias = bf16_round(rng.standard_normal(hv).astype(np.float32))
    pool = _pool(rng, slots, hv)
    idx = np.array([6, 2, 3, 0, 5], dtype=np.int32)  # sequence 3 is null
    cu = np.concatenate(([0], np.cumsum(lens))).astype(np.int32)
    dpool = _d(pool, cuda_device, torch.float32)
    o, st = fused_sigmoid_gating_delta_rule_update(
        _d(a_log, cuda_device, torch.float32), _d(a, cuda_device), _d(b, cuda_device), _d(dt_bias, cuda_device),
        _d(q, cuda_device), _d(k, cuda_device), _d(v, cuda_device), initial_state=dpool,
        cu_seqlens=torch.from_numpy(cu).to(cuda_device), ssm_state_indices=torch.from_numpy(idx).to(cuda_device),
        use_qk_l2norm_in_kernel=l2)
    g, beta = ovd.gating(a, b, a_log, dt_bias)
    ro, rpool = ovd.recurrent(q, k, v, g[None], beta[None], 128 ** -0.5, pool, cu_seqlens=cu, indices=idx,
                              l2=2 if l2 else 0)
    got = o.float().cpu().numpy()
    for s_, (r0, r1) in enumerate(zip(cu[:-1], cu[1:])):
        if r1 > r0 and idx[s_] > 0:
            assert ogdn.rel_err(got[:, r0:r1], ro[:, r0:r1]) < TOL_O, s_
    touched = {int(idx[s_]) for s_ in range(len(lens)) if lens[s_] > 0 and idx[s_] > 0}
    _check_pool(dpool.cpu().numpy(), rpool, pool, touched)


def test_sigmoid_gating_update_speculative_decoding(cuda_device):
    """Speculative decoding: 2-D ssm_state_indices [N, 5] (each sequence's own slots, null
    columns 0), num_accepted_tokens picking the initial state's column, the state after every
    token written to its column."""
    from pseudobrain_b200.vllm_adapter import fused_sigmoid_gating_delta_rule_update
    rng = np.random.default_rng(4)
    lens, acc, h, hv = [3, 1, 4, 2], [2, 1, 3, 1], 1, 2
    nseq, cols = len(lens), 5
    slots = 1 + nseq * cols
    t = sum(lens)
    q = bf16_round(rng.standard_normal((1, t, h, 128)).astype(np.float32))
    k = bf16_round(rng.standard_normal((1, t, h, 128)).astype(np.float32))
    v = bf16_round(rng.standard_normal((1, t, hv, 128)).astype(np.float32))
    a = bf16_round(rng.standard_normal((t, hv)).astype(np.float32))
    b = bf16_round(rng.standard_normal((t, hv)).astype(np.float32))
    a_log = rng.standard_normal(hv).astype(np.float32) * 0.5
    dt_bias = rng.standard_normal(hv).astype(np.float32)
    pool = _pool(rng, slots, hv)
    idx = np.zeros((nseq, cols), dtype=np.int32)
    for s_ in range(nseq):
        for c in range(max(lens[s_], acc[s_])):
            idx[s_, c] = 1 + s_ * cols + c
    idx[2, 1] = 0  # a null column: its state is not written
    cu = np.concatenate(([0], np.cumsum(lens))).astype(np.int32)
    dpool = _d(pool, cuda_device, torch.float32)
    o, _ = fused_sigmoid_gating_delta_rule_update(
        _d(a_log, cuda_device, torch.float32), _d(a, cuda_device), _d(b, cuda_device),
        _d(dt_bias, cuda_device, torch.float32), _d(q, cuda_device), _d(k, cuda_device), _d(v, cuda_device),
        initial_state=dpool, cu_seqlens=torch.from_numpy(cu).to(cuda_device),
        ssm_state_indices=torch.from_numpy(idx).to(cuda_device),
        num_accepted_tokens=torch.tensor(acc, dtype=torch.int32, device=cuda_device), use_qk_l2norm_in_kernel=True)
    g, beta = ovd.gating(a, b, a_log, dt_bias)
    ro, rpool = ovd.recurrent(q, k, v, g[None], beta[None], 128 ** -0.5, pool, cu_seqlens=cu, indices=idx,
                              num_accepted=np.array(acc), l2=2)
    assert ogdn.rel_err(o.float().cpu().numpy(), ro) < TOL_O
    touched = {int(idx[s_, c]) for s_ in range(nseq) for c in range(lens[s_]) if idx[s_, c] > 0}
    _check_pool(dpool.cpu().numpy(), rpool, pool, touched)


def test_fused_recurrent_variable_lengths_and_null_slot(cuda_device):
    """fused_recurrent_gated_delta_rule with given g and beta over sequences of different
    lengths (vLLM's packed layout), the in-kernel norm x / sqrt(sum x^2 + 1e-6), and vLLM's
    null slot (index 0 skipped: no output, no state write)."""
    from pseudobrain_b200.vllm_adapter import fused_recurrent_gated_delta_rule
    rng = np.random.default_rng(5)
    lens, h, hv, slots = [2, 5, 1], 2, 4, 6
    t = sum(lens)
    q = bf16_round(rng.standard_normal((1, t, h, 128)).astype(np.float32))
    k = bf16_round(rng.standard_normal((1, t, h, 128)).astype(np.float32))
    v = bf16_round(rng.standard_normal((1, t, hv, 128)).astype(np.float32))
    g = (-np.logaddexp(0.0, -(rng.standard_normal((1, t, hv)) + 2.0))).astype(np.float32)
    beta = bf16_round((1 / (1 + np.exp(-rng.standard_normal((1, t, hv))))).astype(np.float32))
    pool = _pool(rng, slots, hv)
    idx = np.array([4, 0, 1], dtype=np.int32)
    cu = np.concatenate(([0], np.cumsum(lens))).astype(np.int32)
    dpool = _d(pool, cuda_device, torch.float32)
    o, final = fused_recurrent_gated_delta_rule(
        _d(q, cuda_device), _d(k, cuda_device), _d(v, cuda_device), _d(g, cuda_device, torch.float32),
        _d(beta, cuda_device), None, dpool, True, torch.from_numpy(cu).to(cuda_device),
        torch.from_numpy(idx).to(cuda_device), None, True)
    assert final is dpool
    ro, rpool = ovd.recurrent(q, k, v, g, beta, 128 ** -0.5, pool, cu_seqlens=cu, indices=idx, l2=1)
    got = o.float().cpu().numpy()
    for s_, (r0, r1) in enumerate(zip(cu[:-1], cu[1:])):
        if idx[s_] > 0:
            assert ogdn.rel_err(got[:, r0:r1], ro[:, r0:r1]) < TOL_O, s_
    _check_pool(dpool.cpu().numpy(), rpool, pool, {4, 1})
