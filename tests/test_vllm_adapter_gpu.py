"""GPU parity of the vLLM drop-ins (pseudobrain_b200.vllm_adapter) against the oracle:
ChunkGatedDeltaRule on packed sequences (cu_seqlens) and on a dense batch, with the
in-kernel q/k norm and vLLM's [N, HV, V, K] states, and fused_recurrent_gated_delta_rule on a
state pool through ssm_state_indices (a negative index skipped), in place and not.
bf16 inputs: 2e-2 (outputs and states), as the other bf16 prefill tests."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from oracle.quest import bf16_round

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _rng_inputs(rng, t, hk, hv, bf16=True):
    q = rng.standard_normal((1, t, hk, 128)).astype(np.float32)
    k = rng.standard_normal((1, t, hk, 128)).astype(np.float32)
    v = rng.standard_normal((1, t, hv, 128)).astype(np.float32)
    g = (-np.logaddexp(0.0, -(rng.standard_normal((1, t, hv)) + 2.0))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((1, t, hv))))).astype(np.float32)
    if bf16:
        q, k, v, beta = (bf16_round(x) for x in (q, k, v, beta))
    return q, k, v, g, beta


def _ref(q, k, v, g, beta, h0_vk, hv, norm):
    """oracle: q/k norm (x rsqrt(sum x^2 + 1e-6)), delta_rule_chunked with the [V,K] state."""
    if norm:
        q, k = ogdn.l2_normalize(q, "hf", 1e-6), ogdn.l2_normalize(k, "hf", 1e-6)
    qe, ke = ogdn.expand_key_heads(q, hv), ogdn.expand_key_heads(k, hv)
    o, s = ogdn.delta_rule_chunked(qe, ke, v, g, beta, 128 ** -0.5, h0_vk.transpose(0, 1, 3, 2))
    return o, s.transpose(0, 1, 3, 2)


def _dev(x, dev, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev, dtype)


@pytest.mark.parametrize("norm", [True, False])
def test_chunk_rule_packed_sequences(cuda_device, norm):
    from pseudobrain_b200.vllm_adapter import ChunkGatedDeltaRule
    rng = np.random.default_rng(3 + norm)
    hk, hv, lens = 2, 4, [100, 64, 7, 130]
    t = sum(lens)
    q, k, v, g, beta = _rng_inputs(rng, t, hk, hv)
    if not norm:  # unit rows already, as the caller normalised them
        q, k = bf16_round(ogdn.l2_normalize(q, "max")), bf16_round(ogdn.l2_normalize(k, "max"))
    h0 = (rng.standard_normal((len(lens), hv, 128, 128)) * 0.05).astype(np.float32)
    cu = torch.tensor(np.concatenate(([0], np.cumsum(lens))), dtype=torch.int32, device=cuda_device)
    out_buf = torch.zeros(2 * t * hv * 128, dtype=torch.bfloat16, device=cuda_device)
    o, final = ChunkGatedDeltaRule()(_dev(q, cuda_device), _dev(k, cuda_device), _dev(v, cuda_device),
                                     _dev(g, cuda_device, torch.float32), _dev(beta, cuda_device),
                                     _dev(h0, cuda_device, torch.float32), True, cu_seqlens=cu,
                                     use_qk_l2norm_in_kernel=norm, core_attn_out=out_buf)
    assert o.shape == (1, t, hv, 128) and final.shape == (len(lens), hv, 128, 128)
    for s, (a, b) in enumerate(zip(cu[:-1].tolist(), cu[1:].tolist())):
        ro, rs = _ref(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], beta[:, a:b], h0[s:s + 1], hv, norm)
        assert ogdn.rel_err(o[:, a:b].float().cpu().numpy(), ro) < TOL, s
        assert ogdn.rel_err(final[s:s + 1].cpu().numpy(), rs) < TOL, s
    assert torch.equal(out_buf[: o.numel()], o.reshape(-1))
    assert torch.all(out_buf[o.numel():] == 0)


def test_chunk_rule_dense_batch_without_state(cuda_device):
    from pseudobrain_b200.vllm_adapter import ChunkGatedDeltaRule
    rng = np.random.default_rng(9)
    hk, hv, t = 1, 2, 150
    ins = [_rng_inputs(rng, t, hk, hv) for _ in range(2)]
    q, k, v, g, beta = (np.concatenate(x) for x in zip(*ins))
    o, final = ChunkGatedDeltaRule().forward_cuda(_dev(q, cuda_device), _dev(k, cuda_device), _dev(v, cuda_device),
                                                  _dev(g, cuda_device, torch.float32), _dev(beta, cuda_device), None,
                                                  True)
    for b in range(2):
        ro, rs = _ref(q[b:b + 1], k[b:b + 1], v[b:b + 1], g[b:b + 1], beta[b:b + 1],
                      np.zeros((1, hv, 128, 128), np.float32), hv, True)
        assert ogdn.rel_err(o[b:b + 1].float().cpu().numpy(), ro) < TOL
        assert ogdn.rel_err(final[b:b + 1].cpu().numpy(), rs) < TOL


@pytest.mark.parametrize("inplace", [True, False])
def test_fused_recurrent_on_a_state_pool(cuda_device, inplace):
    """One token per sequence on a state pool: in place through ssm_state_indices (indices 0
    and -1 are vLLM's null block: skipped), or out of place into a new state per sequence."""
    from oracle import vllm_decode as ovd
    from pseudobrain_b200.vllm_adapter import fused_recurrent_gated_delta_rule
    rng = np.random.default_rng(11 + inplace)
    hk, hv, n, slots = 2, 4, 5, 9
    q, k, v, g, beta = _rng_inputs(rng, n, hk, hv)
    pool = (rng.standard_normal((slots, hv, 128, 128)) * 0.05).astype(np.float32)
    idx = np.array([7, 0, -1, 3, 5], dtype=np.int32) if inplace else None
    dpool = _dev(pool if inplace else pool[:n], cuda_device, torch.float32)
    before = dpool.clone()
    cu = torch.arange(n + 1, dtype=torch.int32, device=cuda_device)
    o, final = fused_recurrent_gated_delta_rule(
        _dev(q, cuda_device), _dev(k, cuda_device), _dev(v, cuda_device), _dev(g, cuda_device, torch.float32),
        _dev(beta, cuda_device), None, dpool, inplace, cu,
        torch.from_numpy(idx).to(cuda_device) if idx is not None else None, None, True)
    assert o.shape == (1, n, hv, 128)
    ro, rpool = ovd.recurrent(q, k, v, g, beta, 128 ** -0.5, pool if inplace else pool[:n], cu_seqlens=cu.cpu().numpy(),
                              indices=idx, l2=1)
    for s in range(n):
        slot = int(idx[s]) if inplace else s
        if slot <= 0 and inplace:
            continue
        assert ogdn.rel_err(o[:, s:s + 1].float().cpu().numpy(), ro[:, s:s + 1]) < TOL, s
        assert ogdn.rel_err(final[slot:slot + 1].cpu().numpy(), rpool[slot:slot + 1]) < 1e-4, s
    if inplace:
        assert final is dpool
        for slot in (0, 1, 2, 4, 6, 8):  # untouched slots, the null slot 0 included
            assert torch.equal(dpool[slot], before[slot])
    else:
        assert torch.equal(dpool, before)
