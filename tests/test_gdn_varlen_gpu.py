"""GPU parity of the packed varlen prefill (pbk_gdn_prefill_varlen, vLLM's chunked-prefill
layout: sequences concatenated along T, cu_seqlens offsets) against the oracle run on each
sequence alone. bf16 inputs: 2e-2 norm-wise relative on every sequence's outputs and state
(the bf16 tolerance); rows outside every sequence are never written."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from tests.inputs import gdn_inputs, to_device

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2


def _oracle_seq(inp, lo, hi, h0):
    hv = inp["v"].shape[2]
    sl = slice(lo, hi)
    q, k = (ogdn.expand_key_heads(inp[n][:, sl], hv) for n in ("q", "k"))
    return ogdn.delta_rule_chunked(q, k, inp["v"][:, sl], inp["g"][:, sl], inp["beta"][:, sl], inp["scale"], h0)


@pytest.mark.parametrize("lens,lead,trail,hk,hv", [
    ([100, 0, 64, 257, 1, 130], 5, 11, 1, 2),   # ragged, empty, a whole chunk, a single token
    ([2048], 0, 0, 2, 4),                       # one sequence, no padding around it
    ([63, 65, 128, 190, 33, 7, 300, 64], 0, 40, 2, 4),
])
def test_varlen_matches_per_sequence_oracle(cuda_device, lens, lead, trail, hk, hv):
    from pseudobrain_b200.gdn_prefill import gdn_prefill_varlen_
    t = lead + sum(lens) + trail
    inp = gdn_inputs(t + hv, 1, t, hk, hv, bf16=True, state_std=0.02)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32) + lead
    n = len(lens)
    rng = np.random.default_rng(5)
    h0 = (0.02 * rng.standard_normal((n, hv, 128, 128))).astype(np.float32)
    d = to_device(inp, cuda_device)
    o = torch.full((1, t, hv, 128), 7.0, device=cuda_device)
    state = torch.empty(n, hv, 128, 128, device=cuda_device)
    gdn_prefill_varlen_(d["q"], d["k"], d["v"], d["g"], d["beta"], torch.from_numpy(h0).to(cuda_device), state, o,
                        inp["scale"], torch.from_numpy(cu).to(cuda_device))
    got_o, got_s = o.cpu().numpy(), state.cpu().numpy()
    for s in range(n):
        lo, hi = int(cu[s]), int(cu[s + 1])
        if hi == lo:  # an empty sequence keeps its initial state
            assert np.array_equal(got_s[s], h0[s]), s
            continue
        ro, rs = _oracle_seq(inp, lo, hi, h0[s:s + 1])
        assert ogdn.rel_err(got_o[:, lo:hi], ro) < TOL_BF16, s
        assert ogdn.rel_err(got_s[s:s + 1], rs) < TOL_BF16, s
    assert np.all(got_o[:, :lead] == 7.0) and np.all(got_o[:, cu[-1]:] == 7.0)
    from pseudobrain_b200._capi import device_error
    assert device_error() == 0


def test_varlen_state_pool_in_place_vk_layout(cuda_device):
    """vLLM's pool: [slots, Hv, V, K] updated in place through state_indices, a -1 entry
    skipping its sequence (its rows and slot untouched)."""
    from pseudobrain_b200.gdn_prefill import gdn_prefill_varlen_
    lens = [70, 200, 33]
    t = sum(lens)
    inp = gdn_inputs(41, 1, t, 1, 2, bf16=True, state_std=0.02)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    d = to_device(inp, cuda_device)
    rng = np.random.default_rng(9)
    pool0 = (0.02 * rng.standard_normal((5, 2, 128, 128))).astype(np.float32)
    pool = torch.from_numpy(pool0).to(cuda_device)
    idx = torch.tensor([3, -1, 0], dtype=torch.int32, device=cuda_device)
    o = torch.zeros(1, t, 2, 128, device=cuda_device, dtype=torch.bfloat16)
    gdn_prefill_varlen_(d["q"], d["k"], d["v"], d["g"], d["beta"], pool, pool, o, inp["scale"],
                        torch.from_numpy(cu).to(cuda_device), idx, 1)
    got = pool.cpu().numpy()
    for s, slot in ((0, 3), (2, 0)):
        lo, hi = int(cu[s]), int(cu[s + 1])
        ro, rs = _oracle_seq(inp, lo, hi, pool0[slot:slot + 1].transpose(0, 1, 3, 2))
        assert ogdn.rel_err(o[:, lo:hi].float().cpu().numpy(), ro) < TOL_BF16
        assert ogdn.rel_err(got[slot:slot + 1].transpose(0, 1, 3, 2), rs) < TOL_BF16
    for slot in (1, 2, 4):
        assert np.array_equal(got[slot], pool0[slot])
    assert torch.all(o[:, cu[1]:cu[2]] == 0)


def test_varlen_rejects_bad_arguments(cuda_device):
    from pseudobrain_b200 import _capi
    from pseudobrain_b200.gdn_prefill import gdn_prefill_varlen_
    inp = gdn_inputs(3, 1, 64, 1, 2, bf16=True)
    d = to_device(inp, cuda_device)
    state = torch.empty(1, 2, 128, 128, device=cuda_device)
    o = torch.empty(1, 64, 2, 128, device=cuda_device)
    with pytest.raises(TypeError):
        gdn_prefill_varlen_(d["q"], d["k"], d["v"], d["g"], d["beta"], None, state, o, inp["scale"],
                            torch.tensor([0, 64], device=cuda_device))  # int64 offsets
    d2 = to_device(gdn_inputs(3, 2, 64, 1, 2, bf16=True), cuda_device)
    with pytest.raises(ValueError):
        gdn_prefill_varlen_(d2["q"], d2["k"], d2["v"], d2["g"], d2["beta"], None, state, o, inp["scale"],
                            torch.tensor([0, 64], dtype=torch.int32, device=cuda_device))  # batch 2
    assert _capi.device_error() == 0
