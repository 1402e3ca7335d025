"""GPU parity of the register-resident recurrence (pbk_gdn_decode) against the oracle
and the reference's golden outputs.

The kernel computes in fp32 like the reference (bf16 inputs are widened exactly), so
the tolerance is the fp32 one, 1e-4 norm-wise relative, for every case.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from oracle.quest import bf16_from_bits
from tests.conftest import load_golden
from tests.inputs import gdn_inputs, to_device

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _oracle(inp):
    hv = inp["v"].shape[2]
    return ogdn.delta_rule_sequential(ogdn.expand_key_heads(inp["q"], hv), ogdn.expand_key_heads(inp["k"], hv),
                                      inp["v"], inp["g"], inp["beta"], inp["scale"], inp["h0"])


def test_decode_matches_reference_golden(cuda_device):
    from pseudobrain_b200 import gated_deltanet as G
    f = load_golden("gdn_decode.npz")
    t = {n: torch.from_numpy(bf16_from_bits(f[n])).to(cuda_device, torch.bfloat16)
         for n in ("q", "k", "v", "g", "beta")}
    h0 = torch.from_numpy(f["h0"]).to(cuda_device)
    o, s = G.delta_rule_sequential(t["q"], t["k"], t["v"], t["g"], t["beta"], float(f["scale"]), h0)
    assert ogdn.rel_err(o.cpu().numpy(), f["o_sequential"]) < TOL
    assert ogdn.rel_err(s.cpu().numpy(), f["s_sequential"]) < TOL
    assert torch.equal(h0.cpu(), torch.from_numpy(f["h0"]))  # out of place: h0 untouched


@pytest.mark.parametrize("batch,length,hk,hv,bf16", [
    (1, 1, 1, 1, False), (3, 4, 2, 4, False), (2, 2, 4, 4, True), (5, 1, 2, 8, True), (2, 7, 1, 2, False)])
def test_decode_matches_oracle(cuda_device, batch, length, hk, hv, bf16):
    from pseudobrain_b200 import gated_deltanet as G
    inp = gdn_inputs(batch * 100 + length, batch, length, hk, hv, bf16=bf16, g_bf16=bf16, state_std=0.02)
    d = to_device(inp, cuda_device)
    o, s = G.delta_rule_sequential(d["q"], d["k"], d["v"], d["g"], d["beta"], inp["scale"], d["h0"])
    ro, rs = _oracle(inp)
    assert ogdn.rel_err(o.cpu().numpy(), ro) < TOL
    assert ogdn.rel_err(s.cpu().numpy(), rs) < TOL


@pytest.mark.parametrize("layout", [0, 1])
def test_decode_in_place_layouts_slots_and_bf16_out(cuda_device, layout):
    """vLLM-style call: state pool [slots,Hv,...] in either layout, state_indices with a
    padding slot (-1), in-place update, bf16 output."""
    from pseudobrain_b200 import gated_deltanet as G
    batch, hk, hv = 4, 2, 4
    inp = gdn_inputs(7 + layout, batch, 1, hk, hv, bf16=True, state_std=0.02)
    d = to_device(inp, cuda_device)
    slots = 6
    idx = torch.tensor([5, 0, -1, 3], dtype=torch.int32, device=cuda_device)
    pool_kv = torch.randn(slots, hv, 128, 128, device=cuda_device) * 0.02
    for b in range(batch):
        if idx[b] >= 0:
            pool_kv[idx[b]] = d["h0"][b]
    pool = pool_kv.clone() if layout == 0 else pool_kv.transpose(-1, -2).contiguous()
    before = pool.clone()
    o = torch.full((batch, 1, hv, 128), 7.0, dtype=torch.bfloat16, device=cuda_device)
    G.gdn_recurrent_(d["q"], d["k"], d["v"], d["g"], d["beta"], None, pool, o, inp["scale"], idx, layout)
    ro, rs = _oracle(inp)
    after = pool if layout == 0 else pool.transpose(-1, -2)
    for b in range(batch):
        s = int(idx[b])
        if s < 0:
            assert torch.all(o[b].float() == 7.0)  # skipped sequence: output untouched
            continue
        assert ogdn.rel_err(after[s].cpu().numpy(), rs[b]) < TOL
        assert ogdn.rel_err(o[b, 0].float().cpu().numpy(), ro[b, 0]) < 1e-2  # bf16 output rounding
    untouched = [s for s in range(slots) if s not in idx.tolist()]
    assert torch.equal(pool[untouched], before[untouched])


def test_multi_token_call_equals_token_by_token(cuda_device):
    """T tokens in one launch (state kept in registers) == T launches of one token each,
    bit for bit: the same fp32 operations in the same order."""
    from pseudobrain_b200 import gated_deltanet as G
    inp = gdn_inputs(11, 8, 4, 2, 4, bf16=True, state_std=0.02)
    d = to_device(inp, cuda_device)
    o_all, s_all = G.delta_rule_sequential(d["q"], d["k"], d["v"], d["g"], d["beta"], inp["scale"], d["h0"])
    s = d["h0"].clone()
    o = torch.empty_like(o_all)
    for t in range(4):
        sl = slice(t, t + 1)
        G.gdn_recurrent_(d["q"][:, sl], d["k"][:, sl], d["v"][:, sl], d["g"][:, sl], d["beta"][:, sl],
                         None, s, o[:, sl], inp["scale"])
    assert torch.equal(o, o_all) and torch.equal(s, s_all)


def test_decode_config2_full_size_one_step(cuda_device):
    """benchmark config 2 shape (B=256, 16 key / 32 value heads, 537 MB state), one step."""
    from pseudobrain_b200 import gated_deltanet as G
    inp = gdn_inputs(2, 256, 1, 16, 32, bf16=True, g_bf16=True, state_std=0.02)
    d = to_device(inp, cuda_device)
    state = d["h0"].clone()
    o = torch.empty(256, 1, 32, 128, device=cuda_device)
    G.gdn_recurrent_(d["q"], d["k"], d["v"], d["g"], d["beta"], None, state, o, inp["scale"])
    ro, rs = _oracle(inp)
    assert ogdn.rel_err(o.cpu().numpy(), ro) < TOL
    assert ogdn.rel_err(state.cpu().numpy(), rs) < TOL


def test_decode_rejects_bad_arguments(cuda_device):
    from pseudobrain_b200 import gated_deltanet as G
    from pseudobrain_b200._capi import PbkError
    inp = gdn_inputs(3, 1, 1, 1, 1)
    d = to_device(inp, cuda_device)
    o = torch.empty(1, 1, 1, 128, device=cuda_device)
    with pytest.raises(PbkError):  # dk != 128
        G.gdn_recurrent_(d["q"][..., :64].contiguous(), d["k"][..., :64].contiguous(), d["v"], d["g"],
                         d["beta"], None, d["h0"], o, 1.0)
    with pytest.raises(RuntimeError):  # CPU tensors: no fallback
        G.delta_rule_sequential(*(torch.from_numpy(inp[n]) for n in ("q", "k", "v", "g", "beta")),
                                1.0, torch.from_numpy(inp["h0"]))
