"""GPU parity of the sequence-split prefill (segments of one sequence run in parallel,
chained by pbk_gdn_segment_scan) against the oracle and the unsplit kernel.

The decay and beta are made small here so the state carries across many chunks and the
segment transition matrices are far from zero: the chaining is then what is tested.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from tests.inputs import gdn_inputs, to_device

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2


def _slow_inputs(seed, batch, length, hk, hv):
    inp = gdn_inputs(seed, batch, length, hk, hv, bf16=True, state_std=0.05)
    rng = np.random.default_rng(seed + 1)
    inp["g"] = (-0.002 * rng.random((batch, length, hv))).astype(np.float32)
    from oracle.quest import bf16_round
    inp["beta"] = bf16_round((0.05 + 0.1 * rng.random((batch, length, hv))).astype(np.float32))
    return inp


def _oracle(inp):
    hv = inp["v"].shape[2]
    return ogdn.delta_rule_chunked(ogdn.expand_key_heads(inp["q"], hv), ogdn.expand_key_heads(inp["k"], hv),
                                   inp["v"], inp["g"], inp["beta"], inp["scale"], inp["h0"])


def test_segment_scan_matches_numpy(cuda_device):
    from pseudobrain_b200.gdn_prefill import segment_scan
    rng = np.random.default_rng(3)
    batch, nseg, hv = 2, 5, 3
    b = rng.standard_normal((batch, nseg - 1, hv, 128, 128)).astype(np.float32)
    a = (rng.standard_normal((batch, nseg - 1, hv, 128, 128)) / 16).astype(np.float32)
    m = (a + b).astype(np.float32)
    h0 = rng.standard_normal((batch, hv, 128, 128)).astype(np.float32)
    for init in (h0, None):
        starts = torch.empty(batch, nseg, hv, 128, 128, device=cuda_device)
        segment_scan(torch.from_numpy(b).to(cuda_device), torch.from_numpy(m).to(cuda_device),
                     None if init is None else torch.from_numpy(init).to(cuda_device), starts)
        want = np.zeros((batch, nseg, hv, 128, 128))
        want[:, 0] = 0 if init is None else init
        for p in range(nseg - 1):
            want[:, p + 1] = np.einsum("bhkj,bhjv->bhkv", m[:, p].astype(np.float64) - b[:, p], want[:, p]) + b[:, p]
        assert ogdn.rel_err(starts.cpu().numpy(), want) < 1e-5


def test_state_only_run_equals_full_run(cuda_device):
    """o = NULL computes the same final state bit for bit."""
    from pseudobrain_b200.gdn_prefill import gdn_final_state_, gdn_prefill
    inp = gdn_inputs(8, 2, 700, 1, 2, bf16=True, state_std=0.02)
    d = to_device(inp, cuda_device)
    args = [d[n] for n in ("q", "k", "v", "g", "beta")]
    _, s = gdn_prefill(*args, inp["scale"], d["h0"])
    s2 = torch.empty_like(s)
    gdn_final_state_(*args, d["h0"], s2, inp["scale"])
    assert torch.equal(s, s2)


@pytest.mark.parametrize("batch,length,hk,hv,segments", [(2, 1000, 1, 2, 6), (1, 4096, 2, 4, 8), (1, 640, 1, 1, 10)])
def test_segmented_matches_oracle(cuda_device, batch, length, hk, hv, segments):
    from pseudobrain_b200.gdn_prefill import gdn_prefill, gdn_prefill_segmented
    inp = _slow_inputs(length + segments, batch, length, hk, hv)
    d = to_device(inp, cuda_device)
    args = [d[n] for n in ("q", "k", "v", "g", "beta")]
    o, s = gdn_prefill_segmented(*args, inp["scale"], d["h0"], segments=segments)
    ro, rs = _oracle(inp)
    assert ogdn.rel_err(o.cpu().numpy(), ro) < TOL_BF16
    assert ogdn.rel_err(s.cpu().numpy(), rs) < TOL_BF16
    o1, s1 = gdn_prefill(*args, inp["scale"], d["h0"])
    assert ogdn.rel_err(o.cpu().numpy(), o1.cpu().numpy()) < TOL_BF16
    assert ogdn.rel_err(s.cpu().numpy(), s1.cpu().numpy()) < TOL_BF16


def test_segmented_long_sequence(cuda_device):
    """benchmark config-4 GDN shape per GPU of 8 (4 value heads, 2 key heads), shortened to
    T = 65536 + 100: automatic segment count, against the unsplit kernel."""
    from pseudobrain_b200 import _capi
    from pseudobrain_b200.gdn_prefill import auto_segments, gdn_prefill, gdn_prefill_segmented
    t = 65536 + 100
    inp = _slow_inputs(9, 1, t, 2, 4)
    d = to_device(inp, cuda_device)
    args = [d[n] for n in ("q", "k", "v", "g", "beta")]
    assert auto_segments(1, 4, t) > 1
    o, s = gdn_prefill_segmented(*args, inp["scale"], d["h0"], out_dtype=torch.bfloat16)
    o1, s1 = gdn_prefill(*args, inp["scale"], d["h0"], torch.bfloat16)
    assert ogdn.rel_err(o.float().cpu().numpy(), o1.float().cpu().numpy()) < TOL_BF16
    assert ogdn.rel_err(s.cpu().numpy(), s1.cpu().numpy()) < TOL_BF16
    assert _capi.device_error() == 0


def test_segmented_config4_length_matches_oracle(cuda_device):
    """The config-4 GDN shard of one GPU of 8 (2 key / 4 value heads) over T = 262144 + 100
    tokens, split into segments by auto_segments, against the oracle (the reference's
    algorithm on the host, fp32, the whole sequence in order) with a slow decay, so the
    state carries across every segment boundary. Relative errors printed."""
    from oracle import cpu_reference as cr
    from pseudobrain_b200 import _capi
    from pseudobrain_b200.gdn_prefill import auto_segments, gdn_prefill_segmented
    t = 262144 + 100
    inp = _slow_inputs(21, 1, t, 2, 4)
    d = to_device(inp, cuda_device)
    args = [d[n] for n in ("q", "k", "v", "g", "beta")]
    segs = auto_segments(1, 4, t)
    assert segs > 1
    o, s = gdn_prefill_segmented(*args, inp["scale"], d["h0"], out_dtype=torch.bfloat16)
    cr.use_all_cores()
    hq = {n: torch.from_numpy(inp[n]) for n in ("q", "k", "v", "g", "beta", "h0")}
    ro, rs = cr.chunked_prefill(hq["q"].repeat_interleave(2, dim=2), hq["k"].repeat_interleave(2, dim=2), hq["v"],
                                hq["g"], hq["beta"], inp["scale"], hq["h0"])
    eo = ogdn.rel_err(o.float().cpu().numpy(), ro.numpy())
    es = ogdn.rel_err(s.cpu().numpy(), rs.numpy())
    print(f"[segmented prefill, T={t}, {segs} segments vs oracle] rel err o {eo:.2e}, final state {es:.2e}")
    assert eo < TOL_BF16 and es < TOL_BF16
    assert _capi.device_error() == 0
