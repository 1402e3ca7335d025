"""GPU parity of the sliding-window attention kernel (pbk_swa_prefill) against the
reference's golden outputs and the oracle (oracle/swa.py).

bf16 inputs, fp32 accumulation: 2e-2 norm-wise relative (the bf16 tolerance) on every
case, per head. A window of one key is exact (each query copies its own value row).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import swa as oswa
from oracle.gdn import rel_err
from oracle.quest import bf16_from_bits, bf16_round
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2


def _inputs(seed, b, h, kv, t, q_scale=1.0, d=128):
    rng = np.random.default_rng(seed)
    q = bf16_round(rng.standard_normal((b, h, t, d), dtype=np.float32) * q_scale)
    k = bf16_round(rng.standard_normal((b, kv, t, d), dtype=np.float32))
    v = bf16_round(rng.standard_normal((b, kv, t, d), dtype=np.float32))
    return q, k, v


def _dev(x, device):
    return torch.from_numpy(x).to(device, torch.bfloat16)


def _assert_heads_close(got, want, tol=TOL_BF16):
    for j in range(got.shape[1]):
        assert rel_err(got[:, j], want[:, j]) < tol, f"head {j}: {rel_err(got[:, j], want[:, j])}"


@pytest.mark.parametrize("case", ["win", "full"])
def test_matches_reference_golden(cuda_device, case):
    from pseudobrain_b200.transplant import causal_attention
    f = load_golden("swa.npz")
    q, k, v = (torch.from_numpy(bf16_from_bits(f[f"{case}_{n}"])).to(cuda_device, torch.bfloat16) for n in "qkv")
    window = int(f[f"{case}_window"])
    o = causal_attention(q, k, v, None if window < 0 else window, int(f[f"{case}_sinks"]))
    assert o.dtype == torch.bfloat16 and o.shape == q.shape
    _assert_heads_close(o.float().cpu().numpy(), f[f"{case}_o"])
    # fp32 in -> fp32 out (the kernel reads bf16; these values are exact in bf16)
    o32 = causal_attention(q.float(), k.float(), v.float(), None if window < 0 else window, int(f[f"{case}_sinks"]))
    assert o32.dtype == torch.float32
    _assert_heads_close(o32.cpu().numpy(), f[f"{case}_o"])


@pytest.mark.parametrize("b,h,kv,t,window,sinks", [
    (1, 2, 1, 1, 4096, 0),        # one token
    (1, 4, 1, 127, 64, 0),        # T < one tile
    (2, 4, 2, 1000, 129, 0),      # window not a tile multiple, ragged T, batch 2
    (1, 8, 2, 700, 128, 200),     # sinks spanning two tiles outside the window
    (1, 3, 1, 300, 100, 5),       # odd group: the last pair has one head
    (1, 1, 1, 520, None, 0),      # MHA, full causal
    (1, 8, 8, 384, 4096, 0),      # window longer than T
])
def test_matches_oracle(cuda_device, b, h, kv, t, window, sinks):
    from pseudobrain_b200.transplant import causal_attention
    q, k, v = _inputs(t + h, b, h, kv, t)
    o = causal_attention(_dev(q, cuda_device), _dev(k, cuda_device), _dev(v, cuda_device), window, sinks)
    _assert_heads_close(o.float().cpu().numpy(), oswa.causal_attention(q, k, v, window, sinks))


def test_large_logits_rescale(cuda_device):
    """Scores that grow along the keys force the running maximum up many times (the
    in-place rescale of O and l); scaled queries make the softmax sharp."""
    from pseudobrain_b200.transplant import causal_attention
    q, k, v = _inputs(7, 1, 2, 1, 1024, q_scale=4.0)
    ramp = np.linspace(0.2, 3.0, 1024, dtype=np.float32)[None, None, :, None]
    k = bf16_round(k * ramp)
    o = causal_attention(_dev(q, cuda_device), _dev(k, cuda_device), _dev(v, cuda_device), 512, 0)
    _assert_heads_close(o.float().cpu().numpy(), oswa.causal_attention(q, k, v, 512, 0))


def test_window_of_one_copies_values_exactly(cuda_device):
    from pseudobrain_b200.transplant import causal_attention
    q, k, v = _inputs(3, 1, 4, 2, 300)
    o = causal_attention(_dev(q, cuda_device), _dev(k, cuda_device), _dev(v, cuda_device), 1, 0)
    want = np.repeat(v, 2, axis=1)
    assert np.array_equal(o.float().cpu().numpy(), want)


def test_strided_views_of_packed_projections(cuda_device):
    """q, k, v as column slices of one packed [B,T,(H+2KV)*hd] projection and o written
    into a [B,T,H*hd] buffer: the out-variant op reads and writes through the strides."""
    from pseudobrain_b200.transplant import window_attention_
    b, t, h, kv, d = 1, 600, 4, 1, 128
    q, k, v = _inputs(11, b, h, kv, t)
    packed = np.concatenate([x.transpose(0, 2, 1, 3).reshape(b, t, -1) for x in (q, k, v)], axis=-1)
    p = torch.from_numpy(np.ascontiguousarray(packed)).to(cuda_device, torch.bfloat16)
    qv = p[..., : h * d].view(b, t, h, d)
    kv_ = p[..., h * d:(h + kv) * d].view(b, t, kv, d)
    vv = p[..., (h + kv) * d:].view(b, t, kv, d)
    out = torch.zeros(b, t, h * d, device=cuda_device, dtype=torch.float32)
    window_attention_(qv, kv_, vv, out.view(b, t, h, d), 256, 0, d ** -0.5)
    got = out.view(b, t, h, d).permute(0, 2, 1, 3).cpu().numpy()
    _assert_heads_close(got, oswa.causal_attention(q, k, v, 256, 0))


def test_long_sequence_sampled_rows(cuda_device):
    """benchmark config-4 branch shape per GPU (4 query heads on one key head, window 4096)
    at T=65536: query runs at the start, across tile boundaries and at the end against the
    oracle's row-subset form."""
    from pseudobrain_b200.transplant import causal_attention
    from pseudobrain_b200 import _capi
    t = 65536
    q, k, v = _inputs(5, 1, 4, 1, t)
    o = causal_attention(_dev(q, cuda_device), _dev(k, cuda_device), _dev(v, cuda_device), 4096, 0)
    got = o.float().cpu().numpy()
    for s, want in oswa.causal_attention_at(q, k, v, [0, 4000, 30001, t - 70], 70, 4096, 0).items():
        _assert_heads_close(got[:, :, s:s + 70], want)
    assert _capi.device_error() == 0


def test_rejects_bad_arguments(cuda_device):
    from pseudobrain_b200 import _capi
    from pseudobrain_b200.transplant import window_attention_
    q = torch.zeros(1, 8, 2, 64, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(_capi.PbkError, match="unsupported shape"):
        window_attention_(q, q[:, :, :1], q[:, :, :1], torch.empty_like(q), 0, 0, 0.125)
    q = torch.zeros(1, 8, 2, 128, device=cuda_device, dtype=torch.float32)
    with pytest.raises(_capi.PbkError, match="unsupported dtype"):
        window_attention_(q, q[:, :, :1], q[:, :, :1], torch.empty_like(q), 0, 0, 0.125)
