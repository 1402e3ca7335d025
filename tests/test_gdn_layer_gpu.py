"""GPU parity of the layer pieces around the recurrence (pbk_gdn_conv_norm, pbk_gdn_gating,
pbk_gdn_out_norm) against the reference's outputs (tests/golden/gdn_io.npz) and the oracle.
fp32 outputs: 1e-5 norm-wise relative (fp32 arithmetic in another order); bf16 outputs: the
bf16 rounding bound 4e-3."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu


def _t(x, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev, dtype)


@pytest.mark.parametrize("mode", ["max", "hf"])
@pytest.mark.parametrize("out_dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 4e-3)])
def test_conv_norm_matches_reference(cuda_device, mode, out_dtype, tol):
    from pseudobrain_b200.gdn_layer import conv_qkv
    f = load_golden("gdn_io.npz")
    x, tail, w = (_t(f[n], cuda_device) for n in ("x", "tail", "weight"))
    new_tail = torch.empty_like(tail)
    q, k, v = conv_qkv(x, tail, w, 1, 2, mode, new_tail, out_dtype)
    assert ogdn.rel_err(q.float().cpu().numpy(), f[f"q_{mode}"]) < tol
    assert ogdn.rel_err(k.float().cpu().numpy(), f[f"k_{mode}"]) < tol
    assert ogdn.rel_err(v.float().cpu().numpy(), f["v"]) < tol
    assert np.array_equal(new_tail.cpu().numpy(), f["new_tail"])


def test_conv_short_sequences_and_no_weight(cuda_device):
    """T shorter than the taps (the new tail mixes old tail and inputs), T across several
    token tiles, and SiLU only (no convolution); no normalisation."""
    from pseudobrain_b200.gdn_layer import conv_qkv
    rng = np.random.default_rng(4)
    for t in (1, 2, 33, 97):
        x = rng.standard_normal((2, t, 512)).astype(np.float32)
        tail = rng.standard_normal((2, 3, 512)).astype(np.float32)
        w = (0.5 * rng.standard_normal((512, 4))).astype(np.float32)
        new_tail = torch.empty(2, 3, 512, device=cuda_device)
        q, k, v = conv_qkv(_t(x, cuda_device), _t(tail, cuda_device), _t(w, cuda_device), 1, 2, None, new_tail,
                           torch.float32)
        y, nt = ogdn.short_convolution(x, tail, w)
        got = torch.cat((q.flatten(2), k.flatten(2), v.flatten(2)), -1).cpu().numpy()
        assert ogdn.rel_err(got, y) < 1e-5, t
        assert np.array_equal(new_tail.cpu().numpy(), nt), t
    x = rng.standard_normal((1, 5, 512)).astype(np.float32)
    q, k, v = conv_qkv(_t(x, cuda_device), None, None, 1, 2, None, None, torch.float32)
    got = torch.cat((q.flatten(2), k.flatten(2), v.flatten(2)), -1).cpu().numpy()
    assert ogdn.rel_err(got, ogdn.short_convolution(x, None, None)[0]) < 1e-5


@pytest.mark.parametrize("width", [1, 2, 4, 8])
def test_conv_bf16_staged_path(cuda_device, width):
    """bf16 inputs and outputs with contiguous channels take the staged kernel: against the
    oracle on the same bf16 values (short, ragged and multi-tile T; the tail carried exactly)."""
    from oracle.quest import bf16_round
    from pseudobrain_b200.gdn_layer import conv_qkv
    rng = np.random.default_rng(width)
    for t in (1, 2, 33, 97, 200):
        x = bf16_round(rng.standard_normal((2, t, 640)).astype(np.float32))
        tail = bf16_round(rng.standard_normal((2, width - 1, 640)).astype(np.float32))
        w = (0.5 * rng.standard_normal((640, width))).astype(np.float32)
        new_tail = torch.empty(2, width - 1, 640, device=cuda_device, dtype=torch.bfloat16)
        q, k, v = conv_qkv(_t(x, cuda_device, torch.bfloat16), _t(tail, cuda_device, torch.bfloat16),
                           _t(w, cuda_device), 1, 3, "max", new_tail, torch.bfloat16)
        y, nt = ogdn.short_convolution(x, tail, w)
        y = y.reshape(2, t, 5, 128)
        qn, kn = ogdn.l2_normalize(y[:, :, 0], "max"), ogdn.l2_normalize(y[:, :, 1], "max")
        assert ogdn.rel_err(q[:, :, 0].float().cpu().numpy(), qn) < 4e-3, t
        assert ogdn.rel_err(k[:, :, 0].float().cpu().numpy(), kn) < 4e-3, t
        assert ogdn.rel_err(v.float().cpu().numpy(), y[:, :, 2:]) < 4e-3, t
        assert np.array_equal(new_tail.float().cpu().numpy(), nt), t


def test_gating_matches_reference(cuda_device):
    from pseudobrain_b200.gdn_layer import gdn_gating
    f = load_golden("gdn_io.npz")
    g, beta = gdn_gating(_t(f["decay"], cuda_device), _t(f["a_log"], cuda_device), _t(f["dt_bias"], cuda_device))
    assert ogdn.rel_err(g.cpu().numpy(), f["g"]) < 1e-5
    assert ogdn.rel_err(beta.cpu().numpy(), f["beta"]) < 1e-5


@pytest.mark.parametrize("in_dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 4e-3)])
def test_out_norm_matches_reference(cuda_device, in_dtype, tol):
    from pseudobrain_b200.gdn_layer import gated_out_norm
    f = load_golden("gdn_io.npz")
    o = _t(f["o"], cuda_device, in_dtype)
    gate = _t(f["gate"], cuda_device, in_dtype)
    out = gated_out_norm(o, gate, _t(f["o_norm"], cuda_device), out_dtype=torch.float32)
    want = f["out"] if in_dtype == torch.float32 else ogdn.gated_out_norm(
        o.float().cpu().numpy(), gate.float().cpu().numpy().reshape(o.shape), f["o_norm"])
    assert ogdn.rel_err(out.cpu().numpy(), want) < tol


def test_layer_core_matches_oracle_composition(cuda_device):
    """conv + norm + gating + recurrence (chunked prefill, then a 1-token decode carrying
    state and tail) + gated output norm, against the oracle's pieces composed the way
    GatedDeltaNetLayer.forward composes them (gated_deltanet.py:411-440)."""
    from pseudobrain_b200.gdn_layer import gated_deltanet_core
    rng = np.random.default_rng(6)
    b, hk, hv, c = 1, 1, 2, 512
    w = (0.3 * rng.standard_normal((c, 4))).astype(np.float32)
    a_log = rng.standard_normal(hv).astype(np.float32) * 0.5
    dt_bias = rng.standard_normal(hv).astype(np.float32)
    o_norm = (1.0 + 0.2 * rng.standard_normal(128)).astype(np.float32)
    tail = np.zeros((b, 3, c), np.float32)
    state = np.zeros((b, hv, 128, 128), np.float32)
    d_tail, d_state = _t(tail, cuda_device), _t(state, cuda_device)
    for t in (150, 1):
        qkv = rng.standard_normal((b, t, c)).astype(np.float32)
        gate = rng.standard_normal((b, t, hv * 128)).astype(np.float32)
        decay = rng.standard_normal((b, t, 2 * hv)).astype(np.float32)
        out, d_state, d_tail = gated_deltanet_core(_t(qkv, cuda_device), _t(gate, cuda_device), _t(decay, cuda_device),
                                                   d_tail, _t(w, cuda_device), _t(a_log, cuda_device),
                                                   _t(dt_bias, cuda_device), _t(o_norm, cuda_device), d_state, hk, hv)
        y, tail = ogdn.short_convolution(qkv, tail, w)
        q = ogdn.l2_normalize(y[..., :128].reshape(b, t, hk, 128))
        k = ogdn.l2_normalize(y[..., 128:256].reshape(b, t, hk, 128))
        v = y[..., 256:].reshape(b, t, hv, 128)
        from oracle.quest import bf16_round
        q, k, v = (bf16_round(x.astype(np.float32)) for x in (q, k, v))  # the kernels read bf16 q/k/v
        g, beta = ogdn.gating(decay[..., :hv], decay[..., hv:], a_log, dt_bias)
        beta = bf16_round(beta)
        qe, ke = ogdn.expand_key_heads(q, hv), ogdn.expand_key_heads(k, hv)
        fn = ogdn.delta_rule_sequential if t <= 4 else ogdn.delta_rule_chunked
        o, state = fn(qe, ke, v, g, beta, 128 ** -0.5, state)
        want = ogdn.gated_out_norm(o, gate.reshape(b, t, hv, 128), o_norm)
        assert ogdn.rel_err(out.cpu().numpy(), want) < 2e-2, t
        assert ogdn.rel_err(d_state.cpu().numpy(), state) < 2e-2, t
        assert np.allclose(d_tail.cpu().numpy(), tail), t


def _oracle_decode_layer(qkv, gate, decay, tail, w, a_log, dt_bias, o_norm, state, hk, hv, mode):
    """The reference layer's decode step composed from the oracle's pieces in fp32
    (gated_deltanet.py:411-440: conv, q/k norm, gating, the sequential recurrence, output norm)."""
    b, t, _ = qkv.shape
    y, new_tail = ogdn.short_convolution(qkv, tail, w)
    q = y[..., :hk * 128].reshape(b, t, hk, 128)
    k = y[..., hk * 128:2 * hk * 128].reshape(b, t, hk, 128)
    if mode is not None:
        q, k = ogdn.l2_normalize(q, mode), ogdn.l2_normalize(k, mode)
    v = y[..., 2 * hk * 128:].reshape(b, t, hv, 128)
    g, beta = ogdn.gating(decay[..., :hv], decay[..., hv:], a_log, dt_bias)
    o, new_state = ogdn.delta_rule_sequential(ogdn.expand_key_heads(q, hv), ogdn.expand_key_heads(k, hv), v, g, beta,
                                              128 ** -0.5, state)
    return ogdn.gated_out_norm(o, gate.reshape(b, t, hv, 128), o_norm), new_state, new_tail


@pytest.mark.gpu
@pytest.mark.parametrize("hk,hv,width,layout,mode,in_dtype,out_dtype", [
    (1, 2, 4, "kv", "max", torch.float32, torch.float32),
    (1, 2, 4, "vk", "hf", torch.float32, torch.float32),
    (2, 8, 4, "kv", "max", torch.bfloat16, torch.bfloat16),
    (2, 8, 6, "vk", "max", torch.float32, torch.float32),
    (3, 3, 8, "kv", "hf", torch.float32, torch.bfloat16),
    (2, 4, 1, "vk", None, torch.float32, torch.float32),
])
def test_decode_layer_fused_matches_oracle(cuda_device, hk, hv, width, layout, mode, in_dtype, out_dtype):
    """pbk_gdn_decode_layer (conv + SiLU + q/k norm + gating + recurrence + output norm in one
    kernel) over three decode steps of 1, 3 and 1 tokens, the state and the conv tail carried
    in place (value heads of a key head as one cluster when they share tail channels), against
    the reference layer's pieces composed in fp32; a negative state index skips its sequence
    and leaves its state and tail as they were."""
    from oracle.quest import bf16_round
    from pseudobrain_b200.gdn_layer import gated_deltanet_decode
    rng = np.random.default_rng(11 + hv + width)
    b, c = 3, (2 * hk + hv) * 128
    w = (0.4 * rng.standard_normal((c, width))).astype(np.float32) if width > 1 else None
    a_log = (0.5 * rng.standard_normal(hv)).astype(np.float32)
    dt_bias = rng.standard_normal(hv).astype(np.float32)
    o_norm = (1.0 + 0.2 * rng.standard_normal(128)).astype(np.float32)
    tail = rng.standard_normal((b, max(width - 1, 0), c)).astype(np.float32)
    state = (0.05 * rng.standard_normal((b, hv, 128, 128))).astype(np.float32)
    rnd = (lambda x: bf16_round(x)) if in_dtype == torch.bfloat16 else (lambda x: x)
    tail = rnd(tail)
    d_tail = _t(tail, cuda_device, in_dtype) if width > 1 else None
    d_state = _t(state if layout == "kv" else state.transpose(0, 1, 3, 2).copy(), cuda_device)
    idx = torch.tensor([0, -1, 2], dtype=torch.int32, device=cuda_device)  # sequence 1 skipped
    tol = 1e-4 if out_dtype == torch.float32 and in_dtype == torch.float32 else 2e-2
    for t in (1, 3, 1):
        qkv = rnd(rng.standard_normal((b, t, c)).astype(np.float32))
        gate = rnd(rng.standard_normal((b, t, hv * 128)).astype(np.float32))
        decay = rnd(rng.standard_normal((b, t, 2 * hv)).astype(np.float32))
        out = gated_deltanet_decode(_t(qkv, cuda_device, in_dtype), _t(gate, cuda_device, in_dtype),
                                    _t(decay, cuda_device, in_dtype), d_tail,
                                    _t(w, cuda_device) if w is not None else None, _t(a_log, cuda_device),
                                    _t(dt_bias, cuda_device), _t(o_norm, cuda_device), d_state, hk, hv, mode,
                                    state_layout=layout, state_indices=idx, out_dtype=out_dtype)
        live = [0, 2]
        want, st_new, tl_new = _oracle_decode_layer(qkv[live], gate[live], decay[live],
                                                    tail[live] if width > 1 else None, w, a_log, dt_bias, o_norm,
                                                    state[live], hk, hv, mode)
        got = out.float().cpu().numpy()[live]
        err = ogdn.rel_err(got, want)
        print(f"[decode layer hk={hk} hv={hv} K={width} {layout} t={t}] rel err {err:.2e}")
        assert err < tol
        state[live] = st_new
        if width > 1:
            tail[live] = tl_new
        gs = d_state.cpu().numpy()
        gs = gs if layout == "kv" else gs.transpose(0, 1, 3, 2)
        assert ogdn.rel_err(gs[live], state[live]) < tol
        assert np.array_equal(gs[1], state[1])  # the skipped slot is untouched
        if width > 1:
            assert np.array_equal(d_tail.float().cpu().numpy(), tail)
    from pseudobrain_b200._capi import device_error
    assert device_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("hk,hv,width,t,mode,layout", [
    (1, 2, 4, 150, "max", "kv"),
    (2, 8, 4, 200, "max", "vk"),
    (2, 6, 3, 69, "hf", "kv"),
    (1, 1, 1, 64, "max", "kv"),
    (1, 2, 4, 2, "max", "kv"),
])
def test_prefill_layer_fused_matches_oracle(cuda_device, hk, hv, width, t, mode, layout):
    """pbk_gdn_prefill_layer (the chunk solve with conv + SiLU + q/k norm + gating fused in,
    the tensor-core recurrence, the gated output norm) against the reference layer's pieces
    composed in fp32 with the chunked recurrence, from a nonzero state and tail; then a second
    call continues from the returned state and tail. Sequence 1 is skipped by its state index."""
    from oracle.quest import bf16_round
    from pseudobrain_b200.gdn_layer import gated_deltanet_prefill
    rng = np.random.default_rng(31 + hv + t)
    b, c = 3, (2 * hk + hv) * 128
    w = (0.4 * rng.standard_normal((c, width))).astype(np.float32) if width > 1 else None
    a_log = (0.5 * rng.standard_normal(hv)).astype(np.float32)
    dt_bias = rng.standard_normal(hv).astype(np.float32)
    o_norm = (1.0 + 0.2 * rng.standard_normal(128)).astype(np.float32)
    tail = bf16_round(rng.standard_normal((b, max(width - 1, 0), c)).astype(np.float32))
    state = (0.05 * rng.standard_normal((b, hv, 128, 128))).astype(np.float32)
    d_state = _t(state if layout == "kv" else state.transpose(0, 1, 3, 2).copy(), cuda_device)
    idx = torch.tensor([0, -1, 2], dtype=torch.int32, device=cuda_device)
    live = [0, 2]
    d_tail = _t(tail, cuda_device, torch.bfloat16) if width > 1 else None
    for step in range(2):
        qkv = bf16_round(rng.standard_normal((b, t, c)).astype(np.float32))
        gate = bf16_round(rng.standard_normal((b, t, hv * 128)).astype(np.float32))
        decay = bf16_round(rng.standard_normal((b, t, 2 * hv)).astype(np.float32))
        d_new = torch.full_like(d_tail, 7.0) if width > 1 else None
        out = gated_deltanet_prefill(_t(qkv, cuda_device, torch.bfloat16), _t(gate, cuda_device, torch.bfloat16),
                                     _t(decay, cuda_device, torch.bfloat16), d_tail,
                                     _t(w, cuda_device) if w is not None else None, _t(a_log, cuda_device),
                                     _t(dt_bias, cuda_device), _t(o_norm, cuda_device), d_state, hk, hv, mode,
                                     new_tail=d_new, state_layout=layout, state_indices=idx)
        y, new_tail = ogdn.short_convolution(qkv[live], tail[live] if width > 1 else None, w)
        bl = len(live)
        q = ogdn.l2_normalize(y[..., :hk * 128].reshape(bl, t, hk, 128), mode)
        k = ogdn.l2_normalize(y[..., hk * 128:2 * hk * 128].reshape(bl, t, hk, 128), mode)
        v = y[..., 2 * hk * 128:].reshape(bl, t, hv, 128)
        q, k, v = (bf16_round(x.astype(np.float32)) for x in (q, k, v))  # the tensor cores read bf16
        g, beta = ogdn.gating(decay[live][..., :hv], decay[live][..., hv:], a_log, dt_bias)
        o, st_new = ogdn.delta_rule_chunked(ogdn.expand_key_heads(q, hv), ogdn.expand_key_heads(k, hv), v, g, beta,
                                            128 ** -0.5, state[live])
        want = ogdn.gated_out_norm(o, gate[live].reshape(bl, t, hv, 128), o_norm)
        err = ogdn.rel_err(out.cpu().numpy()[live], want)
        gs = d_state.cpu().numpy()
        gs = gs if layout == "kv" else gs.transpose(0, 1, 3, 2)
        serr = ogdn.rel_err(gs[live], st_new)
        print(f"[prefill layer hk={hk} hv={hv} K={width} T={t} step {step}] rel err out {err:.2e} state {serr:.2e}")
        assert err < 2e-2 and serr < 2e-2
        assert np.array_equal(gs[1], state[1])  # skipped sequence: state untouched
        state[live] = st_new
        if width > 1:
            got_tail = d_new.float().cpu().numpy()
            assert np.array_equal(got_tail[live], new_tail)
            assert np.all(got_tail[1] == 7.0)  # skipped sequence: no tail written
            tail[live] = new_tail
            d_tail = d_new
    from pseudobrain_b200._capi import device_error
    assert device_error() == 0
