"""GPU parity of the RoPE repositioning past the horizon (pbk_quest_rope_gather;
pb27_vllm/memory.py:574-677): moved keys against the reference's own moves
(tests/golden/rope.npz), and the serving twins past a lowered horizon against the
reference's outputs and the oracle.

Moved keys are bf16: both sides turn them in fp32 with the same operation order, so they
agree but for rare last-bit differences of cos/sin (at most 0.1% of the elements, each within
1%). Attention: 5e-3 relative, as the other attention tests.
"""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from oracle import quest as oq
from oracle import serving as osv
from oracle.gdn import rel_err
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.fixture
def lowered_horizon():
    from pseudobrain_b200 import serving as S
    saved = (S.ROPE_HORIZON, S.ROPE_ARC_SPAN, dict(S.MEMORY))
    S.ROPE_HORIZON, S.ROPE_ARC_SPAN = 1500, 600
    yield S
    S.ROPE_HORIZON, S.ROPE_ARC_SPAN = saved[0], saved[1]
    S.MEMORY.clear()
    S.MEMORY.update(saved[2])


def _close_bits(got: np.ndarray, want: np.ndarray) -> None:
    assert np.mean(got != want) < 1e-3
    g, w = oq.bf16_from_bits(got), oq.bf16_from_bits(want)
    assert np.allclose(g, w, rtol=1e-2, atol=1e-2)


def test_moves_match_reference(cuda_device, lowered_horizon):
    S = lowered_horizon
    f = load_golden("rope.npz")
    block, ref_pos, idx = int(f["block"]), int(f["ref_pos"]), f["idx"]
    kv, n = idx.shape
    rk = oq.bf16_from_bits(f["rk"]).reshape(kv, n, block, 128)
    # an archive holding the blocks at their positions (origin 4), other rows random
    rows = S.ORIGIN + (int(idx.max()) + 1) * block + 5
    arc = np.random.default_rng(0).standard_normal((kv, rows, 128)).astype(np.float32)
    for h in range(kv):
        for j, b in enumerate(idx[h]):
            arc[h, S.ORIGIN + b * block:S.ORIGIN + (b + 1) * block] = rk[h, j]
    keys = torch.from_numpy(arc).to(cuda_device, torch.bfloat16)
    values = keys.flip(-1).contiguous()
    blocks = torch.from_numpy(idx).to(cuda_device, torch.int32)
    for mode, want in (("runs", f["rk_runs"]), ("proportional", f["rk_prop"])):
        ok, ov = S.rope_gather(keys, values, blocks, block, S.ORIGIN, n, mode, ref_pos=ref_pos, tail0=7, tail_n=3)
        _close_bits(_bits(ok[:, : n * block]), want)
        ref = osv.reposition_blocks(rk.reshape(kv, n * block, 128), idx, block, ref_pos, mode == "runs", 1500, 600)
        _close_bits(_bits(ok[:, : n * block]), oq.bf16_bits(ref))
        # values gathered unturned; the tail rows copied as they are
        vv = values.float().cpu().numpy()
        for h in range(kv):
            want_v = np.concatenate([vv[h, S.ORIGIN + b * block:S.ORIGIN + (b + 1) * block] for b in idx[h]] +
                                    [vv[h, 7:10]])
            assert np.array_equal(ov[h].float().cpu().numpy(), want_v)
        assert torch.equal(ok[:, n * block:], keys[:, 7:10])
    sk = torch.from_numpy(oq.bf16_from_bits(f["sk"])).to(cuda_device, torch.bfloat16)
    shift = S.sink_shift(ref_pos, 4, n, block)
    ok, _ = S.rope_gather(sk, None, None, 4, 0, 1, "constant", const_delta=shift)
    _close_bits(_bits(ok), f["sk_moved"])


def test_plain_gather_and_out_of_range_rows(cuda_device, lowered_horizon):
    """mode 'none' copies; archive rows past the end read as zeros (no access outside)."""
    S = lowered_horizon
    keys = torch.randn(2, 100, 128, device=cuda_device).to(torch.bfloat16)
    blocks = torch.tensor([[0, 5, 6], [1, 2, 7]], dtype=torch.int32, device=cuda_device)  # block 6, 7 past row 100
    ok, _ = S.rope_gather(keys, None, blocks, 16, 4, 3, "none")
    for h in range(2):
        for j in range(3):
            b = int(blocks[h, j])
            for s in range(16):
                r = 4 + b * 16 + s
                want = keys[h, r] if r < 100 else torch.zeros(128, dtype=keys.dtype, device=cuda_device)
                assert torch.equal(ok[h, j * 16 + s], want)


@pytest.mark.parametrize("case", ["rr", "flat"])
def test_serving_past_horizon(cuda_device, lowered_horizon, case):
    """retrieve_blocks (the rerank on moved candidate keys, or flat scoring with the RoPE dims
    masked) and piece_attention with moved sinks and blocks, against the reference's outputs
    (fp32 keys there, bf16 here) and the oracle on bf16 keys."""
    S = lowered_horizon
    f = load_golden("rope.npz")
    block, groups, window = int(f["block"]), int(f["groups"]), int(f["window"])
    S.MEMORY.update(blocks=4, decode_blocks=4, rerank=12, block_size=block, neighbors=0, window=window)
    keys_np, values_np = oq.bf16_from_bits(f["keys"]), oq.bf16_from_bits(f["values"])
    kv, cap, d = keys_np.shape
    n_blk = cap // block
    arc = types.SimpleNamespace(
        keys=torch.from_numpy(keys_np).to(cuda_device, torch.bfloat16),
        values=torch.from_numpy(values_np).to(cuda_device, torch.bfloat16),
        kmax=torch.zeros(kv, n_blk, d, dtype=torch.bfloat16, device=cuda_device),
        kmin=torch.zeros(kv, n_blk, d, dtype=torch.bfloat16, device=cuda_device),
        size=cap, prompt_len=cap, hole_lo=0, hole_hi=0, smax=None, dirty_lo=0, dirty_hi=n_blk - 1)
    q = torch.from_numpy(oq.bf16_from_bits(f[f"{case}_q"])).to(cuda_device, torch.bfloat16)
    limit = int(f[f"{case}_limit"])
    top = S.retrieve_blocks(arc, q, groups, limit, bool(f[f"{case}_rerank"]))
    assert np.array_equal(top.cpu().numpy(), f[f"{case}_top"])
    pos = torch.from_numpy(f[f"{case}_pos"]).to(cuda_device)
    out = S.piece_attention(arc, q.float(), pos, top, groups, window, 128 ** -0.5)
    assert rel_err(out.cpu().numpy(), f[f"{case}_out"]) < 5e-3
    ref = osv.piece_attention(keys_np, values_np, oq.bf16_from_bits(f[f"{case}_q"]), f[f"{case}_pos"],
                              top.cpu().numpy(), groups, window, 128 ** -0.5, block,
                              rope=(1500, 600, S.ROPE_THETA))
    assert rel_err(out.cpu().numpy(), ref) < 5e-3
