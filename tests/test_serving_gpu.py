"""GPU parity of the serving twins (pb27_vllm/memory.py retrieve_blocks and piece_attention)
against the reference's golden outputs and the oracle (oracle/serving.py): block sets
identical, attention within 5e-3 (bf16 tensor-core products, fp32 accumulation, bf16
probabilities in the P V product)."""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from oracle import serving as osv
from oracle.gdn import rel_err
from oracle.quest import bf16_from_bits, bf16_round
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu
TOL = 5e-3


@pytest.fixture
def memory_settings():
    from pseudobrain_b200 import serving as S
    saved = dict(S.MEMORY)
    yield S.MEMORY
    S.MEMORY.clear()
    S.MEMORY.update(saved)


def _archive(keys, values, block, device, bounds=None):
    kv, cap, d = keys.shape
    n_blk = cap // block
    arc = types.SimpleNamespace(
        keys=torch.from_numpy(keys).to(device, torch.bfloat16), values=torch.from_numpy(values).to(device, torch.bfloat16),
        kmax=torch.zeros(kv, n_blk, d, dtype=torch.bfloat16, device=device),
        kmin=torch.zeros(kv, n_blk, d, dtype=torch.bfloat16, device=device),
        size=cap, prompt_len=cap, hole_lo=0, hole_hi=0, smax=None, dirty_lo=0, dirty_hi=n_blk - 1)
    return arc


@pytest.mark.parametrize("case", ["t1", "t3", "flat"])
def test_matches_reference_golden(cuda_device, memory_settings, case):
    from pseudobrain_b200 import serving as S
    f = load_golden("serving.npz")
    memory_settings.update(blocks=int(f["budget"]), decode_blocks=int(f["budget"]), rerank=int(f["rerank_pool"]),
                           block_size=int(f["block"]), window=int(f["window"]))
    arc = _archive(bf16_from_bits(f["keys"]), bf16_from_bits(f["values"]), int(f["block"]), cuda_device)
    q = torch.from_numpy(bf16_from_bits(f[f"{case}_q"])).to(cuda_device, torch.bfloat16)
    top = S.retrieve_blocks(arc, q, int(f["groups"]), int(f[f"{case}_limit"]), bool(f[f"{case}_rerank"]))
    # the bounds were refreshed from the keys by this package's kernel: bit-exact
    assert np.array_equal(arc.kmax.view(torch.int16).cpu().numpy().view(np.uint16), f["kmax"])
    assert np.array_equal(arc.kmin.view(torch.int16).cpu().numpy().view(np.uint16), f["kmin"])
    assert np.array_equal(top.cpu().numpy(), f[f"{case}_top"])
    pos = torch.from_numpy(f[f"{case}_pos"]).to(cuda_device)
    out = S.piece_attention(arc, q.float(), pos, top, int(f["groups"]), int(f["window"]), 128 ** -0.5)
    assert out.dtype == torch.float32
    assert rel_err(out.cpu().numpy(), f[f"{case}_out"]) < TOL


@pytest.mark.parametrize("t,rerank", [(1, True), (5, True), (1, False), (64, True)])
def test_matches_oracle(cuda_device, memory_settings, t, rerank):
    """PB-27's head layout (24 query / 4 key heads; head dim 128 here), 200 blocks of 64."""
    from pseudobrain_b200 import serving as S
    memory_settings.update(blocks=16, decode_blocks=16, rerank=40, block_size=64, window=512)
    mem = dict(memory_settings)
    rng = np.random.default_rng(t * 7 + rerank)
    kv, groups, d, block = 4, 6, 128, 64
    cap = S.ORIGIN + 200 * block + 33
    keys = bf16_round(rng.standard_normal((kv, cap, d), dtype=np.float32))
    values = bf16_round(rng.standard_normal((kv, cap, d), dtype=np.float32))
    arc = _archive(keys, values, block, cuda_device)
    q_np = bf16_round(rng.standard_normal((t, kv * groups, d), dtype=np.float32))
    q = torch.from_numpy(q_np).to(cuda_device, torch.bfloat16)
    q_pos = np.arange(cap - t, cap)
    limit = int(q_pos[0]) - 512 + 1
    top = S.retrieve_blocks(arc, q, groups, limit, rerank)
    kmax = arc.kmax.float().cpu().numpy()
    kmin = arc.kmin.float().cpu().numpy()
    want = osv.retrieve_blocks(keys, kmax, kmin, q_np, groups, limit, rerank, mem, cap, canonical=True)
    assert np.array_equal(top.cpu().numpy(), want)  # canonical-order scores: bit-exact
    out = S.piece_attention(arc, q, torch.from_numpy(q_pos).to(cuda_device), top, groups, 512, d ** -0.5)
    assert out.dtype == torch.bfloat16
    ref = osv.piece_attention(keys, values, q_np, q_pos, want, groups, 512, d ** -0.5, block)
    assert rel_err(out.float().cpu().numpy(), ref) < 1e-2  # bf16 output


def test_early_piece_without_archive(cuda_device, memory_settings):
    """Queries whose window still covers the sinks: no blocks, attention over the window."""
    from pseudobrain_b200 import serving as S
    memory_settings.update(block_size=64, window=512)
    rng = np.random.default_rng(5)
    keys = bf16_round(rng.standard_normal((2, 300, 128), dtype=np.float32))
    values = bf16_round(rng.standard_normal((2, 300, 128), dtype=np.float32))
    arc = _archive(keys, values, 64, cuda_device)
    q_np = bf16_round(rng.standard_normal((2, 4, 128), dtype=np.float32))
    q_pos = np.array([200, 201])
    assert S.retrieve_blocks(arc, torch.from_numpy(q_np).to(cuda_device, torch.bfloat16), 2, 200 - 512 + 1,
                             True) is None
    out = S.piece_attention(arc, torch.from_numpy(q_np).to(cuda_device), torch.from_numpy(q_pos).to(cuda_device),
                            None, 2, 512, 128 ** -0.5)
    ref = osv.piece_attention(keys, values, q_np, q_pos, None, 2, 512, 128 ** -0.5, 64)
    assert rel_err(out.cpu().numpy(), ref) < TOL
