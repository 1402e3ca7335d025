"""GPU parity of the serving archive's write fused with its block summaries
(pbk_quest_archive_write, pbk_quest_supermeans; pb27_vllm/memory.py:310-430) against the
reference's own Archive.write (tests/golden/archive_write.npz) and the oracle.

Storage, max / min summaries and super-block max / min are bit-exact. Block means are bf16
roundings of fp32 sums in another order than the reference's: within one bf16 rounding step
(relative 2^-8). Super-block means average bf16 block means here and fp32 ones there: within
2% relative or 2e-3 absolute.
"""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from oracle import quest as oq
from oracle import serving as osv
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture
def sblk2():
    from pseudobrain_b200 import serving as S
    saved = S.SBLK
    S.SBLK = 2
    yield S
    S.SBLK = saved


def _archive(kv, d, cap, block, sblk, dev):
    n_blk = cap // block
    n_sb = (n_blk + sblk - 1) // sblk
    z = lambda rows: torch.zeros(kv, rows, d, dtype=torch.bfloat16, device=dev)  # noqa: E731
    return types.SimpleNamespace(keys=z(cap), values=z(cap), kmax=z(n_blk), kmin=z(n_blk), bmean_k=z(n_blk),
                                 bmean_v=z(n_blk), smax=z(n_sb), smin=z(n_sb), smean_k=z(n_sb), smean_v=z(n_sb),
                                 size=0, dirty_lo=1 << 60, dirty_hi=-1, prompt_len=0, hole_lo=0, hole_hi=0)


def _f(t):
    return t.float().cpu().numpy()


def _check(arc, want: dict, size: int, block: int, sblk: int):
    assert arc.size == size
    nb = (size - osv.ORIGIN + block - 1) // block
    nsb = (nb + sblk - 1) // sblk
    assert np.array_equal(_f(arc.keys[:, :size]), want["keys"][:, :size])
    assert np.array_equal(_f(arc.values[:, :size]), want["values"][:, :size])
    for name, n in (("kmax", nb), ("kmin", nb), ("smax", nsb), ("smin", nsb)):
        assert np.array_equal(_f(getattr(arc, name))[:, :n], want[name][:, :n]), name
    for name in ("bmean_k", "bmean_v"):
        assert np.allclose(_f(getattr(arc, name))[:, :nb], want[name][:, :nb], rtol=2 ** -8, atol=1e-6), name
    for name in ("smean_k", "smean_v"):
        assert np.allclose(_f(getattr(arc, name))[:, :nsb], want[name][:, :nsb], rtol=2e-2, atol=2e-3), name


def test_golden_archive_writes(cuda_device, sblk2):
    """The reference's write sequence (a prefill write, short and scattered writes, a long
    write across super-blocks, then the refresh) replayed through archive_write."""
    S = sblk2
    f = load_golden("archive_write.npz")
    block, sblk, cap = int(f["block"]), int(f["sblk"]), int(f["cap"])
    kv, d = f["keys"].shape[0], f["keys"].shape[2]
    arc = _archive(kv, d, cap, block, sblk, cuda_device)
    for i in range(int(f["n_writes"])):
        pos = torch.from_numpy(f[f"w{i}_pos"]).to(cuda_device)
        k = torch.from_numpy(oq.bf16_from_bits(f[f"w{i}_k"])).to(cuda_device, torch.bfloat16)
        v = torch.from_numpy(oq.bf16_from_bits(f[f"w{i}_v"])).to(cuda_device, torch.bfloat16)
        S.archive_write(arc, pos, k, v, block)
    S._refresh(arc, block)
    want = {name: f[name] for name in ("kmax", "kmin", "bmean_k", "bmean_v", "smax", "smin", "smean_k", "smean_v")}
    want["keys"], want["values"] = oq.bf16_from_bits(f["keys"]), oq.bf16_from_bits(f["values"])
    _check(arc, want, int(f["size"]), block, sblk)


@pytest.mark.parametrize("block", [16, 64])
def test_writes_with_growth_match_oracle(cuda_device, sblk2, block):
    """Random contiguous and scattered writes into an archive that starts small and grows
    (Archive.grow), against the oracle's ArchiveState, with a strided (token-major view) input."""
    S = sblk2
    rng = np.random.default_rng(block)
    kv, d = 3, 128
    arc = _archive(kv, d, 4 * block, block, 2, cuda_device)
    ref = osv.ArchiveState(kv, d, 64 * block, block, 2)
    p = 0
    for step in range(12):
        if step % 4 == 3 and p > 8:  # scattered re-writes of earlier positions
            pos = np.sort(rng.choice(p, size=min(5, p), replace=False))
        else:
            n = int(rng.integers(1, 3 * block))
            pos = np.arange(p, p + n)
            p += n
        big = oq.bf16_round(rng.standard_normal((len(pos), kv, 2, d)).astype(np.float32))
        k, v = big[:, :, 0], big[:, :, 1]  # token-major views with a key-head stride of 2 d
        dk = torch.from_numpy(big).to(cuda_device, torch.bfloat16)
        S.archive_write(arc, torch.from_numpy(pos).to(cuda_device), dk[:, :, 0], dk[:, :, 1], block)
        ref.write(pos, k, v)
    S._refresh(arc, block)
    ref.refresh_bounds()
    assert arc.keys.shape[1] >= p
    want = {name: getattr(ref, name) for name in ("keys", "values", "kmax", "kmin", "bmean_k", "bmean_v", "smax",
                                                   "smin", "smean_k", "smean_v")}
    _check(arc, want, p, block, 2)
    from pseudobrain_b200._capi import device_error
    assert device_error() == 0


@pytest.mark.parametrize("rerank,sb", [(False, False), (False, True), (True, False)])
def test_offloaded_archive_equals_hbm_archive(cuda_device, sblk2, rerank, sb, tmp_path):
    """offload_archive (keys and values in unlinked sparse files mapped into host memory, the
    reference's NVMe format; summaries in HBM) gives the same summaries, block selections and
    attention as the same writes into an archive in HBM (the same kernels on the same rows)."""
    S = sblk2
    saved = dict(S.MEMORY)
    try:
        S.MEMORY.update(blocks=6, decode_blocks=6, rerank=12, block_size=16, neighbors=0, window=64)
        kv, d, block, cap, groups = 2, 128, 16, 1600, 3
        host = S.offload_archive(kv, d, cap, block, cuda_device, directory=str(tmp_path))
        dev = _archive(kv, d, cap, block, 2, cuda_device)
        if not sb:
            host.smax = dev.smax = None
        rng = np.random.default_rng(int(rerank) + 2 * int(sb))
        p = 0
        for n in (300, 5, 1, 700, 37, 400):
            kk = torch.from_numpy(oq.bf16_round(rng.standard_normal((n, kv, d)).astype(np.float32))).to(cuda_device,
                                                                                                         torch.bfloat16)
            vv = torch.from_numpy(oq.bf16_round(rng.standard_normal((n, kv, d)).astype(np.float32))).to(cuda_device,
                                                                                                         torch.bfloat16)
            pos = torch.arange(p, p + n, device=cuda_device)
            for arc in (host, dev):
                S.archive_write(arc, pos, kk, vv, block)
            p += n
        scat = torch.tensor([20, 700, 1000], device=cuda_device)  # scattered re-writes
        kk = torch.randn(3, kv, d, device=cuda_device).to(torch.bfloat16)
        for arc in (host, dev):
            S.archive_write(arc, scat, kk, kk, block)
        for arc in (host, dev):
            arc.prompt_len = p
            arc.hole_lo, arc.hole_hi = 4 + 16 * 20, 4 + 16 * 31
        q = torch.randn(2, kv * groups, d, device=cuda_device).to(torch.bfloat16)
        limit = p - 64
        tops = [S.retrieve_blocks(arc, q, groups, limit, rerank) for arc in (host, dev)]
        assert torch.equal(tops[0], tops[1])
        for name in ("kmax", "kmin", "bmean_k", "bmean_v") + (("smax", "smin", "smean_k", "smean_v") if sb else ()):
            assert torch.equal(getattr(host, name), getattr(dev, name)), name
        q_pos = torch.tensor([p - 2, p - 1], device=cuda_device)
        outs = [S.piece_attention(arc, q, q_pos, tops[0], groups, 64, d ** -0.5) for arc in (host, dev)]
        assert torch.equal(outs[0], outs[1])
        assert torch.equal(host.keys[:, :p], dev.keys[:, :p].cpu())
    finally:
        S.MEMORY.clear()
        S.MEMORY.update(saved)
