"""GPU parity of the Quest selection modes beyond the flat one: super-block bounds
(pbk_quest_superbounds), the two-level super-block selection and the hole-masked selection
(pbk_quest_select_levels), the research retrieve's exact rerank, neighbours and kept prompt
selection, and the serving retrieve_blocks' super-block, hole and neighbour paths.

Bounds and page indices must be bit-exact: random cases are compared with the oracle's
canonical-order selections (fp32 sums over d = 0..127 of the exact products, ties to the
lowest index) with no tolerance; the golden cases (the reference's own outputs) have no
near-ties and are compared as they are.
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


def _bf16(bits, dev):
    return torch.from_numpy(oq.bf16_from_bits(bits)).to(dev, torch.bfloat16)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.fixture
def quest_cfg():
    from pseudobrain_b200 import exact_memory as M
    saved = dict(M.EXACT_MEMORY)
    yield M
    M.EXACT_MEMORY.clear()
    M.EXACT_MEMORY.update(saved)


@pytest.fixture
def serving_cfg():
    from pseudobrain_b200 import serving as S
    saved, sblk = dict(S.MEMORY), S.SBLK
    yield S
    S.MEMORY.clear()
    S.MEMORY.update(saved)
    S.SBLK = sblk


@pytest.mark.parametrize("kv,n_blk,sblk,first", [(2, 101, 2, 0), (4, 1000, 64, 0), (3, 77, 8, 5), (1, 5, 16, 0)])
def test_superbounds_bit_exact(cuda_device, kv, n_blk, sblk, first):
    from pseudobrain_b200 import exact_memory as M
    rng = np.random.default_rng(n_blk)
    kmax = oq.bf16_round(rng.standard_normal((kv, n_blk, 128)).astype(np.float32) * 3)
    kmin = oq.bf16_round(kmax - np.abs(rng.standard_normal((kv, n_blk, 128))).astype(np.float32))
    smax_ref, smin_ref = oq.super_bounds(kmax, kmin, sblk)
    dmax = torch.from_numpy(kmax).to(cuda_device, torch.bfloat16)
    dmin = torch.from_numpy(kmin).to(cuda_device, torch.bfloat16)
    n_sb = (n_blk + sblk - 1) // sblk
    smax = torch.full((kv, n_sb, 128), 7.0, dtype=torch.bfloat16, device=cuda_device)
    smin = torch.full_like(smax, 7.0)
    M.super_bounds_(dmax, dmin, n_blk, sblk, smax, smin, first_sb=first)
    assert np.array_equal(_bits(smax)[:, first:], oq.bf16_bits(smax_ref)[:, first:])
    assert np.array_equal(_bits(smin)[:, first:], oq.bf16_bits(smin_ref)[:, first:])
    assert np.all(smax[:, :first].float().cpu().numpy() == 7.0)  # super-blocks before first untouched


@pytest.mark.parametrize("kv,groups,full,extra,page,sblk,nq,t,budget,hole", [
    (2, 4, 1000, 7, 16, 8, 3, 1, 64, (0, 0)),
    (2, 4, 1000, 0, 16, 8, 2, 3, 64, (200, 420)),
    (8, 4, 4000, 3, 16, 64, 2, 1, 256, (0, 0)),
    (4, 2, 333, 1, 64, 4, 1, 5, 40, (10, 30)),
    (1, 8, 130, 0, 16, 8, 1, 2, 300, (0, 0))])
def test_two_level_selection_matches_oracle(cuda_device, kv, groups, full, extra, page, sblk, nq, t, budget, hole):
    from pseudobrain_b200 import exact_memory as M
    rng = np.random.default_rng(full + nq)
    n_arch = full * page + extra
    keys = oq.bf16_round(rng.standard_normal((kv, n_arch, 128)).astype(np.float32))
    q = oq.bf16_round(rng.standard_normal((nq, t, kv * groups, 128)).astype(np.float32))
    kmax, kmin = oq.page_bounds(keys[None], page)
    smax, smin = oq.super_bounds(kmax, kmin, sblk)
    dev = cuda_device
    n_valid = full - (hole[1] - hole[0])
    kb = min(budget, n_valid)
    pages = M.select_pages_levels(torch.from_numpy(q).to(dev, torch.bfloat16),
                                  torch.from_numpy(kmax[0]).to(dev, torch.bfloat16),
                                  torch.from_numpy(kmin[0]).to(dev, torch.bfloat16), n_arch, page, kb,
                                  torch.from_numpy(smax[0]).to(dev, torch.bfloat16),
                                  torch.from_numpy(smin[0]).to(dev, torch.bfloat16), sblk, hole).cpu().numpy()
    for n in range(nq):
        qg = q[n].reshape(t, kv, groups, 128).transpose(1, 2, 0, 3).reshape(kv, groups * t, 128)
        ref = oq.select_two_level(qg, kmax[0], kmin[0], smax[0], smin[0], full, min(kb, full), sblk, hole,
                                  canonical=True)
        assert pages[n].shape == ref.shape
        assert np.array_equal(pages[n], ref), f"group {n}"
    from pseudobrain_b200._capi import device_error
    assert device_error() == 0


@pytest.mark.parametrize("hole", [(0, 0), (5, 140), (0, 299)])
def test_flat_selection_with_hole_matches_oracle(cuda_device, hole):
    from pseudobrain_b200 import exact_memory as M
    rng = np.random.default_rng(hole[1])
    kv, groups, page, full, nq, t = 2, 4, 16, 300, 2, 2
    n_arch = full * page
    keys = oq.bf16_round(rng.standard_normal((kv, n_arch, 128)).astype(np.float32))
    q = oq.bf16_round(rng.standard_normal((nq, t, kv * groups, 128)).astype(np.float32))
    kmax, kmin = oq.page_bounds(keys[None], page)
    kb = min(50, full - (hole[1] - hole[0]))
    pages = M.select_pages_levels(torch.from_numpy(q).to(cuda_device, torch.bfloat16),
                                  torch.from_numpy(kmax[0]).to(cuda_device, torch.bfloat16),
                                  torch.from_numpy(kmin[0]).to(cuda_device, torch.bfloat16), n_arch, page, kb,
                                  hole=hole).cpu().numpy()
    for n in range(nq):
        qg = q[n].reshape(t, kv, groups, 128).transpose(1, 2, 0, 3).reshape(kv, groups * t, 128)
        sc = oq.canonical_bound_scores(qg, kmax[0], kmin[0])
        sc[:, hole[0]:hole[1]] = -np.inf
        assert np.array_equal(pages[n], oq._topk_lowest(sc, kb)), f"group {n}"
        assert not np.any((pages[n] >= hole[0]) & (pages[n] < hole[1]))


LEVEL_CASES = {"sb_t1": {}, "sb_t3": {}, "rerank_t1": {"decode_rerank": 24}, "sb_nb_t1": {"neighbors": 1},
               "prompt_t80": {}, "sb_after_prompt_t1": {}}


def test_golden_retrieve_modes(cuda_device, quest_cfg):
    """retrieve (two-level, rerank, neighbours, kept prompt selection) against the
    reference's own retrieve on the same archive (tests/golden/quest_levels.npz), and
    archive_append's super-block bounds bit-exact."""
    M = quest_cfg
    f = load_golden("quest_levels.npz")
    page, budget, groups, sblk = (int(f[x]) for x in ("page", "budget", "groups", "sblk"))
    base = dict(enabled=True, block_size=page, blocks=budget, decode_blocks=budget, superblock=sblk, rerank=0,
                decode_rerank=0, neighbors=0, keys_like_values=False)
    M.EXACT_MEMORY.update(base)
    keys, values = _bf16(f["keys"], cuda_device), _bf16(f["values"], cuda_device)
    arc = M.archive_append(None, keys[:, :, :700].contiguous(), values[:, :, :700].contiguous())
    arc = M.archive_append(arc, keys[:, :, 700:].contiguous(), values[:, :, 700:].contiguous())
    for name in ("kmax", "kmin", "smax", "smin"):
        assert np.array_equal(_bits(getattr(arc, name)), f[name]), name
    n_arch = keys.shape[2]
    pages = arc.keys[0, :, : (n_arch // page) * page].reshape(keys.shape[1], n_arch // page, page * 128)
    for case, extra in LEVEL_CASES.items():
        M.EXACT_MEMORY.update(base)
        M.EXACT_MEMORY.update(extra)
        if case != "sb_after_prompt_t1":
            arc.prompt_top = None
        rk, rv = M.retrieve(arc, _bf16(f[f"{case}_q"], cuda_device), groups)
        top = f[f"{case}_top"][0]
        sel = top.shape[-1]
        assert rk.shape[2] == sel * page + n_arch % page, case
        want = torch.stack([pages[h, torch.from_numpy(top[h]).to(cuda_device)] for h in range(top.shape[0])])
        assert torch.equal(rk[0, :, : sel * page].reshape(top.shape[0], sel, page * 128), want), case


def test_golden_retrieve_attend_two_level(cuda_device, quest_cfg):
    """retrieve_attend in the two-level mode equals SDPA over [retrieve ; window] (oracle)."""
    M = quest_cfg
    f = load_golden("quest_levels.npz")
    page, budget, groups, sblk = (int(f[x]) for x in ("page", "budget", "groups", "sblk"))
    M.EXACT_MEMORY.update(enabled=True, block_size=page, blocks=budget, decode_blocks=budget, superblock=sblk,
                          rerank=0, decode_rerank=0, neighbors=0, keys_like_values=False)
    keys_all, values_all = oq.bf16_from_bits(f["keys"]), oq.bf16_from_bits(f["values"])
    n_arch = keys_all.shape[2] - 37  # the last 37 keys are the window
    keys, values = _bf16(f["keys"], cuda_device), _bf16(f["values"], cuda_device)
    arc = M.archive_append(None, keys[:, :, :n_arch].contiguous(), values[:, :, :n_arch].contiguous())
    q = _bf16(f["sb_t3_q"], cuda_device)
    qpos = torch.arange(n_arch + 37 - 3, n_arch + 37, device=cuda_device)
    kpos = torch.arange(n_arch, n_arch + 37, device=cuda_device)
    out = M.retrieve_attend(arc, q, groups, keys[:, :, n_arch:], values[:, :, n_arch:], qpos, kpos, 30)
    kmax, kmin = oq.page_bounds(keys_all[:, :, :n_arch], page)
    rk, rv, _ = oq.retrieve_modes(keys_all[:, :, :n_arch], values_all[:, :, :n_arch], kmax, kmin,
                                  oq.bf16_from_bits(f["sb_t3_q"]), groups, page, budget, superblock=sblk)
    ref = oq.attend(oq.bf16_from_bits(f["sb_t3_q"]), rk, rv, keys_all[:, :, n_arch:], values_all[:, :, n_arch:],
                    qpos.cpu().numpy(), kpos.cpu().numpy(), 30, 0, groups)
    from oracle.gdn import rel_err
    assert rel_err(out.cpu().numpy(), ref) < 5e-3


@pytest.mark.parametrize("case", ["s_sb", "s_sb_hole", "s_sb_nb", "s_flat_hole", "s_rerank_hole"])
def test_golden_serving_levels(cuda_device, serving_cfg, case):
    """The serving retrieve_blocks' super-block, hole, neighbour and rerank-with-hole paths
    against pb27_vllm/memory.py (tests/golden/quest_levels.npz); the block and super-block
    bounds are refreshed by this package's kernels, bit-exact."""
    S = serving_cfg
    f = load_golden("quest_levels.npz")
    page, sblk, groups = int(f["page"]), int(f["sblk"]), int(f["groups"])
    S.SBLK = sblk
    S.MEMORY.update(blocks=8, decode_blocks=8, rerank=int(f[f"{case}_pool"]), block_size=page, window=64,
                    neighbors=int(f[f"{case}_neighbors"]))
    keys = _bf16(f["s_keys"], cuda_device)
    kv, cap, d = keys.shape
    n_blk = cap // page
    n_sb = (n_blk + sblk - 1) // sblk
    use_sb = not int(f[f"{case}_nosb"])
    hole = tuple(int(x) for x in f[f"{case}_hole"])
    arc = types.SimpleNamespace(
        keys=keys, values=keys, kmax=torch.zeros(kv, n_blk, d, dtype=torch.bfloat16, device=cuda_device),
        kmin=torch.zeros(kv, n_blk, d, dtype=torch.bfloat16, device=cuda_device),
        smax=torch.zeros(kv, n_sb, d, dtype=torch.bfloat16, device=cuda_device) if use_sb else None,
        smin=torch.zeros(kv, n_sb, d, dtype=torch.bfloat16, device=cuda_device) if use_sb else None,
        size=cap, prompt_len=cap, hole_lo=hole[0], hole_hi=hole[1], dirty_lo=0, dirty_hi=n_blk - 1)
    q = _bf16(f[f"{case}_q"], cuda_device)
    top = S.retrieve_blocks(arc, q, groups, int(f["s_limit"]), bool(f[f"{case}_rerank"]))
    assert np.array_equal(_bits(arc.kmax), f["s_kmax"]) and np.array_equal(_bits(arc.kmin), f["s_kmin"])
    if use_sb:
        assert np.array_equal(_bits(arc.smax), f["s_smax"]) and np.array_equal(_bits(arc.smin), f["s_smin"])
    assert np.array_equal(top.cpu().numpy(), f[f"{case}_top"])


@pytest.mark.parametrize("t,hole,nb", [(1, (0, 0), 0), (4, (4 + 64 * 100, 4 + 64 * 260), 0), (2, (0, 0), 2)])
def test_serving_two_level_matches_oracle(cuda_device, serving_cfg, t, hole, nb):
    """A 2048-block serving archive in 64-token blocks with the reference's super-blocks of 64
    blocks (more than 16 of them: the two-level path), against oracle/serving.py."""
    S = serving_cfg
    S.SBLK = 64
    S.MEMORY.update(blocks=48, decode_blocks=48, rerank=0, block_size=64, window=512, neighbors=nb)
    rng = np.random.default_rng(t * 7 + nb)
    kv, groups, d, block = 2, 4, 128, 64
    n_blk = 2048
    cap = S.ORIGIN + n_blk * block
    keys = oq.bf16_round(rng.standard_normal((kv, cap, d)).astype(np.float32))
    q = oq.bf16_round(rng.standard_normal((t, kv * groups, d)).astype(np.float32))
    dk = torch.from_numpy(keys).to(cuda_device, torch.bfloat16)
    n_sb = (n_blk + 63) // 64
    arc = types.SimpleNamespace(
        keys=dk, values=dk, kmax=torch.zeros(kv, n_blk, d, dtype=torch.bfloat16, device=cuda_device),
        kmin=torch.zeros(kv, n_blk, d, dtype=torch.bfloat16, device=cuda_device),
        smax=torch.zeros(kv, n_sb, d, dtype=torch.bfloat16, device=cuda_device),
        smin=torch.zeros(kv, n_sb, d, dtype=torch.bfloat16, device=cuda_device),
        size=cap, prompt_len=cap, hole_lo=hole[0], hole_hi=hole[1], dirty_lo=0, dirty_hi=n_blk - 1)
    limit = cap - 700
    top = S.retrieve_blocks(arc, torch.from_numpy(q).to(cuda_device, torch.bfloat16), groups, limit, False)
    kmax = oq.bf16_from_bits(_bits(arc.kmax))
    kmin = oq.bf16_from_bits(_bits(arc.kmin))
    smax_ref, smin_ref = osv.super_bounds(kmax, kmin, n_blk, 64)
    assert np.array_equal(_bits(arc.smax), oq.bf16_bits(smax_ref))
    mem = dict(S.MEMORY)
    ref = osv.retrieve_blocks(keys, kmax, kmin, q, groups, limit, False, mem, cap, smax_ref, smin_ref, 64, hole,
                              canonical=True)
    got = top.cpu().numpy()
    assert got.shape == ref.shape
    assert np.array_equal(got, ref)
