"""Head dim 256 (PB-27's attention layers: 24 query / 4 key heads at 256) on the SIMT paths of
the Quest, serving and archive kernels.

* Against the reference (tests/golden/serving256.npz): the archive written from empty
  through archive_write has the reference's block and super-block bounds bit for bit and
  its means within bf16 rounding; retrieve_blocks returns the reference's blocks in the
  flat, super-block, rerank, holed-rerank and past-the-RoPE-horizon rerank paths; and
  piece_attention matches within 5e-3.
* Against the oracle (oracle/quest.py, head-dim generic): page bounds and the gathered
  pages bit-exact, page sets equal to the canonical-order selection (the SIMT score kernel
  sums the dims in order, so no refinement is involved), attention within 5e-3."""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from oracle import quest as oq
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu
TOL = 5e-3


@pytest.fixture
def serving_cfg():
    from pseudobrain_b200 import serving as S
    saved = (dict(S.MEMORY), S.SBLK, S.ROPE_HORIZON)
    yield S
    S.MEMORY.clear()
    S.MEMORY.update(saved[0])
    S.SBLK, S.ROPE_HORIZON = saved[1], saved[2]


def _bf(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def _u16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def test_serving_twins_match_reference(cuda_device, serving_cfg):
    S = serving_cfg
    f = load_golden("serving256.npz")
    dev = cuda_device
    block, groups, window, cap = (int(f[x]) for x in ("block", "groups", "window", "cap"))
    S.SBLK = int(f["sblk"])
    S.MEMORY.update(blocks=6, decode_blocks=6, rerank=12, block_size=block, neighbors=0, window=window)
    keys, values = _bf(f["keys"], dev), _bf(f["values"], dev)
    kv, _, d = keys.shape
    assert d == 256
    n_blk = cap // block
    n_sb = (n_blk + S.SBLK - 1) // S.SBLK
    z = lambda rows: torch.zeros(kv, rows, d, dtype=torch.bfloat16, device=dev)  # noqa: E731
    arc = types.SimpleNamespace(keys=z(cap), values=z(cap), kmax=z(n_blk), kmin=z(n_blk), bmean_k=z(n_blk),
                                bmean_v=z(n_blk), smax=z(n_sb), smin=z(n_sb), smean_k=z(n_sb), smean_v=z(n_sb),
                                size=0, dirty_lo=1 << 60, dirty_hi=-1, prompt_len=0, hole_lo=0, hole_hi=0)
    pos = torch.arange(cap, device=dev)
    for a, b in ((0, 700), (700, 1301), (1301, cap)):  # three writes across block and super-block edges
        S.archive_write(arc, pos[a:b], keys[:, a:b].transpose(0, 1).contiguous(),
                        values[:, a:b].transpose(0, 1).contiguous(), block)
    S._refresh(arc, block)
    arc.prompt_len = cap
    nb = (cap - S.ORIGIN + block - 1) // block
    full_blocks = (cap - S.ORIGIN) // block
    for name in ("kmax", "kmin"):
        assert np.array_equal(_u16(getattr(arc, name))[:, :full_blocks], f[name][:, :full_blocks]), name
    nsb_full = full_blocks // S.SBLK
    for name in ("smax", "smin"):
        assert np.array_equal(_u16(getattr(arc, name))[:, :nsb_full], f[name][:, :nsb_full]), name
    for name in ("bmean_k", "bmean_v"):
        assert np.allclose(getattr(arc, name)[:, :nb].float().cpu().numpy(), f[name][:, :nb], rtol=2 ** -8,
                           atol=1e-6), name
    for name in ("smean_k", "smean_v"):
        assert np.allclose(getattr(arc, name)[:, :nsb_full].float().cpu().numpy(), f[name][:, :nsb_full],
                           rtol=2e-2, atol=2e-3), name
    for case in f["cases"]:
        S.ROPE_HORIZON = int(f[f"{case}_horizon"]) or 262144
        arc.hole_lo, arc.hole_hi = (int(x) for x in f[f"{case}_hole"])
        saved = (arc.smax, arc.smin)
        if not int(f[f"{case}_sb"]):
            arc.smax = arc.smin = None
        q = _bf(f[f"{case}_q"], dev)
        limit = int(f[f"{case}_limit"])
        top = S.retrieve_blocks(arc, q, groups, limit, bool(f[f"{case}_rerank"]))
        arc.smax, arc.smin = saved
        want = f[f"{case}_top"]
        print(f"[hd256 serving] {case}: blocks equal {np.array_equal(top.cpu().numpy(), want)}")
        assert np.array_equal(top.cpu().numpy(), want), case
        t = q.shape[0]
        q_pos = torch.arange(cap - t, cap, device=dev)
        out = S.piece_attention(arc, q.float(), q_pos, top, groups, window, d ** -0.5)
        err = ogdn.rel_err(out.cpu().numpy(), f[f"{case}_out"])
        print(f"[hd256 serving] {case}: attention rel err {err:.2e}")
        assert err < TOL, case
    from pseudobrain_b200._capi import device_error
    assert device_error() == 0


@pytest.mark.parametrize("nq,t,page,budget", [(3, 1, 16, 20), (2, 2, 64, 7)])
def test_quest_core_matches_oracle(cuda_device, nq, t, page, budget):
    from pseudobrain_b200 import exact_memory as M
    rng = np.random.default_rng(41 + t)
    kv, heads, d, n_win = 4, 24, 256, 300
    n_arch = page * 120 + 5
    keys = oq.bf16_round(rng.standard_normal((kv, n_arch + n_win, d), dtype=np.float32))
    values = oq.bf16_round(rng.standard_normal((kv, n_arch + n_win, d), dtype=np.float32))
    q = oq.bf16_round(rng.standard_normal((nq, t, heads, d), dtype=np.float32))
    groups, full = heads // kv, n_arch // page
    dk = torch.from_numpy(keys).to(cuda_device, torch.bfloat16)
    dvv = torch.from_numpy(values).to(cuda_device, torch.bfloat16)
    dq = torch.from_numpy(q).to(cuda_device, torch.bfloat16)
    kmax = torch.empty(kv, full, d, dtype=torch.bfloat16, device=cuda_device)
    kmin = torch.empty_like(kmax)
    M.page_bounds_(dk[:, : full * page], page, kmax, kmin)
    bmax, bmin = oq.page_bounds(keys[None, :, : full * page], page)
    assert np.array_equal(kmax.float().cpu().numpy(), bmax[0]) and np.array_equal(kmin.float().cpu().numpy(), bmin[0])
    pages = M.select_pages(dq, kmax, kmin, n_arch, page, budget)
    s = oq.canonical_page_scores(np.ascontiguousarray(q.transpose(0, 2, 1, 3)), bmax, bmin, groups)
    assert np.array_equal(pages.cpu().numpy(), oq.select_pages(s, budget))
    qpos = (np.full((nq, t), n_arch + n_win - 1) - np.arange(t)[::-1][None]).astype(np.int32)
    kpos = np.arange(n_arch, n_arch + n_win, dtype=np.int32)
    window = 200
    out = M.attend_pages(dq, torch.from_numpy(qpos).to(cuda_device), dk, dvv, n_arch, page, pages,
                         dk[:, n_arch:], dvv[:, n_arch:], torch.from_numpy(kpos).to(cuda_device), window)
    for i in range(nq):
        arc = oq.Archive(keys[None, :, :n_arch], values[None, :, :n_arch], bmax, bmin)
        rk, rv, _ = oq.retrieve(arc, q[i].transpose(1, 0, 2)[None], groups, page, budget)
        ref = oq.attend(q[i].transpose(1, 0, 2)[None], rk, rv, keys[None, :, n_arch:], values[None, :, n_arch:],
                        qpos[i], kpos, window, 0, groups)[0].transpose(1, 0, 2)
        err = ogdn.rel_err(out[i].cpu().numpy(), ref)
        assert err < TOL, err
        gk, gv = M.gather_pages(dk, dvv, n_arch, page, pages[i:i + 1].contiguous(), dq[i:i + 1])
        assert np.array_equal(gk[0].float().cpu().numpy(), rk[0])
        assert np.array_equal(gv[0].float().cpu().numpy(), rv[0])
