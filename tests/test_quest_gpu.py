"""GPU parity of the Quest kernels (bounds, select, gather, attend) against the oracle and
the reference's golden outputs.

Page bounds, page indices and gathered keys must be bit-exact. Scores: both sides sum
exact bf16 x bf16 products in fp32 (orders differ), so selections agree exactly on
these seeded inputs; every test also checks that the selection boundary is not a
near-tie. Attention output: bf16 tensor-core products with fp32 accumulation and the
probabilities rounded to bf16 for the P V product (as flash attention does), ATT_TOL = 5e-3
relative (the bar for bf16 inputs is 2e-2)
(fp32 output) or 1e-2 (bf16 output rounding).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from oracle import quest as oq
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu
ATT_TOL = 5e-3


def _bf16(x, dev):
    return torch.from_numpy(oq.bf16_from_bits(x)).to(dev, torch.bfloat16)


@pytest.fixture
def quest_cfg():
    from pseudobrain_b200 import exact_memory as M
    saved = dict(M.EXACT_MEMORY)
    yield M
    M.EXACT_MEMORY.clear()
    M.EXACT_MEMORY.update(saved)


def test_golden_archive_retrieve_and_attention(cuda_device, quest_cfg):
    M = quest_cfg
    f = load_golden("quest.npz")
    page, budget, groups, window = (int(f[x]) for x in ("page", "budget", "groups", "window"))
    n_arch = int(f["n_arch"])
    M.EXACT_MEMORY.update(enabled=True, block_size=page, blocks=budget, decode_blocks=budget, superblock=0,
                          rerank=0, decode_rerank=0, neighbors=0)
    keys, values = _bf16(f["keys"], cuda_device), _bf16(f["values"], cuda_device)
    arc = M.archive_append(None, keys[:, :, :100].contiguous(), values[:, :, :100].contiguous())
    arc = M.archive_append(arc, keys[:, :, 100:n_arch].contiguous(), values[:, :, 100:n_arch].contiguous())
    assert np.array_equal(oq.bf16_bits(arc.kmax.float().cpu().numpy()), f["kmax"])
    assert np.array_equal(oq.bf16_bits(arc.kmin.float().cpu().numpy()), f["kmin"])
    wk, wv = keys[:, :, n_arch:], values[:, :, n_arch:]
    for case in ("t1", "t3"):
        q = _bf16(f[f"{case}_q"], cuda_device)
        arc.prompt_top = None
        rk, rv = M.retrieve(arc, q, groups)
        assert np.array_equal(oq.bf16_bits(rk.float().cpu().numpy()), f[f"{case}_rk"])
        assert np.array_equal(oq.bf16_bits(rv.float().cpu().numpy()), f[f"{case}_rv"])
        qpos = torch.from_numpy(f[f"{case}_qpos"]).to(cuda_device)
        kpos = torch.from_numpy(f["kpos"]).to(cuda_device)
        out = M.retrieve_attend(arc, q, groups, wk, wv, qpos, kpos, window)
        assert ogdn.rel_err(out.cpu().numpy(), f[f"{case}_out"]) < ATT_TOL


def _random_problem(seed, kv, heads, n_arch, n_win, page, nq, t, dev, plant=True):
    rng = np.random.default_rng(seed)
    keys = oq.bf16_round(rng.standard_normal((kv, n_arch + n_win, 128), dtype=np.float32))
    values = oq.bf16_round(rng.standard_normal((kv, n_arch + n_win, 128), dtype=np.float32))
    q = oq.bf16_round(rng.standard_normal((nq, t, heads, 128), dtype=np.float32))
    planted = rng.choice(n_arch // page, size=nq, replace=False) if plant else []
    groups = heads // kv
    for i, p in enumerate(planted):
        qhat = q[i].reshape(t, kv, groups, 128).mean(axis=(0, 2))
        qhat /= np.linalg.norm(qhat, axis=-1, keepdims=True)
        keys[:, p * page:(p + 1) * page] = oq.bf16_round(45.0 * t * qhat)[:, None]
    return keys, values, q, np.asarray(planted)


def _oracle_select(q, keys, n_arch, page, budget, groups):
    """Per group: page scores and top pages from the oracle (q [nq,t,h,d] -> [B=1,H,T,D])."""
    full = n_arch // page
    kmax, kmin = oq.page_bounds(keys[None, :, : full * page], page)
    tops, scores = [], []
    for i in range(q.shape[0]):
        s = oq.page_scores(q[i].transpose(1, 0, 2)[None], kmax, kmin, groups)[0]
        scores.append(s)
        tops.append(oq.select_pages(s, budget))
    return np.stack(tops), np.stack(scores)


def _assert_same_selection(pages, top_ref, scores_ref, budget):
    """Selected page sets equal the oracle's. A row may differ only where the oracle's own
    scores put the differing pages within fp32 summation noise (1e-5 relative) of the
    selection boundary: both sides sum the same exact products in different orders."""
    pages = np.asarray(pages)
    scores_ref = scores_ref.reshape(-1, scores_ref.shape[-1]).astype(np.float64)
    got, ref = pages.reshape(-1, pages.shape[-1]), top_ref.reshape(-1, top_ref.shape[-1])
    for row in range(got.shape[0]):
        if np.array_equal(got[row], ref[row]):
            continue
        s = scores_ref[row]
        kth = -np.sort(-s)[min(budget, s.size) - 1]
        diff = np.setxor1d(got[row], ref[row])
        assert np.all(np.abs(s[diff] - kth) <= 1e-5 * abs(kth)), f"row {row}: selection differs beyond a near-tie"


@pytest.mark.parametrize("kv,heads,n_arch,page,nq,t,budget", [
    (2, 8, 16 * 300 + 5, 16, 3, 1, 20), (8, 32, 16 * 4000, 16, 8, 1, 256), (4, 16, 64 * 100 + 63, 64, 2, 5, 7),
    (1, 1, 16 * 10, 16, 1, 1, 64)])
def test_select_and_attend_match_oracle(cuda_device, kv, heads, n_arch, page, nq, t, budget):
    from pseudobrain_b200 import exact_memory as M
    n_win = 300
    keys, values, q, planted = _random_problem(kv * 7 + nq, kv, heads, n_arch, n_win, page, nq, t, cuda_device)
    groups = heads // kv
    full = n_arch // page
    top_ref, scores_ref = _oracle_select(q, keys, n_arch, page, budget, groups)
    dk = torch.from_numpy(keys).to(cuda_device, torch.bfloat16)
    dvv = torch.from_numpy(values).to(cuda_device, torch.bfloat16)
    dq = torch.from_numpy(q).to(cuda_device, torch.bfloat16)
    kmax = torch.empty(kv, full, 128, dtype=torch.bfloat16, device=cuda_device)
    kmin = torch.empty_like(kmax)
    M.page_bounds_(dk[:, : full * page], page, kmax, kmin)
    scores = torch.empty(nq, kv, full, device=cuda_device)
    pages = M.select_pages(dq, kmax, kmin, n_arch, page, budget, scores=scores)
    _assert_same_selection(pages.cpu().numpy(), top_ref, scores_ref, budget)
    np.testing.assert_allclose(scores.cpu().numpy(), scores_ref, rtol=2e-6, atol=1e-4)
    for i, p in enumerate(planted):
        assert np.all((pages[i] == int(p)).any(-1).cpu().numpy())
    from pseudobrain_b200._capi import device_error
    assert device_error() == 0  # no bounded device-side wait gave up
    # attention over [pages ; tail ; window]
    qpos = (np.full((nq, t), n_arch + n_win - 1) - np.arange(t)[::-1][None]).astype(np.int32)
    kpos = np.arange(n_arch, n_arch + n_win, dtype=np.int32)
    window = 200
    out = M.attend_pages(dq, torch.from_numpy(qpos).to(cuda_device), dk, dvv, n_arch, page, pages,
                         dk[:, n_arch:], dvv[:, n_arch:], torch.from_numpy(kpos).to(cuda_device), window)
    for i in range(nq):
        arc = oq.Archive(keys[None, :, :n_arch], values[None, :, :n_arch], *oq.page_bounds(keys[None, :, :n_arch], page))
        rk, rv, top = oq.retrieve(arc, q[i].transpose(1, 0, 2)[None], groups, page, budget)
        ref = oq.attend(q[i].transpose(1, 0, 2)[None], rk, rv, keys[None, :, n_arch:], values[None, :, n_arch:],
                        qpos[i], kpos, window, 0, groups)[0].transpose(1, 0, 2)
        assert ogdn.rel_err(out[i].cpu().numpy(), ref) < ATT_TOL
        # and the gather (retrieve's return value) is bit-exact
        gk, gv = M.gather_pages(dk, dvv, n_arch, page, pages[i:i + 1].contiguous(), dq[i:i + 1])
        assert np.array_equal(gk[0].float().cpu().numpy(), rk[0])
        assert np.array_equal(gv[0].float().cpu().numpy(), rv[0])


def test_ties_go_to_lowest_page(cuda_device):
    """Pages with identical bounds score identically: the lowest indices win, like the
    oracle's stable rule."""
    from pseudobrain_b200 import exact_memory as M
    rng = np.random.default_rng(5)
    kv, page, npages = 2, 16, 3000
    # Small integers: every product and partial sum is exact in fp32, so equal pages
    # score bit-identically in any summation order (kernel and oracle alike).
    base = rng.integers(0, 4, size=(kv, 50, 128)).astype(np.float32)
    pick = rng.integers(0, 50, size=npages)
    kmax_np = base[:, pick]
    kmin_np = kmax_np - rng.integers(0, 3, size=(kv, 1, 128)).astype(np.float32)
    q = rng.integers(-2, 3, size=(2, 1, 8, 128)).astype(np.float32)
    kmax = torch.from_numpy(kmax_np).to(cuda_device, torch.bfloat16)
    kmin = torch.from_numpy(kmin_np).to(cuda_device, torch.bfloat16)
    for budget in (1, 7, 100, 2999, 3000, 5000):
        pages = M.select_pages(torch.from_numpy(q).to(cuda_device, torch.bfloat16), kmax, kmin, npages * page, page,
                               budget)
        for i in range(2):
            s = oq.page_scores(q[i].transpose(1, 0, 2)[None], kmax_np[None], kmin_np[None], 4)[0]
            assert np.array_equal(pages[i].cpu().numpy(), oq.select_pages(s, budget))


def test_config3_full_size(cuda_device):
    """benchmark config 3: 1M-token cache, 8 queries, 32/8 heads, page 16, 256-page budget,
    4096 window. Exact page sets vs the oracle's scores on the same bounds, planted pages
    present, and attention within tolerance for two of the queries."""
    from pseudobrain_b200 import exact_memory as M
    from pseudobrain_b200.synthetic import quest_inputs
    x = quest_inputs(device=cuda_device)
    scores = torch.empty(8, 8, x["kmax"].shape[1], device=cuda_device)
    pages = M.select_pages(x["q"], x["kmax"], x["kmin"], x["n_arch"], x["page"], x["budget"], scores=scores)
    kmax = x["kmax"].float().cpu().numpy()[None]
    kmin = x["kmin"].float().cpu().numpy()[None]
    q = x["q"].float().cpu().numpy()
    for i in range(8):
        s = oq.page_scores(q[i].transpose(1, 0, 2)[None], kmax, kmin, 4)[0]
        _assert_same_selection(pages[i].cpu().numpy(), oq.select_pages(s, x["budget"]), s, x["budget"])
        assert bool((pages[i] == int(x["planted"][i])).any(-1).all())
    out = M.attend_pages(x["q"], x["qpos"], x["keys"], x["values"], x["n_arch"], x["page"], pages, x["win_keys"],
                         x["win_values"], x["kpos"], x["window"])
    for i in (0, 5):
        idx = (pages[i].long()[..., None] * 16 + torch.arange(16, device=cuda_device)).view(8, -1)
        rk = torch.gather(x["keys"], 1, idx[..., None].expand(-1, -1, 128)).float().cpu().numpy()[None]
        rv = torch.gather(x["values"], 1, idx[..., None].expand(-1, -1, 128)).float().cpu().numpy()[None]
        ref = oq.attend(q[i].transpose(1, 0, 2)[None], rk, rv, x["win_keys"].float().cpu().numpy()[None],
                        x["win_values"].float().cpu().numpy()[None], x["qpos"][i].cpu().numpy(),
                        x["kpos"].cpu().numpy(), x["window"], 0, 4)[0].transpose(1, 0, 2)
        assert ogdn.rel_err(out[i].cpu().numpy(), ref) < ATT_TOL


def test_quest_rejects_bad_arguments(cuda_device):
    from pseudobrain_b200 import exact_memory as M
    from pseudobrain_b200._capi import PbkError
    q = torch.zeros(1, 1, 8, 128, dtype=torch.bfloat16, device=cuda_device)
    kmax = torch.zeros(3, 10, 128, dtype=torch.bfloat16, device=cuda_device)  # 8 heads over 3 key heads
    with pytest.raises(PbkError):
        M.select_pages(q, kmax, kmax, 160, 16, 4)
    with pytest.raises(ValueError):
        M.page_bounds_(torch.zeros(2, 100, 128, dtype=torch.bfloat16, device=cuda_device), 16, kmax[:2, :5],
                       kmax[:2, :5])
    with pytest.raises(RuntimeError):
        M.select_pages(q.cpu(), kmax, kmax, 160, 16, 4)


def test_select_attend_pages_equals_select_then_attend(cuda_device):
    """select_attend_pages (window attention on a side stream beside the top-k) gives exactly
    select_pages + attend_pages (the same kernels over the same workspace layout), eagerly and
    replayed from a CUDA graph."""
    from pseudobrain_b200 import exact_memory as M
    from pseudobrain_b200.synthetic import quest_inputs
    xq = quest_inputs(device=cuda_device, seed=17, n_tokens=1 << 16, kv=4, heads=16, d=128, page=16, window=512,
                      nq=4, budget_tokens=1024)
    args = (xq["q"], xq["qpos"], xq["keys"], xq["values"], xq["kmax"], xq["kmin"], xq["n_arch"], xq["page"],
            xq["budget"], xq["win_keys"], xq["win_values"], xq["kpos"], xq["window"])
    pages = M.select_pages(xq["q"], xq["kmax"], xq["kmin"], xq["n_arch"], xq["page"], xq["budget"])
    out = M.attend_pages(xq["q"], xq["qpos"], xq["keys"], xq["values"], xq["n_arch"], xq["page"], pages,
                         xq["win_keys"], xq["win_values"], xq["kpos"], xq["window"])
    p2, o2 = M.select_attend_pages(*args)
    assert torch.equal(p2, pages) and torch.equal(o2, out)
    holder = {}

    def step():
        holder["r"] = M.select_attend_pages(*args)

    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(holder["r"][0], pages) and torch.equal(holder["r"][1], out)
