"""Host-side pieces of the per-token selector (pseudobrain_b200.pertoken) on the CPU: the
priority dedup, successor expansion, z-scores, stratified peaks and the global-aggregation
test against the reference's own helpers (pb27_vllm/memory.py:888-992) where the reference
is importable, and the committed fixture's consistency."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

from tests.conftest import ROOT

REFERENCE = "/root/reference"
FIX = os.path.join(ROOT, "tests", "golden", "pertoken.npz")


@pytest.fixture(scope="module")
def mem():
    if not os.path.isdir(os.path.join(REFERENCE, "serving", "pb27_vllm")):
        pytest.skip("reference not present")
    sys.path.insert(0, os.path.join(REFERENCE, "serving", "pb27_vllm"))
    os.environ.setdefault("PB27_MEMORY_OFFLOAD", "")
    try:
        import pb27_vllm.memory as m
    finally:
        sys.path.pop(0)
    return m


def test_dedup_and_successors_match_reference(mem):
    from pseudobrain_b200 import pertoken
    g = torch.Generator().manual_seed(3)
    for m, hi, u in ((12, 5, 4), (40, 30, 40), (64, 100, 17), (9, 3, 9)):
        seq = torch.randint(0, hi, (3, m), generator=g)
        assert torch.equal(pertoken.dedup_priority(seq, u), mem._dedup_priority(seq, u))
        for ms in (1, 5, m):
            a = pertoken.expand_successors_dedup(seq, hi, u, m_succ=ms)
            b = mem._expand_successors_dedup(seq, hi, u, m_succ=ms)
            assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_zscores_peaks_and_global_test_match_reference(mem):
    from pseudobrain_b200 import pertoken, serving
    g = torch.Generator().manual_seed(4)
    score = torch.randn(2, 5, 300, generator=g)
    score[:, :, 40:60] = float("-inf")
    z_rel, z_raw = pertoken.zscores(score)
    s_fin = score.masked_fill(score.isinf(), 0.0)
    s_rel = score - s_fin.mean(1, keepdim=True)
    s_rel_fin = s_rel.masked_fill(score.isinf(), 0.0)
    want_rel = (s_rel - s_rel_fin.mean(-1, keepdim=True)) / s_rel_fin.std(-1, keepdim=True).clamp(min=1e-6)
    assert torch.equal(z_rel, want_rel)
    saved = serving.SBLK
    try:
        serving.SBLK = mem.SBLK = 4
        for max_sb in (1, 8, 100):
            assert torch.equal(pertoken.stratified_peaks(z_raw.amax(1), 300, max_sb),
                               mem._stratified_superblock_peaks(z_raw.amax(1), 300, max_sb))
    finally:
        serving.SBLK, mem.SBLK = saved, 64
    for z in (z_raw, torch.randn(2, 20, 400, generator=g) * 0.3):
        assert pertoken.detect_global_agg(z, z.shape[-1]) == mem._detect_global_agg(z, z.shape[-1])


def test_fixture_steps_are_consistent():
    f = np.load(FIX)
    limit, block, origin = int(f["limit"]), int(f["block"]), int(f["origin"])
    full = (limit - origin) // block
    assert len(f["steps"]) == 7
    for name in f["steps"]:
        top = f[f"{name}_top"]
        assert top.ndim == 2 and top.shape[0] == 2
        assert np.all(np.diff(top, axis=1) >= 0) and top.min() >= 0 and top.max() < full
        lo, hi = (int(x) for x in f[f"{name}_hole"])
        if hi > lo and int(f[f"{name}_lead"]) < 0:  # a prompt piece keeps no block inside the hole
            b0, b1 = max(0, lo - origin) // block, min(full, (hi - origin + block - 1) // block)
            assert not np.any((top >= b0) & (top < b1))


def _stable_reference(mem, monkeypatch):
    """The reference with ties broken by index in its topk and argsort (torch's CPU order
    among equal values is implementation-defined)."""
    orig_sort = torch.Tensor.sort

    def topk(self, k, dim=-1, largest=True, sorted=True):
        idx = orig_sort(self, dim=dim, descending=largest, stable=True).indices.narrow(dim, 0, k)
        return torch.return_types.topk((self.gather(dim, idx), idx))

    def argsort(self, dim=-1, descending=False, stable=False):
        return orig_sort(self, dim=dim, descending=descending, stable=True).indices

    monkeypatch.setattr(torch.Tensor, "topk", topk)
    monkeypatch.setattr(torch.Tensor, "argsort", argsort)


def _cpu_kernels(pertoken, monkeypatch):
    """CPU stand-ins for the three kernels, with the reference's own score arithmetic, so
    that only the selection bookkeeping is compared."""
    def token_scores(q, kmax, kmin, full, n_pool, cand=None, hole=(0, 0), rope_mask=False, kv=None):
        t, h, d = q.shape
        kv = kmax.shape[0] if kv is None else kv
        qg = q.float().permute(1, 0, 2).reshape(kv, h // kv * t, d)
        if rope_mask:
            qg = qg.clone()
            qg[..., : d // 4] = 0
        idx = torch.arange(n_pool).expand(kv, n_pool) if cand is None else cand.long()
        ic = idx.clamp(min=0, max=full - 1)
        bmx = kmax.float().gather(1, ic[..., None].expand(-1, -1, d)).transpose(-1, -2)
        bmn = kmin.float().gather(1, ic[..., None].expand(-1, -1, d)).transpose(-1, -2)
        s = (qg.clamp(min=0) @ bmx + qg.clamp(max=0) @ bmn).view(kv, h // kv, t, n_pool).amax(1)
        bad = (idx >= full) | ((idx >= hole[0]) & (idx < hole[1]))
        return s.masked_fill(bad[:, None, :], float("-inf"))

    def token_rerank(q, keys, block, cand, n_pool, kv=None):
        t, h, d = q.shape
        kv = keys.shape[0] if kv is None else kv
        qg = q.float().permute(1, 0, 2).reshape(kv, h // kv * t, d)
        idx = torch.arange(n_pool).expand(kv, n_pool) if cand is None else cand.long()
        rows = idx[..., None] * block + torch.arange(block)
        ck = keys.float().gather(1, rows.reshape(kv, -1, 1).expand(-1, -1, d))
        return torch.bmm(qg, ck.transpose(-1, -2)).view(kv, h // kv, t, n_pool, block).amax(-1).amax(1)

    def ranks(x):
        order = torch.Tensor.sort(x, dim=-1, descending=True, stable=True).indices
        return torch.empty_like(order).scatter_(-1, order, torch.arange(x.shape[-1]).expand_as(order))

    monkeypatch.setattr(pertoken, "token_scores", token_scores)
    monkeypatch.setattr(pertoken, "token_rerank", token_rerank)
    monkeypatch.setattr(pertoken, "ranks", ranks)
    monkeypatch.setattr(pertoken, "_require_cuda", lambda *a: None)


def test_selection_bookkeeping_matches_reference_with_stable_ties(mem, monkeypatch):
    """Every step of the fixture's sequence (prompt, decode with super-blocks and merges, no
    lead, global aggregation, hole) through both selectors on the CPU with the same scores:
    the selected blocks and the whole selector state after each step are equal when both
    break ties by index."""
    import types
    from pseudobrain_b200 import pertoken, serving
    f = np.load(FIX)
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).float()
    _stable_reference(mem, monkeypatch)
    _cpu_kernels(pertoken, monkeypatch)
    block, groups, limit = int(f["block"]), int(f["groups"]), int(f["limit"])
    cfg = dict(blocks=8, decode_blocks=8, rerank=12, block_size=block, neighbors=0, window=64, chunk=64)
    monkeypatch.setattr(serving, "MEMORY", dict(serving.MEMORY, **cfg))
    monkeypatch.setattr(serving, "SBLK", int(f["sblk"]))
    monkeypatch.setattr(mem, "SBLK", int(f["sblk"]))
    monkeypatch.setattr(mem, "MEMORY", dict(mem.MEMORY, **cfg))
    keys = bf(f["keys"])
    kv, cap, d = keys.shape
    ref = mem.Archive(keys, keys.clone(), bf(f["kmax"]), bf(f["kmin"]))
    ref.smax, ref.smin = bf(f["smax"]), bf(f["smin"])
    ref.size = ref.prompt_len = int(f["prompt_len"])
    ref.dirty_lo, ref.dirty_hi = 1 << 60, -1
    ours = types.SimpleNamespace(keys=keys, values=keys, kmax=ref.kmax, kmin=ref.kmin, smax=ref.smax, smin=ref.smin,
                                 prompt_len=ref.prompt_len, dirty_lo=1 << 60, dirty_hi=-1)
    for name in f["steps"]:
        gagg = "1" if int(f[f"{name}_gagg"]) else "auto"
        monkeypatch.setattr(mem, "GLOBAL_AGG", gagg)
        monkeypatch.setattr(pertoken, "GLOBAL_AGG", gagg)
        for a in (ref, ours):
            a.hole_lo, a.hole_hi = (int(x) for x in f[f"{name}_hole"])
        lead = int(f[f"{name}_lead"])
        lead = None if lead == -9 else lead
        hist = f[f"{name}_hist"]
        q_hist = bf(hist) if hist.size else None
        q = bf(f[f"{name}_q"])
        r1 = mem.retrieve_blocks_per_token(ref, q, groups, limit, 0, lead, 0, q_hist)
        r2 = pertoken.retrieve_blocks_per_token(ours, q, groups, limit, 0, lead, 0, q_hist)
        assert torch.equal(r1[0], r2[0]), name
        for field in ("prompt_top", "decode_top", "last_hop_head", "visit_counts", "last_prio_rank"):
            a, b = getattr(ref, field), getattr(ours, field)
            assert (a is None and b is None) or torch.equal(a, b), (name, field)
        assert ref.is_global_agg == ours.is_global_agg and ref.decode_step == ours.decode_step, name
