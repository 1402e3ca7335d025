"""pbk_quest_select_noalloc: the page selection for callers that cannot allocate device
memory (a host that already owns all free HBM, or a foreign-language caller with no handle
on the framework's allocator). It keeps its page scores in a fixed array inside libpbk
instead of a caller workspace.

Called here through the C ABI and compared with pbk_quest_select (the entry point that
takes a workspace) on the same inputs: page indices must be identical, as for every Quest
test. Two different problems run back to back, so the second call reads the shared array
after the first call left its contents there. This file sorts last, so a run that stops
at the first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _problem(seed, nq, kv, heads, npages, page, budget, device, t=1):
    from pseudobrain_b200 import exact_memory as M
    gen = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(nq, t, heads, 128, generator=gen, device=device).to(torch.bfloat16)
    a = torch.randn(kv, npages, 128, generator=gen, device=device)
    b = torch.randn(kv, npages, 128, generator=gen, device=device)
    kmax, kmin = torch.maximum(a, b).to(torch.bfloat16), torch.minimum(a, b).to(torch.bfloat16)
    k = min(budget, npages)
    pages = torch.full((nq, kv, k), -1, dtype=torch.int32, device=device)
    desc = M._desc(q, page, npages * page, budget, kmax=kmax, kmin=kmin, pages=pages)
    return q, kmax, kmin, pages, desc


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _select_with_workspace(desc, device):
    from pseudobrain_b200._capi import LIB, check
    nbytes = LIB.pbk_quest_select_workspace(ctypes.byref(desc))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
    check(LIB.pbk_quest_select(ctypes.byref(desc), ws.data_ptr(), ws.numel(), _stream(device)), "pbk_quest_select")


def _select_noalloc(desc, device):
    from pseudobrain_b200._capi import LIB, check
    check(LIB.pbk_quest_select_noalloc(ctypes.byref(desc), _stream(device)), "pbk_quest_select_noalloc")


def test_noalloc_select_matches_workspace_select_on_consecutive_calls(cuda_device):
    # config-3 sized selection (8 groups x 8 key heads, 65280 pages: 4,177,920 scores),
    # then a smaller problem that reads the array the first call filled
    for seed, nq, kv, heads, npages, budget in ((11, 8, 8, 32, 65280, 256), (12, 3, 2, 8, 5003, 17)):
        q, kmax, kmin, pages, desc = _problem(seed, nq, kv, heads, npages, 16, budget, cuda_device)
        _select_with_workspace(desc, cuda_device)
        expected = pages.clone()
        pages.fill_(-1)
        _select_noalloc(desc, cuda_device)
        torch.cuda.synchronize()
        assert torch.equal(pages, expected)
        assert bool((pages >= 0).all())
        # the same call again gives the same pages
        pages.fill_(-1)
        _select_noalloc(desc, cuda_device)
        torch.cuda.synchronize()
        assert torch.equal(pages, expected)


def test_noalloc_select_matches_on_the_simt_score_path(cuda_device):
    """More than 64 query rows per key head (3 groups x 6 tokens x 16 query heads over one key
    head: 288 rows) take the SIMT score kernel instead of the tensor-core one; the array then
    holds its scores and segment maxima without tile bound magnitudes."""
    q, kmax, kmin, pages, desc = _problem(14, 3, 1, 16, 4100, 16, 33, cuda_device, t=6)
    _select_with_workspace(desc, cuda_device)
    expected = pages.clone()
    for _ in range(2):
        pages.fill_(-1)
        _select_noalloc(desc, cuda_device)
        torch.cuda.synchronize()
        assert torch.equal(pages, expected)


def test_noalloc_select_writes_caller_scores_when_given(cuda_device):
    q, kmax, kmin, pages, desc = _problem(13, 2, 4, 16, 3000, 16, 40, cuda_device)
    scores_ref = torch.empty(2, 4, 3000, device=cuda_device)
    desc.scores = scores_ref.data_ptr()
    _select_with_workspace(desc, cuda_device)
    expected = pages.clone()
    scores = torch.full_like(scores_ref, float("nan"))
    desc.scores = scores.data_ptr()
    pages.fill_(-1)
    _select_noalloc(desc, cuda_device)
    torch.cuda.synchronize()
    assert torch.equal(pages, expected)
    assert torch.equal(scores, scores_ref)


def test_noalloc_select_rejects_problems_beyond_its_scratch(cuda_device):
    from pseudobrain_b200._capi import LIB, PBK_ERR_TOO_LARGE, PBK_QUEST_NOALLOC_MAX_SCORES
    npages = PBK_QUEST_NOALLOC_MAX_SCORES // 8 + 1  # 1 group x 8 key heads: one score too many
    q = torch.zeros(1, 1, 8, 128, dtype=torch.bfloat16, device=cuda_device)
    kmax = torch.zeros(8, npages, 128, dtype=torch.bfloat16, device=cuda_device)
    pages = torch.full((1, 8, 4), -1, dtype=torch.int32, device=cuda_device)
    from pseudobrain_b200 import exact_memory as M
    desc = M._desc(q, 16, npages * 16, 4, kmax=kmax, kmin=kmax, pages=pages)
    assert LIB.pbk_quest_select_noalloc(ctypes.byref(desc), _stream(cuda_device)) == PBK_ERR_TOO_LARGE
    torch.cuda.synchronize()
    assert bool((pages == -1).all())  # nothing launched
    assert np.isfinite(float(torch.zeros(1, device=cuda_device).sum()))  # the context is still usable
