"""GPU parity of the serving path's per-token selector (pseudobrain_b200.pertoken) with the
reference's retrieve_blocks_per_token (pb27_vllm/memory.py:1009-1294), replayed step by step
from tests/golden/pertoken.npz: before each step the selector state is set to the reference's
state before it (prompt and decode blocks, hop head, visit counts, decode step, the global-
aggregation flag), then the selected blocks and the state after the step must equal the
reference's. The steps cover the prompt branch with exact per-token rescoring and the second
hop, decode steps with a query history over super-blocks with the prompt and decode merges,
a piece without a lead, forced dense global aggregation (stratified peaks, visit counts, the
novelty penalty) and a prompt piece over an archive hole. The fixture's reference ran with
ties in index order (the tie rule of this build; torch's CPU order among equal tier keys is
implementation-defined), so the comparison is exact."""
from __future__ import annotations

import os
import types

import numpy as np
import pytest
import torch

from tests.conftest import ROOT

pytestmark = pytest.mark.gpu
FIX = os.path.join(ROOT, "tests", "golden", "pertoken.npz")


def _bf(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def _opt(a, dev, dtype=torch.int64):
    return None if a.size == 0 else torch.from_numpy(a).to(device=dev, dtype=dtype)


@pytest.fixture()
def selector(cuda_device):
    from pseudobrain_b200 import pertoken, serving
    saved = (dict(serving.MEMORY), serving.SBLK, pertoken.GLOBAL_AGG)
    yield pertoken, serving
    serving.MEMORY.clear()
    serving.MEMORY.update(saved[0])
    serving.SBLK, pertoken.GLOBAL_AGG = saved[1], saved[2]


@pytest.mark.parametrize("fixture", ["pertoken.npz", "pertoken256.npz"])
def test_per_token_selection_matches_reference(cuda_device, selector, fixture):
    """pertoken.npz: 2 key heads x 3 query heads at head dim 128; pertoken256.npz: PB-27's
    attention shape, 4 key heads x 6 query heads at head dim 256."""
    pertoken, serving = selector
    f = np.load(os.path.join(ROOT, "tests", "golden", fixture))
    dev = cuda_device
    serving.MEMORY.update(blocks=8, decode_blocks=8, rerank=12, block_size=int(f["block"]), neighbors=0, window=64,
                          chunk=64)
    serving.SBLK = int(f["sblk"])
    assert int(f["origin"]) == serving.ORIGIN
    keys = _bf(f["keys"], dev)
    arc = types.SimpleNamespace(keys=keys, values=_bf(f["values"], dev), kmax=_bf(f["kmax"], dev),
                                kmin=_bf(f["kmin"], dev), smax=_bf(f["smax"], dev), smin=_bf(f["smin"], dev),
                                smean_k=torch.from_numpy(f["smean_k"]).to(dev),
                                smean_v=torch.from_numpy(f["smean_v"]).to(dev),
                                prompt_len=int(f["prompt_len"]), dirty_lo=1 << 60, dirty_hi=-1)
    groups, limit = int(f["groups"]), int(f["limit"])
    diffs = {}
    for name in f["steps"]:
        for field in ("prompt_top", "decode_top", "last_hop_head"):
            setattr(arc, field, _opt(f[f"{name}_before_{field}"], dev))
        vc = f[f"{name}_before_visit_counts"]
        arc.visit_counts = None if vc.size == 0 else torch.from_numpy(vc).to(dev, torch.int16)
        arc.decode_step = int(f[f"{name}_before_decode_step"])
        arc.is_global_agg = bool(f[f"{name}_before_global"])
        arc.cached_top = None
        arc.hole_lo, arc.hole_hi = (int(x) for x in f[f"{name}_hole"])
        pertoken.GLOBAL_AGG = "1" if int(f[f"{name}_gagg"]) else "auto"
        lead = int(f[f"{name}_lead"])
        lead = None if lead == -9 else lead
        hist = f[f"{name}_hist"]
        q_hist = _bf(hist, dev) if hist.size else None
        res = pertoken.retrieve_blocks_per_token(arc, _bf(f[f"{name}_q"], dev), groups, limit, 0, lead, 0, q_hist)
        top = res[0].cpu().numpy()
        want = f[f"{name}_top"]
        diffs[name] = int((top != want).sum()) if top.shape == want.shape else -1
        print(f"[per-token {fixture}] {name}: {diffs[name]} differing block indices of {want.size}")
        assert top.shape == want.shape and np.array_equal(top, want), name
        assert bool(arc.is_global_agg) == bool(f[f"{name}_after_global"]), name
        assert arc.decode_step == int(f[f"{name}_after_decode_step"]), name
        for field in ("prompt_top", "decode_top"):
            got, ref = getattr(arc, field), f[f"{name}_after_{field}"]
            assert (got is None and ref.size == 0) or np.array_equal(got.cpu().numpy(), ref), (name, field)
        vc_ref = f[f"{name}_after_visit_counts"]
        if vc_ref.size:
            assert np.array_equal(arc.visit_counts.cpu().numpy(), vc_ref), name
        if f"{name}_attn" in f.files:  # the piece's attention (landmarks after the sinks under global aggregation)
            qpos = torch.tensor([limit + 63], device=dev)
            o = serving.piece_attention(arc, _bf(f[f"{name}_q"], dev), qpos, res[0], groups, int(f["window"]),
                                        keys.shape[-1] ** -0.5, None, q_min=limit + 63, q_max=limit + 63)
            ref = f[f"{name}_attn"]
            err = float(np.linalg.norm(o.float().cpu().numpy() - ref) / np.linalg.norm(ref))
            print(f"[per-token {fixture}] {name}: attention rel err {err:.2e}")
            assert err < 2e-2, name
            assert arc.cached_top is res[0]  # the reference caches the set when a prompt set exists


def test_rank_kernel_orders_like_a_stable_descending_sort(cuda_device, selector):
    """Ranks of rows with ties, -inf entries and lengths that are not powers of two equal a
    stable descending argsort's positions."""
    pertoken, _ = selector
    g = torch.Generator(device=cuda_device).manual_seed(5)
    for n in (1, 7, 300, 4096, 12289):
        x = torch.randint(-40, 40, (3, n), device=cuda_device, generator=g).float()
        x[0, : n // 3] = float("-inf")
        got = pertoken.ranks(x)
        order = torch.sort(x, dim=-1, descending=True, stable=True).indices
        want = torch.empty_like(order).scatter_(-1, order, torch.arange(n, device=cuda_device).expand(3, n))
        assert torch.equal(got, want), n


def test_token_scores_and_rerank_match_per_token_products(cuda_device, selector):
    """pbk_quest_token_scores against the per-token bound score computed with fp64 products
    (candidate lists, out-of-range candidates, the hole, the RoPE-dims mask), and
    pbk_quest_token_rerank against fp64 q . k maxima."""
    pertoken, _ = selector
    g = torch.Generator(device=cuda_device).manual_seed(9)
    kv, groups, t, d, nb, block = 2, 5, 9, 128, 70, 16
    q = torch.randn(t, kv * groups, d, device=cuda_device, generator=g).to(torch.bfloat16)
    keys = torch.randn(kv, nb * block, d, device=cuda_device, generator=g).to(torch.bfloat16)
    kb = keys.view(kv, nb, block, d)
    kmax, kmin = kb.amax(2), kb.amin(2)
    cand = torch.randint(0, nb + 6, (kv, 33), device=cuda_device, generator=g)
    for rope in (False, True):
        got = pertoken.token_scores(q, kmax, kmin, nb, 33, cand=cand, hole=(10, 20), rope_mask=rope)
        qd = q.double().view(t, kv, groups, d)
        if rope:
            qd[..., : d // 4] = 0
        cc = cand.clamp(max=nb - 1)
        bmx = kmax.double().gather(1, cc[..., None].expand(-1, -1, d))
        bmn = kmin.double().gather(1, cc[..., None].expand(-1, -1, d))
        want = (torch.einsum("tkgd,kjd->ktgj", qd.clamp(min=0), bmx) +
                torch.einsum("tkgd,kjd->ktgj", qd.clamp(max=0), bmn)).amax(2)
        bad = (cand >= nb) | ((cand >= 10) & (cand < 20))
        want = want.masked_fill(bad[:, None, :], float("-inf"))
        fin = torch.isfinite(want)
        assert torch.equal(torch.isfinite(got), fin)
        assert torch.allclose(got[fin].double(), want[fin], rtol=1e-5, atol=1e-4)
    rc = torch.randint(0, nb, (kv, 21), device=cuda_device, generator=g)
    got = pertoken.token_rerank(q, keys, block, rc, 21)
    kr = keys.double().view(kv, nb, block, d).gather(1, rc[..., None, None].expand(-1, -1, block, d))
    want = torch.einsum("tkgd,kjsd->ktgjs", q.double().view(t, kv, groups, d), kr).amax(-1).amax(2)
    assert torch.allclose(got.double(), want, rtol=1e-5, atol=1e-4)
