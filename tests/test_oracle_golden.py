"""Pin the CPU oracle against the reference's own outputs (tests/golden/*.npz).

The fixtures were produced by tests/golden/make_golden.py from the reference's
pseudobrain.gated_deltanet / pseudobrain.exact_memory functions. Both sides compute
in fp32 with different summation orders, so float outputs agree to ~1e-6 relative;
bounds, page indices and gathered keys must agree bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import gdn as ogdn
from oracle import quest as oq
from tests.conftest import load_golden

FP32_TOL = 1e-5


def _f32(bits):
    return oq.bf16_from_bits(bits)


def test_gdn_fp32_chunked_and_sequential_match_reference():
    f = load_golden("gdn_fp32.npz")
    hv = f["v"].shape[2]
    q, k = ogdn.expand_key_heads(f["q"], hv), ogdn.expand_key_heads(f["k"], hv)
    args = (q, k, f["v"], f["g"], f["beta"], float(f["scale"]), f["h0"])
    o, s = ogdn.delta_rule_chunked(*args)
    assert ogdn.rel_err(o, f["o_chunked"]) < FP32_TOL
    assert ogdn.rel_err(s, f["s_chunked"]) < FP32_TOL
    o, s = ogdn.delta_rule_sequential(*args)
    assert ogdn.rel_err(o, f["o_sequential"]) < FP32_TOL
    assert ogdn.rel_err(s, f["s_sequential"]) < FP32_TOL
    # The reference's two kernels agree with each other too (same recurrence).
    assert ogdn.rel_err(f["o_chunked"], f["o_sequential"]) < FP32_TOL


def test_gdn_bf16_inputs_chunked_matches_reference():
    f = load_golden("gdn_bf16.npz")
    hv = f["v"].shape[2]
    q = ogdn.expand_key_heads(_f32(f["q"]), hv)
    k = ogdn.expand_key_heads(_f32(f["k"]), hv)
    o, s = ogdn.delta_rule_chunked(q, k, _f32(f["v"]), f["g"], _f32(f["beta"]), float(f["scale"]), f["h0"])
    assert ogdn.rel_err(o, f["o_chunked"]) < FP32_TOL
    assert ogdn.rel_err(s, f["s_chunked"]) < FP32_TOL


def test_gdn_decode_sequential_matches_reference():
    f = load_golden("gdn_decode.npz")
    hv = f["v"].shape[2]
    q = ogdn.expand_key_heads(_f32(f["q"]), hv)
    k = ogdn.expand_key_heads(_f32(f["k"]), hv)
    o, s = ogdn.delta_rule_sequential(q, k, _f32(f["v"]), _f32(f["g"]), _f32(f["beta"]),
                                      float(f["scale"]), f["h0"])
    assert ogdn.rel_err(o, f["o_sequential"]) < FP32_TOL
    assert ogdn.rel_err(s, f["s_sequential"]) < FP32_TOL


def test_gdn_fp64_oracle_agrees_with_fp32():
    f = load_golden("gdn_fp32.npz")
    hv = f["v"].shape[2]
    q, k = ogdn.expand_key_heads(f["q"], hv), ogdn.expand_key_heads(f["k"], hv)
    args64 = [x.astype(np.float64) for x in (q, k, f["v"], f["g"], f["beta"])]
    o64, s64 = ogdn.delta_rule_sequential(*args64, float(f["scale"]), f["h0"].astype(np.float64))
    assert ogdn.rel_err(f["o_chunked"], o64) < FP32_TOL
    assert ogdn.rel_err(f["s_chunked"], s64) < FP32_TOL


@pytest.fixture(scope="module")
def quest():
    f = load_golden("quest.npz")
    page, n_arch = int(f["page"]), int(f["n_arch"])
    keys, values = _f32(f["keys"]), _f32(f["values"])
    arc = oq.archive_append(None, keys[:, :, :100], values[:, :, :100], page)
    arc = oq.archive_append(arc, keys[:, :, 100:n_arch], values[:, :, 100:n_arch], page)
    return f, arc, keys, values


def test_quest_bounds_bit_exact(quest):
    f, arc, _, _ = quest
    assert np.array_equal(oq.bf16_bits(arc.kmax), f["kmax"])
    assert np.array_equal(oq.bf16_bits(arc.kmin), f["kmin"])


@pytest.mark.parametrize("case", ["t1", "t3"])
def test_quest_retrieve_and_attend_match_reference(quest, case):
    f, arc, keys, values = quest
    page, budget, groups, window = (int(f[x]) for x in ("page", "budget", "groups", "window"))
    n_arch = int(f["n_arch"])
    q = _f32(f[f"{case}_q"])
    rk, rv, top = oq.retrieve(arc, q, groups, page, budget)
    assert np.array_equal(top, f[f"{case}_top"])
    assert np.array_equal(oq.bf16_bits(rk), f[f"{case}_rk"])
    assert np.array_equal(oq.bf16_bits(rv), f[f"{case}_rv"])
    out = oq.attend(q, rk, rv, keys[:, :, n_arch:], values[:, :, n_arch:], f[f"{case}_qpos"],
                    f["kpos"], window, 0, groups)
    assert ogdn.rel_err(out, f[f"{case}_out"]) < FP32_TOL


def test_select_pages_ties_go_to_lowest_index():
    score = np.array([[3.0, 5.0, 5.0, 1.0, 5.0, 2.0]], dtype=np.float32)
    assert oq.select_pages(score, 2).tolist() == [[1, 2]]
    assert oq.select_pages(score, 4).tolist() == [[0, 1, 2, 4]]
    assert oq.select_pages(score, 10).tolist() == [[0, 1, 2, 3, 4, 5]]


def test_bf16_round_is_round_to_nearest_even():
    import torch
    x = np.random.default_rng(0).standard_normal(4096).astype(np.float32) * 37
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(oq.bf16_round(x), ref)


@pytest.mark.parametrize("case", ["win", "full"])
def test_window_attention_matches_reference(case):
    """oracle/swa.py against transplant.causal_attention (window 100 + 4 sinks through the
    reference's query-chunked path; full causal)."""
    from oracle import swa as oswa
    f = load_golden("swa.npz")
    window = int(f[f"{case}_window"])
    o = oswa.causal_attention(_f32(f[f"{case}_q"]), _f32(f[f"{case}_k"]), _f32(f[f"{case}_v"]),
                              None if window < 0 else window, int(f[f"{case}_sinks"]))
    assert ogdn.rel_err(o, f[f"{case}_o"]) < FP32_TOL
    # the row-subset form used for long sequences agrees with the full one
    part = oswa.causal_attention_at(_f32(f[f"{case}_q"]), _f32(f[f"{case}_k"]), _f32(f[f"{case}_v"]), [0, 130], 50,
                                    None if window < 0 else window, int(f[f"{case}_sinks"]))
    for s, x in part.items():
        assert np.allclose(x, o[:, :, s:s + 50], rtol=0, atol=1e-12)


@pytest.mark.parametrize("case", ["t1", "t3", "flat"])
def test_serving_twins_match_reference(case):
    """oracle/serving.py against pb27_vllm/memory.py's retrieve_blocks and piece_attention."""
    from oracle import serving as osv
    f = load_golden("serving.npz")
    keys, values = _f32(f["keys"]), _f32(f["values"])
    kmax, kmin = _f32(f["kmax"]), _f32(f["kmin"])
    q = _f32(f[f"{case}_q"])
    mem = dict(blocks=int(f["budget"]), decode_blocks=int(f["budget"]), rerank=int(f["rerank_pool"]),
               block_size=int(f["block"]), window=int(f["window"]))
    top = osv.retrieve_blocks(keys, kmax, kmin, q, int(f["groups"]), int(f[f"{case}_limit"]),
                              bool(f[f"{case}_rerank"]), mem, keys.shape[1])
    assert np.array_equal(top, f[f"{case}_top"])
    o = osv.piece_attention(keys, values, q, f[f"{case}_pos"], top, int(f["groups"]), int(f["window"]),
                            q.shape[-1] ** -0.5, int(f["block"]))
    assert ogdn.rel_err(o, f[f"{case}_out"]) < FP32_TOL


def test_gdn_layer_pieces_match_reference():
    """short_convolution, l2_normalize (both modes), gating and the gated output norm of the
    oracle against the reference's outputs."""
    f = load_golden("gdn_io.npz")
    y, new_tail = ogdn.short_convolution(f["x"], f["tail"], f["weight"])
    assert ogdn.rel_err(y, f["y"]) < 1e-5
    assert np.array_equal(new_tail, f["new_tail"])
    b, t = f["x"].shape[:2]
    d = 128
    for mode in ("max", "hf"):
        assert ogdn.rel_err(ogdn.l2_normalize(y[..., :d].reshape(b, t, 1, d), mode), f[f"q_{mode}"]) < 1e-5
        assert ogdn.rel_err(ogdn.l2_normalize(y[..., d:2 * d].reshape(b, t, 1, d), mode), f[f"k_{mode}"]) < 1e-5
    small = np.zeros((1, 1, d), np.float32)
    small[..., 0] = 1e-4
    assert np.allclose(ogdn.l2_normalize(small, "max"), f["small_max"])
    assert np.allclose(ogdn.l2_normalize(small, "hf"), f["small_hf"])
    hv = f["a_log"].shape[0]
    g, beta = ogdn.gating(f["decay"][..., :hv], f["decay"][..., hv:], f["a_log"], f["dt_bias"])
    assert ogdn.rel_err(g, f["g"]) < 1e-6 and ogdn.rel_err(beta, f["beta"]) < 1e-6
    out = ogdn.gated_out_norm(f["o"], f["gate"].reshape(f["o"].shape), f["o_norm"])
    assert ogdn.rel_err(out, f["out"]) < 1e-5


LEVEL_CASES = {"sb_t1": {}, "sb_t3": {}, "rerank_t1": {"rerank": 24}, "sb_nb_t1": {"neighbors": 1},
               "prompt_t80": {}, "sb_after_prompt_t1": {"prompt": "prompt_t80"}}


@pytest.fixture(scope="module")
def levels():
    return load_golden("quest_levels.npz")


def test_super_bounds_bit_exact(levels):
    """oracle super_bounds against the reference archive's smax/smin (exact_memory.py:53-63)."""
    f = levels
    smax, smin = oq.super_bounds(_f32(f["kmax"]), _f32(f["kmin"]), int(f["sblk"]))
    assert np.array_equal(oq.bf16_bits(smax), f["smax"])
    assert np.array_equal(oq.bf16_bits(smin), f["smin"])


@pytest.mark.parametrize("case", list(LEVEL_CASES))
def test_retrieve_modes_match_reference(levels, case):
    """Two-level super-block selection, exact rerank, neighbours and a kept prompt selection
    (exact_memory.py:88-152) against the reference's own retrieve."""
    f = levels
    page, budget, groups, sblk = (int(f[x]) for x in ("page", "budget", "groups", "sblk"))
    opt = LEVEL_CASES[case]
    prompt = f[f"{opt['prompt']}_top"] if "prompt" in opt else None
    _, _, top = oq.retrieve_modes(_f32(f["keys"]), _f32(f["values"]), _f32(f["kmax"]), _f32(f["kmin"]),
                                  _f32(f[f"{case}_q"]), groups, page, budget, superblock=sblk,
                                  rerank=opt.get("rerank", 0), neighbors=opt.get("neighbors", 0), prompt_top=prompt)
    assert np.array_equal(top, f[f"{case}_top"])


@pytest.mark.parametrize("case", ["s_sb", "s_sb_hole", "s_sb_nb", "s_flat_hole", "s_rerank_hole"])
def test_serving_levels_match_reference(levels, case):
    """The serving retrieve_blocks' super-block path, archive hole and neighbours
    (pb27_vllm/memory.py:760-878) against the reference."""
    from oracle import serving as osv
    f = levels
    page, sblk, groups = int(f["page"]), int(f["sblk"]), int(f["groups"])
    kmax, kmin = _f32(f["s_kmax"]), _f32(f["s_kmin"])
    smax, smin = osv.super_bounds(kmax, kmin, kmax.shape[1], sblk)
    assert np.array_equal(oq.bf16_bits(smax), f["s_smax"]) and np.array_equal(oq.bf16_bits(smin), f["s_smin"])
    keys = _f32(f["s_keys"])
    mem = dict(blocks=8, decode_blocks=8, rerank=int(f[f"{case}_pool"]), block_size=page, window=64,
               neighbors=int(f[f"{case}_neighbors"]))
    use_sb = not int(f[f"{case}_nosb"])
    top = osv.retrieve_blocks(keys, kmax, kmin, _f32(f[f"{case}_q"]), groups, int(f["s_limit"]),
                              bool(f[f"{case}_rerank"]), mem, keys.shape[1], smax if use_sb else None,
                              smin if use_sb else None, sblk, tuple(int(x) for x in f[f"{case}_hole"]))
    assert np.array_equal(top, f[f"{case}_top"])


@pytest.fixture(scope="module")
def rope():
    return load_golden("rope.npz")


def test_rope_moves_match_reference(rope):
    """The block moves (contiguous runs, proportional) and the sink move (pb27_vllm/memory.py:
    574-677): bf16 outputs equal the reference's but for rare last-bit differences of cos/sin."""
    from oracle import serving as osv
    f = rope
    args = (int(f["horizon"]), int(f["arc_span"]), float(f["theta"]))
    rk, sk, idx, block, ref_pos = _f32(f["rk"]), _f32(f["sk"]), f["idx"], int(f["block"]), int(f["ref_pos"])
    for got, want in ((osv.reposition_blocks(rk, idx, block, ref_pos, True, *args), f["rk_runs"]),
                      (osv.reposition_blocks(rk, idx, block, ref_pos, False, *args), f["rk_prop"]),
                      (osv.reposition_sinks(sk, ref_pos, idx.shape[1], block, *args), f["sk_moved"])):
        w = _f32(want)
        assert np.mean(oq.bf16_bits(got) != want) < 1e-3
        assert np.allclose(got, w, rtol=1e-2, atol=1e-2)
    assert not np.array_equal(f["rk_runs"], f["rk"])  # the moves did turn the keys


@pytest.mark.parametrize("case", ["rr", "flat"])
def test_rope_serving_matches_reference(rope, case):
    """retrieve_blocks (rerank with moved candidate keys; flat with the RoPE dims masked) and
    piece_attention with moved sinks and blocks, past a lowered horizon."""
    from oracle import serving as osv
    f = rope
    args = (int(f["horizon"]), int(f["arc_span"]), float(f["theta"]))
    keys, values = _f32(f["keys"]), _f32(f["values"])
    block, groups, window = int(f["block"]), int(f["groups"]), int(f["window"])
    kmax, kmin = oq.page_bounds(keys[None, :, 4:4 + ((keys.shape[1] - 4) // block) * block], block)
    mem = dict(blocks=4, decode_blocks=4, rerank=12, block_size=block, window=window)
    q = _f32(f[f"{case}_q"])
    top = osv.retrieve_blocks(keys, kmax[0], kmin[0], q, groups, int(f[f"{case}_limit"]), bool(f[f"{case}_rerank"]),
                              mem, keys.shape[1], rope=args, bf16_keys=False)  # the reference ran on fp32 keys
    assert np.array_equal(top, f[f"{case}_top"])
    o = osv.piece_attention(keys, values, q, f[f"{case}_pos"], top, groups, window, 128 ** -0.5, block, rope=args,
                            bf16_keys=False)
    assert ogdn.rel_err(o, f[f"{case}_out"]) < 1e-4


def test_archive_write_matches_reference():
    """oracle ArchiveState.write / refresh_bounds against pb27_vllm/memory.py's Archive.write
    (fast path, short and scattered writes, a write across super-blocks): storage and max /
    min summaries exact, means to fp32 rounding."""
    from oracle import serving as osv
    f = load_golden("archive_write.npz")
    block, sblk, cap = int(f["block"]), int(f["sblk"]), int(f["cap"])
    kv, d = f["keys"].shape[0], f["keys"].shape[2]
    arc = osv.ArchiveState(kv, d, cap, block, sblk)
    for i in range(int(f["n_writes"])):
        arc.write(f[f"w{i}_pos"], _f32(f[f"w{i}_k"]), _f32(f[f"w{i}_v"]))
    arc.refresh_bounds()
    size = int(f["size"])
    assert arc.size == size
    # the reference allocates with torch.empty: only written rows, blocks and super-blocks count
    assert np.array_equal(oq.bf16_bits(arc.keys[:, :size]), f["keys"][:, :size])
    assert np.array_equal(oq.bf16_bits(arc.values[:, :size]), f["values"][:, :size])
    nb = (size - osv.ORIGIN + block - 1) // block
    nsb = (nb + sblk - 1) // sblk
    for name, n in (("kmax", nb), ("kmin", nb), ("smax", nsb), ("smin", nsb)):
        assert np.array_equal(getattr(arc, name)[:, :n], f[name][:, :n]), name
    for name, n in (("bmean_k", nb), ("bmean_v", nb), ("smean_k", nsb), ("smean_v", nsb)):
        assert np.allclose(getattr(arc, name)[:, :n], f[name][:, :n], rtol=0, atol=1e-6), name


def test_canonical_scores_follow_the_fixed_order():
    """canonical_bound_scores equals a scalar fp32 loop over d = 0..127 (each product exact,
    each addition rounded), row by row, and stays within fp32 summation error of the fp64
    bound scores."""
    rng = np.random.default_rng(9)
    q = oq.bf16_round(rng.standard_normal((2, 3, 128)).astype(np.float32))
    kmax = oq.bf16_round(rng.standard_normal((2, 5, 128)).astype(np.float32) * 3)
    kmin = oq.bf16_round(kmax - np.abs(rng.standard_normal((2, 5, 128))).astype(np.float32))
    got = oq.canonical_bound_scores(q, kmax, kmin)
    for h in range(2):
        for p in range(5):
            best = np.float32(-np.inf)
            for r in range(3):
                acc = np.float32(0)
                for d in range(128):
                    qd = q[h, r, d]
                    acc = np.float32(acc + np.float32(qd * (kmax[h, p, d] if qd > 0 else kmin[h, p, d])))
                best = max(best, acc)
            assert got[h, p] == best
    ref = oq._bound_scores(q, kmax, kmin)
    assert np.allclose(got, ref, rtol=1e-5, atol=1e-5)
    cand = np.array([[0, 2], [1, 4]])
    keys = oq.bf16_round(rng.standard_normal((2, 5 * 4, 128)).astype(np.float32))
    ex = oq.canonical_rerank_scores(q, keys, cand, 4)
    for h in range(2):
        for c in range(2):
            best = np.float32(-np.inf)
            for r in range(3):
                for s in range(4):
                    acc = np.float32(0)
                    for d in range(128):
                        acc = np.float32(acc + np.float32(q[h, r, d] * keys[h, cand[h, c] * 4 + s, d]))
                    best = max(best, acc)
            assert ex[h, c] == best


@pytest.mark.parametrize("case", ["t1", "t3"])
def test_canonical_selection_equals_reference_selection(quest, case):
    """On the reference's golden retrieval the canonical-order selection picks the same pages
    as the reference's own (GEMM-order) scores: no near-tie decides these cases."""
    f, arc, _, _ = quest
    page, budget, groups = (int(f[x]) for x in ("page", "budget", "groups"))
    full = arc.length // page
    s = oq.canonical_page_scores(_f32(f[f"{case}_q"]), arc.kmax[:, :, :full], arc.kmin[:, :, :full], groups)
    assert np.array_equal(oq.select_pages(s, budget), f[f"{case}_top"])


@pytest.mark.parametrize("case", list(LEVEL_CASES))
def test_canonical_retrieve_modes_equal_reference(levels, case):
    """The two-level, rerank, neighbour and prompt modes in the canonical order pick the
    reference's pages on its golden cases."""
    f = levels
    page, budget, groups, sblk = (int(f[x]) for x in ("page", "budget", "groups", "sblk"))
    opt = LEVEL_CASES[case]
    prompt = f[f"{opt['prompt']}_top"] if "prompt" in opt else None
    _, _, top = oq.retrieve_modes(_f32(f["keys"]), _f32(f["values"]), _f32(f["kmax"]), _f32(f["kmin"]),
                                  _f32(f[f"{case}_q"]), groups, page, budget, superblock=sblk,
                                  rerank=opt.get("rerank", 0), neighbors=opt.get("neighbors", 0), prompt_top=prompt,
                                  canonical=True)
    assert np.array_equal(top, f[f"{case}_top"])


@pytest.mark.parametrize("case", ["s_sb", "s_sb_hole", "s_sb_nb", "s_flat_hole", "s_rerank_hole"])
def test_canonical_serving_levels_equal_reference(levels, case):
    from oracle import serving as osv
    f = levels
    page, sblk, groups = int(f["page"]), int(f["sblk"]), int(f["groups"])
    kmax, kmin = _f32(f["s_kmax"]), _f32(f["s_kmin"])
    smax, smin = osv.super_bounds(kmax, kmin, kmax.shape[1], sblk)
    keys = _f32(f["s_keys"])
    mem = dict(blocks=8, decode_blocks=8, rerank=int(f[f"{case}_pool"]), block_size=page, window=64,
               neighbors=int(f[f"{case}_neighbors"]))
    use_sb = not int(f[f"{case}_nosb"])
    top = osv.retrieve_blocks(keys, kmax, kmin, _f32(f[f"{case}_q"]), groups, int(f["s_limit"]),
                              bool(f[f"{case}_rerank"]), mem, keys.shape[1], smax if use_sb else None,
                              smin if use_sb else None, sblk, tuple(int(x) for x in f[f"{case}_hole"]),
                              canonical=True)
    assert np.array_equal(top, f[f"{case}_top"])
