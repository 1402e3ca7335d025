"""Host logic of the multi-GPU sharding on CPU: world-size-2 gloo process groups, with the
oracle as the per-rank kernel (the CUDA kernels need a GPU). The head-sharded result,
after the all-gather, must equal the unsharded computation exactly (same oracle, same
per-chain arithmetic)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_prefill(q, k, v, g, beta, scale, h0):
    from oracle import gdn as ogdn
    hv = v.shape[2]
    h0n = np.zeros((q.shape[0], hv, q.shape[3], v.shape[3]), np.float32) if h0 is None else h0.numpy()
    o, s = ogdn.delta_rule_chunked(ogdn.expand_key_heads(q.numpy(), hv), ogdn.expand_key_heads(k.numpy(), hv),
                                   v.numpy(), g.numpy(), beta.numpy(), scale, h0n)
    return torch.from_numpy(np.ascontiguousarray(o)), torch.from_numpy(np.ascontiguousarray(s))


def _inputs():
    from tests.inputs import gdn_inputs
    inp = gdn_inputs(41, 2, 130, 2, 8, state_std=0.02)
    return {n: torch.from_numpy(inp[n]) for n in ("q", "k", "v", "g", "beta", "h0")}, inp["scale"]


def _oracle_attention(q, k, v, window, sinks):
    from oracle import swa as oswa
    return torch.from_numpy(oswa.causal_attention(q.numpy(), k.numpy(), v.numpy(), window, sinks)).float()


def _attn_inputs():
    g = torch.Generator().manual_seed(12)
    return (torch.randn(1, 8, 150, 128, generator=g), torch.randn(1, 4, 150, 128, generator=g),
            torch.randn(1, 4, 150, 128, generator=g))


def _worker(rank, world, port, mode, outdir):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from pseudobrain_b200 import sharding
        if mode == "hybrid":
            _hybrid_worker(rank, world, outdir)
            return
        if mode == "attention":
            q, k, v = _attn_inputs()
            o = sharding.causal_attention_head_sharded(q, k, v, 50, 3, attention=_oracle_attention)
            torch.save({"o": o}, os.path.join(outdir, f"{mode}_{rank}.pt"))
            return
        x, scale = _inputs()
        fn = sharding.gdn_prefill_head_sharded if mode == "head" else sharding.gdn_prefill_batch_sharded
        o, s = fn(x["q"], x["k"], x["v"], x["g"], x["beta"], scale, x["h0"], prefill=_oracle_prefill)
        torch.save({"o": o, "s": s}, os.path.join(outdir, f"{mode}_{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["head", "batch"])
def test_sharded_prefill_equals_unsharded(tmp_path, mode):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), mode, str(tmp_path)), nprocs=world, start_method="spawn")
    x, scale = _inputs()
    o_ref, s_ref = _oracle_prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], scale, x["h0"])
    for rank in range(world):
        got = torch.load(os.path.join(tmp_path, f"{mode}_{rank}.pt"))
        if mode == "head":  # every rank ends with the full, re-assembled result
            assert torch.equal(got["o"], o_ref) and torch.equal(got["s"], s_ref)
        else:  # each rank has its own sequences
            assert torch.equal(got["o"], o_ref[rank:rank + 1]) and torch.equal(got["s"], s_ref[rank:rank + 1])


def test_head_sharded_window_attention_equals_unsharded(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), "attention", str(tmp_path)), nprocs=world,
                       start_method="spawn")
    q, k, v = _attn_inputs()
    want = _oracle_attention(q, k, v, 50, 3)
    for rank in range(world):
        got = torch.load(os.path.join(tmp_path, f"attention_{rank}.pt"))["o"]
        assert torch.equal(got, want)


def test_shard_maps():
    from pseudobrain_b200.sharding import batch_shard, head_shard
    assert head_shard(32, 16, 8, 3) == (12, 16, 6, 8)
    assert head_shard(32, 16, 1, 0) == (0, 32, 0, 16)
    assert batch_shard(8, 4, 2) == (4, 6)
    with pytest.raises(ValueError):
        head_shard(32, 8, 16, 0)  # 2 value heads per rank would split a key head of 4
    with pytest.raises(ValueError):
        batch_shard(3, 2, 0)


# ---- the hybrid layer pipeline (sharding.hybrid_layer_sharded) with CPU stand-ins -------------
HYB_T, HYB_W = 700, 100


def _hybrid_inputs():
    """Full-layer inputs: GDN 2 key / 4 value heads, attention 4 query / 2 key heads, [1,T,H,D]."""
    from tests.inputs import gdn_inputs
    inp = gdn_inputs(51, 1, HYB_T, 2, 4)
    x = {n: torch.from_numpy(inp[n]) for n in ("q", "k", "v", "g", "beta")}
    x["scale"] = inp["scale"]
    g = torch.Generator().manual_seed(52)
    qa, ka, va = (torch.randn(1, HYB_T, h, 128, generator=g) for h in (4, 2, 2))
    return x, qa, ka, va


def _cpu_gdn(x, o):
    hv = x["v"].shape[2]
    out, _ = _oracle_prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], x["scale"], None)
    o.copy_(out.view(o.shape))


def _cpu_attention(q, k, v, o, window, scale):
    # [1, T, H, D] views -> the oracle's [B, H, T, D]
    got = _oracle_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), window, 0)
    o.copy_(got.transpose(1, 2))


def _hybrid_worker(rank, world, outdir):
    from pseudobrain_b200 import sharding
    x, qa, ka, va = _hybrid_inputs()
    v0, v1, k0, k1 = sharding.head_shard(4, 2, world, rank)
    xs = {"q": x["q"][:, :, k0:k1], "k": x["k"][:, :, k0:k1], "v": x["v"][:, :, v0:v1], "g": x["g"][:, :, v0:v1],
          "beta": x["beta"][:, :, v0:v1], "scale": x["scale"]}
    a0, a1 = rank, rank + 1  # one key head (2 query heads) per rank
    gdn_all, pieces = sharding.hybrid_layer_sharded(xs, qa[:, :, 2 * a0:2 * a1], ka[:, :, a0:a1], va[:, :, a0:a1],
                                                    HYB_W, 128 ** -0.5, swa_chunks=3, gdn=_cpu_gdn,
                                                    attention=_cpu_attention)
    torch.save({"gdn": sharding.assemble_gdn(gdn_all), "swa": sharding.assemble_heads(pieces, HYB_T)},
               os.path.join(outdir, f"hybrid_{rank}.pt"))


def test_hybrid_layer_gdn_parts_join_to_one_launch():
    """The GDN branch run in two launches over groups of whole key heads (each gathered on its
    own at N > 1) joins, by assemble_gdn, to the output of one launch over all heads; a split
    that would cut a key head's group of value heads is refused."""
    from pseudobrain_b200 import sharding
    x, qa, ka, va = _hybrid_inputs()
    kw = dict(swa_chunks=2, gdn=_cpu_gdn, attention=_cpu_attention, gather=False)
    g1, p1 = sharding.hybrid_layer_sharded(x, qa, ka, va, HYB_W, 128 ** -0.5, gdn_parts=1, **kw)
    g2, p2 = sharding.hybrid_layer_sharded(x, qa, ka, va, HYB_W, 128 ** -0.5, gdn_parts=2, **kw)
    assert [(v0, v1) for v0, v1, _ in g2] == [(0, 2), (2, 4)]
    assert torch.equal(sharding.assemble_gdn(g2), sharding.assemble_gdn(g1))
    assert torch.equal(sharding.assemble_heads(p2, HYB_T), sharding.assemble_heads(p1, HYB_T))
    with pytest.raises(ValueError):
        sharding.hybrid_layer_sharded(x, qa, ka, va, HYB_W, 128 ** -0.5, gdn_parts=3, **kw)


def test_hybrid_layer_pipeline_equals_unsharded(tmp_path):
    """Head-sharded hybrid layer on 2 gloo ranks: the attention in halo'd query chunks with a
    gather per chunk, the GDN branch and its gather; the assembled outputs equal the unsharded
    branches (the same CPU stand-ins over all heads) on every rank."""
    from pseudobrain_b200 import sharding
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), "hybrid", str(tmp_path)), nprocs=world,
                       start_method="spawn")
    x, qa, ka, va = _hybrid_inputs()
    o_gdn = torch.empty(1, HYB_T, 4, 128)
    _cpu_gdn(x, o_gdn)
    o_att = torch.empty(1, HYB_T, 4, 128)
    _cpu_attention(qa, ka, va, o_att, HYB_W, 128 ** -0.5)
    want_gdn = o_gdn.view(HYB_T, 2, 2 * 128).transpose(0, 1)  # [N, T, 2 heads * 128]
    want_att = o_att.view(HYB_T, 4 * 128)
    for rank in range(world):
        got = torch.load(os.path.join(tmp_path, f"hybrid_{rank}.pt"))
        assert got["gdn"].dtype == torch.bfloat16  # the gathered GDN output is bf16 (as the model's)
        assert torch.equal(got["gdn"].float(), want_gdn.to(torch.bfloat16).float())
        assert torch.allclose(got["swa"], want_att, rtol=1e-5, atol=1e-6)
    # the chunk plan covers every row once, halos within the window
    plan = sharding.swa_chunk_plan(HYB_T, HYB_W, 3)
    assert plan[0][0] == 0 and plan[-1][1] == HYB_T
    assert all(a[1] == b[0] for a, b in zip(plan, plan[1:]))
    assert all(h == min(s, 128) for s, _, h in plan)


def test_default_transport_by_group_size():
    """The hybrid layer's exchange: copy engines (p2p) only for NCCL groups of 2..4 CUDA ranks
    (measured faster there; at 8 ranks NCCL's all-gather is); one rank or host tensors: nccl."""
    from pseudobrain_b200 import sharding
    assert sharding.default_transport(1, True) == "nccl"
    assert sharding.default_transport(2, False) == "nccl"
    assert sharding.default_transport(8, True) == "nccl"
    assert sharding.P2P_MAX_RANKS == 4
