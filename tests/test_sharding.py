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
