"""The head-sharded hybrid layer on 2 GPUs over NCCL (sharding.hybrid_layer_sharded with the
CUDA kernels): each rank runs its GDN value heads (segmented along T) and its attention key
head in halo'd query chunks, every output chunk is all-gathered as it is written, and the
assembled [T, heads * 128] outputs on every rank equal the unsharded layer (all heads on one
GPU, the same kernels) to bf16 rounding (2e-2, the bar for bf16 inputs; the segment counts and
the attention's tile alignment differ between the two, so the sums associate differently).
Both transports run: NCCL's all-gather, and the copy-engine exchange (CUDA IPC mappings,
cudaMemcpyAsync pushes) twice in a row, which must move the same bytes. Skipped on hosts with
fewer than 2 GPUs. The ranks are child processes with a short process-
group timeout, so a failure ends with an error instead of a wait."""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.conftest import ROOT

pytestmark = pytest.mark.gpu
T, WINDOW = 20000, 1024
GDN_HK, GDN_HV, ATT_H, ATT_KV = 4, 8, 8, 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer_inputs(dev):
    """The full layer's inputs, the same on every rank (seeded on the device)."""
    from pseudobrain_b200.synthetic import gdn_inputs
    x = gdn_inputs(1, T, GDN_HK, GDN_HV, device=dev, seed=71)
    gen = torch.Generator(device=dev).manual_seed(72)
    qa = torch.randn(1, T, ATT_H, 128, device=dev, generator=gen).to(torch.bfloat16)
    ka = torch.randn(1, T, ATT_KV, 128, device=dev, generator=gen).to(torch.bfloat16)
    va = torch.randn(1, T, ATT_KV, 128, device=dev, generator=gen).to(torch.bfloat16)
    return x, qa, ka, va


def _worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from pseudobrain_b200 import sharding
        x, qa, ka, va = _layer_inputs(dev)
        v0, v1, k0, k1 = sharding.head_shard(GDN_HV, GDN_HK, world, rank)
        xs = {"q": x["q"][:, :, k0:k1], "k": x["k"][:, :, k0:k1], "v": x["v"][:, :, v0:v1],
              "g": x["g"][:, :, v0:v1], "beta": x["beta"][:, :, v0:v1], "scale": x["scale"]}
        per = ATT_KV // world
        groups = ATT_H // ATT_KV
        a0, a1 = rank * per, (rank + 1) * per
        out = {}
        # NCCL's all-gather, then the copy-engine exchange twice (the second call reuses the
        # mapped buffers of the first)
        for name, transport in (("nccl", "nccl"), ("p2p", "p2p"), ("p2p_again", "p2p")):
            gdn_all, pieces = sharding.hybrid_layer_sharded(xs, qa[:, :, a0 * groups:a1 * groups], ka[:, :, a0:a1],
                                                            va[:, :, a0:a1], WINDOW, 128 ** -0.5, swa_chunks=4,
                                                            transport=transport)
            out[name] = (sharding.assemble_gdn(gdn_all).cpu(), sharding.assemble_heads(pieces, T).cpu())
        if rank == 0:  # the unsharded layer: all heads on this GPU, no exchange
            g1, p1 = sharding.hybrid_layer_sharded(x, qa, ka, va, WINDOW, 128 ** -0.5, swa_chunks=1, gather=False)
            out["gdn_ref"] = sharding.assemble_gdn(g1).cpu()
            out["swa_ref"] = sharding.assemble_heads(p1, T).cpu()
        from pseudobrain_b200._capi import device_error
        out["device_error"] = device_error()
        torch.save(out, os.path.join(outdir, f"nccl_{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm())


def test_hybrid_layer_two_gpus_equals_unsharded(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    ref = torch.load(os.path.join(tmp_path, "nccl_0.pt"))
    hv_loc = GDN_HV // world
    # unsharded GDN [1, T, 8 heads * 128] -> the rank-major [N, T, 4 heads * 128] gather layout
    want_gdn = ref["gdn_ref"].view(T, world, hv_loc * 128).transpose(0, 1)
    want_swa = ref["swa_ref"]
    for rank in range(world):
        got = torch.load(os.path.join(tmp_path, f"nccl_{rank}.pt"))
        assert got["device_error"] == 0
        gdn, swa = got["nccl"]
        eg, es = _rel(gdn, want_gdn), _rel(swa, want_swa)
        print(f"[2-GPU hybrid layer, rank {rank}] rel err GDN {eg:.2e}, attention {es:.2e}")
        assert eg < 2e-2 and es < 2e-2
        for name in ("p2p", "p2p_again"):  # the same kernels' outputs, moved by the copy engines
            assert torch.equal(got[name][0], gdn) and torch.equal(got[name][1], swa), name
