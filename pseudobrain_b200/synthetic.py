"""Seeded synthetic inputs of the benchmark configurations, generated on the device.

No public dataset is involved: every configuration is defined by shapes and value
distributions (config 0 distributions: q, k ~ N(0,1) L2-normalised per head; v ~ N(0,1);
beta = sigmoid(N(0,1)); g = logsigmoid(N(2,1))).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .exact_memory import page_bounds_


def gdn_inputs(batch: int, length: int, hk: int, hv: int, *, device, seed: int, dtype=torch.bfloat16,
               g_dtype=torch.float32, dk: int = 128, dv: int = 128, state_std: float = 0.0) -> dict:
    gen = torch.Generator(device=device).manual_seed(seed)
    q = F.normalize(torch.randn(batch, length, hk, dk, device=device, generator=gen), dim=-1).to(dtype)
    k = F.normalize(torch.randn(batch, length, hk, dk, device=device, generator=gen), dim=-1).to(dtype)
    v = torch.randn(batch, length, hv, dv, device=device, generator=gen, dtype=dtype)
    beta = torch.sigmoid(torch.randn(batch, length, hv, device=device, generator=gen)).to(dtype)
    g = F.logsigmoid(torch.randn(batch, length, hv, device=device, generator=gen) + 2.0).to(g_dtype)
    h0 = torch.randn(batch, hv, dk, dv, device=device, generator=gen) * state_std if state_std else \
        torch.zeros(batch, hv, dk, dv, device=device)
    return dict(q=q, k=k, v=v, g=g, beta=beta, h0=h0, scale=dk ** -0.5)


def quest_inputs(*, device, seed: int = 3, n_tokens: int = 1 << 20, kv: int = 8, heads: int = 32, d: int = 128,
                 page: int = 16, window: int = 4096, nq: int = 8, budget_tokens: int = 4096,
                 planted_scale: float = 45.0) -> dict:
    """benchmark config 3: a bf16 KV cache of n_tokens (K, V ~ N(0,1)); the last `window`
    positions are the window, the rest is the archive with precomputed page bounds. nq
    single-token queries q ~ N(0,1) at position n_tokens - 1. For query i one seeded archive
    page p_i holds, in every key head g, 16 copies of bf16(planted_scale * unit mean of the
    group's query heads), so it must be selected."""
    gen = torch.Generator(device=device).manual_seed(seed)
    keys = torch.randn(kv, n_tokens, d, device=device, generator=gen, dtype=torch.bfloat16)
    values = torch.randn(kv, n_tokens, d, device=device, generator=gen, dtype=torch.bfloat16)
    q = torch.randn(nq, 1, heads, d, device=device, generator=gen, dtype=torch.bfloat16)
    n_arch = n_tokens - window
    npages = n_arch // page
    groups = heads // kv
    planted = torch.randperm(npages, device=device, generator=gen)[:nq]
    for i in range(nq):
        qhat = F.normalize(q[i, 0].float().view(kv, groups, d).mean(1), dim=-1)  # [kv, d]
        keys[:, planted[i] * page:(planted[i] + 1) * page] = (planted_scale * qhat).to(torch.bfloat16)[:, None]
    kmax = torch.empty(kv, npages, d, device=device, dtype=torch.bfloat16)
    kmin = torch.empty_like(kmax)
    page_bounds_(keys[:, :n_arch], page, kmax, kmin)
    return dict(keys=keys, values=values, q=q, kmax=kmax, kmin=kmin, n_arch=n_arch, page=page,
                budget=budget_tokens // page, window=window, planted=planted,
                qpos=torch.full((nq, 1), n_tokens - 1, dtype=torch.int32, device=device),
                kpos=torch.arange(n_arch, n_tokens, dtype=torch.int32, device=device),
                win_keys=keys[:, n_arch:], win_values=values[:, n_arch:])
