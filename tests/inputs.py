"""Seeded synthetic inputs shared by the parity tests (numpy, deterministic on any host).

Distributions follow benchmark config 0: q, k ~ N(0,1) then L2-normalised per head;
v ~ N(0,1); beta = sigmoid(N(0,1)); g = logsigmoid(N(2,1)); the state ~ N(0, state_std).
bf16 tensors are generated in fp32 and rounded, so the oracle sees exactly the
values the kernel reads.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle.quest import bf16_round


def gdn_inputs(seed: int, batch: int, length: int, hk: int, hv: int, *, dk: int = 128, dv: int = 128,
               bf16: bool = False, g_bf16: bool = False, state_std: float = 0.0) -> dict:
    rng = np.random.default_rng(seed)

    def unit(shape):
        x = rng.standard_normal(shape, dtype=np.float32)
        return (x / np.maximum(np.linalg.norm(x, axis=-1, keepdims=True), 1e-6)).astype(np.float32)

    q, k = unit((batch, length, hk, dk)), unit((batch, length, hk, dk))
    v = rng.standard_normal((batch, length, hv, dv), dtype=np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((batch, length, hv))))).astype(np.float32)
    x = rng.standard_normal((batch, length, hv)) + 2.0
    g = (-np.logaddexp(0.0, -x)).astype(np.float32)  # logsigmoid
    h0 = (rng.standard_normal((batch, hv, dk, dv), dtype=np.float32) * state_std).astype(np.float32)
    if bf16:
        q, k, v, beta = (bf16_round(a) for a in (q, k, v, beta))
    if g_bf16:
        g = bf16_round(g)
    return dict(q=q, k=k, v=v, g=g, beta=beta, h0=h0, scale=dk ** -0.5, bf16=bf16, g_bf16=g_bf16)


def to_device(inp: dict, device) -> dict:
    """Torch tensors on `device`: q/k/v/beta in bf16 when inp['bf16'], g in bf16 when
    inp['g_bf16'], the state fp32."""
    dt = torch.bfloat16 if inp["bf16"] else torch.float32
    out = {n: torch.from_numpy(inp[n]).to(device=device, dtype=dt) for n in ("q", "k", "v", "beta")}
    out["g"] = torch.from_numpy(inp["g"]).to(device=device,
                                             dtype=torch.bfloat16 if inp["g_bf16"] else torch.float32)
    out["h0"] = torch.from_numpy(inp["h0"]).to(device)
    return out
