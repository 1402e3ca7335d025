"""The reference's CPU path for the hot path, restated with torch CPU operations.
TEST AND BASELINE INFRASTRUCTURE ONLY (see oracle/__init__.py).

``bench.py`` times these functions as the CPU baseline and as its ``--impl reference``
arm, and the full-size parity tests use them as the oracle where the numpy restatement
(oracle.gdn, oracle.quest) would take minutes. The reference (pseudobrain/) is plain
PyTorch; its files cannot travel to the GPU host, so this module restates the same
algorithms with the same kinds of torch CPU operations (batched matrix products,
``torch.linalg.solve_triangular``, ``scaled_dot_product_attention``, ``topk``) and so runs
at the reference's speed (a CPU test times the two side by side where the reference is
importable). Every function cites the reference lines it follows; tests/ checks each
against the numpy oracle, which is itself pinned to the reference's golden outputs.

Layouts are the reference's: q, k [B,T,H,K] (already expanded to the value heads, as the
reference's caller does), v [B,T,H,V], g, beta [B,T,H], state [B,H,K,V].
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

CHUNK = 64  # pseudobrain/gated_deltanet.py:48


def use_all_cores() -> int:
    """torch intra-op threads = the host cores this process may run on (reported as
    ``cores``)."""
    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    return n


def _to_heads_first(x: torch.Tensor, dtype) -> torch.Tensor:
    """[B,T,H,*] -> [B,H,T,*] in the compute dtype."""
    return x.to(dtype).transpose(1, 2)


@torch.no_grad()
def chunked_prefill(q, k, v, g, beta, scale: float, h0, chunk: int = CHUNK, head_block: int | None = None):
    """delta_rule_chunked, pseudobrain/gated_deltanet.py:110-165 (fp32; fp64 for fp64 inputs).

    Per chunk of C steps with in-chunk cumulative log decay c:
      A = strict_lower(diag(beta) K K^T o D), D_ti = exp(c_t - c_i);  T = (I + A)^-1;
      W = T diag(beta exp(c)) K;  U' = T diag(beta) V;
    and chunk by chunk: U = U' - W S;  O = diag(exp(c)) Q S + (Q K^T o D) U;
      S <- exp(c_C) S + (diag(exp(c_C - c)) K)^T U.
    A ragged end is padded with identity steps (k = v = 0, g = 0, beta = 0).
    head_block: process this many (batch, head) chains at a time (bounds host memory at full
    size); the chains are independent, so the result does not depend on it.
    Returns (o [B,T,H,V], state [B,H,K,V])."""
    dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    b_, t_, h_, dk = q.shape
    dv = v.shape[-1]
    c_ = min(chunk, t_)
    pad = (-t_) % c_
    n = (t_ + pad) // c_
    qh, kh, vh = (_to_heads_first(x, dt) for x in (q, k, v))
    gh, bh = _to_heads_first(g, dt), _to_heads_first(beta, dt)
    if pad:
        qh, kh, vh = (F.pad(x, (0, 0, 0, pad)) for x in (qh, kh, vh))
        gh, bh = F.pad(gh, (0, pad)), F.pad(bh, (0, pad))
    # chains = (batch, head) pairs, flattened
    qh = qh.reshape(b_ * h_, n, c_, dk) * scale
    kh = kh.reshape(b_ * h_, n, c_, dk)
    vh = vh.reshape(b_ * h_, n, c_, dv)
    cum = gh.reshape(b_ * h_, n, c_).cumsum(-1)
    bh = bh.reshape(b_ * h_, n, c_)
    state = h0.to(dt).reshape(b_ * h_, dk, dv).clone()
    out = torch.empty(b_ * h_, n, c_, dv, dtype=dt)
    lower = torch.ones(c_, c_, dtype=torch.bool).tril()
    strict = torch.ones(c_, c_, dtype=torch.bool).tril(-1)
    eye = torch.eye(c_, dtype=dt)
    step = head_block or b_ * h_
    for lo in range(0, b_ * h_, step):
        sl = slice(lo, min(lo + step, b_ * h_))
        qs, ks, vs, cs, bs = qh[sl], kh[sl], vh[sl], cum[sl], bh[sl]
        dmat = torch.exp((cs[..., :, None] - cs[..., None, :]).masked_fill(~lower, -math.inf))
        amat = ((ks @ ks.transpose(-1, -2)) * dmat * bs[..., :, None]).masked_fill(~strict, 0.0)
        tinv = torch.linalg.solve_triangular(amat + eye, eye.expand_as(amat), upper=False, unitriangular=True)
        gam = torch.exp(cs)
        wmat = tinv @ (ks * (bs * gam)[..., None])
        uprime = tinv @ (vs * bs[..., None])
        qkd = (qs @ ks.transpose(-1, -2)) * dmat
        qgam = qs * gam[..., None]
        ktail = ks * torch.exp(cs[..., -1:] - cs)[..., None]
        glast = gam[..., -1]
        s = state[sl]
        for m in range(n):
            u = uprime[:, m] - wmat[:, m] @ s
            out[sl, m] = qgam[:, m] @ s + qkd[:, m] @ u
            s = s * glast[:, m, None, None] + ktail[:, m].transpose(-1, -2) @ u
        state[sl] = s
    o = out.reshape(b_, h_, n * c_, dv)[:, :, :t_].transpose(1, 2)
    return o, state.reshape(b_, h_, dk, dv)


@torch.no_grad()
def sequential_steps(q, k, v, g, beta, scale: float, h0):
    """delta_rule_sequential, pseudobrain/gated_deltanet.py:93-107 (fp32), the kernel
    select_kernel picks for T <= 4 (:54, :291-294): per step S <- exp(g) S;
    u = (v - S^T k) beta; S <- S + k u^T; o = S^T (scale q). Returns (o, state)."""
    dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    s = h0.to(dt)
    qs, ks, vs = q.to(dt) * scale, k.to(dt), v.to(dt)
    dec, bt = g.to(dt).exp(), beta.to(dt)
    outs = []
    for t in range(q.shape[1]):
        s = s * dec[:, t, :, None, None]
        kt = ks[:, t]
        u = (vs[:, t] - torch.einsum("bhkv,bhk->bhv", s, kt)) * bt[:, t, :, None]
        s = s + kt[..., None] * u[..., None, :]
        outs.append(torch.einsum("bhkv,bhk->bhv", s, qs[:, t]))
    return torch.stack(outs, 1), s


@torch.no_grad()
def page_bounds(keys: torch.Tensor, page: int):
    """_bounds, pseudobrain/exact_memory.py:43-50: elementwise max / min of every page of
    keys [B,KV,N,D] (a partial last page padded with its own last key)."""
    b_, kv, n_, d = keys.shape
    pad = (-n_) % page
    if pad:
        keys = torch.cat((keys, keys[:, :, -1:].expand(b_, kv, pad, d)), dim=2)
    blocks = keys.reshape(b_, kv, -1, page, d)
    return blocks.amax(3), blocks.amin(3)


@torch.no_grad()
def quest_retrieve_attend(q, keys, values, kmax, kmin, n_arch: int, page: int, budget: int, win_keys, win_values,
                          qpos, kpos, window: int, sinks: int = 0):
    """One decode query through the reference's flat Quest path and its attention:
    retrieve (pseudobrain/exact_memory.py:88-152, superblock = rerank = neighbors = 0): page
    score max over the head's rows of pos(q) kmax^T + neg(q) kmin^T (fp32, :94-98,124-125),
    topk (:135), position sort (:144), gather of the pages plus the partial tail (:145-151);
    then SDPA over [retrieved ; window] with the window mask (transplant.py:619-628).
    q [B,H,T,D] (fp32 here, as the CPU reference computes), keys/values [B,KV,n_arch,D],
    bounds [B,KV,P,D], win_keys/values [B,KV,S,D]. Returns ([B,H,T,D], pages [B,KV,k])."""
    b_, h_, t_, d = q.shape
    kv = keys.shape[1]
    groups = h_ // kv
    full = n_arch // page
    qf = q.float().reshape(b_, kv, groups * t_, d)
    pos, neg = qf.clamp(min=0), qf.clamp(max=0)
    score = (pos @ kmax[:, :, :full].float().transpose(-1, -2) + neg @ kmin[:, :, :full].float().transpose(-1, -2))
    score = score.amax(2)                                                   # [B, KV, full]
    top = score.topk(min(budget, full), dim=-1).indices.sort(-1).values
    idx = (top[..., None] * page + torch.arange(page)).reshape(b_, kv, -1)
    rk = torch.gather(keys, 2, idx[..., None].expand(-1, -1, -1, d))
    rv = torch.gather(values, 2, idx[..., None].expand(-1, -1, -1, d))
    if n_arch > full * page:
        rk = torch.cat((rk, keys[:, :, full * page:n_arch]), dim=2)
        rv = torch.cat((rv, values[:, :, full * page:n_arch]), dim=2)
    qp, kp = qpos[:, None], kpos[None, :]
    mask = (kp <= qp) & (((qp - kp) < window) | (kp < sinks))
    mask = torch.cat((torch.ones(t_, rk.shape[2], dtype=torch.bool), mask), dim=1)
    kk = torch.cat((rk, win_keys), dim=2).float().repeat_interleave(groups, dim=1)
    vv = torch.cat((rv, win_values), dim=2).float().repeat_interleave(groups, dim=1)
    return F.scaled_dot_product_attention(q.float(), kk, vv, attn_mask=mask), top


@torch.no_grad()
def window_attention(q, k, v, window: int, sinks: int = 0, chunk: int = 4096):
    """causal_attention's CPU path, pseudobrain/transplant.py:417-436 with its query-chunked
    form :346-362: q [B,H,T,D], k/v [B,KV,T,D] (GQA by repeat); each block of `chunk`
    queries attends to the sinks and the window before it through SDPA with the mask
    s <= t and (t - s < window or s < sinks)."""
    groups = q.shape[1] // k.shape[1]
    if groups > 1:
        k, v = k.repeat_interleave(groups, dim=1), v.repeat_interleave(groups, dim=1)
    t_ = q.shape[2]
    outs = []
    for s0 in range(0, t_, chunk):
        e0 = min(t_, s0 + chunk)
        lo = max(0, s0 - window + 1)
        ns = min(sinks, lo)
        kpos = torch.cat((torch.arange(ns), torch.arange(lo, e0)))
        qp = torch.arange(s0, e0)[:, None]
        mask = (kpos[None, :] <= qp) & (((qp - kpos[None, :]) < window) | (kpos[None, :] < sinks))
        kk = torch.cat((k[:, :, :ns], k[:, :, lo:e0]), dim=2)
        vv = torch.cat((v[:, :, :ns], v[:, :, lo:e0]), dim=2)
        outs.append(F.scaled_dot_product_attention(q[:, :, s0:e0], kk, vv, attn_mask=mask))
    return torch.cat(outs, dim=2)
