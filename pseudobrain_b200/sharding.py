"""(sequence x value-head) sharding of the gated delta rule over the GPUs of one node.

The recurrence of every (sequence, value head) chain is independent
(pseudobrain/gated_deltanet.py:110-165 runs each [b, h] on its own), so a rank can own any
subset of chains with no exchange inside the recurrence. Two layouts:

* batch shard: rank r owns sequences [r B/N, (r+1) B/N) with all heads -- its outputs are
  already in the model's layout; nothing is exchanged (the weak-scaling bench).
* head shard: every rank holds the same tokens and owns value heads
  [r Hv/N, (r+1) Hv/N) with the key heads they read (Hv/N a multiple of the GQA ratio,
  so no key head is split); one all-gather over the process group (NCCL over NVLink on a
  node) restores the [B, T, Hv, V] outputs and [B, Hv, K, V] states.

``prefill`` is the per-rank kernel: pseudobrain_b200.gdn_prefill.gdn_prefill by default.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def batch_shard(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Sequences [b0, b1) of `rank` when `batch` sequences are split over `world` ranks."""
    if batch % world:
        raise ValueError(f"batch {batch} does not split over {world} ranks")
    per = batch // world
    return rank * per, (rank + 1) * per


def head_shard(hv: int, hk: int, world: int, rank: int) -> tuple[int, int, int, int]:
    """(v0, v1, k0, k1): the value heads of `rank` and the key heads they read."""
    if hv % hk or hv % world:
        raise ValueError(f"{hv} value heads do not split over {world} ranks")
    ratio, per = hv // hk, hv // world
    if per % ratio:
        raise ValueError(f"{per} value heads per rank would split a key head shared by {ratio} value heads")
    v0, v1 = rank * per, (rank + 1) * per
    return v0, v1, v0 // ratio, v1 // ratio


def gdn_prefill_head_sharded(q, k, v, g, beta, scale, h0=None, group=None, prefill=None):
    """Chunked gated delta rule with the value heads split over the ranks of `group`.

    Every rank passes the full q, k [B,T,Hk,K], v [B,T,Hv,V], g, beta [B,T,Hv] and h0
    [B,Hv,K,V] (or None); each computes its own heads and the outputs are all-gathered.
    Returns (o [B,T,Hv,V], final state [B,Hv,K,V]) on every rank."""
    if prefill is None:
        from .gdn_prefill import gdn_prefill as prefill
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    b, t, hk, _ = q.shape
    hv = v.shape[2]
    v0, v1, k0, k1 = head_shard(hv, hk, world, rank)
    o_loc, s_loc = prefill(q[:, :, k0:k1], k[:, :, k0:k1], v[:, :, v0:v1], g[:, :, v0:v1], beta[:, :, v0:v1], scale,
                           None if h0 is None else h0[:, v0:v1])
    # rank blocks concatenated along dim 0 (the layout every backend accepts), then viewed
    # as [N, ...]
    o_all = torch.empty((world * o_loc.shape[0],) + tuple(o_loc.shape[1:]), dtype=o_loc.dtype, device=o_loc.device)
    s_all = torch.empty((world * s_loc.shape[0],) + tuple(s_loc.shape[1:]), dtype=s_loc.dtype, device=s_loc.device)
    dist.all_gather_into_tensor(o_all, o_loc.contiguous(), group=group)
    dist.all_gather_into_tensor(s_all, s_loc.contiguous(), group=group)
    o_all = o_all.view((world,) + tuple(o_loc.shape))
    s_all = s_all.view((world,) + tuple(s_loc.shape))
    # [N, B, T, Hv/N, V] -> [B, T, Hv, V];  [N, B, Hv/N, K, V] -> [B, Hv, K, V]
    o = o_all.permute(1, 2, 0, 3, 4).reshape(b, t, hv, o_loc.shape[-1])
    s = s_all.permute(1, 0, 2, 3, 4).reshape(b, hv, s_loc.shape[-2], s_loc.shape[-1])
    return o, s


def gdn_prefill_batch_sharded(q, k, v, g, beta, scale, h0=None, group=None, prefill=None):
    """Chunked gated delta rule on this rank's sequences only (no exchange): returns the
    (o, state) of sequences batch_shard(B, world, rank)."""
    if prefill is None:
        from .gdn_prefill import gdn_prefill as prefill
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    b0, b1 = batch_shard(q.shape[0], world, rank)
    return prefill(q[b0:b1], k[b0:b1], v[b0:b1], g[b0:b1], beta[b0:b1], scale,
                   None if h0 is None else h0[b0:b1])


def causal_attention_head_sharded(q, k, v, window=None, sinks=0, group=None, attention=None):
    """Sliding-window attention (transplant.py:417-436 semantics) with the key heads split
    over the ranks of `group`: rank r computes key heads [r KV/N, (r+1) KV/N) and the query
    heads that read them, then one all-gather restores [B,H,T,hd] on every rank.

    q [B,H,T,hd], k/v [B,KV,T,hd] (the full tensors on every rank). ``attention`` is the
    per-rank function, pseudobrain_b200.transplant.causal_attention by default."""
    if attention is None:
        from .transplant import causal_attention as attention
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    b, h, t, d = q.shape
    kvh = k.shape[1]
    if kvh % world:
        raise ValueError(f"{kvh} key heads do not split over {world} ranks")
    per = kvh // world
    groups = h // kvh
    k0, k1 = rank * per, (rank + 1) * per
    o_loc = attention(q[:, k0 * groups:k1 * groups], k[:, k0:k1], v[:, k0:k1], window, sinks)
    o_all = torch.empty((world * b,) + tuple(o_loc.shape[1:]), dtype=o_loc.dtype, device=o_loc.device)
    dist.all_gather_into_tensor(o_all, o_loc.contiguous(), group=group)
    # [N, B, H/N, T, hd] -> [B, H, T, hd]
    return o_all.view((world,) + tuple(o_loc.shape)).transpose(0, 1).reshape(b, h, t, d)


# ------------------------------------------------------------------------------------------
# The hybrid layer (benchmark config 4) split over the ranks, with its all-gathers overlapped
# ------------------------------------------------------------------------------------------
def swa_chunk_plan(t: int, window: int, chunks: int, first: int | None = None) -> list[tuple[int, int, int]]:
    """Query chunks [s, e) of a T-token sliding-window pass, each with the halo h of earlier
    rows its queries read (s - h >= 0, h >= window - 1 unless the chunk starts earlier): the
    rows [s - h, e) then form a self-contained window-attention problem whose last e - s rows
    are exact. The first chunk is `first` rows (default T / (2 chunks)), so its output is
    ready -- and its all-gather can start -- early; the rest split evenly. Row counts are
    multiples of 128 (the attention kernel's query tile) except at T."""
    if t <= 0:
        return []
    chunks = max(1, chunks)
    first = first if first is not None else max(128, t // (2 * chunks))
    first = min(t, -(-first // 128) * 128)
    bounds = [0, first]
    rest = t - first
    if rest > 0:
        n = max(1, chunks - 1)
        step = -(-(-(-rest // n)) // 128) * 128
        s = first
        while s < t:
            s = min(t, s + step)
            bounds.append(s)
    halo = -(-(window - 1) // 128) * 128 if window > 0 else None
    plan = []
    for s, e in zip(bounds[:-1], bounds[1:]):
        h = s if halo is None else min(s, halo)
        plan.append((s, e, h))
    return plan


class PeerExchange:
    """Rank-major gather buffers on every rank of `group`, filled by copy-engine pushes.

    One bf16 buffer holds, for each piece i of shape (rows_i, width_i), a [N, rows_i, width_i]
    region; rank r's data goes to slot r of every rank's region. The buffer is exported once
    with CUDA IPC (pbk_ipc_handle) and mapped by every other rank (pbk_ipc_open); ``push``
    copies a finished piece from this rank's own slot into the same slot of every peer's buffer
    with one cudaMemcpyAsync per peer, on one stream per peer after an event on the producing
    stream. The copies run on the copy engines over NVLink and use no SMs, so they overlap
    kernels that fill every SM (NCCL's all-gather kernels wait for free SMs). ``start`` and
    ``finish`` are the only collectives: a one-element all-reduce each, so that no rank writes
    into a peer's buffer before the peer's earlier work is done, and no rank reads its buffer
    before every peer's pushes into it have landed. The buffer must come from cudaMalloc (the
    caching allocator's default segments): CUDA IPC cannot export expandable segments, and
    pbk_ipc_handle then fails with an error."""

    def __init__(self, group, pieces: list[tuple[int, int]], device: torch.device):
        from ._capi import LIB, PBK_IPC_HANDLE_BYTES, check
        import ctypes
        self.group, self.device = group, device
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.pieces = list(pieces)
        self.offsets, total = [], 0
        for rows, width in self.pieces:
            self.offsets.append(total)
            total += self.world * rows * width
        self.buf = torch.empty(max(total, 1), dtype=torch.bfloat16, device=device)
        handle = (ctypes.c_uint8 * PBK_IPC_HANDLE_BYTES)()
        off = ctypes.c_int64()
        with torch.cuda.device(device):
            check(LIB.pbk_ipc_handle(self.buf.data_ptr(), handle, ctypes.byref(off)), "pbk_ipc_handle")
        mine = (bytes(handle), off.value)
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=group)
        self.bases, self.peer_ptr = {}, {}
        for p in range(self.world):
            if p == self.rank:
                continue
            base = ctypes.c_void_p()
            h = (ctypes.c_uint8 * PBK_IPC_HANDLE_BYTES).from_buffer_copy(every[p][0])
            with torch.cuda.device(device):
                check(LIB.pbk_ipc_open(h, ctypes.byref(base)), "pbk_ipc_open")
            self.bases[p] = base.value
            self.peer_ptr[p] = base.value + every[p][1]
        self.streams = {p: torch.cuda.Stream(device) for p in self.peer_ptr}
        self.flag = torch.zeros(1, dtype=torch.float32, device=device)
        self._lib = LIB

    def view(self, i: int) -> torch.Tensor:
        """Piece i's region of this rank's buffer, [N, rows, width]."""
        rows, width = self.pieces[i]
        o = self.offsets[i]
        return self.buf[o:o + self.world * rows * width].view(self.world, rows, width)

    def own(self, i: int) -> torch.Tensor:
        """This rank's slot of piece i, [rows, width] (contiguous)."""
        return self.view(i)[self.rank]

    def start(self) -> None:
        dist.all_reduce(self.flag, group=self.group)

    def push(self, i: int) -> None:
        """Copy this rank's slot of piece i (written on the current stream) to every peer."""
        from ._capi import check
        rows, width = self.pieces[i]
        nbytes = rows * width * 2
        elem = self.offsets[i] + self.rank * rows * width
        src = self.buf.data_ptr() + elem * 2
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        for p, st in self.streams.items():
            st.wait_event(ev)
            check(self._lib.pbk_copy_async(self.peer_ptr[p] + elem * 2, src, nbytes, st.cuda_stream), "pbk_copy_async")

    def finish(self) -> None:
        cur = torch.cuda.current_stream(self.device)
        for st in self.streams.values():
            cur.wait_stream(st)
        dist.all_reduce(self.flag, group=self.group)

    def close(self) -> None:
        """Unmap the peers' buffers (after every push has completed)."""
        torch.cuda.synchronize(self.device)
        for base in self.bases.values():
            self._lib.pbk_ipc_close(base)
        self.bases.clear()
        self.peer_ptr.clear()


_EXCHANGES: dict = {}


def peer_exchange(group, pieces, device) -> PeerExchange:
    """The PeerExchange of these piece shapes on `group` (created on first use; every rank
    must ask for the same shapes in the same order)."""
    key = (id(group), tuple(pieces), str(device))
    ex = _EXCHANGES.get(key)
    if ex is None:
        ex = _EXCHANGES[key] = PeerExchange(group, pieces, device)
    return ex


# Above this many ranks the copy engines' egress (about 330 GB/s per B200 measured, pushing
# to 7 peers) is slower than NCCL's SM-driven all-gather (about 660 GB/s), even though NCCL's
# kernels wait for SMs the attention holds.
P2P_MAX_RANKS = 4


def default_transport(world: int, is_cuda: bool, group=None) -> str:
    """"p2p" (copy-engine pushes) for 2..P2P_MAX_RANKS ranks of an NCCL group on CUDA
    tensors, else "nccl"."""
    if world > 1 and world <= P2P_MAX_RANKS and is_cuda and dist.get_backend(group) == "nccl":
        return "p2p"
    return "nccl"


def hybrid_layer_sharded(gdn_in: dict, qa, ka, va, window: int, attn_scale: float, group=None, swa_chunks: int = 8,
                         gdn=None, attention=None, gather: bool = True, gdn_parts: int | None = None,
                         transport: str | None = None):
    """One hybrid layer (GDN branch + sliding-window attention branch, pseudobrain/transplant.py
    WindowedHybridLayer, benchmark config 4) on this rank's heads, with every branch output
    all-gathered over `group` into the head-major layout the output projection reads.

    gdn_in: this rank's GDN shard {q, k [1,T,hk/N,128], v [1,T,hv/N,128], g, beta [1,T,hv/N],
    scale}; qa [1,T,H/N,128], ka, va [1,T,KV/N,128]: this rank's attention heads (window sinks
    0). Order, chosen so the all-gathers (bound by each GPU's NVLink ingress) start early and
    run under the compute: the GDN branch (segmented over T) first, in `gdn_parts` launches over
    consecutive groups of whole key heads (default 2 when N > 1 and the rank's key heads split
    evenly, else 1), each part's output gathered on the communicator's stream while the next
    part and then the attention run; then the attention in query chunks (swa_chunk_plan), each
    chunk's rows gathered as soon as they are written, while the next chunk computes. Only the
    last chunk's gather is left after the compute. Returns ([(v0, v1, gdn_part [N, T,
    (v1 - v0)*128]) for each part: the rank-local value heads [v0, v1)], [(s, e, swa_all [N,
    e - s, H/N*128]) for each chunk]); assemble_gdn joins the parts into [N, T, hv/N*128].
    ``gdn(gdn_in, o)`` and ``attention(q, k, v, o, window, scale)`` replace the CUDA kernels (CPU
    tests); gather=False runs the layer on these heads alone (N = 1 layouts, no exchange).
    transport: "p2p" gathers with copy-engine pushes into every rank's mapped buffers
    (PeerExchange): each piece goes out as soon as it is written, without SMs, so the pushes
    overlap the attention kernel; "nccl" uses all_gather_into_tensor on the communicator's
    stream. The default (default_transport) is "p2p" on NCCL groups of up to P2P_MAX_RANKS. The returned buffers of the p2p
    transport are reused by the next call of the same shapes."""
    world = dist.get_world_size(group) if (gather and dist.is_initialized()) else 1
    if gdn is None:
        from .gdn_prefill import auto_segments, gdn_prefill_segmented

        def gdn(x, o):
            segs = auto_segments(1, x["v"].shape[2], x["q"].shape[1])
            gdn_prefill_segmented(x["q"], x["k"], x["v"], x["g"], x["beta"], x["scale"], None, segments=segs, o=o)
    if attention is None:
        from .transplant import window_attention_

        def attention(q, k, v, o, win, scale):
            window_attention_(q, k, v, o, win, 0, scale)
    t = qa.shape[1]
    heads, d = qa.shape[2], qa.shape[3]
    works, swa_out, gdn_out = [], [], []
    hv, hk, dv = gdn_in["v"].shape[2], gdn_in["k"].shape[2], gdn_in["v"].shape[3]
    if gdn_parts is None:
        gdn_parts = 2 if world > 1 and hk % 2 == 0 else 1
    if gdn_parts < 1 or hk % gdn_parts:
        raise ValueError(f"{hk} key heads do not split into {gdn_parts} parts")
    ratio = hv // hk
    plan = swa_chunk_plan(t, window, swa_chunks)
    if transport is None:
        transport = default_transport(world, qa.is_cuda, group)
    ex = None
    if world > 1 and transport == "p2p":
        pieces = [(t, ((p + 1) * hk // gdn_parts - p * hk // gdn_parts) * ratio * dv) for p in range(gdn_parts)]
        pieces += [(e - s, heads * d) for s, e, _ in plan]
        ex = peer_exchange(group, pieces, qa.device)
        ex.start()
    elif transport not in ("p2p", "nccl"):
        raise ValueError(f"transport must be 'p2p' or 'nccl', not {transport!r}")
    for part in range(gdn_parts):
        k0, k1 = part * hk // gdn_parts, (part + 1) * hk // gdn_parts
        v0, v1 = k0 * ratio, k1 * ratio
        x = {"q": gdn_in["q"][:, :, k0:k1], "k": gdn_in["k"][:, :, k0:k1], "v": gdn_in["v"][:, :, v0:v1],
             "g": gdn_in["g"][:, :, v0:v1], "beta": gdn_in["beta"][:, :, v0:v1], "scale": gdn_in["scale"]}
        if ex is not None:  # written straight into this rank's slot, then pushed to the peers
            gdn(x, ex.own(part).view(1, t, v1 - v0, dv))
            ex.push(part)
            gdn_out.append((v0, v1, ex.view(part)))
            continue
        o_part = torch.empty(1, t, v1 - v0, dv, dtype=torch.bfloat16, device=qa.device)
        gdn(x, o_part)
        if world > 1:
            gathered = torch.empty(world * t, (v1 - v0) * dv, dtype=o_part.dtype, device=o_part.device)
            works.append(dist.all_gather_into_tensor(gathered, o_part.view(t, -1), group=group, async_op=True))
            gdn_out.append((v0, v1, gathered.view(world, t, -1)))
        else:
            gdn_out.append((v0, v1, o_part.view(1, t, -1)))
    for ci, (s, e, h) in enumerate(plan):
        rows = e - s + h
        stage = torch.empty(1, rows, heads, d, dtype=qa.dtype, device=qa.device)
        attention(qa[:, s - h:e], ka[:, s - h:e], va[:, s - h:e], stage, window, attn_scale)
        mine = stage.view(rows, heads * d)[h:]  # this chunk's exact rows (contiguous)
        if ex is not None:
            ex.own(gdn_parts + ci).copy_(mine)
            ex.push(gdn_parts + ci)
            swa_out.append((s, e, ex.view(gdn_parts + ci)))
            continue
        if world > 1:
            gathered = torch.empty(world * (e - s), heads * d, dtype=qa.dtype, device=qa.device)
            works.append(dist.all_gather_into_tensor(gathered, mine, group=group, async_op=True))
            swa_out.append((s, e, gathered.view(world, e - s, heads * d)))
        else:
            swa_out.append((s, e, mine.view(1, e - s, heads * d)))
    for w in works:
        w.wait()
    if ex is not None:
        ex.finish()
    return gdn_out, swa_out


def assemble_gdn(parts) -> torch.Tensor:
    """[(v0, v1, [N, T, (v1 - v0) * V])...] in head order -> [N, T, (heads per rank) * V]: the
    gathered GDN parts joined along each rank's heads (the layout of one gather of all of them)."""
    return torch.cat([x for _, _, x in parts], dim=-1)


def assemble_heads(pieces, t: int) -> torch.Tensor:
    """[(s, e, [N, e - s, W])...] -> [T, N * W]: the gathered attention chunks in the hidden
    layout (token-major, rank-major heads)."""
    n, _, w = pieces[0][2].shape
    out = torch.empty(t, n * w, dtype=pieces[0][2].dtype, device=pieces[0][2].device)
    for s, e, x in pieces:
        out[s:e] = x.permute(1, 0, 2).reshape(e - s, n * w)
    return out
