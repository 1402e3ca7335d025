"""Benchmark of the PseudoBrain hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload all|prefill|decode|quest|hybrid|serving|widen] [--size full|small]

Headline (``value``): GDN chunked prefill of benchmark config 1 (B=4, T=32768, 16 key /
32 value heads, dk=dv=128, chunk 64, bf16 q/k/v/beta, fp32 g and state) in tok/s,
inputs resident in HBM, device-timed with CUDA events, max over ranks. The same line
carries the other two parts of the metric, each with its own roofline:
``decode`` (config 2: B=256 decode step, 537 MB fp32 state, steps/s), ``quest``
(config 3: 8 queries over a 1M-token cache, q/s) and ``hybrid`` (config 4: one GDN +
sliding-window attention layer over a 1M-token sequence, heads split over the ranks with
an NCCL all-gather of each branch's output; tok/s, strong scaling). ``e2e`` times the public API with
pinned host inputs copied in and outputs copied back inside the timed region: streamed (prefill
by sequence, decode by step) so that the copies in, the kernels and the copies out overlap,
with the one-stream figure beside it as ``serial_value``.

``widen`` times the rows around the hot path (the GDN layer's conv / gating / output norm at
config-1 shapes, the two-level Quest selection, the serving archive write and the RoPE move
+ gather), each against the HBM roofline.

Multi-GPU (torchrun, one rank per GPU): weak scaling. Every rank runs its own shard of
(sequence x value head) chains of the same per-GPU size; the recurrence has no
exchange step, so there is no collective inside the timed region.

``serving`` times the serving twins at PB-27's attention shape (head dim 256; the head-dim-128
figures beside them) and the per-token selector's decode selection.

``--impl reference`` times the CPU restatement of the reference algorithm
(oracle/cpu_reference.py: the reference's own torch CPU operations, all host cores) on
bounded samples of the same workload and prints the same metric; under torchrun only rank 0
runs it. ``--workload``/``--size small`` run one part
on a reduced case, for profiler captures only (such a line is not a bench number).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GDN prefill tok/s & decode steps/s per B200; Quest q/s; % TC/HBM roofline"
PREFILL = {"full": dict(batch=4, seqlen=32768), "small": dict(batch=4, seqlen=8192)}
PREFILL_HEADS = dict(hk=16, hv=32, dk=128, dv=128, chunk=64)
DECODE = {"full": dict(batch=256), "small": dict(batch=64)}
DECODE_HEADS = dict(hk=16, hv=32, dk=128, dv=128)
QUEST = {"full": dict(n_tokens=1 << 20), "small": dict(n_tokens=1 << 19)}
HYBRID = {"full": dict(seqlen=1 << 20), "small": dict(seqlen=1 << 16)}
HYBRID_HEADS = dict(hk=16, hv=32, heads=32, kv=8, d=128, window=4096)
QUEST_SHAPE = dict(kv=8, heads=32, d=128, page=16, window=4096, nq=8, budget_tokens=4096)


PREFILL_KERNELS = ("gdn_solve_kernel", "gdn_prefill_tc_kernel")  # the kernels of one prefill step


def prefill_flops_per_token_head(c=64, d=128):
    """5 C x C x d products (KK^T, QK^T, W, U', (QK*D)U) + 3 d x d products per token
    (WS, QS, K^T U) + the triangular inverse (C^2/3 per token)."""
    return 5 * 2 * c * d + 3 * 2 * d * d + 2 * c * c / 3


def solve_flops_per_token_head(c=64, d=128):
    """The chunk solve kernel's share: K K^T and the triangular inverse; the recurrence
    kernel does the other 4 C x C x d and 3 d x d products."""
    return 2 * c * d + 2 * c * c / 3


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return dict(hbm=p["hbm_gbs"], tc=p["bf16_tflops"], tc_sustained=p["bf16_tflops_sustained"], src="measured")
    return dict(hbm=6650.0, tc=1590.0, tc_sustained=1400.0, src="fallback")


def traffic(kernel_key):
    """DRAM bytes per launch of the bench workload from the committed ncu summary
    (profiles/traffic.txt: `<kernel> <bytes per launch>` lines), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel_key:
            return float(parts[1])
    return None


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------------------------
class Timer:
    """Device time of K calls after W warm-ups, bracketed by barrier + synchronize on both
    sides, CUDA events on the launching stream, max over ranks."""

    def __init__(self, torch, dist, dev, world):
        self.torch, self.dist, self.dev, self.world = torch, dist, dev, world

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, x):
        if self.world == 1:
            return x
        t = self.torch.tensor([x], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def __call__(self, fn, steps, warmup):
        torch = self.torch
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        s = torch.cuda.current_stream(self.dev)
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record(s)
        for _ in range(steps):
            fn()
        en.record(s)
        torch.cuda.synchronize()
        self.barrier()
        return self.max_over_ranks(st.elapsed_time(en) / 1e3)


def timed_streams(timed, fn, steps, warmup, first, others):
    """Device time of K calls of a step that spreads its work over several streams: the start
    event on `first` (the stream each step's first work goes to), the end event on the current
    stream after it has waited for `first` and every stream in `others`; barrier + synchronize
    on both sides, max over ranks."""
    torch = timed.torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    timed.barrier()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record(first)
    for _ in range(steps):
        fn()
    cur = torch.cuda.current_stream(timed.dev)
    for s in (first, *others):
        cur.wait_stream(s)
    en.record(cur)
    torch.cuda.synchronize()
    timed.barrier()
    return timed.max_over_ranks(st.elapsed_time(en) / 1e3)


def measure_prefill(args, timed, dev, rank, world, pk):
    import torch
    from pseudobrain_b200.gdn_prefill import chunk_solve, gdn_prefill_, prefill_solved
    from pseudobrain_b200.synthetic import gdn_inputs
    P = {**PREFILL[args.size], **PREFILL_HEADS}
    x = gdn_inputs(P["batch"], P["seqlen"], P["hk"], P["hv"], device=dev, seed=1 + 1000 * rank)
    state = torch.empty(P["batch"], P["hv"], P["dk"], P["dv"], device=dev)
    o = torch.empty(P["batch"], P["seqlen"], P["hv"], P["dv"], device=dev, dtype=torch.bfloat16)

    def step():
        gdn_prefill_(x["q"], x["k"], x["v"], x["g"], x["beta"], None, state, o, x["scale"])

    t = timed(step, args.steps, args.warmup)
    tokens = P["batch"] * P["seqlen"]
    per_step = t / args.steps
    flops = tokens * P["hv"] * prefill_flops_per_token_head(P["chunk"], P["dk"])
    solve_flops = tokens * P["hv"] * solve_flops_per_token_head(P["chunk"], P["dk"])
    algo_bytes = (2 * tokens * P["hk"] * P["dk"] * 2 + tokens * P["hv"] * P["dv"] * 2 * 2 + tokens * P["hv"] * 6
                  + 2 * P["batch"] * P["hv"] * P["dk"] * P["dv"] * 4)
    # the step's two kernels timed apart (CUDA events on the launching stream around each
    # launch, summed over K steps): the roofline is the recurrence kernel's, the dominant one
    ws = chunk_solve(x["q"], x["k"], x["v"], x["g"], x["beta"], state, x["scale"])
    cur = torch.cuda.current_stream(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    for _ in range(args.warmup):
        chunk_solve(x["q"], x["k"], x["v"], x["g"], x["beta"], state, x["scale"], ws)
        prefill_solved(x["q"], x["k"], x["v"], x["g"], x["beta"], None, state, o, x["scale"], ws)
    torch.cuda.synchronize()
    for e in evs:
        e[0].record(cur)
        chunk_solve(x["q"], x["k"], x["v"], x["g"], x["beta"], state, x["scale"], ws)
        e[1].record(cur)
        prefill_solved(x["q"], x["k"], x["v"], x["g"], x["beta"], None, state, o, x["scale"], ws)
        e[2].record(cur)
    torch.cuda.synchronize()
    t_solve = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps / 1e3
    t_rec = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps / 1e3
    del ws
    achieved = (flops - solve_flops) / t_rec / 1e12
    tr_parts = [traffic(kn) for kn in PREFILL_KERNELS]
    step_traffic = sum(tr_parts) if all(x is not None for x in tr_parts) else None
    # e2e through the public API: pinned host inputs in, bf16 outputs back, every step
    host = {n: x[n].cpu().pin_memory() for n in ("q", "k", "v", "g", "beta")}
    dev_in = {n: torch.empty_like(x[n]) for n in host}
    host_o = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)

    def e2e_serial():
        for n, tt in host.items():
            dev_in[n].copy_(tt, non_blocking=True)
        gdn_prefill_(dev_in["q"], dev_in["k"], dev_in["v"], dev_in["g"], dev_in["beta"], None, state, o, x["scale"])
        host_o.copy_(o, non_blocking=True)

    # The same step streamed by sequence: sequence b's inputs go up on a copy stream while
    # sequence b-1 computes, and its output comes back on a second copy stream (PCIe is full
    # duplex) while sequence b+1's inputs go up. Every step still copies all its inputs and
    # reads back all its outputs.
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_comp = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
    nb = P["batch"]
    ev_in, ev_comp, ev_out = ([torch.cuda.Event() for _ in range(nb)] for _ in range(3))
    started = [False]

    def e2e_streamed():
        for bb in range(nb):
            with torch.cuda.stream(s_in):
                if started[0]:
                    s_in.wait_event(ev_comp[bb])  # the previous step's sequence bb has read its inputs
                for n, tt in host.items():
                    dev_in[n][bb].copy_(tt[bb], non_blocking=True)
                ev_in[bb].record(s_in)
            sc = s_comp[bb % 2]
            sc.wait_event(ev_in[bb])
            if started[0]:
                sc.wait_event(ev_out[bb])  # the previous step's output of sequence bb is back
            with torch.cuda.stream(sc):
                sl = slice(bb, bb + 1)
                gdn_prefill_(dev_in["q"][sl], dev_in["k"][sl], dev_in["v"][sl], dev_in["g"][sl], dev_in["beta"][sl],
                             None, state[sl], o[sl], x["scale"])
                ev_comp[bb].record(sc)
            s_out.wait_event(ev_comp[bb])
            with torch.cuda.stream(s_out):
                host_o[bb].copy_(o[bb], non_blocking=True)
                ev_out[bb].record(s_out)
        started[0] = True

    e2e_steps = max(3, args.steps // 2)
    t_e2e_serial = timed(e2e_serial, e2e_steps, min(args.warmup, 3))
    t_e2e = timed_streams(timed, e2e_streamed, e2e_steps, min(args.warmup, 3), s_in, [s_out, *s_comp])
    return {
        "value": world * tokens * args.steps / t, "unit": "tok/s", "ms_per_step": per_step * 1e3,
        "tokens": tokens,
        # the kernel is timed alone over regions of tens of ms: the burst tensor peak applies
        "roofline": {"bound": "tensor", "kernel": "gdn_prefill_tc_kernel", "achieved": achieved,
                     "peak": pk["tc"], "unit": "TFLOP/s", "frac": achieved / pk["tc"],
                     "traffic": traffic("gdn_prefill_tc_kernel"), "peak_source": f"{pk['src']} bf16 burst",
                     "algorithmic_flops": flops - solve_flops, "ms": t_rec * 1e3},
        "kernels": {"gdn_solve_kernel": {"ms": t_solve * 1e3, "tflops": solve_flops / t_solve / 1e12,
                                         "traffic": traffic("gdn_solve_kernel")},
                    "gdn_prefill_tc_kernel": {"ms": t_rec * 1e3, "tflops": (flops - solve_flops) / t_rec / 1e12}},
        "step": {"tflops": flops / per_step / 1e12, "frac": flops / per_step / 1e12 / pk["tc"],
                 "algorithmic_bytes": algo_bytes, "hbm_frac": algo_bytes / per_step / 1e9 / pk["hbm"],
                 "traffic": step_traffic,
                 "traffic_over_algorithmic": step_traffic / algo_bytes if step_traffic else None},
        "e2e": {"value": world * tokens * e2e_steps / t_e2e, "unit": "tok/s",
                "h2d_bytes_per_step": sum(tt.numel() * tt.element_size() for tt in host.values()),
                "d2h_bytes_per_step": host_o.numel() * host_o.element_size(),
                "copies": f"streamed by sequence ({nb} slices): input copies, compute and output copies overlap",
                "serial_value": world * tokens * e2e_steps / t_e2e_serial},
        "gpu_launches": 2 * args.steps,  # chunk solve + recurrence
    }


def measure_decode(args, timed, dev, rank, world, pk):
    import torch
    from pseudobrain_b200 import gated_deltanet as G
    from pseudobrain_b200.synthetic import gdn_inputs
    D = {**DECODE[args.size], **DECODE_HEADS}
    xd = gdn_inputs(D["batch"], 1, D["hk"], D["hv"], device=dev, seed=2 + 1000 * rank, g_dtype=torch.bfloat16,
                    state_std=0.02)
    od = torch.empty(D["batch"], 1, D["hv"], D["dv"], device=dev, dtype=torch.bfloat16)

    def step():
        G.gdn_recurrent_(xd["q"], xd["k"], xd["v"], xd["g"], xd["beta"], None, xd["h0"], od, xd["scale"])

    nsteps = 1000 if args.size == "full" else 20  # config 2: 1000 sequential in-place steps
    t = timed(step, nsteps, max(args.warmup, 10))
    per_step = t / nsteps
    nbytes = 2 * xd["h0"].numel() * 4 + sum(xd[n].numel() * xd[n].element_size()
                                            for n in ("q", "k", "v", "g", "beta")) + od.numel() * 2
    host = {n: xd[n].cpu().pin_memory() for n in ("q", "k", "v", "g", "beta")}
    dev_in = {n: torch.empty_like(xd[n]) for n in host}
    host_o = torch.empty(od.shape, dtype=od.dtype, pin_memory=True)

    def e2e_serial():
        for n, tt in host.items():
            dev_in[n].copy_(tt, non_blocking=True)
        G.gdn_recurrent_(dev_in["q"], dev_in["k"], dev_in["v"], dev_in["g"], dev_in["beta"], None, xd["h0"], od,
                         xd["scale"])
        host_o.copy_(od, non_blocking=True)

    # Streamed: step i+1's inputs go up (into the other of two input slots) while step i
    # computes, and step i's output comes back while step i+1 computes; the steps themselves
    # stay in order on one stream (each updates the state in place).
    s_in, s_c, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    slots = [dev_in, {n: torch.empty_like(xd[n]) for n in host}]
    outs = [od, torch.empty_like(od)]
    host_os = [host_o, torch.empty(od.shape, dtype=od.dtype, pin_memory=True)]
    ev_in, ev_comp, ev_out = ([torch.cuda.Event(), torch.cuda.Event()] for _ in range(3))
    it = [0]

    def e2e_streamed():
        i = it[0]
        sl = i & 1
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_comp[sl])  # step i-2 has read this input slot
            for n, tt in host.items():
                slots[sl][n].copy_(tt, non_blocking=True)
            ev_in[sl].record(s_in)
        s_c.wait_event(ev_in[sl])
        if i >= 2:
            s_c.wait_event(ev_out[sl])  # step i-2's output is back on the host
        with torch.cuda.stream(s_c):
            d = slots[sl]
            G.gdn_recurrent_(d["q"], d["k"], d["v"], d["g"], d["beta"], None, xd["h0"], outs[sl], xd["scale"])
            ev_comp[sl].record(s_c)
        s_out.wait_event(ev_comp[sl])
        with torch.cuda.stream(s_out):
            host_os[sl].copy_(outs[sl], non_blocking=True)
            ev_out[sl].record(s_out)
        it[0] = i + 1

    t_e2e_serial = timed(e2e_serial, 200, 10)
    t_e2e = timed_streams(timed, e2e_streamed, 200, 10, s_in, [s_c, s_out])
    return {
        "metric": "GDN decode steps/s (config 2)", "value": world * nsteps / t, "unit": "steps/s",
        "us_per_step": per_step * 1e6,
        "roofline": {"bound": "hbm", "achieved": nbytes / per_step / 1e9, "peak": pk["hbm"], "unit": "GB/s",
                     "frac": nbytes / per_step / 1e9 / pk["hbm"], "traffic": traffic("gdn_decode_kernel"),
                     "algorithmic_bytes": nbytes},
        "e2e": {"value": world * 200 / t_e2e, "unit": "steps/s",
                "h2d_bytes_per_step": sum(tt.numel() * tt.element_size() for tt in host.values()),
                "d2h_bytes_per_step": host_o.numel() * host_o.element_size(),
                "copies": "streamed: step i+1's input copy and step i-1's output copy overlap step i",
                "serial_value": world * 200 / t_e2e_serial},
        "gpu_launches": nsteps,
    }


def measure_quest(args, timed, dev, rank, world, pk):
    import torch
    from pseudobrain_b200 import exact_memory as M
    from pseudobrain_b200.synthetic import quest_inputs
    Q = {**QUEST[args.size], **QUEST_SHAPE}
    xq = quest_inputs(device=dev, seed=3 + 1000 * rank, **Q)
    kv, npages = Q["kv"], xq["kmax"].shape[1]

    def retrieve_attend(q):  # select_pages then attend_pages, one stream
        pages = M.select_pages(q, xq["kmax"], xq["kmin"], xq["n_arch"], xq["page"], xq["budget"])
        return pages, M.attend_pages(q, xq["qpos"], xq["keys"], xq["values"], xq["n_arch"], xq["page"], pages,
                                     xq["win_keys"], xq["win_values"], xq["kpos"], xq["window"])

    def step():
        retrieve_attend(xq["q"])

    qsteps = max(args.steps, 20)
    t_eager = timed(step, qsteps, max(args.warmup, 3))
    replay, graph = graphed(torch, step)  # the 4 launches of a batch replayed as a CUDA graph
    t = timed(replay, qsteps, max(args.warmup, 3))
    del graph
    per_step = t / qsteps
    bound_bytes = 2 * npages * kv * Q["d"] * 2
    page_bytes = xq["budget"] * Q["page"] * kv * Q["d"] * 2 * 2
    win_bytes = Q["window"] * kv * Q["d"] * 2 * 2
    nbytes = bound_bytes + Q["nq"] * page_bytes + win_bytes
    scores = torch.empty(Q["nq"], kv, npages, device=dev)
    t_sel = timed(lambda: M.select_pages(xq["q"], xq["kmax"], xq["kmin"], xq["n_arch"], xq["page"], xq["budget"],
                                         scores=scores), qsteps, 3)
    host_q = xq["q"].cpu().pin_memory()
    host_out = torch.empty(Q["nq"], 1, Q["heads"], Q["d"], pin_memory=True)
    dev_q = torch.empty_like(xq["q"])

    def e2e():
        dev_q.copy_(host_q, non_blocking=True)
        _, out = retrieve_attend(dev_q)
        host_out.copy_(out, non_blocking=True)

    t_e2e = timed(e2e, qsteps, 3)
    return {
        "metric": "Quest q/s (config 3)", "value": world * Q["nq"] * qsteps / t, "unit": "q/s",
        "us_per_batch": per_step * 1e6, "us_per_batch_eager": t_eager / qsteps * 1e6,
        "timing": "CUDA-graph replay of the batch; the eager figure includes the host's launch cost",
        "roofline": {"bound": "hbm", "achieved": nbytes / per_step / 1e9, "peak": pk["hbm"], "unit": "GB/s",
                     "frac": nbytes / per_step / 1e9 / pk["hbm"], "traffic": traffic("quest_score_tc_kernel"),
                     "algorithmic_bytes": nbytes},
        "select_gbps": bound_bytes / (t_sel / qsteps) / 1e9,
        "e2e": {"value": world * Q["nq"] * qsteps / t_e2e, "unit": "q/s",
                "h2d_bytes_per_step": host_q.numel() * 2, "d2h_bytes_per_step": host_out.numel() * 4},
        "gpu_launches": 4 * qsteps,
    }


def graphed(torch, fn):
    """fn captured once in a CUDA graph (after a warm call on a side stream); returns the
    replay function. Removes the host's per-launch cost from a launch-bound step."""
    fn()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g.replay, g


def _serving_piece(args, timed, dev, rank, world, pk, d):
    """One decode token of a PB-27-shaped layer (24 query / 4 key heads, head dim d) through the
    serving twins (retrieve_blocks with exact rerank + piece_attention): a 262144-token archive
    in 64-token blocks, window 16384 and the reference's defaults (512 candidates reranked
    exactly, 256 blocks kept)."""
    import types
    import torch
    from pseudobrain_b200 import serving as S
    kv, heads, block, window = 4, 24, 64, 16384
    cap = 262144 if args.size == "full" else 65536
    gen = torch.Generator(device=dev).manual_seed(6 + 1000 * rank)
    keys = torch.randn(kv, cap, d, device=dev, generator=gen).to(torch.bfloat16)
    values = torch.randn(kv, cap, d, device=dev, generator=gen).to(torch.bfloat16)
    n_blk = cap // block
    arc = types.SimpleNamespace(keys=keys, values=values, kmax=torch.empty(kv, n_blk, d, dtype=torch.bfloat16, device=dev),
                                kmin=torch.empty(kv, n_blk, d, dtype=torch.bfloat16, device=dev), size=cap,
                                prompt_len=cap, hole_lo=0, hole_hi=0, smax=None, dirty_lo=0, dirty_hi=n_blk - 1)
    q = torch.randn(1, heads, d, device=dev, generator=gen).to(torch.bfloat16)
    q_pos = torch.tensor([cap - 1], device=dev)
    limit = cap - window

    def step():
        top = S.retrieve_blocks(arc, q, heads // kv, limit, True)
        S.piece_attention(arc, q, q_pos, top, heads // kv, window, d ** -0.5, q_min=cap - 1, q_max=cap - 1)

    steps = max(args.steps, 20)
    t_eager = timed(step, steps, max(args.warmup, 3)) / steps
    replay, graph = graphed(torch, step)  # a decode step is launch-bound: replayed as a CUDA graph
    t = timed(replay, steps, max(args.warmup, 3)) / steps
    del graph
    full = (limit - S.ORIGIN) // block
    k = S.budget_for(full, True, cap, limit)
    c = min(max(S.MEMORY["rerank"], 2 * k), full)
    nbytes = (2 * full * kv * d * 2 + c * block * kv * d * 2 + k * block * kv * d * 2 * 2
              + (window + S.SINKS) * kv * d * 2 * 2)
    return {"metric": "serving decode piece (retrieve_blocks + rerank + piece_attention) per s", "value": world / t,
            "unit": "pieces/s", "us_per_piece": t * 1e6, "us_per_piece_eager": t_eager * 1e6,
            "timing": "CUDA-graph replay of the step (8 kernels); the eager figure includes the host's launch cost",
            "config": {"archive_tokens": cap, "kv_heads": kv, "q_heads": heads, "head_dim": d, "block": block,
                       "window": window, "rerank_candidates": c, "blocks_kept": k},
            "roofline": {"bound": "hbm", "achieved": nbytes / t / 1e9, "peak": pk["hbm"], "unit": "GB/s",
                         "frac": nbytes / t / 1e9 / pk["hbm"], "traffic": None, "algorithmic_bytes": nbytes},
            "gpu_launches": 8 * steps}


def _pertoken_decode(args, timed, dev, rank, d):
    """The serving default selector (retrieve_blocks_per_token) on a decode step of the same
    layer: a 16-token query history over the archive's 4096 blocks (super-blocks of 64), merged
    with a prompt selection, recomputed every call (the reference recomputes it every 64th
    decode step and reuses the set in between)."""
    import types
    import torch
    from pseudobrain_b200 import pertoken as P
    from pseudobrain_b200 import serving as S
    kv, heads, block, window = 4, 24, 64, 16384
    cap = 262144 if args.size == "full" else 65536
    gen = torch.Generator(device=dev).manual_seed(8 + 1000 * rank)
    keys = torch.randn(kv, cap, d, device=dev, generator=gen).to(torch.bfloat16)
    n_blk = cap // block
    n_sb = (n_blk + S.SBLK - 1) // S.SBLK
    z = lambda rows: torch.zeros(kv, rows, d, dtype=torch.bfloat16, device=dev)  # noqa: E731
    arc = types.SimpleNamespace(keys=keys, values=keys, kmax=z(n_blk), kmin=z(n_blk), smax=z(n_sb), smin=z(n_sb),
                                size=cap, prompt_len=cap, hole_lo=0, hole_hi=0, dirty_lo=0, dirty_hi=n_blk - 1)
    limit = cap - window
    qp = torch.randn(64, heads, d, device=dev, generator=gen).to(torch.bfloat16)
    P.retrieve_blocks_per_token(arc, qp, heads // kv, limit, 0, -1)  # the prompt's selection (kept)
    hist = torch.randn(16, heads, d, device=dev, generator=gen).to(torch.bfloat16)

    def step():
        arc.cached_top = None
        P.retrieve_blocks_per_token(arc, hist[-1:], heads // kv, limit, 0, 0, 0, hist)

    steps = max(args.steps, 20)
    t = timed(step, steps, max(args.warmup, 3)) / steps
    return {"us_per_selection": t * 1e6, "us_per_decode_step": t * 1e6 / P.DECODE_STRIDE,
            "timing": f"eager, one uncached decode selection per call (recomputed every {P.DECODE_STRIDE}th step)",
            "config": {"archive_tokens": cap, "kv_heads": kv, "q_heads": heads, "head_dim": d, "block": block,
                       "query_history": 16, "decode_blocks": P.DECODE_BLOCKS}}


def measure_serving(args, timed, dev, rank, world, pk):
    """The serving twins at PB-27's attention shape (head dim 256, the SIMT score and attention
    kernels), with the head-dim-128 figures (tensor-core score and attention kernels) and the
    per-token selector's decode selection beside them."""
    main = _serving_piece(args, timed, dev, rank, world, pk, 256)
    hd128 = _serving_piece(args, timed, dev, rank, world, pk, 128)
    main["hd128"] = {key: hd128[key] for key in ("value", "us_per_piece", "roofline")}
    main["pertoken"] = _pertoken_decode(args, timed, dev, rank, 256)
    return main


def measure_widen(args, timed, dev, rank, world, pk):
    """The rows widened around the hot path, each timed alone with its own HBM roofline
    (weak scaling, per-rank shapes): the GDN layer's pieces around the recurrence at config-1
    shapes (short conv + SiLU + q/k L2 norm, gating, gated output norm), the two-level Quest
    selection at the research defaults (64-token pages, super-blocks of 64, 64 pages kept) over
    a 1M-token archive for 8 queries, the serving archive write of a 65536-token piece into a
    1M-token archive (8 key heads, 64-token blocks, max / min / means), and the RoPE move with
    the gather of 1024 retrieved blocks per key head."""
    import types
    import torch
    from pseudobrain_b200 import exact_memory as M
    from pseudobrain_b200 import gdn_layer as L
    from pseudobrain_b200 import serving as S
    small = args.size == "small"
    gen = torch.Generator(device=dev).manual_seed(11 + 1000 * rank)
    steps = max(args.steps, 10)
    hbm = pk["hbm"]

    def entry(seconds, nbytes, launches, **extra):
        return {"us": seconds * 1e6, "achieved_gbps": nbytes / seconds / 1e9, "frac": nbytes / seconds / 1e9 / hbm,
                "algorithmic_bytes": nbytes, "launches_per_call": launches, **extra}

    out = {}
    # GDN layer pieces (config 1 shapes)
    b, t, hk, hv = (1, 8192, 16, 32) if small else (4, 32768, 16, 32)
    c = (2 * hk + hv) * 128
    x = torch.randn(b, t, c, device=dev, generator=gen).to(torch.bfloat16)
    wconv = torch.randn(c, 4, device=dev, generator=gen) * 0.5
    tail = torch.randn(b, 3, c, device=dev, generator=gen).to(torch.bfloat16)
    new_tail = torch.empty_like(tail)
    tc_ = timed(lambda: L.conv_qkv(x, tail, wconv, hk, hv, "max", new_tail), steps, 3) / steps
    out["conv_qkv"] = entry(tc_, 2 * x.numel() * 2 + 2 * tail.numel() * 2 + wconv.numel() * 4, 1,
                            shape=f"x [{b},{t},{c}] bf16 -> q, k [{b},{t},{hk},128], v [{b},{t},{hv},128] bf16",
                            traffic=traffic("gdn_conv_norm_vec_kernel"))
    del x
    decay = torch.randn(b, t, 2 * hv, device=dev, generator=gen).to(torch.bfloat16)
    a_log, dt_bias = torch.randn(hv, device=dev, generator=gen), torch.randn(hv, device=dev, generator=gen)
    tg = timed(lambda: L.gdn_gating(decay, a_log, dt_bias, torch.bfloat16), steps, 3) / steps
    out["gating"] = entry(tg, decay.numel() * 2 + b * t * hv * (4 + 2), 1)
    o = torch.randn(b, t, hv, 128, device=dev, generator=gen)
    gate = torch.randn(b, t, hv * 128, device=dev, generator=gen).to(torch.bfloat16)
    wn = torch.randn(128, device=dev, generator=gen)
    tn = timed(lambda: L.gated_out_norm(o, gate, wn, out_dtype=torch.bfloat16), steps, 3) / steps
    out["gated_out_norm"] = entry(tn, o.numel() * 4 + gate.numel() * 2 + o.numel() * 2, 1,
                                  shape="o fp32, gate bf16 -> out bf16", traffic=traffic("gdn_out_norm_vec_kernel"))
    del o, gate, decay
    torch.cuda.empty_cache()
    out["gdn_layer"] = _gdn_layer_fused(torch, L, dev, gen, small, steps, hbm)
    torch.cuda.empty_cache()
    # two-level Quest selection (research defaults)
    kv, heads, d, page, sblk, nq, budget = 8, 32, 128, 64, 64, 8, 64
    n_tok = (1 << 19) if small else (1 << 20)
    full = n_tok // page
    kmax = torch.randn(kv, full, d, device=dev, generator=gen).to(torch.bfloat16)
    kmin = (kmax.float() - torch.rand(kv, full, d, device=dev, generator=gen) * 2).to(torch.bfloat16)
    smax, smin = M.super_bounds(kmax[None], kmin[None], sblk)
    smax, smin = smax[0], smin[0]
    q = torch.randn(nq, 1, heads, d, device=dev, generator=gen).to(torch.bfloat16)

    def levels():
        M.select_pages_levels(q, kmax, kmin, n_tok, page, budget, smax, smin, sblk)

    replay, graph = graphed(torch, levels)
    tl = timed(replay, steps * 4, 3) / (steps * 4)
    del graph
    m_sb = M.m_superblocks(budget, full, sblk)
    lv_bytes = smax.numel() * 2 * 2 + nq * kv * m_sb * sblk * d * 2 * 2
    tf = timed(lambda: M.select_pages(q, kmax, kmin, n_tok, page, budget), steps * 4, 3) / (steps * 4)
    out["quest_two_level"] = entry(tl, lv_bytes, 5, flat_us=tf * 1e6, flat_bytes=kmax.numel() * 2 * 2,
                                   config=f"{n_tok} tokens, pages of {page}, super-blocks of {sblk}, {nq} queries, "
                                          f"{heads}/{kv} heads, {budget} pages kept, {m_sb} super-blocks",
                                   timing="CUDA-graph replay (5 launches)")
    del kmax, kmin, smax, smin
    torch.cuda.empty_cache()
    # serving archive write
    block, n_new = 64, (16384 if small else 65536)
    cap = n_tok + S.ORIGIN
    n_blk = cap // block
    n_sb = (n_blk + S.SBLK - 1) // S.SBLK
    z = lambda rows: torch.zeros(kv, rows, d, dtype=torch.bfloat16, device=dev)  # noqa: E731
    arc = types.SimpleNamespace(keys=z(cap), values=z(cap), kmax=z(n_blk), kmin=z(n_blk), bmean_k=z(n_blk),
                                bmean_v=z(n_blk), smax=z(n_sb), smin=z(n_sb), smean_k=z(n_sb), smean_v=z(n_sb),
                                size=cap - 4096, dirty_lo=1 << 60, dirty_hi=-1)
    p0 = S.ORIGIN + 40 * block
    kn = torch.randn(n_new, kv, d, device=dev, generator=gen).to(torch.bfloat16)
    vn = torch.randn(n_new, kv, d, device=dev, generator=gen).to(torch.bfloat16)
    pos = torch.arange(p0, p0 + n_new, device=dev)
    tw = timed(lambda: S.archive_write(arc, pos, kn, vn, block, p0, p0 + n_new), steps, 3) / steps
    nb_touch = n_new // block
    w_bytes = 2 * kn.numel() * 2 * 2 + nb_touch * kv * d * 2 * 4
    out["archive_write"] = entry(tw, w_bytes, 4, config=f"{n_new} tokens x {kv} key heads into a {cap}-row archive, "
                                                        f"blocks of {block}, super-blocks of {S.SBLK}",
                                 traffic=traffic("quest_archive_block_kernel"))
    # RoPE move + gather of the retrieved blocks
    nsel = 1024
    blocks = torch.sort(torch.stack([torch.randperm(n_blk - 1, device=dev, generator=gen)[:nsel]
                                     for _ in range(kv)]), dim=-1).values.to(torch.int32)
    tr = timed(lambda: S.rope_gather(arc.keys, arc.values, blocks, block, S.ORIGIN, nsel, "runs",
                                     ref_pos=cap - 1024), steps, 3) / steps
    out["rope_gather"] = entry(tr, 2 * 2 * kv * nsel * block * d * 2, 2,
                               config=f"{nsel} blocks of {block} x {kv} key heads, keys moved, values gathered",
                               traffic=traffic("quest_rope_gather_kernel"))
    del arc, kn, vn
    torch.cuda.empty_cache()
    out["gpu_launches"] = 3 * steps + 5 * (steps * 4 + 3) + 4 * steps + 2 * steps
    lay_p, lay_d = max(3, steps // 3), max(20, steps * 4)  # the fused-layer comparisons
    out["gpu_launches"] += (3 + 5) * (lay_p + 3) + (1 + 4) * (lay_d + 5)
    cv = out["conv_qkv"]  # the line's own fields when this part runs alone
    out.update(metric="widened rows: HBM GB/s of each piece", value=cv["achieved_gbps"], unit="GB/s",
               roofline={"bound": "hbm", "achieved": cv["achieved_gbps"], "peak": hbm, "unit": "GB/s",
                         "frac": cv["frac"], "traffic": cv.get("traffic"), "kernel": "gdn_conv_norm_vec_kernel"})
    return out


def _gdn_layer_fused(torch, L, dev, gen, small, steps, hbm):
    """GatedDeltaNetLayer.forward from the projection's output to the gated, normed output:
    the prefill at config-1 shapes as pbk_gdn_prefill_layer (conv, norm and gating fused into
    the chunk solve; 3 launches) against the same layer as the separate pieces (conv + norm,
    gating, chunk solve, recurrence, output norm: 5 launches), and the decode step at config-2
    shapes as pbk_gdn_decode_layer (1 launch) against conv + gating + decode + output norm."""
    res = {}
    b, t, hk, hv = (1, 8192, 16, 32) if small else (4, 32768, 16, 32)
    c = (2 * hk + hv) * 128
    qkv = torch.randn(b, t, c, device=dev, generator=gen).to(torch.bfloat16)
    gate = torch.randn(b, t, hv * 128, device=dev, generator=gen).to(torch.bfloat16)
    decay = torch.randn(b, t, 2 * hv, device=dev, generator=gen).to(torch.bfloat16)
    wconv = torch.randn(c, 4, device=dev, generator=gen) * 0.5
    tail = torch.randn(b, 3, c, device=dev, generator=gen).to(torch.bfloat16)
    new_tail = torch.empty_like(tail)
    a_log, dt_bias = torch.randn(hv, device=dev, generator=gen) * 0.5, torch.randn(hv, device=dev, generator=gen)
    o_norm = torch.ones(128, device=dev)
    state = torch.zeros(b, hv, 128, 128, device=dev)
    from pseudobrain_b200.gdn_prefill import gdn_prefill_

    def fused():
        L.gated_deltanet_prefill(qkv, gate, decay, tail, wconv, a_log, dt_bias, o_norm, state, hk, hv,
                                 new_tail=new_tail, out_dtype=torch.bfloat16)

    o = torch.empty(b, t, hv, 128, device=dev, dtype=torch.bfloat16)

    def unfused():
        q, k, v = L.conv_qkv(qkv, tail, wconv, hk, hv, "max", new_tail)
        g, beta = L.gdn_gating(decay, a_log, dt_bias, torch.bfloat16)
        gdn_prefill_(q, k, v, g, beta, state, state, o, 128 ** -0.5)
        L.gated_out_norm(o, gate, o_norm, out_dtype=torch.bfloat16)

    reps = max(3, steps // 3)
    tf = timed_plain(torch, fused, reps, 3)
    tu = timed_plain(torch, unfused, reps, 3)
    tokens = b * t
    res["prefill"] = {"config": f"B={b} T={t} Hk={hk} Hv={hv}, conv width 4, bf16 in / out",
                      "fused_ms": tf * 1e3, "unfused_ms": tu * 1e3, "speedup": tu / tf,
                      "fused_tok_s": tokens / tf, "launches": {"fused": 3, "unfused": 5}}
    del qkv, gate, decay, tail, new_tail, state, o
    torch.cuda.empty_cache()
    b, t = 256, 1
    qkv = torch.randn(b, t, c, device=dev, generator=gen).to(torch.bfloat16)
    gate = torch.randn(b, t, hv * 128, device=dev, generator=gen).to(torch.bfloat16)
    decay = torch.randn(b, t, 2 * hv, device=dev, generator=gen).to(torch.bfloat16)
    tail = torch.randn(b, 3, c, device=dev, generator=gen).to(torch.bfloat16)
    tail2 = tail.clone()
    state = torch.randn(b, hv, 128, 128, device=dev, generator=gen) * 0.02

    def dec_fused():
        L.gated_deltanet_decode(qkv, gate, decay, tail, wconv, a_log, dt_bias, o_norm, state, hk, hv,
                                out_dtype=torch.bfloat16)

    o = torch.empty(b, t, hv, 128, device=dev, dtype=torch.bfloat16)
    from pseudobrain_b200.gated_deltanet import gdn_recurrent_

    def dec_unfused():
        q, k, v = L.conv_qkv(qkv, tail, wconv, hk, hv, "max", tail2)
        g, beta = L.gdn_gating(decay, a_log, dt_bias, torch.bfloat16)
        gdn_recurrent_(q, k, v, g, beta, state, state, o, 128 ** -0.5)
        L.gated_out_norm(o, gate, o_norm, out_dtype=torch.bfloat16)

    reps = max(20, steps * 4)
    tdf = timed_plain(torch, dec_fused, reps, 5)
    tdu = timed_plain(torch, dec_unfused, reps, 5)
    sbytes = 2 * state.numel() * 4
    res["decode"] = {"config": f"B={b} T=1 Hk={hk} Hv={hv}, conv width 4, tail in place",
                     "fused_us": tdf * 1e6, "unfused_us": tdu * 1e6, "speedup": tdu / tdf,
                     "fused_steps_s": 1.0 / tdf, "fused_hbm_frac": sbytes / tdf / 1e9 / hbm,
                     "launches": {"fused": 1, "unfused": 4}}
    del qkv, gate, decay, tail, tail2, state, o
    return res


def timed_plain(torch, fn, reps, warmup):
    """Seconds per call: CUDA events around `reps` back-to-back calls on the current stream,
    after `warmup` untimed calls (inputs larger than L2 where the piece's shapes make them)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3 / reps


def swa_pairs(t, window):
    """Visible (query, key) pairs of a causal window over t tokens."""
    w = min(window, t)
    return t * w - w * (w - 1) // 2


def measure_hybrid(args, timed, dev, rank, world, pk):
    """benchmark config 4: one hybrid layer over a 1M-token sequence (B=1). The GDN branch
    (16 key / 32 value heads) is split by value head over the ranks, and within a rank along
    T (segments chained by the segment scan) so a few heads still fill the SMs; the
    sliding-window attention branch (32 query / 8 key heads, window 4096) is split by key
    head. Each branch's output is gathered into rank-major [N, rows, heads/N * 128] buffers
    (the hidden-4096 layout the output projection reads): the GDN branch in two parts, each
    sent as soon as it is written, then the attention in query chunks, each sent while the
    next chunk computes (sharding.hybrid_layer_sharded): by copy-engine pushes into every
    rank's mapped buffers up to 4 GPUs, by NCCL's all-gather above. Strong scaling: the job is one layer pass
    whatever N; at N > 1 rank 0 also times the unsharded layer (all heads on one GPU) for
    the strong-scaling efficiency t1 / (N tN)."""
    import torch
    import torch.distributed as dist
    from pseudobrain_b200.gdn_prefill import auto_segments, gdn_prefill_segmented
    from pseudobrain_b200.sharding import hybrid_layer_sharded
    from pseudobrain_b200.synthetic import gdn_inputs
    from pseudobrain_b200.transplant import window_attention_
    H = HYBRID_HEADS
    t = HYBRID[args.size]["seqlen"]
    if H["hv"] % world or H["kv"] % world:
        return None

    def shard_inputs(nshard, seed):
        hv, hk, heads, kv = H["hv"] // nshard, H["hk"] // nshard, H["heads"] // nshard, H["kv"] // nshard
        x = gdn_inputs(1, t, hk, hv, device=dev, seed=seed)
        gen = torch.Generator(device=dev).manual_seed(seed + 1)
        qa = torch.randn(1, t, heads, H["d"], device=dev, generator=gen).to(torch.bfloat16)
        ka = torch.randn(1, t, kv, H["d"], device=dev, generator=gen).to(torch.bfloat16)
        va = torch.randn(1, t, kv, H["d"], device=dev, generator=gen).to(torch.bfloat16)
        return x, qa, ka, va

    x, qa, ka, va = shard_inputs(world, 4 + 1000 * rank)
    from pseudobrain_b200.sharding import default_transport
    transport = {"p2p": "copy-engine pushes into the peers' mapped buffers (CUDA IPC)",
                 "nccl": "NCCL all_gather_into_tensor"}[default_transport(world, True)] if world > 1 else "none"
    hv, heads = H["hv"] // world, H["heads"] // world
    scale = H["d"] ** -0.5

    def step():
        hybrid_layer_sharded(x, qa, ka, va, H["window"], scale)

    steps = max(3, min(args.steps, 5))
    t_step = timed(step, steps, 3) / steps
    o_gdn = torch.empty(1, t, hv, H["d"], device=dev, dtype=torch.bfloat16)
    o_swa = torch.empty_like(qa)
    segs = auto_segments(1, hv, t)
    t_gdn = timed(lambda: gdn_prefill_segmented(x["q"], x["k"], x["v"], x["g"], x["beta"], x["scale"], None,
                                                segments=segs, o=o_gdn), 2, 1) / 2
    t_swa = timed(lambda: window_attention_(qa, ka, va, o_swa, H["window"], 0, scale), 2, 1) / 2
    t_ag = 0.0
    if world > 1:
        gath_gdn = torch.empty(world * t, hv * H["d"], device=dev, dtype=torch.bfloat16)
        gath_swa = torch.empty(world * t, heads * H["d"], device=dev, dtype=torch.bfloat16)

        def gather():
            dist.all_gather_into_tensor(gath_gdn, o_gdn.view(t, -1))
            dist.all_gather_into_tensor(gath_swa, o_swa.view(t, -1))

        t_ag = timed(gather, 2, 1) / 2
        del gath_gdn, gath_swa
    del o_gdn, o_swa
    gdn_flops = t * H["hv"] * prefill_flops_per_token_head(64, H["d"])
    swa_flops = 4 * H["d"] * swa_pairs(t, H["window"]) * H["heads"]
    per_gpu = (gdn_flops + swa_flops) / world
    ag_bytes = (world - 1) * t * (hv + heads) * H["d"] * 2  # bf16 received per GPU
    out = {
        "metric": "hybrid layer tok/s (config 4)", "value": t / t_step, "unit": "tok/s",
        "per_gpu": t / t_step / world, "scaling": "strong", "ms_per_step": t_step * 1e3,
        "config": {"seqlen": t, "gdn_heads_per_gpu": hv, "gdn_segments": segs, "swa_q_heads_per_gpu": heads,
                   "window": H["window"], "size": args.size, "swa_query_chunks": 8,
                   "transport": transport},
        "roofline": {"bound": "tensor", "achieved": per_gpu / t_step / 1e12, "peak": pk["tc"],
                     "unit": "TFLOP/s", "frac": per_gpu / t_step / 1e12 / pk["tc"],
                     "traffic": None, "peak_source": f"{pk['src']} bf16 burst (timed regions under a second)"},
        "gdn": {"ms": t_gdn * 1e3, "tflops": gdn_flops / world / t_gdn / 1e12},
        "swa": {"ms": t_swa * 1e3, "tflops": swa_flops / world / t_swa / 1e12,
                "frac": swa_flops / world / t_swa / 1e12 / pk["tc"]},
        "e2e": None,
        "gpu_launches": steps * (8 + 1 + 4 + 1),  # attention chunks, chunk solve, 4 recurrence runs, scan
    }
    if world > 1:
        # NCCL's all-gather of the same bytes timed alone (the layer moves them overlapped, by
        # the transport named in its config): its share of the step if it ran serially
        out["all_gather"] = {"ms": t_ag * 1e3, "bytes_received_per_gpu": ag_bytes, "what": "NCCL, alone",
                             "gbps": ag_bytes / t_ag / 1e9 if t_ag > 0 else None,
                             "share_of_step_if_serial": t_ag / (t_ag + t_gdn + t_swa)}
        # strong scaling: the unsharded layer (all heads) on rank 0 while the others wait
        t1 = None
        del x, qa, ka, va
        torch.cuda.empty_cache()
        if rank == 0:
            x1, qa1, ka1, va1 = shard_inputs(1, 4)

            def step1():
                hybrid_layer_sharded(x1, qa1, ka1, va1, H["window"], scale, gather=False)

            step1()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(2):
                step1()
            e1.record()
            torch.cuda.synchronize()
            t1 = e0.elapsed_time(e1) / 2 / 1e3
            del x1, qa1, ka1, va1
            torch.cuda.empty_cache()
        dist.barrier()
        if t1 is not None:
            out["strong_scaling"] = {"t1_ms": t1 * 1e3, "tN_ms": t_step * 1e3, "n": world,
                                     "efficiency": t1 / (world * t_step),
                                     "note": "t1: the same layer, all 32/32 heads on one GPU (rank 0), no exchange"}
    return out


def headline_config(args, world):
    """The `config` object of the line (the reference arm prints the same one)."""
    return {"workload": ("benchmark config 1: GDN chunked prefill B=4 T=32768 Hk=16 Hv=32 dk=dv=128 chunk=64 "
                         "per GPU") if args.workload in ("all", "prefill") else f"{args.workload} part only",
            "size": args.size, "global_batch": PREFILL[args.size]["batch"] * world,
            "seq_len": PREFILL[args.size]["seqlen"],
            "parallelism": f"(sequence x value-head) shards, {world} GPU(s), no collective",
            "l2": "inputs larger than L2 (126 MB) in every timed part"}


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    pk = peaks()
    timed = Timer(torch, dist, dev, world)
    parts = {}
    clk = Clocks(local_rank)
    for name, fn in (("prefill", measure_prefill), ("decode", measure_decode), ("quest", measure_quest),
                     ("hybrid", measure_hybrid), ("serving", measure_serving), ("widen", measure_widen)):
        if args.workload in ("all", name):
            if name == "prefill":
                with clk:
                    parts[name] = fn(args, timed, dev, rank, world, pk)
            else:
                parts[name] = fn(args, timed, dev, rank, world, pk)
            torch.cuda.empty_cache()
    if rank != 0:
        return None
    head = parts.get("prefill") or next(iter(parts.values()))
    ms = head.get("ms_per_step")
    if ms is None:
        ms = head.get("us_per_step", head.get("us_per_batch", 0.0)) / 1e3
    line = {
        "metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 inputs, fp32 state/accumulation", "data": "synthetic (seeded, benchmark config distributions)",
        "config": headline_config(args, world),
        "roofline": head["roofline"], "e2e": head.get("e2e"), "gpu_launches": head["gpu_launches"],
        "clocks": clk.summary(),
    }
    for key in ("kernels", "step"):  # the prefill step's two kernels and its whole-step figures
        if key in head:
            line[key] = head[key]
    # the large, secondary parts first and decode / quest last: a reader of the end of the
    # line (a log tail) sees the two other headline parts of the metric
    for name in ("widen", "serving", "hybrid", "decode", "quest"):
        if name in parts and parts[name] is not None:  # (the head part too: its own figures)
            line[name] = parts[name]
    if world == 1 and not args.no_cpu_baseline:
        if "prefill" in parts:
            line["cpu_baseline"] = cpu_baseline()
        for name, fn in (("hybrid", cpu_baseline_hybrid), ("decode", cpu_baseline_decode),
                         ("quest", cpu_baseline_quest)):
            if line.get(name) is not None and args.size == "full":
                line[name]["cpu_baseline"] = fn()
        for name in ("decode", "quest"):  # keep the two at the end of the line
            if name in line:
                line[name] = line.pop(name)
    return line


# --------------------------------------------------------------------------------------------
# CPU baseline / reference arm: the reference's CPU path restated with the same torch CPU
# operations (oracle/cpu_reference.py), on all host cores, over bounded samples of each config
# --------------------------------------------------------------------------------------------
def _cpu_gdn_inputs(torch, batch, t, hk, hv, seed, state_std=0.0):
    """Config-0 distributions on the host, q and k expanded from the key heads to the value
    heads as the reference's caller does (gated_deltanet.py:422-424)."""
    import torch.nn.functional as F
    g_ = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(batch, t, hk, 128, generator=g_), dim=-1).to(torch.bfloat16).float()
    k = F.normalize(torch.randn(batch, t, hk, 128, generator=g_), dim=-1).to(torch.bfloat16).float()
    v = torch.randn(batch, t, hv, 128, generator=g_).to(torch.bfloat16).float()
    beta = torch.sigmoid(torch.randn(batch, t, hv, generator=g_)).to(torch.bfloat16).float()
    g = F.logsigmoid(torch.randn(batch, t, hv, generator=g_) + 2.0)
    rep = hv // hk
    if state_std:  # a tiled random state: the values do not change the work
        base = torch.randn(1, hv, 128, 128, generator=g_) * state_std
        h0 = base.expand(batch, -1, -1, -1).contiguous()
    else:
        h0 = torch.zeros(batch, hv, 128, 128)
    return q.repeat_interleave(rep, 2), k.repeat_interleave(rep, 2), v, g, beta, h0


def cpu_prefill_step(t=8192, seed=0):
    """One bounded sample of config 1 on the host: B=1, T=t, 16 key / 32 value heads, fp32
    compute (delta_rule_chunked). Returns (tokens, seconds)."""
    import torch
    from oracle import cpu_reference as cr
    q, k, v, g, beta, h0 = _cpu_gdn_inputs(torch, 1, t, PREFILL_HEADS["hk"], PREFILL_HEADS["hv"], seed)
    t0 = time.perf_counter()
    cr.chunked_prefill(q, k, v, g, beta, 128 ** -0.5, h0)
    return t, time.perf_counter() - t0


def cpu_baseline(samples=3, t=8192):
    """Config-1 prefill tok/s of the reference's CPU path (oracle/cpu_reference.py, torch,
    all host cores) over `samples` samples of B=1, T=t, after one warm-up sample."""
    from oracle import cpu_reference as cr
    cores = cr.use_all_cores()
    cpu_prefill_step(t)
    toks = secs = 0.0
    for i in range(samples):
        n, dt = cpu_prefill_step(t, seed=i + 1)
        toks, secs = toks + n, secs + dt
    return {"value": toks / secs, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"delta_rule_chunked (torch fp32 CPU restatement), B=1 T={t} Hk=16 Hv=32, {samples} samples "
                      f"after 1 warm-up, {secs:.1f} s"}


def cpu_baseline_decode(steps=5):
    """Config-2 decode steps/s on the host: gated_delta_rule(..., "sequential") of B=256
    one-token sequences, 32 value heads, the 537 MB fp32 state (the median of `steps` steps
    after one warm-up)."""
    import torch
    from oracle import cpu_reference as cr
    cores = cr.use_all_cores()
    q, k, v, g, beta, h0 = _cpu_gdn_inputs(torch, 256, 1, DECODE_HEADS["hk"], DECODE_HEADS["hv"], 2, state_std=0.02)
    times = []
    for i in range(steps + 1):
        t0 = time.perf_counter()
        _, h0 = cr.sequential_steps(q, k, v, g, beta, 128 ** -0.5, h0)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times[1:])
    return {"value": 1.0 / med, "unit": "steps/s", "cores": cores, "kind": "port",
            "sample": f"delta_rule_sequential (torch fp32 CPU restatement), B=256 Hv=32, median of {steps} in-place "
                      f"steps after 1 warm-up ({med * 1e3:.0f} ms per step)"}


def cpu_baseline_quest(nq=8):
    """Config-3 Quest q/s on the host: per query, the reference's flat retrieve (fp32 bound
    scores, topk, sort, gather + tail) and SDPA over [retrieved ; window] over a 1M-token bf16
    cache with its page bounds precomputed (not timed). The cache is 64 copies of a seeded
    16384-token block, each shifted by its own seeded offset (drawing 2G normals on the host
    would take a minute; the work per query depends only on the sizes)."""
    import torch
    from oracle import cpu_reference as cr
    cores = cr.use_all_cores()
    Q = {**QUEST["full"], **QUEST_SHAPE}
    kv, d, n = Q["kv"], Q["d"], Q["n_tokens"]
    g_ = torch.Generator().manual_seed(3)
    blk = 16384
    reps = n // blk

    def cache():
        base = torch.randn(1, kv, 1, blk, d, generator=g_)
        shift = torch.randn(1, kv, reps, 1, d, generator=g_) * 0.5
        return (base + shift).reshape(1, kv, n, d).to(torch.bfloat16)

    keys, values = cache(), cache()
    n_arch = n - Q["window"]
    kmax, kmin = cr.page_bounds(keys[:, :, :n_arch], Q["page"])
    q = torch.randn(nq, 1, Q["heads"], d, generator=g_).to(torch.bfloat16)
    qpos = torch.tensor([n - 1])
    kpos = torch.arange(n_arch, n)
    times = []
    for i in range(nq + 1):  # the first query warms up
        t0 = time.perf_counter()
        cr.quest_retrieve_attend(q[i % nq].transpose(0, 1)[None], keys[:, :, :n_arch], values[:, :, :n_arch],
                                 kmax, kmin, n_arch, Q["page"], Q["budget_tokens"] // Q["page"], keys[:, :, n_arch:],
                                 values[:, :, n_arch:], qpos, kpos, Q["window"])
        times.append(time.perf_counter() - t0)
    per = statistics.median(times[1:])
    return {"value": 1.0 / per, "unit": "q/s", "cores": cores, "kind": "port",
            "sample": f"retrieve (flat, fp32 scores) + SDPA per query over a 1M-token cache, median of {nq} queries "
                      f"after 1 warm-up ({per * 1e3:.0f} ms per query; page bounds built once, not timed)"}


def cpu_baseline_hybrid(t=16384):
    """Config-4 hybrid layer tok/s on the host, extrapolated from a t-token slice: the GDN
    branch (delta_rule_chunked, 16/32 heads) plus the window attention branch (32/8 heads,
    window 4096, query chunks of 4096 through SDPA), each scaled to 1M tokens by its work
    (GDN linear in T; attention by the visible (query, key) pairs)."""
    import torch
    from oracle import cpu_reference as cr
    cores = cr.use_all_cores()
    H = HYBRID_HEADS
    q, k, v, g, beta, h0 = _cpu_gdn_inputs(torch, 1, t, H["hk"], H["hv"], 4)
    t0 = time.perf_counter()
    cr.chunked_prefill(q, k, v, g, beta, 128 ** -0.5, h0)
    t_gdn = time.perf_counter() - t0
    g_ = torch.Generator().manual_seed(5)
    qa = torch.randn(1, H["heads"], t, H["d"], generator=g_).to(torch.bfloat16).float()
    ka = torch.randn(1, H["kv"], t, H["d"], generator=g_).to(torch.bfloat16).float()
    va = torch.randn(1, H["kv"], t, H["d"], generator=g_).to(torch.bfloat16).float()
    t0 = time.perf_counter()
    cr.window_attention(qa, ka, va, H["window"])
    t_swa = time.perf_counter() - t0
    full = HYBRID["full"]["seqlen"]
    est = t_gdn * full / t + t_swa * swa_pairs(full, H["window"]) / swa_pairs(t, H["window"])
    return {"value": full / est, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{t}-token slice ({t_gdn:.1f} s GDN + {t_swa:.1f} s window attention), extrapolated to "
                      f"{full} tokens ({est:.0f} s): GDN by T, attention by visible (query, key) pairs"}


def run_reference(args, rank, config):
    """The reference arm: the reference's CPU path (torch CPU restatement, all host cores) on
    the headline metric, config 1 prefill tok/s, W warm-up and K timed steps of one bounded
    B=1, T=8192 sample each; plus one CPU figure per other config."""
    if rank != 0:
        return None
    from oracle import cpu_reference as cr
    cores = cr.use_all_cores()
    t = 8192
    for i in range(args.warmup):
        cpu_prefill_step(t, seed=100 + i)
    toks = secs = 0.0
    for i in range(args.steps):
        n, dt = cpu_prefill_step(t, seed=i)
        toks, secs = toks + n, secs + dt
    value = toks / secs
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, benchmark config "
            "distributions)", "impl": "reference", "config": config,
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"delta_rule_chunked (torch fp32 CPU restatement of gated_deltanet.py:110-165),"
                                       f" one B=1 T={t} Hk=16 Hv=32 sample per step"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.workload == "all":
        line["decode"] = cpu_baseline_decode()
        line["quest"] = cpu_baseline_quest()
        line["hybrid"] = cpu_baseline_hybrid()
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=("all", "prefill", "decode", "quest", "hybrid", "serving", "widen"),
                    default="all",
                    help="run one part only (profiling); the JSON line then carries that part")
    ap.add_argument("--size", choices=("full", "small"), default="full",
                    help="small: a reduced case of the same kernels for ncu captures (not a bench number)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, headline_config(args, world))
    else:
        if world > 1:
            import datetime
            import torch
            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local_rank))
        line = run_ours(args, rank, world, local_rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
