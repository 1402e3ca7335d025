"""Benchmark of the PseudoBrain hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (``value``): GDN chunked prefill of BASELINE config 1 (B=4, T=32768, 16 key /
32 value heads, dk=dv=128, chunk 64, bf16 q/k/v/beta, fp32 g and state) in tok/s,
inputs resident in HBM, device-timed with CUDA events, max over ranks. The same line
carries the other two parts of the metric, each with its own roofline:
``decode`` (config 2: B=256 decode step, 537 MB fp32 state, steps/s) and ``quest``
(config 3: 8 queries over a 1M-token cache, q/s). ``e2e`` times the public API with
pinned host inputs copied in and outputs copied back inside the timed region.

Multi-GPU (torchrun, one rank per GPU): weak scaling. Every rank runs its own shard of
(sequence x value head) chains of the same per-GPU size; the recurrence has no
exchange step, so there is no collective inside the timed region.

``--impl reference`` times the CPU restatement of the reference algorithm (oracle/,
numpy, all host cores) on bounded samples of the same workloads and prints the same
metric; under torchrun only rank 0 runs it.
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
PREFILL = dict(batch=4, seqlen=32768, hk=16, hv=32, dk=128, dv=128, chunk=64)
DECODE = dict(batch=256, hk=16, hv=32, dk=128, dv=128, steps_per_rep=1000)
QUEST = dict(n_tokens=1 << 20, kv=8, heads=32, d=128, page=16, window=4096, nq=8, budget_tokens=4096)


def prefill_flops_per_token_head(c=64, d=128):
    """5 C x C x d products (KK^T, QK^T, W, U', (QK*D)U) + 3 d x d products per token
    (WS, QS, K^T U) + the triangular inverse (C^2/3 per token)."""
    return 5 * 2 * c * d + 3 * 2 * d * d + 2 * c * c / 3


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return dict(hbm=p["hbm_gbs"], tc=p["bf16_tflops"], tc_sustained=p["bf16_tflops_sustained"], src="measured")
    return dict(hbm=6650.0, tc=1590.0, tc_sustained=1400.0, src="fallback")


def traffic(kernel_key):
    """DRAM bytes per launch from the committed ncu summary (profiles/traffic.txt), or None."""
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
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from pseudobrain_b200 import gated_deltanet as G
    from pseudobrain_b200 import exact_memory as M
    from pseudobrain_b200.gdn_prefill import gdn_prefill_
    from pseudobrain_b200.synthetic import gdn_inputs, quest_inputs

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    pk = peaks()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, steps, warmup, events_stream=None):
        """Device time of `steps` calls after `warmup`, bracketed by barrier + synchronize."""
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s = torch.cuda.current_stream(dev)
        st.record(s)
        for _ in range(steps):
            fn()
        en.record(s)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(st.elapsed_time(en) / 1e3)

    # ---------------- prefill (headline, config 1) ----------------
    P = PREFILL
    x = gdn_inputs(P["batch"], P["seqlen"], P["hk"], P["hv"], device=dev, seed=1 + 1000 * rank)
    state = torch.empty(P["batch"], P["hv"], P["dk"], P["dv"], device=dev)
    o = torch.empty(P["batch"], P["seqlen"], P["hv"], P["dv"], device=dev, dtype=torch.bfloat16)

    def prefill_step():
        gdn_prefill_(x["q"], x["k"], x["v"], x["g"], x["beta"], None, state, o, x["scale"])

    with Clocks(local_rank) as clk:
        t_prefill = timed(prefill_step, args.steps, args.warmup)
    tokens = P["batch"] * P["seqlen"]
    value = world * tokens * args.steps / t_prefill
    ms_per_step = t_prefill / args.steps * 1e3
    flops = tokens * P["hv"] * prefill_flops_per_token_head(P["chunk"], P["dk"])
    achieved_tf = flops / (t_prefill / args.steps) / 1e12
    algo_bytes = (2 * tokens * P["hk"] * P["dk"] * 2 + tokens * P["hv"] * P["dv"] * 2 * 2 + tokens * P["hv"] * 6
                  + 2 * P["batch"] * P["hv"] * P["dk"] * P["dv"] * 4)

    # e2e through the public API: pinned host inputs in, bf16 outputs back, every step
    host = {n: x[n].cpu().pin_memory() for n in ("q", "k", "v", "g", "beta")}
    dev_in = {n: torch.empty_like(x[n]) for n in host}
    host_o = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = host_o.numel() * host_o.element_size()

    def prefill_e2e():
        for n, t in host.items():
            dev_in[n].copy_(t, non_blocking=True)
        gdn_prefill_(dev_in["q"], dev_in["k"], dev_in["v"], dev_in["g"], dev_in["beta"], None, state, o, x["scale"])
        host_o.copy_(o, non_blocking=True)

    e2e_steps = max(3, args.steps // 2)
    t_e2e = timed(prefill_e2e, e2e_steps, min(args.warmup, 3))
    del x, dev_in, host, host_o, o, state
    torch.cuda.empty_cache()

    # ---------------- decode (config 2) ----------------
    D = DECODE
    xd = gdn_inputs(D["batch"], 1, D["hk"], D["hv"], device=dev, seed=2 + 1000 * rank, g_dtype=torch.bfloat16,
                    state_std=0.02)
    od = torch.empty(D["batch"], 1, D["hv"], D["dv"], device=dev, dtype=torch.bfloat16)

    def decode_step():
        G.gdn_recurrent_(xd["q"], xd["k"], xd["v"], xd["g"], xd["beta"], None, xd["h0"], od, xd["scale"])

    dsteps = D["steps_per_rep"]
    t_dec = timed(decode_step, dsteps, max(args.warmup, 10))
    dec_value = world * dsteps / t_dec
    dec_bytes = 2 * xd["h0"].numel() * 4 + sum(xd[n].numel() * xd[n].element_size() for n in ("q", "k", "v", "g", "beta")) \
        + od.numel() * 2
    hostd = {n: xd[n].cpu().pin_memory() for n in ("q", "k", "v", "g", "beta")}
    devd = {n: torch.empty_like(xd[n]) for n in hostd}
    host_od = torch.empty(od.shape, dtype=od.dtype, pin_memory=True)

    def decode_e2e():
        for n, t in hostd.items():
            devd[n].copy_(t, non_blocking=True)
        G.gdn_recurrent_(devd["q"], devd["k"], devd["v"], devd["g"], devd["beta"], None, xd["h0"], od, xd["scale"])
        host_od.copy_(od, non_blocking=True)

    t_dec_e2e = timed(decode_e2e, 200, 10)
    dec_h2d = sum(t.numel() * t.element_size() for t in hostd.values())
    del xd, devd, hostd, od
    torch.cuda.empty_cache()

    # ---------------- Quest (config 3) ----------------
    Q = QUEST
    xq = quest_inputs(device=dev, seed=3 + 1000 * rank, **{k: Q[k] for k in Q})
    kv, npages = Q["kv"], xq["kmax"].shape[1]
    ws_pages = torch.empty(Q["nq"], kv, xq["budget"], dtype=torch.int32, device=dev)

    def quest_step():
        pages = M.select_pages(xq["q"], xq["kmax"], xq["kmin"], xq["n_arch"], xq["page"], xq["budget"])
        M.attend_pages(xq["q"], xq["qpos"], xq["keys"], xq["values"], xq["n_arch"], xq["page"], pages,
                       xq["win_keys"], xq["win_values"], xq["kpos"], xq["window"])

    qsteps = max(args.steps, 20)
    t_q = timed(quest_step, qsteps, max(args.warmup, 3))
    q_value = world * Q["nq"] * qsteps / t_q
    bound_bytes = 2 * npages * kv * Q["d"] * 2
    page_bytes = xq["budget"] * Q["page"] * kv * Q["d"] * 2 * 2
    win_bytes = Q["window"] * kv * Q["d"] * 2 * 2
    quest_bytes = bound_bytes + Q["nq"] * page_bytes + win_bytes
    # score kernel alone
    scores = torch.empty(Q["nq"], kv, npages, device=dev)
    t_sel = timed(lambda: M.select_pages(xq["q"], xq["kmax"], xq["kmin"], xq["n_arch"], xq["page"], xq["budget"],
                                         scores=scores), qsteps, 3)
    host_q = xq["q"].cpu().pin_memory()
    host_out = torch.empty(Q["nq"], 1, Q["heads"], Q["d"], pin_memory=True)
    dev_q = torch.empty_like(xq["q"])

    def quest_e2e():
        dev_q.copy_(host_q, non_blocking=True)
        pages = M.select_pages(dev_q, xq["kmax"], xq["kmin"], xq["n_arch"], xq["page"], xq["budget"])
        out = M.attend_pages(dev_q, xq["qpos"], xq["keys"], xq["values"], xq["n_arch"], xq["page"], pages,
                             xq["win_keys"], xq["win_values"], xq["kpos"], xq["window"])
        host_out.copy_(out, non_blocking=True)

    t_q_e2e = timed(quest_e2e, qsteps, 3)
    del xq, scores
    torch.cuda.empty_cache()

    if rank != 0:
        return None
    tr = traffic("gdn_prefill")
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 inputs, fp32 state/accumulation", "data": "synthetic (seeded, BASELINE config distributions)",
        "config": {"workload": "BASELINE config 1: GDN chunked prefill B=4 T=32768 Hk=16 Hv=32 dk=dv=128 chunk=64 per GPU",
                   "global_batch": P["batch"] * world, "seq_len": P["seqlen"],
                   "parallelism": f"(sequence x value-head) shards, {world} GPU(s), no collective",
                   "l2": "inputs 1.6 GB per step, larger than L2 (126 MB)"},
        "roofline": {"bound": "tensor", "achieved": achieved_tf, "peak": pk["tc_sustained"], "unit": "TFLOP/s",
                     "frac": achieved_tf / pk["tc_sustained"], "traffic": tr,
                     "peak_source": f"{pk['src']} bf16 sustained", "algorithmic_bytes": algo_bytes,
                     "hbm_frac": algo_bytes / (t_prefill / args.steps) / 1e9 / pk["hbm"]},
        "e2e": {"value": world * tokens * e2e_steps / t_e2e, "unit": "tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
        "decode": {"metric": "GDN decode steps/s (config 2)", "value": dec_value, "unit": "steps/s",
                   "us_per_step": t_dec / dsteps * 1e6,
                   "roofline": {"bound": "hbm", "achieved": dec_bytes / (t_dec / dsteps) / 1e9, "peak": pk["hbm"],
                                "unit": "GB/s", "frac": dec_bytes / (t_dec / dsteps) / 1e9 / pk["hbm"],
                                "traffic": traffic("gdn_decode")},
                   "e2e": {"value": world * 200 / t_dec_e2e, "unit": "steps/s", "h2d_bytes_per_step": dec_h2d,
                           "d2h_bytes_per_step": host_od.numel() * 2},
                   "gpu_launches": dsteps},
        "quest": {"metric": "Quest q/s (config 3)", "value": q_value, "unit": "q/s",
                  "us_per_batch": t_q / qsteps * 1e6,
                  "roofline": {"bound": "hbm", "achieved": quest_bytes / (t_q / qsteps) / 1e9, "peak": pk["hbm"],
                               "unit": "GB/s", "frac": quest_bytes / (t_q / qsteps) / 1e9 / pk["hbm"],
                               "traffic": traffic("quest_score")},
                  "select_gbps": bound_bytes / (t_sel / qsteps) / 1e9,
                  "e2e": {"value": world * Q["nq"] * qsteps / t_q_e2e, "unit": "q/s",
                          "h2d_bytes_per_step": host_q.numel() * 2, "d2h_bytes_per_step": host_out.numel() * 4},
                  "gpu_launches": 4 * qsteps},
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(samples=1)
    return line


# --------------------------------------------------------------------------------------------
# CPU baseline / reference arm: the oracle (numpy restatement of the reference algorithm)
# --------------------------------------------------------------------------------------------
def _cpu_threads():
    n = len(os.sched_getaffinity(0))
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(n)
    except Exception:  # noqa: BLE001 - threadpoolctl is optional
        pass
    return n


def cpu_baseline(samples=1):
    """Prefill tok/s of the oracle's delta_rule_chunked on a bounded slice of config 1:
    B=1, T=4096 (64 chunks), 32 value heads (q, k repeated from 16 key heads), fp32."""
    import numpy as np
    from oracle import gdn as ogdn
    cores = _cpu_threads()
    rng = np.random.default_rng(0)
    t, hk, hv = 4096, PREFILL["hk"], PREFILL["hv"]

    def unit(shape):
        a = rng.standard_normal(shape, dtype=np.float32)
        return a / np.linalg.norm(a, axis=-1, keepdims=True)

    q, k = unit((1, t, hk, 128)), unit((1, t, hk, 128))
    v = rng.standard_normal((1, t, hv, 128), dtype=np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((1, t, hv))))).astype(np.float32)
    g = (-np.logaddexp(0, -(rng.standard_normal((1, t, hv)) + 2))).astype(np.float32)
    h0 = np.zeros((1, hv, 128, 128), np.float32)
    qe, ke = ogdn.expand_key_heads(q, hv), ogdn.expand_key_heads(k, hv)
    times = []
    for _ in range(samples):
        t0 = time.perf_counter()
        ogdn.delta_rule_chunked(qe, ke, v, g, beta, 128 ** -0.5, h0)
        times.append(time.perf_counter() - t0)
    best = min(times)
    return {"value": t / best, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"oracle delta_rule_chunked (numpy fp32), B=1 T={t} Hv={hv}, {samples} run(s), {best:.2f} s"}


def run_reference(args, rank):
    if rank != 0:
        return None
    base = cpu_baseline(samples=1)  # warm-up sample
    vals = [cpu_baseline(samples=1)["value"] for _ in range(max(1, min(args.steps, 5)))]
    value = statistics.median(vals)
    return {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": len(vals),
            "warmup": 1, "ms_per_step": 4096 / value * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE config distributions)",
            "impl": "reference",
            "config": {"workload": "BASELINE config 1 prefill, bounded CPU sample B=1 T=4096 Hv=32 per step"},
            "cpu_baseline": {**base, "value": value},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank)
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
