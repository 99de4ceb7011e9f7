#!/usr/bin/env python
"""Benchmark of the QwenFieldfare MoE-block hot path on B200.

Headline workload: 40 stacked MoE blocks (hidden 2048,
256 experts top-8 + shared expert, intermediate 512, MLX-affine Q4 g64 experts,
Q8 router), batch-1 decode, seeded synthetic weights (seed = layer index) and
fp16 hidden states.  A step is one token batch through all 40 blocks; the
step's inputs rotate over a pool of 64 token batches, so every step routes to
different experts and streams ~659 MB of weights (> the 126 MB L2).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  N > 1 (torchrun) runs N independent replicas
(the decode block does not shard): value = total tokens / max-over-ranks time.
`--impl reference` times the CPU restatement of the reference's kernels
(oracle/, the "port" baseline: the Swift/Metal reference cannot run here).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen-fieldfare_b200"))

N_LAYERS = 40
POOL = 64
ROUTER_BYTES = 256 * 2048 + 2 * 256 * 32 * 2        # 557,056
COEF_BYTES = 2048 + 2 * 32 * 2                      # 2,176
RECORD = 1_769_472
GATE_UP_BYTES = 2 * (524_288 + 2 * 32_768)          # per record: 1,179,648
# the decode kernels' arithmetic: fp16 tensor-core operands (x and the SiLU
# activations), exact Q4 nibbles, fp32 accumulation
DECODE_DTYPE = "fp16 operands (x, SiLU act), fp32 accumulation"
METRIC = "MoE-block tokens/s and achieved HBM GB/s (vs ~8 TB/s) at batch-1 decode and 4K prefill"
PREFILL_T = 4096
EP_T = 16384
HIDDEN, INTER, TOPK = 2048, 512, 8
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# roofline kernels, from one ncu capture each (profiles/): the one-token decode
# kernel moves 17.15 MB per layer (4-layer capture, scaled by the layers of a
# launch); the prefill block's two grouped-GEMM launches move 605 + 512 MB.
DECODE_TRAFFIC_PER_LAYER = 17.15e6
PREFILL_GEMM_TRAFFIC = 1117e6


def gemm_flops(T: int):
    """(routed, shared) FLOPs of the gate/up + down expert GEMMs for T tokens."""
    per_row = 2 * (2 * INTER * HIDDEN + HIDDEN * INTER)
    return float(T * TOPK * per_row), float(T * per_row)


def zipf_bias(seed: int = 3, s: float = 1.1):
    """Harness logit bias: expert popularity ~ Zipf(s) over a seeded permutation of ids."""
    import numpy as np
    rng = np.random.default_rng(seed)
    order = rng.permutation(256)
    p = 1.0 / np.arange(1, 257) ** s
    bias = np.empty(256, np.float32)
    bias[order] = np.log(p / p.max()).astype(np.float32)
    return bias


def cache_trace(n_tokens: int, layers: int, seed: int = 1, s: float = 1.2, reuse: int = 5,
                p_reuse: float = 0.7):
    """Routing of the cached-decode stream: per layer, expert
    popularity ~ Zipf(s) over a seeded permutation of ids; with probability p_reuse a
    token re-uses `reuse` of the previous token's 8 experts at that layer.  Returns
    idx [n_tokens, layers, 8] int32 and routing weights [n_tokens, layers, 8]."""
    import numpy as np
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, 257) ** s
    p /= p.sum()
    perms = [rng.permutation(256) for _ in range(layers)]
    idx = np.zeros((n_tokens, layers, 8), np.int32)
    for t in range(n_tokens):
        for l in range(layers):
            chosen = []
            if t > 0 and rng.random() < p_reuse:
                chosen = [int(e) for e in rng.choice(idx[t - 1, l], reuse, replace=False)]
            while len(chosen) < 8:
                for r in rng.choice(256, 16, p=p):
                    e = int(perms[l][r])
                    if e not in chosen and len(chosen) < 8:
                        chosen.append(e)
            idx[t, l] = chosen
    w = rng.random((n_tokens, layers, 8)).astype(np.float32) + 0.05
    w /= w.sum(-1, keepdims=True)
    return idx, w


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=N_LAYERS)
    ap.add_argument("--no-extras", action="store_true", help="skip the T=8/32/64 lines")
    ap.add_argument("--no-prefill", action="store_true", help="skip the 4096-token prefill block")
    ap.add_argument("--prefill-only", action="store_true",
                    help="measure only the prefill block (profiling runs); value = its tokens/s")
    ap.add_argument("--prefill-tokens", type=int, default=PREFILL_T)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cache-stream", action="store_true",
                    help="skip the cached-decode stream (BASELINE configs[4])")
    ap.add_argument("--cache-only", action="store_true",
                    help="only the cached-decode stream; prints its own line")
    ap.add_argument("--cache-tokens", type=int, default=512)
    ap.add_argument("--cache-slots", type=int, default=2183)
    ap.add_argument("--cache-policy", choices=["lru", "slru", "both"], default="both",
                    help="cache policy of the cached-decode stream (both: LRU, then SLRU)")
    ap.add_argument("--no-ep", action="store_true",
                    help="skip the expert-parallel block (BASELINE configs[3])")
    ap.add_argument("--lm-head-only", action="store_true",
                    help="only the Q4 LM head (248,320 x 2,048, one token); prints its own line")
    ap.add_argument("--ep-only", action="store_true",
                    help="only the expert-parallel block; prints its own line")
    ap.add_argument("--ep-tokens", type=int, default=EP_T)
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock, its maximum, power and the throttle reasons, sampled every
    `period_s` by a reader thread on NVML (read-only queries) from start() to
    stop().  The GPU is found by its PCI bus id, so CUDA_VISIBLE_DEVICES does
    not matter.  Falls back to an nvidia-smi subprocess read line by line."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int, period_s: float = 0.02):
        import threading
        self.rows = []  # (sm_mhz, sm_max_mhz, power_w, [reasons])
        self.period = period_s
        self.err = None
        self._stop = threading.Event()
        self._nvml = None
        self._proc = None
        try:
            import pynvml as N
            import torch
            N.nvmlInit()
            pr = torch.cuda.get_device_properties(device)
            want = (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
            self._h = None
            for i in range(N.nvmlDeviceGetCount()):
                h = N.nvmlDeviceGetHandleByIndex(i)
                pci = N.nvmlDeviceGetPciInfo(h)
                if (pci.domain, pci.bus, pci.device) == want:
                    self._h = h
                    break
            if self._h is None:
                raise RuntimeError("no NVML device with PCI id %s" % (want,))
            self._nvml = N
            self.source = "nvml"
        except Exception as e:  # no NVML: nvidia-smi, read line by line
            self.err = repr(e)
            self.source = "nvidia-smi"
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    def _sample_nvml(self):
        N, h = self._nvml, self._h
        sm = N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)
        smax = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
        try:
            pw = N.nvmlDeviceGetPowerUsage(h) / 1000.0
        except Exception:
            pw = None
        try:
            bits = N.nvmlDeviceGetCurrentClocksEventReasons(h)
        except Exception:
            bits = N.nvmlDeviceGetCurrentClocksThrottleReasons(h)
        self.rows.append((float(sm), float(smax), pw,
                          [k for k, b in self.REASONS.items() if bits & b]))

    def _run(self):
        if self._nvml is not None:
            while not self._stop.is_set():
                try:
                    self._sample_nvml()
                except Exception as e:
                    self.err = repr(e)
                    return
                self._stop.wait(self.period)
            return
        import torch
        try:
            bus = torch.cuda.get_device_properties(torch.cuda.current_device())
            sel = "%08X:%02X:%02X.0" % (bus.pci_domain_id, bus.pci_bus_id, bus.pci_device_id)
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-i", sel, "-lms", str(max(int(self.period * 1000), 20))],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True, bufsize=1)
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for line in self._proc.stdout:
                if self._stop.is_set():
                    break
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 7 and p[0].replace(".", "").isdigit():
                    pw = float(p[2]) if p[2].replace(".", "").isdigit() else None
                    self.rows.append((float(p[0]), float(p[1]), pw,
                                      [names[i] for i in range(4) if p[3 + i] == "Active"]))
        except Exception as e:
            self.err = repr(e)

    def stop(self):
        self._stop.set()
        if self._proc is not None:
            self._proc.terminate()
        self._t.join(timeout=5)
        if self._nvml is not None:
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass
        rows = list(self.rows)
        out = {"source": self.source, "samples": len(rows), "period_ms": self.period * 1e3}
        if not rows:
            out.update({"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": self.err})
            return out
        out["sm_mhz"] = statistics.median(r[0] for r in rows)
        out["sm_min_mhz"] = min(r[0] for r in rows)
        out["sm_max_mhz"] = max(r[1] for r in rows)
        pws = [r[2] for r in rows if r[2] is not None]
        out["power_w_max"] = max(pws) if pws else None
        out["reasons"] = sorted({x for r in rows for x in r[3]})
        return out


# ------------------------------------------------------------------ reference arm
def oracle_stack(layers: int, threads: int):
    """The CPU oracle's copy of the headline model: `layers` MoE layers with the
    bench's seeds (seed = layer index), all 256 expert records of every layer
    resident in host memory (~0.45 GB per layer), generated by `threads`
    workers (the generator releases the GIL)."""
    from concurrent.futures import ThreadPoolExecutor
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    def one(l):
        recs = np.empty((256, RECORD), np.uint8)
        for e in range(256):
            O.lib().qfo_synth_expert_record(l, l, e, 0, recs[e].ctypes.data)
        return O.OracleLayer(O.synth_router(l, l), O.synth_coef(l, l),
                             O.synth_record(l, l, 256), recs)

    with ThreadPoolExecutor(max_workers=max(1, threads)) as ex:
        return list(ex.map(one, range(layers)))


def oracle_step(olayers, x16, threads: int):
    """One step of the stack on the CPU oracle, as qf_moe_stack_forward chains
    it: block l reads x_l and adds its output to the residual h_l; then
    h_{l+1} = out_l and x_{l+1} = fp16(RMSNorm(out_l)) (eps 1e-6)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    x, h = x16, None
    for L in olayers:
        h = O.block(L, x, residual=h, threads=threads)["out"]
        x = O.rmsnorm_to_f16(h, 1e-6)
    return h


def cpu_decode_rate(seconds: float, threads: int, layers: int):
    """cpu_baseline leg: the CPU oracle (restatement of the reference kernels)
    on a bounded sample of the headline workload: whole 40-layer batch-1 steps,
    as many as fit in ~`seconds` (at least one), on `threads` host threads."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    olayers = oracle_stack(layers, threads)
    xs = O.synth_hidden(0, 0, 8)
    oracle_step(olayers, xs[:1], threads)  # warm
    n = 0
    t0 = time.perf_counter()
    while n == 0 or time.perf_counter() - t0 < seconds:
        oracle_step(olayers, xs[n % 8: n % 8 + 1], threads)
        n += 1
    dt = time.perf_counter() - t0
    del olayers
    return n / dt, n, dt / n


def run_reference(args, rank):
    """`--impl reference`: the reference's algorithm for this path on the host
    cores.  The Swift/Metal reference cannot run here (no Swift, Metal or
    Apple GPU), so its CPU restatement (oracle/, kind "port") stands in.  Each
    step is the headline step: one batch-1 token through all `layers` blocks
    chained with the RMSNorm, weights resident in host memory, every thread
    of the box.  Rank 0 only; the other ranks exit without work."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = os.cpu_count() or 1
    t_build = time.perf_counter()
    olayers = oracle_stack(args.layers, threads)
    build_s = time.perf_counter() - t_build
    xs = O.synth_hidden(1000, 0, POOL)  # the headline's seeded token pool (rank 0)
    b = args.batch
    for i in range(args.warmup):
        oracle_step(olayers, xs[(i * b) % POOL: (i * b) % POOL + b], threads)
    t0 = time.perf_counter()
    for i in range(args.steps):
        j = ((args.warmup + i) * b) % POOL
        oracle_step(olayers, xs[j: j + b], threads)
    dt = time.perf_counter() - t0
    ms = dt / max(args.steps, 1) * 1e3
    value = b / (ms / 1e3)
    sample = (f"{args.steps} timed steps, each {b} token(s) through all {args.layers} MoE blocks "
              f"(seed = layer index, all 256 experts resident in host memory, RMSNorm between "
              f"blocks) on the CPU oracle; no extrapolation; weights built in {build_s:.1f} s "
              f"outside the timed region")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (reference order, fp32 activations)",
        "data": "synthetic (seeded weights, seed = layer index; fp16 hidden N(0,1) RMS-normalised)",
        "config": {"workload": f"{args.layers} stacked MoE blocks, batch-{b} decode (BASELINE configs[1])",
                   "batch_tokens": b, "layers": args.layers},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "timing": "time.perf_counter around the timed steps",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)

    import numpy as np
    import torch
    import qfmoe as Q

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    ctx = Q.MoEContext(local)
    hbm_peak, _, peak_kind = peaks()

    layers = [Q.MoELayerWeights.synth(ctx, seed=l, layer=l) for l in range(args.layers)]
    plan = Q.StackPlan(layers)
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def measure(T: int, steps: int, warmup: int, profile: bool, e2e: bool = False):
        # T <= 8 runs one persistent kernel per step (the whole stack); T = 9..64
        # (resident bank) runs the grouped path per block: router, plan (+ top-8
        # up to 32 tokens, a separate top-k launch above), gather, the gate/up and
        # down tcgen05 GEMMs, combine; the gate/up GEMM streams the most bytes
        prof_kernel = "fused" if T <= 8 else "gate_up"
        # clocks sampled over this whole measurement (routing pass, warm-up, timed
        # steps): the timed region alone can be a few milliseconds long
        clocks = ClockSampler(local) if (profile and rank == 0) else None
        pool = torch.stack([Q.synth_hidden(1000 + rank, i * T, T) for i in range(POOL)])
        pool_dev = pool.to(dev)
        x_static = torch.empty((T, 2048), dtype=torch.float16, device=dev)
        out_static = torch.empty((T, 2048), dtype=torch.float32, device=dev)
        ws = ctx.workspace(T)
        idx_all = torch.empty((POOL, args.layers, T, 8), dtype=torch.int32, device=dev)
        # routing of every pool entry -> unique experts per layer (algorithmic bytes)
        for i in range(POOL):
            x_static.copy_(pool_dev[i])
            _, idx, _ = Q.stack_forward(ctx, plan, x_static, out=out_static, return_routing=True,
                                        workspace=ws)
            idx_all[i] = idx
        idx_np = idx_all.cpu().numpy()
        uniq = np.array([[len(np.unique(idx_np[i, l])) for l in range(args.layers)]
                         for i in range(POOL)])
        step_bytes = float(np.mean(
            args.layers * (ROUTER_BYTES + COEF_BYTES + RECORD) + uniq.sum(1) * RECORD))

        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            Q.stack_forward(ctx, plan, x_static, out=out_static, workspace=ws)  # warm on stream
            torch.cuda.synchronize()
            if profile:
                Q.profile_begin(ctx, prof_kernel, 4 * args.layers)
            with torch.cuda.graph(g, stream=s):
                Q.stack_forward(ctx, plan, x_static, out=out_static, workspace=ws)
        torch.cuda.synchronize()

        host_pool = pool.pin_memory() if e2e else None
        host_out = torch.empty((T, 2048), dtype=torch.float32).pin_memory() if e2e else None

        def step(i):
            if e2e:
                x_static.copy_(host_pool[i % POOL], non_blocking=True)
            else:
                x_static.copy_(pool_dev[i % POOL], non_blocking=True)
            g.replay()
            if e2e:
                host_out.copy_(out_static, non_blocking=True)

        with torch.cuda.stream(s):
            for i in range(warmup):
                step(i)
        barrier()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        # e2e: an event after every step gives the per-token latency (input upload,
        # the 40 blocks, output read-back); the kernel-only pass records none
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps)] if e2e else None
        with torch.cuda.stream(s):
            barrier()
            ev0.record(s)
            for i in range(steps):
                step(warmup + i)
                if evs is not None:
                    evs[i].record(s)
            ev1.record(s)
        ev1.synchronize()
        barrier()
        ms = ev0.elapsed_time(ev1) / steps
        clk = clocks.stop() if clocks else None
        ms_max = max_over_ranks(ms)
        res = {"T": T, "ms_per_step": ms_max, "tokens_per_s_rank": T / (ms / 1e3),
               "tokens_per_s": world * T / (ms_max / 1e3), "step_bytes": step_bytes,
               "step_gbs": step_bytes / (ms / 1e3) / 1e9, "clocks": clk}
        if evs is not None:
            from qfmoe.telemetry import LatencySummary
            lat = [ev0.elapsed_time(evs[0])] + [evs[i - 1].elapsed_time(evs[i])
                                                for i in range(1, steps)]
            res["latency"] = LatencySummary.summarize(lat).as_dict()
        if profile:
            last = (warmup + steps - 1) % POOL
            try:
                tot_ms, n = Q.profile_end(ctx)
            except Q.QfError:
                # graph-captured timing nodes unavailable: time the same step eagerly
                x_static.copy_(pool_dev[last])
                Q.profile_begin(ctx, prof_kernel, 4 * args.layers)
                Q.stack_forward(ctx, plan, x_static, out=out_static, workspace=ws)
                tot_ms, n = Q.profile_end(ctx)
                res["kernel_timing"] = "eager replay of the last timed step"
            if prof_kernel == "fused":
                kbytes = float(args.layers * (ROUTER_BYTES + COEF_BYTES + RECORD)
                               + uniq[last].sum() * RECORD)
            else:
                kbytes = float(np.mean((uniq[last] + 1) * GATE_UP_BYTES))
            res["kernel"] = (("k_fused1" if T == 1 else "k_fused") if prof_kernel == "fused"
                             else "k_grouped<0> (gate/up)")
            res["kernel_ms"] = tot_ms / max(n, 1)
            res["kernel_launches"] = n
            res["kernel_bytes"] = kbytes
            res["launches_per_step"] = 1 if prof_kernel == "fused" else (6 if T <= 32 else 7) * args.layers
        del g
        return res

    def measure_block0(steps: int, warmup: int):
        """one MoE block, batch 1, x = seed-0 fp16 hidden.
        Cold: each replay runs 40 single-block launches over the 40 layers' weight
        sets in turn (16.5 MB each, 659 MB per pass > L2), so every block streams
        its weights from HBM.  Warm: 40 launches of layer 0 (seed 0), whose
        16.5 MB stay in L2.  One launch of the one-token kernel per block; CUDA
        graph replay, CUDA events."""
        x = Q.synth_hidden(0, 0, 1).to(dev)
        out = torch.empty((1, 2048), dtype=torch.float32, device=dev)
        ws = ctx.workspace(1)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        res = {}
        for kind, seq in (("cold", list(range(args.layers))), ("warm", [0] * args.layers)):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                Q.block_forward(ctx, layers[seq[0]], x, out=out)
                torch.cuda.synchronize()
                with torch.cuda.graph(g, stream=s):
                    for l in seq:
                        Q.block_forward(ctx, layers[l], x, out=out)
                for _ in range(warmup):
                    g.replay()
                ev0 = torch.cuda.Event(enable_timing=True)
                ev1 = torch.cuda.Event(enable_timing=True)
                ev0.record(s)
                for _ in range(steps):
                    g.replay()
                ev1.record(s)
            ev1.synchronize()
            us = ev0.elapsed_time(ev1) * 1e3 / (steps * len(seq))
            nbytes = ROUTER_BYTES + COEF_BYTES + 9 * RECORD
            gbs = nbytes / (us / 1e6) / 1e9
            res[kind] = {"us_per_block": us, "tokens_per_s": 1e6 / us, "achieved_gbs": gbs,
                         "frac_of_hbm": gbs / hbm_peak, "launches": steps * len(seq)}
            del g
        ctx.check()
        return res

    def measure_prefill(T: int, steps: int, warmup: int):
        """One MoE block over T tokens with Zipf(1.1) routing."""
        L = layers[0]
        bias = torch.from_numpy(zipf_bias()).to(dev)
        xs = [Q.synth_hidden(2000 + rank, i * T, T).to(dev) for i in range(4)]
        out = torch.empty((T, 2048), dtype=torch.float32, device=dev)
        for i in range(warmup):
            Q.block_forward(ctx, L, xs[i % 4], logit_bias=bias, out=out)
        _, idx, _ = Q.block_forward(ctx, L, xs[0], logit_bias=bias, out=out, return_routing=True)
        cnt = np.bincount(idx.cpu().numpy().reshape(-1), minlength=256)
        barrier()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record()
        for i in range(steps):
            Q.block_forward(ctx, L, xs[i % 4], logit_bias=bias, out=out)
        ev1.record()
        ev1.synchronize()
        ms = ev0.elapsed_time(ev1) / steps
        barrier()
        ms_max = max_over_ranks(ms)
        kernels = {}
        for name in ("router", "topk", "gate_up", "down", "combine"):
            Q.profile_begin(ctx, name, 64)
            for i in range(8):
                Q.block_forward(ctx, L, xs[i % 4], logit_bias=bias, out=out)
            tot, n = Q.profile_end(ctx)
            kernels[name] = tot / max(n, 1)
        ctx.check()
        routed, shared = gemm_flops(T)
        gemm_ms = kernels["gate_up"] + kernels["down"]
        return {"T": T, "ms_per_block": ms_max, "tokens_per_s": world * T / (ms_max / 1e3),
                "kernel_ms": kernels, "gemm_ms": gemm_ms,
                "routed_gemm_flops": routed, "shared_gemm_flops": shared,
                "rows_per_expert": {"max": int(cnt.max()), "min": int(cnt.min()), "mean": float(cnt.mean())}}

    def measure_cache_stream(n_tokens: int, slots: int, policies):
        """n_tokens batch-1 decode tokens through all layers with
        routed experts served from `slots` HBM slots, backed by every layer-expert
        record in pinned host memory, once per cache policy (one host tier).  Each
        run starts from a cold cache and is timed end to end through
        qf_moe_stream_step (planning, host->HBM record copies, the block stack,
        and each token's hidden-state upload and output read-back)."""
        from qfmoe.cache import ExpertCache, HostTier, stream_step
        from qfmoe.telemetry import LatencySummary, cache_hit_rate
        idx, w = cache_trace(n_tokens, args.layers, seed=1)
        host = torch.empty((args.layers * 256, RECORD), dtype=torch.uint8, pin_memory=True)
        for l, L in enumerate(layers):
            host[l * 256:(l + 1) * 256].copy_(L.bank)
        torch.cuda.synchronize()
        tier = HostTier(local, slots, host)
        xs = torch.stack([Q.synth_hidden(3000 + rank, t, 1) for t in range(n_tokens)]).pin_memory()
        outs = torch.empty((n_tokens, 1, 2048), dtype=torch.float32).pin_memory()
        x_dev = torch.empty((1, 2048), dtype=torch.float16, device=dev)
        out_dev = torch.empty((1, 2048), dtype=torch.float32, device=dev)
        ws = ctx.workspace(1)
        results = []
        for policy in policies:
            cache = ExpertCache(slots, layer_count=args.layers, policy=policy)
            # warm-up on other tokens, then restart from a cold cache
            wi, ww = cache_trace(8, args.layers, seed=101)
            for t in range(8):
                x_dev.copy_(xs[t], non_blocking=True)
                stream_step(ctx, cache, tier, plan, wi[t], ww[t], x_dev, None, out_dev, 1e-6,
                            workspace=ws)
            torch.cuda.synchronize()
            cache.clear()
            cache.reset_metrics()
            t0 = tier.stats()
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_tokens + 1)]
            barrier()
            evs[0].record()
            for t in range(n_tokens):
                x_dev.copy_(xs[t], non_blocking=True)
                stream_step(ctx, cache, tier, plan, idx[t], w[t], x_dev, None, out_dev, 1e-6,
                            workspace=ws)
                outs[t].copy_(out_dev, non_blocking=True)
                evs[t + 1].record()
            evs[-1].synchronize()
            ms = evs[0].elapsed_time(evs[-1])
            ctx.check()
            barrier()
            ms_max = max_over_ranks(ms)
            m = cache.metrics_snapshot()
            t1 = tier.stats()
            copied = t1["bytes"] - t0["bytes"]
            lat = [evs[t].elapsed_time(evs[t + 1]) for t in range(n_tokens)]
            res = {"tokens": n_tokens, "slots": slots, "policy": policy, "ms_total": ms_max,
                   "tokens_per_s": world * n_tokens / (ms_max / 1e3),
                   "ms_per_token": ms_max / n_tokens,
                   "latency": LatencySummary.summarize(lat).as_dict(),
                   "hits": m["hits"], "misses": m["misses"], "evictions": m["evictions"],
                   "hit_rate": cache_hit_rate(m), "misses_per_token": m["misses"] / n_tokens,
                   "fetched_gib": m["fetched_bytes"] / 2**30,
                   "layer_hit_rates_pct": [round(r, 1) for r in cache.layer_hit_rates()],
                   "h2d_record_bytes": copied, "h2d_gbs": copied / (ms / 1e3) / 1e9,
                   "gpu_launches": n_tokens}
            if rank == 0:
                # the planner's hits against the oracle's restatement on the same trace
                sys.path.insert(0, os.path.join(ROOT, "oracle"))
                import oracle as O
                ref = (O.OracleLRU(slots, args.layers) if policy == "lru"
                       else O.OracleCache(slots, 0.25, args.layers))
                for t in range(n_tokens):
                    for l in range(args.layers):
                        ref.acquire(l, idx[t, l])
                ref_hits = ref.hits if policy == "lru" else ref.metrics()["hits"]
                res["oracle_hits"] = int(ref_hits)
                res["hits_match_oracle"] = int(ref_hits) == m["hits"]
            cache.close()
            results.append(res)
        tier.close()
        del host
        return results

    def measure_ep(T_total: int, steps: int, warmup: int):
        """one MoE block over T_total tokens split evenly over
        the ranks, routed experts' gate/up sharded 256/world per GPU, uniform-random
        top-8 (seeded), rows exchanged by the EP kernels over NVLink.  Timed in
        both modes: down-at-home (the headline: owners return fp16 activation rows,
        each rank runs the down projection of its own tokens with all 256 experts)
        and fully sharded (owners also run the down projection and return fp32
        result rows)."""
        T = T_total // world
        ep = Q.ExpertParallel(ctx, rank, world, max_tokens=T)
        local = ep.local_layer(0, 0)
        full = layers[0]
        rng = np.random.default_rng(5000 + rank)
        idx = np.argsort(rng.random((T, 256)), axis=1)[:, :8].astype(np.int32)
        w = rng.random((T, 8)).astype(np.float32) + 0.05
        w /= w.sum(1, keepdims=True)
        idx_d = torch.from_numpy(idx).to(dev)
        w_d = torch.from_numpy(w).to(dev)
        xs = [Q.synth_hidden(4000 + rank, i * T, T).to(dev) for i in range(2)]
        out = torch.empty((T, 2048), dtype=torch.float32, device=dev)

        def timed(dah: bool) -> float:
            ep.set_down_at_home(dah)
            lay = full if dah else local
            for i in range(warmup):
                ep.forward(lay, xs[i % 2], topk_idx=idx_d, topk_w=w_d, out=out)
            ctx.check()
            barrier()
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
            for i in range(steps):
                ep.forward(lay, xs[i % 2], topk_idx=idx_d, topk_w=w_d, out=out)
            ev1.record()
            ev1.synchronize()
            ms = ev0.elapsed_time(ev1) / steps
            barrier()
            return max_over_ranks(ms)

        ms_sharded = timed(False)
        ms_max = timed(True)  # down-at-home, the headline; the breakdown below is of it
        kernels = {}
        for name in ("router", "dispatch", "gate_up", "down", "combine"):
            Q.profile_begin(ctx, name, 64)
            for i in range(6):
                ep.forward(full, xs[i % 2], topk_idx=idx_d, topk_w=w_d, out=out)
            tot, n = Q.profile_end(ctx)
            kernels[name] = max_over_ranks(tot / max(n, 1))
        ctx.check()
        # token rows this rank sends to other ranks (4 KB each, once per owner)
        # and routed rows whose results come back (1 KB activations here, 8 KB
        # fp32 rows in the sharded mode)
        owner = idx // ep.experts_per_rank
        sent_remote = sum(len(set(o.tolist()) - {rank}) for o in owner)
        routed_remote = int((owner != rank).sum())
        # correctness at this world size: every rank's EP output for all of its
        # tokens against the single-GPU block (all 256 experts resident on this
        # GPU, same tokens, same routing), bit for bit; min over ranks
        equal = True
        for k in range(2):
            ref = Q.block_forward(ctx, layers[0], xs[k], topk_idx=idx_d, topk_w=w_d)
            for dah in (True, False):  # both modes, the same reference
                ep.set_down_at_home(dah)
                got = ep.forward(full if dah else ep.local_layer(0, 0), xs[k], topk_idx=idx_d, topk_w=w_d,
                                 out=out).clone()
                torch.cuda.synchronize()
                equal = equal and bool(torch.equal(got, ref))
        ctx.check()
        flag = torch.tensor([1 if equal else 0, T * 4], dtype=torch.int64, device=dev)
        if dist is not None:
            f_min = flag[:1].clone()
            dist.all_reduce(f_min, op=dist.ReduceOp.MIN)
            n_sum = flag[1:].clone()
            dist.all_reduce(n_sum, op=dist.ReduceOp.SUM)
            flag = torch.cat([f_min, n_sum])
        ep.close()
        # the one-GPU figure of the same run: all T_total tokens through the block
        # on this GPU with all 256 experts (uniform-random top-8 as above)
        rng1 = np.random.default_rng(6000)
        idx1 = torch.from_numpy(np.argsort(rng1.random((T_total, 256)), axis=1)[:, :8]
                                .astype(np.int32)).to(dev)
        w1 = torch.from_numpy(rng1.random((T_total, 8)).astype(np.float32) + 0.05).to(dev)
        w1 /= w1.sum(1, keepdim=True)
        x1 = Q.synth_hidden(4500, 0, T_total).to(dev)
        out1 = torch.empty((T_total, 2048), dtype=torch.float32, device=dev)
        for _ in range(3):
            Q.block_forward(ctx, layers[0], x1, topk_idx=idx1, topk_w=w1, out=out1)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        n1 = max(steps // 2, 3)
        for _ in range(n1):
            Q.block_forward(ctx, layers[0], x1, topk_idx=idx1, topk_w=w1, out=out1)
        e1.record()
        e1.synchronize()
        ms1 = max_over_ranks(e0.elapsed_time(e1) / n1)
        del out1, x1
        routed, shared = gemm_flops(T_total)
        tps = T_total / (ms_max / 1e3)
        tps1 = T_total / (ms1 / 1e3)
        return {"T_total": T_total, "T_rank": T, "ms_per_block": ms_max,
                "tokens_per_s": tps, "kernel_ms": kernels,
                "sharded_ms_per_block": ms_sharded, "sharded_tokens_per_s": T_total / (ms_sharded / 1e3),
                "gemm_flops_per_rank": (routed + shared) / world,
                "remote_rows_sent_rank0": sent_remote,
                "dispatch_remote_bytes_rank0": sent_remote * 4096,
                "return_remote_bytes_rank0": routed_remote * 1024,
                "sharded_return_remote_bytes_rank0": routed_remote * 8192,
                "ep_equal": bool(flag[0].item() == 1), "ep_checked_tokens": int(flag[1].item()),
                "one_gpu_ms_per_block": ms1, "one_gpu_tokens_per_s": tps1,
                "efficiency_vs_one_gpu": tps / (world * tps1)}

    def measure_lm_head(steps: int, warmup: int):
        """Q4 LM head of the 248,320-row vocabulary for one token row (the last
        GEMV of a decode step): 286 MB of weights, larger than L2."""
        rows = 248_320
        gen = torch.Generator(device=dev).manual_seed(5)
        w = torch.randint(0, 256, (rows, 1024), dtype=torch.uint8, device=dev, generator=gen)
        sc = torch.randn((rows, 32), device=dev, generator=gen).abs() * 0.01 + 1e-3
        s, b = sc.half().view(torch.int16), (-8 * sc).half().view(torch.int16)
        x = torch.randn((1, 2048), device=dev, generator=gen)
        x = x / x.pow(2).mean().sqrt()
        out = torch.empty((1, rows), device=dev)
        for _ in range(warmup):
            Q.lm_head(ctx, w, s, b, x, out=out)
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(steps):
            Q.lm_head(ctx, w, s, b, x, out=out)
        ev1.record()
        ev1.synchronize()
        ctx.check()
        ms = ev0.elapsed_time(ev1) / steps
        nbytes = rows * (1024 + 64 + 64) + 2048 * 4 + rows * 4
        gbs = nbytes / (ms / 1e3) / 1e9
        return {"workload": "Q4 LM head, 248,320 x 2,048, one fp32 token row, fp16 scales "
                            "(deltanet.metal:1897-1919 as dispatched at QwenQ4ActiveExpertStreamingRunner.swift:1393-1400)",
                "ms_per_token": ms, "launches": steps,
                "roofline": {"bound": "hbm", "kernel": "k_lm_head", "achieved": gbs, "peak": hbm_peak,
                             "unit": "GB/s", "frac": gbs / hbm_peak, "peak_kind": peak_kind,
                             "bytes_per_launch": nbytes}}

    def ep_line(r):
        _, tc_peak, tc_kind = peaks()
        gemm_ms = r["kernel_ms"]["gate_up"] + r["kernel_ms"]["down"]
        tf = r["gemm_flops_per_rank"] / (gemm_ms / 1e3) / 1e12
        return {
            "workload": f"one MoE block over {r['T_total']} tokens ({r['T_rank']} per GPU), routed experts' "
                        f"gate/up sharded {256 // world} per GPU, down projections of each rank's own tokens "
                        "at home (down-at-home mode), uniform-random top-8 (seeded); token rows out and "
                        "activation rows back by the EP kernels over NVLink peer memory (BASELINE configs[3])",
            "n_gpus": world, "tokens_per_s": r["tokens_per_s"], "ms_per_block": r["ms_per_block"],
            "sharded_tokens_per_s": r["sharded_tokens_per_s"],
            "sharded_note": "fully sharded mode (down projections at the owners, fp32 result rows back), "
                            "timed in the same run",
            "kernel_ms_max_over_ranks": r["kernel_ms"],
            "roofline": {"bound": "tensor", "kernel": "k_grouped (gate/up + down, per rank)", "achieved": tf,
                         "peak": tc_peak, "unit": "TFLOP/s", "frac": tf / tc_peak, "peak_kind": tc_kind},
            "dispatch_remote_bytes_rank0": r["dispatch_remote_bytes_rank0"],
            "return_remote_bytes_rank0": r["return_remote_bytes_rank0"],
            "sharded_return_remote_bytes_rank0": r["sharded_return_remote_bytes_rank0"],
            "ep_equal": r["ep_equal"], "ep_checked_tokens": r["ep_checked_tokens"],
            "ep_check": "every rank's output for all of its tokens (two batches, both modes) equals "
                        "the single-GPU block with all 256 experts on the same tokens and routing, "
                        "bit for bit (torch.equal), min over ranks",
            "one_gpu_tokens_per_s": r["one_gpu_tokens_per_s"],
            "efficiency_vs_one_gpu": r["efficiency_vs_one_gpu"],
            "efficiency_note": "strong scaling: tokens/s at this N / (N x the one-GPU block "
                               "over all %d tokens, timed in the same run)" % r["T_total"],
            "timing": "CUDA events on each rank, max over ranks",
        }

    if args.ep_only:
        r = measure_ep(args.ep_tokens, args.steps, max(args.warmup, 3))
        if rank == 0:
            line = ep_line(r)
            print(json.dumps({
                "metric": "expert-parallel MoE-block tokens/s (BASELINE configs[3])",
                "value": r["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": r["ms_per_block"], "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f16 operands, f32 accumulation",
                "data": "synthetic (seeded weights; fp16 hidden N(0,1) RMS-normalised)",
                "config": {"workload": line["workload"]}, "ep": line,
                "gpu_launches": args.steps * 12}), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    def cache_line(c):
        return {
            "workload": f"{c['tokens']} batch-1 decode tokens through {args.layers} MoE blocks, "
                        f"{c['slots']} HBM expert slots ({c['policy'].upper()}) backed by all "
                        f"{args.layers * 256} layer-expert records in pinned host memory; "
                        "per-layer Zipf(1.2) routing with temporal locality (5 of the previous "
                        "token's 8 experts re-used with probability 0.7), seed 1 (BASELINE configs[4])",
            "policy": c["policy"],
            "tokens_per_s": c["tokens_per_s"], "ms_per_token": c["ms_per_token"],
            "latency": c["latency"],
            "hit_rate": c["hit_rate"], "hits": c["hits"], "misses": c["misses"],
            "misses_per_token": c["misses_per_token"], "evictions": c["evictions"],
            "fetched_gib": c["fetched_gib"], "layer_hit_rates_pct": c["layer_hit_rates_pct"],
            "h2d_gbs": c["h2d_gbs"], "h2d_record_bytes": c["h2d_record_bytes"],
            "oracle_hits": c.get("oracle_hits"), "hits_match_oracle": c.get("hits_match_oracle"),
            "timing": "cold cache; CUDA events around the whole stream and after every token, end "
                      "to end through qf_moe_stream_step with per-token hidden upload and output "
                      "read-back; latency percentiles are nearest-rank (QwenLatencySummary)",
        }

    def cache_policies():
        return ["lru", "slru"] if args.cache_policy == "both" else [args.cache_policy]

    if args.lm_head_only:
        lm = measure_lm_head(args.steps, max(args.warmup, 3))
        if rank == 0:
            print(json.dumps({
                "metric": "Q4 LM-head GB/s (248,320 x 2,048, one fp32 token row)",
                "value": lm["roofline"]["achieved"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": lm["ms_per_token"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (uniform Q4 codes, fp16 scales |N(0,0.01)|+1e-3, bias -8 scale)",
                "config": {"workload": lm["workload"]}, "roofline": lm["roofline"],
                "gpu_launches": args.steps}), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    if args.cache_only:
        cs = measure_cache_stream(args.cache_tokens, args.cache_slots, cache_policies())
        if rank == 0:
            c = cs[0]
            print(json.dumps({
                "metric": "cached-decode MoE tokens/s (BASELINE configs[4])", "value": c["tokens_per_s"],
                "unit": "tokens/s", "n_gpus": world, "steps": c["tokens"], "warmup": 8,
                "ms_per_step": c["ms_per_token"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": DECODE_DTYPE,
                "data": "synthetic (seeded weights, seed = layer index; fp16 hidden N(0,1) RMS-normalised)",
                "config": {"workload": cache_line(c)["workload"]},
                "cache_stream": cache_line(c),
                "cache_stream_by_policy": {x["policy"]: cache_line(x) for x in cs},
                "gpu_launches": c["gpu_launches"]}), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    if args.prefill_only:
        pre = measure_prefill(args.prefill_tokens, args.steps, max(args.warmup, 3))
        if rank == 0:
            _, tc_peak, tc_kind = peaks()
            gemm_tf = (pre["routed_gemm_flops"] + pre["shared_gemm_flops"]) / (pre["gemm_ms"] / 1e3) / 1e12
            print(json.dumps({
                "metric": "MoE-block prefill tokens/s (BASELINE configs[2])", "value": pre["tokens_per_s"],
                "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": pre["ms_per_block"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16 operands, f32 accumulation",
                "data": "synthetic (seeded weights; fp16 hidden N(0,1) RMS-normalised)",
                "config": {"workload": f"one MoE block, {pre['T']} tokens, Zipf(1.1) routing"},
                "kernel_ms": pre["kernel_ms"], "rows_per_expert": pre["rows_per_expert"],
                "roofline": {"bound": "tensor", "achieved": gemm_tf, "peak": tc_peak, "unit": "TFLOP/s",
                             "frac": gemm_tf / tc_peak, "peak_kind": tc_kind,
                             "traffic": PREFILL_GEMM_TRAFFIC if pre["T"] == PREFILL_T else None}}), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    head = measure(args.batch, args.steps, args.warmup, profile=True)
    e2e = measure(args.batch, max(args.steps // 2, 1), max(args.warmup, 3), profile=False,
                  e2e=True)
    extras = {}
    if not args.no_extras:
        for T in (8, 32, 64):
            r = measure(T, max(args.steps // 10, 20), 5, profile=False)
            extras[str(T)] = {"tokens_per_s": r["tokens_per_s"], "ms_per_step": r["ms_per_step"],
                              "step_gbs": r["step_gbs"],
                              "step_frac_of_hbm": r["step_gbs"] / hbm_peak}

    pre = None if args.no_prefill else measure_prefill(args.prefill_tokens, 20, 3)
    # the cached stream is a single-GPU configuration (its host tier pins ~18 GB)
    cst = None if (args.no_cache_stream or world > 1) else measure_cache_stream(
        args.cache_tokens, args.cache_slots, cache_policies())
    blk0 = None if args.no_extras else measure_block0(max(args.steps // 4, 5), 3)
    epr = None if args.no_ep else measure_ep(args.ep_tokens, 20, 3)
    lmh = None if args.no_extras else measure_lm_head(50, 5)

    if rank == 0:
        cpu = None
        if world == 1:
            rate, n, per = cpu_decode_rate(args.cpu_seconds, os.cpu_count() or 1, args.layers)
            cpu = {"value": rate, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": f"{n} whole steps (one batch-1 token through all {args.layers} blocks "
                             f"with the RMSNorm between them, {per * 1e3:.0f} ms each) on the CPU "
                             f"oracle, no extrapolation"}
        achieved = head["kernel_bytes"] / (head["kernel_ms"] / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": head["tokens_per_s"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": DECODE_DTYPE,
            "data": "synthetic (seeded weights, seed = layer index; fp16 hidden N(0,1) RMS-normalised)",
            "config": {"workload": f"{args.layers} stacked MoE blocks, batch-{args.batch} decode "
                                   "(BASELINE configs[1])",
                       "batch_tokens": args.batch, "layers": args.layers,
                       "hidden": 2048, "experts": 256, "top_k": 8, "intermediate": 512,
                       "quant": "Q4 g64 experts, Q8 router, fp16 scales",
                       "parallelism": "replicas" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2: each step streams ~%.0f MB of weights and "
                             "the input rotates over %d token batches" % (head["step_bytes"] / 1e6, POOL)},
            "roofline": {"bound": "hbm", "kernel": head["kernel"], "achieved": achieved,
                         "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                         "peak_kind": peak_kind,
                         "traffic": (DECODE_TRAFFIC_PER_LAYER * args.layers
                                     if args.batch == 1 and args.prefill_tokens == PREFILL_T else None),
                         "bytes_per_launch": head["kernel_bytes"],
                         "ms_per_launch": head["kernel_ms"]},
            "step_hbm": {"achieved": head["step_gbs"], "frac": head["step_gbs"] / hbm_peak,
                         "bytes_per_step": head["step_bytes"]},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e["tokens_per_s"], "unit": "tokens/s",
                    "h2d_bytes_per_step": args.batch * 2048 * 2,
                    "d2h_bytes_per_step": args.batch * 2048 * 4,
                    "latency_per_step": e2e["latency"],
                    "latency_note": "per-step (per-token at batch 1) device time between CUDA "
                                    "events, upload + 40 blocks + read-back; nearest-rank "
                                    "percentiles (QwenLatencySummary)"},
            "gpu_launches": args.steps * head["launches_per_step"],
            "clocks": head["clocks"],
            "decode_batches": extras,
        }
        if pre is not None:
            _, tc_peak, tc_kind = peaks()
            gemm_tf = (pre["routed_gemm_flops"] + pre["shared_gemm_flops"]) / (pre["gemm_ms"] / 1e3) / 1e12
            routed_tf = pre["routed_gemm_flops"] / (pre["gemm_ms"] / 1e3) / 1e12
            line["prefill_4k"] = {
                "workload": f"one MoE block, {pre['T']} tokens, Zipf(1.1) expert popularity through the "
                            "harness logit bias (BASELINE configs[2])",
                "tokens_per_s": pre["tokens_per_s"], "ms_per_block": pre["ms_per_block"],
                "kernel_ms": pre["kernel_ms"], "rows_per_expert": pre["rows_per_expert"],
                "roofline": {"bound": "tensor", "kernel": "k_grouped (gate/up + down launches)",
                             "achieved": gemm_tf, "peak": tc_peak, "unit": "TFLOP/s",
                             "frac": gemm_tf / tc_peak, "peak_kind": tc_kind,
                             "flops_per_block": pre["routed_gemm_flops"] + pre["shared_gemm_flops"],
                             "routed_only_tflops": routed_tf, "routed_only_frac": routed_tf / tc_peak,
                             "traffic": PREFILL_GEMM_TRAFFIC if pre["T"] == PREFILL_T else None},
            }
        if cst is not None:
            line["cache_stream"] = cache_line(cst[0])
            line["cache_stream_by_policy"] = {x["policy"]: cache_line(x) for x in cst}
        if blk0 is not None:
            line["config0"] = {
                "workload": "one MoE block, batch 1, seed-0 fp16 hidden (BASELINE configs[0]); "
                            "cold: 40 weight sets in rotation (659 MB per pass > L2); warm: one "
                            "weight set repeated (16.5 MB, L2-resident)",
                "bytes_per_block": ROUTER_BYTES + COEF_BYTES + 9 * RECORD,
                "cold": blk0["cold"], "warm": blk0["warm"], "peak": hbm_peak,
                "peak_kind": peak_kind, "kernel": "k_fused1 (one launch per block)"}
        if epr is not None:
            line["ep_16k"] = ep_line(epr)
        if lmh is not None:
            line["lm_head"] = lmh
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
