"""Benchmark of the Envision dense-linear hot path on B200 (one JSON line on rank 0).

Workload (the configuration the headline metric is quoted on): the linears of
one FLUX2-Klein-4B-shaped double-stream block at 1024x1024, M = 4096 image + 512 text tokens =
4608, hidden 3072:

    qkv      [4608, 3072] -> 9216   + bias
    out      [4608, 3072] -> 3072   + bias
    gate_up  [4608, 3072] -> 18432  + bias, SiLU-gate epilogue -> [4608, 9216]
    down     [4608, 9216] -> 3072   + bias   (input: the gate_up output)
    adaln    [1, 3072]    -> 18432  + bias   (adaptive-norm modulation, skinny M)

X ~ N(0,1) fp32, W = bf16(0.02 N(0,1)), b = 0.01 N(0,1) fp32, all synthetic and seeded (no model
weights exist in this environment).  One step = the five linears.  The working set (weights
358 MB + activations) exceeds the 126 MB L2, so no flush is needed between steps.

Arms:
  (default)          libenvgemm through its C ABI.  `value` = device-resident throughput
                     (TFLOP/s, whole job); `e2e` = the same through host buffers (pinned), every
                     step copying its inputs H2D and its outputs D2H.  With N > 1 GPUs the weights
                     are N-split by output column and every output is all-gathered over NCCL
                     (strong scaling; the gather is part of the timed step).
  --impl reference   the reference's own CPU GEMM (src/sgemm2.cpp compiled from the reference
                     tree into oracle/_ref, else the C++ restatement of its Pascal qgemm) on the
                     host cores, on a bounded M-slice of the same workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

M_TOK = 4096 + 512
HID = 3072
MLP = 9216
LINEARS = [
    # name, M, K, N (weight rows), kind
    ("qkv", M_TOK, HID, 3 * HID, "bias"),
    ("out", M_TOK, HID, HID, "bias"),
    ("gate_up", M_TOK, HID, 2 * MLP, "silu_gate"),
    ("down", M_TOK, MLP, HID, "bias"),
    ("adaln", 1, HID, 6 * HID, "bias"),
]
FLOPS_PER_STEP = float(sum(2 * M * K * N for _, M, K, N, _ in LINEARS))
WORKLOAD = ("BASELINE config 2: FLUX2-Klein-4B double-stream block linears, M=4608 (4096 img + 512 txt), "
            "hidden 3072: qkv 3072->9216, out 3072->3072, gate_up 3072->18432 (SiLU-gate), down 9216->3072, "
            "adaLN 3072->18432 at M=1; all with fp32 bias")
METRIC = "block_linear_tflops"
UNIT = "TFLOP/s"
# DRAM bytes per k1_gemm launch of this workload, from one ncu capture (profiles/k1_gemm_config2.md);
# None until a capture of the current kernel exists.
K1_TRAFFIC_BYTES_PER_LAUNCH = None


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


# ---------------------------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        busy = [s for s in sm if mx and s > 0.3 * mx] or sm
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------------------------
def dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------
def run_ours(args, world, rank, local):
    import torch
    import torch.distributed as dist

    from invision_b200 import envg
    from invision_b200.nsplit import gather_columns, shard_bounds

    torch.cuda.set_device(local)
    envg.init(local)
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev)

    weights, biases, shards = {}, {}, {}
    for i, (name, M, K, N, kind) in enumerate(LINEARS):
        if name not in ACTIVE:
            continue
        gen.manual_seed(1000 + i)
        w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        b = torch.randn(N, generator=gen, device=dev) * 0.01
        w_host = w.view(torch.int16).cpu().numpy().view(np.uint16)
        layout = envg.LAYOUT_GATE_UP if kind == "silu_gate" else envg.LAYOUT_PLAIN
        if world == 1:
            weights[name] = envg.Weight(w_host, layout=layout)
            biases[name] = b
            shards[name] = (0, N if kind != "silu_gate" else N // 2, None)
        else:
            half = N // 2 if kind == "silu_gate" else N
            n0, n1, per = shard_bounds(half, world, rank, 128)
            weights[name] = envg.Weight(w_host, layout=layout, shard=(n0, n1))
            if kind == "silu_gate":
                biases[name] = torch.cat([b[n0:n1], b[half + n0:half + n1]]).contiguous()
            else:
                biases[name] = b[n0:n1].contiguous()
            shards[name] = (n0, n1, per)
        del w
    xs = {}
    for i, (name, M, K, N, kind) in enumerate(LINEARS):
        if name == "down" and "gate_up" in ACTIVE:
            continue
        gen.manual_seed(2000 + i)
        xs[name] = torch.randn(M, K, generator=gen, device=dev)

    def out_cols(name, N, kind):
        return N // 2 if kind == "silu_gate" else N

    # outputs (full) and per-rank shard outputs for N-split
    ys, ys_shard, gather_bufs = {}, {}, {}
    for name, M, K, N, kind in RUN:
        nout = out_cols(name, N, kind)
        ys[name] = torch.empty(M, nout, device=dev)
        if world > 1:
            n0, n1, per = shards[name]
            ys_shard[name] = torch.zeros(M, per, device=dev)
            gather_bufs[name] = torch.empty(world, M, per, device=dev)

    def step():
        for name, M, K, N, kind in RUN:
            x = ys["gate_up"] if name not in xs else xs[name]
            if world == 1:
                envg.linear(ys[name], x, weights[name], bias=biases[name], sync=False)
                continue
            n0, n1, per = shards[name]
            if n1 - n0 == per:
                envg.linear(ys_shard[name], x, weights[name], bias=biases[name], sync=False)
            elif n1 > n0:  # ragged last shard: compute into the first n1 - n0 columns
                tmp = torch.empty(M, n1 - n0, device=dev)
                envg.linear(tmp, x, weights[name], bias=biases[name], sync=False)
                ys_shard[name][:, : n1 - n0].copy_(tmp)
            gather_columns(ys_shard[name], ys[name].shape[1], out=ys[name], buf=gather_bufs[name])

    def timed(fn, steps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(steps):
            fn()
        s1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = s0.elapsed_time(s1) / steps
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    st0 = envg.stats()
    clk = ClockSampler(local)
    clk.start()
    ms = timed(step, args.steps)
    clocks = clk.stop()
    st1 = envg.stats()
    launches = int(st1["kernel_launches"] - st0["kernel_launches"])
    if world > 1:
        t = torch.tensor([launches], device=dev, dtype=torch.int64)
        dist.all_reduce(t)
        launches = int(t.item())
    value = STEP_FLOPS / (ms * 1e-3) / 1e12

    # GEMM-phase only (no gather) for N > 1: what the N-split itself scales like
    gemm_phase = None
    if world > 1:
        def step_local():
            for name, M, K, N, kind in RUN:
                x = ys["gate_up"] if name not in xs else xs[name]
                n0, n1, per = shards[name]
                if n1 - n0 == per:
                    envg.linear(ys_shard[name], x, weights[name], bias=biases[name], sync=False)
        gms = timed(step_local, args.steps)
        gemm_phase = {"value": STEP_FLOPS / (gms * 1e-3) / 1e12, "ms_per_step": gms}

    # per-kernel device time with CUDA events around each launch (roofline of the top kernel)
    envg.profile(True)
    prof_steps = max(3, min(args.steps, 10))
    for _ in range(prof_steps):
        step()
    torch.cuda.synchronize()
    prof = envg.profile_read()
    envg.profile(False)
    pk, hbm, src = peaks()
    k1 = {"launches": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0}
    for kname in ("k1_gemm", "k1_gemm_silu_gate"):
        for f in k1:
            k1[f] += prof.get(kname, {}).get(f, 0)
    roofline = None
    if k1["launches"]:
        ach = k1["flops"] / (k1["ms"] * 1e-3) / 1e12
        traffic = K1_TRAFFIC_BYTES_PER_LAUNCH
        roofline = {"bound": "tensor", "achieved": round(ach, 1), "peak": pk, "unit": "TFLOP/s",
                    "frac": round(ach / pk, 4), "traffic": traffic, "kernel": "k1_gemm (+ silu_gate variant)",
                    "peak_source": f"{src} (MEASURED_PEAKS.json bf16_tflops, burst)" if src == "measured" else src,
                    "algorithmic_flops_per_launch": k1["flops"] / k1["launches"],
                    "avg_launch_ms": k1["ms"] / k1["launches"]}
    kernels = {k: {"launches": v["launches"], "avg_us": round(1e3 * v["ms"] / v["launches"], 2),
                   "share": None, "tflops": round(v["flops"] / (v["ms"] * 1e-3) / 1e12, 1) if v["flops"] else None,
                   "gbs": round(v["bytes"] / (v["ms"] * 1e-3) / 1e9, 1)} for k, v in prof.items()}
    tot = sum(v["ms"] for v in prof.values()) or 1.0
    for k, v in prof.items():
        kernels[k]["share"] = round(v["ms"] / tot, 4)
    skinny = prof.get("k2_skinny")
    if skinny:
        kernels["k2_skinny"]["hbm_frac"] = round(skinny["bytes"] / (skinny["ms"] * 1e-3) / 1e9 / hbm, 4)

    # end to end through the public API with host (pinned) buffers
    e2e = None
    if not args.no_e2e and world == 1 and len(RUN) == len(LINEARS):
        e2e = run_e2e(args, envg, torch, dev, weights, biases, xs, ys)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and len(RUN) == len(LINEARS):
        cpu = cpu_baseline(args, sample_seconds=args.cpu_seconds)

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": WORKLOAD if len(RUN) == len(LINEARS) else
                           f"one linear of the workload: {[r[0] for r in RUN]}", "M": M_TOK, "hidden": HID, "mlp": MLP,
                           "flops_per_step": STEP_FLOPS,
                           "parallelism": "single GPU" if world == 1 else f"N-split x{world} + NCCL all-gather",
                           "arith": "fp32 activations rounded to bf16 (RNE), bf16 weights, fp32 accumulate",
                           "l2": "working set ~0.6 GB > 126 MB L2; no flush"},
                "clocks": clocks, "gpu_launches": launches, "e2e": e2e, "roofline": roofline,
                "cpu_baseline": cpu, "kernels": kernels}
        if gemm_phase:
            line["gemm_phase"] = gemm_phase
        print(json.dumps(line), flush=True)

    for w in weights.values():
        w.free()


def run_e2e(args, envg, torch, dev, weights, biases, xs, ys):
    """Same step through envg_linear with HOST pointers (pinned numpy views): each call copies its
    input and bias H2D, runs, and copies its output D2H, synchronously, as the Pascal host would."""
    hx = {k: torch.empty(v.shape, dtype=torch.float32, pin_memory=True) for k, v in xs.items()}
    for k in hx:
        hx[k].copy_(xs[k])
    hb = {k: torch.empty(v.shape, dtype=torch.float32, pin_memory=True) for k, v in biases.items()}
    for k in hb:
        hb[k].copy_(biases[k])
    hy = {k: torch.empty(v.shape, dtype=torch.float32, pin_memory=True) for k, v in ys.items()}
    npx = {k: v.numpy() for k, v in hx.items()}
    npb = {k: v.numpy() for k, v in hb.items()}
    npy = {k: v.numpy() for k, v in hy.items()}
    h2d = d2h = 0
    for name, M, K, N, kind in LINEARS:
        x = npy["gate_up"] if name == "down" else npx[name]
        h2d += x.nbytes + npb[name].nbytes
        d2h += npy[name].nbytes

    stream = torch.cuda.Stream(device=dev)
    envg.follow_torch_stream(False)
    envg.set_stream(stream.cuda_stream)

    def step():
        for name, M, K, N, kind in LINEARS:
            x = npy["gate_up"] if name == "down" else npx[name]
            envg.linear(npy[name], x, weights[name], bias=npb[name])

    steps = max(2, min(args.steps, 5))
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    envg.set_stream(None)
    envg.follow_torch_stream(True)
    return {"value": round(FLOPS_PER_STEP / (ms * 1e-3) / 1e12, 2), "unit": UNIT, "ms_per_step": round(ms, 3),
            "steps": steps, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "path": "envg_linear(HOST_PTRS) from pinned host memory, synchronous per call"}


# ---------------------------------------------------------------------------------------------
# CPU side: the reference's own GEMM on the host cores
# ---------------------------------------------------------------------------------------------
class CpuWorkload:
    """Seeded host copies of the workload: fp32-widened bf16 weights (the reference widens at load,
    src/safetensor.pas:584-647), fp32 biases and inputs.  A step runs an M-slice of `rows` rows."""

    def __init__(self):
        import torch

        from oracle import oracle as O

        self.O = O
        g = torch.Generator().manual_seed(7)
        self.w, self.b, self.x = {}, {}, {}
        for name, M, K, N, kind in LINEARS:
            wt = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).float()
            self.w[name] = wt.numpy()
            self.b[name] = (torch.randn(N, generator=g) * 0.01).numpy()
            if name != "down":
                self.x[name] = torch.randn(M, K, generator=g).numpy()
        self.use_ref = O.ref_lib() is not None

    def gemm(self, x, w):
        m, K = x.shape
        N = w.shape[0]
        if self.use_ref:
            return self.O.sgemm2_nt(x, w, m, N, K)
        return self.O.linear_f32(x, w)

    def step(self, rows):
        O = self.O
        flops = 0.0
        y = {}
        for name, M, K, N, kind in LINEARS:
            x = y["gate_up"] if name == "down" else np.ascontiguousarray(self.x[name][: min(M, rows)])
            out = self.gemm(x, self.w[name])
            out += self.b[name]  # QNNAddInplace per row (quicknncpu.pas:1816-1819)
            if kind == "silu_gate":
                h = N // 2
                out = O.silu_mul(np.ascontiguousarray(out[:, :h]), np.ascontiguousarray(out[:, h:]))
            y[name] = out
            flops += 2.0 * x.shape[0] * K * N
        return flops

    def pick_rows(self, target_s):
        """Largest M-slice (multiple of 64, <= 4608) whose step takes about target_s seconds."""
        t = time.perf_counter()
        self.step(64)
        dt = time.perf_counter() - t
        rows = int(64 * target_s / max(dt, 1e-3))
        return max(64, min(M_TOK, (rows // 64) * 64))

    def describe(self):
        return ("reference src/sgemm2.cpp cpp_sgemm (compiled from the reference tree, OpenMP)" if self.use_ref else
                "C++ restatement of the reference Pascal qgemm/gemm_nt (oracle/envg_oracle.cpp)")


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(args, sample_seconds=12.0):
    from oracle import oracle as O

    threads = cpu_threads()
    O.set_threads(threads)
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    wl = CpuWorkload()
    rows = wl.pick_rows(sample_seconds)
    t = time.perf_counter()
    flops = wl.step(rows)
    dt = time.perf_counter() - t
    return {"value": round(flops / dt / 1e12, 5), "unit": UNIT, "cores": threads,
            "kind": "reference" if wl.use_ref else "port",
            "sample": f"one step of the workload on an M-slice of {rows} of 4608 token rows (adaLN M=1 in full); "
                      f"{dt:.1f} s; {wl.describe()}"}


def run_reference(args, world, rank):
    """--impl reference: the reference's CPU GEMM path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    from oracle import oracle as O

    threads = cpu_threads()
    O.set_threads(threads)
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    per_step = max(0.5, min(15.0, 150.0 / max(1, args.steps + args.warmup)))
    wl = CpuWorkload()
    rows = wl.pick_rows(per_step)
    for _ in range(args.warmup):
        wl.step(rows)
    t = time.perf_counter()
    flops = 0.0
    for _ in range(args.steps):
        flops += wl.step(rows)
    dt = time.perf_counter() - t
    value = flops / dt / 1e12
    kind = "reference" if wl.use_ref else "port"
    sample = (f"each step: the workload on an M-slice of {rows} of 4608 token rows (adaLN M=1 in full); "
              f"{wl.describe()}")
    line = {"metric": METRIC, "value": round(value, 5), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "M_slice": rows, "parallelism": f"{threads} host threads"},
            "cpu_baseline": {"value": round(value, 5), "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": round(value, 5), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


ACTIVE = {r[0] for r in LINEARS}
RUN = list(LINEARS)
STEP_FLOPS = FLOPS_PER_STEP


def main():
    global RUN, ACTIVE, STEP_FLOPS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--only", default=None, help="run one linear of the workload (profiling): " +
                    ",".join(r[0] for r in LINEARS))
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.only:
        RUN = [r for r in LINEARS if r[0] == args.only]
        if not RUN:
            ap.error(f"--only: unknown linear {args.only}")
        ACTIVE = {args.only}
        STEP_FLOPS = float(sum(2 * M * K * N for _, M, K, N, _ in RUN))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup()
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
