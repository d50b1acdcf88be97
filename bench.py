"""Benchmark of the Envision dense-linear hot path on B200 (one JSON line on rank 0).

Default workload: BASELINE config 4, the configuration the metric's "at 1/2/4/8 B200" figure is
quoted on (N-split across 1/2/4/8 GPUs) and the largest that fits one GPU: the two linears of a
FLUX2-Klein-9B-shaped single-stream block, batch of 4 images at 1024x1024
(quicknn_transformers.pas:1503 linear1 and :1528 linear2):

    fused_in  [18432, 4096]  -> 36864   QKV (3 x 4096) and gate/up (2 x 12288), no bias
    out       [18432, 16384] -> 4096    no bias

X ~ N(0,1) fp32, W = bf16(0.02 N(0,1)), all synthetic and seeded (no model weights exist in this
environment).  One step = both linears, 8.04 TFLOP.  The working set (weights 436 MB, activations
and outputs 4.5 GB) is far above the 126 MB L2, so no flush is needed between steps.
With N > 1 GPUs (one process per GPU, torchrun) each rank holds a head-aligned output-column
shard of every weight (N-split, strong scaling):
  fused_in  the shard holds whole heads of Q, K and V and whole gate/up pairs; its consumers
            (per-head attention, the per-pair SiLU gate) are column-local, so its output stays
            sharded on the rank (ENVG_KEEP_SHARDED: no transfer);
  out       its output is the residual stream, which every rank needs whole: each rank's columns
            go to every rank's copy of Y from the GEMM epilogue (all-gather fused into the
            epilogue; --gather nccl for NCCL's all-gather instead).
`--config c1|c2|c3|c3_m16|c3_m1|c5` run the other BASELINE shapes (per-config figures);
`--config f2|f3|f4` the fused neighbours (RMSNorm / AdaLN prologues), the VAE ResBlock and
attention.  `--gather-all` gathers fused_in's output too (every linear's Y assembled on every rank).

Arms:
  (default)          libenvgemm through its C ABI.  `value` = device-resident throughput
                     (TFLOP/s, whole job); `e2e` = the same through host buffers (pinned), every
                     call copying its inputs H2D and its output D2H.
  --impl reference   the reference's own CPU GEMM path: the C++ restatement of the Pascal
                     qgemm -> gemm_nt with sDot_x4_avx2 that the Envision binary runs (same
                     tiling, threading and AVX2 instructions), on all host cores, on a bounded
                     M-slice of the same workload.
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

METRIC = "block_linear_tflops"
UNIT = "TFLOP/s"


def lin(name, M, K, N, epi="bias", x_from=None, x_same=None, norm=None, segments=None, keep=False):
    """x_from: the input is that item's output; x_same: the same input tensor as that item;
    norm: "rms" (envg_linear_rmsnorm) or "adaln" (envg_linear_adaln) normalises X in the cast;
    segments: W's row blocks (Q, K, V heads, gate, up) that an N-split shards each in the same
    proportion, so a rank holds whole heads and gate/up pairs; keep: with N > 1 the output stays
    sharded on its rank (its consumers are column-local)."""
    return dict(name=name, op="linear", M=M, K=K, N=N, epi=epi, x_from=x_from, x_same=x_same, norm=norm,
                segments=segments, keep=keep)


def conv(name, B, C, H, W, O, k, stride, pad, epi="silu"):
    return dict(name=name, op="conv", B=B, C=C, H=H, W=W, O=O, k=k, stride=stride, pad=pad, epi=epi)


def attn(name, Sq, Sk, H, KVH, causal=False):
    return dict(name=name, op="attn", Sq=Sq, Sk=Sk, H=H, KVH=KVH, causal=causal, epi="none")


def resblock(name, B, Ci, Co, H, W, G=32):
    return dict(name=name, op="resblock", B=B, Ci=Ci, Co=Co, H=H, W=W, G=G, epi="none")


def qwen(M):
    # q, k and v all read the normalised hidden state (quicknn_qwen3.pas:712-714)
    return [lin("q", M, 2560, 4096, "none"), lin("k", M, 2560, 1024, "none", x_same="q"),
            lin("v", M, 2560, 1024, "none", x_same="q"),
            lin("o", M, 4096, 2560, "none"), lin("gate_up", M, 2560, 2 * 9728, "silu_gate_nobias"),
            lin("down", M, 9728, 2560, "none", x_from="gate_up")]


M_TOK = 4096 + 512
WORKLOADS = {
    "c2": ("BASELINE config 2: FLUX2-Klein-4B double-stream block linears, M=4608 (4096 img + 512 txt), hidden "
           "3072: qkv 3072->9216, out 3072->3072, gate_up 3072->18432 (SiLU-gate), down 9216->3072, adaLN "
           "3072->18432 at M=1; all with fp32 bias",
           [lin("qkv", M_TOK, 3072, 9216), lin("out", M_TOK, 3072, 3072),
            lin("gate_up", M_TOK, 3072, 18432, "silu_gate"), lin("down", M_TOK, 9216, 3072, x_from="gate_up"),
            lin("adaln", 1, 3072, 18432)]),
    "c1": ("BASELINE config 1: FLUX2-Klein-4B QKV linear Y[1024,9216] = X[1024,3072].W^T + b",
           [lin("qkv", 1024, 3072, 9216)]),
    "c3": ("BASELINE config 3: Qwen3-4B layer linears at M=512 (no bias)", qwen(512)),
    "c3_m16": ("BASELINE config 3 at M=16 (skinny)", qwen(16)),
    "c3_m1": ("BASELINE config 3 at M=1 (skinny)", qwen(1)),
    "c4": ("BASELINE config 4: FLUX2-Klein-9B single-stream fused input linear M=18432 (4 x (4096+512) tokens), "
           "K=4096, N=36864 (QKV 3x4096 + gate/up 2x12288), then the output linear K=16384, N=4096 (no bias)",
           [lin("fused_in", 18432, 4096, 36864, "none", segments=(4096, 4096, 4096, 12288, 12288), keep=True),
            lin("out", 18432, 16384, 4096, "none")]),
    "c5": ("BASELINE config 5: VAE-decoder 3x3 conv, [1,512,128,128] -> 512 ch, and [1,256,256,256] -> 256 ch, "
           "fused bias + SiLU",
           [conv("conv512", 1, 512, 128, 128, 512, 3, 1, 1), conv("conv256", 1, 256, 256, 256, 256, 3, 1, 1)]),
    "f3": ("VAE-decoder ResBlocks (GroupNorm 32 + SiLU + 3x3 conv, twice, + residual): 512 ch at 128x128 and "
           "256 ch at 256x256",
           [resblock("rb512", 1, 512, 512, 128, 128), resblock("rb256", 1, 256, 256, 256, 256)]),
    "f2": ("fused prologues: Qwen3-4B q 2560->4096 and gate_up 2560->2x9728 (SiLU-gate) at M=512 behind "
           "QNNRMSNormRows (envg_linear_rmsnorm), and the FLUX2-Klein-4B qkv 3072->9216 + b at M=4608 behind "
           "QNNAdaLN (envg_linear_adaln); one call per linear",
           [lin("rms_q", 512, 2560, 4096, "none", norm="rms"),
            lin("rms_gate_up", 512, 2560, 2 * 9728, "silu_gate_nobias", norm="rms"),
            lin("adaln_qkv", M_TOK, 3072, 9216, norm="adaln")]),
    "f4": ("attention: FLUX2-Klein-4B joint attention (4608 tokens, 24 heads x 128, non-causal) and Qwen3-4B "
           "prefill (512 tokens, 32 query / 8 kv heads x 128, causal)",
           [attn("flux", M_TOK, M_TOK, 24, 24), attn("qwen3", 512, 512, 32, 8, causal=True)]),
}


def item_flops(it):
    if it["op"] == "linear":
        return 2.0 * it["M"] * it["K"] * it["N"]
    if it["op"] == "attn":
        pairs = it["Sq"] * it["Sk"]
        if it["causal"]:
            pairs -= it["Sq"] * (it["Sq"] - 1) / 2
        return 4.0 * 128 * pairs * it["H"]
    if it["op"] == "resblock":
        skip = it["Ci"] * it["Co"] if it["Ci"] != it["Co"] else 0
        return 2.0 * it["B"] * it["H"] * it["W"] * (9 * it["Co"] * it["Ci"] + 9 * it["Co"] * it["Co"] + skip)
    oh = (it["H"] + 2 * it["pad"] - it["k"]) // it["stride"] + 1
    ow = (it["W"] + 2 * it["pad"] - it["k"]) // it["stride"] + 1
    return 2.0 * it["O"] * oh * ow * it["B"] * it["C"] * it["k"] * it["k"]


def is_gate(it):
    return it["op"] == "linear" and it["epi"].startswith("silu_gate")


def out_cols(it):
    return it["N"] // 2 if is_gate(it) else it["N"]


def plain_linear(it):
    """A linear the batch, N-split, end-to-end and CPU-baseline paths take (no fused prologue)."""
    return it["op"] == "linear" and not it.get("norm")


def has_bias(it):
    return it["epi"] in ("bias", "silu_gate", "silu")


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per k1_gemm launch of one step of the
# default workload at one GPU, from an ncu capture of the current kernels (one pass,
# gpu__time_duration and the two dram counters; per-launch mean over the step's launches).
K1_TRAFFIC_BYTES_PER_LAUNCH = {"c4": 3.886e9}


def peaks(clocks=None, region_ms=0.0):
    """(bf16 TFLOP/s, HBM GB/s, which).  The burst cuBLAS figure of MEASURED_PEAKS.json is the
    denominator for a short or unthrottled timed region; the sustained one (cuBLAS looped for
    seconds under the 1 kW power cap) when the clock record shows sw_power_cap over a region of a
    second or more."""
    capped = bool(clocks) and "sw_power_cap" in (clocks.get("reasons") or []) and region_ms >= 1000.0
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        if capped and "bf16_tflops_sustained" in p:
            return float(p["bf16_tflops_sustained"]), float(p["hbm_gbs"]), "measured, sustained"
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured, burst"
    except Exception:
        return (1400.0, 6650.0, "fallback, sustained") if capped else (1590.0, 6650.0, "fallback, burst")


# ---------------------------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    """SM clock and throttle reasons sampled every 5 ms by NVML in a background thread during the
    timed region (nvidia-smi as a fallback)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, device_index):
        self.dev = device_index
        self.samples = []
        self.reasons = set()
        self.stop_flag = False
        self.th = None
        self.mx = None
        self.proc = None

    def _run(self, nv, h):
        while not self.stop_flag:
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def start(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.dev]) if vis else self.dev
            h = nv.nvmlDeviceGetHandleByIndex(idx)
            self.mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self.th = threading.Thread(target=self._run, args=(nv, h), daemon=True)
            self.th.start()
        except Exception:
            self.th = None
            self._start_smi()

    def _start_smi(self):
        fields = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={fields}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return

        def rd():
            names = ["hw_slowdown", "sw_thermal_slowdown", "hw_thermal_slowdown", "sw_power_cap"]
            for line in self.proc.stdout:
                parts = [q.strip() for q in line.split(",")]
                try:
                    self.samples.append(float(parts[0]))
                    self.mx = float(parts[1])
                except (ValueError, IndexError):
                    continue
                for n, v in zip(names, parts[2:6]):
                    if v.lower() == "active":
                        self.reasons.add(n)
        self.th = threading.Thread(target=rd, daemon=True)
        self.th.start()

    def stop(self):
        if self.th is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"], "samples": 0}
        self.stop_flag = True
        src = "NVML, 5 ms"
        if getattr(self, "proc", None) is not None:
            self.proc.terminate()
            src = "nvidia-smi, 50 ms"
        self.th.join(timeout=2)
        sm = list(self.samples)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.mx,
                "reasons": sorted(self.reasons), "samples": len(sm), "source": src}


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
        # stdout carries only the one JSON result line: NCCL's version banner and, with NCCL_DEBUG
        # set, its debug lines, which it prints to stdout while the communicator starts, go to
        # stderr (below), where they stay visible.
        torch.cuda.set_device(local)
        stdout_to_stderr()
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        dist.barrier()
    return world, rank, local


_json_out = None


def stdout_to_stderr():
    """From here on, file descriptor 1 is stderr (NCCL and other libraries print to it); the JSON
    result line goes to the original stdout through emit()."""
    global _json_out
    if _json_out is None:
        sys.stdout.flush()
        _json_out = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def emit(line):
    out = _json_out if _json_out is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------
class Workload:
    """Device-resident weights, inputs and outputs of one workload on this rank."""

    def __init__(self, items, world, rank, dev, gather="peer", force_p2p=False, gather_all=False):
        import torch

        from invision_b200 import envg
        from invision_b200.nsplit import segment_rows, shard_bounds

        self.items, self.world, self.rank, self.dev = items, world, rank, dev
        self.envg = envg
        self.batch = True
        self.gather = gather
        self.force_p2p = force_p2p
        self.sym = {}
        self.keep = set()  # N-split items whose output stays sharded on the rank (no transfer)
        gen = torch.Generator(device=dev)
        self.W, self.b, self.x, self.y, self.shard, self.ys, self.gbuf = {}, {}, {}, {}, {}, {}, {}
        self.nv = {}  # normalisation vectors of the items with a fused prologue
        names = [it["name"] for it in items]
        self.consumed = {it["x_from"] for it in items if it.get("x_from")}
        for i, it in enumerate(items):
            name = it["name"]
            gen.manual_seed(1000 + i)
            if (it["op"] in ("attn", "resblock") or it.get("norm")) and world > 1:
                raise SystemExit(f"{it['op']} workloads run on one GPU")
            if it["op"] == "attn":
                D = 128
                self.x[name] = tuple(torch.randn(n, h * D, generator=gen, device=dev)
                                     for n, h in ((it["Sq"], it["H"]), (it["Sk"], it["KVH"]), (it["Sk"], it["KVH"])))
                self.y[name] = torch.empty(it["Sq"], it["H"] * D, device=dev)
                self.b[name] = None
                continue
            if it["op"] == "resblock":
                Ci, Co = it["Ci"], it["Co"]

                def bfw(shape, sc):
                    w = (torch.randn(*shape, generator=gen, device=dev) * sc).to(torch.bfloat16)
                    return w.view(torch.int16).cpu().numpy().view(np.uint16)

                p = {"conv1_w": bfw((Co, Ci, 3, 3), 0.03), "conv2_w": bfw((Co, Co, 3, 3), 0.03)}
                if Ci != Co:
                    p["skip_w"] = bfw((Co, Ci, 1, 1), 0.1)
                vec = {"norm1_gamma": 1 + 0.1 * torch.randn(Ci, generator=gen, device=dev),
                       "norm1_beta": 0.1 * torch.randn(Ci, generator=gen, device=dev),
                       "conv1_b": 0.01 * torch.randn(Co, generator=gen, device=dev),
                       "norm2_gamma": 1 + 0.1 * torch.randn(Co, generator=gen, device=dev),
                       "norm2_beta": 0.1 * torch.randn(Co, generator=gen, device=dev),
                       "conv2_b": 0.01 * torch.randn(Co, generator=gen, device=dev)}
                if Ci != Co:
                    vec["skip_b"] = 0.01 * torch.randn(Co, generator=gen, device=dev)
                self.W[name] = envg.ResBlock(p)
                self.b[name] = vec
                self.x[name] = torch.randn(it["B"], Ci, it["H"], it["W"], generator=gen, device=dev)
                self.y[name] = torch.empty(it["B"], Co, it["H"], it["W"], device=dev)
                continue
            if it["op"] == "conv":
                if world > 1:
                    raise SystemExit("conv workloads run on one GPU")
                O, C, k = it["O"], it["C"], it["k"]
                w = (torch.randn(O, C * k * k, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
                self.W[name] = envg.Weight(w.view(torch.int16).cpu().numpy().view(np.uint16), conv=(O, C, k, k))
                self.b[name] = torch.randn(O, generator=gen, device=dev) * 0.01
                gen.manual_seed(2000 + i)
                self.x[name] = torch.randn(it["B"], C, it["H"], it["W"], generator=gen, device=dev)
                oh = (it["H"] + 2 * it["pad"] - k) // it["stride"] + 1
                ow = (it["W"] + 2 * it["pad"] - k) // it["stride"] + 1
                self.y[name] = torch.empty(it["B"], O, oh, ow, device=dev)
                continue
            M, K, N = it["M"], it["K"], it["N"]
            w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
            b = torch.randn(N, generator=gen, device=dev) * 0.01 if has_bias(it) else None
            w_host = w.view(torch.int16).cpu().numpy().view(np.uint16)
            del w
            gate = is_gate(it)
            layout = envg.LAYOUT_GATE_UP if gate else envg.LAYOUT_PLAIN
            if world == 1:
                self.W[name] = envg.Weight(w_host, layout=layout)
                self.b[name] = b
            else:
                half = N // 2 if gate else N
                if it.get("segments") and not gate:
                    # head-aligned shard: this rank's heads of Q, K, V and its gate/up rows
                    rows = segment_rows(it["segments"], world, rank, 128)
                    self.W[name] = envg.Weight(np.ascontiguousarray(w_host[rows]), layout=layout)
                    self.b[name] = b[torch.from_numpy(rows).to(dev)].contiguous() if b is not None else None
                    n0, n1, per = 0, len(rows), len(rows)
                else:
                    n0, n1, per = shard_bounds(half, world, rank, 128)
                    self.W[name] = envg.Weight(w_host, layout=layout, shard=(n0, n1))
                    if b is not None:
                        self.b[name] = (torch.cat([b[n0:n1], b[half + n0:half + n1]]) if gate else b[n0:n1]).contiguous()
                    else:
                        self.b[name] = None
                self.shard[name] = (n0, n1, per)
                self.ys[name] = torch.zeros(M, per, device=dev)
                if it.get("keep") and not gather_all and name not in self.consumed:
                    self.keep.add(name)
                elif self.gather == "nccl":
                    self.gbuf[name] = torch.empty(world, M, per, device=dev)
                if name not in self.keep and self.gather == "peer":
                    import torch.distributed as dist
                    import torch.distributed._symmetric_memory as symm_mem

                    ysym = symm_mem.empty(M, out_cols(it), device=dev)
                    h = symm_mem.rendezvous(ysym, dist.group.WORLD)
                    mc = h.multicast_ptr if (h.has_multicast_support and not self.force_p2p) else 0
                    self.sym[name] = (ysym, h, list(h.buffer_ptrs), mc)
            if it.get("x_same"):
                self.x[name] = self.x[it["x_same"]]
            elif it["x_from"] not in names:
                gen.manual_seed(2000 + i)
                self.x[name] = torch.randn(M, K, generator=gen, device=dev)
            self.y[name] = torch.empty(M, out_cols(it), device=dev)
            if it.get("norm") == "rms":
                self.nv[name] = (1 + 0.1 * torch.randn(K, generator=gen, device=dev),)
            elif it.get("norm") == "adaln":
                self.nv[name] = (0.1 * torch.randn(K, generator=gen, device=dev),
                                 0.1 * torch.randn(K, generator=gen, device=dev))

    def input_of(self, it):
        if it["name"] in self.x:
            return self.x[it["name"]]
        return self.sym[it["x_from"]][0] if it["x_from"] in self.sym else self.y[it["x_from"]]

    def out_of(self, name):
        if name in self.keep:
            return self.ys[name]
        return self.sym[name][0] if name in self.sym else self.y[name]

    def run_item(self, it, gather=True):
        envg = self.envg
        name = it["name"]
        if it["op"] == "conv":
            envg.conv2d(self.y[name], self.x[name], self.W[name], self.b[name], it["stride"], it["pad"],
                        epilogue=envg.EPI_SILU if it["epi"] == "silu" else envg.EPI_BIAS, sync=False)
            return
        if it["op"] == "attn":
            q, k, v = self.x[name]
            envg.attention(self.y[name], q, k, v, it["H"], it["KVH"], causal=it["causal"], sync=False)
            return
        if it["op"] == "resblock":
            self.W[name].forward(self.y[name], self.x[name], it["G"], vecs=self.b[name], sync=False)
            return
        x = self.input_of(it)
        if it.get("norm") == "rms":
            envg.linear_rmsnorm(self.y[name], x, self.W[name], weight=self.nv[name][0], bias=self.b[name], sync=False)
            return
        if it.get("norm") == "adaln":
            shift, scale = self.nv[name]
            envg.linear_adaln(self.y[name], x, shift, scale, self.W[name], bias=self.b[name], sync=False)
            return
        if self.world == 1:
            envg.linear(self.y[name], x, self.W[name], bias=self.b[name], sync=False)
            return
        import torch

        from invision_b200.nsplit import gather_columns

        n0, n1, per = self.shard[name]
        if name in self.keep:  # the output stays on this rank: its shard is all there is to compute
            envg.linear(self.ys[name], x, self.W[name], bias=self.b[name], sync=False)
            return
        if gather and name in self.sym:
            # all-gather fused into the epilogue: this rank's columns go to every rank's copy of Y
            ysym, h, peers, mc = self.sym[name]
            if n1 > n0:
                envg.linear_nsplit(ysym, x, self.W[name], n0, peers=None if mc else peers, multicast=mc,
                                   bias=self.b[name], sync=False)
            # the ranks meet only where a copy of Y is read next: before a linear that consumes this
            # output, and at the end of the step (before the next step writes the copies again)
            if name in self.consumed or it is self.items[-1]:
                h.barrier()
            return
        if n1 - n0 == per:
            envg.linear(self.ys[name], x, self.W[name], bias=self.b[name], sync=False)
        elif n1 > n0:  # ragged last shard: compute into the first n1 - n0 columns
            tmp = torch.empty(it["M"], n1 - n0, device=self.dev)
            envg.linear(tmp, x, self.W[name], bias=self.b[name], sync=False)
            self.ys[name][:, : n1 - n0].copy_(tmp)
        if gather:
            gather_columns(self.ys[name], self.y[name].shape[1], out=self.y[name], buf=self.gbuf[name])

    def step(self, gather=True):
        if (self.world > 1 and gather and self.batch and (self.sym or self.keep) and
                all(plain_linear(it) and (it["name"] in self.sym or it["name"] in self.keep) for it in self.items)):
            # N-split shards in envg_linear_nsplit_batch calls, one per segment that ends where a
            # later linear reads a gathered output (the ranks meet there) or at the end of the step.
            # A kept shard names no peers: its epilogue stores into this rank's buffer only.
            seg = []
            handle = next(iter(self.sym.values()))[1] if self.sym else None
            for it in self.items:
                name = it["name"]
                n0, n1, _ = self.shard[name]
                if name in self.keep:
                    seg.append(dict(y=self.ys[name], x=self.input_of(it), W=self.W[name], col0=0, bias=self.b[name]))
                else:
                    ysym, h, peers, mc = self.sym[name]
                    if n1 > n0:
                        seg.append(dict(y=ysym, x=self.input_of(it), W=self.W[name], col0=n0, bias=self.b[name],
                                        peers=None if mc else peers, multicast=mc))
                if (name in self.consumed and name not in self.keep) or it is self.items[-1]:
                    if seg:
                        self.envg.linear_nsplit_batch(seg, sync=False)
                    seg = []
                    if handle is not None:
                        handle.barrier()
            return
        if self.world > 1 and not gather and self.batch and all(plain_linear(it) for it in self.items):
            # the GEMM phase: the same batched step with every shard kept on its rank (the casts
            # overlap the GEMMs as in the full step; no transfer, no barrier)
            seg = [dict(y=self.ys[it["name"]], x=self.input_of(it), W=self.W[it["name"]], col0=0,
                        bias=self.b[it["name"]]) for it in self.items
                   if self.shard[it["name"]][1] > self.shard[it["name"]][0]]
            if seg:
                self.envg.linear_nsplit_batch(seg, sync=False)
            return
        if self.world == 1 and self.batch and all(plain_linear(it) for it in self.items):
            # one envg_linear_batch call: each input cast once, casts overlapped with the GEMMs
            self.envg.linear_batch([dict(dst=self.y[it["name"]], x=self.input_of(it), W=self.W[it["name"]],
                                         bias=self.b[it["name"]]) for it in self.items], sync=False)
            return
        for it in self.items:
            self.run_item(it, gather)

    def free(self):
        for w in self.W.values():
            if isinstance(w, self.envg.ResBlock):
                for c in (w.conv1, w.conv2, w.skip):
                    if c is not None:
                        c.free()
            else:
                w.free()
        self.sym.clear()  # symmetric buffers go before the process group


def workload_config(args, desc, items):
    """The workload, identical on both arms (the driver compares the arms' config objects)."""
    ws = 0.0
    for it in items:
        if it["op"] == "linear":
            ws += 2.0 * it["N"] * it["K"] + 4.0 * it["M"] * (it["K"] + out_cols(it))
    cfg = {"workload": desc, "config": args.config + (f" (only {args.only})" if args.only else ""),
           "flops_per_step": float(sum(item_flops(it) for it in items))}
    if ws:
        cfg["l2"] = (f"working set {ws / 1e9:.2f} GB of weights, inputs and outputs > 126 MB L2: no flush between "
                     "steps")
    else:
        cfg["l2"] = "inputs larger than the 126 MB L2: no flush between steps"
    return cfg


def capture(torch, fn):
    """Capture fn's launches on a side stream into a CUDA graph (the library follows torch's
    current stream)."""
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def run_ours(args, items, desc, world, rank, local):
    import torch
    import torch.distributed as dist

    from invision_b200 import envg

    torch.cuda.set_device(local)
    envg.init(local)
    dev = torch.device("cuda", local)
    wl = Workload(items, world, rank, dev, gather=args.gather, force_p2p=args.p2p,
                  gather_all=args.gather_all)
    wl.batch = not args.no_batch
    step_flops = float(sum(item_flops(it) for it in items))

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
        wl.step()
    torch.cuda.synchronize()

    # One step captured once into a CUDA graph (single GPU): the timed loop replays it, so host
    # launch overhead is out of the device time.  Warm-up above sized every workspace, so the
    # capture allocates nothing.
    graph = None
    if world == 1 and not args.no_graph:
        graph = capture(torch, wl.step)
    run_step = graph.replay if graph is not None else wl.step
    launches_per_step = None
    if graph is not None:
        st_a = envg.stats()
        wl.step()
        torch.cuda.synchronize()
        launches_per_step = int(envg.stats()["kernel_launches"] - st_a["kernel_launches"])
    for _ in range(2):
        run_step()
    torch.cuda.synchronize()

    st0 = envg.stats()
    clk = ClockSampler(local)
    clk.start()
    ms = timed(run_step, args.steps)
    clocks = clk.stop()
    st1 = envg.stats()
    launches = int(st1["kernel_launches"] - st0["kernel_launches"])
    if graph is not None:
        launches = launches_per_step * args.steps  # replays do not pass through the host counter
    if world > 1:
        t = torch.tensor([launches], device=dev, dtype=torch.int64)
        dist.all_reduce(t)
        launches = int(t.item())
    value = step_flops / (ms * 1e-3) / 1e12

    # GEMM-phase only (no gather) for N > 1: what the N-split itself scales like
    gemm_phase = None
    if world > 1:
        for _ in range(2):  # the per-linear calls size their own workspace on first use
            wl.step(gather=False)
        torch.cuda.synchronize()
        gms = timed(lambda: wl.step(gather=False), args.steps)
        gathered = [it for it in items if it["name"] not in wl.keep]
        gbytes = sum(4.0 * it["M"] * out_cols(it) * (world - 1) / world for it in gathered)
        gemm_phase = {"value": round(step_flops / (gms * 1e-3) / 1e12, 2), "ms_per_step": round(gms, 4),
                      "note": "the same batched step with every rank keeping all its shards in local buffers "
                              "(envg_linear_nsplit_batch, casts overlapped as in the step): no transfer, no barrier",
                      "gathered": [it["name"] for it in gathered], "kept_sharded": sorted(wl.keep),
                      "nvlink_bytes_in_per_rank": gbytes,
                      "nvlink_floor_ms": round(gbytes / 770e9 * 1e3, 4),
                      "nvlink_floor_note": "bytes each rank must receive / 770 GB/s (measured peer copy per "
                                          "direction on this pool)"}

    # per-kernel device time: CUDA events the library records around each launch
    pk, hbm, src = peaks(clocks, ms * args.steps)
    envg.profile(True)
    prof_steps = max(3, min(args.steps, 10))
    for _ in range(prof_steps):
        wl.step(gather=False)
    torch.cuda.synchronize()
    prof = envg.profile_read()
    envg.profile(False)
    k1 = {"launches": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0}
    for kname in ("k1_gemm", "k1_gemm_silu_gate", "k1_gemm_conv"):
        for f in k1:
            k1[f] += prof.get(kname, {}).get(f, 0)
    roofline = None
    if not k1["launches"] and prof.get("k_attention", {}).get("launches"):
        fa = prof["k_attention"]
        ach = fa["flops"] / (fa["ms"] * 1e-3) / 1e12
        roofline = {"bound": "tensor", "achieved": round(ach, 1), "peak": pk, "unit": "TFLOP/s",
                    "frac": round(ach / pk, 4), "traffic": None,
                    "kernel": "k_attention (tcgen05 flash-attention forward, fp16 operands)",
                    "peak_source": src + " (MEASURED_PEAKS.json cuBLAS bf16; fp16 runs at the bf16 rate)",
                    "algorithmic_flops_per_launch": fa["flops"] / fa["launches"],
                    "avg_launch_ms": round(fa["ms"] / fa["launches"], 5)}
    if k1["launches"]:
        ach = k1["flops"] / (k1["ms"] * 1e-3) / 1e12
        roofline = {"bound": "tensor", "achieved": round(ach, 1), "peak": pk, "unit": "TFLOP/s",
                    "frac": round(ach / pk, 4),
                    "traffic": (K1_TRAFFIC_BYTES_PER_LAUNCH.get(args.config)
                                if world == 1 and not args.only else None),
                    "kernel": "k1_gemm family (tcgen05 CTA-pair GEMM; plain, SiLU-gate and conv variants)",
                    "peak_source": src + (" (MEASURED_PEAKS.json: cuBLAS bf16 8192^3, burst = best of 10, sustained = "
                                          "looped 4 s under the 1 kW power cap; sustained is used when sw_power_cap "
                                          "was active over a timed region of 1 s or more)"),
                    "algorithmic_flops_per_launch": k1["flops"] / k1["launches"],
                    "avg_launch_ms": round(k1["ms"] / k1["launches"], 5)}
    tot = sum(v["ms"] for v in prof.values()) or 1.0
    kernels = {}
    for k, v in prof.items():
        kernels[k] = {"launches": v["launches"], "avg_us": round(1e3 * v["ms"] / v["launches"], 2),
                      "share": round(v["ms"] / tot, 4),
                      "tflops": round(v["flops"] / (v["ms"] * 1e-3) / 1e12, 1) if v["flops"] else None,
                      "gbs": round(v["bytes"] / (v["ms"] * 1e-3) / 1e9, 1),
                      "hbm_frac": round(v["bytes"] / (v["ms"] * 1e-3) / 1e9 / hbm, 4)}

    # per item (each linear / conv alone): the main kernel's time from per-launch events (these
    # include the launch gap, which dominates kernels of a few microseconds) and the item's time
    # as a CUDA-graph replay of 20 back-to-back calls (no host overhead).
    per_item = {}
    for it in items:
        envg.profile(True)
        reps = 5
        for _ in range(reps):
            wl.run_item(it, gather=False)
        torch.cuda.synchronize()
        p = envg.profile_read()
        envg.profile(False)
        main = {k: v for k, v in p.items()
                if k.startswith("k1") or k.startswith("k2") or
                k in ("k_gemv", "k_attention", "k_split_reduce", "k_skinny_reduce")}
        mms = sum(v["ms"] for v in main.values()) / reps
        mbytes = sum(v["bytes"] for v in main.values()) / reps
        rank_flops = item_flops(it) / (world if it["op"] == "linear" else 1)  # this rank's shard
        rec = {"kernel": "+".join(sorted(main)), "gemm_us": round(1e3 * mms, 2),
               "gemm_tflops": round(rank_flops / (mms * 1e-3) / 1e12, 1) if mms else None,
               "gemm_gbs": round(mbytes / (mms * 1e-3) / 1e9, 1) if mms else None}
        if world == 1 and not args.no_graph:
            # An HBM-bound (skinny) linear is timed over enough copies of its weight that one
            # replay streams more than twice the 126 MB L2, so no call finds its weight in L2.
            name = it["name"]
            copies = [wl.W.get(name)]
            if it["op"] == "linear" and it["M"] <= 64:
                wbytes = 2.0 * it["N"] * it["K"]
                ncopy = int(min(64, -(-2 * 126e6 // wbytes)))
                for _ in range(ncopy - 1):
                    wr = (0.02 * torch.randn(it["N"], it["K"])).to(torch.bfloat16).view(torch.int16)
                    copies.append(envg.Weight(wr.numpy().view(np.uint16), layout=wl.W[name].layout))
            calls = max(20, len(copies))

            def replay_body():
                for c in range(calls):
                    if len(copies) > 1:
                        wl.W[name] = copies[c % len(copies)]
                    wl.run_item(it, gather=False)
                if len(copies) > 1:
                    wl.W[name] = copies[0]

            g = capture(torch, replay_body)
            gms = timed(g.replay, 5) / calls
            rec["graph_us"] = round(1e3 * gms, 2)
            rec["graph_tflops"] = round(item_flops(it) / (gms * 1e-3) / 1e12, 1)
            rec["graph_gbs"] = round(mbytes / (gms * 1e-3) / 1e9, 1)
            if len(copies) > 1:
                rec["weight_copies"] = len(copies)
            del g
            for c in copies[1:]:
                c.free()
        per_item[it["name"]] = rec

    e2e = None
    if not args.no_e2e and world == 1 and all(plain_linear(it) for it in items):
        e2e = run_e2e(args, envg, torch, dev, wl, step_flops)
    elif not args.no_e2e and world > 1 and all(plain_linear(it) for it in items):
        e2e = run_e2e_nsplit(args, torch, dev, wl, step_flops, timed)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and all(plain_linear(it) for it in items):
        cpu = cpu_baseline(items, sample_seconds=args.cpu_seconds)

    if rank == 0:
        if world == 1:
            par = "single GPU"
        elif args.gather == "peer":
            par = (f"N-split x{world}, head-aligned shards; "
                   + (f"{', '.join(sorted(wl.keep))} kept sharded (column-local consumers); " if wl.keep else "")
                   + "all-gather of the rest fused into the GEMM epilogue ("
                   + ("NVLS multimem stores" if any(v[3] for v in wl.sym.values()) else "P2P TMA stores") + ")")
        else:
            par = f"N-split x{world} + NCCL all-gather"
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": workload_config(args, desc, items),
                "arm": {"timing": ("one step captured as a CUDA graph and replayed" if graph is not None
                                   else "steps launched from the host"),
                        "api": ("envg_linear_batch (one call per step)" if world == 1 else
                                "envg_linear_nsplit_batch (one call per barrier-to-barrier segment)")
                               if wl.batch else "envg_linear per linear",
                        "parallelism": par,
                        "arith": "fp32 activations rounded to bf16 (RNE), bf16 weights, fp32 accumulate"},
                "clocks": clocks, "gpu_launches": launches, "e2e": e2e, "roofline": roofline,
                "cpu_baseline": cpu, "kernels": kernels, "per_item": per_item}
        if gemm_phase:
            line["gemm_phase"] = gemm_phase
        emit(line)
    wl.free()


def run_e2e_nsplit(args, torch, dev, wl, step_flops, timed):
    """N > 1: the N-split step through the public API (envg_linear_nsplit_batch) with every step's
    inputs coming from pinned host memory and each rank reading its part of the results back: its
    kept shard, and its block of rows of every gathered output (together the ranks read each
    output once).  Every rank needs the whole X.  Headline: each rank copies only its block of
    rows of each input over its own PCIe link and an NCCL all-gather over NVLink assembles the
    whole input on every rank.  `replicated_copy`: every rank copies the whole input in."""
    import torch.distributed as dist

    world, rank = wl.world, wl.rank
    hx, seen = {}, set()
    for k, v in wl.x.items():
        if v.data_ptr() in seen:  # an input shared by several linears is copied once
            continue
        seen.add(v.data_ptr())
        h = torch.empty(v.shape, dtype=torch.float32, pin_memory=True)
        h.copy_(v)
        hx[k] = h
    outs = []
    for it in wl.items:
        n = it["name"]
        if n in wl.keep:
            src = wl.ys[n]
        else:
            y = wl.out_of(n)
            r0 = rank * y.shape[0] // world
            r1 = (rank + 1) * y.shape[0] // world
            src = y[r0:r1]
        outs.append((src, torch.empty(src.shape, dtype=torch.float32, pin_memory=True)))
    d2h = sum(h.numel() * 4 for _, h in outs)
    steps = max(2, min(args.steps, 5))

    def read_back():
        for src, h in outs:
            h.copy_(src, non_blocking=True)

    def step_replicated():
        for k, h in hx.items():
            wl.x[k].copy_(h, non_blocking=True)
        wl.step()
        read_back()

    # rows of each input this rank brings in (inputs whose rows do not split evenly are copied whole)
    blocks = {}
    for k, h in hx.items():
        M = h.shape[0]
        if M % world == 0 and wl.x[k].is_contiguous():
            r0, r1 = rank * M // world, (rank + 1) * M // world
            blocks[k] = (h[r0:r1], torch.empty((r1 - r0,) + tuple(h.shape[1:]), dtype=torch.float32, device=dev))

    def step_split():
        for k, h in hx.items():
            if k in blocks:
                hb, stage = blocks[k]
                stage.copy_(hb, non_blocking=True)
                dist.all_gather_into_tensor(wl.x[k], stage)
            else:
                wl.x[k].copy_(h, non_blocking=True)
        wl.step()
        read_back()

    for _ in range(2):
        step_split()
        step_replicated()
    torch.cuda.synchronize()
    ms = timed(step_split, steps)
    ms_rep = timed(step_replicated, steps)
    h2d_rep = sum(h.numel() * 4 for h in hx.values())
    h2d = sum((blocks[k][0].numel() if k in blocks else h.numel()) * 4 for k, h in hx.items())
    nvlink = sum((h.numel() - blocks[k][0].numel()) * 4 for k, h in hx.items() if k in blocks)
    return {"value": round(step_flops / (ms * 1e-3) / 1e12, 2), "unit": UNIT, "ms_per_step": round(ms, 3),
            "steps": steps, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "nvlink_in_bytes_per_step": nvlink,
            "path": ("per rank: its row block of each input from pinned host memory (torch copy), NCCL all-gather "
                     "of the inputs over NVLink, envg_linear_nsplit_batch step, its kept shards and its row block "
                     "of every gathered output back to pinned host memory; max over ranks; bytes are this rank's"),
            "replicated_copy": {"value": round(step_flops / (ms_rep * 1e-3) / 1e12, 2), "unit": UNIT,
                                "ms_per_step": round(ms_rep, 3), "h2d_bytes_per_step": h2d_rep,
                                "d2h_bytes_per_step": d2h,
                                "path": "per rank: the whole of every input from pinned host memory, then as above"}}


def run_e2e(args, envg, torch, dev, wl, step_flops):
    """Same step through the public API with HOST pointers (pinned numpy views), timed two ways:
    one envg_linear_batch call over the step's linears (the headline: their copies in and out
    overlap one another and the GEMMs), and one synchronous envg_linear call per linear, as the
    Pascal host calls QNNLinear (each call's copies overlap only its own GEMM)."""
    cache = {}

    def pinned(t):  # one pinned copy per device tensor (items that share an input share it)
        if t.data_ptr() not in cache:
            h = torch.empty(t.shape, dtype=torch.float32, pin_memory=True)
            h.copy_(t)
            cache[t.data_ptr()] = h
        return cache[t.data_ptr()]

    hx = {k: pinned(v) for k, v in wl.x.items()}
    hb = {k: pinned(v) for k, v in wl.b.items() if v is not None}
    hy = {k: torch.empty(v.shape, dtype=torch.float32, pin_memory=True) for k, v in wl.y.items()}
    npx = {k: v.numpy() for k, v in hx.items()}
    npb = {k: v.numpy() for k, v in hb.items()}
    npy = {k: v.numpy() for k, v in hy.items()}
    h2d = d2h = 0
    for it in wl.items:
        n = it["name"]
        x = npx[n] if n in npx else npy[it["x_from"]]
        h2d += x.nbytes + (npb[n].nbytes if n in npb else 0)
        d2h += npy[n].nbytes

    stream = torch.cuda.Stream(device=dev)
    envg.follow_torch_stream(False)
    envg.set_stream(stream.cuda_stream)

    def x_of(it):
        n = it["name"]
        return npx[n] if n in npx else npy[it["x_from"]]

    def step_calls():
        for it in wl.items:
            envg.linear(npy[it["name"]], x_of(it), wl.W[it["name"]], bias=npb.get(it["name"]))

    batch = [dict(dst=npy[it["name"]], x=x_of(it), W=wl.W[it["name"]], bias=npb.get(it["name"])) for it in wl.items]

    def step_batch():
        envg.linear_batch(batch)

    steps = max(2, min(args.steps, 5))

    def timed(step):
        for _ in range(2):
            step()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            step()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps

    ms = timed(step_batch)
    ms_calls = timed(step_calls)
    envg.set_stream(None)
    envg.follow_torch_stream(True)
    # bytes per step: a shared input crosses PCIe once in the batch (once per call in step_calls)
    h2d_batch = sum({c["x"].ctypes.data: c["x"].nbytes for c in batch}.values()) + sum(v.nbytes for v in npb.values())
    return {"value": round(step_flops / (ms * 1e-3) / 1e12, 2), "unit": UNIT, "ms_per_step": round(ms, 3),
            "steps": steps, "h2d_bytes_per_step": h2d_batch, "d2h_bytes_per_step": d2h,
            "path": "one envg_linear_batch(HOST_PTRS) call per step from pinned host memory, synchronous",
            "per_call": {"value": round(step_flops / (ms_calls * 1e-3) / 1e12, 2), "unit": UNIT,
                         "ms_per_step": round(ms_calls, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                         "path": "envg_linear(HOST_PTRS) per linear, synchronous per call"}}


# ---------------------------------------------------------------------------------------------
# CPU side: the reference's own GEMM on the host cores
# ---------------------------------------------------------------------------------------------
class CpuWorkload:
    """Seeded host copies of a linear workload: bf16 weight bits and their fp32 widening (the
    reference widens at load, src/safetensor.pas:584-647, or per call, src/quicknncpu.pas:1830-1847),
    fp32 biases and inputs.  A step runs an M-slice of `rows` rows of every linear whose M exceeds
    it (M = 1 linears run in full) through one of the reference's CPU GEMMs:
      "sgemm2"  src/sgemm2.cpp cpp_sgemm, compiled unmodified from the reference tree (oracle/_ref);
      "o1"      the C++ restatement of the shipped Pascal qgemm -> gemm_nt with sDot_x4_avx2
                (quicknncpu.pas:1241-1337, ops_avx2.inc:1407-1508) on pre-widened fp32 weights."""

    def __init__(self, items):
        import torch

        from oracle import oracle as O

        self.O = O
        self.items = items
        g = torch.Generator().manual_seed(7)
        self.w, self.wb, self.b, self.x = {}, {}, {}, {}
        names = [it["name"] for it in items]
        for it in items:
            n, M, K, N = it["name"], it["M"], it["K"], it["N"]
            wb = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
            self.wb[n] = wb.view(torch.int16).numpy().view(np.uint16)
            self.w[n] = wb.float().numpy()
            self.b[n] = (torch.randn(N, generator=g) * 0.01).numpy() if has_bias(it) else None
            if it["x_from"] not in names:
                self.x[n] = torch.randn(M, K, generator=g).numpy()
        self.has_ref = O.ref_lib() is not None

    def gemm(self, x, n, kind):
        m, K = x.shape
        N = self.w[n].shape[0]
        if kind == "sgemm2":
            return self.O.sgemm2_nt(x, self.w[n], m, N, K)
        return self.O.linear_f32(x, self.w[n])

    def step(self, rows, kind, times=None):
        O = self.O
        flops = 0.0
        y = {}
        for it in self.items:
            n, M, K, N = it["name"], it["M"], it["K"], it["N"]
            t0 = time.perf_counter()
            x = np.ascontiguousarray(self.x[n][: min(M, rows)]) if n in self.x else y[it["x_from"]]
            out = self.gemm(x, n, kind)
            if self.b[n] is not None:
                out += self.b[n]  # QNNAddInplace per row (quicknncpu.pas:1816-1819)
            if is_gate(it):
                h = N // 2
                out = O.silu_mul(np.ascontiguousarray(out[:, :h]), np.ascontiguousarray(out[:, h:]))
            y[n] = out
            if times is not None:
                times[n] = (time.perf_counter() - t0, x.shape[0])
            flops += 2.0 * x.shape[0] * K * N
        return flops

    def widen_seconds(self):
        """One BF16ToSingle widening of every weight (the per-call work of QNNLinearNoBias_BF16)."""
        t = time.perf_counter()
        for n in self.wb:
            self.O.bf16_to_f32(self.wb[n])
        return time.perf_counter() - t

    def pick_rows(self, target_s, kind):
        """Largest M-slice (multiple of 64, <= the largest M) whose step takes about target_s seconds."""
        mmax = max(it["M"] for it in self.items)
        t = time.perf_counter()
        self.step(min(64, mmax), kind)
        dt = time.perf_counter() - t
        rows = int(64 * target_s / max(dt, 1e-3))
        return max(min(64, mmax), min(mmax, (rows // 64) * 64))

    def describe(self, kind):
        return ("reference src/sgemm2.cpp cpp_sgemm (compiled from the reference tree, OpenMP)" if kind == "sgemm2" else
                "C++ restatement of the reference Pascal qgemm/gemm_nt with sDot_x4_avx2 (oracle/envg_oracle.cpp)")


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def use_all_host_threads():
    """The CPU legs run on every host thread (torchrun exports OMP_NUM_THREADS=1, and the
    reference's sgemm2 parallelises with OpenMP, which shares torch's runtime)."""
    import torch

    threads = cpu_threads()
    os.environ["OMP_NUM_THREADS"] = str(threads)
    torch.set_num_threads(threads)
    from oracle import oracle as O

    O.set_threads(threads)
    return threads


def cpu_baseline(items, sample_seconds=8.0):
    """The reference's CPU GEMMs on the host cores, each on a bounded M-slice of the workload.
    `value` is O1, the restated shipped Pascal qgemm -> gemm_nt (the GEMM the Envision binary
    runs; sgemm2.cpp is not linked into it) on pre-widened weights, FLUX's path (use_bf16 is never
    set).  Beside it: O1 with the per-call bf16 -> fp32 widening of QNNLinearNoBias_BF16, and the
    reference's standalone sgemm2.cpp compiled from its tree.  The widened figure is for the whole
    workload: the slice's GEMM time scaled to all rows, plus one widening of every weight per step
    (it does not shrink with the slice)."""
    threads = use_all_host_threads()
    wl = CpuWorkload(items)
    mmax = max(it["M"] for it in items)
    full_flops = float(sum(item_flops(it) for it in items))

    def run(kind):
        rows = wl.pick_rows(sample_seconds, kind)
        times = {}
        t = time.perf_counter()
        flops = wl.step(rows, kind, times)
        dt = time.perf_counter() - t
        full_s = sum(ts * it["M"] / r for it in items for ts, r in [times[it["name"]]])
        return rows, flops, dt, full_s

    o1_rows, o1_flops, o1_dt, o1_full = run("o1")
    widen = wl.widen_seconds()
    o1 = {"value": round(o1_flops / o1_dt / 1e12, 5), "unit": UNIT, "kind": "port", "cores": threads,
          "sample": f"M-slice of {o1_rows} of {mmax} rows, {o1_dt:.1f} s; {wl.describe('o1')}; weights pre-widened "
                    "(the path the shipped FLUX code takes, use_bf16 = false)"}
    o1w = {"value": round(full_flops / (o1_full + widen) / 1e12, 5), "unit": UNIT, "kind": "port", "cores": threads,
           "sample": f"O1 GEMM time of the slice scaled to all {mmax} rows plus {widen:.2f} s of single-threaded "
                     "BF16ToSingle widening of every weight per step (QNNLinearNoBias_BF16, quicknncpu.pas:1830-1847)"}
    out = dict(o1)
    out["cpu_model"] = f"{cpu_model()}, {threads} threads"
    out["o1_qgemm_widened_per_call"] = o1w
    if wl.has_ref:
        rows, flops, dt, _ = run("sgemm2")
        out["sgemm2"] = {"value": round(flops / dt / 1e12, 5), "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": f"M-slice of {rows} of {mmax} rows, {dt:.1f} s; {wl.describe('sgemm2')}"}
    return out


def run_reference(args, items, desc, world, rank):
    """--impl reference: the reference's CPU GEMM path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    if not all(plain_linear(it) for it in items):
        emit({"impl": "reference", "unavailable": "the CPU arm covers linear workloads only"})
        return
    threads = use_all_host_threads()
    per_step = max(0.5, min(15.0, 150.0 / max(1, args.steps + args.warmup)))
    wl = CpuWorkload(items)
    # O1: the restated Pascal qgemm the shipped binary runs (faster here than the unlinked sgemm2.cpp)
    kind = "o1"
    rows = wl.pick_rows(per_step, kind)
    for _ in range(args.warmup):
        wl.step(rows, kind)
    t = time.perf_counter()
    flops = 0.0
    for _ in range(args.steps):
        flops += wl.step(rows, kind)
    dt = time.perf_counter() - t
    value = flops / dt / 1e12
    mmax = max(it["M"] for it in items)
    sample = (f"each step: the workload on an M-slice of {rows} of {mmax} token rows (M=1 linears in full); "
              f"{wl.describe(kind)}")
    line = {"metric": METRIC, "value": round(value, 5), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": workload_config(args, desc, items),
            "arm": {"parallelism": f"{threads} host threads ({cpu_model()})", "M_slice": rows},
            "cpu_baseline": {"value": round(value, 5), "unit": UNIT, "cores": threads,
                             "kind": "reference" if kind == "sgemm2" else "port", "sample": sample},
            "e2e": {"value": round(value, 5), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c4", choices=sorted(WORKLOADS))
    ap.add_argument("--only", default=None, help="run one item of the workload (profiling)")
    ap.add_argument("--rows", type=int, default=0,
                    help="profiling: set M of every linear with M > 64 to this many rows (a smaller case of the same "
                         "kernels for ncu captures; not a bench figure)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch every step from the host")
    ap.add_argument("--no-batch", action="store_true", help="one envg_linear call per linear")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="N>1: all-gather fused into the GEMM epilogue (peer/multicast stores) or NCCL")
    ap.add_argument("--p2p", action="store_true",
                    help="N>1 gather by P2P TMA stores into each rank's copy (default: one multimem store per value "
                         "through an NVLS multicast address where the switch offers one; measured equal at 2 GPUs "
                         "and 3%% faster at 4)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=8.0, help="CPU time per baseline variant")
    ap.add_argument("--gather-all", action="store_true",
                    help="N>1: gather every linear's output, also those whose consumers are column-local")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    desc, items = WORKLOADS[args.config]
    if args.only:
        keep = [it for it in items if it["name"] == args.only]
        if not keep:
            ap.error(f"--only: no item {args.only} in {args.config}")
        items = keep
        desc = f"{args.config}: only {args.only}"
    if args.rows:
        items = [dict(it, M=args.rows) if it["op"] == "linear" and it["M"] > 64 else it for it in items]
        desc = f"{desc} [profiling case: M = {args.rows}]"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if world > 1:
            stdout_to_stderr()
        run_reference(args, items, desc, world, rank)
        return
    world, rank, local = dist_setup()
    try:
        run_ours(args, items, desc, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
