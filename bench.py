#!/usr/bin/env python
"""bench.py -- MoE-layer throughput of the B200-native hot path.

Default workload (N=1): BASELINE config 3 -- one MoE layer over 16384 tokens,
hidden 2048, 32 experts, top-4, expert SwiGLU intermediate 1792, bf16 expert
weights with fp32 accumulation, router logits drawn so that per-expert load
follows Zipf(s=1.1) (injected exactly through the inputs: gate = [I_32 | 0],
x[:, :32] = ln p_e + Gumbel noise; the router GEMM still runs over all 2048
columns).  One step = one full layer forward (route, scan, scatter, W1/W3
SwiGLU grouped GEMM, W2 grouped GEMM, combine) on inputs resident in HBM.

With --gpus N (launched under torchrun) the layer runs expert-parallel: every
rank routes its own 16384 tokens, rows travel to the rank that computes their
expert segment and back (copy-engine writes into CUDA-IPC-mapped peer buffers,
NCCL for the per-forward count all-gather), value = all ranks' tokens /
max-over-ranks device time (weak scaling).  The headline placement is owner
(E/N experts per GPU, BASELINE config 4's sharding) on uniform routing, the
case the scaling target is defined for; the line also carries the other
placement / routing combinations, the staged pipeline, and the same routing
timed on one GPU in the same run (`one_gpu_same_routing.efficiency`).

--impl reference times the reference's own implementation of the path on the
box's host cores (the C restatement in oracle/, since the reference ships no
CPU implementation of this path), on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, E, K, I = 2048, 32, 4, 1792
T_DEFAULT = 16384
ZIPF_S = 1.1
SEED = 1234


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--routing", choices=["zipf", "uniform"], default=None,
                   help="default: zipf on 1 GPU (config 3), uniform on several (config 4's "
                        "4-experts-per-GPU sharding, the case the scaling target is set for)")
    p.add_argument("--tokens", type=int, default=T_DEFAULT)
    p.add_argument("--dtype", choices=["bf16", "tf32"], default="bf16")
    p.add_argument("--cpu-seconds", type=float, default=12.0,
                   help="target CPU work of the bounded cpu_baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-dense", action="store_true", help="skip the dense GEMM sweep")
    p.add_argument("--no-model", action="store_true",
                   help="skip the full-model forward (config 5)")
    p.add_argument("--model-only", action="store_true",
                   help="only time the full-model forward (config 5)")
    p.add_argument("--model-ep", choices=["none", "balanced", "owner"], default="balanced",
                   help="with several GPUs, also time the expert-parallel model in this mode")
    p.add_argument("--ep-mode", choices=["balanced", "owner"], default="owner",
                   help="expert placement when --gpus > 1 (owner: E/N experts per GPU)")
    p.add_argument("--no-variants", action="store_true",
                   help="with --gpus > 1, skip the other placements / routings / pipeline")
    p.add_argument("--gemm-configs", type=int, nargs=3, metavar=("M", "N", "K"),
                   help="time every dense-GEMM kernel configuration on one shape (bf16)")
    p.add_argument("--gemm-launches", type=int, nargs=3, metavar=("M", "N", "K"),
                   help="launch six dense-GEMM configurations and torch.mm four times "
                        "each, eagerly (for a one-pass ncu launch list)")
    p.add_argument("--gemm", type=int, nargs=3, metavar=("M", "N", "K"),
                   help="only time b2_gemm_nt on one dense shape (bf16 operands), "
                        "e.g. for a profiler capture of the dense kernel")
    args = p.parse_args()
    if args.routing is None:
        n = max(int(os.environ.get("WORLD_SIZE", "1")), args.gpus)
        args.routing = "zipf" if n == 1 else "uniform"
    return args


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return dict(hbm=d["hbm_gbs"], bf16=d["bf16_tflops"],
                    bf16_sustained=d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                    source="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sustained=1400.0, source="fallback")


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock, power and clock-event reasons sampled while the timed region
    runs: NVML polled every 5 ms from a host thread (the main thread sits in
    cudaDeviceSynchronize meanwhile), so even a timed region of a few tens of
    ms gets several samples; nvidia-smi at 200 ms if NVML is unavailable.
    Read-only queries: no clock or power setting is touched."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4),
               ("hw_power_brake_slowdown", 0x80))

    def __init__(self, smi_index, period_s=0.005):
        self.idx = smi_index
        self.period = period_s
        self.proc = None
        self.path = None
        self.thread = None
        self.rows = []
        self.nvml = None

    def start(self):
        if self.idx is None:
            return
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self.nvml = pynvml
        except Exception:
            self.nvml = None
        if self.nvml is not None:
            self.stop_flag = threading.Event()
            nv = self.nvml

            def poll():
                while True:
                    try:
                        self.rows.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                          nv.nvmlDeviceGetPowerUsage(h) / 1000.0,
                                          int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
                    except Exception:
                        pass
                    if self.stop_flag.wait(self.period):
                        break

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.idx), "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join()
            self.nvml.nvmlShutdown()
            if not self.rows:
                return None
            sm = sorted(r[0] for r in self.rows)
            reasons = sorted({n for n, bit in self.REASONS for r in self.rows if r[2] & bit})
            return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": self.max_mhz,
                    "sm_mhz_min": sm[0], "power_w_max": max(r[1] for r in self.rows),
                    "reasons": reasons, "samples": len(self.rows), "sampler": "nvml 5 ms"}
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [s.strip() for s in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        os.remove(self.path)
        if not rows:
            return None
        sm = sorted(float(r[1]) for r in rows)
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": float(rows[0][2]),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())
                if any(r[3].replace(".", "").isdigit() for r in rows) else None,
                "reasons": sorted(reasons), "samples": len(rows), "sampler": "nvidia-smi 200 ms"}


def smi_index_for(dev_index: int):
    """nvidia-smi index of torch device `dev_index` (matched by PCI bus id)."""
    import torch
    try:
        props = torch.cuda.get_device_properties(dev_index)
        bus = getattr(props, "pci_bus_id", None)
        dom = getattr(props, "pci_domain_id", 0)
        out = subprocess.run(["nvidia-smi", "--query-gpu=index,pci.bus_id",
                              "--format=csv,noheader"], capture_output=True, text=True,
                             timeout=30).stdout
        if bus is not None:
            for line in out.strip().splitlines():
                idx, pci = [s.strip() for s in line.split(",")]
                # pci like 00000000:1B:00.0
                b = int(pci.split(":")[1], 16)
                d = int(pci.split(":")[0], 16)
                if b == bus and d == dom:
                    return int(idx)
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            return int(vis.split(",")[dev_index])
        return dev_index
    except Exception:
        return None


# ------------------------------------------------------------------ inputs
def make_inputs(T, routing, dev, seed=SEED, token_seed=None):
    """x [T,H] fp32, gate [E,H] fp32, fp32 expert weights -- generated on the
    device.  Weights depend on `seed` only; tokens on `token_seed` (default
    `seed`), so expert-parallel ranks share one layer but hold different tokens."""
    import torch
    gx = torch.Generator(device=dev).manual_seed(seed if token_seed is None else token_seed)
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, H, device=dev, generator=gx)
    if routing == "zipf":
        p = torch.arange(1, E + 1, dtype=torch.float64, device=dev) ** (-ZIPF_S)
        p = p / p.sum()
        u = torch.rand(T, E, device=dev, generator=gx, dtype=torch.float64).clamp_min(1e-300)
        L = (p.log()[None, :] - torch.log(-torch.log(u))).float()
        gate = torch.zeros(E, H, device=dev)
        gate[torch.arange(E), torch.arange(E)] = 1.0
        x[:, :E] = L
        bias = None
    else:
        gate = torch.randn(E, H, device=dev, generator=g) * 0.02
        bias = torch.randn(E, device=dev, generator=g) * 0.02
    w1 = torch.randn(E, I, H, device=dev, generator=g) * 0.02
    w3 = torch.randn(E, I, H, device=dev, generator=g) * 0.02
    w2 = torch.randn(E, H, I, device=dev, generator=g) * 0.02
    return x, gate, bias, w1, w2, w3


def layer_flop(T):
    return T * (2 * H * E + K * (4 * H * I + 2 * I * H))


# ------------------------------------------------------------------ ours
def bench_config(args, world):
    """The workload the line measures -- a function of the arguments alone, so
    the reference arm prints the identical dict."""
    T = args.tokens
    return {"workload": f"moe_layer_{T // 1024}k_{args.routing}", "tokens_per_gpu": T,
            "hidden": H, "experts": E, "top_k": K, "inter": I,
            "routing": ("zipf(1.1) injected logits" if args.routing == "zipf"
                        else "x.gate N(0,1)xN(0,0.02), bias N(0,0.02)"),
            "l2": "inputs larger than L2: x 134 MB fp32, expert weights 705 MB bf16",
            "parallelism": (f"expert-parallel ep{world} ({args.ep_mode} placement), fused "
                            "grouped GEMMs with peer-memory dispatch/return, NCCL count "
                            "all-gather" if world > 1 else "single")}


def exchange_bytes(plan, rank, world, row_bytes):
    """Bytes this rank moved over NVLink in one forward, from its plan."""
    sent = sum(c for d, c in enumerate(plan["send_cnt"]) if d != rank)
    recv = sum(c for s, c in enumerate(plan["recv_cnt"]) if s != rank)
    return {"rank": rank, "rows_computed": plan["recv_rows"],
            "dispatch_sent": sent * row_bytes, "dispatch_received": recv * row_bytes,
            "return_sent": recv * row_bytes, "return_received": sent * row_bytes}


def time_layer(args, rank, world, dev, mode, routing, pipeline="fused", e2e=False,
               keep_host=False):
    """One MoE layer (single-GPU, or expert-parallel over `world` ranks in
    `mode` placement) on `routing` inputs: W warm-up forwards, then K
    forwards timed with CUDA events between barriers (max over ranks), a
    second K-forward pass with stage events, and optionally the end-to-end
    pass through host buffers.  Returns the measurements."""
    import torch
    import torch.distributed as dist
    from final_b200 import SparseMoeBlock, launch_count

    T = args.tokens
    x, gate, bias, w1, w2, w3 = make_inputs(T, routing, dev, SEED, SEED + 1000 * (rank + 1))
    if world > 1:
        from final_b200.ep import ExpertParallelMoE
        layer = ExpertParallelMoE(gate, w1, w2, w3, bias, max_tokens=T, top_k=K, dtype=args.dtype,
                                  mode=mode, timeout_s=120.0, pipeline=pipeline)
    else:
        layer = SparseMoeBlock(gate, w1, w2, w3, bias, max_tokens=T, top_k=K, dtype=args.dtype)
    res = {}
    if keep_host:
        # fp32 weights for the CPU baseline sample (same workload)
        res["host"] = ([t.cpu().numpy() for t in (w1, w3, w2)],
                       (x.cpu().numpy(), gate.cpu().numpy(),
                        None if bias is None else bias.cpu().numpy()))
    del w1, w2, w3
    torch.cuda.empty_cache()
    y = torch.empty(T, H, device=dev)
    row_bytes = H * (4 if args.dtype == "tf32" else 2)
    if world > 1:
        layer.forward_gpu(x, y, T)
        torch.cuda.synchronize()
        plan = layer.last_plan()
        ex = [None] * world
        dist.all_gather_object(ex, exchange_bytes(plan, rank, world, row_bytes))
        res["exchange_bytes_per_step"] = ex
        res["load"] = {"rows_per_rank": [e["rows_computed"] for e in ex]}
    else:
        cnt = layer.forward_traced(x)["counts"].cpu().tolist()
        res["load"] = {"expert_rows_max_min": [max(cnt), min(cnt)]}

    stream = torch.cuda.current_stream()
    fwd = (lambda xi, yi: layer.forward_gpu(xi, yi, T, stream)) if world > 1 else \
        (lambda xi, yi: layer.forward_gpu(xi, yi, 1, T, H, stream))
    def check_status(where):
        # every rank learns every rank's status, so an error stops all of them
        # at the same point (none is left waiting in a collective)
        st = layer.device_status()
        if world > 1:
            t = torch.tensor([st], device=dev, dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            st = int(t.item())
        if st != 0:
            layer.close()
            raise RuntimeError(f"device status 0x{st:x} {where}")

    for _ in range(args.warmup):
        fwd(x, y)
    torch.cuda.synchronize()
    check_status("after warm-up")

    sampler = ClockSampler(smi_index_for(dev.index))
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    n0 = launch_count()
    ev0.record(stream)
    for _ in range(args.steps):
        fwd(x, y)
    ev1.record(stream)
    torch.cuda.synchronize()
    res["clocks"] = sampler.stop()
    res["gpu_launches"] = int(launch_count() - n0)
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    # the same K steps again with CUDA events between the stages (kept out of the
    # timed region above: an event between two kernels stops the second one from
    # starting while the first drains)
    layer.profile(True)
    for _ in range(args.steps):
        fwd(x, y)
    torch.cuda.synchronize()
    layer.profile(False)
    res["stage_ms"], res["nfw"] = layer.profile_read()
    if world > 1:
        tl = [None] * world
        dist.all_gather_object(tl, layer.timeline())
        res["timeline"] = tl
        dist.barrier()
    check_status("in timed region")
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    res["ms"] = ms
    res["ms_per_step"] = ms / args.steps
    res["value"] = T * args.steps * world / (ms / 1e3)

    # ---- end-to-end through the public API with host buffers: every step
    # copies its input batch from pinned host memory and its result back;
    # copies of step i+1 / i-1 overlap the layer of step i (two copy streams,
    # double-buffered device buffers).
    if e2e:
        xh = x.cpu().pin_memory()
        yh = [torch.empty(T, H, dtype=torch.float32).pin_memory() for _ in range(2)]
        xd = [torch.empty_like(x) for _ in range(2)]
        yd = [torch.empty_like(y) for _ in range(2)]
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
        ev = lambda: torch.cuda.Event()

        def pipelined(steps, with_layer=True):
            done_c = [None, None]   # layer of step i finished reading xd / writing yd
            done_o = [None, None]   # D2H of step i finished reading yd
            for i in range(steps):
                b = i & 1
                with torch.cuda.stream(s_in):
                    if done_c[b] is not None:
                        s_in.wait_event(done_c[b])
                    xd[b].copy_(xh, non_blocking=True)
                    e_in = ev(); e_in.record(s_in)
                stream.wait_event(e_in)
                if done_o[b] is not None:
                    stream.wait_event(done_o[b])
                if with_layer:
                    fwd(xd[b], yd[b])
                e_c = ev(); e_c.record(stream); done_c[b] = e_c
                with torch.cuda.stream(s_out):
                    s_out.wait_event(e_c)
                    yh[b].copy_(yd[b], non_blocking=True)
                    e_o = ev(); e_o.record(s_out); done_o[b] = e_o
            for e_o in done_o:
                if e_o is not None:
                    stream.wait_event(e_o)

        pipelined(3)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_stream(stream)
        pipelined(args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
        ems = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = t.item()
        # the same pipeline with the layer left out: the time the two copy
        # streams alone need for these bytes on this box's PCIe link, the
        # bound of the end-to-end figure
        pipelined(3, with_layer=False)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0.record(stream)
        s_in.wait_stream(stream)
        pipelined(args.steps, with_layer=False)
        e1.record(stream)
        torch.cuda.synchronize()
        cms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([cms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            cms = t.item()
        res["e2e"] = {"value": T * args.steps * world / (ems / 1e3), "unit": "tokens/s",
                      "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4,
                      "ms_per_step": ems / args.steps,
                      "copy_bound": {
                          "ms_per_step": cms / args.steps,
                          "value": T * args.steps * world / (cms / 1e3),
                          "h2d_d2h_gbs_each_way": T * H * 4 * args.steps / (cms / 1e3) / 1e9,
                          "frac": cms / ems,
                          "how": "the same pipeline and copies with the layer left out"},
                      "how": "pinned host x -> device, layer, device y -> pinned host every "
                             "step; copies overlap neighbouring steps' layers on two copy "
                             "streams"}
    layer.close()
    del layer, x, y
    torch.cuda.empty_cache()
    return res


def run_ours(args, rank, world, dev):
    import torch.distributed as dist
    T = args.tokens
    keep_host = rank == 0 and world == 1 and not args.no_cpu_baseline
    head = time_layer(args, rank, world, dev, args.ep_mode, args.routing, e2e=not args.no_e2e,
                      keep_host=keep_host)
    stage_ms, nfw = head["stage_ms"], head["nfw"]
    pk = peaks()
    flop = layer_flop(T)
    ms = head["ms"]
    value = head["value"]
    gemm_flop = T * K * 6 * H * I
    w13_flop = T * K * 4 * H * I
    w13_ms = stage_ms["gemm_w13"] / max(nfw, 1)
    w2_ms = stage_ms["gemm_w2"] / max(nfw, 1)
    achieved = w13_flop / (w13_ms / 1e3) / 1e12
    clocks = head["clocks"]
    # denominator: the burst cuBLAS figure when the SM clock stayed at its
    # maximum through the timed region, the power-capped sustained figure if not
    at_max = bool(clocks) and clocks["sm_mhz"] >= 0.95 * clocks["sm_max_mhz"]
    peak = pk["bf16"] if at_max else pk["bf16_sustained"]
    peak_kind = (f"{pk['source']} bf16 {'burst' if at_max else 'sustained'} "
                 f"(burst {pk['bf16']}, sustained {pk['bf16_sustained']})")
    traffic = None
    tf = os.path.join(ROOT, "profiles", "gemm_w13_traffic.json")
    if os.path.exists(tf):
        with open(tf) as f:
            traffic = json.load(f).get("bytes_per_launch_scaled")

    out = {
        "metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": args.dtype, "data": "synthetic",
        "config": bench_config(args, world),
        "weights": f"{args.dtype} packed from fp32 N(0,0.02), random init",
        "load": head["load"],
        "layer_tflops": flop * args.steps * world / (ms / 1e3) / 1e12 / world,
        "grouped_gemm_tflops": gemm_flop / ((w13_ms + w2_ms) / 1e3) / 1e12,
        "frac_of_bf16_peak_layer": flop / (ms / args.steps / 1e3) / 1e12 / pk["bf16"],
        "stages_ms_per_step": {k: v / max(nfw, 1) for k, v in stage_ms.items()},
        "roofline": {"kernel": "gemm_pair_kernel<SwiGLU,bf16> (W1||W3 grouped GEMM, CTA pairs)",
                     "bound": "tensor", "achieved": achieved,
                     "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_kind": peak_kind,
                     "flop_per_launch": w13_flop},
        "gpu_launches": head["gpu_launches"],
        "clocks": clocks,
    }
    if world > 1:
        out["roofline"]["note"] = ("expert-parallel: the W1||W3 stage time includes waiting "
                                   "for remote rows; the 1-GPU line is the kernel figure")
        out["exchange_bytes_per_step"] = head["exchange_bytes_per_step"]
        out["ep_timeline_us"] = head["timeline"]
        if not args.no_variants:
            # the other placements / routings of the same layer, same K / W
            var = {}
            combos = [(m, r, "fused") for m in ("owner", "balanced") for r in ("zipf", "uniform")]
            combos.append((args.ep_mode, args.routing, "staged"))
            for mode, routing, pipe in combos:
                key = f"{mode}_{routing}_{pipe}"
                if (mode, routing, pipe) == (args.ep_mode, args.routing, "fused"):
                    continue
                r = time_layer(args, rank, world, dev, mode, routing, pipe)
                var[key] = {"value": r["value"], "ms_per_step": r["ms_per_step"],
                            "load": r["load"], "timeline_rank0_us": r["timeline"][0]}
            out["variants"] = var
        # the same routing on one GPU (rank 0, the others wait): the weak-scaling
        # efficiency of this line against its own single-GPU rate
        if rank == 0:
            one = time_layer(args, 0, 1, dev, args.ep_mode, args.routing)
            out["one_gpu_same_routing"] = {
                "value": one["value"], "ms_per_step": one["ms_per_step"],
                "efficiency": value / (world * one["value"])}
        dist.barrier()
    if "e2e" in head:
        out["e2e"] = head["e2e"]
    if not args.no_dense and world == 1:
        # single-GPU measurements (with several ranks the others would wait
        # for rank 0 in a barrier meanwhile)
        out["dense_gemm_sweep"] = dense_sweep(dev)
        out["dense_mlp"] = mlp_bench(dev)
    if not args.no_model:
        import torch
        torch.cuda.empty_cache()
        fm = model_bench(dev, rank=rank, world=world)
        if rank == 0:
            out["full_model"] = fm
        if world > 1 and args.model_ep != "none":
            fm = model_bench(dev, rank=rank, world=world, ep=args.model_ep)
            if rank == 0:
                out["full_model_ep"] = fm
    if "host" in head:
        w_host, cpu_inputs = head["host"]
        out["cpu_baseline"] = cpu_baseline(args, cpu_inputs, w_host)
    return out


# ------------------------------------------------------------------ dense
DENSE_M = (512, 4096, 16384)
DENSE_N = (2048, 3072, 65536)


def dense_sweep(dev, K=2048, reps=10):
    """C[M,N] = A[M,2048] . B[N,2048]^T on the tcgen05 core,
    bf16 operands and fp32 operands (TF32 math), fp32 output; TFLOP/s per shape.

    Device time per GEMM: `reps` b2_gemm_nt calls are captured once into a CUDA
    graph and the replay is timed with CUDA events, so the host-side cost of a
    call (ctypes, tensor-map encoding) does not hide the kernel time of the
    small shapes.  cublas_bf16_tflops is torch.mm (cuBLAS, bf16 in and out) on
    the same bf16 operands, timed the same way, for comparison only."""
    import torch
    from final_b200 import gemm_nt, to_bf16
    res = []
    g = torch.Generator(device=dev).manual_seed(2)

    def graph_ms(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / reps

    for M in DENSE_M:
        for N in DENSE_N:
            A = torch.randn(M, K, device=dev, generator=g)
            B = torch.randn(N, K, device=dev, generator=g) * 0.02
            C = torch.empty(M, N, device=dev)
            Ab, Bb = to_bf16(A), to_bf16(B)
            row = {"M": M, "N": N, "K": K}
            flop = 2.0 * M * N * K
            for name, a, b in (("bf16", Ab, Bb), ("tf32", A, B)):
                ms = graph_ms(lambda: gemm_nt(a, b, out=C, dtype=name))
                row[f"{name}_tflops"] = flop / (ms / 1e3) / 1e12
                row[f"{name}_ms"] = ms
            ms = graph_ms(lambda: torch.mm(Ab, Bb.t()))
            row["cublas_bf16_tflops"] = flop / (ms / 1e3) / 1e12
            res.append(row)
            del A, B, C, Ab, Bb
    torch.cuda.empty_cache()
    return res


def gemm_only(args, dev):
    """One dense shape, bf16 operands, fp32 C: warm-up + timed launches."""
    import torch
    from final_b200 import gemm_nt, to_bf16
    M, N, Kd = args.gemm
    g = torch.Generator(device=dev).manual_seed(2)
    A = to_bf16(torch.randn(M, Kd, device=dev, generator=g))
    B = to_bf16(torch.randn(N, Kd, device=dev, generator=g) * 0.02)
    C = torch.empty(M, N, device=dev)
    for _ in range(args.warmup):
        gemm_nt(A, B, out=C)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        gemm_nt(A, B, out=C)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    return {"metric": "dense_gemm_tflops", "M": M, "N": N, "K": Kd, "ms": ms,
            "tflops": 2.0 * M * N * Kd / (ms / 1e3) / 1e12, "steps": args.steps,
            "warmup": args.warmup}


def gemm_configs(args, dev, reps=20):
    """Every kernel configuration of b2_gemm_nt_config on one shape: device
    time per call (CUDA-graph replay of `reps` calls, so launch overhead of
    the host is not measured) and the error against fp64."""
    import torch
    from final_b200 import gemm_nt, to_bf16
    from final_b200.moe import gemm_plan
    M, N, Kd = args.gemm_configs
    g = torch.Generator(device=dev).manual_seed(2)
    A = to_bf16(torch.randn(M, Kd, device=dev, generator=g))
    B = to_bf16(torch.randn(N, Kd, device=dev, generator=g) * 0.02)
    C = torch.empty(M, N, device=dev)
    ref = A.double() @ B.double().T
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    cfgs = ([("single", bn, 1) for bn in (64, 128, 256)] + [("pair", 256, 1)] +
            [("splitk", bn, sp) for bn in (128, 256) for sp in (2, 3, 4, 6, 8)] +
            [("pairsplit", 256, sp) for sp in (2, 3, 4)])
    res = {"metric": "dense_gemm_configs", "M": M, "N": N, "K": Kd,
           "plan": list(gemm_plan(M, N, Kd, "bf16", sms)), "us": {}}
    for cfg in cfgs:
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            try:
                gemm_nt(A, B, out=C, config=cfg, stream=s)
            except Exception:
                continue
            s.synchronize()
            err = ((C.double() - ref).abs().max() / ref.abs().max()).item()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                for _ in range(reps):
                    gemm_nt(A, B, out=C, config=cfg, stream=s)
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        res["us"]["/".join(map(str, cfg))] = [round(e0.elapsed_time(e1) / (5 * reps) * 1e3, 2),
                                              err]
    return res


def gemm_launches(args, dev):
    """Four eager launches of each of six kernel configurations of
    b2_gemm_nt_config, then four of torch.mm (cuBLAS) on the same bf16
    operands: run under `ncu --metrics gpu__time_duration.sum`, the launch
    list gives each kernel's own duration next to cuBLAS's."""
    import torch
    from final_b200 import gemm_nt, to_bf16
    M, N, Kd = args.gemm_launches
    g = torch.Generator(device=dev).manual_seed(2)
    A = to_bf16(torch.randn(M, Kd, device=dev, generator=g))
    B = to_bf16(torch.randn(N, Kd, device=dev, generator=g) * 0.02)
    C = torch.empty(M, N, device=dev)
    cfgs = [("single", 64, 1), ("single", 128, 1), ("pair", 256, 1), ("splitk", 128, 2),
            ("splitk", 128, 4), ("pairsplit", 256, 2)]
    for cfg in cfgs:
        for _ in range(4):
            gemm_nt(A, B, out=C, config=cfg)
        torch.cuda.synchronize()
    for _ in range(4):
        torch.mm(A, B.t())
    torch.cuda.synchronize()
    return {"metric": "dense_gemm_launches", "M": M, "N": N, "K": Kd,
            "configs": ["/".join(map(str, c)) for c in cfgs] + ["torch.mm"], "launches_each": 4}


def mlp_bench(dev, T=16384, Hd=2048, Id=7168, reps=10):
    """Dense SwiGLU MLP of the layers without experts (I = 7168) over T tokens
    on the same GEMM core: tokens/s and TFLOP/s (6*T*H*I FLOP per forward)."""
    import torch
    from final_b200 import MLP
    g = torch.Generator(device=dev).manual_seed(3)
    w1 = torch.randn(Id, Hd, device=dev, generator=g) * 0.02
    w3 = torch.randn(Id, Hd, device=dev, generator=g) * 0.02
    w2 = torch.randn(Hd, Id, device=dev, generator=g) * 0.02
    mlp = MLP(w1, w2, w3, max_tokens=T)
    del w1, w2, w3
    x = torch.randn(T, Hd, device=dev, generator=g)
    y = torch.empty(T, Hd, device=dev)
    out = {"tokens": T, "hidden": Hd, "inter": Id}
    for name, n in (("prefill", T), ("decode_64", 64)):
        for _ in range(3):
            mlp.forward_gpu(x, y, 1, n, Hd)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            mlp.forward_gpu(x, y, 1, n, Hd)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        out[name] = {"tokens": n, "ms": ms, "tokens_per_s": n / (ms / 1e3),
                     "tflops": 6.0 * n * Hd * Id / (ms / 1e3) / 1e12}
    st = mlp.device_status()
    mlp.close()
    if st:
        raise RuntimeError(f"MLP device status 0x{st:x}")
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------ model
def model_bench(dev, B=32, S=512, steps=5, warmup=3, rank=0, world=1, ep=None):
    """Config 5: the whole LFM2-8B-A1B-shaped model (24 layers, random-init
    weights, vocab 65536) over batch 32 x seq 512 token ids uniform in
    [0, 65536): samples/s of the last-token logits, device-timed with inputs
    resident, and end to end with the ids copied from pinned host memory and
    the logits copied back every step.  With several ranks every GPU holds a
    replica of the model (36 GB of its 180 GB) and runs its own batch of 32:
    no activation crosses NVLink; samples/s counts all ranks' samples over the
    slowest rank's time (barrier before and after, max over ranks).  With
    `ep` ("balanced" / "owner") the model is the expert-parallel one instead:
    each rank still runs its own batch of 32, and every MoE layer exchanges
    expert rows with the other ranks over NVLink."""
    import torch
    import torch.distributed as dist
    from final_b200 import launch_count
    from final_b200.lfm2 import LFM2Model, model_flop, synthetic_weights
    t0 = time.time()
    kw = {} if ep is None else dict(expert_parallel=ep, world=world, rank=rank)
    model = LFM2Model(synthetic_weights(dev, seed=11), max_batch=B, max_seq=S, device=dev, **kw)
    torch.cuda.empty_cache()
    build_s = time.time() - t0
    g = torch.Generator(device=dev).manual_seed(12 + 1000 * rank)
    ids = torch.randint(0, 65536, (B, S), device=dev, generator=g, dtype=torch.int32)
    logits = torch.empty(B, 65536, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        model.forward_gpu(ids, logits, B, S, stream)
    torch.cuda.synchronize()
    st = model.device_status()
    if st:
        raise RuntimeError(f"model device status 0x{st:x}")

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    sampler = ClockSampler(smi_index_for(dev.index))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    n0 = launch_count()
    e0.record(stream)
    for _ in range(steps):
        model.forward_gpu(ids, logits, B, S, stream)
    e1.record(stream)
    torch.cuda.synchronize()
    n1 = launch_count()
    clocks = sampler.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    # end to end: ids from pinned host memory, logits back to pinned host memory
    ids_h = ids.cpu().pin_memory()
    logits_h = torch.empty(B, 65536, dtype=torch.float32).pin_memory()
    ids_d = torch.empty_like(ids)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        ids_d.copy_(ids_h, non_blocking=True)
        model.forward_gpu(ids_d, logits, B, S, stream)
        logits_h.copy_(logits, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ems = max_over_ranks(e0.elapsed_time(e1) / steps)
    st = model.device_status()
    if st:
        raise RuntimeError(f"model device status 0x{st:x}")
    flop = model_flop(B, S)
    pk = peaks()
    out = {"workload": "lfm2_8b_a1b_shaped_forward", "batch_per_gpu": B, "seq_len": S,
           "layers": 24, "vocab": 65536, "n_gpus": world,
           "parallelism": ("single" if world == 1 and ep is None else
                           f"replica per GPU x{world}" if ep is None else
                           f"expert-parallel MoE layers ({ep}) x{world}"),
           "scaling": "weak", "weights": "random init (bf16 projections / experts from fp32)",
           "samples_per_s": B * world / (ms / 1e3), "tokens_per_s": B * S * world / (ms / 1e3),
           "ms_per_forward": ms, "tflops_per_gpu": flop / (ms / 1e3) / 1e12,
           "frac_of_bf16_peak": flop / (ms / 1e3) / 1e12 / pk["bf16"],
           "flop_per_forward": flop, "gpu_launches_per_forward": int(n1 - n0) // steps,
           "e2e": {"samples_per_s": B * world / (ems / 1e3), "ms_per_step": ems,
                   "h2d_bytes_per_step": B * S * 4, "d2h_bytes_per_step": B * 65536 * 4},
           "device_bytes": model.device_bytes(), "build_s": build_s, "clocks": clocks,
           "steps": steps, "warmup": warmup}
    model.close()
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------ CPU
def cpu_sample_rate(x, gate, bias, w1, w3, w2, target_s, max_tokens=None):
    """Time the oracle (C restatement of the reference MoE, all host threads)
    on growing token samples until ~target_s of work; returns tokens/s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as o
    o.lib()
    threads = o.num_threads()
    n = 16
    best = None
    while True:
        xs = x[:n]
        t0 = time.perf_counter()
        o.moe_forward(xs, gate, bias, w1, w2, w3, K=K)
        dt = time.perf_counter() - t0
        best = (n, dt)
        if dt * 3 > target_s or (max_tokens and n * 2 > max_tokens) or n * 2 > x.shape[0]:
            break
        n *= 2
    n, dt = best
    return n / dt, n, dt, threads


def cpu_config1_ms(x, gate, bias, w1, w3, w2, reps=5):
    """The oracle on 64 tokens (config 1's size) of the same inputs: best of
    `reps` forwards, in ms."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as o
    best = None
    for _ in range(reps):
        t0 = time.perf_counter()
        o.moe_forward(x[:64], gate, bias, w1, w2, w3, K=K)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    return best * 1e3


def cpu_baseline(args, cpu_inputs, w_host):
    x, gate, bias = cpu_inputs
    w1, w3, w2 = w_host
    rate, n, dt, threads = cpu_sample_rate(x, gate, bias, w1, w3, w2, args.cpu_seconds)
    ms64 = cpu_config1_ms(x, gate, bias, w1, w3, w2)
    return {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} tokens of the same workload (fp32 oracle, {dt:.1f} s)",
            "config1_64_tokens": {"ms_per_forward": ms64, "tokens_per_s": 64 / (ms64 / 1e3),
                                  "sample": "64 tokens of the same inputs, best of 5"}}


def run_reference(args):
    """Reference arm: the reference's MoE semantics on the host cores."""
    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as o
    T = args.tokens
    dev = torch.device("cuda:0") if torch.cuda.is_available() else None
    if dev is not None:
        x, gate, bias, w1, w2, w3 = make_inputs(T, args.routing, dev)
        xc, gc = x.cpu().numpy(), gate.cpu().numpy()
        bc = None if bias is None else bias.cpu().numpy()
        w1c, w3c, w2c = (t.cpu().numpy() for t in (w1, w3, w2))
    else:
        inp = o.moe_inputs(T, H, E, I, SEED, bias=args.routing != "zipf")
        xc, gc, bc = inp["x"], inp["gate"], inp["bias"]
        if args.routing == "zipf":
            o.inject_logits(xc, gc, o.zipf_logits(T, E, SEED))
        w1c, w3c, w2c = inp["w1"], inp["w3"], inp["w2"]
    o.lib()
    threads = o.num_threads()
    # bounded sample per step: size it so warmup+steps take a few minutes at most
    budget_s = max(20.0, min(150.0, 8.0 * (args.steps + args.warmup)))
    per_step = budget_s / (args.steps + args.warmup)
    _, n, _, _ = cpu_sample_rate(xc, gc, bc, w1c, w3c, w2c, per_step)
    rng = np.random.default_rng(0)
    for _ in range(args.warmup):
        s = int(rng.integers(0, T - n + 1))
        o.moe_forward(xc[s:s + n], gc, bc, w1c, w2c, w3c, K=K)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        s = int(rng.integers(0, T - n + 1))
        o.moe_forward(xc[s:s + n], gc, bc, w1c, w2c, w3c, K=K)
    dt = time.perf_counter() - t0
    value = n * args.steps / dt
    out = {"impl": "reference", "metric": "moe_layer_tokens_per_s", "value": value,
           "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": bench_config(args, args.gpus),
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                            "sample": f"{n} tokens per step of the {T}-token workload "
                                      "(C restatement of src/layer.cu MoE, fp32, OpenMP)"},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    if dev is not None:
        out["reference_cuda_kernels_b200"] = ref_gpu_kernels(args, x, gate, bias, w1, w2, w3, dev)
    return out


def ref_gpu_kernels(args, x, gate, bias, w1, w2, w3, dev):
    """The reference's own fp32 CUDA kernels (compiled unmodified for sm_100a,
    oracle/_ref) launched as SparseMoeBlock::forward_gpu does, same workload:
    with the 288 persistent CTAs it ships (src/layer.cu:1474-1490, sized for a
    72-SM part) and, as a tuned variant, with 148*k CTAs for this B200's 148
    SMs (k = 1, 2, 4; its kernels take tasks from an atomic counter, so any
    grid size is valid); the best tuned time is reported beside the shipped one."""
    import ctypes as C
    import torch
    import oracle as o
    r = o.ref_lib()
    if r is None:
        return {"unavailable": "oracle/_ref not built"}
    T = x.shape[0]
    arr = C.c_void_p * E
    p1 = arr(*[w1[e].data_ptr() for e in range(E)])
    p2 = arr(*[w2[e].data_ptr() for e in range(E)])
    p3 = arr(*[w3[e].data_ptr() for e in range(E)])
    vp = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
    y = torch.empty(T, H, device=dev)
    z = [None] * 7

    def timed(ctas, steps=3):
        h = C.c_void_p()
        if r.ref_moe_create(C.cast(p1, C.c_void_p), C.cast(p2, C.c_void_p),
                            C.cast(p3, C.c_void_p), vp(gate), vp(bias), E, K, H, I, T, ctas,
                            C.byref(h)) != 0:
            return None
        for _ in range(2):
            r.ref_moe_forward(h, vp(x), vp(y), T, *z, None)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            r.ref_moe_forward(h, vp(x), vp(y), T, *z, None)
        e1.record()
        torch.cuda.synchronize()
        r.ref_moe_destroy(h)
        return e0.elapsed_time(e1) / steps

    ms = timed(288)
    if ms is None:
        return {"unavailable": "ref_moe_create failed"}
    tuned = {}
    for k in (1, 2, 4):
        t = timed(148 * k)
        if t is not None:
            tuned[148 * k] = t
    out = {"value": T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
           "what": "reference kernels (fp32 FFMA, 288 persistent CTAs as shipped) on this B200"}
    if tuned:
        best = min(tuned, key=tuned.get)
        out["tuned"] = {"persistent_ctas": best, "ms_per_step": tuned[best],
                        "value": T / (tuned[best] / 1e3),
                        "ms_by_ctas": {str(c): v for c, v in tuned.items()},
                        "what": "same kernels with 148*k persistent CTAs (k = 1, 2, 4), best"}
    return out


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(run_reference(args)), flush=True)
        return 0
    import torch
    import torch.distributed as dist
    if args.warmup < 3:
        args.warmup = 3
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    if args.gemm:
        print(json.dumps(gemm_only(args, dev)), flush=True)
        return 0
    if args.gemm_configs:
        print(json.dumps(gemm_configs(args, dev)), flush=True)
        return 0
    if args.gemm_launches:
        print(json.dumps(gemm_launches(args, dev)), flush=True)
        return 0
    if args.model_only:
        fm = model_bench(dev, steps=args.steps, warmup=args.warmup, rank=rank, world=world)
        if rank == 0:
            print(json.dumps(fm), flush=True)
        if world > 1 and args.model_ep != "none":
            fm = model_bench(dev, steps=args.steps, warmup=args.warmup, rank=rank, world=world,
                             ep=args.model_ep)
            if rank == 0:
                print(json.dumps(fm), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return 0
    try:
        out = run_ours(args, rank, world, dev)
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
