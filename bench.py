#!/usr/bin/env python3
"""MoE-block benchmark (one JSON line on rank 0).

Workload: one OLMoE-shaped MoE layer, prefill --
D=2048, 64 experts, top-8 softmax routing (no renorm), SwiGLU FFN 1024, int8
per-row weights with f32 scales, T=512 tokens of f32 activations ~N(0,1),
router and experts N(0,0.02) from a fixed seed.  A step is one pass of the
MoE block over the 512 tokens.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Arms
  ours (default): libomc.so.  `value` = tokens/s with inputs resident in HBM
      (device entry omc_moe_forward_dev: one forward per input buffer is
      captured in a CUDA graph, and the timed region replays it; --stream
      times stream launches instead), timed with CUDA events on the
      launching stream, max over ranks; `e2e` = the same through the host
      entry omc_moe_forward (pinned host x in, host out/top-k back every
      step).  N>1 (--mode ep, the default): expert parallel through the
      library's own NCCL data plane (omc_ep_init with a unique id; each rank
      holds E/N of the layer's experts and routes its own tokens, rows go to
      their experts' ranks and back inside omc_moe_forward[_dev]).  The N>1
      default workload is qwen_ep (the 256-expert
      Qwen-shaped layer, T=8192 tokens in total split over the ranks, router
      bias uniform or --bias zipf); --mode replica runs N independent copies.
  reference: the reference's own CPU MoE (engines/olmoe.c moe(), or the
      workload family's: engines/qwen.c moe_step(), engines/gemma.c route_token
      + expert union; compiled from its sources into oracle/_ref by
      oracle/Makefile) on all host cores, each step a bounded token sample;
      rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

D, I, E, K, T = 2048, 1024, 64, 8, 512
FAMILY, IS, RI8 = "olmoe", 0, 0                      # layer family, shared-expert width, int8 router
SEED_W, SEED_X = 1, 4242
METRIC, UNIT = "MoE-block tokens/s", "tokens/s"
WORKLOAD = "olmoe_layer_prefill_T512"
EXPERT_BYTES = 3 * D * I + 4 * (2 * I + D)          # int8 g,u,d + f32 scales
CONFIG = {"workload": WORKLOAD, "D": D, "I": I, "E": E, "k": K, "T": T,
          "weights": "int8 per-row + f32 scales, N(0,0.02) seed 1",
          "x": "f32 N(0,1) seed 4242, 8 rotating batches",
          "l2": "expert weights 403 MB > 126 MB L2 stream from HBM every step"}

# The BASELINE configs measured by this script (the default line is configs[1]):
#   olmoe_prefill  OLMoE-shaped layer, T=512 (C1)        olmoe_decode  the same, T=1
#   qwen_prefill   Qwen-shaped layer with shared expert, int8 router, T=2048 (C2)
#   qwen_decode    the same, T=1 (C2 decode)
#   olmoe_decode64 / qwen_decode64   one decode step of 64 sequences (T=64), the batched
#                  decode of the next-steps row; run it with --graph (CUDA graph replay)
#   gemma_prefill / gemma_decode / gemma_decode64   a Gemma-4-26B-A4B-shaped layer
#                  (D=2816, 128 experts, top-8, moe_intermediate 704, int8 router;
#                  x is the residual row), T=2048 / 1 / 64
WORKLOADS = {
    "olmoe_prefill": ("olmoe", 512), "olmoe_decode": ("olmoe", 1),
    "qwen_prefill": ("qwen", 2048), "qwen_decode": ("qwen", 1),
    "olmoe_decode64": ("olmoe", 64), "qwen_decode64": ("qwen", 64),
    "gemma_prefill": ("gemma", 2048), "gemma_decode": ("gemma", 1), "gemma_decode64": ("gemma", 64),
    "qwen_ep": ("qwen", 8192),
    "qwen_decode40": ("qwen", 1),
    "qwen_decode64_tier": ("qwen", 64),
}
BIAS = "uniform"                 # qwen_ep: router bias, uniform (none) or zipf
T_TOTAL = None                   # qwen_ep: tokens over all ranks
REF_FN = {"olmoe": "engines/olmoe.c moe()", "qwen": "engines/qwen.c moe_step()",
          "gemma": "engines/gemma.c route_token() + expert union"}


def set_workload(name, tokens=None, world=1, bias="uniform"):
    global D, I, E, K, T, FAMILY, IS, RI8, SEED_W, WORKLOAD, EXPERT_BYTES, CONFIG, BIAS, T_TOTAL
    FAMILY, T = WORKLOADS[name]
    if tokens:
        T = tokens
    if name == "qwen_ep":
        # T tokens in total, T / world per home rank
        T_TOTAL, BIAS = T, bias
        if T % world:
            raise SystemExit(f"qwen_ep: T={T} is not divisible by {world} ranks")
        T = T // world
    if FAMILY == "olmoe":
        D, I, E, K, IS, RI8, SEED_W = 2048, 1024, 64, 8, 0, 0, 1
    elif FAMILY == "gemma":
        D, I, E, K, IS, RI8, SEED_W = 2816, 704, 128, 8, 0, 1, 3
    else:
        D, I, E, K, IS, RI8, SEED_W = 2048, 512, 256, 8, 512, 1, 2
    EXPERT_BYTES = 3 * D * I + 4 * (2 * I + D)
    kind = "decode" if (T == 1 or "decode" in name) else "prefill"
    WORKLOAD = f"{FAMILY}_layer_{kind}_T{T}"
    if name == "qwen_ep":
        WORKLOAD = f"qwen_layer_ep_T{T_TOTAL}_{BIAS}"
    if name == "qwen_decode40":
        WORKLOAD = "qwen_40layers_decode_T1"
    if name == "qwen_decode64_tier":
        WORKLOAD = "qwen_layers_decode64_tiered"
    total = E * EXPERT_BYTES + (3 * D * IS + 4 * (2 * IS + D) if IS else 0)
    CONFIG = {"workload": WORKLOAD, "D": D, "I": I, "E": E, "k": K, "T": T,
              "weights": f"int8 per-row + f32 scales, N(0,0.02) seed {SEED_W}",
              "x": "f32 N(0,1) seed 4242, 8 rotating batches",
              "l2": f"expert weights {total / 1e6:.0f} MB > 126 MB L2 stream from HBM every step"}
    if IS:
        CONFIG.update(shared_expert_I=IS, router="int8 + f32 scale", renorm=1)
    if name == "qwen_ep":
        CONFIG.update(T=T_TOTAL, tokens_total=T_TOTAL, router_bias=BIAS,
                      experts_per_rank=E // world,
                      x="f32 N(0,1), each rank's own seeded tokens, 8 rotating batches")
        if BIAS == "zipf":
            CONFIG["router_bias_rule"] = "bias_e = -1.1 ln(rank_e), rank a seeded permutation of 1..256 (seed 22)"
    if FAMILY == "gemma":
        CONFIG.update(router="int8 + f32 scale (N(0,1) before quantisation)", renorm=1,
                      activation="gelu_tanh", x="f32 N(0,1) residual rows seed 4242, 8 rotating batches")


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return j["hbm_gbs"], j.get("bf16_tflops"), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clocks and throttle reasons sampled every ~5 ms during the timed
    region, read through NVML in a thread (reading only; nothing is set).
    Falls back to `nvidia-smi -lms` when NVML cannot be loaded."""
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))
    SMI_FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                  "clocks_event_reasons.sw_power_cap")

    def __init__(self, cuda_index, period_s=0.005):
        self.cuda_index, self.period = cuda_index, period_s
        self.sm, self.power, self.reasons, self.max_mhz = [], [], set(), None
        self.stop_ev = threading.Event()
        self.thread, self.proc, self.source = None, None, None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(self.cuda_index)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        try:
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except pynvml.NVMLError:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def start(self):
        try:
            nv, h = self._nvml_handle()
        except Exception:  # noqa: BLE001 - any NVML failure selects the fallback
            return self._start_smi()
        self.source = "nvml"
        self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        masks = [(n, getattr(nv, a)) for n, a in self.REASONS]

        def run():
            while not self.stop_ev.is_set():
                try:
                    self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                    self.power.append(nv.nvmlDeviceGetPowerUsage(h) / 1000.0)
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.reasons.update(n for n, m in masks if r & m)
                except nv.NVMLError:
                    pass
                self.stop_ev.wait(self.period)

        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()

    def _start_smi(self):
        self.source = "nvidia-smi"
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.cuda_index), f"--query-gpu={self.SMI_FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return

        def read():
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for ln in self.proc.stdout:
                f = [v.strip() for v in ln.split(",")]
                if len(f) < 7:
                    continue
                try:
                    self.sm.append(float(f[0]))
                    self.max_mhz = float(f[1])
                except ValueError:
                    continue
                self.reasons.update(n for n, v in zip(names, f[3:7]) if v.lower() == "active")

        self.thread = threading.Thread(target=read, daemon=True)
        self.thread.start()

    def stop(self):
        self.stop_ev.set()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no clock samples"],
                    "samples": 0, "source": self.source}
        out = {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.max_mhz,
               "reasons": sorted(self.reasons), "samples": len(self.sm), "source": self.source}
        if self.power:
            out["power_w_median"] = statistics.median(self.power)
        return out


def profiled_traffic(kernel, workload):
    """DRAM bytes (read + write) per launch of `kernel` on `workload` from one
    ncu capture, kept in the data file profiles/traffic.json, or None."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    v = json.load(open(p)).get(f"{kernel}/{workload}")
    return float(v) if isinstance(v, (int, float)) else None


def make_layer():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle
    if FAMILY == "qwen":
        bias = pyoracle.zipf_bias(E, 1.1, seed=22) if BIAS == "zipf" else None
        return pyoracle, pyoracle.make_layer(pyoracle.FAMILY_QWEN, D, I, E, K, SEED_W, renorm=1, router_i8=1,
                                             has_shared=1, Is=IS, router_bias=bias)
    if FAMILY == "gemma":
        return pyoracle, pyoracle.gemma_layer(SEED_W, D=D, I=I, E=E, k=K)
    return pyoracle, pyoracle.olmoe_layer(SEED_W, D=D, I=I, E=E, k=K)


def cpu_reference_tokens_per_s(pyoracle, L, budget_s, kind_pref="reference"):
    """Time the reference's CPU MoE on a bounded token sample; returns
    (tokens/s, sample tokens, kind, cores, seconds)."""
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    fn, kind = None, "port"
    if kind_pref == "reference" and pyoracle.ref_lib(FAMILY) is not None:
        fn, kind = (lambda xx: pyoracle.reference_moe(L, xx)), "reference"
    else:
        fn = lambda xx: pyoracle.oracle_moe(L, xx)[0]  # noqa: E731
    x = pyoracle.normal(SEED_X, (T, D))
    t0 = time.perf_counter()
    fn(x[:16])
    probe = max(time.perf_counter() - t0, 1e-3)
    n = int(min(T, max(16, 16 * budget_s / probe)))
    reps, tot, t0 = 0, 0, time.perf_counter()
    while True:
        fn(x[:n])
        reps += 1
        tot += n
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return tot / dt, n, kind, cores, dt


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    pyoracle, L = make_layer()
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    if pyoracle.ref_lib(FAMILY) is not None:
        kind, fn = "reference", (lambda xx: pyoracle.reference_moe(L, xx))
    else:
        kind, fn = "port", (lambda xx: pyoracle.oracle_moe(L, xx)[0])
    x = pyoracle.normal(SEED_X, (T, D))
    if args.workload == "qwen_decode40":
        # one decode step is one token through every layer: the reference's
        # moe_step once per layer (each layer's weights are the same size)
        one = fn
        fn = lambda xx: [one(xx) for _ in range(args.layers)]  # noqa: E731
    # size each step so the whole run stays within ~150 s of CPU time
    per_step = max(0.25, min(10.0, 150.0 / max(args.steps + args.warmup, 1)))
    t0 = time.perf_counter()
    fn(x[:16])
    probe = max(time.perf_counter() - t0, 1e-3)
    n = int(min(T, max(8, 16 * per_step / probe)))
    for _ in range(args.warmup):
        fn(x[:n])
    samples = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn(x[:n])
        samples.append(time.perf_counter() - t0)
    step_s = sum(samples) / len(samples)
    value = n / step_s
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": dict(CONFIG, sample_tokens_per_step=n),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": f"{n} of {T} tokens per step, {REF_FN[FAMILY]} "
                                       f"OpenMP on {cores} threads"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    rank, world, local = env_rank()
    dist = None
    if world > 1:
        import torch.distributed as dist  # noqa: F811
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    dev = local
    torch.cuda.set_device(dev)
    import overhang_b200 as ob
    ob.init(dev, 1 << 30)      # one layer: 403 MB of experts + router
    ep_mode = world > 1 and args.mode == "ep"
    if ep_mode:
        # the library's own NCCL group: rank 0's unique id, passed over torch.distributed
        uid = [ob.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ob.ep_init(rank, world, uid[0])    # this rank holds experts [rank*E/world, (rank+1)*E/world)
        ob.ep_set_combine(ob.EP_RANKSUM if args.ep_combine == "ranksum" else ob.EP_EXACT)
    pyoracle, L = make_layer()
    tier = args.tier if args.tier and not ep_mode else 0
    layer = ob.MoELayer.from_oracle_layer(0, L, tier=(tier, 1, 0) if tier else None)
    nbuf = 8
    xs = [torch.from_numpy(pyoracle.normal(SEED_X + rank * nbuf + i, (T, D))).to(f"cuda:{dev}")
          for i in range(nbuf)]
    out = torch.empty((T, D), dtype=torch.float32, device=f"cuda:{dev}")
    idx = torch.empty((T, K), dtype=torch.int32, device=f"cuda:{dev}")
    wts = torch.empty((T, K), dtype=torch.float32, device=f"cuda:{dev}")
    # a dedicated stream: the library enqueues on it and the events time it
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream

    def step(i):
        layer.forward_dev(xs[i % nbuf].data_ptr(), T, out.data_ptr(), idx.data_ptr(), wts.data_ptr(),
                          sptr)

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        step(i)
    ob.sync()

    # per-stage device time, a diagnostic pass before the timed region
    # (profiling events between kernels, one synchronised forward at a time)
    ob.decode_stats(reset=True)
    ob.set_profiling(True)
    st = []
    pmiss0 = layer.tier_stats(tier)[5] if tier else 0
    for i in range(5):
        step(i)
        torch.cuda.synchronize()
        st.append(ob.stage_times())
    ob.set_profiling(False)
    # which router the forward took, and the bounded router's counters for the
    # last diagnostic forward (exact chains, retried tokens)
    rstats = ob.router_stats()
    bounded = (ob.router_mode() == ob.ROUTER_BOUNDED or
               (ob.router_mode() == ob.ROUTER_AUTO and E >= 128)) and T >= 16 and FAMILY != "gemma"
    router_info = {"mode": "bounded" if bounded else "exact"}
    dstats = ob.decode_stats(reset=True)
    if dstats["early"] + dstats["waited"]:
        # the fused decode: forwards of the diagnostic pass whose top-k sets
        # the logit intervals decided (streaming before the exact selection)
        router_info["decode_sets_decided_early"] = f'{dstats["early"]}/{dstats["early"] + dstats["waited"]}'

    if bounded:
        router_info.update({"exact_chains_per_token": rstats["jobs"] / T, "retried_tokens": rstats["retried_tokens"],
                            "whole_tokens": rstats["whole_tokens"]})
    prof_misses = ((layer.tier_stats(tier)[5] - pmiss0) / 5) if tier else 0
    stage_names = [n for n, _ in st[-1]] if st and st[-1] else []
    stage_ms = np.array([[v for _, v in row] for row in st]).mean(axis=0).tolist() if stage_names else []
    stages = dict(zip(stage_names, stage_ms))
    # the dominant kernel: the gate/up expert pass (2/3 of the weight bytes)
    # the dominant kernel: the gate/up expert pass (2/3 of the weight bytes),
    # or at decode sizes the fused kernel that is the whole block
    dom = ("gemm_gateup" if "gemm_gateup" in stages else
           "decode_moe" if "decode_moe" in stages else "gemv_gateup")

    graphs = None
    if args.graph and not ep_mode and not tier:
        # one captured forward per input buffer (graph i replays the forward of
        # buffer i); the timed region replays graph i % nbuf at step i, so it
        # runs exactly the requested steps
        ok = 1
        try:
            ob.launch_count(reset=True)
            graphs = []
            for i in range(nbuf):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    step(i)
                graphs.append(g)
            graph_launches = ob.launch_count() / nbuf
            for g in graphs:
                g.replay()
            torch.cuda.synchronize()
        except Exception as exc:   # time stream launches instead, on every rank alike
            print(f"[bench] CUDA graph capture failed ({exc}); timing stream launches", file=sys.stderr)
            ok = 0
            torch.cuda.synchronize()
        if dist:
            f = torch.tensor([ok], device=f"cuda:{dev}")
            dist.all_reduce(f, op=dist.ReduceOp.MIN)
            ok = int(f.item())
        if not ok:
            graphs = None

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed_pass():
        """Exactly args.steps steps between CUDA events on the launching
        stream, bracketed by a barrier and a synchronize; max over ranks."""
        barrier()
        e0.record(stream)
        for i in range(args.steps):
            if graphs is None:
                step(i)
            else:
                graphs[i % nbuf].replay()
        e1.record(stream)
        barrier()
        ms = e0.elapsed_time(e1)
        if dist:
            tt = torch.tensor([ms], device=f"cuda:{dev}")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        return ms

    miss0 = layer.tier_stats(tier)[5] if tier else 0
    clk = ClockSampler(dev)
    clk.start()
    ob.launch_count(reset=True)
    if graphs is None:
        ob.time_stage(dom)      # one event pair around `dom` per step, on the launching stream
    # the timed pass is repeated until the passes add up to >= --min-seconds
    # (every rank runs the same count); the line reports the median pass
    passes = [timed_pass()]
    repeats = max(1, int(np.ceil(args.min_seconds * 1e3 / max(passes[0], 1e-3))))
    if dist:
        rr = torch.tensor([repeats], device=f"cuda:{dev}")
        dist.all_reduce(rr, op=dist.ReduceOp.MAX)
        repeats = int(rr.item())
    while len(passes) < repeats:
        passes.append(timed_pass())
    launches = (ob.launch_count() if graphs is None else graph_launches * args.steps * len(passes)) / len(passes)
    clocks = clk.stop()
    miss1 = layer.tier_stats(tier)[5] if tier else 0
    if graphs is not None:
        # the dominant kernel's launch time, from a short pass outside the graphs
        ob.time_stage(dom)
        for i in range(max(16, args.steps // 8)):
            step(i)
        torch.cuda.synchronize()
    dom_ms, dom_n = ob.stage_timer()
    ob.time_stage(None)
    ob.sync()
    t_max = float(statistics.median(passes))
    other_combine = None
    if ep_mode:
        # the other return mode, timed the same way (three passes), for comparison
        other = "exact" if args.ep_combine == "ranksum" else "ranksum"
        ob.ep_set_combine(ob.EP_EXACT if other == "exact" else ob.EP_RANKSUM)
        for i in range(args.warmup):
            step(i)
        op = float(statistics.median([timed_pass() for _ in range(3)]))
        ob.ep_set_combine(ob.EP_RANKSUM if args.ep_combine == "ranksum" else ob.EP_EXACT)
        other_combine = {"ep_combine": other, "value": world * T * args.steps / (op / 1e3),
                         "ms_per_step": op / args.steps}
    value = world * T * args.steps / (t_max / 1e3)

    # end to end through the host entry: pinned x in, out + routing back
    hx = [torch.from_numpy(pyoracle.normal(SEED_X + rank * nbuf + i, (T, D))).pin_memory() for i in range(nbuf)]
    hout = torch.empty((T, D), dtype=torch.float32).pin_memory()
    hidx = torch.empty((T, K), dtype=torch.int32).pin_memory()
    hw = torch.empty((T, K), dtype=torch.float32).pin_memory()
    lib = ob.lib()

    def step_e2e(i):
        rc = lib.omc_moe_forward(0, C.c_void_p(hx[i % nbuf].data_ptr()), T, C.c_void_p(hout.data_ptr()),
                                 C.c_void_p(hidx.data_ptr()), C.c_void_p(hw.data_ptr()))
        ob.check(rc, "omc_moe_forward")

    def timed_e2e(fn_pass):
        barrier()
        t0 = time.perf_counter()
        fn_pass()
        s_ = time.perf_counter() - t0
        if dist:
            tt = torch.tensor([s_], device=f"cuda:{dev}")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            s_ = float(tt.item())
        return s_

    # the blocking host entry: every call uploads x, runs the forward, downloads out
    for i in range(args.warmup):
        step_e2e(i)
    e2e_block_s = timed_e2e(lambda: [step_e2e(i) for i in range(args.steps)])
    e2e_mode = "omc_moe_forward (blocking)"
    e2e_s = e2e_block_s
    if not ep_mode:
        # the pipelined host entry (omc_moe_forward_async): step i's forward overlaps
        # step i+1's upload and step i-1's download; two calls are kept in flight
        houts = [torch.empty((T, D), dtype=torch.float32).pin_memory() for _ in range(nbuf)]
        hidxs = [torch.empty((T, K), dtype=torch.int32).pin_memory() for _ in range(nbuf)]
        hws = [torch.empty((T, K), dtype=torch.float32).pin_memory() for _ in range(nbuf)]

        def pipelined(n):
            ticks = []
            for i in range(n):
                t = C.c_longlong(-1)
                ob.check(lib.omc_moe_forward_async(0, C.c_void_p(hx[i % nbuf].data_ptr()), T,
                                                   C.c_void_p(houts[i % nbuf].data_ptr()),
                                                   C.c_void_p(hidxs[i % nbuf].data_ptr()),
                                                   C.c_void_p(hws[i % nbuf].data_ptr()), C.byref(t)),
                         "omc_moe_forward_async")
                ticks.append(t.value)
                if i >= 2:
                    ob.check(lib.omc_moe_wait(ticks[i - 2]), "omc_moe_wait")
            ob.check(lib.omc_moe_wait(ticks[-1]), "omc_moe_wait")

        pipelined(args.warmup)
        e2e_s = timed_e2e(lambda: pipelined(args.steps))
        e2e_mode = "omc_moe_forward_async (pipelined, 2 calls in flight)"
    e2e = world * T * args.steps / e2e_s

    hbm, tf, src = peaks()
    # algorithmic bytes of one launch of the dominant kernel: every active
    # expert's int8 gate+up rows and their scales, the f16 copy of the tokens
    # it gathers rows from (T x D) and the f16 h it writes (one row per slot).
    idx_np = idx.cpu().numpy()
    balance = None
    if ep_mode:
        # this rank's gate/up launch: its experts that received slots, those slots,
        # and the token rows it received (one per token with any expert here)
        allidx = [torch.empty_like(idx) for _ in range(world)]
        dist.all_gather(allidx, idx)
        full = np.concatenate([a.cpu().numpy() for a in allidx])
        lo, hi = rank * E // world, (rank + 1) * E // world
        here = (full >= lo) & (full < hi)
        n_active = int(len(np.unique(full[here])))
        rows = int(here.sum())
        recv_rows = int(here.any(axis=1).sum())
        per_rank = [int(((full >= r * E // world) & (full < (r + 1) * E // world)).sum()) for r in range(world)]
        balance = {"slots_per_rank": per_rank, "max_over_mean": max(per_rank) / (sum(per_rank) / world)}
    else:
        n_active, rows = int(len(np.unique(idx_np))), T * K
        recv_rows = T
    shared_w = (2 * IS * D + 2 * IS * 4) if IS else 0          # the shared expert's gate+up
    srows = T if IS else 0
    # the whole step's weight bytes (every active expert + shared + router) over the step time
    router_bytes = (E * D * (1 if RI8 else 4) + (4 * E if RI8 else 0) + (4 * D if IS else 0)
                    + (2 * 4 * D + 4 * E if FAMILY == "gemma" else 0))
    step_bytes = n_active * EXPERT_BYTES + (3 * D * IS + 4 * (2 * IS + D) if IS else 0) + router_bytes
    # one GPU's algorithmic FLOP per step (per token: k experts' three projections, the
    # router, and the shared expert with its gate)
    step_flop = T * (2 * K * 3 * D * I + 2 * D * E + ((2 * 3 * D * IS + 2 * D) if IS else 0))
    if dom == "gemm_gateup":
        xh_rows = recv_rows + (T if IS and ep_mode else 0)
        alg_bytes = (n_active * (2 * I * D + 2 * I * 4) + shared_w + xh_rows * D * 2
                     + (rows + srows) * max(I, IS) * 2)
    elif dom == "decode_moe":
        # one launch is the block: every weight byte of the step, x in, out back
        alg_bytes = step_bytes + 2 * T * D * 4
    else:
        alg_bytes = n_active * (2 * I * D + 2 * I * 4) + shared_w + T * D * 4 + (T * K + srows) * max(I, IS) * 4
    achieved = alg_bytes / (dom_ms / 1e3) / 1e9 if dom_ms > 0 else None
    traffic = profiled_traffic(dom, args.workload)
    # the gate/up GEMM's FLOP per launch (every slot's two I x D products, and the
    # shared expert's for the home tokens): the tensor roofline of the large-T rows
    dom_flop = 2 * 2 * I * D * rows + (2 * 2 * IS * D * T if IS else 0)
    roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm if achieved else None, "traffic": traffic}
    if args.workload == "qwen_ep" and dom == "gemm_gateup" and dom_ms > 0 and tf:
        # M_avg = 256 rows per expert: compute-bound, judged against the bf16 peak
        ach_t = dom_flop / (dom_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": ach_t, "peak": tf, "unit": "TFLOP/s", "frac": ach_t / tf,
                "traffic": traffic, "hbm_achieved_gbs": achieved}
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max / args.steps, "higher_is_better": True,
            "scaling": "strong" if args.workload == "qwen_ep" else "weak", "vs_baseline": None,
            "dtype": "f16xint8->f32",
            "data": "synthetic",
            "config": dict(CONFIG, parallelism=(f"ep{world}" if ep_mode else f"replica{world}"),
                           launch=("cuda_graph" if graphs is not None else "stream"),
                           tokens_per_rank=T),
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": T * D * 4,
                    "d2h_bytes_per_step": T * D * 4 + T * K * 8, "entry": e2e_mode,
                    "blocking_value": world * T * args.steps / e2e_block_s},
            "gpu_launches": launches,
            "repeats": len(passes), "pass_ms": [round(p, 4) for p in passes],
            "stage_ms": stages,
            "router": router_info,
            "roofline": dict(roof, **{
                         "kernel": dom, "peak_source": src, "alg_bytes_per_launch": alg_bytes,
                         "launch_ms": dom_ms, "launches_timed": dom_n,
                         "step_weight_bytes": step_bytes,
                         "step_hbm_frac": step_bytes / (t_max / args.steps / 1e3) / (hbm * 1e9),
                         "step_flop": step_flop,
                         "step_tensor_frac": (step_flop / (t_max / args.steps / 1e3) / (tf * 1e12)
                                              if tf else None), "flop_per_launch": dom_flop}),
            "clocks": clocks}
    if balance:
        line["ep_balance"] = balance
    if other_combine:
        line["config"]["ep_combine"] = args.ep_combine
        line["ep_other_combine"] = other_combine
    if tier:
        # the tiered store: experts outside the HBM slots cross the host link
        # once per step that routes to them (the tier_fetch stage)
        swaps = layer.tier_stats(tier)[4]
        misses = (miss1 - miss0) / (args.steps * len(passes))   # counted on the device over the timed steps
        f_ms = stages.get("tier_fetch", 0.0)
        line["config"]["tier_hbm_slots"] = tier
        line["tier"] = {"hbm_slots": tier, "experts": E, "swaps": swaps, "misses_per_step": misses,
                        "miss_bytes_per_step": misses * EXPERT_BYTES,
                        # the fetch stage (routing step + copies) timed over the five profiled steps,
                        # against the misses of those same steps
                        "fetch_stage_ms": f_ms, "fetch_misses_per_step": prof_misses,
                        "fetch_gbs": (prof_misses * EXPERT_BYTES / (f_ms / 1e3) / 1e9
                                      if f_ms > 0 and prof_misses else None)}
    if rank == 0 and world == 1 and not args.no_cpu:
        tps, n, kind, cores, dt = cpu_reference_tokens_per_s(pyoracle, L, args.cpu_seconds)
        line["cpu_baseline"] = {"value": tps, "unit": UNIT, "cores": cores, "kind": kind,
                                "sample": f"{n} of {T} tokens per call for {dt:.1f} s, "
                                          f"{REF_FN[FAMILY]} OpenMP"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ob.shutdown()
    if dist:
        dist.destroy_process_group()


def run_layers(args):
    """configs[2] decode: the Qwen-shaped layer's int8 weights for every one of
    args.layers layers resident in HBM at once (40 layers: ~32 GB of experts),
    one decode step = one token through every layer in turn (each layer's
    forward_dev on its own input row, all captured in one CUDA graph).  The
    layers share one seeded expert set, stored once per layer in its own HBM
    (layer l's expert e is seeded expert (e + 37 l) mod E, and layer l's router
    its own seed), so every step streams every layer's routed experts from
    HBM: no layer reads another's weights from L2."""
    import torch
    rank, world, local = env_rank()
    if world > 1:
        raise SystemExit("--workload qwen_decode40 runs on one GPU")
    dev = local
    torch.cuda.set_device(dev)
    import overhang_b200 as ob
    NL = args.layers
    ob.init(dev, 0)
    pyoracle, L = make_layer()
    a = L.arrays
    t0 = time.perf_counter()
    layers = []
    for l in range(NL):
        perm = (np.arange(E) + 37 * l) % E
        rq, rs = pyoracle.quantize_c(pyoracle.normal(SEED_W * 1000003 + 7 + 101 * l, (E, D), 0.02))
        m = ob.MoELayer(l, ob.FAMILY_QWEN, D, I, E, K, rq, rs, 1, 1, IS)
        m.set_experts_packed(a["g"][perm], a["gs"][perm], a["u"][perm], a["us"][perm], a["d"][perm],
                             a["ds"][perm])
        m.set_shared(a["sh_g"], a["sh_gs"], a["sh_u"], a["sh_us"], a["sh_d"], a["sh_ds"], a["sh_gate"])
        layers.append(m)
    t_up = time.perf_counter() - t0
    nbuf = 4
    xs = [[torch.from_numpy(pyoracle.normal(SEED_X + 97 * l + i, (T, D))).cuda() for l in range(NL)]
          for i in range(nbuf)]
    outs = [torch.empty((T, D), dtype=torch.float32, device="cuda") for _ in range(NL)]
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, K), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream

    def step(i):
        for l, m in enumerate(layers):
            m.forward_dev(xs[i % nbuf][l].data_ptr(), T, outs[l].data_ptr(), idx.data_ptr(), wts.data_ptr(), sptr)

    for i in range(args.warmup):
        step(i)
    ob.sync()
    ob.set_profiling(True)
    stage = []
    for i in range(3):
        step(i)
        torch.cuda.synchronize()
        stage.append(ob.stage_times())
    ob.set_profiling(False)
    ob.launch_count(reset=True)
    graphs = []
    for i in range(nbuf):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(i)
        graphs.append(g)
    per_step_launches = ob.launch_count() / nbuf
    for g in graphs:
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed_pass():
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(args.steps):
            graphs[i % nbuf].replay()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    clk = ClockSampler(dev)
    clk.start()
    passes = [timed_pass()]
    repeats = max(1, int(np.ceil(args.min_seconds * 1e3 / max(passes[0], 1e-3))))
    while len(passes) < repeats:
        passes.append(timed_pass())
    clocks = clk.stop()
    t_ms = float(statistics.median(passes))
    step_s = t_ms / args.steps / 1e3
    value = T * args.steps / (t_ms / 1e3)
    hbm, tf, src = peaks()
    # one step's algorithmic bytes: in every layer, each routed expert a token
    # chose (distinct per layer), the shared expert, the int8 router and its
    # scales, the shared gate vector, and x in / out back
    idx_all = []
    for l, m in enumerate(layers):
        _, li, _ = m.forward(xs[0][l].cpu().numpy())
        idx_all.append(len(np.unique(li)))
    shared_bytes = 3 * D * IS + 4 * (2 * IS + D)
    router_bytes = E * D + 4 * E + 4 * D
    step_bytes = sum(n * EXPERT_BYTES + shared_bytes + router_bytes + 2 * T * D * 4 for n in idx_all)
    ach = step_bytes / step_s / 1e9
    # the host entry, one call per layer (x in, out + routing back), every step
    hx = [torch.from_numpy(xs[0][l].cpu().numpy()).pin_memory() for l in range(NL)]
    hout = torch.empty((T, D), dtype=torch.float32).pin_memory()
    lib = ob.lib()

    def host_step():
        for l in range(NL):
            ob.check(lib.omc_moe_forward(l, C.c_void_p(hx[l].data_ptr()), T, C.c_void_p(hout.data_ptr()), None,
                                         None), "omc_moe_forward")

    for _ in range(args.warmup):
        host_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_step()
    e2e = T * args.steps / (time.perf_counter() - t0)
    names = [n for n, _ in stage[-1]]
    st = dict(zip(names, np.array([[v for _, v in row] for row in stage]).mean(axis=0).tolist()))
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32xint8->f32", "data": "synthetic",
            "config": dict(CONFIG, workload=WORKLOAD, layers=NL, parallelism="single",
                           launch="cuda_graph (one step = every layer)",
                           resident_expert_bytes=NL * (E * EXPERT_BYTES + shared_bytes),
                           upload_s=round(t_up, 1),
                           l2="every step streams each layer's own routed experts: distinct HBM per layer"),
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": NL * T * D * 4,
                    "d2h_bytes_per_step": NL * T * D * 4, "entry": "omc_moe_forward per layer (blocking)"},
            "gpu_launches": per_step_launches * args.steps, "repeats": len(passes),
            "pass_ms": [round(v, 4) for v in passes],
            "stage_ms_last_layer": st,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                         "traffic": None, "kernel": "decode_moe (every layer of a step)", "peak_source": src,
                         "alg_bytes_per_step": step_bytes, "layer_us": t_ms / args.steps / NL * 1e3},
            "clocks": clocks}
    print(json.dumps(line), flush=True)
    ob.shutdown()


def run_tier_sweep(args):
    """C4 on the configs[2] set: args.layers Qwen-shaped layers, each a tiered
    store (omc_tier_enable) holding round(args.tier_frac * E) of its routed
    experts in HBM and every expert's home in pinned host memory; one step =
    one decode step of 64 sequences (T = 64) through every layer.  Routed
    experts outside HBM cross the host link once per forward that routes them;
    the hot-store policy (LFRU, include/tier.h) swaps one expert per forward
    at most.  Layer l's expert e is seeded expert (e + 37 l) mod E, as in
    qwen_decode40.  Two extra fully resident copies of layers 0 and 1 check
    that the tiered forwards are bit-identical."""
    import torch
    rank, world, local = env_rank()
    if world > 1:
        raise SystemExit("--workload qwen_decode64_tier runs on one GPU")
    dev = local
    torch.cuda.set_device(dev)
    import overhang_b200 as ob
    NL = args.layers
    ob.init(dev, 0)
    pyoracle, L = make_layer()
    a = L.arrays
    slots = max(1, min(E, int(round(args.tier_frac * E))))
    tiered = slots < E
    t0 = time.perf_counter()
    layers = []
    routers = []

    def build(lid, l, tier_slots):
        perm = (np.arange(E) + 37 * l) % E
        if len(routers) <= l:
            routers.append(pyoracle.quantize_c(pyoracle.normal(SEED_W * 1000003 + 7 + 101 * l, (E, D), 0.02)))
        rq, rs = routers[l]
        m = ob.MoELayer(lid, ob.FAMILY_QWEN, D, I, E, K, rq, rs, 1, 1, IS)
        if tier_slots:
            m.tier_enable(tier_slots, 1, 0)
        m.set_experts_packed(a["g"][perm], a["gs"][perm], a["u"][perm], a["us"][perm], a["d"][perm], a["ds"][perm])
        m.set_shared(a["sh_g"], a["sh_gs"], a["sh_u"], a["sh_us"], a["sh_d"], a["sh_ds"], a["sh_gate"])
        return m

    for l in range(NL):
        layers.append(build(l, l, slots if tiered else 0))
    refs = [build(NL + l, l, 0) for l in range(min(2, NL))] if tiered else []
    t_up = time.perf_counter() - t0
    nbuf = 2
    xs = [[torch.from_numpy(pyoracle.normal(SEED_X + 97 * l + i, (T, D))).cuda() for l in range(NL)]
          for i in range(nbuf)]
    out = torch.empty((T, D), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, K), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream

    def step(i):
        for l, m in enumerate(layers):
            m.forward_dev(xs[i % nbuf][l].data_ptr(), T, out.data_ptr(), idx.data_ptr(), wts.data_ptr(), sptr)

    # bit-identity of tiered forwards (layers 0 and 1) against their resident copies
    identical = None
    if refs:
        identical = True
        for l, r in enumerate(refs):
            xh = xs[0][l].cpu().numpy()
            o1, i1, _ = layers[l].forward(xh)
            o2, i2, _ = r.forward(xh)
            identical &= bool(np.array_equal(i1, i2) and np.array_equal(o1.view(np.uint32), o2.view(np.uint32)))
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    ob.set_profiling(True)
    step(0)
    torch.cuda.synchronize()
    ob.set_profiling(False)
    last_stages = dict(ob.stage_times())
    miss0 = sum(m.tier_stats(slots)[5] for m in layers) if tiered else 0
    swaps0 = sum(m.tier_stats(slots)[4] for m in layers) if tiered else 0
    clk = ClockSampler(dev)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    clocks = clk.stop()
    t_ms = e0.elapsed_time(e1)
    misses = ((sum(m.tier_stats(slots)[5] for m in layers) - miss0) / args.steps) if tiered else 0.0
    swaps = ((sum(m.tier_stats(slots)[4] for m in layers) - swaps0) / args.steps) if tiered else 0.0
    step_s = t_ms / args.steps / 1e3
    miss_bytes = misses * EXPERT_BYTES
    line = {"metric": METRIC, "value": T * args.steps / (t_ms / 1e3), "unit": UNIT, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16xint8->f32",
            "data": "synthetic",
            "config": dict(CONFIG, workload=WORKLOAD, layers=NL, sequences=T, hbm_expert_fraction=slots / E,
                           hbm_slots_per_layer=slots, launch="stream", upload_s=round(t_up, 1),
                           host_expert_bytes=(NL * E * EXPERT_BYTES if tiered else 0)),
            "tier": {"misses_per_step": misses, "miss_bytes_per_step": miss_bytes, "swaps_per_step": swaps,
                     "link_gbs_over_step": miss_bytes / step_s / 1e9,
                     "link_roofline_gbs": 51.0,
                     "step_ms_if_link_bound": miss_bytes / 51e9 * 1e3,
                     "last_layer_stage_ms": last_stages,
                     "bit_identical_to_resident_layers_0_1": identical},
            "clocks": clocks}
    print(json.dumps(line), flush=True)
    ob.shutdown()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--min-seconds", type=float, default=0.5,
                    help="repeat the timed pass of --steps steps until the passes add up to this many seconds; "
                         "the line reports the median pass")
    ap.add_argument("--workload", default=None, choices=sorted(WORKLOADS),
                    help="olmoe_prefill (BASELINE configs[1], the default line on one GPU), olmoe_decode, "
                         "qwen_prefill, qwen_decode, ...; qwen_ep (configs[3], the default on N>1 GPUs)")
    ap.add_argument("--tier-frac", type=float, default=0.5,
                    help="qwen_decode64_tier: fraction of each layer's experts kept in HBM (the rest in pinned "
                         "host memory)")
    ap.add_argument("--ep-combine", default="ranksum", choices=["ranksum", "exact"],
                    help="N>1 expert parallel: results back as one row per (token, rank) summed there "
                         "(ranksum) or one row per slot summed at home (exact: bit-equal to one GPU)")
    ap.add_argument("--layers", type=int, default=40,
                    help="qwen_decode40: layers resident at once (each with its own copy of the expert set)")
    ap.add_argument("--bias", default="uniform", choices=["uniform", "zipf"],
                    help="qwen_ep: router bias (zipf: bias_e = -1.1 ln(rank_e), skewed expert load)")
    ap.add_argument("--graph", action="store_true", default=True,
                    help="capture one forward per input buffer in a CUDA graph and time graph replays "
                         "(the default; --mode ep always times stream launches)")
    ap.add_argument("--stream", dest="graph", action="store_false",
                    help="time stream launches of the forward instead of graph replays")
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per rank instead of the workload's T (the T sweep of the prefill rows)")
    ap.add_argument("--tier", type=int, default=0,
                    help="tiered expert store: keep this many experts in HBM, the rest in pinned host memory "
                         "(LFRU swaps every step; stream launches)")
    ap.add_argument("--mode", default="ep", choices=["ep", "replica"],
                    help="N>1: expert parallel through the library's NCCL data plane (each rank holds E/N "
                         "experts and routes its own tokens), or N independent replicas")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = env_rank()[1]
    if args.workload is None:
        args.workload = "olmoe_prefill" if world == 1 or args.mode == "replica" else "qwen_ep"
    set_workload(args.workload, args.tokens, world, args.bias)
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "qwen_decode40":
        run_layers(args)
    elif args.workload == "qwen_decode64_tier":
        run_tier_sweep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
