#!/usr/bin/env python3
"""MoE-layer tokens/s on B200 for the GPT-OSS-120B-shaped stack.

One step = one pass of T tokens through the 36-layer MoE stack
(h <- h + MoE(RMSNorm(h)), 128 MXFP4 experts per layer, top-4, hidden 2880,
expert FFN 2880; attention omitted, as the config says).  Weights are
generated on the device from seed 0 (~61 GB); inputs are seeded bf16 N(0,1)
tokens drawn from a pool of 16 batches so that routing changes every step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--mode decode|prefill]
                  [--tokens T] [--layers L] [--impl umsx|reference] [--ep]

With N > 1 (torchrun, one rank per GPU) decode runs expert-parallel: rank g holds
experts [g*E/N, (g+1)*E/N) of every layer (61 GB / N) and one token per step
(global batch N), the router is replicated and the dispatch / combine travel as
P2P NVLink stores inside the exchange kernels (ep.EpStack); the value is all
ranks' tokens over the slowest rank's time, and a 2-layer parity check against
one GPU's whole layers runs first (parity_ok).  `--replicas` runs N independent whole-stack
replicas instead.  `--impl reference` times the
reference's own CPU implementation of the path (tools/trace/exact_packed_cpu.h
packed MXFP4 GEMV compiled from the reference sources into oracle/_ref/) on
this host's cores, on rank 0 only.

`--ep` (prefill, T tokens split T/N per rank) splits every layer's experts over the N ranks
(ep.EpPrefill): per layer the token rows travel to the experts' ranks and the outputs come back as
P2P NVLink stores inside the exchange kernels; with `--config skew` it runs configs[3] (Qwen3-30B-A3B
shapes, Zipf(1.2) router bias) and reports every GPU's rows and jobs per layer.  Total work is
fixed as N grows (strong scaling).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HBM_FALLBACK_GBS = 6650.0
PREFILL_MIN_TOKENS = 65  # from this many tokens the MXFP4 layers run the tensor-core prefill path


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--mode", choices=("decode", "prefill"), default="decode")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--experts", type=int, default=None,
                    help="override the expert count (profiling runs that must hold only a few GB)")
    ap.add_argument("--impl", choices=("umsx", "reference"), default="umsx")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the bounded CPU sample")
    ap.add_argument("--ref-seconds", type=float, default=150.0, help="timed budget of the --impl reference arm")
    ap.add_argument("--no-prefill", action="store_true", help="decode line without the prefill sub-record")
    ap.add_argument("--no-extra", action="store_true",
                    help="decode line without the configs[3] skew and residency-bank sub-records")
    ap.add_argument("--ep", action="store_true", help="expert parallelism over the ranks (prefill)")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1 decode as independent replicas instead of expert parallelism")
    ap.add_argument("--config", choices=("stack", "skew", "bank", "configs"), default="stack",
                    help="stack: configs[2] (the headline); skew: configs[3] load-skew layers at T=4096; "
                         "bank: a residency-banked GPT-OSS-120B-shaped layer (LFU / LRU); "
                         "configs: configs[1] (T=1, 16) and configs[4] (27 layers, T=1)")
    a = ap.parse_args()
    if a.tokens is None:
        a.tokens = 1 if a.mode == "decode" else 4096
    a.warmup = max(a.warmup, 3)
    return a


TENSOR_FALLBACK_TFLOPS = 1590.0


def peaks(kind: str = "hbm_gbs"):
    """A measured peak from MEASURED_PEAKS.json (hbm_gbs, bf16_tflops, bf16_tflops_sustained), else the fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p[kind]), "measured"
    except Exception:
        return (HBM_FALLBACK_GBS if kind == "hbm_gbs" else TENSOR_FALLBACK_TFLOPS), "fallback"


def metric_name(a):
    return (f"MoE-layer tokens/s, GPT-OSS-120B-shaped {a.layers}-layer MXFP4 stack, "
            f"{a.mode} T={a.tokens}")


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


# ----------------------------------------------------------------------------- clocks

class Clocks:
    """SM clock and clock-event reasons sampled every 2 ms during the timed region, read-only, by an
    NVML polling thread (nvidia_ml_py); nvidia-smi's CSV sampler is the fallback."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.thread = None
        self.stop = False
        self.nvml = None
        self.proc = None
        self.path = None

    def _handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _poll(self, h):
        import pynvml
        mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop:
            try:
                self.rows.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), mx, get_reasons(h),
                                  pynvml.nvmlDeviceGetPowerUsage(h) / 1e3))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        import threading
        try:
            h = self._handle()
            self.nvml = True
            self.thread = threading.Thread(target=self._poll, args=(h,), daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.rows and time.time() - t0 < 1.0:  # the sampler is running before timing starts
                time.sleep(0.001)
        except Exception:
            self.nvml = None
            q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap")
            self.path = tempfile.mktemp(prefix="clocks_", suffix=".csv")
            try:
                self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                              "--format=csv,noheader,nounits", "-lms", "20"],
                                             stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            except Exception:
                self.proc = None
        return self

    def __exit__(self, *exc):
        self.stop = True
        if self.thread:
            self.thread.join(timeout=2)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.nvml:
            if not self.rows:
                return None
            sm = [r[0] for r in self.rows]
            reasons = sorted({name for r in self.rows for bit, name in self.REASONS.items() if r[2] & bit})
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(r[1] for r in self.rows), "reasons": reasons,
                    "samples": len(self.rows), "power_w_max": max(r[3] for r in self.rows), "source": "nvml"}
        try:
            rows = [r.split(",") for r in open(self.path).read().strip().splitlines() if r.strip()]
            os.unlink(self.path)
        except Exception:
            return None
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if len(r) > 5 + i and r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi"}


# ----------------------------------------------------------------------------- CPU baseline

REF_HOST_LAYERS = 4   # distinct host layers the CPU legs rotate through (about 1.7 GB each)
REF_TOKEN_POOL = 16   # seeded tokens cycled over the steps


def bench_host_weights(orc, cfg, layer: int, threads: int):
    """The GPU stack's layer `layer` (the same seeded tensors umsx_moe_create_synthetic draws),
    drawn on the host with `threads` generator threads."""
    import numpy as np
    from oracle.oracle import LayerWeights
    from tests.helpers import C, U
    E, H, I, s = cfg.experts, cfg.hidden, cfg.intermediate, cfg.seed
    gu = np.empty((E, 2 * I, H // 32 * 17), np.uint8)
    orc.gen_blocks_into(U.QUANT_MXFP4, gu, s, C.stream_id(layer, C.KIND_GATE_UP), 0, E * 2 * I * (H // 32), threads)
    dn = np.empty((E, H, I // 32 * 17), np.uint8)
    orc.gen_blocks_into(U.QUANT_MXFP4, dn, s, C.stream_id(layer, C.KIND_DOWN), 0, E * H * (I // 32), threads)
    rw = orc.gen_normal_f32(s, C.stream_id(layer, C.KIND_ROUTER_W), 0, E * H, cfg.router_sigma).reshape(E, H)
    rb = orc.gen_normal_f32(s, C.stream_id(layer, C.KIND_ROUTER_B), 0, E, cfg.router_bias_sigma)
    gub = orc.gen_normal_bf16(s, C.stream_id(layer, C.KIND_GU_BIAS), 0, E * 2 * I, cfg.bias_sigma).reshape(E, 2 * I)
    db = orc.gen_normal_bf16(s, C.stream_id(layer, C.KIND_DOWN_BIAS), 0, E * H, cfg.bias_sigma).reshape(E, H)
    return LayerWeights(rw, rb, gu, None, None, dn, gub, db)


class ReferenceStack:
    """The reference's exact packed MXFP4 CPU path (oracle/_ref: tools/trace/exact_packed_cpu.h and
    cpu_mxfp4_vnni.cpp compiled from the reference sources), or the oracle port where that build is
    absent, driving the GPT-OSS-120B-shaped stack h <- h + MoE(RMSNorm(h)) on the host cores.  The
    stack's `layers` layers rotate through REF_HOST_LAYERS distinct host layers (layer l uses host
    layer l mod 4, each drawn from the generator's seed for that layer index), so consecutive layers
    touch different expert bytes, as the GPU's 36 distinct layers do."""

    def __init__(self, layers: int):
        from concurrent.futures import ThreadPoolExecutor

        from oracle.oracle import Oracle, RefKernels
        from tests.helpers import oracle_desc
        pkg = load_pkg()
        self.cfg = pkg.configs.GPT_OSS_120B
        self.orc = Oracle()
        self.cores = len(os.sched_getaffinity(0))
        self.layers = layers
        self.ref = None
        try:
            ref = RefKernels()
            if ref.supported():
                self.ref = ref
        except Exception:
            self.ref = None
        self.kind = "reference" if self.ref else "port"
        self.desc = oracle_desc(self.cfg)
        t0 = time.time()
        n = self.n_host = min(REF_HOST_LAYERS, layers)
        self.host = [bench_host_weights(self.orc, self.cfg, l, self.cores) for l in range(n)]
        if self.ref:  # the reference driver packs each layer into its own layout (in parallel)
            with ThreadPoolExecutor(max_workers=n) as ex:
                self.handles = list(ex.map(lambda w: self.ref.layer(self.desc, w), self.host))
            self.host = None  # the packed copies are what it reads
        self.setup_s = time.time() - t0

    def layer(self, l: int, x):
        if self.ref:
            return self.ref.layer_forward(self.handles[l % len(self.handles)], x, self.cfg.hidden, self.cores)
        return self.orc.moe_layer(self.desc, self.host[l % len(self.host)], x, threads=self.cores)["out"]

    def step(self, x):
        import numpy as np
        h = x.astype(np.float32)
        for l in range(self.layers):
            h = (h + self.layer(l, self.orc.rmsnorm(h, 1e-5))).astype(np.float32)
        return h

    def timed(self, tokens: int, steps: int, warmup: int, budget_s: float):
        """Runs `warmup` then up to `steps` timed steps (fewer if the budget runs out); returns the
        per-step seconds of the steps timed."""
        import numpy as np
        rng = np.random.default_rng(7)
        pool = [rng.standard_normal((tokens, self.cfg.hidden)).astype(np.float32) for _ in range(REF_TOKEN_POOL)]
        for i in range(warmup):
            self.step(pool[i % REF_TOKEN_POOL])
        times = []
        t_start = time.time()
        for i in range(steps):
            s = time.perf_counter()
            self.step(pool[(warmup + i) % REF_TOKEN_POOL])
            times.append(time.perf_counter() - s)
            if time.time() - t_start > budget_s:
                break
        return times

    def close(self):
        if self.ref:
            for h in self.handles:
                self.ref.layer_destroy(h)
            self.handles = []

    def sample_text(self, tokens: int, timed: int, warmup: int):
        return (f"{tokens} token(s) per step through all {self.layers} layers of the GPT-OSS-120B-shaped stack "
                f"(RMSNorm + residual; 128 MXFP4 experts per layer, top-4), the layers rotating through "
                f"{self.n_host} distinct host layers of the seeded weights "
                f"(about 1.7 GB each) and {REF_TOKEN_POOL} seeded tokens cycling over the steps; {warmup} warm-up "
                f"and {timed} timed steps on {self.cores} host threads; no extrapolation across layers")


def cpu_baseline(a, budget_s: float) -> dict:
    """A bounded sample of the same workload on the CPU path (see ReferenceStack)."""
    T = a.tokens if a.mode == "decode" else min(a.tokens, 4)
    rs = ReferenceStack(a.layers)
    try:
        times = rs.timed(T, steps=10 ** 6, warmup=2, budget_s=budget_s)
    finally:
        rs.close()
    step_s = statistics.mean(times)
    return {"value": T / step_s, "unit": "tokens/s", "cores": rs.cores, "kind": rs.kind,
            "sample": rs.sample_text(T, len(times), 2) + (f"; prefill sampled at T={T}" if a.mode != "decode" else ""),
            "ms_per_step": step_s * 1e3, "setup_s": rs.setup_s}


# ----------------------------------------------------------------------------- GPU arm

def load_pkg():
    import __graft_entry__
    return __graft_entry__.load_package()


def algorithmic_bytes(cfg, tokens: int):
    """Per-launch algorithmic bytes of gate_up and down, averaged over layers.

    Distinct experts touched by T tokens with top-k of E: E*(1-(1-k/E)^T) (exactly k at T=1)."""
    E, k, H, I = cfg.experts, cfg.top_k, cfg.hidden, cfg.intermediate
    distinct = k if tokens == 1 else E * (1 - (1 - k / E) ** tokens)
    jobs = tokens * k
    gu = distinct * (2 * I * H // 32 * 17 + 2 * I * 2) + tokens * H * (1 + 4 / 32) + jobs * I * (1 + 4 / 32)
    dn = distinct * (H * I // 32 * 17 + H * 2) + jobs * I * (1 + 4 / 32) + jobs * H * 4
    return gu, dn, distinct


def ep_decode_arm(a):
    """N > 1 decode: the stack split over the ranks by expert (rank g holds experts [g*E/N, (g+1)*E/N) of
    every layer, 61 GB / N), one token per rank per step (global batch N), the router replicated, the
    dispatch and combine exchanged by P2P stores over NVLink inside the kernels (EpStack).  Before
    timing, every rank's token goes through a 2-layer slice and rank 0 recomputes the same tokens on one
    GPU with whole layers: the bits must agree (parity_ok); a mismatch ends the run with a non-zero
    status."""
    import datetime
    import importlib

    import numpy as np
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    pkg = load_pkg()
    ep = importlib.import_module(pkg.__name__ + ".ep")
    cfg = pkg.configs.GPT_OSS_120B
    if a.experts:
        import dataclasses
        cfg = dataclasses.replace(cfg, experts=a.experts)
    H = cfg.hidden
    layers = [pkg.MoeLayer(cfg.desc(max_tokens=world, ep_rank=rank, ep_world=world), synthetic=cfg.synthetic(layer=l),
                           device=dev.index, reserve_bytes=2 << 30) for l in range(a.layers)]
    group = ep.EpGroup(H, cfg.top_k, dev.index)
    stream = torch.cuda.current_stream(dev)

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # parity: every rank's token through the first two layers, against rank 0's one-GPU recompute of the
    # same tokens with whole layers (the one-GPU stack is bit-exact with the oracle in the GPU tests)
    xcheck = torch.from_numpy(np.random.default_rng(99).standard_normal((world, H)).astype(np.float32)).to(dev)
    slice_st = ep.EpStack(group, layers[:2])
    got = slice_st.forward(xcheck[rank:rank + 1].contiguous())
    slice_st.close()
    gathered = [torch.empty_like(got) for _ in range(world)]
    dist.all_gather(gathered, got)
    ok = torch.ones(1, dtype=torch.int32, device=dev)
    if rank == 0:
        whole = [pkg.MoeLayer(cfg.desc(max_tokens=world), synthetic=cfg.synthetic(layer=l), device=dev.index,
                              reserve_bytes=2 << 30) for l in range(2)]
        ref_st = pkg.MoeStack(whole, max_tokens=world)
        want = ref_st.forward(xcheck)
        ok[0] = int(torch.equal(torch.cat(gathered).view(torch.int32), want.view(torch.int32)))
        ref_st.close()
        for l in whole:
            l.close()
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    parity_ok = bool(ok.item())

    est = ep.EpStack(group, layers)
    pool = 16
    rng = np.random.default_rng(1000)  # the same batches on every rank: rank g takes row g
    xs = torch.from_numpy(rng.standard_normal((pool, world, H)).astype(np.float32)).to(torch.bfloat16)
    xs_dev = xs[:, rank:rank + 1].contiguous().to(dev)
    out = torch.empty((1, H), dtype=torch.float32, device=dev)
    for i in range(a.warmup):
        est.forward(xs_dev[i % pool], out)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    launches0 = pkg.kernel_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index) as clk:
        ev0.record(stream)
        for i in range(a.steps):
            est.forward(xs_dev[i % pool], out)
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = pkg.kernel_launches() - launches0
    est.status()
    dist.barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    ms_step = ms / a.steps
    # end to end: the token from pinned host memory, the result back, every step
    e2e = None
    if not a.no_e2e:
        xh = xs[:, rank:rank + 1].contiguous().pin_memory()
        oh = torch.empty((1, H), dtype=torch.float32).pin_memory()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(a.steps):
            est.forward_host(xh[i % pool], oh)
        e1.record(stream)
        torch.cuda.synchronize()
        ems = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": world * a.steps / (ems / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": int(H * 2),
               "d2h_bytes_per_step": int(H * 4), "ms_per_step": ems / a.steps,
               "api": "umsx_ep_stack_forward_host (per rank)"}
    peak, peak_kind = peaks()
    E, k = cfg.experts, cfg.top_k
    distinct = E * (1 - (1 - k / E) ** world)
    expert_b = cfg.expert_bytes()
    step_bytes = a.layers * (distinct * expert_b + world * cfg.router_bytes())  # all ranks together
    per_gpu = step_bytes / world / (ms_step / 1e3) / 1e9
    one_launch = launches == a.steps  # the one-launch expert-parallel decode kernel served every step
    if one_launch:  # token rows once per step, every job's output row to every other rank per layer
        xbytes = world * (world - 1) * H * 4 + a.layers * world * k * H * 4 * (world - 1)
        exch = ("P2P NVLink stores inside the one-launch decode kernel k_decode (CUDA IPC mappings): token rows once "
                "per step, each job's output row into every rank, a release/acquire flag exchange per layer; no "
                "collective in the data path")
        kern = ("k_decode, expert-parallel form (one launch per step per GPU: replicated router over all ranks' "
                "tokens, this rank's experts, cross-rank flag exchange per layer)")
    else:
        xbytes = a.layers * (world * (world - 1) * H * 4 + world * k * H * 4 * (world - 1) / world)
        exch = ("P2P NVLink stores inside k_ep_share / k_ep_combine (CUDA IPC mappings), release/acquire flags; "
                "no collective in the data path")
        kern = "whole decode step per GPU (per-stage exact kernels + exchange kernels)"
    res = {"metric": metric_name(a), "value": world * a.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
           "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "int8 dot (MXFP4 x Q8_0), fp32 accumulate", "data": "synthetic",
           "parity_ok": parity_ok,
           "config": {"workload": f"gpt-oss-120b-stack {a.mode}, expert parallel", "layers": a.layers,
                      "experts": cfg.experts, "experts_per_gpu": cfg.experts // world, "top_k": k, "hidden": H,
                      "ffn": cfg.intermediate, "quant": "mxfp4", "tokens_per_step_per_gpu": 1, "global_batch": world,
                      "parallelism": f"ep{world}",
                      "exchange": exch,
                      "l2": "inputs larger than L2", "expected_distinct_experts_per_layer": distinct,
                      "parity": "every rank's token through a 2-layer slice, bit-exact with one GPU running whole layers"},
           "roofline": {"kernel": kern,
                        "bound": "hbm", "achieved": per_gpu, "peak": peak, "unit": "GB/s", "frac": per_gpu / peak,
                        "peak_source": f"{peak_kind} hbm_gbs", "algorithmic_bytes_per_step_all_gpus": step_bytes,
                        "traffic": None},
           "exchange_bytes_per_step": xbytes, "gpu_launches": launches, "clocks": clk.summary(), "e2e": e2e}
    est.close()
    group.close()
    for l in layers:
        l.close()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res))
    if not parity_ok:
        raise SystemExit(3)


def gpu_arm(a):
    import numpy as np
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    if world > 1 and a.mode == "decode" and not a.replicas:
        return ep_decode_arm(a)
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    pkg = load_pkg()
    cfg = pkg.configs.GPT_OSS_120B
    if a.experts:
        import dataclasses
        cfg = dataclasses.replace(cfg, experts=a.experts)
    T = a.tokens
    layers = [pkg.MoeLayer(cfg.desc(max_tokens=1), synthetic=cfg.synthetic(layer=l), device=dev.index,
                           reserve_bytes=2 << 30) for l in range(a.layers)]
    stack = pkg.MoeStack(layers, max_tokens=T)
    pool = 16
    rng = np.random.default_rng(1000 + rank)
    xs = torch.from_numpy(rng.standard_normal((pool, T, cfg.hidden)).astype(np.float32)).to(torch.bfloat16)
    xs_dev = xs.to(dev)
    out = torch.empty((T, cfg.hidden), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # device-resident timed region (the stack replays one CUDA graph per step)
    for i in range(a.warmup):
        stack.forward(xs_dev[i % pool], out)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches0 = pkg.kernel_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index) as clk:
        ev0.record(stream)
        for i in range(a.steps):
            stack.forward(xs_dev[i % pool], out)
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = pkg.kernel_launches() - launches0
    barrier()
    torch.cuda.synchronize()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    ms_step = ms / a.steps
    per_step_launches = launches / a.steps
    persistent = per_step_launches == 1  # the whole stack ran as one persistent decode kernel per step
    stages = None
    if not persistent:
        # per-stage durations: the same steps again with CUDA events between the stages (the
        # combine then runs as a kernel of its own so that every stage has a boundary)
        stack.set_timing(True)
        for i in range(a.warmup):
            stack.forward(xs_dev[i % pool], out)
        stage_sum = dict.fromkeys(stack.STAGES, 0.0)
        for i in range(a.steps):
            stack.forward(xs_dev[i % pool], out)
            for k, v in stack.stage_times().items():
                stage_sum[k] += v
        stages = {k: v / a.steps for k, v in stage_sum.items()}
        stack.set_timing(False)
    value = world * T * a.steps / (ms / 1e3)
    clocks = clk.summary()

    # end-to-end through the C ABI with host buffers (pinned), copies inside the timed region
    e2e = None
    if not a.no_e2e:
        xh = xs.pin_memory()
        oh = torch.empty((T, cfg.hidden), dtype=torch.float32).pin_memory()
        for i in range(a.warmup):
            stack.forward_host(xh[i % pool], oh)
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(a.steps):
            stack.forward_host(xh[i % pool], oh)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ems = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": world * T * a.steps / (ems / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": int(T * cfg.hidden * 2), "d2h_bytes_per_step": int(T * cfg.hidden * 4),
               "ms_per_step": ems / a.steps, "api": "umsx_stack_forward_host"}

    peak, peak_kind = peaks()
    gu_bytes, dn_bytes, distinct = algorithmic_bytes(cfg, T)
    stack_bytes = a.layers * (gu_bytes + dn_bytes + cfg.router_bytes())
    if persistent:
        # one launch per step: its duration is the device-timed step (events on the launching stream)
        roof = {"kernel": "k_decode (persistent: RMSNorm, router, top-k, exact MXFP4 x Q8_0 gate_up + SwiGLU-OAI, "
                          "down, rank-order combine; all layers in one launch)", "bound": "hbm",
                "achieved": stack_bytes / (ms_step / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                "frac": stack_bytes / (ms_step / 1e3) / 1e9 / peak, "peak_source": f"{peak_kind} hbm_gbs",
                "algorithmic_bytes_per_launch": stack_bytes, "avg_launch_ms": ms_step,
                "traffic": traffic_for(a, "k_decode")}
    elif T >= PREFILL_MIN_TOKENS:
        # tensor-core prefill: the gate_up grouped GEMM (k_moe_gemm) dominates; useful FLOPs =
        # 2 x jobs x 2I x H per launch (the kernel issues twice that: activation hi + lo)
        gu_ms = stages["gate_up"] / a.layers
        gu_flops = 2.0 * T * cfg.top_k * 2 * cfg.intermediate * cfg.hidden
        tpeak, tkind = peaks("bf16_tflops_sustained")
        roof = {"kernel": "k_moe_gemm gate_up (tcgen05 kind::f16, exact f16 MXFP4 weights x hi+lo f16 Q8_0 "
                          "activations, fp32 TMEM accumulators, fused bias + SwiGLU-OAI + Q8_0)", "bound": "tensor",
                "achieved": gu_flops / (gu_ms / 1e3) / 1e12, "peak": tpeak, "unit": "TFLOP/s",
                "frac": gu_flops / (gu_ms / 1e3) / 1e12 / tpeak, "peak_source": f"{tkind} bf16_tflops_sustained",
                "algorithmic_flops_per_launch": gu_flops, "mma_flops_issued_per_launch": 2 * gu_flops,
                "avg_launch_ms": gu_ms, "traffic": traffic_for(a, "k_moe_gemm")}
    else:
        gu_ms = stages["gate_up"] / a.layers
        roof = {"kernel": "k_gate_up (MXFP4 x Q8_0 exact GEMV, fused SwiGLU-OAI + Q8_0)", "bound": "hbm",
                "achieved": gu_bytes / (gu_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                "frac": gu_bytes / (gu_ms / 1e3) / 1e9 / peak, "peak_source": f"{peak_kind} hbm_gbs",
                "algorithmic_bytes_per_launch": gu_bytes, "avg_launch_ms": gu_ms, "traffic": None}
    res = {"metric": metric_name(a), "value": value, "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None,
           "dtype": ("f16 tensor-core MMA (exact f16 MXFP4 weights x hi+lo f16 Q8_0 activations), fp32 accumulate"
                     if T >= PREFILL_MIN_TOKENS else "int8 dot (MXFP4 x Q8_0), fp32 accumulate"),
           "data": "synthetic",
           "config": {"workload": f"gpt-oss-120b-stack {a.mode}", "layers": a.layers, "experts": cfg.experts,
                      "top_k": cfg.top_k, "hidden": cfg.hidden, "ffn": cfg.intermediate, "quant": "mxfp4",
                      "tokens_per_step_per_gpu": T, "global_batch": T * world,
                      "parallelism": "replicas" if world > 1 else "single",
                      "l2": f"inputs larger than L2: {stack_bytes / 1e9:.2f} GB of weights read per step",
                      "expected_distinct_experts_per_layer": distinct},
           "roofline": roof,
           "stack_roofline": {"bytes_per_step": stack_bytes, "achieved_gbs": stack_bytes / (ms_step / 1e3) / 1e9,
                              "frac": stack_bytes / (ms_step / 1e3) / 1e9 / peak},
           "stages_ms_per_step": stages, "gpu_launches": launches, "clocks": clocks, "e2e": e2e}
    if world == 1 and a.mode == "decode" and not a.no_prefill:
        try:
            res["prefill"] = prefill_record(pkg, cfg, layers, dev, a)
        except Exception as exc:  # the decode line must still be printed
            res["prefill"] = {"error": str(exc)[:200]}
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        try:
            res["cpu_baseline"] = cpu_baseline(a, a.cpu_seconds)
        except Exception as exc:  # the GPU line must still be printed
            res["cpu_baseline"] = {"value": None, "error": str(exc)[:200]}
    stack.close()
    for l in layers:
        l.close()
    if world == 1 and a.mode == "decode" and not a.no_extra:
        # configs[3] (load skew, T = 4096) and the residency bank, measured in the same run
        import argparse
        torch.cuda.empty_cache()
        for name, fn, steps, warmup in (("skew", skew_arm, 20, 3), ("bank", bank_arm, 128, 64),
                                        ("configs", configs_record, 64, 8)):
            sub = argparse.Namespace(**vars(a))
            sub.steps, sub.warmup, sub.tokens, sub.experts = steps, warmup, 4096, None
            try:
                r = fn(sub, emit=False)
                res[name] = {k: r.get(k) for k in ("metric", "value", "unit", "steps", "warmup", "ms_per_step", "config")}
                res[name]["detail"] = r.get("skew") or r.get("configs") or {
                    "resident_ms_per_token": r.get("resident_ms_per_token"), "bank": r.get("bank")}
            except Exception as exc:  # the decode line must still be printed
                res[name] = {"error": str(exc)[:200]}
            torch.cuda.empty_cache()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res))


def prefill_record(pkg, cfg, layers, dev, a, tokens: int = 4096, steps: int = 5, warmup: int = 3) -> dict:
    """The metric's second regime on the same 36 layers: one step = `tokens` tokens through the stack
    (router, tcgen05 grouped GEMMs for gate_up and down, rank-order combine + residual per layer),
    inputs resident in HBM (far larger than L2), CUDA events on the launching stream."""
    import numpy as np
    import torch
    T, H = tokens, cfg.hidden
    st = pkg.MoeStack(layers, max_tokens=T)
    rng = np.random.default_rng(2000)
    xs = [torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(torch.bfloat16).to(dev)
          for _ in range(2)]
    out = torch.empty((T, H), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    for i in range(warmup):
        st.forward(xs[i % 2], out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index) as clk:
        e0.record(stream)
        for i in range(steps):
            st.forward(xs[i % 2], out)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    st.set_timing(True)
    st.forward(xs[0], out)
    stages = {k: v / a.layers for k, v in st.stage_times().items()}
    st.set_timing(False)
    st.close()
    gu_flops = 2.0 * T * cfg.top_k * 2 * cfg.intermediate * H
    dn_flops = 2.0 * T * cfg.top_k * H * cfg.intermediate
    bf16_sus, kind = peaks("bf16_tflops_sustained")
    gu_tf = gu_flops / (stages["gate_up"] / 1e3) / 1e12
    return {"tokens_per_step": T, "value": T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "warmup": warmup, "layers": a.layers,
            "stage_ms_per_layer": stages,
            "roofline": {"kernel": "k_moe_gemm gate_up (tcgen05 kind::f16, exact f16 MXFP4 weights x hi+lo f16 "
                                   "Q8_0 activations)", "bound": "tensor",
                         "achieved": gu_tf, "unit": "TFLOP/s", "useful_flops_per_launch": gu_flops,
                         "peak": bf16_sus, "frac": gu_tf / bf16_sus, "peak_source": f"{kind} bf16_tflops_sustained",
                         "frac_of_nominal_fp4_dense_9000": gu_tf / 9000.0},
            "layer_tflops_useful": (gu_flops + dn_flops) / ((stages["gate_up"] + stages["down"]) / 1e3) / 1e12,
            "clocks": clk.summary(), "l2": "inputs larger than L2 (61 GB of weights, 4096 x 2880 activations)"}


def configs_record(a, emit: bool = False) -> dict:
    """The other BASELINE configurations timed on one GPU through the public API: configs[1] (Qwen3-30B-
    A3B-shaped Q8_0 layer, T = 1 and 16; four seeded layers cycled so that consecutive calls read other
    weights) and configs[4] (the DeepSeek-V2-Lite-shaped 27-layer block: dense layer 0, 26 MoE layers
    with shared experts, T = 1).  Tokens/s, and the HBM roofline fraction of the algorithmic bytes
    (the expected distinct experts a call touches, the router, and for configs[4] the dense and shared
    FFNs) over the measured copy peak."""
    import torch
    pkg = load_pkg()
    C = pkg.configs
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    torch.manual_seed(5)
    peak, kind = peaks()
    stream = torch.cuda.current_stream(dev)
    out = {}

    def clocked(fn, steps, warmup):
        for i in range(warmup):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            fn(warmup + i)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    c1 = C.QWEN3_30B
    layers = [pkg.MoeLayer(c1.desc(16), synthetic=c1.synthetic(layer=l), device=0) for l in range(4)]
    for T in (1, 16):
        xs = [torch.randn(T, c1.hidden, device=dev).to(torch.bfloat16) for _ in range(7)]
        o = torch.empty((T, c1.hidden), dtype=torch.float32, device=dev)
        ms = clocked(lambda i: layers[i % 4].forward(xs[i % 7], o), max(a.steps, 64), 8)
        distinct = c1.experts * (1 - (1 - c1.top_k / c1.experts) ** T)
        b = distinct * c1.expert_bytes() + c1.router_bytes()
        out[f"qwen3_30b_T{T}"] = {"tokens_per_s": T / (ms / 1e3), "ms_per_layer": ms, "bytes_per_call": b,
                                 "achieved_gbs": b / (ms / 1e3) / 1e9, "frac": b / (ms / 1e3) / 1e9 / peak}
    for l in layers:
        l.close()
    torch.cuda.empty_cache()
    import importlib
    mixed = importlib.import_module(pkg.__name__ + ".mixed")
    stack, layers, shared = mixed.deepseek_v2_lite_stack(C.DEEPSEEK_V2_LITE.layers, max_tokens=1)
    xs = [torch.randn(1, C.DEEPSEEK_V2_LITE.hidden, device=dev).to(torch.bfloat16) for _ in range(16)]
    o = torch.empty((1, C.DEEPSEEK_V2_LITE.hidden), dtype=torch.float32, device=dev)
    ms = clocked(lambda i: stack.forward(xs[i % 16], o), max(a.steps // 4, 20), 3)
    r, sh, dn = C.DEEPSEEK_V2_LITE, C.DEEPSEEK_V2_LITE_SHARED, C.DEEPSEEK_V2_LITE_DENSE
    b = (dn.expert_bytes() + dn.router_bytes() +
         26 * (r.top_k * r.expert_bytes() + r.router_bytes() + sh.expert_bytes() + sh.router_bytes()))
    out["deepseek_v2_lite_27_T1"] = {"tokens_per_s": 1e3 / ms, "ms_per_token": ms, "bytes_per_token": b,
                                     "achieved_gbs": b / (ms / 1e3) / 1e9, "frac": b / (ms / 1e3) / 1e9 / peak}
    stack.close()
    for l in layers + [x for x in shared if x is not None]:
        l.close()
    torch.cuda.empty_cache()
    res = {"metric": "MoE tokens/s on the other BASELINE configurations (configs[1], configs[4])",
           "value": out["qwen3_30b_T1"]["tokens_per_s"], "unit": "tokens/s", "steps": max(a.steps, 64),
           "warmup": 8, "ms_per_step": out["qwen3_30b_T1"]["ms_per_layer"],
           "config": {"workload": "configs[1] Qwen3-30B-A3B layer (Q8_0) T=1 headline value; T=16 and "
                                  "configs[4] DeepSeek-V2-Lite 27-layer T=1 in the detail",
                      "peak_source": f"{kind} hbm_gbs"},
           "configs": out}
    if emit:
        print(json.dumps(res))
    return res


def skew_router(pkg, cfg):
    """configs[3]'s router: weights N(0, router_sigma) (seeded numpy draws) and the bias
    log(Zipf(1.2) popularity) + N(0, 0.5) over the experts (configs.zipf_router_bias)."""
    import numpy as np
    rng = np.random.default_rng(cfg.seed + 77)
    rw = (rng.standard_normal((cfg.experts, cfg.hidden)) * cfg.router_sigma).astype(np.float32)
    return rw, pkg.configs.zipf_router_bias(cfg.experts, seed=cfg.seed)


def random_host_layer(cfg, seed: int) -> dict:
    """Host weights of one MXFP4 fused layer in ggml layout, drawn with numpy: codes uniform over the
    16 e2m1 codes, block exponents 119..123 (2^-8 .. 2^-4), bf16 biases N(0, bias_sigma)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    E, H, I = cfg.experts, cfg.hidden, cfg.intermediate

    def blocks(rows, cols):
        b = rng.integers(0, 256, size=(E, rows, cols // 32, 17), dtype=np.uint8)
        b[..., 0] = rng.integers(119, 124, size=(E, rows, cols // 32), dtype=np.uint8)
        return b.reshape(E, rows, cols // 32 * 17)

    def bf16(n):
        return ((rng.standard_normal(n) * cfg.bias_sigma).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)

    return {"router_w": (rng.standard_normal((E, H)) * cfg.router_sigma).astype(np.float32),
            "router_b": (rng.standard_normal(E) * cfg.router_bias_sigma).astype(np.float32),
            "gate_up": blocks(2 * I, H), "down": blocks(H, I),
            "gate_up_bias": bf16(E * 2 * I).reshape(E, 2 * I), "down_bias": bf16(E * H).reshape(E, H)}


def bank_arm(a, emit: bool = True):
    """Expert residency (the reference's hybrid expert cache, row (f)4): a GPT-OSS-120B-shaped layer
    (128 MXFP4 experts, 1.7 GB) kept in pinned host memory, `slots` experts resident in a device bank
    admitted by the reference's LFU or LRU rule, the others uploaded for the call that needs them; one
    token per call (the reference admits on single-token dispatches), routed by configs[3]'s Zipf(1.2)
    router bias so that a bank of a quarter or half of the experts can hold the hot ones.  Per policy and
    bank size: tokens/s (CUDA events around the timed calls; every call synchronises with the host once
    for its routing), hit rate, uploads per token; the resident layer on the same weights times the same
    calls for comparison."""
    import numpy as np
    import torch
    pkg = load_pkg()
    U = pkg.umsx
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = pkg.configs.GPT_OSS_120B
    if a.experts:
        import dataclasses
        cfg = dataclasses.replace(cfg, experts=a.experts)
    w = random_host_layer(cfg, 2024)
    rw, rb = skew_router(pkg, cfg)
    w["router_w"], w["router_b"] = rw, rb
    steps, warmup = max(a.steps, 64), max(a.warmup, 32)
    rng = np.random.default_rng(5)
    pool = warmup + steps  # every call routes a token of its own
    xs = torch.from_numpy(rng.standard_normal((pool, 1, cfg.hidden)).astype(np.float32)).to(torch.bfloat16).to(dev)
    out = torch.empty((1, cfg.hidden), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def run(layer, first, n):
        for i in range(first, first + n):
            layer.forward(xs[i % pool], out)

    def timed(layer, first, steps):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run(layer, first, steps)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    resident = pkg.MoeLayer(cfg.desc(1), w, device=0)
    run(resident, 0, warmup)
    res_ms = timed(resident, warmup, steps)
    resident.close()
    per_expert = 3 * cfg.intermediate * (cfg.hidden // 32) * 17
    records = {}
    with Clocks(0) as clk:
        for policy, pname in ((U.BANK_LFU, "lfu"), (U.BANK_LRU, "lru")):
            for slots in (cfg.experts // 8, cfg.experts // 4, cfg.experts // 2):
                layer = pkg.MoeLayer(cfg.desc(1), w, bank=(slots, policy), device=0)
                run(layer, 0, warmup)  # the warm-up calls fill the bank
                before = layer.bank_stats()
                ms = timed(layer, warmup, steps)
                after = layer.bank_stats()
                d = {k: after[k] - before[k] for k in U.BANK_STAT_NAMES}
                records[f"{pname}_{slots}"] = {
                    "policy": pname, "slots": slots, "tokens_per_s": 1e3 / ms, "ms_per_token": ms,
                    "hit_rate": d["hits"] / max(1, d["demands"]), "admissions_per_token": d["admissions"] / steps,
                    "transient_uploads_per_token": d["transient"] / steps,
                    "upload_gb_per_s": d["upload_bytes"] / (ms * steps / 1e3) / 1e9,
                    "upload_bytes_per_token": d["upload_bytes"] / steps}
                layer.close()
    head = records[f"lfu_{cfg.experts // 4}"]
    res = {"metric": "banked MoE-layer tokens/s (GPT-OSS-120B-shaped layer, 128 experts in host memory, "
                     "one token per call, Zipf(1.2) routing)",
           "value": head["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "steps": steps, "warmup": warmup,
           "ms_per_step": head["ms_per_token"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "int8 dot (MXFP4 x Q8_0), fp32 accumulate", "data": "synthetic",
           "config": {"workload": "gpt-oss-120b layer, residency bank (LFU, 32 of 128 experts resident)",
                      "experts": cfg.experts, "top_k": cfg.top_k, "hidden": cfg.hidden, "ffn": cfg.intermediate,
                      "expert_bytes": per_expert, "routing": "configs[3] Zipf(1.2) router bias"},
           "resident_ms_per_token": res_ms, "bank": records, "clocks": clk.summary()}
    if emit:
        print(json.dumps(res))
    return res


def skew_arm(a, emit: bool = True):
    """Qwen3-30B-A3B layer shapes in Q8_0 and MXFP4 with the Zipf(1.2) router bias, T = 4096
    tokens per step on one GPU: tokens/s, p50 / p99 layer latency over the steps (CUDA events per step,
    inputs from a pool of 8 seeded batches), per-expert load and the per-GPU load an expert-parallel
    split over G = 2 / 4 / 8 GPUs would see (contiguous expert blocks): max / mean jobs per GPU."""
    import numpy as np
    import torch
    rank, world, local = dist_env()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pkg = load_pkg()
    T = a.tokens if a.tokens != 1 else 4096
    out_rec = {}
    for name in ("qwen3-skew-q8_0", "qwen3-skew-mxfp4"):
        cfg = pkg.configs.CONFIGS[name]
        layer = pkg.MoeLayer(cfg.desc(max_tokens=T), synthetic=cfg.synthetic(), device=0)
        layer.set_router(*skew_router(pkg, cfg))
        rng = np.random.default_rng(3000)
        xs = [torch.from_numpy(rng.standard_normal((T, cfg.hidden)).astype(np.float32)).to(torch.bfloat16).to(dev)
              for _ in range(8)]
        out = torch.empty((T, cfg.hidden), dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream(dev)
        for i in range(a.warmup):
            layer.forward(xs[i % 8], out)
        torch.cuda.synchronize()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(a.steps + 1)]
        with Clocks(0) as clk:
            evs[0].record(stream)
            for i in range(a.steps):
                layer.forward(xs[i % 8], out)
                evs[i + 1].record(stream)
            torch.cuda.synchronize()
        ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(a.steps)]
        _, _, counts = layer.route(xs[0])
        c = counts.cpu().numpy().astype(np.int64)
        per_gpu = {f"G{G}": {"jobs": c.reshape(G, -1).sum(1).tolist(),
                             "max_over_mean": float(c.reshape(G, -1).sum(1).max() / c.reshape(G, -1).sum(1).mean())}
                   for G in (2, 4, 8)}
        out_rec[name] = {"tokens_per_s": T * a.steps / (sum(ms) / 1e3), "layer_ms_p50": float(np.percentile(ms, 50)),
                         "layer_ms_p99": float(np.percentile(ms, 99)), "layer_ms_mean": float(np.mean(ms)),
                         "expert_load_max_over_mean": float(c.max() / c.mean()), "experts_unused": int((c == 0).sum()),
                         "ep_partition": per_gpu, "clocks": clk.summary()}
        layer.close()
    res = {"metric": f"MoE-layer tokens/s, configs[3] load skew (Qwen3-30B-A3B shapes, Zipf 1.2 router bias), T={T}",
           "value": out_rec["qwen3-skew-q8_0"]["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "steps": a.steps,
           "warmup": a.warmup, "higher_is_better": True, "data": "synthetic",
           "config": {"workload": "qwen3-30b-a3b skew layer (Q8_0 headline value; MXFP4 in the sub-record)",
                      "tokens": T, "experts": 128, "top_k": 8, "hidden": 2048, "ffn": 768},
           "skew": out_rec}
    if emit:
        print(json.dumps(res))
    return res


def ep_arm(a):
    """Expert-parallel prefill (--ep): every layer's experts split over the N ranks (rank g holds
    [g*E/N, (g+1)*E/N)), the step's T tokens split over the ranks (T/N each, strong scaling), the
    token rows sent to the experts' ranks and the outputs returned as P2P NVLink stores inside the
    exchange kernels (ep.EpPrefill); no collective carries layer data.  --config stack: the
    GPT-OSS-120B-shaped stack; --config skew: configs[3] (Qwen3-30B-A3B shapes with the Zipf(1.2) router
    bias, Q8_0 headline and MXFP4 sub-record), with every rank's rows and jobs per layer (the per-GPU
    load the skew produces) and p50 / p99 step latency.  Before timing, rank 0 recomputes the first
    layers on one GPU with whole layers for every rank's tokens: the bits must agree (parity_ok)."""
    import dataclasses
    import datetime
    import importlib

    import numpy as np
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    for k, v in (("MASTER_ADDR", "127.0.0.1"), ("MASTER_PORT", "29511"), ("RANK", "0"), ("WORLD_SIZE", "1")):
        os.environ.setdefault(k, v)  # a single-GPU run without torchrun
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    pkg = load_pkg()
    ep = importlib.import_module(pkg.__name__ + ".ep")
    T = a.tokens if a.tokens and a.tokens > 1 else 4096
    if T % world:
        raise SystemExit("--ep needs tokens divisible by the number of GPUs")
    Tr = T // world

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if a.config == "skew":
        names, n_layers = ["qwen3-skew-q8_0", "qwen3-skew-mxfp4"], a.layers if a.layers != 36 else 1
    else:
        names, n_layers = ["gpt-oss-120b"], a.layers
    stream = torch.cuda.current_stream(dev)
    records = {}
    parity_ok = True
    for name in names:
        cfg = pkg.configs.CONFIGS[name] if name in pkg.configs.CONFIGS else pkg.configs.GPT_OSS_120B
        if a.experts:
            cfg = dataclasses.replace(cfg, experts=a.experts)
        H, K = cfg.hidden, cfg.top_k
        router = None
        if a.config == "skew":
            router = skew_router(pkg, cfg)

        def make(l, **kw):
            m = pkg.MoeLayer(cfg.desc(max_tokens=kw.pop("max_tokens"), **kw), synthetic=cfg.synthetic(layer=l),
                             device=dev.index, reserve_bytes=2 << 30)
            if router is not None:
                m.set_router(*router)
            return m

        layers = [make(l, max_tokens=T, ep_rank=rank, ep_world=world) for l in range(n_layers)]
        group = ep.EpGroup(H, K, dev.index)
        rng = np.random.default_rng(1000)  # the same batches on every rank: rank g takes rows [g*T/N, (g+1)*T/N)
        pool = 4
        xs = torch.from_numpy(rng.standard_normal((pool, T, H)).astype(np.float32)).to(torch.bfloat16)
        # parity: the first (up to) two layers for every rank's tokens against one GPU with whole layers
        n_chk = min(2, n_layers)
        chk = ep.EpPrefill(group, layers[:n_chk], max_tokens=Tr)
        got = chk.forward(xs[0, rank * Tr:(rank + 1) * Tr].contiguous().to(dev))
        chk.close()
        gathered = [torch.empty_like(got) for _ in range(world)]
        dist.all_gather(gathered, got)
        ok = torch.ones(1, dtype=torch.int32, device=dev)
        if rank == 0:
            whole = [make(l, max_tokens=T) for l in range(n_chk)]
            ref = pkg.MoeStack(whole, max_tokens=T)
            want = ref.forward(xs[0].to(dev))
            ok[0] = int(torch.equal(torch.cat(gathered).view(torch.int32), want.view(torch.int32)))
            ref.close()
            for l in whole:
                l.close()
            torch.cuda.empty_cache()
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        parity_ok = parity_ok and bool(ok.item())

        pf = ep.EpPrefill(group, layers, max_tokens=Tr)
        xs_dev = xs[:, rank * Tr:(rank + 1) * Tr].contiguous().to(dev)
        out = torch.empty((Tr, H), dtype=torch.float32, device=dev)
        for i in range(a.warmup):
            pf.forward(xs_dev[i % pool], out)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        launches0 = pkg.kernel_launches()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(a.steps + 1)]
        with Clocks(dev.index) as clk:
            evs[0].record(stream)
            for i in range(a.steps):
                pf.forward(xs_dev[i % pool], out)
                evs[i + 1].record(stream)
            torch.cuda.synchronize()
        launches = pkg.kernel_launches() - launches0
        pf.status()
        dist.barrier()
        step_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(a.steps)]
        ms = max_over_ranks(sum(step_ms))
        p50, p99 = max_over_ranks(float(np.percentile(step_ms, 50))), max_over_ranks(float(np.percentile(step_ms, 99)))
        loads = [None] * world
        dist.all_gather_object(loads, pf.loads().tolist())
        jobs = np.array([[lj[1] for lj in r] for r in loads], dtype=np.int64)  # [rank][layer]
        rows = np.array([[lj[0] for lj in r] for r in loads], dtype=np.int64)
        e2e = None
        if not a.no_e2e:
            xh = xs[:, rank * Tr:(rank + 1) * Tr].contiguous().pin_memory()
            oh = torch.empty((Tr, H), dtype=torch.float32).pin_memory()
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(a.steps):
                pf.forward_host(xh[i % pool], oh)
            e1.record(stream)
            torch.cuda.synchronize()
            ems = max_over_ranks(e0.elapsed_time(e1))
            e2e = {"value": T * a.steps / (ems / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": int(Tr * H * 2),
                   "d2h_bytes_per_step": int(Tr * H * 4), "ms_per_step": ems / a.steps,
                   "api": "umsx_ep_prefill_forward_host (per rank)"}
        ms_step = ms / a.steps
        flops = n_layers * 2.0 * T * K * 3 * cfg.intermediate * H  # gate_up (2I x H) + down (H x I) per job
        tpeak, tkind = peaks("bf16_tflops_sustained")
        achieved = flops / world / (ms_step / 1e3) / 1e12
        records[name] = {
            "tokens_per_s": T * a.steps / (ms / 1e3), "ms_per_step": ms_step, "step_ms_p50": p50, "step_ms_p99": p99,
            "jobs_per_gpu_per_layer": jobs.tolist(), "rows_received_per_gpu_per_layer": rows.tolist(),
            "jobs_max_over_mean": float((jobs.max(0) / jobs.mean(0)).max()),
            "exchange_bytes_per_step": int(rows.sum() * (H + H // 32 * 4 + K * 4 + 8) + T * K * H * 4 * n_layers),
            "roofline": {"kernel": "whole step, expert FLOPs per GPU (useful, not the hi+lo MMAs issued)",
                         "bound": "tensor", "achieved": achieved, "peak": tpeak, "unit": "TFLOP/s",
                         "frac": achieved / tpeak, "peak_source": f"{tkind} bf16_tflops_sustained", "traffic": None},
            "gpu_launches": launches, "clocks": clk.summary(), "e2e": e2e,
            "config": {"layers": n_layers, "experts": cfg.experts, "experts_per_gpu": cfg.experts // world,
                       "top_k": K, "hidden": H, "ffn": cfg.intermediate,
                       "quant": "mxfp4" if cfg.quant == pkg.umsx.QUANT_MXFP4 else "q8_0"}}
        pf.close()
        group.close()
        for l in layers:
            l.close()
        torch.cuda.empty_cache()
    head = records[names[0]]
    workload = ("qwen3-30b-a3b skew layer (configs[3], Zipf 1.2 router bias), prefill, expert parallel"
                if a.config == "skew" else "gpt-oss-120b-stack prefill, expert parallel")
    res = {"metric": (f"MoE-layer tokens/s, configs[3] load skew, T={T}, expert parallel over {world} GPU(s)"
                      if a.config == "skew" else
                      f"MoE-layer tokens/s, GPT-OSS-120B-shaped {n_layers}-layer MXFP4 stack, prefill T={T}, "
                      f"expert parallel over {world} GPU(s)"),
           "value": head["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
           "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "f16 tensor-core MMA (exact f16 weights x hi+lo f16 Q8_0 activations), fp32 accumulate",
           "data": "synthetic", "parity_ok": parity_ok,
           "config": {"workload": workload, **head["config"], "global_batch": T, "tokens_per_gpu": Tr,
                      "parallelism": f"ep{world}",
                      "exchange": "P2P NVLink stores inside k_ep_count / k_ep_dispatch / k_ep_return (CUDA IPC "
                                  "mappings), release/acquire flags; no collective in the data path",
                      "l2": "inputs larger than L2",
                      "parity": "every rank's tokens through the first layers, bit-exact with one GPU"},
           "roofline": head["roofline"], "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
           "e2e": head["e2e"], "layers_detail": records}
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res))
    if not parity_ok:
        raise SystemExit(3)


def traffic_for(a, kernel: str):
    """Per-launch DRAM bytes of the kernel, from the committed ncu capture (profiles/traffic.json):
    bytes per layer measured on a small stack, times this run's layer count."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            t = json.load(f)[f"{a.mode}_T{a.tokens}"][kernel]
        return t["dram_bytes_per_layer"] * a.layers
    except Exception:
        return None


def reference_arm(a):
    """The reference's CPU path on this host's cores, for the GPU arm's metric and config: each
    step runs the same token count through all stack layers (ReferenceStack), --warmup steps
    untimed, then up to --steps timed steps within a budget of a few minutes (the line reports the
    count actually timed)."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    T = a.tokens if a.mode == "decode" else min(a.tokens, 4)
    rs = ReferenceStack(a.layers)
    try:
        times = rs.timed(T, steps=a.steps, warmup=a.warmup, budget_s=a.ref_seconds)
    finally:
        rs.close()
    step_s = statistics.mean(times)
    value = T / step_s
    res = {"metric": metric_name(a), "value": value, "unit": "tokens/s", "n_gpus": world, "steps": len(times),
           "steps_requested": a.steps, "warmup": a.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot (MXFP4 x Q8_0), fp32 accumulate",
           "data": "synthetic", "impl": "reference",
           "config": {"workload": f"gpt-oss-120b-stack {a.mode}", "layers": a.layers, "experts": 128, "top_k": 4,
                      "hidden": 2880, "ffn": 2880, "quant": "mxfp4", "tokens_per_step_per_gpu": T,
                      "global_batch": T, "parallelism": "single"},
           "cpu_baseline": {"kind": rs.kind, "cores": rs.cores, "value": value, "unit": "tokens/s",
                            "sample": rs.sample_text(T, len(times), a.warmup)
                            + (f"; prefill sampled at T={T}" if a.mode != "decode" else "")},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(res))


def main():
    a = parse()
    if a.ep and a.impl != "reference":
        ep_arm(a)
    elif a.config == "skew":
        skew_arm(a)
    elif a.config == "bank":
        bank_arm(a)
    elif a.config == "configs":
        configs_record(a, emit=True)
    elif a.impl == "reference":
        reference_arm(a)
    else:
        gpu_arm(a)


if __name__ == "__main__":
    main()
