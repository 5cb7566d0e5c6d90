#!/usr/bin/env python
"""bench.py -- MoE-layer tokens/s and expert-weight HBM GB/s on B200.

Workload (the north-star layer): GLM-style sigmoid
MoE, d_model 7168, 256 routed experts of d_ff 2048 in Q4_K plus one shared
expert in Q8_0, top-8 with router bias N(0,0.01), weights renormalised and
scaled by 2.5, router logits skewed by per-expert offsets N(0,1.5); weights
N(0,0.02) from a seed, activations N(0,1) then RMSNorm.  A step is one
forward of the layer over --tokens tokens per GPU (decode: 1).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T]
  python bench.py --impl reference ...   # the reference CPU algorithm on the host cores

Timing: W untimed warm-up steps, then K steps each timed with CUDA events on
the forward's stream; L2 is flushed (256 MiB write) before every step outside
the events, and each step feeds new tokens (so new experts).  Multi-GPU: one
process per GPU under torchrun; value = all ranks' tokens / max-over-ranks time.
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = dict(name="c5_glm_sigmoid_256e_top8_q4k_shared_q8_0", d_model=7168, expert_ffn=2048, n_experts=256,
                n_active=8, moe_sigmoid=1, routed_scale=2.5, n_shared=1, swiglu_limit=0.0, rms_eps=1e-5,
                fmt=(6, 6, 6), shared_fmt=(4, 4, 4), weight_sigma=0.02, router_sigma=0.02, bias_sigma=0.01,
                offset_sigma=1.5)
METRIC = "MoE-layer tokens/s + expert-weight HBM GB/s vs 8 TB/s peak, 1/2/4/8 B200"
SEED = 0x51520000 + 5 * 0x100  # config 5, layer 0
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
L2_FLUSH_BYTES = 256 << 20


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            return json.load(fh), "measured"
    except Exception:
        return {"hbm_gbs": FALLBACK_HBM_GBS}, "fallback"


# ------------------------------------------------------------------ clocks

class NvmlClockSampler:
    """SM clock and clock-event reasons read through NVML by a background
    thread every ~1 ms between start() and stop(), so that even a timed region
    of a few milliseconds holds many samples."""
    NAMES = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
             ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
             ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
             ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, uuid):
        import threading
        import pynvml as N
        self.N = N
        N.nvmlInit()
        self.h = N.nvmlDeviceGetHandleByUUID(uuid)
        self.max_mhz = float(N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM))
        self.samples = []
        self.reasons = 0
        self.stop_ev = threading.Event()
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        N = self.N
        while not self.stop_ev.is_set():
            try:
                self.samples.append(float(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM)))
                self.reasons |= int(N.nvmlDeviceGetCurrentClocksEventReasons(self.h))
            except Exception:
                pass
            time.sleep(0.001)

    def start(self):
        self.thread.start()
        t0 = time.time()
        while not self.samples and time.time() - t0 < 1.0:
            time.sleep(0.001)

    def stop(self):
        self.stop_ev.set()
        self.thread.join(timeout=5)
        N = self.N
        reasons = sorted(n for n, c in self.NAMES if self.reasons & getattr(N, c))
        try:
            N.nvmlShutdown()
        except Exception:
            pass
        if not self.samples:
            return {"error": "no NVML samples"}
        return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "source": "nvml"}


def clock_sampler(ident):
    """NVML sampler when pynvml works on this box, else nvidia-smi."""
    try:
        return NvmlClockSampler(ident)
    except Exception:
        return ClockSampler(ident)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 20 ms in the background;
    start() returns once the first sample is written (at most ~3 s), so a short
    timed region still falls inside the sampling."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, ident):
        self.ident = ident
        self.path = tempfile.mktemp(prefix="qrm_clocks_", suffix=".csv")
        self.proc = None
        self.error = None

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.errf = open(self.path + ".err", "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.ident}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=self.fh, stderr=self.errf)
            t0 = time.time()
            while time.time() - t0 < 3.0 and self.proc.poll() is None:
                if os.path.getsize(self.path) > 0:
                    break
                time.sleep(0.01)
        except Exception as ex:
            self.proc = None
            self.error = str(ex)

    def stop(self):
        if self.proc is None:
            return {"error": self.error}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        self.errf.close()
        with open(self.path + ".err") as fh:
            err = fh.read().strip()
        os.unlink(self.path + ".err")
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = max(mx, float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"error": err[-300:] or "no samples"}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU leg

def cpu_sample(steps, warmup, budget_s=None, seed=SEED):
    """Times the reference CPU algorithm (the oracle restatement of
    StreamingEngine.GlmMoeFfn, MatVecParallel over nproc-1 threads) one token
    per step on the host cores.  Expert matrices come from a pool of 8
    distinct seeded experts (expert e uses pool entry e % 8): the CPU cost does
    not depend on the values, and generating all 256 on the host would take
    minutes.  Returns (tokens/s, threads, sample description)."""
    from tests import oracle_api as O  # the oracle: CPU baseline only
    W = WORKLOAD
    d, f, E = W["d_model"], W["expert_ffn"], W["n_experts"]
    rng = np.random.default_rng(seed)
    pool = 8

    def q(fmt, rows, cols):
        return O.quantize(fmt, (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(W["weight_sigma"])))

    gates = [q(6, f, d) for _ in range(pool)]
    ups = [q(6, f, d) for _ in range(pool)]
    downs = [q(6, d, f) for _ in range(pool)]

    class Case:
        pass

    c = Case()
    c.cfg = dict(d_model=d, n_experts=E, n_active=W["n_active"], expert_ffn=f, moe_sigmoid=1,
                 routed_scale=W["routed_scale"], n_shared=1, swiglu_limit=0.0, rms_eps=W["rms_eps"])
    c.norm_w = np.ones(d, np.float32)
    c.router = (rng.standard_normal((E, d), dtype=np.float32) * np.float32(W["router_sigma"]))
    c.router_bias = (rng.standard_normal(E) * W["bias_sigma"]).astype(np.float32)
    c.logit_offset = (rng.standard_normal(E) * W["offset_sigma"]).astype(np.float32)
    c.gate = [gates[e % pool] for e in range(E)]
    c.up = [ups[e % pool] for e in range(E)]
    c.down = [downs[e % pool] for e in range(E)]
    c.fmt_gate = c.fmt_up = c.fmt_down = 6
    c.shared = (q(4, f, d), q(4, f, d), q(4, d, f))
    c.fmt_sh = (4, 4, 4)
    threads = max(1, (os.cpu_count() or 2) - 1)
    xs = rng.standard_normal((warmup + steps, 1, d), dtype=np.float32)
    for i in range(warmup):
        O.moe_forward(c, xs[i], O.APPLY_NORM, threads)
    t0 = time.perf_counter()
    done = 0
    for i in range(steps):
        O.moe_forward(c, xs[warmup + i], O.APPLY_NORM, threads)
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    desc = (f"{done} decode tokens (T=1 each) of the full-size layer through the C++ restatement of "
            f"StreamingEngine.GlmMoeFfn with MatVecParallel over {threads} threads; 8 distinct seeded experts "
            f"reused across the 256 expert slots")
    return done / dt, threads, desc


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    val, threads, desc = cpu_sample(args.steps, args.warmup)
    line = dict(metric=METRIC, value=val, unit="tokens/s", n_gpus=args.gpus, steps=args.steps, warmup=args.warmup,
                ms_per_step=1000.0 / val, higher_is_better=True, scaling="weak", vs_baseline=None, dtype="f32",
                data="synthetic", impl="reference",
                config=dict(workload=WORKLOAD["name"], tokens_per_step=1, parallelism="host threads"),
                cpu_baseline=dict(value=val, unit="tokens/s", cores=threads, kind="port", sample=desc),
                e2e=dict(value=val, unit="tokens/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU leg

def build_layer(torch, Q, dev, T, seed=SEED, rank=0, world=1, nccl_id=None):
    """The workload's layer; with world > 1 an expert-parallel layer holding
    this rank's block of routed experts (the weights are the same on every
    rank: each expert is generated from its own seed)."""
    W = WORKLOAD
    d, f, E = W["d_model"], W["expert_ffn"], W["n_experts"]
    layer = Q.MoeLayer(d, E, W["n_active"], f, moe_sigmoid=True, routed_scale=W["routed_scale"],
                       n_shared=W["n_shared"], swiglu_limit=W["swiglu_limit"], rms_eps=W["rms_eps"],
                       fmt=W["fmt"], shared_fmt=W["shared_fmt"], device=dev, max_tokens=T,
                       rank=rank, world=world, nccl_id=nccl_id)
    n = f * d
    tmp = torch.empty(n, dtype=torch.float32, device=f"cuda:{dev}")
    qbuf = torch.empty(Q.tensor_bytes(n, 4), dtype=torch.uint8, device=f"cuda:{dev}")

    def synth(expert, which, fmt, s):
        Q.synth_gaussian(tmp.data_ptr(), n, s, W["weight_sigma"])
        nb = Q.tensor_bytes(n, fmt)
        Q.synth_quantize(fmt, tmp.data_ptr(), n, qbuf.data_ptr())
        layer.upload_expert_device(expert, which, fmt, qbuf.data_ptr(), nb)

    first, count = layer.expert_range()
    for e in range(first, first + count):
        for w in range(3):
            synth(e, w, W["fmt"][w], seed * 4096 + e * 3 + w)
    for w in range(3):
        synth(Q.SHARED_EXPERT, w, W["shared_fmt"][w], seed * 4096 + E * 3 + w)
    small = torch.empty(E * d, dtype=torch.float32, device=f"cuda:{dev}")
    Q.synth_gaussian(small.data_ptr(), E * d, seed + 1, W["router_sigma"])
    router = small.cpu().numpy().reshape(E, d)
    Q.synth_gaussian(small.data_ptr(), E, seed + 2, W["bias_sigma"])
    bias = small[:E].cpu().numpy()
    Q.synth_gaussian(small.data_ptr(), E, seed + 3, W["offset_sigma"])
    offset = small[:E].cpu().numpy()
    layer.upload_router(router, bias)
    layer.upload_logit_offset(offset)
    layer.upload_norm(np.ones(d, np.float32))  # synthetic norms are ones (Program.cs:357-360)
    torch.cuda.synchronize()
    return layer


def traffic_from_profiles():
    """dram bytes per gate/up launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "expert_stream_c5_decode.md")
    try:
        with open(p) as fh:
            for line in fh:
                if line.startswith("dram_bytes_per_launch:"):
                    return float(line.split(":")[1])
    except Exception:
        pass
    return None


def run_ours(args, rank, world, dist):
    import torch
    import qauntrunner_b200 as Q
    dev = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(dev)
    T = args.tokens
    W = WORKLOAD
    d = W["d_model"]
    t_build = time.perf_counter()
    nccl_id = None
    if world > 1:
        # expert parallelism: one NCCL id, made on rank 0, for the library's communicator
        idt = torch.zeros(Q.NCCL_ID_BYTES, dtype=torch.uint8, device=f"cuda:{dev}")
        if rank == 0:
            idt.copy_(torch.frombuffer(bytearray(Q.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(idt, 0)
        nccl_id = bytes(idt.cpu().numpy().tobytes())
    layer = build_layer(torch, Q, dev, T, seed=SEED, rank=rank, world=world, nccl_id=nccl_id)
    log(f"[rank {rank}] layer built in {time.perf_counter() - t_build:.1f}s")
    nsteps = args.warmup + args.steps
    g = torch.Generator(device=f"cuda:{dev}")
    g.manual_seed(SEED + 17 + rank)
    xs = torch.randn((nsteps, T, d), generator=g, device=f"cuda:{dev}", dtype=torch.float32)
    out = torch.empty((T, d), dtype=torch.float32, device=f"cuda:{dev}")
    idx = torch.empty((T, layer.k), dtype=torch.int32, device=f"cuda:{dev}")
    wts = torch.empty((T, layer.k), dtype=torch.float32, device=f"cuda:{dev}")
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{dev}")
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    flags = Q.APPLY_NORM

    def step(i):
        layer.forward_device(xs[i].data_ptr(), T, out.data_ptr(), flags, idx.data_ptr(), wts.data_ptr(), sp)

    # expert parallel: the ranks' forwards wait for one another, so every rank
    # leaves the L2 flush together (a one-element all-reduce on the stream,
    # outside the timed events) and no rank's step absorbs another's flush
    sync_buf = torch.zeros(1, device=f"cuda:{dev}") if world > 1 else None

    def flush_l2(i):
        flush.fill_(float(i))
        if sync_buf is not None:
            dist.all_reduce(sync_buf)

    with torch.cuda.stream(stream):
        for prof in ((False, True) if world == 1 else (False,)):   # capture the forward graphs before timing
            layer.set_profiling(prof)
            for i in range(args.warmup):
                flush_l2(i)
                step(i)
    torch.cuda.synchronize()
    layer.sync()

    # ---- timed region: device-resident inputs, K back-to-back steps
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    try:
        ident = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        ident = str(dev)
    clocks = clock_sampler(ident)
    layer.set_profiling(False)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            flush_l2(i)
            ev0[i].record(stream)
            step(args.warmup + i)
            ev1[i].record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clock_info = clocks.stop()
    layer.sync()
    step_ms = [ev0[i].elapsed_time(ev1[i]) for i in range(args.steps)]
    total_ms = float(sum(step_ms))

    # ---- per-stage breakdown (library events inside the forward graph), same inputs
    stage_ms = np.zeros(Q.STAGE_COUNT)
    stage_bytes = np.zeros(Q.STAGE_COUNT)
    nprof = min(args.steps, 64)
    if world == 1:
        layer.set_profiling(True)
        with torch.cuda.stream(stream):
            for i in range(nprof):
                flush.fill_(float(i))
                step(args.warmup + i)
                ms, by = layer.last_profile()
                stage_ms += ms
                stage_bytes += by
        layer.set_profiling(False)
        torch.cuda.synchronize()
        layer.sync()

    # ---- e2e: host (pinned) buffers through the C ABI, copies inside the timed region
    xh = xs.cpu().pin_memory()
    oh = torch.empty((T, d), dtype=torch.float32).pin_memory()
    xd = torch.empty((T, d), dtype=torch.float32, device=f"cuda:{dev}")
    e0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            xd.copy_(xh[i], non_blocking=True)
            layer.forward_device(xd.data_ptr(), T, out.data_ptr(), flags, None, None, sp)
            oh.copy_(out, non_blocking=True)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        for i in range(args.steps):
            flush_l2(i)
            e0[i].record(stream)
            xd.copy_(xh[args.warmup + i], non_blocking=True)
            layer.forward_device(xd.data_ptr(), T, out.data_ptr(), flags, None, None, sp)
            oh.copy_(out, non_blocking=True)
            e1[i].record(stream)
    torch.cuda.synchronize()
    layer.sync()
    if dist:
        dist.barrier()
    e2e_ms = float(sum(e0[i].elapsed_time(e1[i]) for i in range(args.steps)))

    # ---- max over ranks
    vals = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=f"cuda:{dev}")
    if dist:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms = float(vals[0]), float(vals[1])
    tokens = args.steps * T * world
    value = tokens / (total_ms / 1000.0)
    e2e_value = tokens / (e2e_ms / 1000.0)

    peaks, peak_kind = measured_peaks()
    peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    gu_ms, gu_bytes = stage_ms[3], stage_bytes[3]   # over the nprof breakdown steps
    achieved = gu_bytes / (gu_ms / 1000.0) / 1e9 if gu_ms > 0 else 0.0
    traffic = traffic_from_profiles()
    if world == 1:
        layer_bytes = (stage_bytes[3] + stage_bytes[4]) / nprof + (W["n_experts"] * d * 4 + T * d * 4 * 2)
        roof_kernel = "expert gate/up fused dequant GEMV + SwiGLU"
    else:
        # expert parallelism (no per-stage events): compressed bytes this rank streamed in
        # the last step (its experts that the gathered batch selected + shared expert +
        # router) over the step time of the timed region
        _, off = layer.last_dispatch(T)
        first, count = layer.expert_range()
        used = int(np.count_nonzero(np.diff(off)[first:first + count]))
        f = W["expert_ffn"]
        ebytes = 3 * Q.tensor_bytes(d * f, W["fmt"][0])
        sbytes = 3 * Q.tensor_bytes(d * f, W["shared_fmt"][0])
        layer_bytes = used * ebytes + sbytes + W["n_experts"] * d * 4
        achieved = layer_bytes / (total_ms / args.steps / 1000.0) / 1e9
        traffic = None
        roof_kernel = "whole layer step per rank (expert parallel: no per-stage events)"
    layer_gbs = layer_bytes / (total_ms / args.steps / 1000.0) / 1e9

    # the library counts the kernel launches of its forward (one graph replay)
    launches_per_step = layer.last_launch_count()
    transport = layer.ep_transport()
    # an expert-parallel layer's close is collective: every rank closes here
    layer.close()
    if rank != 0:
        return 0
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        try:
            v, cores, desc = cpu_sample(steps=64, warmup=1, budget_s=15.0)
            cpu = dict(value=v, unit="tokens/s", cores=cores, kind="port", sample=desc)
        except Exception as ex:  # the baseline must never block the GPU number
            cpu = dict(value=None, unit="tokens/s", cores=None, kind="port", sample=f"failed: {ex}")
    line = dict(
        metric=METRIC, value=value, unit="tokens/s", n_gpus=world, steps=args.steps, warmup=args.warmup,
        ms_per_step=total_ms / args.steps, higher_is_better=True, scaling="weak", vs_baseline=None,
        dtype="f32", data="synthetic",
        config=dict(workload=WORKLOAD["name"], tokens_per_rank=T, d_model=d, n_experts=W["n_experts"],
                    top_k=W["n_active"], expert_ffn=W["expert_ffn"], formats="routed Q4_K, shared Q8_0",
                    l2="flushed before every step (256 MiB write, outside the timed events)",
                    parallelism="single GPU" if world == 1 else f"ep{world} (expert parallel, {transport} exchanges)"),
        roofline=dict(bound="hbm", kernel=roof_kernel, achieved=achieved,
                      peak=peak, unit="GB/s", frac=achieved / peak if peak else None, peak_kind=peak_kind,
                      traffic=traffic),
        layer_hbm=dict(achieved_gbs=layer_gbs, frac_of_8tbs=layer_gbs / NOMINAL_HBM_GBS,
                       frac_of_measured=layer_gbs / peak, bytes_per_step=layer_bytes),
        stage_ms_per_step={n: float(stage_ms[i] / nprof) for i, n in enumerate(Q.STAGES)},
        cpu_baseline=cpu,
        e2e=dict(value=e2e_value, unit="tokens/s", h2d_bytes_per_step=T * d * 4, d2h_bytes_per_step=T * d * 4),
        gpu_launches=launches_per_step * args.steps,
        clocks=clock_info,
    )
    print(json.dumps(line), flush=True)
    layer.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--experts", type=int, default=None, help="profiling runs only: fewer experts")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.experts:
        WORKLOAD["n_experts"] = args.experts
        WORKLOAD["name"] += f"_e{args.experts}"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist = None
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1:
        import datetime
        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        dist = tdist
    try:
        return run_ours(args, rank, world, dist)
    finally:
        if dist:
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
