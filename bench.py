#!/usr/bin/env python
"""bench.py -- MoE-layer tokens/s and expert-weight HBM GB/s on B200.

Default workload (the north-star layer): GLM-style
sigmoid MoE, d_model 7168, 256 routed experts of d_ff 2048 in Q4_K plus one
shared expert in Q8_0, top-8 with router bias N(0,0.01), weights
renormalised and scaled by 2.5, router logits skewed by per-expert offsets
N(0,1.5); weights N(0,0.02) from seeds, activations N(0,1) then RMSNorm.  A
step is one forward of the layer over --tokens tokens per GPU (decode: 1).
--config c1..c5 selects another BASELINE config (one layer of it), --sweep
prints one line per (config, T) of the measurement plan.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--config c5]
  python bench.py --sweep [--steps K]
  python bench.py --impl reference ...   # the reference CPU algorithm on the host cores

Timing: W untimed warm-up steps, then K steps each timed with CUDA events on
the forward's stream; L2 is flushed (256 MiB written, then another 256 MiB read,
so no dirty lines are left to write back) before every step outside
the events, and each step feeds new tokens (so new experts).  Multi-GPU: one
process per GPU under torchrun; value = all ranks' tokens / max-over-ranks
time.  e2e = the drop-in call (qrm_forward: pageable host arrays in and out,
synchronous) timed by wall clock; e2e_pinned = the same forward with pinned
host buffers, the copies inside CUDA events.  The first timed step's tokens
are checked against the CPU oracle after the timed region (routing bit for
bit, outputs as max relative error).
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

from tests.moe_case import CONFIGS  # noqa: E402  (shapes only)

METRIC = "MoE-layer tokens/s + expert-weight HBM GB/s vs 8 TB/s peak, 1/2/4/8 B200"
NAMES = {
    "c1": "c1_mixtral_small_8e_top2_q4_0",
    "c2": "c2_mixtral_8x7b_layer_8e_top2_q4k",
    "c3": "c3_glm_sigmoid_160e_top8_q4k_q6k_shared",
    "c4": "c4_ternary_prefill_64e_top6_tri",
    "c5": "c5_glm_sigmoid_256e_top8_q4k_shared_q8_0",
}
FORMATS = {"c1": "Q4_0", "c2": "Q4_K", "c3": "gate/up Q4_K, down Q6_K, shared same",
           "c4": "TRI (QuantizeTriLegacy)", "c5": "routed Q4_K, shared Q8_0"}
SWEEP = [("c5", 1), ("c5", 4), ("c5", 16), ("c5", 64), ("c5", 256), ("c5", 1024), ("c5", 4096),
         ("c1", 1), ("c1", 32), ("c2", 1), ("c2", 8), ("c2", 64), ("c3", 1), ("c3", 16), ("c3", 256),
         ("c4", 2048)]
NOMINAL_HBM_GBS = 8000.0
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            return json.load(fh), "measured"
    except Exception:
        return dict(FALLBACK), "fallback"


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


class SmiClockSampler:
    """nvidia-smi clocks / throttle reasons every 20 ms (used when NVML is not
    reachable from Python)."""
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
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.ident}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
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
            return {"error": "no samples"}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvidia-smi"}


def clock_sampler(ident):
    try:
        return NvmlClockSampler(ident)
    except Exception:
        return SmiClockSampler(ident)


# ------------------------------------------------------------------ CPU leg

def cpu_case(cfg_name, seed=1):
    """The config's full-size layer for the CPU restatement, on the host.
    Expert matrices come from a pool of at most 8 distinct seeded experts
    (expert e uses pool entry e % 8): the CPU cost does not depend on the
    values, and generating every expert on the host would take minutes."""
    from tests import oracle_api as O  # the oracle: CPU baseline only
    from tests.moe_case import MoeCase, storage_fmt
    c = CONFIGS[cfg_name]
    d, f, E = c["d_model"], c["expert_ffn"], c["n_experts"]
    rng = np.random.default_rng(seed)
    pool = min(8, E)

    def q(fmt, rows, cols):
        return O.quantize(fmt, rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))

    fq = c["fmt"]
    mats = [[q(fq[w], *((d, f) if w == 2 else (f, d))) for _ in range(pool)] for w in range(3)]
    shared, fmt_sh = None, (0, 0, 0)
    if c["n_shared"] and c["moe_sigmoid"]:
        sf = c.get("shared_fmt", fq)
        shared = tuple(q(sf[w], *((d, f) if w == 2 else (f, d))) for w in range(3))
        fmt_sh = tuple(storage_fmt(x) for x in sf)
    case = MoeCase(cfg=c, norm_w=np.ones(d, np.float32),
                   router=rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.02),
                   router_bias=(rng.standard_normal(E) * c["bias_sigma"]).astype(np.float32)
                   if c.get("bias_sigma") else None,
                   logit_offset=(rng.standard_normal(E) * c["offset_sigma"]).astype(np.float32)
                   if c.get("offset_sigma") else None,
                   gate=[mats[0][e % pool] for e in range(E)], up=[mats[1][e % pool] for e in range(E)],
                   down=[mats[2][e % pool] for e in range(E)], fmt_gate=storage_fmt(fq[0]),
                   fmt_up=storage_fmt(fq[1]), fmt_down=storage_fmt(fq[2]), shared=shared, fmt_sh=fmt_sh)
    case.pool = pool
    return case


def cpu_time(case, cfg_name, T, budget_s, seed=2):
    """Times the reference CPU algorithm (the oracle restatement of
    StreamingEngine.MoeFfn / GlmMoeFfn with MatVecParallel over nproc-1
    threads, one Forward call per token as the engine runs) on host tokens
    until budget_s has passed (at most the T tokens of one step).  Returns
    (tokens/s, threads, sample description)."""
    from tests import oracle_api as O  # the oracle: CPU baseline only
    c = CONFIGS[cfg_name]
    d = c["d_model"]
    rng = np.random.default_rng(seed)
    threads = max(1, (os.cpu_count() or 2) - 1)
    flags = O.APPLY_NORM | (0 if c["moe_sigmoid"] else O.ADD_RESIDUAL)
    O.moe_forward(case, rng.standard_normal((1, d), dtype=np.float32), flags, threads)   # warm-up
    t0 = time.perf_counter()
    done = 0
    while done < T:
        O.moe_forward(case, rng.standard_normal((1, d), dtype=np.float32), flags, threads)
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    desc = (f"{done} of the {T} tokens of a step of the full-size {cfg_name} layer, one Forward call each, through "
            f"the C++ restatement of StreamingEngine.{'GlmMoeFfn' if c['moe_sigmoid'] else 'MoeFfn'} with "
            f"MatVecParallel over {threads} threads; {case.pool} distinct seeded experts reused across the "
            f"{c['n_experts']} slots")
    return done / dt, threads, desc


def cpu_sample(cfg_name, T, budget_s):
    return cpu_time(cpu_case(cfg_name), cfg_name, T, budget_s)


def run_reference(args, rank, world, out):
    if rank != 0:
        return 0
    cfg_name, T = args.config, args.tokens
    # each step a bounded sample of that step's tokens, the whole run within a few minutes
    per_step = max(0.5, min(10.0, 120.0 / (args.steps + args.warmup)))
    vals = []
    case = cpu_case(cfg_name)
    for i in range(args.warmup + args.steps):
        v, threads, desc = cpu_time(case, cfg_name, T, per_step, seed=2 + i)
        if i >= args.warmup:
            vals.append(v)
    val = float(np.mean(vals))
    line = dict(metric=METRIC, value=val, unit="tokens/s", n_gpus=args.gpus, steps=args.steps, warmup=args.warmup,
                ms_per_step=1000.0 * T / val, higher_is_better=True, scaling="weak", vs_baseline=None, dtype="f32",
                data="synthetic", impl="reference",
                config=dict(workload=NAMES[cfg_name], tokens_per_rank=T, parallelism="host threads"),
                cpu_baseline=dict(value=val, unit="tokens/s", cores=threads, kind="port", sample=desc),
                e2e=dict(value=val, unit="tokens/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), file=out, flush=True)
    return 0


# ------------------------------------------------------------------ GPU leg

def profile_traffic(cfg_name, T, gateup):
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summary of this workload (profiles/), with the capture it comes from; None
    when no capture covers the workload."""
    if cfg_name != "c5" or T != 1 or not gateup:
        return None
    path = os.path.join(ROOT, "profiles", "expert_stream_c5_decode.md")
    try:
        with open(path) as fh:
            for line in fh:
                if line.startswith("dram_bytes_per_launch:"):
                    return (float(line.split(":")[1]),
                            "ncu dram__bytes_read.sum + dram__bytes_write.sum of the gate/up launch, "
                            "profiles/expert_stream_c5_decode.md (32-expert capture of the same shapes and "
                            "routing width; per-launch bytes do not depend on the expert count)")
    except OSError:
        pass
    return None


def expert_flops(cfg, counts, T, shared):
    """2 * MACs of the expert products of one forward: per routed assignment
    and shared token 3 d*f (gate, up, down)."""
    d, f = cfg["d_model"], cfg["expert_ffn"]
    rows = int(counts.sum()) + (T if shared else 0)
    return 2.0 * rows * 3 * d * f, 2.0 * rows * 2 * d * f, 2.0 * rows * d * f


def run_one(args, cfg_name, T, rank, world, dist, torch, Q):
    from tests.synth_layer import SynthLayer
    dev = int(os.environ.get("LOCAL_RANK", 0))
    cfg = CONFIGS[cfg_name]
    d, E = cfg["d_model"], cfg["n_experts"]
    spec = SynthLayer(cfg_name, **({"n_experts": args.experts} if args.experts else {}))
    t_build = time.perf_counter()
    nccl_id = None
    if world > 1:
        # expert parallelism: one NCCL id, made on rank 0, for the library's communicator
        idt = torch.zeros(Q.NCCL_ID_BYTES, dtype=torch.uint8, device=f"cuda:{dev}")
        if rank == 0:
            idt.copy_(torch.frombuffer(bytearray(Q.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(idt, 0)
        nccl_id = bytes(idt.cpu().numpy().tobytes())
    layer = spec.build(torch, Q, dev, T, rank=rank, world=world, nccl_id=nccl_id)
    log(f"[rank {rank}] {cfg_name} layer built in {time.perf_counter() - t_build:.1f}s")
    flags = Q.APPLY_NORM | (0 if cfg["moe_sigmoid"] else Q.ADD_RESIDUAL)
    nsteps = args.warmup + args.steps
    nx = min(nsteps, max(2, (1 << 30) // max(1, T * d * 4)))     # distinct input batches (<= 1 GiB)
    g = torch.Generator(device=f"cuda:{dev}")
    g.manual_seed(spec.seed + 17 + rank)
    xs = torch.randn((nx, T, d), generator=g, device=f"cuda:{dev}", dtype=torch.float32)
    out = torch.empty((T, d), dtype=torch.float32, device=f"cuda:{dev}")
    idx = torch.empty((T, layer.k), dtype=torch.int32, device=f"cuda:{dev}")
    wts = torch.empty((T, layer.k), dtype=torch.float32, device=f"cuda:{dev}")
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{dev}")
    # write-read: a second buffer larger than L2 is read after the write, so
    # the written lines are cleaned out of L2 before the step instead of being
    # written back to HBM inside it (L2 holds no layer data either way)
    flush_rd = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{dev}") \
        if args.flush == "write-read" else None
    flush_out = torch.empty(1, dtype=torch.float32, device=f"cuda:{dev}")

    def flush_cache(i):
        flush.fill_(float(i))
        if flush_rd is not None:
            torch.sum(flush_rd, dim=0, keepdim=True, out=flush_out)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream

    def step(i):
        layer.forward_device(xs[i % nx].data_ptr(), T, out.data_ptr(), flags, idx.data_ptr(), wts.data_ptr(), sp)

    # expert parallel: the ranks' forwards wait for one another, so every rank
    # leaves the L2 flush together (a one-element all-reduce on the stream,
    # outside the timed events) and no rank's step absorbs another's flush
    sync_buf = torch.zeros(1, device=f"cuda:{dev}") if world > 1 else None

    def flush_l2(i):
        flush_cache(i)
        if sync_buf is not None:
            dist.all_reduce(sync_buf)

    with torch.cuda.stream(stream):
        for prof in (False, True):   # capture the forward graphs before timing
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
    launches_per_step = layer.last_launch_count()

    # ---- per-stage breakdown (library events inside the forward graph), same inputs
    stage_ms = np.zeros(Q.STAGE_COUNT)
    stage_bytes = np.zeros(Q.STAGE_COUNT)
    stage_flops = np.zeros(3)
    nprof = min(args.steps, 64)
    if world == 1:
        layer.set_profiling(True)
        with torch.cuda.stream(stream):
            for i in range(nprof):
                flush_cache(i)
                step(args.warmup + i)
                ms, by = layer.last_profile()
                stage_ms += ms
                stage_bytes += by
                _, off = layer.last_dispatch(T)
                stage_flops += np.array(expert_flops(cfg, np.diff(off), T, spec.shared))
        layer.set_profiling(False)
        torch.cuda.synchronize()
        layer.sync()
    ep_stage = None
    if world > 1:
        # expert parallel: every rank runs the same profiled forwards
        ep_ms = np.zeros(len(Q.EP_STAGES))
        layer.set_profiling(True)
        with torch.cuda.stream(stream):
            for i in range(nprof):
                flush_l2(i)
                step(args.warmup + i)
                ep_ms += layer.last_profile_ep()
        layer.set_profiling(False)
        torch.cuda.synchronize()
        layer.sync()
        mx = torch.tensor(ep_ms / nprof, dtype=torch.float64, device=f"cuda:{dev}")
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        ep_stage = dict(rank0={n: float(v) for n, v in zip(Q.EP_STAGES, ep_ms / nprof)},
                        max_over_ranks={n: float(v) for n, v in zip(Q.EP_STAGES, mx.cpu().numpy())})

    # ---- e2e (pinned): host buffers, copies inside the events
    nh = min(nx, args.steps + args.warmup)
    xh = xs[:nh].cpu().pin_memory()
    oh = torch.empty((T, d), dtype=torch.float32).pin_memory()
    xd = torch.empty((T, d), dtype=torch.float32, device=f"cuda:{dev}")
    e0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            xd.copy_(xh[i % nh], non_blocking=True)
            layer.forward_device(xd.data_ptr(), T, out.data_ptr(), flags, None, None, sp)
            oh.copy_(out, non_blocking=True)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        for i in range(args.steps):
            flush_l2(i)
            e0[i].record(stream)
            xd.copy_(xh[(args.warmup + i) % nh], non_blocking=True)
            layer.forward_device(xd.data_ptr(), T, out.data_ptr(), flags, None, None, sp)
            oh.copy_(out, non_blocking=True)
            e1[i].record(stream)
    torch.cuda.synchronize()
    layer.sync()
    if dist:
        dist.barrier()
    e2e_pinned_ms = float(sum(e0[i].elapsed_time(e1[i]) for i in range(args.steps)))

    # ---- e2e (drop-in call): qrm_forward on ordinary (pageable) numpy arrays, wall clock
    xp = [np.ascontiguousarray(xh[i].numpy()) for i in range(nh)]
    outp = np.empty((T, d), np.float32)
    idxp = np.empty((T, layer.k), np.int32)
    wp = np.empty((T, layer.k), np.float32)
    for i in range(args.warmup):
        layer.forward_into(xp[i % nh], flags, outp, idxp, wp)
    if dist:
        dist.barrier()
    e2e_ms = 0.0
    for i in range(args.steps):
        flush_cache(i)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        layer.forward_into(xp[(args.warmup + i) % nh], flags, outp, idxp, wp)
        e2e_ms += (time.perf_counter() - t0) * 1000.0

    # ---- parity of the first timed step's tokens against the oracle (after timing)
    parity = None
    if not args.no_parity:
        from tests.gpu_helpers import check_synth_batch
        r = check_synth_batch(spec, layer, xh[args.warmup % nh].numpy(), flags, full_limit=8,
                              check_dispatch=world == 1)
        parity = dict(routing_bit_exact=r["routing_bit_exact"], max_rel_err=r["err"],
                      tokens_checked=r["tokens_checked"], tolerance=1e-3)

    # ---- max over ranks
    vals = torch.tensor([total_ms, e2e_ms, e2e_pinned_ms, parity["max_rel_err"] if parity else 0.0],
                        dtype=torch.float64, device=f"cuda:{dev}")
    if dist:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms, e2e_pinned_ms = float(vals[0]), float(vals[1]), float(vals[2])
    if parity:
        parity["max_rel_err"] = float(vals[3])
    tokens = args.steps * T * world
    value = tokens / (total_ms / 1000.0)

    peaks, peak_kind = measured_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK["hbm_gbs"]))
    tensor = float(peaks.get("bf16_tflops_sustained", FALLBACK["bf16_tflops_sustained"]))
    roofline, layer_hbm = None, None
    if world == 1:
        gu_ms, dn_ms = stage_ms[3] / nprof, stage_ms[4] / nprof
        gu_bytes, dn_bytes = stage_bytes[3] / nprof, stage_bytes[4] / nprof
        _, gu_flops, dn_flops = stage_flops / nprof
        # the dominant expert stage, bounded by HBM or by the tensor pipe
        # (whichever its arithmetic intensity says: machine balance = tensor / hbm)
        if dn_ms > gu_ms:
            kern, ms_k, by_k, fl_k = "expert down (fused dequant product)", dn_ms, dn_bytes, dn_flops
        else:
            kern, ms_k, by_k, fl_k = "expert gate/up (fused dequant product + SwiGLU)", gu_ms, gu_bytes, gu_flops
        tensor_bound = fl_k / max(by_k, 1.0) > tensor * 1e12 / (hbm * 1e9)
        if tensor_bound:
            ach = fl_k / (ms_k / 1000.0) / 1e12 if ms_k > 0 else 0.0
            roofline = dict(bound="tensor", kernel=kern, achieved=ach, peak=tensor, unit="TFLOP/s",
                            frac=ach / tensor, peak_kind=f"{peak_kind} bf16_tflops_sustained",
                            flops_per_launch=fl_k, traffic=None)
        else:
            ach = by_k / (ms_k / 1000.0) / 1e9 if ms_k > 0 else 0.0
            roofline = dict(bound="hbm", kernel=kern, achieved=ach, peak=hbm, unit="GB/s", frac=ach / hbm,
                            peak_kind=f"{peak_kind} hbm_gbs", bytes_per_launch=by_k, traffic=None)
        layer_bytes = gu_bytes + dn_bytes + E * d * 4 + T * d * 4 * 2
    else:
        # expert parallelism (no per-stage events): compressed bytes this rank streamed in
        # the last step (its experts that the gathered batch selected + shared expert +
        # router) over the step time of the timed region
        _, off = layer.last_dispatch(T)
        first, count = layer.expert_range()
        used = int(np.count_nonzero(np.diff(off)[first:first + count]))
        f = cfg["expert_ffn"]
        ebytes = sum(Q.tensor_bytes(d * f, x) for x in spec.fmt)
        sbytes = sum(Q.tensor_bytes(d * f, x) for x in spec.fmt_sh) if spec.shared else 0
        layer_bytes = used * ebytes + sbytes + E * d * 4
        ach = layer_bytes / (total_ms / args.steps / 1000.0) / 1e9
        roofline = dict(bound="hbm", kernel="whole layer step per rank (expert parallel: no per-stage events)",
                        achieved=ach, peak=hbm, unit="GB/s", frac=ach / hbm, peak_kind=f"{peak_kind} hbm_gbs",
                        traffic=None)
    if world == 1 and roofline and roofline.get("bound") == "hbm":
        tr = profile_traffic(cfg_name, T, "gate/up" in roofline["kernel"])
        if tr:
            roofline["traffic"], roofline["traffic_source"] = tr
    layer_gbs = layer_bytes / (total_ms / args.steps / 1000.0) / 1e9
    layer_hbm = dict(achieved_gbs=layer_gbs, frac_of_8tbs=layer_gbs / NOMINAL_HBM_GBS, frac_of_measured=layer_gbs / hbm,
                     bytes_per_step=layer_bytes)
    transport = layer.ep_transport()
    # an expert-parallel layer's close is collective: every rank closes here
    layer.close()
    if rank != 0:
        return None
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        try:
            v, cores, desc = cpu_sample(cfg_name, T, budget_s=12.0)
            cpu = dict(value=v, unit="tokens/s", cores=cores, kind="port", sample=desc)
        except Exception as ex:  # the baseline must never block the GPU number
            cpu = dict(value=None, unit="tokens/s", cores=None, kind="port", sample=f"failed: {ex}")
    line = dict(
        metric=METRIC, value=value, unit="tokens/s", n_gpus=world, steps=args.steps, warmup=args.warmup,
        ms_per_step=total_ms / args.steps, higher_is_better=True, scaling="weak", vs_baseline=None,
        dtype="expert products: weight codes x 16-bit fixed-point activations (integer MMA, exact int32 sums, "
              "f32 scales) or dequantised f16 x f16 (tensor MMA, f32 accumulate); routing and combine f32",
        data="synthetic",
        config=dict(workload=NAMES[cfg_name], tokens_per_rank=T, d_model=d, n_experts=E, top_k=cfg["n_active"],
                    expert_ffn=cfg["expert_ffn"], formats=FORMATS[cfg_name],
                    l2=("flushed before every step outside the timed events: 256 MiB written" +
                        (", then another 256 MiB buffer read (no dirty lines left to write back)"
                         if args.flush == "write-read" else "")),
                    parallelism="single GPU" if world == 1 else f"ep{world} (expert parallel, {transport} exchanges)"),
        roofline=roofline,
        layer_hbm=layer_hbm,
        stage_ms_per_step={n: float(stage_ms[i] / nprof) for i, n in enumerate(Q.STAGES)} if world == 1 else ep_stage,
        cpu_baseline=cpu,
        e2e=dict(value=tokens / (e2e_ms / 1000.0), unit="tokens/s", h2d_bytes_per_step=T * d * 4,
                 d2h_bytes_per_step=T * d * 4 + T * layer.k * 8,
                 call="qrm_forward, pageable host arrays, wall clock per synchronous call"),
        e2e_pinned=dict(value=tokens / (e2e_pinned_ms / 1000.0), unit="tokens/s", h2d_bytes_per_step=T * d * 4,
                        d2h_bytes_per_step=T * d * 4),
        parity=parity,
        gpu_launches=launches_per_step * args.steps,
        clocks=clock_info,
    )
    return line


def run_stack(args, cfg_name, T, torch, Q):
    """One step = T tokens through args.layers MoE layers of the config on a
    device-resident residual stream (qrm_stack): BASELINE config 2 is a
    32-layer Mixtral-8x7B-shaped stack.  --hbm-budget-gb below the stack's
    expert bytes keeps only the first layers resident and streams the others
    from pinned host memory."""
    from tests.synth_layer import SEED_BASE, SynthLayer
    dev = 0
    cfg = CONFIGS[cfg_name]
    d, E, f = cfg["d_model"], cfg["n_experts"], cfg["expert_ffn"]
    nL = args.layers
    specs = [SynthLayer(cfg_name, seed=SEED_BASE + int(cfg_name[1:]) * 0x100 + 0x10000 * l) for l in range(nL)]
    sp0 = specs[0]
    t0 = time.perf_counter()
    budget = int(args.hbm_budget_gb * (1 << 30))
    S = Q.MoeStack(nL, d, E, cfg["n_active"], f, hbm_budget=budget, moe_sigmoid=bool(cfg["moe_sigmoid"]),
                   routed_scale=cfg["routed_scale"], n_shared=cfg["n_shared"], swiglu_limit=cfg["swiglu_limit"],
                   rms_eps=cfg["rms_eps"], fmt=sp0.fmt, shared_fmt=sp0.fmt_sh if sp0.shared else sp0.fmt,
                   device=dev, max_tokens=T)
    for sp, L in zip(specs, S.layers):
        sp.upload_into(torch, Q, dev, L)
    n_res, lbytes = S.info()
    log(f"[rank 0] {cfg_name} stack of {nL} layers built in {time.perf_counter() - t0:.1f}s "
        f"({n_res} resident, {nL - n_res} streamed, {lbytes / 1e9:.2f} GB per layer)")
    flags = Q.APPLY_NORM | Q.ADD_RESIDUAL
    nsteps = args.warmup + args.steps
    nx = min(nsteps, max(2, (1 << 30) // max(1, T * d * 4)))
    g = torch.Generator(device=f"cuda:{dev}")
    g.manual_seed(sp0.seed + 17)
    xs = torch.randn((nx, T, d), generator=g, device=f"cuda:{dev}", dtype=torch.float32)
    out = torch.empty((T, d), dtype=torch.float32, device=f"cuda:{dev}")
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{dev}")
    flush_rd = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{dev}")
    flush_out = torch.empty(1, dtype=torch.float32, device=f"cuda:{dev}")
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream

    def flush_l2(i):
        flush.fill_(float(i))
        torch.sum(flush_rd, dim=0, keepdim=True, out=flush_out)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            flush_l2(i)
            S.forward_device(xs[i % nx].data_ptr(), T, out.data_ptr(), flags, sp)
    torch.cuda.synchronize()
    S.sync()
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    try:
        ident = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        ident = str(dev)
    clocks = clock_sampler(ident)
    clocks.start()
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            flush_l2(i)
            ev0[i].record(stream)
            S.forward_device(xs[(args.warmup + i) % nx].data_ptr(), T, out.data_ptr(), flags, sp)
            ev1[i].record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    S.sync()
    total_ms = float(sum(ev0[i].elapsed_time(ev1[i]) for i in range(args.steps)))
    launches = sum(L.last_launch_count() for L in S.layers)
    # expert bytes the last step's batch selected, over all layers (+ routers)
    ebytes = sum(Q.tensor_bytes(d * f, x) for x in sp0.fmt)
    used = 0
    for L in S.layers:
        _, off = L.last_dispatch(T)
        used += int(np.count_nonzero(np.diff(off)))
    step_bytes = used * ebytes + nL * (E * d * 4 + 2 * T * d * 4)
    # e2e: pinned host tokens in, the stack's output back, copies inside the events
    xh = xs[:min(nx, nsteps)].cpu().pin_memory()
    oh = torch.empty((T, d), dtype=torch.float32).pin_memory()
    xd = torch.empty((T, d), dtype=torch.float32, device=f"cuda:{dev}")
    e0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            flush_l2(i)
            e0[i].record(stream)
            xd.copy_(xh[i % xh.shape[0]], non_blocking=True)
            S.forward_device(xd.data_ptr(), T, out.data_ptr(), flags, sp)
            oh.copy_(out, non_blocking=True)
            e1[i].record(stream)
    torch.cuda.synchronize()
    S.sync()
    e2e_ms = float(sum(e0[i].elapsed_time(e1[i]) for i in range(args.steps)))
    S.close()
    peaks, peak_kind = measured_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK["hbm_gbs"]))
    step_s = total_ms / args.steps / 1000.0
    ach = step_bytes / step_s / 1e9
    cpu = None
    if not args.no_cpu_baseline:
        try:
            # one token through one full-size layer, times the layer count
            v, cores, desc = cpu_sample(cfg_name, 1, budget_s=12.0)
            cpu = dict(value=v / nL, unit="tokens/s", cores=cores, kind="port",
                       sample=desc + f"; tokens/s of one layer divided by the {nL} layers of the stack")
        except Exception as ex:
            cpu = dict(value=None, unit="tokens/s", cores=None, kind="port", sample=f"failed: {ex}")
    streamed = nL - n_res
    return dict(
        metric=METRIC, value=args.steps * T / (total_ms / 1000.0), unit="tokens/s", n_gpus=1, steps=args.steps,
        warmup=args.warmup, ms_per_step=total_ms / args.steps, higher_is_better=True, scaling="weak", vs_baseline=None,
        dtype="expert products: weight codes x 16-bit fixed-point activations (integer MMA, exact int32 sums, "
              "f32 scales) or dequantised f16 x f16 (tensor MMA, f32 accumulate); routing and combine f32",
        data="synthetic",
        config=dict(workload=NAMES[cfg_name] + f"_stack{nL}", tokens_per_rank=T, layers=nL, resident_layers=n_res,
                    streamed_layers=streamed, hbm_budget_gb=args.hbm_budget_gb or None, d_model=d, n_experts=E,
                    top_k=cfg["n_active"], expert_ffn=f, formats=FORMATS[cfg_name],
                    l2="flushed before every step outside the timed events: 256 MiB written, then another 256 MiB "
                       "buffer read", parallelism="single GPU"),
        roofline=dict(bound="hbm", kernel=f"whole {nL}-layer stack step (expert bytes the batch selected + routers)",
                      achieved=ach, peak=hbm, unit="GB/s", frac=ach / hbm, peak_kind=f"{peak_kind} hbm_gbs",
                      bytes_per_launch=step_bytes, traffic=None),
        layer_hbm=dict(achieved_gbs=ach, frac_of_8tbs=ach / NOMINAL_HBM_GBS, frac_of_measured=ach / hbm,
                       bytes_per_step=step_bytes),
        h2d_stream=dict(bytes_per_step=streamed * lbytes, gbs=streamed * lbytes / step_s / 1e9) if streamed else None,
        cpu_baseline=cpu,
        e2e=dict(value=args.steps * T / (e2e_ms / 1000.0), unit="tokens/s", h2d_bytes_per_step=T * d * 4,
                 d2h_bytes_per_step=T * d * 4, call="qrm_stack_forward_device, pinned host buffers, copies inside "
                                                    "the events"),
        parity=dict(note="per-layer parity and stack == chain of single layers: tests/test_gpu_stack.py"),
        gpu_launches=launches * args.steps,
        clocks=clock_info,
    )


def main():
    # the JSON lines go to the original stdout; everything else written to
    # fd 1 (NCCL's version banner, library prints) goes to stderr
    out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--config", choices=sorted(NAMES), default="c5")
    ap.add_argument("--sweep", action="store_true", help="one line per (config, T) of the measurement plan")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--experts", type=int, default=0, help="routed experts (a smaller case of the config)")
    ap.add_argument("--layers", type=int, default=32, help="config c2: layers of the stack (1: one layer)")
    ap.add_argument("--hbm-budget-gb", type=float, default=0.0,
                    help="config c2 stack: expert bytes kept in HBM (0: all); the other layers stream from host")
    ap.add_argument("--flush", choices=["write", "write-read"], default="write-read",
                    help="L2 flush between steps: write a buffer larger than L2, then (write-read) read another")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world, out)
    import torch
    import qauntrunner_b200 as Q
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as tdist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        dist = tdist
    try:
        runs = SWEEP if args.sweep else [(args.config, args.tokens)]
        for cfg_name, T in runs:
            if cfg_name == "c2" and args.layers > 1 and world == 1:
                line = run_stack(args, cfg_name, T, torch, Q)
            else:
                line = run_one(args, cfg_name, T, rank, world, dist, torch, Q)
            if line is not None:
                print(json.dumps(line), file=out, flush=True)
        return 0
    finally:
        if dist:
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
