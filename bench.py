"""Benchmark: π0.5 action chunks (prefill of 968 prefix tokens + 10 denoise steps, batch 1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--batch B]

One process per GPU (torchrun for N > 1). Every rank holds a full replica of the fp16 model
(random N(0, 0.02) weights, seeded) and runs its own independent requests; there is no
collective on the data path (the only collectives are the timing barrier and the max over
ranks). One step = one action chunk per request: ``prefill`` (18 prefix-expert layers over
968 tokens, writing the per-layer K/V cache) + ``denoise_loop_kv`` (10 Euler steps of the
action expert, replayed as one CUDA graph), inputs resident in HBM. ``e2e`` times the public
API ``PiZeroRunner.sample_graph`` from pinned host buffers (prefix embeddings and noise up,
actions down) over the same steps.

Prints one JSON line on rank 0 (schema in the project's build notes): value = chunks/s over all
GPUs, ms_per_step = ms per chunk (per GPU), roofline of the dominant kernel family measured
live with CUDA events, the CPU oracle timed on one whole chunk as ``cpu_baseline``, SM clocks
sampled during the timed region, and the number of library kernels launched.

``--impl reference`` times the reference's CPU implementation of the path — the numpy oracle
that restates it (the reference itself needs TVM, absent here) — on all host cores, one whole
chunk per step (until the steps are done or two minutes of chunks have run), and prints the same
line with ``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "mlc-vla_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "pi0.5 ms/action-chunk (prefill968+10 steps, bs1); chunks/s at 1/2/4/8 GPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def full_config(logits="float32"):
    """The benchmarked π0.5 configuration; ``logits`` is the reference's attn_logits_dtype
    (its default "float32", or "float16" for its tensor-core option)."""
    from mlc_vla.model.pi0 import Pi0Config

    return Pi0Config(action_horizon=50, action_dim=32, num_denoise_steps=10, dtype="float16",
                     attn_logits_dtype=logits)


# ------------------------------------------------------------------------------------------
# algorithmic work per kernel family (per chunk), for the roofline
# ------------------------------------------------------------------------------------------
def work_model(cfg, batch):
    """family -> (work per chunk, unit, bound). FLOPs for the compute-bound prefill, HBM bytes
    (weights + K/V + activations, each read or written once) for the weight-bound denoise."""
    vlm, ae = cfg.vlm, cfg.action_expert
    L, H, KV, hd = vlm.depth, vlm.num_heads, vlm.num_kv_heads, vlm.head_dim
    hq, hkv = H * hd, KV * hd
    W0, F0, W1, F1 = vlm.width, vlm.mlp_dim, ae.width, ae.mlp_dim
    P, S, D, N = cfg.prefix_len, cfg.suffix_len, cfg.action_dim, cfg.num_denoise_steps
    M0, M1 = batch * P, batch * S
    e = 2
    w = {}
    w["prefill.qkv_rope_gemm"] = (2 * M0 * W0 * ((L - 1) * (hq + 2 * hkv) + 2 * hkv), "flop", "tensor")
    w["prefill.attention"] = ((L - 1) * 4 * batch * H * P * P * hd, "flop", "tensor")
    w["prefill.o_gemm"] = ((L - 1) * 2 * M0 * W0 * hq, "flop", "tensor")
    w["prefill.gate_up_geglu_gemm"] = ((L - 1) * 2 * M0 * W0 * 2 * F0, "flop", "tensor")
    w["prefill.down_gemm"] = ((L - 1) * 2 * M0 * W0 * F0, "flop", "tensor")
    w["prefill.rmsnorm"] = ((2 * L - 1) * 2 * M0 * W0 * e, "byte", "hbm")
    nmod = (2 * L + 1) * 3 * W1
    w["denoise.time_mlp_modulation_gemm"] = ((2 * W1 * W1 + nmod * W1) * e, "byte", "hbm")
    per_step = {
        "denoise.qkv_rope_gemm": L * ((hq + 2 * hkv) * W1 * e + M1 * (W1 * e + hq * 4 + 2 * hkv * 4)),
        "denoise.attention": L * batch * KV * (P + S) * hd * (4 + e),
        "denoise.o_gemm": L * (W1 * hq * e + M1 * (hq + 2 * W1) * e),
        "denoise.gate_up_geglu_gemm": L * (2 * F1 * W1 * e + M1 * (W1 + F1) * e),
        "denoise.down_gemm": L * (W1 * F1 * e + M1 * (F1 + 2 * W1) * e),
        "denoise.ada_rmsnorm": (2 * L + 1) * 2 * M1 * W1 * e,
        "denoise.action_in": (W1 * D + M1 * W1) * e,
        "denoise.action_out_euler": (W1 * D) * e + M1 * W1 * e,
    }
    for k, v in per_step.items():
        w[k] = (N * v, "byte", "hbm")
    return w


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from one ncu capture of each
# kernel at the bench's configuration, reported as the roofline's "traffic" when that family is the
# dominant one; traffic near the algorithmic bytes means no operand is read twice.
NCU_TRAFFIC = {
    "denoise.gate_up_geglu_gemm": 16936704,
    "denoise.qkv_rope_gemm": 5465344,
    "denoise.o_gemm": 4541440,
    "denoise.down_gemm": 8940544,
    "denoise.attention": 2054144,  # fp32 logits (K hi + lo read); NCU_TRAFFIC_F16 with fp16 logits
    "prefill.gate_up_geglu_gemm": 138220032 + 17278720,
    "prefill.attention": 5023232,
}


NCU_TRAFFIC_F16 = {"denoise.attention": 1315584}


def roofline_of(fam, wm, traffic):
    """Roofline of the dominant kernel family of `fam` ({family: (launches, device ms)}) against
    the measured peaks: achieved = the family's algorithmic work (`wm`) ÷ its device time."""
    pk, pk_kind = peaks()
    dom = max(fam, key=lambda k: fam[k][1])
    work, unit, bound = wm.get(dom, (0, "byte", "hbm"))
    ms = fam[dom][1]
    if bound == "tensor":
        achieved = work / (ms / 1e3) / 1e12
        peak = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
        runit = "TFLOP/s"
    else:
        achieved = work / (ms / 1e3) / 1e9
        peak = pk["hbm_gbs"]
        runit = "GB/s"
    families = {}
    for k, (n, tot) in sorted(fam.items(), key=lambda kv: -kv[1][1]):
        wk = wm.get(k)
        ent = {"launches": n, "ms": round(tot, 4), "share": round(tot / sum(v[1] for v in fam.values()), 4)}
        if wk:
            if wk[2] == "tensor":
                ent["tflops"] = round(wk[0] / (tot / 1e3) / 1e12, 1)
            else:
                ent["gbs"] = round(wk[0] / (tot / 1e3) / 1e9, 1)
        families[k] = ent
    return {"bound": bound, "kernel": dom, "achieved": round(achieved, 2), "peak": peak,
            "unit": runit, "frac": round(achieved / peak, 4), "traffic": traffic.get(dom),
            "traffic_unit": "bytes per launch (ncu)",
            "peak_source": f"{pk_kind} ({'bf16_tflops_sustained' if bound == 'tensor' else 'hbm_gbs'})",
            "work_per_launch": work / max(1, fam[dom][0]), "families": families}


# ------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ------------------------------------------------------------------------------------------
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        # samples go to a private temporary file (removed after the summary is read)
        fd, self.path = tempfile.mkstemp(prefix=f"pi0_clocks_gpu{gpu_index}_", suffix=".csv")
        os.close(fd)

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        try:
            os.unlink(self.path)
        except OSError:
            pass
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------
# CPU baseline: the oracle on whole chunks
# ------------------------------------------------------------------------------------------
def cpu_threads():
    """Use every host core for the oracle's BLAS calls, also under torchrun (which exports
    OMP_NUM_THREADS=1), and return the count in use."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info, threadpool_limits

        threadpool_limits(n)
        got = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(got) if got else n
    except Exception:  # noqa: BLE001
        return n


class CpuChunk:
    """The numpy oracle on the benchmarked workload: prefill of 968 tokens through all 18 prefix
    layers plus the 10-step denoise loop through all 18 action-expert layers, fp16 rounding
    emulated on fp32 BLAS. Every layer computes in full; to keep set-up short, all layers of an
    expert share one seeded draw of that expert's layer weights (the arithmetic and the bytes
    streamed per layer are those of distinct weights: a layer's 0.4 GB fp32 copy is far larger
    than the host caches)."""

    SAMPLE = ("numpy oracle (fp32 BLAS, fp16 rounding emulated): one whole chunk per step, "
              "prefill(968) through 18 prefix layers + denoise_loop_kv (10 steps x 18 layers), "
              "batch 1; layers of an expert share one weight draw")

    def __init__(self):
        from mlc_vla.model.pi0 import Pi0Config
        from mlc_vla.model.pi0.pi0_model import backbone_named_params
        from oracle import pi0_oracle as O

        self.O = O
        self.cores = cpu_threads()
        cfg = Pi0Config(action_horizon=50, action_dim=32, num_denoise_steps=10, dtype="float16")
        self.cfg = cfg
        named = backbone_named_params(cfg)
        rng = np.random.default_rng(0)
        drawn, self.p = {}, {}
        for name, spec in named:
            # backbone.layers.<i>.<rest>: one draw per <rest>, shared by every layer i
            parts = name.split(".")
            key = ".".join(parts[3:]) if name.startswith("backbone.layers.") else name
            if key not in drawn:
                w = rng.standard_normal(tuple(int(x) for x in spec.shape), dtype=np.float32)
                drawn[key] = O.rnd(w * np.float32(0.02), "float16")
            self.p[name] = drawn[key]
        P, S, D = cfg.prefix_len, cfg.suffix_len, cfg.action_dim
        self.prefix = rng.standard_normal((1, P, cfg.vlm.width), dtype=np.float32)
        self.noise = rng.standard_normal((1, S, D), dtype=np.float32)
        self.pm = O.prefix_mask(P)
        self.sc, self.ss = O.suffix_rope(cfg, P)
        self.te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)

    def chunk_ms(self):
        O = self.O
        t0 = time.perf_counter()
        k, v = O.prefill(self.p, self.cfg, self.prefix, self.pm)
        O.denoise_loop_kv(self.p, self.cfg, k, v, self.noise, self.te, self.sc, self.ss, self.pm)
        return (time.perf_counter() - t0) * 1e3

    def warm(self):
        """A short untimed pass (one denoise step on a zero cache) that touches every code path."""
        O, cfg = self.O, self.cfg
        kv = (cfg.vlm.depth, 1, cfg.vlm.num_kv_heads, cfg.prefix_len, cfg.vlm.head_dim)
        z = np.zeros(kv, np.float32)
        O.denoise_step_kv(self.p, cfg, z, z, self.noise, self.te[:1], self.sc, self.ss, self.pm)


# ------------------------------------------------------------------------------------------
# reference arm
# ------------------------------------------------------------------------------------------
# the reference arm times whole samples until --steps are done or this much host time has gone,
# so that `--steps K` with the GPU arm's K still ends within a few minutes
REFERENCE_BUDGET_S = 120.0


def timed_samples(fn, steps):
    """Times fn() (returns ms) up to `steps` times, stopping early once REFERENCE_BUDGET_S of
    samples have run (at least one sample)."""
    t, spent = [], 0.0
    for _ in range(max(1, steps)):
        t.append(fn())
        spent += t[-1] / 1e3
        if spent >= REFERENCE_BUDGET_S:
            break
    return t


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cpu = CpuChunk()
    for _ in range(args.warmup):
        cpu.warm()
    t = timed_samples(cpu.chunk_ms, args.steps)
    ms = float(np.mean(t))
    value = 1000.0 / ms
    line = {
        "metric": METRIC, "value": value, "unit": "chunks/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": "pi0.5 fp16 bs1: prefill(968) + 10 Euler steps (host CPU)",
                   "global_batch": 1, "seq_len": 968, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "chunks/s", "cores": cpu.cores, "kind": "port",
                         "sample": CpuChunk.SAMPLE + f"; {len(t)} whole chunks timed (of "
                         f"{args.steps} steps asked; at most {REFERENCE_BUDGET_S:.0f} s of samples), "
                         f"warm-up: {args.warmup} single denoise steps"},
        "e2e": {"value": value, "unit": "chunks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------
# B200 arm
# ------------------------------------------------------------------------------------------
def make_weights(named_params, device, seed=0):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for _, spec in named_params:
        t = torch.randn(spec.shape, generator=g, device=device, dtype=torch.float32).mul_(0.02)
        out.append(t.to(torch.float16))
    return out


def family_times(rt, fn, vision=False):
    """{kernel family: (launches, device ms)} of one call of `fn`, replayed from a captured graph
    in which every launch is bracketed by event-record nodes (the profiled pass). `vision`: `rt`
    is a VisionRuntime."""
    import ctypes

    import torch

    from mlc_vla import _lib

    lib = _lib.load()
    enable = lib.pi0_vision_profile_enable if vision else lib.pi0_profile_enable
    read = lib.pi0_vision_profile_read if vision else lib.pi0_profile_read
    enable(rt._ctx, 1)
    fn()
    torch.cuda.synchronize()
    nf = lib.pi0_profile_families()
    launches = (ctypes.c_int64 * nf)()
    total = (ctypes.c_double * nf)()
    _lib.check(read(rt._ctx, nf, launches, total), rt._ctx, vision=vision)
    enable(rt._ctx, 0)
    return {lib.pi0_profile_family_name(i).decode(): (int(launches[i]), float(total[i]))
            for i in range(nf) if launches[i]}


def make_quant_weights(cfg, preset, device, seed=0):
    """The quantised parameter table of `preset` (q_weight, q_scale and bias per Linear): the
    make_weights draws, each Linear weight group-quantised on the GPU."""
    from mlc_vla.model.pi0.pi0_model import backbone_named_params
    from mlc_vla.runtime import quantize_weight

    fp = dict(zip([n for n, _ in backbone_named_params(cfg)],
                  make_weights(backbone_named_params(cfg), device, seed)))
    out = []
    for name, _ in backbone_named_params(cfg, quant=preset):
        if name.endswith(".q_weight"):
            out += quantize_weight(fp[name[: -len(".q_weight")] + ".weight"], preset)
        elif not name.endswith(".q_scale"):
            out.append(fp[name])
    return out


def run_b200(args):
    import torch
    import torch.distributed as dist

    from mlc_vla import _lib
    from mlc_vla.replicas import whole_job_throughput
    from mlc_vla.sample import PiZeroRunner, make_prefix_mask_np, make_rope_np, make_time_embs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    cfg = full_config(args.attn_logits)
    B = args.batch
    quant = None
    if args.quant != "none":
        from mlc_vla.quant import PRESETS

        quant = PRESETS[args.quant]
    runner = PiZeroRunner(cfg, target="cuda", max_batch=B, device=local, quant=quant)
    rt = runner.ex
    params = (make_weights(rt.named_params, dev, seed=0) if quant is None
              else rt.to_params(make_quant_weights(cfg, quant, dev, seed=0)))
    rt.bind(params)
    lib = _lib.load()

    # device-resident inputs (per-rank seeds: independent requests)
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    P, S, D, W0 = cfg.prefix_len, cfg.suffix_len, cfg.action_dim, cfg.vlm.width
    prefix = torch.randn((B, P, W0), generator=gen, device=dev).to(torch.float16)
    noise = torch.randn((B, S, D), generator=gen, device=dev)
    # --pad: per-request valid prefix length ~ U[700, 968] (seeded per rank), padded to 968 with
    # the mask, suffix RoPE offset = valid length (the throughput sweep's inputs)
    if args.pad:
        nvs = np.random.default_rng(2000 + rank).integers(700, P + 1, size=B)
    else:
        nvs = np.full(B, P)
    pads = np.stack([(np.arange(P) < nv).astype(np.float32) for nv in nvs])
    pm = torch.from_numpy(np.concatenate(
        [make_prefix_mask_np(P, pad_mask=pads[i]) for i in range(B)], 0)).to(dev)
    ropes = [make_rope_np(S, cfg.vlm.head_dim, cfg.rope_theta, offset=int(nv)) for nv in nvs]
    sc = torch.from_numpy(np.concatenate([r[0] for r in ropes], 0)).to(dev)
    ss = torch.from_numpy(np.concatenate([r[1] for r in ropes], 0)).to(dev)
    te = torch.from_numpy(np.concatenate(make_time_embs(cfg.num_denoise_steps, cfg.action_expert.width), 0)).to(dev, torch.float16)
    vlm = cfg.vlm
    kv_shape = (vlm.depth, B, vlm.num_kv_heads, P, vlm.head_dim)
    keys = torch.empty(kv_shape, dtype=torch.float32, device=dev)
    values = torch.empty(kv_shape, dtype=torch.float16, device=dev)
    x = torch.empty((B, S, D), dtype=torch.float32, device=dev)

    def chunk():
        rt.prefill(prefix, pm, keys=keys, values=values)
        rt.denoise_loop_kv(keys, values, noise, te, sc, ss, pm, out=x)

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        chunk()
    torch.cuda.synchronize(dev)

    fam = family_times(rt, chunk)
    for _ in range(2):
        chunk()  # re-warm the graph path
    torch.cuda.synchronize(dev)

    # timed region (device-resident inputs)
    barrier()
    torch.cuda.synchronize(dev)
    n0 = lib.pi0_launch_count(rt._ctx)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            chunk()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    n_launch = lib.pi0_launch_count(rt._ctx) - n0
    elapsed = e0.elapsed_time(e1)
    barrier()
    # whole-job chunks/s: every rank's chunks over the slowest rank's device time
    value, elapsed_max = whole_job_throughput(elapsed, B * args.steps)
    ms_chunk = elapsed_max / args.steps

    # end to end through the public API: pinned host prefix + noise up, actions down
    e2e = None
    if not args.no_e2e:
        host_prefix = prefix.cpu().pin_memory()
        host_noise = noise.cpu().numpy()
        for _ in range(max(1, args.warmup)):
            runner.sample_graph(params, host_prefix, noise=host_noise, prefix_pad=pads if args.pad else None)
        torch.cuda.synchronize(dev)
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            runner.sample_graph(params, host_prefix, noise=host_noise, prefix_pad=pads if args.pad else None)
        f1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_value, e2e_ms = whole_job_throughput(f0.elapsed_time(f1), B * args.steps)
        # per step: the prefix embeddings and the noise; the pad mask, suffix RoPE tables and
        # time embeddings depend on the (unchanging) pad pattern and step count only, and the
        # runner keeps them on the device after the first call
        h2d = host_prefix.numel() * host_prefix.element_size() + host_noise.nbytes
        e2e = {"value": e2e_value, "unit": "chunks/s", "ms_per_step": e2e_ms / args.steps,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(B * S * D * 4)}

    traffic = dict(NCU_TRAFFIC, **(NCU_TRAFFIC_F16 if args.attn_logits == "float16" else {}))
    roofline = roofline_of(fam, work_model(cfg, B), traffic)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        c = CpuChunk()
        c.warm()
        cms = c.chunk_ms()
        cpu = {"value": 1000.0 / cms, "unit": "chunks/s", "cores": c.cores, "kind": "port",
               "sample": CpuChunk.SAMPLE + "; one chunk timed", "ms_per_chunk": round(cms, 1)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "chunks/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_chunk,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (random N(0,0.02) weights, N(0,1) prefix_embs and noise, seeded)",
            "config": {"workload": "pi0.5 fp16, per GPU batch %d: prefill(968) + denoise_loop_kv "
                                   "(10 Euler steps, one CUDA graph); horizon 50, action_dim 32%s%s"
                                   % (B, "; valid prefix lengths U[700,968], padded with the mask"
                                      if args.pad else "",
                                      "" if quant is None else f"; weights {args.quant} (the denoise "
                                      "GEMMs read the codes, prefill reads them dequantised)"),
                       "model": "pi0.5 (gemma_2b prefix expert + gemma_300m action expert)",
                       "global_batch": world * B, "seq_len": P, "parallelism": f"dp{world} (replicas)",
                       "attn_logits_dtype": args.attn_logits,
                       "l2": "inputs larger than L2 (4.8 GB of weights streamed per chunk)"},
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk.summary(),
            "gpu_launches": int(n_launch),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    rt.close()
    return 0


def run_part(args):
    """``--part prefill`` / ``--part step``: time one half of the chunk on one GPU (the prefill
    alone, or one ``denoise_step_kv`` on a seeded random K/V cache), for per-kernel profiling.
    Prints a JSON line with the part's mean ms; the chunk metric is the default mode."""
    import torch

    from mlc_vla.runtime import Pi0Runtime
    from mlc_vla.sample import make_prefix_mask_np, make_rope_np, make_time_embs

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = full_config(args.attn_logits)
    if args.layers == 2:  # profiling aid: every width of the full model, two layers
        cfg = dataclasses.replace(cfg, paligemma_variant="gemma_2b_2l",
                                  action_expert_variant="gemma_300m_2l")
    if args.quant != "none":
        from mlc_vla.quant import PRESETS

        q = PRESETS[args.quant]
        rt = Pi0Runtime(cfg, device=0, quant=q)
        rt.bind(rt.to_params(make_quant_weights(cfg, q, dev, seed=0)))
    else:
        rt = Pi0Runtime(cfg, device=0)
        rt.bind(make_weights(rt.named_params, dev, seed=0))
    P, S, D, W0 = cfg.prefix_len, cfg.suffix_len, cfg.action_dim, cfg.vlm.width
    g = torch.Generator(device=dev).manual_seed(1)
    pm = torch.from_numpy(make_prefix_mask_np(P)).to(dev)
    vlm = cfg.vlm
    kv = (vlm.depth, 1, vlm.num_kv_heads, P, vlm.head_dim)
    if args.part == "prefill":
        prefix = torch.randn((1, P, W0), generator=g, device=dev).half()
        keys = torch.empty(kv, device=dev)
        values = torch.empty(kv, device=dev, dtype=torch.float16)

        def once():
            rt.prefill(prefix, pm, keys=keys, values=values)
    else:
        keys = torch.randn(kv, generator=g, device=dev) * 0.5
        values = (torch.randn(kv, generator=g, device=dev) * 0.5).half()
        c, s_ = make_rope_np(S, vlm.head_dim, cfg.rope_theta, offset=P)
        sc, ss = torch.from_numpy(c).to(dev), torch.from_numpy(s_).to(dev)
        te = torch.from_numpy(make_time_embs(1, cfg.action_expert.width)[0]).to(dev, torch.float16)
        x = torch.randn((1, S, D), generator=g, device=dev)
        v = torch.empty_like(x)

        def once():
            rt.denoise_step_kv(keys, values, x, te, sc, ss, pm, out=v)
    for _ in range(args.warmup):
        once()
    torch.cuda.synchronize(dev)
    fam = family_times(rt, once)
    for _ in range(2):
        once()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        once()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / max(1, args.steps)
    print(json.dumps({"part": args.part, "ms": ms, "steps": args.steps, "warmup": args.warmup,
                      "config": f"pi0.5 fp16 batch 1 (full widths, {cfg.vlm.depth} layers), "
                                f"weights {args.quant}",
                      "families_ms": {k: round(v[1], 4) for k, v in sorted(
                          fam.items(), key=lambda kv: -kv[1][1])}}),
          flush=True)
    rt.close()
    return 0


# ------------------------------------------------------------------------------------------
# --workload embed_image: the vision stage (SigLIP So400m/14 + projector), 3 images per step
# ------------------------------------------------------------------------------------------
METRIC_VISION = ("pi0.5 embed_image images/s (SigLIP So400m/14 27 layers + projector, "
                 "224x224x3 -> 256x2048, fp16); one step = one 3-camera observation")
VISION_IMAGES = 3


def vision_work_model(cfg, n):
    """family -> (work per call of n images, unit, bound): GEMM and attention FLOPs (the patch
    GEMM at the unpadded K = p·p·C), LayerNorm bytes (read + write once)."""
    s = cfg.siglip
    L, W, F, H = s.num_hidden_layers, s.hidden_size, s.intermediate_size, s.num_attention_heads
    T, hd, pd = s.num_patches, s.head_dim, s.patch_size * s.patch_size * s.num_channels
    M = n * T
    return {
        "vision.patchify_embed_gemm": (2 * M * pd * W, "flop", "tensor"),
        "vision.qkv_gemm": (L * 2 * M * W * 3 * W, "flop", "tensor"),
        "vision.attention": (L * 4 * n * H * T * T * hd, "flop", "tensor"),
        "vision.out_gemm": (L * 2 * M * W * W, "flop", "tensor"),
        "vision.fc1_gelu_gemm": (L * 2 * M * W * F, "flop", "tensor"),
        "vision.fc2_gemm": (L * 2 * M * F * W, "flop", "tensor"),
        "vision.projector_gemm": (2 * M * W * s.projection_dim, "flop", "tensor"),
        "vision.layernorm": ((2 * L + 1) * 2 * M * W * 2, "byte", "hbm"),
    }


def vision_weights(named_params, device, seed=0):
    """make_weights draws with 1 added to every LayerNorm weight."""
    out = make_weights(named_params, device, seed)
    for t, (name, _) in zip(out, named_params):
        if name.endswith(("layer_norm1.weight", "layer_norm2.weight", "post_layernorm.weight")):
            t.add_(1.0)
    return out


class CpuVision:
    """The numpy SigLIP oracle on one 224×224×3 image per step (27 layers + projector, fp16
    rounding emulated on fp32 BLAS)."""

    SAMPLE = ("numpy SigLIP oracle (fp32 BLAS, fp16 rounding emulated): one image per step, "
              "27 layers + post LayerNorm + projector; layers share one weight draw")

    def __init__(self):
        from mlc_vla.model.pi0 import Pi0Config
        from mlc_vla.model.pi0.pi0_model import vision_named_params
        from oracle import pi0_oracle as O
        from oracle import siglip_oracle as S

        self.S = S
        self.cores = cpu_threads()
        self.cfg = Pi0Config(dtype="float16")
        rng = np.random.default_rng(0)
        drawn, self.p = {}, {}
        for name, spec in vision_named_params(self.cfg):
            # vision.layers.<i>.<rest>: one draw per <rest>, shared by every layer i (each layer
            # still computes in full; set-up stays short)
            key = ".".join(name.split(".")[3:]) if name.startswith("vision.layers.") else name
            if key not in drawn:
                w = rng.standard_normal(tuple(int(x) for x in spec.shape), dtype=np.float32)
                w *= np.float32(0.02)
                if name.endswith(("layer_norm1.weight", "layer_norm2.weight", "post_layernorm.weight")):
                    w += np.float32(1.0)
                drawn[key] = O.rnd(w, "float16")
            self.p[name] = drawn[key]
        sg = self.cfg.siglip
        self.image = rng.uniform(-1, 1, (1, sg.image_size, sg.image_size, sg.num_channels)).astype(np.float32)

    def image_ms(self):
        t0 = time.perf_counter()
        self.S.embed_image(self.p, self.cfg, self.image)
        return (time.perf_counter() - t0) * 1e3


def run_vision_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    cpu = CpuVision()
    for _ in range(min(args.warmup, 1)):
        cpu.image_ms()
    t = timed_samples(cpu.image_ms, args.steps)
    ms = float(np.mean(t))
    value = 1000.0 / ms
    line = {
        "metric": METRIC_VISION, "value": value, "unit": "images/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms * VISION_IMAGES,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": "embed_image fp16, SigLIP So400m/14 (host CPU, one image per step)",
                   "global_batch": 1, "seq_len": 256, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": cpu.cores, "kind": "port",
                         "sample": CpuVision.SAMPLE + f"; {len(t)} images timed (of "
                         f"{args.steps} steps asked; at most {REFERENCE_BUDGET_S:.0f} s of samples), "
                         f"{min(args.warmup, 1)} untimed"},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_vision(args):
    import torch
    import torch.distributed as dist

    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.replicas import whole_job_throughput
    from mlc_vla.vision import VisionRuntime

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    cfg = Pi0Config(dtype="float16")
    n = VISION_IMAGES * args.batch
    rt = VisionRuntime(cfg, device=local, max_images=n)
    params = vision_weights(rt.named_params, dev, seed=0)
    rt.bind(params)
    sg = cfg.siglip
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    images = (torch.rand((n, sg.image_size, sg.image_size, sg.num_channels), generator=gen,
                         device=dev) * 2 - 1).to(torch.float16)
    out = torch.empty((n, sg.num_patches, sg.projection_dim), dtype=torch.float16, device=dev)

    def once():
        rt.embed_image(images, out=out)

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        once()
    torch.cuda.synchronize(dev)
    fam = family_times(rt, once, vision=True)
    for _ in range(2):
        once()
    torch.cuda.synchronize(dev)

    barrier()
    torch.cuda.synchronize(dev)
    n0 = rt.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            once()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    n_launch = rt.launch_count() - n0
    elapsed = e0.elapsed_time(e1)
    barrier()
    value, elapsed_max = whole_job_throughput(elapsed, n * args.steps)
    ms_step = elapsed_max / args.steps

    # end to end through the public API: pinned host images up, image tokens down
    e2e = None
    if not args.no_e2e:
        host = images.cpu().pin_memory()
        host_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        dimg = torch.empty_like(images)

        def e2e_once():
            dimg.copy_(host, non_blocking=True)
            rt.embed_image(dimg, out=out)
            host_out.copy_(out, non_blocking=True)

        for _ in range(max(1, args.warmup)):
            e2e_once()
        torch.cuda.synchronize(dev)
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            e2e_once()
        f1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_value, e2e_ms = whole_job_throughput(f0.elapsed_time(f1), n * args.steps)
        e2e = {"value": e2e_value, "unit": "images/s", "ms_per_step": e2e_ms / args.steps,
               "h2d_bytes_per_step": int(host.numel() * host.element_size()),
               "d2h_bytes_per_step": int(host_out.numel() * host_out.element_size())}

    roofline = roofline_of(fam, vision_work_model(cfg, n), NCU_TRAFFIC_VISION)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        c = CpuVision()
        c.image_ms()
        cms = c.image_ms()
        cpu = {"value": 1000.0 / cms, "unit": "images/s", "cores": c.cores, "kind": "port",
               "sample": CpuVision.SAMPLE + "; one image timed after one untimed",
               "ms_per_image": round(cms, 1)}
    if rank == 0:
        line = {
            "metric": METRIC_VISION, "value": value, "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (random N(0,0.02) weights, LayerNorm weights 1 + N(0,0.02); "
                    "U(-1,1) images; seeded)",
            "config": {"workload": f"embed_image fp16, {n} images of 224x224x3 per call (one CUDA "
                                   "graph): patchify + 27 SigLIP layers + post LayerNorm + projector",
                       "model": "SigLIP So400m/14 + PaliGemma projector",
                       "global_batch": world * n, "seq_len": sg.num_patches,
                       "parallelism": f"dp{world} (replicas)",
                       "l2": "inputs larger than L2 (0.83 GB of weights streamed per call)"},
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk.summary(),
            "gpu_launches": int(n_launch),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    rt.close()
    return 0


# DRAM bytes per launch of the dominant vision family from one ncu capture at the bench's
# configuration (dram__bytes_read.sum + dram__bytes_write.sum)
NCU_TRAFFIC_VISION = {"vision.fc2_gemm": 18330368}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--pad", action="store_true",
                    help="per-request valid prefix lengths U[700,968] padded to 968 (throughput sweep)")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--part", default="chunk", choices=["chunk", "prefill", "step"],
                    help="profiling aid: time only the prefill or one denoise step")
    ap.add_argument("--quant", default="none", choices=["none", "q4f16_1", "q3f16_1"],
                    help="group-quantised weights (the denoise GEMMs dequantise in shared memory)")
    ap.add_argument("--attn-logits", default="float32", choices=["float32", "float16"],
                    help="attention logits operands (the reference's attn_logits_dtype; its "
                         "default float32, or float16 for its tensor-core option)")
    ap.add_argument("--layers", type=int, default=18, choices=[2, 18],
                    help="with --part: 2 = full widths with two layers, for small profiler captures")
    ap.add_argument("--workload", default="chunk", choices=["chunk", "embed_image"],
                    help="chunk: the action-chunk hot path (default); embed_image: the vision "
                         "stage, 3 images per step")
    args = ap.parse_args()
    if args.workload == "embed_image":
        return run_vision_reference(args) if args.impl == "reference" else run_vision(args)
    if args.part != "chunk":
        return run_part(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
