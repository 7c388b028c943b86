#!/usr/bin/env python
"""bench.py -- LTX-2.5's w8g64 qlinear and the joint AV DiT on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload stack|sweep|qlinear|i8|block|...]

The default line is BASELINE config 5, the metric's "DiT s/denoise-step
@960x544x121": a step is one forward of the 48-block joint audio-video stack
over 8160 video + 126 audio + 256 text tokens, random-init w8g64 weights
(seeded, generated and packed on the device), bf16 activations.  Under
torchrun the stack is tensor parallel over the N ranks (column-split q/k/v
and FF-up, row-split out-projections and FF-down, NCCL over NVLink): strong
scaling, the same step at every N, time = max over ranks.

value     s/step, inputs resident in HBM (weights ~21 GB / N stream every step).
e2e       the same through the C ABI (ltx_stack_forward) with the stream
          activations copied in from and out to pinned host memory each step.
roofline  algorithmic FLOPs of the step (GEMMs 2*M*N*K + attention 4*tq*tk*d)
          per GPU / time, against MEASURED_PEAKS.json: the sustained bf16 peak
          for a timed region of a second or more, else the burst one; both
          fractions are printed.
sweep     BASELINE config 2, the w8g64 linear-shape sweep (nine shapes, each
          through ltx_qlinear), measured on the same contexts after the stack:
          roofline_sweep (tensor, the six M=8160 shapes) and roofline_hbm (HBM,
          the three M=126 audio shapes) ride on the line.
cpu_baseline  the reference's own CPU block_forward (oracle/_ref, compiled
          from the reference sources) on a bounded full-width sample on all
          host cores, extrapolated to the step by FLOPs; rank 0 at N=1.

--impl reference  that reference CPU path alone, same metric and config
        (the reference's GPU path is Apple Metal, unavailable here).
Other workloads (--workload): sweep (config 2 alone, N replicas), qlinear
(config 1), i8 (config 3), block (config 4), attn, lora, trunk, connector,
adaln.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "vpipe-ltx-2.5_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

SHAPES = [  # (name, M, K, N)
    ("video attn-out 4096->4096", 8160, 4096, 4096),
    ("video fused-QKV 4096->12288", 8160, 4096, 12288),
    ("video FFN-up 4096->16384", 8160, 4096, 16384),
    ("video FFN-down 16384->4096", 8160, 16384, 4096),
    ("audio 2048->2048", 126, 2048, 2048),
    ("audio FFN-up 2048->8192", 126, 2048, 8192),
    ("audio FFN-down 8192->2048", 126, 8192, 2048),
    ("a2v out 2048->4096", 8160, 2048, 4096),
    ("v2a k/v 4096->2048", 8160, 4096, 2048),
]
METRIC = "w8g64 qlinear TFLOP/s, DiT linear-shape sweep (BASELINE config 2)"
UNIT = "TFLOP/s"
CPU_ROWS = 64        # cpu sample: first 64 tokens ...
CPU_FEATURES = 1024  # ... x first 1024 output features of every shape


def flops(M, K, N):
    return 2.0 * M * N * K


def hbm_bytes(M, K, N):
    return N * K * (1.0 + 4.0 / 64.0) + 2.0 * M * (K + N)


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


# A timed region at least this long is a seconds-long loop under the power
# cap, the regime MEASURED_PEAKS.json's sustained figure was measured in;
# shorter regions are bursts.  Chosen by the region's length, never by a
# clock sample, so the choice cannot flip on one nvidia-smi reading.
SUSTAINED_REGION_S = 1.0


def tensor_peak_for(region_s, clocks=None):
    """The bf16 tensor peak for a timed region of `region_s` seconds.
    Returns a dict: peak (the one the fraction uses), kind, burst, sustained
    (both MEASURED_PEAKS.json figures, so either fraction can be read)."""
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        burst, sus = float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"])
        src = "measured"
    except Exception:
        burst, sus, src = 1590.0, 1400.0, "fallback"
    if region_s >= SUSTAINED_REGION_S:
        peak, kind = sus, f"{src} bf16_tflops_sustained (timed region {region_s:.2f} s >= " \
                          f"{SUSTAINED_REGION_S:.0f} s)"
    else:
        peak, kind = burst, f"{src} bf16_tflops (burst; timed region {region_s * 1e3:.0f} ms)"
    return {"peak": peak, "kind": kind, "burst": burst, "sustained": sus}


def roofline_fracs(achieved, pk, clocks):
    """Both fractions and the clock-normalized rate (TFLOP/s per GHz of the
    median SM clock) so the clock dependence can be read off the line."""
    out = {"frac_of_burst": round(achieved / pk["burst"], 4),
           "frac_of_sustained": round(achieved / pk["sustained"], 4)}
    mhz = (clocks or {}).get("sm_mhz")
    if mhz:
        out["tflops_per_ghz"] = round(achieved / (mhz / 1e3), 1)
    return out


def traffic_from_profile():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/traffic.json), or None."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            return json.load(f)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,"
              "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100", "-i",
                 str(self.gpu_id)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi takes a while to print its first sample; the timed
            # region starts only once it does (at most 5 s), so short regions
            # are sampled too
            t0 = time.monotonic()
            while not self.lines and time.monotonic() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        self.t_start = time.monotonic()
        self.t_stop = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def __exit__(self, *a):
        self.t_stop = time.monotonic()
        if self.proc is not None:
            # one more sample period so the region's tail is covered
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.t.join(timeout=5)

    def summary(self):
        """Median SM clock and the throttle reasons seen over the samples
        taken inside the timed region (the sample just after it included)."""
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        stop = (self.t_stop if self.t_stop is not None else time.monotonic()) + 0.15
        for ts, ln in self.lines:
            if ts < self.t_start or ts > stop:
                continue
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [],
                    "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def gpu_index(local):
    """The nvidia-smi index of this rank's GPU (CUDA_VISIBLE_DEVICES aware)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    return vis.split(",")[local] if vis else str(local)


def make_weights(L, ctx, torch, dev, K, N, gen):
    w = torch.randn((N, K), generator=gen, device=dev, dtype=torch.float32) * 0.02
    codes, scales, biases = L.pack_w8g64(ctx, w)
    del w
    qw = L.QWeight.upload(ctx, codes, scales, biases, N, K, sb_dtype=L.SB_BF16,
                          on_device=True)
    del codes, scales, biases
    return qw


def cpu_reference_sample(threads):
    """The reference CPU qlinear (dequantise-then-dense, linear_ with f64
    accumulation) on the bounded sample.  Returns (flops, seconds, kind)."""
    import concurrent.futures as cf
    import numpy as np
    from oracle import lib as olib
    from oracle import ref as oref
    kind = "reference" if oref.available() else "port"
    rng = np.random.default_rng(7)
    jobs = []
    for _, M, K, N in SHAPES:
        m, n = min(M, CPU_ROWS), min(N, CPU_FEATURES)
        x = olib.bf16_to_f32(olib.f32_to_bf16(rng.standard_normal((m, K)).astype(np.float32)))
        w = (rng.standard_normal((n, K)) * 0.02).astype(np.float32)
        _, _, _, deq = (oref.pack(w, 8, 64) if kind == "reference"
                        else olib.pack_affine(w, 8, 64))
        jobs.append((x, deq))
    linear = oref.linear if kind == "reference" else (
        lambda x, w: olib.linear_f64(x, w, None, 1))

    def run_one(x, w):
        return linear(x, w)

    total = sum(flops(x.shape[0], x.shape[1], w.shape[0]) for x, w in jobs)
    t0 = time.perf_counter()
    if threads <= 1:
        for x, w in jobs:
            run_one(x, w)
    else:
        with cf.ThreadPoolExecutor(max_workers=threads) as ex:
            futs = []
            for x, w in jobs:
                step = max(1, (x.shape[0] + threads - 1) // threads)
                for r in range(0, x.shape[0], step):
                    futs.append(ex.submit(run_one, x[r:r + step], w))
            for f in futs:
                f.result()
    return total, time.perf_counter() - t0, kind


def sample_desc():
    return (f"first {CPU_ROWS} tokens x first {CPU_FEATURES} output features of "
            "each of the 9 sweep shapes (full K), weights dequantized once "
            "outside the timing")


def block_flops(vt, at, tt, vdim, adim):
    """Algorithmic FLOPs of one joint block: its 20 GEMMs (fused q/k/v and
    k/v counted as one) and the six attentions' QK^T and PV."""
    gemm = 0.0
    for (M, K, N) in [(vt, vdim, 3 * vdim), (vt, vdim, vdim), (vt, vdim, vdim), (tt, vdim, 2 * vdim),
                      (vt, vdim, vdim), (vt, vdim, 4 * vdim), (vt, 4 * vdim, vdim),
                      (at, adim, 3 * adim), (at, adim, adim), (at, adim, adim), (tt, adim, 2 * adim),
                      (at, adim, adim), (at, adim, 4 * adim), (at, 4 * adim, adim),
                      (vt, vdim, adim), (at, adim, 2 * adim), (vt, adim, vdim),
                      (at, adim, adim), (vt, vdim, 2 * adim), (at, adim, adim)]:
        gemm += flops(M, K, N)
    attn = 4.0 * (vt * vt * vdim + vt * tt * vdim + at * at * adim + at * tt * adim
                  + vt * at * adim + at * vt * adim)
    return gemm, attn


def run_stack(args):
    """one denoise step = the 48-block stack over 8160
    video + 126 audio + 256 text tokens, synthetic w8g64 weights, one shared
    scratch arena per GPU.  Under torchrun the stack is tensor-parallel over
    the ranks (Megatron split, NCCL all-reduce): strong scaling, the same
    step on every N."""
    import datetime
    import torch
    import ltx25_b200 as L
    from ltx25_b200 import synth
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
        pg = dist
    ctx = L.Context(local)
    if world > 1:
        uid = torch.zeros(L.TP_ID_BYTES, dtype=torch.uint8, device=dev)
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(L.tp_unique_id()), dtype=torch.uint8))
        pg.broadcast(uid, src=0)
        join = ctx.set_sp if args.parallel == "sp" else ctx.set_tp
        join(rank, world, bytes(uid.cpu().numpy().tobytes()))
    vdim, vh, adim, ah = 4096, 32, 2048, 32
    frames, hh, ww, at, tt = 16, 17, 30, 126, 256
    vt = frames * hh * ww
    nblk = args.blocks
    st = L.Stack(ctx)
    for i in range(nblk):
        # the same seed on every rank: each keeps its shard of the same weights
        st.add(synth.load_random_block(ctx, vdim, vh, adim, ah, seed=7 + i, device=dev))
    st.reserve(vt, at, tt)
    v_self, a_self, v_cross, a_cross = L.geometry_tables(frames, hh, ww, at, vdim, vh, adim, ah)
    dt = lambda t: (torch.from_numpy(t[0]).to(dev), torch.from_numpy(t[1]).to(dev))
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    v = synth.random_stream_inputs(vdim, vt, tt, vh, gen, device=dev, pe=dt(v_self),
                                   cross_pe=dt(v_cross))
    a = synth.random_stream_inputs(adim, at, tt, ah, gen, device=dev, pe=dt(a_self),
                                   cross_pe=dt(a_cross))
    x0v, x0a = v["x"].clone(), a["x"].clone()
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        v["x"].copy_(x0v)
        a["x"].copy_(x0a)
        st.forward(v, a)
    torch.cuda.synchronize()
    ctx.check()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    n0 = L.launch_count()
    with ClockSampler(gpu_index(local)) as clk:
        for e0, e1 in evs:
            # x is reset outside the timed pair; weights (>19 GB / N) and the
            # activations stream through HBM every step, far above L2
            v["x"].copy_(x0v)
            a["x"].copy_(x0a)
            e0.record(stream)
            st.forward(v, a, stream=stream)
            e1.record(stream)
        torch.cuda.synchronize()
    launches = L.launch_count() - n0
    if pg is not None:
        pg.barrier()
    ctx.check()
    times = [e0.elapsed_time(e1) for e0, e1 in evs]
    ms = sum(times) / len(times)          # the K timed steps, x resets excluded
    region_s = sum(times) * 1e-3
    if pg is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    ok = bool(torch.isfinite(v["x"].float()).all() and torch.isfinite(a["x"].float()).all())

    # end to end through the public API: host x in, host x out, every step
    hv = x0v.cpu().pin_memory()
    ha = x0a.cpu().pin_memory()
    ov = torch.empty_like(hv).pin_memory()
    oa = torch.empty_like(ha).pin_memory()
    e2e_steps = max(1, min(args.steps, 3))
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(e2e_steps):
        v["x"].copy_(hv, non_blocking=True)
        a["x"].copy_(ha, non_blocking=True)
        st.forward(v, a, stream=stream)
        ov.copy_(v["x"], non_blocking=True)
        oa.copy_(a["x"], non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1) / e2e_steps
    if pg is not None:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    ctx.check()

    g, at_fl = block_flops(vt, at, tt, vdim, adim)
    step_flops = nblk * (g + at_fl)
    achieved = step_flops / (ms * 1e-3) / 1e12
    io_bytes = (vt * vdim + at * adim) * 2
    clocks = clk.summary()
    pk = tensor_peak_for(region_s)
    per_gpu = achieved / world
    line = {
        "metric": "DiT s/denoise-step @960x544x121 (BASELINE config 5, 48-block stack)",
        "value": round(ms / 1e3, 4), "unit": "s/step", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded device-generated weights, w8g64)",
        "config": {"workload": f"{nblk}-block joint AV stack, one denoise step: video 8160x4096 "
                               "(16x17x30), audio 126x2048, text 256",
                   "parallelism": f"{args.parallel}{world}",
                   "l2": "weights (~21 GB / N) and activations far above L2 every step"},
        "e2e": {"value": round(e2e_ms / 1e3, 4), "unit": "s/step",
                "h2d_bytes_per_step": io_bytes, "d2h_bytes_per_step": io_bytes,
                "api": "ltx_stack_forward, x copied in from and out to pinned host memory"},
        "gpu_launches": int(launches),
        "algorithmic_tflop": round(step_flops / 1e12, 2),
        "tflops": round(achieved, 1),
        "roofline": dict({"bound": "tensor", "achieved": round(per_gpu, 1),
                          "peak": pk["peak"], "peak_source": pk["kind"],
                          "unit": "TFLOP/s per GPU", "frac": round(per_gpu / pk["peak"], 4),
                          "traffic": None},
                         **roofline_fracs(per_gpu, pk, clocks)),
        "finite": ok, "clocks": clocks,
    }
    st.close()
    for b in st.blocks:
        b.close()
    if not args.no_sweep:
        # BASELINE config 2 on the same contexts after the stack is freed
        # (replicas under torchrun), so the qlinear evidence rides the line
        sw = measure_sweep(args_for_sweep(args), ctx, dev, rank, world, pg, local)
        line["sweep"] = sw
        line["roofline_sweep"] = sw["roofline"]
        line["roofline_hbm"] = sw["roofline_hbm"]
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = ref_block_baseline(blocks=nblk)
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def args_for_sweep(args):
    """The sweep's own step count (its steps are ~3 ms, the stack's ~300)."""
    import copy
    a = copy.copy(args)
    a.steps = max(args.steps, 20)
    return a


def run_attn(args):
    """The video stream's self-attention (8160 x 8160 tokens, 32 heads of
    128) alone: the tcgen05 flash kernel (or, with --sage, the int8-QK
    tier), with q/k/v (200 MB) above L2."""
    import torch
    import ltx25_b200 as L
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = L.Context(local)
    tq = tk = 8160
    heads, D = 32, 128
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    q = torch.randn((tq, heads * D), generator=gen, device=dev).to(torch.bfloat16)
    kv = torch.randn((tk, 2 * heads * D), generator=gen, device=dev).to(torch.bfloat16)
    gate = torch.randn((tq, heads), generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    ctx.set_tiers(sage_attn=args.sage)
    run = lambda: L.attention(ctx, q, kv[:, :heads * D], kv[:, heads * D:], heads, D,
                              gate=gate, out=out)
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    ctx.check()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    gpu_id = os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local] \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else str(local)
    n0 = L.launch_count()
    with ClockSampler(gpu_id) as clk:
        for e0, e1 in evs:
            e0.record()
            run()
            e1.record()
        torch.cuda.synchronize()
    launches = (L.launch_count() - n0) // max(args.steps, 1)
    ctx.check()
    ms = statistics.median([e0.elapsed_time(e1) for e0, e1 in evs])
    fl = 4.0 * tq * tk * heads * D
    peak_tf, _, peak_kind = peaks()
    tf = fl / (ms * 1e-3) / 1e12
    line = {
        "metric": "video self-attention TFLOP/s (8160x8160, 32 heads x 128)" +
                  (" [sage int8 QK]" if args.sage else ""),
        "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "dtype": "int8 QK / bf16 PV" if args.sage else "bf16",
        "data": "synthetic N(0,1) q/k/v, gated",
        "config": {"workload": "attention 8160x8160x32x128 + gate; q/k/v 200 MB > L2"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak_tf,
                     "peak_kind": peak_kind, "unit": "TFLOP/s", "frac": round(tf / peak_tf, 3),
                     "traffic": None},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    ctx.set_tiers()
    ctx.close()
    return 0


def run_lora(args):
    """Low-rank adapters on a qlinear at the reference's own adapter
    benchmark shapes (tests/ltx25-lora-apply-test.cc:498-510): the x2
    upscaler's rank-32 projection and feed-forward widening over 32640
    tokens, and the distilled adapter's rank 450 over 8160.  Arms: the
    plain qlinear, the adapted qlinear with the delta in the same GEMM
    (ltx_qlinear_lora), and the plain qlinear followed by the standalone
    lora_add (the reference's form).  The adapter's arithmetic is 2*rank/K
    of the linear, the floor for its cost."""
    import torch
    import ltx25_b200 as L
    world, rank_, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = L.Context(local)
    shapes = [("x2 upscaler attn proj, rank 32", 32640, 4096, 4096, 32),
              ("x2 upscaler ff widening, rank 32", 32640, 4096, 16384, 32),
              ("distilled adapter, rank 450", 8160, 4096, 4096, 450)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(13)
    gpu_id = os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local] \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else str(local)
    rows = []
    n0 = L.launch_count()
    total = {"plain": 0.0, "fused": 0.0, "separate": 0.0}
    with ClockSampler(gpu_id) as clk:
        for name, M, K, N, r in shapes:
            w = torch.randn((N, K), generator=gen, device=dev) * 0.02
            c, s_, b_ = L.pack_w8g64(ctx, w)
            del w
            q = L.QWeight.upload(ctx, c, s_, b_, N, K, on_device=True)
            a = (torch.randn((r, K), generator=gen, device=dev) * (3.0 / (r * K) ** 0.5)).to(
                torch.bfloat16)
            b = torch.randn((N, r), generator=gen, device=dev).to(torch.bfloat16)
            lo = L.Lora(ctx, a, b)
            x = torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
            y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            arms = {"plain": lambda: L.qlinear(ctx, q, x, out=y),
                    "fused": lambda: L.qlinear_lora(ctx, q, lo, x, out=y),
                    "separate": lambda: (L.qlinear(ctx, q, x, out=y), L.lora_add(ctx, lo, x, y))}
            # arms interleaved step by step, rotating the order, so clock and
            # power drift fall on all three alike
            names = list(arms)
            for _ in range(args.warmup):
                for arm in names:
                    arms[arm]()
            torch.cuda.synchronize()
            evs = {arm: [(torch.cuda.Event(enable_timing=True),
                          torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
                   for arm in names}
            for i in range(args.steps):
                for j in range(len(names)):
                    arm = names[(i + j) % len(names)]
                    e0, e1 = evs[arm][i]
                    e0.record()
                    arms[arm]()
                    e1.record()
            torch.cuda.synchronize()
            res = {arm: statistics.median([e0.elapsed_time(e1) for e0, e1 in evs[arm]])
                   for arm in names}
            for arm in names:
                total[arm] += res[arm]
            ctx.check()
            rows.append({"shape": name, "M": M, "K": K, "N": N, "rank": r,
                         "plain_us": round(res["plain"] * 1e3, 1),
                         "fused_us": round(res["fused"] * 1e3, 1),
                         "separate_us": round(res["separate"] * 1e3, 1),
                         "fused_overhead": round(res["fused"] / res["plain"] - 1, 4),
                         "separate_overhead": round(res["separate"] / res["plain"] - 1, 4),
                         "arithmetic_overhead": round(2.0 * r / K, 4)})
            lo.free()
            q.free()
            del x, y, a, b
    launches = L.launch_count() - n0
    fl = sum(2.0 * M * K * N + 2.0 * M * r * (K + N) for _, M, K, N, r in shapes)
    tf = fl / (total["fused"] * 1e-3) / 1e12
    clocks = clk.summary()
    pk = tensor_peak_for(total["fused"] * 1e-3)
    tpeak, tpeak_kind = pk["peak"], pk["kind"]
    line = {
        "metric": "adapted w8g64 qlinear TFLOP/s (linear + rank-r adapter), reference LoRA shapes",
        "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total["fused"], 4), "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic N(0,1) x, N(0,0.02) w8g64 weights, adapter pairs "
                                 "scaled like the reference test's",
        "config": {"workload": "qlinear + LoRA at tests/ltx25-lora-apply-test.cc:498-510 shapes"},
        "per_shape": rows, "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": tpeak,
                     "peak_source": tpeak_kind, "unit": "TFLOP/s", "frac": round(tf / tpeak, 3),
                     "traffic": None},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    ctx.close()
    return 0


def run_trunk(args):
    """The trunk around the block loop at BASELINE config 4's geometry: video
    patchify (8160 tokens, 128 latent channels -> 4096, channel-major input,
    the keyframe embedding on the first frame's 510 tokens) and output head
    (LayerNorm, modulation, 4096 -> 128, channel-major out), and the audio
    pair (126 tokens, 128 <-> 2048).  HBM-bound: the algorithmic bytes are
    the activations in and out plus the packed weights."""
    import torch
    import ltx25_b200 as L
    world, rank_, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = L.Context(local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(17)
    z, oc = 128, 128
    legs = []
    nbytes = 0.0
    for T, dim, first in ((8160, 4096, 17 * 30), (126, 2048, 0)):
        wi = torch.randn((dim, z), generator=gen, device=dev) * 0.05
        wo = torch.randn((oc, dim), generator=gen, device=dev) * 0.02
        qi = L.QWeight.upload(ctx, *L.pack_w8g64(ctx, wi), dim, z, on_device=True)
        qo = L.QWeight.upload(ctx, *L.pack_w8g64(ctx, wo), oc, dim, on_device=True)
        lat = torch.randn((z, T), generator=gen, device=dev).to(torch.bfloat16)
        pre = torch.randn((dim,), generator=gen, device=dev).to(torch.bfloat16)
        bi = torch.zeros((dim,), device=dev, dtype=torch.bfloat16)
        bo = torch.zeros((oc,), device=dev, dtype=torch.bfloat16)
        ss = (torch.randn((2, dim), generator=gen, device=dev) * 0.2).float().contiguous()
        x = torch.empty((T, dim), device=dev, dtype=torch.bfloat16)
        out = torch.empty((oc, T), device=dev, dtype=torch.bfloat16)
        legs.append(lambda qi=qi, qo=qo, lat=lat, pre=pre, bi=bi, bo=bo, ss=ss, x=x, out=out,
                    first=first: (L.patchify(ctx, qi, lat, bias=bi, channel_major=True,
                                             prefix=pre, prefix_rows=first, out=x),
                                  L.output_head(ctx, qo, x, ss, bias=bo, channel_major=True,
                                                out=out)))
        nbytes += 2.0 * T * z + 2.0 * T * dim + dim * z * (1 + 4 / 64)      # patchify
        nbytes += 2.0 * T * dim + 2.0 * T * oc + oc * dim * (1 + 4 / 64)     # head
    step = lambda: [f() for f in legs]
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    ctx.check()
    gpu_id = os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local] \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else str(local)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    n0 = L.launch_count()
    with ClockSampler(gpu_id) as clk:
        for e0, e1 in evs:
            e0.record()
            step()
            e1.record()
        torch.cuda.synchronize()
    launches = (L.launch_count() - n0) // max(args.steps, 1)
    ms = statistics.median([e0.elapsed_time(e1) for e0, e1 in evs])
    _, hbm_peak, peak_kind = peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    line = {
        "metric": "DiT trunk (patchify + output head, video and audio) GB/s of activations",
        "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4), "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic N(0,1) latents, w8g64 weights",
        "config": {"workload": "patchify 8160x128->4096 (+keyframe rows) and head "
                               "8160x4096->128, audio 126x128<->2048; channel-major ends"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": round(gbs / hbm_peak, 3),
                     "traffic": None},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    ctx.close()
    return 0


def run_i8(args):
    """BASELINE config 3, the i8_gemm tier: per-token symmetric int8
    quantization of X [8160][4096] (N(0,1), 0.1 % of entries x20) and the
    kind::i8 tcgen05 GEMM against W [16384][4096] (w8g64 from N(0, 0.02),
    requantized per output channel once, in the warm-up), int32 accumulate,
    rescaled to bf16.  A step is one ltx_qlinear call with the tier on: the
    activation quantization kernel plus the GEMM.  The working set (X 67 MB,
    int8 W 67 MB, Y 267 MB) is above L2."""
    import torch
    import ltx25_b200 as L
    world, rank_, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = L.Context(local)
    M, K, N = 8160, 4096, 16384
    gen = torch.Generator(device=dev)
    gen.manual_seed(29)
    x = torch.randn((M, K), generator=gen, device=dev)
    x = torch.where(torch.rand((M, K), generator=gen, device=dev) < 1e-3, x * 20.0, x)
    x = x.to(torch.bfloat16)
    w32 = torch.randn((N, K), generator=gen, device=dev) * 0.02
    codes, scales, zps = L.pack_w8g64(ctx, w32)
    qw = L.QWeight.upload(ctx, codes, scales, zps, N, K, on_device=True)
    del w32
    y = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
    ctx.set_tiers(i8_gemm=True)
    if not ctx.i8_takes(M, K, N):
        raise RuntimeError("the int8 tier does not take BASELINE config 3's shape")
    run = lambda: L.qlinear(ctx, qw, x, out=y)
    for _ in range(max(args.warmup, 3)):
        run()
    torch.cuda.synchronize()
    ctx.check()
    steps = max(1, args.steps)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    gpu_id = os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local] \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else str(local)
    n0 = L.launch_count()
    with ClockSampler(gpu_id) as clk:
        for e0, e1 in evs:
            e0.record()
            run()
            e1.record()
        torch.cuda.synchronize()
    launches = (L.launch_count() - n0) // steps
    ctx.check()
    ms = statistics.median([e0.elapsed_time(e1) for e0, e1 in evs])
    ops = 2.0 * M * N * K
    tops = ops / (ms * 1e-3) / 1e12
    clocks = clk.summary()
    pk = tensor_peak_for(ms * steps * 1e-3)
    bf16_peak, bf16_kind = pk["peak"], pk["kind"]
    peak = 2.0 * bf16_peak
    line = {
        "metric": "i8_gemm tier qlinear TOP/s (BASELINE config 3)",
        "value": round(tops, 1), "unit": "TOP/s", "n_gpus": 1, "steps": steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4), "higher_is_better": True,
        "vs_baseline": None, "dtype": "int8 x int8 -> int32, bf16 out",
        "data": "synthetic N(0,1) activations with 0.1 % x20 outliers; N(0, 0.02) weights "
                "w8g64-packed on device",
        "config": {"workload": "BASELINE config 3: X [8160][4096] per-token int8, "
                               "W [16384][4096] per-channel int8; quantization + GEMM",
                   "l2": "working set 400 MB > L2"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor (int8)", "achieved": round(tops, 1),
                     "peak": round(peak, 1), "unit": "TOP/s", "frac": round(tops / peak, 3),
                     "traffic": None,
                     "peak_source": "2 x " + bf16_kind + " (assumption: dense int8 rate = "
                                    "2 x dense bf16, NVIDIA's nominal ratio)"},
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        # the C restatement of the tier (oracle/ltx_oracle.c: per-token
        # quantizer + integer GEMM) on a bounded sample: 256 tokens x 2048
        # output features, full K, all host threads
        import numpy as np
        from oracle import lib
        rows, feats = 256, 2048
        xs = x[:rows].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        cs = codes[:feats].cpu().numpy().view(np.uint32)
        ss = scales[:feats].cpu().numpy().view(np.uint16)
        zs = zps[:feats].cpu().numpy().view(np.uint16)
        deq = lib.dequant_bf16(cs, ss, zs, K)
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        xq, sx = lib.quant_rows_i8(xs, K)
        wq, sw = lib.quant_rows_i8(deq, K)
        lib.i8_gemm(xq, sx, wq, sw, None, K, threads=threads)
        t = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": round(2.0 * rows * feats * K / t / 1e12, 5),
                                "unit": "TOP/s", "cores": threads, "kind": "port",
                                "sample": f"oracle/ltx_oracle.c quantizer + integer GEMM, first "
                                          f"{rows} tokens x first {feats} output features, "
                                          f"full K",
                                "seconds": round(t, 2)}
    print(json.dumps(line), flush=True)
    ctx.set_tiers(i8_gemm=False)
    ctx.close()
    return 0


# The adaLN chains of one denoise step (Ltx25Dit::compute_adaln_step_,
# src/ltx25-dit.cc:178-236), one noise level each: (name, width, rows of the
# root linear's output).
ADALN_CHAINS = [("video", 4096, 9), ("prompt", 4096, 2), ("av_video_ss", 4096, 4),
                ("av_a2v_gate", 4096, 1), ("audio", 2048, 9), ("audio_prompt", 2048, 2),
                ("av_audio_ss", 2048, 4), ("av_v2a_gate", 2048, 1)]


def host_read_gbs(threads, nbytes=1 << 30):
    """Host memory read rate with `threads` threads: a torch CPU sum over a
    1 GiB f32 tensor (best of 3), the roofline for host streaming code."""
    import torch
    old = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        a = torch.ones(nbytes // 4, dtype=torch.float32)
        a.sum()
        best = float("inf")
        for _ in range(3):
            t0 = time.perf_counter()
            a.sum()
            best = min(best, time.perf_counter() - t0)
        return nbytes / best / 1e9
    finally:
        torch.set_num_threads(old)


def run_adaln(args):
    """The trunk's adaLN chains for one denoise step on the HOST (no GPU):
    the eight chains of ADALN_CHAINS at BASELINE config 4's widths (video 4096,
    audio 2048), each sinusoid -> linear_1 -> SiLU -> linear_2 -> SiLU ->
    linear as f64-sum GEMVs over bf16 weights, split over the host's threads.
    Host-memory-bound: the algorithmic bytes are the bf16 weights (~851 MB a
    step)."""
    import numpy as np
    import ltx25_b200 as L
    rng = np.random.default_rng(23)

    def bits(*shape, sc):
        a = (rng.standard_normal(shape, dtype=np.float32) * np.float32(sc))
        return (a.view(np.uint32) >> 16).astype(np.uint16)

    chains, nbytes, video_w = [], 0, None
    for name, dim, rows in ADALN_CHAINS:
        w = (bits(dim, 256, sc=0.05), bits(dim, sc=0.01), bits(dim, dim, sc=0.02),
             bits(dim, sc=0.01), bits(rows * dim, dim, sc=0.02), bits(rows * dim, sc=0.01))
        chains.append(L.AdaLN(*w))
        nbytes += 2 * (w[0].size + w[1].size + w[2].size + w[3].size + w[4].size + w[5].size)
        if name == "video":
            video_w = w
    threads = os.cpu_count() or 1
    sigma = 0.725
    tsteps = [sigma * 1000.0] * len(chains)
    # the step's chains at once (ltx_adaln_run_many), and one after another
    # (ltx_adaln_run per chain, the reference's order) for comparison
    step = lambda: L.adaln_run_many(chains, tsteps, threads=threads)
    one_by_one = lambda: [c(t, threads=threads) for c, t in zip(chains, tsteps)]
    for _ in range(max(args.warmup, 3)):
        step()
        one_by_one()
    steps = max(1, min(args.steps, 50))
    ts, ts1 = [], []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        one_by_one()
        ts1.append(time.perf_counter() - t0)
    sec = statistics.median(ts)
    sec1 = statistics.median(ts1)
    gbs = nbytes / sec / 1e9
    peak = host_read_gbs(threads)
    line = {
        "metric": "host adaLN chains of one denoise step, GB/s of bf16 weights",
        "value": round(gbs, 2), "unit": "GB/s", "n_gpus": 0, "steps": steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(sec * 1e3, 3),
        "higher_is_better": True, "dtype": "bf16 weights, f64 sums",
        "data": "synthetic N(0, 0.02) bf16 weights",
        "config": {"workload": "8 adaLN chains (video / audio timestep 9 rows, prompt 2, "
                               "a2v / v2a scale-shift 4, gates 1; widths 4096 / 2048), "
                               "one noise level each; host code, no GPU",
                   "threads": threads, "weight_bytes": int(nbytes),
                   "api": "ltx_adaln_run_many (rows over all of the step's chains split over the threads)",
                   "one_chain_at_a_time_ms": round(sec1 * 1e3, 3)},
        "gpu_launches": 0,
        "roofline": {"bound": "host memory", "achieved": round(gbs, 2), "peak": round(peak, 2),
                     "unit": "GB/s", "frac": round(gbs / peak, 3), "traffic": None,
                     "peak_source": f"measured here: torch CPU sum over 1 GiB, {threads} threads"},
    }
    if not args.no_cpu_baseline:
        # the numpy restatement of the chain (the port), video chain only
        from oracle import adaln_np
        t0 = time.perf_counter()
        adaln_np.chain(sigma * 1000.0, *video_w)
        t = time.perf_counter() - t0
        vb = 2 * sum(a.size for a in video_w)
        line["cpu_baseline"] = {"value": round(vb / t / 1e9, 3), "unit": "GB/s", "cores": threads,
                                "kind": "port",
                                "sample": "oracle/adaln_np.chain on the video chain (one run)"}
    print(json.dumps(line), flush=True)
    for c in chains:
        c.close()
    return 0


def run_connector(args):
    """The video embeddings connector at the model's geometry: 8 blocks of
    32 x 128 heads over 256 caption tokens (100 real, the rest registers),
    w8g64 linears; tensor-bound GEMMs on a short sequence."""
    import torch
    import ltx25_b200 as L
    from ltx25_b200.synth import connector_tensors
    world, rank_, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = L.Context(local)
    heads, hd, layers, regs, T, nv = 32, 128, 8, 128, 256, 100
    dim = heads * hd
    c = L.Connector(ctx, heads, hd, layers, regs)
    c.load(connector_tensors(dim, heads, layers, regs, seed=3, device=dev), want_deq=False)
    c.finalize()
    c.reserve(T)
    x = (torch.randn((T, dim), device=dev)).to(torch.bfloat16)
    out = torch.empty_like(x)
    for _ in range(max(args.warmup, 3)):
        c.forward(x, nv, out=out)
    torch.cuda.synchronize()
    ctx.check()
    gpu_id = os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local] \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else str(local)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    n0 = L.launch_count()
    with ClockSampler(gpu_id) as clk:
        for e0, e1 in evs:
            e0.record()
            c.forward(x, nv, out=out)
            e1.record()
        torch.cuda.synchronize()
    launches = (L.launch_count() - n0) // max(args.steps, 1)
    ms = statistics.median([e0.elapsed_time(e1) for e0, e1 in evs])
    fl = layers * (2.0 * T * dim * dim * 4 + 2.0 * T * dim * 4 * dim * 2 +
                   4.0 * T * T * dim + 2.0 * T * dim * heads)
    tf = fl / (ms * 1e-3) / 1e12
    peak_tf, _, peak_kind = peaks()
    line = {
        "metric": "video embeddings connector TFLOP/s (8 blocks, 256 tokens, 4096 wide)",
        "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4), "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic N(0,1) captions, random w8g64 weights",
        "config": {"workload": "connector 8 x (attn 32x128, ff 4x), 256 tokens, 100 valid"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak_tf,
                     "peak_kind": peak_kind, "unit": "TFLOP/s", "frac": round(tf / peak_tf, 3),
                     "traffic": None},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    c.close()
    ctx.close()
    return 0


# ------------------------------------------------------ reference CPU block
# The reference's own block_forward (src/ltx25-block-ref.cc:308-389, compiled
# into oracle/_ref) on a bounded sample at the real widths: one random-init
# block (video 4096 x 32 heads, audio 2048 x 32 heads), 8 video tokens (a
# 2x2x2 grid), 4 audio, 8 text.  Its rate in algorithmic FLOP/s extrapolates
# to the full geometry by FLOPs.
REF_SAMPLE = {"vt": 8, "grid": (2, 2, 2), "at": 4, "tt": 8}
_REF_BLOCK = {}


def ref_block_setup():
    if _REF_BLOCK:
        return _REF_BLOCK
    from oracle import block_np
    from oracle import ref as oref
    t0 = time.perf_counter()
    kind = "reference" if oref.available() else "port"
    tensors = block_np.random_block_tensors(4096, 32, 2048, 32, seed=3, f32_draws=True)
    cfg = dict(vdim=4096, vheads=32, adim=2048, aheads=32, vt=REF_SAMPLE["vt"],
               at=REF_SAMPLE["at"], tt=REF_SAMPLE["tt"])
    inp = block_np.random_block_inputs(cfg, seed=4, video_grid=REF_SAMPLE["grid"])
    if kind == "reference":
        blk = oref.RefBlock(tensors, 4096, 32, 2048, 32)
        del tensors

        def fwd():
            blk.forward(inp["video"], inp["audio"])
        _REF_BLOCK["blk"] = blk
    else:
        def fwd():
            block_np.block_forward(tensors, inp["video"], inp["audio"], 4096, 32, 2048, 32)
    g, a = block_flops(REF_SAMPLE["vt"], REF_SAMPLE["at"], REF_SAMPLE["tt"], 4096, 2048)
    _REF_BLOCK.update(fwd=fwd, kind=kind, sample_flops=g + a,
                      setup_s=time.perf_counter() - t0)
    return _REF_BLOCK


def ref_block_round(threads):
    """`threads` concurrent block_forward calls on the sample (ctypes drops
    the GIL, so they run on as many cores).  Returns (FLOPs, seconds)."""
    import concurrent.futures as cf
    r = ref_block_setup()
    t0 = time.perf_counter()
    if threads <= 1:
        r["fwd"]()
    else:
        with cf.ThreadPoolExecutor(max_workers=threads) as ex:
            for f in [ex.submit(r["fwd"]) for _ in range(threads)]:
                f.result()
    return threads * r["sample_flops"], time.perf_counter() - t0


def ref_block_desc(threads):
    s = REF_SAMPLE
    return (f"{threads} concurrent block_forward calls (src/ltx25-block-ref.cc:308-389, "
            f"f32 with f64 dot products) per round, each one random-init block at the real "
            f"widths (video 4096x32 heads, audio 2048x32) on {s['vt']} video tokens "
            f"({s['grid'][0]}x{s['grid'][1]}x{s['grid'][2]}), {s['at']} audio, {s['tt']} "
            f"text; extrapolated to 8160/126/256 tokens by algorithmic FLOPs")


def full_block_flops():
    g, a = block_flops(8160, 126, 256, 4096, 2048)
    return g + a


def ref_block_baseline(blocks, rounds=2):
    """cpu_baseline of the block and stack lines: the reference block on all
    host cores, one warm-up round then `rounds` timed; returns the dict."""
    threads = os.cpu_count() or 1
    ref_block_round(threads)
    fl = sec = 0.0
    for _ in range(rounds):
        f, t = ref_block_round(threads)
        fl += f
        sec += t
    rate = fl / sec
    per_block = full_block_flops() / rate
    r = _REF_BLOCK
    return {"value": round(per_block * blocks, 2) if blocks > 1 else round(per_block * 1e3, 1),
            "unit": "s/step" if blocks > 1 else "ms", "cores": threads, "kind": r["kind"],
            "sample": ref_block_desc(threads),
            "gflops": round(rate / 1e9, 2), "seconds": round(sec, 2),
            "setup_s": round(r["setup_s"], 1)}


# ------------------------------------------------------------------ block
def run_block(args):
    """one joint AV block, 8160 video + 126 audio + 256
    text tokens at the real widths, synthetic w8g64 weights."""
    import torch
    import ltx25_b200 as L
    from ltx25_b200 import synth
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = L.Context(local)
    vdim, vh, adim, ah = 4096, 32, 2048, 32
    frames, hh, ww, at, tt = 16, 17, 30, 126, 256
    vt = frames * hh * ww
    blk = synth.load_random_block(ctx, vdim, vh, adim, ah, seed=7)
    blk.reserve(vt, at, tt)
    v_self, a_self, v_cross, a_cross = L.geometry_tables(frames, hh, ww, at, vdim, vh, adim, ah)
    dt = lambda t: (torch.from_numpy(t[0]).to(dev), torch.from_numpy(t[1]).to(dev))
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    v = synth.random_stream_inputs(vdim, vt, tt, vh, gen, pe=dt(v_self), cross_pe=dt(v_cross))
    a = synth.random_stream_inputs(adim, at, tt, ah, gen, pe=dt(a_self), cross_pe=dt(a_cross))
    x0v, x0a = v["x"].clone(), a["x"].clone()
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        blk.forward(v, a)
    torch.cuda.synchronize()
    ctx.check()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    torch.cuda.synchronize()
    n0 = L.launch_count()
    with ClockSampler(gpu_index(local)) as clk:
        for e0, e1 in evs:
            # x is reset outside the timed pair; the block's weights (0.44 GB)
            # and activations stream far above L2 every step
            v["x"].copy_(x0v)
            a["x"].copy_(x0a)
            e0.record(stream)
            blk.forward(v, a, stream=stream)
            e1.record(stream)
        torch.cuda.synchronize()
    launches = L.launch_count() - n0
    ctx.check()
    times = [e0.elapsed_time(e1) for e0, e1 in evs]
    ms = statistics.median(times)
    region_s = sum(times) * 1e-3

    # end to end through the public API: host x in, host x out, every step
    hv, ha = x0v.cpu().pin_memory(), x0a.cpu().pin_memory()
    ov, oa = torch.empty_like(hv).pin_memory(), torch.empty_like(ha).pin_memory()
    e2e_steps = max(1, min(args.steps, 20))
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(e2e_steps):
        v["x"].copy_(hv, non_blocking=True)
        a["x"].copy_(ha, non_blocking=True)
        blk.forward(v, a, stream=stream)
        ov.copy_(v["x"], non_blocking=True)
        oa.copy_(a["x"], non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1) / e2e_steps
    ctx.check()
    io_bytes = (vt * vdim + at * adim) * 2

    gemm_flops, attn_flops = block_flops(vt, at, tt, vdim, adim)
    achieved = (gemm_flops + attn_flops) / (ms * 1e-3) / 1e12
    clocks = clk.summary()
    pk = tensor_peak_for(region_s)
    line = {
        "metric": "DiT joint AV block forward ms @960x544x121 (BASELINE config 4)",
        "value": round(ms, 3), "unit": "ms", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False,
        "scaling": "none", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded device-generated weights, w8g64)",
        "config": {"workload": "one block: video 8160x4096 (16x17x30), audio 126x2048, "
                               "text 256, 3-axis video RoPE, 1-D audio RoPE",
                   "l2": "weights 0.44 GB and activations above L2 every step"},
        "e2e": {"value": round(e2e_ms, 3), "unit": "ms", "h2d_bytes_per_step": io_bytes,
                "d2h_bytes_per_step": io_bytes,
                "api": "ltx_block_forward, x copied in from and out to pinned host memory"},
        "gpu_launches": int(launches),
        "algorithmic_tflop": round((gemm_flops + attn_flops) / 1e12, 3),
        "gemm_tflop": round(gemm_flops / 1e12, 3), "attention_tflop": round(attn_flops / 1e12, 3),
        "roofline": dict({"bound": "tensor", "achieved": round(achieved, 1),
                          "peak": pk["peak"], "peak_source": pk["kind"], "unit": "TFLOP/s",
                          "frac": round(achieved / pk["peak"], 4), "traffic": None},
                         **roofline_fracs(achieved, pk, clocks)),
        "clocks": clocks,
    }
    blk.close()
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = ref_block_baseline(blocks=1)
    print(json.dumps(line), flush=True)
    ctx.close()
    return 0


# ------------------------------------------------------------------ sweep
def measure_sweep(args, ctx, dev, rank, world, pg, local):
    """BASELINE config 2 on one context: every shape of SHAPES through
    ltx_qlinear, K timed steps (inputs resident), then the end-to-end leg
    through host buffers.  Returns the sweep's figures as a dict."""
    import torch
    import ltx25_b200 as L
    route = {"auto": L.ROUTE_AUTO, "fused": L.ROUTE_FUSED,
             "dequant": L.ROUTE_DEQUANT_ONCE}[args.route]
    ctx.set_route(route)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    weights, xs, ys = [], [], []
    for _, M, K, N in SHAPES:
        weights.append(make_weights(L, ctx, torch, dev, K, N, gen))
        xs.append(torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16))
        ys.append(torch.empty((M, N), device=dev, dtype=torch.bfloat16))
    ctx.reserve(max(s[1] for s in SHAPES), max(s[3] for s in SHAPES),
                max(s[2] for s in SHAPES))
    stream = torch.cuda.current_stream()
    ctx.check()

    def step(evs=None):
        for i, (w, x, y) in enumerate(zip(weights, xs, ys)):
            if evs is not None:
                evs[i][0].record(stream)
            L.qlinear(ctx, w, x, out=y, stream=stream)
            if evs is not None:
                evs[i][1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.check()

    evs = [[[torch.cuda.Event(enable_timing=True),
             torch.cuda.Event(enable_timing=True)] for _ in SHAPES]
           for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    n_launch0 = L.launch_count()
    with ClockSampler(gpu_index(local)) as clk:
        t_start.record(stream)
        for s in range(args.steps):
            step(evs[s])
        t_end.record(stream)
        torch.cuda.synchronize()
    launches = L.launch_count() - n_launch0
    if pg is not None:
        pg.barrier()
    ctx.check()
    ms_total = t_start.elapsed_time(t_end)
    per_shape_ms = [0.0] * len(SHAPES)
    for s in range(args.steps):
        for i in range(len(SHAPES)):
            per_shape_ms[i] += evs[s][i][0].elapsed_time(evs[s][i][1])
    if pg is not None:
        t = torch.tensor([ms_total], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms_total = float(t.item())
    step_flops = sum(flops(M, K, N) for _, M, K, N in SHAPES)
    ms_per_step = ms_total / args.steps
    value = world * step_flops / (ms_per_step * 1e-3) / 1e12

    # end to end: each step uploads every shape's input and downloads every
    # result; the uploads run on one copy stream and the downloads on
    # another, each shape's GEMM waits only for its own input, and the device
    # buffers are double-buffered across steps, so PCIe in, PCIe out and the
    # GEMMs overlap (a serving loop's pipelining) while every byte still
    # crosses per step.
    xh = [torch.empty(x.shape, dtype=x.dtype, pin_memory=True) for x in xs]
    yh = [torch.empty(y.shape, dtype=y.dtype, pin_memory=True) for y in ys]
    for a, b in zip(xh, xs):
        a.copy_(b)
    h2d = sum(x.numel() * 2 for x in xs)
    d2h = sum(y.numel() * 2 for y in ys)
    copy_in = torch.cuda.Stream(dev)
    copy_out = torch.cuda.Stream(dev)
    xs2 = [xs, [torch.empty_like(x) for x in xs]]
    ys2 = [ys, [torch.empty_like(y) for y in ys]]
    ev = {kind: [[torch.cuda.Event() for _ in SHAPES] for _ in range(2)]
          for kind in ("in", "done", "out")}
    nstep = {"k": 0}

    def e2e_step():
        k = nstep["k"]
        nstep["k"] += 1
        bs = k % 2
        for i, (w, a, b) in enumerate(zip(weights, xh, yh)):
            x, y = xs2[bs][i], ys2[bs][i]
            if k >= 2:
                copy_in.wait_event(ev["done"][bs][i])      # x free
            with torch.cuda.stream(copy_in):
                x.copy_(a, non_blocking=True)
            ev["in"][bs][i].record(copy_in)
            stream.wait_event(ev["in"][bs][i])
            if k >= 2:
                stream.wait_event(ev["out"][bs][i])        # y free
            L.qlinear(ctx, w, x, out=y, stream=stream)
            ev["done"][bs][i].record(stream)
            copy_out.wait_event(ev["done"][bs][i])
            with torch.cuda.stream(copy_out):
                b.copy_(y, non_blocking=True)
            ev["out"][bs][i].record(copy_out)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    copy_in.wait_event(e0)
    copy_out.wait_event(e0)
    for _ in range(args.e2e_steps):
        e2e_step()
    stream.wait_stream(copy_in)
    stream.wait_stream(copy_out)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
    if pg is not None:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    ctx.check()
    e2e_value = world * step_flops / (e2e_ms * 1e-3) / 1e12

    _, hbm_peak, _ = peaks()
    vid = [i for i, s in enumerate(SHAPES) if s[1] > 1024]
    aud = [i for i, s in enumerate(SHAPES) if s[1] <= 1024]
    vid_fl = sum(flops(*SHAPES[i][1:]) for i in vid) * args.steps
    vid_s = sum(per_shape_ms[i] for i in vid) * 1e-3
    aud_b = sum(hbm_bytes(*SHAPES[i][1:]) for i in aud) * args.steps
    aud_s = sum(per_shape_ms[i] for i in aud) * 1e-3
    achieved = vid_fl / vid_s / 1e12 if vid_s > 0 else 0.0
    achieved_hbm = aud_b / aud_s / 1e9 if aud_s > 0 else 0.0
    prof = traffic_from_profile() or {}
    per_shape = []
    for i, (name, M, K, N) in enumerate(SHAPES):
        t = per_shape_ms[i] / args.steps * 1e-3
        per_shape.append({"shape": name, "M": M, "K": K, "N": N,
                          "us": round(t * 1e6, 2),
                          "tflops": round(flops(M, K, N) / t / 1e12, 1),
                          "gbs": round(hbm_bytes(M, K, N) / t / 1e9, 1)})
    clocks = clk.summary()
    pk = tensor_peak_for(ms_total * 1e-3)
    out = {
        "value": round(value, 2), "unit": UNIT, "ms_per_step": round(ms_per_step, 4),
        "steps": args.steps,
        "shapes": [f"{n}: M={M} K={K} N={N}" for n, M, K, N in SHAPES],
        "route": args.route,
        "l2": "inputs larger than L2: the sweep's operands total ~1.5 GB and each shape's "
              "are evicted by the others between repeats",
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 3),
                "api": "ltx_qlinear via ctypes, pinned host buffers; uploads and downloads on "
                       "two copy streams overlapped with the GEMMs, device buffers double-"
                       "buffered across steps"},
        "gpu_launches": int(launches),
        "clocks": clocks,
        "roofline": dict({
            "bound": "tensor", "achieved": round(achieved, 1),
            "peak": pk["peak"], "unit": "TFLOP/s",
            "frac": round(achieved / pk["peak"], 4), "peak_source": pk["kind"],
            "kernel": ("dequant_w8_kernel + gemm_tc_kernel<MODE_BF16,TN=256> (route auto: "
                       "M >= %d expands the weight once per call, src/ltx25-metal-ops.cc:"
                       "468-545) over the 6 M=8160 shapes; time covers both" % L.DEQUANT_MIN_M)
                      if args.route != "fused" else
                      "gemm_tc_kernel<MODE_W8G64,TN=256> over the 6 M=8160 shapes",
            "traffic": prof.get("video_bytes_per_launch_" + args.route)},
            **roofline_fracs(achieved, pk, clocks)),
        "roofline_hbm": {
            "bound": "hbm", "achieved": round(achieved_hbm, 1),
            "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved_hbm / hbm_peak, 4),
            "kernel": "the small-M w8g64 path over the 3 M=126 shapes",
            "traffic": prof.get("audio_bytes_per_launch")},
        "per_shape": per_shape,
    }
    for w in weights:
        w.free()
    del xs, ys, xs2, ys2, xh, yh
    torch.cuda.synchronize()
    return out


def run_sweep(args):
    """BASELINE config 2 as its own line (--workload sweep): N replicas."""
    import torch
    import ltx25_b200 as L
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        pg = dist
    ctx = L.Context(local)
    sw = measure_sweep(args, ctx, dev, rank, world, pg, local)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        f, s, kind = cpu_reference_sample(1)
        cpu = {"value": f / s / 1e12, "unit": UNIT, "cores": 1, "kind": kind,
               "sample": sample_desc(), "seconds": round(s, 2)}
    line = {
        "metric": METRIC, "value": sw["value"], "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sw["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 activations; N(0,0.02) weights "
                "w8g64-packed on device, bit-identical to the reference packer)",
        "config": {"workload": "BASELINE config 2: DiT linear-shape sweep, all w8g64",
                   "shapes": sw["shapes"], "l2": sw["l2"],
                   "parallelism": f"replicas x{world} (no data-path collective)",
                   "route": args.route},
        "e2e": sw["e2e"], "gpu_launches": sw["gpu_launches"], "clocks": sw["clocks"],
        "roofline": sw["roofline"], "roofline_hbm": sw["roofline_hbm"],
        "per_shape": sw["per_shape"], "cpu_baseline": cpu,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if pg is not None:
        pg.destroy_process_group()
    return 0


# ------------------------------------------------------- config 1 qlinear
Q1 = (1024, 4096, 4096)          # M, K, N
Q1_CPU_ROWS = 512                # cpu sample: the first 512 tokens, all N, full K
L2_FLUSH_BYTES = 256 << 20       # > the 126 MB L2


def run_qlinear(args):
    """one w8g64 qlinear, X [1024][4096] ~ N(0, 1) bf16,
    W [4096][4096] ~ N(0, 0.02) packed w8g64, bias [4096] ~ N(0, 0.01), bf16
    out, through ltx_qlinear.  Its operands (34.6 MB) fit in L2, so a 256 MB
    buffer is written between timed iterations (outside each event pair) and
    every iteration starts from DRAM."""
    import torch
    import ltx25_b200 as L
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = L.Context(local)
    M, K, N = Q1
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    x = torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
    w32 = torch.randn((N, K), generator=gen, device=dev) * 0.02
    bias = (torch.randn((N,), generator=gen, device=dev) * 0.01).to(torch.bfloat16)
    codes, scales, zps = L.pack_w8g64(ctx, w32)
    qw = L.QWeight.upload(ctx, codes, scales, zps, N, K, on_device=True)
    y = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    ctx.reserve(M, N, K)
    for _ in range(args.warmup):
        flush.zero_()
        L.qlinear(ctx, qw, x, bias=bias, out=y, stream=stream)
    torch.cuda.synchronize()
    ctx.check()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    n0 = L.launch_count()
    with ClockSampler(gpu_index(local)) as clk:
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            L.qlinear(ctx, qw, x, bias=bias, out=y, stream=stream)
            e1.record(stream)
        torch.cuda.synchronize()
    launches = L.launch_count() - n0
    ctx.check()
    times = [e0.elapsed_time(e1) for e0, e1 in evs]
    ms = sum(times) / len(times)
    fl = flops(M, K, N)
    byts = N * K + 4.0 * N * K / 64 + 2.0 * M * K + 2.0 * M * N + 2.0 * N
    tf = fl / (ms * 1e-3) / 1e12

    # end to end: x from pinned host memory in, y out, every step
    xh = x.cpu().pin_memory()
    yh = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    e2e = []
    for _ in range(args.steps):
        flush.zero_()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        x.copy_(xh, non_blocking=True)
        L.qlinear(ctx, qw, x, bias=bias, out=y, stream=stream)
        yh.copy_(y, non_blocking=True)
        f1.record(stream)
        e2e.append((f0, f1))
    torch.cuda.synchronize()
    ctx.check()
    e2e_ms = sum(a.elapsed_time(b) for a, b in e2e) / len(e2e)
    clocks = clk.summary()
    pk = tensor_peak_for(sum(times) * 1e-3)
    _, hbm_peak, _ = peaks()
    line = {
        "metric": "w8g64 qlinear TFLOP/s (BASELINE config 1)",
        "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic N(0,1) bf16 x, N(0,0.02) w8g64 weights, N(0,0.01) bias, seed 7",
        "config": {"workload": "BASELINE config 1: qlinear 1024x4096 -> 4096 with bias",
                   "l2": "operands 34.6 MB fit in L2: a 256 MB buffer is written between "
                         "timed iterations, outside the event pairs"},
        "e2e": {"value": round(fl / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
                "ms_per_step": round(e2e_ms, 4),
                "api": "ltx_qlinear, x in from and y out to pinned host memory"},
        "gpu_launches": int(launches),
        "roofline": dict({"bound": "tensor", "achieved": round(tf, 1), "peak": pk["peak"],
                          "peak_source": pk["kind"], "unit": "TFLOP/s",
                          "frac": round(tf / pk["peak"], 4), "traffic": None,
                          "kernel": "gemm_tc_kernel<MODE_W8G64> (fused route below "
                                    "LTX_DEQUANT_MIN_M rows)"},
                         **roofline_fracs(tf, pk, clocks)),
        "hbm": {"algorithmic_bytes": int(byts), "gbs": round(byts / (ms * 1e-3) / 1e9, 1),
                "frac": round(byts / (ms * 1e-3) / 1e9 / hbm_peak, 4)},
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        f, s, kind = ref_linear_sample(1)
        line["cpu_baseline"] = {"value": round(f / s / 1e12, 6), "unit": "TFLOP/s", "cores": 1,
                                "kind": kind, "sample": q1_sample_desc(), "seconds": round(s, 2)}
    print(json.dumps(line), flush=True)
    qw.free()
    ctx.close()
    return 0


_Q1_CPU = {}


def ref_linear_sample(threads):
    """The reference's CPU qlinear for config 1 (dequantise-then-dense,
    linear_ with f64 accumulation, src/ltx25-block-ref.cc:13-29) on the first
    Q1_CPU_ROWS tokens, all N, full K; the weight is packed and dequantized
    once, outside the timing.  Rows are split over `threads`.  Returns
    (FLOPs, seconds, kind)."""
    import concurrent.futures as cf
    import numpy as np
    from oracle import lib as olib
    from oracle import ref as oref
    if not _Q1_CPU:
        M, K, N = Q1
        kind = "reference" if oref.available() else "port"
        rng = np.random.default_rng(7)
        x = olib.bf16_to_f32(olib.f32_to_bf16(
            rng.standard_normal((Q1_CPU_ROWS, K)).astype(np.float32)))
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        b = olib.bf16_to_f32(olib.f32_to_bf16((rng.standard_normal(N) * 0.01).astype(np.float32)))
        _, _, _, deq = oref.pack(w, 8, 64) if kind == "reference" else olib.pack_affine(w, 8, 64)
        if kind != "reference":
            deq = olib.bf16_to_f32(deq) if deq.dtype == np.uint16 else deq
        _Q1_CPU.update(x=x, w=deq, b=b, kind=kind)
    c = _Q1_CPU
    lin = oref.linear if c["kind"] == "reference" else (
        lambda x, w, b: olib.linear_f64(x, w, b, 1))
    rows = c["x"].shape[0]
    t0 = time.perf_counter()
    if threads <= 1:
        lin(c["x"], c["w"], c["b"])
    else:
        step = max(1, (rows + threads - 1) // threads)
        with cf.ThreadPoolExecutor(max_workers=threads) as ex:
            for f in [ex.submit(lin, c["x"][r:r + step], c["w"], c["b"])
                      for r in range(0, rows, step)]:
                f.result()
    return flops(rows, Q1[1], Q1[2]), time.perf_counter() - t0, c["kind"]


def q1_sample_desc():
    return (f"reference linear_ (dequantise-then-dense, f64 accumulation) on the first "
            f"{Q1_CPU_ROWS} of 1024 tokens x all 4096 output features, full K, bias; weight "
            f"packed and dequantized once outside the timing")


# ------------------------------------------------- dense GEMM against cuBLAS
def run_cublas_ab(args):
    """The dense tcgen05 GEMM (gemm_tc_kernel<MODE_BF16>, the expand-once
    route's second half) against cuBLAS (torch.matmul, a library GEMM) on
    the six M=8160 sweep shapes with the same bf16 operands, arms
    interleaved step by step so clocks and power fall on both alike: how
    close the hand-written dense GEMM comes to the library one."""
    import numpy as np
    import torch
    import ltx25_b200 as L
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    ctx = L.Context(0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    rows = []
    tot = {"ours": 0.0, "cublas": 0.0}
    fl_all = 0.0
    n0 = L.launch_count()
    with ClockSampler(gpu_index(0)) as clk:
        for name, M, K, N in SHAPES:
            if M <= 1024:
                continue
            x = torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
            w = (torch.randn((N, K), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
            qw = L.QWeight.upload_dense(ctx, w.view(torch.int16).cpu().numpy().view(np.uint16),
                                        N, K)
            y = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
            arms = {"ours": lambda: L.qlinear(ctx, qw, x, out=y),
                    "cublas": lambda: torch.matmul(x, w.t(), out=y)}
            for _ in range(args.warmup):
                for f in arms.values():
                    f()
            evs = {a: [] for a in arms}
            for i in range(args.steps):
                for a in (list(arms) if i % 2 == 0 else list(arms)[::-1]):
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    arms[a]()
                    e1.record()
                    evs[a].append((e0, e1))
            torch.cuda.synchronize()
            ctx.check()
            fl = flops(M, K, N)
            row = {"shape": name, "M": M, "K": K, "N": N}
            for a in arms:
                ms = statistics.median([e0.elapsed_time(e1) for e0, e1 in evs[a]])
                tot[a] += ms * args.steps
                row[a + "_tflops"] = round(fl / (ms * 1e-3) / 1e12, 1)
            row["ratio"] = round(row["ours_tflops"] / row["cublas_tflops"], 3)
            fl_all += fl * args.steps
            rows.append(row)
            qw.free()
            del x, w, y
    launches = L.launch_count() - n0
    ours = fl_all / (tot["ours"] * 1e-3) / 1e12
    cub = fl_all / (tot["cublas"] * 1e-3) / 1e12
    pk = tensor_peak_for(tot["ours"] * 1e-3 / 2)
    line = {
        "metric": "dense bf16 tcgen05 GEMM vs cuBLAS, six M=8160 sweep shapes",
        "value": round(ours, 1), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic N(0,1) x, N(0,0.02) bf16 weights",
        "config": {"workload": "gemm_tc_kernel<MODE_BF16> vs torch.matmul, arms interleaved"},
        "cublas_tflops": round(cub, 1), "ratio_to_cublas": round(ours / cub, 3),
        "per_shape": rows, "gpu_launches": int(launches),
        "roofline": dict({"bound": "tensor", "achieved": round(ours, 1), "peak": pk["peak"],
                          "peak_source": pk["kind"], "unit": "TFLOP/s",
                          "frac": round(ours / pk["peak"], 4), "traffic": None},
                         **roofline_fracs(ours, pk, clk.summary())),
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    ctx.close()
    return 0


# --------------------------------------------------------- GEMM phase trace
TRACE_NAMES = ["entry", "setup", "first_tma", "last_tma", "first_full_deq", "first_mma",
               "last_commit", "first_acc", "epi_done", "reduced", "end"]


def run_gemm_trace(args):
    """The w8g64 GEMM's own phase trace (ltx_ctx_set_trace: clock64 stamps
    and per-role wait counters of every CTA) on the three audio shapes of
    the sweep, one uncontended long-K shape, and the video FFN-up shape on
    the fused route (single CTAs and CTA pairs).  Prints per-CTA medians:
    phase stamps from entry, and per-k-block cycles of the MMA issuer's span
    and of each role's waits.  L2 flushed before every traced call: where
    the small-M and fused kernels spend their cycles."""
    import numpy as np
    import torch
    import ltx25_b200 as L
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    ctx = L.Context(0)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(13)
    small, big = 128 * 128 + 128 * 64 + 512, 256 * 128 + 128 * 64 + 512   # bytes a k-block stages
    cases = [("audio 2048->2048", 126, 2048, 2048, None, small),
             ("audio FFN-up", 126, 2048, 8192, None, small),
             ("audio FFN-down", 126, 8192, 2048, None, small),
             ("uncontended K=65536", 126, 65536, 128, None, small),
             ("video FFN-up fused", 8160, 4096, 16384, 0, big),
             ("video FFN-up fused pair", 8160, 4096, 16384, 1, small)]   # a pair CTA: half the tokens
    out = []
    for name, M, K, N, pair, stage_bytes in cases:
        w32 = torch.randn((N, K), generator=gen, device=dev) * 0.02
        c, sc, zp = L.pack_w8g64(ctx, w32)
        del w32
        qw = L.QWeight.upload(ctx, c, sc, zp, N, K, on_device=True)
        x = torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
        y = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
        if pair is not None:
            ctx.set_route(L.ROUTE_FUSED)
            ctx.set_tile_plan(pair=pair)
        for _ in range(3):
            L.qlinear(ctx, qw, x, out=y)
        ts = []
        for _ in range(5):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            L.qlinear(ctx, qw, x, out=y)
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        tr = torch.zeros((148, 24), dtype=torch.int64, device=dev)
        flush.zero_()
        torch.cuda.synchronize()
        ctx.set_trace(tr, 148)
        L.qlinear(ctx, qw, x, out=y)
        torch.cuda.synchronize()
        ctx.set_trace(None, 0)
        ctx.set_tile_plan()
        ctx.set_route(L.ROUTE_AUTO)
        ctx.check()
        t = tr.cpu().numpy().astype(np.int64)
        t = t[t[:, 0] != 0]
        rel = t[:, :11] - t[:, 0:1]
        tiles = float(np.median(t[:, 11]))
        kbs = float(np.median(t[:, 21])) * 2       # the traced dequant group takes every other
        span = float(np.median(rel[:, 6] - rel[:, 5]))
        per = lambda col, n: round(float(np.median(t[:, col])) / max(n, 1), 1)
        out.append({
            "case": name, "M": M, "K": K, "N": N, "us": round(min(ts) * 1e3, 2),
            "ctas": int(len(t)), "tiles_per_cta": tiles, "kblocks_per_cta": kbs,
            "phase_cycles": {n: int(np.median(rel[:, i])) for i, n in enumerate(TRACE_NAMES)},
            "mma_span_cycles_per_kblock": round(span / max(kbs, 1), 1),
            "stage_bytes_per_clk": round(stage_bytes * max(kbs, 1) / max(span, 1), 1),
            "mma_wait_full_per_kblock": per(12, kbs), "mma_wait_a_per_kblock": per(13, kbs),
            "mma_wait_acc_per_tile": per(14, tiles), "producer_wait_empty_per_kblock": per(15, kbs),
            "dequant_per_block": {"wait_full": per(16, kbs / 2), "load": per(17, kbs / 2),
                                  "math": per(18, kbs / 2), "store": per(19, kbs / 2),
                                  "wait_aempty": per(20, kbs / 2)},
        })
        qw.free()
        del x, y
    print(json.dumps({"metric": "w8g64 GEMM phase trace (cycles, per-CTA medians)",
                      "value": None, "unit": "cycles", "cases": out}), flush=True)
    ctx.close()
    return 0


# ------------------------------------------------------------- reference arm
def run_reference(args):
    """--impl reference: the reference's own CPU implementation of the path
    (oracle/_ref, compiled from the reference sources; the reference's GPU
    path is Apple Metal, unavailable on this box) on the host cores, for the
    same metric and config as the matching --workload.  Rank 0 only."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    wl = args.workload
    if wl in ("stack", "block"):
        ref_block_setup()
        for _ in range(args.warmup):
            ref_block_round(threads)
        fl = sec = 0.0
        for _ in range(args.steps):
            f, s = ref_block_round(threads)
            fl += f
            sec += s
        rate = fl / sec
        per_block = full_block_flops() / rate
        kind = _REF_BLOCK["kind"]
        if wl == "stack":
            value, unit = per_block * args.blocks, "s/step"
            metric = "DiT s/denoise-step @960x544x121 (BASELINE config 5, 48-block stack)"
            cfg = {"workload": f"{args.blocks}-block joint AV stack: video 8160x4096 "
                               "(16x17x30), audio 126x2048, text 256; extrapolated from a "
                               "bounded sample",
                   "parallelism": f"{args.parallel}{args.gpus} (the CPU arm runs on rank 0's "
                                  "host cores)"}
        else:
            value, unit = per_block * 1e3, "ms"
            metric = "DiT joint AV block forward ms @960x544x121 (BASELINE config 4)"
            cfg = {"workload": "one block: video 8160x4096 (16x17x30), audio 126x2048, text "
                               "256; extrapolated from a bounded sample"}
        desc = ref_block_desc(threads)
        line = {"impl": "reference", "metric": metric, "value": round(value, 3), "unit": unit,
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(sec / args.steps * 1e3, 1), "higher_is_better": False,
                "scaling": "strong" if wl == "stack" else "none", "vs_baseline": None,
                "dtype": "f32/f64-accumulate", "data": "synthetic (seeded random-init block)",
                "config": dict(cfg, sample=desc),
                "cpu_baseline": {"value": round(value, 3), "unit": unit, "cores": threads,
                                 "kind": kind, "sample": desc,
                                 "gflops": round(rate / 1e9, 2)},
                "e2e": {"value": round(value, 3), "unit": unit, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0},
                "note": "the reference's GPU path is Apple Metal (unavailable on this box); "
                        "this arm is its CPU block_forward on all host cores, each step one "
                        "round of concurrent calls, extrapolated to the full geometry by "
                        "algorithmic FLOPs"}
        print(json.dumps(line), flush=True)
        return 0
    if wl == "qlinear":
        for _ in range(args.warmup):
            ref_linear_sample(threads)
        fl = sec = 0.0
        kind = "port"
        for _ in range(args.steps):
            f, s, kind = ref_linear_sample(threads)
            fl += f
            sec += s
        value = fl / sec / 1e12
        line = {"impl": "reference", "metric": "w8g64 qlinear TFLOP/s (BASELINE config 1)",
                "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": sec / args.steps * 1e3,
                "higher_is_better": True, "scaling": "none", "vs_baseline": None,
                "dtype": "f32/f64-accumulate", "data": "synthetic, seed 7",
                "config": {"workload": "BASELINE config 1, bounded CPU sample",
                           "sample": q1_sample_desc()},
                "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads,
                                 "kind": kind, "sample": q1_sample_desc()},
                "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    if wl == "sweep":
        for _ in range(args.warmup):
            cpu_reference_sample(threads)
        fl = sec = 0.0
        kind = "port"
        for _ in range(args.steps):
            f, s, kind = cpu_reference_sample(threads)
            fl += f
            sec += s
        value = fl / sec / 1e12
        line = {
            "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": sec / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32/f64-accumulate",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights)",
            "config": {"workload": "BASELINE config 2 sweep, bounded CPU sample",
                       "sample": sample_desc()},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads,
                             "kind": kind, "sample": sample_desc()},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "the reference's GPU path is Apple Metal (unavailable on this "
                    "box); this arm is its CPU dequantise-then-dense qlinear",
        }
        print(json.dumps(line), flush=True)
        return 0
    print(json.dumps({"impl": "reference",
                      "unavailable": f"no reference CPU arm for --workload {wl}: the reference "
                                     "implements it only in Metal"}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 10 for stack, 200 otherwise)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true",
                    help="stack: skip the config-2 sweep carried on the line")
    ap.add_argument("--only", type=int, default=None,
                    help="profile one sweep shape (index into SHAPES)")
    ap.add_argument("--blocks", type=int, default=48, help="stack depth (--workload stack)")
    ap.add_argument("--parallel", default="tp", choices=["tp", "sp"],
                    help="stack under torchrun: tensor parallel (BASELINE config 5) or "
                         "sequence/head parallel")
    ap.add_argument("--sage", action="store_true", help="sage_attn tier (--workload attn)")
    ap.add_argument("--route", default="auto", choices=["auto", "fused", "dequant"],
                    help="qlinear route for quantized weights (sweep)")
    ap.add_argument("--workload", default="stack",
                    choices=["stack", "sweep", "qlinear", "block", "attn", "lora", "trunk",
                             "connector", "adaln", "i8", "cublas_ab", "gemm_trace"],
                    help="stack: BASELINE config 5, the 48-block denoise step (the "
                         "headline, carrying the config-2 sweep); sweep: config 2 alone; "
                         "qlinear: config 1; i8: config 3; block: config 4")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 10 if args.workload == "stack" else 200
    args.warmup = max(args.warmup, 3)
    if args.only is not None:
        SHAPES[:] = [SHAPES[args.only]]
    if args.impl == "reference":
        return run_reference(args)
    runs = {"stack": run_stack, "sweep": run_sweep, "qlinear": run_qlinear,
            "block": run_block, "attn": run_attn, "lora": run_lora, "trunk": run_trunk,
            "connector": run_connector, "adaln": run_adaln, "i8": run_i8,
            "cublas_ab": run_cublas_ab, "gemm_trace": run_gemm_trace}
    return runs[args.workload](args)


if __name__ == "__main__":
    sys.exit(main())
