"""Benchmark: 1008px Hiera-L image encodes per second on B200 (sam3.c's
sam3_vit_build hot path), plus the encoder-GEMM TFLOP/s and the reference CPU
backend timed on the same host.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]

Workload: a batch of 64 synthetic 1008x1008 images
(seeded, see sam3.c_b200/synth.py) encoded by the 32-block ViT (width 1024,
16 heads, MLP 4736, 24x24 windows, global blocks 7/15/23/31) with BF16
weights ~N(0, 0.02), sharded by image over the N GPUs (one weight replica
per GPU, no collective on the data path): strong scaling, total work fixed.
One step = the 64-image batch.  Under torchrun every rank encodes its
shard; the step time is the max over ranks of CUDA-event time.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "sam3.c_b200"))

import dp  # noqa: E402
import synth  # noqa: E402

CFG = synth.HIERA_L
ATTN_GFLOP_PER_IMAGE = 28 * 12.23 + 4 * 110.08
TOTAL_GFLOP_PER_IMAGE = 5399.0
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) per launch of the dominant kernel, gemm2_kernel,
# averaged over the four GEMMs of one ViT block at 8 images: one ncu capture
# of `python bench.py --images 8 --batch 8 --steps 1 --warmup 1
# --no-cpu-baseline` with --metrics dram__bytes_read.sum,dram__bytes_write.sum
# -k regex:gemm2_kernel -s 4 -c 4 (per launch: 746.0, 292.8, 363.7, 434.6 MB).
GEMM_TRAFFIC_BYTES_PER_LAUNCH = 459.3e6


def gemm_gflop_per_image(cfg=CFG):
    gs = cfg["img_size"] // cfg["patch_size"]
    M, e, m = gs * gs, cfg["embed_dim"], cfg["mlp_dim"]
    per_block = 2 * M * e * (3 * e + e + m + m)
    patch = 2 * M * cfg["patch_size"] ** 2 * 3 * e
    return (cfg["depth"] * per_block + patch) / 1e9


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- reference arm
def cpu_reference_full(threads: int = 0, with_extrapolation: bool = True):
    """Time the UNMODIFIED reference CPU backend (oracle/_ref, compiled from
    the sam3.c sources) on one full 1008px encode: sam3_vit_build with all
    32 blocks (globals 7/15/23/31) through the reference's own graph and CPU
    kernels, its thread pool over all host threads, warm-up 0 and one
    iteration (about 75-110 s on 16 threads).  Beside it, the per-block
    extrapolation a shorter sample would give (depth-0 and depth-2 runs,
    a global block costed at a window block x (144.05 + 110.08) /
    (144.05 + 12.23) GFLOP) and its error against the full run."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if not O.ref_available():
        return None
    n = O.ref_set_threads(threads)
    img = synth.images(CFG, 1, seed=100)[0]
    w = synth.vit_weights(CFG, seed=0)
    t = time.perf_counter()
    O.ref_vit_encode(CFG, w, img)
    t_full = time.perf_counter() - t
    res = {"value": 1.0 / t_full, "unit": "images/s", "cores": os.cpu_count() if n == 0 else n,
           "kind": "reference", "seconds_per_image": t_full,
           "sample": (f"reference sam3_vit_build on its CPU backend (oracle/_ref), 1 image 1008px, all 32 blocks, "
                      f"measured once (warm-up 0, 1 iteration): {t_full:.1f} s/image")}
    if with_extrapolation:
        w2 = dict(w, blocks=w["blocks"][:2])
        t = time.perf_counter()
        O.ref_vit_encode(dict(CFG, depth=0), w2, img)
        t_embed = time.perf_counter() - t
        t = time.perf_counter()
        O.ref_vit_encode(dict(CFG, depth=2), w2, img)
        t2 = time.perf_counter() - t
        t_blk = max((t2 - t_embed) / 2, 1e-9)
        g = (144.05 + 110.08) / (144.05 + 12.23)
        t_x = t_embed + 28 * t_blk + 4 * g * t_blk
        res["extrapolated_from_2_blocks"] = {"seconds_per_image": t_x,
                                             "error_vs_full": (t_x - t_full) / t_full}
    O.ref_set_threads(1)  # release the pool's workers
    return res


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    r = cpu_reference_full(args.cpu_threads, with_extrapolation=not args.cpu_json)
    if r is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libsam3_ref.so not built"}))
        return 0
    if args.cpu_json:  # the cpu_baseline object alone, for the repo arm
        print(json.dumps({k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}))
        return 0
    v = r["value"]
    line = {"impl": "reference", "metric": "images_per_sec_1008px_hiera_l", "value": v,
            "unit": "images/s", "n_gpus": args.gpus, "steps": 1, "warmup": 0,
            "ms_per_step": 1000.0 * r["seconds_per_image"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config4_batched_encode_64x1008px_hiera_l",
                       "global_batch": args.images, "parallelism": "cpu",
                       "step": "one full 32-block 1008px encode of one image of the workload (BASELINE: the "
                               "full encoder is timed warm-up 0, 1 iteration; --steps / --warmup do not "
                               "apply to this ~100 s step)"},
            "cpu_baseline": {"value": v, "unit": "images/s", "cores": r["cores"],
                             "kind": "reference", "sample": r["sample"]},
            "extrapolated_from_2_blocks": r.get("extrapolated_from_2_blocks"),
            "e2e": {"value": v, "unit": "images/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def cpu_baseline_subprocess(args):
    """The full-encode CPU baseline in a fresh process (no CUDA context or
    torch threads competing for the host cores), after the GPU legs."""
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--cpu-json",
           "--cpu-threads", str(args.cpu_threads)]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    try:
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env).stdout
        for ln in out.splitlines()[::-1]:
            if ln.startswith("{"):
                d = json.loads(ln)
                return None if "unavailable" in d else d
    except (subprocess.TimeoutExpired, ValueError) as e:
        return {"unavailable": str(e)}
    return None


# ---------------------------------------------------------------- our arm
def run_ours(args):
    import torch
    import torch.distributed as dist
    import sam3cu

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl")
    torch.cuda.set_device(local)
    sam3cu.init(local)
    dev = torch.device("cuda", local)

    n_total = args.images
    first, n_local = dp.shard_range(n_total, world, rank)
    B = min(args.batch, max(n_local, 1))
    wdt = {"bf16": sam3cu.BF16, "f16": sam3cu.F16, "q8": sam3cu.Q8_0}[args.dtype]

    w = synth.vit_weights(CFG, seed=0)
    enc = sam3cu.VitEncoder(CFG, w, wdt, max_batch=B)
    del w
    s = CFG["img_size"]
    np_ = enc.np
    e = CFG["embed_dim"]
    # this rank's images: image i of the job uses seed 100 + i
    host_imgs = torch.empty((n_local, 3, s, s), dtype=torch.float32).pin_memory()
    for i in range(n_local):
        host_imgs[i] = torch.from_numpy(synth.images(CFG, 1, seed=dp.image_seed(first + i))[0])
    host_out = torch.empty((max(n_local, 1), np_, e), dtype=torch.float32).pin_memory()
    dev_imgs = host_imgs.to(dev)
    dev_out = torch.empty((B, np_, e), dtype=torch.float32, device=dev)
    stream = torch.cuda.ExternalStream(enc.stream, device=dev)
    chunks = [(i, min(B, n_local - i)) for i in range(0, n_local, B)]

    def step_device():
        for i, n in chunks:
            enc.encode_async(dev_imgs[i:i + n], dev_out[:n])

    def step_e2e():
        # public API with host buffers: one call for this rank's images; the
        # library encodes them in chunks of B and overlaps each chunk's H2D
        # and D2H copies with the neighbouring chunks' compute
        enc.encode_ptr(host_imgs.data_ptr(), n_local, host_out.data_ptr(), on_device=False)

    def timed(fn, k):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(k):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        return dp.max_over_ranks(a.elapsed_time(b), device=dev)

    for _ in range(args.warmup):
        step_device()
    torch.cuda.synchronize()
    sam3cu.launch_count(reset=True)
    clk = ClockSampler(local)
    clk.start()
    ms = timed(step_device, args.steps)
    clocks = clk.stop()
    launches = sam3cu.launch_count()
    assert sam3cu.device_error() == 0, "device-side error during the timed region"
    ms_step = ms / args.steps
    value = n_total / (ms_step / 1000.0)

    # end-to-end through the public API with host buffers
    for _ in range(max(1, args.warmup // 2)):
        step_e2e()
    ms_e2e = timed(step_e2e, max(1, args.steps // 2)) / max(1, args.steps // 2)
    e2e_value = n_total / (ms_e2e / 1000.0)
    h2d = n_total * 3 * s * s * 4
    d2h = n_total * np_ * e * 4

    # per-kernel-kind device time of one encode of B images (direct
    # launches with events between them, same stream)
    prof = enc.profile(dev_imgs[:B], dev_out)
    gemm_ms, gemm_n = prof["gemm"]
    attn_ms, attn_n = prof["attention"]
    ln_ms, ln_n = prof["layernorm"]
    gemm_tflops = gemm_gflop_per_image() * B / gemm_ms  # GFLOP/ms = TFLOP/s
    attn_tflops = ATTN_GFLOP_PER_IMAGE * B / attn_ms
    # LN1/LN2 read the f32 stream and write 16-bit; ln_pre reads and writes f32
    ln_bytes = (2 * CFG["depth"] * np_ * e * (4 + 2) + np_ * e * 8) * B
    pk, pk_src = peaks()
    peak = pk.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])

    if rank == 0:
        cpu = None
        total = gemm_ms + attn_ms + ln_ms + prof["other"][0]
        line = {
            "metric": "images_per_sec_1008px_hiera_l", "value": value, "unit": "images/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": {"bf16": "bf16", "f16": "f16", "q8": "q8_0w+bf16"}[args.dtype],
            "data": "synthetic (seeded images and random-init weights of the Hiera-L ViT)",
            "config": {"workload": "config4_batched_encode_64x1008px_hiera_l",
                       "global_batch": n_total, "images_per_encode_call": B, "seq_len": 5184,
                       "parallelism": f"dp{world} (image shards, weight replica per GPU)",
                       "l2": "inputs and weights larger than L2 (0.8 GB images, 0.9 GB weights)"},
            "e2e": {"value": e2e_value, "unit": "images/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor",
                         "kernel": "gemm2_kernel (2-SM tcgen05 linear + fused epilogue)",
                         "achieved": gemm_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": gemm_tflops / peak,
                         "traffic": GEMM_TRAFFIC_BYTES_PER_LAUNCH if args.dtype != "q8" else None,
                         "traffic_unit": "bytes per launch (ncu, 8 images, BF16)",
                         "peak_source": f"{pk_src} bf16_tflops_sustained"},
            "gemm_tflops": gemm_tflops,
            "attention_tflops": attn_tflops,
            "layernorm_gbs": ln_bytes / (ln_ms / 1000.0) / 1e9,
            "kernel_share": {k: round(prof[k][0] / total, 4) for k in prof},
            "kernel_launches_per_encode": {k: prof[k][1] for k in prof},
            "model_tflops": TOTAL_GFLOP_PER_IMAGE * value / 1000.0,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if world == 1 and not args.no_tinyvit:
            enc.close()
            line["tinyvit_config5"] = tinyvit_leg(args, dev, sam3cu)
            line["fpn_neck"] = neck_leg(args, dev, sam3cu)
            line["gemm_sweep_config1"] = gemm_sweep_leg(args, dev, sam3cu)
            line["dropin_vtable_f32"] = dropin_leg(args, dev, sam3cu)
            line.update(q8_legs(args, dev, sam3cu))
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_subprocess(args)
        print(json.dumps(line))
    enc.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def _event_ms(fn, iters, stream=None):
    """Mean ms per call of fn, CUDA events on `stream` (the stream fn's
    kernels run on; torch's current stream by default)."""
    import torch
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(stream)
    for _ in range(iters):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def q8_legs(args, dev, sam3cu):
    """BASELINE configs 0 and 2 (parity cases, reported beside the headline):
    the single Q8_0 linear [5184 x 1024] . [4736 x 1024]^T + bias through
    sam3cu_linear_q8 (F32 activations as configured, rounded to BF16 inside
    the timed call; F32 out), and the full 1008px ViT
    encode of one image with Q8_0 weights (F16 activations).  Device-
    resident inputs; CUDA-event times after warm-up."""
    import torch
    rng = np.random.default_rng(1)
    M, K, N = 5184, 1024, 4736
    x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).to(dev)
    w = torch.from_numpy((rng.standard_normal((N, K)) * 0.02).astype(np.float32)).to(dev)
    b = torch.from_numpy((rng.standard_normal(N) * 0.01).astype(np.float32)).to(dev)
    q, sc = sam3cu.q8_repack(sam3cu.q8_quantize(w), N, K)
    y = torch.empty((M, N), dtype=torch.float32, device=dev)
    f = lambda: sam3cu.linear_q8(x, q, sc, bias=b, out=y)
    for _ in range(3):
        f()
    torch.cuda.synchronize()
    ms_lin = _event_ms(f, 20)
    # breakdown: the same call with BF16 activations (no cast), and the bare
    # 16-bit GEMM on the dequantised weight (no cast, no dequantisation)
    xb = x.bfloat16()
    fb = lambda: sam3cu.linear_q8(xb, q, sc, bias=b, out=y)
    wdq = w.bfloat16()  # same shape and layout as the dequantised weight
    fg = lambda: sam3cu.linear(xb, wdq, bias=b, out=y)
    for g_ in (fb, fg):
        for _ in range(3):
            g_()
    ms_bf = _event_ms(fb, 20)
    ms_gemm = _event_ms(fg, 20)
    lin = {"tflops": 2 * M * K * N / ms_lin / 1e9, "ms": ms_lin,
           "dtype": "q8_0w x f32a (bf16 on chip), f32 out",
           "note": "F32 activations cast inside the call + dequantise-once path (M >= 2048) of sam3cu_linear_q8",
           "breakdown_ms": {"f32_x_call": ms_lin, "bf16_x_call": ms_bf, "bf16_gemm_only_f32_out": ms_gemm}}
    if args.leg == "q8lin":  # config 0 alone (the ncu capture of its kernels)
        return {"q8_linear_config0": lin}
    enc = sam3cu.VitEncoder(CFG, synth.vit_weights(CFG, seed=0), sam3cu.Q8_0, max_batch=1)
    img = torch.from_numpy(synth.images(CFG, 1, seed=100)).to(dev)
    out = torch.empty((1, enc.np, CFG["embed_dim"]), dtype=torch.float32, device=dev)
    g = lambda: enc.encode_async(img, out)
    for _ in range(3):
        g()
    torch.cuda.synchronize()
    ms_enc = _event_ms(g, 10, torch.cuda.ExternalStream(enc.stream, device=dev))
    prof = enc.profile(img, out)
    enc.close()
    # BASELINE config 4's batch with Q8_0 weights: 64 images, 8 per call
    enc = sam3cu.VitEncoder(CFG, synth.vit_weights(CFG, seed=0), sam3cu.Q8_0, max_batch=8)
    imgs = torch.from_numpy(synth.images(CFG, 8, seed=100)).to(dev)
    out8 = torch.empty((8, enc.np, CFG["embed_dim"]), dtype=torch.float32, device=dev)
    h = lambda: [enc.encode_async(imgs, out8) for _ in range(8)]
    h()
    torch.cuda.synchronize()
    ms64 = _event_ms(h, 3, torch.cuda.ExternalStream(enc.stream, device=dev))
    prof8 = enc.profile(imgs, out8)
    enc.close()
    assert sam3cu.device_error() == 0
    return {
        "q8_encode_64img": {"value": 64 * 1000.0 / ms64, "unit": "images/s", "ms_per_64": ms64,
                            "gemm_tflops": gemm_gflop_per_image() * 8 / prof8["gemm"][0],
                            "dtype": "q8_0w+bf16a", "images_per_call": 8},
        "q8_linear_config0": lin,
        "q8_encode_config2": {"value": 1000.0 / ms_enc, "unit": "images/s", "ms_per_image": ms_enc,
                              "gemm_tflops": gemm_gflop_per_image() / prof["gemm"][0],
                              # the per-launch profile adds an event and a ramp to every launch,
                              # so its intervals sum to more than the encode; scaled to the
                              # measured encode time by the GEMMs' share of the profile:
                              "gemm_tflops_share_of_encode":
                                  gemm_gflop_per_image() / (ms_enc * prof["gemm"][0] /
                                                            sum(v[0] for v in prof.values())),
                              "profile_sum_ms": sum(v[0] for v in prof.values()),
                              "dtype": "q8_0w+bf16a", "batch": 1},
    }


# (name, K, N, epilogue) of the four ViT-block linears
SWEEP_SHAPES = (("qkv", 1024, 3072, "bias"), ("proj", 1024, 1024, "residual"), ("fc1", 1024, 4736, "gelu"),
                ("fc2", 4736, 1024, "residual"))


def gemm_sweep_leg(args, dev, sam3cu):
    """the ViT-block linears at M = 5184*B for B in
    {1, 2, 4, 8}, values ~N(0,1)/sqrt(K), FP32 accumulation, each with the
    encoder's epilogue (bias; tanh-GELU on fc1; F32 residual added in place
    on proj / fc2).  BF16 at every B, F16 at B = 8, F32 (3xTF32: three
    kind::tf32 MMAs per product, hi*hi + hi*lo + lo*hi) at B = 1 and 8,
    whose TFLOP/s count the F32 product once.  Device-resident
    operands, CUDA events over 20 launches after 3 warm-ups.  With the CPU
    baseline on, the reference's cpu_kernel_matmul_bf16 (oracle/_ref) is
    timed on the proj shape at B = 1 beside it."""
    import torch
    res = {"unit": "TFLOP/s", "m_per_image": 5184, "shapes": {}}
    g = torch.Generator(device=dev).manual_seed(0)
    for dt_name, dt, Bs in (("bf16", torch.bfloat16, (1, 2, 4, 8)), ("f16", torch.float16, (8,)),
                            ("f32", torch.float32, (1, 8))):
        for name, K, N, epi in SWEEP_SHAPES:
            w = (torch.randn(N, K, device=dev, generator=g) / K ** 0.5).to(dt)
            b = torch.randn(N, device=dev, generator=g) / K ** 0.5
            for B in Bs:
                M = 5184 * B
                x = (torch.randn(M, K, device=dev, generator=g) / K ** 0.5).to(dt)
                if epi == "residual":
                    y = torch.randn(M, N, device=dev, generator=g)
                    f = lambda: sam3cu.linear(x, w, bias=b, residual=y, out=y)
                else:
                    y = torch.empty(M, N, device=dev, dtype=dt)
                    act = sam3cu.ACT_GELU_TANH if epi == "gelu" else sam3cu.ACT_NONE
                    f = lambda: sam3cu.linear(x, w, bias=b, act=act, out=y)
                for _ in range(3):
                    f()
                ms = _event_ms(f, 20)
                res["shapes"][f"{dt_name}_{name}_B{B}"] = round(2.0 * M * K * N / ms / 1e9, 1)
                del x, y
    assert sam3cu.device_error() == 0
    pk, pk_src = peaks()
    tf32 = 0.5 * pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    res["f32_peak"] = {"tf32_tflops": tf32, "f32_via_3xtf32_tflops": tf32 / 3.0,
                       "source": f"{pk_src} bf16_tflops x 1/2 (B200 datasheet TF32:BF16 dense ratio; "
                                 "no TF32 peak is measured); 3 MMAs per F32 product"}
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        if O.ref_available():
            O.ref_set_threads(args.cpu_threads)
            rng = np.random.default_rng(0)
            a = rng.standard_normal((5184, 1024)).astype(np.float32)
            wt = (rng.standard_normal((1024, 1024)) / 32.0).astype(np.float32)
            bits = lambda v: (np.ascontiguousarray(v).view(np.uint32) >> 16).astype(np.uint16)
            O.ref_matmul(bits(a[:64]), bits(wt), "bf16")
            t = time.perf_counter()
            O.ref_matmul(bits(a), bits(wt), "bf16")
            s = time.perf_counter() - t
            res["cpu_reference_bf16_proj_B1_gflops"] = round(2.0 * 5184 * 1024 * 1024 / s / 1e9, 1)
            # release the reference's worker threads: left alive they keep the
            # host cores busy and starve the launches of the legs that follow
            O.ref_set_threads(1)
    return res


NECK_SCALES = (4.0, 2.0, 1.0, 0.5)


def neck_gflop_per_image(d_model=256, dim=1024, grid=72):
    """Algorithmic GFLOP of the FPN neck (2 per multiply-add), per image."""
    fl = 0.0
    for sf in NECK_SCALES:
        H = (grid - 2) // 2 + 1 if sf < 0.75 else grid
        for kind, ci, co, k in synth.neck_layer_dims(d_model, dim, sf):
            if kind == "t":  # k2 s2 transposed conv: every input pixel feeds 4 outputs
                fl += 2.0 * H * H * ci * 4 * co
                H *= 2
            else:
                fl += 2.0 * H * H * ci * k * k * co
    return fl / 1e9


def neck_leg(args, dev, sam3cu):
    """The FPN neck after the encoder (sam3_neck_build,
    necks.c): ViT features [8, 5184, 1024] f32 -> 4 scales of d_model 256,
    BF16 compute.  Device-resident input; CUDA events on the neck's stream.
    With the CPU baseline on, the reference's own sam3_neck_build on its CPU
    backend (oracle/_ref) is timed on one image beside it."""
    import torch
    B = 8
    w = synth.neck_weights(256, 1024, NECK_SCALES, seed=0)
    neck = sam3cu.FpnNeck(256, 1024, 72, NECK_SCALES, w, sam3cu.BF16, max_batch=B)
    feat = torch.randn(B, 5184, 1024, device=dev)
    outs = neck.outputs(B, dev)
    f = lambda: neck.forward(feat, outs, sync=False)
    for _ in range(3):
        f()
    torch.cuda.synchronize()
    ms = _event_ms(f, 10, torch.cuda.ExternalStream(neck.stream, device=dev))
    neck.close()
    assert sam3cu.device_error() == 0
    gf = neck_gflop_per_image()
    res = {"workload": "sam3 FPN neck 72x72x1024 -> 288/144/72/36 x 256, 8 images per call",
           "dtype": "bf16", "value": B / (ms / 1000.0), "unit": "images/s", "ms_per_image": ms / B,
           "tflops": gf * B / ms, "gflop_per_image": gf}
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        if O.ref_available():
            O.ref_set_threads(args.cpu_threads)
            x = np.random.default_rng(0).standard_normal((5184, 1024)).astype(np.float32)
            t = time.perf_counter()
            try:
                O.ref_neck(256, 1024, 72, NECK_SCALES, w, x)
                res["cpu_reference_s_per_image"] = time.perf_counter() - t
                res["cpu_reference"] = ("reference sam3_neck_build on its CPU backend (oracle/_ref), 1 image, "
                                        f"the backend's own thread pool over {os.cpu_count()} host threads")
            except RuntimeError as e:
                res["cpu_reference_unavailable"] = str(e)
    return res


def attention_leg(args, dev, sam3cu):
    """The tcgen05 attention alone at the encoder's shapes for 8 images:
    global (8 groups x 5184 tokens) and windowed (72 windows x 576 tokens),
    16 heads of 64, BF16 Q|K|V packed as the QKV GEMM writes them.  CUDA
    events over 10 launches after 3 warm-ups; 4*S^2*64 FLOP per (group,
    head)."""
    import torch
    res = {"unit": "TFLOP/s"}
    g = torch.Generator(device=dev).manual_seed(0)
    for name, groups, seq in (("global_8img", 8, 5184), ("window_8img", 72, 576)):
        qkv = torch.randn(groups * seq, 3 * 1024, device=dev, generator=g).bfloat16()
        out = torch.empty(groups * seq, 1024, device=dev, dtype=torch.bfloat16)
        f = lambda: sam3cu.sdpa_packed(qkv, groups, seq, 16, 64, out=out)
        for _ in range(3):
            f()
        ms = _event_ms(f, 10)
        res[name] = 4.0 * seq * seq * 64 * 16 * groups / ms / 1e9
        del qkv, out
    assert sam3cu.device_error() == 0
    return res


def sdpa_f32_leg(args, dev, sam3cu):
    """The drop-in path's F32 attention kernel (sam3cu_sdpa_f32_strided)
    alone: Q|K|V read with strides from a packed [groups*seq, 3*1024] F32
    buffer (the QKV layout), 16 heads of 64; checked against torch's SDPA in
    float64; CUDA events over 5 launches after 2 warm-ups."""
    import ctypes as C
    import torch
    L = sam3cu.lib()
    f = L.sam3cu_sdpa_f32_strided
    P = C.POINTER(C.c_int64)
    f.argtypes = [C.c_void_p, P, C.c_void_p, P, C.c_void_p, P, C.c_void_p, C.c_void_p, P] + [C.c_int] * 5 + \
        [C.c_void_p]
    S, B, H, D = args.sdpa_seq, args.sdpa_groups, 16, 64
    E = H * D
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = torch.randn(B * S, 3 * E, device=dev, generator=g)
    o = torch.empty(B * S, E, device=dev)
    st = (C.c_int64 * 3)(S * 3 * E, D, 3 * E)
    so = (C.c_int64 * 3)(S * E, D, E)
    base = qkv.data_ptr()

    def run():
        sam3cu.check(f(base, st, base + 4 * E, st, base + 8 * E, st, None, o.data_ptr(), so, B, H, S, S, D,
                       torch.cuda.current_stream().cuda_stream), "sam3cu_sdpa_f32_strided")
    for _ in range(2):
        run()
    ms = _event_ms(run, 5)
    q, k, v = [qkv[:, i * E:(i + 1) * E].reshape(B, S, H, D).transpose(1, 2).double() for i in range(3)]
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B * S, E)
    err = float((o.double() - ref).abs().max() / ref.abs().max())
    assert sam3cu.device_error() == 0
    return {"groups": B, "seq": S, "ms": ms, "tflops": 4.0 * S * S * D * H * B / ms / 1e9,
            "rel_err_vs_torch_f64": err}


def dropin_leg(args, dev, sam3cu):
    """The drop-in path: the reference's own sam3_vit_build (compiled from
    the sam3.c sources, dropin/_ref) evaluating its F32 Hiera-L graph on one
    1008 px image through sam3_cuda_backend_ops(), host buffers in and out,
    exactly the call sequence of a sam3.c build with the CUDA backend
    registered (16 graph_evals, the residual stream read back to the host
    between them).  One untimed encode uploads the weights (the session
    keeps them, as a sam3_ctx does); then the host wall time of each
    sam3_vit_build call is taken (the call returns after its last
    synchronous read-back)."""
    sys.path.insert(0, os.path.join(ROOT, "dropin"))
    import dropin as D
    if not D.available():
        return {"unavailable": "dropin/_ref/libsam3_dropin.so not built"}
    w = synth.vit_weights(CFG, seed=0)
    img = synth.images(CFG, 1, seed=100)[0]
    dv = D.DropinVit(CFG, w, dev.index or 0)
    del w
    dv.encode(img)
    dv.profile_dump()  # SAM3CU_VTABLE_PROFILE only: drop the weight-upload encode
    secs = [dv.encode(img)[1] for _ in range(args.dropin_iters)]
    dv.profile_dump()
    dv.close()
    assert sam3cu.device_error() == 0
    t = float(np.median(secs))
    return {"workload": "reference sam3_vit_build (F32 graph, 32 blocks) on sam3_cuda_backend_ops, "
                        "1 image 1008px, host image in / host features out",
            "dtype": "f32 (3xTF32 GEMMs, F32 attention)", "value": 1.0 / t, "unit": "images/s",
            "ms_per_image": 1000.0 * t, "iters": len(secs),
            "ms_min": 1000.0 * min(secs), "ms_max": 1000.0 * max(secs)}


def tinyvit_leg(args, dev, sam3cu):
    """BASELINE config 5 (a parity case, reported beside the headline): the
    TinyViT-21M backbone at 1008 px, batch 32, F16, random-init weights,
    device-resident images, CUDA-event time of 5 encodes after 3 warm-ups."""
    import torch
    cfg = dict(synth.TINYVIT_21M)
    B = args.tinyvit_batch
    tv = sam3cu.TinyViT(cfg, synth.tinyvit_weights(cfg, seed=0), sam3cu.F16, max_batch=B)
    imgs = torch.from_numpy(synth.tinyvit_images(cfg, B, seed=1)).to(dev)
    out = torch.empty((B, tv.grid * tv.grid, cfg["embed_dim"]), dtype=torch.float32, device=dev)
    for _ in range(3):
        tv.encode_ptr(imgs.data_ptr(), B, out.data_ptr(), on_device=True)
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(5):
        tv.encode_ptr(imgs.data_ptr(), B, out.data_ptr(), on_device=True)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / 5
    tv.close()
    assert sam3cu.device_error() == 0
    return {"workload": f"config5_tinyvit21m_1008px_batch{B}", "dtype": "f16", "value": B / (ms / 1000.0),
            "unit": "images/s", "ms_per_batch": ms, "data": "synthetic (seeded images, random-init weights)"}


def run_leg(args):
    import torch
    import sam3cu
    torch.cuda.set_device(0)
    sam3cu.init(0)
    dev = torch.device("cuda", 0)
    fn = {"dropin": dropin_leg, "sweep": gemm_sweep_leg, "q8": q8_legs, "q8lin": q8_legs, "neck": neck_leg,
          "tinyvit": tinyvit_leg, "attn": attention_leg, "sdpa_f32": sdpa_f32_leg}[args.leg]
    print(json.dumps({"leg": args.leg, "result": fn(args, dev, sam3cu)}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--images", type=int, default=64)
    ap.add_argument("--batch", type=int, default=8, help="images per encode call")
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "f16", "q8"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-threads", type=int, default=0)
    ap.add_argument("--cpu-json", action="store_true",
                    help="with --impl reference: print only the cpu_baseline object (no extrapolation)")
    ap.add_argument("--no-tinyvit", action="store_true", help="skip the config-5 TinyViT leg")
    ap.add_argument("--dropin-iters", type=int, default=3)
    ap.add_argument("--sdpa-seq", type=int, default=5184, help="sdpa_f32 leg: tokens per group")
    ap.add_argument("--sdpa-groups", type=int, default=1, help="sdpa_f32 leg: groups (images or windows)")
    ap.add_argument("--tinyvit-batch", type=int, default=32, help="tinyvit leg: images per call")
    ap.add_argument("--leg", default=None,
                    choices=["dropin", "sweep", "q8", "q8lin", "neck", "tinyvit", "attn", "sdpa_f32"],
                    help="run one side leg alone on GPU 0 and print its result")
    args = ap.parse_args()
    if args.leg:
        return run_leg(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
