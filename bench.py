"""Benchmark of the SAM 3 PE backbone hot path on B200 (one JSON line).

Workload ("config 5"): 64 independent 1008 x 1008
x 3 uint8 tiles (uniform, seeded) through the random-init 32-block PE
backbone (width 1024, 16 heads, MLP 4096, 24 x 24 windows, global blocks
7/15/23/31), bf16 tensor-core operands with fp32 accumulation, tiles
sharded evenly across the GPUs (one process per GPU, no collective in the
data path). The total is fixed at 64 tiles, so "scaling" is "strong". A step
= one pass of every rank's tile shard through the backbone. The line also
carries, measured on rank 0, the attention configs 1 and 2 (the metric's "PE
attention TFLOP/s" part) and the decoder attention of config 3 (GB/s against
the HBM peak); at N = 1 it adds the reference kernels' CPU times of configs
1-3 (`cpu_configs`) beside the tiles/s `cpu_baseline`.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

--impl reference times the reference's own CPU kernels (sam3_kernels.cl
compiled for the host by oracle/Makefile) on the host cores, rank 0 only.
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
sys.path.insert(0, ROOT)

METRIC = "PE attention TFLOP/s (% bf16 peak); backbone tiles/sec at 1/2/4/8 B200"
TOTAL_TILES = 64
SEED = 1
TILE_FLOP = 4.964e12  # algorithmic FLOPs of one backbone tile
SIDE = 1008


def load_product():
    import importlib.util
    name = "sam3_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(ROOT, "i.sam3.opencl_b200", "sam3_b200.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def image_stream(tile):
    return 3 * 1000003 + tile  # SAM3_IMAGE_STREAM_TILE


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return dict(hbm=p["hbm_gbs"], bf16=p["bf16_tflops"],
                    bf16_sus=p.get("bf16_tflops_sustained", p["bf16_tflops"]),
                    src="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sus=1400.0, src="fallback")


class Clocks:
    """nvidia-smi sampling during the timed region (one sampler, on rank 0,
    for all the job's GPUs). Entering waits for the first sample, so that
    a short timed region (8 GPUs: a few hundred ms) still has samples
    inside it."""

    def __init__(self, gpus, active=True):
        self.gpus = gpus
        self.active = active
        self.proc = None
        self.path = f"/tmp/sam3_bench_clocks_{os.getpid()}.csv"

    def __enter__(self):
        if not self.active:
            return self
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(str(g) for g in self.gpus),
                 f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        t0 = time.time()
        while self.proc and self.proc.poll() is None and time.time() - t0 < 5.0:
            try:
                if os.path.getsize(self.path) > 0:
                    break
            except OSError:
                pass
            time.sleep(0.01)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()
            self.f.close()

    def summary(self):
        if not self.active:
            return None
        try:
            rows = [r.split(",") for r in open(self.path).read().strip().splitlines()]
        except Exception:
            return None
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def smi_indices(devs):
    """nvidia-smi indices of CUDA devices (through CUDA_VISIBLE_DEVICES when
    it lists plain indices)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    try:
        phys = [int(x) for x in vis.split(",")] if vis else None
    except ValueError:
        phys = None
    if phys is None:
        return devs
    return [phys[d] for d in devs if d < len(phys)]


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            sys.exit("run multi-GPU benchmarks under torchrun (one process per GPU)")
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if args.impl == "ours" else "gloo"
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
        pg = dist
    return world, rank, local, pg


# ---------------------------------------------------------------- reference arm
def reference_arm(args, world, rank):
    """The reference's CPU kernels on a bounded sample, extrapolated to
    tiles/s: the prologue, one windowed and one global block of one tile per
    step are timed; a tile = prologue + 28 windowed + 4 global blocks."""
    from oracle import binding as ob
    from oracle.reference_cpu import RefTrunk

    if rank != 0:
        return None
    if not ob.have_ref():
        return {"impl": "reference", "unavailable":
                "oracle/_ref/libsam3ref.so was not built (reference tree absent at build time)"}
    rt = RefTrunk(SEED, depth=2, global_blocks=(1,))
    img = ob.u8(SEED, image_stream(0), (SIDE, SIDE, 3))
    times = []
    for step in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        x = rt.prologue(img)
        t1 = time.perf_counter()
        rt.block(x, 0)
        t2 = time.perf_counter()
        rt.block(x, 1)
        t3 = time.perf_counter()
        if step >= args.warmup:
            times.append((t1 - t0, t2 - t1, t3 - t2))
    pro = statistics.median(t[0] for t in times)
    win = statistics.median(t[1] for t in times)
    glob = statistics.median(t[2] for t in times)
    tile_s = pro + 28 * win + 4 * glob
    value = 1.0 / tile_s
    sample = (f"reference kernels (sam3_kernels.cl compiled as host C++: gemm_cpu_t/"
              f"gemm_cpu_n, layernorm, rope_apply, softmax_rows, window (un)partition) "
              f"orchestrated as vit_block; per step: prologue {pro:.2f}s + 1 windowed "
              f"block {win:.2f}s + 1 global block {glob:.2f}s of one tile; tile time "
              f"extrapolated as prologue + 28 windowed + 4 global = {tile_s:.1f}s")
    cores = ob.ref().ref_num_threads()
    return {"metric": METRIC, "value": value, "unit": "tiles/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": (pro + win + glob) * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded uint8 tiles, random-init weights)",
            "config": {"workload": "config 5: 64 tiles x 32-block PE backbone "
                                   "(bounded CPU sample, see cpu_baseline.sample)"},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tiles/s", "cores": cores,
                             "kind": "reference", "sample": sample},
            "e2e": {"value": value, "unit": "tiles/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------- our arm
L2_BYTES = 126 * 1024 * 1024  # B200 L2


def flush_l2(buf):
    buf.add_(1)


def attention_bench(sb, cb, torch, pk, iters=10):
    """Configs 1 and 2: the fused attention kernel on bf16 qkv (RoPE already
    applied, as the QKV GEMM epilogue leaves it), L2 flushed (256 MiB write)
    between timed iterations; TFLOP/s = 4 N^2 d per (sequence, head) / kernel
    time. Also timed: the op with fp32 Q/K/V in (RoPE + bf16 cast pass +
    kernel), and config 2 in the fp32 reference mode (CUDA cores)."""
    stream = torch.cuda.ExternalStream(cb.stream)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(SEED)
    res = {}
    for name, side, nseq in (("config1_window_9x576", 24, 9), ("config2_global_5184", 72, 1)):
        E, N = 1024, side * side
        qkv = torch.randn(nseq * N, 3 * E, device="cuda", generator=g)
        q16 = qkv.to(torch.bfloat16)
        cs = torch.empty(N * 64, dtype=torch.float32)
        sb.lib().sam3_synth_rope_axial(side, 64, 10000.0, cs.data_ptr())
        cs = cs.cuda()
        out16 = torch.empty(nseq * N, E, dtype=torch.bfloat16, device="cuda")
        out32 = torch.empty(nseq * N, E, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        mq, mq16, mcs = cb.wrap(qkv), cb.wrap(q16), cb.wrap(cs)
        mo16, mo32 = cb.wrap(out16), cb.wrap(out32)
        flops = 4.0 * nseq * 16 * N * N * 64
        runs = [("tc_kernel", lambda: cb.attention(mq16, nseq, N, E, 16, 64, None, N, 0.125,
                                                    sb.ATTN_TC, mo16)),
                ("tc_from_f32_qkv", lambda: cb.attention(mq, nseq, N, E, 16, 64, mcs, N,
                                                               0.125, sb.ATTN_TC, mo32))]
        if nseq == 1:
            runs.append(("f32_reference_mode",
                         lambda: cb.attention(mq, nseq, N, E, 16, 64, None, N, 0.125,
                                              sb.ATTN_F32, mo32)))
        for mode_name, fn in runs:
            times = []
            for it in range(iters + 3):
                with torch.cuda.stream(stream):
                    flush_l2(flush)
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    fn()
                    e1.record(stream)
                stream.synchronize()
                if it >= 3:
                    times.append(e0.elapsed_time(e1))
            t = statistics.median(times)
            tf = flops / (t * 1e-3) / 1e12
            res[f"{name}.{mode_name}"] = {"ms": t, "tflops": tf,
                                          "frac_bf16_peak": tf / pk["bf16"]}
        cb.sync()
    res["peak_bf16_tflops"] = pk["bf16"]
    res["peak_source"] = pk["src"] + " bf16_tflops (burst: kernels timed alone)"
    return res


# Config 3: the mask decoder's fused attention for one batch of 64 prompts
# (sam3_model.c:419-451; dint 128, 8 heads of 16, 5184 image tokens), with the
# reference's 8 tokens per prompt (sam3_model.c:34-35) and the 7 BASELINE
# names. t2i: prompt tokens over the image (per-prompt K/V, as the decoder's
# two-way layers feed it, or one shared K/V); i2t: image tokens over the
# prompt tokens. HBM-bound: GB/s = algorithmic bytes / kernel time.
DEC_P, DEC_NK, DEC_D = 64, 5184, 128


def decoder_cases(ntok):
    P, N, D = DEC_P, DEC_NK, DEC_D
    return [  # name, Nq, Nk, q rows, kv rows, shared kv, algorithmic bytes
        (f"t2i_per_prompt_kv_{ntok}tok", ntok, N, P * ntok, P * N, False,
         4 * (P * ntok * D * 2 + 2 * P * N * D)),
        (f"t2i_shared_kv_{ntok}tok", ntok, N, P * ntok, N, True,
         4 * (P * ntok * D * 2 + 2 * N * D)),
        (f"i2t_{ntok}tok", N, ntok, P * N, P * ntok, False,
         4 * (P * N * D * 2 + 2 * P * ntok * D)),
    ]


def decoder_bench(cb, torch, pk, iters=10):
    stream = torch.cuda.ExternalStream(cb.stream)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(SEED + 3)
    res = {}
    for ntok in (8, 7):
        for name, nq, nk, qrows, kvrows, shared, nbytes in decoder_cases(ntok):
            q = torch.randn(qrows, DEC_D, device="cuda", generator=g)
            k = torch.randn(kvrows, DEC_D, device="cuda", generator=g)
            v = torch.randn(kvrows, DEC_D, device="cuda", generator=g)
            o = torch.empty(qrows, DEC_D, device="cuda")
            torch.cuda.synchronize()
            mq, mk, mv, mo = cb.wrap(q), cb.wrap(k), cb.wrap(v), cb.wrap(o)
            skv = 0 if shared else nk * DEC_D
            # Inputs far larger than L2 stream from HBM on every call: those
            # cases run back to back between one event pair (no flush, whose
            # dirty lines would be written back inside the timed region);
            # the shared-K/V case, whose 5.8 MB would stay in L2, has L2
            # flushed before each timed call.
            big = nbytes > 2 * L2_BYTES
            times = []
            for it in range(iters + 3):
                with torch.cuda.stream(stream):
                    if not big:
                        flush_l2(flush)
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    for _ in range(8 if big else 1):
                        cb.mha(DEC_P, nq, nk, DEC_D, mq, nq * DEC_D, mk, skv, mv, skv, mo)
                    e1.record(stream)
                stream.synchronize()
                if it >= 3:
                    times.append(e0.elapsed_time(e1) / (8 if big else 1))
            t = statistics.median(times)
            gbs = nbytes / (t * 1e-3) / 1e9
            res[name] = {"ms": t, "gbs": gbs, "frac_hbm": gbs / pk["hbm"],
                         "bytes": nbytes,
                         "l2": "inputs > L2, 8 calls back to back" if big
                         else "L2 flushed before each call"}
        cb.sync()
    res["peak_hbm_gbs"] = pk["hbm"]
    res["batch"] = f"{DEC_P} prompts, dint {DEC_D}, 8 heads, {DEC_NK} image tokens"
    return res


NECK_TILES = 8
# multiply-adds per token of point_neck (E = 1024): ConvT 1024->512 (x2
# levels), ConvT 512->256 (4 sub-pixels), 1x1 and 3x3 convolutions and the
# conv_s0 / conv_s1 projections at 16x, 4x and 1x the token count
NECK_MAC_PER_TOKEN = (2 * 1024 * 2048 + 4 * 512 * 1024 + 16 * 256 * 256 + 16 * 2304 * 256
                      + 16 * 256 * 32 + 4 * 512 * 256 + 4 * 2304 * 256 + 4 * 256 * 64
                      + 1024 * 256 + 2304 * 256)


def neck_bench(sb, cb, torch, iters=5):
    """The SimpleFPN neck (cb_neck_run) on NECK_TILES trunk outputs per call,
    random-init weights, synthetic fp32 tokens; device-timed, plus one
    profiled call for the per-kernel shares."""
    stream = torch.cuda.ExternalStream(cb.stream)
    T = 5184
    neck = sb.Neck(cb, grid=72, embed=1024, max_tiles=NECK_TILES)
    neck.init_random(SEED, 0.02)
    x = cb.alloc(NECK_TILES * T * 1024 * 4, sb.F32)
    cb.synth_normal(SEED, 9400, 0.0, 1.0, x, NECK_TILES * T * 1024)
    outs = [cb.alloc(NECK_TILES * T * 256 * 4, sb.F32),
            cb.alloc(NECK_TILES * 16 * T * 32 * 4, sb.F32),
            cb.alloc(NECK_TILES * 4 * T * 64 * 4, sb.F32)]
    times = []
    for it in range(iters + 2):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        neck.run(x, NECK_TILES, *outs)
        e1.record(stream)
        e1.synchronize()
        if it >= 2:
            times.append(e0.elapsed_time(e1))
    cb.profile(True)
    neck.run(x, NECK_TILES, *outs)
    cb.profile(False)
    prof = cb.profile_table()
    neck.close()
    t = statistics.median(times)
    flop = 2.0 * NECK_MAC_PER_TOKEN * T * NECK_TILES
    total = sum(v["ms"] for v in prof.values())
    kernels = {k: {"share": v["ms"] / total, "launches": v["calls"],
                   "gbs": v["bytes"] / (v["ms"] * 1e-3) / 1e9,
                   "tflops": v["flops"] / (v["ms"] * 1e-3) / 1e12 if v["flops"] else None}
               for k, v in prof.items()}
    return {"tiles": NECK_TILES, "ms_per_call": t, "ms_per_tile": t / NECK_TILES,
            "tflops": flop / (t * 1e-3) / 1e12, "gflop_per_tile": flop / NECK_TILES / 1e9,
            "kernels": kernels,
            "work": "cb_neck_run: point_neck of 8 tiles (72 x 72 x 1024 fp32 tokens) "
                    "-> emb, feat_s0, feat_s1"}


def input_bench(sb, cb, torch, iters=10):
    """The input path (cb_image_encoder_input) on a 2100 x 1500 crop of a
    seeded uint8 image resized to one 1008 x 1008 tile, uint8 tile output
    (what cb_encode_tiles reads); device-timed."""
    stream = torch.cuda.ExternalStream(cb.stream)
    rows, cols = 1600, 2200
    img = cb.alloc(rows * cols * 3, sb.U8)
    h = np.random.default_rng(SEED).integers(0, 256, size=(rows, cols, 3), dtype=np.uint8)
    cb.write(img, h)
    tiles = cb.alloc(1008 * 1008 * 3, sb.U8)
    times = []
    for it in range(iters + 3):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        cb.image_encoder_input(img, cols, rows, 40, 60, 2100, 1500, 1008, tiles=tiles)
        e1.record(stream)
        e1.synchronize()
        if it >= 3:
            times.append(e0.elapsed_time(e1))
    t = statistics.median(times)
    nbytes = 2100 * 1500 * 3 + 2 * 1500 * 1008 * 3 + 1008 * 1008 * 3
    return {"ms_per_crop": t, "crops_per_s": 1e3 / t, "gbs": nbytes / (t * 1e-3) / 1e9,
            "work": "2100 x 1500 RGB crop -> 1008 x 1008 uint8 tile (antialiased bilinear)"}


def detector_attention_bench(sb, cb, torch, pk, iters=10):
    """cb_attend on the detector's two image-sized shapes: the fusion
    encoder's self-attention (5184 tokens, 8 heads of 32) and the decoder's
    201 queries over the image with the box relative position bias, both on
    the tensor cores (CB_ATTN_TC; the biased one also in the fp32 mode for
    comparison); synthetic N(0, 1) inputs, device-timed."""
    stream = torch.cuda.ExternalStream(cb.stream)
    g = torch.Generator(device="cuda").manual_seed(SEED + 5)
    heads, hd, T = 8, 32, 5184
    res = {}
    for name, nq, rpb, mode in (("fusion_self_5184", T, False, 0),
                                ("decoder_image_rpb_201", 201, True, 0),
                                ("decoder_image_rpb_201_fp32_mode", 201, True, 1)):
        q = torch.randn(nq, heads * hd, device="cuda", generator=g)
        k = torch.randn(T, heads * hd, device="cuda", generator=g)
        v = torch.randn(T, heads * hd, device="cuda", generator=g)
        o = torch.empty(nq, heads * hd, device="cuda")
        dy = torch.randn(nq * 72 * heads, device="cuda", generator=g) if rpb else None
        dx = torch.randn(nq * 72 * heads, device="cuda", generator=g) if rpb else None
        torch.cuda.synchronize()
        w = [cb.wrap(t) for t in (q, k, v, o)]
        wb = [cb.wrap(t) for t in (dy, dx)] if rpb else [None, None]
        times = []
        for it in range(iters + 3):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            cb.attend(nq, T, heads, hd, w[0], heads * hd, w[1], heads * hd, w[2], heads * hd,
                      w[3], heads * hd, 0, wb[0], wb[1], 72 if rpb else 0, mode)
            e1.record(stream)
            e1.synchronize()
            if it >= 3:
                times.append(e0.elapsed_time(e1))
        t = statistics.median(times)
        flop = 4.0 * nq * T * hd * heads
        res[name] = {"ms": t, "tflops": flop / (t * 1e-3) / 1e12,
                     "path": "CUDA cores (fp32)" if mode else (
                         "tcgen05 (bf16), box bias as a dense term, keys split over CTAs"
                         if rpb else "tcgen05 (bf16)")}
    return res


MASK_P = 64  # prompts per decode (config 3: batches of 64)


def mask_decoder_bench(sb, cb, torch, iters=5):
    """The whole point-prompt decoder (cb_decode: prompt tokens from host
    points, two-way transformer, output upscaling, heads, low-res logits,
    IoU back to the host) on MASK_P prompts per call, synthetic image
    features and random-init weights; device-timed with CUDA events on the
    backend stream around each blocking call, plus one profiled call for the
    per-kernel shares."""
    stream = torch.cuda.ExternalStream(cb.stream)
    dec = sb.Decoder(cb, MASK_P)
    dec.init_random(SEED, 0.02)
    T = 5184
    feats = []
    for k, n in enumerate((T * 256, 16 * T * 32, 4 * T * 64)):
        m = cb.alloc(n * 4, sb.F32)
        cb.synth_normal(SEED, 9216 + k, 0.0, 1.0, m, n)
        feats.append(m)
    dec.set_image(*feats)
    rng = np.random.default_rng(SEED)
    pts = rng.uniform(0, 1008, size=(MASK_P, 2)).astype(np.float32)
    low = cb.alloc(MASK_P * 3 * 288 * 288 * 4, sb.F32)
    times = []
    for it in range(iters + 2):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dec.decode(pts, low)
        e1.record(stream)
        e1.synchronize()
        if it >= 2:
            times.append(e0.elapsed_time(e1))
    cb.profile(True)
    dec.decode(pts, low)
    cb.profile(False)
    prof = cb.profile_table()
    dec.close()
    t = statistics.median(times)
    total = sum(v["ms"] for v in prof.values())
    kernels = {k: {"share": v["ms"] / total, "launches": v["calls"],
                   "gbs": v["bytes"] / (v["ms"] * 1e-3) / 1e9,
                   "tflops": v["flops"] / (v["ms"] * 1e-3) / 1e12 if v["flops"] else None}
               for k, v in prof.items()}
    return {"prompts": MASK_P, "ms_per_decode": t, "prompts_per_s": MASK_P / (t * 1e-3),
            "kernel_ms": total,  # sum of the profiled launches' event times
            "kernels": kernels,
            "work": "cb_decode: 64 one-point prompts on one 72 x 72 image embedding, "
                    "lowres [64, 3, 288, 288] on the device, IoU to the host"}


def cpu_configs_sample():
    """Configs 1-3 on the reference's kernels (oracle/_ref) on all host
    cores, rank 0 at N=1: C1 and C2 RoPE + QK^T gemm_cpu_t + softmax_rows +
    P.V gemm_cpu_n as vit_block launches them (C2 heads chunked by
    head_chunk), C3 the attn_fewkeys / attn_manykeys kernels for one batch.
    softmax_rows runs with one work-item per group (the host executor turns
    work-group barriers into fiber switches; a one-item group needs none),
    as the tiles/s baseline does. For C3 the faster of the reference kernel
    and the oracle's restatement is reported, with its kind: attn_manykeys
    needs its 256-item work-group barriers, which the host executor runs as
    fibers, far slower than a CPU OpenCL compiler's work-item loops."""
    from oracle import binding as ob
    if not ob.have_ref():
        return None
    out = {"cores": ob.num_threads(), "kind": "reference"}
    E = 1024
    for name, side, nseq, hc in (("config1_window_9x576", 24, 9, 16),
                                 ("config2_global_5184", 72, 1, 4)):
        N = side * side
        qkv = ob.normal(SEED, 70, (nseq * N, 3 * E))
        cs = ob.rope_axial(side, 64)
        t0 = time.perf_counter()
        ob.rope_apply(qkv, E, 64, N, cs, use_ref=True)
        ob.ref_attention(qkv, nseq, N, E, 16, 64, 0.125, head_chunk=hc, softmax_local=1)
        t = time.perf_counter() - t0
        out[name] = {"s": t, "tflops": 4.0 * nseq * 16 * N * N * 64 / t / 1e12}
    for cname, nq, nk, qrows, kvrows, shared, nbytes in decoder_cases(8):
        q = ob.normal(SEED, 71, (qrows, DEC_D))
        k = ob.normal(SEED, 72, (kvrows, DEC_D))
        v = ob.normal(SEED, 73, (kvrows, DEC_D))
        skv = 0 if shared else nk * DEC_D
        best = None
        for kind, use_ref in (("reference", True), ("port", False)):
            t0 = time.perf_counter()
            ob.mha(DEC_P, nq, nk, DEC_D, q, nq * DEC_D, k, skv, v, skv, use_ref=use_ref)
            t = time.perf_counter() - t0
            if best is None or t < best[0]:
                best = (t, kind)
        out["config3_" + cname] = {"s": best[0], "gbs": nbytes / best[0] / 1e9,
                                   "kind": best[1]}
    # the whole mask decoder, oracle restatement of sam_decode (its kernels are
    # the reference's, pinned bit-exact), 2 prompts
    w = ob.DecoderWeights(SEED, 0.02)
    img = ob.decoder_image(SEED)
    pts = np.array([[100.0, 200.0], [700.0, 800.0]], np.float32)
    t0 = time.perf_counter()
    ob.sam_decode(w, *img, pts)
    t = time.perf_counter() - t0
    out["mask_decoder_2_prompts"] = {"s": t, "prompts_per_s": 2 / t, "kind": "port"}
    # the neck on one tile, oracle restatement (im2col pinned to the reference)
    x = ob.normal(SEED, 9400, (5184, 1024))
    nw = ob.NeckWeights(SEED, 0.02)
    t0 = time.perf_counter()
    ob.point_neck(nw, x, 72)
    t = time.perf_counter() - t0
    out["neck_1_tile"] = {"s": t, "tflops": 2.0 * NECK_MAC_PER_TOKEN * 5184 / t / 1e12,
                          "kind": "port"}
    img = ob.u8(SEED, 9600, (1500, 2100, 3))
    t0 = time.perf_counter()
    ob.aa_resize(img, 1008, 1008)
    out["input_resize_1_crop"] = {"s": time.perf_counter() - t0, "kind": "port"}
    # detector attention: the decoder's 201 queries with the box bias in full,
    # the fusion encoder's self-attention for one of its 8 heads (x 8)
    qd = ob.normal(SEED, 9700, (201, 256))
    kd = ob.normal(SEED, 9701, (5184, 256))
    dyb = ob.normal(SEED, 9702, (201 * 72 * 8,))
    t0 = time.perf_counter()
    ob.attend(qd, kd, kd, 8, 32, 0, dyb, dyb, 72)
    out["detector_rpb_201x5184"] = {"s": time.perf_counter() - t0, "kind": "port"}
    qf = ob.normal(SEED, 9703, (5184, 32))
    t0 = time.perf_counter()
    ob.attend(qf, qf, qf, 1, 32)
    out["detector_fusion_self_5184"] = {"s": 8 * (time.perf_counter() - t0), "kind": "port",
                                        "sample": "one head of 8, x 8"}
    return out


def cpu_baseline_sample():
    """Rank 0, N=1: the reference's CPU kernels on a bounded sample."""
    try:
        r = reference_arm(argparse.Namespace(warmup=0, steps=1), 1, 0)
    except Exception as e:  # the baseline is reported, never required
        return {"value": None, "unit": "tiles/s", "cores": 0, "kind": "reference",
                "sample": f"failed: {e}"}
    if r is None or "unavailable" in r:
        return None
    return r["cpu_baseline"]


def our_arm(args, world, rank, local, pg):
    import torch
    sb = load_product()

    torch.cuda.set_device(local)
    pk = peaks()
    cb = sb.Backend(local)
    first, n = sb.tile_shard(TOTAL_TILES, world, rank)
    enc = sb.Encoder(cb, max_tiles=n)
    enc.init_random(SEED)
    # this rank's shard of the 64 tiles, pinned host memory and device copy
    host = torch.empty(n, SIDE, SIDE, 3, dtype=torch.uint8).pin_memory()
    for i in range(n):  # the product's seeded generator (include/sam3_synth.h)
        sb.lib().sam3_synth_u8(SEED, image_stream(first + i), SIDE * SIDE * 3,
                               host[i].data_ptr())
    dev_tiles = host.cuda()
    out = torch.empty(n, 5184, 1024, dtype=torch.float32, device="cuda")
    host_out = torch.empty(n, 5184, 1024, dtype=torch.float32).pin_memory()
    torch.cuda.synchronize()
    m_tiles, m_out = cb.wrap(dev_tiles), cb.wrap(out)
    stream = torch.cuda.ExternalStream(cb.stream)

    def barrier():
        cb.sync()
        torch.cuda.synchronize()
        if pg:
            pg.barrier()

    def max_over_ranks(v):
        return sb.max_over_ranks(v, pg, "cuda")

    # configs 1 and 2 alone first, on rank 0, before the long backbone run
    # heats the GPU into its power cap: the burst conditions their peak
    # (bf16_tflops, burst) is measured under
    attn = attention_bench(sb, cb, torch, pk) if rank == 0 else None
    for _ in range(args.warmup):
        enc.encode_tiles(m_tiles, n, m_out)
    barrier()
    # `value`: the timed steps with the backend's per-launch profiler off
    with Clocks(smi_indices([local] if world == 1 else list(range(world))),
                active=rank == 0) as clk:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            enc.encode_tiles(m_tiles, n, m_out)
        e1.record(stream)
        barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    value = TOTAL_TILES * args.steps / (ms * 1e-3)

    # per-kernel shares and the roofline: the same steps again with a CUDA
    # event pair around every launch, on the launching stream
    cb.profile(True)
    p0 = torch.cuda.Event(enable_timing=True)
    p1 = torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for _ in range(args.steps):
        enc.encode_tiles(m_tiles, n, m_out)
    p1.record(stream)
    barrier()
    cb.profile(False)
    prof_ms = max_over_ranks(p0.elapsed_time(p1))
    prof = cb.profile_table()

    # end to end through the public host API: pinned host tiles in, tokens
    # out; encode_tiles_host blocks, so a host clock brackets each call
    enc.encode_tiles_host(host.numpy(), host_out.numpy())
    barrier()
    e2e_ms = []
    for _ in range(max(1, args.steps)):
        t0 = time.perf_counter()
        enc.encode_tiles_host(host.numpy(), host_out.numpy())
        t1 = time.perf_counter()
        barrier()
        e2e_ms.append((t1 - t0) * 1e3)
    e2e_step = max_over_ranks(sum(e2e_ms) / len(e2e_ms))
    e2e_value = TOTAL_TILES / (e2e_step * 1e-3)

    line = None
    if rank == 0:
        total_ms = sum(v["ms"] for v in prof.values())
        dom_name, dom = max(prof.items(), key=lambda kv: kv[1]["ms"])
        achieved = dom["flops"] / (dom["ms"] * 1e-3) / 1e12
        traffic = None
        tpath = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tpath):
            traffic = json.load(open(tpath)).get(dom_name)
        kernels = {k: {"share": v["ms"] / total_ms,
                       "tflops": v["flops"] / (v["ms"] * 1e-3) / 1e12 if v["flops"] else None,
                       "gbs": v["bytes"] / (v["ms"] * 1e-3) / 1e9,
                       "launches": v["calls"]} for k, v in prof.items()}
        dec = decoder_bench(cb, torch, pk)
        mdec = mask_decoder_bench(sb, cb, torch)
        nk = neck_bench(sb, cb, torch)
        inp = input_bench(sb, cb, torch)
        det = detector_attention_bench(sb, cb, torch, pk)
        line = {
            "metric": METRIC, "value": value, "unit": "tiles/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded uint8 tiles, random-init N(0,0.02) weights)",
            "config": {"workload": "config 5: 64 tiles x 32-block PE backbone, sharded "
                                   f"{n} tiles/GPU", "tiles": TOTAL_TILES, "tiles_per_gpu": n,
                       "parallelism": f"tile-sharded x{world}, no collective",
                       "l2": "inputs larger than L2 (805 MB weights + activations per step)"},
            "backbone_tflops": value * TILE_FLOP / 1e12,
            "roofline": {"bound": "tensor", "kernel": dom_name, "achieved": achieved,
                         "peak": pk["bf16_sus"], "unit": "TFLOP/s",
                         "frac": achieved / pk["bf16_sus"],
                         "peak_source": f"{pk['src']} bf16_tflops_sustained",
                         "traffic": traffic,
                         "timing": "CUDA events around each launch in a second pass of "
                                   f"the same {args.steps} steps ({prof_ms / args.steps:.1f} "
                                   "ms/step with the events vs "
                                   f"{ms / args.steps:.1f} without)"},
            "kernels": kernels,
            "attention": attn,
            "decoder_attention": dec,
            "mask_decoder": mdec,
            "neck": nk,
            "input_path": inp,
            "detector_attention": det,
            "e2e": {"value": e2e_value, "unit": "tiles/s", "timing": "host clock around "
                    "each blocking encode_tiles_host call, max over ranks",
                    "h2d_bytes_per_step": TOTAL_TILES * SIDE * SIDE * 3,
                    "d2h_bytes_per_step": TOTAL_TILES * 5184 * 1024 * 4},
            "gpu_launches": int(sum(v["calls"] for v in prof.values())),  # per timed region
            "clocks": clk.summary(),
        }
    enc.close()
    cb.close()
    return line


def profile_case(ntile):
    """Small case for ncu captures: a 2-block trunk (one windowed, one global
    block) on `ntile` tiles, encoded twice. Per encode the launches are
    patch_in, gemm (patch), layernorm, then per block layernorm, gemm (qkv),
    attention, gemm (proj), layernorm, gemm (fc1), gemm (fc2), and the final
    unpermute; so with -k regex:gemm_bf16 the 13th GEMM launch is the second
    encode's fc1, and with -k regex:attn_tc launches 3-4 are the second
    encode's windowed and global attention."""
    import torch
    sb = load_product()
    cb = sb.Backend(0)
    enc = sb.Encoder(cb, max_tiles=ntile, depth=2, global_blocks=(1,))
    enc.init_random(SEED)
    tiles = torch.empty(ntile, SIDE, SIDE, 3, dtype=torch.uint8)
    for i in range(ntile):
        sb.lib().sam3_synth_u8(SEED, image_stream(i), SIDE * SIDE * 3, tiles[i].data_ptr())
    dev = tiles.cuda()
    out = torch.empty(ntile, 5184, 1024, device="cuda")
    torch.cuda.synchronize()
    for _ in range(2):
        enc.encode_tiles(cb.wrap(dev), ntile, cb.wrap(out))
    cb.sync()
    enc.close()
    cb.close()
    print(f"profile case done: {ntile} tiles, 2 blocks, 2 encodes")


def profile_part(part):
    """Small cases of the parts beyond the backbone for ncu captures, each
    run twice (the second run is the one to capture): `decoder` = cb_decode
    of 16 prompts, `neck` = cb_neck_run on 2 tiles, `detector` = the two
    cb_attend shapes of the bench, `input` = one 2100 x 1500 crop,
    `elementwise` = the backbone's element-wise kernels (patch_embed_in,
    LayerNorm, the RoPE + bf16 cast of the fp32 attention op),
    `decoder_attention` = config 3's two cb_mha forms at 64 prompts."""
    import torch
    sb = load_product()
    cb = sb.Backend(0)
    T = 5184
    if part == "decoder":
        dec = sb.Decoder(cb, 16)
        dec.init_random(SEED, 0.02)
        feats = []
        for k, n in enumerate((T * 256, 16 * T * 32, 4 * T * 64)):
            m = cb.alloc(n * 4, sb.F32)
            cb.synth_normal(SEED, 9216 + k, 0.0, 1.0, m, n)
            feats.append(m)
        dec.set_image(*feats)
        pts = np.random.default_rng(SEED).uniform(0, 1008, size=(16, 2)).astype(np.float32)
        low = cb.alloc(16 * 3 * 288 * 288 * 4, sb.F32)
        for _ in range(2):
            dec.decode(pts, low)
        dec.close()
    elif part == "neck":
        neck = sb.Neck(cb, grid=72, embed=1024, max_tiles=2)
        neck.init_random(SEED, 0.02)
        x = cb.alloc(2 * T * 1024 * 4, sb.F32)
        cb.synth_normal(SEED, 9400, 0.0, 1.0, x, 2 * T * 1024)
        outs = [cb.alloc(2 * T * 256 * 4, sb.F32), cb.alloc(2 * 16 * T * 32 * 4, sb.F32),
                cb.alloc(2 * 4 * T * 64 * 4, sb.F32)]
        for _ in range(2):
            neck.run(x, 2, *outs)
        neck.close()
    elif part == "detector":
        for _ in range(2):
            detector_attention_bench(sb, cb, torch, None, iters=1)
    elif part == "decoder_attention":
        # config 3's cb_mha forms at 64 prompts, two calls each: token ->
        # image over per-prompt K/V (split + merge), then image -> token
        P, N, D = DEC_P, DEC_NK, DEC_D
        g = torch.Generator(device="cuda").manual_seed(SEED + 3)
        for nq, nk, qrows, kvrows in ((8, N, P * 8, P * N), (N, 8, P * N, P * 8)):
            q = torch.randn(qrows, D, device="cuda", generator=g)
            k = torch.randn(kvrows, D, device="cuda", generator=g)
            v = torch.randn(kvrows, D, device="cuda", generator=g)
            o = torch.empty(qrows, D, device="cuda")
            torch.cuda.synchronize()
            mq, mk, mv, mo = cb.wrap(q), cb.wrap(k), cb.wrap(v), cb.wrap(o)
            for _ in range(2):
                cb.mha(P, nq, nk, D, mq, nq * D, mk, nk * D, mv, nk * D, mo)
            cb.sync()
    elif part == "input":
        for _ in range(2):
            input_bench(sb, cb, torch, iters=1)
    elif part == "elementwise":
        # the element-wise kernels on inputs larger than L2: 4 tiles through a
        # 1-block trunk (patch_embed_in, ln_pre and the two block LayerNorms
        # on 20736 x 1024 rows), then config 2's fp32 attention op, whose
        # RoPE + bf16 cast pass (rope_cast) reads the 64 MB fp32 qkv
        enc = sb.Encoder(cb, max_tiles=4, depth=1, global_blocks=(0,))
        enc.init_random(SEED)
        tiles = torch.empty(4, SIDE, SIDE, 3, dtype=torch.uint8)
        for i in range(4):
            sb.lib().sam3_synth_u8(SEED, image_stream(i), SIDE * SIDE * 3, tiles[i].data_ptr())
        dev = tiles.cuda()
        out = torch.empty(4, T, 1024, device="cuda")
        qkv = torch.randn(T, 3 * 1024, device="cuda")
        cs = torch.empty(T * 64, dtype=torch.float32)
        sb.lib().sam3_synth_rope_axial(72, 64, 10000.0, cs.data_ptr())
        cs = cs.cuda()
        o = torch.empty(T, 1024, device="cuda")
        torch.cuda.synchronize()
        for _ in range(2):
            enc.encode_tiles(cb.wrap(dev), 4, cb.wrap(out))
            cb.attention(cb.wrap(qkv), 1, T, 1024, 16, 64, cb.wrap(cs), T, 0.125, sb.ATTN_TC,
                         cb.wrap(o))
        enc.close()
    cb.sync()
    cb.close()
    print(f"profile part done: {part}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-case", type=int, default=0, metavar="TILES",
                    help="run the small ncu case on TILES tiles and exit")
    ap.add_argument("--profile-part", choices=["decoder", "neck", "detector", "input", "elementwise",
                                               "decoder_attention"],
                    help="run a small case of one part (beyond the backbone, or its "
                         "element-wise kernels) and exit")
    args = ap.parse_args()
    if args.profile_part:
        profile_part(args.profile_part)
        return
    if args.profile_case:
        profile_case(args.profile_case)
        return
    world, rank, local, pg = dist_setup(args)
    if args.impl == "reference":
        line = reference_arm(args, world, rank)
    else:
        line = our_arm(args, world, rank, local, pg)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample()
            try:
                line["cpu_configs"] = cpu_configs_sample()
            except Exception as e:  # reported, never required
                line["cpu_configs"] = {"failed": str(e)}
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
