#!/usr/bin/env python3
"""Encoder throughput benchmark (frames/s) of the B200 engine for sam3.cpp.

Headline: SAM 3 ViT-L image encoder + tracker SimpleFPN neck, q4_0 weights
(seeded synthetic, random-init), a 64-frame batch of seeded 1008x1008 frames split 64/N over N GPUs (strong
scaling; one process per GPU, no data-path collective). One step = encode the rank's frames; `value` = 64 /
the slowest rank's step time. The q4_0 weights stay in block form in HBM (engine option weights_quantised = 1:
each layer's weight is dequantised into an L2-resident f16 staging buffer right before its GEMM).

The same line carries the other configurations:
  vit_f16_b1       configs[2]: SAM 3 ViT-L f16, batch 1 (latency)
  hiera_t_f16_b1   configs[0]: SAM 2.1 Hiera-T f16, batch 1 (latency)
  hiera_t_q4_0     configs[1]: SAM 2.1 Hiera-T q4_0, 16 frames per GPU
  video_hiera_l_q8_0  configs[4]: Hiera-L q8_0 on 64 frames over the GPUs, each frame's neck_trk_0/1/2 moved
                   to the tracking GPU (rank 0) over NVLink (CUDA IPC + peer copy), one tracking step per
                   frame there (memory attention from a device-resident memory bank, SAM mask decoder,
                   memory encoder, object pointer: s3b_track_step); the end-to-end pipeline rate and its
                   limiter.

  python bench.py [--gpus N] [--steps K] [--warmup W]
  python bench.py --impl reference ...   # the CPU restatement (oracle) of the same path, timed

`value` is measured with the frames resident in HBM; `e2e` goes through the public C ABI with pinned host
frames every step (s3b_encode_u8: host->device copy inside the timed region) and reads back neck_trk_0..2
(f32, the maps sam3_propagate_single hands downstream) of every frame into pinned host memory through
s3b_output_host_bind (copies overlap the next encoder pass). Inputs plus activations per step are far
larger than L2 (126 MB), so no separate flush is added.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
FRAMES_TOTAL = 64
# 1: q4_0 / q8_0 linear weights stay in block form in HBM and each layer's weight is dequantised into an
# f16 staging buffer (L2-resident) before its GEMM; 2: the GEMM dequantises in shared memory; 0: f16 at load
WEIGHTS_QUANTISED = 1
WEIGHTS_DESC = {0: "f16, dequantised once at load",
                1: "block form (q4_0 / q8_0 planes); each layer dequantised into an L2-resident f16 staging "
                   "buffer right before its GEMM",
                2: "block form; dequantised inside the GEMM's shared-memory stages"}
# measured with ncu (one --set full capture of ViT block 0): mean DRAM read+write per launch of the
# qkv / proj / fc1 / fc2 GEMMs of a ViT block at 8 frames per pass, and their algorithmic bytes
GEMM_TRAFFIC_BYTES = 4.728e8  # (294.5 + 374.3 + 435.7 + 786.5) MB / 4
GEMM_ALG_BYTES = 5.007e8  # (346.4 + 426.8 + 487.4 + 742.3) MB / 4


def load_pkg():
    name = "sam3_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = os.path.join(ROOT, "sam3.cpp_b200")
    spec = importlib.util.spec_from_file_location(name, os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def shard_frames(total: int, rank: int, world: int) -> tuple[int, int]:
    """Frames [first, first + count) encoded by `rank`: contiguous blocks whose sizes differ by at most one;
    frame f keeps its seed on any world size."""
    first = total * rank // world
    return first, total * (rank + 1) // world - first


def rank_frames(per_gpu: int, rank: int) -> tuple[int, int]:
    """Frames [first, first + per_gpu) of `rank` when every rank encodes per_gpu frames of its own."""
    return rank * per_gpu, per_gpu


def max_over_ranks(x: float, world: int, device) -> float:
    """Max of a per-rank time over all ranks (the job's time); identity on one rank."""
    if world <= 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


class _CudaArray:
    """Zero-copy view of engine-owned device memory for torch.as_tensor (the CUDA array interface)."""

    def __init__(self, ptr: int, n: int, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


def model_file(s3b, kind: str) -> str:
    """Seeded synthetic .ggml files of the configurations (written once per box under the temp dir)."""
    import dataclasses
    from sam3_b200 import synth
    path = os.path.join(tempfile.gettempdir(), f"s3b_bench_{kind}_v2.ggml")
    if os.path.exists(path):
        return path
    tmp = path + f".tmp{os.getpid()}"
    if kind in ("vit_q4_0", "vit_q8_0", "vit_f16"):
        qtype = {"vit_q4_0": 2, "vit_q8_0": 8, "vit_f16": None}[kind]
        synth.write_sam3(tmp, synth.SAM3_VIT_L, seed=0, ftype=1, qtype=qtype, quantize=s3b.quantize_rows)
    elif kind in ("hiera_t_q4_0", "hiera_t_f16"):
        synth.write_sam2(tmp, synth.HIERA_T, seed=0, ftype=1, qtype=2 if kind == "hiera_t_q4_0" else None,
                         quantize=s3b.quantize_rows)
    elif kind == "hiera_l_q8_0":
        # the video configuration carries the tracker: memory attention, SAM mask decoder, memory encoder
        from sam3_b200 import ggml_io
        cfg = dataclasses.replace(synth.HIERA_L, with_mem_attn=True, with_sam_dec=True)
        T = synth.sam2_tensors(cfg, seed=0)
        T.update(synth.mem_enc_tensors(1))
        synth.write_model(tmp, T, cfg.hparams(), ggml_io.MAGIC_SAM2, 1, 1, 8, s3b.quantize_rows)
    else:
        raise ValueError(kind)
    os.replace(tmp, path)
    return path


def prepare_models(s3b, kinds, local, world):
    """Local rank 0 writes the model files; the other ranks wait for them."""
    if local == 0:
        for k in kinds:
            model_file(s3b, k)
    barrier(world)
    return {k: model_file(s3b, k) for k in kinds}


def vit_flops_per_frame(cfg, with_neck=True):
    """Algorithmic FLOPs of one frame (2*M*N*K per GEMM, 4*Nq*Nk*d per attention head)."""
    G, E, M = cfg.grid, cfg.embed, cfg.mlp
    T = G * G
    hd = E // cfg.heads
    gemm = 2 * T * 588 * E  # patch embed
    attn = 0
    for i in range(cfg.depth):
        gemm += 2 * T * E * (3 * E + E + 2 * M)
        n = T if i in cfg.global_idx else cfg.window ** 2
        nwin = 1 if i in cfg.global_idx else (G // cfg.window) ** 2
        attn += 4 * nwin * cfg.heads * n * n * hd
    neck = 0
    if with_neck:
        D, mid = cfg.neck_dim, cfg.neck_mid
        neck += 2 * T * E * 4 * mid + 2 * 4 * T * mid * 4 * D + 2 * 16 * T * D * D + 2 * 16 * T * 9 * D * D
        neck += 2 * T * E * 4 * mid + 2 * 4 * T * mid * D + 2 * 4 * T * 9 * D * D
        neck += 2 * T * E * D + 2 * T * 9 * D * D
        neck += 2 * (T // 4) * E * D + 2 * (T // 4) * 9 * D * D
    return gemm, attn, neck


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    def __init__(self, index: int):
        self.path = tempfile.mktemp(suffix=".csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def timed_calls(eng, stream, fn, steps, world, profiled):
    """Device time of `steps` calls of fn on `stream` (CUDA events, barrier + synchronize on both sides, max
    over ranks), in ms per call, and the engine's launch profile of those calls. Unprofiled calls replay the
    encoder's CUDA graph (what a caller gets); profiled calls (CUDA events around every launch, the kernel
    breakdown and roofline) run eagerly."""
    import torch
    barrier(world)
    torch.cuda.synchronize()
    eng.profile_begin(profiled)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    prof = eng.profile_end()
    return max_over_ranks(e0.elapsed_time(e1) / steps, world, "cuda"), prof


def tflops(part):
    return part["flops"] / (part["ms"] / 1000.0) / 1e12 if part["ms"] > 0 else 0.0


# ---------------------------------------------------------------- CPU reference (oracle port)
def cpu_reference(workload: str, steps: int, warmup: int) -> dict:
    """Times the CPU restatement of the path (oracle, numpy; BLAS on every host core) on configs[3]'s
    per-frame forward, for real: one step = one eighth of a frame's forward, four of the 32 ViT blocks
    in order (the prefix rides with the first eighth, the tracker neck with the last), so eight steps
    compute one complete frame. The reference's own CPU backend (ggml) is not in the checkout."""
    from threadpoolctl import threadpool_limits
    cores = os.cpu_count() or 1
    sys.path.insert(0, ROOT)
    load_pkg()
    from oracle import quant as oq
    from oracle import vit as ov
    from sam3_b200 import synth
    cfg = synth.SAM3_VIT_L
    qtype = {"vit_q4_0": 2, "vit_q8_0": 8, "vit_f16": None}[workload]
    t_setup = time.perf_counter()
    W = synth.stored_values(synth.sam3_tensors(cfg, seed=0), 1, qtype, oq.quantize, oq.dequantize)
    setup_s = time.perf_counter() - t_setup
    per = cfg.depth // 8

    state = {"x": None, "frame": 0}

    def eighth(e):
        if e == 0:
            chw = ov.preprocess_u8(synth.frames_u8(1, cfg.img_size, base_seed=1000 + state["frame"]))
            state["x"] = ov.prefix(W, chw, cfg)
        for b in range(e * per, (e + 1) * per):
            state["x"] = ov.block(W, state["x"], b, cfg)
        if e == 7:
            ov.neck(W, state["x"])
            state["frame"] += 1

    with threadpool_limits(limits=cores):
        for k in range(warmup):
            eighth(k % 8)
        # the timed steps start a fresh frame
        step_s = []
        t0 = time.perf_counter()
        for k in range(steps):
            t = time.perf_counter()
            eighth(k % 8)
            step_s.append(time.perf_counter() - t)
        total = time.perf_counter() - t0
    frames = steps / 8.0
    return {"value": frames / total, "ms_per_step": 1000.0 * total / steps, "total_s": total, "frames": frames,
            "cores": cores, "setup_s": setup_s,
            "sample": f"{steps} timed eighths of the SAM 3 ViT-L + tracker-neck forward ({frames:g} frame(s)), "
                      f"each eighth 4 of the 32 blocks in order (prefix with the first, neck with the last); "
                      f"per-step seconds min {min(step_s):.2f} max {max(step_s):.2f}; oracle (numpy f32, "
                      f"BLAS threads = {cores}); weights {workload.split('_', 1)[1]} (dequantised)"}


# ---------------------------------------------------------------- GPU measurements
def bench_vit(s3b, path, args, rank, world, local, stream) -> dict:
    """64 frames split 64/N; device-resident timing, then e2e through the public API."""
    import torch
    from sam3_b200 import synth
    cfg = synth.SAM3_VIT_L
    first, nf = shard_frames(args.frames, rank, world)
    eng = s3b.Engine(local)
    eng.set_option("weights_quantised", args.weights_quantised)
    eng.set_option("frames_per_pass", min(args.frames_per_pass, max(nf, 1)))
    eng.set_option("gemm_pairs", args.gemm_pairs)
    t0 = time.time()
    eng.load_model(path)
    load_s = time.time() - t0
    # the persistent device-weight cache: written by a first cached load, then a timed load from it
    cache = os.path.join(tempfile.gettempdir(), f"s3b_bench_{args.workload}_wq{args.weights_quantised}_{local}.s3bc")
    ce = s3b.Engine(local)
    ce.set_option("weights_quantised", args.weights_quantised)
    ce.load_model_cached(path, cache)
    t0 = time.time()
    cache_hit = ce.load_model_cached(path, cache)
    load_cached_s = time.time() - t0
    ce.close()
    host = synth.frames_u8(nf, cfg.img_size, base_seed=1000 + first)
    host_t = torch.from_numpy(host).pin_memory()
    dev = host_t.cuda()
    for _ in range(args.warmup):
        eng.encode_u8(dev)
    eng.sync()

    # --- timed region (device-resident inputs): the headline, every call replayed from the encoder's CUDA
    # graph; then the same steps again with CUDA events around every launch (kernel breakdown, roofline)
    eng.set_stream(stream.cuda_stream)
    enc = lambda: eng.encode_u8(dev)
    clocks = ClockSampler(local)
    ms, prof_plain = timed_calls(eng, stream, enc, args.steps, world, False)
    clk = clocks.stop()
    prof_ms, prof = timed_calls(eng, stream, enc, args.steps, world, True)
    value = args.frames / (ms / 1000.0)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # --- end to end through the public API: pinned host frames in, neck_trk_0..2 (f32) of every frame out
    G = cfg.grid
    sizes = [4 * G, 2 * G, G]
    outs = {f"neck_trk_{i}": torch.empty(nf, S, S, cfg.neck_dim, dtype=torch.float32).pin_memory()
            for i, S in enumerate(sizes)}
    for n, t in outs.items():
        eng.output_host_bind(n, t)
    eng.encode_u8(host_t.numpy())  # one untimed call with the bindings in place
    eng.sync()
    barrier(world)
    torch.cuda.synchronize()
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host_np = host_t.numpy()
    ev2.record(stream)
    for _ in range(args.steps):
        eng.encode_u8(host_np)  # H2D inside the public call; outputs land in `outs` per pass
    eng.sync()  # the last pass's read-back included
    ev3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(ev2.elapsed_time(ev3) / args.steps, world, "cuda")
    # the read-back is the real output: spot-check one frame against s3b_output_copy
    readback_ok = bool(np.array_equal(outs["neck_trk_2"][nf - 1].numpy(), eng.output("neck_trk_2", nf - 1)))
    for n in outs:
        eng.output_host_bind(n, None)
    d2h = sum(int(t.numel()) * 4 for t in outs.values())

    peak_burst, peak_sust, hbm, src = measured_peaks()
    g, a, ln, wst = prof["gemm"], prof["attention"], prof["layernorm"], prof["weight_staging"]
    gemm_tf = tflops(g)
    fl_gemm, fl_attn, fl_neck = vit_flops_per_frame(cfg)
    line = {
        "value": value, "ms_per_step": ms,
        "timing": {"value": "CUDA events around K steps, every encoder call replayed from its CUDA graph",
                   "profiled_ms_per_step": prof_ms,
                   "profiled": "the same K steps again with CUDA events around every launch (eager): the kernel "
                               "times behind roofline, attention, layernorm and weight_staging"},
        "e2e": {"value": args.frames / (e2e_ms / 1000.0), "unit": "frames/s", "h2d_bytes_per_step": int(host.nbytes),
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "outputs_read_back": "neck_trk_0, neck_trk_1, neck_trk_2 (f32, every frame), via s3b_output_host_bind",
                "readback_matches_output_copy": readback_ok},
        "roofline": {"bound": "tensor", "achieved": gemm_tf, "peak": peak_sust, "unit": "TFLOP/s",
                     "frac": gemm_tf / peak_sust,
                     # DRAM bytes per GEMM launch (read + write), mean of the four block-0 GEMMs at 8 frames
                     # from one ncu capture of ViT block 0; algorithmic 5.0e8
                     "traffic": GEMM_TRAFFIC_BYTES, "traffic_algorithmic": GEMM_ALG_BYTES,
                     "kernel": "gemm_f16_tc_kernel (tcgen05/TMEM, TMA)",
                     "peak_source": f"{src} bf16_tflops_sustained (kernel timed inside a long step)",
                     "gemm_ms_per_step": g["ms"] / args.steps, "gemm_launches_per_step": g["launches"] / args.steps},
        "attention": {"achieved_tflops": tflops(a), "ms_per_step": a["ms"] / args.steps,
                      "frac_of_peak": tflops(a) / peak_sust},
        "layernorm": {"achieved_gbs": ln["bytes"] / (ln["ms"] / 1000.0) / 1e9 if ln["ms"] > 0 else 0.0,
                      "peak_gbs": hbm, "frac_of_peak": (ln["bytes"] / (ln["ms"] / 1000.0) / 1e9 / hbm)
                      if ln["ms"] > 0 else 0.0, "ms_per_step": ln["ms"] / args.steps,
                      "launches_per_step": ln["launches"] / args.steps,
                      "bound": "hbm (algorithmic bytes: f32 rows in + f16 rows out)"},
        "weight_staging": {"ms_per_step": wst["ms"] / args.steps, "launches_per_step": wst["launches"] / args.steps,
                           "achieved_gbs": wst["bytes"] / (wst["ms"] / 1000.0) / 1e9 if wst["ms"] > 0 else 0.0,
                           "what": "block-form weight planes read from HBM, f16 staging written (L2)"},
        "whole_step_tflops": (fl_gemm + fl_attn + fl_neck) * value / 1e12, "flops_per_frame": fl_gemm + fl_attn + fl_neck,
        "gpu_launches": int(prof_plain["launches"]), "clocks": clk,
        "setup": {"load_s": load_s, "load_cached_s": load_cached_s if cache_hit else None,
                  "weights_mib": eng.model_info()["weights_mib"], "frames_this_rank": nf}}
    eng.set_stream(None)
    eng.close()
    return line


def bench_latency(s3b, path, label, img, args, rank, world, local, stream) -> dict:
    """Batch-1 latency: one frame per call, K calls back to back (device-resident frame)."""
    import torch
    from sam3_b200 import synth
    eng = s3b.Engine(local)
    eng.set_option("frames_per_pass", 1)
    eng.load_model(path)
    frame = torch.from_numpy(synth.frames_u8(1, img, base_seed=1000 + rank)).cuda()
    eng.set_stream(stream.cuda_stream)
    for _ in range(args.warmup):
        eng.encode_u8(frame)
    eng.sync()
    enc = lambda: eng.encode_u8(frame)
    ms, _ = timed_calls(eng, stream, enc, args.steps, world, False)
    prof_ms, prof = timed_calls(eng, stream, enc, args.steps, world, True)
    eng.set_stream(None)
    eng.close()
    g, a = prof["gemm"], prof["attention"]
    return {"workload": label, "latency_ms": ms, "frames_per_s_per_gpu": 1000.0 / ms,
            "latency_ms_profiled": prof_ms,
            "timing": "CUDA events around K back-to-back calls replayed from the encoder's CUDA graph; the kernel "
                      "rates from the same calls again with CUDA events around every launch (eager)",
            "gemm_tflops": tflops(g), "attention_tflops": tflops(a),
            "algorithmic_tflop_per_frame": (g["flops"] + a["flops"]) / args.steps / 1e12,
            "gpu_launches_per_frame": prof["launches"] / args.steps}


HIERA_FRAMES_PER_GPU = 16


def bench_hiera(s3b, path, args, rank, world, local, stream) -> dict:
    """SAM 2.1 Hiera-T + FPN neck, q4_0, a batch of 16 seeded 1024^2 frames per GPU."""
    import torch
    from sam3_b200 import synth
    eng = s3b.Engine(local)
    eng.set_option("weights_quantised", args.weights_quantised)
    eng.set_option("frames_per_pass", HIERA_FRAMES_PER_GPU)
    eng.load_model(path)
    n = HIERA_FRAMES_PER_GPU
    frames = torch.from_numpy(synth.frames_u8(n, 1024, base_seed=1000 + rank * n)).cuda()
    eng.set_stream(stream.cuda_stream)
    for _ in range(args.warmup):
        eng.encode_u8(frames)
    eng.sync()
    enc = lambda: eng.encode_u8(frames)
    ms, _ = timed_calls(eng, stream, enc, args.steps, world, False)
    prof_ms, prof = timed_calls(eng, stream, enc, args.steps, world, True)
    g, a = prof["gemm"], prof["attention"]
    eng.set_stream(None)
    eng.close()
    return {"workload": f"configs[1]: SAM 2.1 Hiera-T image encoder + FPN neck, q4_0 weights "
                        f"({WEIGHTS_DESC[args.weights_quantised]}), {n} seeded 1024^2 frames per GPU "
                        f"(device-resident) x {world} GPU(s)",
            "value": n * world / (ms / 1000.0), "unit": "frames/s", "ms_per_step": ms,
            "profiled_ms_per_step": prof_ms, "gemm_tflops": tflops(g), "gemm_ms_per_step": g["ms"] / args.steps,
            "attention_tflops": tflops(a), "attention_ms_per_step": a["ms"] / args.steps,
            "algorithmic_tflop_per_step": (g["flops"] + a["flops"]) / args.steps / 1e12,
            "gpu_launches_per_step": prof["launches"] / args.steps}


def bench_video(s3b, path, args, rank, world, local, stream) -> dict:
    """Hiera-L q8_0 on 64 frames over N GPUs, then per-frame memory attention on the tracking GPU
    (rank 0) from a device-resident memory bank (7 slots of 64x64x64 + 16 object pointers: M = 28,736).

    Encoder throughput: every rank encodes its share of the 64 frames (64/N).
    Pipeline (N > 1): ranks 1..N-1 encode the 64 frames of step k and copy each frame's neck_trk_2 (4 MB)
    into rank 0's receive buffer k % 2 over NVLink (CUDA IPC + s3b_peer_copy_output); meanwhile rank 0 runs
    memory attention on the 64 frames of step k - 1 from buffer (k - 1) % 2. A host barrier between steps
    orders the two. With N = 1 one GPU does both, one after the other. Rate = 64 frames x K steps / the
    slowest rank's time; the copies' contents are checked against the encoders' outputs."""
    import torch
    import torch.distributed as dist
    from sam3_b200 import synth
    cfg = synth.HIERA_L
    eng = s3b.Engine(local)
    eng.set_option("weights_quantised", args.weights_quantised)
    eng.load_model(path)
    out = {"workload": f"configs[4]: SAM 2.1 Hiera-L image encoder + FPN neck, q8_0 weights "
                       f"({WEIGHTS_DESC[args.weights_quantised]}), {FRAMES_TOTAL} seeded 1024^2 frames over "
                       f"{world} GPU(s); memory attention per frame on GPU 0 from a device memory bank"}

    # --- encoder throughput (every rank its 64/N share)
    first, nf = shard_frames(FRAMES_TOTAL, rank, world)
    frames = torch.from_numpy(synth.frames_u8(nf, 1024, base_seed=1000 + first)).cuda()
    eng.set_stream(stream.cuda_stream)
    for _ in range(args.warmup):
        eng.encode_u8(frames)
    eng.sync()
    enc = lambda: eng.encode_u8(frames)
    ms, _ = timed_calls(eng, stream, enc, args.steps, world, False)
    _, prof = timed_calls(eng, stream, enc, args.steps, world, True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out.update({"encoder_frames_per_s": FRAMES_TOTAL / (ms / 1000.0), "encoder_ms_per_step": ms,
                "encoder_gemm_tflops": tflops(prof["gemm"]), "encoder_attention_tflops": tflops(prof["attention"])})

    # --- the tracker's per-frame work on the tracking GPU (rank 0), from a device memory bank (seeded):
    # 7 slots [4096][64] (slot 0 the conditioning frame), 16 object pointers [256]
    feat, n_slots, n_ptrs = 64, cfg.num_maskmem, cfg.max_obj_ptrs
    levels = [("neck_trk_0", 4 * feat), ("neck_trk_1", 2 * feat), ("neck_trk_2", feat)]
    lbytes = [s * s * 256 * 4 for _, s in levels]
    fbytes = sum(lbytes)  # the three feature maps a tracking step reads
    slot_tpos = [0] + [n_slots - s for s in range(1, n_slots)]
    ptr_tpos = list(range(1, n_ptrs + 1))

    def timed(fn, n):
        for _ in range(max(args.warmup, 2)):
            fn()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    if rank == 0:
        g2 = torch.Generator(device="cuda").manual_seed(5)
        bank = [torch.randn(feat * feat, 64, device="cuda", generator=g2) for _ in range(n_slots)]
        ptrs = torch.randn(n_ptrs, 256, device="cuda", generator=g2)
        lv = [torch.from_numpy(eng.output(name, 0).reshape(-1, 256)).cuda() for name, _ in levels]
        res = torch.empty_like(lv[2])
        touts = {"mask": torch.empty(16 * feat * feat, device="cuda"), "scores": torch.empty(3, device="cuda"),
                 "mem": torch.empty(feat * feat, 64, device="cuda"), "ptr": torch.empty(256, device="cuda")}
        dec_outs = (torch.empty(4, 4 * feat, 4 * feat, device="cuda"), torch.empty(4, device="cuda"),
                    torch.empty(1, device="cuda"), torch.empty(4, 256, device="cuda"))
        mms = timed(lambda: eng.mem_attn_bank(lv[2], feat, bank, slot_tpos, ptrs, ptr_tpos, out=res), args.steps)
        dms = timed(lambda: eng.sam_decode(feat, res, lv[0], lv[1], None, outs=dec_outs), args.steps)
        ems = timed(lambda: eng.mem_encode(feat, lv[2], dec_outs[0][0], dec_outs[2], out=touts["mem"]), args.steps)
        tms = timed(lambda: eng.track_step(feat, lv[0], lv[1], lv[2], bank, slot_tpos, ptrs, ptr_tpos, outs=touts),
                    args.steps)
        eng.profile_begin(True)
        eng.mem_attn_bank(lv[2], feat, bank, slot_tpos, ptrs, ptr_tpos, out=res)
        torch.cuda.synchronize()
        p2 = eng.profile_end()
        fl = p2["gemm"]["flops"] + p2["attention"]["flops"]
        eng.profile_begin(False)
        eng.track_step(feat, lv[0], lv[1], lv[2], bank, slot_tpos, ptrs, ptr_tpos, outs=touts)
        torch.cuda.synchronize()
        p3 = eng.profile_end()
        out.update({"mem_attn_ms_per_frame": mms, "mem_attn_tflop_per_frame": fl / 1e12,
                    "mem_attn_tflops": fl / (mms / 1000.0) / 1e12, "mem_attn_attention_tflops": tflops(p2["attention"]),
                    "mem_attn_memory_tokens": n_slots * feat * feat + 4 * n_ptrs,
                    "mask_decoder_ms_per_frame": dms, "memory_encoder_ms_per_frame": ems,
                    "track_step_ms_per_frame": tms, "track_step_launches": p3["launches"],
                    "track_timing": "CUDA events around the timed calls; s3b_mem_attn_bank (prompt built on the "
                                    "device from the bank, layers replayed from a CUDA graph), s3b_sam_decode, "
                                    "s3b_mem_encode, and s3b_track_step = all of them + the mask choice + the "
                                    "object pointer"})

    # --- the pipeline: encode, hand the three feature maps to the tracking GPU, one tracking step per frame
    encoders = list(range(1, world)) if world > 1 else [0]
    e_idx = encoders.index(rank) if rank in encoders else -1
    efirst, enf = shard_frames(FRAMES_TOTAL, e_idx, len(encoders)) if e_idx >= 0 else (0, 0)
    if enf:
        eframes = torch.from_numpy(synth.frames_u8(enf, 1024, base_seed=1000 + efirst)).cuda()
    recv = None
    if rank == 0 and world > 1:
        recv = eng.device_alloc(2 * FRAMES_TOTAL * fbytes)
        handle = [eng.ipc_export(recv)]
    else:
        handle = [None]
    if world > 1:
        dist.broadcast_object_list(handle, src=0)
    dst_base = None if world == 1 else (recv if rank == 0 else eng.ipc_open(handle[0]))

    def frame_slot(base, f):
        return [base + f * fbytes + sum(lbytes[:i]) for i in range(3)]

    def encode_step(k):
        if not enf:
            return
        eng.encode_u8(eframes)
        if world == 1:
            return
        buf = dst_base + (k % 2) * FRAMES_TOTAL * fbytes
        for f in range(enf):
            for (name, _), dst, nb in zip(levels, frame_slot(buf, efirst + f), lbytes):
                eng.peer_copy_output(name, f, dst, 0, nb)

    def track_frames(k):
        for f in range(FRAMES_TOTAL):
            if world == 1:
                t = [eng.output_device_ptr(name, f) for name, _ in levels]
            else:
                t = frame_slot(recv + (k % 2) * FRAMES_TOTAL * fbytes, f)
            # the step's memory and pointer go back into the bank rings (slot 0 stays the conditioning frame)
            touts["mem"] = bank[1 + f % (n_slots - 1)]
            touts["ptr"] = ptrs[f % n_ptrs]
            eng.track_step(feat, t[0], t[1], t[2], bank, slot_tpos, ptrs, ptr_tpos, outs=touts)

    def pipeline_step(k):
        if world == 1:
            encode_step(k)
            track_frames(k)
        else:
            encode_step(k)
            if rank == 0 and k > 0:
                track_frames(k - 1)
        eng.sync()
        barrier(world)

    n_warm = max(args.warmup, 2)
    for k in range(n_warm):
        pipeline_step(k)
    barrier(world)
    torch.cuda.synchronize()
    e0.record(stream)
    steps = args.steps
    for k in range(n_warm, n_warm + steps):
        pipeline_step(k)
    e1.record(stream)
    torch.cuda.synchronize()
    pms = max_over_ranks(e0.elapsed_time(e1) / steps, world, "cuda")
    # content check (N > 1): the frames rank 0 tracked in the last step came from the encoders' last outputs
    ok = None
    if world > 1:
        last = n_warm + steps - 1  # buffer last % 2 holds the frames encoded in step `last`
        sums = []
        for f in range(enf):
            for (name, s), nb in zip(levels, lbytes):
                p = eng.output_device_ptr(name, f)
                v = torch.as_tensor(_CudaArray(p, nb // 4, "<i4"), device="cuda")
                sums.append((efirst + f, name, int(v.to(torch.int64).sum().item())))
        all_sums = [None] * world
        dist.all_gather_object(all_sums, sums)
        if rank == 0:
            buf = recv + (last % 2) * FRAMES_TOTAL * fbytes
            ok = True
            n_checked = 0
            for part in all_sums:
                for f, name, sref in part:
                    i = [n for n, _ in levels].index(name)
                    v = torch.as_tensor(_CudaArray(frame_slot(buf, f)[i], lbytes[i] // 4, "<i4"), device="cuda")
                    ok = ok and int(v.to(torch.int64).sum().item()) == sref
                    n_checked += 1
            ok = ok and n_checked == 3 * FRAMES_TOTAL
        barrier(world)
        if rank != 0:
            eng.ipc_close(dst_base)
        barrier(world)
    if rank == 0:
        track_total = FRAMES_TOTAL * out["track_step_ms_per_frame"]
        out.update({"pipeline_frames_per_s": FRAMES_TOTAL / (pms / 1000.0), "pipeline_ms_per_step": pms,
                    "pipeline": ("one GPU: encode 64 frames, then one tracking step per frame (memory attention, "
                                 "mask decoder, memory encoder, object pointer)" if world == 1 else
                                 f"{len(encoders)} encoder GPU(s) -> NVLink peer copies of neck_trk_0/1/2 (CUDA IPC) "
                                 f"-> tracking GPU 0 (one tracking step per frame), double-buffered, one host "
                                 f"barrier per step"),
                    "pipeline_limiter": ("encoder + tracking in series on one GPU" if world == 1 else
                                         ("tracking steps on the tracking GPU"
                                          if track_total >= pms * 0.8 else "encoders")),
                    "p2p_bytes_per_frame": fbytes})
        if ok is not None:
            out["p2p_content_check"] = "pass" if ok else "FAIL"
        if world == 1:
            out["pipeline_encoder_ms"] = ms
        if recv is not None:
            eng.device_free(recv)
    eng.set_stream(None)
    eng.close()
    return out


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="vit_q4_0", choices=["vit_q4_0", "vit_q8_0", "vit_f16"])
    ap.add_argument("--frames", type=int, default=FRAMES_TOTAL, help="frames of the batch (split over the GPUs)")
    ap.add_argument("--frames-per-pass", type=int, default=8)
    ap.add_argument("--gemm-pairs", type=int, default=2, choices=[0, 1, 2],
                    help="256-row GEMM tiles on SM pairs: 2 (default) every wide GEMM, 1 K >= 2048 and the "
                         "f16-output ones, 0 never")
    ap.add_argument("--weights-quantised", type=int, default=WEIGHTS_QUANTISED, choices=[0, 1, 2],
                    help="1 (default): block form in HBM, staged per layer; 2: dequantised inside the GEMM; "
                         "0: f16 at load")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-headline", action="store_true",
                    help="skip the configs[3] headline and print only the --only lines (for profiling them)")
    ap.add_argument("--only", default="", help="comma list of extra lines to run (vit_f16_b1, hiera_t_f16_b1, "
                                               "hiera_t_q4_0, video); 'none' for the headline only")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n_gpus = max(world, 1)
    metric = "encoder frames/sec (SAM 3 ViT 1008^2 + SimpleFPN neck)"
    cfg_json = {"workload": f"configs[3]: SAM 3 ViT-L encoder + tracker neck, {args.workload.split('_', 1)[1]} "
                            f"weights, a {args.frames}-frame batch of seeded 1008^2 frames split {args.frames}/N "
                            f"over {n_gpus} GPU(s)",
                "frames_total": args.frames, "frames_per_gpu": args.frames / n_gpus, "img_size": 1008,
                "parallelism": f"frame-sharded x{n_gpus} (no collective)",
                "weights_in_hbm": WEIGHTS_DESC[args.weights_quantised],
                "l2_flush": "inputs + activations per step >> 126 MB L2"}

    if args.impl == "reference":
        # the CPU restatement of the reference path (the reference's ggml CPU backend is not in the checkout)
        if rank != 0:
            return
        r = cpu_reference(args.workload, args.steps, args.warmup)
        line = {"impl": "reference", "metric": metric, "value": r["value"], "unit": "frames/s", "n_gpus": n_gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded random-init weights, seeded uniform uint8 frames)", "config": cfg_json,
                "cpu_baseline": {"value": r["value"], "unit": "frames/s", "cores": r["cores"], "kind": "port",
                                 "sample": r["sample"]},
                "e2e": {"value": r["value"], "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "setup_s": r["setup_s"]}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=600))
    torch.cuda.set_device(local)
    s3b = load_pkg()
    extra = {"vit_f16_b1", "hiera_t_f16_b1", "hiera_t_q4_0", "video"}
    if args.only == "none":
        extra = set()
    elif args.only:
        extra = set(args.only.split(","))
    kinds = ([] if args.no_headline else [args.workload]) + (["vit_f16"] if "vit_f16_b1" in extra and args.workload != "vit_f16" else []) + \
        (["hiera_t_f16"] if "hiera_t_f16_b1" in extra else []) + (["hiera_t_q4_0"] if "hiera_t_q4_0" in extra else []) + \
        (["hiera_l_q8_0"] if "video" in extra else [])
    t0 = time.time()
    paths = prepare_models(s3b, kinds, local, world)
    gen_s = time.time() - t0
    stream = torch.cuda.Stream()

    if args.no_headline:
        line = {"metric": metric, "n_gpus": n_gpus, "steps": args.steps, "warmup": args.warmup,
                "note": "--no-headline: the configs[3] headline was not run", "setup": {"model_gen_s": gen_s}}
    else:
        v = bench_vit(s3b, paths[args.workload], args, rank, world, local, stream)
        line = {"metric": metric, "value": v.pop("value"), "unit": "frames/s", "n_gpus": n_gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": v.pop("ms_per_step"), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f16 (f32 accumulate)",
                "data": "synthetic (seeded random-init weights, seeded uniform uint8 frames)", "config": cfg_json}
        line.update(v)
        line["setup"]["model_gen_s"] = gen_s
    if "vit_f16_b1" in extra:
        line["vit_f16_b1"] = bench_latency(s3b, paths["vit_f16"], "configs[2]: SAM 3 ViT-L encoder + tracker neck, "
                                           "f16 weights, batch 1 (one seeded 1008^2 frame per call)", 1008,
                                           args, rank, world, local, stream)
    if "hiera_t_f16_b1" in extra:
        line["hiera_t_f16_b1"] = bench_latency(s3b, paths["hiera_t_f16"], "configs[0]: SAM 2.1 Hiera-T encoder + "
                                               "FPN neck, f16 weights, batch 1 (one seeded 1024^2 frame per call)",
                                               1024, args, rank, world, local, stream)
    if "hiera_t_q4_0" in extra:
        line["hiera_t_q4_0"] = bench_hiera(s3b, paths["hiera_t_q4_0"], args, rank, world, local, stream)
    if "video" in extra:
        line["video_hiera_l_q8_0"] = bench_video(s3b, paths["hiera_l_q8_0"], args, rank, world, local, stream)
    if rank == 0 and not args.no_cpu_baseline and not args.no_headline and world == 1:
        r = cpu_reference(args.workload, 8, 1)
        line["cpu_baseline"] = {"value": r["value"], "unit": "frames/s", "cores": r["cores"], "kind": "port",
                                "sample": r["sample"]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
