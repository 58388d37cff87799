#!/usr/bin/env python3
"""Encoder throughput benchmark (frames/s) of the B200 engine for sam3.cpp.

Workload: SAM 3 ViT image encoder + tracker
SimpleFPN neck, q4_0 weights (seeded synthetic, random-init), 64 seeded
1008x1008 frames per GPU (rank r encodes frames [64 r, 64 r + 64): weak
scaling, one process per GPU, no data-path collective). One step = encode
all frames of the rank; `value` = all ranks' frames / the slowest rank's time.
The same line carries `hiera_t_q4_0` (configs[1]: SAM 2.1 Hiera-T + FPN
neck, q4_0, 16 seeded 1024x1024 frames per GPU) and `video_hiera_l_q8_0`
(configs[4]: Hiera-L q8_0 on 64 frames per GPU, then memory attention per
frame on GPU 0), timed the same way.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload vit_q4_0|vit_f16]
  python bench.py --impl reference ...   # CPU restatement (oracle) of the same path

`value` is measured with inputs resident in HBM (device uint8 frames);
`e2e` goes through the public C ABI with pinned host frames every step
(s3b_encode_u8: host->device copy inside the timed region) and reads the
tracker's level-2 feature map (neck_trk_2, the memory-attention input) back
to the host. Inputs (64 x 3 MB frames + 2.5 GB of activations per pass) are
far larger than L2 (126 MB), so no separate flush is needed.
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
# 1: q4_0 / q8_0 linear weights stay in block form in HBM and the GEMMs dequantise them in shared
# memory (engine option weights_quantised); 0: dequantised to f16 at load (--weights-quantised)
WEIGHTS_QUANTISED = 0
# measured with ncu (one --set full capture of ViT block 0): mean DRAM read+write per launch of the
# qkv / proj / fc1 / fc2 GEMMs of a ViT block at 8 frames per pass, and their algorithmic bytes
GEMM_TRAFFIC_BYTES = 4.696e8
GEMM_ALG_BYTES = 5.006e8


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


def rank_frames(per_gpu: int, rank: int) -> tuple[int, int]:
    """Frames [first, first + per_gpu) encoded by `rank` (weak scaling: every rank encodes per_gpu frames
    of its own; frame f keeps its seed on any world size)."""
    return rank * per_gpu, per_gpu


def shard_frames(total: int, rank: int, world: int) -> tuple[int, int]:
    """Frames [first, first + count) encoded by `rank`: contiguous blocks whose
    sizes differ by at most one; frame f keeps its seed on any world size."""
    first = total * rank // world
    return first, total * (rank + 1) // world - first


def max_over_ranks(x: float, world: int, device) -> float:
    """Max of a per-rank time over all ranks (the job's time); identity on one rank."""
    if world <= 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


HIERA_FRAMES_PER_GPU = 16


def bench_hiera(s3b, local: int, rank: int, world: int, steps: int, warmup: int, stream, device) -> dict:
    """SAM 2.1 Hiera-T image encoder + FPN neck, q4_0 weights, a batch of 16 seeded
    1024^2 frames per GPU (device-resident), CUDA events on the engine stream, max over ranks."""
    import torch
    import torch.distributed as dist
    from sam3_b200 import synth
    path = os.path.join(tempfile.gettempdir(), "s3b_bench_hiera_t_q4_0.ggml")
    if local == 0 and not os.path.exists(path):
        synth.write_sam2(path + ".tmp", synth.HIERA_T, seed=0, ftype=1, qtype=2, quantize=s3b.quantize_rows)
        os.replace(path + ".tmp", path)
    if world > 1:
        dist.barrier()
    eng = s3b.Engine(local)
    eng.set_option("weights_quantised", WEIGHTS_QUANTISED)
    eng.set_option("frames_per_pass", HIERA_FRAMES_PER_GPU)
    eng.load_model(path)
    n = HIERA_FRAMES_PER_GPU
    frames = torch.from_numpy(synth.frames_u8(n, 1024, base_seed=1000 + rank * n)).to(device)
    for _ in range(warmup):
        eng.encode_u8(frames)
    eng.sync()
    eng.set_stream(stream.cuda_stream)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    eng.profile_begin(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        eng.encode_u8(frames)
    e1.record(stream)
    torch.cuda.synchronize()
    prof = eng.profile_end()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world, device)
    g, a = prof["gemm"], prof["attention"]
    eng.set_stream(None)
    eng.close()
    return {"workload": f"configs[1]: SAM 2.1 Hiera-T image encoder + FPN neck, q4_0 weights, {n} seeded 1024^2 "
                        f"frames per GPU (device-resident) x {world} GPU(s)",
            "value": n * world / (ms / 1000.0), "unit": "frames/s", "ms_per_step": ms,
            "gemm_tflops": g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] > 0 else 0.0,
            "gemm_ms_per_step": g["ms"] / steps,
            "attention_tflops": a["flops"] / (a["ms"] / 1000.0) / 1e12 if a["ms"] > 0 else 0.0,
            "attention_ms_per_step": a["ms"] / steps,
            "algorithmic_tflop_per_step": (g["flops"] + a["flops"]) / steps / 1e12,
            "gpu_launches_per_step": prof["launches"] / steps}


def bench_video(s3b, local: int, rank: int, world: int, steps: int, warmup: int, stream, device) -> dict:
    """SAM 2.1 Hiera-L image encoder + FPN neck, q8_0 weights, 64 seeded 1024^2 frames
    sharded over the GPUs (frames/s of the job, max over ranks); then, on rank 0 (the tracking GPU), memory
    attention per frame: 4 layers, d = 256, 64x64 current tokens from the encoder's level-2 map, cross-attention
    to 7 memory frames of 64x64 tokens + 16 object pointers x 4 tokens (M = 28736, random memory bank)."""
    import dataclasses

    import torch
    import torch.distributed as dist
    from sam3_b200 import synth
    cfg = dataclasses.replace(synth.HIERA_L, with_mem_attn=True)
    path = os.path.join(tempfile.gettempdir(), "s3b_bench_hiera_l_q8_0.ggml")
    if local == 0 and not os.path.exists(path):
        synth.write_sam2(path + ".tmp", cfg, seed=0, ftype=1, qtype=8, quantize=s3b.quantize_rows)
        os.replace(path + ".tmp", path)
    if world > 1:
        dist.barrier()
    eng = s3b.Engine(local)
    eng.set_option("weights_quantised", WEIGHTS_QUANTISED)
    eng.load_model(path)
    first, nf = rank_frames(FRAMES_TOTAL, rank)
    frames = torch.from_numpy(synth.frames_u8(nf, 1024, base_seed=1000 + first)).to(device)
    for _ in range(warmup):
        eng.encode_u8(frames)
    eng.sync()
    eng.set_stream(stream.cuda_stream)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    eng.profile_begin(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        eng.encode_u8(frames)
    e1.record(stream)
    torch.cuda.synchronize()
    prof = eng.profile_end()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world, device)
    g, a = prof["gemm"], prof["attention"]
    out = {"workload": f"configs[4]: SAM 2.1 Hiera-L image encoder + FPN neck, q8_0 weights, {FRAMES_TOTAL} seeded "
                       f"1024^2 frames per GPU x {world} GPU(s); memory attention per frame on GPU 0",
           "encoder_frames_per_s": FRAMES_TOTAL * world / (ms / 1000.0), "encoder_ms_per_step": ms,
           "encoder_gemm_tflops": g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] > 0 else 0.0,
           "encoder_attention_tflops": a["flops"] / (a["ms"] / 1000.0) / 1e12 if a["ms"] > 0 else 0.0}
    # hand-off of per-frame features to the tracking GPU (rank 0): every other rank copies its frame 0's
    # neck_trk_2 (the memory-attention input) into its slot of a rank-0 buffer opened through CUDA IPC
    # (s3b_peer_copy_output over NVLink); rank 0 then runs memory attention on the frame rank 1 encoded
    ne = eng.output_shape("neck_trk_2")
    fbytes = ne[0] * ne[1] * ne[2] * 4
    recv = None
    if world > 1:
        import torch.distributed as dist
        if rank == 0:
            recv = eng.device_alloc(fbytes * (world - 1))
            handle = [eng.ipc_export(recv)]
        else:
            handle = [None]
        dist.broadcast_object_list(handle, src=0)
        ms_copy = 0.0
        if rank > 0:
            ptr = eng.ipc_open(handle[0])
            dst = ptr + (rank - 1) * fbytes
            for _ in range(warmup):
                eng.peer_copy_output("neck_trk_2", 0, dst, 0, fbytes)
            eng.sync()
            e0.record(stream)
            for _ in range(steps):
                eng.peer_copy_output("neck_trk_2", 0, dst, 0, fbytes)
            e1.record(stream)
            torch.cuda.synchronize()
            ms_copy = e0.elapsed_time(e1) / steps
            eng.ipc_close(ptr)
        dist.barrier()
        t = max_over_ranks(ms_copy, world, device)
        out["p2p_neck_trk_2"] = {"bytes_per_frame": fbytes, "senders": world - 1, "ms_per_copy_max": t,
                                 "gbs_per_sender": fbytes / (t / 1000.0) / 1e9 if t > 0 else None,
                                 "path": "s3b_peer_copy_output into a rank-0 buffer opened with s3b_ipc_open"}
    if rank == 0:
        # current frame = frame 0 of rank 1 (received above) or of this rank's own batch; its PE; random
        # memory bank and pointer tokens
        if recv is not None:
            curr = torch.as_tensor(_CudaArray(recv, fbytes // 4), device=device).view(-1, 256)
        else:
            curr = torch.from_numpy(eng.output("neck_trk_2", 0).reshape(-1, 256)).to(device)
        pos = torch.from_numpy(eng.output("neck_trk_pe_2", 0).reshape(-1, 256)).to(device)
        g2 = torch.Generator(device=device).manual_seed(5)
        m_total, n_ptr = cfg.num_maskmem * 4096 + cfg.max_obj_ptrs * 4, cfg.max_obj_ptrs * 4
        prompt = torch.randn(m_total, 64, device=device, generator=g2)
        prompt_pos = torch.randn(m_total, 64, device=device, generator=g2) * 0.1
        res = torch.empty_like(curr)
        # timed without per-launch profiling (the layers replay from a CUDA graph from the second call on);
        # one more profiled pass gives the algorithmic FLOPs and the attention kernels' share
        for _ in range(max(warmup, 2)):
            eng.mem_attn(curr, pos, 64, prompt, prompt_pos, n_ptr, out=res)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(steps):
            eng.mem_attn(curr, pos, 64, prompt, prompt_pos, n_ptr, out=res)
        e1.record(stream)
        torch.cuda.synchronize()
        mms = e0.elapsed_time(e1) / steps
        eng.profile_begin(True)
        eng.mem_attn(curr, pos, 64, prompt, prompt_pos, n_ptr, out=res)
        torch.cuda.synchronize()
        p2 = eng.profile_end()
        fl = p2["gemm"]["flops"] + p2["attention"]["flops"]
        out.update({"mem_attn_ms_per_frame": mms, "mem_attn_tflop_per_frame": fl / 1e12,
                    "mem_attn_tflops": fl / (mms / 1000.0) / 1e12,
                    "mem_attn_attention_tflops": p2["attention"]["flops"] / (p2["attention"]["ms"] / 1000.0) / 1e12
                    if p2["attention"]["ms"] > 0 else 0.0,
                    "mem_attn_timing": "CUDA events around the timed calls, no per-launch profiling; the layers "
                                       "replay from a CUDA graph",
                    "mem_attn_memory_tokens": m_total,
                    "mem_attn_input": "frame 0 of rank 1 (peer-copied)" if recv is not None else "own frame 0"})
        if recv is not None:
            eng.device_free(recv)
    eng.set_stream(None)
    eng.close()
    return out


class _CudaArray:
    """Zero-copy view of engine-owned device memory for torch.as_tensor (the CUDA array interface)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


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


def make_model(s3b, workload: str, path: str):
    from sam3_b200 import synth
    cfg = synth.SAM3_VIT_L
    qtype = {"vit_q4_0": 2, "vit_q8_0": 8, "vit_f16": None}[workload]
    synth.write_sam3(path, cfg, seed=0, ftype=1, qtype=qtype, quantize=s3b.quantize_rows)
    return cfg


def cpu_sample(workload: str, steps: int = 1):
    """Times the oracle (numpy, all host threads) on a bounded sample of one
    frame: prefix + one windowed block + one global block + the tracker neck,
    and extrapolates to frames/s (28 windowed + 4 global blocks)."""
    s3b = load_pkg()
    sys.path.insert(0, ROOT)
    from oracle import quant as oq
    from oracle import vit as ov
    from sam3_b200 import synth
    cfg = synth.SAM3_VIT_L
    qtype = {"vit_q4_0": 2, "vit_q8_0": 8, "vit_f16": None}[workload]
    rng_cfg = synth.Sam3Config(depth=8, global_idx=(7,))  # blocks 0 (windowed) and 7 (global)
    T = synth.sam3_tensors(rng_cfg, seed=0)
    T = {k: v for k, v in T.items() if not k.startswith("vit.blocks.") or k.split(".")[2] in ("0", "7")}
    W = synth.stored_values(T, 1, qtype, oq.quantize, oq.dequantize)
    chw = ov.preprocess_u8(synth.frames_u8(1, cfg.img_size))
    vals = []
    parts = None
    for _ in range(steps):
        t0 = time.perf_counter()
        x = ov.prefix(W, chw, cfg)
        t1 = time.perf_counter()
        x = ov.block(W, x, 0, rng_cfg)
        t2 = time.perf_counter()
        x = ov.block(W, x, 7, rng_cfg)
        t3 = time.perf_counter()
        ov.neck(W, x)
        t4 = time.perf_counter()
        t_frame = (t1 - t0) + 28 * (t2 - t1) + 4 * (t3 - t2) + (t4 - t3)
        vals.append(1.0 / t_frame)
        parts = {"prefix_s": t1 - t0, "win_block_s": t2 - t1, "global_block_s": t3 - t2, "neck_s": t4 - t3}
    return float(np.median(vals)), parts


def main():
    global WEIGHTS_QUANTISED
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="vit_q4_0", choices=["vit_q4_0", "vit_q8_0", "vit_f16"])
    ap.add_argument("--frames", type=int, default=FRAMES_TOTAL, help="frames per GPU")
    ap.add_argument("--frames-per-pass", type=int, default=8)
    ap.add_argument("--gemm-pairs", type=int, default=1, choices=[0, 1, 2],
                    help="256-row GEMM tiles on SM pairs: 1 (default) for K >= 2048, 2 for all, 0 never")
    ap.add_argument("--weights-quantised", type=int, default=WEIGHTS_QUANTISED, choices=[0, 1],
                    help="1: quantised weights stay in block form in HBM, dequantised inside the GEMMs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-hiera", action="store_true", help="skip the Hiera-T (configs[1]) measurement")
    ap.add_argument("--only-hiera", action="store_true",
                    help="run only the Hiera-T (configs[1]) measurement and print its numbers (a profiling case)")
    ap.add_argument("--no-video", action="store_true",
                    help="skip the Hiera-L + memory attention (configs[4]) measurement")
    args = ap.parse_args()
    WEIGHTS_QUANTISED = args.weights_quantised

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n_gpus = max(world, 1)
    metric = "encoder frames/sec (SAM 3 ViT 1008^2 + SimpleFPN neck)"
    cfg_json = {"workload": f"configs[3]: SAM 3 ViT-L encoder + tracker neck, {args.workload.split('_', 1)[1]} "
                            f"weights, {args.frames} seeded 1008^2 frames per GPU x {n_gpus} GPU(s)",
                "frames_total": args.frames * n_gpus, "frames_per_gpu": args.frames,
                "img_size": 1008,
                "parallelism": f"frame-sharded x{n_gpus} (no collective)",
                "weights_in_hbm": ("block form, dequantised inside the GEMMs" if args.weights_quantised
                                   else "f16, dequantised once at load"),
                "l2_flush": "inputs + activations per step >> 126 MB L2"}

    if args.impl == "reference":
        # CPU restatement of the reference path (the reference's ggml CPU backend cannot be built here)
        if rank != 0:
            return
        steps = max(1, min(args.steps, 3))
        for _ in range(min(args.warmup, 1)):
            cpu_sample(args.workload, 1)
        t0 = time.perf_counter()
        v, parts = cpu_sample(args.workload, steps)
        elapsed = time.perf_counter() - t0
        ms = 1000.0 * args.frames / v
        line = {"impl": "reference", "metric": metric, "value": v, "unit": "frames/s", "n_gpus": n_gpus,
                "steps": steps, "warmup": min(args.warmup, 1), "ms_per_step": ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init)",
                "config": cfg_json,
                "cpu_baseline": {"value": v, "unit": "frames/s", "cores": os.cpu_count(), "kind": "port",
                                 "sample": f"1 frame: prefix + 1 windowed + 1 global ViT block + tracker neck, "
                                           f"extrapolated to 28+4 blocks; {steps} step(s), {elapsed:.1f} s; {parts}"},
                "e2e": {"value": v, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
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
    from sam3_b200 import synth

    if args.only_hiera:
        h = bench_hiera(s3b, local, rank, world, args.steps, args.warmup, torch.cuda.Stream(), "cuda")
        if rank == 0:
            print(json.dumps({"impl": "b200", "n_gpus": n_gpus, "steps": args.steps, "warmup": args.warmup,
                              "hiera_t_q4_0": h}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    path = os.path.join(tempfile.gettempdir(), f"s3b_bench_{args.workload}.ggml")
    t0 = time.time()
    if local == 0 and not os.path.exists(path):
        make_model(s3b, args.workload, path + ".tmp")
        os.replace(path + ".tmp", path)
    if world > 1:
        dist.barrier()
    cfg = synth.SAM3_VIT_L
    gen_s = time.time() - t0
    eng = s3b.Engine(local)
    eng.set_option("weights_quantised", WEIGHTS_QUANTISED)
    eng.set_option("frames_per_pass", args.frames_per_pass)
    eng.set_option("gemm_pairs", args.gemm_pairs)
    t0 = time.time()
    eng.load_model(path)
    load_s = time.time() - t0

    first, nf = rank_frames(args.frames, rank)
    host = synth.frames_u8(nf, cfg.img_size, base_seed=1000 + first)
    host_t = torch.from_numpy(host).pin_memory()
    dev = host_t.cuda()
    out_host = torch.empty((nf, 72, 72, 256), dtype=torch.float32).pin_memory()

    def step_device():
        eng.encode_u8(dev)

    for _ in range(args.warmup):
        step_device()
    eng.sync()

    # --- timed region (device-resident inputs), profiled with CUDA events on the engine stream
    stream = torch.cuda.Stream()
    eng.set_stream(stream.cuda_stream)
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    eng.profile_begin(True)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step_device()
    ev1.record(stream)
    torch.cuda.synchronize()
    prof = eng.profile_end()
    clk = clocks.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world, "cuda")
    value = args.frames * n_gpus / (ms / 1000.0)

    # --- end-to-end through the public API with host buffers
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev2 = torch.cuda.Event(enable_timing=True)
    ev3 = torch.cuda.Event(enable_timing=True)
    out_np = out_host.numpy()
    host_np = host_t.numpy()  # pinned host frames
    ev2.record(stream)
    for _ in range(args.steps):
        eng.encode_u8(host_np)                      # H2D inside the public call
        for f in range(nf):                         # D2H of the tracker-level map, per frame
            eng.output("neck_trk_2", f, out=out_np[f])
    ev3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(ev2.elapsed_time(ev3) / args.steps, world, "cuda")
    e2e = args.frames * n_gpus / (e2e_ms / 1000.0)

    # --- roofline of the dominant kernel (tensor-core GEMM)
    peak_burst, peak_sust, hbm, src = measured_peaks()
    g = prof["gemm"]
    gemm_tflops = g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] > 0 else 0.0
    a = prof["attention"]
    ln = prof["layernorm"]
    attn_tflops = a["flops"] / (a["ms"] / 1000.0) / 1e12 if a["ms"] > 0 else 0.0
    fl_gemm, fl_attn, fl_neck = vit_flops_per_frame(cfg)
    total_tflops = (fl_gemm + fl_attn + fl_neck) * value / 1e12

    line = {"metric": metric, "value": value, "unit": "frames/s", "n_gpus": n_gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 (f32 accumulate)", "data": "synthetic (seeded random-init weights, seeded uniform uint8 frames)",
            "config": cfg_json,
            "e2e": {"value": e2e, "unit": "frames/s", "h2d_bytes_per_step": int(host.nbytes),
                    "d2h_bytes_per_step": int(out_host.numel() * 4)},
            "roofline": {"bound": "tensor", "achieved": gemm_tflops, "peak": peak_sust, "unit": "TFLOP/s",
                         "frac": gemm_tflops / peak_sust,
                         # DRAM bytes per GEMM launch (read + write), mean of the four block-0 GEMMs at 8 frames
                         # from one ncu capture of ViT block 0; algorithmic 5.0e8
                         "traffic": GEMM_TRAFFIC_BYTES, "traffic_algorithmic": GEMM_ALG_BYTES,
                         "kernel": "gemm_f16_tc_kernel (tcgen05/TMEM, TMA)",
                         "peak_source": f"{src} bf16_tflops_sustained (kernel timed inside a long step)",
                         "gemm_ms_per_step": g["ms"] / args.steps, "gemm_launches_per_step": g["launches"] / args.steps},
            "attention": {"achieved_tflops": attn_tflops, "ms_per_step": a["ms"] / args.steps,
                          "frac_of_peak": attn_tflops / peak_sust},
            "layernorm": {"achieved_gbs": ln["bytes"] / (ln["ms"] / 1000.0) / 1e9 if ln["ms"] > 0 else 0.0,
                          "peak_gbs": hbm, "frac_of_peak": (ln["bytes"] / (ln["ms"] / 1000.0) / 1e9 / hbm)
                          if ln["ms"] > 0 else 0.0, "ms_per_step": ln["ms"] / args.steps,
                          "launches_per_step": ln["launches"] / args.steps,
                          "bound": "hbm (algorithmic bytes: f32 rows in + f16 rows out)"},
            "whole_step_tflops": total_tflops, "flops_per_frame": fl_gemm + fl_attn + fl_neck,
            "gpu_launches": int(prof["launches"]), "clocks": clk,
            "setup": {"model_gen_s": gen_s, "load_s": load_s, "weights_mib": eng.model_info()["weights_mib"]}}
    eng.set_stream(None)
    eng.close()
    if not args.no_hiera:
        line["hiera_t_q4_0"] = bench_hiera(s3b, local, rank, world, args.steps, args.warmup, stream, "cuda")
    if not args.no_video:
        line["video_hiera_l_q8_0"] = bench_video(s3b, local, rank, world, args.steps, args.warmup, stream, "cuda")
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        v, parts = cpu_sample(args.workload, 1)
        line["cpu_baseline"] = {"value": v, "unit": "frames/s", "cores": os.cpu_count(), "kind": "port",
                                "sample": f"oracle (numpy) on 1 frame: prefix + 1 windowed + 1 global block + "
                                          f"tracker neck, extrapolated to 28+4 blocks; {parts}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
