#!/usr/bin/env python3
"""Generates the full-size oracle fixtures in tests/golden/ (no reference checkout needed).

The oracle (oracle/, a numpy restatement of the reference path pinned to the reference's own dumps by
make_golden.py) takes minutes per frame at the configurations' full sizes, too long to run inside a GPU
test. This script runs it once on seeded synthetic models and frames and stores deterministic samples
(indices + values) and summary statistics of every output:

1. fullsize_vit_l_q4_0.npz — SAM 3 ViT-L + tracker neck, q4_0 weights (synth.SAM3_VIT_L, weight seed 0),
   frames 0 and 7 of the 8-frame pass made by synth.frames_u8(8, 1008, base_seed=1000):
   vit_output, neck_trk_0..3.
2. fullsize_hiera_l_q8_0.npz — SAM 2.1 Hiera-L + FPN neck, q8_0 weights (synth.HIERA_L, weight seed 0),
   frames 0 and 1 of synth.frames_u8(2, 1024, base_seed=1000): neck_trk_0..2.

    python tests/golden/make_oracle_fixtures.py [--only vit|hiera]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from make_golden import load_pkg, sample  # noqa: E402

WEIGHT_SEED = 0
FRAME_SEED = 1000


def make_vit(out_path: str):
    load_pkg()
    from oracle import quant as oq
    from oracle import vit as ov
    from sam3_b200 import synth
    cfg = synth.SAM3_VIT_L
    t0 = time.time()
    W = synth.stored_values(synth.sam3_tensors(cfg, seed=WEIGHT_SEED), 1, 2, oq.quantize, oq.dequantize)
    frames = synth.frames_u8(8, cfg.img_size, base_seed=FRAME_SEED)
    out = {}
    for k, f in enumerate((0, 7)):
        x, _ = ov.backbone(W, ov.preprocess_u8(frames[f:f + 1]), cfg)
        necks = ov.neck(W, x)
        out.update(sample(x[0], f"frame{f}_vit_output", 300 + 10 * k))
        for i in range(4):
            out.update(sample(necks[i][0], f"frame{f}_neck_trk_{i}", 301 + 10 * k + i))
        print(f"vit frame {f} done ({time.time() - t0:.0f} s)", flush=True)
    meta = {"weights_seed": WEIGHT_SEED, "frame_seed": FRAME_SEED, "frames_in_pass": 8, "frames": [0, 7],
            "qtype": 2, "ftype": 1, "config": "synth.SAM3_VIT_L (configs[3]), tracker neck",
            "generator": "oracle.vit backbone + neck on the q4_0-dequantised stored values"}
    np.savez_compressed(out_path, meta=json.dumps(meta), **out)
    print("wrote", out_path)


def make_hiera(out_path: str):
    load_pkg()
    from oracle import hiera as oh
    from oracle import quant as oq
    from sam3_b200 import synth
    cfg = synth.HIERA_L
    t0 = time.time()
    W = synth.stored_values(synth.sam2_tensors(cfg, seed=WEIGHT_SEED), 1, 8, oq.quantize, oq.dequantize)
    frames = synth.frames_u8(2, cfg.img_size, base_seed=FRAME_SEED)
    out = {}
    for k, f in enumerate((0, 1)):
        stages = oh.backbone(W, oh.preprocess_u8(frames[f:f + 1]), cfg)
        fpn = oh.fpn(W, stages, cfg)
        for i in range(len(fpn)):
            out.update(sample(fpn[i][0], f"frame{f}_neck_trk_{i}", 400 + 10 * k + i))
        print(f"hiera frame {f} done ({time.time() - t0:.0f} s)", flush=True)
    meta = {"weights_seed": WEIGHT_SEED, "frame_seed": FRAME_SEED, "frames": [0, 1], "qtype": 8, "ftype": 1,
            "config": "synth.HIERA_L (configs[4] encoder)",
            "generator": "oracle.hiera backbone + fpn on the q8_0-dequantised stored values"}
    np.savez_compressed(out_path, meta=json.dumps(meta), **out)
    print("wrote", out_path)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", choices=["vit", "hiera"], default=None)
    a = ap.parse_args()
    if a.only in (None, "hiera"):
        make_hiera(os.path.join(HERE, "fullsize_hiera_l_q8_0.npz"))
    if a.only in (None, "vit"):
        make_vit(os.path.join(HERE, "fullsize_vit_l_q4_0.npz"))


if __name__ == "__main__":
    main()
