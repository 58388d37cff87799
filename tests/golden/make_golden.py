#!/usr/bin/env python3
"""Generates the golden fixtures in tests/golden/ from the reference's own code.

Run in a container that has the reference checkout (read-only) and torch:

    python tests/golden/make_golden.py --reference /path/to/sam3.cpp

1. vit_golden.npz — the reference's PyTorch ViT + SimpleFPN forward
   (tests/dump_vit_reference.py main(), run unmodified as a subprocess) on a
   seeded synthetic checkpoint whose tensors are exactly the values a f16
   .ggml file written by sam3_b200.synth stores (same seed, same rounding),
   and on a seeded 1008x1008 uint8 frame. The script's detector neck
   ("convs.*") is given the tracker neck weights ("neck.trk.*" in .ggml
   naming), so its outputs are the engine's neck_trk_0..3.
2. mem_attn_golden.npz — run_memory_attention() imported from the
   reference's tests/dump_phase7_reference.py on seeded synthetic tracker
   weights, current features, memory prompt and prompt PE.
3. window_golden.npz — window_partition / window_unpartition imported from
   the reference's tests/dump_vit_reference.py on seeded padded inputs (the
   Hiera window path: 64 -> 70 at ws 14, q-pooled unpartition at ws // 2).
4. sam_dec_golden.npz — dump_case() imported from the reference's
   tests/dump_phase6_reference.py (SAM prompt encoder + SAM mask decoder) on
   seeded synthetic decoder weights, seeded neck_trk_0..2 feature maps at the
   SAM 3 size (72^2 image tokens) and three prompt cases of our own.
5. mem_enc_golden.npz — run_memory_encoder() and run_obj_ptr() imported
   from the reference's tests/dump_phase7_reference.py on seeded synthetic
   memory-encoder weights, a seeded neck_trk_2 map and seeded 288^2 mask
   logits (object present and absent).

Each dumped tensor is stored as deterministic samples (indices + values)
plus summary statistics, so the fixtures stay small; tests regenerate the
same weights from the seeds and compare.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
N_SAMPLES = 4096

VIT_SEED = 2024
FRAME_SEED = 1000
MEM_SEED = 77
MEM_FRAMES = 2
MEM_PTRS = 2


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


def sample(arr: np.ndarray, key: str, seed: int):
    flat = np.ascontiguousarray(arr, np.float32).ravel()
    rng = np.random.default_rng(seed)
    idx = np.sort(rng.choice(flat.size, size=min(N_SAMPLES, flat.size), replace=False)).astype(np.int64)
    return {f"{key}__shape": np.array(arr.shape, np.int64), f"{key}__idx": idx, f"{key}__val": flat[idx],
            f"{key}__stats": np.array([flat.mean(dtype=np.float64), flat.std(dtype=np.float64),
                                       np.abs(flat).mean(dtype=np.float64), np.abs(flat).max()], np.float64)}


def vit_checkpoint(W: dict):
    """.ggml-named stored values -> the state dict keys dump_vit_reference.py reads."""
    import torch
    sd = {}
    tp = "detector.backbone.vision_backbone.trunk."
    for k, v in W.items():
        if k.startswith("vit."):
            name = k[len("vit."):].replace(".mlp.lin1.", ".mlp.fc1.").replace(".mlp.lin2.", ".mlp.fc2.")
            t = torch.from_numpy(np.ascontiguousarray(v))
            if name == "pos_embed":  # [g, g, E] -> [1, 1 + g*g, E] with a (unused) cls slot
                g, _, E = v.shape
                t = torch.cat([torch.zeros(1, 1, E), t.reshape(1, g * g, E)], dim=1)
            elif name.endswith("attn.freqs_cis"):  # [N, 32, 2] (cos, sin) -> complex [N, 32]
                t = torch.complex(t[..., 0].contiguous(), t[..., 1].contiguous())
            sd[tp + name] = t
        elif k.startswith("neck.trk."):
            sd["detector.backbone.vision_backbone.convs." + k[len("neck.trk."):]] = torch.from_numpy(
                np.ascontiguousarray(v))
    return sd


def make_vit(reference: str, out_path: str):
    import torch
    from PIL import Image
    s3b = load_pkg()
    from sam3_b200 import synth
    cfg = synth.SAM3_VIT_L
    T = synth.sam3_tensors(cfg, seed=VIT_SEED, ln_random=True)
    W = synth.stored_values(T, 1, None)
    frame = synth.frames_u8(1, cfg.img_size, base_seed=FRAME_SEED)[0]
    with tempfile.TemporaryDirectory() as d:
        ck = os.path.join(d, "synthetic_sam3.pt")
        torch.save(vit_checkpoint(W), ck)
        img = os.path.join(d, "frame.png")
        Image.fromarray(frame).save(img)
        outdir = os.path.join(d, "ref")
        script = os.path.join(reference, "tests", "dump_vit_reference.py")
        subprocess.run([sys.executable, script, "--checkpoint", ck, "--image", img, "--outdir", outdir],
                       check=True, cwd=d)

        def load(name):
            shape = tuple(int(x) for x in open(os.path.join(outdir, name + ".shape")).read().split(","))
            return np.fromfile(os.path.join(outdir, name + ".bin"), dtype=np.float32).reshape(shape)

        out = {}
        taps = ["preprocessed", "after_ln_pre", "block_0_out", "block_7_out", "vit_final",
                "neck_det_0", "neck_det_1", "neck_det_2", "neck_det_3"]
        for i, name in enumerate(taps):
            a = load(name)
            if name.startswith("neck_det_"):
                a = a[0].transpose(1, 2, 0)  # [1, C, H, W] -> channel-last [H, W, C]
            elif name == "preprocessed":
                a = a[0]
            else:
                a = a[0]  # [H, W, C]
            out.update(sample(a, name, 100 + i))
    meta = {"weights_seed": VIT_SEED, "frame_seed": FRAME_SEED, "ln_random": True, "ftype": 1,
            "generator": "tests/dump_vit_reference.py main() of the reference, unmodified",
            "config": "SAM 3 ViT-L 1008^2 (synth.SAM3_VIT_L), tracker neck weights as the script's convs.*"}
    np.savez_compressed(out_path, meta=json.dumps(meta), **out)
    print("wrote", out_path)


def mem_attn_tracker_weights(T: dict):
    import torch
    sd = {}
    for k, v in T.items():
        if not k.startswith("mem_attn."):
            continue
        name = k.replace("mem_attn.layers.", "transformer.encoder.layers.").replace("mem_attn.norm.",
                                                                                   "transformer.encoder.norm.")
        name = name.replace(".sa.", ".self_attn.").replace(".ca.", ".cross_attn_image.")
        sd[name] = torch.from_numpy(np.ascontiguousarray(v))
    return sd


def mem_inputs(seed: int, H: int = 72):
    """Seeded current features, memory prompt (MEM_FRAMES spatial slots + MEM_PTRS pointers x 4 tokens)."""
    sys.path.insert(0, ROOT)
    from oracle.mem_attn import golden_inputs
    return golden_inputs({"feat": H, "inputs_seed": seed, "mem_frames": MEM_FRAMES, "ptrs": MEM_PTRS})


def make_mem_attn(reference: str, out_path: str):
    import torch
    s3b = load_pkg()
    from sam3_b200 import synth
    cfg = synth.Sam3Config(depth=1, global_idx=(), with_mem_attn=True)
    T = synth.sam3_tensors(cfg, seed=MEM_SEED, ln_random=True)
    W = synth.stored_values({k: v for k, v in T.items() if k.startswith("mem_attn.")}, 1, None)
    spec = importlib.util.spec_from_file_location("dump_phase7_reference",
                                                  os.path.join(reference, "tests", "dump_phase7_reference.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    curr, prompt, prompt_pos, n_ptr = mem_inputs(MEM_SEED + 1)
    curr_nchw = torch.from_numpy(curr.reshape(72, 72, 256).transpose(2, 0, 1).copy())[None]
    with torch.no_grad():
        res = ref.run_memory_attention(mem_attn_tracker_weights(W), curr_nchw,
                                       torch.from_numpy(prompt)[:, None, :], torch.from_numpy(prompt_pos)[:, None, :],
                                       n_ptr)
    out = {}
    for i, key in enumerate(["input", "layer0_after_sa", "layer0_after_ca", "layer0_after_ffn", "output"]):
        a = res[key].numpy()  # batch-first [1, N, 256]
        assert a.shape == (1, 72 * 72, 256), a.shape
        out.update(sample(a[0], key, 200 + i))
    meta = {"weights_seed": MEM_SEED, "inputs_seed": MEM_SEED + 1, "mem_frames": MEM_FRAMES, "ptrs": MEM_PTRS,
            "feat": 72, "generator": "run_memory_attention() of the reference's tests/dump_phase7_reference.py"}
    np.savez_compressed(out_path, meta=json.dumps(meta), **out)
    print("wrote", out_path)


WINDOW_SEED = 31
# (input shape [B, H, W, C], window size): padded grids of the Hiera stages (64 -> 70 at ws 14, the
# q-pooled 32 -> 35 at ws 7), an exact fit and a non-square padded one
WINDOW_CASES = [((1, 64, 64, 3), 14), ((2, 32, 32, 2), 7), ((1, 32, 32, 2), 8), ((1, 20, 30, 3), 8)]


def make_window(reference: str, out_path: str):
    """window_partition / window_unpartition of the reference's tests/dump_vit_reference.py (imported, not
    modified) on seeded padded inputs, plus the Hiera q-stride path: partition at ws, 2x2 max pool of every
    window (torch max_pool2d, as sam2's do_pool), unpartition at ws // 2 onto the halved, padded grid."""
    import torch
    spec = importlib.util.spec_from_file_location("dump_vit_reference",
                                                  os.path.join(reference, "tests", "dump_vit_reference.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    rng = np.random.default_rng(WINDOW_SEED)
    out = {}
    for c, (shape, ws) in enumerate(WINDOW_CASES):
        x = rng.standard_normal(shape).astype(np.float32)
        win, pad_hw = ref.window_partition(torch.from_numpy(x), ws)
        back = ref.window_unpartition(win, ws, pad_hw, shape[1:3])
        B, H, W, C = shape
        # the inputs are regenerated by the tests from the seed (standard normals in case order)
        assert np.array_equal(back.numpy(), x)  # the reference's own round trip
        out[f"case{c}_windows"] = win.numpy()
        out[f"case{c}_pad_hw"] = np.array(pad_hw, np.int64)
        if ws % 2 == 0:  # q-stride blocks have even windows (Hiera pools 8 -> 4 and 14 -> 7)
            pooled = torch.nn.functional.max_pool2d(win.permute(0, 3, 1, 2), 2, 2).permute(0, 2, 3, 1)
            ws2 = ws // 2
            th, tw = H // 2, W // 2
            pad2 = (th + (ws2 - th % ws2) % ws2, tw + (ws2 - tw % ws2) % ws2)
            out[f"case{c}_qpool_unpartition"] = ref.window_unpartition(pooled, ws2, pad2, (th, tw)).numpy()
    meta = {"seed": WINDOW_SEED, "cases": WINDOW_CASES,
            "generator": "window_partition / window_unpartition of the reference's tests/dump_vit_reference.py "
                         "(lines 64-86), torch max_pool2d for the q pooling"}
    np.savez_compressed(out_path, meta=json.dumps(meta), **out)
    print("wrote", out_path)


SAMDEC_SEED = 91
SAMDEC_FEAT_SEED = 92
# (case name, positive points, negative points, box) in 1008^2 input coordinates
SAMDEC_CASES = [
    ("point", [(412.0, 530.0)], [], None),
    ("box", [], [], (150.0, 210.0, 790.0, 880.0)),
    ("box_points", [(600.0, 610.0)], [(300.0, 280.0)], (150.0, 210.0, 790.0, 880.0)),
]


def sam_dec_weights():
    """Stored (f16-rounded) values of the seeded synthetic prompt-encoder / mask-decoder tensors."""
    load_pkg()
    from sam3_b200 import synth
    return synth.stored_values(synth.sam_dec_tensors(SAMDEC_SEED), 1, None)


def sam_dec_features(H=72, seed=SAMDEC_FEAT_SEED):
    """neck_trk_0..2 stand-ins, channel-last f32 [4H, 4H, 256], [2H, 2H, 256], [H, H, 256]."""
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((s, s, 256), dtype=np.float32) for s in (4 * H, 2 * H, H)]


def sam_dec_torch_names(W: dict):
    """.ggml decoder names -> (prompt encoder dict, mask decoder dict, no_mem_embed) as dump_phase6 reads them
    (the converter's renames, convert_sam3_to_ggml.py:167-187, undone)."""
    import torch
    pe, dec = {}, {}
    for k, v in W.items():
        t = torch.from_numpy(np.ascontiguousarray(v))
        if k == "sam_pe.pe_gaussian":
            pe["pe_layer.positional_encoding_gaussian_matrix"] = t
        elif k.startswith("sam_pe."):
            pe[k[len("sam_pe."):]] = t
        elif k.startswith("sam_dec."):
            n = k[len("sam_dec."):]
            n = n.replace("final_attn.", "transformer.final_attn_token_to_image.")
            n = n.replace("final_norm.", "transformer.norm_final_attn.")
            n = n.replace("upscale.", "output_upscaling.").replace("hyper.", "output_hypernetworks_mlps.")
            if n.startswith("twoway."):
                n = "transformer.layers." + n[len("twoway."):].replace(".sa.", ".self_attn.")
            dec[n] = t
    return pe, dec, torch.from_numpy(W["no_mem_embed"].reshape(-1))


def make_sam_dec(reference: str, out_path: str):
    import torch
    spec = importlib.util.spec_from_file_location("dump_phase6_reference",
                                                  os.path.join(reference, "tests", "dump_phase6_reference.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    W = sam_dec_weights()
    pe, dec, no_mem = sam_dec_torch_names(W)
    f0, f1, f2 = sam_dec_features()
    nchw = [torch.from_numpy(np.ascontiguousarray(f.transpose(2, 0, 1)))[None] for f in (f0, f1, f2)]
    out = {}

    def load(d, name):
        shape = tuple(int(x) for x in open(os.path.join(d, name + ".shape")).read().split(","))
        return np.fromfile(os.path.join(d, name + ".bin"), dtype=np.float32).reshape(tuple(reversed(shape)))

    for c, (name, pos, neg, box) in enumerate(SAMDEC_CASES):
        case = ref.PromptCase(case_id=name, multimask=False, pos_points=[list(p) for p in pos],
                              neg_points=[list(p) for p in neg], box=list(box) if box else [])
        with tempfile.TemporaryDirectory() as d, torch.no_grad():
            ref.dump_case(case, pe, dec, no_mem, nchw[0], nchw[1], nchw[2], d)
            masks = load(d, "sam_dec_masks")[0]                # [4, 288*288]
            out[f"{name}_sparse"] = load(d, "sam_pe_sparse")[0]  # [n, 256]
            out[f"{name}_iou"] = load(d, "sam_dec_iou")[0]
            out[f"{name}_obj_score"] = load(d, "sam_dec_obj_score")[0]
            out[f"{name}_sam_token"] = load(d, "sam_dec_sam_token")[0]
            out[f"{name}_mask_tokens"] = load(d, "sam_dec_mask_tokens")[0]
            out[f"{name}_final_queries"] = load(d, "sam_dec_final_queries")[0]
            out.update(sample(load(d, "sam_dec_block1_keys")[0], f"{name}_block1_keys", 300 + 10 * c))
            out.update(sample(load(d, "sam_dec_upscaled")[0], f"{name}_upscaled", 301 + 10 * c))
            out.update(sample(masks, f"{name}_masks", 302 + 10 * c))
    meta = {"weights_seed": SAMDEC_SEED, "features_seed": SAMDEC_FEAT_SEED, "feat": 72, "input_size": 1008,
            "cases": SAMDEC_CASES,
            "generator": "dump_case() of the reference's tests/dump_phase6_reference.py, imported unmodified"}
    np.savez_compressed(out_path, meta=json.dumps(meta), **out)
    print("wrote", out_path)


MEMENC_SEED = 61
MEMENC_FEAT_SEED = 62


def mem_enc_weights():
    load_pkg()
    from sam3_b200 import synth
    return synth.stored_values(synth.mem_enc_tensors(MEMENC_SEED), 1, None)


def mem_enc_inputs(H=72, seed=MEMENC_FEAT_SEED):
    """neck_trk_2 stand-in [H, H, 256], mask logits [4H, 4H] (a smooth blob plus noise), SAM token [256]."""
    rng = np.random.default_rng(seed)
    pix = rng.standard_normal((H, H, 256), dtype=np.float32)
    S = 4 * H
    yy, xx = np.mgrid[0:S, 0:S].astype(np.float32) / np.float32(S)
    logits = (8.0 * np.exp(-((xx - 0.45) ** 2 + (yy - 0.55) ** 2) / 0.03) - 4.0).astype(np.float32)
    logits += rng.standard_normal((S, S), dtype=np.float32) * np.float32(0.5)
    token = rng.standard_normal(256, dtype=np.float32)
    return pix, logits, token


def mem_enc_torch_names(W: dict):
    import torch
    sd = {}
    for k, v in W.items():
        n = k.replace("mem_enc.ds.", "maskmem_backbone.mask_downsampler.encoder.")
        n = n.replace("mem_enc.fuser.", "maskmem_backbone.fuser.layers.").replace("mem_enc.", "maskmem_backbone.")
        sd[n] = torch.from_numpy(np.ascontiguousarray(v))
    sd["no_obj_ptr"] = sd["no_obj_ptr"].reshape(-1)
    return sd


def make_mem_enc(reference: str, out_path: str):
    import torch
    spec = importlib.util.spec_from_file_location("dump_phase7_reference",
                                                  os.path.join(reference, "tests", "dump_phase7_reference.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    W = mem_enc_weights()
    sd = mem_enc_torch_names(W)
    pix, logits, token = mem_enc_inputs()
    out = {}
    with torch.no_grad():
        pix_t = torch.from_numpy(np.ascontiguousarray(pix.transpose(2, 0, 1)))[None]
        m_t = torch.from_numpy(logits)[None, None]
        for c, score in enumerate((2.5, -1.5)):
            r = ref.run_memory_encoder(sd, pix_t, m_t, torch.tensor([[score]]))
            name = "present" if score > 0 else "absent"
            for i, key in enumerate(("mask_downsampled", "fuser0", "fuser1", "output")):
                a = r[key][0].permute(1, 2, 0).numpy()  # channel-last
                out.update(sample(a, f"{name}_{key}", 400 + 10 * c + i))
            out[f"{name}_obj_ptr"] = ref.run_obj_ptr(sd, torch.from_numpy(token)[None], torch.tensor([[score]]))[0].numpy()
    meta = {"weights_seed": MEMENC_SEED, "inputs_seed": MEMENC_FEAT_SEED, "feat": 72, "img_size": 1008,
            "scores": [2.5, -1.5], "gelu": "erf (the Python reference's F.gelu)",
            "generator": "run_memory_encoder() / run_obj_ptr() of the reference's tests/dump_phase7_reference.py"}
    np.savez_compressed(out_path, meta=json.dumps(meta), **out)
    print("wrote", out_path)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the sam3.cpp checkout (read-only)")
    ap.add_argument("--only", choices=["vit", "mem_attn", "window", "sam_dec", "mem_enc"], default=None)
    a = ap.parse_args()
    if a.only in (None, "vit"):
        make_vit(a.reference, os.path.join(HERE, "vit_golden.npz"))
    if a.only in (None, "mem_attn"):
        make_mem_attn(a.reference, os.path.join(HERE, "mem_attn_golden.npz"))
    if a.only in (None, "window"):
        make_window(a.reference, os.path.join(HERE, "window_golden.npz"))
    if a.only in (None, "sam_dec"):
        make_sam_dec(a.reference, os.path.join(HERE, "sam_dec_golden.npz"))
    if a.only in (None, "mem_enc"):
        make_mem_enc(a.reference, os.path.join(HERE, "mem_enc_golden.npz"))


if __name__ == "__main__":
    main()
