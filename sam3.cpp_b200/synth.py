"""Seeded synthetic models and frames in sam3.cpp's .ggml format.

There are no checkpoints on this machine, so benchmarks and parity tests use
random-init weights of the reference architectures: every weight and bias
N(0, 0.02), LayerNorm gamma = 1, beta = 0 (or a seeded random affine for
tests), drawn from numpy.random.default_rng(seed) in file-record order.
Values are rounded to the file dtype chosen by the reference converter
(convert_sam3_to_ggml.py write_tensor) and, for q4_0 / q4_1 / q8_0 models,
quantised with the reference quantiser's selection rule
(examples/quantize.cpp:195-223). RoPE tables (`attn.freqs_cis`) are not
random: they follow compute_axial_cis (sam3.cpp:3555-3586; window blocks
scale 1, global blocks scale window/grid).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import ggml_io


# ---------------------------------------------------------------- configs
@dataclass
class Sam3Config:
    img_size: int = 1008
    patch: int = 14
    embed: int = 1024
    depth: int = 32
    heads: int = 16
    mlp_ratio_x1000: int = 4625
    window: int = 24
    global_idx: tuple = (7, 15, 23, 31)
    neck_dim: int = 256
    neck_mid: int = 512
    visual_only: int = 1
    with_mem_attn: bool = False
    mem_out_dim: int = 64
    mem_attn_layers: int = 4
    num_maskmem: int = 7
    max_obj_ptrs: int = 16
    mem_ffn: int = 2048
    with_sam_dec: bool = False

    @property
    def grid(self) -> int:
        return self.img_size // self.patch

    @property
    def mlp(self) -> int:
        return int(np.float32(self.embed) * np.float32(self.mlp_ratio_x1000 / 1000.0))

    @property
    def pretrain_grid(self) -> int:
        return self.grid // 3 if self.grid % 3 == 0 else self.grid

    def hparams(self) -> list[int]:
        # sam3_load_hparams order (sam3.cpp:1477-1520); n_global entries of global_attn_idx
        hp = [self.img_size, self.patch, self.embed, self.depth, self.heads, self.mlp_ratio_x1000, self.window,
              len(self.global_idx), *self.global_idx]
        hp += [1024, 16, 24, 32, 49408, 256]              # text encoder (unused by the engine)
        hp += [self.neck_dim]
        hp += [6, 8, 2048, 6, 8, 2048, 200, 3, 1, 4]      # fenc, ddec, geom, presence, geom queries
        hp += [256, 2, 3, 3]                              # sam decoder
        hp += [self.mem_out_dim, self.mem_attn_layers, self.num_maskmem, self.max_obj_ptrs]
        hp += [2, self.visual_only]                       # n_amb_experts, visual_only
        return hp


SAM3_VIT_L = Sam3Config()


@dataclass
class Sam2Config:
    """SAM 2 / 2.1 Hiera image encoder + FPN neck (+ optional memory attention)."""
    img_size: int = 1024
    embed: int = 96
    heads: int = 1
    stages: tuple = (1, 2, 7, 2)
    global_idx: tuple = (5, 7, 9)
    q_pool: int = 3
    window_spec: tuple = (8, 4, 14, 7)
    bkg: tuple = (7, 7)
    scalp: int = 1
    neck_dim: int = 256
    fpn_top_down_levels: tuple = (2, 3)
    with_mem_attn: bool = False
    mem_out_dim: int = 64
    mem_attn_layers: int = 4
    num_maskmem: int = 7
    max_obj_ptrs: int = 16
    mem_ffn: int = 2048
    with_sam_dec: bool = False

    def hparams(self) -> list[int]:
        # sam2_load_hparams order (sam3.cpp:1564-1626), 57 fields for the Hiera backbone
        g = list(self.global_idx) + [0] * (8 - len(self.global_idx))
        td = list(self.fpn_top_down_levels) + [0] * (4 - len(self.fpn_top_down_levels))
        hp = [self.img_size, 1, self.embed, self.heads, len(self.stages), *self.stages, len(self.global_idx), *g,
              self.q_pool, *self.window_spec, self.bkg[0], self.bkg[1], self.scalp, self.neck_dim,
              len(self.fpn_top_down_levels), *td]
        hp += [256, 2, 3, 3]                                       # sam decoder
        hp += [self.mem_out_dim, self.mem_attn_layers, self.num_maskmem, self.max_obj_ptrs]
        hp += [2000, -1000]                                        # sigmoid scale / bias x100
        hp += [1, 1, 1, 1, 1, 1, 0, 1, 0, 1, 1, 1, 1, 1, 1]        # tracking flags, is_sam2_1 = 1
        return hp

    def blocks(self):
        """Per-block (dim_in, dim_out, heads, window, q_stride) following sam3.cpp:1676-1742."""
        ends, cum = [], 0
        for s in self.stages:
            cum += s
            ends.append(cum - 1)
        qpool_blocks = [ends[s] + 1 for s in range(len(self.stages) - 1)][:self.q_pool]
        out, cur, embed, heads = [], 0, self.embed, self.heads
        for i in range(sum(self.stages)):
            ws = 0 if i in self.global_idx else self.window_spec[cur]
            dout = embed
            if i > 0 and i - 1 == ends[cur]:
                dout = embed * 2
                heads *= 2
                cur += 1
            out.append((embed, dout, heads, ws, i in qpool_blocks))
            embed = dout
        return out

    def stage_dims(self):
        return [self.embed * (2 ** s) for s in range(len(self.stages))]


HIERA_T = Sam2Config()
HIERA_L = Sam2Config(embed=144, heads=2, stages=(2, 6, 36, 4), global_idx=(23, 33, 43), window_spec=(8, 4, 16, 8))


def sam2_tensors(cfg: Sam2Config, seed: int = 0, ln_random: bool = False) -> dict:
    """name -> f32 array (PyTorch shape) of a SAM 2.1 Hiera image encoder + FPN neck."""
    g = _Gen(seed, ln_random)
    E0 = cfg.embed
    T: dict[str, np.ndarray] = {}
    T["hiera.patch_embed.weight"] = g.w(E0, 3, 7, 7)
    T["hiera.patch_embed.bias"] = g.w(E0)
    T["hiera.pos_embed"] = g.w(1, E0, cfg.bkg[0], cfg.bkg[1])
    T["hiera.pos_embed_window"] = g.w(1, E0, cfg.window_spec[0], cfg.window_spec[0])
    for i, (din, dout, heads, ws, qs) in enumerate(cfg.blocks()):
        p = f"hiera.blocks.{i}"
        T[f"{p}.norm1.weight"], T[f"{p}.norm1.bias"] = g.ln(din)
        T[f"{p}.attn.qkv.weight"] = g.w(3 * dout, din)
        T[f"{p}.attn.qkv.bias"] = g.w(3 * dout)
        T[f"{p}.attn.proj.weight"] = g.w(dout, dout)
        T[f"{p}.attn.proj.bias"] = g.w(dout)
        T[f"{p}.norm2.weight"], T[f"{p}.norm2.bias"] = g.ln(dout)
        T[f"{p}.mlp.fc1.weight"] = g.w(4 * dout, dout)
        T[f"{p}.mlp.fc1.bias"] = g.w(4 * dout)
        T[f"{p}.mlp.fc2.weight"] = g.w(dout, 4 * dout)
        T[f"{p}.mlp.fc2.bias"] = g.w(dout)
        if din != dout:
            T[f"{p}.proj.weight"] = g.w(dout, din)
            T[f"{p}.proj.bias"] = g.w(dout)
    dims = cfg.stage_dims()
    for i in range(4):
        T[f"fpn.convs.{i}.weight"] = g.w(cfg.neck_dim, dims[3 - i], 1, 1)
        T[f"fpn.convs.{i}.bias"] = g.w(cfg.neck_dim)
    if cfg.with_mem_attn:
        _mem_attn(g, T, cfg.neck_dim, cfg.mem_out_dim, cfg.mem_attn_layers, cfg.mem_ffn, cfg.num_maskmem)
    if cfg.with_sam_dec:
        _sam_dec(g, T, cfg.neck_dim)
    return T


# ---------------------------------------------------------------- RoPE / PE
def axial_cis(dim: int, end_x: int, end_y: int, theta: float = 10000.0, scale: float = 1.0) -> np.ndarray:
    """compute_axial_cis as (cos, sin) pairs: [end_x*end_y, dim//2, 2] f32."""
    q = dim // 4
    freqs = (1.0 / (np.float32(theta) ** (np.arange(0, dim, 4, dtype=np.float32)[:q] / np.float32(dim)))).astype(np.float32)
    t = np.arange(end_x * end_y, dtype=np.float32)
    tx = (t % end_x).astype(np.float32) * np.float32(scale)
    ty = np.floor(t / end_x).astype(np.float32) * np.float32(scale)
    ax = np.outer(tx, freqs).astype(np.float32)
    ay = np.outer(ty, freqs).astype(np.float32)
    ang = np.concatenate([ax, ay], axis=1)
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32)


# ---------------------------------------------------------------- tensors
class _Gen:
    def __init__(self, seed: int, ln_random: bool):
        self.rng = np.random.default_rng(seed)
        self.ln_random = ln_random

    def w(self, *shape, std=0.02):
        return (self.rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    def ln(self, n):
        if self.ln_random:
            g = 1.0 + self.w(n, std=0.1)
            b = self.w(n, std=0.1)
            return g.astype(np.float32), b
        return np.ones(n, np.float32), np.zeros(n, np.float32)


def _neck(g: _Gen, T: dict, pfx: str, E: int, D: int, mid: int):
    T[pfx + "0.dconv_2x2_0.weight"] = g.w(E, mid, 2, 2)       # ConvTranspose2d [Cin, Cout, kH, kW]
    T[pfx + "0.dconv_2x2_0.bias"] = g.w(mid)
    T[pfx + "0.dconv_2x2_1.weight"] = g.w(mid, D, 2, 2)
    T[pfx + "0.dconv_2x2_1.bias"] = g.w(D)
    T[pfx + "0.conv_1x1.weight"] = g.w(D, D, 1, 1)
    T[pfx + "0.conv_1x1.bias"] = g.w(D)
    T[pfx + "0.conv_3x3.weight"] = g.w(D, D, 3, 3)
    T[pfx + "0.conv_3x3.bias"] = g.w(D)
    T[pfx + "1.dconv_2x2.weight"] = g.w(E, mid, 2, 2)
    T[pfx + "1.dconv_2x2.bias"] = g.w(mid)
    T[pfx + "1.conv_1x1.weight"] = g.w(D, mid, 1, 1)
    T[pfx + "1.conv_1x1.bias"] = g.w(D)
    T[pfx + "1.conv_3x3.weight"] = g.w(D, D, 3, 3)
    T[pfx + "1.conv_3x3.bias"] = g.w(D)
    for s in (2, 3):
        T[pfx + f"{s}.conv_1x1.weight"] = g.w(D, E, 1, 1)
        T[pfx + f"{s}.conv_1x1.bias"] = g.w(D)
        T[pfx + f"{s}.conv_3x3.weight"] = g.w(D, D, 3, 3)
        T[pfx + f"{s}.conv_3x3.bias"] = g.w(D)


def _mem_attn(g: _Gen, T: dict, D: int, MD: int, layers: int, ffn: int, num_maskmem: int):
    for i in range(layers):
        p = f"mem_attn.layers.{i}"
        for a in ("sa.q_proj", "sa.k_proj", "sa.v_proj", "sa.out_proj", "ca.q_proj"):
            T[f"{p}.{a}.weight"] = g.w(D, D)
            T[f"{p}.{a}.bias"] = g.w(D)
        T[f"{p}.ca.k_proj.weight"] = g.w(D, MD)
        T[f"{p}.ca.k_proj.bias"] = g.w(D)
        T[f"{p}.ca.v_proj.weight"] = g.w(D, MD)
        T[f"{p}.ca.v_proj.bias"] = g.w(D)
        T[f"{p}.ca.out_proj.weight"] = g.w(D, D)
        T[f"{p}.ca.out_proj.bias"] = g.w(D)
        T[f"{p}.linear1.weight"] = g.w(ffn, D)
        T[f"{p}.linear1.bias"] = g.w(ffn)
        T[f"{p}.linear2.weight"] = g.w(D, ffn)
        T[f"{p}.linear2.bias"] = g.w(D)
        for n in ("norm1", "norm2", "norm3"):
            T[f"{p}.{n}.weight"], T[f"{p}.{n}.bias"] = g.ln(D)
    T["mem_attn.norm.weight"], T["mem_attn.norm.bias"] = g.ln(D)
    T["mem_enc.tpos_enc"] = g.w(num_maskmem, 1, 1, MD)
    T["obj_ptr_tpos_proj.weight"] = g.w(MD, D)
    T["obj_ptr_tpos_proj.bias"] = g.w(MD)


def _sam_dec(g: _Gen, T: dict, D: int, ffn: int = 2048, n_mask: int = 4, depth: int = 2):
    """SAM prompt-encoder embeddings + SAM mask decoder + the tracker's no_mem_embed, in .ggml naming
    (convert_sam3_to_ggml.py:167-185; shapes as registered at sam3.cpp:1848-1966). Embeddings and the
    Gaussian PE matrix are N(0, 1) like their PyTorch initialisation, linear weights N(0, 0.02)."""
    Di = D // 2  # the cross-attention internal dim (downsample rate 2)
    T["sam_pe.pe_gaussian"] = g.w(2, D // 2, std=1.0)
    for i in range(4):
        T[f"sam_pe.point_embeddings.{i}.weight"] = g.w(1, D, std=1.0)
    T["sam_pe.not_a_point_embed.weight"] = g.w(1, D, std=1.0)
    T["sam_pe.no_mask_embed.weight"] = g.w(1, D, std=1.0)
    T["sam_dec.iou_token.weight"] = g.w(1, D, std=1.0)
    T["sam_dec.mask_tokens.weight"] = g.w(n_mask, D, std=1.0)
    T["sam_dec.obj_score_token.weight"] = g.w(1, D, std=1.0)

    def attn(pfx, di):
        for a in ("q_proj", "k_proj", "v_proj"):
            T[f"{pfx}.{a}.weight"] = g.w(di, D)
            T[f"{pfx}.{a}.bias"] = g.w(di)
        T[f"{pfx}.out_proj.weight"] = g.w(D, di)
        T[f"{pfx}.out_proj.bias"] = g.w(D)

    for i in range(depth):
        p = f"sam_dec.twoway.{i}"
        attn(p + ".sa", D)
        attn(p + ".cross_attn_token_to_image", Di)
        attn(p + ".cross_attn_image_to_token", Di)
        for n in ("norm1", "norm2", "norm3", "norm4"):
            T[f"{p}.{n}.weight"], T[f"{p}.{n}.bias"] = g.ln(D)
        T[f"{p}.mlp.lin1.weight"] = g.w(ffn, D)
        T[f"{p}.mlp.lin1.bias"] = g.w(ffn)
        T[f"{p}.mlp.lin2.weight"] = g.w(D, ffn)
        T[f"{p}.mlp.lin2.bias"] = g.w(D)
    attn("sam_dec.final_attn", Di)
    T["sam_dec.final_norm.weight"], T["sam_dec.final_norm.bias"] = g.ln(D)
    T["sam_dec.upscale.0.weight"] = g.w(D, D // 4, 2, 2)          # ConvTranspose2d [Cin, Cout, kH, kW]
    T["sam_dec.upscale.0.bias"] = g.w(D // 4)
    T["sam_dec.upscale.1.weight"], T["sam_dec.upscale.1.bias"] = g.ln(D // 4)   # LayerNorm2d
    T["sam_dec.upscale.3.weight"] = g.w(D // 4, D // 8, 2, 2)
    T["sam_dec.upscale.3.bias"] = g.w(D // 8)
    T["sam_dec.conv_s0.weight"] = g.w(D // 8, D, 1, 1)
    T["sam_dec.conv_s0.bias"] = g.w(D // 8)
    T["sam_dec.conv_s1.weight"] = g.w(D // 4, D, 1, 1)
    T["sam_dec.conv_s1.bias"] = g.w(D // 4)
    for m in range(n_mask):
        for j in range(3):
            T[f"sam_dec.hyper.{m}.layers.{j}.weight"] = g.w(D // 8 if j == 2 else D, D)
            T[f"sam_dec.hyper.{m}.layers.{j}.bias"] = g.w(D // 8 if j == 2 else D)
    for j in range(3):
        T[f"sam_dec.iou_prediction_head.layers.{j}.weight"] = g.w(n_mask if j == 2 else D, D)
        T[f"sam_dec.iou_prediction_head.layers.{j}.bias"] = g.w(n_mask if j == 2 else D)
        T[f"sam_dec.pred_obj_score_head.layers.{j}.weight"] = g.w(1 if j == 2 else D, D)
        T[f"sam_dec.pred_obj_score_head.layers.{j}.bias"] = g.w(1 if j == 2 else D)
    T["no_mem_embed"] = g.w(1, 1, D)


def _mem_enc(g: _Gen, T: dict, D: int = 256, MD: int = 64, ffn: int = 1024):
    """Memory encoder (mask downsampler, pixel projection, 2 CXBlock fusers, out projection), object-
    pointer MLP and the no-object embeddings, in .ggml naming (convert_sam3_to_ggml.py:158-187; shapes as
    registered at sam3.cpp:1968-2056). gamma is the CXBlocks' layer scale (PyTorch init 1e-6; drawn
    around 0.5 here so the fusers matter)."""
    ch = [1, 4, 16, 64, D]
    for s, (ci, ni) in enumerate(((0, 1), (3, 4), (6, 7), (9, 10))):
        T[f"mem_enc.ds.{ci}.weight"] = g.w(ch[s + 1], ch[s], 3, 3, std=0.3)
        T[f"mem_enc.ds.{ci}.bias"] = g.w(ch[s + 1])
        T[f"mem_enc.ds.{ni}.weight"], T[f"mem_enc.ds.{ni}.bias"] = g.ln(ch[s + 1])
    T["mem_enc.ds.12.weight"] = g.w(D, D, 1, 1, std=0.05)
    T["mem_enc.ds.12.bias"] = g.w(D)
    T["mem_enc.pix_feat_proj.weight"] = g.w(D, D, 1, 1, std=0.05)
    T["mem_enc.pix_feat_proj.bias"] = g.w(D)
    for i in range(2):
        p = f"mem_enc.fuser.{i}"
        T[p + ".dwconv.weight"] = g.w(D, 1, 7, 7, std=0.1)
        T[p + ".dwconv.bias"] = g.w(D)
        T[p + ".norm.weight"], T[p + ".norm.bias"] = g.ln(D)
        T[p + ".pwconv1.weight"] = g.w(ffn, D, std=0.05)
        T[p + ".pwconv1.bias"] = g.w(ffn)
        T[p + ".pwconv2.weight"] = g.w(D, ffn, std=0.05)
        T[p + ".pwconv2.bias"] = g.w(D)
        T[p + ".gamma"] = (0.5 + g.w(D, std=0.1)).astype(np.float32)
    T["mem_enc.out_proj.weight"] = g.w(MD, D, 1, 1, std=0.05)
    T["mem_enc.out_proj.bias"] = g.w(MD)
    for j in range(3):
        T[f"obj_ptr_proj.layers.{j}.weight"] = g.w(D, D, std=0.05)
        T[f"obj_ptr_proj.layers.{j}.bias"] = g.w(D)
    T["no_obj_ptr"] = g.w(1, D, std=1.0)
    T["no_obj_embed_spatial"] = g.w(1, MD, std=1.0)


def mem_enc_tensors(seed: int, D: int = 256, MD: int = 64, ln_random: bool = True) -> dict:
    """The memory-encoder + object-pointer tensors alone (the names and shapes _mem_enc writes)."""
    g = _Gen(seed, ln_random)
    T: dict[str, np.ndarray] = {}
    _mem_enc(g, T, D, MD)
    return T


def sam_dec_tensors(seed: int, D: int = 256, ln_random: bool = True) -> dict:
    """The SAM prompt encoder + mask decoder tensors alone (the names and shapes _sam_dec writes)."""
    g = _Gen(seed, ln_random)
    T: dict[str, np.ndarray] = {}
    _sam_dec(g, T, D)
    return T


def sam3_tensors(cfg: Sam3Config, seed: int = 0, ln_random: bool = False, neck_det: bool = False) -> dict:
    """name -> f32 array (PyTorch shape) of a SAM 3 image encoder (+ optional memory attention)."""
    g = _Gen(seed, ln_random)
    E, G, W = cfg.embed, cfg.grid, cfg.window
    T: dict[str, np.ndarray] = {}
    T["vit.patch_embed.proj.weight"] = g.w(E, 3, cfg.patch, cfg.patch)
    T["vit.pos_embed"] = g.w(cfg.pretrain_grid, cfg.pretrain_grid, E)
    T["vit.ln_pre.weight"], T["vit.ln_pre.bias"] = g.ln(E)
    for i in range(cfg.depth):
        p = f"vit.blocks.{i}"
        T[f"{p}.norm1.weight"], T[f"{p}.norm1.bias"] = g.ln(E)
        T[f"{p}.attn.qkv.weight"] = g.w(3 * E, E)
        T[f"{p}.attn.qkv.bias"] = g.w(3 * E)
        T[f"{p}.attn.proj.weight"] = g.w(E, E)
        T[f"{p}.attn.proj.bias"] = g.w(E)
        T[f"{p}.norm2.weight"], T[f"{p}.norm2.bias"] = g.ln(E)
        T[f"{p}.mlp.lin1.weight"] = g.w(cfg.mlp, E)
        T[f"{p}.mlp.lin1.bias"] = g.w(cfg.mlp)
        T[f"{p}.mlp.lin2.weight"] = g.w(E, cfg.mlp)
        T[f"{p}.mlp.lin2.bias"] = g.w(E)
        hd = E // cfg.heads
        if i in cfg.global_idx:
            T[f"{p}.attn.freqs_cis"] = axial_cis(hd, G, G, scale=W / G)
        else:
            T[f"{p}.attn.freqs_cis"] = axial_cis(hd, W, W, scale=1.0)
    if neck_det and not cfg.visual_only:
        _neck(g, T, "neck.det.", E, cfg.neck_dim, cfg.neck_mid)
    _neck(g, T, "neck.trk.", E, cfg.neck_dim, cfg.neck_mid)
    if cfg.with_mem_attn:
        _mem_attn(g, T, cfg.neck_dim, cfg.mem_out_dim, cfg.mem_attn_layers, cfg.mem_ffn, cfg.num_maskmem)
    if cfg.with_sam_dec:
        _sam_dec(g, T, cfg.neck_dim)
    return T


# ---------------------------------------------------------------- files
def _round_to_dtype(name: str, a: np.ndarray, ftype: int) -> tuple[int, np.ndarray]:
    dt = ggml_io.file_dtype(name, a.ndim, ftype)
    if dt == ggml_io.F16:
        a = a.astype(np.float16).astype(np.float32)
    return dt, a


def stored_values(T: dict, ftype: int = 1, qtype: int | None = None, quantize=None, dequantize=None) -> dict:
    """The f32 values the engine sees after file-dtype rounding and quantisation."""
    out = {}
    for name, a in T.items():
        dt, v = _round_to_dtype(name, a, ftype)
        if qtype is not None and ggml_io.quantisable(name, v.shape, dt):
            raw = quantize(qtype, v.reshape(-1, v.shape[-1]))
            v = dequantize(qtype, raw, v.shape[-1]).reshape(v.shape)
        out[name] = v
    return out


def write_model(path: str, T: dict, hparams: list[int], magic: int, version: int, ftype: int = 1,
                qtype: int | None = None, quantize=None):
    """Writes T (name -> f32 array, PyTorch shape) as a .ggml file.

    ftype 0/1 follows the converter's dtype rule; with `qtype` the quantisable
    tensors are then stored as q4_0 / q4_1 / q8_0 blocks (quantize(qtype, rows)
    returns the raw blocks, e.g. sam3_b200.quantize_rows)."""
    recs = []
    for name, a in T.items():
        dt, v = _round_to_dtype(name, a, ftype)
        if qtype is not None and ggml_io.quantisable(name, v.shape, dt):
            raw = quantize(qtype, v.reshape(-1, v.shape[-1]))
            recs.append(ggml_io.Record(name, qtype, v.shape, raw.tobytes()))
        elif dt == ggml_io.F16:
            recs.append(ggml_io.Record(name, dt, v.shape, v.astype(np.float16).tobytes()))
        else:
            recs.append(ggml_io.Record(name, dt, v.shape, np.ascontiguousarray(v, np.float32).tobytes()))
    file_ftype = qtype if qtype is not None else ftype
    ggml_io.write(path, magic, version, file_ftype, hparams, recs)


def write_sam3(path: str, cfg: Sam3Config, seed: int = 0, ftype: int = 1, qtype: int | None = None,
               quantize=None, ln_random: bool = False, neck_det: bool = False) -> dict:
    T = sam3_tensors(cfg, seed, ln_random=ln_random, neck_det=neck_det)
    write_model(path, T, cfg.hparams(), ggml_io.MAGIC_SAM3, 3, ftype, qtype, quantize)
    return T


def write_sam2(path: str, cfg: Sam2Config, seed: int = 0, ftype: int = 1, qtype: int | None = None,
               quantize=None, ln_random: bool = False) -> dict:
    T = sam2_tensors(cfg, seed, ln_random=ln_random)
    write_model(path, T, cfg.hparams(), ggml_io.MAGIC_SAM2, 1, ftype, qtype, quantize)
    return T


def frames_u8(n: int, size: int, base_seed: int = 1000) -> np.ndarray:
    """Seeded uniform uint8 frames [n, size, size, 3] (frame i from default_rng(base_seed + i))."""
    out = np.empty((n, size, size, 3), dtype=np.uint8)
    for i in range(n):
        out[i] = np.random.default_rng(base_seed + i).integers(0, 256, size=(size, size, 3), dtype=np.uint8)
    return out
