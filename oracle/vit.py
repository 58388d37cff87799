"""SAM 3 ViT backbone + SimpleFPN neck — numpy oracle (test infrastructure only).

Follows sam3.cpp: prefix sam3_build_vit_prefix_graph (3806-3830), blocks
sam3_vit_block_forward (3710-3801), neck sam3_build_neck_graph (3863-3921),
preprocessing sam3_preprocess_image (3486-3514). Weights are the dict of f32
arrays (PyTorch shapes, ggml tensor names) the engine sees after file dtype
rounding / quantisation (sam3_b200.synth.stored_values).
"""
import numpy as np

from . import nn


def preprocess_u8(frames):
    """uint8 [B, S, S, 3] -> f32 [B, 3, S, S], (p/255 - 0.5)/0.5 (sam3.cpp:3505-3511)."""
    v = frames.astype(np.float32) / np.float32(255.0)
    v = (v - np.float32(0.5)) / np.float32(0.5)
    return np.ascontiguousarray(v.transpose(0, 3, 1, 2))


def prefix(W, chw, cfg, f16_inputs=False):
    """Patch embed (conv 14/s14, no bias) + tiled pos + ln_pre -> [B, G, G, E]."""
    x = nn.conv2d_cl(np.ascontiguousarray(chw.transpose(0, 2, 3, 1)), W["vit.patch_embed.proj.weight"], None,
                     stride=cfg.patch, pad=0, f16_inputs=f16_inputs)
    G = cfg.grid
    pos = W["vit.pos_embed"]  # [g, g, E]
    g = pos.shape[0]
    tiled = np.tile(pos, (G // g, G // g, 1)) if G % g == 0 else pos[:G, :G]
    x = x + tiled[None]
    return nn.layer_norm(x, W["vit.ln_pre.weight"], W["vit.ln_pre.bias"], 1e-5)


def block(W, x, i, cfg, f16_inputs=False):
    """One ViT block on x [B, G, G, E]."""
    p = f"vit.blocks.{i}"
    E, NH = cfg.embed, cfg.heads
    HD = E // NH
    is_global = i in cfg.global_idx
    shortcut = x
    xn = nn.layer_norm(x, W[p + ".norm1.weight"], W[p + ".norm1.bias"], 1e-5)
    B, H, Wd, _ = xn.shape
    if not is_global:
        xn, pad_hw = nn.window_partition(xn, cfg.window)
    Bw, Hc, Wc, _ = xn.shape
    L = Hc * Wc
    qkv = nn.linear(xn.reshape(Bw, L, E), W[p + ".attn.qkv.weight"], W[p + ".attn.qkv.bias"], f16_inputs)
    qkv = qkv.reshape(Bw, L, 3, NH, HD).transpose(2, 0, 3, 1, 4)  # [3, Bw, NH, L, HD]
    q, k, v = qkv[0], qkv[1], qkv[2]
    cis = W[p + ".attn.freqs_cis"]
    q = nn.rope(q, cis)
    k = nn.rope(k, cis)
    o = nn.attention(q.reshape(Bw * NH, L, HD), k.reshape(Bw * NH, L, HD), v.reshape(Bw * NH, L, HD),
                     1.0 / np.sqrt(HD), f16_inputs)
    o = o.reshape(Bw, NH, L, HD).transpose(0, 2, 1, 3).reshape(Bw, Hc, Wc, E)
    o = nn.linear(o, W[p + ".attn.proj.weight"], W[p + ".attn.proj.bias"], f16_inputs)
    if not is_global:
        o = nn.window_unpartition(o, cfg.window, pad_hw, (H, Wd))
    x = shortcut + o
    xn = nn.layer_norm(x, W[p + ".norm2.weight"], W[p + ".norm2.bias"], 1e-5)
    h = nn.gelu_erf(nn.linear(xn, W[p + ".mlp.lin1.weight"], W[p + ".mlp.lin1.bias"], f16_inputs))
    h = nn.linear(h, W[p + ".mlp.lin2.weight"], W[p + ".mlp.lin2.bias"], f16_inputs)
    return (x + h).astype(np.float32)


def backbone(W, chw, cfg, f16_inputs=False, depth=None, taps=()):
    """Full ViT; returns (output [B, G, G, E], {block_idx: output} for idx in taps)."""
    x = prefix(W, chw, cfg, f16_inputs)
    out = {}
    for i in range(cfg.depth if depth is None else depth):
        x = block(W, x, i, cfg, f16_inputs)
        if i in taps:
            out[i] = x.copy()
    return x, out


def neck(W, x, pfx="neck.trk.", f16_inputs=False):
    """SimpleFPN path on x [B, G, G, E] -> 4 maps [B, S, S, D] (4x, 2x, 1x, 0.5x)."""
    o0 = nn.deconv2x2_cl(x, W[pfx + "0.dconv_2x2_0.weight"], W[pfx + "0.dconv_2x2_0.bias"], f16_inputs)
    o0 = nn.gelu_erf(o0)
    o0 = nn.deconv2x2_cl(o0, W[pfx + "0.dconv_2x2_1.weight"], W[pfx + "0.dconv_2x2_1.bias"], f16_inputs)
    o0 = nn.conv2d_cl(o0, W[pfx + "0.conv_1x1.weight"], W[pfx + "0.conv_1x1.bias"], f16_inputs=f16_inputs)
    o0 = nn.conv2d_cl(o0, W[pfx + "0.conv_3x3.weight"], W[pfx + "0.conv_3x3.bias"], pad=1, f16_inputs=f16_inputs)
    o1 = nn.deconv2x2_cl(x, W[pfx + "1.dconv_2x2.weight"], W[pfx + "1.dconv_2x2.bias"], f16_inputs)
    o1 = nn.conv2d_cl(o1, W[pfx + "1.conv_1x1.weight"], W[pfx + "1.conv_1x1.bias"], f16_inputs=f16_inputs)
    o1 = nn.conv2d_cl(o1, W[pfx + "1.conv_3x3.weight"], W[pfx + "1.conv_3x3.bias"], pad=1, f16_inputs=f16_inputs)
    o2 = nn.conv2d_cl(x, W[pfx + "2.conv_1x1.weight"], W[pfx + "2.conv_1x1.bias"], f16_inputs=f16_inputs)
    o2 = nn.conv2d_cl(o2, W[pfx + "2.conv_3x3.weight"], W[pfx + "2.conv_3x3.bias"], pad=1, f16_inputs=f16_inputs)
    o3 = nn.maxpool2(x)
    o3 = nn.conv2d_cl(o3, W[pfx + "3.conv_1x1.weight"], W[pfx + "3.conv_1x1.bias"], f16_inputs=f16_inputs)
    o3 = nn.conv2d_cl(o3, W[pfx + "3.conv_3x3.weight"], W[pfx + "3.conv_3x3.bias"], pad=1, f16_inputs=f16_inputs)
    return [o0, o1, o2, o3]
