"""SAM 2 / 2.1 Hiera backbone + FPN neck — numpy oracle (test infrastructure only).

Follows sam3.cpp: bicubic background PE + tiled window PE
(sam2_bicubic_interpolate_cpu 4072-4109, sam2_compute_pos_embed 4114-4171),
the MultiScaleBlock (sam2_hiera_block_forward 4295-4457: LN 1e-6, shortcut
dim-projection of the normed input + 2x2 max pool on q-stride blocks, zero
padding after the norm + window partition, qkv, q max-pooled inside each
window, attention 1/sqrt(head_dim), projection, unpartition with window
ws//2 after pooling, residual, LN, MLP with tanh GELU, residual), the
backbone (sam2_build_hiera_graph 4462-4527: conv 7x7/s4/p3 + bias + PE) and
the FPN neck (sam2_build_fpn_neck_graph 4532-4603: lateral 1x1 convs,
nearest-2x top-down adds at fpn_top_down_levels, scalp). Not pinned to a
reference dump (the SAM 2 dump script needs the external sam2 package);
its shared pieces (window partition, LayerNorm, attention, convolutions)
are the ones pinned through the ViT / memory-attention fixtures.
"""
import numpy as np

from . import nn

IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def preprocess_u8(frames):
    """uint8 [B, S, S, 3] -> f32 [B, 3, S, S], ImageNet mean/std (sam3.cpp:3518-3544)."""
    v = frames.astype(np.float32) / np.float32(255.0)
    v = (v - np.array(IMAGENET_MEAN, np.float32)) / np.array(IMAGENET_STD, np.float32)
    return np.ascontiguousarray(v.transpose(0, 3, 1, 2)).astype(np.float32)


def _cubic(x):
    x = np.abs(x)
    return np.where(x < 1, (1.25 * x - 2.25) * x * x + 1.0,
                    np.where(x < 2, ((-0.75 * x + 3.75) * x - 6.0) * x + 3.0, 0.0)).astype(np.float32)


def bicubic(src, H_out, W_out):
    """Keys cubic (a = -0.75), half-pixel centres, clamped taps: [C, Hi, Wi] -> [C, Ho, Wo]."""
    C, H_in, W_in = src.shape

    def axis(n_out, n_in):
        f = (np.arange(n_out, dtype=np.float32) + np.float32(0.5)) * np.float32(n_in) / np.float32(n_out) - np.float32(0.5)
        i0 = np.floor(f).astype(np.int64)
        d = (f - i0).astype(np.float32)
        idx = np.stack([np.clip(i0 + j, 0, n_in - 1) for j in (-1, 0, 1, 2)], 1)
        w = np.stack([_cubic(d - j) for j in (-1, 0, 1, 2)], 1)
        return idx, w

    iy, wy = axis(H_out, H_in)
    ix, wx = axis(W_out, W_in)
    out = np.zeros((C, H_out, W_out), np.float32)
    for a in range(4):
        rows = src[:, iy[:, a], :]  # [C, Ho, Wi]
        for b in range(4):
            out += (wy[:, a][None, :, None] * wx[:, b][None, None, :]) * rows[:, :, ix[:, b]]
    return out


def pos_embed(W, H, Wd):
    """Background PE resized to (H, W) plus the tiled window PE, channel-last [H, W, E]."""
    bkg = W["hiera.pos_embed"][0]          # [E, 7, 7]
    win = W["hiera.pos_embed_window"][0]   # [E, ws, ws]
    ws = win.shape[1]
    pe = bicubic(bkg, H, Wd)
    pe = pe + np.tile(win, (1, H // ws + 1, Wd // ws + 1))[:, :H, :Wd]
    return np.ascontiguousarray(pe.transpose(1, 2, 0))


def block(W, x, i, meta, f16_inputs=False):
    din, dout, heads, ws, qs = meta
    p = f"hiera.blocks.{i}"
    B, H, Wd, _ = x.shape
    normed = nn.layer_norm(x, W[p + ".norm1.weight"], W[p + ".norm1.bias"], 1e-6)
    if din != dout:
        shortcut = nn.linear(normed, W[p + ".proj.weight"], W[p + ".proj.bias"], f16_inputs)
        if qs:
            shortcut = nn.maxpool2(shortcut)
    elif qs:
        shortcut = nn.maxpool2(x)
    else:
        shortcut = x
    if ws > 0:
        xw, pad_hw = nn.window_partition(normed, ws)
    else:
        xw = normed
    Bw, Hc, Wc, _ = xw.shape
    qkv = nn.linear(xw.reshape(Bw, Hc * Wc, din), W[p + ".attn.qkv.weight"], W[p + ".attn.qkv.bias"], f16_inputs)
    q, k, v = qkv[..., :dout], qkv[..., dout:2 * dout], qkv[..., 2 * dout:]
    oh, ow = Hc, Wc
    if qs:
        q = nn.maxpool2(q.reshape(Bw, Hc, Wc, dout))
        oh, ow = q.shape[1], q.shape[2]
        q = q.reshape(Bw, oh * ow, dout)
    hd = dout // heads
    sh = lambda t: t.reshape(Bw, t.shape[1], heads, hd).transpose(0, 2, 1, 3).reshape(Bw * heads, t.shape[1], hd)
    o = nn.attention(sh(q), sh(k), sh(v), 1.0 / np.sqrt(hd), f16_inputs)
    o = o.reshape(Bw, heads, oh * ow, hd).transpose(0, 2, 1, 3).reshape(Bw, oh, ow, dout)
    o = nn.linear(o, W[p + ".attn.proj.weight"], W[p + ".attn.proj.bias"], f16_inputs)
    if ws > 0:
        if qs:
            ws_out = ws // 2
            th, tw = H // 2, Wd // 2
            pad = (th + (ws_out - th % ws_out) % ws_out, tw + (ws_out - tw % ws_out) % ws_out)
            o = nn.window_unpartition(o, ws_out, pad, (th, tw))
        else:
            o = nn.window_unpartition(o, ws, pad_hw, (H, Wd))
    res1 = shortcut + o
    n2 = nn.layer_norm(res1, W[p + ".norm2.weight"], W[p + ".norm2.bias"], 1e-6)
    h = nn.gelu_tanh(nn.linear(n2, W[p + ".mlp.fc1.weight"], W[p + ".mlp.fc1.bias"], f16_inputs))
    h = nn.linear(h, W[p + ".mlp.fc2.weight"], W[p + ".mlp.fc2.bias"], f16_inputs)
    return (res1 + h).astype(np.float32)


def backbone(W, chw, cfg, f16_inputs=False):
    """Returns the 4 stage outputs, channel-last [B, S_i, S_i, C_i]."""
    x = nn.conv2d_cl(np.ascontiguousarray(chw.transpose(0, 2, 3, 1)), W["hiera.patch_embed.weight"],
                     W["hiera.patch_embed.bias"], stride=4, pad=3, f16_inputs=f16_inputs)
    x = x + pos_embed(W, x.shape[1], x.shape[2])[None]
    ends, cum = [], 0
    for s in cfg.stages:
        cum += s
        ends.append(cum - 1)
    outs = []
    for i, meta in enumerate(cfg.blocks()):
        x = block(W, x, i, meta, f16_inputs)
        if i in ends:
            outs.append(x)
    return outs


def fpn(W, stages, cfg, f16_inputs=False):
    """Lateral convs (convs[3-i] maps stage i), nearest-2x top-down adds, scalp."""
    lat = [nn.conv2d_cl(stages[i], W[f"fpn.convs.{3 - i}.weight"], W[f"fpn.convs.{3 - i}.bias"],
                        f16_inputs=f16_inputs) for i in range(4)]
    raw = [None] * 4
    prev = None
    for i in range(3, -1, -1):
        td = i in cfg.fpn_top_down_levels
        if td and prev is not None:
            up = prev.repeat(2, axis=1).repeat(2, axis=2)
            raw[i] = lat[i] + up
            prev = raw[i]
        else:
            raw[i] = lat[i]
            if td or prev is None:
                prev = raw[i]
    return raw[:4 - cfg.scalp]
