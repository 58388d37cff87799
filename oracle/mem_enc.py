"""Memory encoder + object-pointer MLP of the tracker — numpy oracle (test infrastructure only).

Restates sam3_encode_memory (sam3.cpp:11506-11603): the chosen mask's logits are resized to the
model input size (sam3_bilinear_interpolate, 9614-9639), passed through sigmoid * scale + bias
(scale 20, bias -10 from the hparams' x100 fields, 226-227), resized to 16 H; the learned mask
downsampler (4 x [3x3 / stride 2 / pad 1 conv, LayerNorm2d eps 1e-6, GELU] then a 1x1 conv); the
1x1 pixel-feature projection of neck_trk_2; their sum through two CXBlocks (sam3_cxblock_forward,
9058-9104: depthwise 7x7 pad 3, LayerNorm2d, pointwise MLP 256 -> 1024 -> 256 with GELU, x + gamma h);
the 1x1 output projection to 64 channels; no_obj_embed_spatial added when the object score is <= 0.
And sam3_extract_obj_ptr_cpu (9344-9418): a 3-layer ReLU MLP of the SAM output token, replaced by
no_obj_ptr when the object score is <= 0.

`gelu` selects the GELU: "tanh" is ggml_gelu, the form sam3.cpp's graph uses (and the engine);
"erf" is PyTorch's F.gelu, the form of the reference's Python dump (tests/dump_phase7_reference.py),
against which the oracle's structure is pinned. Convolution inputs are rounded to f16 when
`f16_inputs` (ggml_conv_2d's im2col runs in the f16 kernel's type). Maps are channel-last.
"""
import numpy as np

from . import nn


def bilinear(src, dst_w, dst_h):
    """sam3_bilinear_interpolate (sam3.cpp:9614-9639): half-pixel centres, f64 source coordinates
    clamped to [0, n - 1], taps x0 = min(floor, n - 2), x0 + 1; f32 weights and f32 blend in the
    reference's order."""
    src = np.asarray(src, np.float32)
    src_h, src_w = src.shape

    def axis(n_dst, n_src):
        s = n_src / n_dst
        f = (np.arange(n_dst, dtype=np.float64) + 0.5) * s - 0.5
        f = np.clip(f, 0.0, n_src - 1)
        i0 = np.minimum(f.astype(np.int64), n_src - 2)
        return i0, (f - i0).astype(np.float32)

    y0, wy = axis(dst_h, src_h)
    x0, wx = axis(dst_w, src_w)
    a = src[y0][:, x0]
    b = src[y0][:, x0 + 1]
    c = src[y0 + 1][:, x0]
    d = src[y0 + 1][:, x0 + 1]
    wx = wx[None, :]
    wy = wy[:, None]
    one = np.float32(1.0)
    top = (one - wx) * a + wx * b
    bot = (one - wx) * c + wx * d
    return ((one - wy) * top + wy * bot).astype(np.float32)


def mask_input(mask_logits, img_size, feat, scale=20.0, bias=-10.0):
    """Mask preprocessing of sam3_encode_memory (sam3.cpp:11516-11520) -> [16 feat, 16 feat]."""
    m = bilinear(mask_logits, img_size, img_size)
    s = (1.0 / (1.0 + np.exp(-m.astype(np.float64)))).astype(np.float32)
    m = (s * np.float32(scale) + np.float32(bias)).astype(np.float32)
    return bilinear(m, 16 * feat, 16 * feat)


def _gelu(x, kind):
    return nn.gelu_tanh(x) if kind == "tanh" else nn.gelu_erf(x)


def _ln2d(x, W, name):
    return nn.layer_norm(x, W[name + ".weight"], W[name + ".bias"], 1e-6)


def dwconv7(x, w, b):
    """Depthwise 7x7 / pad 3 convolution on channel-last [H, W, C], weight [C, 1, 7, 7] (f32 math)."""
    H, Wd, C = x.shape
    xp = np.pad(x, ((3, 3), (3, 3), (0, 0)))
    out = np.zeros((H, Wd, C), np.float32)
    for ky in range(7):
        for kx in range(7):
            out += xp[ky:ky + H, kx:kx + Wd, :] * w[:, 0, ky, kx].astype(np.float32)
    return (out + b.astype(np.float32)).astype(np.float32)


def encode(W, pix_feat, mask_logits, obj_score, img_size, gelu="tanh", f16_inputs=True, taps=None, scale=20.0,
           bias=-10.0):
    """pix_feat [H, H, 256] (neck_trk_2), mask_logits [4H, 4H] -> memory features [H, H, 64]."""
    H = pix_feat.shape[0]
    x = mask_input(mask_logits, img_size, H, scale, bias)[None, :, :, None]  # [1, 16H, 16H, 1]
    for conv_id, norm_id in ((0, 1), (3, 4), (6, 7), (9, 10)):
        x = nn.conv2d_cl(x, W[f"mem_enc.ds.{conv_id}.weight"], W[f"mem_enc.ds.{conv_id}.bias"], stride=2, pad=1,
                         f16_inputs=f16_inputs)
        x = _gelu(_ln2d(x, W, f"mem_enc.ds.{norm_id}"), gelu)
    x = nn.conv2d_cl(x, W["mem_enc.ds.12.weight"], W["mem_enc.ds.12.bias"], f16_inputs=f16_inputs)[0]
    pix = nn.conv2d_cl(pix_feat[None], W["mem_enc.pix_feat_proj.weight"], W["mem_enc.pix_feat_proj.bias"],
                       f16_inputs=f16_inputs)[0]
    h = (pix + x).astype(np.float32)
    if taps is not None:
        taps["mask_downsampled"] = x.copy()
        taps["fused_input"] = h.copy()
    for i in range(2):
        p = f"mem_enc.fuser.{i}"
        t = dwconv7(h, W[p + ".dwconv.weight"], W[p + ".dwconv.bias"])
        t = _ln2d(t, W, p + ".norm")
        t = _gelu(nn.linear(t, W[p + ".pwconv1.weight"], W[p + ".pwconv1.bias"], f16_inputs=f16_inputs), gelu)
        t = nn.linear(t, W[p + ".pwconv2.weight"], W[p + ".pwconv2.bias"], f16_inputs=f16_inputs)
        h = (h + W[p + ".gamma"].astype(np.float32) * t).astype(np.float32)
        if taps is not None:
            taps[f"fuser{i}"] = h.copy()
    out = nn.conv2d_cl(h[None], W["mem_enc.out_proj.weight"], W["mem_enc.out_proj.bias"], f16_inputs=f16_inputs)[0]
    if float(obj_score) <= 0.0 and "no_obj_embed_spatial" in W:
        out = out + W["no_obj_embed_spatial"].reshape(1, 1, -1).astype(np.float32)
    return out.astype(np.float32)


def obj_ptr(W, sam_token, obj_score, f16_inputs=False):
    """sam3_extract_obj_ptr_cpu (sam3.cpp:9344-9418): [256] -> [256]."""
    if float(obj_score) <= 0.0:
        return W["no_obj_ptr"].reshape(-1).astype(np.float32)
    h = np.asarray(sam_token, np.float32)[None]
    for j in range(3):
        h = nn.linear(h, W[f"obj_ptr_proj.layers.{j}.weight"], W[f"obj_ptr_proj.layers.{j}.bias"],
                      f16_inputs=f16_inputs)
        if j < 2:
            h = np.maximum(h, 0)
    return h[0].astype(np.float32)
