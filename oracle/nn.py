"""Shared numpy building blocks of the oracle (test infrastructure only).

Each function restates the ggml op sequence the reference builds; the
`f16_inputs` switch rounds GEMM operands to f16 the way ggml's CPU mul_mat
does for f16 weights (sam3.cpp:6635-6636 host reference rounds its input).
"""
import ctypes
import ctypes.util

import numpy as np


def f16r(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def layer_norm(x, w, b, eps):
    """ggml_norm + mul + add over the last dim (sam3.cpp:1036-1060); f64 statistics."""
    x = np.asarray(x, np.float32)
    mean = x.mean(axis=-1, keepdims=True, dtype=np.float64)
    xc = x - mean.astype(np.float32)
    var = np.square(xc).mean(axis=-1, keepdims=True, dtype=np.float64)
    y = xc * (1.0 / np.sqrt(var + eps)).astype(np.float32)
    y = y * w.astype(np.float32)
    if b is not None:
        y = y + b.astype(np.float32)
    return y.astype(np.float32)


def linear(x, w, b=None, f16_inputs=False):
    """ggml_mul_mat(w, x) + b: x [..., K], w [N, K] -> [..., N] (f32 accumulate)."""
    if f16_inputs:
        x, w = f16r(x), f16r(w)
    y = np.matmul(x.reshape(-1, x.shape[-1]).astype(np.float32), w.astype(np.float32).T)
    if b is not None:
        y = y + b.astype(np.float32)
    return y.reshape(*x.shape[:-1], w.shape[0]).astype(np.float32)


def gelu_erf(x):
    from scipy.special import erf
    x = np.asarray(x, np.float32)
    return (np.float32(0.5) * x * (np.float32(1.0) + erf(x * np.float32(0.7071067811865476)))).astype(np.float32)


def gelu_tanh(x):
    xd = x.astype(np.float64)
    return (0.5 * xd * (1.0 + np.tanh(0.7978845608028654 * (xd + 0.044715 * xd ** 3)))).astype(np.float32)


def relu(x):
    return np.maximum(x, 0).astype(np.float32)


def rope(x, cis):
    """sam3_apply_rope (sam3.cpp:3667-3706): x [..., N, D] pairs (2i, 2i+1), cis [N, D/2, 2]."""
    xr = x[..., 0::2]
    xi = x[..., 1::2]
    c = cis[..., 0]
    s = cis[..., 1]
    out = np.empty_like(x)
    out[..., 0::2] = xr * c - xi * s
    out[..., 1::2] = xr * s + xi * c
    return out


def attention(q, k, v, scale, f16_inputs=False):
    """softmax(q k^T * scale) v for q [B, Nq, D], k/v [B, Nk, D] (no mask), f32 softmax."""
    if f16_inputs:
        q, k, v = f16r(q), f16r(k), f16r(v)
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    out = np.empty((q.shape[0], q.shape[1], v.shape[2]), np.float32)
    for b in range(q.shape[0]):
        # chunk queries to bound memory for the global / memory-attention sizes
        for s in range(0, q.shape[1], 2048):
            sc = np.matmul(q[b, s:s + 2048], k[b].T)
            sc *= np.float32(scale)
            sc -= sc.max(axis=-1, keepdims=True)
            np.exp(sc, out=sc)
            sc /= sc.sum(axis=-1, keepdims=True, dtype=np.float64).astype(np.float32)
            out[b, s:s + 2048] = np.matmul(sc, v[b])
    return out


def window_partition(x, ws):
    """[B, H, W, C] -> ([B*nw, ws, ws, C], (Hp, Wp)); zero pad after the norm (sam3.cpp:4190-4228)."""
    B, H, W, C = x.shape
    ph = (ws - H % ws) % ws
    pw = (ws - W % ws) % ws
    if ph or pw:
        x = np.pad(x, ((0, 0), (0, ph), (0, pw), (0, 0)))
    Hp, Wp = H + ph, W + pw
    x = x.reshape(B, Hp // ws, ws, Wp // ws, ws, C).transpose(0, 1, 3, 2, 4, 5).reshape(-1, ws, ws, C)
    return x, (Hp, Wp)


def window_unpartition(w, ws, pad_hw, hw):
    """Inverse of window_partition (sam3.cpp:4240-4277)."""
    Hp, Wp = pad_hw
    H, W = hw
    B = w.shape[0] // ((Hp // ws) * (Wp // ws))
    x = w.reshape(B, Hp // ws, Wp // ws, ws, ws, -1).transpose(0, 1, 3, 2, 4, 5).reshape(B, Hp, Wp, -1)
    return x[:, :H, :W, :]


def maxpool2(x):
    """2x2/s2 max pool on [B, H, W, C] (floor), ggml_pool_2d MAX k=2 s=2 p=0."""
    B, H, W, C = x.shape
    H2, W2 = H // 2, W // 2
    x = x[:, :2 * H2, :2 * W2, :].reshape(B, H2, 2, W2, 2, C)
    return x.max(axis=(2, 4))


def conv2d_cl(x, w, b, stride=1, pad=0, f16_inputs=False):
    """Conv2d on channel-last x [B, H, W, Cin] with PyTorch weight [Cout, Cin, k, k]."""
    B, H, W, Cin = x.shape
    Cout, _, k, _ = w.shape
    xp = np.pad(x, ((0, 0), (pad, pad), (pad, pad), (0, 0))) if pad else x
    OH = (H + 2 * pad - k) // stride + 1
    OW = (W + 2 * pad - k) // stride + 1
    wf = w.transpose(2, 3, 1, 0).reshape(k * k * Cin, Cout)  # (ky, kx, ci) x co
    if f16_inputs:
        xp, wf = f16r(xp), f16r(wf)
    out = np.zeros((B, OH, OW, Cout), np.float32)
    for ky in range(k):
        for kx in range(k):
            patch = xp[:, ky:ky + stride * OH:stride, kx:kx + stride * OW:stride, :]
            out += np.matmul(patch.reshape(-1, Cin), wf[(ky * k + kx) * Cin:(ky * k + kx + 1) * Cin]).reshape(
                B, OH, OW, Cout)
    if b is not None:
        out += b.astype(np.float32)
    return out


def deconv2x2_cl(x, w, b, f16_inputs=False):
    """ConvTranspose2d k=2 s=2 on channel-last x [B, H, W, Cin], weight [Cin, Cout, 2, 2]."""
    B, H, W, Cin = x.shape
    Cout = w.shape[1]
    if f16_inputs:
        x, w = f16r(x), f16r(w)
    out = np.zeros((B, 2 * H, 2 * W, Cout), np.float32)
    xf = x.reshape(-1, Cin)
    for ky in range(2):
        for kx in range(2):
            out[:, ky::2, kx::2, :] = np.matmul(xf, w[:, :, ky, kx]).reshape(B, H, W, Cout)
    if b is not None:
        out += b.astype(np.float32)
    return out


# The C library's single-precision sinf / cosf / powf, the functions sam3.cpp calls for its
# sinusoidal encodings (numpy's own float32 sin / cos may differ from them in the last bit).
_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
for _fn, _n in (("sinf", 1), ("cosf", 1), ("powf", 2)):
    getattr(_libm, _fn).restype = ctypes.c_float
    getattr(_libm, _fn).argtypes = [ctypes.c_float] * _n


def libm_f32(fn, *args):
    """Elementwise libm `fn` ("sinf", "cosf", "powf") over float32 arrays (broadcast), float32 result."""
    f = getattr(_libm, fn)
    arrs = np.broadcast_arrays(*[np.asarray(a, dtype=np.float32) for a in args])
    out = np.empty(arrs[0].shape, np.float32)
    flat = [a.ravel() for a in arrs]
    o = out.ravel()
    for k in range(o.size):
        o[k] = f(*[float(a[k]) for a in flat])
    return out


def sine_pe_2d(H, W, d_model):
    """sam3_sinusoidal_pe_2d (sam3.cpp:3597-3633) as channel-last [H, W, d_model]: the same float32
    operations (pos = (p + 1) / n * 2pi, dim_t = powf(1e4, paired / half), sinf / cosf of pos / dim_t)
    and the same libm functions, so the values are bit-exact."""
    half = d_model // 2
    scale = np.float32(2.0) * np.float32(np.pi)
    y = ((np.arange(H, dtype=np.float32) + np.float32(1)) / np.float32(H)) * scale
    x = ((np.arange(W, dtype=np.float32) + np.float32(1)) / np.float32(W)) * scale
    i = np.arange(half)
    dim_t = libm_f32("powf", np.float32(10000.0), (i & ~1).astype(np.float32) / np.float32(half))
    py = (y[:, None] / dim_t[None, :]).astype(np.float32)
    px = (x[:, None] / dim_t[None, :]).astype(np.float32)
    even = (i % 2 == 0)[None, :]
    vy = np.where(even, libm_f32("sinf", py), libm_f32("cosf", py)).astype(np.float32)
    vx = np.where(even, libm_f32("sinf", px), libm_f32("cosf", px)).astype(np.float32)
    pe = np.empty((H, W, d_model), np.float32)
    pe[:, :, :half] = vy[:, None, :]
    pe[:, :, half:] = vx[None, :, :]
    return pe


def resize_bilinear_u8(img, dst_w, dst_h):
    """sam3_resize_bilinear (sam3.cpp:3441-3481): uint8 [H, W, 3] -> uint8 [dst_h, dst_w, 3].

    Half-pixel centres (o + 0.5) * (src / dst) - 0.5 clamped at 0, the second tap clamped at
    the last row / column, v = wy0 (wx0 p00 + wx p01) + wy (wx0 p10 + wx p11) in f64 with every
    operation rounded on its own (numpy never fuses), then (int)(v + 0.5) clamped to [0, 255].
    """
    img = np.asarray(img, np.uint8)
    H, W = img.shape[0], img.shape[1]

    def taps(n_out, n_in):
        s = np.float64(n_in) / np.float64(n_out)
        f = (np.arange(n_out, dtype=np.float64) + 0.5) * s - 0.5
        f = np.maximum(f, 0.0)
        i0 = f.astype(np.int64)
        i1 = np.where(i0 < n_in - 1, i0 + 1, i0)
        return i0, i1, f - i0

    y0, y1, wy = taps(dst_h, H)
    x0, x1, wx = taps(dst_w, W)
    src = img.astype(np.float64)
    wy, wx = wy[:, None, None], wx[None, :, None]
    wy0, wx0 = 1.0 - wy, 1.0 - wx
    p00 = src[y0][:, x0]
    p01 = src[y0][:, x1]
    p10 = src[y1][:, x0]
    p11 = src[y1][:, x1]
    v = wy0 * (wx0 * p00 + wx * p01) + wy * (wx0 * p10 + wx * p11)
    return np.clip((v + 0.5).astype(np.int64), 0, 255).astype(np.uint8)
