"""ggml block formats q4_0 / q4_1 / q8_0 — oracle restatement (numpy).

Reference call sites: examples/quantize.cpp:195-265 (selection rule and
ggml_quantize_chunk), sam3.cpp:1065-1081 and 3167-3174 (type-traits to_float).
The algorithm is ggml's reference quantiser (ggml-quants.c, *_ref), an
unvendored dependency of the reference; restated from its published form:
  q4_0  block = f16 d + 16 B nibbles;  d = v/-8 (v: element of max |x|),
        q = min(15, trunc(x/d + 8.5)), value = (q - 8) * d
  q4_1  block = f16 d, f16 m + 16 B;   d = (max-min)/15, m = min,
        q = min(15, trunc((x-m)/d + 0.5)), value = q*d + m
  q8_0  block = f16 d + 32 int8;       d = amax/127, q = roundf(x/d), value = q*d
Nibble j holds element j (low) and element j+16 (high).
"""
import numpy as np

QK = 32
BLOCK_BYTES = {2: 18, 3: 20, 8: 34}


def _roundf(x):
    # C roundf: half away from zero
    return np.sign(x) * np.floor(np.abs(x) + np.float32(0.5))


def quantize(qtype: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    nrows = x.size // x.shape[-1]
    blocks = x.reshape(-1, QK)
    nb = blocks.shape[0]
    if qtype == 2:
        imax = np.abs(blocks).argmax(axis=1)
        vmax = blocks[np.arange(nb), imax][:, None]
        d = (vmax / np.float32(-8)).astype(np.float32)
        with np.errstate(divide="ignore"):
            idv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
        q = np.trunc(blocks * idv + np.float32(8.5)).astype(np.int32)
        q = np.minimum(q, 15).astype(np.uint8)
        qs = q[:, :16] | (q[:, 16:] << 4)
        out = np.concatenate([d.astype(np.float16).view(np.uint8), qs.astype(np.uint8)], axis=1)
    elif qtype == 3:
        vmin = blocks.min(axis=1, keepdims=True)
        vmax = blocks.max(axis=1, keepdims=True)
        d = ((vmax - vmin) / np.float32(15)).astype(np.float32)
        with np.errstate(divide="ignore"):
            idv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
        q = np.trunc((blocks - vmin) * idv + np.float32(0.5)).astype(np.int32)
        q = np.minimum(q, 15).astype(np.uint8)
        qs = q[:, :16] | (q[:, 16:] << 4)
        out = np.concatenate([d.astype(np.float16).view(np.uint8), vmin.astype(np.float16).view(np.uint8),
                              qs.astype(np.uint8)], axis=1)
    elif qtype == 8:
        amax = np.abs(blocks).max(axis=1, keepdims=True)
        d = (amax / np.float32(127)).astype(np.float32)
        with np.errstate(divide="ignore"):
            idv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
        q = _roundf(blocks * idv).astype(np.int8)
        out = np.concatenate([d.astype(np.float16).view(np.uint8), q.view(np.uint8)], axis=1)
    else:
        raise ValueError(qtype)
    return out.reshape(nrows, -1)


def dequantize(qtype: int, raw: np.ndarray, ne0: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1, BLOCK_BYTES[qtype])
    d = raw[:, 0:2].copy().view(np.float16).astype(np.float32)
    if qtype == 2:
        qs = raw[:, 2:18]
        q = np.concatenate([qs & 0x0F, qs >> 4], axis=1).astype(np.int32) - 8
        v = q.astype(np.float32) * d
    elif qtype == 3:
        m = raw[:, 2:4].copy().view(np.float16).astype(np.float32)
        qs = raw[:, 4:20]
        q = np.concatenate([qs & 0x0F, qs >> 4], axis=1).astype(np.float32)
        v = (q * d).astype(np.float32) + m
    else:
        v = raw[:, 2:34].view(np.int8).astype(np.float32) * d
    return v.astype(np.float32).reshape(-1, ne0)
