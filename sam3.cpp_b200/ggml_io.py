"""Writer / reader of sam3.cpp's .ggml model files (Python side).

Format (the reader is sam3.cpp:3200-3344 / 3091-3194; the writers are
convert_sam3_to_ggml.py:160-240 and convert_sam2_to_ggml.py:206-318):
  u32 magic ("sam3" 0x73616D33 or "sam2" 0x73616D32), i32 version, i32 ftype,
  i32 n_tensors, the model's i32 hyper-parameters, then per tensor
  i32 n_dims, i32 name_len, i32 dtype, i32 ne[n_dims] (reversed, ggml order),
  name bytes, zero padding to a 32-byte file offset, raw data.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

MAGIC_SAM3 = 0x73616D33
MAGIC_SAM2 = 0x73616D32
F32, F16, Q4_0, Q4_1, Q8_0 = 0, 1, 2, 3, 8
QTYPES = (Q4_0, Q4_1, Q8_0)
BLOCK_BYTES = {Q4_0: 18, Q4_1: 20, Q8_0: 34}

# Substrings that keep a tensor in f32 when the converter writes f16 files
# (convert_sam3_to_ggml.py write_tensor: 1-D tensors and these names).
F32_NAME_PARTS = ("embed", "pos_embed", "tpos", "pe_gaussian", "freqs_cis", "token", "no_obj", "no_mem", "gamma")

# Names the reference quantiser never quantises (examples/quantize.cpp:203-219).
NO_QUANT_PARTS = ("token_embed", "pos_embed", "query_embed", "label_embed", "cls_embed", "point_embeddings",
                  "not_a_point_embed", "no_mask_embed", "no_mem_embed", "no_obj_embed", "presence_token.weight",
                  "iou_token", "mask_tokens", "obj_score_token", "pe_gaussian", "freqs_cis", "gamma", "tpos_enc",
                  "no_obj_ptr", "no_mem_pos_enc", "trk_mask_ds", "latents")


@dataclass
class Record:
    name: str
    dtype: int
    shape: tuple  # PyTorch order (outermost first)
    data: bytes


def file_dtype(name: str, ndim: int, ftype: int) -> int:
    if ftype == F16 and ndim >= 2 and not any(p in name for p in F32_NAME_PARTS):
        return F16
    return F32


def quantisable(name: str, shape: tuple, dtype: int, qblock: int = 32) -> bool:
    """examples/quantize.cpp:220-223: 2-D+, ne0 % 32 == 0, not quantised, not an embedding."""
    return len(shape) >= 2 and shape[-1] % qblock == 0 and dtype not in QTYPES and \
        not any(p in name for p in NO_QUANT_PARTS)


def write(path: str, magic: int, version: int, ftype: int, hparams: list[int], records: list[Record]):
    with open(path, "wb") as f:
        f.write(struct.pack("<I", magic))
        f.write(struct.pack("<iii", version, ftype, len(records)))
        for v in hparams:
            f.write(struct.pack("<i", int(v)))
        for r in records:
            nb = r.name.encode()
            f.write(struct.pack("<iii", len(r.shape), len(nb), r.dtype))
            for d in reversed(r.shape):
                f.write(struct.pack("<i", int(d)))
            f.write(nb)
            pad = (32 - f.tell() % 32) % 32
            f.write(b"\x00" * pad)
            f.write(r.data)


def read(path: str, n_hparams: int):
    """Returns (magic, version, ftype, hparams, {name: Record})."""
    recs = {}
    with open(path, "rb") as f:
        magic, = struct.unpack("<I", f.read(4))
        version, ftype, n = struct.unpack("<iii", f.read(12))
        hp = list(struct.unpack(f"<{n_hparams}i", f.read(4 * n_hparams)))
        for _ in range(n):
            nd, nl, dt = struct.unpack("<iii", f.read(12))
            ne = struct.unpack(f"<{nd}i", f.read(4 * nd))
            name = f.read(nl).decode()
            f.seek((32 - f.tell() % 32) % 32, 1)
            n_el = int(np.prod(ne))
            if dt in QTYPES:
                nbytes = (ne[0] // 32) * BLOCK_BYTES[dt] * (n_el // ne[0])
            else:
                nbytes = n_el * (2 if dt == F16 else 4)
            recs[name] = Record(name, dt, tuple(reversed(ne)), f.read(nbytes))
    return magic, version, ftype, hp, recs
