"""B200 encoder engine for sam3.cpp — Python host side over the C ABI.

The product is ``libsam3b200.so`` (sm_100a kernels + C++14 host engine) built
from ``csrc/`` and declared in ``include/sam3_b200.h``. This module binds it
with ctypes and adds the Python-side plumbing a caller needs: device buffers
come from PyTorch (``tensor.data_ptr()``), the engine owns its own weights
and workspace.

The directory is named ``sam3.cpp_b200``; import it through ``load()`` in
``__graft_entry__.py`` / ``tests/conftest.py`` which registers it as the
module ``sam3_b200``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libsam3b200.so")
CSRC = os.path.join(PKG_DIR, "csrc")

S3B_F32, S3B_F16, S3B_Q4_0, S3B_Q4_1, S3B_Q8_0 = 0, 1, 2, 3, 8
ACT_NONE, ACT_GELU_ERF, ACT_GELU_TANH, ACT_RELU = 0, 1, 2, 3
ENCODE_NO_NECK, ENCODE_NO_DET = 1, 2
DEC_ADD_NO_MEM, DEC_DEVICE_PTRS = 1, 2

ERRORS = {
    0: "S3B_OK", -1: "S3B_ERR_ARG", -2: "S3B_ERR_IO", -3: "S3B_ERR_FORMAT", -4: "S3B_ERR_CUDA",
    -5: "S3B_ERR_STATE", -6: "S3B_ERR_UNSUPPORTED", -7: "S3B_ERR_DEVICE", -8: "S3B_ERR_OOM",
}

class TensorDesc(ctypes.Structure):
    """s3b_tensor_desc: one caller-owned host tensor for s3b_load_weights."""
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int32), ("n_dims", ctypes.c_int32),
                ("ne", ctypes.c_int64 * 4), ("data", ctypes.c_void_p)]


# Every symbol declared in include/sam3_b200.h: (name, restype, argtypes)
_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
_S = ctypes.c_char_p
SYMBOLS = [
    ("s3b_create", _I, [_I, ctypes.POINTER(_P)]),
    ("s3b_destroy", None, [_P]),
    ("s3b_last_error", _S, [_P]),
    ("s3b_set_stream", _I, [_P, _P]),
    ("s3b_reset_stream", _I, [_P]),
    ("s3b_sync", _I, [_P]),
    ("s3b_set_option", _I, [_P, _S, _I64]),
    ("s3b_profile_begin", _I, [_P, _I]),
    ("s3b_profile_end", _I, [_P, ctypes.POINTER(ctypes.c_double), _I]),
    ("s3b_load_model", _I, [_P, _S]),
    ("s3b_load_model_cached", _I, [_P, _S, _S]),
    ("s3b_load_weights", _I, [_P, _I, ctypes.POINTER(ctypes.c_int32), _I, _I, ctypes.POINTER(TensorDesc), _I]),
    ("s3b_inspect_model", _I, [_S, ctypes.POINTER(ctypes.c_int32), _I, _S, _I]),
    ("s3b_model_info", _I, [_P, ctypes.POINTER(ctypes.c_int32), _I]),
    ("s3b_encode_u8", _I, [_P, _P, _I, _I, _I]),
    ("s3b_encode_chw", _I, [_P, _P, _I, _I, _I]),
    ("s3b_encode_u8_device", _I, [_P, _P, _I, _I, _I]),
    ("s3b_encode_chw_device", _I, [_P, _P, _I, _I, _I]),
    ("s3b_encode_image_u8", _I, [_P, _P, _I, _I, _I, _I]),
    ("s3b_encode_image_u8_device", _I, [_P, _P, _I, _I, _I, _I]),
    ("s3b_output_shape", _I, [_P, _S, ctypes.POINTER(_I64)]),
    ("s3b_output_copy", _I, [_P, _S, _I, _P, _I64]),
    ("s3b_output_device_ptr", _I, [_P, _S, _I, ctypes.POINTER(_P)]),
    ("s3b_output_host_bind", _I, [_P, _S, _P, _I64]),
    ("s3b_peer_copy_output", _I, [_P, _S, _I, _P, _I, _I64]),
    ("s3b_device_alloc", _I, [_P, _I64, ctypes.POINTER(_P)]),
    ("s3b_device_free", _I, [_P, _P]),
    ("s3b_ipc_export", _I, [_P, _P, _P]),
    ("s3b_ipc_open", _I, [_P, _P, ctypes.POINTER(_P)]),
    ("s3b_ipc_close", _I, [_P, _P]),
    ("s3b_mem_attn", _I, [_P, _P, _P, _I, _P, _P, _I, _I, _P, _I]),
    ("s3b_mem_attn_bank", _I, [_P, _P, _P, _I, _P, _P, _P, _I, _P, _P, _I, _P]),
    ("s3b_op_build_prompt", _I, [_P, _I, _P, _P, _P, _I, _P, _P, _I, _P, _P, _I64, ctypes.POINTER(_I),
                                 ctypes.POINTER(_I)]),
    ("s3b_sam_decode", _I, [_P, _I, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P]),
    ("s3b_sam_prompt_tokens", _I, [_P, _P, _P, _I, _P, _I, _I, _I, _P, _I]),
    ("s3b_sam_dense_pe", _I, [_P, _I, _P]),
    ("s3b_sam_best_mask", _I, [_P, _I, _I]),
    ("s3b_mem_encode", _I, [_P, _I, _P, _P, _I, _I, _P, _P, _I]),
    ("s3b_obj_ptr", _I, [_P, _P, _P, _P, _I]),
    ("s3b_track_step", _I, [_P, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P, _I, _P, _P, _P, _P]),
    ("s3b_test_wait_timeout", _I, [_P, _I64, _I]),
    ("s3b_select_memory_frames", _I, [_I, _I, ctypes.POINTER(_I), _I]),
    ("s3b_sine_pe_2d", _I, [_I, _I, _I, _P]),
    ("s3b_op_gemm", _I, [_P, _P, _I64, _P, _I64, _I, _I, _I, _P, _I, _P, _I, _I64, _P, _I64]),
    ("s3b_op_gemm_rope", _I, [_P, _P, _I64, _P, _I64, _I, _I, _I, _P, _P, _I, _I, _I64, _P, _I, _I64]),
    ("s3b_op_gemm_q", _I, [_P, _P, _I64, _P, _I, _I, _I, _I, _P, _I, _P, _I, _I64, _P, _I64]),
    ("s3b_op_attention", _I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F]),
    ("s3b_op_attention_qkv", _I, [_P, _P, _I64, _P, _I64, _I, _I, _I, _I, _F]),
    ("s3b_op_resize_bilinear_u8", _I, [_P, _P, _I, _I, _I, _P, _I, _I]),
    ("s3b_op_layernorm", _I, [_P, _P, _P, _I, _I64, _I, _P, _P, _F]),
    ("s3b_op_conv3x3", _I, [_P, _P, _I, _I, _I, _I, _P, _P, _P, _I]),
    ("s3b_op_deconv2x2", _I, [_P, _P, _I, _I, _I, _I, _P, _P, _I, _P, _I, _I]),
    ("s3b_conv3x3_noalloc", _I, [_P, _I, _I, _I, _I, _P, _P, _P, _I, _P]),
    ("s3b_conv3x3_noalloc_status", _I, [ctypes.POINTER(_I)]),
    ("s3b_op_dequantize", _I, [_P, _P, _I, _I64, _I64, _P]),
    ("s3b_row_size", _I64, [_I, _I64]),
    ("s3b_quantize_rows", _I, [_I, _P, _I64, _I64, _P]),
    ("s3b_dequantize_rows", _I, [_I, _P, _I64, _I64, _P]),
]

_lib = None


def build(verbose: bool = False) -> str:
    """Compiles libsam3b200.so for sm_100a with the Makefile in csrc/."""
    cmd = ["make", "-C", CSRC, "-j", str(min(8, os.cpu_count() or 1))]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode != 0:
        print(r.stdout[-4000:], r.stderr[-4000:])
    if r.returncode != 0:
        raise RuntimeError("building libsam3b200.so failed")
    return LIB_PATH


def lib() -> ctypes.CDLL:
    """Loads the in-tree shared library (fails loudly when it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: run build() (make -C {CSRC}) first")
    L = ctypes.CDLL(LIB_PATH)
    for name, res, args in SYMBOLS:
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


class S3BError(RuntimeError):
    pass


def _ptr(x) -> int | None:
    """Raw address of a torch tensor, numpy array, int, or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    raise TypeError(type(x))


# ---------------------------------------------------------------- host format helpers
def row_size(qtype: int, ne0: int) -> int:
    return int(lib().s3b_row_size(qtype, ne0))


def quantize_rows(qtype: int, x: np.ndarray) -> np.ndarray:
    """Quantises f32 rows [nrows, ne0] to raw ggml blocks (uint8 [nrows, row_size])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    ne0 = x.shape[-1]
    nrows = x.size // ne0
    out = np.empty((nrows, row_size(qtype, ne0)), dtype=np.uint8)
    rc = lib().s3b_quantize_rows(qtype, x.ctypes.data, ne0, nrows, out.ctypes.data)
    if rc != 0:
        raise S3BError(f"s3b_quantize_rows: {ERRORS.get(rc, rc)}")
    return out


def dequantize_rows(qtype: int, raw: np.ndarray, ne0: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    nrows = raw.size // row_size(qtype, ne0)
    out = np.empty((nrows, ne0), dtype=np.float32)
    rc = lib().s3b_dequantize_rows(qtype, raw.ctypes.data, ne0, nrows, out.ctypes.data)
    if rc != 0:
        raise S3BError(f"s3b_dequantize_rows: {ERRORS.get(rc, rc)}")
    return out


def sam_best_mask(iou, multimask: bool) -> int:
    """Index of the mask sam3_propagate_single keeps (s3b_sam_best_mask)."""
    a = np.ascontiguousarray(np.asarray(iou, np.float32).reshape(-1))
    r = lib().s3b_sam_best_mask(_ptr(a), a.size, 1 if multimask else 0)
    if r < 0:
        raise S3BError(f"s3b_sam_best_mask: {ERRORS.get(r, r)}")
    return r


def select_memory_frames(bank_size: int, max_slots: int) -> list[int]:
    """Memory-bank slots memory attention reads (s3b_select_memory_frames)."""
    buf = (ctypes.c_int * max(bank_size, 1))()
    n = lib().s3b_select_memory_frames(bank_size, max_slots, buf, max(bank_size, 1))
    if n < 0:
        raise S3BError(f"s3b_select_memory_frames: {ERRORS.get(n, n)}")
    return list(buf[:n])


def sine_pe_2d(H: int, W: int, d_model: int) -> np.ndarray:
    """Sinusoidal 2D PE [H, W, d_model] as the engine computes it (s3b_sine_pe_2d)."""
    out = np.empty((H, W, d_model), dtype=np.float32)
    rc = lib().s3b_sine_pe_2d(H, W, d_model, out.ctypes.data)
    if rc != 0:
        raise S3BError(f"s3b_sine_pe_2d: {ERRORS.get(rc, rc)}")
    return out


def inspect_model(path: str) -> dict:
    """Host-only parse of a .ggml file (s3b_inspect_model); raises S3BError on corrupt files."""
    info = (ctypes.c_int32 * 7)()
    err = ctypes.create_string_buffer(512)
    rc = lib().s3b_inspect_model(path.encode(), info, 7, err, 512)
    if rc != 0:
        raise S3BError(f"s3b_inspect_model: {ERRORS.get(rc, rc)}: {err.value.decode()}")
    keys = ["is_sam2", "img_size", "n_tensors", "ftype", "depth", "embed_dim", "n_quantised"]
    return dict(zip(keys, list(info)))


# ---------------------------------------------------------------- engine
class Engine:
    """One engine context on one CUDA device (s3b_create / s3b_destroy)."""

    def __init__(self, device: int = 0):
        self._L = lib()
        h = ctypes.c_void_p()
        rc = self._L.s3b_create(device, ctypes.byref(h))
        if rc != 0:
            raise S3BError(f"s3b_create({device}) failed: {ERRORS.get(rc, rc)}")
        self.h = h
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            self._L.s3b_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int, what: str):
        if rc != 0:
            msg = self._L.s3b_last_error(self.h)
            raise S3BError(f"{what}: {ERRORS.get(rc, rc)}: {msg.decode() if msg else ''}")

    def last_error(self) -> str:
        m = self._L.s3b_last_error(self.h)
        return m.decode() if m else ""

    def set_stream(self, stream_handle: int | None):
        """Runs on `stream_handle` (a cudaStream_t value; 0 = legacy default stream);
        None returns to a stream owned by the context."""
        if stream_handle is None:
            self._check(self._L.s3b_reset_stream(self.h), "s3b_reset_stream")
        else:
            self._check(self._L.s3b_set_stream(self.h, stream_handle), "s3b_set_stream")

    def sync(self):
        self._check(self._L.s3b_sync(self.h), "s3b_sync")

    def set_option(self, key: str, value: int):
        self._check(self._L.s3b_set_option(self.h, key.encode(), value), "s3b_set_option")

    def profile_begin(self, with_events: bool = True):
        self._check(self._L.s3b_profile_begin(self.h, 1 if with_events else 0), "s3b_profile_begin")

    def profile_end(self) -> dict:
        buf = (ctypes.c_double * 17)()
        self._check(self._L.s3b_profile_end(self.h, buf, 17), "s3b_profile_end")
        v = list(buf)
        return {"gemm": {"launches": v[0], "ms": v[1], "flops": v[2], "bytes": v[3]},
                "attention": {"launches": v[4], "ms": v[5], "flops": v[6], "bytes": v[7]},
                "layernorm": {"launches": v[9], "ms": v[10], "bytes": v[12]},
                "weight_staging": {"launches": v[13], "ms": v[14], "bytes": v[16]},
                "launches": int(v[8])}

    def load_model(self, path: str):
        self._check(self._L.s3b_load_model(self.h, path.encode()), "s3b_load_model")

    def load_model_cached(self, path: str, cache_path: str) -> bool:
        """s3b_load_model through the device-weight cache; True when the model came from the cache."""
        rc = self._L.s3b_load_model_cached(self.h, path.encode(), cache_path.encode())
        self._check(min(rc, 0), "s3b_load_model_cached")
        return rc == 1

    def load_weights(self, is_sam2: int, hparams, ftype: int, tensors):
        """s3b_load_weights from host tensors: tensors = [(name, dtype, shape (PyTorch order), bytes-like)]."""
        descs = (TensorDesc * len(tensors))()
        keep = []
        for i, (name, dtype, shape, data) in enumerate(tensors):
            buf = np.frombuffer(data, dtype=np.uint8)
            keep.append(buf)
            ne = list(reversed(shape)) + [1] * (4 - len(shape))
            descs[i] = TensorDesc(name.encode(), dtype, len(shape), (ctypes.c_int64 * 4)(*ne), buf.ctypes.data)
        hp = (ctypes.c_int32 * len(hparams))(*[int(v) for v in hparams])
        self._check(self._L.s3b_load_weights(self.h, is_sam2, hp, len(hparams), ftype, descs, len(tensors)),
                    "s3b_load_weights")

    def model_info(self) -> dict:
        buf = (ctypes.c_int32 * 7)()
        self._check(self._L.s3b_model_info(self.h, buf, 7), "s3b_model_info")
        keys = ["is_sam2", "img_size", "n_blocks", "embed_dim", "neck_dim", "mem_attn_layers", "weights_mib"]
        return dict(zip(keys, list(buf)))

    # -- encoder
    def encode_u8(self, frames, flags: int = 0):
        """frames: uint8 [n, S, S, 3] numpy (host) or torch CUDA tensor (device)."""
        n, S = int(frames.shape[0]), int(frames.shape[1])
        if hasattr(frames, "is_cuda") and frames.is_cuda:
            rc = self._L.s3b_encode_u8_device(self.h, frames.data_ptr(), n, S, flags)
        else:
            frames = np.ascontiguousarray(frames, dtype=np.uint8)
            rc = self._L.s3b_encode_u8(self.h, frames.ctypes.data, n, S, flags)
        self._check(rc, "s3b_encode_u8")

    def encode_image_u8(self, frames, flags: int = 0):
        """frames: uint8 [n, H, W, 3] of any size, numpy (host) or torch CUDA tensor (device);
        resized to the model size on the device unless already at it."""
        n, H, W = int(frames.shape[0]), int(frames.shape[1]), int(frames.shape[2])
        if hasattr(frames, "is_cuda") and frames.is_cuda:
            rc = self._L.s3b_encode_image_u8_device(self.h, frames.data_ptr(), n, W, H, flags)
        else:
            frames = np.ascontiguousarray(frames, dtype=np.uint8)
            rc = self._L.s3b_encode_image_u8(self.h, frames.ctypes.data, n, W, H, flags)
        self._check(rc, "s3b_encode_image_u8")

    def encode_chw(self, frames, flags: int = 0):
        """frames: f32 [n, 3, S, S] numpy (host) or torch CUDA tensor (device)."""
        n, S = int(frames.shape[0]), int(frames.shape[2])
        if hasattr(frames, "is_cuda") and frames.is_cuda:
            rc = self._L.s3b_encode_chw_device(self.h, frames.data_ptr(), n, S, flags)
        else:
            frames = np.ascontiguousarray(frames, dtype=np.float32)
            rc = self._L.s3b_encode_chw(self.h, frames.ctypes.data, n, S, flags)
        self._check(rc, "s3b_encode_chw")

    def output_shape(self, name: str) -> tuple:
        ne = (ctypes.c_int64 * 4)()
        self._check(self._L.s3b_output_shape(self.h, name.encode(), ne), "s3b_output_shape")
        return tuple(ne)

    def output(self, name: str, frame: int = 0, out: np.ndarray | None = None) -> np.ndarray:
        """Frame `frame` of an output as numpy [H][W][C] (ggml [C, W, H])."""
        ne = self.output_shape(name)
        if out is None:
            out = np.empty((ne[2], ne[1], ne[0]), dtype=np.float32)
        assert out.dtype == np.float32 and out.flags.c_contiguous and out.size == ne[0] * ne[1] * ne[2]
        self._check(self._L.s3b_output_copy(self.h, name.encode(), frame, out.ctypes.data, out.size),
                    "s3b_output_copy")
        return out

    def output_host_bind(self, name: str, host=None):
        """Binds host memory (a pinned torch CPU tensor or numpy array of f32, frames x frame elements) to
        output `name`: every later encode copies each pass's frames into it, overlapped with the next pass
        (s3b_output_host_bind). None unbinds."""
        if host is None:
            self._check(self._L.s3b_output_host_bind(self.h, name.encode(), None, 0), "s3b_output_host_bind")
            return
        n = host.numel() if hasattr(host, "numel") else host.size
        self._check(self._L.s3b_output_host_bind(self.h, name.encode(), _ptr(host), n), "s3b_output_host_bind")

    def output_device_ptr(self, name: str, frame: int = 0) -> int:
        p = ctypes.c_void_p()
        self._check(self._L.s3b_output_device_ptr(self.h, name.encode(), frame, ctypes.byref(p)),
                    "s3b_output_device_ptr")
        return int(p.value)

    # -- per-frame features to the tracking GPU
    def peer_copy_output(self, name: str, frame: int, dst_ptr: int, dst_device: int, dst_bytes: int):
        self._check(self._L.s3b_peer_copy_output(self.h, name.encode(), frame, dst_ptr, dst_device, dst_bytes),
                    "s3b_peer_copy_output")

    def device_alloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p()
        self._check(self._L.s3b_device_alloc(self.h, nbytes, ctypes.byref(p)), "s3b_device_alloc")
        return int(p.value)

    def device_free(self, ptr: int):
        self._check(self._L.s3b_device_free(self.h, ptr), "s3b_device_free")

    def ipc_export(self, ptr: int) -> bytes:
        h = ctypes.create_string_buffer(64)
        self._check(self._L.s3b_ipc_export(self.h, ptr, h), "s3b_ipc_export")
        return h.raw

    def ipc_open(self, handle: bytes) -> int:
        assert len(handle) == 64
        p = ctypes.c_void_p()
        self._check(self._L.s3b_ipc_open(self.h, ctypes.create_string_buffer(handle, 64), ctypes.byref(p)),
                    "s3b_ipc_open")
        return int(p.value)

    def ipc_close(self, ptr: int):
        self._check(self._L.s3b_ipc_close(self.h, ptr), "s3b_ipc_close")

    # -- memory attention
    def mem_attn(self, curr, src_pos, feat: int, prompt, prompt_pos, n_ptr_tokens: int, out=None):
        """All numpy (host) or all torch CUDA tensors (device)."""
        dev = hasattr(curr, "is_cuda") and curr.is_cuda
        m_total = int(prompt.shape[0])
        if out is None:
            if dev:
                import torch
                out = torch.empty_like(curr)
            else:
                out = np.empty_like(np.asarray(curr, dtype=np.float32))
        if not dev:
            curr = np.ascontiguousarray(curr, dtype=np.float32)
            src_pos = np.ascontiguousarray(src_pos, dtype=np.float32)
            prompt = np.ascontiguousarray(prompt, dtype=np.float32)
            prompt_pos = np.ascontiguousarray(prompt_pos, dtype=np.float32)
        rc = self._L.s3b_mem_attn(self.h, _ptr(curr), _ptr(src_pos), feat, _ptr(prompt), _ptr(prompt_pos),
                                  m_total, n_ptr_tokens, _ptr(out), 1 if dev else 0)
        self._check(rc, "s3b_mem_attn")
        return out

    @staticmethod
    def _bank_args(slot_feats, slot_pes, slot_tpos, obj_ptrs, ptr_tpos):
        n_slots = len(slot_feats)
        feats = (ctypes.c_void_p * max(n_slots, 1))(*[_ptr(f) for f in slot_feats])
        pes = None
        if slot_pes is not None:
            pes = (ctypes.c_void_p * max(n_slots, 1))(*[_ptr(p) for p in slot_pes])
        tpos = (ctypes.c_int * max(n_slots, 1))(*[int(t) for t in slot_tpos])
        n_ptrs = 0 if obj_ptrs is None else int(obj_ptrs.shape[0])
        ptpos = (ctypes.c_int * max(n_ptrs, 1))(*[int(t) for t in (ptr_tpos if n_ptrs else [])])
        return n_slots, feats, pes, tpos, n_ptrs, ptpos

    def mem_attn_bank(self, curr, feat: int, slot_feats, slot_tpos, obj_ptrs=None, ptr_tpos=(), slot_pes=None,
                      src_pos=None, out=None):
        """Memory attention with the prompt built on the device from a memory bank (s3b_mem_attn_bank).
        All tensors are torch CUDA tensors: curr [N, 256], slot_feats list of [N, 64], obj_ptrs [P, 256]."""
        if out is None:
            import torch
            out = torch.empty_like(curr)
        n_slots, feats, pes, tpos, n_ptrs, ptpos = self._bank_args(slot_feats, slot_pes, slot_tpos, obj_ptrs, ptr_tpos)
        rc = self._L.s3b_mem_attn_bank(self.h, _ptr(curr), _ptr(src_pos), feat, feats, pes, tpos, n_slots,
                                       _ptr(obj_ptrs), ptpos, n_ptrs, _ptr(out))
        self._check(rc, "s3b_mem_attn_bank")
        return out

    def build_prompt(self, feat: int, slot_feats, slot_tpos, obj_ptrs=None, ptr_tpos=(), slot_pes=None):
        """The device prompt build alone: (prompt [M, 64], prompt_pos [M, 64], n_ptr_tokens) as torch CUDA tensors."""
        import torch
        n_slots, feats, pes, tpos, n_ptrs, ptpos = self._bank_args(slot_feats, slot_pes, slot_tpos, obj_ptrs, ptr_tpos)
        cap = n_slots * feat * feat + 4 * n_ptrs
        dev = slot_feats[0].device if n_slots else obj_ptrs.device
        prompt = torch.empty(max(cap, 1), 64, device=dev, dtype=torch.float32)
        pos = torch.empty_like(prompt)
        m_total, n_ptr = ctypes.c_int(0), ctypes.c_int(0)
        rc = self._L.s3b_op_build_prompt(self.h, feat, feats, pes, tpos, n_slots, _ptr(obj_ptrs), ptpos, n_ptrs,
                                         prompt.data_ptr(), pos.data_ptr(), cap, ctypes.byref(m_total),
                                         ctypes.byref(n_ptr))
        self._check(rc, "s3b_op_build_prompt")
        return prompt[:m_total.value], pos[:m_total.value], n_ptr.value

    # -- SAM mask decoder
    def sam_prompt_tokens(self, box=None, pos_points=(), neg_points=(), orig_size=None) -> np.ndarray:
        """Sparse prompt tokens [n, 256] (box corners, positive, negative points, padding token)."""
        pos = np.ascontiguousarray(np.asarray(pos_points, np.float32).reshape(-1, 2))
        neg = np.ascontiguousarray(np.asarray(neg_points, np.float32).reshape(-1, 2))
        bx = None if box is None else np.ascontiguousarray(np.asarray(box, np.float32).reshape(4))
        w, h = orig_size if orig_size is not None else (self.model_info()["img_size"],) * 2
        cap = 32
        out = np.empty((cap, 256), np.float32)
        n = self._L.s3b_sam_prompt_tokens(self.h, _ptr(bx), _ptr(pos) if len(pos) else None, len(pos),
                                          _ptr(neg) if len(neg) else None, len(neg), int(w), int(h), _ptr(out), cap)
        self._check(min(n, 0), "s3b_sam_prompt_tokens")
        return out[:n].copy()

    def sam_dense_pe(self, feat: int) -> np.ndarray:
        out = np.empty((feat * feat, 256), np.float32)
        self._check(self._L.s3b_sam_dense_pe(self.h, feat, _ptr(out)), "s3b_sam_dense_pe")
        return out

    def sam_decode(self, feat: int, image_feats, feat_s0, feat_s1, sparse=None, add_no_mem=False, outs=None):
        """SAM mask decoder: all numpy (host) or all torch CUDA tensors (device, asynchronous on the engine's
        stream). Returns (masks [4, 4 feat, 4 feat], iou [4], obj_score [1], mask_tokens [4, 256])."""
        dev = hasattr(image_feats, "is_cuda") and image_feats.is_cuda
        S = 4 * feat
        if outs is None:
            if dev:
                import torch
                mk = lambda *s: torch.empty(*s, device=image_feats.device, dtype=torch.float32)
            else:
                mk = lambda *s: np.empty(s, np.float32)
            outs = (mk(4, S, S), mk(4), mk(1), mk(4, 256))
        if not dev:
            image_feats, feat_s0, feat_s1 = (np.ascontiguousarray(x, dtype=np.float32)
                                             for x in (image_feats, feat_s0, feat_s1))
            if sparse is not None:
                sparse = np.ascontiguousarray(sparse, dtype=np.float32)
        n_sparse = 0 if sparse is None else int(sparse.shape[0])
        flags = (DEC_ADD_NO_MEM if add_no_mem else 0) | (DEC_DEVICE_PTRS if dev else 0)
        rc = self._L.s3b_sam_decode(self.h, feat, _ptr(image_feats), _ptr(feat_s0), _ptr(feat_s1), _ptr(sparse),
                                    n_sparse, flags, *[_ptr(o) for o in outs])
        self._check(rc, "s3b_sam_decode")
        return outs

    # -- memory encoder / object pointer
    def mem_encode(self, feat: int, pix_feat, mask_logits, obj_score=None, out=None):
        """Memory features [feat*feat, 64]: all numpy (host) or all torch CUDA tensors (device; obj_score a
        1-element device tensor or None)."""
        dev = hasattr(pix_feat, "is_cuda") and pix_feat.is_cuda
        mh, mw = int(mask_logits.shape[-2]), int(mask_logits.shape[-1])
        if out is None:
            if dev:
                import torch
                out = torch.empty(feat * feat, 64, device=pix_feat.device, dtype=torch.float32)
            else:
                out = np.empty((feat * feat, 64), np.float32)
        if not dev:
            pix_feat = np.ascontiguousarray(pix_feat, dtype=np.float32)
            mask_logits = np.ascontiguousarray(mask_logits, dtype=np.float32)
            if obj_score is not None:
                obj_score = np.ascontiguousarray(np.asarray(obj_score, np.float32).reshape(1))
        rc = self._L.s3b_mem_encode(self.h, feat, _ptr(pix_feat), _ptr(mask_logits), mh, mw, _ptr(obj_score),
                                    _ptr(out), 0 if not dev else 2)
        self._check(rc, "s3b_mem_encode")
        return out

    def obj_ptr(self, sam_token, obj_score=None, out=None):
        dev = hasattr(sam_token, "is_cuda") and sam_token.is_cuda
        if out is None:
            if dev:
                import torch
                out = torch.empty(256, device=sam_token.device, dtype=torch.float32)
            else:
                out = np.empty(256, np.float32)
        if not dev:
            sam_token = np.ascontiguousarray(sam_token, dtype=np.float32)
            if obj_score is not None:
                obj_score = np.ascontiguousarray(np.asarray(obj_score, np.float32).reshape(1))
        self._check(self._L.s3b_obj_ptr(self.h, _ptr(sam_token), _ptr(obj_score), _ptr(out), 0 if not dev else 2),
                    "s3b_obj_ptr")
        return out

    def track_step(self, feat: int, trk0, trk1, trk2, slot_feats, slot_tpos, obj_ptrs=None, ptr_tpos=(),
                   slot_pes=None, want=("mask", "scores", "mem", "ptr"), outs=None):
        """One tracking step (s3b_track_step) on torch CUDA tensors (or raw device addresses for the inputs);
        returns a dict of the outputs asked for (or fills `outs`, a dict of preallocated tensors)."""
        import torch
        if outs is None:
            dev = trk2.device
            outs = {"mask": torch.empty(16 * feat * feat, device=dev) if "mask" in want else None,
                    "scores": torch.empty(3, device=dev) if "scores" in want else None,
                    "mem": torch.empty(feat * feat, 64, device=dev) if "mem" in want else None,
                    "ptr": torch.empty(256, device=dev) if "ptr" in want else None}
        outs = {k: outs.get(k) for k in ("mask", "scores", "mem", "ptr")}
        n_slots, feats, pes, tpos, n_ptrs, ptpos = self._bank_args(slot_feats, slot_pes, slot_tpos, obj_ptrs, ptr_tpos)
        rc = self._L.s3b_track_step(self.h, feat, _ptr(trk0), _ptr(trk1), _ptr(trk2), feats, pes, tpos, n_slots,
                                    _ptr(obj_ptrs), ptpos, n_ptrs, _ptr(outs["mask"]), _ptr(outs["scores"]),
                                    _ptr(outs["mem"]), _ptr(outs["ptr"]))
        self._check(rc, "s3b_track_step")
        return {k: v for k, v in outs.items() if v is not None}

    # -- operators on device pointers (torch CUDA tensors)
    def gemm(self, A, B, out, bias=None, act=ACT_NONE, resid=None, K=None):
        M, lda = A.shape[0], A.stride(0)
        N, ldb = B.shape[0], B.stride(0)
        K = K if K is not None else A.shape[1]
        out_f32 = 1 if out.dtype.itemsize == 4 else 0
        rc = self._L.s3b_op_gemm(self.h, A.data_ptr(), lda, B.data_ptr(), ldb, M, N, K, _ptr(bias), act,
                                 out.data_ptr(), out_f32, out.stride(0), _ptr(resid),
                                 resid.stride(0) if resid is not None else 0)
        self._check(rc, "s3b_op_gemm")

    def gemm_q(self, A, blocks, qtype: int, N: int, out, bias=None, act=ACT_NONE, resid=None):
        """out = A B^T (+ bias, act, resid) with B as N rows of q4_0 / q8_0 blocks (a uint8 CUDA tensor of
        N * row_size(qtype, K) bytes, ggml row layout)."""
        M, lda, K = A.shape[0], A.stride(0), A.shape[1]
        out_f32 = 1 if out.dtype.itemsize == 4 else 0
        rc = self._L.s3b_op_gemm_q(self.h, A.data_ptr(), lda, blocks.data_ptr(), qtype, M, N, K, _ptr(bias), act,
                                   out.data_ptr(), out_f32, out.stride(0), _ptr(resid),
                                   resid.stride(0) if resid is not None else 0)
        self._check(rc, "s3b_op_gemm_q")

    def gemm_rope(self, A, B, out, bias, table, rope_d: int, rope_cols: int, rope_mod: int):
        M, lda = A.shape[0], A.stride(0)
        N, ldb = B.shape[0], B.stride(0)
        out_f32 = 1 if out.dtype.itemsize == 4 else 0
        rc = self._L.s3b_op_gemm_rope(self.h, A.data_ptr(), lda, B.data_ptr(), ldb, M, N, A.shape[1], _ptr(bias),
                                      table.data_ptr(), rope_d, rope_cols, rope_mod, out.data_ptr(), out_f32,
                                      out.stride(0))
        self._check(rc, "s3b_op_gemm_rope")

    def attention(self, q, k, v, out, scale: float):
        B, H, nq, d = q.shape
        nk = k.shape[2]
        rc = self._L.s3b_op_attention(self.h, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, nq,
                                      nk, d, scale)
        self._check(rc, "s3b_op_attention")

    def attention_qkv(self, qkv, out, nwin: int, heads: int, ntok: int, d: int, scale: float):
        """qkv f16 [nwin*ntok][ld] (q | k | v, heads*d each), out f16 [nwin*ntok][ld_out]."""
        rc = self._L.s3b_op_attention_qkv(self.h, qkv.data_ptr(), qkv.stride(0), out.data_ptr(), out.stride(0), nwin,
                                          heads, ntok, d, scale)
        self._check(rc, "s3b_op_attention_qkv")

    def resize_bilinear_u8(self, src, out):
        """src uint8 CUDA [n, H, W, 3] -> out uint8 CUDA [n, H', W', 3]."""
        n, H, W = int(src.shape[0]), int(src.shape[1]), int(src.shape[2])
        rc = self._L.s3b_op_resize_bilinear_u8(self.h, src.data_ptr(), n, W, H, out.data_ptr(), int(out.shape[2]),
                                               int(out.shape[1]))
        self._check(rc, "s3b_op_resize_bilinear_u8")

    def layernorm(self, x, out, g, b, eps: float):
        rows, C = x.shape
        out_f32 = 1 if out.dtype.itemsize == 4 else 0
        rc = self._L.s3b_op_layernorm(self.h, x.data_ptr(), out.data_ptr(), out_f32, rows, C, g.data_ptr(),
                                      _ptr(b), eps)
        self._check(rc, "s3b_op_layernorm")

    def conv3x3(self, x, w, bias, out):
        """x f16 [B,H,W,C], w f16 [Cout,3,3,C], bias f32 [Cout] or None, out f32 [B,H,W,Cout]."""
        B, H, W, C = x.shape
        Cout = w.shape[0]
        rc = self._L.s3b_op_conv3x3(self.h, x.data_ptr(), B, H, W, C, w.data_ptr(), _ptr(bias), out.data_ptr(), Cout)
        self._check(rc, "s3b_op_conv3x3")

    def deconv2x2(self, x, w, bias, out, act: int = 0):
        """x f16 [B,H,W,Cin], w f16 [2,2,Cout,Cin], bias f32 [Cout] or None, out f16 / f32 [B,2H,2W,Cout]."""
        B, H, W, Cin = x.shape
        Cout = w.shape[2]
        rc = self._L.s3b_op_deconv2x2(self.h, x.data_ptr(), B, H, W, Cin, w.data_ptr(), _ptr(bias), act,
                                      out.data_ptr(), 1 if out.dtype.itemsize == 4 else 0, Cout)
        self._check(rc, "s3b_op_deconv2x2")

    def dequantize(self, raw, qtype: int, ne0: int, nrows: int, out):
        rc = self._L.s3b_op_dequantize(self.h, raw.data_ptr(), qtype, ne0, nrows, out.data_ptr())
        self._check(rc, "s3b_op_dequantize")
