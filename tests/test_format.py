""".ggml format, block quantisation and C ABI surface (CPU only)."""
import os
import re
import struct

import numpy as np
import pytest

from oracle import quant as oq

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_header_symbols_exported(s3b):
    """Every function declared in include/sam3_b200.h is exported by libsam3b200.so."""
    hdr = open(os.path.join(ROOT, "include", "sam3_b200.h")).read()
    names = set(re.findall(r"\b(s3b_[a-z0-9_]+)\s*\(", hdr))
    assert len(names) >= 20
    L = s3b.lib()
    missing = [n for n in sorted(names) if not hasattr(L, n)]
    assert not missing, missing
    bound = {n for n, _, _ in s3b.SYMBOLS}
    assert names == bound, names ^ bound


@pytest.mark.parametrize("qtype", [2, 3, 8])
def test_oracle_quant_matches_gguf(qtype):
    """The oracle's block formats are bit-identical to gguf-py's (independent ggml port)."""
    gguf_quants = pytest.importorskip("gguf.quants")
    from gguf.constants import GGMLQuantizationType as Q
    qt = {2: Q.Q4_0, 3: Q.Q4_1, 8: Q.Q8_0}[qtype]
    rng = np.random.default_rng(qtype)
    x = rng.standard_normal((256, 1024)).astype(np.float32) * 0.02
    x[0, :32] = 0.0                      # all-zero block (d == 0)
    x[1, :32] = 1e-3                     # constant block
    x[2, 5] = 3.0                        # outlier
    x = x.astype(np.float16).astype(np.float32)
    ours = oq.quantize(qtype, x)
    ref = gguf_quants.quantize(x, qt)
    assert np.array_equal(ours, ref.reshape(ours.shape))
    assert np.array_equal(oq.dequantize(qtype, ours, 1024).view(np.uint32),
                          gguf_quants.dequantize(ref, qt).reshape(256, 1024).astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("qtype", [2, 3, 8])
def test_library_quant_matches_oracle(s3b, qtype):
    """The product's host quantiser / dequantiser (C ABI) == oracle, bit for bit."""
    rng = np.random.default_rng(10 + qtype)
    x = (rng.standard_normal((64, 4736)) * 0.02).astype(np.float16).astype(np.float32)
    raw = s3b.quantize_rows(qtype, x)
    assert np.array_equal(raw, oq.quantize(qtype, x))
    assert np.array_equal(s3b.dequantize_rows(qtype, raw, 4736).view(np.uint32),
                          oq.dequantize(qtype, raw, 4736).view(np.uint32))
    assert s3b.row_size(qtype, 4736) == raw.shape[1]


def _tiny(synth):
    return synth.Sam3Config(img_size=336, patch=14, embed=256, depth=3, heads=4, window=8, global_idx=(1,),
                            neck_dim=64, neck_mid=128)


@pytest.mark.parametrize("qtype", [None, 2, 3, 8])
def test_writer_reader_roundtrip(s3b, tmp_path, qtype):
    from sam3_b200 import ggml_io, synth
    cfg = _tiny(synth)
    p = str(tmp_path / "m.ggml")
    T = synth.write_sam3(p, cfg, seed=1, qtype=qtype, quantize=s3b.quantize_rows)
    info = s3b.inspect_model(p)
    assert info["is_sam2"] == 0 and info["img_size"] == 336 and info["depth"] == 3 and info["embed_dim"] == 256
    assert info["n_tensors"] == len(T)
    magic, version, ftype, hp, recs = ggml_io.read(p, len(cfg.hparams()))
    assert magic == ggml_io.MAGIC_SAM3 and hp == cfg.hparams()
    nq = sum(r.dtype in ggml_io.QTYPES for r in recs.values())
    assert nq == info["n_quantised"]
    if qtype is None:
        assert nq == 0
        assert recs["vit.blocks.0.attn.qkv.weight"].dtype == ggml_io.F16
    else:
        # quantisation rule: 2-D, ne0 % 32 == 0, not embeddings / pos / freqs_cis
        assert recs["vit.blocks.0.mlp.lin2.weight"].dtype == qtype
        assert recs["vit.patch_embed.proj.weight"].dtype == ggml_io.F32   # ne0 = 14 and "embed" -> f32
        assert recs["vit.blocks.0.attn.freqs_cis"].dtype == ggml_io.F32
        assert recs["neck.trk.0.conv_3x3.weight"].dtype == ggml_io.F16   # ne0 = 3
    # records are 32-byte aligned and the data round-trips
    r = recs["vit.blocks.1.attn.proj.weight"]
    if r.dtype == ggml_io.F16:
        np.testing.assert_array_equal(np.frombuffer(r.data, np.float16).astype(np.float32).reshape(r.shape),
                                      T["vit.blocks.1.attn.proj.weight"].astype(np.float16).astype(np.float32))


def test_loader_rejects_corrupt_files(s3b, tmp_path):
    from sam3_b200 import synth
    cfg = _tiny(synth)
    p = str(tmp_path / "m.ggml")
    synth.write_sam3(p, cfg, seed=1)
    data = open(p, "rb").read()
    bad = str(tmp_path / "bad.ggml")
    open(bad, "wb").write(b"XXXX" + data[4:])
    with pytest.raises(s3b.S3BError, match="FORMAT"):
        s3b.inspect_model(bad)
    open(bad, "wb").write(data[: len(data) // 2])
    with pytest.raises(s3b.S3BError):
        s3b.inspect_model(bad)
    with pytest.raises(s3b.S3BError, match="IO"):
        s3b.inspect_model(str(tmp_path / "missing.ggml"))
    # a quantised record whose ne0 is not a multiple of 32 is rejected
    from sam3_b200 import ggml_io
    rec = ggml_io.Record("x.weight", 2, (4, 20), b"\x00" * 100)
    ggml_io.write(bad, ggml_io.MAGIC_SAM3, 3, 2, cfg.hparams(), [rec])
    with pytest.raises(s3b.S3BError, match="FORMAT"):
        s3b.inspect_model(bad)
