"""The B200 engine against the reference's own PyTorch outputs (fixtures made
by tests/golden/make_golden.py from tests/dump_vit_reference.py and
tests/dump_phase7_reference.py of the reference), at full size, through the
C ABI.

Tolerances: the engine computes GEMM / attention operands in f16 with f32
accumulation, as ggml's CPU path does for f16 weights. The reference's own
acceptance bar for this stage is cos > 0.999 and mean-abs < 0.05 against
its PyTorch dump (tests/test_phase3.cpp:516-577) and 5e-3 max-abs per
memory-attention layer (tests/test_phase7.cpp:100-112); here we require
cos >= 0.999 and mean-abs <= 2% of the reference's mean |value| on every
tap, plus max-abs <= 5e-3 * max|ref| for memory attention."""
import json
import os

import numpy as np
import pytest

from oracle import mem_attn as om
from test_golden import check_samples, gold

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def vit_model(s3b, tmp_path_factory):
    from sam3_b200 import synth
    g = gold("vit_golden.npz")
    meta = json.loads(str(g["meta"]))
    path = str(tmp_path_factory.mktemp("golden") / "sam3_vit_l_f16.ggml")
    synth.write_sam3(path, synth.SAM3_VIT_L, seed=meta["weights_seed"], ftype=1, ln_random=True)
    return path, g, meta


@pytest.mark.parametrize("stop,key", [(0, "after_ln_pre"), (1, "block_0_out"), (8, "block_7_out"),
                                      (-1, "vit_final")])
def test_vit_taps_vs_reference(engine, vit_model, stop, key):
    from sam3_b200 import synth
    path, g, meta = vit_model
    engine.load_model(path)
    engine.set_option("stop_after_blocks", stop)
    try:
        engine.encode_u8(synth.frames_u8(1, 1008, base_seed=meta["frame_seed"]))
        got = engine.output("vit_output", 0)
    finally:
        engine.set_option("stop_after_blocks", -1)
    print(check_samples(got, g, key, 0.02, 0.2, 0.999))


def test_neck_vs_reference(engine, vit_model):
    from sam3_b200 import synth
    path, g, meta = vit_model
    engine.load_model(path)
    engine.encode_u8(synth.frames_u8(1, 1008, base_seed=meta["frame_seed"]))
    for i in range(4):
        print(check_samples(engine.output(f"neck_trk_{i}", 0), g, f"neck_det_{i}", 0.02, 0.2, 0.999))


def test_mem_attn_vs_reference(engine, s3b, tmp_path):
    from sam3_b200 import synth
    g = gold("mem_attn_golden.npz")
    meta = json.loads(str(g["meta"]))
    cfg = synth.Sam3Config(depth=1, global_idx=(), with_mem_attn=True)
    path = str(tmp_path / "mem.ggml")
    synth.write_sam3(path, cfg, seed=meta["weights_seed"], ftype=1, ln_random=True)
    engine.load_model(path)
    assert engine.model_info()["mem_attn_layers"] == 4
    curr, prompt, prompt_pos, n_ptr = om.golden_inputs(meta)
    out = engine.mem_attn(curr, om.src_pos(meta["feat"]), meta["feat"], prompt, prompt_pos, n_ptr)
    print(check_samples(out, g, "output", 0.02, 5e-3 * 5, 0.999))


@pytest.mark.parametrize("qtype,feat,slots,ptrs", [(None, 16, 3, 3), (8, 24, 2, 0), (2, 32, 1, 16)])
def test_mem_attn_vs_oracle(engine, s3b, tmp_path, qtype, feat, slots, ptrs):
    """Other feature sizes, slot / pointer counts and weight formats, device pointers, against the oracle."""
    from oracle import quant as oq
    from sam3_b200 import synth
    cfg = synth.Sam3Config(img_size=336, patch=14, embed=128, depth=1, heads=2, window=8, global_idx=(),
                           neck_dim=256, neck_mid=128, with_mem_attn=True)
    path = str(tmp_path / "mem.ggml")
    T = synth.write_sam3(path, cfg, seed=9, ftype=1, qtype=qtype, quantize=s3b.quantize_rows, ln_random=True)
    W = synth.stored_values({k: v for k, v in T.items() if k.startswith("mem_attn.")}, 1, qtype, oq.quantize,
                            oq.dequantize)
    engine.load_model(path)
    rng = np.random.default_rng(feat)
    N = feat * feat
    curr = rng.standard_normal((N, 256), dtype=np.float32)
    M = slots * N + 4 * ptrs
    prompt = rng.standard_normal((M, 64), dtype=np.float32)
    ppos = rng.standard_normal((M, 64), dtype=np.float32)
    pos = om.src_pos(feat)
    ref = om.mem_attn(W, curr, pos, feat, prompt, ppos, 4 * ptrs)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = engine.mem_attn(d(curr), d(pos), feat, d(prompt), d(ppos), 4 * ptrs)
    engine.sync()
    got = out.cpu().numpy()
    diff = np.abs(got - ref)
    cos = float((got * ref).sum() / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert cos >= 0.9995 and diff.mean() <= 0.01 * np.abs(ref).mean(), (cos, diff.mean(), diff.max())


def test_mem_attn_graph_replay_equals_eager(engine, s3b, tmp_path):
    """Option "graphs": from the second call with the same shapes and buffers, the memory-attention layers
    replay from a CUDA graph (on a stream that can be captured). Replays give the same bits as eager runs,
    and a model reload or an option change recaptures."""
    from sam3_b200 import synth
    cfg = synth.Sam3Config(img_size=336, patch=14, embed=128, depth=1, heads=2, window=8, global_idx=(),
                           neck_dim=256, neck_mid=128, with_mem_attn=True)
    path = str(tmp_path / "mem_g.ggml")
    synth.write_sam3(path, cfg, seed=9, ftype=1, qtype=8, quantize=s3b.quantize_rows, ln_random=True)
    rng = np.random.default_rng(7)
    feat, slots, ptrs = 16, 2, 4
    N, M = feat * feat, slots * feat * feat + 4 * ptrs
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    curr = d(rng.standard_normal((N, 256), dtype=np.float32))
    pos = d(om.src_pos(feat))
    prompt = d(rng.standard_normal((M, 64), dtype=np.float32))
    ppos = d(rng.standard_normal((M, 64), dtype=np.float32))
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    engine.set_stream(stream.cuda_stream)
    try:
        engine.load_model(path)
        outs = []
        for i in range(5):
            if i == 4:
                engine.set_option("graphs", 0)
            out = torch.empty_like(curr)
            engine.mem_attn(curr, pos, feat, prompt, ppos, 4 * ptrs, out=out)
            engine.sync()
            outs.append(out.cpu())
        engine.set_option("graphs", 1)
        engine.load_model(path)  # new weight buffers: the next calls run eagerly, then recapture
        for _ in range(3):
            out = torch.empty_like(curr)
            engine.mem_attn(curr, pos, feat, prompt, ppos, 4 * ptrs, out=out)
            engine.sync()
            outs.append(out.cpu())
    finally:
        engine.set_option("graphs", 1)
        engine.set_stream(torch.cuda.current_stream().cuda_stream)
    for i, o in enumerate(outs[1:], 1):
        assert torch.equal(o, outs[0]), i
