"""Encoder calls replayed from CUDA graphs (option "graphs", s3b_encode_*): from the second call with the
same entry point, input pointer, frame count, size, flags, options and buffers, the whole launch sequence
is captured once and replayed. Replays must give the bits of eager runs, read the input buffer's current
contents, and never replay into buffers that were reallocated (another frame count, a model reload)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _models(s3b, synth, tmp_path):
    sam3 = synth.Sam3Config(img_size=336, patch=14, embed=256, depth=3, heads=4, mlp_ratio_x1000=4625, window=8,
                            global_idx=(1,), neck_dim=64, neck_mid=128, visual_only=1)
    p3 = str(tmp_path / "vit_graph.ggml")
    synth.write_sam3(p3, sam3, seed=4, ftype=1, qtype=2, quantize=s3b.quantize_rows, ln_random=True)
    sam2 = synth.Sam2Config(img_size=256, embed=96, heads=1, stages=(1, 2, 2, 1), global_idx=(4,),
                            window_spec=(8, 4, 14, 7))
    p2 = str(tmp_path / "hiera_graph.ggml")
    synth.write_sam2(p2, sam2, seed=6, ftype=1, qtype=2, quantize=s3b.quantize_rows)
    return [(p3, sam3.img_size, ["vit_output", "neck_trk_0", "neck_trk_2"]),
            (p2, sam2.img_size, ["neck_trk_0", "neck_trk_1", "neck_trk_2"])]


def _outs(engine, names, n):
    return {(nm, f): engine.output(nm, f).copy() for nm in names for f in range(n)}


@pytest.mark.parametrize("which", [0, 1])
def test_encode_graph_replay_equals_eager(engine, s3b, tmp_path, which):
    from sam3_b200 import synth
    path, img, names = _models(s3b, synth, tmp_path)[which]
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    engine.set_stream(stream.cuda_stream)
    try:
        engine.load_model(path)
        a = torch.from_numpy(synth.frames_u8(2, img, base_seed=31)).cuda()
        b = torch.from_numpy(synth.frames_u8(2, img, base_seed=32)).cuda()
        buf = a.clone()
        # eager reference results (graphs off)
        engine.set_option("graphs", 0)
        engine.encode_u8(a)
        engine.sync()
        ref_a = _outs(engine, names, 2)
        engine.encode_u8(b)
        engine.sync()
        ref_b = _outs(engine, names, 2)
        engine.set_option("graphs", 1)
        # same input buffer four times: eager, eager (the first call of this key after allocation), then
        # capture + replay; every call gives the eager bits
        for i in range(4):
            engine.encode_u8(buf)
            engine.sync()
            got = _outs(engine, names, 2)
            for k, v in ref_a.items():
                assert np.array_equal(got[k], v), (i, k)
        # new contents in the same buffer: the replay reads them
        buf.copy_(b)
        engine.encode_u8(buf)
        engine.sync()
        got = _outs(engine, names, 2)
        for k, v in ref_b.items():
            assert np.array_equal(got[k], v), ("refill", k)
        # one frame: other output buffers (reallocated), then back to two frames
        one = buf[:1].clone()
        for _ in range(3):
            engine.encode_u8(one)
            engine.sync()
        for nm in names:
            assert np.array_equal(engine.output(nm, 0), ref_b[(nm, 0)]), nm
        buf.copy_(a)
        for _ in range(3):
            engine.encode_u8(buf)
            engine.sync()
            got = _outs(engine, names, 2)
            for k, v in ref_a.items():
                assert np.array_equal(got[k], v), ("back", k)
        # a model reload moves the weights: the next calls must not replay the old graph
        engine.load_model(path)
        for _ in range(3):
            engine.encode_u8(buf)
            engine.sync()
        got = _outs(engine, names, 2)
        for k, v in ref_a.items():
            assert np.array_equal(got[k], v), ("reload", k)
        # launches are still counted for replays
        engine.profile_begin(False)
        engine.encode_u8(buf)
        prof = engine.profile_end()
        assert prof["launches"] > 0
    finally:
        engine.set_option("graphs", 1)
        engine.set_stream(torch.cuda.current_stream().cuda_stream)


def test_encode_graph_host_bound_outputs_stay_correct(engine, s3b, tmp_path):
    """With an output bound to host memory the call stays eager (its copies run on a second stream); the
    bound host buffer receives the same values as s3b_output_copy, before and after replays."""
    from sam3_b200 import synth
    path, img, names = _models(s3b, synth, tmp_path)[1]
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    engine.set_stream(stream.cuda_stream)
    try:
        engine.load_model(path)
        frames = torch.from_numpy(synth.frames_u8(2, img, base_seed=41)).cuda()
        for _ in range(3):
            engine.encode_u8(frames)  # replayed from the third call
        engine.sync()
        ref = engine.output("neck_trk_2", 1).copy()
        shape = engine.output_shape("neck_trk_2")
        host = torch.zeros(2, shape[2], shape[1], shape[0], dtype=torch.float32).pin_memory()
        engine.output_host_bind("neck_trk_2", host)
        for _ in range(2):
            engine.encode_u8(frames)
            engine.sync()
            assert np.array_equal(host[1].numpy(), ref)
        engine.output_host_bind("neck_trk_2", None)
        for _ in range(3):
            engine.encode_u8(frames)
        engine.sync()
        assert np.array_equal(engine.output("neck_trk_2", 1), ref)
    finally:
        engine.set_stream(torch.cuda.current_stream().cuda_stream)
