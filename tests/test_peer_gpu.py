"""Hand-off of per-frame features to the tracking GPU (s3b_peer_copy_output, s3b_device_alloc and the
CUDA IPC entry points): same-device copy, cross-GPU peer copy (when the box gives more than one GPU), and
the one-process-per-GPU path through an IPC handle (two processes, here on one GPU)."""
import os
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _tiny_model(s3b, path):
    from sam3_b200 import synth
    cfg = synth.Sam3Config(img_size=336, patch=14, embed=256, depth=2, heads=4, mlp_ratio_x1000=4625, window=8,
                           global_idx=(1,), neck_dim=64, neck_mid=128, visual_only=1)
    synth.write_sam3(path, cfg, seed=9, ftype=1)
    return cfg


def test_peer_copy_same_device(engine, s3b, tmp_path):
    from sam3_b200 import synth
    path = str(tmp_path / "tiny.ggml")
    cfg = _tiny_model(s3b, path)
    engine.load_model(path)
    engine.encode_u8(synth.frames_u8(2, cfg.img_size, base_seed=5))
    engine.sync()
    ne = engine.output_shape("neck_trk_2")
    n = ne[0] * ne[1] * ne[2]
    dst = torch.full((n,), float("nan"), device="cuda:0")
    engine.peer_copy_output("neck_trk_2", 1, dst.data_ptr(), 0, n * 4)
    engine.sync()
    assert np.array_equal(dst.cpu().numpy(), engine.output("neck_trk_2", 1).reshape(-1))
    with pytest.raises(Exception):
        engine.peer_copy_output("neck_trk_2", 1, dst.data_ptr(), 0, n * 4 - 4)  # too small


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_copy_other_gpu(engine, s3b, tmp_path):
    from sam3_b200 import synth
    path = str(tmp_path / "tiny.ggml")
    cfg = _tiny_model(s3b, path)
    engine.load_model(path)
    engine.encode_u8(synth.frames_u8(1, cfg.img_size, base_seed=6))
    engine.sync()
    ne = engine.output_shape("neck_trk_2")
    n = ne[0] * ne[1] * ne[2]
    dst = torch.zeros(n, device="cuda:1")
    engine.peer_copy_output("neck_trk_2", 0, dst.data_ptr(), 1, n * 4)
    engine.sync()
    assert np.array_equal(dst.cpu().numpy(), engine.output("neck_trk_2", 0).reshape(-1))


def test_ipc_handoff_two_processes(s3b, tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    path = str(tmp_path / "tiny.ggml")
    _tiny_model(s3b, path)
    worker = os.path.join(ROOT, "tests", "peer_ipc_worker.py")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    track = subprocess.Popen([sys.executable, worker, "track", path, str(tmp_path)], env=env, cwd=ROOT,
                             stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    enc = subprocess.Popen([sys.executable, worker, "encode", path, str(tmp_path)], env=env, cwd=ROOT,
                           stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    out_e, _ = enc.communicate(timeout=300)
    out_t, _ = track.communicate(timeout=300)
    assert enc.returncode == 0, out_e[-3000:]
    assert track.returncode == 0, out_t[-3000:]
    assert open(tmp_path / "result").read() == "equal"
