"""Worker of tests/test_peer_gpu.py::test_ipc_handoff_two_processes (one process per GPU, here both on
GPU 0). Role "track": allocates the receive buffer, exports its IPC handle, waits for the encoder, then
checks the buffer against its own encoding of the same frame. Role "encode": encodes the frame, opens the
handle and copies neck_trk_2 into the tracker's buffer with s3b_peer_copy_output."""
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))


def wait_for(path, limit_s=120.0):
    t0 = time.time()
    while not os.path.exists(path):
        if time.time() - t0 > limit_s:
            raise TimeoutError(path)
        time.sleep(0.05)


class CudaArray:
    """Zero-copy view of device memory for torch.as_tensor (the CUDA array interface)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


def main():
    role, model, workdir = sys.argv[1], sys.argv[2], sys.argv[3]
    import torch
    from conftest import load_pkg
    s3b = load_pkg()
    from sam3_b200 import synth
    eng = s3b.Engine(0)
    eng.load_model(model)
    frames = synth.frames_u8(1, 336, base_seed=42)
    eng.encode_u8(frames)
    eng.sync()
    ne = eng.output_shape("neck_trk_2")
    n = ne[0] * ne[1] * ne[2]
    if role == "track":
        ptr = eng.device_alloc(n * 4)
        with open(os.path.join(workdir, "handle.tmp"), "wb") as f:
            f.write(eng.ipc_export(ptr))
        os.replace(os.path.join(workdir, "handle.tmp"), os.path.join(workdir, "handle"))
        wait_for(os.path.join(workdir, "copied"))
        got = torch.as_tensor(CudaArray(ptr, n), device="cuda:0").cpu().numpy()
        want = eng.output("neck_trk_2", 0).reshape(-1)
        ok = got.tobytes() == want.tobytes()
        eng.device_free(ptr)
        with open(os.path.join(workdir, "result"), "w") as f:
            f.write("equal" if ok else "differ")
    else:
        wait_for(os.path.join(workdir, "handle"))
        handle = open(os.path.join(workdir, "handle"), "rb").read()
        ptr = eng.ipc_open(handle)
        eng.peer_copy_output("neck_trk_2", 0, ptr, 0, n * 4)
        eng.sync()
        eng.ipc_close(ptr)
        open(os.path.join(workdir, "copied"), "w").close()


if __name__ == "__main__":
    main()
