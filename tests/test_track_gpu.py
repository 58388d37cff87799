"""One tracking step of one object on the GPU (s3b_track_step): memory attention from the object's memory
bank -> SAM mask decoder -> kept mask -> memory encoder -> object pointer, all on the device.

- The step equals the same operations called one by one through the C ABI (s3b_mem_attn_bank,
  s3b_sam_decode, the mask rule of sam3_propagate_single, s3b_mem_encode, s3b_obj_ptr), bit for bit, for
  SAM 2 (multimask: best of tokens 1-3, its token for the pointer) and SAM 3 (token 0).
- A 3-frame loop that appends each step's memory features and pointer to the bank agrees with the
  oracle's composition of the same steps (cosine >= 0.999 on the masks and memory features)."""
import numpy as np
import pytest

from oracle import mask_decoder as md
from oracle import mem_attn as om
from oracle import mem_enc as me
from oracle import nn

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


def _model(tmp_path, sam2, seed):
    from sam3_b200 import ggml_io, synth
    if sam2:
        cfg = synth.Sam2Config(img_size=256, embed=96, heads=1, stages=(1, 2, 2, 1), global_idx=(4,),
                               window_spec=(8, 4, 14, 7), with_mem_attn=True, with_sam_dec=True)
        T = synth.sam2_tensors(cfg, seed=seed, ln_random=True)
        magic, ver = ggml_io.MAGIC_SAM2, 1
    else:
        cfg = synth.Sam3Config(img_size=224, patch=14, embed=128, depth=1, heads=2, window=8, global_idx=(),
                               neck_dim=256, neck_mid=128, with_mem_attn=True, with_sam_dec=True)
        T = synth.sam3_tensors(cfg, seed=seed, ln_random=True)
        magic, ver = ggml_io.MAGIC_SAM3, 3
    T.update(synth.mem_enc_tensors(seed + 1))
    path = str(tmp_path / f"trk_{int(sam2)}_{seed}.ggml")
    synth.write_model(path, T, cfg.hparams(), magic, ver, 1)
    return cfg, path, synth.stored_values(T, 1, None)


def _frame(H, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(s * s, 256, device="cuda", generator=g) for s in (4 * H, 2 * H, H)]


@pytest.mark.parametrize("sam2", [True, False], ids=["sam2", "sam3"])
def test_track_step_equals_its_parts(tmp_path, engine, sam2):
    cfg, path, W = _model(tmp_path, sam2, 31)
    engine.load_model(path)
    H = 16
    t0, t1, t2 = _frame(H, 1)
    g = torch.Generator(device="cuda").manual_seed(2)
    feats = [torch.randn(H * H, 64, device="cuda", generator=g) for _ in range(3)]
    ptrs = torch.randn(2, 256, device="cuda", generator=g)
    slot_tpos, ptr_tpos = [0, 2, 1], [1, 2]
    out = engine.track_step(H, t0, t1, t2, feats, slot_tpos, ptrs, ptr_tpos)
    cond = engine.mem_attn_bank(t2, H, feats, slot_tpos, ptrs, ptr_tpos)
    masks, iou, obj, toks = engine.sam_decode(H, cond, t0, t1, None)
    engine.sync()
    iou_h = iou.cpu().numpy()
    k = int(np.argmax(iou_h[1:]) + 1) if sam2 else 0
    kept = masks[k].contiguous()
    mem = engine.mem_encode(H, t2, kept, obj)
    ptr = engine.obj_ptr(toks[k if sam2 else 0].contiguous(), obj)
    engine.sync()
    assert torch.equal(out["mask"], kept.reshape(-1))
    sc = out["scores"].cpu().numpy()
    assert sc[2] == k and sc[0] == iou_h[k] and sc[1] == obj.cpu().numpy()[0]
    assert torch.equal(out["mem"], mem)
    assert torch.equal(out["ptr"], ptr)


def test_track_loop_vs_oracle(tmp_path, engine):
    cfg, path, W = _model(tmp_path, True, 41)
    engine.load_model(path)
    H = 16
    img = cfg.img_size
    g = torch.Generator(device="cuda").manual_seed(7)
    # the bank starts with a conditioning frame's memory (tpos 0) and its pointer
    bank = [torch.randn(H * H, 64, device="cuda", generator=g)]
    ptrs = [torch.randn(256, device="cuda", generator=g)]
    tpos_enc = W["mem_enc.tpos_enc"].reshape(cfg.num_maskmem, 64)
    ref_bank = [b.cpu().numpy() for b in bank]
    ref_ptrs = [p.cpu().numpy() for p in ptrs]
    for f in range(3):
        t0, t1, t2 = _frame(H, 100 + f)
        slot_tpos = [0] + [len(bank) - s for s in range(1, len(bank))]
        ptr_tpos = [f + 1 - i for i in range(len(ptrs))]
        out = engine.track_step(H, t0, t1, t2, bank, slot_tpos, torch.stack(ptrs), ptr_tpos)
        engine.sync()
        # oracle composition of the same step, from the oracle's own bank
        pe64 = nn.sine_pe_2d(H, H, 64).reshape(H * H, 64)
        prompt, ppos, n_ptr = om.build_prompt(ref_bank, [pe64] * len(ref_bank), slot_tpos, tpos_enc, ref_ptrs,
                                              ptr_tpos, W["obj_ptr_tpos_proj.weight"], W["obj_ptr_tpos_proj.bias"],
                                              cfg.num_maskmem)
        x2 = t2.cpu().numpy()
        cond = om.mem_attn(W, x2, om.src_pos(H), H, prompt, ppos, n_ptr)
        rm, ri, ro, rt = md.decode(W, cond.reshape(H, H, 256), t0.cpu().numpy().reshape(4 * H, 4 * H, 256),
                                   t1.cpu().numpy().reshape(2 * H, 2 * H, 256),
                                   W["sam_pe.not_a_point_embed.weight"].reshape(1, 256))
        taps = {}
        _, _, _, _ = md.decode(W, cond.reshape(H, H, 256), t0.cpu().numpy().reshape(4 * H, 4 * H, 256),
                               t1.cpu().numpy().reshape(2 * H, 2 * H, 256),
                               W["sam_pe.not_a_point_embed.weight"].reshape(1, 256), taps=taps)
        k = int(np.argmax(ri[1:]) + 1)
        mask_tokens = taps["final_queries"][2:6]
        assert int(out["scores"][2].item()) == k
        assert _cos(out["mask"].cpu().numpy(), rm[k]) >= 0.999
        rmem = me.encode(W, x2.reshape(H, H, 256), rm[k], ro[0], img).reshape(H * H, 64)
        rptr = me.obj_ptr(W, mask_tokens[k], ro[0])
        assert _cos(out["mem"].cpu().numpy(), rmem) >= 0.999
        assert _cos(out["ptr"].cpu().numpy(), rptr) >= 0.999
        bank.append(out["mem"])
        ptrs.insert(0, out["ptr"])
        ref_bank.append(rmem)
        ref_ptrs.insert(0, rptr)


@pytest.mark.parametrize("sam2", [True, False], ids=["sam2", "sam3"])
def test_track_step_graph_replay_equals_eager(tmp_path, engine, sam2):
    """On a capturable stream, the second tracking step with the same buffers, bank layout and positions is
    captured into a CUDA graph and later steps replay it: they give the eager bits, read the current
    contents of the same buffers, and a changed position or buffer runs (and later captures) its own key."""
    cfg, path, W = _model(tmp_path, sam2, 37)
    H = 16
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    engine.set_stream(stream.cuda_stream)
    try:
        engine.load_model(path)
        with torch.cuda.stream(stream):
            t0, t1, t2 = _frame(H, 3)
            g = torch.Generator(device="cuda").manual_seed(4)
            feats = [torch.randn(H * H, 64, device="cuda", generator=g) for _ in range(3)]
            ptrs = torch.randn(2, 256, device="cuda", generator=g)
            new_feats = [torch.randn(H * H, 64, device="cuda", generator=g) for _ in range(3)]
            outs = {"mask": torch.empty(16 * H * H, device="cuda"), "scores": torch.empty(3, device="cuda"),
                    "mem": torch.empty(H * H, 64, device="cuda"), "ptr": torch.empty(256, device="cuda")}

        def step(slot_tpos=(0, 2, 1), ptr_tpos=(1, 2)):
            engine.track_step(H, t0, t1, t2, feats, list(slot_tpos), ptrs, list(ptr_tpos), outs=outs)
            engine.sync()
            return {k: v.cpu().clone() for k, v in outs.items()}

        engine.set_option("graphs", 0)
        ref = step()
        ref_tpos = step(slot_tpos=(0, 1, 2))
        for f, nf in zip(feats, new_feats):
            f.copy_(nf)
        ref_new = step()
        engine.set_option("graphs", 1)
        with torch.cuda.stream(stream):
            g = torch.Generator(device="cuda").manual_seed(4)
            old = [torch.randn(H * H, 64, device="cuda", generator=g) for _ in range(3)]
        for f, o in zip(feats, old):
            f.copy_(o)
        for i in range(4):  # eager, eager, capture + replay, replay
            got = step()
            for k in ref:
                assert torch.equal(got[k], ref[k]), (i, k)
        got = step(slot_tpos=(0, 1, 2))  # another key
        for k in ref:
            assert torch.equal(got[k], ref_tpos[k]), ("tpos", k)
        for f, nf in zip(feats, new_feats):  # new contents, same buffers: the replay reads them
            f.copy_(nf)
        got = step()
        for k in ref:
            assert torch.equal(got[k], ref_new[k]), ("refill", k)
    finally:
        engine.set_option("graphs", 1)
        engine.set_stream(torch.cuda.current_stream().cuda_stream)
