"""Memory attention — numpy oracle (test infrastructure only).

Restates sam3_build_mem_attn_graph (sam3.cpp:9224-9337): x = curr + 0.1*pos,
then per layer a single-head RoPE self-attention, a RoPE cross-attention to
the memory prompt (K from prompt + prompt_pos, V from prompt, RoPE on the
spatial keys only, pointer tokens excluded), a ReLU FFN, each pre-normed
with a residual, and a final LayerNorm. RoPE tables follow
sam3_ensure_tracker_pe_caches (sam3.cpp:11126-11169): axial CIS, dim 256,
theta 1e4, scale 1, over the feat x feat grid, repeated for every memory
slot (sam3.cpp:11262-11263). The prompt builder follows
sam3_build_prompt_and_pos (sam3.cpp:9123-9209).
"""
import numpy as np

from . import nn


def axial_cis(dim, end_x, end_y, theta=10000.0, scale=1.0):
    """sam3_compute_axial_cis (sam3.cpp:3555-3586) as [N, dim/2, 2] (cos, sin)."""
    q = dim // 4
    freqs = (1.0 / (np.float32(theta) ** (np.arange(0, dim, 4, dtype=np.float32)[:q] / np.float32(dim)))).astype(
        np.float32)
    t = np.arange(end_x * end_y)
    tx = (t % end_x).astype(np.float32) * np.float32(scale)
    ty = (t // end_x).astype(np.float32) * np.float32(scale)
    ang = np.concatenate([np.outer(tx, freqs), np.outer(ty, freqs)], axis=1).astype(np.float32)
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32)


def src_pos(feat, D=256):
    """Sinusoidal PE of the current tokens, [N, D] (sam3_sinusoidal_pe_2d)."""
    return nn.sine_pe_2d(feat, feat, D).reshape(feat * feat, D)


def mem_attn(W, curr, pos, feat, prompt, prompt_pos, n_ptr, taps=None, f16_inputs=False):
    """curr/pos [N, 256], prompt/prompt_pos [M, 64] -> [N, 256]."""
    N = feat * feat
    D = curr.shape[1]
    rope_q = axial_cis(D, feat, feat)
    M = prompt.shape[0]
    m_sp = M - n_ptr
    rope_k = rope_q[np.arange(m_sp) % N] if m_sp > 0 else None
    x = (curr + np.float32(0.1) * pos).astype(np.float32)
    if taps is not None:
        taps["input"] = x.copy()
    scale = 1.0 / np.sqrt(D)
    n_layers = len({k.split(".")[2] for k in W if k.startswith("mem_attn.layers.")})
    for l in range(n_layers):
        p = f"mem_attn.layers.{l}"
        L = lambda a, n: nn.linear(a, W[f"{p}.{n}.weight"], W[f"{p}.{n}.bias"], f16_inputs)
        xn = nn.layer_norm(x, W[f"{p}.norm1.weight"], W[f"{p}.norm1.bias"], 1e-5)
        q = nn.rope(L(xn, "sa.q_proj"), rope_q)
        k = nn.rope(L(xn, "sa.k_proj"), rope_q)
        v = L(xn, "sa.v_proj")
        o = nn.attention(q[None], k[None], v[None], scale, f16_inputs)[0]
        x = x + L(o, "sa.out_proj")
        if taps is not None:
            taps[f"layer{l}_after_sa"] = x.copy()
        xn = nn.layer_norm(x, W[f"{p}.norm2.weight"], W[f"{p}.norm2.bias"], 1e-5)
        q = nn.rope(L(xn, "ca.q_proj"), rope_q)
        k = L((prompt + prompt_pos).astype(np.float32), "ca.k_proj")
        v = L(prompt, "ca.v_proj")
        if m_sp > 0:
            k[:m_sp] = nn.rope(k[:m_sp], rope_k)
        o = nn.attention(q[None], k[None], v[None], scale, f16_inputs)[0]
        x = x + L(o, "ca.out_proj")
        if taps is not None:
            taps[f"layer{l}_after_ca"] = x.copy()
        xn = nn.layer_norm(x, W[f"{p}.norm3.weight"], W[f"{p}.norm3.bias"], 1e-5)
        x = x + L(nn.relu(L(xn, "linear1")), "linear2")
        if taps is not None:
            taps[f"layer{l}_after_ffn"] = x.copy()
    return nn.layer_norm(x, W["mem_attn.norm.weight"], W["mem_attn.norm.bias"], 1e-5)


def one_d_sine_pe(pos, dim, temperature=10000.0):
    """sam3_get_1d_sine_pe (sam3.cpp:3636-3647): first dim/2 sinf, then cosf of pos / powf(T, paired / (dim/2)),
    float32 operations and libm functions as the reference."""
    pe_dim = dim // 2
    i = np.arange(pe_dim)
    dim_t = nn.libm_f32("powf", np.float32(temperature), (i & ~1).astype(np.float32) / np.float32(pe_dim))
    val = (np.float32(pos) / dim_t).astype(np.float32)
    return np.concatenate([nn.libm_f32("sinf", val), nn.libm_f32("cosf", val)]).astype(np.float32)


def project_tpos(sine, tpos_w, tpos_b):
    """obj_ptr_tpos_proj on the host (sam3.cpp:9186-9195): y[j] = b[j] + sum_i W[j][i] x[i], accumulated in
    float32 from the bias, i in order, each product and sum rounded."""
    acc = np.asarray(tpos_b, np.float32).copy()
    w = np.asarray(tpos_w, np.float32)
    for i in range(sine.shape[0]):
        acc = (acc + (w[:, i] * np.float32(sine[i])).astype(np.float32)).astype(np.float32)
    return acc


def build_prompt(slot_feats, slot_pes, spatial_tpos, tpos_enc, obj_ptrs, ptr_tpos, tpos_w, tpos_b, num_maskmem,
                 max_obj_ptrs=16, MD=64):
    """sam3_build_prompt_and_pos (sam3.cpp:9123-9209): memory tokens + (PE + temporal PE), then each 256-d
    object pointer split into 4 tokens of 64 with the projected 1-D sine PE of rel / 15 (9183). Returns
    (prompt [M, 64], prompt_pos [M, 64], pointer tokens)."""
    prompt, pos = [], []
    for f, pe, tp in zip(slot_feats, slot_pes, spatial_tpos):
        prompt.append(np.asarray(f, np.float32))
        pp = np.asarray(pe, np.float32).copy()
        if 0 <= tp < num_maskmem:
            pp = (pp + np.asarray(tpos_enc, np.float32)[num_maskmem - tp - 1][None, :]).astype(np.float32)
        pos.append(pp)
    n_ptr = 0
    for ptr, rel in zip(obj_ptrs, ptr_tpos):
        if rel < 0:
            continue
        sine = one_d_sine_pe(np.float32(rel) / np.float32(15.0), ptr.shape[0])
        proj = project_tpos(sine, tpos_w, tpos_b)  # [MD]
        split = ptr.shape[0] // MD
        prompt.append(np.asarray(ptr, np.float32).reshape(split, MD))
        pos.append(np.repeat(proj[None, :], split, axis=0))
        n_ptr += split
    if not prompt:
        return np.zeros((0, MD), np.float32), np.zeros((0, MD), np.float32), 0
    return np.concatenate(prompt).astype(np.float32), np.concatenate(pos).astype(np.float32), n_ptr


def select_memory_frames(bank_size, max_slots):
    """sam3_select_memory_frames (sam3.cpp:9423-9447) for a bank of `bank_size` slots."""
    if bank_size <= max_slots:
        return list(range(bank_size))
    sel = [0, bank_size - 1]
    remaining = max_slots - 2
    if remaining > 0:
        step = np.float32(bank_size - 2) / np.float32(remaining + 1)
        for i in range(remaining):
            idx = 1 + int(np.float32(i + 1) * step)
            sel.append(min(idx, bank_size - 2))
    return sorted(set(sel))


def golden_inputs(meta, D=256, MD=64):
    """The seeded inputs of tests/golden/mem_attn_golden.npz (same generator as make_golden.py)."""
    H = meta["feat"]
    rng = np.random.default_rng(meta["inputs_seed"])
    curr = rng.standard_normal((H * H, D), dtype=np.float32)
    m_sp = meta["mem_frames"] * H * H
    n_ptr = 4 * meta["ptrs"]
    prompt = rng.standard_normal((m_sp + n_ptr, MD), dtype=np.float32)
    prompt_pos = (rng.standard_normal((m_sp + n_ptr, MD), dtype=np.float32) * np.float32(0.5)).astype(np.float32)
    return curr, prompt, prompt_pos, n_ptr
