"""Kernel-level parity through the C ABI: tensor-core GEMM, flash attention,
LayerNorm and block dequantisation against fp32 references on the same inputs."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _ref_gemm(A, B, bias, act, resid):
    y = A.float() @ B.float().T
    if bias is not None:
        y = y + bias
    if act == 1:
        y = torch.nn.functional.gelu(y)
    elif act == 2:
        y = torch.nn.functional.gelu(y, approximate="tanh")
    elif act == 3:
        y = torch.relu(y)
    if resid is not None:
        y = y + resid
    return y


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 96, 96), (5184, 3072, 1024), (1000, 4736, 1024),
                                   (777, 1024, 4736), (64, 128, 592), (4097, 288, 152), (256, 512, 2304)])
@pytest.mark.parametrize("act", [0, 1])
def test_gemm(engine, M, N, K, act):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K + act)
    A = (torch.randn(M, K, device="cuda", generator=g) * 0.5).half()
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    resid = torch.randn(M, N, device="cuda", generator=g) if act == 0 else None
    out = torch.empty(M, N, device="cuda", dtype=torch.float32)
    engine.gemm(A, B, out, bias=bias, act=act, resid=resid)
    engine.sync()
    ref = _ref_gemm(A, B, bias, act, resid)
    err = (out - ref).abs().max().item()
    tol = 2e-3 * max(1.0, ref.abs().max().item()) + 1e-4 * K ** 0.5
    assert err < tol, f"max abs err {err} (tol {tol})"


@pytest.mark.parametrize("wide", [0, 1])
@pytest.mark.parametrize("pairs", [0, 1, 2])
@pytest.mark.parametrize("M,N,K,resid", [(41472 // 8 + 130, 3072, 1024, False), (1000, 4736, 1024, False),
                                         (5184, 1024, 4736, True), (4097, 288, 152, True), (257, 512, 64, True),
                                         (5184, 1024, 1024, True)])
def test_gemm_pairs_and_single(engine, wide, pairs, M, N, K, resid):
    """256-row tiles on SM pairs (cta_group::2) and 128-row tiles on single SMs, 8 or 16 epilogue warps
    (16: one staging buffer per column group), ragged M / N / K tails, f16 and f32 (in-place residual)
    outputs, against the fp32 reference."""
    engine.set_option("gemm_pairs", pairs)
    engine.set_option("gemm_wide_epilogue", wide)
    try:
        g = torch.Generator(device="cuda").manual_seed(M + N + K + pairs)
        A = (torch.randn(M, K, device="cuda", generator=g) * 0.5).half()
        B = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
        bias = torch.randn(N, device="cuda", generator=g) * 0.1
        if resid:
            out = torch.randn(M, N, device="cuda", generator=g)
            ref = out + A.float() @ B.float().T + bias
            engine.gemm(A, B, out, bias=bias, resid=out)
        else:
            out = torch.empty(M, N, device="cuda", dtype=torch.float16)
            ref = A.float() @ B.float().T + bias
            engine.gemm(A, B, out, bias=bias)
        engine.sync()
        err = (out.float() - ref).abs().max().item()
        assert err < 2e-3 * max(1.0, ref.abs().max().item()) + 1e-4 * K ** 0.5 + (0 if resid else 1e-2), err
    finally:
        engine.set_option("gemm_pairs", 2)  # the default
        engine.set_option("gemm_wide_epilogue", 1)


@pytest.mark.parametrize("pairs", [1, 2])
@pytest.mark.parametrize("wide", [0, 1])
@pytest.mark.parametrize("M,N,K,act", [(5184, 4736, 1024, 1), (1000, 3072, 256, 0), (777, 288, 96, 2),
                                       (130, 1000, 1024, 3)])
def test_gemm_f16_epilogue_warps(engine, pairs, wide, M, N, K, act):
    """f16-output GEMMs with 8 or 16 epilogue warps (column groups of 128 or 64), on single SMs
    or SM pairs, ragged M / N."""
    engine.set_option("gemm_wide_epilogue", wide)
    engine.set_option("gemm_pairs", pairs)
    try:
        g = torch.Generator(device="cuda").manual_seed(M * 3 + N + act)
        A = (torch.randn(M, K, device="cuda", generator=g) * 0.5).half()
        B = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
        bias = torch.randn(N, device="cuda", generator=g) * 0.1
        out = torch.full((M, N), 3.0, device="cuda", dtype=torch.float16)
        engine.gemm(A, B, out, bias=bias, act=act)
        engine.sync()
        ref = _ref_gemm(A, B, bias, act, None)
        assert (out.float() - ref).abs().max().item() < 1e-2 * max(1.0, ref.abs().max().item())
    finally:
        engine.set_option("gemm_wide_epilogue", 1)
        engine.set_option("gemm_pairs", 2)  # the default


@pytest.mark.parametrize("wide", [0, 1])
def test_gemm_rope_epilogue_warps(engine, wide):
    """QKV-shaped GEMM with RoPE on q, k (ViT window layout) with 8 or 16 epilogue warps."""
    engine.set_option("gemm_wide_epilogue", wide)
    try:
        M, E, HD = 576 * 9, 1024, 64
        g = torch.Generator(device="cuda").manual_seed(11)
        A = torch.randn(M, E, device="cuda", generator=g).half()
        B = (torch.randn(3 * E, E, device="cuda", generator=g) * 0.03).half()
        bias = torch.randn(3 * E, device="cuda", generator=g) * 0.1
        ang = torch.rand(576, HD // 2, device="cuda", generator=g) * 6.28
        table = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
        out = torch.empty(M, 3 * E, device="cuda", dtype=torch.float16)
        engine.gemm_rope(A, B, out, bias, table, HD, 2 * E, 576)
        engine.sync()
        y = A.float() @ B.float().T + bias
        pos = torch.arange(M, device="cuda") % 576
        c = table[pos, :, 0].repeat(1, 2 * E // HD)
        s = table[pos, :, 1].repeat(1, 2 * E // HD)
        a, b = y[:, 0:2 * E:2], y[:, 1:2 * E:2]
        ref = y.clone()
        ref[:, 0:2 * E:2] = a * c - b * s
        ref[:, 1:2 * E:2] = a * s + b * c
        assert (out.float() - ref).abs().max().item() < 2e-2
    finally:
        engine.set_option("gemm_wide_epilogue", 1)


@pytest.mark.parametrize("M,N,K", [(5184, 1024, 1024), (1000, 96, 256), (333, 1024, 4736)])
def test_gemm_inplace_residual(engine, M, N, K):
    """out += A B^T + bias with the residual being the output itself (the
    epilogue loads the residual chunk by TMA into its staging buffer)."""
    g = torch.Generator(device="cuda").manual_seed(M + N)
    A = torch.randn(M, K, device="cuda", generator=g).half()
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(N, device="cuda", generator=g)
    x = torch.randn(M, N, device="cuda", generator=g)
    ref = x + A.float() @ B.float().T + bias
    engine.gemm(A, B, x, bias=bias, resid=x)
    engine.sync()
    assert (x - ref).abs().max().item() < 2e-3 * max(1.0, ref.abs().max().item())


def test_gemm_rope_f16(engine):
    """RoPE on the first 2*E columns (q, k) of a fused qkv projection, f16 TMA-store epilogue."""
    M, E, HD = 576 * 2, 256, 64
    g = torch.Generator(device="cuda").manual_seed(7)
    A = torch.randn(M, E, device="cuda", generator=g).half()
    B = (torch.randn(3 * E, E, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(3 * E, device="cuda", generator=g) * 0.1
    ang = torch.rand(576, HD // 2, device="cuda", generator=g) * 6.28
    table = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
    out = torch.empty(M, 3 * E, device="cuda", dtype=torch.float16)
    engine.gemm_rope(A, B, out, bias, table, HD, 2 * E, 576)
    engine.sync()
    y = A.float() @ B.float().T + bias
    pos = torch.arange(M, device="cuda") % 576
    c = table[pos, :, 0].repeat(1, 2 * E // HD)
    s = table[pos, :, 1].repeat(1, 2 * E // HD)
    a, b = y[:, 0:2 * E:2], y[:, 1:2 * E:2]
    ref = y.clone()
    ref[:, 0:2 * E:2] = a * c - b * s
    ref[:, 1:2 * E:2] = a * s + b * c
    assert (out.float() - ref).abs().max().item() < 2e-2


@pytest.mark.parametrize("act", [1, 2])
def test_gemm_activation_accuracy(engine, act):
    """The epilogue GELUs (erf by Abramowitz-Stegun 7.1.26; tanh via exp) against
    float64 references: A holds f16-exact inputs, B = I, so out = act(x) exactly up
    to the activation's own error (bound 2e-6 absolute + 1e-6 relative)."""
    x = torch.linspace(-9.0, 9.0, 128 * 64, device="cuda").half().reshape(-1, 64)
    eye = torch.eye(64, device="cuda").half()
    out = torch.empty(x.shape[0], 64, device="cuda", dtype=torch.float32)
    engine.gemm(x, eye, out, act=act)
    engine.sync()
    xd = x.double()
    if act == 1:
        ref = 0.5 * xd * (1 + torch.erf(xd / 2 ** 0.5))
    else:
        ref = 0.5 * xd * (1 + torch.tanh(0.7978845608028654 * (xd + 0.044715 * xd ** 3)))
    err = (out.double() - ref).abs()
    assert (err <= 2e-6 + 1e-6 * ref.abs()).all(), err.max().item()


def test_gemm_f16_out_strided(engine):
    M, N, K = 513, 640, 320
    A_full = torch.randn(M, K + 64, device="cuda").half()
    A = A_full[:, :K]
    B = (torch.randn(N, K, device="cuda") * 0.05).half()
    out = torch.zeros(M, N, device="cuda", dtype=torch.float16)
    engine.gemm(A, B, out, act=3)
    engine.sync()
    ref = torch.relu(A.float() @ B.float().T)
    assert (out.float() - ref).abs().max().item() < 1e-2


@pytest.mark.parametrize("D,nq,nk,heads,batch", [(64, 576, 576, 16, 2), (64, 5184, 5184, 2, 1), (96, 49, 196, 8, 3),
                                                 (96, 4096, 4096, 1, 1), (80, 100, 100, 2, 2),
                                                 (256, 1000, 3000, 1, 1), (128, 70, 33, 3, 2),
                                                 (72, 196, 196, 2, 3), (72, 49, 196, 16, 2),
                                                 # more (batch, head) pairs than a grid's y extent (Hiera-T
                                                 # stage-1 windows at 16 frames per pass)
                                                 (96, 16, 16, 4, 16400),
                                                 # d = 256 on the tcgen05 kernel: heads as row blocks, ragged keys
                                                 (256, 300, 500, 2, 2), (256, 128, 64, 1, 3), (256, 1, 77, 3, 1),
                                                 # d = 72 / 96 with a full query tile on the tcgen05 kernel
                                                 (72, 300, 500, 3, 2), (96, 1000, 300, 2, 1), (72, 4096, 4096, 1, 1),
                                                 # small windows, one warp per (batch, head): every key padding
                                                 # (16 / 32 / 48 / 64), ragged query counts, pad d = 72
                                                 (96, 16, 16, 2, 301), (96, 4, 16, 4, 99), (72, 16, 64, 2, 50),
                                                 (64, 9, 40, 3, 7), (128, 1, 5, 2, 3), (72, 4, 16, 8, 33)])
def test_attention(engine, D, nq, nk, heads, batch):
    g = torch.Generator(device="cuda").manual_seed(D + nq + nk)
    q = torch.randn(batch, heads, nq, D, device="cuda", generator=g).half()
    k = torch.randn(batch, heads, nk, D, device="cuda", generator=g).half()
    v = torch.randn(batch, heads, nk, D, device="cuda", generator=g).half()
    out = torch.empty(batch, nq, heads * D, device="cuda", dtype=torch.float16)
    scale = 1.0 / D ** 0.5
    engine.attention(q, k, v, out, scale)
    engine.sync()
    ref = torch.softmax((q.float() @ k.float().transpose(-1, -2)) * scale, dim=-1) @ v.float()
    ref = ref.permute(0, 2, 1, 3).reshape(batch, nq, heads * D)
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, err


def _ref_attention_qkv(qkv, nwin, heads, ntok, d, scale):
    E = heads * d
    x = qkv[:, :3 * E].float().view(nwin, ntok, 3, heads, d).permute(2, 0, 3, 1, 4)
    q, k, v = x[0], x[1], x[2]
    o = torch.softmax((q @ k.transpose(-1, -2)) * scale, dim=-1) @ v
    return o.permute(0, 2, 1, 3).reshape(nwin * ntok, E)


# d = 64 over one fused qkv buffer runs the tcgen05 kernel (ViT window / global
# attention shapes, ragged token counts, padded row strides); other d use the
# mma.sync kernel through the same entry point.
@pytest.mark.parametrize("nwin,heads,ntok,d,pad", [(9, 16, 576, 64, 0), (1, 16, 5184, 64, 0), (3, 2, 64, 64, 0),
                                                   (2, 3, 200, 64, 64), (5, 1, 129, 64, 8), (1, 4, 1, 64, 0),
                                                   (4, 2, 300, 72, 0), (2, 2, 256, 96, 32)])
@pytest.mark.parametrize("impl", [0, 3, 4])
def test_attention_qkv(engine, nwin, heads, ntok, d, pad, impl):
    """impl 0 (and 4): one persistent CTA per SM with two query tiles and one thread per query row; 3: one
    query tile per CTA, each row's softmax split over two warps."""
    g = torch.Generator(device="cuda").manual_seed(nwin * 1000 + heads * 10 + ntok)
    E = heads * d
    qkv = (torch.randn(nwin * ntok, 3 * E + pad, device="cuda", generator=g) * 1.5).half()
    out = torch.full((nwin * ntok, E + pad), 7.0, device="cuda", dtype=torch.float16)
    scale = 1.0 / d ** 0.5
    engine.set_option("attention_impl", impl)
    try:
        engine.attention_qkv(qkv, out, nwin, heads, ntok, d, scale)
        engine.sync()
    finally:
        engine.set_option("attention_impl", 0)
    ref = _ref_attention_qkv(qkv, nwin, heads, ntok, d, scale)
    err = (out[:, :E].float() - ref).abs().max().item()
    assert err < 2e-2, err
    if pad:
        assert torch.all(out[:, E:] == 7.0), "wrote past the head columns"


def test_attention_qkv_impls_agree(engine):
    """The mma.sync kernel and the tcgen05 kernel (MUFU-only and polynomial exponentials) agree."""
    nwin, heads, ntok, d = 4, 16, 576, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    qkv = (torch.randn(nwin * ntok, 3 * heads * d, device="cuda", generator=g) * 2).half()
    outs = []
    for impl, poly in ((1, 0), (0, 0), (0, 2), (0, 4), (3, 0), (3, 3), (4, 0), (4, 2), (4, 4)):
        engine.set_option("attention_impl", impl)
        engine.set_option("attention_exp_poly", poly)
        engine.set_option("attention_fa_exp_poly", poly)
        out = torch.empty(nwin * ntok, heads * d, device="cuda", dtype=torch.float16)
        engine.attention_qkv(qkv, out, nwin, heads, ntok, d, 0.125)
        engine.sync()
        outs.append(out.float())
    engine.set_option("attention_impl", 0)
    engine.set_option("attention_exp_poly", 0)
    engine.set_option("attention_fa_exp_poly", 1)
    for o in outs[1:]:
        assert (o - outs[0]).abs().max().item() < 1e-2


@pytest.mark.parametrize("impl", [0, 3, 4])
def test_attention_qkv_growing_max(engine, impl):
    """Keys whose logits grow tile by tile, so the running reference max of the d = 64 kernels moves
    after the first key tile and the running O rows are rescaled in TMEM (both kernels)."""
    nwin, heads, ntok, d = 2, 4, 600, 64
    E = heads * d
    g = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn(nwin, ntok, 3, heads, d, device="cuda", generator=g)
    grow = 1.0 + torch.arange(ntok, device="cuda").float() / 128.0  # key tile j scaled by about 1 + j
    x[:, :, 1] *= grow.view(1, ntok, 1, 1) * 3.0
    x[:, :, 0] *= 3.0
    qkv = x.reshape(nwin * ntok, 3 * E).half()
    out = torch.empty(nwin * ntok, E, device="cuda", dtype=torch.float16)
    engine.set_option("attention_impl", impl)
    try:
        engine.attention_qkv(qkv, out, nwin, heads, ntok, d, 0.125)
        engine.sync()
    finally:
        engine.set_option("attention_impl", 0)
    ref = _ref_attention_qkv(qkv, nwin, heads, ntok, d, 0.125)
    assert torch.isfinite(out).all()
    assert (out.float() - ref).abs().max().item() < 3e-2


@pytest.mark.parametrize("D", [72, 96])
@pytest.mark.parametrize("k128", [0, 1])
def test_attention_wide_key_tiles(engine, D, k128):
    """d = 72 / 96 on both tcgen05 kernels (option attention_wide_k128): 64-key tiles with two CTAs per SM and
    128-key tiles with P in TMEM, heads as column offsets of a fused qkv buffer (Hiera) and as row blocks,
    ragged query and key counts (the last 128-key tile masked), key splits."""
    engine.set_option("attention_wide_k128", k128)
    try:
        nwin, heads, ntok = 2, 3, 1300
        g = torch.Generator(device="cuda").manual_seed(D + 7 * k128)
        E = heads * D
        qkv = (torch.randn(nwin * ntok, 3 * E, device="cuda", generator=g) * 1.5).half()
        out = torch.empty(nwin * ntok, E, device="cuda", dtype=torch.float16)
        engine.attention_qkv(qkv, out, nwin, heads, ntok, D, D ** -0.5)
        engine.sync()
        assert (out.float() - _ref_attention_qkv(qkv, nwin, heads, ntok, D, D ** -0.5)).abs().max().item() < 2e-2
        q = torch.randn(1, 2, 4096, D, device="cuda", generator=g).half()
        k = torch.randn(1, 2, 1500, D, device="cuda", generator=g).half()
        v = torch.randn(1, 2, 1500, D, device="cuda", generator=g).half()
        o = torch.empty(1, 4096, 2 * D, device="cuda", dtype=torch.float16)
        engine.attention(q, k, v, o, D ** -0.5)
        engine.sync()
        ref = torch.softmax((q.float() @ k.float().transpose(-1, -2)) * D ** -0.5, dim=-1) @ v.float()
        assert (o.float() - ref.permute(0, 2, 1, 3).reshape(1, 4096, 2 * D)).abs().max().item() < 2e-2
    finally:
        engine.set_option("attention_wide_k128", -1)


@pytest.mark.parametrize("nq,nk", [(4096, 1100), (300, 777)])
def test_attention_d256_growing_max(engine, nq, nk):
    """d = 256 (memory attention): keys whose logits grow tile by tile, so the reference max moves after
    the first 128-key tile and the O rows are rescaled in TMEM; with 4096 queries the keys are also split
    over CTAs and merged by the combine kernel."""
    g = torch.Generator(device="cuda").manual_seed(nq + nk)
    q = torch.randn(1, 1, nq, 256, device="cuda", generator=g) * 0.5
    k = torch.randn(1, 1, nk, 256, device="cuda", generator=g) * 0.5
    k *= (1.0 + torch.arange(nk, device="cuda").float() / 96.0).view(1, 1, nk, 1)
    v = torch.randn(1, 1, nk, 256, device="cuda", generator=g)
    q, k, v = q.half(), k.half(), v.half()
    out = torch.empty(1, nq, 256, device="cuda", dtype=torch.float16)
    engine.attention(q, k, v, out, 1.0 / 16)
    engine.sync()
    ref = torch.softmax((q.float() @ k.float().transpose(-1, -2)) / 16, dim=-1) @ v.float()
    assert torch.isfinite(out).all()
    assert (out.float() - ref.reshape(1, nq, 256)).abs().max().item() < 3e-2


@pytest.mark.parametrize("rows,C,f32", [(5184, 1024, 0), (1000, 96, 1), (37, 256, 0), (64, 1152, 1), (5000, 144, 0),
                                        (777, 192, 1), (301, 288, 0), (129, 576, 1), (65, 64, 0), (33, 80, 1),
                                        (70001, 96, 0)])
def test_layernorm(engine, rows, C, f32):
    """Widths whose float4 count is a multiple of 32 run one row per warp; the others (Hiera's 96, 144,
    192, 288, 576, ...) run L-lane row groups, several rows per warp."""
    x = torch.randn(rows, C, device="cuda") * 3 + 1
    g = torch.randn(C, device="cuda")
    b = torch.randn(C, device="cuda")
    out = torch.empty(rows, C, device="cuda", dtype=torch.float32 if f32 else torch.float16)
    engine.layernorm(x, out, g, b, 1e-6)
    engine.sync()
    ref = torch.nn.functional.layer_norm(x, (C,), g, b, 1e-6)
    assert (out.float() - ref).abs().max().item() < (2e-5 * C ** 0.5 + 1e-4 if f32 else 2e-2)


@pytest.mark.parametrize("implicit,pairs", [(1, 1), (1, 0), (0, 1)])
@pytest.mark.parametrize("B,H,W,C,Cout", [(1, 36, 36, 256, 256), (2, 17, 23, 64, 128), (1, 72, 72, 256, 256),
                                          (3, 9, 40, 128, 64), (1, 5, 7, 64, 256), (2, 144, 144, 256, 256)])
def test_conv3x3(engine, implicit, pairs, B, H, W, C, Cout):
    """3x3 / pad 1 conv: implicit GEMM (8 x 16 pixel blocks by 4-D TMA, zero-filled border taps, clipped
    stores at ragged edges) on single SMs or SM pairs, and im2col + GEMM, against the fp32 reference."""
    g = torch.Generator(device="cuda").manual_seed(H * W + C)
    x = torch.randn(B, H, W, C, device="cuda", generator=g).half()
    w = (torch.randn(Cout, 3, 3, C, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(Cout, device="cuda", generator=g) * 0.1
    out = torch.full((B, H, W, Cout), float("nan"), device="cuda", dtype=torch.float32)
    engine.set_option("conv_implicit", implicit)
    engine.set_option("gemm_pairs", pairs)
    try:
        engine.conv3x3(x, w, bias, out)
        engine.sync()
    finally:
        engine.set_option("conv_implicit", 1)
        engine.set_option("gemm_pairs", 2)  # the default
    ref = torch.nn.functional.conv2d(x.float().permute(0, 3, 1, 2), w.float().permute(0, 3, 1, 2), bias, padding=1)
    ref = ref.permute(0, 2, 3, 1)
    err = (out - ref).abs().max().item()
    assert err < 2e-3 * max(1.0, ref.abs().max().item()), err


@pytest.mark.parametrize("blocks,pairs", [(1, 1), (1, 0), (0, 1)])
@pytest.mark.parametrize("B,H,W,Cin,Cout,act,f32", [(1, 72, 72, 1024, 512, 1, 0), (2, 17, 23, 64, 256, 0, 0),
                                                    (1, 36, 40, 512, 256, 0, 1), (3, 9, 5, 96, 64, 1, 1)])
def test_deconv2x2(engine, blocks, pairs, B, H, W, Cin, Cout, act, f32):
    """2x2 / stride 2 transposed conv: pixel-block GEMM with 5-D TMA output stores (ragged blocks
    clipped) on single SMs or SM pairs, and the scattered-store GEMM, against the fp32 reference."""
    g = torch.Generator(device="cuda").manual_seed(H * W + Cin + Cout)
    x = torch.randn(B, H, W, Cin, device="cuda", generator=g).half()
    w = (torch.randn(2, 2, Cout, Cin, device="cuda", generator=g) * (0.5 / Cin ** 0.5)).half()
    bias = torch.randn(Cout, device="cuda", generator=g) * 0.1
    out = torch.full((B, 2 * H, 2 * W, Cout), float("nan"), device="cuda",
                     dtype=torch.float32 if f32 else torch.float16)
    engine.set_option("conv_implicit", blocks)
    engine.set_option("gemm_pairs", pairs)
    try:
        engine.deconv2x2(x, w, bias, out, act)
        engine.sync()
    finally:
        engine.set_option("conv_implicit", 1)
        engine.set_option("gemm_pairs", 2)  # the default
    # torch weight layout for conv_transpose2d: [Cin][Cout][kh][kw]
    wt = w.float().permute(3, 2, 0, 1).contiguous()
    ref = torch.nn.functional.conv_transpose2d(x.float().permute(0, 3, 1, 2), wt, bias, stride=2)
    if act:
        ref = torch.nn.functional.gelu(ref)
    ref = ref.permute(0, 2, 3, 1)
    err = (out.float() - ref).abs().max().item()
    assert err < (2e-3 if f32 else 1e-2) * max(1.0, ref.abs().max().item()), err


def test_conv3x3_implicit_equals_im2col(engine):
    """The implicit GEMM reads the same products in the same K order (tap, channel) as the GEMM over
    the column matrix, so both paths give the same bits."""
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(2, 40, 56, 256, device="cuda", generator=g).half()
    w = (torch.randn(256, 3, 3, 256, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(256, device="cuda", generator=g) * 0.1
    outs = []
    for implicit in (1, 0):
        engine.set_option("conv_implicit", implicit)
        out = torch.empty(2, 40, 56, 256, device="cuda", dtype=torch.float32)
        engine.conv3x3(x, w, bias, out)
        engine.sync()
        outs.append(out)
    engine.set_option("conv_implicit", 1)
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("qtype", [2, 3, 8])
def test_dequant_bit_exact(engine, s3b, qtype):
    from oracle import quant
    rng = np.random.default_rng(qtype)
    x = rng.standard_normal((64, 4736)).astype(np.float32) * 0.02
    raw = quant.quantize(qtype, x)
    ref = quant.dequantize(qtype, raw, 4736)
    d_raw = torch.from_numpy(raw).cuda()
    out = torch.empty(64, 4736, device="cuda", dtype=torch.float32)
    engine.dequantize(d_raw, qtype, 4736, 64, out)
    engine.sync()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
