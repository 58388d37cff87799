"""SAM prompt encoder (dense / point embeddings) + SAM mask decoder — numpy oracle (test infrastructure only).

Restates the reference's decoder graph sam3_build_sam_dec_graph (sam3.cpp:10538-10757) with its TwoWay
blocks (sam3_twoway_block_forward, 10436-10495), attention (sam3_sam_attention, 10164-10262: q / k / v
projections, 8 heads, scale 1/sqrt(head dim), out projection), LayerNorm eps 1e-5 (sam3_layer_norm,
1036-1047) and the LayerNorm2d of the upscaling (eps 1e-6, 1049-1060); the dense positional encoding
(sam3_pe_encode_coord / sam3_populate_pe_cache, 10269-10345) and the point prompt embedding of the
image predictor (box corners, points, then one padding point: 10355-10380). Weights are the dict of f32
arrays in .ggml tensor names and PyTorch shapes (sam3_b200.synth.stored_values); feature maps are
channel-last [H, W, C].
"""
import numpy as np

from . import nn


def pe_encode(coords_norm, gauss):
    """[..., 2] coordinates in [0, 1] -> [..., 256] (sam3_pe_encode_coord, sam3.cpp:10269-10282):
    c = 2 x - 1; dot_i = c_x G[0][i] + c_y G[1][i], times 2 pi (f32 steps); sin then cos."""
    c = (np.float32(2.0) * coords_norm.astype(np.float32) - np.float32(1.0)).astype(np.float32)
    g = gauss.astype(np.float32).reshape(2, -1)
    dot = c[..., 0:1] * g[0] + c[..., 1:2] * g[1]
    enc = (dot * np.float32(2.0 * np.pi)).astype(np.float32)
    e64 = enc.astype(np.float64)
    return np.concatenate([np.sin(e64), np.cos(e64)], axis=-1).astype(np.float32)


def dense_pe(W, H):
    """The image PE of the H x H grid at pixel centres, channel-last [H, H, 256] (sam3.cpp:10330-10341)."""
    g = W["sam_pe.pe_gaussian"]
    c = (np.arange(H, dtype=np.float32) + np.float32(0.5)) / np.float32(H)
    xx, yy = np.meshgrid(c, c)  # xx varies along columns
    return pe_encode(np.stack([xx, yy], axis=-1), g)


def prompt_points(pos_points=(), neg_points=(), box=None):
    """sam3_collect_pvs_prompt_tokens (sam3.cpp:10361-10391): box corners (labels 2, 3), positive points
    (1), negative points (0), then one padding point (0, 0) with label -1."""
    coords, labs = [], []
    if box is not None:
        coords += [[box[0], box[1]], [box[2], box[3]]]
        labs += [2, 3]
    coords += [list(p) for p in pos_points]
    labs += [1] * len(pos_points)
    coords += [list(p) for p in neg_points]
    labs += [0] * len(neg_points)
    coords.append([0.0, 0.0])
    labs.append(-1)
    return np.array(coords, np.float32).reshape(-1, 2), labs


def sparse_embeddings(W, coords, labs, input_size=1008, orig_w=None, orig_h=None):
    """Sparse prompt tokens [n, 256] of sam3_segment_pvs (sam3.cpp:10880-10900): each coordinate is
    scaled from the original image to the model input, shifted to the pixel centre and normalised
    (px = x / orig_w * input + 0.5, x_norm = px / input), encoded (pe_encode) and added to
    point_embeddings[label]; the padding point (label -1) is not_a_point_embed alone."""
    orig_w = orig_w or input_size
    orig_h = orig_h or input_size
    c = np.asarray(coords, np.float32).reshape(-1, 2)
    s = np.float32(input_size)
    px = c[:, 0] / np.float32(orig_w) * s + np.float32(0.5)
    py = c[:, 1] / np.float32(orig_h) * s + np.float32(0.5)
    emb = pe_encode(np.stack([px / s, py / s], axis=-1), W["sam_pe.pe_gaussian"])
    out = np.empty_like(emb)
    for i, l in enumerate(labs):
        if l == -1:
            out[i] = W["sam_pe.not_a_point_embed.weight"][0]
        else:
            out[i] = emb[i] + W[f"sam_pe.point_embeddings.{l}.weight"][0]
    return out.astype(np.float32)


def _linear(x, W, name):
    return nn.linear(x, W[name + ".weight"], W[name + ".bias"])


def attention(W, pfx, q, k, v, heads=8):
    """sam3_sam_attention: project, split heads (head h = columns h*hd ..), softmax(q k^T / sqrt(hd)) v, merge, out."""
    Q, K, V = _linear(q, W, pfx + ".q_proj"), _linear(k, W, pfx + ".k_proj"), _linear(v, W, pfx + ".v_proj")
    di = Q.shape[-1]
    hd = di // heads
    sh = lambda t: t.reshape(t.shape[0], heads, hd).transpose(1, 0, 2)
    o = nn.attention(sh(Q), sh(K), sh(V), 1.0 / np.sqrt(hd))  # [heads, nq, hd]
    o = o.transpose(1, 0, 2).reshape(q.shape[0], di)
    return _linear(o, W, pfx + ".out_proj")


def _ln(x, W, name, eps=1e-5):
    return nn.layer_norm(x, W[name + ".weight"], W[name + ".bias"], eps)


def mlp(W, pfx, x, n=3, sigmoid=False):
    for j in range(n):
        x = _linear(x, W, f"{pfx}.layers.{j}")
        if j < n - 1:
            x = np.maximum(x, 0)
    if sigmoid:
        x = (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)
    return x.astype(np.float32)


def decode(W, image_feats, feat_s0, feat_s1, sparse, add_no_mem=False, depth=2, taps=None):
    """image_feats [H, H, 256], feat_s0 [4H, 4H, 256], feat_s1 [2H, 2H, 256], sparse [n, 256] ->
    (masks [4, 4H, 4H], iou [4], obj_score [1], sam_token [256])."""
    H = image_feats.shape[0]
    D = image_feats.shape[-1]
    if add_no_mem:
        image_feats = image_feats + W["no_mem_embed"].reshape(1, 1, D)
    tokens = np.concatenate([W["sam_dec.obj_score_token.weight"], W["sam_dec.iou_token.weight"],
                             W["sam_dec.mask_tokens.weight"], sparse], axis=0).astype(np.float32)
    keys = (image_feats + W["sam_pe.no_mask_embed.weight"].reshape(1, 1, D)).reshape(H * H, D).astype(np.float32)
    key_pe = dense_pe(W, H).reshape(H * H, D)
    queries, query_pe = tokens, tokens
    for i in range(depth):
        p = f"sam_dec.twoway.{i}"
        if i == 0:
            queries = attention(W, p + ".sa", queries, queries, queries)
        else:
            q = queries + query_pe
            queries = queries + attention(W, p + ".sa", q, q, queries)
        queries = _ln(queries, W, p + ".norm1")
        q, k = queries + query_pe, keys + key_pe
        queries = _ln(queries + attention(W, p + ".cross_attn_token_to_image", q, k, keys), W, p + ".norm2")
        h = np.maximum(_linear(queries, W, p + ".mlp.lin1"), 0)
        queries = _ln(queries + _linear(h, W, p + ".mlp.lin2"), W, p + ".norm3")
        q, k = queries + query_pe, keys + key_pe
        keys = _ln(keys + attention(W, p + ".cross_attn_image_to_token", k, q, queries), W, p + ".norm4")
        if taps is not None:
            taps[f"block{i}_queries"] = queries.copy()
            taps[f"block{i}_keys"] = keys.copy()
    q, k = queries + query_pe, keys + key_pe
    queries = _ln(queries + attention(W, "sam_dec.final_attn", q, k, keys), W, "sam_dec.final_norm")
    if taps is not None:
        taps["final_queries"] = queries.copy()
    iou_tok, mask_toks, obj_tok = queries[1], queries[2:6], queries[0]
    # upscaling: deconv -> + conv_s1(feat_s1) -> LayerNorm2d -> GELU -> deconv -> + conv_s0(feat_s0) -> GELU
    src = keys.reshape(1, H, H, D)
    up1 = nn.deconv2x2_cl(src, W["sam_dec.upscale.0.weight"], W["sam_dec.upscale.0.bias"])
    up1 = up1 + nn.conv2d_cl(feat_s1[None], W["sam_dec.conv_s1.weight"], W["sam_dec.conv_s1.bias"])
    up1 = nn.gelu_erf(nn.layer_norm(up1, W["sam_dec.upscale.1.weight"], W["sam_dec.upscale.1.bias"], 1e-6))
    up2 = nn.deconv2x2_cl(up1, W["sam_dec.upscale.3.weight"], W["sam_dec.upscale.3.bias"])
    up2 = nn.gelu_erf(up2 + nn.conv2d_cl(feat_s0[None], W["sam_dec.conv_s0.weight"], W["sam_dec.conv_s0.bias"]))[0]
    if taps is not None:
        taps["upscaled"] = up2.copy()
    hyper = np.stack([mlp(W, f"sam_dec.hyper.{m}", mask_toks[m][None])[0] for m in range(mask_toks.shape[0])])
    masks = np.einsum("mc,hwc->mhw", hyper.astype(np.float64), up2.astype(np.float64)).astype(np.float32)
    iou = mlp(W, "sam_dec.iou_prediction_head", iou_tok[None], sigmoid=True)[0]
    obj = mlp(W, "sam_dec.pred_obj_score_head", obj_tok[None])[0]
    return masks, iou, obj, mask_toks[0].copy()
