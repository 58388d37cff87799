"""The arithmetic of the block-form weight path (option weights_quantised), checked on the CPU.

Inside the GEMM a block value q becomes an f16 weight by the 0x6400-exponent trick: the f16 with bits
0x6400 | u is exactly 1024 + u for u < 1024, so subtracting 1032 (q4_0: u = q) or 1152 (q8_0: u = q ^ 0x80 =
q + 128) gives the integer exactly, and one rounded f16 multiply by the block scale d gives round_f16(q' * d).
The load-time path computes the same value as round_f16(f32(q' * d)); the product of two f16 values is exact
in f32, so both round the same real number once and must agree bit for bit, subnormal scales included.

numpy's float16 arithmetic rounds each operation's exact result once, as the device's sub.rn / mul.rn.f16x2
do, so it stands in for the device instructions here. The q4_0 nibble plane packs 8 values per 32-bit word
(value 2p in nibble p, value 2p + 1 in nibble p + 4), so that pair p of the word is (w >> 4p) & 0x000F000F.
"""
import numpy as np

from oracle import quant as oq


def _f16_from_bits(b):
    return np.asarray(b, dtype=np.uint16).view(np.float16)


def _scales():
    # every exponent of f16, several mantissas each, both signs: normals, subnormals and the largest values
    bits = np.concatenate([np.arange(0x0001, 0x7C00, 37, dtype=np.uint16), np.array([0x0001, 0x03FF, 0x0400, 0x7BFF],
                                                                                    dtype=np.uint16)])
    bits = np.concatenate([bits, bits | 0x8000])
    return _f16_from_bits(bits)


def _load_time(qprime, d):
    # the load-time dequantisation: f32 product, then one rounding to f16
    return (qprime.astype(np.float32) * d.astype(np.float32)).astype(np.float16)


def test_q4_0_exponent_trick_equals_load_time_rounding():
    d = _scales()[None, :]
    q = np.arange(16, dtype=np.uint16)[:, None]
    x = _f16_from_bits(0x6400 | q)                       # 1024 + q, exact
    with np.errstate(over="ignore"):                      # the largest scales overflow to inf in both paths
        v = (x - np.float16(1032.0)) * d                  # (q - 8) exact, then one rounded multiply
        ref = _load_time((q.astype(np.int32) - 8), d)
    assert np.array_equal(v.view(np.uint16), ref.view(np.uint16))


def test_q8_0_exponent_trick_equals_load_time_rounding():
    d = _scales()[None, :]
    q = np.arange(-128, 128, dtype=np.int32)[:, None]
    u = (q.astype(np.int8).view(np.uint8) ^ 0x80).astype(np.uint16)  # q + 128 in [0, 255]
    x = _f16_from_bits(0x6400 | u)
    with np.errstate(over="ignore"):
        v = (x - np.float16(1152.0)) * d
        ref = _load_time(q, d)
    assert np.array_equal(v.view(np.uint16), ref.view(np.uint16))


def _pack_q4_words(vals8):
    """8 nibbles (values 0..15 of 8 consecutive weights) -> one 32-bit word of the q4_0 value plane."""
    w = 0
    for p in range(4):
        w |= int(vals8[2 * p]) << (4 * p)
        w |= int(vals8[2 * p + 1]) << (16 + 4 * p)
    return w


def test_q4_0_plane_word_pairs():
    rng = np.random.default_rng(0)
    for _ in range(200):
        vals = rng.integers(0, 16, 8)
        w = _pack_q4_words(vals)
        for p in range(4):
            pair = (w >> (4 * p)) & 0x000F000F
            assert pair & 0xFFFF == vals[2 * p] and pair >> 16 == vals[2 * p + 1]


def test_q4_0_plane_from_ggml_blocks_dequantises_like_the_oracle():
    """ggml q4_0 rows -> value plane words + scales -> the exponent trick, against the oracle's dequantisation
    rounded to f16 (the load-time values)."""
    rng = np.random.default_rng(1)
    K = 96
    w = (rng.standard_normal((8, K)) * 0.05).astype(np.float32)
    raw = oq.quantize(2, w)
    ref = oq.dequantize(2, raw, K).astype(np.float16)
    got = np.empty_like(ref)
    for n in range(raw.shape[0]):
        for b in range(K // 32):
            blk = raw[n, b * 18:(b + 1) * 18]
            d = blk[:2].view(np.float16)[0]
            qs = blk[2:]
            q = np.concatenate([qs & 0x0F, qs >> 4])          # ggml order: value j and value j + 16 share byte j
            for g in range(4):
                word = _pack_q4_words(q[8 * g:8 * g + 8])
                for p in range(4):
                    pair = (word >> (4 * p)) & 0x000F000F
                    for half, lo in ((pair & 0xFFFF, 0), (pair >> 16, 1)):
                        x = _f16_from_bits(0x6400 | half)
                        got[n, b * 32 + 8 * g + 2 * p + lo] = (x - np.float16(1032.0)) * d
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
