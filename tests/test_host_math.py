"""Host-side arithmetic of the engine checked against the oracle on the CPU (no GPU):

- the sinusoidal 2D PE the engine serves as the "neck_trk_pe_i" outputs and as memory attention's src_pos
  and slot PEs (sam3_sinusoidal_pe_2d, sam3.cpp:3597-3633), bit-exact at every size the configurations use;
- the memory-bank frame selection (sam3_select_memory_frames, sam3.cpp:9423-9447), exact for every bank
  size and slot count in a sweep.
"""
import numpy as np
import pytest

from oracle import mem_attn as om
from oracle import nn


@pytest.mark.parametrize("S,d", [(288, 256), (144, 256), (72, 256), (36, 256),  # SAM 3 ViT neck levels
                                 (256, 256), (128, 256), (64, 256),            # Hiera FPN levels
                                 (64, 64), (16, 64), (5, 8)])                  # memory slots, odd sizes
def test_sine_pe_2d_bit_exact(s3b, S, d):
    got = s3b.sine_pe_2d(S, S, d)
    ref = nn.sine_pe_2d(S, S, d)
    assert got.shape == ref.shape
    assert np.array_equal(got, ref), np.abs(got - ref).max()


def test_sine_pe_2d_rectangular_and_rejects_bad_sizes(s3b):
    assert np.array_equal(s3b.sine_pe_2d(7, 9, 64), nn.sine_pe_2d(7, 9, 64))
    with pytest.raises(s3b.S3BError):
        s3b.sine_pe_2d(4, 4, 63)  # odd channel count


def test_select_memory_frames_matches_reference_rule(s3b):
    for bank in range(0, 41):
        for max_slots in range(0, 12):
            got = s3b.select_memory_frames(bank, max_slots)
            assert got == om.select_memory_frames(bank, max_slots), (bank, max_slots, got)
    # the documented examples of the rule: everything when it fits, first + last + evenly spaced otherwise
    assert s3b.select_memory_frames(5, 7) == [0, 1, 2, 3, 4]
    assert s3b.select_memory_frames(20, 7) == [0, 4, 7, 10, 13, 16, 19]


def test_one_d_sine_pe_is_libm_exact():
    # the oracle's 1-D PE uses the C library's sinf / cosf / powf on float32 arguments (sam3.cpp:3636-3647);
    # pin two entries computed independently through ctypes
    pe = om.one_d_sine_pe(np.float32(3) / np.float32(15), 256)
    assert pe.dtype == np.float32 and pe.shape == (256,)
    v0 = np.float32(3) / np.float32(15)  # dim_t = 1 for i = 0
    assert pe[0] == nn.libm_f32("sinf", v0) and pe[128] == nn.libm_f32("cosf", v0)
