"""Properties of the quantised-weight oracle: packing order, round trips,
known-answer cases and quantiser error bounds."""
import numpy as np

from oracle import quant_oracle as qo


def test_nibble_order_low_is_even_k():
    q = np.array([[1, 2, 3, 4, 15, 0]], np.uint8)
    p = qo.pack_nibbles(q)
    assert p.tolist() == [[0x21, 0x43, 0x0F]]
    np.testing.assert_array_equal(qo.unpack_nibbles(p, 6), q)


def test_nf4_levels_are_reference_literals():
    assert qo.NF4_LEVELS.dtype == np.float32 and qo.NF4_LEVELS.shape == (16,)
    assert qo.NF4_LEVELS[7] == 0.0 and qo.NF4_LEVELS[0] == -1.0 and qo.NF4_LEVELS[15] == 1.0
    assert np.all(np.diff(qo.NF4_LEVELS) > 0)
    assert qo.NF4_LEVELS[8] == np.float32(0.0796)


def test_nf4_known_answer():
    # one row, one block of 4: absmax 2.0, values map to levels exactly
    W = np.array([[2.0, -2.0, 0.0, 2.0 * 0.4407]], np.float32)
    p, am = qo.quantize_nf4(W, block_size=4)
    codes = qo.unpack_nibbles(p, 4)
    assert am.tolist() == [[2.0]]
    assert codes.tolist() == [[15, 0, 7, 12]]
    np.testing.assert_array_equal(qo.dequant_nf4(p, am, 4, 4), [[2.0, -2.0, 0.0,
                                                                 np.float32(0.4407) * 2]])


def test_nf4_zero_block_and_ragged_tail():
    W = np.zeros((2, 10), np.float32)
    W[1, 8:] = [0.5, -0.25]
    p, am = qo.quantize_nf4(W, block_size=8)
    assert am.shape == (2, 2)
    assert am[0].tolist() == [0.0, 0.0]
    Wd = qo.dequant_nf4(p, am, 10, 8)
    np.testing.assert_array_equal(Wd[0], 0)
    assert Wd[1, 8] == 0.5 and Wd[1, 9] == np.float32(-0.5251) * 0.5


def test_nf4_error_bound():
    rng = np.random.default_rng(0)
    W = (rng.standard_normal((64, 512)) / 64).astype(np.float32)
    p, am = qo.quantize_nf4(W, 64)
    Wd = qo.dequant_nf4(p, am, 512, 64)
    # half the largest gap between levels, times absmax
    gap = np.max(np.diff(qo.NF4_LEVELS)) / 2
    am_full = np.repeat(am, 64, axis=1)
    assert np.all(np.abs(Wd - W) <= gap * am_full + 1e-7)


def test_int_grouped_round_trip_and_bounds():
    rng = np.random.default_rng(1)
    W = (rng.standard_normal((16, 384)) / 64).astype(np.float32)
    for bits in (4, 8):
        q, s, z = qo.quantize_int_grouped(W, bits, 128)
        assert q.max() <= 2 ** bits - 1
        assert s.dtype == np.float16 and z.dtype == np.float16 and s.shape == (16, 3)
        Wd = qo.dequant_int_grouped(q, s, z, 384, 128)
        step = np.repeat(s.astype(np.float32), 128, axis=1)
        err = np.abs(Wd - W) / step
        # rounding error <= half a step; the two roundings of zero and w/scale
        # can push a group extreme one code past the range, where it clips
        assert err.max() <= 1.0 + 1e-3
        assert np.mean(err <= 0.5 + 1e-3) > 0.99
    p4, s4, z4 = qo.quantize_int4_grouped(W, 128)
    assert p4.shape == (16, 192)
    np.testing.assert_array_equal(qo.dequant_int4_grouped(p4, s4, z4, 384, 128),
                                  qo.dequant_int_grouped(qo.unpack_nibbles(p4, 384), s4, z4, 384,
                                                         128))


def test_int4_per_row_reduces_to_reference_layout():
    """group == K is the reference's per-row int4 (lora_quantized.metal:64-65)."""
    rng = np.random.default_rng(2)
    W = rng.standard_normal((4, 64)).astype(np.float32)
    p, s, z = qo.quantize_int4_grouped(W, 64)
    assert s.shape == (4, 1)
    q = qo.unpack_nibbles(p, 64)
    ref_style = (q.astype(np.float32) - z.astype(np.float32)) * s.astype(np.float32)
    np.testing.assert_array_equal(ref_style, qo.dequant_int4_grouped(p, s, z, 64, 64))
