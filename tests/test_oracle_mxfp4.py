"""Pins the oracle's MXFP4 codec and quantizer to the reference.

Known answers come from the reference's own tests:
engine/src/mxfp4.rs:51-65, engine/tests/mxfp4.rs:9-40 and :88-105,
python/tests/test_mxfp4.py:18-83.  Golden vectors come from running the
reference's python/quantize_mxfp4.py (tests/golden/make_golden.py).
"""
import numpy as np
import pytest

import oracle as O


def test_smallest_e8m0_scale_and_signed_zero_decode():
    # engine/src/mxfp4.rs:56-65
    packed = np.full(16, 0x82, np.uint8)
    scales = np.zeros(1, np.uint8)
    decoded = O.mxfp4_values(packed, scales, 0, 32)
    assert decoded.view(np.uint32)[0] == 0x0040_0000
    assert decoded.view(np.uint32)[1] == np.float32(-0.0).view(np.uint32)


def packed_weight():
    # engine/tests/mxfp4.rs:5-9: all 16 codes twice, scaled by 2^-1
    row = np.array([0x10, 0x32, 0x54, 0x76, 0x98, 0xBA, 0xDC, 0xFE], np.uint8)
    return O.Matrix(1, 32, packed=np.tile(row, 2), scales=np.array([126], np.uint8))


def test_matrix_multiply_decodes_nibbles_and_scales():
    # engine/tests/mxfp4.rs:11-33
    x = np.eye(32, dtype=np.float32)
    y = O.matmul_raw(packed_weight(), x)
    levels = [0.0, 0.25, 0.5, 0.75, 1.0, 1.5, 2.0, 3.0]
    expected = [(-levels[i % 8] if i % 16 >= 8 else levels[i % 8]) for i in range(32)]
    assert y.shape == (32, 1)
    np.testing.assert_array_equal(y[:, 0], np.array(expected, np.float32))


def test_invalid_quantized_storage_is_rejected():
    # engine/tests/mxfp4.rs:35-40 (Tensor::quantized -> Mxfp4::validate)
    assert O.mxfp4_validate(1, 31, np.zeros(16, np.uint8), np.array([127], np.uint8)) != 0
    assert O.mxfp4_validate(1, 32, np.zeros(15, np.uint8), np.array([127], np.uint8)) != 0
    assert O.mxfp4_validate(1, 32, np.zeros(16, np.uint8), np.array([255], np.uint8)) != 0
    assert O.mxfp4_validate(1, 32, np.zeros(16, np.uint8), np.array([254], np.uint8)) == 0


def test_matrix_rows_and_blocks_use_different_scales():
    # engine/tests/mxfp4.rs:88-105
    w = O.Matrix(2, 64, packed=np.full(64, 0x77, np.uint8),
                 scales=np.array([127, 126, 125, 124], np.uint8))
    x = np.zeros((3, 64), np.float32)
    x[0, 0] = 1.0
    x[1, 32] = 1.0
    x[2, 0] = 1.0
    x[2, 32] = 1.0
    y = O.matmul_raw(w, x)
    np.testing.assert_array_equal(y.reshape(-1), [6.0, 1.5, 3.0, 0.75, 9.0, 2.25])


# -- python/tests/test_mxfp4.py ------------------------------------------------

LEVELS = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)


def test_all_codes_round_trip_with_signed_zero():
    values = np.tile(np.concatenate([LEVELS, -LEVELS]), 2)[None, :]
    packed, scales = O.mxfp4_quantize(values)
    np.testing.assert_array_equal(packed[0, :8], [0x10, 0x32, 0x54, 0x76, 0x98, 0xBA, 0xDC, 0xFE])
    np.testing.assert_array_equal(scales, [[127]])
    actual = O.mxfp4_dequantize(packed, scales)
    np.testing.assert_array_equal(actual, values)
    np.testing.assert_array_equal(np.signbit(actual), np.signbit(values))


def test_midpoints_round_to_even_and_overflow_saturates():
    values = np.zeros((1, 32), np.float32)
    values[0, :8] = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0]
    packed, scales = O.mxfp4_quantize(values)
    np.testing.assert_array_equal(scales, [[127]])
    np.testing.assert_array_equal(O.mxfp4_dequantize(packed, scales)[0, :8], [0, 1, 1, 2, 2, 4, 4, 6])


def test_each_block_gets_its_own_scale():
    values = np.zeros((2, 64), np.float32)
    values[0, :32] = 6
    values[0, 32:] = -0.75
    packed, scales = O.mxfp4_quantize(values)
    np.testing.assert_array_equal(scales, [[127, 124], [0, 0]])
    np.testing.assert_array_equal(O.mxfp4_dequantize(packed, scales), values)


@pytest.mark.parametrize("invalid", [np.nan, np.inf, -np.inf])
def test_non_finite_weights_are_rejected(invalid):
    values = np.zeros((1, 32), np.float32)
    values[0, 1] = invalid
    with pytest.raises(ValueError, match="non-finite"):
        O.mxfp4_quantize(values)


def test_invalid_row_width_is_rejected():
    with pytest.raises(ValueError, match="divisible"):
        O.mxfp4_quantize(np.zeros((1, 31), np.float32))


# -- golden vectors from the reference quantizer ------------------------------


def golden_cases(golden_dir):
    data = np.load(golden_dir / "mxfp4_quantize.npz")
    names = sorted({k.split(".")[0] for k in data.files})
    return data, names


def test_quantize_matches_reference_bit_exact(golden_dir):
    data, names = golden_cases(golden_dir)
    assert len(names) >= 10
    for name in names:
        packed, scales = O.mxfp4_quantize(data[f"{name}.values"])
        np.testing.assert_array_equal(packed, data[f"{name}.packed"], err_msg=name)
        np.testing.assert_array_equal(scales, data[f"{name}.scales"], err_msg=name)


def test_decode_matches_reference_dequantize_bit_exact(golden_dir):
    data, names = golden_cases(golden_dir)
    for name in names:
        ours = O.mxfp4_dequantize(data[f"{name}.packed"], data[f"{name}.scales"])
        ref = data[f"{name}.dequantized"]
        np.testing.assert_array_equal(ours.view(np.uint32), ref.view(np.uint32), err_msg=name)
