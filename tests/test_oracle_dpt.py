"""CPU pins of the oracle's DPT-consumer restatements (token_to_chw, the two
bilinear resizes, the Winograd F(2x2, 3x3) convolution) against the
reference's own known answers and properties (src/resample.rs:250-482,
src/conv.rs:1105-1590), on the reference tests' xorshift32 inputs."""
import numpy as np
import pytest

from conftest import xorshift32_values


def draws(seed, *sizes):
    """Consecutive random_vec draws from one Xorshift32 (the reference tests' rng)."""
    v = xorshift32_values(sum(sizes), seed)
    out, o = [], 0
    for n in sizes:
        out.append(v[o:o + n])
        o += n
    return out


def test_token_to_chw_is_a_transpose(oracle_lib):
    x = np.arange(6 * 5, dtype=np.float32).reshape(6, 5)
    np.testing.assert_array_equal(oracle_lib.token_to_chw(x, 6, 5), x.T)


def test_resize_hand_checked(oracle_lib):
    o = oracle_lib
    ident = np.arange(1, 10, dtype=np.float32).reshape(1, 3, 3)
    np.testing.assert_array_equal(o.bilinear_resize(ident, 3, 3), ident)  # bilinear_resize_identity_hand_checked
    np.testing.assert_array_equal(o.bilinear_resize(ident, 3, 3, True), ident)  # align_corners_identity
    up = o.bilinear_resize(np.array([[[10, 20]]], np.float32), 1, 4).ravel()  # upsample_2x_hand_checked
    np.testing.assert_allclose(up, [10.0, 12.5, 17.5, 20.0], atol=1e-6)
    ac = o.bilinear_resize(np.array([[[10, 20]]], np.float32), 1, 5, True).ravel()  # endpoints_are_exact
    assert ac[0] == 10.0 and ac[4] == 20.0
    np.testing.assert_allclose(ac, [10.0, 12.5, 15.0, 17.5, 20.0], atol=1e-6)
    one = o.bilinear_resize(np.array([[[5, 7, 9]]], np.float32), 1, 1, True)  # degenerate_output_size_one
    assert one.ravel()[0] == 5.0


def test_resize_conventions_differ(oracle_lib):
    (x,) = draws(0x2222AAAA, 2 * 4 * 4)
    x = x.reshape(2, 4, 4)
    a = oracle_lib.bilinear_resize(x, 7, 5, True)
    b = oracle_lib.bilinear_resize(x, 7, 5, False)
    assert np.any(np.abs(a - b) > 1e-4)


def test_conv2d_1x1_hand_checked(oracle_lib):
    x = np.arange(1, 13, dtype=np.float32).reshape(3, 2, 2)
    w = np.array([1, 0, 0, 0, 0, 1], np.float32).reshape(2, 3, 1, 1)
    out = oracle_lib.conv2d_naive(x, w, 1, 0, np.array([10.0, -1.0], np.float32))
    np.testing.assert_array_equal(out.ravel(), [11, 12, 13, 14, 8, 9, 10, 11])


def test_winograd_matches_direct(oracle_lib):
    # winograd_f2_matches_direct_3x3_oracle: (3, 5, 7, 9), bound 2e-5
    in_c, out_c, h, w = 3, 5, 7, 9
    x, wt, b = draws(0xF2F20001, in_c * h * w, out_c * in_c * 9, out_c)
    x = x.reshape(in_c, h, w)
    wt = wt.reshape(out_c, in_c, 3, 3)
    got = oracle_lib.conv3x3_winograd_f2(x, wt, b)
    want = oracle_lib.conv2d_naive(x, wt, 1, 1, b)
    assert np.abs(got - want).max() < 2e-5


def test_winograd_relu_and_fused_resize_are_bitwise(oracle_lib):
    o = oracle_lib
    in_c, out_c, h, w = 3, 5, 7, 9
    i = np.arange(in_c * h * w, dtype=np.float32)
    x = ((np.sin(i * np.float32(0.17)) - np.float32(0.4)) * np.float32(1.3)).astype(np.float32).reshape(in_c, h, w)
    wt = (np.cos(np.arange(out_c * in_c * 9, dtype=np.float32) * np.float32(0.11)) * np.float32(0.2)).astype(
        np.float32).reshape(out_c, in_c, 3, 3)
    b = (np.arange(out_c, dtype=np.float32) * np.float32(0.03) - np.float32(0.05)).astype(np.float32)
    np.testing.assert_array_equal(o.conv3x3_winograd_f2(x, wt, b, relu_input=True),
                                  o.conv3x3_winograd_f2(np.maximum(x, 0), wt, b))
    # fused_resize_align_corners_winograd_matches_materialized_route
    in_c, out_c, ih, iw, oh, ow = 16, 16, 7, 5, 11, 9
    x, add, wt, b = draws(0xF05E0001, in_c * ih * iw, in_c * oh * ow, out_c * in_c * 9, out_c)
    x = x.reshape(in_c, ih, iw)
    add = add.reshape(in_c, oh, ow)
    wt = wt.reshape(out_c, in_c, 3, 3)
    mat = o.bilinear_resize(x, oh, ow, True) + add
    np.testing.assert_array_equal(o.conv3x3_winograd_f2_resize_ac(x, oh, ow, add, wt, b),
                                  o.conv3x3_winograd_f2(mat, wt, b))
