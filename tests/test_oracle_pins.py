"""Pins the CPU oracle against the reference's own known-answer tests.

The reference crate (Rust) cannot be built in this image, so the oracle is
pinned by (1) the hand-checked values and tolerance tests the reference
ships (cited per test), transcribed in tests/golden/reference_kat.json, and
(2) independent restatements (numpy float16 for the RNE half conversion,
math.erf for the A&S erf bound, an order-free numpy softmax attention).
"""
import json
import math
import os

import numpy as np
import pytest

from conftest import xorshift32_values

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_kat.json")


@pytest.fixture(scope="module")
def kat():
    with open(GOLDEN) as f:
        return json.load(f)


# ---- tests/scalar_ops.rs ------------------------------------------------

def test_gemm_2x2_identity(oracle_lib, kat):
    case = kat["scalar_ops.gemm_2x2_identity"]
    a = np.array(case["a"], np.float32).reshape(2, 2)
    i = np.array(case["identity"], np.float32).reshape(2, 2)
    assert oracle_lib.gemm_f32(a, i).ravel().tolist() == case["expected"]


def test_softmax_rows_sums_to_one(oracle_lib, kat):
    case = kat["scalar_ops.softmax_rows_sums_to_one"]
    x = oracle_lib.softmax_rows(np.array(case["x"], np.float32).reshape(2, 3))
    assert abs(x[0].sum() - 1) < 1e-6 and abs(x[1].sum() - 1) < 1e-6
    assert abs(x[1, 0] - 1.0 / 3.0) < 1e-6


def test_gelu_zero_and_large(oracle_lib):
    x = oracle_lib.gelu(np.array([0.0, 10.0, -10.0], np.float32))
    assert abs(x[0]) < 1e-6 and abs(x[1] - 10.0) < 1e-3 and abs(x[2]) < 1e-3


def test_layernorm_zero_mean(oracle_lib):
    x = oracle_lib.layernorm(np.array([[1, 2, 3, 4]], np.float32), np.ones(4), np.zeros(4), 1e-5)
    assert abs(x.mean()) < 1e-4


def test_layerscale_known_values(oracle_lib, kat):
    case = kat["scalar_ops.layerscale"]
    x = oracle_lib.layerscale(np.array(case["x"], np.float32).reshape(2, 3), np.array(case["gamma"], np.float32))
    assert x.ravel().tolist() == case["expected"]


# ---- src/cuda.rs:1399-1417 (hand-checked GEMM and bias/scale epilogue) ---

def test_cuda_module_gemm_and_bias_scale_values(oracle_lib, kat):
    case = kat["cuda.gemm_bias_scale"]
    a = np.array(case["left"], np.float32).reshape(2, 3)
    b = np.array(case["right"], np.float32).reshape(3, 2)
    assert oracle_lib.gemm_f32(a, b).ravel().tolist() == case["product"]
    c = oracle_lib.linear_bias_scale(a, b, case["bias"], case["gamma"])
    assert c.ravel().tolist() == case["epilogue"]


def test_cuda_module_prepared_linear_chain(oracle_lib, kat):
    case = kat["cuda.prepared_linear_chain"]
    left = np.array(case["left"], np.float32).reshape(case["rows"], -1)
    f, g = case["first"], case["second"]
    h = oracle_lib.linear_bias_scale(left, np.array(f["weight"], np.float32).reshape(f["k"], f["n"]), f["bias"],
                                     f["scale"])
    out = oracle_lib.linear_bias_scale(h, np.array(g["weight"], np.float32).reshape(g["k"], g["n"]), g["bias"],
                                       np.ones(g["n"], np.float32))
    assert out.ravel().tolist() == case["expected"]


def test_cuda_module_patchify_values(oracle_lib, kat):
    case = kat["cuda.patchify_nchw"]
    image = np.arange(48, dtype=np.float32)
    got = oracle_lib.patchify_nchw(image, case["height"], case["width"], case["patch"], case["channels"])
    assert got.ravel().tolist() == case["expected"]


@pytest.mark.parametrize("h,w,p,c", [(5, 4, 2, 3), (4, 4, 0, 3), (0, 4, 2, 3), (4, 6, 4, 1)])
def test_patchify_rejects_invalid_shapes(oracle_lib, h, w, p, c):
    with pytest.raises(ValueError):
        oracle_lib.patchify_nchw(np.zeros(max(c * h * w, 1), np.float32), h, w, p, c)


def test_cuda_module_prepend_cls_add_pos_values(oracle_lib, kat):
    case = kat["cuda.prepend_cls_add_pos"]
    got = oracle_lib.prepend_cls_add_pos(case["patches"], case["cls"], case["position"], case["tokens"],
                                         case["channels"])
    assert got.ravel().tolist() == case["expected"]


# ---- tests/attention_matches_naive.rs -----------------------------------

@pytest.mark.parametrize("heads,n,hd,seed", [(2, 8, 16, 0x12345678), (4, 37, 32, 0xDEADBEEF), (1, 130, 8, 0x0BADF00D)])
def test_attention_tiled_matches_naive(oracle_lib, heads, n, hd, seed):
    vals = xorshift32_values(3 * heads * n * hd, seed)
    q, k, v = (vals[i * heads * n * hd:(i + 1) * heads * n * hd].reshape(heads, n, hd) for i in range(3))
    naive = oracle_lib.attention_naive(q, k, v)
    tiled = oracle_lib.attention(q, k, v)
    assert np.abs(naive - tiled).max() < 1e-4
    # independent float64 softmax restatement
    s = np.einsum("hid,hjd->hij", q.astype(np.float64), k.astype(np.float64)) / math.sqrt(hd)
    p = np.exp(s - s.max(-1, keepdims=True))
    ref = np.einsum("hij,hjd->hid", p / p.sum(-1, keepdims=True), v.astype(np.float64))
    assert np.abs(naive - ref).max() < 1e-5


# ---- tests/q8_0_dot_matches_f32.rs --------------------------------------

def test_q8_0_gemm_close_to_f32(oracle_lib):
    m, n, k = 8, 8, 64
    a = ((np.arange(m * k) % 17).astype(np.float32) - 8.0) * np.float32(0.1)
    b = ((np.arange(k * n) % 13).astype(np.float32) - 6.0) * np.float32(0.1)
    a = a.reshape(m, k)
    b = b.reshape(k, n)
    aq = oracle_lib.quantize_rows_q8_0(a)
    bq = oracle_lib.quantize_rows_q8_0(np.ascontiguousarray(b.T))
    c = oracle_lib.gemm_q8_0(m, n, k, aq, bq)
    a_de = oracle_lib.dequantize_q8_0(aq)
    b_de = oracle_lib.dequantize_q8_0(bq).T
    c_ref = oracle_lib.gemm_f32(a_de, np.ascontiguousarray(b_de))
    assert np.all(np.abs(c - c_ref) < 1e-2 + 1e-2 * np.abs(c_ref))


def _quantize_numpy(x):
    """Independent numpy restatement of src/q8_0_dot.rs:34-45."""
    x = x.reshape(-1, 32).astype(np.float32)
    amax = np.abs(x).max(1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    y = (x * inv[:, None]).astype(np.float32)
    q = np.sign(y) * np.floor(np.abs(y) + 0.5)  # half away from zero, exact in f64
    # floor(|y| + 0.5) in float64 is exact for |y| < 2^52
    q = np.clip(q, -127, 127).astype(np.int8)
    return d.astype(np.float16).view(np.uint16), q


def test_quantize_matches_numpy_restatement(oracle_lib):
    rng = np.random.default_rng(7)
    x = np.concatenate([
        rng.standard_normal(32 * 200).astype(np.float32),
        (rng.standard_normal(32 * 50) * 1e-6).astype(np.float32),  # f16-subnormal scales
        np.zeros(32, np.float32),
        np.array([0.5, -0.5, 1.5, -2.5] * 8, np.float32) * np.float32(127 / 2.5),  # ties
    ])
    blocks = oracle_lib.quantize_rows_q8_0(x.reshape(1, -1))[0]
    d_ref, q_ref = _quantize_numpy(x)
    assert np.array_equal(blocks["d"], d_ref)
    assert np.array_equal(blocks["qs"], q_ref)


def test_f16_rne_matches_numpy(oracle_lib):
    rng = np.random.default_rng(3)
    vals = np.concatenate([
        rng.standard_normal(2000).astype(np.float32) * 10,
        rng.standard_normal(2000).astype(np.float32) * 1e-5,
        np.array([65504, 65520, 65519.996, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8, 0.0, -0.0, np.inf, -np.inf], np.float32),
    ])
    # exact ties at the f16 mantissa boundary
    ties = (np.arange(1, 200, dtype=np.float32) * np.float32(2.0 ** -11) + np.float32(1.0)).astype(np.float32)
    vals = np.concatenate([vals, ties])
    got = np.array([oracle_lib.f16_from_f32(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, vals.astype(np.float16).view(np.uint16))


# ---- src/scalar.rs:124-134 (erf bound), tests/simd_matches_scalar.rs ---

def test_erf_within_abramowitz_stegun_bound(oracle_lib):
    for x in np.linspace(-4, 4, 801):
        assert abs(oracle_lib.erf(float(x)) - math.erf(float(np.float32(x)))) < 1.5e-7 + 4e-7


def test_gelu_ramp_matches_exact_erf(oracle_lib):
    x = np.arange(1000, dtype=np.float32) * np.float32(0.017) - np.float32(3.0)
    got = oracle_lib.gelu(x)
    ref = np.array([0.5 * v * (1 + math.erf(v / math.sqrt(2))) for v in x.astype(np.float64)])
    assert np.abs(got - ref).max() < 1e-4


# ---- src/rope.rs:95-154, src/specialized.rs:3444-3470 --------------------

def test_rope2d_cached_matches_uncached_rotation(oracle_lib):
    heads, n, hd = 3, 7, 16
    pos = np.array([[i, 3 * i] for i in range(n)], np.int64)
    x = (np.arange(heads * n * hd, dtype=np.float32) - np.float32(43.0)) * np.float32(0.0625)
    x = x.reshape(heads, n, hd)
    got = oracle_lib.rope2d(x, pos, 100.0)
    # uncached restatement (src/rope.rs:98-127) in float32 with libm sin/cos
    import ctypes
    libm = ctypes.CDLL("libm.so.6")
    for fn in ("sinf", "cosf", "powf"):
        getattr(libm, fn).restype = ctypes.c_float
    libm.sinf.argtypes = libm.cosf.argtypes = [ctypes.c_float]
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    half, quarter = hd // 2, hd // 4
    inv = [libm.powf(100.0, float(np.float32(-2.0 * i) / np.float32(half))) for i in range(quarter)]
    ref = x.copy()
    for p in range(n):
        for h in range(heads):
            for axis in range(2):
                posf = np.float32(pos[p, axis])
                off = axis * half
                for i in range(quarter):
                    ang = float(posf * np.float32(inv[i]))
                    s, c = np.float32(libm.sinf(ang)), np.float32(libm.cosf(ang))
                    a, b = ref[h, p, off + i], ref[h, p, off + i + quarter]
                    ref[h, p, off + i] = a * c - b * s
                    ref[h, p, off + i + quarter] = b * c + a * s
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_rope_cls_token_unrotated_and_norm_preserved(oracle_lib):
    pos = oracle_lib.da3_positions(24, 36)
    assert pos.shape == (865, 2) and pos[0].tolist() == [0, 0]
    assert pos[1].tolist() == [1, 1] and pos[36].tolist() == [1, 36] and pos[37].tolist() == [2, 1]
    x = np.random.default_rng(1).standard_normal((2, 865, 64)).astype(np.float32)
    y = oracle_lib.rope2d(x, pos, 100.0)
    assert np.array_equal(y[:, 0], x[:, 0])
    assert np.allclose(np.linalg.norm(y, axis=-1), np.linalg.norm(x, axis=-1), rtol=1e-5)


def test_fused_qk_norm_rope_equals_separate_passes(oracle_lib):
    """src/specialized.rs:3403-3441: fused == LayerNorm then rope, bitwise."""
    rng = np.random.default_rng(5)
    pos = oracle_lib.da3_positions(24, 36)
    q = rng.standard_normal((12, 865, 64)).astype(np.float32)
    k = rng.standard_normal((12, 865, 64)).astype(np.float32)
    g = (0.5 + rng.random(64)).astype(np.float32)
    b = rng.standard_normal(64).astype(np.float32) * np.float32(0.1)
    fq, fk = oracle_lib.qk_norm_rope(q, k, g, b, g, b, pos, 100.0, 1e-6)
    sq = oracle_lib.rope2d(oracle_lib.layernorm(q.reshape(-1, 64), g, b, 1e-6).reshape(q.shape), pos, 100.0)
    assert np.array_equal(fq, sq)


def test_qkv_head_major_layout(oracle_lib):
    """Layout pin of src/cuda.rs:1523-1545 (split to [H,T,D])."""
    rng = np.random.default_rng(2)
    t, heads = 5, 2
    e = heads * 64
    x = rng.standard_normal((t, e)).astype(np.float32)
    w = rng.standard_normal((e, 3 * e)).astype(np.float32)
    b = rng.standard_normal(3 * e).astype(np.float32)
    q, k, v = oracle_lib.qkv(x, w, b, heads)
    full = x.astype(np.float64) @ w.astype(np.float64) + b
    for g, out in enumerate((q, k, v)):
        for h in range(heads):
            np.testing.assert_allclose(out[h], full[:, g * e + h * 64:g * e + (h + 1) * 64], rtol=1e-5, atol=1e-5)
