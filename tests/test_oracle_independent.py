"""An independent float64 restatement, written from the reference's Rust
source, of the oracle's ops that carry the GPU parity claims.  The oracle
(oracle/vk_oracle.c) reproduces the reference's f32 rounding sequence; these
checks pin it against the same mathematics computed without that code:

  layernorm_row            src/scalar.rs:99-113
  erf (A&S 7.1.26), gelu   src/scalar.rs:116-134
  quantize_row_q8_0        src/q8_0_dot.rs:27-46 (scale and block values)
  gemm_q8_0                src/scalar.rs:25-56
  rope rotation tables     src/specialized.rs:389-410, src/rope.rs:42-60
  attention_naive          src/attention.rs:10-59
  DA3 positions            src/specialized.rs:359-366

Bars are the f32 rounding the oracle carries (relative ~1e-6), not looser.
"""
import math

import numpy as np
import pytest


def rng(seed):
    return np.random.default_rng(seed)


def test_layernorm_float64(oracle_lib):
    x = (rng(1).standard_normal((67, 768)) * 3 + 0.5).astype(np.float32)
    g = (1 + 0.1 * rng(2).standard_normal(768)).astype(np.float32)
    b = (0.1 * rng(3).standard_normal(768)).astype(np.float32)
    xd = x.astype(np.float64)
    mean = xd.mean(axis=1, keepdims=True)
    var = ((xd - mean) ** 2).mean(axis=1, keepdims=True)
    ref = (xd - mean) / np.sqrt(var + 1e-6) * g + b
    got = oracle_lib.layernorm(x, g, b, 1e-6).astype(np.float64)
    assert np.abs(got - ref).max() < 2e-6 * np.abs(ref).max()


def as_erf64(x):
    """Abramowitz-Stegun 7.1.26 as src/scalar.rs:125-134 writes it, in float64."""
    s = np.sign(x)
    a = np.abs(x)
    t = 1.0 / (1.0 + 0.3275911 * a)
    poly = ((((1.061405429 * t - 1.453152027) * t) + 1.421413741) * t - 0.284496736) * t + 0.254829592
    return s * (1.0 - poly * t * np.exp(-a * a))


def test_erf_and_gelu_float64(oracle_lib):
    xs = np.linspace(-6, 6, 2401).astype(np.float32)
    got = np.array([oracle_lib.erf(float(v)) for v in xs])
    ref = as_erf64(xs.astype(np.float64))
    assert np.abs(got - ref).max() < 5e-7  # a few f32 ulps of the f32 evaluation
    # and A&S itself against the true erf: the published |error| < 1.5e-7
    true = np.array([math.erf(float(v)) for v in xs])
    assert np.abs(ref - true).max() < 1.5e-7
    g = oracle_lib.gelu(xs).astype(np.float64)
    xd = xs.astype(np.float64)
    gref = 0.5 * xd * (1 + as_erf64(xd / math.sqrt(2.0)))
    assert np.abs(g - gref).max() < 1e-6


def test_quantize_float64(oracle_lib):
    x = (rng(4).standard_normal((16, 256)) * 0.7).astype(np.float32)
    x[3, :32] = 0.0  # an all-zero block
    blocks = oracle_lib.quantize_rows_q8_0(x)
    xb = x.astype(np.float64).reshape(16, 8, 32)
    amax = np.abs(xb).max(axis=2)
    d = amax / 127.0
    got_d = blocks["d"].view(np.float16).astype(np.float64)
    # the stored scale is d rounded to f16 (relative 2^-11)
    assert np.all(np.abs(got_d - d) <= d * 2.0 ** -11 + 1e-12)
    # each quant is x / d rounded to the nearest integer, clamped to 127
    q = blocks["qs"].astype(np.float64)
    with np.errstate(divide="ignore", invalid="ignore"):
        ideal = np.where(d[..., None] > 0, xb / d[..., None], 0.0)
    assert np.all(np.abs(q - ideal) <= 0.5 + 1e-4)
    assert np.all(q[3, 0] == 0) and got_d[3, 0] == 0.0


def test_gemm_q8_0_float64(oracle_lib):
    m, n, k = 5, 7, 256
    a = oracle_lib.quantize_rows_q8_0(rng(5).standard_normal((m, k)).astype(np.float32))
    b = oracle_lib.quantize_rows_q8_0((rng(6).standard_normal((n, k)) * 0.02).astype(np.float32))
    got = oracle_lib.gemm_q8_0(m, n, k, a, b).astype(np.float64)
    da = a["d"].view(np.float16).astype(np.float64)
    db = b["d"].view(np.float16).astype(np.float64)
    qa = a["qs"].astype(np.float64)
    qb = b["qs"].astype(np.float64)
    isum = np.einsum("ibl,jbl->ijb", qa, qb)
    ref = np.einsum("ib,jb,ijb->ij", da, db, isum)
    assert np.abs(got - ref).max() < 1e-5 * np.abs(ref).max()


def test_rope_tables_float64(oracle_lib):
    pos = oracle_lib.da3_positions(48, 72)
    assert pos[0].tolist() == [0, 0] and pos[1].tolist() == [1, 1] and pos[72].tolist() == [1, 72]
    assert pos[73].tolist() == [2, 1] and pos[-1].tolist() == [48, 72]
    rot = oracle_lib.rope_rotations(pos, 100.0)  # [T, 2, 16, (sin, cos)]
    inv = 100.0 ** (-2.0 * np.arange(16) / 32.0)
    ang = pos[:, :, None].astype(np.float64) * inv[None, None, :]
    assert np.abs(rot[..., 0] - np.sin(ang)).max() < 2e-5  # f32 angle: |ang| <= 72 carries ~4e-6
    assert np.abs(rot[..., 1] - np.cos(ang)).max() < 2e-5


def test_attention_naive_float64(oracle_lib):
    heads, n, hd = 3, 130, 64
    q, k, v = (rng(7 + i).standard_normal((heads, n, hd)).astype(np.float32) for i in range(3))
    got = oracle_lib.attention_naive(q, k, v).astype(np.float64)
    s = np.einsum("hid,hjd->hij", q.astype(np.float64), k.astype(np.float64)) / math.sqrt(hd)
    p = np.exp(s - s.max(axis=2, keepdims=True))
    ref = np.einsum("hij,hjd->hid", p / p.sum(axis=2, keepdims=True), v.astype(np.float64))
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-6
