"""GPU parity of the operator entry points, through the C ABI, against the
CPU oracle (oracle/) on the same seeded inputs.

Bars (written per test): bit-exact for Q8_0 quantisation, int32 block dots
and the Q8_0 f32 sums (the kernel keeps the reference's rounding order), and
for the f32 projections / RoPE (same FMA chain and rounding); relative L2
for everything else: 1e-5 for f32 math, 1e-3 for bf16 math against the
oracle fed the same bf16-rounded operands.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def vk():
    import vestra_kernels

    return vestra_kernels


@pytest.fixture(scope="module")
def ctx(vk):
    c = vk.Context(0)
    yield c
    c.close()


def dev(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device="cuda", dtype=dtype)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def rng_inputs(seed, *shapes, scale=1.0):
    r = np.random.default_rng(seed)
    return [(r.standard_normal(s) * scale).astype(np.float32) for s in shapes]


# ---------------------------------------------------------------- Q8_0 (bit-exact)
def test_quantize_row_q8_0_bit_exact(vk, ctx, oracle_lib):
    (x,) = rng_inputs(11, (865, 768))
    x[3, :32] = 0.0                      # all-zero block: d = 0, inv = 0
    x[4, :32] = np.float32(1e-7)         # f16-subnormal scale
    nblocks = x.size // 32
    out = torch.zeros(nblocks * 34, dtype=torch.uint8, device="cuda")
    vk.quantize_row_q8_0(dev(x), out, ctx=ctx)
    got = host(out).view(oracle_lib.BLOCK_Q8_0)
    ref = oracle_lib.quantize_rows_q8_0(x.reshape(1, -1)).ravel()
    assert np.array_equal(got["d"], ref["d"])
    assert np.array_equal(got["qs"], ref["qs"])


@pytest.mark.parametrize("m,n,k", [(865, 768, 768), (130, 256, 3072), (1, 128, 128)])
def test_gemm_q8_0_block_dots_and_sums_bit_exact(vk, ctx, oracle_lib, m, n, k):
    a, w = rng_inputs(12 + k, (m, k), (n, k), scale=1.0)
    w *= np.float32(0.02)
    aq = oracle_lib.quantize_rows_q8_0(a)
    bq = oracle_lib.quantize_rows_q8_0(w)
    da = dev(aq.view(np.uint8).ravel(), torch.uint8)
    db = dev(bq.view(np.uint8).ravel(), torch.uint8)
    dots = torch.empty(m * n * (k // 32), dtype=torch.int32, device="cuda")
    assert vk.gemm_q8_0_block_dots(m, n, k, da, db, dots, ctx=ctx)
    assert np.array_equal(host(dots).reshape(m, n, k // 32), oracle_lib.q8_0_block_dots(m, n, k, aq, bq))
    c = torch.empty(m * n, dtype=torch.float32, device="cuda")
    assert vk.gemm_q8_0(m, n, k, da, db, c, ctx=ctx)
    ref = oracle_lib.gemm_q8_0(m, n, k, aq, bq)
    assert np.array_equal(host(c).reshape(m, n).view(np.uint32), ref.view(np.uint32))


def test_gemm_q8_0_rejects_unsupported_shape(vk, ctx):
    z = torch.zeros(34 * 16, dtype=torch.uint8, device="cuda")
    c = torch.zeros(64, dtype=torch.float32, device="cuda")
    assert not vk.gemm_q8_0(8, 8, 64, z, z, c, ctx=ctx)  # the reference test's (8, 8, 64)
    assert float(c.abs().sum()) == 0.0


def test_gemm_q8_0_empty_is_a_no_op(vk, ctx):
    z = torch.zeros(34 * 4, dtype=torch.uint8, device="cuda")
    c = torch.full((8,), 7.0, device="cuda")
    assert vk.gemm_q8_0(0, 128, 128, z, z, c, ctx=ctx)
    assert vk.gemm_q8_0(1, 0, 128, z, z, c, ctx=ctx)
    assert float(c.sum()) == 56.0


# ---------------------------------------------------------------- projections
SHAPES = [(768, 2304), (768, 768), (768, 3072), (3072, 768)]


@pytest.mark.parametrize("k,n", SHAPES)
def test_linear_f32_bit_exact(vk, ctx, oracle_lib, k, n):
    ctx.set_math(vk.MATH_F32)
    x, w = rng_inputs(20 + n, (865, k), (k, n))
    w *= np.float32(0.02)
    out = torch.empty(865 * n, device="cuda")
    assert vk.linear_f32_da3_base(865, n, k, dev(x), dev(w), out, ctx=ctx)
    ref = oracle_lib.linear_fma(x, w)
    assert np.array_equal(host(out).reshape(865, n), ref)


@pytest.mark.parametrize("k,n", SHAPES)
def test_linear_bf16_rel_l2(vk, ctx, oracle_lib, k, n):
    ctx.set_math(vk.MATH_BF16)
    try:
        x, w = rng_inputs(30 + n, (865, k), (k, n))
        w *= np.float32(0.02)
        out = torch.empty(865 * n, device="cuda")
        assert vk.linear_f32_da3_base(865, n, k, dev(x), dev(w), out, ctx=ctx)
        ref = oracle_lib.linear_fma(oracle_lib.round_bf16(x), oracle_lib.round_bf16(w))
        err = rel_l2(host(out).reshape(865, n), ref)
        assert err < 1e-3, err
        assert err < 1e-5, f"accumulation-order error only expected, got {err}"
    finally:
        ctx.set_math(vk.MATH_F32)


@pytest.mark.parametrize("math", ["f32", "bf16", "q8"])
@pytest.mark.parametrize("k", [768, 3072])
def test_linear_bias_scale(vk, ctx, oracle_lib, math, k):
    ctx.set_math({"f32": vk.MATH_F32, "bf16": vk.MATH_BF16, "q8": vk.MATH_Q8_0}[math])
    try:
        x, w, b, s = rng_inputs(40 + k, (865, k), (k, 768), (768,), (768,))
        w *= np.float32(0.02)
        b *= np.float32(0.01)
        out = torch.empty(865 * 768, device="cuda")
        assert vk.linear_bias_scale_f32_da3_base(865, 768, k, dev(x), dev(w), dev(b), dev(s), out, ctx=ctx)
        got = host(out).reshape(865, 768)
        if math == "f32":
            assert np.array_equal(got, oracle_lib.linear_bias_scale(x, w, b, s))
        elif math == "bf16":
            ref = oracle_lib.linear_bias_scale(oracle_lib.round_bf16(x), oracle_lib.round_bf16(w), b, s)
            assert rel_l2(got, ref) < 1e-3
        else:
            aq = oracle_lib.quantize_rows_q8_0(x)
            wq = oracle_lib.quantize_rows_q8_0(np.ascontiguousarray(w.T))
            acc = oracle_lib.gemm_q8_0(865, 768, k, aq, wq)
            ref = ((acc + b) * s).astype(np.float32)
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
            # and the quantised product stays close to the f32 one (tests/q8_0_dot_matches_f32.rs)
            assert rel_l2(got, oracle_lib.linear_bias_scale(x, w, b, s)) < 2e-2
    finally:
        ctx.set_math(vk.MATH_F32)


@pytest.mark.parametrize("math", ["f32", "bf16"])
@pytest.mark.parametrize("tokens", [865, 3457, 37])
def test_qkv_head_major(vk, ctx, oracle_lib, math, tokens):
    ctx.set_math(vk.MATH_F32 if math == "f32" else vk.MATH_BF16)
    try:
        x, w, b = rng_inputs(50 + tokens, (tokens, 768), (768, 2304), (2304,))
        w *= np.float32(0.02)
        b *= np.float32(0.01)
        q = torch.empty(12 * tokens * 64, device="cuda")
        k = torch.empty_like(q)
        v = torch.empty_like(q)
        assert vk.qkv_f32_da3_base(dev(x), dev(w), dev(b), q, k, v, ctx=ctx)
        if math == "f32":
            rq, rk, rv = oracle_lib.qkv(x, w, b, 12)
            for g, r in ((q, rq), (k, rk), (v, rv)):
                assert np.array_equal(host(g).reshape(12, tokens, 64), r)
        else:
            rq, rk, rv = oracle_lib.qkv(oracle_lib.round_bf16(x), oracle_lib.round_bf16(w), b, 12)
            for g, r in ((q, rq), (k, rk), (v, rv)):
                assert rel_l2(host(g).reshape(12, tokens, 64), r) < 1e-3
    finally:
        ctx.set_math(vk.MATH_F32)


def test_linear_rejects_non_da3_shape(vk, ctx):
    out = torch.zeros(10 * 100, device="cuda")
    assert not vk.linear_f32_da3_base(10, 100, 64, torch.zeros(640, device="cuda"), torch.zeros(6400, device="cuda"), out, ctx=ctx)
    assert float(out.abs().sum()) == 0.0


def test_dimensions_beyond_32_bits_are_rejected(vk, ctx):
    # The kernels index with 32-bit ints; the entry points refuse larger
    # dimensions before touching any buffer (the pointers are never read).
    import ctypes

    lib, big, dummy = vk.lib(), 1 << 31, ctypes.c_void_p(16)
    assert lib.vk_linear_f32_da3_base(ctx.handle, big, 768, 768, dummy, dummy, dummy) == vk.VK_UNSUPPORTED_SHAPE
    assert "32-bit" in vk.last_error()
    assert lib.vk_gemm_q8_0(ctx.handle, big, 128, 128, dummy, dummy, dummy) == vk.VK_UNSUPPORTED_SHAPE
    assert lib.vk_layernorm(ctx.handle, dummy, big, 768, dummy, dummy, ctypes.c_float(1e-6)) == vk.VK_UNSUPPORTED_SHAPE


def test_prepared_linear_chain_matches_reference_values(vk, ctx):
    """src/cuda.rs:1433-1447: two prepared linears run back to back (f32)."""
    import json
    import os

    with open(os.path.join(os.path.dirname(__file__), "golden", "reference_kat.json")) as fh:
        case = json.load(fh)["cuda.prepared_linear_chain"]
    f, g = case["first"], case["second"]
    first = vk.Linear(ctx, np.array(f["weight"], np.float32).reshape(f["k"], f["n"]), f["bias"], f["scale"],
                      math=vk.MATH_F32)
    second = vk.Linear(ctx, np.array(g["weight"], np.float32).reshape(g["k"], g["n"]), g["bias"], None,
                       math=vk.MATH_F32)
    mid = torch.empty(case["rows"] * f["n"], device="cuda")
    out = torch.empty(case["rows"] * g["n"], device="cuda")
    first(dev(np.array(case["left"], np.float32)), mid)
    second(mid, out)
    assert host(out).tolist() == case["expected"]


def test_prepared_linear_matches_raw(vk, ctx, oracle_lib):
    x, w, b, s = rng_inputs(60, (300, 768), (768, 768), (768,), (768,))
    w *= np.float32(0.02)
    for math in (vk.MATH_F32, vk.MATH_BF16, vk.MATH_Q8_0):
        lin = vk.Linear(ctx, w, b, s, math=math)
        out = torch.empty(300 * 768, device="cuda")
        lin(dev(x), out)
        ref = oracle_lib.linear_bias_scale(x, w, b, s)
        tol = {vk.MATH_F32: 1e-6, vk.MATH_BF16: 1e-2, vk.MATH_Q8_0: 2e-2}[math]
        assert rel_l2(host(out).reshape(300, 768), ref) < tol


# ---------------------------------------------------------------- attention
def xorshift_qkv(heads, n, hd, seed):
    from conftest import xorshift32_values

    vals = xorshift32_values(3 * heads * n * hd, seed)
    return [vals[i * heads * n * hd:(i + 1) * heads * n * hd].reshape(heads, n, hd) for i in range(3)]


@pytest.mark.parametrize("heads,n,hd,seed", [(2, 8, 16, 0x12345678), (4, 37, 32, 0xDEADBEEF), (1, 130, 8, 0x0BADF00D)])
def test_attention_generic_matches_naive(vk, ctx, oracle_lib, heads, n, hd, seed):
    """tests/attention_matches_naive.rs cases, |diff| < 1e-4."""
    q, k, v = xorshift_qkv(heads, n, hd, seed)
    out = torch.empty(q.size, device="cuda")
    vk.attention(dev(q), dev(k), dev(v), heads, n, hd, out, ctx=ctx)
    ref = oracle_lib.attention_naive(q, k, v)
    assert np.abs(host(out).reshape(q.shape) - ref).max() < 1e-4


@pytest.mark.parametrize("tokens", [865, 2 * 865, 33, 1])
def test_flash_attention_f32(vk, ctx, oracle_lib, tokens):
    q, k, v = rng_inputs(70 + tokens, (12, tokens, 64), (12, tokens, 64), (12, tokens, 64))
    out = torch.empty(q.size, device="cuda")
    assert vk.flash_attention_f32_da3_base(dev(q), dev(k), dev(v), 12, tokens, out, ctx=ctx)
    got = host(out).reshape(q.shape)
    tiled = oracle_lib.attention(q, k, v)
    naive = oracle_lib.attention_naive(q, k, v)
    assert rel_l2(got, tiled) < 1e-5
    d = np.abs(got - naive)
    assert d.mean() <= 5e-5 and d.max() <= 5e-4  # src/cuda.rs:1613-1648 bounds


@pytest.mark.parametrize("tokens,heads", [(865, 12), (865, 48), (865, 75), (300, 101), (1000, 40), (3457, 2), (64, 3),
                                           (65, 1), (1, 2), (97, 301)])
def test_flash_attention_bf16(vk, ctx, oracle_lib, tokens, heads):
    """(865, 48), (865, 75), (300, 101), (97, 301): enough heads for tile
    pairs with an odd tile count per head, so the heads' last tiles pair up
    across heads (75, 101, 301: one left alone).  (865, 48) and (1000, 40):
    168 and 160 items on 148 CTAs, so the last round's items run as single
    tiles."""
    ctx.set_math(vk.MATH_BF16)
    try:
        q, k, v = (oracle_lib.round_bf16(t) for t in rng_inputs(80 + tokens, *[(heads, tokens, 64)] * 3))
        out = torch.empty(q.size, device="cuda")
        assert vk.flash_attention_f32_da3_base(dev(q), dev(k), dev(v), heads, tokens, out, ctx=ctx)
        got = host(out).reshape(q.shape)
        err = rel_l2(got, oracle_lib.attention_naive(q, k, v))
        print(f"bf16 attention tokens={tokens} rel_l2={err:.3e}")
        assert err < 2e-5  # P V as f16 P_hi + P_lo: about 22 bits of P
    finally:
        ctx.set_math(vk.MATH_F32)


@pytest.mark.parametrize("boost", [1.0, 40.0, 400.0])
@pytest.mark.parametrize("span", [(600, 610), (100, 105)])
@pytest.mark.parametrize("split", ["1", "0"])
def test_flash_attention_bf16_logit_jumps(vk, ctx, oracle_lib, boost, span, split, monkeypatch):
    """Keys whose logits exceed every earlier one by far (up to ~3000 in
    score units), in a late block or in block 0 past the 64 keys the first
    reference is taken from: the online softmax must re-reference its
    running maximum without overflowing.  Both kernels: split P (the
    operator's) and single f16 P (the bf16 encoder's, VK_ATT_API_SPLIT=0)."""
    monkeypatch.setenv("VK_ATT_API_SPLIT", split)
    ctx.set_math(vk.MATH_BF16)
    try:
        heads, tokens = 2, 865
        q, k, v = rng_inputs(91, *[(heads, tokens, 64)] * 3)
        k[:, span[0]:span[1]] *= np.float32(boost)  # a late block, or block 0's second half
        q, k, v = (oracle_lib.round_bf16(t) for t in (q, k, v))
        out = torch.empty(q.size, device="cuda")
        assert vk.flash_attention_f32_da3_base(dev(q), dev(k), dev(v), heads, tokens, out, ctx=ctx)
        got = host(out).reshape(q.shape)
        assert np.isfinite(got).all()
        err = rel_l2(got, oracle_lib.attention_naive(q, k, v))
        assert err < (2e-5 if split == "1" else 1e-3), err
    finally:
        ctx.set_math(vk.MATH_F32)


# ---------------------------------------------------------------- norms, RoPE, pointwise
@pytest.mark.parametrize("rows,cols", [(865, 768), (67, 64), (5, 100), (20011, 768), (33, 3072)])
def test_layernorm(vk, ctx, oracle_lib, rows, cols):
    x, g, b = rng_inputs(90 + cols, (rows, cols), (cols,), (cols,))
    t = dev(x)
    vk.layernorm(t, rows, cols, dev(g), dev(b), 1e-6, ctx=ctx)
    # bit-exact: the same ascending folds and separately rounded operations
    assert np.array_equal(host(t).reshape(rows, cols), oracle_lib.layernorm(x, g, b, 1e-6))


def test_rope2d_bit_exact(vk, ctx, oracle_lib):
    pos = oracle_lib.da3_positions(24, 36)
    (x,) = rng_inputs(100, (12, 865, 64))
    t = dev(x)
    vk.rope2d(t, 12, 865, 64, dev(pos, torch.int64), 100.0, ctx=ctx)
    assert np.array_equal(host(t).reshape(x.shape), oracle_lib.rope2d(x, pos, 100.0))
    # generic head_dim (src/rope.rs:132-154 case)
    pos2 = np.array([[i, 3 * i] for i in range(7)], np.int64)
    x2 = ((np.arange(3 * 7 * 16, dtype=np.float32) - np.float32(43.0)) * np.float32(0.0625)).reshape(3, 7, 16)
    t2 = dev(x2)
    vk.rope2d(t2, 3, 7, 16, dev(pos2, torch.int64), 100.0, ctx=ctx)
    assert np.array_equal(host(t2).reshape(x2.shape), oracle_lib.rope2d(x2, pos2, 100.0))


def test_rope2d_device_tables(vk, ctx, oracle_lib):
    """Rotations are built on the device from device positions (no host
    round trip): a 72-wide grid and a second frequency are bit-exact through
    the cached lookup table; positions outside it (negative, >= 4096) take
    double-precision sin / cos, within an ulp of the host's f32 functions;
    changed positions at the same address are picked up."""
    pos = oracle_lib.da3_positions(48, 72)
    (x,) = rng_inputs(101, (2, 3457, 64))
    for freq in (100.0, 10000.0):
        t = dev(x)
        vk.rope2d(t, 2, 3457, 64, dev(pos, torch.int64), freq, ctx=ctx)
        assert np.array_equal(host(t).reshape(x.shape), oracle_lib.rope2d(x, pos, freq))
    pd = dev(pos, torch.int64)
    pd += 3  # same buffer, new contents
    t = dev(x)
    vk.rope2d(t, 2, 3457, 64, pd, 100.0, ctx=ctx)
    assert np.array_equal(host(t).reshape(x.shape), oracle_lib.rope2d(x, pos + 3, 100.0))
    far = np.array([[-5, 4096], [70000, 12], [4095, -1]], np.int64)
    (x3,) = rng_inputs(102, (1, 3, 64))
    t3 = dev(x3)
    vk.rope2d(t3, 1, 3, 64, dev(far, torch.int64), 100.0, ctx=ctx)
    ref = oracle_lib.rope2d(x3, far, 100.0)
    assert np.abs(host(t3).reshape(x3.shape) - ref).max() <= 4e-7 * max(1.0, float(np.abs(x3).max())) * 4
    # head_dim above 128 (40 frequencies): the host-built table, bit-exact
    pos4 = oracle_lib.da3_positions(3, 5)
    (x4,) = rng_inputs(103, (2, 16, 160))
    t4 = dev(x4)
    vk.rope2d(t4, 2, 16, 160, dev(pos4, torch.int64), 100.0, ctx=ctx)
    assert np.array_equal(host(t4).reshape(x4.shape), oracle_lib.rope2d(x4, pos4, 100.0))


def test_qk_norm_rope(vk, ctx, oracle_lib):
    pos = oracle_lib.da3_positions(24, 36)
    q, k, g, b = rng_inputs(110, (12, 865, 64), (12, 865, 64), (64,), (64,))
    tq, tk = dev(q), dev(k)
    assert vk.qk_norm_rope_f32_da3_base(tq, tk, dev(g), dev(b), dev(g), dev(b), dev(pos.ravel(), torch.int64),
                                        100.0, 1e-6, ctx=ctx)
    rq, rk = oracle_lib.qk_norm_rope(q, k, g, b, g, b, pos, 100.0, 1e-6)
    assert np.array_equal(host(tq).reshape(q.shape), rq)
    assert np.array_equal(host(tk).reshape(k.shape), rk)


def test_gelu_add_bias_layerscale(vk, ctx, oracle_lib):
    x = np.arange(1000, dtype=np.float32) * np.float32(0.017) - np.float32(3.0)
    t = dev(x)
    vk.gelu(t, ctx=ctx)
    assert np.abs(host(t) - oracle_lib.gelu(x)).max() < 1e-6
    a, b2, bias, g = rng_inputs(120, (67, 64), (67, 64), (64,), (64,))
    ta = dev(a)
    vk.add(ta, dev(b2), ctx=ctx)
    assert np.array_equal(host(ta), oracle_lib.add(a, b2))
    vk.add_bias_rows(ta, 67, 64, dev(bias), ctx=ctx)
    vk.layerscale(ta, 67, 64, dev(g), ctx=ctx)
    assert np.array_equal(host(ta), oracle_lib.layerscale(oracle_lib.add_bias_rows(oracle_lib.add(a, b2), bias), g))
    # src/cuda.rs:1375-1381 known answer
    d = dev(np.array([1.0, -2.0, 3.5], np.float32))
    vk.add(d, dev(np.array([0.5, 2.0, -1.0], np.float32)), ctx=ctx)
    assert host(d).tolist() == [1.5, 0.0, 2.5]


@pytest.mark.parametrize("k,n", SHAPES)
def test_linear_bf16_pair_kernel_large_m(vk, ctx, k, n):
    """M large enough for the CTA-pair (256 x 256) kernel; torch fp32 matmul
    of the same bf16-rounded operands as reference (TF32 off)."""
    ctx.set_math(vk.MATH_BF16)
    try:
        m = 4096 + 37
        g = torch.Generator(device="cuda").manual_seed(n + k)
        x = torch.randn(m, k, device="cuda", generator=g)
        w = torch.randn(k, n, device="cuda", generator=g) * 0.02
        b = torch.randn(n, device="cuda", generator=g) * 0.01
        s = torch.randn(n, device="cuda", generator=g)
        out = torch.empty(m * n, device="cuda")
        torch.cuda.synchronize()  # ctx runs on its own stream
        assert vk.linear_f32_da3_base(m, n, k, x, w, out, ctx=ctx)
        ctx.synchronize()
        torch.backends.cuda.matmul.allow_tf32 = False
        ref = x.bfloat16().float() @ w.bfloat16().float()
        err = (out.view(m, n) - ref).norm() / ref.norm()
        assert float(err) < 1e-5, float(err)
        if n == 768:
            out2 = torch.empty(m * n, device="cuda")
            torch.cuda.synchronize()
            assert vk.linear_bias_scale_f32_da3_base(m, n, k, x, w, b, s, out2, ctx=ctx)
            ctx.synchronize()
            ref2 = (ref + b) * s
            assert float((out2.view(m, n) - ref2).norm() / ref2.norm()) < 1e-5
    finally:
        ctx.set_math(vk.MATH_F32)
