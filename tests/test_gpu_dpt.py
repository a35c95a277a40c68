"""GPU parity of the DPT head's consumers of the encoder output, through the C
ABI, against the CPU oracle and the reference's own known answers.

Bars: bit-exact for token_to_chw and both bilinear resizes (data movement and
the reference's f32 operations in its order); for the Winograd convolution,
1e-5 relative L2 (and the reference's 2e-5 absolute bound against direct
convolution) -- the transform-domain sums use fused multiply-adds where the
scalar fallback rounds each product -- and bit-exact for the reference's two
bitwise properties (ReLU input == materialised ReLU; fused resize + add ==
the materialised route).
"""
import numpy as np
import pytest

from conftest import xorshift32_values

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def draws(seed, *sizes):
    v = xorshift32_values(sum(sizes), seed)
    out, o = [], 0
    for n in sizes:
        out.append(v[o:o + n])
        o += n
    return out


@pytest.fixture(scope="module")
def vk():
    import vestra_kernels

    return vestra_kernels


@pytest.fixture(scope="module")
def ctx(vk):
    c = vk.Context(0)
    yield c
    c.close()


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("tokens,channels", [(864, 768), (37, 50), (1, 1), (3456, 96)])
def test_token_to_chw_bitexact(vk, ctx, oracle_lib, tokens, channels):
    x = np.random.default_rng(tokens).standard_normal((tokens, channels)).astype(np.float32)
    out = torch.empty(channels * tokens, device="cuda")
    vk.token_to_chw_f32(dev(x), tokens, channels, out, ctx=ctx)
    np.testing.assert_array_equal(host(out).reshape(channels, tokens), oracle_lib.token_to_chw(x, tokens, channels))


def test_token_to_chw_rejects_empty(vk, ctx):
    t = torch.empty(4, device="cuda")
    with pytest.raises(vk.VestraError):
        vk.token_to_chw_f32(t, 0, 4, t, ctx=ctx)


RESIZE_CASES = [(3, 5, 7, 9, 4, 0xABCD1234), (2, 16, 16, 5, 5, 0x13579BDF), (2, 4, 4, 7, 5, 0x2222AAAA),
                (3, 5, 7, 9, 4, 0x99995555), (128, 96, 144, 192, 288, 7), (64, 192, 288, 336, 504, 8),
                (4, 1, 3, 1, 1, 9), (5, 3, 1, 6, 2, 10)]


@pytest.mark.parametrize("ac", [False, True])
@pytest.mark.parametrize("c,ih,iw,oh,ow,seed", RESIZE_CASES)
def test_bilinear_resize_bitexact(vk, ctx, oracle_lib, ac, c, ih, iw, oh, ow, seed):
    (x,) = draws(seed, c * ih * iw) if c * ih * iw < 100000 else (
        np.random.default_rng(seed).standard_normal(c * ih * iw).astype(np.float32),)
    x = x.reshape(c, ih, iw)
    out = torch.empty(c * oh * ow, device="cuda")
    fn = vk.bilinear_resize_align_corners if ac else vk.bilinear_resize
    fn(dev(x), c, ih, iw, oh, ow, out, ctx=ctx)
    np.testing.assert_array_equal(host(out).reshape(c, oh, ow), oracle_lib.bilinear_resize(x, oh, ow, ac))


def test_resize_hand_checked(vk, ctx):
    out = torch.empty(4, device="cuda")
    vk.bilinear_resize(dev([10.0, 20.0]), 1, 1, 2, 1, 4, out, ctx=ctx)
    np.testing.assert_allclose(host(out), [10.0, 12.5, 17.5, 20.0], atol=1e-6)
    out = torch.empty(5, device="cuda")
    vk.bilinear_resize_align_corners(dev([10.0, 20.0]), 1, 1, 2, 1, 5, out, ctx=ctx)
    r = host(out)
    assert r[0] == 10.0 and r[4] == 20.0
    np.testing.assert_allclose(r, [10.0, 12.5, 15.0, 17.5, 20.0], atol=1e-6)
    ident = dev(np.arange(1, 10))
    out = torch.empty(9, device="cuda")
    vk.bilinear_resize(ident, 1, 3, 3, 3, 3, out, ctx=ctx)
    np.testing.assert_array_equal(host(out), np.arange(1, 10, dtype=np.float32))
    out = torch.full((1,), -1.0, device="cuda")
    vk.bilinear_resize_align_corners(dev([5.0, 7.0, 9.0]), 1, 1, 3, 1, 1, out, ctx=ctx)
    assert host(out)[0] == 5.0
    # zero sizes are a no-op, as the reference's early return
    keep = torch.full((3,), 7.0, device="cuda")
    vk.bilinear_resize(dev([1.0, 2.0, 3.0]), 1, 1, 3, 0, 3, keep, ctx=ctx)
    assert (host(keep) == 7.0).all()


def conv_inputs(seed, in_c, out_c, h, w, rng_kind="xorshift"):
    if rng_kind == "xorshift":
        x, wt, b = draws(seed, in_c * h * w, out_c * in_c * 9, out_c)
    else:
        r = np.random.default_rng(seed)
        x = r.standard_normal(in_c * h * w).astype(np.float32)
        wt = (r.standard_normal(out_c * in_c * 9) * 0.05).astype(np.float32)
        b = (r.standard_normal(out_c) * 0.1).astype(np.float32)
    return x.reshape(in_c, h, w), wt.reshape(out_c, in_c, 3, 3), b


CONV_CASES = [(3, 5, 7, 9, "xorshift"), (16, 16, 11, 9, "xorshift"), (20, 40, 13, 6, "normal"),
              (128, 128, 48, 72, "normal"), (64, 32, 96, 144, "normal"), (1, 1, 1, 1, "normal"),
              (33, 7, 2, 65, "normal")]


@pytest.mark.parametrize("in_c,out_c,h,w,kind", CONV_CASES)
def test_conv3x3_matches_oracle(vk, ctx, oracle_lib, in_c, out_c, h, w, kind):
    x, wt, b = conv_inputs(0xF2F20001 if kind == "xorshift" else in_c * 131 + h, in_c, out_c, h, w, kind)
    f = vk.WinogradF2Filter(ctx, wt, in_c, out_c)
    out = torch.empty(out_c * h * w, device="cuda")
    vk.conv3x3_winograd_f2_prepared(dev(x), in_c, h, w, f, out_c, dev(b), out, ctx=ctx)
    got = host(out).reshape(out_c, h, w)
    want = oracle_lib.conv3x3_winograd_f2(x, wt, b)
    assert rel_l2(got, want) <= 1e-5
    if in_c * out_c * h * w <= 64 * 32 * 96 * 144:
        direct = oracle_lib.conv2d_naive(x, wt, 1, 1, b)
        scale = max(1.0, float(np.abs(direct).max()))
        assert np.abs(got - direct).max() < 2e-5 * scale  # winograd_f2_matches_direct_3x3_oracle


def test_conv3x3_no_bias_and_relu_bitwise(vk, ctx, oracle_lib):
    in_c, out_c, h, w = 3, 5, 7, 9
    i = np.arange(in_c * h * w, dtype=np.float32)
    x = ((np.sin(i * np.float32(0.17)) - np.float32(0.4)) * np.float32(1.3)).astype(np.float32).reshape(in_c, h, w)
    wt = (np.cos(np.arange(out_c * in_c * 9, dtype=np.float32) * np.float32(0.11)) * np.float32(0.2)).astype(
        np.float32)
    b = (np.arange(out_c, dtype=np.float32) * np.float32(0.03) - np.float32(0.05)).astype(np.float32)
    f = vk.WinogradF2Filter(ctx, wt, in_c, out_c)
    relu = torch.empty(out_c * h * w, device="cuda")
    mat = torch.empty_like(relu)
    vk.conv3x3_winograd_f2_prepared(dev(x), in_c, h, w, f, out_c, dev(b), relu, relu_input=True, ctx=ctx)
    vk.conv3x3_winograd_f2_prepared(dev(np.maximum(x, 0)), in_c, h, w, f, out_c, dev(b), mat, ctx=ctx)
    # winograd_relu_input_matches_materialized_relu_bitwise
    np.testing.assert_array_equal(host(relu).view(np.uint32), host(mat).view(np.uint32))
    nob = torch.empty_like(relu)
    vk.conv3x3_winograd_f2_prepared(dev(x), in_c, h, w, f, out_c, None, nob, ctx=ctx)
    assert rel_l2(host(nob).reshape(out_c, h, w), oracle_lib.conv3x3_winograd_f2(x, wt.reshape(out_c, in_c, 3, 3))) \
        <= 1e-5


@pytest.mark.parametrize("in_c,out_c,ih,iw,oh,ow,with_add", [(16, 16, 7, 5, 11, 9, True),
                                                              (64, 32, 48, 72, 84, 126, True),
                                                              (8, 8, 5, 5, 5, 5, False)])
def test_fused_resize_conv(vk, ctx, oracle_lib, in_c, out_c, ih, iw, oh, ow, with_add):
    x, add, wt, b = draws(0xF05E0001, in_c * ih * iw, in_c * oh * ow, out_c * in_c * 9, out_c)
    x = x.reshape(in_c, ih, iw)
    add = add.reshape(in_c, oh, ow)
    wt = wt.reshape(out_c, in_c, 3, 3)
    f = vk.WinogradF2Filter(ctx, wt, in_c, out_c)
    fused = torch.empty(out_c * oh * ow, device="cuda")
    vk.conv3x3_winograd_f2_prepared_resize_align_corners(dev(x), in_c, ih, iw, oh, ow, dev(add) if with_add else None,
                                                         f, out_c, dev(b), fused, ctx=ctx)
    # the materialised route on the GPU: resize, add, convolve
    rs = torch.empty(in_c * oh * ow, device="cuda")
    vk.bilinear_resize_align_corners(dev(x), in_c, ih, iw, oh, ow, rs, ctx=ctx)
    if with_add:
        rs += dev(add).reshape(-1)
    mat = torch.empty_like(fused)
    vk.conv3x3_winograd_f2_prepared(rs, in_c, oh, ow, f, out_c, dev(b), mat, ctx=ctx)
    # fused_resize_align_corners_winograd_matches_materialized_route
    np.testing.assert_array_equal(host(fused).view(np.uint32), host(mat).view(np.uint32))
    want = oracle_lib.conv3x3_winograd_f2_resize_ac(x, oh, ow, add if with_add else None, wt, b)
    assert rel_l2(host(fused).reshape(out_c, oh, ow), want) <= 1e-5


def test_conv3x3_batched_equals_single(vk, ctx):
    in_c, out_c, h, w, n = 24, 40, 17, 23, 3
    x, wt, b = conv_inputs(5, in_c * n, out_c, h, w, "normal")
    wt = wt[:, :in_c].copy()
    f = vk.WinogradF2Filter(ctx, wt, in_c, out_c)
    xs = dev(x)
    batched = torch.empty(n * out_c * h * w, device="cuda")
    vk.conv3x3_batched(xs, n, h, w, f, dev(b), batched, ctx=ctx)
    for i in range(n):
        one = torch.empty(out_c * h * w, device="cuda")
        vk.conv3x3_winograd_f2_prepared(xs[i * in_c:(i + 1) * in_c], in_c, h, w, f, out_c, dev(b), one, ctx=ctx)
        np.testing.assert_array_equal(host(batched)[i * out_c * h * w:(i + 1) * out_c * h * w], host(one))


def test_conv3x3_rejects_mismatched_channels(vk, ctx):
    f = vk.WinogradF2Filter(ctx, np.zeros(2 * 3 * 9, np.float32), 3, 2)
    t = torch.zeros(3 * 4 * 4, device="cuda")
    o = torch.zeros(2 * 4 * 4, device="cuda")
    with pytest.raises(vk.VestraError):
        vk.conv3x3_winograd_f2_prepared(t, 4, 4, 4, f, 2, None, o, ctx=ctx)


def test_token_to_chw_batched(vk, ctx, oracle_lib):
    n, tokens, channels = 3, 100, 70
    x = np.random.default_rng(1).standard_normal((n, tokens, channels)).astype(np.float32)
    out = torch.empty(n * channels * tokens, device="cuda")
    vk.token_to_chw_batched(dev(x), n, tokens, channels, out, ctx=ctx)
    got = host(out).reshape(n, channels, tokens)
    for i in range(n):
        np.testing.assert_array_equal(got[i], oracle_lib.token_to_chw(x[i], tokens, channels))


# bf16 math: the 16 transform-domain products on the tensor cores (V and U
# rounded to bf16, f32 accumulation).  Bar: 1e-2 relative L2 against the f32
# oracle, the precision class of the encoder's bf16 math.
BF16_BAR = 1e-2


@pytest.mark.parametrize("in_c,out_c,h,w", [(3, 5, 7, 9), (16, 16, 11, 9), (20, 40, 13, 6), (128, 128, 48, 72),
                                            (64, 32, 96, 144), (33, 7, 2, 65), (1, 1, 1, 1), (48, 96, 33, 130)])
def test_conv3x3_bf16_matches_oracle(vk, ctx, oracle_lib, in_c, out_c, h, w):
    x, wt, b = conv_inputs(in_c * 7 + w, in_c, out_c, h, w, "normal")
    f = vk.WinogradF2Filter(ctx, wt, in_c, out_c, math=vk.MATH_BF16)
    out = torch.empty(out_c * h * w, device="cuda")
    vk.conv3x3_winograd_f2_prepared(dev(x), in_c, h, w, f, out_c, dev(b), out, ctx=ctx)
    assert rel_l2(host(out).reshape(out_c, h, w), oracle_lib.conv3x3_winograd_f2(x, wt, b)) <= BF16_BAR


def test_conv3x3_bf16_relu_fused_and_batched(vk, ctx, oracle_lib):
    in_c, out_c, ih, iw, oh, ow, n = 24, 40, 17, 23, 30, 41, 3
    r = np.random.default_rng(11)
    x = r.standard_normal((n, in_c, ih, iw)).astype(np.float32)
    add = r.standard_normal((in_c, oh, ow)).astype(np.float32)
    wt = (r.standard_normal((out_c, in_c, 3, 3)) * 0.05).astype(np.float32)
    b = (r.standard_normal(out_c) * 0.1).astype(np.float32)
    f = vk.WinogradF2Filter(ctx, wt, in_c, out_c, math=vk.MATH_BF16)
    relu = torch.empty(n * out_c * ih * iw, device="cuda")
    vk.conv3x3_batched(dev(x), n, ih, iw, f, dev(b), relu, relu_input=True, ctx=ctx)
    fused = torch.empty(n * out_c * oh * ow, device="cuda")
    vk.conv3x3_batched(dev(x), n, ih, iw, f, dev(b), fused, resize_to=(oh, ow), add=dev(add), ctx=ctx)
    relu_h = host(relu).reshape(n, out_c, ih, iw)
    fused_h = host(fused).reshape(n, out_c, oh, ow)
    for i in range(n):
        assert rel_l2(relu_h[i], oracle_lib.conv3x3_winograd_f2(x[i], wt, b, relu_input=True)) <= BF16_BAR
        assert rel_l2(fused_h[i], oracle_lib.conv3x3_winograd_f2_resize_ac(x[i], oh, ow, add, wt, b)) <= BF16_BAR
