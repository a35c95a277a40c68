"""GPU parity of the patch embedding and token assembly (the step before the
encoder), through the C ABI, against the reference's own values
(tests/golden, src/cuda.rs:1576-1605) and the CPU oracle.

Bars: bit-exact for patchify and the cls / position assembly (data movement
and one f32 add, as the reference kernels); bit-exact for the f32 patch
embedding (ascending-K FMA projection + bias, as the f32 operators); 1e-3
relative L2 for the bf16 embedding against the oracle fed bf16-rounded
operands.
"""
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_kat.json")


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


@pytest.fixture(scope="module")
def kat():
    with open(GOLDEN) as f:
        return json.load(f)


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def test_patchify_matches_reference_values(vk, ctx, kat):
    case = kat["cuda.patchify_nchw"]
    out = torch.empty(len(case["expected"]), device="cuda")
    vk.patchify_nchw_f32(dev(np.arange(48)), case["height"], case["width"], case["patch"], case["channels"], out,
                         ctx=ctx)
    assert host(out).tolist() == case["expected"]


def test_prepend_cls_add_pos_matches_reference_values(vk, ctx, kat):
    case = kat["cuda.prepend_cls_add_pos"]
    out = torch.empty(len(case["expected"]), device="cuda")
    vk.prepend_cls_add_pos_f32(dev(case["patches"]), dev(case["cls"]), dev(case["position"]), case["tokens"],
                               case["channels"], out, ctx=ctx)
    assert host(out).tolist() == case["expected"]


@pytest.mark.parametrize("h,w,p,c", [(336, 504, 14, 3), (28, 42, 14, 1), (6, 4, 2, 5)])
def test_patchify_bit_exact_with_oracle(vk, ctx, oracle_lib, h, w, p, c):
    img = np.random.default_rng(h + w).standard_normal((c, h, w)).astype(np.float32)
    out = torch.empty((h // p) * (w // p) * c * p * p, device="cuda")
    vk.patchify_nchw_f32(dev(img), h, w, p, c, out, ctx=ctx)
    assert np.array_equal(host(out).reshape((h // p) * (w // p), -1), oracle_lib.patchify_nchw(img, h, w, p, c))


def test_patchify_rejects_invalid_shape(vk, ctx):
    img = torch.zeros(3 * 30 * 42, device="cuda")
    out = torch.zeros(3 * 30 * 42, device="cuda")
    with pytest.raises(vk.VestraError):
        vk.patchify_nchw_f32(img, 30, 42, 14, 3, out, ctx=ctx)  # 30 is not a multiple of 14
    assert float(out.abs().sum()) == 0.0


def test_prepend_bit_exact_with_oracle(vk, ctx, oracle_lib):
    r = np.random.default_rng(5)
    n, e = 864, 768
    patches, cls, pos = r.standard_normal((n, e)), r.standard_normal(e), r.standard_normal((n + 1, e))
    out = torch.empty((n + 1) * e, device="cuda")
    vk.prepend_cls_add_pos_f32(dev(patches), dev(cls), dev(pos), n, e, out, ctx=ctx)
    assert np.array_equal(host(out).reshape(n + 1, e), oracle_lib.prepend_cls_add_pos(patches, cls, pos, n, e))


def reference_embedding(oracle_lib, images, w, b, cls, pos, patch, round_bf16=False):
    """patchify -> [K, E] projection + bias -> [cls; .] + position, per image."""
    out = []
    c, h, wd = images.shape[1:]
    n = (h // patch) * (wd // patch)
    ww = oracle_lib.round_bf16(w) if round_bf16 else w
    for img in images:
        p = oracle_lib.patchify_nchw(img, h, wd, patch, c)
        if round_bf16:
            p = oracle_lib.round_bf16(p)
        proj = oracle_lib.linear_bias_scale(p, ww, b, np.ones(w.shape[1], np.float32))
        out.append(oracle_lib.prepend_cls_add_pos(proj, cls, pos, n, w.shape[1]))
    return np.stack(out)


def embedding_inputs(images, h, w, c=3, p=14, e=768, seed=7):
    r = np.random.default_rng(seed)
    n = (h // p) * (w // p)
    imgs = r.random((images, c, h, w), dtype=np.float32)
    wt = (r.standard_normal((c * p * p, e)) * 0.02).astype(np.float32)
    b = (r.standard_normal(e) * 0.01).astype(np.float32)
    cls = (r.standard_normal(e) * 0.02).astype(np.float32)
    pos = (r.standard_normal((n + 1, e)) * 0.02).astype(np.float32)
    return imgs, wt, b, cls, pos, n


def test_patch_embed_f32_bit_exact(vk, ctx, oracle_lib):
    h, w = 336, 504
    imgs, wt, b, cls, pos, n = embedding_inputs(2, h, w)
    pe = vk.PatchEmbed(ctx, wt, b, cls, channels=3, patch=14, math=vk.MATH_F32)
    out = torch.empty((2, n + 1, 768), device="cuda")
    assert pe(dev(imgs), dev(pos), out, 2, h, w)
    ref = reference_embedding(oracle_lib, imgs, wt, b, cls, pos, 14)
    assert np.array_equal(host(out), ref)


@pytest.mark.parametrize("images,h,w", [(3, 336, 504), (1, 28, 70), (3, 98, 140), (5, 112, 168)])
def test_patch_embed_bf16(vk, ctx, oracle_lib, images, h, w):
    imgs, wt, b, cls, pos, n = embedding_inputs(images, h, w, seed=images + h)
    pe = vk.PatchEmbed(ctx, wt, b, cls, channels=3, patch=14, math=vk.MATH_BF16)
    out = torch.empty((images, n + 1, 768), device="cuda")
    assert pe(dev(imgs), dev(pos), out, images, h, w)
    got = host(out)
    ref = reference_embedding(oracle_lib, imgs, wt, b, cls, pos, 14, round_bf16=True)
    err = rel_l2(got, ref)
    print(f"bf16 patch embedding {images}x{h}x{w}: rel_l2 {err:.2e}")
    assert err < 1e-3
    # the cls rows are exactly cls + position[0]
    assert np.array_equal(got[:, 0], np.broadcast_to(cls + pos[0], got[:, 0].shape))


def test_patch_embed_batch_equals_single_images(vk, ctx):
    h, w = 336, 504
    imgs, wt, b, cls, pos, n = embedding_inputs(4, h, w, seed=3)
    pe = vk.PatchEmbed(ctx, wt, b, cls, channels=3, patch=14, math=vk.MATH_BF16)
    whole = torch.empty((4, n + 1, 768), device="cuda")
    assert pe(dev(imgs), dev(pos), whole, 4, h, w)
    for i in range(4):
        one = torch.empty((1, n + 1, 768), device="cuda")
        assert pe(dev(imgs[i:i + 1]), dev(pos), one, 1, h, w)
        assert np.array_equal(host(one)[0], host(whole)[i])


def test_patch_embed_pair_tiles(vk, ctx, oracle_lib):
    """8 images at 504x336 (6,912 patch rows): the projection runs on CTA-pair
    tiles, its epilogue writing each patch at its token row.  Against the
    single-image runs (single-CTA tiles) and the oracle for two images."""
    h, w = 336, 504
    imgs, wt, b, cls, pos, n = embedding_inputs(8, h, w, seed=11)
    pe = vk.PatchEmbed(ctx, wt, b, cls, channels=3, patch=14, math=vk.MATH_BF16)
    whole = torch.empty((8, n + 1, 768), device="cuda")
    assert pe(dev(imgs), dev(pos), whole, 8, h, w)
    got = host(whole)
    for i in (0, 5, 7):
        one = torch.empty((1, n + 1, 768), device="cuda")
        assert pe(dev(imgs[i:i + 1]), dev(pos), one, 1, h, w)
        assert rel_l2(host(one)[0], got[i]) < 1e-6, i
    ref = reference_embedding(oracle_lib, imgs[6:8], wt, b, cls, pos, 14, round_bf16=True)
    assert rel_l2(got[6:8], ref) < 1e-3


def test_patch_embed_rejects_non_multiple_grid(vk, ctx):
    imgs, wt, b, cls, pos, n = embedding_inputs(1, 28, 28)
    pe = vk.PatchEmbed(ctx, wt, b, cls, channels=3, patch=14, math=vk.MATH_BF16)
    out = torch.zeros((1, 5, 768), device="cuda")
    assert not pe(torch.zeros(3 * 30 * 28, device="cuda"), dev(pos), out, 1, 30, 28)
    assert float(out.abs().sum()) == 0.0

