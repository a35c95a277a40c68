"""GPU parity of the DA3-BASE encoder (vk_encoder_*) against the oracle's
block composition on the same seeded random-init weights.

The bars are stated on a block's *update* (out - in), which is what the
kernels compute, with LayerScale 1 so the update is as large as the stream
(at the DA3 init of 1e-5 the update sits below the f32 resolution of the
residual it is added to).  Relative L2 per layer, at the DA3-BASE shapes:
  bf16  <= 1e-3 against the oracle rounding to bf16 (v to f16) where the
        kernels store;
  f32   <= 1e-5 against the f32 oracle;
  Q8_0  <= 3e-3 against the oracle composing the reference's Q8_0 ops
        (quantize_row_q8_0, gemm_q8_0) at the kernels' quantisation points.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

E, H, F = 768, 12, 3072


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def make_layers(n, seed, ls=1e-5):
    r = np.random.default_rng(seed)
    f = lambda *s, sc=1.0: (r.standard_normal(s) * sc).astype(np.float32)
    out = []
    for _ in range(n):
        out.append({
            "ln1_g": np.ones(E, np.float32) + f(E, sc=0.05), "ln1_b": f(E, sc=0.02),
            "qkv_w": f(E, 3 * E, sc=0.02), "qkv_b": f(3 * E, sc=0.01),
            "proj_w": f(E, E, sc=0.02), "proj_b": f(E, sc=0.01), "ls1": np.full(E, ls, np.float32),
            "ln2_g": np.ones(E, np.float32) + f(E, sc=0.05), "ln2_b": f(E, sc=0.02),
            "fc1_w": f(E, F, sc=0.02), "fc1_b": f(F, sc=0.01),
            "fc2_w": f(F, E, sc=0.02), "fc2_b": f(E, sc=0.01), "ls2": np.full(E, ls, np.float32),
        })
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


def run_encoder(vk, ctx, layers, x, images, gh, gw, math):
    enc = vk.Encoder(ctx, layers, math=math)
    t = torch.from_numpy(x).cuda()
    out = torch.empty_like(t)
    enc.forward(t, out, images, gh, gw)
    ctx.synchronize()
    return out.cpu().numpy(), enc


MATHS = ["bf16", "f32", "q8"]
# Q8_0: the int32 block dots and the f32 fold are bit-exact (test_gpu_ops);
# what is left is how Q8_0 quantisation amplifies last-bit differences
# upstream of it (the LayerNorm's reduction order, attention's f32
# accumulation): a value that sits near a rounding boundary of d / 127 moves
# by a whole step.  Emulated on the oracle, a 1e-7 relative perturbation of
# the LayerNorm output alone gives 2e-3 on the update; measured here:
# 1.2e-3 - 2.3e-3.
BAR = {"bf16": 1e-3, "f32": 1e-5, "q8": 3e-3}


def math_mode(vk, math):
    return {"bf16": vk.MATH_BF16, "f32": vk.MATH_F32, "q8": vk.MATH_Q8_0}[math]


def oracle_points(math):
    return {"bf16_points": math == "bf16", "q8_points": math == "q8"}


@pytest.mark.parametrize("math", MATHS)
def test_one_block_full_size(vk, ctx, oracle_lib, math):
    gh, gw = 24, 36
    T = gh * gw + 1
    layers = make_layers(1, 7, ls=1.0)  # LayerScale 1 so the update is visible
    x = np.random.default_rng(8).standard_normal((1, T, E)).astype(np.float32)
    got, enc = run_encoder(vk, ctx, layers, x, 1, gh, gw, math_mode(vk, math))
    ref = oracle_lib.encoder(x[0], layers, gh, gw, **oracle_points(math))
    err = rel_l2(got[0] - x[0], ref - x[0])
    print(f"encoder block math={math} update rel_l2={err:.3e} launches={enc.last_launches()}")
    assert err < BAR[math]
    assert rel_l2(got[0], ref) < BAR[math]


@pytest.mark.parametrize("math", MATHS)
def test_twelve_layers_per_layer_full_size(vk, ctx, oracle_lib, math):
    """The 12-layer DA3-BASE encoder at 504x336 (24 x 36 patches, 865
    tokens): every layer's update against the oracle layer fed the same
    input (the GPU's own output of the layer before), and the 12-layer
    forward equal to the chain of single-layer forwards."""
    gh, gw = 24, 36
    T = gh * gw + 1
    layers = make_layers(12, 41, ls=1.0)
    x0 = np.random.default_rng(42).standard_normal((1, T, E)).astype(np.float32)
    m = math_mode(vk, math)
    x = x0
    errs = []
    for layer in layers:
        got, _ = run_encoder(vk, ctx, [layer], x, 1, gh, gw, m)
        ref = oracle_lib.encoder_layer(x[0], layer, gh, gw, **oracle_points(math))
        errs.append(rel_l2(got[0] - x[0], ref - x[0]))
        x = got
    print(f"12-layer {math} per-layer update rel_l2: " + " ".join(f"{e:.2e}" for e in errs))
    assert max(errs) < BAR[math], errs
    full, enc = run_encoder(vk, ctx, layers, x0, 1, gh, gw, m)
    assert enc.last_launches() == 12 * (10 if math == "f32" else 7)
    assert np.array_equal(full, x)


@pytest.mark.parametrize("math", MATHS)
def test_one_block_1008x672(vk, ctx, oracle_lib, math):
    """One block at 1008x672: 48 x 72 patches + cls = 3457 tokens, the RoPE
    grid 72 wide (src/specialized.rs:359-366) and 28 key blocks."""
    gh, gw = 48, 72
    T = gh * gw + 1
    layers = make_layers(1, 51, ls=1.0)
    x = np.random.default_rng(52).standard_normal((1, T, E)).astype(np.float32)
    got, _ = run_encoder(vk, ctx, layers, x, 1, gh, gw, math_mode(vk, math))
    ref = oracle_lib.encoder(x[0], layers, gh, gw, **oracle_points(math))
    err = rel_l2(got[0] - x[0], ref - x[0])
    print(f"encoder block 3457 tokens math={math} update rel_l2={err:.3e}")
    assert err < BAR[math]


def test_da3_layerscale_twelve_layers(vk, ctx, oracle_lib):
    """BASELINE's random init (LayerScale 1e-5), 12 layers chained, bf16:
    the whole output against the chained oracle."""
    gh, gw = 24, 36
    T = gh * gw + 1
    layers = make_layers(12, 61, ls=1e-5)
    x = np.random.default_rng(62).standard_normal((1, T, E)).astype(np.float32)
    got, _ = run_encoder(vk, ctx, layers, x, 1, gh, gw, vk.MATH_BF16)
    ref = oracle_lib.encoder(x[0], layers, gh, gw, bf16_points=True)
    err = rel_l2(got[0], ref)
    print(f"12-layer LayerScale 1e-5 output rel_l2={err:.3e}")
    assert err < 1e-6


def test_batch_images_independent(vk, ctx, oracle_lib):
    gh, gw = 24, 36
    T = gh * gw + 1
    layers = make_layers(2, 9)
    x = np.random.default_rng(10).standard_normal((3, T, E)).astype(np.float32)
    got3, _ = run_encoder(vk, ctx, layers, x, 3, gh, gw, vk.MATH_BF16)
    got1, _ = run_encoder(vk, ctx, layers, x[1:2].copy(), 1, gh, gw, vk.MATH_BF16)
    assert np.array_equal(got3[1], got1[0])


def test_twelve_layers_small_grid(vk, ctx, oracle_lib):
    """Two 25-token images through 12 chained layers: a whole-stack bar,
    since 12 chained bf16 layers compound their rounding."""
    gh, gw = 4, 6
    T = gh * gw + 1
    layers = make_layers(12, 11, ls=0.1)
    x = np.random.default_rng(12).standard_normal((2, T, E)).astype(np.float32)
    got, enc = run_encoder(vk, ctx, layers, x, 2, gh, gw, vk.MATH_BF16)
    for i in range(2):
        ref = oracle_lib.encoder(x[i], layers, gh, gw, bf16_points=True)
        err = rel_l2(got[i] - x[i], ref - x[i])
        print(f"12-layer image {i} stacked update rel_l2={err:.3e}")
        assert err < 3e-3
    assert enc.last_launches() == 12 * 7


def test_graph_replay_and_host_path_match(vk, ctx, oracle_lib):
    gh, gw = 24, 36
    T = gh * gw + 1
    layers = make_layers(2, 13)
    x = np.random.default_rng(14).standard_normal((5, T, E)).astype(np.float32)
    enc = vk.Encoder(ctx, layers, math=vk.MATH_BF16)
    t = torch.from_numpy(x).cuda()
    outs = []
    for _ in range(3):  # eager, capture, replay
        o = torch.empty_like(t)
        enc.forward(t, o, 5, gh, gw)
        ctx.synchronize()
        outs.append(o.cpu().numpy())
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])
    import os

    os.environ["VK_E2E_CHUNK"] = "2"
    try:
        hin = torch.from_numpy(x).pin_memory()
        hout = torch.empty_like(hin).pin_memory()
        for _ in range(2):
            enc.forward_host(hin, hout, 5, gh, gw)
            assert np.array_equal(hout.numpy(), outs[0])
        # back-to-back asynchronous calls on different buffers, interleaved
        # with a device-path forward, all ordered through the shared ring
        hin2 = torch.from_numpy(x[::-1].copy()).pin_memory()
        hout2 = torch.empty_like(hin2).pin_memory()
        hout.zero_()
        enc.forward_host_async(hin, hout, 5, gh, gw)
        enc.forward_host_async(hin2, hout2, 5, gh, gw)
        o = torch.empty_like(t)
        enc.forward(t, o, 5, gh, gw)
        ctx.synchronize()
        assert np.array_equal(hout.numpy(), outs[0])
        assert np.array_equal(hout2.numpy(), outs[0][::-1])
        assert np.array_equal(o.cpu().numpy(), outs[0])
    finally:
        del os.environ["VK_E2E_CHUNK"]


def test_large_batch_matches_single_images(vk, ctx, oracle_lib):
    """16 images (every GEMM on the CTA-pair kernel) against the same images
    run alone (single-CTA kernels)."""
    gh, gw = 24, 36
    T = gh * gw + 1
    layers = make_layers(1, 15, ls=1.0)
    x = np.random.default_rng(16).standard_normal((16, T, E)).astype(np.float32)
    big, _ = run_encoder(vk, ctx, layers, x, 16, gh, gw, vk.MATH_BF16)
    for i in (0, 7, 15):
        one, _ = run_encoder(vk, ctx, layers, x[i:i + 1].copy(), 1, gh, gw, vk.MATH_BF16)
        err = rel_l2(big[i] - x[i], one[0] - x[i])
        assert err < 1e-3, (i, err)


def test_eight_images_wide_residual_tiles(vk, ctx, oracle_lib):
    """8 images (M = 6,920 rows, a GPU's shard at 8-way strong scaling): the
    out-proj and fc2 GEMMs take 256 x 384 CTA-pair tiles (one round on 74 SM
    pairs).  Every image against the same image run alone, and image 0's
    update against the oracle."""
    gh, gw = 24, 36
    T = gh * gw + 1
    layers = make_layers(1, 17, ls=1.0)
    x = np.random.default_rng(18).standard_normal((8, T, E)).astype(np.float32)
    big, _ = run_encoder(vk, ctx, layers, x, 8, gh, gw, vk.MATH_BF16)
    for i in (0, 3, 7):
        one, _ = run_encoder(vk, ctx, layers, x[i:i + 1].copy(), 1, gh, gw, vk.MATH_BF16)
        assert rel_l2(big[i] - x[i], one[0] - x[i]) < 1e-3, i
    ref = oracle_lib.encoder(x[0], layers, gh, gw, bf16_points=True)
    err = rel_l2(big[0] - x[0], ref - x[0])
    print(f"8-image block (256 x 384 residual tiles) update rel_l2={err:.3e}")
    assert err < 1e-3


def oracle_views_layer(oracle_lib, views, layer, gh, gw, joint, bf):
    """One layer over a group of views: jointly (a global layer) or per view."""
    T = gh * gw + 1
    if joint:
        out = oracle_lib.encoder_layer(np.concatenate(views), layer, gh, gw, bf16_points=bf)
        return [out[i * T:(i + 1) * T] for i in range(len(views))]
    return [oracle_lib.encoder_layer(v, layer, gh, gw, bf16_points=bf) for v in views]


def per_layer_views(vk, ctx, oracle_lib, layers, x, gh, gw, V, global_layers, math, tag):
    """Every layer of a multi-view stack against the oracle layer fed the
    GPU's own input; the whole stack equal to the chained layers."""
    m = {"bf16": vk.MATH_BF16, "f32": vk.MATH_F32}[math]
    bf = math == "bf16"
    images = x.shape[0]
    cur = x
    errs = []
    for li, layer in enumerate(layers):
        g = li in global_layers
        enc = vk.Encoder(ctx, [layer], math=m, views=V, global_layers=(0,) if g else ())
        t = torch.from_numpy(cur).cuda()
        out = torch.empty_like(t)
        assert enc.forward(t, out, images, gh, gw)
        ctx.synchronize()
        got = out.cpu().numpy()
        for grp in range(images // V):
            views = [cur[grp * V + i] for i in range(V)]
            ref = oracle_views_layer(oracle_lib, views, layer, gh, gw, g, bf)
            for i in range(V):
                img = grp * V + i
                errs.append(rel_l2(got[img] - cur[img], ref[i] - cur[img]))
        cur = got
    print(f"{tag} {math}: per-layer update rel_l2 max {max(errs):.2e}")
    assert max(errs) < BAR[math], errs
    enc = vk.Encoder(ctx, layers, math=m, views=V, global_layers=tuple(global_layers))
    t = torch.from_numpy(x).cuda()
    out = torch.empty_like(t)
    assert enc.forward(t, out, images, gh, gw)
    ctx.synchronize()
    assert np.array_equal(out.cpu().numpy(), cur)
    return enc, t


@pytest.mark.parametrize("math", ["bf16", "f32"])
def test_multiview_global_layers(vk, ctx, oracle_lib, math):
    """Two views of 504x336 (one sequence of 2 x 865 tokens, RoPE positions
    repeating per view) in global layers 1 and 2, per-view layer 0.
    Oracle: the same composition from the restated block."""
    gh, gw, V = 24, 36, 2
    T = gh * gw + 1
    layers = make_layers(3, 21, ls=1.0)
    x = np.random.default_rng(22).standard_normal((2, T, E)).astype(np.float32)
    enc, t = per_layer_views(vk, ctx, oracle_lib, layers, x, gh, gw, V, (1, 2), math, "multi-view")
    # an image count that is not whole groups is refused, output untouched
    out2 = torch.zeros((1, T, E), device="cuda")
    assert not enc.forward(t[:1].contiguous(), out2, 1, gh, gw)
    assert float(out2.abs().sum()) == 0.0


def test_multiview_small_grid(vk, ctx, oracle_lib):
    """Four 25-token images as two pairs of views, global layers 1 and 3,
    f32 (the bf16 bar is set at the DA3-BASE shapes above)."""
    gh, gw, V = 4, 6, 2
    T = gh * gw + 1
    layers = make_layers(4, 25, ls=1.0)
    x = np.random.default_rng(26).standard_normal((4, T, E)).astype(np.float32)
    per_layer_views(vk, ctx, oracle_lib, layers, x, gh, gw, V, (1, 3), "f32", "multi-view 25")


def add_qk_norm(layer, seed):
    r = np.random.default_rng(seed)
    layer = dict(layer)
    layer["q_norm_g"] = (1.0 + 0.1 * r.standard_normal(64)).astype(np.float32)
    layer["q_norm_b"] = (0.05 * r.standard_normal(64)).astype(np.float32)
    layer["k_norm_g"] = (1.0 + 0.1 * r.standard_normal(64)).astype(np.float32)
    layer["k_norm_b"] = (0.05 * r.standard_normal(64)).astype(np.float32)
    return layer


@pytest.mark.parametrize("math", ["bf16", "f32"])
def test_qk_norm_layers(vk, ctx, oracle_lib, math):
    """Layers 1 and 2 LayerNorm each q / k head before RoPE (DA3's late
    blocks, qk_norm_rope_f32_da3_base); layer 2 is also a global cross-view
    layer.  Two 504x336 views.  Oracle: the restated block with the same
    options."""
    gh, gw, V = 24, 36, 2
    T = gh * gw + 1
    layers = make_layers(3, 31, ls=1.0)
    layers[1] = add_qk_norm(layers[1], 32)
    layers[2] = add_qk_norm(layers[2], 33)
    x = np.random.default_rng(34).standard_normal((2, T, E)).astype(np.float32)
    enc, t = per_layer_views(vk, ctx, oracle_lib, layers, x, gh, gw, V, (2,), math, "qk-norm")
    out = torch.empty_like(t)
    slots = enc.profile(t, out, 2, gh, gw)
    assert len(slots) == (10 if math == "f32" else 7) and all(s >= 0.0 for s in slots)


def test_qk_norm_needs_bf16_or_f32(vk, ctx):
    layers = make_layers(1, 35)
    layers[0] = add_qk_norm(layers[0], 36)
    with pytest.raises(vk.VestraError):
        vk.Encoder(ctx, layers, math=vk.MATH_Q8_0)
