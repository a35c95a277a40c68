"""The timed CPU baseline (oracle/vk_cpu_ref.c, the reference's AVX-512 path
restated) agrees with the scalar oracle within the reference's own bounds."""
import numpy as np
import pytest


def test_cpu_ref_flash_attention_matches_serial(oracle_lib):
    """src/specialized.rs:2871-2910: flash vs serial tiled, MAE <= 2e-5, max <= 2e-4."""
    r = np.random.default_rng(0)
    q, k, v = (r.uniform(-1, 1, (2, 865, 64)).astype(np.float32) for _ in range(3))
    got = oracle_lib.cpu_ref_flash_attention(q, k, v)
    ref = oracle_lib.attention(q, k, v)
    d = np.abs(got - ref)
    assert d.mean() <= 2e-5 and d.max() <= 2e-4


def test_cpu_ref_block_matches_oracle(oracle_lib):
    E, F = 768, 3072
    r = np.random.default_rng(1)
    f = lambda *s, sc=1.0: (r.standard_normal(s) * sc).astype(np.float32)
    layer = {"ln1_g": np.ones(E, np.float32), "ln1_b": f(E, sc=0.02), "qkv_w": f(E, 3 * E, sc=0.02),
             "qkv_b": f(3 * E, sc=0.01), "proj_w": f(E, E, sc=0.02), "proj_b": f(E, sc=0.01),
             "ls1": np.ones(E, np.float32), "ln2_g": np.ones(E, np.float32), "ln2_b": f(E, sc=0.02),
             "fc1_w": f(E, F, sc=0.02), "fc1_b": f(F, sc=0.01), "fc2_w": f(F, E, sc=0.02),
             "fc2_b": f(E, sc=0.01), "ls2": np.ones(E, np.float32)}
    x = f(25, E)
    got = oracle_lib.cpu_ref_encoder_layer(x, layer, 4, 6)
    ref = oracle_lib.encoder_layer(x, layer, 4, 6)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref - x)
    assert err < 1e-5, err
