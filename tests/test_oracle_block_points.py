"""The oracle's block composition (vko_encoder_layer) at its three rounding
modes, restated here from the oracle's own operators in Python and checked
bit for bit: pre-LN -> QKV (+bias) -> RoPE on q, k -> attention ->
out-proj (+bias) * LS1 + residual -> LN -> fc1 (+bias) -> GELU -> fc2
(+bias) * LS2 + residual, with
  bf16 points: weights and the stored activations rounded to bf16, v to f16;
  Q8_0 points: every projection is quantize_row_q8_0 + gemm_q8_0
               (src/q8_0_dot.rs:27-46, src/scalar.rs:25-56) on Q8_0 weights
               (the [K, N] weight transposed, src/dispatch.rs:85-90), q and k
               rounded to bf16 and v to f16.
"""
import numpy as np
import pytest

E, H, F = 768, 12, 3072


def layer(seed):
    r = np.random.default_rng(seed)
    f = lambda *s, sc=1.0: (r.standard_normal(s) * sc).astype(np.float32)
    return {"ln1_g": 1 + f(E, sc=0.05), "ln1_b": f(E, sc=0.02), "qkv_w": f(E, 3 * E, sc=0.02),
            "qkv_b": f(3 * E, sc=0.01), "proj_w": f(E, E, sc=0.02), "proj_b": f(E, sc=0.01),
            "ls1": np.full(E, 0.5, np.float32), "ln2_g": 1 + f(E, sc=0.05), "ln2_b": f(E, sc=0.02),
            "fc1_w": f(E, F, sc=0.02), "fc1_b": f(F, sc=0.01), "fc2_w": f(F, E, sc=0.02),
            "fc2_b": f(E, sc=0.01), "ls2": np.full(E, 0.5, np.float32)}


def f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def block(O, x, L, gh, gw, mode):
    T = x.shape[0]
    pos = O.da3_positions(gh, gw)
    bf = mode == "bf16"
    R = O.round_bf16 if bf else (lambda t: t)

    def lin(a, w):
        if mode == "q8":
            wq = O.quantize_rows_q8_0(np.ascontiguousarray(w.T))
            return O.gemm_q8_0(a.shape[0], w.shape[1], a.shape[1], O.quantize_rows_q8_0(a), wq)
        return O.linear_fma(a, R(w))

    h = R(O.layernorm(x, L["ln1_g"], L["ln1_b"], 1e-6))
    c = (lin(h, L["qkv_w"]) + L["qkv_b"]).astype(np.float32)
    q, k, v = [c[:, i * E:(i + 1) * E].reshape(T, H, 64).transpose(1, 0, 2).copy() for i in range(3)]
    q, k = O.rope2d(q, pos, 100.0), O.rope2d(k, pos, 100.0)
    if mode != "f32":
        q, k, v = O.round_bf16(q), O.round_bf16(k), f16(v)
    att = O.attention_naive(q, k, v).transpose(1, 0, 2).reshape(T, E).copy()
    o = ((lin(R(att), L["proj_w"]) + L["proj_b"]) * L["ls1"]).astype(np.float32)
    x = O.add(x, o)
    h = R(O.layernorm(x, L["ln2_g"], L["ln2_b"], 1e-6))
    g = R(O.gelu((lin(h, L["fc1_w"]) + L["fc1_b"]).astype(np.float32)))
    o = ((lin(g, L["fc2_w"]) + L["fc2_b"]) * L["ls2"]).astype(np.float32)
    return O.add(x, o)


@pytest.mark.parametrize("mode", ["f32", "bf16", "q8"])
def test_block_points_composition(oracle_lib, mode):
    gh, gw = 4, 6
    L = layer(3)
    x = np.random.default_rng(4).standard_normal((gh * gw + 1, E)).astype(np.float32)
    got = oracle_lib.encoder_layer(x, L, gh, gw, bf16_points=mode == "bf16", q8_points=mode == "q8")
    ref = block(oracle_lib, x, L, gh, gw, mode)
    assert np.array_equal(got, ref)
