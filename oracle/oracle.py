"""ctypes view of the CPU parity checker (oracle/libvk_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg.  The product (vestra-kernels_b200/) never
imports this module.  Each wrapper names the reference function it restates;
the C sources carry the reference file:line citations.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

QK8_0 = 32
# BlockQ8_0 {d: f16, qs: [i8; 32]}, #[repr(C)], 34 bytes (src/lib.rs:33-38).
BLOCK_Q8_0 = np.dtype([("d", "<u2"), ("qs", "i1", (QK8_0,))], align=False)
assert BLOCK_Q8_0.itemsize == 34

_f = ctypes.POINTER(ctypes.c_float)
_sz = ctypes.c_size_t


def build() -> str:
    """Compile the oracle libraries (make in oracle/)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", _HERE, "all"], check=True)
    return os.path.join(_HERE, "libvk_oracle.so")


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "libvk_oracle.so")
        if not os.path.exists(path):
            build()
        _LIB = ctypes.CDLL(path)
    return _LIB


def _p(a: np.ndarray, ctype=ctypes.c_float):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().vko_set_threads(ctypes.c_int(n))


def f16_from_f32(x: float) -> int:
    lib().vko_f16_from_f32.restype = ctypes.c_uint16
    return int(lib().vko_f16_from_f32(ctypes.c_float(x)))


def round_bf16(x) -> np.ndarray:
    """bfloat16 round-to-nearest-even, returned as f32."""
    x = _f32(x)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    nan = np.isnan(x)
    out = r.view(np.float32).copy()
    out[nan] = np.nan
    return out.reshape(x.shape)


def gemm_f32(a, b) -> np.ndarray:
    """scalar::gemm_f32 (src/scalar.rs:3-18)."""
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().vko_gemm_f32(_sz(m), _sz(n), _sz(k), _p(a), _p(b), _p(c))
    return c


def quantize_rows_q8_0(x) -> np.ndarray:
    """quantize_row_q8_0 applied per row (src/q8_0_dot.rs:27-46)."""
    x = _f32(x)
    rows, k = x.shape
    assert k % QK8_0 == 0
    out = np.zeros((rows, k // QK8_0), BLOCK_Q8_0)
    lib().vko_quantize_row_q8_0(_p(x), _sz(rows * (k // QK8_0)), out.ctypes.data_as(ctypes.c_void_p))
    return out


def dequantize_q8_0(blocks: np.ndarray) -> np.ndarray:
    """dequantize_q8_0 (src/lib.rs:42-50); returns [..., K]."""
    blocks = np.ascontiguousarray(blocks)
    out = np.empty(blocks.size * QK8_0, np.float32)
    lib().vko_dequantize_q8_0(blocks.ctypes.data_as(ctypes.c_void_p), _sz(blocks.size), _p(out))
    return out.reshape(blocks.shape[:-1] + (blocks.shape[-1] * QK8_0,))


def gemm_q8_0(m, n, k, a_q, b_q) -> np.ndarray:
    """scalar::gemm_q8_0 (src/scalar.rs:25-56); B is pre-transposed [N, K/32]."""
    a_q, b_q = np.ascontiguousarray(a_q), np.ascontiguousarray(b_q)
    c = np.empty((m, n), np.float32)
    lib().vko_gemm_q8_0(_sz(m), _sz(n), _sz(k), a_q.ctypes.data_as(ctypes.c_void_p),
                        b_q.ctypes.data_as(ctypes.c_void_p), _p(c))
    return c


def q8_0_block_dots(m, n, k, a_q, b_q) -> np.ndarray:
    """The int32 per-block dot products of src/scalar.rs:47-50: [M, N, K/32]."""
    a_q, b_q = np.ascontiguousarray(a_q), np.ascontiguousarray(b_q)
    out = np.empty((m, n, k // QK8_0), np.int32)
    lib().vko_q8_0_block_dots(_sz(m), _sz(n), _sz(k), a_q.ctypes.data_as(ctypes.c_void_p),
                              b_q.ctypes.data_as(ctypes.c_void_p), _p(out, ctypes.c_int32))
    return out


def add(dst, src) -> np.ndarray:
    dst = _f32(dst).copy()
    src = _f32(src)
    lib().vko_add(_p(dst), _p(src), _sz(dst.size))
    return dst


def add_bias_rows(x, bias) -> np.ndarray:
    x = _f32(x).copy()
    rows, cols = x.shape
    lib().vko_add_bias_rows(_p(x), _sz(rows), _sz(cols), _p(_f32(bias)))
    return x


def layernorm(x, gamma, beta, eps) -> np.ndarray:
    """scalar::layernorm (src/scalar.rs:83-114)."""
    x = _f32(x).copy()
    rows, cols = x.reshape(-1, x.shape[-1]).shape
    lib().vko_layernorm(_p(x), _sz(rows), _sz(cols), _p(_f32(gamma)), _p(_f32(beta)), ctypes.c_float(eps))
    return x


def gelu(x) -> np.ndarray:
    """scalar::gelu (src/scalar.rs:116-134)."""
    x = _f32(x).copy()
    lib().vko_gelu(_p(x), _sz(x.size))
    return x


def erf(x: float) -> float:
    lib().vko_erf.restype = ctypes.c_float
    return float(lib().vko_erf(ctypes.c_float(x)))


def layerscale(x, gamma) -> np.ndarray:
    x = _f32(x).copy()
    rows, cols = x.shape
    lib().vko_layerscale(_p(x), _sz(rows), _sz(cols), _p(_f32(gamma)))
    return x


def softmax_rows(x) -> np.ndarray:
    x = _f32(x).copy()
    rows, cols = x.shape
    lib().vko_softmax_rows(_p(x), _sz(rows), _sz(cols))
    return x


def attention_naive(q, k, v) -> np.ndarray:
    """attention_naive (src/attention.rs:10-59); q,k,v [heads, n, head_dim]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    heads, n, hd = q.shape
    out = np.empty_like(q)
    lib().vko_attention_naive(_p(q), _p(k), _p(v), _sz(heads), _sz(n), _sz(hd), _p(out))
    return out


def attention(q, k, v) -> np.ndarray:
    """attention, tiled online route (src/attention.rs:66-201)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    heads, n, hd = q.shape
    out = np.empty_like(q)
    lib().vko_attention(_p(q), _p(k), _p(v), _sz(heads), _sz(n), _sz(hd), _p(out))
    return out


def rope2d(x, pos_yx, freq) -> np.ndarray:
    """rope2d (src/rope.rs:30-93); x [heads, n, head_dim], pos_yx [n, 2] int64."""
    x = _f32(x).copy()
    heads, n, hd = x.shape
    pos = np.ascontiguousarray(pos_yx, dtype=np.int64)
    lib().vko_rope2d(_p(x), _sz(heads), _sz(n), _sz(hd), _p(pos, ctypes.c_int64), ctypes.c_float(freq))
    return x


def rope_rotations(pos_yx, freq) -> np.ndarray:
    """rope_rotations (src/specialized.rs:389-410): [tokens, 2, 16, 2] (sin, cos)."""
    pos = np.ascontiguousarray(pos_yx, dtype=np.int64)
    t = pos.shape[0]
    out = np.empty((t, 2, 16, 2), np.float32)
    lib().vko_rope_rotations(_p(pos, ctypes.c_int64), _sz(t), ctypes.c_float(freq), _p(out))
    return out


def qk_norm_rope(q, k, qg, qb, kg, kb, pos_yx, freq, eps):
    """qk_norm_rope_f32_da3_base (src/specialized.rs:278-454)."""
    q, k = _f32(q).copy(), _f32(k).copy()
    heads, t, _ = q.shape
    pos = np.ascontiguousarray(pos_yx, dtype=np.int64)
    lib().vko_qk_norm_rope(_p(q), _p(k), _sz(heads), _sz(t), _p(_f32(qg)), _p(_f32(qb)),
                           _p(_f32(kg)), _p(_f32(kb)), _p(pos, ctypes.c_int64),
                           ctypes.c_float(freq), ctypes.c_float(eps))
    return q, k


def da3_positions(grid_h, grid_w) -> np.ndarray:
    out = np.empty((grid_h * grid_w + 1, 2), np.int64)
    lib().vko_da3_positions(_sz(grid_h), _sz(grid_w), _p(out, ctypes.c_int64))
    return out


def qkv(x, w, b, heads):
    """qkv_f32_da3_base (src/specialized.rs:996-1167) generalised in tokens."""
    x, w, b = _f32(x), _f32(w), _f32(b)
    t = x.shape[0]
    q = np.empty((heads, t, 64), np.float32)
    k = np.empty_like(q)
    v = np.empty_like(q)
    lib().vko_qkv(_sz(t), _sz(heads), _p(x), _p(w), _p(b), _p(q), _p(k), _p(v))
    return q, k, v


def linear_bias_scale(a, b, bias, scale) -> np.ndarray:
    """linear_bias_scale_f32_da3_base arithmetic (src/specialized.rs:880-991)."""
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().vko_linear_bias_scale(_sz(m), _sz(n), _sz(k), _p(a), _p(b), _p(_f32(bias)),
                                _p(_f32(scale)), _p(c))
    return c


def linear_fma(a, b) -> np.ndarray:
    """linear_f32_da3_base arithmetic: ascending-K FMA (src/specialized.rs:1171-1300)."""
    return linear_bias_scale(a, b, np.zeros(np.shape(b)[1], np.float32), np.ones(np.shape(b)[1], np.float32))


def patchify_nchw(image, height, width, patch, channels) -> np.ndarray:
    """vestra_patchify_nchw_f32 (src/cuda.rs:295-316); raises on an invalid shape."""
    image = _f32(image)
    rows = (height // patch) * (width // patch) if patch else 0
    out = np.empty((rows, channels * patch * patch), np.float32)
    lib().vko_patchify_nchw.restype = ctypes.c_int
    if lib().vko_patchify_nchw(_p(image), _sz(height), _sz(width), _sz(patch), _sz(channels), _p(out)) != 0:
        raise ValueError("invalid NCHW patchify shape")
    return out


def prepend_cls_add_pos(patches, cls, position, patch_count, embed) -> np.ndarray:
    """vestra_prepend_cls_add_pos_f32 (src/cuda.rs:321-334)."""
    out = np.empty((patch_count + 1, embed), np.float32)
    lib().vko_prepend_cls_add_pos(_p(_f32(patches)), _p(_f32(cls)), _p(_f32(position)), _sz(patch_count), _sz(embed),
                                  _p(out))
    return out


# ---- DPT head consumers (the step after the encoder)

def token_to_chw(token_major, tokens, channels) -> np.ndarray:
    """vestra_token_to_chw_f32 (src/cuda.rs:278-291): [tokens, channels] -> [channels, tokens]."""
    out = np.empty((channels, tokens), np.float32)
    lib().vko_token_to_chw(_p(_f32(token_major)), _sz(tokens), _sz(channels), _p(out))
    return out


def bilinear_resize(x, oh, ow, align_corners=False) -> np.ndarray:
    """bilinear_resize / bilinear_resize_align_corners (src/resample.rs:10-99, 151-249); x [c, ih, iw]."""
    x = _f32(x)
    c, ih, iw = x.shape
    out = np.zeros((c, oh, ow), np.float32)
    fn = lib().vko_bilinear_resize_align_corners if align_corners else lib().vko_bilinear_resize
    fn(_p(x), _sz(c), _sz(ih), _sz(iw), _sz(oh), _sz(ow), _p(out))
    return out


def winograd_f2_filter(weight, in_c, out_c) -> np.ndarray:
    """transformed_winograd_filter (src/conv.rs:121-171): OIHW -> U [16, in_c, out_c]."""
    u = np.empty((16, in_c, out_c), np.float32)
    lib().vko_winograd_f2_filter(_p(_f32(weight)), _sz(in_c), _sz(out_c), _p(u))
    return u


def conv3x3_winograd_f2(x, weight, bias=None, relu_input=False) -> np.ndarray:
    """conv3x3_winograd_f2 / _relu_input (src/conv.rs:266-280, 651-831); x [in_c, h, w], OIHW weight."""
    x = _f32(x)
    in_c, h, w = x.shape
    out_c = np.shape(weight)[0]
    u = winograd_f2_filter(weight, in_c, out_c)
    out = np.empty((out_c, h, w), np.float32)
    b = _f32(bias) if bias is not None else None
    lib().vko_conv3x3_winograd_f2(_p(x), _sz(in_c), _sz(h), _sz(w), _p(u), _sz(out_c),
                                  _p(b) if b is not None else None, ctypes.c_int(int(relu_input)), _p(out))
    return out


def conv3x3_winograd_f2_resize_ac(x, oh, ow, add, weight, bias=None) -> np.ndarray:
    """conv3x3_winograd_f2_prepared_resize_align_corners (src/conv.rs:304-484)."""
    x = _f32(x)
    in_c, ih, iw = x.shape
    out_c = np.shape(weight)[0]
    u = winograd_f2_filter(weight, in_c, out_c)
    out = np.empty((out_c, oh, ow), np.float32)
    a = _f32(add) if add is not None else None
    b = _f32(bias) if bias is not None else None
    lib().vko_conv3x3_winograd_f2_resize_ac(_p(x), _sz(in_c), _sz(ih), _sz(iw), _sz(oh), _sz(ow),
                                            _p(a) if a is not None else None, _p(u), _sz(out_c),
                                            _p(b) if b is not None else None, _p(out))
    return out


def conv2d_naive(x, weight, stride=1, pad=1, bias=None) -> np.ndarray:
    """conv2d_naive (src/conv.rs:950-1000): direct convolution, OIHW weight."""
    x = _f32(x)
    weight = _f32(weight)
    in_c, ih, iw = x.shape
    out_c, _, kh, kw = weight.shape
    oh, ow = (ih + 2 * pad - kh) // stride + 1, (iw + 2 * pad - kw) // stride + 1
    out = np.empty((out_c, oh, ow), np.float32)
    b = _f32(bias) if bias is not None else None
    lib().vko_conv2d_naive(_p(x), _sz(in_c), _sz(ih), _sz(iw), _p(weight), _sz(out_c), _sz(kh), _sz(kw),
                           _sz(stride), _sz(pad), _p(b) if b is not None else None, _p(out))
    return out


LAYER_KEYS = ["ln1_g", "ln1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "ls1",
              "ln2_g", "ln2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "ls2"]
# optional Q/K LayerNorm vectors of a layer dict -> struct fields
QK_NORM_KEYS = {"q_norm_g": "qn_g", "q_norm_b": "qn_b", "k_norm_g": "kn_g", "k_norm_b": "kn_b"}


class _Layer(ctypes.Structure):
    _fields_ = [(n, _f) for n in LAYER_KEYS + list(QK_NORM_KEYS.values())]


def _layer_struct(layer: dict):
    keep = {kk: _f32(layer[kk]) for kk in LAYER_KEYS}
    for kk, field in QK_NORM_KEYS.items():
        if layer.get(kk) is not None:
            keep[field] = _f32(layer[kk])
    return keep, _Layer(**{kk: _p(vv) for kk, vv in keep.items()})


def encoder_layer(x, layer: dict, grid_h, grid_w, heads=12, eps=1e-6, freq=100.0, bf16_points=False,
                  q8_points=False):
    """One DA3-BASE block composed from the restated operators; x [T, E].

    bf16_points rounds to bf16 (v to f16) where the bf16 kernels store;
    q8_points runs the projections as gemm_q8_0 over Q8_0 weights and
    activations, where the Q8_0 kernels quantise."""
    assert not (bf16_points and q8_points)
    x = _f32(x).copy()
    t, e = x.shape
    ffn = np.shape(layer["fc1_w"])[1]
    keep, st = _layer_struct(layer)
    lib().vko_encoder_layer(_p(x), _sz(t), _sz(grid_h), _sz(grid_w), _sz(e), _sz(heads), _sz(ffn),
                            ctypes.byref(st), ctypes.c_float(eps), ctypes.c_float(freq),
                            ctypes.c_int(2 if q8_points else (1 if bf16_points else 0)))
    return x


def encoder(x, layers, grid_h, grid_w, heads=12, eps=1e-6, freq=100.0, bf16_points=False, q8_points=False):
    for layer in layers:
        x = encoder_layer(x, layer, grid_h, grid_w, heads, eps, freq, bf16_points, q8_points)
    return x


# ---------------------------------------------------------------- timed CPU baseline
_REF = None


def cpu_ref():
    """libvk_cpu_ref.so: the AVX-512 + OpenMP restatement of the reference's
    timed fast path (the CPU baseline bench.py reports)."""
    global _REF
    if _REF is None:
        path = os.path.join(_HERE, "libvk_cpu_ref.so")
        if not os.path.exists(path):
            build()
        _REF = ctypes.CDLL(path)
    return _REF


def set_cpu_ref_threads(n: int) -> None:
    """OpenMP threads of the timed CPU baseline (libvk_cpu_ref.so).  torchrun
    exports OMP_NUM_THREADS=1 to every rank, so the baseline sets its own."""
    cpu_ref().vko_set_threads(ctypes.c_int(n))


def cpu_ref_encoder_layer(x, layer: dict, grid_h, grid_w, eps=1e-6, freq=100.0):
    """One block on the restated AVX-512 path; x [T, 768], modified copy returned."""
    x = _f32(x).copy()
    keep, st = _layer_struct(layer)
    cpu_ref().vkr_encoder_layer(_p(x), _sz(x.shape[0]), _sz(grid_h), _sz(grid_w), ctypes.byref(st),
                                ctypes.c_float(eps), ctypes.c_float(freq))
    return x


def cpu_ref_flash_attention(q, k, v):
    q, k, v = _f32(q), _f32(k), _f32(v)
    heads, n, _ = q.shape
    out = np.empty_like(q)
    cpu_ref().vkr_flash_attention(_p(q), _p(k), _p(v), _sz(heads), _sz(n), _p(out))
    return out
