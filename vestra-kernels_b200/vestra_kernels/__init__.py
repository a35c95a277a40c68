"""vestra_kernels -- Python mirror of the vestra-kernels public API on B200.

The functions keep the names, argument order and meaning of the reference
crate's public API (src/lib.rs:52-130, src/attention.rs, src/rope.rs,
src/scalar.rs, src/dispatch.rs, src/q8_0_dot.rs): buffers are CUDA tensors
(torch is used only to own device memory and streams), shapes are explicit,
the DA3-BASE specialised operators return ``False`` when the shape is
unsupported and leave the output untouched, generic operators raise on
length mismatches as the reference's ``assert_eq!`` panics do.

Every call goes through the C ABI of ``libvestra_b200.so``
(include/vestra_b200.h).  There is no CPU fallback: importing this module
without the built library, or calling it without a B200, raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvestra_b200.so")

VK_OK = 0
VK_UNSUPPORTED_SHAPE = 1
VK_ERR_INVALID_ARGUMENT = 2
VK_ERR_CUDA = 3
VK_ERR_TIMEOUT = 4
VK_ERR_NO_DEVICE = 5
VK_ERR_OUT_OF_MEMORY = 6

MATH_F32 = 0
MATH_BF16 = 1
MATH_Q8_0 = 2

QK8_0 = 32
DA3_BASE_TOKENS = 865

# Exported entry points of include/vestra_b200.h, with ctypes signatures.
_P = ctypes.c_void_p
_S = ctypes.c_size_t
_I = ctypes.c_int
_F = ctypes.c_float
SIGNATURES = {
    "vk_init": (_I, [_I, ctypes.POINTER(_P)]),
    "vk_destroy": (_I, [_P]),
    "vk_stream_set": (_I, [_P, _P]),
    "vk_set_math": (_I, [_P, _I]),
    "vk_synchronize": (_I, [_P]),
    "vk_last_error": (ctypes.c_char_p, []),
    "vk_version": (ctypes.c_char_p, []),
    "vk_qkv_f32_da3_base": (_I, [_P, _S, _P, _P, _P, _P, _P, _P]),
    "vk_linear_f32_da3_base": (_I, [_P, _S, _S, _S, _P, _P, _P]),
    "vk_linear_bias_scale_f32_da3_base": (_I, [_P, _S, _S, _S, _P, _P, _P, _P, _P]),
    "vk_flash_attention_f32_da3_base": (_I, [_P, _P, _P, _P, _S, _S, _P]),
    "vk_qk_norm_rope_f32_da3_base": (_I, [_P, _P, _P, _S, _S, _P, _P, _P, _P, _P, _F, _F]),
    "vk_attention": (_I, [_P, _P, _P, _P, _S, _S, _S, _P]),
    "vk_rope2d": (_I, [_P, _P, _S, _S, _S, _P, _F]),
    "vk_layernorm": (_I, [_P, _P, _S, _S, _P, _P, _F]),
    "vk_gelu": (_I, [_P, _P, _S]),
    "vk_add": (_I, [_P, _P, _P, _S]),
    "vk_add_bias_rows": (_I, [_P, _P, _S, _S, _P]),
    "vk_layerscale": (_I, [_P, _P, _S, _S, _P]),
    "vk_quantize_row_q8_0": (_I, [_P, _P, _S, _P]),
    "vk_gemm_q8_0": (_I, [_P, _S, _S, _S, _P, _P, _P]),
    "vk_gemm_q8_0_block_dots": (_I, [_P, _S, _S, _S, _P, _P, _P]),
    "vk_gemm_q8_0_noalloc": (_I, [_P, _S, _S, _S, _P, _P, _P]),
    "vk_prepare_linear": (_I, [_P, _S, _S, _P, _P, _P, _I, ctypes.POINTER(_P)]),
    "vk_prepare_linear_q8_0": (_I, [_P, _S, _S, _P, _P, _P, ctypes.POINTER(_P)]),
    "vk_linear_run": (_I, [_P, _P, _S, _P, _P]),
    "vk_release_linear": (_I, [_P]),
    "vk_encoder_prepare": (_I, [_P, _P, _P, ctypes.POINTER(_P)]),
    "vk_encoder_forward": (_I, [_P, _P, _S, _S, _S, _P, _P]),
    "vk_encoder_forward_host": (_I, [_P, _P, _S, _S, _S, _P, _P]),
    "vk_encoder_forward_host_async": (_I, [_P, _P, _S, _S, _S, _P, _P]),
    "vk_encoder_profile": (_I, [_P, _P, _S, _S, _S, _P, _P, _P, _I]),
    "vk_encoder_last_launches": (_I, [_P]),
    "vk_encoder_release": (_I, [_P]),
    "vk_patchify_nchw_f32": (_I, [_P, _P, _S, _S, _S, _S, _P]),
    "vk_prepend_cls_add_pos_f32": (_I, [_P, _P, _P, _P, _S, _S, _P]),
    "vk_patch_embed_prepare": (_I, [_P, _S, _S, _S, _P, _P, _P, _I, ctypes.POINTER(_P)]),
    "vk_patch_embed_forward": (_I, [_P, _P, _S, _S, _S, _P, _P, _P]),
    "vk_patch_embed_release": (_I, [_P]),
    "vk_token_to_chw_f32": (_I, [_P, _P, _S, _S, _P]),
    "vk_token_to_chw_f32_batched": (_I, [_P, _P, _S, _S, _S, _P]),
    "vk_bilinear_resize_f32": (_I, [_P, _P, _S, _S, _S, _S, _S, _P]),
    "vk_bilinear_resize_align_corners_f32": (_I, [_P, _P, _S, _S, _S, _S, _S, _P]),
    "vk_conv3x3_prepare": (_I, [_P, _P, _S, _S, ctypes.POINTER(_P)]),
    "vk_conv3x3_prepare_math": (_I, [_P, _P, _S, _S, _I, ctypes.POINTER(_P)]),
    "vk_conv3x3_forward": (_I, [_P, _P, _P, _S, _S, _S, _S, _P, _I, _P]),
    "vk_conv3x3_resize_ac_forward": (_I, [_P, _P, _P, _S, _S, _S, _S, _S, _P, _S, _P, _P]),
    "vk_conv3x3_forward_batched": (_I, [_P, _P, _S, _P, _S, _S, _P, _I, _P]),
    "vk_conv3x3_resize_ac_forward_batched": (_I, [_P, _P, _S, _P, _S, _S, _S, _S, _P, _P, _P]),
    "vk_conv3x3_release": (_I, [_P]),
}

_lib = None
_lock = threading.Lock()


class VestraError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"status {status}: {msg}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Loads libvestra_b200.so (raises if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is missing: run `python vestra-kernels_b200/build.py`")
            l = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(l, name)
                fn.restype = res
                fn.argtypes = args
            _lib = l
    return _lib


def last_error() -> str:
    return lib().vk_last_error().decode()


def _check(status: int) -> int:
    if status not in (VK_OK, VK_UNSUPPORTED_SHAPE):
        raise VestraError(status, last_error())
    return status


def _ptr(t):
    if t is None:
        return None
    import torch

    if not isinstance(t, torch.Tensor):
        raise TypeError("expected a torch tensor")
    if not t.is_contiguous():
        raise ValueError("tensors must be contiguous")
    return ctypes.c_void_p(t.data_ptr())


class Context:
    """One vk_ctx per GPU (replaces CudaRuntime, src/cuda.rs:356-443)."""

    def __init__(self, device: int = 0, math: int = MATH_F32, stream=None):
        h = ctypes.c_void_p()
        _check(lib().vk_init(device, ctypes.byref(h)))
        self.handle = h
        self.device = device
        self.set_math(math)
        if stream is not None:
            self.set_stream(stream)

    def set_math(self, math: int) -> None:
        _check(lib().vk_set_math(self.handle, math))
        self.math = math

    def set_stream(self, stream) -> None:
        """stream: a torch.cuda.Stream or raw cudaStream_t (int)."""
        raw = getattr(stream, "cuda_stream", stream)
        _check(lib().vk_stream_set(self.handle, ctypes.c_void_p(raw)))

    def synchronize(self) -> None:
        _check(lib().vk_synchronize(self.handle))

    def close(self) -> None:
        if self.handle:
            lib().vk_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default = {}


def default_context(device: int | None = None) -> Context:
    import torch

    dev = torch.cuda.current_device() if device is None else device
    if dev not in _default:
        _default[dev] = Context(dev)
    ctx = _default[dev]
    ctx.set_stream(torch.cuda.current_stream(dev))
    return ctx


def _len(t) -> int:
    return t.numel()


# ---------------------------------------------------------------- src/lib.rs
def qkv_f32_da3_base(input, weight, bias, q, k, v, ctx: Context | None = None) -> bool:
    """src/lib.rs:52.  input [T*768], weight [768*2304], bias [2304] -> q, k, v [12*T*64]."""
    ctx = ctx or default_context()
    t = _len(input) // 768
    if (_len(input) != t * 768 or t == 0 or _len(weight) != 768 * 2304 or _len(bias) != 2304
            or _len(q) != t * 768 or _len(k) != _len(q) or _len(v) != _len(q)):
        return False
    return _check(lib().vk_qkv_f32_da3_base(ctx.handle, t, _ptr(input), _ptr(weight), _ptr(bias),
                                            _ptr(q), _ptr(k), _ptr(v))) == VK_OK


def linear_f32_da3_base(m, n, k, input, weight, output, ctx: Context | None = None) -> bool:
    """src/lib.rs:67."""
    ctx = ctx or default_context()
    if _len(input) != m * k or _len(weight) != k * n or _len(output) != m * n:
        return False
    return _check(lib().vk_linear_f32_da3_base(ctx.handle, m, n, k, _ptr(input), _ptr(weight), _ptr(output))) == VK_OK


def linear_bias_scale_f32_da3_base(m, n, k, a, b, bias, scale, c, ctx: Context | None = None) -> bool:
    """src/lib.rs:94."""
    ctx = ctx or default_context()
    if _len(a) != m * k or _len(b) != k * n or _len(bias) != n or _len(scale) != n or _len(c) != m * n:
        return False
    return _check(lib().vk_linear_bias_scale_f32_da3_base(ctx.handle, m, n, k, _ptr(a), _ptr(b), _ptr(bias),
                                                          _ptr(scale), _ptr(c))) == VK_OK


def flash_attention_f32_da3_base(query, key, value, heads, tokens, output, ctx: Context | None = None) -> bool:
    """src/lib.rs:82."""
    ctx = ctx or default_context()
    n = heads * tokens * 64
    if tokens == 0 or _len(query) != n or _len(key) != n or _len(value) != n or _len(output) != n:
        return False
    return _check(lib().vk_flash_attention_f32_da3_base(ctx.handle, _ptr(query), _ptr(key), _ptr(value), heads,
                                                        tokens, _ptr(output))) == VK_OK


def qk_norm_rope_f32_da3_base(q, k, q_gamma, q_beta, k_gamma, k_beta, positions_yx, frequency, epsilon,
                              heads: int = 12, ctx: Context | None = None) -> bool:
    """src/lib.rs:108; positions_yx is an int64 CUDA tensor [tokens * 2]."""
    ctx = ctx or default_context()
    tokens = _len(positions_yx) // 2
    if (tokens == 0 or _len(q) != heads * tokens * 64 or _len(k) != _len(q)
            or any(_len(x) != 64 for x in (q_gamma, q_beta, k_gamma, k_beta))):
        return False
    return _check(lib().vk_qk_norm_rope_f32_da3_base(ctx.handle, _ptr(q), _ptr(k), heads, tokens, _ptr(q_gamma),
                                                     _ptr(q_beta), _ptr(k_gamma), _ptr(k_beta), _ptr(positions_yx),
                                                     float(frequency), float(epsilon))) == VK_OK


# ---------------------------------------------------------------- generic
def attention(q, k, v, heads, n, head_dim, out, ctx: Context | None = None) -> None:
    """src/attention.rs:66 (panics -> ValueError on length mismatch)."""
    ctx = ctx or default_context()
    for x in (q, k, v, out):
        if _len(x) != heads * n * head_dim:
            raise ValueError("attention: length mismatch")
    if _check(lib().vk_attention(ctx.handle, _ptr(q), _ptr(k), _ptr(v), heads, n, head_dim, _ptr(out))) != VK_OK:
        raise VestraError(VK_UNSUPPORTED_SHAPE, last_error())


def rope2d(x, heads, n, head_dim, pos_yx, freq, ctx: Context | None = None) -> None:
    """src/rope.rs:30."""
    ctx = ctx or default_context()
    if _len(x) != heads * n * head_dim:
        raise ValueError("rope2d: x size mismatch")
    if _len(pos_yx) != n * 2:
        raise ValueError("rope2d: pos_yx size mismatch")
    if head_dim % 4 != 0:
        raise ValueError(f"rope2d: head_dim must be divisible by 4, got {head_dim}")
    _check(lib().vk_rope2d(ctx.handle, _ptr(x), heads, n, head_dim, _ptr(pos_yx), float(freq)))


def layernorm(x, rows, cols, gamma, beta, eps, ctx: Context | None = None) -> None:
    """scalar::layernorm (src/scalar.rs:83)."""
    ctx = ctx or default_context()
    if _len(x) != rows * cols:
        raise ValueError("layernorm: length mismatch")
    _check(lib().vk_layernorm(ctx.handle, _ptr(x), rows, cols, _ptr(gamma), _ptr(beta), float(eps)))


def gelu(x, ctx: Context | None = None) -> None:
    """Kernels::gelu (src/dispatch.rs:56)."""
    ctx = ctx or default_context()
    _check(lib().vk_gelu(ctx.handle, _ptr(x), _len(x)))


def add(dst, src, ctx: Context | None = None) -> None:
    """Kernels::add (src/dispatch.rs:77)."""
    ctx = ctx or default_context()
    if _len(dst) != _len(src):
        raise ValueError("add: length mismatch")
    _check(lib().vk_add(ctx.handle, _ptr(dst), _ptr(src), _len(dst)))


def add_bias_rows(x, rows, cols, bias, ctx: Context | None = None) -> None:
    ctx = ctx or default_context()
    _check(lib().vk_add_bias_rows(ctx.handle, _ptr(x), rows, cols, _ptr(bias)))


def layerscale(x, rows, cols, gamma, ctx: Context | None = None) -> None:
    ctx = ctx or default_context()
    _check(lib().vk_layerscale(ctx.handle, _ptr(x), rows, cols, _ptr(gamma)))


def quantize_row_q8_0(x, out, ctx: Context | None = None) -> None:
    """src/q8_0_dot.rs:27; out is a uint8 CUDA tensor of nblocks * 34 bytes."""
    ctx = ctx or default_context()
    nblocks = _len(out) // 34
    if _len(x) != nblocks * QK8_0:
        raise ValueError("x.len() must be out.len()*QK8_0")
    _check(lib().vk_quantize_row_q8_0(ctx.handle, _ptr(x), nblocks, _ptr(out)))


def gemm_q8_0(m, n, k, a_q, b_q, c, ctx: Context | None = None) -> bool:
    """Kernels::gemm_q8_0 (src/dispatch.rs:91); a_q/b_q uint8 tensors of 34-byte blocks."""
    ctx = ctx or default_context()
    return _check(lib().vk_gemm_q8_0(ctx.handle, m, n, k, _ptr(a_q), _ptr(b_q), _ptr(c))) == VK_OK


def gemm_q8_0_block_dots(m, n, k, a_q, b_q, dots, ctx: Context | None = None) -> bool:
    ctx = ctx or default_context()
    return _check(lib().vk_gemm_q8_0_block_dots(ctx.handle, m, n, k, _ptr(a_q), _ptr(b_q), _ptr(dots))) == VK_OK


# ---------------------------------------------------------------- prepared values
class Linear:
    """Prepared projection (mirrors CudaLinearF32, src/cuda.rs:1291-1334)."""

    def __init__(self, ctx: Context, weight_kn, bias=None, scale=None, math: int = MATH_BF16):
        import numpy as np

        w = np.ascontiguousarray(weight_kn, dtype=np.float32)
        self.k, self.n = w.shape
        keep = [w] + [None if x is None else np.ascontiguousarray(x, dtype=np.float32) for x in (bias, scale)]
        ptrs = [None if x is None else x.ctypes.data_as(ctypes.c_void_p) for x in keep]
        h = ctypes.c_void_p()
        st = _check(lib().vk_prepare_linear(ctx.handle, self.k, self.n, ptrs[0], ptrs[1], ptrs[2], math, ctypes.byref(h)))
        if st != VK_OK:
            raise VestraError(st, last_error())
        self.handle, self.ctx = h, ctx

    def __call__(self, x, out) -> None:
        m = _len(x) // self.k
        _check(lib().vk_linear_run(self.ctx.handle, self.handle, m, _ptr(x), _ptr(out)))

    def __del__(self):
        try:
            if self.handle:
                lib().vk_release_linear(self.handle)
                self.handle = None
        except Exception:
            pass


# ---------------------------------------------------------------- patch embedding
def patchify_nchw_f32(image, height, width, patch, channels, patches, ctx: Context | None = None) -> None:
    """CudaRuntime::patchify_nchw_f32 (src/cuda.rs:1073): image [C, H, W] ->
    patches [(H/p)(W/p), C p p]; invalid shapes raise, as the reference's Err."""
    ctx = ctx or default_context()
    _check(lib().vk_patchify_nchw_f32(ctx.handle, _ptr(image), height, width, patch, channels, _ptr(patches)))


def prepend_cls_add_pos_f32(patches, cls, position, patch_count, embed, tokens, ctx: Context | None = None) -> None:
    """CudaRuntime::prepend_cls_add_pos_f32 (src/cuda.rs:1130): tokens = [cls; patches] + position."""
    ctx = ctx or default_context()
    _check(lib().vk_prepend_cls_add_pos_f32(ctx.handle, _ptr(patches), _ptr(cls), _ptr(position), patch_count, embed,
                                            _ptr(tokens)))


class PatchEmbed:
    """Batched DA3 patch embedding: tokens[b] = [cls; patchify(image[b]) . W + b] + position."""

    def __init__(self, ctx: Context, weight_kn, bias, cls, channels: int, patch: int, math: int = MATH_BF16):
        import numpy as np

        w = np.ascontiguousarray(weight_kn, dtype=np.float32)
        self.k, self.embed = w.shape
        if self.k != channels * patch * patch:
            raise ValueError(f"weight has {self.k} rows, expected channels * patch^2 = {channels * patch * patch}")
        b = np.ascontiguousarray(bias, dtype=np.float32)
        c = np.ascontiguousarray(cls, dtype=np.float32)
        h = ctypes.c_void_p()
        st = _check(lib().vk_patch_embed_prepare(ctx.handle, channels, patch, self.embed,
                                                 w.ctypes.data_as(ctypes.c_void_p), b.ctypes.data_as(ctypes.c_void_p),
                                                 c.ctypes.data_as(ctypes.c_void_p), math, ctypes.byref(h)))
        if st != VK_OK:
            raise VestraError(st, last_error())
        self.handle, self.ctx, self.patch, self.channels = h, ctx, patch, channels

    def __call__(self, images, position, tokens, count: int, height: int, width: int) -> bool:
        """images [count, C, H, W], position [(H/p)(W/p) + 1, E], tokens [count, tokens, E] (CUDA tensors)."""
        return _check(lib().vk_patch_embed_forward(self.ctx.handle, self.handle, count, height, width, _ptr(images),
                                                   _ptr(position), _ptr(tokens))) == VK_OK

    def __del__(self):
        try:
            if self.handle:
                lib().vk_patch_embed_release(self.handle)
                self.handle = None
        except Exception:
            pass


# ---------------------------------------------------------------- DPT head consumers

def token_to_chw_f32(token_major, tokens: int, channels: int, chw, ctx: Context | None = None) -> None:
    """CudaRuntime::token_to_chw_f32 (src/cuda.rs:1032-1068): [tokens, channels] -> [channels, tokens];
    zero sizes raise, as the reference's LengthMismatch."""
    ctx = ctx or default_context()
    _check(lib().vk_token_to_chw_f32(ctx.handle, _ptr(token_major), tokens, channels, _ptr(chw)))


def token_to_chw_batched(token_major, images: int, tokens: int, channels: int, chw,
                         ctx: Context | None = None) -> None:
    """`images` token-major matrices back to back -> `images` CHW maps."""
    ctx = ctx or default_context()
    _check(lib().vk_token_to_chw_f32_batched(ctx.handle, _ptr(token_major), images, tokens, channels, _ptr(chw)))


def bilinear_resize(x, c: int, ih: int, iw: int, oh: int, ow: int, out, ctx: Context | None = None) -> None:
    """resample::bilinear_resize (src/resample.rs:10): half-pixel centres, clamp to edge."""
    ctx = ctx or default_context()
    _check(lib().vk_bilinear_resize_f32(ctx.handle, _ptr(x), c, ih, iw, oh, ow, _ptr(out)))


def bilinear_resize_align_corners(x, c: int, ih: int, iw: int, oh: int, ow: int, out,
                                  ctx: Context | None = None) -> None:
    """resample::bilinear_resize_align_corners (src/resample.rs:184)."""
    ctx = ctx or default_context()
    _check(lib().vk_bilinear_resize_align_corners_f32(ctx.handle, _ptr(x), c, ih, iw, oh, ow, _ptr(out)))


class WinogradF2Filter:
    """prepare_winograd_f2_filter (src/conv.rs:175): an OIHW [out_c, in_c, 3, 3]
    filter transformed once to U [16, in_c, out_c] on the device."""

    def __init__(self, ctx: Context, weight, in_c: int, out_c: int, math: int = MATH_F32):
        """math: MATH_F32 (the reference's f32 Winograd arithmetic on the SIMT cores) or MATH_BF16 (the
        convolution as an implicit GEMM on the tensor cores, bf16 operands, f32 accumulation)."""
        import numpy as np

        w = np.ascontiguousarray(weight, dtype=np.float32)
        if w.size != out_c * in_c * 9:
            raise ValueError(f"weight has {w.size} values, expected out_c * in_c * 9 = {out_c * in_c * 9}")
        h = ctypes.c_void_p()
        st = _check(lib().vk_conv3x3_prepare_math(ctx.handle, w.ctypes.data_as(ctypes.c_void_p), in_c, out_c, math,
                                                  ctypes.byref(h)))
        if st != VK_OK:
            raise VestraError(st, last_error())
        self.handle, self.ctx, self.in_c, self.out_c = h, ctx, in_c, out_c

    def __del__(self):
        try:
            if self.handle:
                lib().vk_conv3x3_release(self.handle)
                self.handle = None
        except Exception:
            pass


def conv3x3_winograd_f2_prepared(x, in_c: int, ih: int, iw: int, filt: WinogradF2Filter, out_c: int, bias, out,
                                 relu_input: bool = False, ctx: Context | None = None) -> None:
    """conv3x3_winograd_f2_prepared / _prepared_relu_input (src/conv.rs:282, 667): stride 1, pad 1."""
    ctx = ctx or filt.ctx
    _check(lib().vk_conv3x3_forward(ctx.handle, filt.handle, _ptr(x), in_c, ih, iw, out_c, _ptr(bias),
                                    int(relu_input), _ptr(out)))


def conv3x3_winograd_f2_prepared_resize_align_corners(x, in_c: int, ih: int, iw: int, oh: int, ow: int, add,
                                                      filt: WinogradF2Filter, out_c: int, bias, out,
                                                      ctx: Context | None = None) -> None:
    """conv3x3_winograd_f2_prepared_resize_align_corners (src/conv.rs:304): resize + add fused into the conv."""
    ctx = ctx or filt.ctx
    _check(lib().vk_conv3x3_resize_ac_forward(ctx.handle, filt.handle, _ptr(x), in_c, ih, iw, oh, ow, _ptr(add),
                                              out_c, _ptr(bias), _ptr(out)))


def conv3x3_batched(x, images: int, ih: int, iw: int, filt: WinogradF2Filter, bias, out, relu_input: bool = False,
                    resize_to=None, add=None, ctx: Context | None = None) -> None:
    """`images` convolutions back to back; resize_to=(oh, ow) fuses the align-corners resize (+ shared add)."""
    ctx = ctx or filt.ctx
    if resize_to is None:
        _check(lib().vk_conv3x3_forward_batched(ctx.handle, filt.handle, images, _ptr(x), ih, iw, _ptr(bias),
                                                int(relu_input), _ptr(out)))
    else:
        oh, ow = resize_to
        _check(lib().vk_conv3x3_resize_ac_forward_batched(ctx.handle, filt.handle, images, _ptr(x), ih, iw, oh, ow,
                                                          _ptr(add), _ptr(bias), _ptr(out)))


class _LayerWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "ln1_gamma", "ln1_beta", "qkv_weight", "qkv_bias", "proj_weight", "proj_bias", "ls1",
        "ln2_gamma", "ln2_beta", "fc1_weight", "fc1_bias", "fc2_weight", "fc2_bias", "ls2",
        "q_norm_gamma", "q_norm_beta", "k_norm_gamma", "k_norm_beta")]


class _EncoderConfig(ctypes.Structure):
    _fields_ = [("layers", ctypes.c_int), ("heads", ctypes.c_int), ("ffn", ctypes.c_int),
                ("eps", ctypes.c_float), ("rope_freq", ctypes.c_float), ("math", ctypes.c_int),
                ("views", ctypes.c_int), ("global_layers", ctypes.c_uint64)]


LAYER_KEYS = ["ln1_g", "ln1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "ls1",
              "ln2_g", "ln2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "ls2"]
# optional per layer: Q/K LayerNorm before RoPE ([64] each; all four or none)
QK_NORM_KEYS = ["q_norm_g", "q_norm_b", "k_norm_g", "k_norm_b"]


class Encoder:
    """DA3-BASE ViT encoder (vk_encoder_*); layers are dicts of host f32 arrays
    keyed by LAYER_KEYS in the reference layout ([K, N] weights)."""

    def __init__(self, ctx: Context, layers, heads: int = 12, ffn: int = 3072, eps: float = 1e-6,
                 rope_freq: float = 100.0, math: int = MATH_BF16, views: int = 1, global_layers=()):
        """views / global_layers: layers listed in global_layers attend across
        each group of `views` consecutive images (multi-view global attention)."""
        import numpy as np

        self.ctx = ctx
        self.math = math
        self.embed = heads * 64
        keep, structs = [], (_LayerWeights * len(layers))()
        for i, layer in enumerate(layers):
            vals = [np.ascontiguousarray(layer[kk], dtype=np.float32) for kk in LAYER_KEYS]
            vals += [None if layer.get(kk) is None else np.ascontiguousarray(layer[kk], dtype=np.float32)
                     for kk in QK_NORM_KEYS]
            keep.append(vals)
            for fname, arr in zip((f for f, _ in _LayerWeights._fields_), vals):
                setattr(structs[i], fname, None if arr is None else arr.ctypes.data)
        mask = 0
        for li in global_layers:
            if not 0 <= li < min(len(layers), 64):
                raise ValueError(f"global layer {li} outside 0..{len(layers) - 1}")
            mask |= 1 << li
        cfg = _EncoderConfig(len(layers), heads, ffn, eps, rope_freq, math, views, mask)
        h = ctypes.c_void_p()
        st = _check(lib().vk_encoder_prepare(ctx.handle, ctypes.byref(cfg), structs, ctypes.byref(h)))
        if st != VK_OK:
            raise VestraError(st, last_error())
        self.handle = h

    def forward(self, tokens, out, images: int, grid_h: int, grid_w: int) -> bool:
        """Device tensors [images, 1 + grid_h * grid_w, E] f32 (may alias); False
        (output untouched) for an unsupported shape."""
        return _check(lib().vk_encoder_forward(self.ctx.handle, self.handle, images, grid_h, grid_w, _ptr(tokens),
                                               _ptr(out))) == VK_OK

    def forward_host(self, tokens, out, images: int, grid_h: int, grid_w: int) -> None:
        """Host tensors (pinned for overlap); copies are pipelined with compute."""
        _check(lib().vk_encoder_forward_host(self.ctx.handle, self.handle, images, grid_h, grid_w,
                                             ctypes.c_void_p(tokens.data_ptr()), ctypes.c_void_p(out.data_ptr())))

    def forward_host_async(self, tokens, out, images: int, grid_h: int, grid_w: int) -> None:
        """forward_host without waiting: `out` is complete after ctx.synchronize()
        (or later work on the context stream); back-to-back calls overlap."""
        _check(lib().vk_encoder_forward_host_async(self.ctx.handle, self.handle, images, grid_h, grid_w,
                                                   ctypes.c_void_p(tokens.data_ptr()),
                                                   ctypes.c_void_p(out.data_ptr())))

    def profile(self, tokens, out, images: int, grid_h: int, grid_w: int):
        """Per-kernel device ms of one eager forward, summed over blocks."""
        ms = (ctypes.c_float * 16)()
        _check(lib().vk_encoder_profile(self.ctx.handle, self.handle, images, grid_h, grid_w, _ptr(tokens),
                                        _ptr(out), ms, 16))
        n = 10 if self.math == MATH_F32 else 7
        return [float(ms[i]) for i in range(n)]

    def last_launches(self) -> int:
        return int(lib().vk_encoder_last_launches(self.handle))

    def __del__(self):
        try:
            if self.handle:
                lib().vk_encoder_release(self.handle)
                self.handle = None
        except Exception:
            pass
