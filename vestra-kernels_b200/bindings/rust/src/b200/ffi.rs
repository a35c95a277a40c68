//! Raw declarations of include/vestra_b200.h, one per C entry point, in the
//! header's order and argument names.  `BlockQ8_0` is the crate's own
//! `#[repr(C)] { d: f16, qs: [i8; 32] }` (src/lib.rs:33-38), 34 bytes, which
//! is `vk_block_q8_0` byte for byte (tests/abi_layout.c asserts the C side).
#![allow(non_camel_case_types, dead_code)]
use core::ffi::{c_char, c_int, c_void};

use crate::BlockQ8_0;

pub const VK_OK: c_int = 0;
pub const VK_UNSUPPORTED_SHAPE: c_int = 1;
pub const VK_ERR_INVALID_ARGUMENT: c_int = 2;
pub const VK_ERR_CUDA: c_int = 3;
pub const VK_ERR_TIMEOUT: c_int = 4;
pub const VK_ERR_NO_DEVICE: c_int = 5;
pub const VK_ERR_OUT_OF_MEMORY: c_int = 6;

pub const VK_MATH_F32: c_int = 0;
pub const VK_MATH_BF16: c_int = 1;
pub const VK_MATH_Q8_0: c_int = 2;

#[repr(C)]
pub struct VkCtx { _p: [u8; 0] }
#[repr(C)]
pub struct VkLinear { _p: [u8; 0] }
#[repr(C)]
pub struct VkEncoder { _p: [u8; 0] }
#[repr(C)]
pub struct VkConv3x3 { _p: [u8; 0] }
#[repr(C)]
pub struct VkPatchEmbed { _p: [u8; 0] }

/// vk_layer_weights: host f32 arrays of one block, [K, N] weights.
#[repr(C)]
pub struct VkLayerWeights {
    pub ln1_gamma: *const f32, pub ln1_beta: *const f32,
    pub qkv_weight: *const f32, pub qkv_bias: *const f32,
    pub proj_weight: *const f32, pub proj_bias: *const f32, pub ls1: *const f32,
    pub ln2_gamma: *const f32, pub ln2_beta: *const f32,
    pub fc1_weight: *const f32, pub fc1_bias: *const f32,
    pub fc2_weight: *const f32, pub fc2_bias: *const f32, pub ls2: *const f32,
    /// NULL unless the block LayerNorms q / k before RoPE
    pub q_norm_gamma: *const f32, pub q_norm_beta: *const f32,
    pub k_norm_gamma: *const f32, pub k_norm_beta: *const f32,
}

/// vk_encoder_config (40 bytes: global_layers at offset 32).
#[repr(C)]
pub struct VkEncoderConfig {
    pub layers: c_int,
    pub heads: c_int,
    pub ffn: c_int,
    pub eps: f32,
    pub rope_freq: f32,
    pub math: c_int,
    pub views: c_int,
    pub global_layers: u64,
}

extern "C" {
    pub fn vk_init(device: c_int, out: *mut *mut VkCtx) -> c_int;
    pub fn vk_destroy(ctx: *mut VkCtx) -> c_int;
    pub fn vk_stream_set(ctx: *mut VkCtx, stream: *mut c_void) -> c_int;
    pub fn vk_set_math(ctx: *mut VkCtx, math: c_int) -> c_int;
    pub fn vk_synchronize(ctx: *mut VkCtx) -> c_int;
    pub fn vk_last_error() -> *const c_char;
    pub fn vk_version() -> *const c_char;
    pub fn vk_qkv_f32_da3_base(ctx: *mut VkCtx, tokens: usize, input: *const f32, weight: *const f32, bias: *const f32, q: *mut f32, k: *mut f32, v: *mut f32) -> c_int;
    pub fn vk_linear_f32_da3_base(ctx: *mut VkCtx, m: usize, n: usize, k: usize, input: *const f32, weight: *const f32, output: *mut f32) -> c_int;
    pub fn vk_linear_bias_scale_f32_da3_base(ctx: *mut VkCtx, m: usize, n: usize, k: usize, a: *const f32, b: *const f32, bias: *const f32, scale: *const f32, c: *mut f32) -> c_int;
    pub fn vk_flash_attention_f32_da3_base(ctx: *mut VkCtx, query: *const f32, key: *const f32, value: *const f32, heads: usize, tokens: usize, output: *mut f32) -> c_int;
    pub fn vk_qk_norm_rope_f32_da3_base(ctx: *mut VkCtx, q: *mut f32, k: *mut f32, heads: usize, tokens: usize, q_gamma: *const f32, q_beta: *const f32, k_gamma: *const f32, k_beta: *const f32, positions_yx: *const i64, frequency: f32, epsilon: f32) -> c_int;
    pub fn vk_attention(ctx: *mut VkCtx, q: *const f32, k: *const f32, v: *const f32, heads: usize, n: usize, head_dim: usize, out: *mut f32) -> c_int;
    pub fn vk_rope2d(ctx: *mut VkCtx, x: *mut f32, heads: usize, n: usize, head_dim: usize, pos_yx: *const i64, freq: f32) -> c_int;
    pub fn vk_layernorm(ctx: *mut VkCtx, x: *mut f32, rows: usize, cols: usize, gamma: *const f32, beta: *const f32, eps: f32) -> c_int;
    pub fn vk_gelu(ctx: *mut VkCtx, x: *mut f32, n: usize) -> c_int;
    pub fn vk_add(ctx: *mut VkCtx, dst: *mut f32, src: *const f32, n: usize) -> c_int;
    pub fn vk_add_bias_rows(ctx: *mut VkCtx, x: *mut f32, rows: usize, cols: usize, bias: *const f32) -> c_int;
    pub fn vk_layerscale(ctx: *mut VkCtx, x: *mut f32, rows: usize, cols: usize, gamma: *const f32) -> c_int;
    pub fn vk_quantize_row_q8_0(ctx: *mut VkCtx, x: *const f32, nblocks: usize, out: *mut BlockQ8_0) -> c_int;
    pub fn vk_gemm_q8_0(ctx: *mut VkCtx, m: usize, n: usize, k: usize, a_q: *const BlockQ8_0, b_q: *const BlockQ8_0, c: *mut f32) -> c_int;
    pub fn vk_gemm_q8_0_block_dots(ctx: *mut VkCtx, m: usize, n: usize, k: usize, a_q: *const BlockQ8_0, b_q: *const BlockQ8_0, dots: *mut i32) -> c_int;
    pub fn vk_gemm_q8_0_noalloc(stream: *mut c_void, m: usize, n: usize, k: usize, a_q: *const BlockQ8_0, b_q: *const BlockQ8_0, c: *mut f32) -> c_int;
    pub fn vk_patchify_nchw_f32(ctx: *mut VkCtx, image: *const f32, height: usize, width: usize, patch: usize, channels: usize, patches: *mut f32) -> c_int;
    pub fn vk_prepend_cls_add_pos_f32(ctx: *mut VkCtx, patches: *const f32, cls: *const f32, position: *const f32, patch_count: usize, embed: usize, tokens: *mut f32) -> c_int;
    pub fn vk_patch_embed_prepare(ctx: *mut VkCtx, channels: usize, patch: usize, embed: usize, weight_host: *const f32, bias_host: *const f32, cls_host: *const f32, math: c_int, out: *mut *mut VkPatchEmbed) -> c_int;
    pub fn vk_patch_embed_forward(ctx: *mut VkCtx, pe: *const VkPatchEmbed, images: usize, height: usize, width: usize, images_dev: *const f32, position_dev: *const f32, tokens_dev: *mut f32) -> c_int;
    pub fn vk_patch_embed_release(pe: *mut VkPatchEmbed) -> c_int;
    pub fn vk_prepare_linear(ctx: *mut VkCtx, k: usize, n: usize, weight_host: *const f32, bias_host: *const f32, scale_host: *const f32, math: c_int, out: *mut *mut VkLinear) -> c_int;
    pub fn vk_prepare_linear_q8_0(ctx: *mut VkCtx, k: usize, n: usize, blocks_host: *const BlockQ8_0, bias_host: *const f32, scale_host: *const f32, out: *mut *mut VkLinear) -> c_int;
    pub fn vk_linear_run(ctx: *mut VkCtx, lin: *const VkLinear, m: usize, input: *const f32, output: *mut f32) -> c_int;
    pub fn vk_release_linear(lin: *mut VkLinear) -> c_int;
    pub fn vk_encoder_prepare(ctx: *mut VkCtx, cfg: *const VkEncoderConfig, layers_host: *const VkLayerWeights, out: *mut *mut VkEncoder) -> c_int;
    pub fn vk_encoder_forward(ctx: *mut VkCtx, enc: *mut VkEncoder, images: usize, grid_h: usize, grid_w: usize, tokens_dev: *const f32, out_dev: *mut f32) -> c_int;
    pub fn vk_encoder_forward_host(ctx: *mut VkCtx, enc: *mut VkEncoder, images: usize, grid_h: usize, grid_w: usize, tokens_host: *const f32, out_host: *mut f32) -> c_int;
    pub fn vk_encoder_forward_host_async(ctx: *mut VkCtx, enc: *mut VkEncoder, images: usize, grid_h: usize, grid_w: usize, tokens_host: *const f32, out_host: *mut f32) -> c_int;
    pub fn vk_encoder_profile(ctx: *mut VkCtx, enc: *mut VkEncoder, images: usize, grid_h: usize, grid_w: usize, tokens_dev: *const f32, out_dev: *mut f32, ms_per_slot: *mut f32, slots: c_int) -> c_int;
    pub fn vk_encoder_last_launches(enc: *const VkEncoder) -> c_int;
    pub fn vk_encoder_release(enc: *mut VkEncoder) -> c_int;
    pub fn vk_token_to_chw_f32(ctx: *mut VkCtx, token_major: *const f32, tokens: usize, channels: usize, chw: *mut f32) -> c_int;
    pub fn vk_token_to_chw_f32_batched(ctx: *mut VkCtx, token_major: *const f32, images: usize, tokens: usize, channels: usize, chw: *mut f32) -> c_int;
    pub fn vk_bilinear_resize_f32(ctx: *mut VkCtx, input: *const f32, c: usize, ih: usize, iw: usize, oh: usize, ow: usize, out: *mut f32) -> c_int;
    pub fn vk_bilinear_resize_align_corners_f32(ctx: *mut VkCtx, input: *const f32, c: usize, ih: usize, iw: usize, oh: usize, ow: usize, out: *mut f32) -> c_int;
    pub fn vk_conv3x3_prepare(ctx: *mut VkCtx, weight_host: *const f32, in_c: usize, out_c: usize, out: *mut *mut VkConv3x3) -> c_int;
    pub fn vk_conv3x3_prepare_math(ctx: *mut VkCtx, weight_host: *const f32, in_c: usize, out_c: usize, math: c_int, out: *mut *mut VkConv3x3) -> c_int;
    pub fn vk_conv3x3_forward(ctx: *mut VkCtx, conv: *const VkConv3x3, input: *const f32, in_c: usize, ih: usize, iw: usize, out_c: usize, bias: *const f32, relu_input: c_int, out: *mut f32) -> c_int;
    pub fn vk_conv3x3_resize_ac_forward(ctx: *mut VkCtx, conv: *const VkConv3x3, input: *const f32, in_c: usize, ih: usize, iw: usize, oh: usize, ow: usize, add: *const f32, out_c: usize, bias: *const f32, out: *mut f32) -> c_int;
    pub fn vk_conv3x3_forward_batched(ctx: *mut VkCtx, conv: *const VkConv3x3, images: usize, input: *const f32, ih: usize, iw: usize, bias: *const f32, relu_input: c_int, out: *mut f32) -> c_int;
    pub fn vk_conv3x3_resize_ac_forward_batched(ctx: *mut VkCtx, conv: *const VkConv3x3, images: usize, input: *const f32, ih: usize, iw: usize, oh: usize, ow: usize, add: *const f32, bias: *const f32, out: *mut f32) -> c_int;
    pub fn vk_conv3x3_release(conv: *mut VkConv3x3) -> c_int;
}
