/* Layout of the C-ABI records that the Rust binding
 * (vestra-kernels_b200/bindings/rust/src/b200/ffi.rs) mirrors with
 * #[repr(C)] structs: BlockQ8_0 (src/lib.rs:33-38) is 34 packed bytes, the
 * layer weights 18 pointers, the encoder config 40 bytes.  Compiled and run
 * by tests/test_rust_binding.py; exits non-zero on a mismatch. */
#include <stddef.h>
#include <stdio.h>

#include "vestra_b200.h"

#define CHECK(cond)                                          \
  do {                                                       \
    if (!(cond)) {                                           \
      fprintf(stderr, "layout check failed: %s\n", #cond);   \
      return 1;                                              \
    }                                                        \
  } while (0)

int main(void) {
  CHECK(sizeof(vk_block_q8_0) == 34);
  CHECK(offsetof(vk_block_q8_0, d) == 0);
  CHECK(offsetof(vk_block_q8_0, qs) == 2);
  CHECK(sizeof(vk_layer_weights) == 18 * sizeof(void*));
  CHECK(offsetof(vk_layer_weights, ln1_gamma) == 0 * sizeof(void*));
  CHECK(offsetof(vk_layer_weights, qkv_weight) == 2 * sizeof(void*));
  CHECK(offsetof(vk_layer_weights, ls1) == 6 * sizeof(void*));
  CHECK(offsetof(vk_layer_weights, fc2_bias) == 12 * sizeof(void*));
  CHECK(offsetof(vk_layer_weights, ls2) == 13 * sizeof(void*));
  CHECK(offsetof(vk_layer_weights, q_norm_gamma) == 14 * sizeof(void*));
  CHECK(offsetof(vk_layer_weights, k_norm_beta) == 17 * sizeof(void*));
  CHECK(sizeof(vk_encoder_config) == 40);
  CHECK(offsetof(vk_encoder_config, layers) == 0);
  CHECK(offsetof(vk_encoder_config, heads) == 4);
  CHECK(offsetof(vk_encoder_config, ffn) == 8);
  CHECK(offsetof(vk_encoder_config, eps) == 12);
  CHECK(offsetof(vk_encoder_config, rope_freq) == 16);
  CHECK(offsetof(vk_encoder_config, math) == 20);
  CHECK(offsetof(vk_encoder_config, views) == 24);
  CHECK(offsetof(vk_encoder_config, global_layers) == 32);
  printf("abi layout ok\n");
  return 0;
}
