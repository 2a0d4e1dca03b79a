// Host-side probe of the product's fp16 conversions (mini_ai_b200/csrc/mq_common.cuh):
// f32_to_f16_rne and f16_to_f32, the same inline functions the quantizer and
// the kernels' host paths use, exported over a range of inputs so a CPU test
// can compare them with the reference build over every input. Test support
// only: compiled by tests/test_fp16_product.py into a temporary directory.
#include "mq_common.cuh"

extern "C" {

void probe_f32_to_f16_range(uint32_t start, uint16_t *dst, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = mq::f32_to_f16_rne(mq::bits_f32(start + (uint32_t)i));
}

void probe_f16_to_f32_all(float *dst) {
  for (uint32_t h = 0; h < 65536u; ++h) dst[h] = mq::f16_to_f32((uint16_t)h);
}

}  // extern "C"
