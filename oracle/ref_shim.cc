// ORACLE — test infrastructure only.
//
// extern "C" wrapper around the reference's own, unmodified C++ sources for
// the quantized-linear path, compiled in place by oracle/Makefile:
//   src/quantized_tensor.cc  QuantizeTensor / DequantizeTensor / HalfToFloat /
//                            FloatToHalf / TensorFromQuantized / QuantizedDotRow
//   src/matmul_optimized.cc  LinearDispatch (kThreadedSimd), SetMatmulThreads
//   src/thread_pool.cc, src/tensor.cc
// Used to pin the C restatement (oracle/mq_oracle.c), to generate the golden
// fixtures under tests/golden/, and as the timed CPU baseline.
#include "mini_llama/matmul_dispatch.h"
#include "mini_llama/quantized_tensor.h"
#include "mini_llama/tensor.h"

#include <cstdint>
#include <cstring>
#include <exception>
#include <string>

using namespace mini_llama;

namespace {
thread_local std::string g_error;

int Fail(const std::exception &e) {
  g_error = e.what();
  return -1;
}

Tensor WrapPacked(int qtype, const uint8_t *blocks, size_t nbytes, int rows, int cols) {
  std::vector<uint8_t> bytes(blocks, blocks + nbytes);
  return TensorFromQuantized(std::move(bytes), rows, cols, static_cast<QuantType>(qtype));
}
}  // namespace

extern "C" {

const char *ref_last_error() { return g_error.c_str(); }

float ref_half_to_float(uint16_t h) { return HalfToFloat(h); }
uint16_t ref_float_to_half(float f) { return FloatToHalf(f); }

void ref_float_to_half_range(uint32_t start, uint16_t *dst, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    const uint32_t bits = start + static_cast<uint32_t>(i);
    float f;
    std::memcpy(&f, &bits, 4);
    dst[i] = FloatToHalf(f);
  }
}

void ref_half_to_float_batch(const uint16_t *src, float *dst, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = HalfToFloat(src[i]);
}

// QuantizeTensor on a rows x cols F32 matrix; dst receives the packed blocks.
int ref_quantize(int qtype, const float *src, int rows, int cols, uint8_t *dst, size_t dst_bytes) {
  try {
    Tensor t({rows, cols});
    std::memcpy(t.data.data(), src, sizeof(float) * static_cast<size_t>(rows) * cols);
    const Tensor q = QuantizeTensor(t, static_cast<QuantType>(qtype));
    if (q.quantized->bytes.size() != dst_bytes) {
      g_error = "destination size mismatch";
      return -3;
    }
    std::memcpy(dst, q.quantized->bytes.data(), dst_bytes);
    return 0;
  } catch (const std::exception &e) {
    return Fail(e);
  }
}

int ref_dequantize(int qtype, const uint8_t *blocks, size_t nbytes, int rows, int cols, float *dst) {
  try {
    const Tensor d = DequantizeTensor(WrapPacked(qtype, blocks, nbytes, rows, cols));
    std::memcpy(dst, d.data.data(), sizeof(float) * d.data.size());
    return 0;
  } catch (const std::exception &e) {
    return Fail(e);
  }
}

// y[m] = LinearDispatch(x[m], W, kThreadedSimd) for each of the m activation
// rows, with SetMatmulThreads(threads). The packed weight is wrapped once.
struct RefWeight {
  Tensor w;
};

void *ref_weight_create(int qtype, const uint8_t *blocks, size_t nbytes, int rows, int cols) {
  try {
    return new RefWeight{WrapPacked(qtype, blocks, nbytes, rows, cols)};
  } catch (const std::exception &e) {
    Fail(e);
    return nullptr;
  }
}

void ref_weight_destroy(void *w) { delete static_cast<RefWeight *>(w); }

int ref_set_threads(unsigned threads) {
  try {
    SetMatmulThreads(threads);
    return 0;
  } catch (const std::exception &e) {
    return Fail(e);
  }
}

int ref_linear(void *handle, const float *x, int m, int ldx, float *y, int ldy) {
  try {
    const Tensor &w = static_cast<RefWeight *>(handle)->w;
    const int cols = w.shape[1], rows = w.shape[0];
    Tensor xin({cols});
    for (int i = 0; i < m; ++i) {
      std::memcpy(xin.data.data(), x + static_cast<size_t>(i) * ldx, sizeof(float) * cols);
      const Tensor out = LinearDispatch(xin, w, MatmulMode::kThreadedSimd);
      std::memcpy(y + static_cast<size_t>(i) * ldy, out.data.data(), sizeof(float) * rows);
    }
    return 0;
  } catch (const std::exception &e) {
    return Fail(e);
  }
}

float ref_dot_row(int qtype, const uint8_t *blocks, size_t nbytes, int rows, int cols, int row, const float *x) {
  try {
    const Tensor w = WrapPacked(qtype, blocks, nbytes, rows, cols);
    return QuantizedDotRow(*w.quantized, row, x);
  } catch (const std::exception &e) {
    Fail(e);
    return 0.0f;
  }
}

}  // extern "C"
