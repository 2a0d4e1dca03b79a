/*
 * ORACLE — test infrastructure only, never part of the product path.
 *
 * Plain-C restatement of mini_ai's CPU quantized-linear path (GGUF Q8_0 /
 * Q4_0 / Q4_1 block packing, decoding and the per-row block dot product).
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this file's shared library, and only to check or time against it.
 *
 * Parity pins:
 *   - the .npz files under tests/golden hold outputs of the reference's own C++ sources
 *     (src/quantized_tensor.cc, src/matmul_optimized.cc) built by
 *     oracle/Makefile, plus the reference test-suite known-answer vectors
 *     (tests/test_compute.cc:54-68);
 *   - tests/test_oracle.py compares this file against those fixtures and,
 *     where the reference build is present, exhaustively over fp16/fp32.
 *
 * Each function cites the reference lines it restates (paths relative to
 * the mini_ai project root). Build with -ffp-contract=off: the reference
 * accumulates with separate fp32 multiply and add (no FMA), and parity on
 * the CPU side is bit-exact.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_OK 0
#define ORACLE_ERR_INVALID (-1)
#define ORACLE_ERR_SIZE (-3)
#define ORACLE_ERR_NONFINITE (-4)
#define ORACLE_ERR_RANGE (-5)

/* GGML type ids: include/mini_llama/quantized_tensor.h:10 (== gguf.h:15-17). */
enum { Q8_0 = 8, Q4_0 = 2, Q4_1 = 3 };

/* Bytes per 32-weight block: src/quantized_tensor.cc:13-23. */
size_t oracle_block_bytes(int qtype) {
  switch (qtype) {
  case Q8_0: return 34; /* fp16 d + 32 x int8 */
  case Q4_0: return 18; /* fp16 d + 16 bytes of nibbles */
  case Q4_1: return 20; /* fp16 d + fp16 m + 16 bytes of nibbles */
  default: return 0;
  }
}

size_t oracle_quantized_bytes(int qtype, int rows, int cols) {
  const size_t bb = oracle_block_bytes(qtype);
  if (!bb || rows <= 0 || cols <= 0) return 0;
  return (size_t)rows * (((size_t)cols + 31) / 32) * bb;
}

static float bits_to_float(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t float_to_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/*
 * fp16 -> fp32, exact: src/quantized_tensor.cc:46-55.
 * The reference returns a positive quiet NaN for every NaN input and scales
 * subnormals by 2^-24; both are reproduced here by building the fp32 bits.
 */
float oracle_half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 31u;
  const uint32_t frac = h & 1023u;
  if (exp == 31) return frac ? bits_to_float(0x7fc00000u) : bits_to_float(sign | 0x7f800000u);
  if (exp == 0) {
    /* frac * 2^-24 is exact in fp32 (frac < 2^10). */
    const float mag = (float)frac * 5.9604644775390625e-8f;
    return bits_to_float(float_to_bits(mag) | sign);
  }
  return bits_to_float(sign | ((exp - 15 + 127) << 23) | (frac << 13));
}

/*
 * fp32 -> fp16 with round-to-nearest-even: src/quantized_tensor.cc:57-86.
 * NaN keeps its sign and becomes 0x7e00; overflow saturates to infinity;
 * magnitudes below 2^-25 flush to signed zero.
 */
uint16_t oracle_float_to_half(float f) {
  const uint32_t b = float_to_bits(f);
  const uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
  const uint32_t e8 = (b >> 23) & 255u;
  uint32_t man = b & 0x7fffffu;
  if (e8 == 255) return sign | (man ? 0x7e00u : 0x7c00u);
  const int e = (int)e8 - 112; /* rebias 127 -> 15 */
  if (e >= 31) return sign | 0x7c00u;
  if (e <= 0) {
    if (e < -10) return sign;
    /* subnormal half: shift the 24-bit significand right by 14 - e. */
    const uint32_t sig = man | 0x800000u;
    const int sh = 14 - e;
    const uint32_t q = sig >> sh, rem = sig & ((1u << sh) - 1u), half = 1u << (sh - 1);
    const uint32_t r = q + ((rem > half) || (rem == half && (q & 1u)));
    return sign | (uint16_t)r; /* a carry into bit 10 yields the smallest normal */
  }
  /* normal half: keep 10 of the 23 mantissa bits, round to nearest even. */
  const uint32_t q = man >> 13, rem = man & 0x1fffu;
  uint32_t r = q + ((rem > 0x1000u) || (rem == 0x1000u && (q & 1u)));
  uint32_t ee = (uint32_t)e;
  if (r == 1024u) { r = 0; ++ee; }
  if (ee >= 31) return sign | 0x7c00u;
  return sign | (uint16_t)(ee << 10) | (uint16_t)r;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void wr16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)(v & 255); p[1] = (uint8_t)(v >> 8); }

/* std::round: half away from zero (src/quantized_tensor.cc:146). */
static int round_half_away(float v) { return (int)roundf(v); }

/*
 * Pack one 32-slot block. Restates the inner body of QuantizeTensor,
 * src/quantized_tensor.cc:114-155:
 *  - slots past `n` are zero (values[32] = {} at :115);
 *  - min, max and the signed absolute maximum start at 0 (:116), so a Q4_1
 *    block always satisfies min <= 0 <= max, and the signed maximum keeps
 *    the FIRST element of largest magnitude (strict '>' at :124);
 *  - the scale is stored as fp16 and read back before use (:132-133);
 *  - q = scale == 0 ? 0 : round((v - offset) / scale) for all 32 slots.
 */
static int quantize_block(int qtype, const float *src, int n, uint8_t *blk) {
  float v[32] = {0};
  float mn = 0.0f, mx = 0.0f, smax = 0.0f;
  for (int i = 0; i < n; ++i) {
    const float x = src[i];
    if (!isfinite(x)) return ORACLE_ERR_NONFINITE;
    v[i] = x;
    mn = (x < mn) ? x : mn; /* std::min(mn, x) */
    mx = (mx < x) ? x : mx; /* std::max(mx, x) */
    if (fabsf(x) > fabsf(smax)) smax = x;
  }
  const size_t bb = oracle_block_bytes(qtype);
  memset(blk, 0, bb);
  float d = qtype == Q8_0 ? fabsf(smax) / 127.0f : qtype == Q4_0 ? smax / -8.0f : (mx - mn) / 15.0f;
  wr16(blk, oracle_float_to_half(d));
  d = oracle_half_to_float(rd16(blk));
  if (!isfinite(d)) return ORACLE_ERR_RANGE;
  float m = 0.0f;
  if (qtype == Q4_1) {
    wr16(blk + 2, oracle_float_to_half(mn));
    m = oracle_half_to_float(rd16(blk + 2));
    if (!isfinite(m)) return ORACLE_ERR_RANGE;
  }
  for (int i = 0; i < 32; ++i) {
    int q = d == 0.0f ? 0 : round_half_away((v[i] - m) / d);
    if (qtype == Q8_0) {
      q = q < -127 ? -127 : q > 127 ? 127 : q;
      blk[2 + i] = (uint8_t)(int8_t)q;
    } else {
      q = qtype == Q4_0 ? q + 8 : q;
      q = q < 0 ? 0 : q > 15 ? 15 : q;
      const int base = qtype == Q4_1 ? 4 : 2;
      blk[base + (i & 15)] |= (uint8_t)(q << (i < 16 ? 0 : 4));
    }
  }
  return ORACLE_OK;
}

/* QuantizeTensor: src/quantized_tensor.cc:104-159 (row-major, row r block b
 * at (r * ceil(cols/32) + b) * BlockBytes). Returns 0 or a negative code. */
int oracle_quantize(int qtype, const float *src, int rows, int cols, uint8_t *dst, size_t dst_bytes) {
  const size_t need = oracle_quantized_bytes(qtype, rows, cols);
  if (!need) return ORACLE_ERR_INVALID;
  if (dst_bytes != need) return ORACLE_ERR_SIZE;
  const size_t nb = ((size_t)cols + 31) / 32, bb = oracle_block_bytes(qtype);
  for (int r = 0; r < rows; ++r)
    for (size_t b = 0; b < nb; ++b) {
      const size_t c0 = b * 32;
      const int n = (size_t)cols - c0 < 32 ? (int)((size_t)cols - c0) : 32;
      const int rc = quantize_block(qtype, src + (size_t)r * cols + c0, n, dst + ((size_t)r * nb + b) * bb);
      if (rc) return rc;
    }
  return ORACLE_OK;
}

/* Decode element i of a block: Value, src/quantized_tensor.cc:32-43.
 * Q8_0: d*int8; Q4_0: d*(q-8); Q4_1: d*q + m. Nibble i<16 is the low half of
 * byte i, nibble i>=16 the high half of byte i-16. */
static float decode(int qtype, const uint8_t *blk, int i) {
  const float d = oracle_half_to_float(rd16(blk));
  if (qtype == Q8_0) return d * (float)(int8_t)blk[2 + i];
  const int base = qtype == Q4_1 ? 4 : 2;
  const int byte = blk[base + (i & 15)];
  const int q = i < 16 ? (byte & 15) : (byte >> 4);
  if (qtype == Q4_1) return d * (float)q + oracle_half_to_float(rd16(blk + 2));
  return d * (float)(q - 8);
}

/* DequantizeTensor: src/quantized_tensor.cc:193-206. */
int oracle_dequantize(int qtype, const uint8_t *blocks, size_t nbytes, int rows, int cols, float *dst) {
  const size_t need = oracle_quantized_bytes(qtype, rows, cols);
  if (!need) return ORACLE_ERR_INVALID;
  if (nbytes != need) return ORACLE_ERR_SIZE;
  const size_t nb = ((size_t)cols + 31) / 32, bb = oracle_block_bytes(qtype);
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < cols; ++c)
      dst[(size_t)r * cols + c] = decode(qtype, blocks + ((size_t)r * nb + c / 32) * bb, c % 32);
  return ORACLE_OK;
}

/*
 * QuantizedDotRow: src/quantized_tensor.cc:161-191. One fp32 accumulator,
 * blocks in order, elements in order, tail elements past `cols` skipped;
 * the per-block scale (and Q4_1 min) is decoded once per block (:170-172)
 * and each element is value = d*q (+ m) before `sum += value * x`.
 */
float oracle_dot_row(int qtype, const uint8_t *blocks, int cols, int row, const float *x) {
  const size_t nb = ((size_t)cols + 31) / 32, bb = oracle_block_bytes(qtype);
  float sum = 0.0f;
  for (size_t b = 0; b < nb; ++b) {
    const uint8_t *blk = blocks + ((size_t)row * nb + b) * bb;
    const float d = oracle_half_to_float(rd16(blk));
    const float m = qtype == Q4_1 ? oracle_half_to_float(rd16(blk + 2)) : 0.0f;
    for (int i = 0; i < 32 && b * 32 + (size_t)i < (size_t)cols; ++i) {
      float value;
      if (qtype == Q8_0) {
        value = d * (float)(int8_t)blk[2 + i];
      } else {
        const int byte = blk[(qtype == Q4_1 ? 4 : 2) + (i & 15)];
        const int q = i < 16 ? (byte & 15) : (byte >> 4);
        value = qtype == Q4_1 ? d * (float)q + m : d * (float)(q - 8);
      }
      sum += value * x[b * 32 + i];
    }
  }
  return sum;
}

/*
 * y[m, n] = dot(row n, x[m]) for m in [0, M): the reference linear
 * (LinearDispatch, src/matmul_optimized.cc:146-182) applied to each of the M
 * activation rows in turn, which is what its per-token prefill does
 * (src/forward.cc:189-193). Rows are split into contiguous chunks across
 * `threads` POSIX threads as ThreadPool::ParallelFor does
 * (src/thread_pool.cc:51-86); each output is computed by exactly one thread
 * in a fixed order, so results do not depend on the thread count.
 */
typedef struct {
  int qtype, cols, m, r0, r1, ldx, ldy, n_rows;
  const uint8_t *blocks;
  const float *x;
  float *y;
} task_t;

static void *run_rows(void *arg) {
  const task_t *t = (const task_t *)arg;
  for (int mm = 0; mm < t->m; ++mm)
    for (int r = t->r0; r < t->r1; ++r)
      t->y[(size_t)mm * t->ldy + r] = oracle_dot_row(t->qtype, t->blocks, t->cols, r, t->x + (size_t)mm * t->ldx);
  return NULL;
}

int oracle_linear(int qtype, const uint8_t *blocks, size_t nbytes, int rows, int cols, const float *x, int m,
                  int ldx, float *y, int ldy, int threads) {
  const size_t need = oracle_quantized_bytes(qtype, rows, cols);
  if (!need || m < 0 || ldx < cols || ldy < rows) return ORACLE_ERR_INVALID;
  if (nbytes != need) return ORACLE_ERR_SIZE;
  if (m == 0) return ORACLE_OK;
  if (threads < 1) threads = 1;
  if (threads > rows) threads = rows;
  if (threads > 256) threads = 256;
  task_t tasks[256];
  pthread_t tid[256];
  for (int t = 0; t < threads; ++t) {
    tasks[t] = (task_t){qtype, cols, m, (int)((long long)rows * t / threads), (int)((long long)rows * (t + 1) / threads),
                        ldx, ldy, rows, blocks, x, y};
  }
  int started = 0;
  for (int t = 1; t < threads; ++t) {
    if (pthread_create(&tid[t], NULL, run_rows, &tasks[t]) != 0) break;
    started = t;
  }
  run_rows(&tasks[0]);
  for (int t = started + 1; t < threads; ++t) run_rows(&tasks[t]); /* rows whose thread failed to start */
  for (int t = 1; t <= started; ++t) pthread_join(tid[t], NULL);
  return ORACLE_OK;
}

/* Batch helpers for exhaustive fp16 checks from Python. */
void oracle_float_to_half_batch(const float *src, uint16_t *dst, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = oracle_float_to_half(src[i]);
}
void oracle_half_to_float_batch(const uint16_t *src, float *dst, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = oracle_half_to_float(src[i]);
}
/* Fills dst with float_to_half of the bit patterns [start, start + n). */
void oracle_float_to_half_range(uint32_t start, uint16_t *dst, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = oracle_float_to_half(bits_to_float(start + (uint32_t)i));
}
