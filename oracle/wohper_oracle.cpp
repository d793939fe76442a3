// wohper_oracle.cpp -- TEST INFRASTRUCTURE ONLY (see wohper_oracle.h).
//
// Restates the reference's Rust CPU kernels (crate engine/zc_infer_core) in
// C++.  Every function cites the reference file:line it follows.  Build flags
// (oracle/Makefile): -O2 -mavx2 -mfma -ffp-contract=off, so scalar `a*b+c`
// stays two roundings exactly like Rust, and only the explicit _mm256_fmadd_ps
// calls fuse.
#include "wohper_oracle.h"

#include <immintrin.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// a1 decoders (src/deepseek_v4.rs:151-204, 358-372)
// ---------------------------------------------------------------------------
float powi2(int e) { return std::ldexp(1.0f, e); }  // Rust 2f32.powi(e): exact

float decode_fp8(uint8_t byte, float scale) {
  float sign = (byte & 0x80) ? -1.0f : 1.0f;
  int exponent = (byte >> 3) & 0x0f;
  int mantissa = byte & 0x07;
  if (exponent == 0 && mantissa == 0) return 0.0f;
  float value;
  if (exponent == 0) {
    value = ((float)mantissa / 8.0f) * powi2(-6);
  } else {
    value = (1.0f + (float)mantissa / 8.0f) * powi2(exponent - 7);
  }
  return sign * value * scale;
}

float decode_ue8m0(uint8_t byte) { return byte == 0 ? 0.0f : powi2((int)byte - 127); }

float decode_fp4(uint8_t nibble, float scale) {
  nibble &= 0x0f;
  float sign = (nibble & 0x08) ? -1.0f : 1.0f;
  int exponent = (nibble >> 1) & 0x03;
  int mantissa = nibble & 0x01;
  if (exponent == 0 && mantissa == 0) return 0.0f;
  float value;
  if (exponent == 0) {
    value = ((float)mantissa / 2.0f) * powi2(-2);
  } else {
    value = (1.0f + (float)mantissa / 2.0f) * powi2(exponent - 1);
  }
  return sign * value * scale;
}

// FP4_E2M1_BASE_LUT (src/deepseek_v4.rs:177-180)
const float kFp4BaseLut[16] = {0.0f, 0.125f, 1.0f,  1.5f,  2.0f,  3.0f,  4.0f,  6.0f,
                               0.0f, -0.125f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};
// fp4_avx2::FP4_BASE_X8_I8 (src/deepseek_v4.rs:285-287)
const int8_t kFp4BaseX8[16] = {0, 1, 8, 12, 16, 24, 32, 48, 0, -1, -8, -12, -16, -24, -32, -48};

struct Luts {
  float fp8[256];
  float ue8m0[256];
  float sorted[256];
  Luts() {
    for (int b = 0; b < 256; ++b) {
      fp8[b] = decode_fp8((uint8_t)b, 1.0f);
      ue8m0[b] = decode_ue8m0((uint8_t)b);
      sorted[b] = fp8[b];
    }
    // src/compute.rs:2547-2558: values.sort_by(f32::total_cmp).  No NaN in
    // the table and +0.0 twice (0x00 and 0x80 both decode to +0.0).
    std::sort(sorted, sorted + 256, [](float a, float b) { return a < b; });
  }
};
const Luts& luts() {
  static Luts l;
  return l;
}

// ---------------------------------------------------------------------------
// Threading: compute_thread_count / parallel_rows_f32 (src/deepseek_v4.rs:206-262)
// Per-row results do not depend on the split, so any split is bit-identical.
// ---------------------------------------------------------------------------
int g_threads = 0;
int thread_count() {
  if (g_threads > 0) return g_threads;
  const char* env = std::getenv("ZC_COMPUTE_THREADS");
  if (env) {
    int v = std::atoi(env);
    if (v > 0) return v;
  }
  int n = (int)std::thread::hardware_concurrency();
  return std::max(1, n - 2);
}

// work(row_offset, count) -> status; first error wins.
int parallel_rows(size_t total, size_t min_rows, const std::function<int(size_t, size_t)>& work) {
  int threads = thread_count();
  min_rows = std::max<size_t>(min_rows, 1);
  if (threads <= 1 || total < min_rows * 2) return work(0, total);
  size_t chunk = std::max((total + threads - 1) / threads, min_rows);
  std::vector<std::thread> pool;
  std::mutex mu;
  int first = ORC_OK;
  for (size_t off = 0; off < total; off += chunk) {
    size_t take = std::min(chunk, total - off);
    pool.emplace_back([&, off, take]() {
      int st = work(off, take);
      if (st != ORC_OK) {
        std::lock_guard<std::mutex> g(mu);
        if (first == ORC_OK) first = st;
      }
    });
  }
  for (auto& t : pool) t.join();
  return first;
}

__attribute__((target("avx2,fma"))) float hsum256(__m256 v) {
  alignas(32) float l[8];
  _mm256_storeu_ps(l, v);
  return ((l[0] + l[1]) + (l[2] + l[3])) + ((l[4] + l[5]) + (l[6] + l[7]));
}

// ---------------------------------------------------------------------------
// a2 FP8 row dot
// ---------------------------------------------------------------------------
// simd_x86::fp8_ue8m0_dot_row_avx2 (src/compute.rs:5977-6018).  When
// dequant_out != nullptr this is fp8_ue8m0_dot_row_avx2_store_dequant
// (src/compute.rs:6028-6074): same arithmetic, also stores the LUT values.
__attribute__((target("avx2,fma"))) float fp8_dot_avx2(const uint8_t* w, const uint8_t* srow,
                                                       size_t scale_cols, size_t col_group,
                                                       const float* x, float* dequant_out) {
  const float* lut = luts().fp8;
  const float* slut = luts().ue8m0;
  __m256 acc = _mm256_setzero_ps();
  float tail = 0.0f;
  for (size_t g = 0; g < scale_cols; ++g) {
    float scale = slut[srow[g]];
    const uint8_t* bytes = w + g * col_group;
    const float* cols = x + g * col_group;
    __m256 g0 = _mm256_setzero_ps();
    __m256 g1 = _mm256_setzero_ps();
    size_t chunks = col_group / 16;
    for (size_t c = 0; c < chunks; ++c) {
      size_t base = c * 16;
      __m256i idx0 = _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i*)(bytes + base)));
      __m256i idx1 = _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i*)(bytes + base + 8)));
      __m256 w0 = _mm256_i32gather_ps(lut, idx0, 4);
      __m256 w1 = _mm256_i32gather_ps(lut, idx1, 4);
      if (dequant_out) {
        _mm256_storeu_ps(dequant_out + g * col_group + base, w0);
        _mm256_storeu_ps(dequant_out + g * col_group + base + 8, w1);
      }
      g0 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(cols + base), g0);
      g1 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(cols + base + 8), g1);
    }
    float rem = 0.0f;
    for (size_t i = chunks * 16; i < col_group; ++i) {
      float v = lut[bytes[i]];
      if (dequant_out) dequant_out[g * col_group + i] = v;
      rem += v * cols[i];
    }
    acc = _mm256_fmadd_ps(_mm256_add_ps(g0, g1), _mm256_set1_ps(scale), acc);
    tail += rem * scale;
  }
  return hsum256(acc) + tail;
}

// simd_x86::fp8_ue8m0_dot_dequant_row_avx2 (src/compute.rs:6080-6112)
__attribute__((target("avx2,fma"))) float fp8_dot_dequant_avx2(const float* dq,
                                                               const uint8_t* srow,
                                                               size_t scale_cols,
                                                               size_t col_group, const float* x) {
  const float* slut = luts().ue8m0;
  __m256 acc = _mm256_setzero_ps();
  float tail = 0.0f;
  for (size_t g = 0; g < scale_cols; ++g) {
    float scale = slut[srow[g]];
    const float* weights = dq + g * col_group;
    const float* cols = x + g * col_group;
    __m256 g0 = _mm256_setzero_ps();
    __m256 g1 = _mm256_setzero_ps();
    size_t chunks = col_group / 16;
    for (size_t c = 0; c < chunks; ++c) {
      size_t base = c * 16;
      g0 = _mm256_fmadd_ps(_mm256_loadu_ps(weights + base), _mm256_loadu_ps(cols + base), g0);
      g1 = _mm256_fmadd_ps(_mm256_loadu_ps(weights + base + 8), _mm256_loadu_ps(cols + base + 8),
                           g1);
    }
    float rem = 0.0f;
    for (size_t i = chunks * 16; i < col_group; ++i) rem += weights[i] * cols[i];
    acc = _mm256_fmadd_ps(_mm256_add_ps(g0, g1), _mm256_set1_ps(scale), acc);
    tail += rem * scale;
  }
  return hsum256(acc) + tail;
}

// scalar fp8_ue8m0_dot_row (src/compute.rs:5936-5960)
float fp8_dot_scalar(const uint8_t* w, const uint8_t* srow, size_t scale_cols, size_t col_group,
                     const float* x) {
  const float* lut = luts().fp8;
  const float* slut = luts().ue8m0;
  float acc = 0.0f;
  for (size_t g = 0; g < scale_cols; ++g) {
    float scale = slut[srow[g]];
    const uint8_t* bytes = w + g * col_group;
    const float* cols = x + g * col_group;
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    size_t quads = col_group / 4;
    for (size_t q = 0; q < quads; ++q) {
      size_t i = q * 4;
      s0 += lut[bytes[i]] * cols[i];
      s1 += lut[bytes[i + 1]] * cols[i + 1];
      s2 += lut[bytes[i + 2]] * cols[i + 2];
      s3 += lut[bytes[i + 3]] * cols[i + 3];
    }
    for (size_t i = quads * 4; i < col_group; ++i) s0 += lut[bytes[i]] * cols[i];
    acc += scale * ((s0 + s1) + (s2 + s3));
  }
  return acc;
}

bool avx2_available() {
  static bool ok = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
  return ok;
}

// shape checks shared by the three FP8 GEMV forms (src/compute.rs:6184-6216)
int fp8_validate(size_t weight_len, size_t rows, size_t cols, size_t scale_len, size_t scale_rows,
                 size_t scale_cols, size_t row_start, size_t row_end) {
  if (rows == 0 || cols == 0 || scale_rows == 0 || scale_cols == 0 || rows % scale_rows != 0 ||
      cols % scale_cols != 0)
    return ORC_ERR_INVALID_SHAPE;
  if (row_start >= row_end || row_end > rows) return ORC_ERR_INVALID_SHAPE;
  if (weight_len < cols * row_end) return ORC_ERR_INVALID_SHAPE;
  if (scale_len < scale_rows * scale_cols) return ORC_ERR_INVALID_SHAPE;
  return ORC_OK;
}

// ---------------------------------------------------------------------------
// a7 act quant (src/compute.rs:2504-2545)
// ---------------------------------------------------------------------------
float nearest_in_sorted_lut(const float* lut, float target) {
  // lut.partition_point(|v| *v < target)
  size_t idx = (size_t)(std::partition_point(lut, lut + 256, [&](float v) { return v < target; }) -
                        lut);
  size_t lo_i = idx == 0 ? 0 : idx - 1;
  if (lo_i > 255) lo_i = 255;
  size_t up_i = idx > 255 ? 255 : idx;
  float lower = lut[lo_i];
  float upper = lut[up_i];
  return std::fabs(upper - target) < std::fabs(lower - target) ? upper : lower;
}

void act_quant(float* values, size_t n, size_t block_size) {
  if (block_size == 0 || n == 0) return;
  const float* lut = luts().sorted;
  for (size_t b0 = 0; b0 < n; b0 += block_size) {
    size_t b1 = std::min(n, b0 + block_size);
    float amax = 0.0f;
    for (size_t i = b0; i < b1; ++i) amax = std::fmax(amax, std::fabs(values[i]));
    amax = std::fmax(amax, 1.0e-4f);
    float scale = exp2f(ceilf(log2f(amax / 448.0f)));
    for (size_t i = b0; i < b1; ++i) {
      float scaled = values[i] / scale;
      // f32::clamp: NaN passes through
      if (scaled < -448.0f) scaled = -448.0f;
      if (scaled > 448.0f) scaled = 448.0f;
      values[i] = nearest_in_sorted_lut(lut, scaled) * scale;
    }
  }
}

// ---------------------------------------------------------------------------
// BF16 dot (src/compute.rs:6115-6136 AVX2; 2910-2944 scalar)
// ---------------------------------------------------------------------------
inline float bf16_to_f32(uint16_t raw) {
  uint32_t bits = (uint32_t)raw << 16;
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

__attribute__((target("avx2,fma"))) float bf16_dot_avx2(const uint16_t* row, const float* x,
                                                        size_t n) {
  __m256 acc0 = _mm256_setzero_ps();
  __m256 acc1 = _mm256_setzero_ps();
  size_t chunks = n / 16;
  for (size_t c = 0; c < chunks; ++c) {
    size_t i = c * 16;
    __m128i raw0 = _mm_loadu_si128((const __m128i*)(row + i));
    __m128i raw1 = _mm_loadu_si128((const __m128i*)(row + i + 8));
    __m256 w0 = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(raw0), 16));
    __m256 w1 = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(raw1), 16));
    acc0 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(x + i), acc0);
    acc1 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(x + i + 8), acc1);
  }
  float tail = 0.0f;
  for (size_t i = chunks * 16; i < n; ++i) tail += bf16_to_f32(row[i]) * x[i];
  return hsum256(_mm256_add_ps(acc0, acc1)) + tail;
}

float bf16_dot_scalar(const uint16_t* row, const float* x, size_t n) {
  float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  size_t quads = n / 4;
  for (size_t q = 0; q < quads; ++q) {
    size_t i = q * 4;
    s0 += bf16_to_f32(row[i]) * x[i];
    s1 += bf16_to_f32(row[i + 1]) * x[i + 1];
    s2 += bf16_to_f32(row[i + 2]) * x[i + 2];
    s3 += bf16_to_f32(row[i + 3]) * x[i + 3];
  }
  for (size_t i = quads * 4; i < n; ++i) s0 += bf16_to_f32(row[i]) * x[i];
  return (s0 + s1) + (s2 + s3);
}

// ---------------------------------------------------------------------------
// a9 FP4 row dot: fp4_avx2::dot_row (src/deepseek_v4.rs:294-347)
// ---------------------------------------------------------------------------
__attribute__((target("avx2,fma"))) float fp4_dot_avx2(const uint8_t* w, const uint8_t* srow,
                                                       size_t scale_cols, size_t group_bytes,
                                                       size_t group_cols, const float* x) {
  const float* slut = luts().ue8m0;
  const __m128i lut = _mm_loadu_si128((const __m128i*)kFp4BaseX8);
  const __m128i low_mask = _mm_set1_epi8(0x0f);
  __m256 acc = _mm256_setzero_ps();
  float tail = 0.0f;
  for (size_t g = 0; g < scale_cols; ++g) {
    float scale = slut[srow[g]];
    const uint8_t* bytes = w + g * group_bytes;
    const float* cols = x + g * group_cols;
    size_t chunks = group_bytes / 16;
    __m256 gacc = _mm256_setzero_ps();
    for (size_t c = 0; c < chunks; ++c) {
      __m128i wv = _mm_loadu_si128((const __m128i*)(bytes + c * 16));
      __m128i lo = _mm_and_si128(wv, low_mask);
      __m128i hi = _mm_and_si128(_mm_srli_epi16(wv, 4), low_mask);
      __m128i vlo = _mm_shuffle_epi8(lut, lo);
      __m128i vhi = _mm_shuffle_epi8(lut, hi);
      __m128i il = _mm_unpacklo_epi8(vlo, vhi);
      __m128i ih = _mm_unpackhi_epi8(vlo, vhi);
      const float* base = cols + c * 32;
      __m256 c0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(il));
      __m256 c1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(il, 8)));
      __m256 c2 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(ih));
      __m256 c3 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(ih, 8)));
      gacc = _mm256_fmadd_ps(c0, _mm256_loadu_ps(base), gacc);
      gacc = _mm256_fmadd_ps(c1, _mm256_loadu_ps(base + 8), gacc);
      gacc = _mm256_fmadd_ps(c2, _mm256_loadu_ps(base + 16), gacc);
      gacc = _mm256_fmadd_ps(c3, _mm256_loadu_ps(base + 24), gacc);
    }
    acc = _mm256_fmadd_ps(gacc, _mm256_set1_ps(scale * 0.125f), acc);
    float rem = 0.0f;
    for (size_t i = chunks * 16; i < group_bytes; ++i) {
      uint8_t byte = bytes[i];
      rem += kFp4BaseLut[byte & 0x0f] * cols[2 * i];
      rem += kFp4BaseLut[byte >> 4] * cols[2 * i + 1];
    }
    tail += rem * scale;
  }
  return hsum256(acc) + tail;
}

size_t packed_row_bytes(size_t cols) { return (cols + 1) / 2; }

// validate_fp4_matvec (src/deepseek_v4.rs:434-462)
int fp4_validate(const orc_fp4_spec& s, size_t input_len, size_t output_len) {
  if (s.rows == 0 || s.cols == 0 || s.scale_cols == 0) return ORC_ERR_EMPTY_SHAPE;
  if (input_len < s.cols) return ORC_ERR_INPUT_TOO_SMALL;
  if (output_len < s.rows) return ORC_ERR_OUTPUT_TOO_SMALL;
  if (s.cols % s.scale_cols != 0) return ORC_ERR_INVALID_SHAPE;
  if (s.packed_len < s.rows * packed_row_bytes(s.cols)) return ORC_ERR_PACKED_WEIGHT_TOO_SMALL;
  if (s.scales_len < s.rows * s.scale_cols) return ORC_ERR_SCALE_TOO_SMALL;
  return ORC_OK;
}

// fp4_e2m1_ue8m0_matvec_scalar (src/deepseek_v4.rs:464-549)
int fp4_matvec(const orc_fp4_spec& s, const float* input, size_t input_len, float* output,
               size_t output_len, int path) {
  int st = fp4_validate(s, input_len, output_len);
  if (st != ORC_OK) return st;
  size_t row_bytes = packed_row_bytes(s.cols);
  size_t group_cols = s.cols / s.scale_cols;
  const float* slut = luts().ue8m0;
  if (path != 2 && s.cols % 2 == 0 && group_cols % 2 == 0) {
    size_t group_bytes = group_cols / 2;
    if (path == 0 && avx2_available()) {
      return parallel_rows(s.rows, 64, [&](size_t off, size_t cnt) {
        for (size_t r = off; r < off + cnt; ++r) {
          float acc = fp4_dot_avx2(s.packed_weight + r * row_bytes, s.ue8m0_scales + r * s.scale_cols,
                                   s.scale_cols, group_bytes, group_cols, input);
          if (!std::isfinite(acc)) return (int)ORC_ERR_NON_FINITE_OUTPUT;
          output[r] = acc;
        }
        return (int)ORC_OK;
      });
    }
    for (size_t r = 0; r < s.rows; ++r) {
      const uint8_t* wr = s.packed_weight + r * row_bytes;
      const uint8_t* sr = s.ue8m0_scales + r * s.scale_cols;
      float acc = 0.0f;
      for (size_t g = 0; g < s.scale_cols; ++g) {
        float scale = slut[sr[g]];
        const uint8_t* bytes = wr + g * group_bytes;
        const float* cols = input + g * group_cols;
        float low = 0.0f, high = 0.0f;
        for (size_t i = 0; i < group_bytes; ++i) {
          low += kFp4BaseLut[bytes[i] & 0x0f] * cols[2 * i];
          high += kFp4BaseLut[bytes[i] >> 4] * cols[2 * i + 1];
        }
        acc += scale * (low + high);
      }
      if (!std::isfinite(acc)) return ORC_ERR_NON_FINITE_OUTPUT;
      output[r] = acc;
    }
    return ORC_OK;
  }
  for (size_t r = 0; r < s.rows; ++r) {
    size_t ro = r * row_bytes, so = r * s.scale_cols;
    float acc = 0.0f;
    for (size_t col = 0; col < s.cols; ++col) {
      uint8_t packed = s.packed_weight[ro + col / 2];
      uint8_t nibble = (col & 1) == 0 ? (packed & 0x0f) : (packed >> 4);
      float scale = decode_ue8m0(s.ue8m0_scales[so + col / group_cols]);
      acc += decode_fp4(nibble, scale) * input[col];
    }
    if (!std::isfinite(acc)) return ORC_ERR_NON_FINITE_OUTPUT;
    output[r] = acc;
  }
  return ORC_OK;
}

inline float silu(float x) { return x / (1.0f + expf(-x)); }  // src/deepseek_v4.rs:551-554
const float kSwigluLimit = 10.0f;                             // src/deepseek_v4.rs:559

// deepseek_v4_fp4_expert_forward_scalar (src/deepseek_v4.rs:561-601)
int fp4_expert_forward(const orc_fp4_expert& e, const float* input, size_t input_len,
                       float* output, size_t output_len, float* scratch, size_t scratch_len) {
  if (e.w1.cols != input_len || e.w3.cols != input_len || e.w1.rows != e.w3.rows ||
      e.w2.cols != e.w1.rows)
    return ORC_ERR_INVALID_SHAPE;
  if (output_len < e.w2.rows) return ORC_ERR_OUTPUT_TOO_SMALL;
  size_t inter = e.w1.rows;
  if (scratch_len < 2 * inter) return ORC_ERR_SCRATCH_TOO_SMALL;
  float* gate = scratch;
  float* up = scratch + inter;
  std::vector<float> xq(input, input + e.w1.cols);
  act_quant(xq.data(), xq.size(), 64);
  int st = fp4_matvec(e.w1, xq.data(), xq.size(), gate, inter, 0);
  if (st != ORC_OK) return st;
  st = fp4_matvec(e.w3, xq.data(), xq.size(), up, inter, 0);
  if (st != ORC_OK) return st;
  for (size_t i = 0; i < inter; ++i) {
    float gated = std::fmin(gate[i], kSwigluLimit);
    float upped = up[i];
    // f32::clamp(-10, 10)
    if (upped < -kSwigluLimit) upped = -kSwigluLimit;
    if (upped > kSwigluLimit) upped = kSwigluLimit;
    gate[i] = silu(gated) * upped;
  }
  act_quant(gate, inter, 64);
  st = fp4_matvec(e.w2, gate, inter, output, output_len, 0);
  if (st != ORC_OK) return st;
  for (size_t i = 0; i < e.w2.rows; ++i)
    if (!std::isfinite(output[i])) return ORC_ERR_NON_FINITE_OUTPUT;
  return ORC_OK;
}

int fp8_gemv_full(const orc_fp8_matrix& m, const float* x, float* y) {
  return orc_fp8_gemv_rows(m.weight, m.rows * m.cols, m.rows, m.cols, m.scale,
                           m.scale_rows * m.scale_cols, m.scale_rows, m.scale_cols, 0, m.rows, x,
                           m.cols, y, m.rows);
}

// sqrt_softplus (src/compute.rs:2238-2248)
float sqrt_softplus(float v) {
  float sp;
  if (v > 20.0f)
    sp = v;
  else if (v < -20.0f)
    sp = expf(v);
  else
    sp = log1pf(expf(v));
  return sqrtf(std::fmax(sp, 0.0f));
}

// Combine the routed experts for one token (src/compute.rs:1948-2030).
int combine_routed(const orc_fp4_expert* experts, const int32_t* ids, const float* weights,
                   size_t topk, const float* x, size_t hidden, float* out) {
  if (topk == 0) return ORC_OK;
  size_t inter = experts[ids[0]].w1.rows;
  std::vector<float> scratch(2 * std::max<size_t>(inter, 1));
  if (topk == 1) {
    // single expert: hidden = expert(hidden), no weighting (src/compute.rs:1960-1966)
    std::vector<float> tmp(hidden);
    int st = fp4_expert_forward(experts[ids[0]], x, hidden, tmp.data(), hidden, scratch.data(),
                                scratch.size());
    if (st != ORC_OK) return st;
    std::copy(tmp.begin(), tmp.end(), out);
    return ORC_OK;
  }
  // valid_route_weight_sum (src/compute.rs:2015-2030)
  bool valid = true;
  float sum = 0.0f;
  for (size_t k = 0; k < topk; ++k) {
    float w = weights[k];
    if (std::isfinite(w) && w >= 0.0f)
      sum = sum + w;
    else {
      valid = false;
      break;
    }
  }
  if (valid && sum <= 1.1920929e-07f) valid = false;
  float uniform = 1.0f / (float)topk;
  std::vector<float> acc(hidden, 0.0f), y(hidden);
  for (size_t k = 0; k < topk; ++k) {
    float w = valid ? weights[k] / sum : uniform;
    const orc_fp4_expert& e = experts[ids[k]];
    std::vector<float> scr(2 * e.w1.rows);
    int st = fp4_expert_forward(e, x, hidden, y.data(), hidden, scr.data(), scr.size());
    if (st != ORC_OK) return st;
    for (size_t i = 0; i < hidden; ++i) acc[i] += y[i] * w;
  }
  std::copy(acc.begin(), acc.end(), out);
  return ORC_OK;
}

}  // namespace

// ===========================================================================
// extern "C" surface
// ===========================================================================
extern "C" {

void orc_set_threads(int threads) { g_threads = threads; }
int orc_get_threads(void) { return thread_count(); }

float orc_decode_fp8_e4m3(uint8_t byte, float scale) { return decode_fp8(byte, scale); }
float orc_decode_ue8m0_scale(uint8_t byte) { return decode_ue8m0(byte); }
float orc_decode_fp4_e2m1(uint8_t nibble, float scale) { return decode_fp4(nibble, scale); }
void orc_fp8_e4m3_base_lut(float out[256]) { std::memcpy(out, luts().fp8, sizeof(luts().fp8)); }
void orc_ue8m0_scale_lut(float out[256]) { std::memcpy(out, luts().ue8m0, sizeof(luts().ue8m0)); }
void orc_fp4_e2m1_base_lut(float out[16]) { std::memcpy(out, kFp4BaseLut, sizeof(kFp4BaseLut)); }
void orc_fp8_e4m3_sorted_lut(float out[256]) {
  std::memcpy(out, luts().sorted, sizeof(luts().sorted));
}

float orc_fp8_dot_row(const uint8_t* weight_row, const uint8_t* scale_row, size_t scale_cols,
                      size_t col_group, const float* input, int avx2) {
  if (avx2 && avx2_available())
    return fp8_dot_avx2(weight_row, scale_row, scale_cols, col_group, input, nullptr);
  return fp8_dot_scalar(weight_row, scale_row, scale_cols, col_group, input);
}

// gemv_fp8_e4m3_ue8m0_tensorwise / _rows (src/compute.rs:6174-6321)
int orc_fp8_gemv_rows(const uint8_t* weight, size_t weight_len, size_t rows, size_t cols,
                      const uint8_t* scale, size_t scale_len, size_t scale_rows, size_t scale_cols,
                      size_t row_start, size_t row_end, const float* input, size_t input_len,
                      float* output, size_t output_len) {
  int st = fp8_validate(weight_len, rows, cols, scale_len, scale_rows, scale_cols, row_start,
                        row_end);
  if (st != ORC_OK) return st;
  if (input_len < cols) return ORC_ERR_INVALID_SHAPE;
  size_t n = row_end - row_start;
  if (output_len < n) return ORC_ERR_OUTPUT_TOO_SMALL;
  size_t row_group = rows / scale_rows, col_group = cols / scale_cols;
  bool avx = avx2_available();
  return parallel_rows(n, 32, [&](size_t off, size_t cnt) {
    for (size_t i = off; i < off + cnt; ++i) {
      size_t row = row_start + i;
      const uint8_t* wr = weight + row * cols;
      const uint8_t* sr = scale + (row / row_group) * scale_cols;
      float acc = avx ? fp8_dot_avx2(wr, sr, scale_cols, col_group, input, nullptr)
                      : fp8_dot_scalar(wr, sr, scale_cols, col_group, input);
      if (!std::isfinite(acc)) return (int)ORC_ERR_NON_FINITE_OUTPUT;
      output[i] = acc;
    }
    return (int)ORC_OK;
  });
}

// gemv_fp8_e4m3_ue8m0_rows_multi (src/compute.rs:6384-6577): the first input
// decodes and stores the row, the others reuse it; bit-identical to the
// single-input kernel.
int orc_fp8_gemv_rows_multi(const uint8_t* weight, size_t weight_len, size_t rows, size_t cols,
                            const uint8_t* scale, size_t scale_len, size_t scale_rows,
                            size_t scale_cols, size_t row_start, size_t row_end,
                            const float* inputs, size_t count, size_t ldx, float* outputs,
                            size_t ldy) {
  if (count == 0) return ORC_ERR_INVALID_SHAPE;
  int st = fp8_validate(weight_len, rows, cols, scale_len, scale_rows, scale_cols, row_start,
                        row_end);
  if (st != ORC_OK) return st;
  size_t n = row_end - row_start;
  if (ldx < cols) return ORC_ERR_INVALID_SHAPE;
  if (ldy < n) return ORC_ERR_OUTPUT_TOO_SMALL;
  size_t row_group = rows / scale_rows, col_group = cols / scale_cols;
  bool avx = avx2_available();
  int threads = std::max(1, thread_count());
  size_t chunk_rows = std::max<size_t>((n + threads - 1) / threads, 8);
  auto worker = [&](size_t off, size_t cnt) -> int {
    std::vector<float> dq(cols);
    const float* lut = luts().fp8;
    for (size_t i = off; i < off + cnt; ++i) {
      size_t row = row_start + i;
      const uint8_t* wr = weight + row * cols;
      const uint8_t* sr = scale + (row / row_group) * scale_cols;
      for (size_t k = 0; k < count; ++k) {
        const float* x = inputs + k * ldx;
        float acc;
        if (avx) {
          acc = k == 0 ? fp8_dot_avx2(wr, sr, scale_cols, col_group, x, dq.data())
                       : fp8_dot_dequant_avx2(dq.data(), sr, scale_cols, col_group, x);
        } else {
          if (k == 0)
            for (size_t c = 0; c < cols; ++c) dq[c] = lut[wr[c]];
          // fp8_ue8m0_dot_dequant_row scalar (src/compute.rs:6338-6370)
          const float* slut = luts().ue8m0;
          acc = 0.0f;
          for (size_t g = 0; g < scale_cols; ++g) {
            float sc = slut[sr[g]];
            const float* wv = dq.data() + g * col_group;
            const float* cv = x + g * col_group;
            float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
            size_t quads = col_group / 4;
            for (size_t q = 0; q < quads; ++q) {
              size_t j = q * 4;
              s0 += wv[j] * cv[j];
              s1 += wv[j + 1] * cv[j + 1];
              s2 += wv[j + 2] * cv[j + 2];
              s3 += wv[j + 3] * cv[j + 3];
            }
            for (size_t j = quads * 4; j < col_group; ++j) s0 += wv[j] * cv[j];
            acc += sc * ((s0 + s1) + (s2 + s3));
          }
        }
        if (!std::isfinite(acc)) return ORC_ERR_NON_FINITE_OUTPUT;
        outputs[k * ldy + i] = acc;
      }
    }
    return ORC_OK;
  };
  if (threads <= 1 || n <= chunk_rows) return worker(0, n);
  std::vector<std::thread> pool;
  std::mutex mu;
  int first = ORC_OK;
  for (size_t off = 0; off < n; off += chunk_rows) {
    size_t take = std::min(chunk_rows, n - off);
    pool.emplace_back([&, off, take]() {
      int s = worker(off, take);
      if (s != ORC_OK) {
        std::lock_guard<std::mutex> g(mu);
        if (first == ORC_OK) first = s;
      }
    });
  }
  for (auto& t : pool) t.join();
  return first;
}

void orc_fp8_act_quant_dequant_in_place(float* values, size_t n, size_t block_size) {
  act_quant(values, n, block_size);
}

float orc_bf16_dot_row(const uint16_t* row, const float* input, size_t n, int avx2) {
  if (avx2 && avx2_available()) return bf16_dot_avx2(row, input, n);
  return bf16_dot_scalar(row, input, n);
}

// gemv_bf16_tensorwise (src/compute.rs:6139-6172)
int orc_bf16_gemv(const uint16_t* weight, size_t rows, size_t cols, const float* input,
                  float* output) {
  if (rows == 0 || cols == 0) return ORC_ERR_INVALID_SHAPE;
  bool avx = avx2_available();
  return parallel_rows(rows, 32, [&](size_t off, size_t cnt) {
    for (size_t r = off; r < off + cnt; ++r)
      output[r] = avx ? bf16_dot_avx2(weight + r * cols, input, cols)
                      : bf16_dot_scalar(weight + r * cols, input, cols);
    return (int)ORC_OK;
  });
}

int orc_fp4_matvec(const orc_fp4_spec* spec, const float* input, size_t input_len,
                   float* output, size_t output_len, int path) {
  return fp4_matvec(*spec, input, input_len, output, output_len, path);
}

int orc_fp4_expert_forward(const orc_fp4_expert* expert, const float* input, size_t input_len,
                           float* output, size_t output_len, float* scratch, size_t scratch_len) {
  return fp4_expert_forward(*expert, input, input_len, output, output_len, scratch, scratch_len);
}

size_t orc_fp4_expert_scratch_len(size_t intermediate) { return intermediate * 2; }

// compute_deepseek_fp8_shared_expert_into_hidden (src/compute.rs:5545-5614)
int orc_fp8_expert_forward(const orc_fp8_expert* e, const float* input, size_t hidden,
                           float* output) {
  if (e->w1.cols != hidden || e->w3.cols != hidden) return ORC_ERR_INVALID_SHAPE;
  if (e->w1.rows != e->w3.rows || e->w2.cols != e->w1.rows) return ORC_ERR_INVALID_SHAPE;
  size_t inter = e->w1.rows;
  std::vector<float> xq(input, input + hidden), gate(inter), up(inter);
  act_quant(xq.data(), hidden, 64);
  int st = fp8_gemv_full(e->w1, xq.data(), gate.data());
  if (st != ORC_OK) return st;
  st = fp8_gemv_full(e->w3, xq.data(), up.data());
  if (st != ORC_OK) return st;
  for (size_t i = 0; i < inter; ++i) {
    float gated = std::fmin(gate[i], kSwigluLimit);
    float upped = up[i];
    if (upped < -kSwigluLimit) upped = -kSwigluLimit;
    if (upped > kSwigluLimit) upped = kSwigluLimit;
    gate[i] = silu(gated) * upped;
  }
  act_quant(gate.data(), inter, 64);
  return fp8_gemv_full(e->w2, gate.data(), output);
}

int orc_router(const uint16_t* gate_bf16, size_t experts, size_t hidden, const float* x,
               size_t topk, int mode, const float* bias, float route_scale,
               const int32_t* hash_ids, int32_t* ids_out, float* weights_out, float* logits_out) {
  if (experts == 0 || hidden == 0) return ORC_ERR_INVALID_SHAPE;
  std::vector<float> scores(experts);
  int st = orc_bf16_gemv(gate_bf16, experts, hidden, x, scores.data());
  if (st != ORC_OK) return st;
  if (logits_out) std::copy(scores.begin(), scores.end(), logits_out);
  if (mode == 1)
    for (auto& v : scores) v = sqrt_softplus(v);
  std::vector<std::pair<int32_t, float>> routes;  // (expert, score)
  if (mode == 1 && hash_ids) {
    // tid2eid hash routing (src/compute.rs:2190-2206)
    for (size_t k = 0; k < topk; ++k) {
      int32_t e = hash_ids[k];
      if (e >= 0 && (size_t)e < experts) routes.push_back({e, scores[e]});
    }
  } else {
    std::vector<std::pair<float, int32_t>> sel(experts);
    for (size_t e = 0; e < experts; ++e) {
      float s = scores[e];
      if (mode == 1 && bias) s = s + bias[e];
      sel[e] = {s, (int32_t)e};
    }
    // selected.sort_by(|l, r| r.0.total_cmp(&l.0)): stable, descending
    auto key = [](float f) {
      int32_t b;
      std::memcpy(&b, &f, 4);
      return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);  // total_cmp key
    };
    std::stable_sort(sel.begin(), sel.end(),
                     [&](const std::pair<float, int32_t>& l, const std::pair<float, int32_t>& r) {
                       return key(l.first) > key(r.first);
                     });
    for (size_t k = 0; k < std::min(topk, experts); ++k)
      routes.push_back({sel[k].second, scores[sel[k].second]});
  }
  size_t n = routes.size();
  if (mode == 1) {
    // finalize_route_weights (src/compute.rs:2253-2268)
    float sum = 0.0f;
    for (auto& r : routes) sum = sum + r.second;
    if (n > 0) {
      if (sum > 0.0f && std::isfinite(sum)) {
        for (auto& r : routes) r.second = r.second / sum * route_scale;
      } else {
        float u = route_scale / (float)n;
        for (auto& r : routes) r.second = u;
      }
    }
  } else if (n > 0) {
    // normalize_route_weights_legacy (src/server/generation.rs:3152-3180)
    bool finite = true;
    for (auto& r : routes) finite = finite && std::isfinite(r.second);
    bool uniform = !finite;
    if (!uniform) {
      float mx = -INFINITY;
      for (auto& r : routes) mx = std::fmax(mx, r.second);
      float sum = 0.0f;
      for (auto& r : routes) {
        r.second = expf(r.second - mx);
        sum += r.second;
      }
      if (!std::isfinite(sum) || sum <= 1.1920929e-07f)
        uniform = true;
      else
        for (auto& r : routes) r.second /= sum;
    }
    if (uniform)
      for (auto& r : routes) r.second = 1.0f / (float)n;
  }
  for (size_t k = 0; k < topk; ++k) {
    ids_out[k] = k < n ? routes[k].first : -1;
    weights_out[k] = k < n ? routes[k].second : 0.0f;
  }
  return (int)n;
}

size_t orc_deepseek_sqrtsoftplus_route(const float* logits, size_t n, const float* bias,
                                       size_t topk, float route_scale, int32_t* ids_out,
                                       float* weights_out) {
  struct S {
    size_t idx;
    float sel, w;
  };
  std::vector<S> scored(n);
  for (size_t i = 0; i < n; ++i) {
    float x = logits[i];
    float sp = x > 20.0f ? x : logf(1.0f + expf(x));
    float w = sqrtf(sp);
    scored[i] = {i, w + (bias ? bias[i] : 0.0f), w};
  }
  // sort_by(b.1.partial_cmp(&a.1)) -- stable merge sort, descending
  std::stable_sort(scored.begin(), scored.end(), [](const S& a, const S& b) { return a.sel > b.sel; });
  size_t k = std::min(topk, n);
  float denom = 0.0f;
  for (size_t i = 0; i < k; ++i) denom += scored[i].w;
  for (size_t i = 0; i < k; ++i) {
    ids_out[i] = (int32_t)scored[i].idx;
    weights_out[i] = denom <= 1.1920929e-07f ? route_scale / (float)std::max<size_t>(topk, 1)
                                              : scored[i].w / denom * route_scale;
  }
  return k;
}

// ---------------------------------------------------------------------------
// mHC hyper-connections (src/compute.rs:4945-5132)

static inline float hc_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

// normalize_comb_rows / normalize_comb_cols (src/compute.rs:4993-5013)
static void hc_norm_rows(float* comb, size_t hc, float eps) {
  for (size_t j = 0; j < hc; ++j) {
    float sum = 0.0f;  // row.iter().sum(): in order
    for (size_t k = 0; k < hc; ++k) sum += comb[j * hc + k];
    for (size_t k = 0; k < hc; ++k) comb[j * hc + k] /= sum + eps;
  }
}
static void hc_norm_cols(float* comb, size_t hc, float eps) {
  for (size_t k = 0; k < hc; ++k) {
    float sum = 0.0f;
    for (size_t j = 0; j < hc; ++j) sum += comb[j * hc + k];
    for (size_t j = 0; j < hc; ++j) comb[j * hc + k] /= sum + eps;
  }
}

// hc_split_sinkhorn_scalar (src/compute.rs:4945-4991)
int orc_hc_split_sinkhorn(const float* mixes, size_t mixes_len, const float* scale,
                          size_t scale_len, const float* base, size_t base_len, size_t hc,
                          size_t iters, float eps, float* pre, float* post, float* comb) {
  size_t mix_hc = (2 + hc) * hc;
  if (mixes_len < mix_hc || base_len < mix_hc || scale_len < 3) return ORC_ERR_INVALID_SHAPE;
  for (size_t j = 0; j < hc; ++j) {
    pre[j] = hc_sigmoid(mixes[j] * scale[0] + base[j]) + eps;
    post[j] = 2.0f * hc_sigmoid(mixes[j + hc] * scale[1] + base[j + hc]);
  }
  for (size_t j = 0; j < hc; ++j)
    for (size_t k = 0; k < hc; ++k)
      comb[j * hc + k] = mixes[2 * hc + j * hc + k] * scale[2] + base[2 * hc + j * hc + k];
  for (size_t j = 0; j < hc; ++j) {
    float* row = comb + j * hc;
    float mx = -INFINITY;  // fold(NEG_INFINITY, f32::max): NaN-ignoring
    for (size_t k = 0; k < hc; ++k) mx = std::fmax(mx, row[k]);
    float sum = 0.0f;
    for (size_t k = 0; k < hc; ++k) {
      row[k] = expf(row[k] - mx);
      sum += row[k];
    }
    for (size_t k = 0; k < hc; ++k) row[k] = row[k] / sum + eps;
  }
  hc_norm_cols(comb, hc, eps);
  for (size_t it = 1; it < iters; ++it) {
    hc_norm_rows(comb, hc, eps);
    hc_norm_cols(comb, hc, eps);
  }
  return ORC_OK;
}

// sum of squares / hc_dim, then 1 / sqrt(. + eps) (src/compute.rs:5028-5034)
static float hc_inv_rms(const float* x, size_t hc_dim, float eps) {
  float sum = 0.0f;
  for (size_t i = 0; i < hc_dim; ++i) sum += x[i] * x[i];
  float mean_square = sum / (float)hc_dim;
  return 1.0f / std::sqrt(mean_square + eps);
}

// dot_f32_row (src/compute.rs:4875-4884)
static float hc_dot(const float* row, const float* x, size_t n) {
  float acc = 0.0f;
  for (size_t i = 0; i < n; ++i) acc += row[i] * x[i];
  return acc;
}

// hc_pre_into (src/compute.rs:5016-5053)
int orc_hc_pre(const float* fn, size_t mix_hc, size_t fn_hc_dim, const float* scale,
               size_t scale_len, const float* base, const float* x, size_t hc, size_t hidden,
               size_t iters, float eps, float* y, float* post, float* comb) {
  size_t hc_dim = hc * hidden;
  if (fn_hc_dim != hc_dim) return ORC_ERR_INVALID_SHAPE;
  float inv_rms = hc_inv_rms(x, hc_dim, eps);
  std::vector<float> mixes(mix_hc), pre(hc);
  for (size_t j = 0; j < mix_hc; ++j) mixes[j] = hc_dot(fn + j * hc_dim, x, hc_dim) * inv_rms;
  int st = orc_hc_split_sinkhorn(mixes.data(), mix_hc, scale, scale_len, base, mix_hc, hc, iters,
                                 eps, pre.data(), post, comb);
  if (st != ORC_OK) return st;
  for (size_t d = 0; d < hidden; ++d) {
    float acc = 0.0f;
    for (size_t i = 0; i < hc; ++i) acc += pre[i] * x[i * hidden + d];
    y[d] = acc;
  }
  return ORC_OK;
}

// hc_post_into (src/compute.rs:5055-5089): out[k] = post[k] y + sum_i comb[k][i] res[i]
void orc_hc_post(const float* y, const float* residual, const float* post, const float* comb,
                 float* out, size_t hc, size_t hidden) {
  for (size_t k = 0; k < hc; ++k)
    for (size_t d = 0; d < hidden; ++d) {
      float acc = post[k] * y[d];
      for (size_t i = 0; i < hc; ++i) acc += comb[k * hc + i] * residual[i * hidden + d];
      out[k * hidden + d] = acc;
    }
}

// hc_head_pool (src/compute.rs:5091-5132)
void orc_hc_head(const float* fn, float scale, const float* base, const float* x, size_t hc,
                 size_t hidden, float eps, float* pooled) {
  size_t hc_dim = hc * hidden;
  float inv_rms = hc_inv_rms(x, hc_dim, eps);
  std::vector<float> pre(hc);
  for (size_t j = 0; j < hc; ++j) {
    float mix = hc_dot(fn + j * hc_dim, x, hc_dim) * inv_rms;
    pre[j] = hc_sigmoid(mix * scale + base[j]) + eps;
  }
  for (size_t d = 0; d < hidden; ++d) {
    float acc = 0.0f;
    for (size_t i = 0; i < hc; ++i) acc += pre[i] * x[i * hidden + d];
    pooled[d] = acc;
  }
}

void orc_expf_n(const float* x, float* y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = expf(x[i]);
}

// rope_inv_freqs (src/compute.rs:2591-2621)
void orc_rope_inv_freqs(size_t rope_dim, float theta, float yarn_factor, float beta_fast,
                        float beta_slow, size_t original_seq_len, float* out) {
  size_t pairs = rope_dim / 2;
  for (size_t pair = 0; pair < pairs; ++pair)
    out[pair] = powf(theta, -((float)(2 * pair)) / (float)rope_dim);
  if (yarn_factor <= 0.0f || original_seq_len == 0) return;
  float dim = (float)rope_dim;
  float base_ln = logf(theta);
  const float PI = 3.14159265358979323846f;  // std::f32::consts::PI
  auto find_correction_dim = [&](float num_rotations) {
    return dim * logf((float)original_seq_len / (num_rotations * 2.0f * PI)) / (2.0f * base_ln);
  };
  float low = std::fmax(floorf(find_correction_dim(beta_fast)), 0.0f);
  float high = std::fmin(ceilf(find_correction_dim(beta_slow)), dim - 1.0f);
  if (std::fabs(low - high) < 1.1920929e-07f) high = low + 0.001f;
  for (size_t pair = 0; pair < pairs; ++pair) {
    float ramp = (((float)pair) - low) / (high - low);
    ramp = ramp < 0.0f ? 0.0f : (ramp > 1.0f ? 1.0f : ramp);  // clamp(0.0, 1.0): NaN stays
    float smooth = 1.0f - ramp;
    out[pair] = out[pair] / yarn_factor * (1.0f - smooth) + out[pair] * smooth;
  }
}

// apply_rope_interleaved_with_freqs (src/compute.rs:2623-2651)
static void rope_pairs(float* values, size_t position, const float* inv_freqs, size_t pairs,
                       bool inverse) {
  float pos = (float)position;
  for (size_t pair = 0; pair < pairs; ++pair) {
    float angle = pos * inv_freqs[pair];
    float s = sinf(angle), c = cosf(angle);
    if (inverse) s = -s;
    float even = values[2 * pair], odd = values[2 * pair + 1];
    values[2 * pair] = even * c - odd * s;
    values[2 * pair + 1] = even * s + odd * c;
  }
}

// the attention core of compute_deepseek_v4_mla_attention (src/compute.rs:4080-4185)
void orc_mla_attention(const float* q, size_t heads, size_t head_dim, size_t nope_dim,
                       const float* keys, size_t key_stride, size_t token_pos, size_t window,
                       const float* compressed, size_t compressed_count, const float* sink,
                       const float* inv_freqs, float* out) {
  const float scale = powf((float)head_dim, -0.5f);
  size_t context = token_pos + 1;
  size_t window_start = context > window ? context - window : 0;
  for (size_t i = 0; i < heads * head_dim; ++i) out[i] = 0.0f;
  auto dot = [&](const float* a, const float* b) {
    float score = 0.0f;
    for (size_t d = 0; d < head_dim; ++d) score += a[d] * b[d];
    return score;
  };
  for (size_t head = 0; head < heads; ++head) {
    const float* qh = q + head * head_dim;
    float max_score = -INFINITY;
    for (size_t pos = window_start; pos < context; ++pos) {
      float score = dot(qh, keys + pos * key_stride) * scale;
      if (score > max_score) max_score = score;
    }
    for (size_t b = 0; b < compressed_count; ++b) {
      float score = dot(qh, compressed + b * head_dim) * scale;
      if (score > max_score) max_score = score;
    }
    float denom = 0.0f;
    if (sink) denom += expf(sink[head] - max_score);
    float* oh = out + head * head_dim;
    float weights_sum = 0.0f;
    for (size_t pos = window_start; pos < context; ++pos) {
      const float* key = keys + pos * key_stride;
      float score = dot(qh, key);
      float weight = expf((score * scale) - max_score);
      weights_sum += weight;
      for (size_t d = 0; d < head_dim; ++d) oh[d] += weight * key[d];
    }
    for (size_t b = 0; b < compressed_count; ++b) {
      const float* key = compressed + b * head_dim;
      float score = dot(qh, key);
      float weight = expf((score * scale) - max_score);
      weights_sum += weight;
      for (size_t d = 0; d < head_dim; ++d) oh[d] += weight * key[d];
    }
    denom += weights_sum;
    if (denom > 0.0f)
      for (size_t d = 0; d < head_dim; ++d) oh[d] /= denom;
    rope_pairs(oh + nope_dim, token_pos, inv_freqs, (head_dim - nope_dim) / 2, true);
  }
}

// score_bf16_lm_head_topk + push_topk_candidate + the final sort
// (src/compute.rs:2838-2962)
int orc_lm_head_topk(const uint16_t* weight, size_t rows, size_t cols, const float* x,
                     size_t top_k, uint32_t row_base, uint32_t* tokens_out, float* logits_topk,
                     float* logits_out) {
  if (rows == 0) return -1;
  top_k = std::max<size_t>(top_k, 1);
  std::vector<float> logits(rows);
  orc_bf16_gemv(weight, rows, cols, x, logits.data());
  if (logits_out) std::copy(logits.begin(), logits.end(), logits_out);
  auto key = [](float f) {  // f32::total_cmp key
    int32_t b;
    std::memcpy(&b, &f, 4);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
  };
  std::vector<std::pair<uint32_t, float>> best;
  best.reserve(std::min<size_t>(top_k, 64));
  for (size_t r = 0; r < rows; ++r) {
    const uint32_t token = row_base + (uint32_t)r;
    const float logit = logits[r];
    if (best.size() < top_k) {
      best.push_back({token, logit});
      continue;
    }
    // min_by(total_cmp): the first of equal minima
    size_t worst = 0;
    for (size_t i = 1; i < best.size(); ++i)
      if (key(best[i].second) < key(best[worst].second)) worst = i;
    if (logit > best[worst].second) best[worst] = {token, logit};
  }
  // sort_by(|l, r| r.total_cmp(l)): stable, descending
  std::stable_sort(best.begin(), best.end(),
                   [&](const std::pair<uint32_t, float>& l, const std::pair<uint32_t, float>& r) {
                     return key(l.second) > key(r.second);
                   });
  for (size_t i = 0; i < best.size(); ++i) {
    tokens_out[i] = best[i].first;
    logits_topk[i] = best[i].second;
  }
  return (int)best.size();
}

// compute_active_and_shared_experts (src/compute.rs:1872-1946)
int orc_moe_combine_token(const orc_fp4_expert* experts, const int32_t* ids, const float* weights,
                          size_t topk, const orc_fp4_expert* shared_fp4,
                          const orc_fp8_expert* shared_fp8, const float* x, size_t hidden,
                          float* y) {
  std::vector<float> routed(hidden, 0.0f), shared(hidden, 0.0f);
  bool applied = shared_fp4 || shared_fp8;
  if (topk > 0) {
    int st = combine_routed(experts, ids, weights, topk, x, hidden, routed.data());
    if (st != ORC_OK) return st;
  }
  if (shared_fp4) {
    std::vector<float> scr(2 * shared_fp4->w1.rows);
    int st = fp4_expert_forward(*shared_fp4, x, hidden, shared.data(), hidden, scr.data(),
                                scr.size());
    if (st != ORC_OK) return st;
  } else if (shared_fp8) {
    int st = orc_fp8_expert_forward(shared_fp8, x, hidden, shared.data());
    if (st != ORC_OK) return st;
  }
  for (size_t i = 0; i < hidden; ++i) {
    if (topk == 0)
      y[i] = applied ? shared[i] : x[i];
    else
      y[i] = applied ? shared[i] + routed[i] : routed[i];
  }
  return ORC_OK;
}

// Expert-major batched MoE (src/compute.rs:1779-1810,1817-1870;
// src/server/generation.rs:2487-2606).  Per-position weights are
// score/sum(scores) (uniform if not finite); the union is walked in ascending
// expert id (the BTreeMap order; the engine's I/O-completion order inside a
// chunk makes its own cross-expert order vary run to run).
int orc_moe_batched(const orc_fp4_expert* experts, size_t num_experts, const int32_t* ids,
                    const float* weights, size_t tokens, size_t topk,
                    const orc_fp4_expert* shared_fp4, const float* x, size_t hidden, float* y) {
  std::map<int32_t, std::vector<std::pair<size_t, float>>> uni;
  for (size_t t = 0; t < tokens; ++t) {
    const int32_t* id = ids + t * topk;
    const float* w = weights + t * topk;
    float sum = 0.0f;
    bool finite = true;
    for (size_t k = 0; k < topk; ++k) {
      sum += w[k];
      finite = finite && std::isfinite(w[k]);
    }
    finite = finite && std::isfinite(sum) && sum > 0.0f;
    float uniform = 1.0f / (float)topk;
    for (size_t k = 0; k < topk; ++k) {
      if (id[k] < 0 || (size_t)id[k] >= num_experts) return ORC_ERR_INVALID_SHAPE;
      uni[id[k]].push_back({t, finite ? w[k] / sum : uniform});
    }
  }
  std::vector<float> acc(tokens * hidden, 0.0f);
  std::vector<char> seen(tokens, 0);
  std::vector<std::pair<int32_t, std::vector<std::pair<size_t, float>>*>> order;
  for (auto& kv : uni) order.push_back({kv.first, &kv.second});
  // experts are independent: parallelise over experts, then accumulate in
  // expert-id order so the result does not depend on the thread split.
  std::vector<std::vector<float>> outs(order.size());
  int threads = std::max(1, thread_count());
  std::vector<std::thread> pool;
  std::mutex mu;
  int first = ORC_OK;
  size_t next = 0;
  for (int th = 0; th < threads; ++th) {
    pool.emplace_back([&]() {
      int saved = orc_get_threads();
      (void)saved;
      for (;;) {
        size_t i;
        {
          std::lock_guard<std::mutex> g(mu);
          if (next >= order.size() || first != ORC_OK) return;
          i = next++;
        }
        const orc_fp4_expert& e = experts[order[i].first];
        auto& targets = *order[i].second;
        std::vector<float> out(targets.size() * hidden), scr(2 * e.w1.rows);
        for (size_t j = 0; j < targets.size(); ++j) {
          int st = fp4_expert_forward(e, x + targets[j].first * hidden, hidden,
                                      out.data() + j * hidden, hidden, scr.data(), scr.size());
          if (st != ORC_OK) {
            std::lock_guard<std::mutex> g(mu);
            if (first == ORC_OK) first = st;
            return;
          }
        }
        outs[i] = std::move(out);
      }
    });
  }
  for (auto& t : pool) t.join();
  if (first != ORC_OK) return first;
  for (size_t i = 0; i < order.size(); ++i) {
    auto& targets = *order[i].second;
    for (size_t j = 0; j < targets.size(); ++j) {
      size_t pos = targets[j].first;
      float w = targets[j].second;
      seen[pos] = 1;
      float* a = acc.data() + pos * hidden;
      const float* v = outs[i].data() + j * hidden;
      for (size_t h = 0; h < hidden; ++h) a[h] += v[h] * w;
    }
  }
  // finish_layer_deepseek_mhc_phase2_batch (src/compute.rs:1817-1870)
  std::vector<float> sh(hidden);
  for (size_t t = 0; t < tokens; ++t) {
    float* out = y + t * hidden;
    const float* xt = x + t * hidden;
    bool applied = shared_fp4 != nullptr;
    if (applied) {
      std::vector<float> scr(2 * shared_fp4->w1.rows);
      int st = fp4_expert_forward(*shared_fp4, xt, hidden, sh.data(), hidden, scr.data(),
                                  scr.size());
      if (st != ORC_OK) return st;
    }
    for (size_t h = 0; h < hidden; ++h) {
      float r = acc[t * hidden + h];
      if (seen[t])
        out[h] = applied ? sh[h] + r : r;
      else
        out[h] = applied ? sh[h] : xt[h];
    }
  }
  return ORC_OK;
}


static inline float bf16_value(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// apply_weighted_rms_norm (src/compute.rs:3077-3115) / rms_norm_in_place
// (src/compute.rs:7110-7122): the mean of squares summed in index order
// (Iterator::sum), eps 1e-6, then (x * inv_rms) * weight.
void orc_rms_norm(const float* in, size_t n, const uint16_t* weight_bf16, float* out) {
  if (n == 0) return;
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) sum += in[i] * in[i];
  const float mean_square = sum / (float)n;
  const float inv_rms = 1.0f / sqrtf(mean_square + 1.0e-6f);
  for (size_t i = 0; i < n; ++i)
    out[i] = weight_bf16 ? in[i] * inv_rms * bf16_value(weight_bf16[i]) : in[i] * inv_rms;
}

// compute_deepseek_v4_mla_attention (src/compute.rs:3924-4293), the compressor's
// rows given: q path (:3994-4040), kv path (:4041-4075), the attention core
// (orc_mla_attention, :4080-4185), the grouped output projection (:4230-4293).
int orc_v4_attention(const orc_v4_attn* L, size_t token_pos, float* hidden, float* kv_cache,
                     size_t kv_stride, const float* compressed, size_t compressed_count,
                     const float* inv_freqs) {
  const size_t hd = L->head_dim, nope = L->nope_dim, heads = L->heads, hidden_n = L->hidden;
  const size_t q_full = heads * hd, groups = L->o_groups, o_lora = L->o_lora_rank;
  if (groups == 0 || o_lora == 0 || q_full % groups != 0) return ORC_ERR_INVALID_SHAPE;
  const size_t group_in = q_full / groups, o_mid_len = groups * o_lora;
  std::vector<float> x_fp8(hidden, hidden + hidden_n), q_lora(L->q_lora_rank), q(q_full),
      kv(hd), attn(q_full), o_mid(o_mid_len);
  act_quant(x_fp8.data(), x_fp8.size(), 64);
  int st = fp8_gemv_full(L->wq_a, x_fp8.data(), q_lora.data());
  if (st != ORC_OK) return st;
  orc_rms_norm(q_lora.data(), q_lora.size(), L->q_norm, q_lora.data());
  act_quant(q_lora.data(), q_lora.size(), 64);
  if ((st = fp8_gemv_full(L->wq_b, q_lora.data(), q.data())) != ORC_OK) return st;
  for (size_t h = 0; h < heads; ++h) orc_rms_norm(&q[h * hd], hd, nullptr, &q[h * hd]);
  for (size_t h = 0; h < heads; ++h)
    rope_pairs(&q[h * hd + nope], token_pos, inv_freqs, (hd - nope) / 2, false);
  if ((st = fp8_gemv_full(L->wkv, x_fp8.data(), kv.data())) != ORC_OK) return st;
  orc_rms_norm(kv.data(), hd, L->kv_norm, kv.data());
  rope_pairs(&kv[nope], token_pos, inv_freqs, (hd - nope) / 2, false);
  act_quant(kv.data(), nope, 64);
  std::copy(kv.begin(), kv.end(), kv_cache + token_pos * kv_stride);
  orc_mla_attention(q.data(), heads, hd, nope, kv_cache, kv_stride, token_pos, L->window,
                    compressed, compressed_count, L->sink, inv_freqs, attn.data());
  act_quant(attn.data(), attn.size(), 64);
  for (size_t g = 0; g < groups; ++g) {
    const orc_fp8_matrix& m = L->wo_a;
    st = orc_fp8_gemv_rows(m.weight, m.rows * m.cols, m.rows, m.cols, m.scale,
                           m.scale_rows * m.scale_cols, m.scale_rows, m.scale_cols, g * o_lora,
                           (g + 1) * o_lora, &attn[g * group_in], group_in, &o_mid[g * o_lora],
                           o_lora);
    if (st != ORC_OK) return st;
  }
  act_quant(o_mid.data(), o_mid.size(), 64);
  return fp8_gemv_full(L->wo_b, o_mid.data(), hidden);
}

}  // extern "C"
