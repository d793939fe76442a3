// kernels.cuh -- argument blocks and launchers of the wohper_b200 kernels
// (internal to the library; the public surface is include/wohper_b200.h).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"

namespace wh {

// Raise a kernel's dynamic shared-memory limit once per (device, kernel); the
// attribute call is not repeated on the launch path.
cudaError_t ensure_smem_attr(const void* kernel, size_t bytes);
template <class K>
inline cudaError_t ensure_smem(K* kernel, size_t bytes) {
  return ensure_smem_attr(reinterpret_cast<const void*>(kernel), bytes);
}

// ---------------- the host libm's expf on the device ----------------
// Inputs where the host's expf differs from exp((double)x) rounded once, or
// lies too close to a rounding midpoint to trust the device's double exp:
// keys ascending (float bits as uint32), vals the host expf.
struct ExpfTable {
  const uint32_t* keys;
  const float* vals;
  const uint32_t* bucket;  // [2^20 + 1]: first key index of each (bits >> 12) bucket
  int n;
  // relative distance from a rounding midpoint within which x is looked up: a
  // power of two at least twice the farthest host difference measured, and at
  // least the 2^-44 band the table holds in full
  double near;
};
constexpr int kExpfBucketShift = 12;
constexpr uint32_t kExpfBuckets = 1u << (32 - kExpfBucketShift);
bool expf_table_host(const uint32_t** keys, const float** vals, int* n);
bool expf_bucket_host(const uint32_t** bucket);
double expf_near_host();

__device__ __forceinline__ float ref_expf(float x, const ExpfTable& t) {
  const double yd = exp((double)x);
  const float c = __double2float_rn(yd);
  const uint32_t cb = __float_as_uint(c);
  const double dc = (double)c;
  const double other = (double)__uint_as_float(yd > dc ? cb + 1u : cb - 1u);
  if (fabs(yd - 0.5 * (dc + other)) <= yd * t.near) {
    // near a rounding midpoint (about 0.14 % of inputs with glibc 2.39's
    // 2^-32): x's bucket bounds, then a binary search over the bucket's few keys
    const uint32_t xb = __float_as_uint(x);
    const uint32_t b = xb >> kExpfBucketShift;
    int lo = (int)__ldg(t.bucket + b), hi = (int)__ldg(t.bucket + b + 1);
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(t.keys + mid) < xb) lo = mid + 1; else hi = mid;
    }
    if (lo < t.n && __ldg(t.keys + lo) == xb) return __ldg(t.vals + lo);
  }
  return c;
}
// The table of the current device, installed by install_expf_table (wh_ctx_create).
__constant__ ExpfTable c_expf;
__device__ __forceinline__ float libm_expf(float x) { return ref_expf(x, c_expf); }
// Builds the host table once per process and installs it on the current device
// (once per device).  Returns false when the table cannot reproduce the host expf.
bool install_expf_table(cudaError_t* err);
cudaError_t launch_ref_expf(const float* x, float* y, long long n, cudaStream_t s);

// ---------------- mHC hyper-connections ----------------
constexpr int kHcMaxHc = 8;
constexpr int kHcMaxMix = (2 + kHcMaxHc) * kHcMaxHc;
struct HcArgs {
  const float* fn;     // [rows][hc * hidden]: (2 + hc) * hc rows (hc_pre) or hc (hc_head)
  const float* scale;  // [3] (hc_pre)
  const float* base;   // [rows]
  const float* x;      // [tokens][hc * hidden]
  float* y;            // [tokens][hidden]
  float* post;         // [tokens][hc] (hc_pre)
  float* comb;         // [tokens][hc][hc] (hc_pre)
  float* dots;         // scratch [tokens][rows + 1]: x . x, then fn_j . x
  int tokens, hc, hidden, iters, head, vec4;
  float eps, head_scale;
};
size_t hc_dots_bytes(int tokens, int rows);
struct HcPostArgs {
  const float* y;         // [tokens][hidden]
  const float* residual;  // [tokens][hc * hidden]
  const float* post;      // [tokens][hc]
  const float* comb;      // [tokens][hc][hc]
  float* out;             // [tokens][hc * hidden]
  int tokens, hc, hidden;
};
cudaError_t launch_hc_mix(const HcArgs& a, cudaStream_t s);
cudaError_t launch_hc_post(const HcPostArgs& a, int num_sms, cudaStream_t s);

// ---------------- MLA attention core ----------------
struct MlaArgs {
  const float* q;           // [heads][head_dim]
  const float* keys;        // layer cache rows [positions][key_stride]
  const float* compressed;  // [compressed_count][head_dim]
  const float* sink;        // [heads] or nullptr
  float* out;               // [heads][head_dim]
  float* scores;            // scratch [window_len + compressed_count][heads]
  float* tile_max;          // scratch [tiles][heads]
  float* weights;           // scratch [heads][window_len + compressed_count]
  float* head_max;          // scratch [heads]
  int heads, head_dim, nope_dim, key_stride;
  int window_start, window_len, compressed_count;
  int smem_ld, head_group, stages, vec4;  // launch plan (mla_plan)
  float scale;
  float rope_cos[64], rope_sin[64];  // per rope pair at the token's position
};
// The launches take the arguments of up to N tokens; token z of the grid's z
// dimension reads t[z] (its own q, cache, compressed rows, window and rope).
constexpr int kMlaMaxTok = 32;
template <int N>
struct MlaBatch {
  MlaArgs t[N];
};
bool mla_plan(MlaArgs& a, size_t* smem_scores, size_t* smem_output);
size_t mla_scratch_bytes(int heads, int positions);
size_t mla_tile_count(int positions);
// every token's plan fields (smem_ld, head_group, stages) must be equal;
// smem sizes and grids are those of the token with the most positions
template <int N>
cudaError_t launch_mla_attention(const MlaBatch<N>& b, int tokens, size_t smem_scores,
                                 size_t smem_output, cudaStream_t s);

// ---------------- BF16 lm_head top-k ----------------
struct LmHeadArgs {
  const uint16_t* weight;  // [rows][cols] bf16 bits
  const float* x;          // [cols]
  long long rows;
  int cols;
  int top_k;
  uint32_t row_base;
  float* logits;      // [rows]
  uint32_t* flags;    // bit 0: a NaN logit (zeroed before the launch)
  uint32_t* counter;  // passes handed out (zeroed before the launch)
  uint32_t* cand_count;  // candidates collected (zeroed before the launch)
  int* hist;             // [4096] histogram (zeroed before the launch)
  uint64_t* cand;        // [8192] candidate keys
  uint32_t* out_tokens;
  float* out_logits;
  // several tokens in one call: token t reads x + t * ldx and owns
  // logits + t * rows, the words flags + t * kLmTokWords (flags, counter,
  // candidate count, -, histogram), cand + t * 8192 and out_* + t * top_k
  int tokens;  // 1 for the one-token call
  int ldx;
};
constexpr int kLmTokWords = 4 + 4096;
size_t lm_head_scratch_bytes(long long rows, int top_k);
size_t lm_head_batch_scratch_bytes(long long rows, int top_k, int tokens);
cudaError_t launch_lm_head_batch(const LmHeadArgs& a, bool pdl, cudaStream_t s);
bool lm_head_supported(long long rows, int cols, int top_k);
cudaError_t launch_lm_head_stage(const LmHeadArgs& a, int stage, bool pdl, cudaStream_t s);

// ---------------- FP8 GEMV ----------------
struct Fp8GemvArgs {
  const uint8_t* weight;  // [rows][cols] E4M3
  const uint8_t* scale;   // [scale_rows][scale_cols] UE8M0
  int rows, cols, scale_rows, scale_cols;
  int row_start, row_end;
  const float* x;  // [batch][ldx]
  int ldx;
  float* y;  // [batch][ldy], y[b*ldy + r - row_start]
  int ldy;
  int batch;
  int act_quant_block;  // 0 or the block size of a fused act quant of x
  int box_rows;         // rows per CTA (fast path)
  uint32_t* status;
  const float* addend;  // nullable, laid out like y: y = gemv + addend (after the finite check)
  // grouped input (the reference's grouped wo_a): row r reads x + (r / x_group_rows) *
  // x_group_off (+ b * ldx); 0 = every row reads x
  int x_group_rows;
  long long x_group_off;
};

void set_act_quant_table(const ActQuantTable& t, cudaStream_t s);
const ActQuantTable* act_quant_table_device();
// true when the one-input kernel takes the call (it then act-quantises x itself)
bool fp8_gemv_rowgroup_fits(const Fp8GemvArgs& a, int num_sms);
// wmap == nullptr selects the generic kernel; the batched kernel (2..N
// inputs, or one input the one-input kernel does not take) needs xmap: x as
// f32 [batch][ldx] with box [16 inputs][136 floats], no swizzle.
cudaError_t launch_fp8_gemv(const CUtensorMap* wmap, const CUtensorMap* xmap,
                            const Fp8GemvArgs& a, int num_sms, cudaStream_t stream, bool pdl);
cudaError_t launch_act_quant(float* v, long long n, int block, uint32_t* status, int num_sms,
                             cudaStream_t stream);

// ---------------- FP4 matvec (standalone, f32 input) ----------------
struct Fp4MatvecArgs {
  const uint8_t* packed;  // [rows][(cols+1)/2]
  const uint8_t* scales;  // [rows][scale_cols]
  int rows, cols, scale_cols;
  const float* x;
  float* y;
  uint32_t* status;
};
cudaError_t launch_fp4_matvec(const Fp4MatvecArgs& a, int num_sms, cudaStream_t stream);

// ---------------- router ----------------
struct RouterArgs {
  const uint16_t* gate;  // [experts][hidden] bf16 bits
  int experts, hidden;
  const float* x;  // [tokens][hidden]
  int tokens;
  int topk;
  int mode;            // 0 = RawLogits (softmax over the selected), 1 = DeepSeek sqrt-softplus
  const float* bias;   // nullable, mode 1 selection bias
  float route_scale;   // mode 1
  const int32_t* hash_ids;  // nullable [tokens][topk] (tid2eid rows), mode 1
  float* logits;       // [tokens][experts] scratch/output
  int32_t* ids;        // [tokens][topk]
  float* weights;      // [tokens][topk] route weights after the mode's normalisation
  float* combine_w;    // [tokens][topk] w_k / sum(w) as the combine applies them (nullable)
  uint32_t* counters;  // [tokens] zero-initialised, reset by the kernel
  uint32_t* status;
};

// ---------------- MoE (FP4 experts, one token per call or a few) ----------------
// Tensor maps for every expert's w1/w3 (box [kMoeUpRows rows][128 B]) and w2
// (box [kMoeDownRows rows][128 B]) live in device memory (built once per
// weight set).  The host builds the maps with these box heights and the
// kernels size their shared-memory stages and transaction counts from them.
constexpr int kMoeUpRows = 32;
constexpr int kMoeDownRows = 16;
struct Fp4ExpertDev {
  const uint8_t* w1_scale;  // [inter][hidden/32]
  const uint8_t* w3_scale;
  const uint8_t* w2_scale;  // [hidden][inter/32]
  const uint8_t* w1;        // packed (used by the exact fallback)
  const uint8_t* w3;
  const uint8_t* w2;
};
struct MoeArgs {
  const CUtensorMap* maps;     // [num_experts + has_shared][3] (w1, w3, w2)
  const Fp4ExpertDev* experts; // [num_experts + has_shared]
  int num_experts;             // routed experts
  int has_shared;              // slot num_experts is the shared expert
  int hidden, inter;
  const float* x;              // [tokens][hidden]
  int tokens;
  int topk;
  const int32_t* ids;          // [tokens][topk]
  const float* combine_w;      // [tokens][topk]
  float* h;                    // scratch [tokens][slots][inter] (SwiGLU hidden, f32)
  uint32_t* blk_counters;      // zeroed [tokens][slots][inter/64] arrival counters
  float* y;                    // [tokens][hidden]
  float* expert_out;           // nullable [tokens][slots][hidden] (per-expert outputs)
  int combine;                 // 1: routed combine + shared; 0: write expert_out only
  uint32_t* status;
};
cudaError_t launch_moe_up(const MoeArgs& a, int num_sms, cudaStream_t stream, bool pdl);
cudaError_t launch_moe_down(const MoeArgs& a, int num_sms, cudaStream_t stream, bool pdl);
size_t moe_up_smem_bytes(int hidden);
size_t moe_down_smem_bytes(int inter, int slots);

}  // namespace wh
