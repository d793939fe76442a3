// v4attn.cu -- the projection path of DeepSeek-V4's MLA attention for one
// decode token (compute_deepseek_v4_mla_attention, src/compute.rs:3924-4293)
// around the attention core of mla.cu, and the weighted RMS norm the layer
// applies before it and before the MoE (apply_weighted_rms_norm,
// src/compute.rs:3077-3115; rms_norm_in_place, src/compute.rs:7110-7122).
//
//   x_fp8 = act_quant(x)                       (fused into the FP8 GEMVs)
//   q_lora = wq_a x_fp8; q_norm; act_quant     (wh_fp8_gemv + norm_kernel)
//   q = wq_b q_lora; per-head RMS; RoPE        (wh_fp8_gemv + norm_kernel)
//   kv = wkv x_fp8; kv_norm; RoPE on the rope dims; act_quant of the nope
//   dims; the row stored into the layer's KV cache at token_pos  (norm_kernel)
//   attention core (wh_mla_attention)
//   o_mid = grouped wo_a act_quant(attn)       (wh_fp8_gemv_grouped)
//   out = wo_b act_quant(o_mid)                (wh_fp8_gemv)
//
// Every step is the reference's arithmetic in its order: the mean of squares
// is summed in index order by one thread (the sum is a dependent chain, as in
// the reference's Iterator::sum), then 1/sqrt(ms + 1e-6) and (x * inv) * w
// without fused multiply-adds; RoPE pairs as (e*c - o*s, e*s + o*c) with the
// cos/sin of pos * inv_freq from the host C library (f32::sin_cos).
#include "common.cuh"
#include "kernels.cuh"
#include <vector>

namespace wh {

constexpr int kNormThreads = 256;
constexpr int kNormMaxLen = 4096;   // floats of one segment staged in shared memory
constexpr int kNormMaxPairs = 64;

constexpr int kNormMaxTok = 32;      // tokens of one launch when segments are per token

struct NormArgs {
  const float* in;
  float* out;
  int segments, n, in_stride, out_stride;
  const uint16_t* weight;  // bf16 [n] or null (unweighted)
  int rope_off, rope_pairs;
  float rope_cos[kNormMaxPairs], rope_sin[kNormMaxPairs];
  int aq_len;              // act quant (block 64) of [0, aq_len) after the rope
  // token mapping (seg_per_tok > 0): segment s is segment s % seg_per_tok of
  // token tok[s / seg_per_tok], at in/out + tok * tok_stride + (s % seg_per_tok) * stride
  int seg_per_tok;
  long long tok_stride;
  int tok[kNormMaxTok];
  float* copy[kNormMaxTok];  // nullable: a copy of the token's output segment (KV row)
  uint32_t* status;
};

__device__ __forceinline__ long long norm_seg_off(const NormArgs& a, int seg, int stride) {
  if (a.seg_per_tok <= 0) return (long long)seg * stride;
  return (long long)a.tok[seg / a.seg_per_tok] * a.tok_stride +
         (long long)(seg % a.seg_per_tok) * stride;
}

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

__global__ void __launch_bounds__(kNormThreads) norm_kernel(NormArgs a) {
  __shared__ float v[kNormMaxLen];
  __shared__ float sq[kNormMaxLen];
  __shared__ float inv_s;
  const int seg = blockIdx.x;
  const float* in = a.in + norm_seg_off(a, seg, a.in_stride);
  pdl_wait_prior();
  for (int i = threadIdx.x; i < a.n; i += blockDim.x) {
    const float x = in[i];
    v[i] = x;
    sq[i] = __fmul_rn(x, x);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // the reference's sum in index order (one dependent chain)
    float s = 0.0f;
    int i = 0;
    for (; i + 8 <= a.n; i += 8) {
      float t[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) t[k] = sq[i + k];
#pragma unroll
      for (int k = 0; k < 8; ++k) s = __fadd_rn(s, t[k]);
    }
    for (; i < a.n; ++i) s = __fadd_rn(s, sq[i]);
    const float ms = __fdiv_rn(s, (float)a.n);
    inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, 1.0e-6f)));
  }
  __syncthreads();
  const float inv = inv_s;
  for (int i = threadIdx.x; i < a.n; i += blockDim.x) {
    const float t = __fmul_rn(v[i], inv);
    v[i] = a.weight ? __fmul_rn(t, bf16_to_f32(a.weight[i])) : t;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < a.rope_pairs; p += blockDim.x) {
    const float c = a.rope_cos[p], s = a.rope_sin[p];
    float* e = v + a.rope_off + 2 * p;
    const float even = e[0], odd = e[1];
    e[0] = __fsub_rn(__fmul_rn(even, c), __fmul_rn(odd, s));
    e[1] = __fadd_rn(__fmul_rn(even, s), __fmul_rn(odd, c));
  }
  __syncthreads();
  if (a.aq_len > 0) {
    act_quant_smem_warp(v, a.aq_len, 64, threadIdx.x >> 5, blockDim.x >> 5, threadIdx.x & 31,
                        &c_aq);
    __syncthreads();
  }
  float* out = a.out + norm_seg_off(a, seg, a.out_stride);
  float* cp = a.seg_per_tok > 0 && seg < kNormMaxTok * a.seg_per_tok
                  ? a.copy[seg / a.seg_per_tok]
                  : nullptr;
  if (cp) cp += (long long)(seg % a.seg_per_tok) * a.n;
  for (int i = threadIdx.x; i < a.n; i += blockDim.x) {
    const float x = v[i];
    out[i] = x;
    if (cp) cp[i] = x;
  }
  pdl_launch_dependents();
}

cudaError_t launch_norm(const NormArgs& a, cudaStream_t stream) {
  norm_kernel<<<a.segments, kNormThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace wh

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
namespace {

wh_status norm_check(int segments, int n, int in_stride, int out_stride) {
  if (segments < 1 || n < 1 || in_stride < n || out_stride < n)
    return fail(WH_ERR_INVALID_SHAPE, "rms norm shape");
  if (n > wh::kNormMaxLen) return fail(WH_ERR_UNSUPPORTED, "rms norm segment > 4096 floats");
  return WH_OK;
}

void rope_cos_sin(wh::NormArgs& a, int token_pos, const float* inv_freqs, int pairs) {
  const float pos = (float)token_pos;
  for (int i = 0; i < pairs; ++i) {
    const float angle = pos * inv_freqs[i];
    a.rope_sin[i] = sinf(angle);
    a.rope_cos[i] = cosf(angle);
  }
}

}  // namespace

extern "C" {

wh_status wh_rms_norm(wh_ctx* c, const float* in, float* out, int segments, int n,
                      const uint16_t* weight_bf16, wh_stream_t stream) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "ctx is null");
  if (wh_status st = norm_check(segments, n, n, n)) return st;
  if (!in || !out) return fail(WH_ERR_INVALID_POINTER, "null pointer");
  wh::NormArgs a{};
  a.in = in;
  a.out = out;
  a.segments = segments;
  a.n = n;
  a.in_stride = n;
  a.out_stride = n;
  a.weight = weight_bf16;
  a.status = c->status;
  WH_CUDA(wh::launch_norm(a, (cudaStream_t)stream));
  return WH_OK;
}

size_t wh_v4_attention_scratch_len(const wh_v4_attn* L, int tokens) {
  if (!L || tokens < 1) return 0;
  auto up64 = [](size_t n) { return (n + 63) & ~size_t(63); };
  const size_t q_full = (size_t)L->heads * L->head_dim;
  return (size_t)tokens * (up64(L->q_lora_rank) + up64(q_full) + up64(L->head_dim) +
                           up64(q_full) + up64((size_t)L->o_groups * L->o_lora_rank));
}

wh_status wh_v4_attention(wh_ctx* c, const wh_v4_attn* L, int tokens, const int* token_pos,
                          float* hidden, float* const* kv_caches, int kv_stride,
                          const float* const* compressed, const int* compressed_count,
                          const float* inv_freqs, float* scratch, size_t scratch_len,
                          wh_stream_t stream) {
  if (!c || !L) return fail(WH_ERR_INVALID_POINTER, "null ctx/layer");
  const int hd = L->head_dim, nope = L->nope_dim, heads = L->heads;
  const int q_full = heads * hd;
  if (tokens < 1 || !token_pos || !kv_caches)
    return fail(tokens < 1 ? WH_ERR_EMPTY_SHAPE : WH_ERR_INVALID_POINTER, "tokens");
  if (tokens > wh::kNormMaxTok) return fail(WH_ERR_UNSUPPORTED, "more than 32 tokens per call");
  if (hd < 1 || heads < 1 || nope < 0 || nope > hd || (hd - nope) % 2 != 0 ||
      L->q_lora_rank < 1 || L->o_groups < 1 || L->o_lora_rank < 1 || q_full % L->o_groups != 0 ||
      L->hidden < 1 || kv_stride < hd || L->window < 1)
    return fail(WH_ERR_INVALID_SHAPE, "MLA o_groups configuration");
  for (int t = 0; t < tokens; ++t)
    if (token_pos[t] < 0 || (compressed_count && compressed_count[t] < 0))
      return fail(WH_ERR_INVALID_SHAPE, "token position / compressed count");
  const int group_in = q_full / L->o_groups, o_mid = L->o_groups * L->o_lora_rank;
  // the projections' shapes (tensor_by_role_with_cols, src/compute.rs:3994-4260)
  if (L->wq_a.cols != L->hidden || L->wq_a.rows != L->q_lora_rank ||
      L->wq_b.cols != L->q_lora_rank || L->wq_b.rows != q_full || L->wkv.cols != L->hidden ||
      L->wkv.rows != hd || L->wo_a.cols != group_in || L->wo_a.rows != o_mid ||
      L->wo_b.cols != o_mid || L->wo_b.rows != L->hidden)
    return fail(WH_ERR_INVALID_SHAPE, "MLA projection shapes");
  const int pairs = (hd - nope) / 2;
  if (pairs > wh::kNormMaxPairs || (pairs > 0 && nope % 2 != 0))
    return fail(WH_ERR_UNSUPPORTED, "rope part > 128 or odd nope_dim");
  if (hd > wh::kNormMaxLen || L->q_lora_rank > wh::kNormMaxLen)
    return fail(WH_ERR_UNSUPPORTED, "norm segment > 4096 floats");
  if (scratch_len < wh_v4_attention_scratch_len(L, tokens))
    return fail(WH_ERR_SCRATCH_TOO_SMALL, "v4 attention scratch too small");
  if (!hidden || !scratch || (pairs > 0 && !inv_freqs))
    return fail(WH_ERR_INVALID_POINTER, "null pointer");
  for (int t = 0; t < tokens; ++t)
    if (!kv_caches[t] || (compressed_count && compressed_count[t] > 0 &&
                          (!compressed || !compressed[t])))
      return fail(WH_ERR_INVALID_POINTER, "null KV cache / compressed rows");
  // scratch, each part [tokens][len] with 64-float aligned rows:
  // q_lora | q | kv | attn_out | o_mid
  auto up64 = [](size_t n) { return (n + 63) & ~size_t(63); };
  const int ld_ql = (int)up64(L->q_lora_rank), ld_q = (int)up64(q_full), ld_kv = (int)up64(hd),
            ld_om = (int)up64(o_mid);
  float* q_lora = scratch;
  float* q = q_lora + (size_t)tokens * ld_ql;
  float* kv = q + (size_t)tokens * ld_q;
  float* attn = kv + (size_t)tokens * ld_kv;
  float* omid = attn + (size_t)tokens * ld_q;
  cudaStream_t s = (cudaStream_t)stream;
  wh_status st;
  // q path: wq_a over every token (the weights are read once for the batch)
  if ((st = wh_fp8_gemv(c, L->wq_a.weight, L->wq_a.scale, L->wq_a.rows, L->wq_a.cols,
                        L->wq_a.scale_rows, L->wq_a.scale_cols, 0, L->wq_a.rows, hidden, tokens,
                        L->hidden, q_lora, ld_ql, 64, stream)) != WH_OK)
    return st;
  wh::NormArgs nq{};
  nq.in = q_lora;
  nq.out = q_lora;
  nq.segments = tokens;
  nq.n = L->q_lora_rank;
  nq.in_stride = nq.out_stride = ld_ql;
  nq.weight = L->q_norm;
  nq.aq_len = L->q_lora_rank;
  nq.status = c->status;
  WH_CUDA(wh::launch_norm(nq, s));
  if ((st = wh_fp8_gemv(c, L->wq_b.weight, L->wq_b.scale, L->wq_b.rows, L->wq_b.cols,
                        L->wq_b.scale_rows, L->wq_b.scale_cols, 0, L->wq_b.rows, q_lora, tokens,
                        ld_ql, q, ld_q, 0, stream)) != WH_OK)
    return st;
  // kv path
  if ((st = wh_fp8_gemv(c, L->wkv.weight, L->wkv.scale, L->wkv.rows, L->wkv.cols,
                        L->wkv.scale_rows, L->wkv.scale_cols, 0, L->wkv.rows, hidden, tokens,
                        L->hidden, kv, ld_kv, 64, stream)) != WH_OK)
    return st;
  // per-head RMS + RoPE of q, and kv_norm + RoPE + act quant + cache store,
  // one launch each per distinct position (the cos/sin are launch arguments)
  std::vector<char> done(tokens, 0);
  for (int t0 = 0; t0 < tokens; ++t0) {
    if (done[t0]) continue;
    wh::NormArgs nh{};
    nh.in = q;
    nh.out = q;
    nh.n = hd;
    nh.in_stride = nh.out_stride = hd;
    nh.rope_off = nope;
    nh.rope_pairs = pairs;
    rope_cos_sin(nh, token_pos[t0], inv_freqs, pairs);
    nh.seg_per_tok = heads;
    nh.tok_stride = ld_q;
    nh.status = c->status;
    wh::NormArgs nk = nh;
    nk.in = kv;
    nk.out = kv;
    nk.seg_per_tok = 1;
    nk.tok_stride = ld_kv;
    nk.weight = L->kv_norm;
    nk.aq_len = nope;
    int m = 0;
    for (int t = t0; t < tokens; ++t)
      if (!done[t] && token_pos[t] == token_pos[t0]) {
        done[t] = 1;
        nh.tok[m] = nk.tok[m] = t;
        nk.copy[m] = kv_caches[t] + (long long)token_pos[t] * kv_stride;
        ++m;
      }
    nh.segments = m * heads;
    nk.segments = m;
    WH_CUDA(wh::launch_norm(nh, s));
    WH_CUDA(wh::launch_norm(nk, s));
  }
  // attention core, every token in one set of launches
  MlaToken mt[wh::kNormMaxTok];
  for (int t = 0; t < tokens; ++t) {
    const int cc = compressed_count ? compressed_count[t] : 0;
    mt[t] = MlaToken{q + (size_t)t * ld_q, kv_caches[t], token_pos[t],
                     cc > 0 ? compressed[t] : nullptr, cc, attn + (size_t)t * ld_q};
  }
  if ((st = mla_attention_tokens(c, heads, hd, nope, kv_stride, L->window, L->sink, inv_freqs, mt,
                                 tokens, stream)) != WH_OK)
    return st;
  // grouped low-rank output projection (src/compute.rs:4244-4293)
  if ((st = wh_fp8_gemv_grouped(c, L->wo_a.weight, L->wo_a.scale, L->wo_a.rows, L->wo_a.cols,
                                L->wo_a.scale_rows, L->wo_a.scale_cols, 0, o_mid, attn, tokens,
                                ld_q, L->o_lora_rank, group_in, omid, ld_om, 64, stream)) != WH_OK)
    return st;
  return wh_fp8_gemv(c, L->wo_b.weight, L->wo_b.scale, L->wo_b.rows, L->wo_b.cols,
                     L->wo_b.scale_rows, L->wo_b.scale_cols, 0, L->wo_b.rows, omid, tokens, ld_om,
                     hidden, L->hidden, 64, stream);
}

}  // extern "C"
