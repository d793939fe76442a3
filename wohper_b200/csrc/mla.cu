// mla.cu -- the attention core of DeepSeek-V4's MLA decode for sm_100a.
//
// Replaces the part of compute_deepseek_v4_mla_attention
// (engine/zc_infer_core/src/compute.rs:4080-4185) between the query/key path
// and the output projections.  For each head:
//   scores  s_p = (sum_d q_d * k_p,d) * scale over the sliding window
//           [max(0, pos + 1 - window), pos] of the layer's key cache, then over
//           the compressed rows; products and sums rounded one by one, in d
//           order (no fused multiply-add, as the reference's scalar loop)
//   softmax max over all s_p; denom = exp(sink - max) (when the layer has a
//           sink) + the in-order sum of w_p = exp(s_p - max), exp being the
//           host libm's expf reproduced bit for bit (ref_expf)
//   output  o_d = in-order sum over p of w_p * k_p,d (the keys are the values),
//           divided by denom when it is positive, then inverse RoPE on the
//           rope pairs (cos and sin of pos * inv_freq computed on the host with
//           the C library, as the reference does)
//
// Every sum above is a dependent chain in the reference's order, so the work
// is spread over chains, never inside one:
//   mla_scores_kernel  one CTA per tile of positions, all heads: one thread per
//                      (head, position) chain over d; q and the tile's key rows
//                      copied into shared memory (rows padded by 16 B so that a
//                      warp's 16-byte reads of 32 heads hit distinct banks).
//                      Writes the scaled scores [P][heads] and the tile's
//                      per-head max.
//   mla_weights_kernel one CTA per (head, 256 positions): the head's max over
//                      the tile maxima and w = exp(s - max), each weight once.
//   mla_output_kernel  one CTA per (64-feature slice, group of heads): the
//                      group's weight rows into shared memory, one thread per
//                      (head, feature) chain over the positions, the slice's
//                      key rows streamed through a 4-stage cp.async ring of 64
//                      rows, a denominator warp running the in-order weight
//                      sums in the same stages, then division, inverse RoPE
//                      (pair partner by shuffle) and the store.
// Each kernel is launched as a programmatic dependent of the one before; the
// staging copies are cp.async, so all of a CTA's loads are in flight at once.
#include "common.cuh"
#include "kernels.cuh"

namespace wh {

constexpr int kMlaScoreThreads = 512;
constexpr int kMlaSlice = 64;  // features per output CTA (two warps per head)
constexpr int kMlaRingRows = 64;  // key rows per ring stage of the output kernel
constexpr int kMlaStages = 4;
constexpr int kMlaWeightThreads = 256;

__device__ __forceinline__ const float* mla_key_row(const MlaArgs& a, int p) {
  return p < a.window_len ? a.keys + (long long)(a.window_start + p) * a.key_stride
                          : a.compressed + (long long)(p - a.window_len) * a.head_dim;
}

__device__ __forceinline__ void cp_async(void* smem, const void* gmem, bool vec16) {
  const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
  if (vec16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kMlaScoreThreads) mla_scores_kernel(MlaArgs a) {
  extern __shared__ __align__(16) float mla_s[];
  const int tid = threadIdx.x;
  const int H = a.heads, D = a.head_dim, ld = a.smem_ld;
  const int P = a.window_len + a.compressed_count;
  const int p0 = blockIdx.x * a.tile_pos;
  const int np = min(a.tile_pos, P - p0);
  float* q_s = mla_s;                           // [H][ld]
  float* k_s = q_s + (size_t)H * ld;            // [tile_pos][ld]
  float* sc_s = k_s + (size_t)a.tile_pos * ld;  // [tile_pos][H]
  pdl_wait_prior();
  // stage q and the tile's key rows; every copy in flight at once
  const int cw = a.vec4 ? 4 : 1;
  const int per_row = D / cw;
  for (int i = tid; i < H * per_row; i += blockDim.x) {
    const int h = i / per_row, c = (i - h * per_row) * cw;
    cp_async(q_s + h * ld + c, a.q + (long long)h * D + c, a.vec4);
  }
  for (int i = tid; i < np * per_row; i += blockDim.x) {
    const int r = i / per_row, c = (i - r * per_row) * cw;
    cp_async(k_s + r * ld + c, mla_key_row(a, p0 + r) + c, a.vec4);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  // one chain per (head, position): lanes are consecutive heads at one position
  for (int c = tid; c < H * a.tile_pos; c += blockDim.x) {
    const int h = c % H, r = c / H;
    if (r >= np) continue;
    const float* qh = q_s + h * ld;
    const float* kr = k_s + r * ld;
    float s = 0.0f;
    int d = 0;
#pragma unroll 4
    for (; d + 4 <= D; d += 4) {
      const float4 qv = *reinterpret_cast<const float4*>(qh + d);
      const float4 kv = *reinterpret_cast<const float4*>(kr + d);
      s = __fadd_rn(s, __fmul_rn(qv.x, kv.x));
      s = __fadd_rn(s, __fmul_rn(qv.y, kv.y));
      s = __fadd_rn(s, __fmul_rn(qv.z, kv.z));
      s = __fadd_rn(s, __fmul_rn(qv.w, kv.w));
    }
    for (; d < D; ++d) s = __fadd_rn(s, __fmul_rn(qh[d], kr[d]));
    s = __fmul_rn(s, a.scale);
    a.scores[(long long)(p0 + r) * H + h] = s;
    sc_s[r * H + h] = s;
  }
  __syncthreads();
  // the tile's max per head (a NaN score never becomes the max)
  for (int h = tid; h < H; h += blockDim.x) {
    float m = -INFINITY;
    for (int r = 0; r < np; ++r) {
      const float v = sc_s[r * H + h];
      m = v > m ? v : m;
    }
    a.tile_max[(long long)blockIdx.x * H + h] = m;
  }
  pdl_launch_dependents();
}

// w[h][p] = exp(s_p - max_h) for a chunk of positions of one head; the head's
// max over the tile maxima.
__global__ void __launch_bounds__(kMlaWeightThreads) mla_weights_kernel(MlaArgs a) {
  __shared__ float s_red[kMlaWeightThreads / 32];
  const int tid = threadIdx.x, h = blockIdx.y;
  const int H = a.heads;
  const int P = a.window_len + a.compressed_count;
  const int ntiles = (P + a.tile_pos - 1) / a.tile_pos;
  pdl_wait_prior();
  float m = -INFINITY;
  for (int t = tid; t < ntiles; t += blockDim.x) {
    const float v = a.tile_max[(long long)t * H + h];
    m = v > m ? v : m;
  }
  for (int o = 16; o; o >>= 1) {
    const float other = __shfl_xor_sync(0xffffffffu, m, o);
    m = other > m ? other : m;
  }
  if ((tid & 31) == 0) s_red[tid >> 5] = m;
  __syncthreads();
  m = -INFINITY;
  for (int w = 0; w < kMlaWeightThreads / 32; ++w) m = s_red[w] > m ? s_red[w] : m;
  const int p = blockIdx.x * kMlaWeightThreads + tid;
  if (p < P)
    a.weights[(long long)h * P + p] =
        ref_expf(__fsub_rn(a.scores[(long long)p * H + h], m), a.expf);
  if (blockIdx.x == 0 && tid == 0) a.head_max[h] = m;
  pdl_launch_dependents();
}

// Copies rows [r0, r0 + kMlaRingRows) of the CTA's feature slice into a ring slot.
__device__ __forceinline__ void mla_issue_rows(const MlaArgs& a, float* slot, int r0, int P,
                                               int f0, int nf) {
  const int cw = a.vec4 ? 4 : 1;  // floats per copy
  const int per_row = (nf + cw - 1) / cw;
  const int rows = min(kMlaRingRows, P - r0);
  for (int i = threadIdx.x; i < rows * per_row; i += blockDim.x) {
    const int r = i / per_row, c = (i - r * per_row) * cw;
    cp_async(slot + r * kMlaSlice + c, mla_key_row(a, r0 + r) + f0 + c, a.vec4);
  }
}

__global__ void __launch_bounds__(4 * kMlaSlice + 32) mla_output_kernel(MlaArgs a) {
  extern __shared__ __align__(16) float mla_w[];  // [group][P] weights | key ring
  __shared__ float s_den[4];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int D = a.head_dim, G = a.head_group;
  const int P = a.window_len + a.compressed_count;
  const int h0 = blockIdx.y * G;
  const int fw = 2 * G;  // feature warps; warp fw is the denominator warp
  const int f0 = blockIdx.x * kMlaSlice, nf = min(kMlaSlice, D - f0);
  float* ring = mla_w + ((G * P + 3) & ~3);  // [kMlaStages][kMlaRingRows][kMlaSlice]
  const int nst = (P + kMlaRingRows - 1) / kMlaRingRows;
  pdl_wait_prior();
  // the key rows do not depend on the scores: start the ring first
#pragma unroll
  for (int st = 0; st < kMlaStages - 1; ++st) {
    if (st < nst)
      mla_issue_rows(a, ring + st * kMlaRingRows * kMlaSlice, st * kMlaRingRows, P, f0, nf);
    cp_async_commit();
  }
  // the group's weight rows (contiguous [h][P]) behind the ring's first stages
  for (int i = tid; i < G * P; i += blockDim.x)
    cp_async(mla_w + i, a.weights + (long long)h0 * P + i, false);
  cp_async_commit();
  cp_async_wait<0>();
  const int g = warp >> 1;
  const int fl = (warp & 1) * 32 + lane;  // feature within the slice
  const bool feature = warp < fw && fl < nf;
  const bool dwarp = warp == fw && lane < G;
  const float* w = mla_w + (warp < fw ? g : (lane < G ? lane : 0)) * P;
  float acc = 0.0f;  // feature chain, or the denominator warp's weight sum
  for (int st = 0; st < nst; ++st) {
    cp_async_wait<kMlaStages - 2>();
    __syncthreads();  // stage st (and the weights) landed for every thread; slot st - 1 is free
    const int nx = st + kMlaStages - 1;
    if (nx < nst)
      mla_issue_rows(a, ring + (nx % kMlaStages) * kMlaRingRows * kMlaSlice, nx * kMlaRingRows,
                     P, f0, nf);
    cp_async_commit();
    const float* slot = ring + (st % kMlaStages) * kMlaRingRows * kMlaSlice;
    const int r0 = st * kMlaRingRows, rows = min(kMlaRingRows, P - r0);
    if (feature) {
#pragma unroll 8
      for (int r = 0; r < rows; ++r)
        acc = __fadd_rn(acc, __fmul_rn(w[r0 + r], slot[r * kMlaSlice + fl]));
    } else if (dwarp) {
      // the in-order sum of the weights, stage by stage
      for (int r = 0; r < rows; ++r) acc = __fadd_rn(acc, w[r0 + r]);
    }
  }
  cp_async_wait<0>();
  if (dwarp) {
    float denom = 0.0f;
    if (a.sink)
      denom = __fadd_rn(denom, ref_expf(__fsub_rn(a.sink[h0 + lane], a.head_max[h0 + lane]), a.expf));
    s_den[lane] = __fadd_rn(denom, acc);
  }
  __syncthreads();
  if (warp < fw) {
    const int f = f0 + fl;
    const float den = s_den[g];
    if (den > 0.0f) acc = __fdiv_rn(acc, den);
    // inverse RoPE: sin negated; the pair partner is the neighbouring lane
    // (nope_dim and the slice start are even)
    const float partner = __shfl_xor_sync(0xffffffffu, acc, 1);
    if (fl < nf) {
      if (f >= a.nope_dim) {
        const int i = (f - a.nope_dim) >> 1;
        const float c = a.rope_cos[i], sn = -a.rope_sin[i];
        if (((f - a.nope_dim) & 1) == 0)
          acc = __fsub_rn(__fmul_rn(acc, c), __fmul_rn(partner, sn));
        else
          acc = __fadd_rn(__fmul_rn(partner, sn), __fmul_rn(acc, c));
      }
      a.out[(long long)(h0 + g) * D + f] = acc;
    }
  }
  pdl_launch_dependents();
}

// Plans the two launches: tile_pos, smem_ld and head_group.  Returns false
// when the shape does not fit shared memory.
bool mla_plan(MlaArgs& a, size_t* smem_scores, size_t* smem_output) {
  const int H = a.heads, D = a.head_dim;
  const int P = a.window_len + a.compressed_count;
  constexpr size_t kBudget = 220 * 1024;
  if (H > kMlaScoreThreads) return false;
  a.smem_ld = ((D + 3) & ~3) + 4;
  // as many positions as threads allow, fewer when the key rows would not fit
  const size_t q_bytes = sizeof(float) * (size_t)H * a.smem_ld;
  const size_t per_pos = sizeof(float) * (size_t)(a.smem_ld + H);
  const size_t fit = q_bytes < kBudget ? (kBudget - q_bytes) / per_pos : 0;
  a.tile_pos = (int)std::min<size_t>(kMlaScoreThreads / H, fit);
  if (a.tile_pos < 1) return false;
  *smem_scores = q_bytes + per_pos * a.tile_pos;
  const size_t ring = sizeof(float) * kMlaStages * kMlaRingRows * kMlaSlice;
  const size_t wbytes = sizeof(float) * (size_t)P, wbudget = kBudget - ring - 16;
  a.head_group = (H % 4 == 0 && 4 * wbytes <= wbudget) ? 4
               : (H % 2 == 0 && 2 * wbytes <= wbudget) ? 2 : 1;
  *smem_output = sizeof(float) * (((size_t)a.head_group * P + 3) & ~(size_t)3) + ring;
  return *smem_scores <= kBudget && *smem_output <= kBudget;
}

size_t mla_scratch_bytes(int heads, int positions, int tile_pos) {
  const int ntiles = (positions + tile_pos - 1) / tile_pos;
  return sizeof(float) * (2 * (size_t)positions * heads + (size_t)ntiles * heads + heads);
}

cudaError_t launch_mla_attention(const MlaArgs& a, size_t smem_scores, size_t smem_output,
                                 cudaStream_t s) {
  const int P = a.window_len + a.compressed_count;
  cudaError_t e = ensure_smem(mla_scores_kernel, smem_scores);
  if (e != cudaSuccess) return e;
  e = ensure_smem(mla_output_kernel, smem_output);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3((P + a.tile_pos - 1) / a.tile_pos);
  cfg.blockDim = dim3(kMlaScoreThreads);
  cfg.dynamicSmemBytes = smem_scores;
  e = cudaLaunchKernelEx(&cfg, mla_scores_kernel, a);
  if (e != cudaSuccess) return e;
  cfg.gridDim = dim3((P + kMlaWeightThreads - 1) / kMlaWeightThreads, a.heads);
  cfg.blockDim = dim3(kMlaWeightThreads);
  cfg.dynamicSmemBytes = 0;
  e = cudaLaunchKernelEx(&cfg, mla_weights_kernel, a);
  if (e != cudaSuccess) return e;
  cfg.gridDim = dim3((a.head_dim + kMlaSlice - 1) / kMlaSlice, a.heads / a.head_group);
  cfg.blockDim = dim3(2 * 32 * a.head_group + 32);
  cfg.dynamicSmemBytes = smem_output;
  return cudaLaunchKernelEx(&cfg, mla_output_kernel, a);
}

}  // namespace wh
