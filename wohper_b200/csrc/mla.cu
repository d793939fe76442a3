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
//           host libm's expf reproduced bit for bit (libm_expf)
//   output  o_d = in-order sum over p of w_p * k_p,d (the keys are the values),
//           divided by denom when it is positive, then inverse RoPE on the
//           rope pairs (cos and sin of pos * inv_freq computed on the host with
//           the C library, as the reference does)
//
// Every sum above is a dependent chain in the reference's order, so the work
// is spread over chains, never inside one:
//   mla_scores_kernel  one CTA per (16 positions, 32 heads): lane = head, and
//                      each thread runs the chains over d of two positions, so
//                      one 16-byte q read from shared memory serves two chains
//                      and the key reads are warp broadcasts (rows padded by
//                      16 B so that the 32 lanes' q reads hit distinct banks).
//                      Writes the scaled scores [P][heads] and the tile's
//                      per-head max.
//   mla_weights_kernel one CTA per (head, 256 positions): the head's max over
//                      the tile maxima and w = exp(s - max), each weight once.
//   mla_output_kernel  one CTA per (16-feature slice, group of up to 16 heads):
//                      the group's weight rows into shared memory, one thread
//                      per (head, feature) chain over the positions (a warp is
//                      two heads x 16 features, so each key value read from
//                      shared memory serves 16 heads' chains, and the 16 head
//                      groups of 64 heads re-read the keys 4 times from L2,
//                      not 16), the slice's
//                      key rows streamed through a cp.async ring of 12 (8, 4)
//                      stages of 64 rows by the feature warps alone (on a named
//                      barrier), a denominator warp running the in-order weight
//                      sums beside them, then division, inverse RoPE (pair
//                      partner by shuffle) and the store.
// Each kernel is launched as a programmatic dependent of the one before; the
// staging copies are cp.async, so all of a CTA's loads are in flight at once.
#include "common.cuh"
#include "kernels.cuh"
#include <algorithm>

namespace wh {

constexpr int kMlaScoreHeads = 32;  // heads per scores CTA (one per lane)
constexpr int kMlaScoreChains = 2;  // positions per thread
constexpr int kMlaScoreTile = 16;   // positions per scores CTA
constexpr int kMlaScoreThreads = kMlaScoreHeads * kMlaScoreTile / kMlaScoreChains;
constexpr int kMlaSlice = 16;       // features per output CTA (half a warp per head)
constexpr int kMlaMaxGroup = 16;    // heads per output CTA at most
constexpr int kMlaRingRows = 64;    // key rows per ring stage of the output kernel
constexpr size_t kMlaStageBytes = sizeof(float) * kMlaRingRows * kMlaSlice;
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

template <int N>
__global__ void __launch_bounds__(kMlaScoreThreads)
    mla_scores_kernel(const __grid_constant__ MlaBatch<N> b) {
  const MlaArgs& a = b.t[blockIdx.z];
  extern __shared__ __align__(16) float mla_s[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = a.heads, D = a.head_dim, ld = a.smem_ld;
  const int P = a.window_len + a.compressed_count;
  if ((int)blockIdx.x * kMlaScoreTile >= P) return;  // beyond this token's positions
  const int p0 = blockIdx.x * kMlaScoreTile, np = min(kMlaScoreTile, P - p0);
  const int hb = blockIdx.y * kMlaScoreHeads, nh = min(kMlaScoreHeads, H - hb);
  float* q_s = mla_s;                              // [kMlaScoreHeads][ld]
  float* k_s = q_s + (size_t)kMlaScoreHeads * ld;  // [kMlaScoreTile][ld]
  float* sc_s = k_s + (size_t)kMlaScoreTile * ld;  // [kMlaScoreTile][kMlaScoreHeads]
  pdl_wait_prior();
  // the block's q rows and the tile's key rows; every copy in flight at once
  const int cw = a.vec4 ? 4 : 1;
  const int per_row = D / cw;
  for (int i = tid; i < nh * per_row; i += blockDim.x) {
    const int h = i / per_row, c = (i - h * per_row) * cw;
    cp_async(q_s + h * ld + c, a.q + (long long)(hb + h) * D + c, a.vec4);
  }
  for (int i = tid; i < np * per_row; i += blockDim.x) {
    const int r = i / per_row, c = (i - r * per_row) * cw;
    cp_async(k_s + r * ld + c, mla_key_row(a, p0 + r) + c, a.vec4);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  // lane = head, two positions per thread (a row beyond np is computed on
  // whatever the buffer holds and never stored)
  const int r0 = warp * kMlaScoreChains;
  if (lane < nh && r0 < np) {
    const float* qh = q_s + lane * ld;
    const float* kr = k_s + r0 * ld;
    float s0 = 0.0f, s1 = 0.0f;
    int d = 0;
#pragma unroll 4
    for (; d + 4 <= D; d += 4) {
      const float4 qv = *reinterpret_cast<const float4*>(qh + d);
      const float4 k0 = *reinterpret_cast<const float4*>(kr + d);
      const float4 k1 = *reinterpret_cast<const float4*>(kr + ld + d);
      // the two chains interleaved, so that each addition waits on its own
      // chain only
      const float m0x = __fmul_rn(qv.x, k0.x), m1x = __fmul_rn(qv.x, k1.x);
      const float m0y = __fmul_rn(qv.y, k0.y), m1y = __fmul_rn(qv.y, k1.y);
      const float m0z = __fmul_rn(qv.z, k0.z), m1z = __fmul_rn(qv.z, k1.z);
      const float m0w = __fmul_rn(qv.w, k0.w), m1w = __fmul_rn(qv.w, k1.w);
      s0 = __fadd_rn(s0, m0x);
      s1 = __fadd_rn(s1, m1x);
      s0 = __fadd_rn(s0, m0y);
      s1 = __fadd_rn(s1, m1y);
      s0 = __fadd_rn(s0, m0z);
      s1 = __fadd_rn(s1, m1z);
      s0 = __fadd_rn(s0, m0w);
      s1 = __fadd_rn(s1, m1w);
    }
    for (; d < D; ++d) {
      const float qd = qh[d];
      s0 = __fadd_rn(s0, __fmul_rn(qd, kr[d]));
      s1 = __fadd_rn(s1, __fmul_rn(qd, kr[ld + d]));
    }
    const float sv[2] = {__fmul_rn(s0, a.scale), __fmul_rn(s1, a.scale)};
#pragma unroll
    for (int j = 0; j < 2; ++j)
      if (r0 + j < np) {
        a.scores[(long long)(p0 + r0 + j) * H + hb + lane] = sv[j];
        sc_s[(r0 + j) * kMlaScoreHeads + lane] = sv[j];
      }
  }
  __syncthreads();
  // the tile's max per head (a NaN score never becomes the max)
  if (tid < nh) {
    float m = -INFINITY;
    for (int r = 0; r < np; ++r) {
      const float v = sc_s[r * kMlaScoreHeads + tid];
      m = v > m ? v : m;
    }
    a.tile_max[(long long)blockIdx.x * H + hb + tid] = m;
  }
  pdl_launch_dependents();
}

// w[h][p] = exp(s_p - max_h) for a chunk of positions of one head; the head's
// max over the tile maxima.
template <int N>
__global__ void __launch_bounds__(kMlaWeightThreads)
    mla_weights_kernel(const __grid_constant__ MlaBatch<N> b) {
  const MlaArgs& a = b.t[blockIdx.z];
  __shared__ float s_red[kMlaWeightThreads / 32];
  const int tid = threadIdx.x, h = blockIdx.y;
  const int H = a.heads;
  const int P = a.window_len + a.compressed_count;
  if ((int)blockIdx.x * kMlaWeightThreads >= P) return;  // beyond this token's positions
  const int ntiles = (P + kMlaScoreTile - 1) / kMlaScoreTile;
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
    a.weights[(long long)h * P + p] = libm_expf(__fsub_rn(a.scores[(long long)p * H + h], m));
  if (blockIdx.x == 0 && tid == 0) a.head_max[h] = m;
  pdl_launch_dependents();
}

// Copies rows [r0, r0 + kMlaRingRows) of the CTA's feature slice into a ring
// slot; threads [0, nthreads) take part.
__device__ __forceinline__ void mla_issue_rows(const MlaArgs& a, float* slot, int r0, int P,
                                               int f0, int nf, int nthreads) {
  const int rows = min(kMlaRingRows, P - r0);
  if (a.vec4 && nf == kMlaSlice) {
    constexpr int kPerRow = kMlaSlice / 4;
    for (int i = threadIdx.x; i < rows * kPerRow; i += nthreads) {
      const int r = i / kPerRow, c = (i % kPerRow) * 4;
      cp_async(slot + r * kMlaSlice + c, mla_key_row(a, r0 + r) + f0 + c, true);
    }
    return;
  }
  const int cw = a.vec4 ? 4 : 1;  // floats per copy
  const int per_row = (nf + cw - 1) / cw;
  for (int i = threadIdx.x; i < rows * per_row; i += nthreads) {
    const int r = i / per_row, c = (i - r * per_row) * cw;
    cp_async(slot + r * kMlaSlice + c, mla_key_row(a, r0 + r) + f0 + c, a.vec4);
  }
}

template <int kStages, int N>
__global__ void __launch_bounds__(kMlaMaxGroup * kMlaSlice + 32)
    mla_output_kernel(const __grid_constant__ MlaBatch<N> b) {
  const MlaArgs& a = b.t[blockIdx.z];
  extern __shared__ __align__(16) float mla_w[];  // [group][P] weights | key ring
  __shared__ float s_den[kMlaMaxGroup];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int D = a.head_dim, G = a.head_group;
  const int P = a.window_len + a.compressed_count;
  const int h0 = blockIdx.y * G;
  const int fw = (G + 1) / 2;  // feature warps (two heads each); warp fw: denominators
  const int nfeat = fw * 32;  // threads of the feature warps
  const int f0 = blockIdx.x * kMlaSlice, nf = min(kMlaSlice, D - f0);
  // weight rows padded to wld = P rounded up to 4, plus 4: the denominator
  // lanes read distinct banks
  const int wld = ((P + 3) & ~3) + 4;
  float* ring = mla_w + G * wld;  // [kStages][kMlaRingRows][kMlaSlice]
  const int nst = (P + kMlaRingRows - 1) / kMlaRingRows;
  const int g = 2 * warp + (lane >> 4);  // the lane's head within the group
  const int fl = lane & 15;              // the lane's feature within the slice
  const bool feature = warp < fw && g < G && fl < nf;
  const bool dwarp = warp == fw && lane < G;
  pdl_wait_prior();
  // copy group 0, by every thread: the group's weight rows (contiguous [h][P])
  if ((P & 3) == 0) {
    const int q4 = P / 4;
    for (int i = tid; i < G * q4; i += blockDim.x) {
      const int gg = i / q4, c = (i - gg * q4) * 4;
      cp_async(mla_w + gg * wld + c, a.weights + (long long)(h0 + gg) * P + c, true);
    }
  } else {
    for (int i = tid; i < G * P; i += blockDim.x) {
      const int gg = i / P, c = i - gg * P;
      cp_async(mla_w + gg * wld + c, a.weights + (long long)(h0 + gg) * P + c, false);
    }
  }
  cp_async_commit();
  // the feature warps own the key ring; its first stages are groups 1 .. S-1
  if (warp < fw) {
#pragma unroll
    for (int st = 0; st < kStages - 1; ++st) {
      if (st < nst)
        mla_issue_rows(a, ring + st * kMlaRingRows * kMlaSlice, st * kMlaRingRows, P, f0, nf,
                       nfeat);
      cp_async_commit();
    }
    cp_async_wait<kStages - 1>();  // group 0: the weights
  } else {
    cp_async_wait<0>();
  }
  __syncthreads();  // the weights are visible to every thread
  const float* w = mla_w + (warp < fw ? (g < G ? g : 0) : (lane < G ? lane : 0)) * wld;
  float acc = 0.0f;  // a feature chain, or a denominator's weight sum
  if (warp < fw) {
    for (int st = 0; st < nst; ++st) {
      cp_async_wait<kStages - 2>();
      // stage st landed for every feature thread, and slot st - 1 is free
      asm volatile("bar.sync 1, %0;" ::"r"(nfeat) : "memory");
      const int nx = st + kStages - 1;
      if (nx < nst)
        mla_issue_rows(a, ring + (nx % kStages) * kMlaRingRows * kMlaSlice, nx * kMlaRingRows,
                       P, f0, nf, nfeat);
      cp_async_commit();
      const float* slot = ring + (st % kStages) * kMlaRingRows * kMlaSlice;
      const int r0 = st * kMlaRingRows, rows = min(kMlaRingRows, P - r0);
      if (feature) {
        if (rows == kMlaRingRows) {
          // a full stage: the loads of eight rows ahead of their multiplies,
          // the weights four rows per 16-byte read
          const float4* wq = reinterpret_cast<const float4*>(w + r0);
#pragma unroll
          for (int r = 0; r < kMlaRingRows; r += 8) {
            const float4 wa = wq[r / 4], wb = wq[r / 4 + 1];
            float kv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) kv[j] = slot[(r + j) * kMlaSlice + fl];
            const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
            float pr[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) pr[j] = __fmul_rn(wv[j], kv[j]);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, pr[j]);
          }
        } else {
#pragma unroll 8
          for (int r = 0; r < rows; ++r)
            acc = __fadd_rn(acc, __fmul_rn(w[r0 + r], slot[r * kMlaSlice + fl]));
        }
      }
    }
    cp_async_wait<0>();
  } else if (dwarp) {
    // the in-order sum of the weights, beside the ring
#pragma unroll 8
    for (int p = 0; p < P; ++p) acc = __fadd_rn(acc, w[p]);
    float denom = 0.0f;
    if (a.sink)
      denom = __fadd_rn(denom, libm_expf(__fsub_rn(a.sink[h0 + lane], a.head_max[h0 + lane])));
    s_den[lane] = __fadd_rn(denom, acc);
  }
  __syncthreads();
  if (warp < fw) {
    const int f = f0 + fl;
    const float den = s_den[g < G ? g : 0];
    if (den > 0.0f) acc = __fdiv_rn(acc, den);
    // inverse RoPE: sin negated; the pair partner is the neighbouring lane
    // (nope_dim and the slice start are even)
    const float partner = __shfl_xor_sync(0xffffffffu, acc, 1);
    if (g < G && fl < nf) {
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

// Plans the launches: smem_ld, head_group and the output ring's depth (12, 8
// or 4 stages of 64 rows).  Returns false when the shape does not fit shared
// memory.
bool mla_plan(MlaArgs& a, size_t* smem_scores, size_t* smem_output) {
  constexpr size_t kBudget = 220 * 1024;
  const int H = a.heads, D = a.head_dim;
  const int P = a.window_len + a.compressed_count;
  a.smem_ld = ((D + 3) & ~3) + 4;
  *smem_scores = sizeof(float) * ((size_t)(kMlaScoreHeads + kMlaScoreTile) * a.smem_ld +
                                  (size_t)kMlaScoreTile * kMlaScoreHeads);
  if (*smem_scores > kBudget) return false;
  for (int stages : {12, 8, 4})
    for (int g : {16, 8, 4, 2, 1}) {
      if (H % g) continue;
      const size_t bytes =
          sizeof(float) * (size_t)g * ((((size_t)P + 3) & ~(size_t)3) + 4) + stages * kMlaStageBytes;
      if (bytes <= kBudget) {
        a.head_group = g;
        a.stages = stages;
        *smem_output = bytes;
        return true;
      }
    }
  return false;
}

size_t mla_scratch_bytes(int heads, int positions) {
  const int ntiles = (positions + kMlaScoreTile - 1) / kMlaScoreTile;
  return sizeof(float) * (2 * (size_t)positions * heads + (size_t)ntiles * heads + heads);
}

size_t mla_tile_count(int positions) {
  return (size_t)(positions + kMlaScoreTile - 1) / kMlaScoreTile;
}

template <int S, int N>
static cudaError_t launch_mla_output(const cudaLaunchConfig_t& cfg, const MlaBatch<N>& b) {
  cudaError_t e = ensure_smem(mla_output_kernel<S, N>, cfg.dynamicSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaLaunchKernelEx(&cfg, mla_output_kernel<S, N>, b);
}

template <int N>
cudaError_t launch_mla_attention(const MlaBatch<N>& b, int tokens, size_t smem_scores,
                                 size_t smem_output, cudaStream_t s) {
  int P = 0;
  for (int t = 0; t < tokens; ++t) P = std::max(P, b.t[t].window_len + b.t[t].compressed_count);
  const MlaArgs& a = b.t[0];
  cudaError_t e = ensure_smem(mla_scores_kernel<N>, smem_scores);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3((P + kMlaScoreTile - 1) / kMlaScoreTile,
                     (a.heads + kMlaScoreHeads - 1) / kMlaScoreHeads, tokens);
  cfg.blockDim = dim3(kMlaScoreThreads);
  cfg.dynamicSmemBytes = smem_scores;
  e = cudaLaunchKernelEx(&cfg, mla_scores_kernel<N>, b);
  if (e != cudaSuccess) return e;
  cfg.gridDim = dim3((P + kMlaWeightThreads - 1) / kMlaWeightThreads, a.heads, tokens);
  cfg.blockDim = dim3(kMlaWeightThreads);
  cfg.dynamicSmemBytes = 0;
  e = cudaLaunchKernelEx(&cfg, mla_weights_kernel<N>, b);
  if (e != cudaSuccess) return e;
  cfg.gridDim = dim3((a.head_dim + kMlaSlice - 1) / kMlaSlice, a.heads / a.head_group, tokens);
  cfg.blockDim = dim3(32 * ((a.head_group + 1) / 2) + 32);
  cfg.dynamicSmemBytes = smem_output;
  switch (a.stages) {
    case 12: return launch_mla_output<12, N>(cfg, b);
    case 8: return launch_mla_output<8, N>(cfg, b);
    default: return launch_mla_output<4, N>(cfg, b);
  }
}
template cudaError_t launch_mla_attention<1>(const MlaBatch<1>&, int, size_t, size_t,
                                             cudaStream_t);
template cudaError_t launch_mla_attention<kMlaMaxTok>(const MlaBatch<kMlaMaxTok>&, int, size_t,
                                                      size_t, cudaStream_t);

}  // namespace wh
