// moe.cu -- router, FP4 expert matvecs and the routed-expert combine (sm_100a).
//
// Replaces, for one or a few tokens:
//   route_experts_from_dense_block + finalize_route_weights
//     (engine/zc_infer_core/src/compute.rs:2129-2268) and
//     normalize_route_weights_legacy (src/server/generation.rs:3152-3180),
//   deepseek_v4_fp4_expert_forward_scalar (src/deepseek_v4.rs:561-601),
//   fp4_e2m1_ue8m0_matvec_scalar (src/deepseek_v4.rs:464-549),
//   compute_active_experts / compute_active_and_shared_experts
//     (src/compute.rs:1872-2030).
//
// Kernels (one token = one pass; all weights HBM-resident, caller-owned):
//   router_kernel   bf16 gate GEMV in the reference's dot_bf16_row_avx2 order
//                   (two 8-lane FMA chains over 16-column chunks), then the
//                   last CTA of each token does top-k + weights.  It also
//                   writes the token's act-quantised input as f16 grid values
//                   q (x = q * 2^k per 64-block) for the expert kernels.
//   moe_up_kernel   for every (token, slot, 64-row block): w1 and w3 FP4
//                   matvecs streamed by TMA, SwiGLU with the reference's
//                   clamps, and the act quant of the 64 hidden values; writes
//                   f16 grid values + block multipliers.
//   moe_down_kernel for every (token, 16 output rows): the w2 matvecs of all
//                   slots, then the weighted combine in route order plus the
//                   shared expert.
// Arithmetic: each row reproduces fp4_avx2::dot_row bit for bit.  The
// reference multiplies 8*base(nibble) (an integer) by x in fp32 FMA chains;
// here the FMA multiplies base(nibble) (f16) by q = x/2^k (f16, an E4M3 grid
// value) -- both products are exact, so every partial sum is the reference's
// scaled by 2^-(k+3) exactly, and the group sum is rescaled exactly before the
// fma with scale/8.
#include "common.cuh"
#include "kernels.cuh"

namespace wh {

// Quantise value v with block scale `scale` and return the E4M3 grid value q
// (|q| <= 448) -- v/scale clamped and rounded as the reference does.
__device__ __forceinline__ float aq_grid(float v, float scale) {
  float t = __fdiv_rn(v, scale);
  t = t < -448.0f ? -448.0f : t;
  t = t > 448.0f ? 448.0f : t;
  return e4m3_nearest_ties_lower(t);
}

__device__ __forceinline__ float glibc_like_expf(float x) {
  // exp in double then one rounding to float: agrees with glibc expf except
  // when exp(x) lies within ~1e-16 relative of a float rounding boundary.
  return (float)exp((double)x);
}

__device__ __forceinline__ float silu_ref(float x) {  // src/deepseek_v4.rs:551-554
  return __fdiv_rn(x, __fadd_rn(1.0f, glibc_like_expf(-x)));
}

__device__ __forceinline__ float sqrt_softplus_ref(float v) {  // src/compute.rs:2238-2248
  float sp;
  if (v > 20.0f)
    sp = v;
  else if (v < -20.0f)
    sp = glibc_like_expf(v);
  else
    sp = (float)log1p((double)glibc_like_expf(v));
  return __fsqrt_rn(fmaxf(sp, 0.0f));
}

// total_cmp ordering key of f32::total_cmp
__device__ __forceinline__ int32_t total_key(float f) {
  int32_t b = __float_as_int(f);
  return b ^ int32_t(uint32_t(b >> 31) >> 1);
}

// ---------------------------------------------------------------------------
// Router
// ---------------------------------------------------------------------------
constexpr int kRouterWarps = 8;
constexpr int kRouterRowsPerCta = kRouterWarps * 4;

__global__ void __launch_bounds__(kRouterWarps * 32) router_kernel(RouterArgs a, __half* xq,
                                                                  float* xq_mult) {
  const int t = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait_prior();
  const float* x = a.x + (long long)t * a.hidden;

  // (1) act-quantised copy of x for the expert kernels (one warp per 64-block)
  if (xq != nullptr) {
    const int nblk = a.hidden / 64;
    for (int blk = blockIdx.x * kRouterWarps + warp; blk < nblk; blk += gridDim.x * kRouterWarps) {
      float v0 = x[blk * 64 + lane], v1 = x[blk * 64 + 32 + lane];
      float amax = fmaxf(fabsf(v0), fabsf(v1));
      for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      amax = fmaxf(amax, 1.0e-4f);
      float scale = exp2i(ceil_log2f_ref(__fdiv_rn(amax, 448.0f), &c_aq));
      xq[(long long)t * a.hidden + blk * 64 + lane] = __float2half_rn(aq_grid(v0, scale));
      xq[(long long)t * a.hidden + blk * 64 + 32 + lane] = __float2half_rn(aq_grid(v1, scale));
      if (lane == 0) xq_mult[(long long)t * nblk + blk] = __fmul_rn(scale, 8.0f);
    }
  }

  // (2) logits: 8 lanes per expert row, lane p owns chains 2p,2p+1 of acc0
  // (p<4) or of acc1 (p>=4); dot_bf16_row_avx2 (src/compute.rs:6115-6136)
  const int p = lane & 7;
  const int e = blockIdx.x * kRouterRowsPerCta + warp * 4 + (lane >> 3);
  const int ee = e < a.experts ? e : a.experts - 1;  // every lane joins the shuffles
  const int chunks = a.hidden / 16;
  {
    const uint16_t* row = a.gate + (long long)ee * a.hidden;
    const uint32_t* w32 = reinterpret_cast<const uint32_t*>(row) + p;  // 2 bf16 at 16c+2p
    const float2* x2 = reinterpret_cast<const float2*>(x) + p;
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll 8
    for (int c = 0; c < chunks; ++c) {
      uint32_t wv = __ldg(w32 + c * 8);
      float2 wf = make_float2(__uint_as_float(wv << 16), __uint_as_float(wv & 0xffff0000u));
      acc = ffma2(wf, __ldg(x2 + c * 8), acc);
    }
    // v_j = acc0_j + acc1_j (lanes p and p^4)
    float o0 = __shfl_xor_sync(0xffffffffu, acc.x, 4);
    float o1 = __shfl_xor_sync(0xffffffffu, acc.y, 4);
    float s = __fadd_rn(__fadd_rn(acc.x, o0), __fadd_rn(acc.y, o1));  // lane p: v_{2p}+v_{2p+1}
    float s1 = __shfl_xor_sync(0xffffffffu, s, 1);
    float s2 = __fadd_rn(s, s1);  // p=0: (v0+v1)+(v2+v3); p=2: (v4+v5)+(v6+v7)
    float s3 = __shfl_xor_sync(0xffffffffu, s2, 2);
    float hs = __fadd_rn(s2, s3);
    if (p == 0 && e < a.experts) {
      float tail = 0.0f;
      for (int i = chunks * 16; i < a.hidden; ++i)
        tail = __fadd_rn(tail, __fmul_rn(__uint_as_float(uint32_t(row[i]) << 16), x[i]));
      a.logits[(long long)t * a.experts + e] = __fadd_rn(hs, tail);
    }
  }

  // (3) last CTA of this token: top-k + weights
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    uint32_t prev = atomicAdd(&a.counters[t], 1u);
    last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!last) {
    pdl_launch_dependents();
    return;
  }
  __threadfence();
  if (warp == 0) {
    const float* L = a.logits + (long long)t * a.experts;
    constexpr int kMaxPerLane = 32;  // experts <= 1024
    float sc[kMaxPerLane];
    int32_t key[kMaxPerLane];
    for (int i = 0; i < kMaxPerLane; ++i) {
      int ex = i * 32 + lane;
      float v = ex < a.experts ? __ldcg(L + ex) : 0.0f;
      if (a.mode == 1 && ex < a.experts) v = sqrt_softplus_ref(v);
      sc[i] = v;
      float sel = v;
      if (a.mode == 1 && a.bias != nullptr && ex < a.experts) sel = __fadd_rn(v, a.bias[ex]);
      key[i] = ex < a.experts ? total_key(sel) : INT32_MIN;
    }
    int32_t ids[32];
    float score[32];
    int n = 0;
    uint32_t taken = 0;  // bit i: entry i*32+lane already selected
    auto score_of = [&](int ex) {
      float mine = 0.0f;
      for (int i = 0; i < kMaxPerLane; ++i)
        if (i * 32 + lane == ex) mine = sc[i];
      return __shfl_sync(0xffffffffu, mine, ex & 31);
    };
    if (a.mode == 1 && a.hash_ids != nullptr) {
      // tid2eid hash routing (src/compute.rs:2190-2206)
      for (int k = 0; k < a.topk; ++k) {
        const int ex = a.hash_ids[(long long)t * a.topk + k];
        if (ex >= 0 && ex < a.experts) {
          const float got = score_of(ex);
          ids[n] = ex;
          score[n] = got;
          ++n;
        }
      }
    } else {
      // stable descending sort by total_cmp, truncated: max key, lowest id on ties
      const int kk = min(a.topk, a.experts);
      for (int k = 0; k < kk; ++k) {
        int32_t bk = INT32_MIN;
        int bi = 0x7fffffff;
        for (int i = 0; i < kMaxPerLane; ++i) {
          const int ex = i * 32 + lane;
          if (ex < a.experts && !((taken >> i) & 1u) && (key[i] > bk || (key[i] == bk && ex < bi))) {
            bk = key[i];
            bi = ex;
          }
        }
        for (int o = 16; o; o >>= 1) {
          const int32_t ok2 = __shfl_xor_sync(0xffffffffu, bk, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ok2 > bk || (ok2 == bk && oi < bi)) {
            bk = ok2;
            bi = oi;
          }
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        ids[k] = bi;
        score[k] = score_of(bi);
        n = k + 1;
      }
    }
    if (lane == 0) {
      float w[32];
      for (int k = 0; k < n; ++k) w[k] = score[k];
      if (a.mode == 1) {
        float sum = 0.0f;
        for (int k = 0; k < n; ++k) sum = __fadd_rn(sum, w[k]);
        if (n > 0) {
          if (sum > 0.0f && isfinite(sum)) {
            for (int k = 0; k < n; ++k) w[k] = __fmul_rn(__fdiv_rn(w[k], sum), a.route_scale);
          } else {
            float u = __fdiv_rn(a.route_scale, (float)n);
            for (int k = 0; k < n; ++k) w[k] = u;
          }
        }
      } else if (n > 0) {
        bool uniform = false;
        for (int k = 0; k < n; ++k) uniform = uniform || !isfinite(w[k]);
        if (!uniform) {
          float mx = -INFINITY;
          for (int k = 0; k < n; ++k) mx = fmaxf(mx, w[k]);
          float sum = 0.0f;
          for (int k = 0; k < n; ++k) {
            w[k] = glibc_like_expf(__fsub_rn(w[k], mx));
            sum = __fadd_rn(sum, w[k]);
          }
          if (!isfinite(sum) || sum <= 1.1920929e-07f)
            uniform = true;
          else
            for (int k = 0; k < n; ++k) w[k] = __fdiv_rn(w[k], sum);
        }
        if (uniform)
          for (int k = 0; k < n; ++k) w[k] = __fdiv_rn(1.0f, (float)n);
      }
      // combine weights w_k / sum(w) (valid_route_weight_sum, src/compute.rs:2015-2030)
      bool valid = true;
      float sum = 0.0f;
      for (int k = 0; k < n; ++k) {
        if (isfinite(w[k]) && w[k] >= 0.0f)
          sum = __fadd_rn(sum, w[k]);
        else {
          valid = false;
          break;
        }
      }
      if (valid && sum <= 1.1920929e-07f) valid = false;
      for (int k = 0; k < a.topk; ++k) {
        a.ids[(long long)t * a.topk + k] = k < n ? ids[k] : -1;
        a.weights[(long long)t * a.topk + k] = k < n ? w[k] : 0.0f;
        if (a.combine_w)
          a.combine_w[(long long)t * a.topk + k] =
              k < n ? (valid ? __fdiv_rn(w[k], sum) : __fdiv_rn(1.0f, (float)n)) : 0.0f;
      }
      a.counters[t] = 0;  // ready for the next call
    }
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// Shared FP4 group kernel: one lane = one row; 16 packed bytes = one group of
// 32 columns; x given as 16 f16x2 words of E4M3 grid values.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fp4_group_chains(const uint4 wb, const uint4* xq4, float gacc[8]) {
  const uint32_t ws[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) gacc[j] = 0.0f;
  // c-th fma of every lane chain: columns 8c + j  (word c, nibble j)
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 xv = xq4[c];  // f16 pairs for columns 8c..8c+7
    const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t wh2 = fp4x2_to_f16x2_ref(ws[c] >> (8 * i));
      gacc[2 * i] = fma_f16lo(wh2, xs[i], gacc[2 * i]);
      gacc[2 * i + 1] = fma_f16hi(wh2, xs[i], gacc[2 * i + 1]);
    }
  }
}

__device__ __forceinline__ float hsum8(const float a[8]) {
  return __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                   __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
}

// ---------------------------------------------------------------------------
// moe_up: grid (inter/64, slots, tokens); 2 consumer warps (64 rows) + 1 producer
// ---------------------------------------------------------------------------
constexpr int kUpStages = 6;
constexpr int kUpRows = 64;
constexpr int kUpStageBytes = kUpRows * 128;  // 8 KB

size_t moe_up_smem_bytes(int hidden) {
  return 1024 + kUpStages * kUpStageBytes + 2 * kUpStages * 8 + hidden * 2 + (hidden / 64) * 4 +
         64;
}

__global__ void __launch_bounds__(96) moe_up_kernel(MoeArgs a, const __half* __restrict__ xq,
                                                    const float* __restrict__ xq_mult,
                                                    __half* hq, float* hq_mult) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kUpStages * kUpStageBytes);
  uint64_t* empty = full + kUpStages;
  __half* xs = reinterpret_cast<__half*>(empty + kUpStages);
  float* xm = reinterpret_cast<float*>(xs + a.hidden);
  float* red = xm + a.hidden / 64;  // [2] block amax exchange

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.z, slot = blockIdx.y;
  const int row0 = blockIdx.x * kUpRows;
  const int nslots = a.topk + a.has_shared;
  const int nbox = a.hidden / 256;  // 128 B = 256 columns per box
  const int nstage = 2 * nbox;      // w1, w3 interleaved

  if (threadIdx.x == 0) {
    for (int s = 0; s < kUpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2);
    }
    fence_barrier_init();
  }
  __syncthreads();

  int expert;
  if (slot >= a.topk) {
    expert = a.num_experts;  // shared expert slot
  } else {
    pdl_wait_prior();  // ids come from the router
    expert = a.ids[(long long)t * a.topk + slot];
  }
  const bool valid_expert = expert >= 0 && expert < a.num_experts + a.has_shared;

  if (warp == 2) {
    if (lane == 0 && valid_expert) {
      const CUtensorMap* m1 = a.maps + expert * 3 + 0;
      const CUtensorMap* m3 = a.maps + expert * 3 + 1;
      prefetch_tensormap(m1);
      prefetch_tensormap(m3);
      for (int i = 0; i < nstage; ++i) {
        const int s = i % kUpStages;
        if (i >= kUpStages && !mbar_wait(&empty[s], ((i / kUpStages) - 1) & 1, a.status)) break;
        mbar_arrive_expect_tx(&full[s], kUpStageBytes);
        tma_load_2d(stages + s * kUpStageBytes, (i & 1) ? m3 : m1, &full[s], (i >> 1) * 128, row0);
      }
      // leave no copy in flight if the consumers stopped early
      for (int i = max(0, nstage - kUpStages); i < nstage; ++i)
        mbar_wait(&full[i % kUpStages], (i / kUpStages) & 1, a.status);
    }
    return;
  }
  if (slot >= a.topk) pdl_wait_prior();
  if (!valid_expert) {
    if (threadIdx.x == 0) flag(a.status, WH_DEV_BADARG);
    return;
  }
  pdl_launch_dependents();

  // stage the token's quantised input
  {
    const uint4* src = reinterpret_cast<const uint4*>(xq + (long long)t * a.hidden);
    uint4* dst = reinterpret_cast<uint4*>(xs);
    for (int i = threadIdx.x; i < a.hidden / 8; i += 64) dst[i] = src[i];
    for (int i = threadIdx.x; i < a.hidden / 64; i += 64) xm[i] = xq_mult[(long long)t * (a.hidden / 64) + i];
    asm volatile("bar.sync 1, 64;");
  }

  const int r = warp * 32 + lane;  // row within the 64-row block
  const int row = row0 + r;
  const Fp4ExpertDev ed = a.experts[expert];
  const int scols = a.hidden / 32;
  const uint8_t* s1 = ed.w1_scale + (long long)row * scols;
  const uint8_t* s3 = ed.w3_scale + (long long)row * scols;
  float acc1[8], acc3[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc1[j] = acc3[j] = 0.0f;

  bool ok = true;
  for (int i = 0; i < nstage; ++i) {
    const int s = i % kUpStages;
    if (!mbar_wait(&full[s], (i / kUpStages) & 1, a.status)) {
      ok = false;
      break;
    }
    const int box = i >> 1;
    const uint8_t* base = stages + s * kUpStageBytes + r * 128;
    uint4 wb[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) wb[g] = *reinterpret_cast<const uint4*>(base + 16 * (g ^ (r & 7)));
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    const uint2 sb = __ldg(reinterpret_cast<const uint2*>(((i & 1) ? s3 : s1) + box * 8));
    const uint32_t sbw[2] = {sb.x, sb.y};
    float* acc = (i & 1) ? acc3 : acc1;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const int G = box * 8 + g;  // 32-column group index
      float gacc[8];
      fp4_group_chains(wb[g], reinterpret_cast<const uint4*>(xs + G * 32), gacc);
      const float m = xm[G >> 1];
      const float s8 = __fmul_rn(decode_ue8m0((sbw[g >> 2] >> (8 * (g & 3))) & 0xff), 0.125f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = fmaf(__fmul_rn(gacc[j], m), s8, acc[j]);
    }
  }
  if (!ok) return;

  const float gate = __fadd_rn(hsum8(acc1), 0.0f);
  const float up = __fadd_rn(hsum8(acc3), 0.0f);
  if (!isfinite(gate) || !isfinite(up)) flag(a.status, WH_DEV_NONFINITE);
  // SwiGLU with the reference clamps (src/deepseek_v4.rs:556-596)
  const float gated = fminf(gate, 10.0f);
  float upped = up;
  upped = upped < -10.0f ? -10.0f : upped;
  upped = upped > 10.0f ? 10.0f : upped;
  const float h = __fmul_rn(silu_ref(gated), upped);
  // act quant over this 64-row block (src/deepseek_v4.rs:595)
  float amax = fabsf(h);
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) red[warp] = amax;
  asm volatile("bar.sync 1, 64;");
  amax = fmaxf(fmaxf(red[0], red[1]), 1.0e-4f);
  const float scale = exp2i(ceil_log2f_ref(__fdiv_rn(amax, 448.0f), &c_aq));
  const long long hb = ((long long)t * nslots + slot) * a.inter;
  hq[hb + row] = __float2half_rn(aq_grid(h, scale));
  if (r == 0) hq_mult[hb / 64 + row / 64] = __fmul_rn(scale, 8.0f);
  if (a.h) a.h[hb + row] = h;
}

// ---------------------------------------------------------------------------
// moe_down: grid (hidden/16, tokens); 4 consumer warps (8 slots x 16 rows) + producer
// ---------------------------------------------------------------------------
constexpr int kDownStages = 4;
constexpr int kDownRows = 16;
constexpr int kDownSlots = 8;
constexpr int kDownBox = kDownRows * 128;              // 2 KB
constexpr int kDownStageBytes = kDownSlots * kDownBox;  // 16 KB

size_t moe_down_smem_bytes(int inter, int slots) {
  (void)slots;
  return 1024 + kDownStages * kDownStageBytes + 2 * kDownStages * 8 +
         kDownSlots * (inter * 2 + 16) + kDownSlots * (inter / 64) * 4 +
         kDownSlots * kDownRows * 4 + 64;
}

__global__ void __launch_bounds__(160) moe_down_kernel(MoeArgs a, const __half* __restrict__ hq,
                                                       const float* __restrict__ hq_mult) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kDownStages * kDownStageBytes);
  uint64_t* empty = full + kDownStages;
  const int hstride = a.inter * 2 + 16;  // bytes per slot (padded: slots of a warp hit other banks)
  uint8_t* hs = reinterpret_cast<uint8_t*>(empty + kDownStages);
  float* hm = reinterpret_cast<float*>(hs + kDownSlots * hstride);
  float* ys = hm + kDownSlots * (a.inter / 64);
  __shared__ int slot_expert[kDownSlots];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.y;
  const int row0 = blockIdx.x * kDownRows;
  const int nslots = a.topk + a.has_shared;
  const int nbox = a.inter / 256;

  if (threadIdx.x < kDownSlots) {
    int e = -1;
    if (threadIdx.x < a.topk)
      e = a.ids[(long long)t * a.topk + threadIdx.x];  // written by the router, 2 kernels back
    else if (threadIdx.x < nslots)
      e = a.num_experts;
    if (e < -1 || e >= a.num_experts + a.has_shared) e = -1;
    slot_expert[threadIdx.x] = e;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kDownStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 4) {
    if (lane == 0) {
      int nvalid = 0;
      for (int k = 0; k < nslots; ++k) nvalid += slot_expert[k] >= 0;
      for (int i = 0; i < nbox; ++i) {
        const int s = i % kDownStages;
        if (i >= kDownStages && !mbar_wait(&empty[s], ((i / kDownStages) - 1) & 1, a.status)) break;
        mbar_arrive_expect_tx(&full[s], nvalid * kDownBox);
        for (int k = 0; k < nslots; ++k) {
          const int e = slot_expert[k];
          if (e >= 0)
            tma_load_2d(stages + s * kDownStageBytes + k * kDownBox, a.maps + e * 3 + 2, &full[s],
                        i * 128, row0);
        }
      }
      for (int i = max(0, nbox - kDownStages); i < nbox; ++i)
        mbar_wait(&full[i % kDownStages], (i / kDownStages) & 1, a.status);
    }
    return;
  }

  pdl_wait_prior();  // hq from moe_up
  pdl_launch_dependents();
  // stage hq of every slot
  for (int k = 0; k < nslots; ++k) {
    const uint4* src = reinterpret_cast<const uint4*>(hq + ((long long)t * nslots + k) * a.inter);
    uint4* dst = reinterpret_cast<uint4*>(hs + k * hstride);
    for (int i = threadIdx.x; i < a.inter / 8; i += 128) dst[i] = src[i];
    for (int i = threadIdx.x; i < a.inter / 64; i += 128)
      hm[k * (a.inter / 64) + i] = hq_mult[((long long)t * nslots + k) * (a.inter / 64) + i];
  }
  asm volatile("bar.sync 1, 128;");

  const int slot = warp * 2 + (lane >> 4);
  const int r = lane & 15;
  const int row = row0 + r;
  const int e = slot < nslots ? slot_expert[slot] : -1;
  const bool active = e >= 0;
  const int scols = a.inter / 32;
  const uint8_t* srow = active ? a.experts[e].w2_scale + (long long)row * scols : nullptr;
  const __half* hslot = reinterpret_cast<const __half*>(hs + (active ? slot : 0) * hstride);
  const float* hmul = hm + (active ? slot : 0) * (a.inter / 64);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  bool ok = true;
  for (int i = 0; i < nbox; ++i) {
    const int s = i % kDownStages;
    if (!mbar_wait(&full[s], (i / kDownStages) & 1, a.status)) {
      ok = false;
      break;
    }
    uint4 wb[8];
    if (active) {
      const uint8_t* base = stages + s * kDownStageBytes + slot * kDownBox + r * 128;
#pragma unroll
      for (int g = 0; g < 8; ++g) wb[g] = *reinterpret_cast<const uint4*>(base + 16 * (g ^ (r & 7)));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (active) {
      const uint2 sb = __ldg(reinterpret_cast<const uint2*>(srow + i * 8));
      const uint32_t sbw[2] = {sb.x, sb.y};
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const int G = i * 8 + g;
        float gacc[8];
        fp4_group_chains(wb[g], reinterpret_cast<const uint4*>(hslot + G * 32), gacc);
        const float m = hmul[G >> 1];
        const float s8 = __fmul_rn(decode_ue8m0((sbw[g >> 2] >> (8 * (g & 3))) & 0xff), 0.125f);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = fmaf(__fmul_rn(gacc[j], m), s8, acc[j]);
      }
    }
  }
  if (!ok) return;
  if (active) {
    const float yv = __fadd_rn(hsum8(acc), 0.0f);
    if (!isfinite(yv)) flag(a.status, WH_DEV_NONFINITE);
    ys[slot * kDownRows + r] = yv;
    if (a.expert_out)
      a.expert_out[((long long)t * nslots + slot) * a.hidden + row] = yv;
  }
  asm volatile("bar.sync 1, 128;");
  if (a.combine && threadIdx.x < kDownRows) {
    const int rr = threadIdx.x;
    const float* cw = a.combine_w + (long long)t * a.topk;
    float routed = 0.0f;
    if (a.topk == 1) {
      routed = ys[0 * kDownRows + rr];  // one expert: unweighted (src/compute.rs:1960-1966)
    } else {
      for (int k = 0; k < a.topk; ++k)
        routed = __fadd_rn(routed, __fmul_rn(ys[k * kDownRows + rr], cw[k]));
    }
    float out = routed;
    if (a.has_shared) out = a.topk > 0 ? __fadd_rn(ys[a.topk * kDownRows + rr], routed)
                                       : ys[a.topk * kDownRows + rr];
    a.y[(long long)t * a.hidden + row0 + rr] = out;
  }
}

// ---------------------------------------------------------------------------
// Generic exact FP4 matvec (fp4_e2m1_ue8m0_matvec_scalar dispatch), one thread
// per row: AVX2 dot_row order when cols and the group width are even, else
// the per-element order.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fp4_base(uint32_t n) {
  const float lut[16] = {0.0f, 0.125f, 1.0f,  1.5f,  2.0f,  3.0f,  4.0f,  6.0f,
                         0.0f, -0.125f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};
  return lut[n & 15];
}

__global__ void fp4_matvec_generic_kernel(Fp4MatvecArgs a) {
  pdl_wait_prior();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= a.rows) return;
  const int row_bytes = (a.cols + 1) / 2;
  const uint8_t* w = a.packed + (long long)row * row_bytes;
  const uint8_t* s = a.scales + (long long)row * a.scale_cols;
  const int group_cols = a.cols / a.scale_cols;
  float out;
  if (a.cols % 2 == 0 && group_cols % 2 == 0) {
    const int group_bytes = group_cols / 2;
    const int chunks = group_bytes / 16;
    float acc[8];
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    float tail = 0.0f;
    for (int g = 0; g < a.scale_cols; ++g) {
      const float scale = decode_ue8m0(s[g]);
      const uint8_t* bytes = w + (long long)g * group_bytes;
      const float* cols = a.x + (long long)g * group_cols;
      float gacc[8];
      for (int j = 0; j < 8; ++j) gacc[j] = 0.0f;
      for (int c = 0; c < chunks; ++c) {
        for (int q = 0; q < 4; ++q) {  // c0..c3: columns 8q + j of this 32-column chunk
          for (int j = 0; j < 8; ++j) {
            const int col = 8 * q + j;
            const uint32_t byte = bytes[16 * c + col / 2];
            const uint32_t nib = (col & 1) ? (byte >> 4) : (byte & 15);
            gacc[j] = fmaf(8.0f * fp4_base(nib), cols[32 * c + col], gacc[j]);
          }
        }
      }
      const float s8 = __fmul_rn(scale, 0.125f);
      for (int j = 0; j < 8; ++j) acc[j] = fmaf(gacc[j], s8, acc[j]);
      float rem = 0.0f;
      for (int i = chunks * 16; i < group_bytes; ++i) {
        rem = __fadd_rn(rem, __fmul_rn(fp4_base(bytes[i] & 15), cols[2 * i]));
        rem = __fadd_rn(rem, __fmul_rn(fp4_base(bytes[i] >> 4), cols[2 * i + 1]));
      }
      tail = __fadd_rn(tail, __fmul_rn(rem, scale));
    }
    out = __fadd_rn(hsum8(acc), tail);
  } else {
    float acc = 0.0f;
    for (int col = 0; col < a.cols; ++col) {
      const uint32_t byte = w[col / 2];
      const uint32_t nib = (col & 1) ? (byte >> 4) : (byte & 15);
      const float scale = decode_ue8m0(s[col / group_cols]);
      acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(fp4_base(nib), scale), a.x[col]));
    }
    out = acc;
  }
  if (!isfinite(out)) flag(a.status, WH_DEV_NONFINITE);
  a.y[row] = out;
}

cudaError_t launch_fp4_matvec(const Fp4MatvecArgs& a, int num_sms, cudaStream_t stream) {
  (void)num_sms;
  fp4_matvec_generic_kernel<<<(a.rows + 127) / 128, 128, 0, stream>>>(a);
  return cudaGetLastError();
}

// SwiGLU of the generic expert path (gate/up in place into gate)
__global__ void swiglu_kernel(float* gate, const float* up, int n, uint32_t* status) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float g = gate[i], u = up[i];
  if (!isfinite(g) || !isfinite(u)) flag(status, WH_DEV_NONFINITE);
  float gated = fminf(g, 10.0f);
  u = u < -10.0f ? -10.0f : u;
  u = u > 10.0f ? 10.0f : u;
  gate[i] = __fmul_rn(silu_ref(gated), u);
}

cudaError_t launch_swiglu(float* gate, const float* up, int n, uint32_t* status, cudaStream_t s) {
  swiglu_kernel<<<(n + 255) / 256, 256, 0, s>>>(gate, up, n, status);
  return cudaGetLastError();
}

// Host launchers ------------------------------------------------------------
static cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                  cudaLaunchAttribute* attr, bool pdl) {
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

cudaError_t launch_router_ex(const RouterArgs& a, __half* xq, float* xq_mult, cudaStream_t s,
                             bool pdl) {
  cudaLaunchAttribute attr[1];
  dim3 grid((a.experts + kRouterRowsPerCta - 1) / kRouterRowsPerCta, a.tokens);
  cudaLaunchConfig_t cfg = pdl_cfg(grid, dim3(kRouterWarps * 32), 0, s, attr, pdl);
  return cudaLaunchKernelEx(&cfg, router_kernel, a, xq, xq_mult);
}

cudaError_t launch_moe_up_ex(const MoeArgs& a, const __half* xq, const float* xq_mult, __half* hq,
                             float* hq_mult, cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  const size_t smem = moe_up_smem_bytes(a.hidden);
  cudaError_t e = cudaFuncSetAttribute(moe_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.inter / kUpRows, a.topk + a.has_shared, a.tokens);
  cudaLaunchConfig_t cfg = pdl_cfg(grid, dim3(96), smem, s, attr, pdl);
  return cudaLaunchKernelEx(&cfg, moe_up_kernel, a, xq, xq_mult, hq, hq_mult);
}

cudaError_t launch_moe_down_ex(const MoeArgs& a, const __half* hq, const float* hq_mult,
                               cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  const size_t smem = moe_down_smem_bytes(a.inter, a.topk + a.has_shared);
  cudaError_t e = cudaFuncSetAttribute(moe_down_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.hidden / kDownRows, a.tokens);
  cudaLaunchConfig_t cfg = pdl_cfg(grid, dim3(160), smem, s, attr, pdl);
  return cudaLaunchKernelEx(&cfg, moe_down_kernel, a, hq, hq_mult);
}

// Stand-alone act quant to f16 grid values + block multipliers (x = q*mult/8)
__global__ void xq_kernel(const float* x, int n, int tokens, __half* xq, float* xq_mult) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  pdl_wait_prior();
  const int nblk = n / 64;
  if (warp >= nblk * tokens) return;
  const int t = warp / nblk, blk = warp % nblk;
  const float* v = x + (long long)t * n + blk * 64;
  float v0 = v[lane], v1 = v[32 + lane];
  float amax = fmaxf(fabsf(v0), fabsf(v1));
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fmaxf(amax, 1.0e-4f);
  float scale = exp2i(ceil_log2f_ref(__fdiv_rn(amax, 448.0f), &c_aq));
  xq[(long long)t * n + blk * 64 + lane] = __float2half_rn(aq_grid(v0, scale));
  xq[(long long)t * n + blk * 64 + 32 + lane] = __float2half_rn(aq_grid(v1, scale));
  if (lane == 0) xq_mult[(long long)t * nblk + blk] = __fmul_rn(scale, 8.0f);
  pdl_launch_dependents();
}

cudaError_t launch_xq(const float* x, int n, int tokens, __half* xq, float* xq_mult,
                      cudaStream_t s) {
  long long warps = (long long)(n / 64) * tokens;
  xq_kernel<<<(unsigned)((warps * 32 + 127) / 128), 128, 0, s>>>(x, n, tokens, xq, xq_mult);
  return cudaGetLastError();
}

}  // namespace wh
