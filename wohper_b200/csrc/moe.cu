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

__device__ __forceinline__ float silu_ref(float x) {  // src/deepseek_v4.rs:551-554
  return __fdiv_rn(x, __fadd_rn(1.0f, libm_expf(-x)));
}

__device__ __forceinline__ float sqrt_softplus_ref(float v) {  // src/compute.rs:2238-2248
  float sp;
  if (v > 20.0f)
    sp = v;
  else if (v < -20.0f)
    sp = libm_expf(v);
  else
    sp = (float)log1p((double)libm_expf(v));
  return __fsqrt_rn(fmaxf(sp, 0.0f));
}

// total_cmp ordering key of f32::total_cmp
__device__ __forceinline__ int32_t total_key(float f) {
  int32_t b = __float_as_int(f);
  return b ^ int32_t(uint32_t(b >> 31) >> 1);
}

// ---------------------------------------------------------------------------
// Router: a CTA of two warps covers 4 expert rows.  Each half-warp owns one
// row and each of its 16 lanes one of the 16 FMA chains of dot_bf16_row_avx2
// (lanes 0-7: acc0 lane j, columns 16c+j; lanes 8-15: acc1 lane j, columns
// 16c+8+j).  The rows and the token's x are bulk copied into shared memory
// first (rows padded by 32 B so the two rows of a warp hit different banks).
// The CTA that arrives last selects the top-k and computes the route weights.
// ---------------------------------------------------------------------------
constexpr int kRouterRowsPerCta = 4;
constexpr int kRouterWorkers = 64;                  // warps 0-1: logits, act quant, top-k
constexpr int kRouterThreads = kRouterWorkers + 32;  // warp 2: the dry top-k pass

struct RouterSmemPlan {
  int row_stride;  // bytes
  size_t bytes;
};
__host__ __device__ inline RouterSmemPlan router_smem_plan(int hidden) {
  RouterSmemPlan p;
  p.row_stride = hidden * 2 + 32;
  p.bytes = 64 + size_t(kRouterRowsPerCta) * p.row_stride + size_t(hidden) * 4;
  return p;
}

__device__ __forceinline__ float key_to_float(int32_t k) {  // inverse of total_key
  return __int_as_float(k ^ int32_t(uint32_t(k >> 31) >> 1));
}

// Arrival counter with release (this CTA's logits) and acquire (everyone
// else's, for the last arriver) at GPU scope.
__device__ __forceinline__ uint32_t atomic_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(p), "r"(v)
               : "memory");
  return old;
}

// Top-k selection and route weights for token t by one warp, all in
// registers.  PER = logits held per lane (candidate i of lane l is expert
// i*32+l; experts <= 32*PER).  Lane k ends up owning route k.  Each step of the
// selection is a warp-wide arg-max (redux max of the total_cmp key, then redux
// min of the expert id among the lanes holding it), which is the order of the
// reference's stable descending sort.  Ordered sums (the reference adds left
// to right) gather their terms with independent shuffles first.
// ld(sc): loads the logits of experts i*32 + lane (i < PER) into sc, all in
// flight together; entries past the last expert are cleared below.
template <int PER, class Ld>
__device__ __forceinline__ void router_topk_and_weights(const RouterArgs& a, int t, int lane,
                                                        bool dry, Ld ld) {
  constexpr unsigned kFull = 0xffffffffu;
  const bool biased = a.mode == 1 && a.bias != nullptr;
  float sc[PER];
  int32_t key[PER];
  uint32_t avail = 0;  // bit i: candidate i exists and is not selected yet
  ld(sc);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const bool in = i * 32 + lane < a.experts;
    if (!in) sc[i] = 0.0f;
    avail |= uint32_t(in) << i;
  }
  if (a.mode == 1) {
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if ((avail >> i) & 1u) sc[i] = sqrt_softplus_ref(sc[i]);
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int ex = i * 32 + lane;
    key[i] = total_key((biased && ex < a.experts) ? __fadd_rn(sc[i], __ldg(a.bias + ex)) : sc[i]);
  }

  auto score_of = [&](int ex) {  // warp-uniform ex
    float mine = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (i == (ex >> 5)) mine = sc[i];
    return __shfl_sync(kFull, mine, ex & 31);
  };
  int my_id = -1;
  float my_score = 0.0f;
  int n = 0;
  if (a.mode == 1 && a.hash_ids != nullptr) {
    // tid2eid hash routing (src/compute.rs:2190-2206): keep valid ids in order
    for (int k = 0; k < a.topk; ++k) {
      const int ex = a.hash_ids[(long long)t * a.topk + k];
      if (ex >= 0 && ex < a.experts) {
        const float got = score_of(ex);
        if (lane == n) {
          my_id = ex;
          my_score = got;
        }
        ++n;
      }
    }
  } else {
    // stable descending sort by total_cmp, truncated: max key, lowest id on ties
    const int kk = min(a.topk, a.experts);
    for (int k = 0; k < kk; ++k) {
      int32_t bk = INT32_MIN;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        // ids grow with i on a lane: a strict '>' keeps the lowest id on ties
        if (((avail >> i) & 1u) && (bi == 0x7fffffff || key[i] > bk)) {
          bk = key[i];
          bi = i * 32 + lane;
        }
      }
      const int32_t m = __reduce_max_sync(kFull, bk);
      const int win = int(__reduce_min_sync(
          kFull, (bi != 0x7fffffff && bk == m) ? uint32_t(bi) : 0xffffffffu));
      if ((win & 31) == lane) avail &= ~(1u << (win >> 5));
      const float got = score_of(win);
      if (lane == k) {
        my_id = win;
        my_score = got;
      }
      n = k + 1;
    }
  }
  const bool mine = lane < n;
  auto ordered_sum = [&](float v) {  // v_0 + v_1 + ... + v_{n-1}, left to right
    float g[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) g[k] = __shfl_sync(kFull, v, k);
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (k < n) acc = __fadd_rn(acc, g[k]);
    for (int k = 8; k < n; ++k) acc = __fadd_rn(acc, __shfl_sync(kFull, v, k));
    return acc;  // uniform
  };
  float w = my_score;
  if (a.mode == 1) {
    // finalize_route_weights (src/compute.rs:2253-2268)
    const float sum = ordered_sum(mine ? w : 0.0f);
    if (n > 0) {
      if (sum > 0.0f && isfinite(sum))
        w = __fmul_rn(__fdiv_rn(w, sum), a.route_scale);
      else
        w = __fdiv_rn(a.route_scale, (float)n);
    }
  } else if (n > 0) {
    // normalize_route_weights_legacy (src/server/generation.rs:3152-3180)
    bool uniform = __any_sync(kFull, mine && !isfinite(w));
    if (!uniform) {
      // every selected w is finite here, where total_cmp order is numeric
      // order (a -0/+0 tie gives the same exp(w - max) either way)
      const float mx = key_to_float(__reduce_max_sync(kFull, mine ? total_key(w) : INT32_MIN));
      const float e = mine ? libm_expf(__fsub_rn(w, mx)) : 0.0f;
      const float sum = ordered_sum(e);
      if (!isfinite(sum) || sum <= 1.1920929e-07f)
        uniform = true;
      else
        w = __fdiv_rn(e, sum);
    }
    if (uniform) w = __fdiv_rn(1.0f, (float)n);
  }
  // combine weights w_k / sum(w) (valid_route_weight_sum, src/compute.rs:2015-2030)
  const bool bad = __any_sync(kFull, mine && !(isfinite(w) && w >= 0.0f));
  const float wsum = ordered_sum(mine ? w : 0.0f);
  const bool valid = !bad && wsum > 1.1920929e-07f;
  if (dry) return;
  if (lane < a.topk) {
    const long long o = (long long)t * a.topk + lane;
    a.ids[o] = mine ? my_id : -1;
    a.weights[o] = mine ? w : 0.0f;
    if (a.combine_w)
      a.combine_w[o] = mine ? (valid ? __fdiv_rn(w, wsum) : __fdiv_rn(1.0f, (float)n)) : 0.0f;
  }
  if (lane == 0) a.counters[t] = 0;  // ready for the next call
}

// Candidate logits of token t from global memory: every load is issued before
// the first is used (indices clamped to the last expert; the top-k clears the
// entries past it).
template <int PER>
__device__ __forceinline__ void router_load_global(const RouterArgs& a, int t, int lane,
                                                   float (&sc)[PER]) {
  const float* L = a.logits + (long long)t * a.experts;
#pragma unroll
  for (int i = 0; i < PER; ++i) sc[i] = __ldcg(L + min(i * 32 + lane, a.experts - 1));
}

// The top-k runs once per token, in one warp of the last CTA, usually on code
// that is in no cache (the weights streamed since the last call evict it).
// A third warp of every CTA runs it once "dry" (no stores; logits of an
// earlier call or of this one, whichever are there) while the other two
// compute the logits, so that the last CTA's real pass fetches its
// instructions on chip (not inlined: both passes run the same code).
__device__ __noinline__ void router_topk_any(const RouterArgs& a, int t, int lane, bool dry) {
  auto ld = [&](auto& sc) { router_load_global(a, t, lane, sc); };
  if (a.experts <= 32) router_topk_and_weights<1>(a, t, lane, dry, ld);
  else if (a.experts <= 64) router_topk_and_weights<2>(a, t, lane, dry, ld);
  else if (a.experts <= 128) router_topk_and_weights<4>(a, t, lane, dry, ld);
  else if (a.experts <= 256) router_topk_and_weights<8>(a, t, lane, dry, ld);
  else if (a.experts <= 512) router_topk_and_weights<16>(a, t, lane, dry, ld);
  else router_topk_and_weights<32>(a, t, lane, dry, ld);
}

// kSmem: rows and x staged in shared memory (hidden % 8 == 0, 16-byte aligned
// rows); otherwise read straight from global memory.
template <bool kSmem>
__global__ void __launch_bounds__(kRouterThreads) router_kernel(RouterArgs a, __half* xq,
                                                                float* xq_mult) {
  extern __shared__ __align__(16) uint8_t rsmem[];
  const int t = blockIdx.y;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int e0 = blockIdx.x * kRouterRowsPerCta;
  const int nrows = min(kRouterRowsPerCta, a.experts - e0);
  const RouterSmemPlan plan = router_smem_plan(a.hidden);
  uint64_t* bar = reinterpret_cast<uint64_t*>(rsmem);
  uint32_t* last_s = reinterpret_cast<uint32_t*>(rsmem + 8);
  uint8_t* rows_s = rsmem + 64;
  float* x_s = reinterpret_cast<float*>(rows_s + kRouterRowsPerCta * plan.row_stride);

  if (kSmem && tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (kSmem && tid == 0) {
    // gate rows do not depend on earlier kernels: start them before the PDL wait
    mbar_arrive_expect_tx(bar, nrows * a.hidden * 2 + a.hidden * 4);
    for (int r = 0; r < nrows; ++r)
      bulk_load(rows_s + r * plan.row_stride, a.gate + (long long)(e0 + r) * a.hidden,
                a.hidden * 2, bar);
  }
  if (warp == 2) {
    router_topk_any(a, t, lane, true);
    return;  // the barriers below count warps 0-1 only
  }
  pdl_wait_prior();
  const float* x = a.x + (long long)t * a.hidden;
  if (kSmem && tid == 0) bulk_load(x_s, x, a.hidden * 4, bar);

  // (1) act-quantised copy of x for the expert kernels: 64-blocks over the warps
  if (xq != nullptr) {
    const int nblk = a.hidden / 64;
    for (int blk = blockIdx.x * 2 + warp; blk < nblk; blk += gridDim.x * 2) {
      const float v0 = x[blk * 64 + lane], v1 = x[blk * 64 + 32 + lane];
      float amax = fmaxf(fabsf(v0), fabsf(v1));
      for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      amax = fmaxf(amax, 1.0e-4f);
      const float scale = exp2i(ceil_log2f_ref(__fdiv_rn(amax, 448.0f), &c_aq));
      xq[(long long)t * a.hidden + blk * 64 + lane] = __float2half_rn(aq_grid(v0, scale));
      xq[(long long)t * a.hidden + blk * 64 + 32 + lane] = __float2half_rn(aq_grid(v1, scale));
      if (lane == 0) xq_mult[(long long)t * nblk + blk] = __fmul_rn(scale, 8.0f);
    }
  }

  // (2) logits -- dot_bf16_row_avx2 (src/compute.rs:6115-6136)
  const int p = lane & 15;
  const int r = warp * 2 + (lane >> 4);
  const int rr = r < nrows ? r : nrows - 1;  // every lane joins the shuffles
  const int chunks = a.hidden / 16;
  const uint16_t* grow = a.gate + (long long)(e0 + rr) * a.hidden;
  const uint16_t* wv;
  const float* xv;
  if (kSmem) {
    mbar_wait(bar, 0, a.status);  // a timeout is flagged; the CTA still finishes
    wv = reinterpret_cast<const uint16_t*>(rows_s + rr * plan.row_stride) + p;
    xv = x_s + p;
  } else {
    wv = grow + p;
    xv = x + p;
  }
  float acc = 0.0f;
#pragma unroll 16
  for (int c = 0; c < chunks; ++c)
    acc = __fmaf_rn(__uint_as_float(uint32_t(wv[c * 16]) << 16), xv[c * 16], acc);
  // v_j = acc0_j + acc1_j, then the pairwise horizontal sum of v_0..v_7
  const float v = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 8));
  const float h1 = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
  const float h2 = __fadd_rn(h1, __shfl_xor_sync(0xffffffffu, h1, 2));
  const float h3 = __fadd_rn(h2, __shfl_xor_sync(0xffffffffu, h2, 4));
  if (p == 0 && r < nrows) {
    float tail = 0.0f;
    for (int i = chunks * 16; i < a.hidden; ++i)
      tail = __fadd_rn(tail, __fmul_rn(__uint_as_float(uint32_t(grow[i]) << 16), x[i]));
    a.logits[(long long)t * a.experts + e0 + r] = __fadd_rn(h3, tail);
  }
  bar_and(1, kRouterWorkers, 1);
  if (tid == 0) *last_s = atomic_add_acq_rel(&a.counters[t], 1u) == gridDim.x - 1;
  bar_and(1, kRouterWorkers, 1);
  pdl_launch_dependents();
  // (3) the last CTA of this token does top-k + weights
  if (!*last_s || warp != 0) return;
  router_topk_any(a, t, lane, false);
}

// ---------------------------------------------------------------------------
// Shared FP4 group kernel: one lane = one row; 16 packed bytes = one group of
// 32 columns; x given as 4 uint4 (16 f16x2 words) of E4M3 grid values.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fp4_group_chains(const uint4 wb, const uint4 (&xv)[4],
                                                 float gacc[8]) {
  const uint32_t ws[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) gacc[j] = 0.0f;
  // c-th fma of every lane chain: columns 8c + j  (word c, nibble j)
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t xs[4] = {xv[c].x, xv[c].y, xv[c].z, xv[c].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t wh2 = fp4x2_to_f16x2_ref(ws[c] >> (8 * i));
      gacc[2 * i] = fma_f16lo(wh2, xs[i], gacc[2 * i]);
      gacc[2 * i + 1] = fma_f16hi(wh2, xs[i], gacc[2 * i + 1]);
    }
  }
}

__device__ __forceinline__ void load_x4(const __half* base, int G, uint4 (&xv)[4]) {
  const uint4* p = reinterpret_cast<const uint4*>(base + G * 32);
#pragma unroll
  for (int c = 0; c < 4; ++c) xv[c] = p[c];
}

// 8 groups (one 128-byte box column) of one row: wb[g] = the row's 16 bytes of
// group g, xs = the input's f16 grid values, xm = the 64-block multipliers.
__device__ __forceinline__ void fp4_box_accumulate(const uint4 (&wb)[8], const __half* xs,
                                                   const float* xm, int box, uint2 sb,
                                                   float acc[8]) {
  const uint32_t sbw[2] = {sb.x, sb.y};
  uint4 xv[2][4];
  load_x4(xs, box * 8, xv[0]);
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const int G = box * 8 + g;
    if (g + 1 < 8) load_x4(xs, G + 1, xv[(g + 1) & 1]);
    float gacc[8];
    fp4_group_chains(wb[g], xv[g & 1], gacc);
    const float m = xm[G >> 1];
    const float s8 = __fmul_rn(decode_ue8m0((sbw[g >> 2] >> (8 * (g & 3))) & 0xff), 0.125f);
    const float2 mm = make_float2(m, m), ss = make_float2(s8, s8);
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      const float2 r = ffma2(fmul2(make_float2(gacc[j], gacc[j + 1]), mm), ss,
                             make_float2(acc[j], acc[j + 1]));
      acc[j] = r.x;
      acc[j + 1] = r.y;
    }
  }
}

// The same over half of a row's chains: lane half hf = 0 runs chains 0-3 (bytes
// 0 and 1 of every word, columns 8c + 0..3), hf = 1 chains 4-7 (bytes 2 and 3,
// columns 8c + 4..7); acc[j] is chain 4 hf + j.  Each chain sees the same FMAs
// in the same order as in fp4_box_accumulate.
__device__ __forceinline__ void fp4_box_accumulate_half(const uint4 (&wb)[8], const __half* xs,
                                                        const float* xm, int box, uint2 sb,
                                                        int hf, float acc[4]) {
  const uint32_t sbw[2] = {sb.x, sb.y};
  const int sh = 16 * hf;
  // x pair words of columns 8c + 4hf + {0,1} and {2,3}: uint2 index 8G + 2c + hf
  const uint2* xp = reinterpret_cast<const uint2*>(xs) + hf;
  uint2 xv[2][4];
#pragma unroll
  for (int c = 0; c < 4; ++c) xv[0][c] = xp[8 * (box * 8) + 2 * c];
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const int G = box * 8 + g;
    if (g + 1 < 8) {
#pragma unroll
      for (int c = 0; c < 4; ++c) xv[(g + 1) & 1][c] = xp[8 * (G + 1) + 2 * c];
    }
    const uint32_t ws[4] = {wb[g].x, wb[g].y, wb[g].z, wb[g].w};
    float gacc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t hw = ws[c] >> sh;
      const uint32_t w0 = fp4x2_to_f16x2_ref(hw);
      const uint32_t w1 = fp4x2_to_f16x2_ref(hw >> 8);
      const uint2 xc = xv[g & 1][c];
      gacc[0] = fma_f16lo(w0, xc.x, gacc[0]);
      gacc[1] = fma_f16hi(w0, xc.x, gacc[1]);
      gacc[2] = fma_f16lo(w1, xc.y, gacc[2]);
      gacc[3] = fma_f16hi(w1, xc.y, gacc[3]);
    }
    const float m = xm[G >> 1];
    const float s8 = __fmul_rn(decode_ue8m0((sbw[g >> 2] >> (8 * (g & 3))) & 0xff), 0.125f);
    const float2 mm = make_float2(m, m), ss = make_float2(s8, s8);
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      const float2 r = ffma2(fmul2(make_float2(gacc[j], gacc[j + 1]), mm), ss,
                             make_float2(acc[j], acc[j + 1]));
      acc[j] = r.x;
      acc[j + 1] = r.y;
    }
  }
}

// hsum8 of a row whose chains are split over lanes 2r (chains 0-3) and 2r+1
// (chains 4-7): the same association, ((a0+a1)+(a2+a3)) + ((a4+a5)+(a6+a7)).
__device__ __forceinline__ float hsum8_pair(const float a[4]) {
  const float q = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
  const float o = __shfl_xor_sync(0xffffffffu, q, 1);
  return __fadd_rn(q, o);
}

__device__ __forceinline__ float hsum8(const float a[8]) {
  return __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                   __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
}

// ---------------------------------------------------------------------------
// moe_up: grid (inter/32, slots, tokens).  Warps 0-1 compute the 32 w1 (gate)
// rows, warps 2-3 the same w3 (up) rows, two lanes per row (each lane four of
// the row's eight FMA chains); warp 4 streams both with TMA.  Four consumer
// warps per CTA spread the FMA work evenly over an SM's four schedulers.  The
// SwiGLU hidden of the 32 rows goes to global memory; the second CTA of each
// 64-row act-quant block to finish quantises the block (atomic arrival
// counter, no waiting).
// ---------------------------------------------------------------------------
constexpr int kUpConsumers = 4;
constexpr int kUpThreads = (kUpConsumers + 1) * 32;
constexpr int kUpStages = 4;
constexpr int kUpRows = kMoeUpRows;
constexpr int kUpBox = kUpRows * 128;         // 4 KB
constexpr int kUpStageBytes = 2 * kUpBox;     // w1 box + w3 box

size_t moe_up_smem_bytes(int hidden) {
  return 1024 + kUpStages * kUpStageBytes + 2 * kUpStages * 8 + 16 + hidden * 2 +
         (hidden / 64) * 4 + 128 + 2 * kUpRows * (hidden / 32) + 64;
}

__global__ void __launch_bounds__(kUpThreads) moe_up_kernel(MoeArgs a, const __half* __restrict__ xq,
                                                    const float* __restrict__ xq_mult,
                                                    __half* hq, float* hq_mult) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kUpStages * kUpStageBytes);
  uint64_t* empty = full + kUpStages;
  uint64_t* xbar = empty + kUpStages;
  __half* xs = reinterpret_cast<__half*>(xbar + 2);
  float* xm = reinterpret_cast<float*>(xs + a.hidden);
  float* gsh = xm + a.hidden / 64;  // [32] gate values handed to the up warp
  uint8_t* ssm = reinterpret_cast<uint8_t*>(gsh + 32);  // [2][32 rows][hidden/32] scales

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.z, slot = blockIdx.y;
  const int row0 = blockIdx.x * kUpRows;
  const int nslots = a.topk + a.has_shared;
  const int nbox = a.hidden / 256;  // 128 B = 256 columns per box

  if (threadIdx.x == 0) {
    for (int s = 0; s < kUpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kUpConsumers);
    }
    mbar_init(xbar, 1);
    fence_barrier_init();
  }
  __syncthreads();

  int expert;
  if (slot >= a.topk) {
    expert = a.num_experts;  // shared expert slot: no dependency on the router
  } else {
    pdl_wait_prior();  // ids come from the router
    expert = a.ids[(long long)t * a.topk + slot];
  }
  const bool valid_expert = expert >= 0 && expert < a.num_experts + a.has_shared;

  if (warp == kUpConsumers) {
    if (lane == 0 && valid_expert) {
      const CUtensorMap* m1 = a.maps + expert * 3 + 0;
      const CUtensorMap* m3 = a.maps + expert * 3 + 1;
      prefetch_tensormap(m1);
      prefetch_tensormap(m3);
      auto issue = [&](int i) {
        const int s = i % kUpStages;
        mbar_arrive_expect_tx(&full[s], kUpStageBytes);
        tma_load_2d(stages + s * kUpStageBytes, m1, &full[s], i * 128, row0);
        tma_load_2d(stages + s * kUpStageBytes + kUpBox, m3, &full[s], i * 128, row0);
      };
      const int scols = a.hidden / 32;
      const Fp4ExpertDev& ex = a.experts[expert];
      // x and its multipliers (produced by the router) and this CTA's scale
      // rows ([32 rows][hidden/32] per matrix, contiguous) on one barrier
      mbar_arrive_expect_tx(xbar, a.hidden * 2 + (a.hidden / 64) * 4 + 2 * kUpRows * scols);
      auto load_scales = [&]() {
        bulk_load(ssm, ex.w1_scale + (long long)row0 * scols, kUpRows * scols, xbar);
        bulk_load(ssm + kUpRows * scols, ex.w3_scale + (long long)row0 * scols, kUpRows * scols,
                  xbar);
      };
      auto load_x = [&]() {
        bulk_load(xs, xq + (long long)t * a.hidden, a.hidden * 2, xbar);
        bulk_load(xm, xq_mult + (long long)t * (a.hidden / 64), (a.hidden / 64) * 4, xbar);
      };
      int i = 0;
      if (slot >= a.topk) {
        // shared expert: weights and scales do not depend on the router, so
        // they stream while it runs; x once it has completed
        load_scales();
        for (; i < nbox && i < kUpStages; ++i) issue(i);  // first pass needs no free slot
        pdl_wait_prior();
        load_x();
      } else {
        // routed (the router has completed): the small inputs go ahead of the
        // ring so that they do not queue behind 32 KB of weights
        load_x();
        load_scales();
        for (; i < nbox && i < kUpStages; ++i) issue(i);
      }
      for (; i < nbox; ++i) {
        if (!mbar_wait(&empty[i % kUpStages], ((i / kUpStages) - 1) & 1, a.status)) break;
        issue(i);
      }
      // leave no copy in flight if the consumers stopped early
      for (int k = max(0, i - kUpStages); k < i; ++k)
        if (!mbar_drain(&full[k % kUpStages], (k / kUpStages) & 1, a.status)) break;
      mbar_drain(xbar, 0, a.status);
    }
    return;
  }
  if (!valid_expert) {
    if (threadIdx.x == 0) flag(a.status, WH_DEV_BADARG);
    return;
  }
  // the next kernel reads the router's ids before its own wait: only release it
  // once the router has completed (shared-slot CTAs have not waited yet)
  if (slot >= a.topk) pdl_wait_prior();
  pdl_launch_dependents();
  // a failed (timed-out) wait skips the work but still reaches the named
  // barrier below, so the partner warp is never stranded
  bool ok = __all_sync(0xffffffffu, mbar_wait(xbar, 0, a.status));

  const int mat = warp >> 1;                      // 0: w1, 1: w3
  const int rl = (warp & 1) * 16 + (lane >> 1);   // row within the CTA's 32
  const int hf = lane & 1;                        // chain half
  const int row = row0 + rl;
  const int scols = a.hidden / 32;
  const uint8_t* srow = ssm + (mat * kUpRows + rl) * scols;
  float acc[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] = 0.0f;

  for (int i = 0; ok && i < nbox; ++i) {
    const int s = i % kUpStages;
    const uint2 sb = *reinterpret_cast<const uint2*>(srow + i * 8);
    // warp-uniform: the lane pairs exchange partial sums with shuffles
    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (i / kUpStages) & 1, a.status))) {
      ok = false;
      break;
    }
    const uint8_t* base = stages + s * kUpStageBytes + mat * kUpBox + rl * 128;
    uint4 wb[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) wb[g] = *reinterpret_cast<const uint4*>(base + 16 * (g ^ (rl & 7)));
    fp4_box_accumulate_half(wb, xs, xm, i, sb, hf, acc);
    // release the slot only after every lane has consumed its loads: an
    // arrive issued while shared-memory loads are still outstanding lets the
    // next TMA overwrite the slot under them (seen with several CTAs per SM)
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  const float v = __fadd_rn(hsum8_pair(acc), 0.0f);
  if (!isfinite(v)) flag(a.status, WH_DEV_NONFINITE);
  if (mat == 0 && hf == 0) gsh[rl] = v;
  const int ok_all = bar_and(1, kUpConsumers * 32, ok);
  if (mat == 0 || !ok_all) return;

  // SwiGLU with the reference clamps (src/deepseek_v4.rs:556-596)
  const float gated = fminf(gsh[rl], 10.0f);
  float upped = v;
  upped = upped < -10.0f ? -10.0f : upped;
  upped = upped > 10.0f ? 10.0f : upped;
  const float hv = __fmul_rn(silu_ref(gated), upped);
  const long long hb = ((long long)t * nslots + slot) * a.inter;
  if (hf == 0) a.h[hb + row] = hv;
  // act quant over the 64-row block (src/deepseek_v4.rs:595): the later of the
  // two 32-row CTAs quantises the whole block.  Every thread fences its store
  // before warp 2's lane 0 publishes the arrival.
  __threadfence();
  bar_and(2, 64, 1);
  if (warp != 2) return;
  uint32_t prev = 0;
  const long long blk = hb / 64 + row0 / 64;
  if (lane == 0) prev = atomicAdd(&a.blk_counters[blk], 1u);
  prev = __shfl_sync(0xffffffffu, prev, 0);
  if (prev == 0) return;
  __threadfence();
  const int b0 = (row0 / 64) * 64;
  const float h0 = __ldcg(a.h + hb + b0 + lane), h1 = __ldcg(a.h + hb + b0 + 32 + lane);
  float amax = fmaxf(fabsf(h0), fabsf(h1));
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fmaxf(amax, 1.0e-4f);
  const float scale = exp2i(ceil_log2f_ref(__fdiv_rn(amax, 448.0f), &c_aq));
  hq[hb + b0 + lane] = __float2half_rn(aq_grid(h0, scale));
  hq[hb + b0 + 32 + lane] = __float2half_rn(aq_grid(h1, scale));
  if (lane == 0) {
    hq_mult[blk] = __fmul_rn(scale, 8.0f);
    a.blk_counters[blk] = 0;  // ready for the next call
  }
}

// ---------------------------------------------------------------------------
// moe_down: grid (hidden/16, tokens); 8 consumer warps (warp k = slot k, 16 rows,
// two lanes per row) + a TMA producer warp
// ---------------------------------------------------------------------------
constexpr int kDownConsumers = 8;
constexpr int kDownThreads = (kDownConsumers + 1) * 32;
constexpr int kDownStages = 4;
constexpr int kDownRows = kMoeDownRows;
constexpr int kDownSlots = 8;
constexpr int kDownBox = kDownRows * 128;              // 2 KB
constexpr int kDownStageBytes = kDownSlots * kDownBox;  // 16 KB

size_t moe_down_smem_bytes(int inter, int slots) {
  (void)slots;
  return 1024 + kDownStages * kDownStageBytes + 2 * kDownStages * 8 + 16 +
         kDownSlots * (inter * 2 + 16) + kDownSlots * (inter / 64) * 4 +
         kDownSlots * kDownRows * 4 + kDownSlots * kDownRows * (inter / 32) + 64;
}

__global__ void __launch_bounds__(kDownThreads) moe_down_kernel(MoeArgs a, const __half* __restrict__ hq,
                                                       const float* __restrict__ hq_mult) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kDownStages * kDownStageBytes);
  uint64_t* empty = full + kDownStages;
  uint64_t* xbar = empty + kDownStages;
  const int hstride = a.inter * 2 + 16;  // bytes per slot (padded: slots of a warp hit other banks)
  uint8_t* hs = reinterpret_cast<uint8_t*>(xbar + 2);
  float* hm = reinterpret_cast<float*>(hs + kDownSlots * hstride);
  float* ys = hm + kDownSlots * (a.inter / 64);
  uint8_t* ssm = reinterpret_cast<uint8_t*>(ys + kDownSlots * kDownRows);  // [slot][16][inter/32]
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
  uint64_t* sbar = xbar + 1;  // the slots' w2 scale rows
  if (threadIdx.x == 0) {
    for (int s = 0; s < kDownStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDownConsumers);
    }
    mbar_init(xbar, 1);
    mbar_init(sbar, 1);
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kDownConsumers) {
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
        if (!mbar_drain(&full[i % kDownStages], (i / kDownStages) & 1, a.status)) break;
    }
    return;
  }

  // the w2 scale rows depend only on the router's ids: stage them before the
  // wait for moe_up (this CTA's 16 rows of each slot's w2 scales are contiguous)
  const int scols = a.inter / 32;
  if (threadIdx.x == 0) {
    int nvalid = 0;
    for (int k = 0; k < nslots; ++k) nvalid += slot_expert[k] >= 0;
    mbar_arrive_expect_tx(sbar, nvalid * kDownRows * scols);
    for (int k = 0; k < nslots; ++k) {
      const int e = slot_expert[k];
      if (e >= 0)
        bulk_load(ssm + k * kDownRows * scols, a.experts[e].w2_scale + (long long)row0 * scols,
                  kDownRows * scols, sbar);
    }
  }
  pdl_wait_prior();  // hq from moe_up
  pdl_launch_dependents();
  // stage hq of every slot (bulk copies, one barrier)
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(xbar, nslots * (a.inter * 2 + (a.inter / 64) * 4));
    for (int k = 0; k < nslots; ++k) {
      bulk_load(hs + k * hstride, hq + ((long long)t * nslots + k) * a.inter, a.inter * 2, xbar);
      bulk_load(hm + k * (a.inter / 64), hq_mult + ((long long)t * nslots + k) * (a.inter / 64),
                (a.inter / 64) * 4, xbar);
    }
  }
  bool ok = __all_sync(0xffffffffu, mbar_wait(sbar, 0, a.status) && mbar_wait(xbar, 0, a.status));

  const int slot = warp;
  const int r = lane >> 1;
  const int hf = lane & 1;
  const int row = row0 + r;
  const int e = slot < nslots ? slot_expert[slot] : -1;
  const bool active = e >= 0;
  const uint8_t* srow = ssm + ((active ? slot : 0) * kDownRows + r) * scols;
  const __half* hslot = reinterpret_cast<const __half*>(hs + (active ? slot : 0) * hstride);
  const float* hmul = hm + (active ? slot : 0) * (a.inter / 64);
  float acc[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] = 0.0f;
  for (int i = 0; ok && i < nbox; ++i) {
    const int s = i % kDownStages;
    uint2 sb = make_uint2(0, 0);
    if (active) sb = *reinterpret_cast<const uint2*>(srow + i * 8);
    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (i / kDownStages) & 1, a.status))) {
      ok = false;
      break;
    }
    uint4 wb[8];
    if (active) {
      const uint8_t* base = stages + s * kDownStageBytes + slot * kDownBox + r * 128;
#pragma unroll
      for (int g = 0; g < 8; ++g) wb[g] = *reinterpret_cast<const uint4*>(base + 16 * (g ^ (r & 7)));
    }
    if (active) fp4_box_accumulate_half(wb, hslot, hmul, i, sb, hf, acc);
    __syncwarp();  // slot released after its data has been consumed
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (ok && active) {  // warp-uniform
    const float yv = __fadd_rn(hsum8_pair(acc), 0.0f);
    if (!isfinite(yv)) flag(a.status, WH_DEV_NONFINITE);
    if (hf == 0) {
      ys[slot * kDownRows + r] = yv;
      if (a.expert_out)
        a.expert_out[((long long)t * nslots + slot) * a.hidden + row] = yv;
    }
  }
  const int ok_all = bar_and(1, kDownConsumers * 32, ok);
  if (ok_all && a.combine && threadIdx.x < kDownRows) {
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

// ---------------------------------------------------------------------------
// Batched router (many tokens, no act-quantised copy needed): the logits as a
// tiled CUDA-core GEMM and then one warp per token for the top-k.  A thread
// owns one expert x 4 tokens and keeps, for each of them, the 16 FMA chains
// of dot_bf16_row_avx2 (src/compute.rs:6115-6136: chain p accumulates
// columns 16c + p; logit = pairwise hsum of chain p + chain p+8, p < 8), so
// every logit -- and therefore every selected id -- is the reference's bit
// for bit.  Tiles: 32 experts x 32 tokens x 64 columns, double-buffered in
// shared memory with a register prefetch of the next tile.
// ---------------------------------------------------------------------------
constexpr int kRbTile = 32, kRbK = 64, kRbStride = kRbK + 4;  // floats per padded smem row

__global__ void __launch_bounds__(256) router_logits_batched_kernel(RouterArgs a) {
  __shared__ __align__(16) float ws[2][kRbTile * kRbStride];
  __shared__ __align__(16) float xs[2][kRbTile * kRbStride];
  const int e0 = blockIdx.x * kRbTile, t0 = blockIdx.y * kRbTile;
  const int tid = threadIdx.x, lane = tid & 31, tg = tid >> 5;  // expert e0+lane, tokens 4tg..
  // loaders: gate row gr, 8 bf16 at column 8*gc; x rows xr[j], 4 floats at 4*xc[j]
  const int gr = tid >> 3, gc = tid & 7;
  const uint4* gsrc = reinterpret_cast<const uint4*>(
      a.gate + (long long)min(e0 + gr, a.experts - 1) * a.hidden + gc * 8);
  const float4* xsrc[2];
  int xoff[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = tid + 256 * j, r = i >> 4, c = i & 15;
    xsrc[j] = reinterpret_cast<const float4*>(a.x + (long long)min(t0 + r, a.tokens - 1) * a.hidden +
                                              c * 4);
    xoff[j] = r * kRbStride + c * 4;
  }
  uint4 gv;
  float4 xv[2];
  auto fetch = [&](int k0) {
    gv = __ldg(gsrc + k0 / 8);
    xv[0] = __ldg(xsrc[0] + k0 / 4);
    xv[1] = __ldg(xsrc[1] + k0 / 4);
  };
  auto stash = [&](int st) {
    float* w = &ws[st][gr * kRbStride + gc * 8];
    *reinterpret_cast<float4*>(w) =
        make_float4(__uint_as_float(gv.x << 16), __uint_as_float(gv.x & 0xffff0000u),
                    __uint_as_float(gv.y << 16), __uint_as_float(gv.y & 0xffff0000u));
    *reinterpret_cast<float4*>(w + 4) =
        make_float4(__uint_as_float(gv.z << 16), __uint_as_float(gv.z & 0xffff0000u),
                    __uint_as_float(gv.w << 16), __uint_as_float(gv.w & 0xffff0000u));
    *reinterpret_cast<float4*>(&xs[st][xoff[0]]) = xv[0];
    *reinterpret_cast<float4*>(&xs[st][xoff[1]]) = xv[1];
  };
  float acc[4][16];
#pragma unroll
  for (int t = 0; t < 4; ++t)
#pragma unroll
    for (int p = 0; p < 16; ++p) acc[t][p] = 0.0f;
  const int nk = a.hidden / kRbK;
  fetch(0);
  stash(0);
  __syncthreads();
  for (int kc = 0; kc < nk; ++kc) {
    if (kc + 1 < nk) fetch((kc + 1) * kRbK);
    const float* wr = &ws[kc & 1][lane * kRbStride];
    const float* xr = &xs[kc & 1][(tg * 4) * kRbStride];
#pragma unroll
    for (int c = 0; c < kRbK / 16; ++c) {
      float w[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(wr + c * 16 + 4 * q);
        w[4 * q] = v.x;
        w[4 * q + 1] = v.y;
        w[4 * q + 2] = v.z;
        w[4 * q + 3] = v.w;
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = *reinterpret_cast<const float4*>(xr + t * kRbStride + c * 16 + 4 * q);
          acc[t][4 * q] = __fmaf_rn(w[4 * q], v.x, acc[t][4 * q]);
          acc[t][4 * q + 1] = __fmaf_rn(w[4 * q + 1], v.y, acc[t][4 * q + 1]);
          acc[t][4 * q + 2] = __fmaf_rn(w[4 * q + 2], v.z, acc[t][4 * q + 2]);
          acc[t][4 * q + 3] = __fmaf_rn(w[4 * q + 3], v.w, acc[t][4 * q + 3]);
        }
      }
    }
    if (kc + 1 < nk) stash((kc + 1) & 1);
    __syncthreads();
  }
  const int e = e0 + lane;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int tok = t0 + tg * 4 + t;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(acc[t][j], acc[t][8 + j]);
    const float h = __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3])),
                              __fadd_rn(__fadd_rn(v[4], v[5]), __fadd_rn(v[6], v[7])));
    // + the (empty) column tail, as the reference adds it: -0 becomes +0
    if (e < a.experts && tok < a.tokens) a.logits[(long long)tok * a.experts + e] = __fadd_rn(h, 0.0f);
  }
}

template <int PER>
__global__ void __launch_bounds__(128) router_topk_kernel(RouterArgs a) {
  const int t = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t >= a.tokens) return;  // warp-uniform
  const int lane = threadIdx.x & 31;
  router_topk_and_weights<PER>(a, t, lane, false,
                               [&](auto& sc) { router_load_global(a, t, lane, sc); });
}

// Router logits of a decode batch (up to 128 tokens): the 32 x 32 tiles above
// give such a batch only experts/32 x tokens/32 CTAs (8 for 256 experts and 32
// tokens), each walking the whole hidden dimension.  Here a warp owns 16
// experts x TB tokens with two lanes per expert row, the lanes holding chains
// 8h + j over columns 16c + 8h + j -- the same 16 chains in the same order as
// the tile kernel's, summed the same way -- and the grid has experts/64 x
// tokens/TB CTAs of four warps (TB = 1 up to 32 tokens, 4 up to 128).  The
// gate rows are read through L2 (2 MB for 256 x 4096), 16 chunks in flight per
// lane.
constexpr int kRsWarps = 4;
constexpr int kRsDepth = 16;
template <int TB>
__global__ void __launch_bounds__(32 * kRsWarps) router_logits_small_kernel(RouterArgs a) {
  extern __shared__ __align__(16) float rs_x[];  // [TB][hidden]
  const int t0 = blockIdx.y * TB;
  const int nt = min(TB, a.tokens - t0);
  for (int i = threadIdx.x * 4; i < TB * a.hidden; i += blockDim.x * 4) {
    const int tt = i / a.hidden, col = i - tt * a.hidden;
    *reinterpret_cast<float4*>(rs_x + i) =
        tt < nt ? __ldg(reinterpret_cast<const float4*>(a.x + (long long)(t0 + tt) * a.hidden + col))
                : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, half = lane & 1;
  const int e = (blockIdx.x * kRsWarps + warp) * 16 + (lane >> 1);
  const bool active = e < a.experts;
  const uint8_t* wp = reinterpret_cast<const uint8_t*>(a.gate + (long long)(active ? e : a.experts - 1) *
                                                                    a.hidden) + 16 * half;
  const int chunks = a.hidden / 16;
  float2 acc[TB][4];
#pragma unroll
  for (int tt = 0; tt < TB; ++tt)
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[tt][k] = make_float2(0.0f, 0.0f);
  auto step = [&](const uint4 w, int c) {
    const float2 w0 = make_float2(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u));
    const float2 w1 = make_float2(__uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u));
    const float2 w2 = make_float2(__uint_as_float(w.z << 16), __uint_as_float(w.z & 0xffff0000u));
    const float2 w3 = make_float2(__uint_as_float(w.w << 16), __uint_as_float(w.w & 0xffff0000u));
#pragma unroll
    for (int tt = 0; tt < TB; ++tt) {
      const float* xp = rs_x + tt * a.hidden + 8 * half + 16 * c;
      const float4 xa = *reinterpret_cast<const float4*>(xp);
      const float4 xb = *reinterpret_cast<const float4*>(xp + 4);
      acc[tt][0] = ffma2(w0, make_float2(xa.x, xa.y), acc[tt][0]);
      acc[tt][1] = ffma2(w1, make_float2(xa.z, xa.w), acc[tt][1]);
      acc[tt][2] = ffma2(w2, make_float2(xb.x, xb.y), acc[tt][2]);
      acc[tt][3] = ffma2(w3, make_float2(xb.z, xb.w), acc[tt][3]);
    }
  };
  int c = 0;
  for (; c + kRsDepth <= chunks; c += kRsDepth) {
    uint4 w[kRsDepth];
#pragma unroll
    for (int k = 0; k < kRsDepth; ++k) w[k] = __ldg(reinterpret_cast<const uint4*>(wp + 32 * (c + k)));
#pragma unroll
    for (int k = 0; k < kRsDepth; ++k) step(w[k], c + k);
  }
  for (; c < chunks; ++c) step(__ldg(reinterpret_cast<const uint4*>(wp + 32 * c)), c);
#pragma unroll
  for (int tt = 0; tt < TB; ++tt) {
    // v_j = chain j + chain 8 + j (the partner lane), then
    // ((v0 + v1) + (v2 + v3)) + ((v4 + v5) + (v6 + v7)), then the empty column tail
    float p[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      p[2 * k] = __fadd_rn(acc[tt][k].x, __shfl_xor_sync(0xffffffffu, acc[tt][k].x, 1));
      p[2 * k + 1] = __fadd_rn(acc[tt][k].y, __shfl_xor_sync(0xffffffffu, acc[tt][k].y, 1));
    }
    if (half == 0 && active && tt < nt) {
      const float h = __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])),
                                __fadd_rn(__fadd_rn(p[4], p[5]), __fadd_rn(p[6], p[7])));
      a.logits[(long long)(t0 + tt) * a.experts + e] = __fadd_rn(h, 0.0f);
    }
  }
}

template <int TB>
static cudaError_t launch_router_small(const RouterArgs& a, cudaStream_t s) {
  const size_t smem = size_t(TB) * a.hidden * 4;
  cudaError_t e = ensure_smem(router_logits_small_kernel<TB>, smem);
  if (e != cudaSuccess) return e;
  dim3 grid((a.experts + 16 * kRsWarps - 1) / (16 * kRsWarps), (a.tokens + TB - 1) / TB);
  router_logits_small_kernel<TB><<<grid, 32 * kRsWarps, smem, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_router_batched(const RouterArgs& a, cudaStream_t s) {
  if (a.tokens <= 32 && a.hidden % 16 == 0) {
    cudaError_t e = launch_router_small<1>(a, s);
    if (e != cudaSuccess) return e;
  } else if (a.tokens <= 128 && a.hidden % 16 == 0) {
    cudaError_t e = launch_router_small<4>(a, s);
    if (e != cudaSuccess) return e;
  } else {
    dim3 grid((a.experts + kRbTile - 1) / kRbTile, (a.tokens + kRbTile - 1) / kRbTile);
    router_logits_batched_kernel<<<grid, 256, 0, s>>>(a);
  }
  const int blocks = (a.tokens + 3) / 4;
  if (a.experts <= 32) router_topk_kernel<1><<<blocks, 128, 0, s>>>(a);
  else if (a.experts <= 64) router_topk_kernel<2><<<blocks, 128, 0, s>>>(a);
  else if (a.experts <= 128) router_topk_kernel<4><<<blocks, 128, 0, s>>>(a);
  else if (a.experts <= 256) router_topk_kernel<8><<<blocks, 128, 0, s>>>(a);
  else if (a.experts <= 512) router_topk_kernel<16><<<blocks, 128, 0, s>>>(a);
  else router_topk_kernel<32><<<blocks, 128, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_router_ex(const RouterArgs& a, __half* xq, float* xq_mult, cudaStream_t s,
                             bool pdl) {
  if (xq == nullptr && a.tokens >= 32 && a.hidden % kRbK == 0 &&
      (reinterpret_cast<uintptr_t>(a.gate) % 16) == 0 &&
      (reinterpret_cast<uintptr_t>(a.x) % 16) == 0)
    return launch_router_batched(a, s);
  cudaLaunchAttribute attr[1];
  dim3 grid((a.experts + kRouterRowsPerCta - 1) / kRouterRowsPerCta, a.tokens);
  const bool smem_ok = a.hidden % 8 == 0 && (reinterpret_cast<uintptr_t>(a.gate) % 16) == 0 &&
                       (reinterpret_cast<uintptr_t>(a.x) % 16) == 0 &&
                       router_smem_plan(a.hidden).bytes <= 200 * 1024;
  if (smem_ok) {
    const size_t smem = router_smem_plan(a.hidden).bytes;
    cudaError_t e = ensure_smem(router_kernel<true>, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = pdl_cfg(grid, dim3(kRouterThreads), smem, s, attr, pdl);
    return cudaLaunchKernelEx(&cfg, router_kernel<true>, a, xq, xq_mult);
  }
  cudaLaunchConfig_t cfg = pdl_cfg(grid, dim3(kRouterThreads), 64, s, attr, pdl);
  return cudaLaunchKernelEx(&cfg, router_kernel<false>, a, xq, xq_mult);
}

cudaError_t launch_moe_up_ex(const MoeArgs& a, const __half* xq, const float* xq_mult, __half* hq,
                             float* hq_mult, cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  const size_t smem = moe_up_smem_bytes(a.hidden);
  cudaError_t e = ensure_smem(moe_up_kernel, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.inter / kUpRows, a.topk + a.has_shared, a.tokens);
  cudaLaunchConfig_t cfg = pdl_cfg(grid, dim3(kUpThreads), smem, s, attr, pdl);
  return cudaLaunchKernelEx(&cfg, moe_up_kernel, a, xq, xq_mult, hq, hq_mult);
}

cudaError_t launch_moe_down_ex(const MoeArgs& a, const __half* hq, const float* hq_mult,
                               cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  const size_t smem = moe_down_smem_bytes(a.inter, a.topk + a.has_shared);
  cudaError_t e = ensure_smem(moe_down_kernel, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.hidden / kDownRows, a.tokens);
  cudaLaunchConfig_t cfg = pdl_cfg(grid, dim3(kDownThreads), smem, s, attr, pdl);
  return cudaLaunchKernelEx(&cfg, moe_down_kernel, a, hq, hq_mult);
}

// Stand-alone act quant to f16 grid values + block multipliers (x = q*mult/8)
// x from pinned host memory into device memory (n floats, 16-byte aligned):
// one pass over the bus, no copy engine
__global__ void __launch_bounds__(256) stage_rows_kernel(const float4* __restrict__ src,
                                                         float4* __restrict__ dst, size_t n4) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

cudaError_t launch_stage_rows(const float* src, float* dst, size_t n, cudaStream_t s) {
  const size_t n4 = n / 4;
  const unsigned grid = (unsigned)std::min<size_t>((n4 + 255) / 256, 1024);
  stage_rows_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const float4*>(src),
                                         reinterpret_cast<float4*>(dst), n4);
  return cudaGetLastError();
}

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
