// lmhead.cu -- BF16 lm_head top-k for sm_100a.
//
// Replaces score_bf16_lm_head_topk (engine/zc_infer_core/src/compute.rs:
// 2867-2913) and RowIndex::topk_bf16_lm_head (src/row_index.rs:208-300): the
// logit of every row is dot_bf16_row (AVX2 order, src/compute.rs:6116-6136: 16
// FMA chains over the whole row, acc0 lanes j on columns 16c+j, acc1 lanes j
// on 16c+8+j, then hsum256(acc0 + acc1) + tail), and the k best rows are those
// push_topk_candidate keeps (src/compute.rs:2948-2962), sorted descending by
// total_cmp.
//
//   lm_logits_kernel        persistent (4 CTAs per SM); a warp takes 16-row
//                           passes from a counter, 2 lanes per row (a lane
//                           holds one accumulator's 8 chains as f32 pairs), x
//                           in shared memory, streaming 16-byte weight loads
//                           It also builds a histogram of the logits'
//                           total-order keys (top 12 bits).
//   lm_collect_kernel       the bin above which k+1 rows lie; those rows are
//                           compacted into a candidate list
//   lm_select_kernel        one CTA sorts the candidates by (value desc in
//                           total order, row asc).  When the k best values are
//                           distinct and above the (k+1)-th (IEEE comparison)
//                           and no logit is NaN, the reference's result is
//                           exactly the sorted top k.  Otherwise one warp
//                           replays push_topk_candidate over all logits in
//                           row order (its vector positions decide ties).
#include "common.cuh"
#include "kernels.cuh"

namespace wh {

constexpr int kLmRowsPerWarp = 16;
constexpr int kLmWarps = 8;
constexpr int kLmMaxK = 511;
constexpr int kLmSelCap = 8192;
constexpr int kLmBins = 4096;

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// f32::total_cmp key as an unsigned value that grows with the float
__device__ __forceinline__ uint32_t total_ukey(float f) {
  const int32_t b = __float_as_int(f);
  return uint32_t(b ^ int32_t(uint32_t(b >> 31) >> 1)) ^ 0x80000000u;
}
// ascending order of the 64-bit key = value descending (total order), row ascending
__device__ __forceinline__ uint64_t lm_key(float v, uint32_t row) {
  return (uint64_t(~total_ukey(v)) << 32) | row;
}
__device__ __forceinline__ float lm_key_value(uint64_t k) {
  const uint32_t u = ~uint32_t(k >> 32) ^ 0x80000000u;  // total key
  const int32_t b = int32_t(u);
  return __int_as_float(b ^ int32_t(uint32_t(b >> 31) >> 1));
}

__global__ void __launch_bounds__(32 * kLmWarps) lm_logits_kernel(LmHeadArgs a) {
  extern __shared__ __align__(16) float lm_xs[];
  pdl_wait_prior();
  for (int i = threadIdx.x; i < a.cols; i += blockDim.x) lm_xs[i] = a.x[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int half = lane & 1;
  const int chunks = a.cols / 16;
  const float* xp = lm_xs + 8 * half;
  const long long passes = (a.rows + kLmRowsPerWarp - 1) / kLmRowsPerWarp;
  // warps take 16-row passes from a counter, so the launch ends within about one
  // pass of its average instead of a whole extra wave
  for (;;) {
    long long pass = 0;
    if (lane == 0) pass = (long long)atomicAdd(a.counter, 1u);
    pass = __shfl_sync(0xffffffffu, pass, 0);
    if (pass >= passes) break;
    const long long row = pass * kLmRowsPerWarp + (lane >> 1);
    const bool active = row < a.rows;
    const long long rr = active ? row : a.rows - 1;  // every lane joins the shuffles
    const uint16_t* wrow = a.weight + rr * a.cols;
    const uint8_t* wp = reinterpret_cast<const uint8_t*>(wrow) + 16 * half;
    float2 acc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] = make_float2(0.0f, 0.0f);
    auto step = [&](const uint4 w, int c) {
      const float4 xa = *reinterpret_cast<const float4*>(xp + 16 * c);
      const float4 xb = *reinterpret_cast<const float4*>(xp + 16 * c + 4);
      acc[0] = ffma2(make_float2(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u)),
                     make_float2(xa.x, xa.y), acc[0]);
      acc[1] = ffma2(make_float2(__uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u)),
                     make_float2(xa.z, xa.w), acc[1]);
      acc[2] = ffma2(make_float2(__uint_as_float(w.z << 16), __uint_as_float(w.z & 0xffff0000u)),
                     make_float2(xb.x, xb.y), acc[2]);
      acc[3] = ffma2(make_float2(__uint_as_float(w.w << 16), __uint_as_float(w.w & 0xffff0000u)),
                     make_float2(xb.z, xb.w), acc[3]);
    };
    int c = 0;
    for (; c + 8 <= chunks; c += 8) {
      uint4 w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) w[k] = ld_stream_v4(wp + 32 * (c + k));
#pragma unroll
      for (int k = 0; k < 8; ++k) step(w[k], c + k);
    }
    for (; c < chunks; ++c) step(ld_stream_v4(wp + 32 * c), c);
    // P_j = acc0_j + acc1_j (the partner lane holds the other accumulator), then
    // hsum256: ((P0 + P1) + (P2 + P3)) + ((P4 + P5) + (P6 + P7))
    float p[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      p[2 * k] = __fadd_rn(acc[k].x, __shfl_xor_sync(0xffffffffu, acc[k].x, 1));
      p[2 * k + 1] = __fadd_rn(acc[k].y, __shfl_xor_sync(0xffffffffu, acc[k].y, 1));
    }
    int bin = -1;
    if (half == 0 && active) {
      const float h = __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])),
                                __fadd_rn(__fadd_rn(p[4], p[5]), __fadd_rn(p[6], p[7])));
      float tail = 0.0f;
      for (int i = chunks * 16; i < a.cols; ++i)
        tail = __fadd_rn(tail, __fmul_rn(__uint_as_float(uint32_t(wrow[i]) << 16), lm_xs[i]));
      const float v = __fadd_rn(h, tail);
      a.logits[row] = v;
      if (isnan(v)) atomicOr(a.flags, 1u);
      bin = int(total_ukey(v) >> 20);
    }
    // histogram of the top 12 bits of the total-order key (the selection's
    // first step), one atomic per distinct bin of the warp's 16 rows
    const uint32_t peers = __match_any_sync(0xffffffffu, bin);
    if (bin >= 0 && lane == __ffs(peers) - 1) atomicAdd(&a.hist[bin], __popc(peers));
  }
  pdl_launch_dependents();
}

// Logits of TB tokens per weight pass (several-token call): the same row
// passes, lanes and chain order as lm_logits_kernel, with the tile's inputs
// in shared memory and TB accumulator sets per lane, so the weights stream
// once per tile of tokens instead of once per token.  Grid y = token tiles;
// each tile hands out its passes from the counter of its first token.
template <int TB>
constexpr int lm_batch_threads() { return TB >= 8 ? 256 : 512; }  // 8 tokens: registers
template <int TB>
__global__ void __launch_bounds__(lm_batch_threads<TB>(), 1) lm_logits_batch_kernel(LmHeadArgs a) {
  extern __shared__ __align__(16) float lm_xt[];  // [TB][cols]
  const int t0 = blockIdx.y * TB;
  const int nt = min(TB, a.tokens - t0);
  pdl_wait_prior();
  for (int i = threadIdx.x; i < TB * a.cols; i += blockDim.x) {
    const int tt = i / a.cols, col = i - tt * a.cols;
    lm_xt[i] = tt < nt ? a.x[(long long)(t0 + tt) * a.ldx + col] : 0.0f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int half = lane & 1;
  const int chunks = a.cols / 16;
  uint32_t* counter = a.flags + (long long)t0 * kLmTokWords + 1;
  const long long passes = (a.rows + kLmRowsPerWarp - 1) / kLmRowsPerWarp;
  for (;;) {
    long long pass = 0;
    if (lane == 0) pass = (long long)atomicAdd(counter, 1u);
    pass = __shfl_sync(0xffffffffu, pass, 0);
    if (pass >= passes) break;
    const long long row = pass * kLmRowsPerWarp + (lane >> 1);
    const bool active = row < a.rows;
    const long long rr = active ? row : a.rows - 1;  // every lane joins the shuffles
    const uint16_t* wrow = a.weight + rr * a.cols;
    const uint8_t* wp = reinterpret_cast<const uint8_t*>(wrow) + 16 * half;
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
        const float* xp = lm_xt + tt * a.cols + 8 * half + 16 * c;
        const float4 xa = *reinterpret_cast<const float4*>(xp);
        const float4 xb = *reinterpret_cast<const float4*>(xp + 4);
        acc[tt][0] = ffma2(w0, make_float2(xa.x, xa.y), acc[tt][0]);
        acc[tt][1] = ffma2(w1, make_float2(xa.z, xa.w), acc[tt][1]);
        acc[tt][2] = ffma2(w2, make_float2(xb.x, xb.y), acc[tt][2]);
        acc[tt][3] = ffma2(w3, make_float2(xb.z, xb.w), acc[tt][3]);
      }
    };
    int c = 0;
    for (; c + 4 <= chunks; c += 4) {
      uint4 w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) w[k] = ld_stream_v4(wp + 32 * (c + k));
#pragma unroll
      for (int k = 0; k < 4; ++k) step(w[k], c + k);
    }
    for (; c < chunks; ++c) step(ld_stream_v4(wp + 32 * c), c);
#pragma unroll
    for (int tt = 0; tt < TB; ++tt) {
      // P_j = acc0_j + acc1_j, then ((P0 + P1) + (P2 + P3)) + ((P4 + P5) + (P6 + P7))
      float p[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        p[2 * k] = __fadd_rn(acc[tt][k].x, __shfl_xor_sync(0xffffffffu, acc[tt][k].x, 1));
        p[2 * k + 1] = __fadd_rn(acc[tt][k].y, __shfl_xor_sync(0xffffffffu, acc[tt][k].y, 1));
      }
      int bin = -1;
      if (half == 0 && active && tt < nt) {
        const float h = __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])),
                                  __fadd_rn(__fadd_rn(p[4], p[5]), __fadd_rn(p[6], p[7])));
        const float* xt = lm_xt + tt * a.cols;
        float tail = 0.0f;
        for (int i = chunks * 16; i < a.cols; ++i)
          tail = __fadd_rn(tail, __fmul_rn(__uint_as_float(uint32_t(wrow[i]) << 16), xt[i]));
        const float v = __fadd_rn(h, tail);
        const long long t = t0 + tt;
        a.logits[t * a.rows + row] = v;
        if (isnan(v)) atomicOr(a.flags + t * kLmTokWords, 1u);
        bin = int(total_ukey(v) >> 20);
      }
      const uint32_t peers = __match_any_sync(0xffffffffu, bin);
      if (bin >= 0 && lane == __ffs(peers) - 1)
        atomicAdd(reinterpret_cast<int*>(a.flags + (long long)(t0 + tt) * kLmTokWords + 4) + bin,
                  __popc(peers));
    }
  }
  pdl_launch_dependents();
}

// The arguments of token t of a several-token call (t = 0: the call itself).
__device__ __forceinline__ LmHeadArgs lm_token(const LmHeadArgs& a0, int t) {
  LmHeadArgs a = a0;
  if (t > 0) {
    a.x = a0.x + (long long)t * a0.ldx;
    a.logits = a0.logits + (long long)t * a0.rows;
    a.flags = a0.flags + (long long)t * kLmTokWords;
    a.counter = a.flags + 1;
    a.cand_count = a.flags + 2;
    a.hist = reinterpret_cast<int*>(a.flags + 4);
    a.cand = a0.cand + (long long)t * kLmSelCap;
    a.out_tokens = a0.out_tokens + (long long)t * a0.top_k;
    a.out_logits = a0.out_logits + (long long)t * a0.top_k;
  }
  return a;
}

// in-place ascending bitonic sort of n (a power of two) keys in shared memory
__device__ void bitonic_sort(uint64_t* k, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint64_t x = k[lo], y = k[hi];
        if ((x > y) == up) {
          k[lo] = y;
          k[hi] = x;
        }
      }
    }
  }
  __syncthreads();
}

// push_topk_candidate replayed in row order by one warp (the tie / NaN path).
// best_* hold the reference's vector; lanes test 32 rows at a time against the
// current minimum and the entering rows are applied one by one in row order.
__device__ void lm_replay(const LmHeadArgs& a, uint32_t* best_row, float* best_val, int* n_out) {
  const int lane = threadIdx.x & 31;
  const int k = a.top_k;
  int n = 0;
  float mval = 0.0f;  // current minimum (total_cmp), first position among equals
  int mpos = 0;
  auto recompute_min = [&]() {
    uint64_t best = ~0ull;  // (total key, position): smallest first
    for (int i = lane; i < n; i += 32) {
      const uint64_t key = (uint64_t(total_ukey(best_val[i])) << 32) | uint32_t(i);
      best = key < best ? key : best;
    }
    for (int o = 16; o; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other < best ? other : best;
    }
    mpos = int(uint32_t(best));
    mval = best_val[mpos];
  };
  for (long long base = 0; base < a.rows; base += 32) {
    const long long r = base + lane;
    const bool in = r < a.rows;
    const float v = in ? a.logits[r] : 0.0f;
    uint32_t todo = __ballot_sync(0xffffffffu, in);
    while (todo) {
      if (n < k) {
        // filling: the next row in order is appended
        const int src = __ffs(todo) - 1;
        const float vv = __shfl_sync(0xffffffffu, v, src);
        if (lane == 0) {
          best_row[n] = uint32_t(base + src);
          best_val[n] = vv;
        }
        __syncwarp();
        ++n;
        todo &= todo - 1;
        if (n == k) recompute_min();
        continue;
      }
      // the first remaining row that beats the current minimum replaces it
      const uint32_t enter = __ballot_sync(0xffffffffu, in && v > mval) & todo;
      if (!enter) break;
      const int src = __ffs(enter) - 1;
      const float vv = __shfl_sync(0xffffffffu, v, src);
      if (lane == 0) {
        best_row[mpos] = uint32_t(base + src);
        best_val[mpos] = vv;
      }
      __syncwarp();
      todo &= ~((2u << src) - 1u);  // rows up to src are done
      recompute_min();
    }
  }
  *n_out = n;
}

// The rows whose logit lies in the histogram bin that leaves at least k+1
// rows at or above it, or in a higher bin: about k+1 plus the few that share
// the boundary bin.  Every CTA finds the bin from the histogram itself.
constexpr int kLmCollectRows = 8 * 1024;  // rows per collect CTA

__global__ void __launch_bounds__(1024) lm_collect_kernel(LmHeadArgs a0) {
  const LmHeadArgs a = lm_token(a0, blockIdx.y);
  __shared__ int s_bin;
  __shared__ int hist[kLmBins];
  const int tid = threadIdx.x, lane = tid & 31;
  pdl_wait_prior();
  // the logits this CTA examines, loaded before the histogram work
  const long long r0 = (long long)blockIdx.x * kLmCollectRows;
  float v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const long long r = r0 + k * 1024 + tid;
    v[k] = r < a.rows ? a.logits[r] : 0.0f;
  }
  for (int i = tid; i < kLmBins; i += blockDim.x) hist[i] = a.hist[i];
  __syncthreads();
  const long long want = a.rows < a.top_k + 1 ? a.rows : (long long)a.top_k + 1;
  if (tid < 32) {
    // lane l sums 128 bins from the top: [4095 - 128 l - 127, 4095 - 128 l]
    int sum = 0;
    for (int i = 0; i < 128; ++i) sum += hist[kLmBins - 1 - 128 * lane - i];
    int incl = sum;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int excl = incl - sum;
    const uint32_t hit = __ballot_sync(0xffffffffu, incl >= want && excl < want);
    const int src = hit ? __ffs(hit) - 1 : 31;
    if (lane == src) {
      int acc = excl, b = kLmBins - 1 - 128 * lane;
      for (int i = 0; i < 128; ++i, --b) {
        acc += hist[b];
        if (acc >= want) break;
      }
      s_bin = b < 0 ? 0 : b;
    }
  }
  __syncthreads();
  const int bmin = s_bin;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const long long r = r0 + k * 1024 + tid;
    if (r < a.rows && int(total_ukey(v[k]) >> 20) >= bmin) {
      const uint32_t slot = atomicAdd(a.cand_count, 1u);
      if (slot < uint32_t(kLmSelCap)) a.cand[slot] = lm_key(v[k], uint32_t(r));
    }
  }
  pdl_launch_dependents();
}

// One CTA sorts the candidates.  When the k best values are distinct and above
// the (k+1)-th (IEEE comparison) and no logit is NaN, the reference's result
// is exactly the sorted top k; ties, NaNs or more candidates than fit take the
// exact replay of push_topk_candidate.
__global__ void __launch_bounds__(256) lm_select_kernel(LmHeadArgs a0) {
  const LmHeadArgs a = lm_token(a0, blockIdx.x);
  extern __shared__ __align__(16) uint64_t lm_sel[];  // cand[kLmSelCap] | replay state
  __shared__ int s_n;
  uint64_t* cand = lm_sel;
  uint32_t* best_row = reinterpret_cast<uint32_t*>(cand + kLmSelCap);
  float* best_val = reinterpret_cast<float*>(best_row + kLmMaxK + 1);
  const int tid = threadIdx.x;
  pdl_wait_prior();
  const uint32_t n = *a.cand_count;
  bool replay = n > uint32_t(kLmSelCap);
  if (!replay) {
    int n2 = 1;
    while (n2 < int(n)) n2 <<= 1;
    for (int i = tid; i < n2; i += blockDim.x) cand[i] = i < int(n) ? a.cand[i] : ~0ull;
    bitonic_sort(cand, n2);
    // rows <= k: nothing was ever replaced and the key order is the answer;
    // otherwise an IEEE tie among the first k + 1 (or a NaN) needs the replay
    bool fb = false;
    if (a.rows > a.top_k) {
      for (int i = tid; i < a.top_k; i += blockDim.x)
        fb |= lm_key_value(cand[i]) == lm_key_value(cand[i + 1]);
      if (tid == 0) fb |= (*a.flags & 1u) != 0;
    }
    replay = __syncthreads_or(fb) != 0;
    if (!replay) {
      const int count = int(a.rows < a.top_k ? a.rows : (long long)a.top_k);
      for (int i = tid; i < count; i += blockDim.x) {
        a.out_tokens[i] = a.row_base + uint32_t(cand[i]);
        a.out_logits[i] = lm_key_value(cand[i]);
      }
      pdl_launch_dependents();
      return;
    }
  }
  if (tid < 32) {
    int nn = 0;
    lm_replay(a, best_row, best_val, &nn);
    if (tid == 0) s_n = nn;
  }
  __syncthreads();
  // sort_by(|l, r| r.total_cmp(l)) is stable: ties keep vector order
  const int nb = s_n;
  int m2 = 1;
  while (m2 < nb) m2 <<= 1;
  for (int i = tid; i < m2; i += blockDim.x)
    cand[i] = i < nb ? (uint64_t(~total_ukey(best_val[i])) << 32) | uint32_t(i) : ~0ull;
  bitonic_sort(cand, m2);
  for (int i = tid; i < nb; i += blockDim.x) {
    const int pos = int(uint32_t(cand[i]));
    a.out_tokens[i] = a.row_base + best_row[pos];
    a.out_logits[i] = best_val[pos];
  }
  pdl_launch_dependents();
}

size_t lm_head_scratch_bytes(long long rows, int top_k) {
  (void)top_k;
  return 1024 + size_t(rows) * 4 + size_t(kLmBins) * 4 + size_t(kLmSelCap) * 8;
}

bool lm_head_supported(long long rows, int cols, int top_k) {
  return top_k >= 1 && top_k <= kLmMaxK && cols >= 1 && cols <= 16384 && rows >= 1 &&
         rows < (1ll << 31);
}

// stage 0: logits + histogram; 1: candidates; 2: the selection (or the replay).
// pdl: launch stages 1 and 2 with programmatic dependent launch.
cudaError_t launch_lm_head_stage(const LmHeadArgs& a, int stage, bool pdl, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = (stage > 0 && pdl) ? 1 : 0;
  cudaError_t e;
  switch (stage) {
    case 0: {
      int dev = 0, sms = 148;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      const long long passes = (a.rows + kLmRowsPerWarp - 1) / kLmRowsPerWarp;
      const long long ctas = std::min<long long>(4LL * sms, (passes + kLmWarps - 1) / kLmWarps);
      cfg.blockDim = dim3(32 * kLmWarps);
      cfg.gridDim = dim3(unsigned(ctas));
      cfg.dynamicSmemBytes = size_t(a.cols) * 4;
      e = ensure_smem(lm_logits_kernel, cfg.dynamicSmemBytes);
      return e != cudaSuccess ? e : cudaLaunchKernelEx(&cfg, lm_logits_kernel, a);
    }
    case 1:
      cfg.blockDim = dim3(1024);
      cfg.gridDim = dim3(unsigned((a.rows + kLmCollectRows - 1) / kLmCollectRows));
      return cudaLaunchKernelEx(&cfg, lm_collect_kernel, a);
    default:
      cfg.blockDim = dim3(256);
      cfg.gridDim = dim3(1);
      cfg.dynamicSmemBytes = size_t(kLmSelCap) * 8 + 2 * (kLmMaxK + 1) * 4;
      e = ensure_smem(lm_select_kernel, cfg.dynamicSmemBytes);
      return e != cudaSuccess ? e : cudaLaunchKernelEx(&cfg, lm_select_kernel, a);
  }
}

size_t lm_head_batch_scratch_bytes(long long rows, int top_k, int tokens) {
  (void)top_k;
  return 1024 + size_t(tokens) * (size_t(rows) * 4 + size_t(kLmTokWords) * 4 +
                                  size_t(kLmSelCap) * 8);
}

// Tokens per weight pass: as many as fit (with x) in 192 KB of shared memory,
// and no more than the call's token count rounded up to a power of two.
static int lm_batch_tile(int cols, int tokens) {
  const size_t bytes = size_t(cols) * 4;
  int tb = bytes * 8 <= 192 * 1024 ? 8 : bytes * 4 <= 192 * 1024 ? 4 : bytes * 2 <= 192 * 1024 ? 2 : 1;
  while (tb > 1 && tb / 2 >= tokens) tb /= 2;
  return tb;
}

template <int TB>
static cudaError_t launch_lm_logits_batch(const LmHeadArgs& a, cudaLaunchConfig_t cfg) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long passes = (a.rows + kLmRowsPerWarp - 1) / kLmRowsPerWarp;
  const int tiles = (a.tokens + TB - 1) / TB;
  const long long per_tile = std::max<long long>(1, sms / tiles);
  cfg.blockDim = dim3(lm_batch_threads<TB>());
  cfg.gridDim = dim3(unsigned(std::min<long long>(per_tile, (passes + 15) / 16)), tiles);
  cfg.dynamicSmemBytes = size_t(TB) * a.cols * 4;
  cudaError_t e = ensure_smem(lm_logits_batch_kernel<TB>, cfg.dynamicSmemBytes);
  return e != cudaSuccess ? e : cudaLaunchKernelEx(&cfg, lm_logits_batch_kernel<TB>, a);
}

// Several tokens: the logits of every token (weights streamed once per tile of
// tokens), then the candidates and the selection of every token, one grid each.
cudaError_t launch_lm_head_batch(const LmHeadArgs& a, bool pdl, cudaStream_t s) {
  if (a.tokens == 1) {  // token 0's words are the single call's layout
    cudaError_t e = cudaSuccess;
    for (int stage = 0; stage < 3 && e == cudaSuccess; ++stage) e = launch_lm_head_stage(a, stage, pdl, s);
    return e;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  cudaError_t e;
  switch (lm_batch_tile(a.cols, a.tokens)) {
    case 8: e = launch_lm_logits_batch<8>(a, cfg); break;
    case 4: e = launch_lm_logits_batch<4>(a, cfg); break;
    case 2: e = launch_lm_logits_batch<2>(a, cfg); break;
    default: e = launch_lm_logits_batch<1>(a, cfg); break;
  }
  if (e != cudaSuccess) return e;
  cfg.numAttrs = pdl ? 1 : 0;
  cfg.blockDim = dim3(1024);
  cfg.gridDim = dim3(unsigned((a.rows + kLmCollectRows - 1) / kLmCollectRows), a.tokens);
  cfg.dynamicSmemBytes = 0;
  if ((e = cudaLaunchKernelEx(&cfg, lm_collect_kernel, a)) != cudaSuccess) return e;
  cfg.blockDim = dim3(256);
  cfg.gridDim = dim3(a.tokens);
  cfg.dynamicSmemBytes = size_t(kLmSelCap) * 8 + 2 * (kLmMaxK + 1) * 4;
  if ((e = ensure_smem(lm_select_kernel, cfg.dynamicSmemBytes)) != cudaSuccess) return e;
  return cudaLaunchKernelEx(&cfg, lm_select_kernel, a);
}

}  // namespace wh
