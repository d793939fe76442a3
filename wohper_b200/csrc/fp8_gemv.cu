// fp8_gemv.cu -- FP8 E4M3 x UE8M0(128x128) GEMV / batched GEMV for sm_100a.
//
// Replaces gemv_fp8_e4m3_ue8m0_{tensorwise,rows,rows_multi}
// (engine/zc_infer_core/src/compute.rs:6174-6577).  Every output equals the
// reference's AVX2 row kernel fp8_ue8m0_dot_row_avx2 (src/compute.rs:5977-6018)
// bit for bit: per 128-column group, 16 FMA chains of 8 steps (g0 lanes j over
// columns 16c+j, g1 lanes over 16c+8+j), P_j = g0_j + g1_j,
// acc_j = fma(P_j, scale_g, acc_j) over the groups in order, then the pairwise
// 8-lane sum.  The batched form keeps the same per-(row,input) arithmetic, so
// it is batch-invariant like the reference's rows_multi.
//
// Layout / data movement (fast path, col_group == 128):
//   * one CTA per block of <= 32 rows (block size chosen so the grid covers
//     the SMs once); a producer warp streams [rows x 128 B] boxes of W with TMA
//     (SWIZZLE_128B) through an 8-stage mbarrier ring; the swizzle makes the
//     consumers' row-per-lane reads bank-conflict free;
//   * 4 lanes per row, each owning 4 of the 16 chains (4 bytes per 16-byte
//     chunk), so a warp covers 8 rows; x sits in shared memory (optionally
//     act-quantised in the prologue) and is read as broadcast float4s;
//   * E4M3 -> f16x2 by the hardware converter, f16 -> f32, fma.rn.f32x2.
//     0x7F/0xFF (the reference's +-480, NaN for the hardware) make the row
//     non-finite; such rows are recomputed with the exact bit decoder.
// Shapes the fast path does not cover (col_group != 128, cols % 16 != 0) run
// fp8_gemv_generic_kernel, one thread per (row, input), same arithmetic.
#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace wh {

// The input of the rows from `row0` on (grouped mode: the group row0 lies in).
__device__ __forceinline__ const float* fp8_x_rows(const Fp8GemvArgs& a, int row0) {
  return a.x_group_rows ? a.x + (long long)(row0 / a.x_group_rows) * a.x_group_off : a.x;
}


__constant__ ActQuantTable c_aq;

cudaError_t ensure_smem_attr(const void* kernel, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, size_t> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> g(mu);
  auto key = std::make_pair(dev, kernel);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) done[key] = bytes;
  return e;
}

void set_act_quant_table(const ActQuantTable& t, cudaStream_t s) {
  cudaMemcpyToSymbolAsync(c_aq, &t, sizeof(t), 0, cudaMemcpyHostToDevice, s);
}
const ActQuantTable* act_quant_table_device() {
  void* p = nullptr;
  cudaGetSymbolAddress(&p, c_aq);
  return reinterpret_cast<const ActQuantTable*>(p);
}

// Block-wise act quant-dequant of a shared-memory vector, by one warp per
// block of `block` values (block <= 64*8).  Exact reference semantics.
__device__ void act_quant_smem_warp(float* v, int n, int block, int warp, int nwarps, int lane,
                                    const ActQuantTable* tab) {
  for (int b0 = warp * block; b0 < n; b0 += nwarps * block) {
    int b1 = min(n, b0 + block);
    float amax = 0.0f;
    for (int i = b0 + lane; i < b1; i += 32) amax = fmaxf(amax, fabsf(v[i]));
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    amax = fmaxf(amax, 1.0e-4f);
    float q = __fdiv_rn(amax, 448.0f);
    float scale = exp2i(ceil_log2f_ref(q, tab));
    for (int i = b0 + lane; i < b1; i += 32) {
      float t = __fdiv_rn(v[i], scale);
      t = t < -448.0f ? -448.0f : t;
      t = t > 448.0f ? 448.0f : t;
      v[i] = __fmul_rn(e4m3_nearest_ties_lower(t), scale);
    }
  }
}

// Standalone in-place act quant (fp8_act_quant_dequant_in_place).
__global__ void act_quant_kernel(float* v, long long n, int block, uint32_t* status) {
  int lane = threadIdx.x & 31;
  long long warp = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  pdl_wait_prior();
  for (long long b0 = warp * block; b0 < n; b0 += nw * block) {
    long long b1 = b0 + block < n ? b0 + block : n;
    float amax = 0.0f;
    for (long long i = b0 + lane; i < b1; i += 32) amax = fmaxf(amax, fabsf(v[i]));
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    amax = fmaxf(amax, 1.0e-4f);
    float scale = exp2i(ceil_log2f_ref(__fdiv_rn(amax, 448.0f), &c_aq));
    for (long long i = b0 + lane; i < b1; i += 32) {
      float t = __fdiv_rn(v[i], scale);
      t = t < -448.0f ? -448.0f : t;
      t = t > 448.0f ? 448.0f : t;
      v[i] = __fmul_rn(e4m3_nearest_ties_lower(t), scale);
    }
  }
  pdl_launch_dependents();
}

// Exact scalar restatement of fp8_ue8m0_dot_row_avx2 for one (row, input),
// used by the generic kernel and for the rare non-finite recompute.
__device__ float fp8_row_dot_exact(const uint8_t* __restrict__ w, const uint8_t* __restrict__ srow,
                                   int scale_cols, int col_group, const float* __restrict__ x) {
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  float tail = 0.0f;
  const int chunks = col_group / 16;
  for (int g = 0; g < scale_cols; ++g) {
    float scale = decode_ue8m0(srow[g]);
    const uint8_t* bytes = w + (long long)g * col_group;
    const float* cols = x + (long long)g * col_group;
    float g0[8], g1[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) g0[j] = g1[j] = 0.0f;
    for (int c = 0; c < chunks; ++c) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        g0[j] = fmaf(decode_fp8_exact(bytes[16 * c + j]), cols[16 * c + j], g0[j]);
        g1[j] = fmaf(decode_fp8_exact(bytes[16 * c + 8 + j]), cols[16 * c + 8 + j], g1[j]);
      }
    }
    float rem = 0.0f;
    for (int i = chunks * 16; i < col_group; ++i)
      rem = __fadd_rn(rem, __fmul_rn(decode_fp8_exact(bytes[i]), cols[i]));
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = fmaf(__fadd_rn(g0[j], g1[j]), scale, acc[j]);
    tail = __fadd_rn(tail, __fmul_rn(rem, scale));
  }
  float h = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3])),
                      __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7])));
  return __fadd_rn(h, tail);
}

__global__ void fp8_gemv_generic_kernel(Fp8GemvArgs a) {
  pdl_wait_prior();
  long long n = (long long)(a.row_end - a.row_start) * a.batch;
  const int row_group = a.rows / a.scale_rows;
  const int col_group = a.cols / a.scale_cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    int b = int(i / (a.row_end - a.row_start));
    int r = a.row_start + int(i % (a.row_end - a.row_start));
    const uint8_t* w = a.weight + (long long)r * a.cols;
    const uint8_t* s = a.scale + (long long)(r / row_group) * a.scale_cols;
    float acc = fp8_row_dot_exact(w, s, a.scale_cols, col_group,
                                  fp8_x_rows(a, r) + (long long)b * a.ldx);
    if (!isfinite(acc)) flag(a.status, WH_DEV_NONFINITE);
    const long long o = (long long)b * a.ldy + (r - a.row_start);
    a.y[o] = a.addend ? __fadd_rn(acc, a.addend[o]) : acc;
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// Fast path
// ---------------------------------------------------------------------------
constexpr int kFp8StageBytes = 32 * 128;  // up to 32 rows x 128 B, 1024-aligned
constexpr int kFp8MaxStages = 48;
constexpr size_t kFp8SmemBudget = 200 * 1024;


// ---------------------------------------------------------------------------
// Batched path (2..N inputs): the inputs stream with the weights.  Each ring
// stage holds one 128-column group: the weight box [32 rows][128 B] (TMA) and
// the group's 128 columns of each of the tile's TB inputs (one 512-byte bulk
// copy per input), so nothing is staged before the first group and a CTA
// holds 4 stages.  Lane mapping as fp8_gemv_tma_kernel (8 lanes per row, lane
// q the chains 2(q&3), 2(q&3)+1 of g0 or g1); the row's weights of a group
// are decoded once and applied to the TB inputs.  Inputs are act-quantised
// beforehand when the call asks for it.
// ---------------------------------------------------------------------------
constexpr int kFbStages = 4;
constexpr int kFbTB = 16;                           // inputs per CTA
constexpr int kFbStageBytes = 4096 + kFbTB * 512;   // weight box + x tile
constexpr int kFbThreads = 32 * (8 + 1);            // 8 consumer warps + producer

size_t fp8_gemv_batch_smem_bytes(int scale_cols) {
  return 1024 + (size_t)kFbStages * kFbStageBytes + 2 * kFbStages * 8 + 32 * (size_t)scale_cols +
         64;
}

__global__ void __launch_bounds__(kFbThreads) fp8_gemv_batch_kernel(
    const __grid_constant__ CUtensorMap wmap, Fp8GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kFbStages * kFbStageBytes);
  uint64_t* empty = full + kFbStages;
  uint8_t* scale_s = reinterpret_cast<uint8_t*>(empty + kFbStages);  // CTA's scale rows

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int box_rows = a.box_rows;  // <= 32
  const int row0 = a.row_start + blockIdx.x * box_rows;
  const int ngroups = a.scale_cols;
  const int tile = blockIdx.y;
  const int tb = min(kFbTB, a.batch - tile * kFbTB);
  const float* xbase = fp8_x_rows(a, row0) + (long long)tile * kFbTB * a.ldx;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFbStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 8) {
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      pdl_wait_prior();  // the inputs may come from the previous kernel
      int g = 0;
      for (; g < ngroups; ++g) {
        const int s = g % kFbStages;
        if (g >= kFbStages && !mbar_wait(&empty[s], ((g / kFbStages) - 1) & 1, a.status)) break;
        uint8_t* st = stages + s * kFbStageBytes;
        mbar_arrive_expect_tx(&full[s], box_rows * 128 + tb * 512);
        tma_load_2d(st, &wmap, &full[s], g * 128, row0);
        for (int b = 0; b < tb; ++b)
          bulk_load(st + 4096 + b * 512, xbase + (long long)b * a.ldx + g * 128, 512, &full[s]);
      }
      for (int i = max(0, g - kFbStages); i < g; ++i)
        if (!mbar_drain(&full[i % kFbStages], (i / kFbStages) & 1, a.status)) break;
    }
    return;
  }

  const int row_group = a.rows / a.scale_rows;
  const int last_row = min(row0 + box_rows, a.row_end) - 1;
  const int srow0 = row0 / row_group;
  const int nsrows = last_row / row_group - srow0 + 1;
  for (int i = threadIdx.x; i < nsrows * a.scale_cols; i += 256)
    scale_s[i] = a.scale[(long long)srow0 * a.scale_cols + i];
  asm volatile("bar.sync 1, 256;" ::: "memory");

  const int rloc = warp * 4 + (lane >> 3);  // row within the box
  const int q = lane & 7;
  const int row = row0 + rloc;
  const bool active = rloc < box_rows && row < a.row_end;
  const uint8_t* srow_s = scale_s + ((active ? row : row0) / row_group - srow0) * a.scale_cols;
  // the lane's two columns within each 16-column chunk
  const int cofs = (q < 4 ? 0 : 8) + 2 * (q & 3);

  float2 acc[kFbTB];
#pragma unroll
  for (int b = 0; b < kFbTB; ++b) acc[b] = make_float2(0.0f, 0.0f);
  bool ok = true;
  for (int g = 0; g < ngroups; ++g) {
    const int s = g % kFbStages;
    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (g / kFbStages) & 1, a.status))) {
      ok = false;
      break;
    }
    const uint8_t* st = stages + s * kFbStageBytes;
    float2 wf[8];
#pragma unroll
    for (int c = 0; c < 8; ++c)
        wf[c] = h2_to_f2(e4m3x2_to_f16x2(
          *reinterpret_cast<const uint16_t*>(st + rloc * 128 + 16 * (c ^ (rloc & 7)) + cofs)));
    const float scale = decode_ue8m0(srow_s[g]);
    const float2 sc = make_float2(scale, scale);
    const float* xt = reinterpret_cast<const float*>(st + 4096) + cofs;
#pragma unroll
    for (int b = 0; b < kFbTB; ++b) {
      if (b < tb) {
        float2 pj = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          pj = ffma2(wf[c], *reinterpret_cast<const float2*>(xt + b * 128 + 16 * c), pj);
        // P_j = g0_j + g1_j: lanes q and q ^ 4 hold g0 / g1 of the same j
        float2 o;
        o.x = __shfl_xor_sync(0xffffffffu, pj.x, 4);
        o.y = __shfl_xor_sync(0xffffffffu, pj.y, 4);
        acc[b] = ffma2(fadd2(pj, o), sc, acc[b]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (!ok) return;
  const uint8_t* srow = a.scale + (long long)((active ? row : a.row_start) / row_group) * a.scale_cols;
#pragma unroll
  for (int b = 0; b < kFbTB; ++b) {
    if (b < tb) {
      // hsum256: ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7))
      const float s2 = __fadd_rn(acc[b].x, acc[b].y);
      const float s4 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, 1));
      const float s8 = __fadd_rn(s4, __shfl_xor_sync(0xffffffffu, s4, 2));
      if (q == 0 && active) {
        float tot = __fadd_rn(s8, 0.0f);
        const int bi = tile * kFbTB + b;
        if (!isfinite(tot)) {
          // 0x7F/0xFF bytes (or a genuine overflow): exact recompute
          tot = fp8_row_dot_exact(a.weight + (long long)row * a.cols, srow, a.scale_cols, 128,
                                  xbase + (long long)b * a.ldx);
          if (!isfinite(tot)) flag(a.status, WH_DEV_NONFINITE);
        }
        const long long o = (long long)bi * a.ldy + (row - a.row_start);
        a.y[o] = a.addend ? __fadd_rn(tot, a.addend[o]) : tot;
      }
    }
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// One-input fast path: lane = row, warp = column group.
//
// The reference's g0/g1 chains restart at every 128-column group, so a
// (row, group) pair is an independent unit of 16 chains x 8 FMAs; only
// acc_j = fma(P_j, scale_g, acc_j) runs across the groups.  Phase 1 gives each
// lane one row of the tile and each warp a column group: the lane runs all 16
// chains of its (row, group) with the group's x read as shared-memory
// broadcasts and its weight row read as 16-byte words (bank-conflict free
// under the 128-byte swizzle), and stores P_j = g0_j + g1_j.  Eight chain
// warps give each (row, j) a thread that runs the acc_j chain over the groups
// in order, each group as soon as its P_j are stored (one mbarrier per group),
// so the chain runs under the weight stream; then the pairwise 8-lane sum.
// Same arithmetic as fp8_gemv_tma_kernel.
// ---------------------------------------------------------------------------
constexpr int kRgConsumers = 8;   // phase-1 warps
constexpr int kRgRing = 12;       // weight stages in flight per CTA
constexpr int kRgMaxGroups = 64;  // cols <= 8192
constexpr int kRgThreads = 32 * (kRgConsumers + 1);

static int fp8_rg_stages(int cols) {
  const int ngroups = cols / 128;
  if (ngroups > kRgMaxGroups) return 0;
  long long room = (long long)kFp8SmemBudget - 1024 - (long long)cols * 4 -
                   (long long)ngroups * 32 * 8 * 4 - (2 * kFp8MaxStages + kRgMaxGroups) * 8 -
                   (32LL * ngroups + 16);
  int ns = (int)std::max(0LL, room / kFp8StageBytes);
  return std::min({ns, kRgRing, ngroups});
}

size_t fp8_gemv_rg_smem_bytes(int cols) {
  const int ns = fp8_rg_stages(cols);
  if (ns < 4) return size_t(1) << 30;
  const int ngroups = cols / 128;
  return 1024 + size_t(ns) * kFp8StageBytes +
         (2 * kFp8MaxStages + kRgMaxGroups) * sizeof(uint64_t) + size_t(cols) * sizeof(float) +
         size_t(ngroups) * 32 * 8 * sizeof(float) + size_t(32) * ngroups + 16;
}

__global__ void __launch_bounds__(kRgThreads)
    fp8_gemv_rowgroup_kernel(const __grid_constant__ CUtensorMap wmap, Fp8GemvArgs a,
                             int nstages) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + nstages * kFp8StageBytes);
  uint64_t* empty = full + kFp8MaxStages;
  float* xs = reinterpret_cast<float*>(empty + kFp8MaxStages + kRgMaxGroups);  // cols
  const int ngroups = a.scale_cols;                               // col_group == 128
  float* ps = xs + a.cols;                                        // [ngroups][32][8]
  uint8_t* scale_s = reinterpret_cast<uint8_t*>(ps + ngroups * 32 * 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int box_rows = a.box_rows;
  const int row0 = a.row_start + blockIdx.x * box_rows;
  // the next kernel in the stream may start now: it streams its own weights
  // while this one finishes (it waits for this grid before reading results)
  pdl_launch_dependents();

  // one barrier per thread: a single thread initialising them one after the
  // other delays the first TMA issue by about a microsecond
  {
    const int t = threadIdx.x;
    const bool ring = ngroups > nstages;  // empty barriers only when slots are reused
    if (t < nstages) mbar_init(&full[t], 1);
    else if (t < 2 * kFp8MaxStages && t - kFp8MaxStages < nstages && ring)
      mbar_init(&empty[t - kFp8MaxStages], 1);  // one warp consumes each group
    if (t < 2 * kFp8MaxStages) fence_barrier_init();
  }
  __syncthreads();

  if (warp == kRgConsumers) {
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      int g = 0, s = 0;
      uint32_t phase = 0;
      for (; g < ngroups; ++g) {
        if (g >= nstages && !mbar_wait(&empty[s], phase, a.status)) break;
        mbar_arrive_expect_tx(&full[s], box_rows * 128);
        tma_load_2d(stages + s * kFp8StageBytes, &wmap, &full[s], g * 128, row0);
        if (++s == nstages) {
          s = 0;
          if (g >= nstages) phase ^= 1u;
        }
      }
      for (int i = max(0, g - nstages); i < g; ++i)
        if (!mbar_drain(&full[i % nstages], (i / nstages) & 1, a.status)) break;
    }
    return;
  }

  constexpr int nthr = kRgConsumers * 32;
  const int row_group = a.rows / a.scale_rows;
  const int last_row = min(row0 + box_rows, a.row_end) - 1;
  const int srow0 = row0 / row_group;
  const int nsrows = last_row / row_group - srow0 + 1;
  // the UE8M0 scale rows of the box (used by the chains at the end)
  for (int i = threadIdx.x; i < nsrows * a.scale_cols; i += nthr)
    scale_s[i] = a.scale[(long long)srow0 * a.scale_cols + i];
  pdl_wait_prior();
  // x: when no act-quant block straddles a 128-column group, each warp stages
  // (and act-quantises) only the groups it computes, so phase 1 starts without
  // a CTA-wide barrier and the x loads overlap the weight stream
  const float4* x4 = reinterpret_cast<const float4*>(fp8_x_rows(a, row0));
  float4* xs4 = reinterpret_cast<float4*>(xs);
  const bool own_x = a.act_quant_block == 0 || 128 % a.act_quant_block == 0;
  if (own_x) {
    for (int g0 = warp; g0 < ngroups; g0 += 4 * kRgConsumers) {
      float4 v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (g0 + k * kRgConsumers < ngroups) v[k] = __ldg(x4 + (g0 + k * kRgConsumers) * 32 + lane);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (g0 + k * kRgConsumers < ngroups) xs4[(g0 + k * kRgConsumers) * 32 + lane] = v[k];
    }
  } else {
    const int n4 = a.cols / 4;
    for (int i0 = threadIdx.x; i0 < n4; i0 += 4 * nthr) {
      float4 v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (i0 + k * nthr < n4) v[k] = __ldg(x4 + i0 + k * nthr);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (i0 + k * nthr < n4) xs4[i0 + k * nthr] = v[k];
    }
  }
  if (own_x) {
    __syncwarp();
    if (a.act_quant_block > 0) {
      for (int g = warp; g < ngroups; g += kRgConsumers)
        act_quant_smem_warp(xs + g * 128, 128, a.act_quant_block, 0, 1, lane, &c_aq);
      __syncwarp();
    }
  } else {
    asm volatile("bar.sync 1, %0;" ::"r"(nthr));
    act_quant_smem_warp(xs, a.cols, a.act_quant_block, warp, kRgConsumers, lane, &c_aq);
    asm volatile("bar.sync 1, %0;" ::"r"(nthr));
  }

  // ---- phase 1: P_j of (row = lane, group) ----
  bool ok = true;
  const int r = lane;
  const bool has_row = r < box_rows;
  for (int g = warp; g < ngroups; g += kRgConsumers) {
    const int s = g % nstages;
    ok = ok && mbar_wait(&full[s], (uint32_t)((g / nstages) & 1), a.status);
    if (ok && has_row) {
      const uint8_t* wrow = stages + s * kFp8StageBytes + r * 128;
      const float4* xg = reinterpret_cast<const float4*>(xs + g * 128);
      float2 g0[4], g1[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) g0[k] = g1[k] = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 w = *reinterpret_cast<const uint4*>(wrow + 16 * (c ^ (r & 7)));
        const float4 x0 = xg[4 * c], x1 = xg[4 * c + 1], x2 = xg[4 * c + 2], x3 = xg[4 * c + 3];
        // bytes 0..7 (w.x, w.y): g0 chains j = 0..7; bytes 8..15: g1 chains
        g0[0] = ffma2(h2_to_f2(e4m3x2_to_f16x2(w.x)), make_float2(x0.x, x0.y), g0[0]);
        g0[1] = ffma2(h2_to_f2(e4m3x2_to_f16x2(w.x >> 16)), make_float2(x0.z, x0.w), g0[1]);
        g0[2] = ffma2(h2_to_f2(e4m3x2_to_f16x2(w.y)), make_float2(x1.x, x1.y), g0[2]);
        g0[3] = ffma2(h2_to_f2(e4m3x2_to_f16x2(w.y >> 16)), make_float2(x1.z, x1.w), g0[3]);
        g1[0] = ffma2(h2_to_f2(e4m3x2_to_f16x2(w.z)), make_float2(x2.x, x2.y), g1[0]);
        g1[1] = ffma2(h2_to_f2(e4m3x2_to_f16x2(w.z >> 16)), make_float2(x2.z, x2.w), g1[1]);
        g1[2] = ffma2(h2_to_f2(e4m3x2_to_f16x2(w.w)), make_float2(x3.x, x3.y), g1[2]);
        g1[3] = ffma2(h2_to_f2(e4m3x2_to_f16x2(w.w >> 16)), make_float2(x3.z, x3.w), g1[3]);
      }
      float4* pd = reinterpret_cast<float4*>(ps + (g * 32 + r) * 8);
      const float2 p0 = fadd2(g0[0], g1[0]), p1 = fadd2(g0[1], g1[1]);
      const float2 p2 = fadd2(g0[2], g1[2]), p3 = fadd2(g0[3], g1[3]);
      pd[0] = make_float4(p0.x, p0.y, p1.x, p1.y);
      pd[1] = make_float4(p2.x, p2.y, p3.x, p3.y);
    }
    // release the slot after the warp's weight loads (after a timed-out wait
    // the arrivals still come, so the producer never waits on a dead slot)
    __syncwarp();
    if (lane == 0 && ngroups > nstages) mbar_arrive(&empty[s]);
  }
  // ---- the chains: acc_j = fma(P_j, scale_g, acc_j) over the groups in
  // order, one consumer thread per (row, j), once every P_j is stored ----
  const int ok_all = bar_and(1, nthr, ok);
  const int t = threadIdx.x;
  const int rr = t >> 3, j = t & 7;
  const int row = row0 + rr;
  const bool active = rr < box_rows && row < a.row_end;
  const uint8_t* srow_s = scale_s + ((active ? row : row0) / row_group - srow0) * a.scale_cols;
  const float* pj = ps + rr * 8 + j;
  float acc = 0.0f;
  if (active && ok_all) {
#pragma unroll 4
    for (int g = 0; g < ngroups; ++g) acc = fmaf(pj[g * 256], decode_ue8m0(srow_s[g]), acc);
  }
  // hsum256: ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7))
  const float s2 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
  const float s4 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, 2));
  const float s8 = __fadd_rn(s4, __shfl_xor_sync(0xffffffffu, s4, 4));
  if (j == 0 && active && ok_all) {
    float tot = __fadd_rn(s8, 0.0f);
    if (!isfinite(tot)) {
      // 0x7F/0xFF bytes (or a genuine overflow): exact recompute
      const uint8_t* srow = a.scale + (long long)(row / row_group) * a.scale_cols;
      tot = fp8_row_dot_exact(a.weight + (long long)row * a.cols, srow, a.scale_cols, 128, xs);
      if (!isfinite(tot)) flag(a.status, WH_DEV_NONFINITE);
    }
    a.y[row - a.row_start] = a.addend ? __fadd_rn(tot, a.addend[row - a.row_start]) : tot;
  }
}

static size_t fp8_scale_smem(int cols) { return size_t(32) * (cols / 128) + 16; }


cudaError_t launch_fp8_gemv(const CUtensorMap* wmap, const Fp8GemvArgs& a, int num_sms,
                            cudaStream_t stream, bool pdl) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (wmap == nullptr) {
    long long n = (long long)(a.row_end - a.row_start) * a.batch;
    cfg.blockDim = dim3(128);
    cfg.gridDim = dim3((unsigned)std::min<long long>((n + 127) / 128, 4LL * num_sms));
    cfg.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&cfg, fp8_gemv_generic_kernel, a);
  }
  const int nrows = a.row_end - a.row_start;
  if (a.batch == 1 && a.ldx >= a.cols && fp8_gemv_rg_smem_bytes(a.cols) <= kFp8SmemBudget + 1024) {
    const int ns = fp8_rg_stages(a.cols);
    cfg.blockDim = dim3(kRgThreads);
    cfg.gridDim = dim3((nrows + a.box_rows - 1) / a.box_rows);
    cfg.dynamicSmemBytes = fp8_gemv_rg_smem_bytes(a.cols);
    cudaError_t e = ensure_smem(fp8_gemv_rowgroup_kernel, cfg.dynamicSmemBytes);
    if (e != cudaSuccess) return e;
    return cudaLaunchKernelEx(&cfg, fp8_gemv_rowgroup_kernel, *wmap, a, ns);
  }
  // 2..N inputs: the streaming batched kernel, kFbTB inputs per CTA
  cfg.blockDim = dim3(kFbThreads);
  cfg.gridDim = dim3((nrows + a.box_rows - 1) / a.box_rows, (a.batch + kFbTB - 1) / kFbTB);
  cfg.dynamicSmemBytes = fp8_gemv_batch_smem_bytes(a.scale_cols);
  cudaError_t e = ensure_smem(fp8_gemv_batch_kernel, cfg.dynamicSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaLaunchKernelEx(&cfg, fp8_gemv_batch_kernel, *wmap, a);
}

cudaError_t launch_act_quant(float* v, long long n, int block, uint32_t* status, int num_sms,
                             cudaStream_t stream) {
  long long blocks = (n + block - 1) / block;
  long long warps = std::min<long long>(blocks, 8LL * num_sms * 4);
  unsigned grid = (unsigned)std::max<long long>(1, (warps + 3) / 4);
  act_quant_kernel<<<grid, 128, 0, stream>>>(v, n, block, status);
  return cudaGetLastError();
}

}  // namespace wh
