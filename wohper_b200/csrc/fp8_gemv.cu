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
//   * one CTA per box of <= 32 rows (box height chosen so the grid covers the
//     SMs once); a producer warp streams [rows x 128 B] boxes of W with TMA
//     (SWIZZLE_128B) through an mbarrier ring; the swizzle makes the
//     consumers' row-per-lane reads bank-conflict free;
//   * one input: fp8_gemv_rowgroup_kernel, a lane per row and a warp per
//     column group, x staged (and act-quantised) in shared memory;
//   * 2..N inputs: fp8_gemv_batch_kernel, the inputs streamed with the
//     weights, 8 lanes per row, the decoded weights applied to 16 inputs;
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

// the same thresholds in global memory, for kernels that stage them in shared
// memory with one coalesced load (a constant-bank read with 256 distinct
// indices per warp would serialise)
__device__ ActQuantTable g_aq;

void set_act_quant_table(const ActQuantTable& t, cudaStream_t s) {
  cudaMemcpyToSymbolAsync(c_aq, &t, sizeof(t), 0, cudaMemcpyHostToDevice, s);
  cudaMemcpyToSymbolAsync(g_aq, &t, sizeof(t), 0, cudaMemcpyHostToDevice, s);
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
    const AqScale sc = aq_block_scale(amax, tab->thr);
    for (int i = b0 + lane; i < b1; i += 32) v[i] = aq_value(v[i], sc);
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
    const AqScale sc = aq_block_scale(amax, c_aq.thr);
    for (long long i = b0 + lane; i < b1; i += 32) v[i] = aq_value(v[i], sc);
  }
  pdl_launch_dependents();
}

// Exact scalar restatement of fp8_ue8m0_dot_row_avx2 for one (row, input),
// used by the generic kernel and for the rare non-finite recompute.
// x_pad: floats of padding after every 8 groups of x (the one-input kernel's
// shared-memory layout), 0 for a plain vector.
__device__ float fp8_row_dot_exact(const uint8_t* __restrict__ w, const uint8_t* __restrict__ srow,
                                   int scale_cols, int col_group, const float* __restrict__ x,
                                   int x_pad = 0) {
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  float tail = 0.0f;
  const int chunks = col_group / 16;
  for (int g = 0; g < scale_cols; ++g) {
    float scale = decode_ue8m0(srow[g]);
    const uint8_t* bytes = w + (long long)g * col_group;
    const float* cols = x + (long long)g * col_group + (g >> 3) * x_pad;
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
constexpr size_t kFp8SmemBudget = 200 * 1024;


// ---------------------------------------------------------------------------
// Batched path (2..N inputs): a CTA takes a box of up to 32 rows and a tile of
// 16 inputs; per 128-column group one ring stage holds the weight box
// [rows][128 B] (TMA, 128-byte swizzle) and the x tile [16 inputs][136 floats]
// (TMA from a [batch][cols] map: the 8 floats past the group pad every input
// row onto other banks, and are never read).
//
// A group of 4 lanes (a quad) owns 2 rows x 4 inputs; lane q of the quad holds
// the chains 2q and 2q+1 of both halves (g0: columns 16c + 2q, +1; g1:
// 16c + 8 + 2q, +1) as f32 pairs, so P_j = g0_j + g1_j is local and the
// reference's acc_j = fma(P_j, scale, acc_j) follows once per group.  Each
// weight pair is decoded once and used for 4 inputs; each x pair is read once
// and used for 2 rows.  The pairwise 8-lane sum of the end is two shuffles
// inside the quad.  Inputs are act-quantised beforehand when the call asks.
// ---------------------------------------------------------------------------
constexpr int kFbStages = 4;
constexpr int kFbTB = 16;                           // inputs per CTA
constexpr int kFbXStride = 136;                     // floats per input row of a stage
constexpr int kFbXBytes = kFbTB * kFbXStride * 4;   // 8704
constexpr int kFbStageBytes = 13 * 1024;            // weight box (4 KB) + x tile, 1 KiB multiple
constexpr int kFbThreads = 32 * (8 + 1);            // 8 consumer warps + producer

size_t fp8_gemv_batch_smem_bytes(int scale_cols) {
  return 1024 + (size_t)kFbStages * kFbStageBytes + 2 * kFbStages * 8 + 32 * (size_t)scale_cols +
         64;
}

__global__ void __launch_bounds__(kFbThreads, 2) fp8_gemv_batch_kernel(
    const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
    Fp8GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kFbStages * kFbStageBytes);
  uint64_t* empty = full + kFbStages;
  uint8_t* scale_s = reinterpret_cast<uint8_t*>(empty + kFbStages);  // the box's scale rows

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int box_rows = a.box_rows;  // <= 32
  const int tile = blockIdx.x;      // inputs [16 tile, 16 tile + 16): neighbours share weights
  const int row0 = a.row_start + blockIdx.y * box_rows;
  const int ngroups = a.scale_cols;
  // grouped mode: the box's rows read their group's slice of every input
  const int xcol0 = a.x_group_rows ? (int)((row0 / a.x_group_rows) * a.x_group_off) : 0;
  // the next kernel may start its weight stream now (it waits for this grid
  // before reading y)
  pdl_launch_dependents();

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
      prefetch_tensormap(&xmap);
      const uint32_t stage_tx = box_rows * 128 + kFbXBytes;
      // the first stages' weights do not depend on the previous kernel
      const int pre = min(ngroups, kFbStages);
      for (int g = 0; g < pre; ++g) {
        mbar_arrive_expect_tx(&full[g], stage_tx);
        tma_load_2d(stages + g * kFbStageBytes, &wmap, &full[g], g * 128, row0);
      }
      pdl_wait_prior();  // the inputs may come from the previous kernel
      for (int g = 0; g < pre; ++g)
        tma_load_2d(stages + g * kFbStageBytes + 4096, &xmap, &full[g], xcol0 + g * 128,
                    tile * kFbTB);
      int g = pre, s = 0;
      uint32_t phase = 0;
      for (; g < ngroups; ++g) {
        if (!mbar_wait(&empty[s], phase, a.status)) break;  // slot of group g - kFbStages
        uint8_t* st = stages + s * kFbStageBytes;
        mbar_arrive_expect_tx(&full[s], stage_tx);
        tma_load_2d(st, &wmap, &full[s], g * 128, row0);
        tma_load_2d(st + 4096, &xmap, &full[s], xcol0 + g * 128, tile * kFbTB);
        if (++s == kFbStages) {
          s = 0;
          phase ^= 1u;
        }
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

  const int quad = lane >> 2, q = lane & 3;
  const int rl0 = warp * 4 + (quad >> 2) * 2;  // the quad's two rows within the box
  const int ig = quad & 3;                      // its inputs: ig + 4m, m = 0..3
  const uint8_t* srow_s[2];
  bool rvalid[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int row = row0 + rl0 + k;
    rvalid[k] = rl0 + k < box_rows && row < a.row_end;
    srow_s[k] = scale_s + ((rvalid[k] ? row : row0) / row_group - srow0) * a.scale_cols;
  }
  const int tb = min(kFbTB, a.batch - tile * kFbTB);

  float2 acc[2][4];
#pragma unroll
  for (int k = 0; k < 2; ++k)
#pragma unroll
    for (int m = 0; m < 4; ++m) acc[k][m] = make_float2(0.0f, 0.0f);
  bool ok = true;
  int s = 0;
  uint32_t phase = 0;
  for (int g = 0; g < ngroups; ++g) {
    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], phase, a.status))) {
      ok = false;
      break;
    }
    const uint8_t* wst = stages + s * kFbStageBytes;
    const float* xst = reinterpret_cast<const float*>(wst + 4096) + ig * kFbXStride + 2 * q;
    float2 g0[2][4], g1[2][4];
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
      for (int m = 0; m < 4; ++m) g0[k][m] = g1[k][m] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float2 w0[2], w1[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int r = rl0 + k;
        const uint4 ch = *reinterpret_cast<const uint4*>(wst + r * 128 + 16 * (c ^ (r & 7)));
        // bytes 2q, 2q+1 (g0) and 8 + 2q, 9 + 2q (g1) of the 16-column chunk
        const uint32_t lo = (q >> 1) ? ch.y : ch.x, hi = (q >> 1) ? ch.w : ch.z;
        const int sh = 16 * (q & 1);
        w0[k] = h2_to_f2(e4m3x2_to_f16x2(lo >> sh));
        w1[k] = h2_to_f2(e4m3x2_to_f16x2(hi >> sh));
      }
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float* xp = xst + 4 * m * kFbXStride + 16 * c;
        const float2 x0 = *reinterpret_cast<const float2*>(xp);
        const float2 x1 = *reinterpret_cast<const float2*>(xp + 8);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          g0[k][m] = ffma2(w0[k], x0, g0[k][m]);
          g1[k][m] = ffma2(w1[k], x1, g1[k][m]);
        }
      }
    }
    // release the slot after the warp's reads of it
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float sc = decode_ue8m0(srow_s[k][g]);
      const float2 sc2 = make_float2(sc, sc);
#pragma unroll
      for (int m = 0; m < 4; ++m) acc[k][m] = ffma2(fadd2(g0[k][m], g1[k][m]), sc2, acc[k][m]);
    }
    if (++s == kFbStages) {
      s = 0;
      phase ^= 1u;
    }
  }
  if (!ok) return;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int row = row0 + rl0 + k;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      // hsum256: ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7)); lane q holds
      // a_2q, a_2q+1
      const float s2 = __fadd_rn(acc[k][m].x, acc[k][m].y);
      const float s4 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, 1));
      const float s8 = __fadd_rn(s4, __shfl_xor_sync(0xffffffffu, s4, 2));
      const int b = ig + 4 * m;
      if (q == 0 && rvalid[k] && b < tb) {
        float tot = __fadd_rn(s8, 0.0f);
        const int bi = tile * kFbTB + b;
        if (!isfinite(tot)) {
          // 0x7F/0xFF bytes (or a genuine overflow): exact recompute
          const uint8_t* srow = a.scale + (long long)(row / row_group) * a.scale_cols;
          tot = fp8_row_dot_exact(a.weight + (long long)row * a.cols, srow, a.scale_cols, 128,
                                  fp8_x_rows(a, row) + (long long)bi * a.ldx);
          if (!isfinite(tot)) flag(a.status, WH_DEV_NONFINITE);
        }
        const long long o = (long long)bi * a.ldy + (row - a.row_start);
        a.y[o] = a.addend ? __fadd_rn(tot, a.addend[o]) : tot;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// One-input fast path: lanes = rows, warps = column groups.
//
// The reference's g0/g1 chains restart at every 128-column group, so a
// (row, group) pair is an independent unit of 16 chains x 8 FMAs; only
// acc_j = fma(P_j, scale_g, acc_j) runs across the groups.  Phase 1 gives each
// warp every 8th column group and each lane one (row, group) pair of the
// CTA's box of rows: the lane runs all 16 chains with the group's x read as
// shared-memory broadcasts and its weight row read as 16-byte words
// (bank-conflict free under the 128-byte swizzle), and stores
// P_j = g0_j + g1_j.  A box of R <= 16 rows puts 32/R groups side by side in
// the warp (R rounded up to a power of two), so short boxes keep the lanes
// busy.  After a barrier each (row, j) thread runs its acc_j chain over the
// groups in order, then the pairwise 8-lane sum.
//
// Each group has its own full barrier, so a consumer waits for exactly its
// group's copy whatever order the copies land in (ring slots are reused by
// groups that other warps consume).
//
// At decode sizes latency, not arithmetic, bounds this kernel, so:
//   * a ring slot is the box rounded up to 1 KiB (the 128-byte swizzle repeats
//     every 1 KiB), so a short box keeps more groups in flight.  The ring is
//     sized for two CTAs per SM when that leaves at least 8 slots (the next
//     kernel's CTAs then issue their weight loads while this one finishes),
//     else one CTA per SM takes a deeper ring;
//   * weights, scales and the act-quant thresholds do not depend on the
//     previous kernel: they are requested before the programmatic-dependency
//     wait, x after it;
//   * x is act-quantised in registers as it is loaded: a block of 4L values
//     spans L lanes of the warp, and a warp quantises 4 groups at once.
// Shared-memory x is padded by 4 floats after every 8 groups, so the groups a
// quarter-warp reads side by side (8 apart) sit in different banks.
// ---------------------------------------------------------------------------
constexpr int kRgConsumers = 8;   // phase-1 warps
constexpr int kRgMaxGroups = 64;  // cols <= 8192
constexpr int kRgXBatch = 4;      // x float4s a lane loads at once
constexpr int kRgThreads = 32 * (kRgConsumers + 1);
constexpr long long kRgTwoPerSm = 112 * 1024;  // dynamic smem per CTA with two CTAs per SM
constexpr int kRgMinRing = 8;
constexpr int kRgMaxRing = 64;
constexpr int kRgXPad = 4;

__host__ __device__ constexpr int fp8_rg_slot(int box_rows) {
  return ((box_rows * 128 + 1023) / 1024) * 1024;
}
__host__ __device__ constexpr int fp8_rg_xs_len(int ngroups) {
  return ngroups * 128 + ((ngroups + 7) / 8) * kRgXPad;
}
__host__ __device__ constexpr int fp8_rg_lane_rows(int box_rows) {  // power of two >= box_rows
  return box_rows <= 1 ? 1 : box_rows <= 2 ? 2 : box_rows <= 4 ? 4 : box_rows <= 8 ? 8
       : box_rows <= 16 ? 16 : 32;
}

// bytes besides the ring: alignment pad, barriers, x, P, thresholds, scale rows
static long long fp8_rg_fixed(int ngroups, int box_rows) {
  return 1024 + 2LL * kRgMaxGroups * 8 + 4LL * fp8_rg_xs_len(ngroups) +
         4LL * ngroups * box_rows * 8 + 256 * 4 + 32LL * ngroups + 16;
}

struct RgPlan {
  int ns;  // ring slots
  size_t smem;
};

static bool fp8_rg_plan(const Fp8GemvArgs& a, RgPlan* p) {
  const int ngroups = a.scale_cols, box = a.box_rows, aqb = a.act_quant_block;
  if (a.batch != 1 || a.ldx < a.cols || ngroups < 1 || ngroups > kRgMaxGroups ||
      a.cols != ngroups * 128 || box < 1 || box > 32)
    return false;
  if (aqb != 0 && (aqb < 4 || 128 % aqb != 0)) return false;  // quantised in registers
  const long long fixed = fp8_rg_fixed(ngroups, box);
  const int slot = fp8_rg_slot(box);
  // A warp waits for its 32/R side-by-side groups together before it frees
  // their slots, so the ring must hold one such pass of every warp: with
  // fewer slots a pass could wait for a copy that only a later pass frees.
  const int need = std::min(ngroups, kRgConsumers * (32 / fp8_rg_lane_rows(box)));
  const int two = (int)std::max(0LL, (kRgTwoPerSm - fixed) / slot);
  int ns = std::min(two, ngroups);
  if (two < std::max(need, std::min(ngroups, kRgMinRing)))
    ns = std::min((int)std::max(0LL, ((long long)kFp8SmemBudget - fixed) / slot), ngroups);
  ns = std::min(ns, kRgMaxRing);
  if (ns < std::max(need, std::min(ngroups, 4))) return false;
  p->ns = ns;
  p->smem = (size_t)(fixed + (long long)ns * slot);
  return true;
}

bool fp8_gemv_rowgroup_fits(const Fp8GemvArgs& a, int) {
  RgPlan p;
  return fp8_rg_plan(a, &p);
}

// Act quant-dequant of the float4 `v` a lane holds, in blocks of 4 * lanes
// values over aligned groups of `lanes` lanes (lanes a power of two <= 32).
__device__ __forceinline__ float4 act_quant_lanes(float4 v, int lanes, const uint32_t* thr) {
  // max|v| ignoring NaN (as the reference's f32::max): a NaN operand of fmaxf
  // yields the other one, and the 1e-4 floor comes after
  float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  for (int o = lanes >> 1; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const AqScale sc = aq_block_scale(m, thr);
  return make_float4(aq_value(v.x, sc), aq_value(v.y, sc), aq_value(v.z, sc), aq_value(v.w, sc));
}

// R: the box height rounded up to a power of two (lanes per group)
template <int R>
__global__ void __launch_bounds__(kRgThreads, 4)
    fp8_gemv_rowgroup_kernel(const __grid_constant__ CUtensorMap wmap, Fp8GemvArgs a,
                             int nstages) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  const int box_rows = a.box_rows;
  const int slot = fp8_rg_slot(box_rows);
  const int ngroups = a.scale_cols;  // col_group == 128
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + nstages * slot);  // [group]
  uint64_t* empty = full + kRgMaxGroups;                                 // [ring slot]
  float* xs = reinterpret_cast<float*>(empty + kRgMaxGroups);            // padded x
  float* ps = xs + fp8_rg_xs_len(ngroups);                               // [group][row][8]
  uint32_t* thr_s = reinterpret_cast<uint32_t*>(ps + ngroups * box_rows * 8);  // 256
  uint8_t* scale_s = reinterpret_cast<uint8_t*>(thr_s + 256);  // the box's scale rows

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = a.row_start + blockIdx.x * box_rows;
  // the next kernel in the stream may start now: it streams its own weights
  // while this one finishes (it waits for this grid before reading results)
  pdl_launch_dependents();

  // one barrier per thread: a single thread initialising them one after the
  // other delays the first TMA issue by about a microsecond
  {
    const int t = threadIdx.x;
    if (t < ngroups) mbar_init(&full[t], 1);
    else if (t >= kRgMaxGroups && t - kRgMaxGroups < nstages)
      mbar_init(&empty[t - kRgMaxGroups], 1);  // the lane group that read the slot
    if (t < 2 * kRgMaxGroups) fence_barrier_init();
  }
  __syncthreads();

  if (warp == kRgConsumers) {
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      // slot and phase advance without a division: the producer's turn
      // between a freed slot and the next copy is on the stream's critical path
      int g = 0, s = 0;
      uint32_t phase = 0;
      for (; g < ngroups; ++g) {
        if (g >= nstages && !mbar_wait(&empty[s], phase, a.status)) break;
        mbar_arrive_expect_tx(&full[g], box_rows * 128);
        tma_load_2d(stages + s * slot, &wmap, &full[g], g * 128, row0);
        if (++s == nstages) {
          s = 0;
          if (g >= nstages) phase ^= 1u;
        }
      }
      // the copies still in flight land before the CTA leaves
      for (int i = max(0, g - nstages); i < g; ++i)
        if (!mbar_drain(&full[i], 0, a.status)) break;
    }
    return;
  }

  constexpr int nthr = kRgConsumers * 32;
  const int t = threadIdx.x;
  const int aqb = a.act_quant_block;
  const int row_group = a.rows / a.scale_rows;
  const int srow0 = row0 / row_group;
  // constant inputs first: the act-quant thresholds (one per thread) and the
  // UE8M0 scale rows of the box (read by the chains)
  const uint32_t thr_v = aqb > 0 ? __ldg(&g_aq.thr[t]) : 0u;
  {
    const int nsr = (min(row0 + box_rows, a.row_end) - 1) / row_group - srow0 + 1;
    for (int i = t; i < nsr * ngroups; i += nthr)
      scale_s[i] = a.scale[(long long)srow0 * a.scale_cols + i];
  }
  pdl_wait_prior();

  // ---- x: each warp stages (and act-quantises) only the groups it computes ----
  const int jw = (ngroups - warp + kRgConsumers - 1) / kRgConsumers;  // this warp's groups
  {
    const float4* x4 = reinterpret_cast<const float4*>(fp8_x_rows(a, row0));
    float4* xs4 = reinterpret_cast<float4*>(xs);
    for (int j0 = 0; j0 < kRgMaxGroups / kRgConsumers; j0 += kRgXBatch) {
      if (j0 > 0 && j0 >= jw) break;  // the first batch runs in every warp (barrier)
      float4 v[kRgXBatch];
#pragma unroll
      for (int u = 0; u < kRgXBatch; ++u)
        if (j0 + u < jw) v[u] = __ldg(x4 + (warp + kRgConsumers * (j0 + u)) * 32 + lane);
      if (j0 == 0 && aqb > 0) {
        thr_s[t] = thr_v;
        asm volatile("bar.sync 2, %0;" ::"r"(nthr) : "memory");
      }
#pragma unroll
      for (int u = 0; u < kRgXBatch; ++u) {
        const int g = warp + kRgConsumers * (j0 + u);
        if (j0 + u < jw) {
          if (aqb > 0) v[u] = act_quant_lanes(v[u], aqb / 4, thr_s);
          xs4[(g * 128 + (g >> 3) * kRgXPad) / 4 + lane] = v[u];
        }
      }
    }
    __syncwarp();
  }

  // ---- phase 1: P_j of (row r, group g) ----
  constexpr int gpw = 32 / R;  // groups side by side in a warp
  const int r = lane & (R - 1), q = lane / R;
  bool ok = true;
  for (int j0 = 0; j0 < jw; j0 += gpw) {
    const int j = j0 + q;
    const bool has_g = j < jw;
    const int g = warp + kRgConsumers * j;
    const int s = g % nstages;
    bool landed = false;
    if (has_g) {
      ok = ok && mbar_wait(&full[g], 0, a.status);
      landed = ok;
    }
    if (landed && r < box_rows) {
      const uint8_t* wrow = stages + s * slot + r * 128;
      const float4* xg = reinterpret_cast<const float4*>(xs + g * 128 + (g >> 3) * kRgXPad);
      float2 g0[4], g1[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) g0[u] = g1[u] = make_float2(0.0f, 0.0f);
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
      float4* pd = reinterpret_cast<float4*>(ps + (g * box_rows + r) * 8);
      const float2 p0 = fadd2(g0[0], g1[0]), p1 = fadd2(g0[1], g1[1]);
      const float2 p2 = fadd2(g0[2], g1[2]), p3 = fadd2(g0[3], g1[3]);
      pd[0] = make_float4(p0.x, p0.y, p1.x, p1.y);
      pd[1] = make_float4(p2.x, p2.y, p3.x, p3.y);
    }
    // release the slot once the group's lanes have read it (after a timed-out
    // wait the arrivals still come, so the producer never waits on a dead slot)
    __syncwarp();
    if (has_g && r == 0) mbar_arrive(&empty[s]);
  }

  // ---- the chains: acc_j = fma(P_j, scale_g, acc_j) over the groups in
  // order, one consumer thread per (row, j), once every P_j is stored ----
  const int ok_all = bar_and(1, nthr, ok);
  const int rr = t >> 3, j8 = t & 7;
  const int row = row0 + rr;
  const bool active = rr < box_rows && row < a.row_end;
  const uint8_t* srow_s = scale_s + ((active ? row : row0) / row_group - srow0) * ngroups;
  const float* pj = ps + rr * 8 + j8;
  const int pstride = box_rows * 8;
  float acc = 0.0f;
  if (active && ok_all) {
#pragma unroll 4
    for (int g = 0; g < ngroups; ++g) acc = fmaf(pj[g * pstride], decode_ue8m0(srow_s[g]), acc);
  }
  // hsum256: ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7))
  const float s2 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
  const float s4 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, 2));
  const float s8 = __fadd_rn(s4, __shfl_xor_sync(0xffffffffu, s4, 4));
  if (j8 == 0 && active && ok_all) {
    float tot = __fadd_rn(s8, 0.0f);
    if (!isfinite(tot)) {
      // 0x7F/0xFF bytes (or a genuine overflow): exact recompute
      const uint8_t* srow = a.scale + (long long)(row / row_group) * a.scale_cols;
      tot = fp8_row_dot_exact(a.weight + (long long)row * a.cols, srow, a.scale_cols, 128, xs,
                              kRgXPad);
      if (!isfinite(tot)) flag(a.status, WH_DEV_NONFINITE);
    }
    a.y[row - a.row_start] = a.addend ? __fadd_rn(tot, a.addend[row - a.row_start]) : tot;
  }
}

cudaError_t launch_fp8_gemv(const CUtensorMap* wmap, const CUtensorMap* xmap,
                            const Fp8GemvArgs& a, int num_sms, cudaStream_t stream, bool pdl) {
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
  RgPlan p;
  if (fp8_rg_plan(a, &p)) {
    cfg.blockDim = dim3(kRgThreads);
    cfg.gridDim = dim3((nrows + a.box_rows - 1) / a.box_rows);
    cfg.dynamicSmemBytes = p.smem;
    auto* kern = fp8_gemv_rowgroup_kernel<32>;
    switch (fp8_rg_lane_rows(a.box_rows)) {
      case 1:
      case 2:
      case 4: kern = fp8_gemv_rowgroup_kernel<4>; break;
      case 8: kern = fp8_gemv_rowgroup_kernel<8>; break;
      case 16: kern = fp8_gemv_rowgroup_kernel<16>; break;
      default: break;
    }
    cudaError_t e = ensure_smem(kern, cfg.dynamicSmemBytes);
    if (e != cudaSuccess) return e;
    return cudaLaunchKernelEx(&cfg, kern, *wmap, a, p.ns);
  }
  // 2..N inputs: the batched kernel, 16 inputs x one row box per CTA; the
  // input tiles of a row box are neighbours in launch order (they read the
  // same weights)
  if (xmap == nullptr) return cudaErrorInvalidValue;
  cfg.blockDim = dim3(kFbThreads);
  cfg.gridDim = dim3((a.batch + kFbTB - 1) / kFbTB, (nrows + a.box_rows - 1) / a.box_rows);
  cfg.dynamicSmemBytes = fp8_gemv_batch_smem_bytes(a.scale_cols);
  cudaError_t e = ensure_smem(fp8_gemv_batch_kernel, cfg.dynamicSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaLaunchKernelEx(&cfg, fp8_gemv_batch_kernel, *wmap, *xmap, a);
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
