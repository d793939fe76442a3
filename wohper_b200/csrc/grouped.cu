// grouped.cu -- batched MoE FFN (many tokens) on the 5th-generation tensor
// cores: expert-major grouped GEMMs with block-scaled FP8 MMA.
//
// The reference processes a batch expert by expert, one matvec per
// (token, expert) row (accumulate_expert_for_positions, src/compute.rs:1779-1810;
// union in ascending expert id, src/server/generation.rs:2487-2569).  Here the
// rows of each expert are gathered into one contiguous block and every
// expert's w1/w3 and w2 run as GEMMs:
//
//   route (router_kernel) -> count + units -> dispatch (act quant of each token,
//   scattered to its 7 expert rows) -> grouped up GEMM (w1, w3, SwiGLU, act
//   quant of h) -> grouped down GEMM (w2) -> combine in ascending expert id.
//
// FP4 weights: the reference's E2M1 table has 0.125 at code 1, which the
// hardware's OCP E2M1 decode (0.5) does not match, but every value of it is
// exact in E4M3.  Converter warps therefore turn each FP4 tile into E4M3 in
// shared memory and the MMA is kind::mxf8f6f4 with UE8M0 scales: the weight's
// per-32 scale bytes as SFA, the activation's act-quant exponent as SFB.
// Products are exact; the accumulation order is the tensor core's, so results
// match the reference within floating-point tolerance (not bit for bit).
#include <cuda_fp8.h>

#include "tc.cuh"

namespace wh {

// Below this many tokens a call is decode-sized and takes the single-token
// (route-order) combine; from here on the batched (ascending expert id)
// combine.  The tile size is chosen apart from it (grouped_tile_n): 16 tokens
// while the routed experts average at most 4 rows, kGN beyond.
constexpr int kGroupedMinTokens = 32;
// K (hidden and inter) must be a multiple of 512: scale bytes are read 16 at a
// time (4 K tiles of 128)
// tokens per tile (MMA N) of batches: 112, not 128, so that two accumulator
// sets of both up matrices (2 x 2 x 112 columns) and the scale columns fit in
// TMEM's 512 columns
constexpr int kGN = 112;
constexpr int kGNSmall = 16;    // tokens per tile for decode-sized batches
// TMA ring depth (raw FP4 A + E4M3 B per K tile): deeper for the small tile,
// whose stages are smaller.  The 16-token up GEMM trades two TMA stages for a
// third converted-A slot (its converters wait less on the MMA); for the
// 112-token tiles a third slot measured no better.
template <bool kUp, int kN>
struct GRing {
  static constexpr int stages = kN <= 16 ? (kUp ? 6 : 8) : 4;
  static constexpr int conv = kN <= 16 && kUp ? 3 : 2;  // converted-A ring depth
};
constexpr int kGWork = 16;      // act-quant exchange slots (barrier pairs, amax rows)
// Warp roles: epilogue-only warps (SwiGLU with the exact expf, act quant,
// stores; latency-bound, a third of a unit's time or more) on one of two TMEM
// accumulator sets, while 8 converter warps and the MMA go on with the next
// unit; then the TMA producer warp and the MMA warp.  Epilogue warp w reads TMEM
// lane quadrant w % 4; 16-token tiles take 4, the larger tiles 8 (two column
// halves).
template <int kN>
struct GWarps {
  static constexpr int epi = kN <= 16 ? 4 : 8;
  static constexpr int conv = 8;
  static constexpr int threads = (epi + conv + 2) * 32;
};
constexpr int kGRawA = 128 * 64;    // FP4 A tile: 128 rows x 128 K
constexpr int kGConvA = 128 * 128;  // E4M3 A tile

constexpr uint32_t kGTmemCols = 512;

struct GroupedArgs {
  const CUtensorMap* amaps;  // [experts][3] FP4 maps, box {64 B, 128 rows}
  const Fp4ExpertDev* experts;
  int K, M;                  // reduction length; rows of each weight matrix
  const uint8_t* bsf;        // UE8M0 of the B rows, row r at bsf + r * bsf_stride
  int bsf_stride;            // bytes (K/32 for a dense [rows][K/32] array)
  int rows_total;
  const int4* units;         // (expert, m tile, first row, valid rows)
  const int* n_units;
  uint8_t* hq;               // up: [rows][M] E4M3 of act-quantised h
  uint8_t* hsf;              // up: [rows][M/32] UE8M0
  float* y;                  // down: [rows][M]
  const int* y_row_map;      // down, nullable: output row of each B row
  // down, peer transport: output rows m < y_peer_rows belong to source rank
  // m / y_cap and go to row y_self_off + m % y_cap of y_peers[m / y_cap] (that
  // rank's window); rows m >= y_peer_rows go to row m - y_peer_rows of y
  float* const* y_peers;
  int y_peer_rows, y_cap, y_self_off;
  // nullable: after its last store, the kernel's last CTA releases
  // *sig_flags[i] = sig_epoch for i < sig_n (arrival counter sig_done)
  uint64_t* const* sig_flags;
  uint32_t* sig_done;
  int sig_n;
  uint64_t sig_epoch;
  uint32_t* status;
};

template <bool kUp, int kN>
struct GroupedSmem {
  static constexpr int kGStages = GRing<kUp, kN>::stages;
  static constexpr int kGConv = GRing<kUp, kN>::conv;
  static constexpr int kGB = kN * 128;  // E4M3 B tile (1024-byte multiple)
  static constexpr int kRawStage = kGB + (kUp ? 2 : 1) * kGRawA;
  static constexpr int kConvStage = (kUp ? 2 : 1) * kGConvA;
  static constexpr int kSfStage = (kUp ? 3 : 2) * 512;
  static constexpr size_t kBytes = 1024 + size_t(kGStages) * kRawStage +
                                   size_t(kGConv) * kConvStage + size_t(kGConv) * kSfStage +
                                   (2 * kGStages + 2 * kGConv + 5 + kGWork / 2) * 8 + 16 +
                                   2 * kGWork * 16 * 4;
  static_assert(kBytes <= 232448, "grouped GEMM shared memory over 227 KB");
  static_assert(2 * 2 * kN + 16 * kGConv <= 512, "two accumulator sets and the scales exceed TMEM");
};

// 8 FP4 codes (one 32-bit word, code i in bits 4i..4i+3) -> 8 E4M3 bytes of
// the reference values {0, 0.125, 1, 1.5, 2, 3, 4, 6} with the code's sign.
__device__ __forceinline__ uint2 fp4x8_to_e4m3x8(uint32_t w) {
  const uint32_t mag = w & 0x77777777u;
  const uint32_t lo = __byte_perm(0x3C382000u, 0x4C484440u, mag);
  const uint32_t hi = __byte_perm(0x3C382000u, 0x4C484440u, mag >> 16);
  const uint32_t w4 = w << 4;
  const uint32_t slo = __byte_perm(w4, w, 0x5140);  // sign of code i at bit 7 of byte i
  const uint32_t shi = __byte_perm(w4, w, 0x7362);
  return make_uint2(lo | (slo & 0x80808080u), hi | (shi & 0x80808080u));
}

// FP4 tiles [128 rows][64 B] -> E4M3 [128 rows][128 B] with 128-byte
// swizzle; 32 * kWork threads, 512 / (32 * kWork) 16-byte chunks of each
// of the kMats tiles per thread.  Every load is issued before the first
// conversion.
template <int kMats, int kWork>
__device__ __forceinline__ void convert_tiles(const uint8_t* raw, int raw_stride, uint8_t* dst,
                                              int dst_stride, int tid) {
  constexpr int kPer = 512 / (32 * kWork);
  uint4 v[kMats][kPer];
#pragma unroll
  for (int m = 0; m < kMats; ++m)
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = tid + 32 * kWork * j;
      v[m][j] = *reinterpret_cast<const uint4*>(raw + m * raw_stride + (i >> 2) * 64 + (i & 3) * 16);
    }
#pragma unroll
  for (int m = 0; m < kMats; ++m)
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = tid + 32 * kWork * j;
      const int r = i >> 2, ch = i & 3;
      const uint2 a = fp4x8_to_e4m3x8(v[m][j].x), b = fp4x8_to_e4m3x8(v[m][j].y);
      const uint2 c = fp4x8_to_e4m3x8(v[m][j].z), d = fp4x8_to_e4m3x8(v[m][j].w);
      uint8_t* row = dst + m * dst_stride + r * 128;
      *reinterpret_cast<uint4*>(row + (((2 * ch) ^ (r & 7)) << 4)) = make_uint4(a.x, a.y, b.x, b.y);
      *reinterpret_cast<uint4*>(row + (((2 * ch + 1) ^ (r & 7)) << 4)) =
          make_uint4(c.x, c.y, d.x, d.y);
    }
}

// word k of a 16-byte group without local memory
__device__ __forceinline__ uint32_t pick4(const uint4& v, int k) {
  return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

__device__ __forceinline__ uint8_t e4m3_byte(float q) {
  return (uint8_t)__nv_cvt_float_to_fp8(q, __NV_SATFINITE, __NV_E4M3);
}
// two values -> E4M3 bytes, round to nearest even, saturated to +-448 (exact
// for values already on the E4M3 grid)
__device__ __forceinline__ uint32_t e4m3x2_rn(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// The reference's act-quant rounding of t = v / scale (src/compute.rs:2504-2545):
// clamp to +-448 (a NaN stays NaN, as f32::clamp keeps it), then the nearest
// E4M3 grid value with ties to the lower entry; returned as the E4M3 byte.
// A NaN maps to the reference's lut[0] = -480, which has no E4M3 encoding
// other than 0xFF (NaN to the tensor core); the layer's output is then
// non-finite and the call reports NonFiniteOutput.
__device__ __forceinline__ float aq_clamp448(float t) {
  return t < -448.0f ? -448.0f : (t > 448.0f ? 448.0f : t);
}
__device__ __forceinline__ uint32_t e4m3x2_ref(float lo, float hi) {
  const float a = e4m3_nearest_ties_lower(aq_clamp448(lo));
  const float b = e4m3_nearest_ties_lower(aq_clamp448(hi));
  uint32_t r = e4m3x2_rn(a, b);
  if (a == -480.0f) r |= 0xFFu;
  if (b == -480.0f) r |= 0xFF00u;
  return r;
}

template <bool kUp, int kN>
__global__ void __launch_bounds__(GWarps<kN>::threads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap bmap, GroupedArgs a) {
  using L = GroupedSmem<kUp, kN>;
  constexpr int kGB = L::kGB;
  constexpr int kGStages = L::kGStages;
  constexpr int kGConv = L::kGConv;
  using WR = GWarps<kN>;
  constexpr int kEpiW = WR::epi, kConvW = WR::conv, kAccBufs = 2;
  constexpr int kProducer = kEpiW + kConvW, kMmaWarp = kProducer + 1;
  constexpr int kEpiWarps = kEpiW;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* raw = smem;                                        // [stages][B | A1 | A3]
  uint8_t* conv = raw + kGStages * L::kRawStage;              // [conv][A1 | A3]
  uint8_t* sfs = conv + kGConv * L::kConvStage;               // [conv][SFA1 | SFA3 | SFB]
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(sfs + kGConv * L::kSfStage);
  uint64_t* raw_empty = raw_full + kGStages;
  uint64_t* conv_full = raw_empty + kGStages;
  uint64_t* conv_empty = conv_full + kGConv;
  uint64_t* acc_full = conv_empty + kGConv;  // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  uint64_t* mma_done = acc_empty + 2;
  uint64_t* pair_bar = mma_done + 1;  // [kGWork/2]: warps 2p, 2p+1 (act-quant amax exchange)
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(pair_bar + kGWork / 2);
  float* amax_s = reinterpret_cast<float*>(tmem_base_s + 4);  // [2 parity][8 warps][16]
  __shared__ uint32_t aq_thr[256];  // act-quant ceil(log2f) thresholds

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ktiles = a.K / 128;
  constexpr int kMats = kUp ? 2 : 1;
  for (int i = tid; i < 256; i += WR::threads) aq_thr[i] = c_aq.thr[i];

  if (tid == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kConvW + 1);
    }
    for (int c = 0; c < kGConv; ++c) {
      mbar_init(&conv_full[c], kConvW);
      mbar_init(&conv_empty[c], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    for (int p = 0; p < kGWork / 2; ++p) mbar_init(&pair_bar[p], 64);
    fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_base_s, kGTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_base_s;
  const int n_units = *a.n_units;

  if (warp == kProducer) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      bool ok = true;
      uint32_t g = 0;
      prefetch_tensormap(&bmap);
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x) {
        const int4 un = a.units[u];
        const CUtensorMap* m1 = a.amaps + un.x * 3 + (kUp ? 0 : 2);
        const CUtensorMap* m3 = a.amaps + un.x * 3 + 1;
        prefetch_tensormap(m1);
        if (kUp) prefetch_tensormap(m3);
        for (int kt = 0; kt < ktiles; ++kt, ++g) {
          const int s = g % kGStages;
          if (g >= kGStages && !mbar_wait(&raw_empty[s], ((g / kGStages) - 1) & 1, a.status)) {
            ok = false;
            break;
          }
          uint8_t* st = raw + s * L::kRawStage;
          mbar_arrive_expect_tx(&raw_full[s], kGB + kMats * kGRawA);
          tma_load_2d(st, &bmap, &raw_full[s], kt * 128, un.z);
          tma_load_2d(st + kGB, m1, &raw_full[s], kt * 64, un.y * 128);
          if (kUp) tma_load_2d(st + kGB + kGRawA, m3, &raw_full[s], kt * 64, un.y * 128);
        }
      }
      // no copy may be in flight when the CTA exits
      for (uint32_t i = g > kGStages ? g - kGStages : 0; i < g; ++i)
        if (!mbar_drain(&raw_full[i % kGStages], (i / kGStages) & 1, a.status)) break;
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = true;
      uint32_t g = 0, gc = 0, nu = 0;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++nu) {
        const uint32_t ab = nu % kAccBufs;
        if (nu >= kAccBufs && !mbar_wait(&acc_empty[ab], ((nu / kAccBufs) - 1) & 1, a.status))
          break;
        tc::fence_after_sync();
        const uint32_t tacc = tmem + ab * 2 * kN;
        for (int kt = 0; kt < ktiles; ++kt, ++g, ++gc) {
          const int s = g % kGStages, c = gc % kGConv;
          if (!mbar_wait(&conv_full[c], (gc / kGConv) & 1, a.status) ||
              !mbar_wait(&raw_full[s], (g / kGStages) & 1, a.status)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t tsf = tmem + kAccBufs * 2 * kN + 16 * c;
          const uint8_t* sf = sfs + c * L::kSfStage;
          tc::cp_sf_block(tsf, tc::desc_sf_block(smem_u32(sf)));
          if (kUp) tc::cp_sf_block(tsf + 4, tc::desc_sf_block(smem_u32(sf + 512)));
          const uint32_t tsfb = tsf + 8;
          tc::cp_sf_block(tsfb, tc::desc_sf_block(smem_u32(sf + (kUp ? 1024 : 512))));
          const uint8_t* bt = raw + s * L::kRawStage;
          const uint8_t* ct = conv + c * L::kConvStage;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t acc = (kt | k) != 0;
            const uint32_t id = tc::idesc_mxf8(kN, k, k);
            const uint64_t db = tc::desc_sw128(smem_u32(bt + 32 * k));
            tc::mma_mxf8(tacc, tc::desc_sw128(smem_u32(ct + 32 * k)), db, id,
                         tsf | (uint32_t(k) << 30), tsfb | (uint32_t(k) << 30), acc);
            if (kUp)
              tc::mma_mxf8(tacc + kN, tc::desc_sw128(smem_u32(ct + kGConvA + 32 * k)), db, id,
                           (tsf + 4) | (uint32_t(k) << 30), tsfb | (uint32_t(k) << 30), acc);
          }
          tc::commit(&conv_empty[c]);
          tc::commit(&raw_empty[s]);
        }
        if (ok) tc::commit(&acc_full[ab]);
      }
      // every MMA and scale copy has finished before TMEM is released
      tc::commit(mma_done);
      mbar_wait(mma_done, 0, a.status);
    }
  } else {
    // ------- epilogue: warp w reads TMEM lanes 32*(w%4).. and columns -------
    // ------- [kCols*(w/4), +kCols) of the tile                         -------
    uint32_t chunk = 0;  // act-quant exchange parity
    auto epilogue = [&](const int4& un, uint32_t tacc) -> bool {
      bool ok = true;
      const int q4 = warp & 3;
      const int feat = un.y * 128 + q4 * 32 + lane;
      const uint32_t trow = tacc + ((uint32_t)(q4 * 32) << 16);
      // columns of this warp: the tile split over the kEpiWarps/4 groups of 4
      // warps in 16-column chunks (the small tile's single chunk goes to warps 0-3)
      constexpr int kGroups = kEpiWarps / 4;
      constexpr int kCols = (kN / 16 + kGroups - 1) / kGroups * 16;  // whole 16-column chunks
      const int col0 = (warp >> 2) * kCols;
      for (int n0 = col0; n0 < col0 + kCols && n0 < kN; n0 += 16) {
        if (n0 >= un.w) break;  // every remaining column is past the expert's rows
        uint32_t v1[16];
        tc::ld_32x32b_x16(trow + n0, v1);
        if (kUp) {
          uint32_t v3[16];
          tc::ld_32x32b_x16(trow + kN + n0, v3);
          tc::wait_ld();
          float h[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            // SwiGLU with the reference clamps and its silu, x / (1 + expf(-x)),
            // with the host libm's expf (src/deepseek_v4.rs:551-554,589-593)
            const float gte = fminf(__uint_as_float(v1[j]), 10.0f);
            float upv = __uint_as_float(v3[j]);
            upv = upv < -10.0f ? -10.0f : upv;
            upv = upv > 10.0f ? 10.0f : upv;
            h[j] = __fmul_rn(silu_ref(gte), upv);
          }
          // act quant of h per token over the 64 features of warps 2p, 2p+1
          float mine = 0.0f;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float m = fabsf(h[j]);
#pragma unroll
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == j) mine = m;
          }
          float* xs_amax = amax_s + (chunk & 1) * (kGWork * 16);
          if (lane < 16) xs_amax[warp * 16 + lane] = mine;
          mbar_arrive(&pair_bar[warp >> 1]);
          if (!mbar_wait(&pair_bar[warp >> 1], chunk & 1, a.status)) ok = false;
          ++chunk;
          // lane j < 16: exponent of token n0 + j
          int kj = 0;
          if (lane < 16) {
            const float m = fmaxf(fmaxf(mine, xs_amax[(warp ^ 1) * 16 + lane]), 1.0e-4f);
            kj = ceil_log2f_thr(__fdiv_rn(m, 448.0f), aq_thr);
            const int row = un.z + n0 + lane;
            if ((warp & 1) == 0 && n0 + lane < un.w)
              *reinterpret_cast<uint16_t*>(a.hsf + (long long)row * (a.M / 32) +
                                           (un.y * 128 + q4 * 32) / 32) =
                  (uint16_t)((kj + 127) * 0x0101);
          }
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const int k0 = __shfl_sync(0xffffffffu, kj, j);
            const int k1 = __shfl_sync(0xffffffffu, kj, j + 1);
            // h / 2^k == h * 2^-k exactly
            const uint32_t b2 = e4m3x2_ref(__fmul_rn(h[j], exp2i(-k0)), __fmul_rn(h[j + 1], exp2i(-k1)));
            const long long row = un.z + n0 + j;
            if (n0 + j < un.w) a.hq[row * a.M + feat] = (uint8_t)(b2 & 0xff);
            if (n0 + j + 1 < un.w) a.hq[(row + 1) * a.M + feat] = (uint8_t)(b2 >> 8);
          }
        } else {
          tc::wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (n0 + j < un.w) {
              const int row = un.z + n0 + j;
              const int m = a.y_row_map ? a.y_row_map[row] : row;
              float* dst;
              if (m < a.y_peer_rows) {
                const int src = m / a.y_cap;
                dst = a.y_peers[src] + (long long)(a.y_self_off + m - src * a.y_cap) * a.M;
              } else {
                dst = a.y + (long long)(m - a.y_peer_rows) * a.M;
              }
              dst[feat] = __uint_as_float(v1[j]);
            }
        }
      }
      return ok;
    };
    if (warp < kEpiW) {
      // ---------------- epilogue warps ----------------
      bool ok = true;
      uint32_t nu = 0;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++nu) {
        const uint32_t ab = nu % kAccBufs;
        if (!mbar_wait(&acc_full[ab], (nu / kAccBufs) & 1, a.status)) break;
        tc::fence_after_sync();
        ok = epilogue(a.units[u], tmem + ab * 2 * kN);
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[ab]);
      }
    } else {
      // ---------------- converters ----------------
      const int ctid = tid - 32 * kEpiW;
      bool ok = true;
      uint32_t g = 0, gc = 0, nu = 0;
      // scale factors: converter threads 0-127 stage SFA1 (+ SFB) of row ctid,
      // threads 128-255 stage SFA3 of row ctid-128, the others none
      const int r = ctid & 127;
      const bool second = ctid >= 128;
      const bool stages_sf = ctid < 256;
      const int sfk = a.K / 32;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++nu) {
        const int4 un = a.units[u];
        const Fp4ExpertDev& ex = a.experts[un.x];
        const uint8_t* sfa = (second ? ex.w3_scale : (kUp ? ex.w1_scale : ex.w2_scale)) +
                             (long long)(un.y * 128 + r) * sfk;
        const bool need_a = stages_sf && (!second || kUp);
        const bool brow_ok = un.z + r < a.rows_total;
        const uint8_t* sfb = a.bsf + (long long)(brow_ok ? un.z + r : 0) * a.bsf_stride;
        // scale bytes of 4 K tiles per 16-byte load, one group ahead
        auto sf_group = [&](int kt0, uint4& qa, uint4& qb) {
          qa = need_a ? __ldg(reinterpret_cast<const uint4*>(sfa + kt0 * 4)) : make_uint4(0, 0, 0, 0);
          qb = (!second && stages_sf && brow_ok) ? __ldg(reinterpret_cast<const uint4*>(sfb + kt0 * 4))
                                    : make_uint4(0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu);
        };
        uint4 ca, cb, na, nb;
        sf_group(0, na, nb);
        for (int kt = 0; kt < ktiles; ++kt, ++g, ++gc) {
          const int s = g % kGStages, c = gc % kGConv;
          if ((kt & 3) == 0) {
            ca = na;
            cb = nb;
            if (kt + 4 < ktiles) sf_group(kt + 4, na, nb);
          }
          if (!mbar_wait(&raw_full[s], (g / kGStages) & 1, a.status) ||
              (gc >= kGConv && !mbar_wait(&conv_empty[c], ((gc / kGConv) - 1) & 1, a.status))) {
            ok = false;
            break;
          }
          const uint8_t* st = raw + s * L::kRawStage;
          uint8_t* ct = conv + c * L::kConvStage;
          convert_tiles<kMats, kConvW>(st + kGB, kGRawA, ct, kGConvA, ctid);
          uint8_t* sf = sfs + c * L::kSfStage;
          const int atom = (r & 31) * 16 + (r >> 5) * 4;
          if (!stages_sf) {
          } else if (!second) {
            *reinterpret_cast<uint32_t*>(sf + atom) = pick4(ca, kt & 3);
            *reinterpret_cast<uint32_t*>(sf + (kUp ? 1024 : 512) + atom) = pick4(cb, kt & 3);
          } else if (kUp) {
            *reinterpret_cast<uint32_t*>(sf + 512 + atom) = pick4(ca, kt & 3);
          }
          tc::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&conv_full[c]);
            mbar_arrive(&raw_empty[s]);
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, kGTmemCols);
  if (a.sig_flags && last_cta_arrival(a.sig_done) && tid < a.sig_n)
    st_release_sys(a.sig_flags[tid], a.sig_epoch);
}

// ---------------------------------------------------------------------------
// routing bookkeeping
// ---------------------------------------------------------------------------
struct GroupedPlanArgs {
  const int32_t* ids;  // [T][topk]
  int tokens, topk, num_experts, has_shared;
  int* counts;         // [experts + 1], zeroed before the count kernel
  int* slot;           // [T][topk] row of (t, k) within its expert
  int* offsets;        // [experts + 2] first row of each expert (shared = experts)
  int4* units_up;      // (expert, m tile, first row, valid rows)
  int4* units_down;
  int* n_units;        // [2]
  int mt_up, mt_down;  // 128-row tiles of inter / hidden
  int tile_n;          // tokens per tile of the grouped GEMMs
  int route_order;     // combine in route order (single-token semantics) instead of id order
  uint32_t* status;
};

__global__ void grouped_count_kernel(GroupedPlanArgs a) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.tokens * a.topk) return;
  const int e = a.ids[i];
  if (e < 0 || e >= a.num_experts) {
    flag(a.status, WH_DEV_BADARG);
    a.slot[i] = -1;
    return;
  }
  a.slot[i] = atomicAdd(&a.counts[e], 1);
}

// One CTA: exclusive scans of rows and tiles over the experts, then the unit
// lists (expert-major so that CTAs running together share B rows).
__global__ void __launch_bounds__(1024) grouped_units_kernel(GroupedPlanArgs a) {
  __shared__ int tiles_s[1056];
  __shared__ int rows_s[1056];
  const int ne = a.num_experts + a.has_shared;
  const int tn = a.tile_n;
  for (int e = threadIdx.x; e < ne; e += blockDim.x) {
    const int n = e < a.num_experts ? a.counts[e] : a.tokens;
    rows_s[e] = n;
    tiles_s[e] = (n + tn - 1) / tn;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // exclusive scans of rows and tiles, 32 experts per step
    const int lane = threadIdx.x;
    int row = 0, tile = 0;
    for (int base = 0; base < ne; base += 32) {
      const int e = base + lane;
      const int n = e < ne ? rows_s[e] : 0, t = e < ne ? tiles_s[e] : 0;
      int sn = n, st = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int pn = __shfl_up_sync(0xffffffffu, sn, o), pt = __shfl_up_sync(0xffffffffu, st, o);
        if (lane >= o) {
          sn += pn;
          st += pt;
        }
      }
      if (e < ne) {
        rows_s[e] = row + sn - n;
        tiles_s[e] = tile + st - t;
        a.offsets[e] = row + sn - n;
      }
      row += __shfl_sync(0xffffffffu, sn, 31);
      tile += __shfl_sync(0xffffffffu, st, 31);
    }
    if (lane == 0) {
      a.offsets[ne] = row;
      a.n_units[0] = tile * a.mt_up;
      a.n_units[1] = tile * a.mt_down;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < ne; e += blockDim.x) {
    const int n = a.offsets[e + 1] - a.offsets[e];
    const int nt = (n + tn - 1) / tn;
    for (int t = 0; t < nt; ++t) {
      const int row0 = a.offsets[e] + t * tn;
      const int nv = min(tn, n - t * tn);
      const int u = tiles_s[e] + t;
      for (int m = 0; m < a.mt_up; ++m) a.units_up[u * a.mt_up + m] = make_int4(e, m, row0, nv);
      for (int m = 0; m < a.mt_down; ++m)
        a.units_down[u * a.mt_down + m] = make_int4(e, m, row0, nv);
    }
  }
}

// Act quant of each token (src/compute.rs:2504-2545, block 64) written as E4M3
// bytes + UE8M0 exponents to the token's rows of every expert it routes to.
__global__ void __launch_bounds__(128) grouped_dispatch_kernel(GroupedPlanArgs a, const float* x,
                                                               int hidden, uint8_t* xq,
                                                               uint8_t* xsf) {
  const int t = blockIdx.x;  // blockIdx.y: 4 of the token's 64-blocks
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int rows[33];
  if (threadIdx.x < a.topk) {
    const int i = t * a.topk + threadIdx.x;
    const int e = a.ids[i];
    rows[threadIdx.x] = (e >= 0 && e < a.num_experts && a.slot[i] >= 0) ? a.offsets[e] + a.slot[i]
                                                                         : -1;
  }
  if (threadIdx.x == 0) rows[a.topk] = a.has_shared ? a.offsets[a.num_experts] + t : -1;
  __syncthreads();
  const int nrows = a.topk + 1;
  const float* xt = x + (long long)t * hidden;
  for (int blk = blockIdx.y * 4 + warp; blk < hidden / 64; blk += 4 * gridDim.y) {
    const float v0 = xt[blk * 64 + 2 * lane], v1 = xt[blk * 64 + 2 * lane + 1];
    float amax = fmaxf(fabsf(v0), fabsf(v1));
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    amax = fmaxf(amax, 1.0e-4f);
    const int k = ceil_log2f_ref(__fdiv_rn(amax, 448.0f), &c_aq);
    const float sc = exp2i(k);
    const uint32_t b2 = uint32_t(e4m3_byte(aq_grid(v0, sc))) | uint32_t(e4m3_byte(aq_grid(v1, sc))) << 8;
    for (int j = 0; j < nrows; ++j) {
      const int row = rows[j];
      if (row < 0) continue;
      reinterpret_cast<uint16_t*>(xq + (long long)row * hidden + blk * 64)[lane] = (uint16_t)b2;
      if (lane < 2) xsf[(long long)row * (hidden / 32) + blk * 2 + lane] = (uint8_t)(k + 127);
    }
  }
}

// y[t] = shared(x_t) + sum over t's experts in ascending id of y_e * w/sum(w)
// (finish of the batched path, src/compute.rs:1817-1870 with the union order of
// src/server/generation.rs:2487-2569).
__global__ void __launch_bounds__(256) grouped_combine_kernel(GroupedPlanArgs a, const float* yrows,
                                                              const float* combine_w, const float* x,
                                                              float* y, int hidden) {
  const int t = blockIdx.x;
  __shared__ int rows[33];
  __shared__ float ws[33];
  if (threadIdx.x == 0) {
    int n = 0;
    // insertion order by expert id ascending
    int ids[32];
    for (int k = 0; k < a.topk; ++k) {
      const int i = t * a.topk + k;
      const int e = a.ids[i];
      if (e < 0 || e >= a.num_experts || a.slot[i] < 0) continue;
      int p = n++;
      while (!a.route_order && p > 0 && ids[p - 1] > e) {
        ids[p] = ids[p - 1];
        rows[p] = rows[p - 1];
        ws[p] = ws[p - 1];
        --p;
      }
      ids[p] = e;
      rows[p] = a.offsets[e] + a.slot[i];
      ws[p] = combine_w[i];
    }
    rows[32] = n;
  }
  __syncthreads();
  const int n = rows[32];
  const long long sh = a.has_shared ? (long long)(a.offsets[a.num_experts] + t) * hidden : -1;
  for (int h = blockIdx.y * blockDim.x + threadIdx.x; h < hidden; h += blockDim.x * gridDim.y) {
    float acc = 0.0f;
    if (a.route_order && n == 1)  // one expert: unweighted (src/compute.rs:1960-1966)
      acc = yrows[(long long)rows[0] * hidden + h];
    else
      for (int j = 0; j < n; ++j)
        acc = __fadd_rn(acc, __fmul_rn(yrows[(long long)rows[j] * hidden + h], ws[j]));
    float out;
    if (n > 0)
      out = sh >= 0 ? __fadd_rn(yrows[sh + h], acc) : acc;
    else
      out = sh >= 0 ? yrows[sh + h] : x[(long long)t * hidden + h];
    y[(long long)t * hidden + h] = out;
  }
}

// Any UE8M0 scale byte equal to 0 or 255 in any expert matrix -> *flag = 1.
__global__ void grouped_scale_check_kernel(const Fp4ExpertDev* ex, int hidden, int inter,
                                           uint32_t* flag) {
  const Fp4ExpertDev& e = ex[blockIdx.y];
  const uint8_t* p = blockIdx.z == 0 ? e.w1_scale : blockIdx.z == 1 ? e.w3_scale : e.w2_scale;
  const long long n4 = (long long)hidden * inter / 32 / 4;
  const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
  bool bad = false;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const uint32_t v = q[i];
    bad |= (((v - 0x01010101u) & ~v & 0x80808080u) | ((~v - 0x01010101u) & v & 0x80808080u)) != 0;
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flag, 1u);
}

cudaError_t launch_scale_check(const Fp4ExpertDev* ex, int n, int hidden, int inter,
                               uint32_t* flag, cudaStream_t s) {
  grouped_scale_check_kernel<<<dim3(16, n, 3), 256, 0, s>>>(ex, hidden, inter, flag);
  return cudaGetLastError();
}

template <bool kUp, int kN>
cudaError_t launch_grouped_t(const CUtensorMap& bmap, const GroupedArgs& a, int num_sms,
                             cudaStream_t s) {
  const size_t smem = GroupedSmem<kUp, kN>::kBytes;
  cudaError_t e = ensure_smem(grouped_gemm_kernel<kUp, kN>, smem);
  if (e != cudaSuccess) return e;
  grouped_gemm_kernel<kUp, kN><<<num_sms, GWarps<kN>::threads, smem, s>>>(bmap, a);
  return cudaGetLastError();
}

// tile_n: kGN (batches) or kGNSmall (decode-sized)
cudaError_t launch_grouped_gemm(bool up, int tile_n, const CUtensorMap& bmap, const GroupedArgs& a,
                                int num_sms, cudaStream_t s) {
  if (tile_n == kGNSmall)
    return up ? launch_grouped_t<true, kGNSmall>(bmap, a, num_sms, s)
              : launch_grouped_t<false, kGNSmall>(bmap, a, num_sms, s);
  return up ? launch_grouped_t<true, kGN>(bmap, a, num_sms, s)
            : launch_grouped_t<false, kGN>(bmap, a, num_sms, s);
}

cudaError_t launch_grouped_route(const GroupedPlanArgs& p, const float* x, int hidden,
                                 uint8_t* xq, uint8_t* xsf, cudaStream_t s) {
  const int n = p.tokens * p.topk;
  grouped_count_kernel<<<(n + 255) / 256, 256, 0, s>>>(p);
  grouped_units_kernel<<<1, 1024, 0, s>>>(p);
  grouped_dispatch_kernel<<<dim3(p.tokens, hidden / 256), 128, 0, s>>>(p, x, hidden, xq, xsf);
  return cudaGetLastError();
}

cudaError_t launch_grouped_combine(const GroupedPlanArgs& p, const float* yrows,
                                   const float* combine_w, const float* x, float* y, int hidden,
                                   cudaStream_t s) {
  grouped_combine_kernel<<<dim3(p.tokens, (hidden + 1023) / 1024), 256, 0, s>>>(p, yrows, combine_w,
                                                                              x, y, hidden);
  return cudaGetLastError();
}

}  // namespace wh
