// decode.cu -- the one-token MoE FFN step (router, w1/w3 + SwiGLU + act quant,
// w2 + combine) as ONE persistent kernel on sm_100a.
//
// Same arithmetic as router_kernel -> moe_up_kernel -> moe_down_kernel, bit
// for bit (the reference functions are cited there); what changes is the
// schedule.  One cooperative CTA per SM:
//
//   warps 0-15  four consumer groups of four warps.  A group runs one task at
//               a time: an up task (32 rows of w1 and w3 of one slot, two
//               lanes per row, SwiGLU, act quant of the 64-row block by the
//               block's second finisher) or a down task (8 rows of w2 of
//               every slot, two lanes per row, then the route-order combine).
//   warps 16-19 TMA producers, one per group: group g of CTA c takes up task
//               c + G g (the shared expert's blocks first -- they need no
//               routing --, then the routed ones; three or four per SM), then
//               down tasks from a global queue, and streams each task's
//               weight boxes into the group's 5-stage ring.  w2 of a group's
//               first down task streams while it still computes its up task.
//   warp 20     control: this CTA's two gate rows (logits) and one 64-block
//               of the act-quantised token; a grid-wide arrival count; the
//               top-k (every CTA, redundantly, on code warmed by a dry pass at
//               kernel start); staging x for the up tasks and, once every
//               act-quant block is done, the quantised hidden for the down
//               tasks.
//
// Compared with three launches this removes two kernel boundaries (dependency
// release + staging loads), takes the down tasks from a shared queue (256
// CTAs on 148 SMs leave 109 SMs with two) and overlaps the w2 stream with the
// w1/w3 compute.  Measured on B200 it is still slower than the three kernels
// (70-90 us against 59 us), so it is opt-in (wh_moe_plan_set_fused_decode).
//
// Every wait is bounded (%globaltimer); a timeout sets WH_DEV_TIMEOUT and the
// kernel unwinds (later waits fail at once).  The cooperative launch keeps all
// CTAs resident, which the grid-wide waits need.  Global counters in
// `sync` start at zero; the last CTA to leave resets them.
namespace wh {

constexpr int kDecGroups = 4;
constexpr int kDecStages = 5;
constexpr int kDecStageBytes = 8192;  // w1 + w3 boxes [32][128 B], or 8 slots x w2 [8][128 B]
constexpr int kDecUpRows = 32;
constexpr int kDecDownRows = 8;
constexpr int kDecSlots = 8;
constexpr int kDecConsumerWarps = 4 * kDecGroups;
constexpr int kDecProducerWarp = kDecConsumerWarps;               // + group: one per group
constexpr int kDecControlWarp = kDecConsumerWarps + kDecGroups;
constexpr int kDecThreads = (kDecConsumerWarps + kDecGroups + 1) * 32;
constexpr int kDecSkip = 0x40000000;  // task flag: expert id out of range, nothing streamed

struct DecodeArgs {
  RouterArgs r;              // one token
  MoeArgs m;                 // maps: w1/w3 boxes [32 rows][128 B]
  const CUtensorMap* dmaps;  // [experts + shared] w2, boxes [8 rows][128 B]
  __half* xq;                // [hidden] act-quantised token (E4M3 grid values)
  float* xq_mult;            // [hidden / 64]
  __half* hq;                // [slots][inter]
  float* hq_mult;            // [slots][inter / 64]
  uint32_t* sync;            // [4], zero at rest: logits arrivals, task queue, hq blocks, exits
};

struct DecodeSmem {
  int ring, region, xs, xm, hm, bars, hdr, ids, cw, gsh, ys, total;
};
// region: the router's staged gate rows + x, later the quantised hidden of
// every slot (rows padded by 32 / 16 bytes so that lanes of different rows or
// slots hit different banks)
__host__ __device__ inline DecodeSmem decode_smem(int hidden, int inter) {
  DecodeSmem s{};
  int off = 0;
  auto take = [&](int bytes, int align) {
    off = (off + align - 1) / align * align;
    const int at = off;
    off += bytes;
    return at;
  };
  s.ring = take(kDecGroups * kDecStages * kDecStageBytes, 1024);
  const int router_bytes = 2 * (hidden * 2 + 32) + hidden * 4;
  const int hs_bytes = kDecSlots * (inter * 2 + 16);
  s.region = take(router_bytes > hs_bytes ? router_bytes : hs_bytes, 128);
  s.xs = take(hidden * 2, 128);
  s.xm = take((hidden / 64) * 4, 16);
  s.hm = take(kDecSlots * (inter / 64) * 4, 16);
  s.bars = take((2 * kDecGroups * kDecStages + 4 + 3 * kDecGroups) * 8, 8);
  s.hdr = take(kDecGroups * kDecStages * 4, 4);
  s.ids = take(kDecSlots * 4, 4);
  s.cw = take(kDecSlots * 4, 4);
  s.gsh = take(kDecGroups * 2 * 32 * 4, 16);
  s.ys = take(kDecGroups * 2 * kDecSlots * kDecDownRows * 4, 16);
  s.total = off + 1024;  // + alignment slack of the dynamic shared base
  return s;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// wait until *p >= target (bounded; gives up at once after an earlier timeout)
__device__ __forceinline__ bool wait_count(const uint32_t* p, uint32_t target, uint32_t* status) {
  if (ld_acquire_gpu(p) >= target) return true;
  const uint64_t start = globaltimer();
  while (ld_acquire_gpu(p) < target) {
    if ((*(volatile uint32_t*)status & WH_DEV_TIMEOUT) || globaltimer() - start > WH_WAIT_NS) {
      flag(status, WH_DEV_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}
// mbarrier wait that also gives up soon after a timeout elsewhere.  The status
// word is global memory: it is read only every 64th poll, so that a wait that
// succeeds sees the phase within one poll, not one L2 round trip, late.
__device__ __forceinline__ bool dec_wait(uint64_t* bar, uint32_t phase, uint32_t* status) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t start = globaltimer();
  for (uint32_t n = 1; !mbar_try_wait(bar, phase); ++n) {
    if (globaltimer() - start > WH_WAIT_NS ||
        ((n & 63) == 0 && (*(volatile uint32_t*)status & WH_DEV_TIMEOUT))) {
      flag(status, WH_DEV_TIMEOUT);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// up task t: slot and first row.  The shared expert's blocks come first.
__device__ __forceinline__ void dec_up_task(const MoeArgs& m, int t, int& slot, int& row0) {
  const int per = m.inter / kDecUpRows;
  if (m.has_shared) {
    slot = t < per ? m.topk : (t - per) / per;
  } else {
    slot = t / per;
  }
  row0 = (t % per) * kDecUpRows;
}

// (the argument is taken by value and never by address outside the one-off
// top-k calls, which get a local copy: field reads stay constant-bank loads)
__global__ void __launch_bounds__(kDecThreads, 1) moe_decode_kernel(DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* sm = align_smem_1024(smem_raw);
  const MoeArgs m = a.m;
  const DecodeSmem L = decode_smem(m.hidden, m.inter);
  uint8_t* ring = sm + L.ring;
  uint8_t* region = sm + L.region;
  __half* xs = reinterpret_cast<__half*>(sm + L.xs);
  float* xm = reinterpret_cast<float*>(sm + L.xm);
  float* hm = reinterpret_cast<float*>(sm + L.hm);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.bars);
  uint64_t* empty = full + kDecGroups * kDecStages;
  uint64_t* xbar = empty + kDecGroups * kDecStages;  // x staged
  uint64_t* idsbar = xbar + 1;                        // routes known (ids_s, cw_s)
  uint64_t* hsbar = xbar + 2;                         // quantised hidden staged
  uint64_t* rbar = xbar + 3;                          // router rows staged
  uint64_t* gbar = xbar + 4;                          // [groups]: w1 values for SwiGLU
  uint64_t* qbar = gbar + kDecGroups;                 // [groups]: h stored (act quant)
  uint64_t* ybar = qbar + kDecGroups;                 // [groups]: down outputs for the combine
  int* hdr = reinterpret_cast<int*>(sm + L.hdr);
  int* ids_s = reinterpret_cast<int*>(sm + L.ids);
  float* cw_s = reinterpret_cast<float*>(sm + L.cw);
  float* gsh_all = reinterpret_cast<float*>(sm + L.gsh);
  float* ys_all = reinterpret_cast<float*>(sm + L.ys);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int nslots = m.topk + m.has_shared;
  const int n_up = nslots * (m.inter / kDecUpRows);
  const int n_down = m.hidden / kDecDownRows;
  const int hstride = m.inter * 2 + 16;
  uint32_t* status = m.status;

  if (tid == 0) {
    for (int i = 0; i < kDecGroups * kDecStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    mbar_init(xbar, 1);
    mbar_init(idsbar, 1);
    mbar_init(hsbar, 1);
    mbar_init(rbar, 1);
    for (int g = 0; g < kDecGroups; ++g) {
      mbar_init(&gbar[g], 2);
      mbar_init(&qbar[g], 2);
      mbar_init(&ybar[g], 4);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kDecControlWarp) {
    // ------------------------------------------------------------ control
    const RouterArgs r = a.r;
    const int hidden = m.hidden;
    const int e0 = cta * 2;
    const int nrows = max(0, min(2, r.experts - e0));
    const bool do_aq = cta < hidden / 64;
    const int row_stride = hidden * 2 + 32;
    float* x_s = reinterpret_cast<float*>(region + 2 * row_stride);
    bool ok = true;
    if (nrows > 0 || do_aq) {
      if (lane == 0) {
        mbar_arrive_expect_tx(rbar, nrows * hidden * 2 + hidden * 4);
        for (int k = 0; k < nrows; ++k)
          bulk_load(region + k * row_stride, r.gate + (long long)(e0 + k) * hidden, hidden * 2, rbar);
        bulk_load(x_s, r.x, hidden * 4, rbar);
      }
      ok = __all_sync(0xffffffffu, dec_wait(rbar, 0, status));
    }
    if (ok && do_aq) {
      // act-quantised token, block `cta` (src/compute.rs:2504-2545)
      const int blk = cta;
      const float v0 = x_s[blk * 64 + lane], v1 = x_s[blk * 64 + 32 + lane];
      float amax = fmaxf(fabsf(v0), fabsf(v1));
      for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      amax = fmaxf(amax, 1.0e-4f);
      const float scale = exp2i(ceil_log2f_ref(__fdiv_rn(amax, 448.0f), &c_aq));
      a.xq[blk * 64 + lane] = __float2half_rn(aq_grid(v0, scale));
      a.xq[blk * 64 + 32 + lane] = __float2half_rn(aq_grid(v1, scale));
      if (lane == 0) a.xq_mult[blk] = __fmul_rn(scale, 8.0f);
    }
    if (ok && nrows > 0) {
      // logits: dot_bf16_row_avx2 order (src/compute.rs:6115-6136), as router_kernel
      const int p = lane & 15;
      const int rr0 = lane >> 4;
      const int rr = rr0 < nrows ? rr0 : nrows - 1;
      const uint16_t* wv = reinterpret_cast<const uint16_t*>(region + rr * row_stride) + p;
      const float* xv = x_s + p;
      const int chunks = hidden / 16;
      float acc = 0.0f;
#pragma unroll 16
      for (int c = 0; c < chunks; ++c)
        acc = __fmaf_rn(__uint_as_float(uint32_t(wv[c * 16]) << 16), xv[c * 16], acc);
      const float v = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 8));
      const float h1 = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
      const float h2 = __fadd_rn(h1, __shfl_xor_sync(0xffffffffu, h1, 2));
      const float h3 = __fadd_rn(h2, __shfl_xor_sync(0xffffffffu, h2, 4));
      if (p == 0 && rr0 < nrows) r.logits[e0 + rr0] = __fadd_rn(h3, 0.0f);
    }
    // every CTA's logits and x blocks, then the routes (each CTA computes them)
    __threadfence();
    __syncwarp();
    if (lane == 0) atomicAdd(&a.sync[0], 1u);
    ok = __all_sync(0xffffffffu, wait_count(&a.sync[0], (uint32_t)G, status)) && ok;
    fence_proxy_async_global();
    if (lane == 0) {
      mbar_arrive_expect_tx(xbar, hidden * 2 + (hidden / 64) * 4);
      bulk_load(xs, a.xq, hidden * 2, xbar);
      bulk_load(xm, a.xq_mult, (hidden / 64) * 4, xbar);
    }
    {
      const RouterArgs rcopy = a.r;
      router_topk_any(rcopy, 0, lane, false);
    }
    __syncwarp();
    if (lane < m.topk) {
      ids_s[lane] = r.ids[lane];
      cw_s[lane] = r.combine_w ? r.combine_w[lane] : 0.0f;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(idsbar);
    // quantised hidden of every valid slot, once all of its 64-row blocks exist
    int nvalid = m.has_shared;
    for (int k = 0; k < m.topk; ++k) {
      const int e = ids_s[k];
      nvalid += e >= 0 && e < m.num_experts;
    }
    ok = __all_sync(0xffffffffu,
                    wait_count(&a.sync[2], (uint32_t)(nvalid * (m.inter / 64)), status)) && ok;
    fence_proxy_async_global();
    if (lane == 0) {
      mbar_arrive_expect_tx(hsbar, nvalid * (m.inter * 2 + (m.inter / 64) * 4));
      for (int k = 0; k < nslots; ++k) {
        const int e = k < m.topk ? ids_s[k] : m.num_experts;
        if (k < m.topk && !(e >= 0 && e < m.num_experts)) continue;
        bulk_load(region + k * hstride, a.hq + (long long)k * m.inter, m.inter * 2, hsbar);
        bulk_load(hm + k * (m.inter / 64), a.hq_mult + (long long)k * (m.inter / 64),
                  (m.inter / 64) * 4, hsbar);
      }
    }
    // leave no copy in flight
    dec_wait(xbar, 0, status);
    dec_wait(hsbar, 0, status);
  } else if (warp >= kDecProducerWarp) {
    // ------------------------------------------------------------ producers
    // one warp per group, so that each streams with its own task's tensor
    // maps only (one lane issues; a map it has not used lately costs a
    // descriptor fetch per copy)
    const int g = warp - kDecProducerWarp;
    if (lane == 0) {
      int slot_e[kDecSlots];
      bool ids_known = false;
      const int n_total = n_up + n_down;
      uint32_t i = 0;
      // up task cta + G * g (as one CTA per 32-row block on each of the
      // groups: every SM gets three or four), then down tasks from the queue
      int next_up = cta + G * g;
      for (;;) {
        int t;
        if (next_up >= 0 && next_up < n_up) {
          t = next_up;
          next_up = -1;
        } else {
          t = n_up + (int)atomicAdd(&a.sync[1], 1u);
          if (t >= n_total) t = -1;
        }
        const int s0 = i % kDecStages;
        if (i >= kDecStages &&
            !dec_wait(&empty[g * kDecStages + s0], ((i / kDecStages) - 1) & 1, status))
          break;
        if (t < 0) {
          hdr[g * kDecStages + s0] = -1;
          mbar_arrive(&full[g * kDecStages + s0]);
          ++i;
          break;
        }
        int slot = 0, row0 = 0;
        if (t < n_up) dec_up_task(m, t, slot, row0);
        const bool needs_ids = t >= n_up || slot < m.topk;
        if (needs_ids && !ids_known) {
          if (!dec_wait(idsbar, 0, status)) break;
          for (int k = 0; k < kDecSlots; ++k) {
            int e = -1;
            if (k < m.topk) e = ids_s[k];
            else if (k < nslots) e = m.num_experts;
            if (e < -1 || e >= m.num_experts + m.has_shared || (k < m.topk && e >= m.num_experts))
              e = -1;
            slot_e[k] = e;
          }
          ids_known = true;
        }
        int nb;
        const CUtensorMap *m1 = nullptr, *m3 = nullptr;
        int nv = 0;
        if (t < n_up) {
          const int e = slot < m.topk ? slot_e[slot] : m.num_experts;
          if (e < 0) {  // nothing to stream: one header-only stage
            flag(status, WH_DEV_BADARG);
            hdr[g * kDecStages + s0] = t | kDecSkip;
            mbar_arrive(&full[g * kDecStages + s0]);
            ++i;
            continue;
          }
          m1 = m.maps + e * 3 + 0;
          m3 = m.maps + e * 3 + 1;
          prefetch_tensormap(m1);
          prefetch_tensormap(m3);
          nb = m.hidden / 256;
        } else {
          row0 = (t - n_up) * kDecDownRows;
          for (int k = 0; k < nslots; ++k)
            if (slot_e[k] >= 0) {
              prefetch_tensormap(a.dmaps + slot_e[k]);
              ++nv;
            }
          nb = m.inter / 256;
        }
        bool failed = false;
        for (int b = 0; b < nb; ++b, ++i) {
          const int s = i % kDecStages;
          uint64_t* f = &full[g * kDecStages + s];
          if (b > 0 && i >= kDecStages &&
              !dec_wait(&empty[g * kDecStages + s], ((i / kDecStages) - 1) & 1, status)) {
            failed = true;
            break;
          }
          hdr[g * kDecStages + s] = t;
          uint8_t* stage = ring + (g * kDecStages + s) * kDecStageBytes;
          if (t < n_up) {
            mbar_arrive_expect_tx(f, kDecStageBytes);
            tma_load_2d(stage, m1, f, b * 128, row0);
            tma_load_2d(stage + kDecStageBytes / 2, m3, f, b * 128, row0);
          } else {
            mbar_arrive_expect_tx(f, nv * kDecDownRows * 128);
            for (int k = 0; k < nslots; ++k)
              if (slot_e[k] >= 0)
                tma_load_2d(stage + k * kDecDownRows * 128, a.dmaps + slot_e[k], f, b * 128,
                            row0);
          }
        }
        if (failed) break;
      }
      // leave no copy in flight
      for (uint32_t k = i > kDecStages ? i - kDecStages : 0; k < i; ++k)
        dec_wait(&full[g * kDecStages + k % kDecStages], (k / kDecStages) & 1, status);
    }
    __syncwarp();  // lanes 1-31 wait here for lane 0, not at the CTA barrier below
  } else {
    // ------------------------------------------------------------ consumers
    const int g = warp >> 2, wg = warp & 3;
    if (warp == kDecConsumerWarps - 1) {  // warm the top-k code
      const RouterArgs rcopy = a.r;
      router_topk_any(rcopy, 0, lane, true);
    }
    bool have_x = false, have_ids = false, have_hs = false;
    uint32_t i = 0;
    int n_up_done = 0, n_down_done = 0;
    for (;;) {
      const int s = i % kDecStages;
      if (!__all_sync(0xffffffffu, dec_wait(&full[g * kDecStages + s], (i / kDecStages) & 1, status)))
        break;
      const int t = hdr[g * kDecStages + s];
      if (t == -1) break;
      if (t & kDecSkip) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[g * kDecStages + s]);
        ++i;
        continue;
      }
      if (t < n_up) {
        // ---- up task: 32 rows of w1 (warps 0-1) and w3 (warps 2-3)
        int slot, row0;
        dec_up_task(m, t, slot, row0);
        if (!have_x) have_x = __all_sync(0xffffffffu, dec_wait(xbar, 0, status));
        if (slot < m.topk && !have_ids) have_ids = __all_sync(0xffffffffu, dec_wait(idsbar, 0, status));
        if (!have_x || (slot < m.topk && !have_ids)) break;
        const int e = slot < m.topk ? ids_s[slot] : m.num_experts;
        const int mat = wg >> 1;
        const int rl = (wg & 1) * 16 + (lane >> 1);
        const int hf = lane & 1;
        const int row = row0 + rl;
        const int scols = m.hidden / 32;
        const Fp4ExpertDev& ex = m.experts[e];
        const uint8_t* srow = (mat ? ex.w3_scale : ex.w1_scale) + (long long)row * scols;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const int nbox = m.hidden / 256;
        bool ok = true;
        // the row's scale bytes (hidden/32 <= 128), all loaded at task start:
        // box b uses bytes 8b..8b+7, i.e. half of sr[0] after b/2 shifts
        uint4 sr[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          sr[q] = q * 16 < scols ? __ldg(reinterpret_cast<const uint4*>(srow) + q) : make_uint4(0, 0, 0, 0);
        for (int b = 0; b < nbox; ++b) {
          const int sb_s = i % kDecStages;
          if (b > 0 &&
              !__all_sync(0xffffffffu,
                          dec_wait(&full[g * kDecStages + sb_s], (i / kDecStages) & 1, status))) {
            ok = false;
            break;
          }
          const uint2 sb = (b & 1) ? make_uint2(sr[0].z, sr[0].w) : make_uint2(sr[0].x, sr[0].y);
          if (b & 1) {
#pragma unroll
            for (int q = 0; q < 7; ++q) sr[q] = sr[q + 1];
          }
          const uint8_t* base = ring + (g * kDecStages + sb_s) * kDecStageBytes +
                                mat * (kDecStageBytes / 2) + rl * 128;
          uint4 wb[8];
#pragma unroll
          for (int q = 0; q < 8; ++q)
            wb[q] = *reinterpret_cast<const uint4*>(base + 16 * (q ^ (rl & 7)));
          fp4_box_accumulate_half(wb, xs, xm, b, sb, hf, acc);
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[g * kDecStages + sb_s]);
          ++i;
        }
        if (!ok) break;
        const float v = __fadd_rn(hsum8_pair(acc), 0.0f);
        if (!isfinite(v)) flag(status, WH_DEV_NONFINITE);
        const int par = n_up_done & 1;
        float* gsh = gsh_all + (g * 2 + par) * 32;
        ++n_up_done;
        if (mat == 0) {
          if (hf == 0) gsh[rl] = v;
          __syncwarp();
          if (lane == 0) mbar_arrive(&gbar[g]);
          continue;
        }
        if (!__all_sync(0xffffffffu, dec_wait(&gbar[g], par, status))) break;
        // SwiGLU with the reference clamps (src/deepseek_v4.rs:556-596)
        const float gated = fminf(gsh[rl], 10.0f);
        float upped = v;
        upped = upped < -10.0f ? -10.0f : upped;
        upped = upped > 10.0f ? 10.0f : upped;
        const float hv = __fmul_rn(silu_ref(gated), upped);
        const long long hb = (long long)slot * m.inter;
        if (hf == 0) m.h[hb + row] = hv;
        // act quant of the 64-row block (src/deepseek_v4.rs:595) by the
        // block's second finisher; stores fenced before the arrival
        __threadfence();
        __syncwarp();
        if (lane == 0) mbar_arrive(&qbar[g]);
        if (wg != 2) continue;
        if (!__all_sync(0xffffffffu, dec_wait(&qbar[g], par, status))) break;
        uint32_t prev = 0;
        const long long blk = hb / 64 + row0 / 64;
        if (lane == 0) prev = atomicAdd(&m.blk_counters[blk], 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == 0) continue;
        __threadfence();
        const int b0 = (row0 / 64) * 64;
        const float h0 = __ldcg(m.h + hb + b0 + lane), h1 = __ldcg(m.h + hb + b0 + 32 + lane);
        float amax = fmaxf(fabsf(h0), fabsf(h1));
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        amax = fmaxf(amax, 1.0e-4f);
        const float scale = exp2i(ceil_log2f_ref(__fdiv_rn(amax, 448.0f), &c_aq));
        a.hq[hb + b0 + lane] = __float2half_rn(aq_grid(h0, scale));
        a.hq[hb + b0 + 32 + lane] = __float2half_rn(aq_grid(h1, scale));
        if (lane == 0) {
          a.hq_mult[blk] = __fmul_rn(scale, 8.0f);
          m.blk_counters[blk] = 0;  // ready for the next call
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(&a.sync[2], 1u);
      } else {
        // ---- down task: 8 rows of w2 for every slot (warp wg: slots 2wg, 2wg+1)
        const int row0 = (t - n_up) * kDecDownRows;
        if (!have_ids) have_ids = __all_sync(0xffffffffu, dec_wait(idsbar, 0, status));
        if (!have_hs) have_hs = __all_sync(0xffffffffu, dec_wait(hsbar, 0, status));
        if (!have_ids || !have_hs) break;
        const int slot = wg * 2 + (lane >> 4);
        const int r = (lane >> 1) & 7;
        const int hf = lane & 1;
        const int row = row0 + r;
        int e = -1;
        if (slot < m.topk) e = ids_s[slot];
        else if (slot < nslots) e = m.num_experts;
        const bool active = slot < nslots && e >= 0 && (slot >= m.topk || e < m.num_experts);
        const int scols = m.inter / 32;
        const uint8_t* srow = active ? m.experts[e].w2_scale + (long long)row * scols : nullptr;
        const __half* hslot = reinterpret_cast<const __half*>(region + (active ? slot : 0) * hstride);
        const float* hmul = hm + (active ? slot : 0) * (m.inter / 64);
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const int nbox = m.inter / 256;
        bool ok = true;
        uint4 sr[8];  // the row's scale bytes (inter/32 <= 128), loaded at task start
#pragma unroll
        for (int q = 0; q < 8; ++q)
          sr[q] = active && q * 16 < scols ? __ldg(reinterpret_cast<const uint4*>(srow) + q)
                                           : make_uint4(0, 0, 0, 0);
        for (int b = 0; b < nbox; ++b) {
          const int sb_s = i % kDecStages;
          if (b > 0 &&
              !__all_sync(0xffffffffu,
                          dec_wait(&full[g * kDecStages + sb_s], (i / kDecStages) & 1, status))) {
            ok = false;
            break;
          }
          const uint2 sb = (b & 1) ? make_uint2(sr[0].z, sr[0].w) : make_uint2(sr[0].x, sr[0].y);
          if (b & 1) {
#pragma unroll
            for (int q = 0; q < 7; ++q) sr[q] = sr[q + 1];
          }
          if (active) {  // the two halves of a warp may differ: no shuffles inside
            const uint8_t* base = ring + (g * kDecStages + sb_s) * kDecStageBytes +
                                  slot * kDecDownRows * 128 + r * 128;
            uint4 wb[8];
#pragma unroll
            for (int q = 0; q < 8; ++q)
              wb[q] = *reinterpret_cast<const uint4*>(base + 16 * (q ^ (r & 7)));
            fp4_box_accumulate_half(wb, hslot, hmul, b, sb, hf, acc);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[g * kDecStages + sb_s]);
          ++i;
        }
        if (!ok) break;
        const float q = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
        const float o = __shfl_xor_sync(0xffffffffu, q, 1);
        const float yv = __fadd_rn(__fadd_rn(q, o), 0.0f);
        const int par = n_down_done & 1;
        ++n_down_done;
        float* ys = ys_all + (g * 2 + par) * kDecSlots * kDecDownRows;
        if (active && !isfinite(yv)) flag(status, WH_DEV_NONFINITE);
        if (hf == 0) ys[slot * kDecDownRows + r] = active ? yv : 0.0f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&ybar[g]);
        if (wg != 0) continue;
        if (!__all_sync(0xffffffffu, dec_wait(&ybar[g], par, status))) break;
        if (lane < kDecDownRows) {
          // route-order weighted combine + shared expert, as moe_down_kernel
          float routed = 0.0f;
          if (m.topk == 1) {
            routed = ys[0 * kDecDownRows + lane];
          } else {
            for (int k = 0; k < m.topk; ++k)
              routed = __fadd_rn(routed, __fmul_rn(ys[k * kDecDownRows + lane], cw_s[k]));
          }
          float out = routed;
          if (m.has_shared)
            out = m.topk > 0 ? __fadd_rn(ys[m.topk * kDecDownRows + lane], routed)
                             : ys[m.topk * kDecDownRows + lane];
          m.y[row0 + lane] = out;
        }
      }
    }
  }

  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&a.sync[3], 1u) == (uint32_t)G - 1) {
      a.sync[0] = 0;
      a.sync[1] = 0;
      a.sync[2] = 0;
      __threadfence();
      a.sync[3] = 0;
    }
  }
}

size_t decode_smem_bytes(int hidden, int inter) { return (size_t)decode_smem(hidden, inter).total; }

// grid = SM count (one resident CTA each, cooperative)
cudaError_t launch_moe_decode(const DecodeArgs& a, int num_sms, cudaStream_t s) {
  const size_t smem = decode_smem_bytes(a.m.hidden, a.m.inter);
  cudaError_t e = ensure_smem(moe_decode_kernel, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, moe_decode_kernel, a);
}

// can the decode kernel run here: shapes, one resident CTA per SM
bool decode_supported(int experts, int hidden, int inter, int topk, int has_shared, int num_sms) {
  if (topk + has_shared > kDecSlots || topk < 0) return false;
  if (experts > 2 * num_sms || experts < 1) return false;
  if (hidden % 512 || inter % 256 || hidden / 64 > num_sms) return false;
  if (hidden > 4096 || inter > 4096) return false;  // a row's scales held in 8 uint4
  if (hidden / 256 <= kDecStages || inter / 256 <= kDecStages) return false;  // >= 1 task apart
  const size_t smem = decode_smem_bytes(hidden, inter);
  if (smem > 227 * 1024) return false;
  if (ensure_smem(moe_decode_kernel, smem) != cudaSuccess) return false;
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, moe_decode_kernel, kDecThreads, smem) !=
          cudaSuccess ||
      blocks < 1)
    return false;
  return true;
}

}  // namespace wh
