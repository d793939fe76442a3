// ep.cu -- expert parallelism: the MoE FFN with the routed experts sharded
// contiguously over `world` ranks (rank r owns experts [r*E_l, (r+1)*E_l)) and
// the shared expert replicated on every rank.
//
// One step on every rank (the collectives run between these calls, over NCCL):
//   wh_ep_dispatch    act quant of the rank's tokens, rows packed per
//                     destination rank and local expert (E4M3 bytes + UE8M0
//                     exponents, one row per route), counts per (dest, expert)
//   all-to-all        counts, then rows
//   wh_ep_expert_ffn  grouped up/down GEMMs over the received rows (segments
//                     (source rank, local expert)) and over the rank's own
//                     tokens for the shared expert
//   all-to-all        f32 result rows back to their token's rank
//   wh_ep_combine     y = shared(x) + sum over routes in ascending expert id of
//                     y_e * w/sum(w) (the batched path of the reference,
//                     src/compute.rs:1779-1810, 1817-1870)
//
// The peer-memory transport (wh_ep_p2p_*) runs the same step without NCCL and
// without a host synchronisation: every rank exports one window (receive rows,
// receive counts, returned result rows, arrival flags) to the others over CUDA
// IPC; the dispatch kernel stores each route's row straight into its
// destination's window over NVLink and releases a per-source flag; the
// receiving rank's first kernel waits (bounded) for every source's flag; the
// down GEMM's epilogue stores each result row straight into the window of the
// rank that owns the token and the kernel's last CTA releases a per-destination
// flag; the combine waits for those.  Windows are laid out with a fixed
// capacity of rows per source (cap = max_tokens * topk), so no count exchange
// has to precede the row transfer.
namespace wh {

// One rank's view of a peer's window (device array, one entry per rank).
struct EpPeer {
  uint8_t* recv;       // [world][cap][row_bytes] rows received from each source
  int* counts;         // [world][E_l] rows per (source, local expert)
  uint64_t* row_flag;  // [world] epoch of the last rows+counts stored by each source
  uint64_t* res_flag;  // [world] epoch of the last results stored by each destination
  float* yback;        // [world][cap][hidden] result rows returned by each destination
};

struct EpArgs {
  int world, local_experts, topk, hidden, row_bytes;
  const int32_t* ids;  // [tokens][topk] global expert ids
  int tokens;
  int* cnt;            // [world * local_experts] routes per (dest, local expert), zeroed
  int* slot;           // [tokens][topk] index of the route within its (dest, expert)
  int* off;            // [world * local_experts] first send row of each (dest, expert)
  int* pos;            // [tokens][topk] send row of each route
  uint32_t* status;
};

__global__ void ep_count_kernel(EpArgs a) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.tokens * a.topk) return;
  const int e = a.ids[i];
  if (e < 0 || e >= a.world * a.local_experts) {
    flag(a.status, WH_DEV_BADARG);
    a.slot[i] = -1;
    return;
  }
  a.slot[i] = atomicAdd(&a.cnt[e], 1);  // e = dest * local_experts + local id
}

// exclusive scan of n counts by one warp
__device__ __forceinline__ int warp_exclusive_scan(const int* in, int* out, int n, int lane) {
  int base = 0;
  for (int b = 0; b < n; b += 32) {
    const int v = b + lane < n ? in[b + lane] : 0;
    int s = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int p = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += p;
    }
    if (b + lane < n) out[b + lane] = base + s - v;
    base += __shfl_sync(0xffffffffu, s, 31);
  }
  return base;
}

__global__ void ep_scan_kernel(EpArgs a) {
  warp_exclusive_scan(a.cnt, a.off, a.world * a.local_experts, threadIdx.x);
}

// act quant (block 64, src/compute.rs:2504-2545) of token row x into E4M3
// bytes + per-32 exponents, written to each of the nrows rows listed
__device__ __forceinline__ void pack_token_rows(const float* x, int hidden, uint8_t* base,
                                                int row_bytes, const int* rows, int nrows,
                                                int warp, int nwarps, int lane) {
  for (int blk = warp; blk < hidden / 64; blk += nwarps) {
    const float v0 = x[blk * 64 + 2 * lane], v1 = x[blk * 64 + 2 * lane + 1];
    float amax = fmaxf(fabsf(v0), fabsf(v1));
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    amax = fmaxf(amax, 1.0e-4f);
    const int k = ceil_log2f_ref(__fdiv_rn(amax, 448.0f), &c_aq);
    const float sc = exp2i(k);
    const uint16_t b2 = uint16_t(e4m3_byte(aq_grid(v0, sc))) | uint16_t(e4m3_byte(aq_grid(v1, sc))) << 8;
    for (int j = 0; j < nrows; ++j) {
      if (rows[j] < 0) continue;
      uint8_t* row = base + (long long)rows[j] * row_bytes;
      reinterpret_cast<uint16_t*>(row + blk * 64)[lane] = b2;
      if (lane < 2) row[hidden + blk * 2 + lane] = (uint8_t)(k + 127);
    }
  }
}

__global__ void __launch_bounds__(128) ep_pack_kernel(EpArgs a, const float* x, uint8_t* send) {
  const int t = blockIdx.x;
  __shared__ int rows[32];
  if (threadIdx.x < a.topk) {
    const int i = t * a.topk + threadIdx.x;
    const int e = a.ids[i];
    const int r = a.slot[i] >= 0 ? a.off[e] + a.slot[i] : -1;
    rows[threadIdx.x] = r;
    a.pos[i] = r;
  }
  __syncthreads();
  pack_token_rows(x + (long long)t * a.hidden, a.hidden, send, a.row_bytes, rows, a.topk,
                  threadIdx.x >> 5, 4, threadIdx.x & 31);
}

// the rank's own tokens as rows *first_row + t (shared expert input; the first
// row is the shared expert's block start, behind the received rows)
__global__ void __launch_bounds__(128) ep_pack_local_kernel(const float* x, int hidden,
                                                            uint8_t* base, int row_bytes,
                                                            const int* first_row) {
  const int t = blockIdx.x;
  __shared__ int rows[1];
  if (threadIdx.x == 0) rows[0] = *first_row + t;
  __syncthreads();
  pack_token_rows(x + (long long)t * hidden, hidden, base, row_bytes, rows, 1, threadIdx.x >> 5,
                  4, threadIdx.x & 31);
}

// Received rows arrive source-major ((source rank, local expert) segments).
// They are regrouped expert-major so that every local expert's rows form one
// block (each weight tile is then converted once per 128 rows, not once per
// source): per-expert totals and, per segment, its offset inside its
// expert's block; grouped_units_kernel then scans the totals into expert
// offsets (shared expert last, over the rank's own tokens) and the units.
struct EpSortArgs {
  const int* recv_counts;  // [world][local_experts]
  int world, local_experts;
  int seg_stride;          // 0: segments packed back to back (at most max_rows rows);
                           // else source s's segments start at row s * seg_stride
  int max_rows;            // rows available to the received segments
  const uint64_t* wait;    // nullable: [world] arrival flags to wait for (>= epoch)
  uint64_t epoch;
  uint32_t* status;
  int* seg_cnt;            // [world * local_experts] checked counts
  int* totals;             // [local_experts] rows per local expert
  int* seg_off;            // [world * local_experts] first received row of each segment
  int* src_off;            // [world * local_experts] offset of the segment in its expert block
  const int* exp_off;      // [local_experts + 2] expert block starts (from grouped_units_kernel)
  const uint8_t* recv;     // received rows
  uint8_t* sorted;         // expert-major rows (+ the own tokens at the tail)
  int* row_map;            // [rows] received row of each sorted row
  int row_bytes;
};

// One CTA of 1024 threads.  Waits for the sources (peer transport), checks the
// counts (a negative count, or more rows than the layout holds, zeroes the
// offending source's segments and flags WH_DEV_BADARG; a source that timed out
// contributes no rows), then the per-expert totals and segment offsets.
__global__ void __launch_bounds__(1024) ep_totals_kernel(EpSortArgs a) {
  __shared__ int cnt[1024];
  __shared__ int base[1024];
  const int El = a.local_experts, nseg = a.world * El;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ int arrived[1024];
  if (tid < a.world) arrived[tid] = a.wait ? (int)wait_epoch(a.wait + tid, a.epoch, a.status) : 1;
  __syncthreads();
  for (int i = tid; i < nseg; i += blockDim.x) cnt[i] = arrived[i / El] ? a.recv_counts[i] : 0;
  __syncthreads();
  if (a.seg_stride > 0) {
    for (int s = tid; s < a.world; s += blockDim.x) {
      long long sum = 0;
      bool bad = false;
      for (int l = 0; l < El; ++l) {
        bad |= cnt[s * El + l] < 0;
        sum += cnt[s * El + l];
      }
      if (bad || sum > a.seg_stride) {
        flag(a.status, WH_DEV_BADARG);
        for (int l = 0; l < El; ++l) cnt[s * El + l] = 0;
      }
    }
  } else if (tid == 0) {
    long long sum = 0;
    bool bad = false;
    for (int i = 0; i < nseg; ++i) {
      bad |= cnt[i] < 0;
      sum += cnt[i];
    }
    if (bad || sum > a.max_rows) {
      flag(a.status, WH_DEV_BADARG);
      for (int i = 0; i < nseg; ++i) cnt[i] = 0;
    }
  }
  __syncthreads();
  if (a.seg_stride > 0) {
    for (int s = warp; s < a.world; s += blockDim.x >> 5)
      warp_exclusive_scan(cnt + s * El, base + s * El, El, lane);
  } else if (warp == 0) {
    warp_exclusive_scan(cnt, base, nseg, lane);
  }
  __syncthreads();
  for (int i = tid; i < nseg; i += blockDim.x) {
    a.seg_cnt[i] = cnt[i];
    a.seg_off[i] = base[i] + (a.seg_stride > 0 ? (i / El) * a.seg_stride : 0);
  }
  for (int l = tid; l < El; l += blockDim.x) {
    int acc = 0;
    for (int s = 0; s < a.world; ++s) {
      a.src_off[s * El + l] = acc;
      acc += cnt[s * El + l];
    }
    a.totals[l] = acc;
  }
}

__global__ void __launch_bounds__(256) ep_permute_kernel(EpSortArgs a) {
  const int s = blockIdx.x;  // segment (source, local expert)
  const int l = s % a.local_experts;
  const int n = a.seg_cnt[s];
  const int src0 = a.seg_off[s], dst0 = a.exp_off[l] + a.src_off[s];
  const int chunks = a.row_bytes / 16;
  for (int i = threadIdx.x; i < n * chunks; i += blockDim.x) {
    const int r = i / chunks, c = i % chunks;
    reinterpret_cast<uint4*>(a.sorted + (long long)(dst0 + r) * a.row_bytes)[c] =
        reinterpret_cast<const uint4*>(a.recv + (long long)(src0 + r) * a.row_bytes)[c];
  }
  for (int r = threadIdx.x; r < n; r += blockDim.x) a.row_map[dst0 + r] = src0 + r;
}

// output row of the shared expert's rows: tail_base + own token index
__global__ void ep_map_tail_kernel(int* row_map, const int* first, int tail_base, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) row_map[*first + i] = tail_base + i;
}

// y[t] = y_shared[t] + sum over routes in ascending expert id of y_back[pos] * w/sum(w)
// (peer transport: first waits for the result flags of every destination)
__global__ void __launch_bounds__(256) ep_combine_kernel(const int32_t* ids, const float* weights,
                                                         const int* pos, int topk,
                                                         const float* y_back,
                                                         const float* y_shared, int has_shared,
                                                         float* y, int hidden, int tokens,
                                                         const uint64_t* wait, int world,
                                                         uint64_t epoch, uint32_t* status) {
  const int t = blockIdx.x;
  __shared__ int rows[33];
  __shared__ float ws[32];
  // (a rank without tokens still waits: its next dispatch may only store into
  // a destination's window after that destination has consumed this step)
  if (wait && threadIdx.x < world) wait_epoch(wait + threadIdx.x, epoch, status);
  if (t >= tokens) return;
  if (threadIdx.x == 0) {
    float sum = 0.0f;
    bool finite = true;
    for (int k = 0; k < topk; ++k) {
      const float w = weights[t * topk + k];
      sum = __fadd_rn(sum, w);
      finite = finite && isfinite(w);
    }
    finite = finite && isfinite(sum) && sum > 0.0f;
    int key[32];
    int n = 0;
    for (int k = 0; k < topk; ++k) {
      const int i = t * topk + k;
      if (pos[i] < 0) continue;
      const int e = ids[i];
      int p = n++;
      while (p > 0 && key[p - 1] > e) {
        key[p] = key[p - 1];
        rows[p] = rows[p - 1];
        ws[p] = ws[p - 1];
        --p;
      }
      key[p] = e;
      rows[p] = pos[i];
      ws[p] = finite ? __fdiv_rn(weights[i], sum) : __fdiv_rn(1.0f, (float)topk);
    }
    rows[32] = n;
  }
  __syncthreads();
  const int n = rows[32];
  for (int h = threadIdx.x; h < hidden; h += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < n; ++j)
      acc = __fadd_rn(acc, __fmul_rn(y_back[(long long)rows[j] * hidden + h], ws[j]));
    const float sh = has_shared ? y_shared[(long long)t * hidden + h] : 0.0f;
    y[(long long)t * hidden + h] = has_shared ? (n > 0 ? __fadd_rn(sh, acc) : sh) : acc;
  }
}

// ---------------------------------------------------------------------------
// peer-memory transport
// ---------------------------------------------------------------------------
struct EpP2pArgs {
  int world, rank, local_experts, topk, hidden, row_bytes, cap;
  const int32_t* ids;  // [tokens][topk] global expert ids
  int tokens;
  const int* cnt;      // [world * E_l] routes per (dest, local expert)
  const int* slot;     // [tokens][topk] index of the route within its (dest, expert), -1 invalid
  const int* off;      // [world * E_l] first row of each (dest, expert) in the dest's region
  int* pos;            // [tokens][topk] row of the route's result in this rank's returned rows
  const EpPeer* peers;
  uint32_t* done;      // arrival counter (zero at rest)
  uint64_t epoch;
  uint32_t* status;
};

// off[d][l]: exclusive scan of cnt[d][.] (rows from this rank in d's region)
__global__ void ep_scan_dest_kernel(const int* cnt, int* off, int world, int El, int cap,
                                    uint32_t* status) {
  const int lane = threadIdx.x & 31;
  for (int d = threadIdx.x >> 5; d < world; d += blockDim.x >> 5) {
    const int n = warp_exclusive_scan(cnt + d * El, off + d * El, El, lane);
    if (n > cap && lane == 0) flag(status, WH_DEV_BADARG);  // rows past cap are not sent
  }
}

// One CTA per token (at least one CTA: the last one signals even with no
// tokens).  Act quant of the token (block 64, src/compute.rs:2504-2545; lane =
// 16 consecutive features, a warp = 512 features = 8 blocks), then one 16-byte
// store per lane and route into the destination rank's window (E4M3 bytes; the
// 16 exponent bytes of the 512 features by lane 0).  The last CTA stores this
// rank's counts into every destination and releases its arrival flags.
__global__ void __launch_bounds__(256) ep_p2p_pack_kernel(EpP2pArgs a, const float* x) {
  __shared__ uint8_t* dst[32];
  const int t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int El = a.local_experts;
  if (t < a.tokens) {
    if (tid < a.topk) {
      const int i = t * a.topk + tid;
      uint8_t* p = nullptr;
      int r = -1;
      if (a.slot[i] >= 0) {
        const int e = a.ids[i];
        const int j = a.off[e] + a.slot[i];
        const int d = e / El;
        if (j < a.cap) {
          p = a.peers[d].recv + ((long long)a.rank * a.cap + j) * a.row_bytes;
          r = d * a.cap + j;
        }
      }
      dst[tid] = p;
      a.pos[i] = r;
    }
    __syncthreads();
    const float* xr = x + (long long)t * a.hidden;
    for (int c = warp; c < a.hidden / 512; c += blockDim.x >> 5) {
      const float4* src = reinterpret_cast<const float4*>(xr + c * 512 + lane * 16);
      float v[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 f = src[q];
        v[4 * q] = f.x;
        v[4 * q + 1] = f.y;
        v[4 * q + 2] = f.z;
        v[4 * q + 3] = f.w;
      }
      float amax = 0.0f;
#pragma unroll
      for (int q = 0; q < 16; ++q) amax = fmaxf(amax, fabsf(v[q]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, 1.0e-4f);
      const int k = ceil_log2f_ref(__fdiv_rn(amax, 448.0f), &c_aq);
      const float sc = exp2i(k);
      uint32_t w[4], ex[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        w[q] = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) w[q] |= uint32_t(e4m3_byte(aq_grid(v[4 * q + b], sc))) << (8 * b);
        // exponent bytes 4q..4q+3 = blocks 2q, 2q+1 (lanes 8q, 8q+4), twice each
        const uint32_t ka = (uint32_t)(__shfl_sync(0xffffffffu, k, 8 * q) + 127) & 0xffu;
        const uint32_t kb = (uint32_t)(__shfl_sync(0xffffffffu, k, 8 * q + 4) + 127) & 0xffu;
        ex[q] = ka | ka << 8 | kb << 16 | kb << 24;
      }
      const uint4 data = make_uint4(w[0], w[1], w[2], w[3]);
      const uint4 exps = make_uint4(ex[0], ex[1], ex[2], ex[3]);
      for (int r = 0; r < a.topk; ++r) {
        uint8_t* p = dst[r];
        if (!p) continue;
        *reinterpret_cast<uint4*>(p + c * 512 + lane * 16) = data;
        if (lane == 0) *reinterpret_cast<uint4*>(p + a.hidden + c * 16) = exps;
      }
    }
  }
  if (last_cta_arrival(a.done)) {
    for (int i = tid; i < a.world * El; i += blockDim.x)
      a.peers[i / El].counts[a.rank * El + i % El] = a.cnt[i];
    __threadfence_system();
    __syncthreads();
    if (tid < a.world) st_release_sys(a.peers[tid].row_flag + a.rank, a.epoch);
  }
}

// dispatch with the peer transport: counts (cnt zeroed here), per-destination
// offsets, then pack + store + signal
cudaError_t launch_ep_p2p_dispatch(const EpP2pArgs& p, const EpArgs& c, const float* x,
                                   cudaStream_t s) {
  const int n = c.tokens * c.topk;
  cudaError_t e = cudaMemsetAsync(c.cnt, 0, sizeof(int) * c.world * c.local_experts, s);
  if (e != cudaSuccess) return e;
  if (n > 0) ep_count_kernel<<<(n + 255) / 256, 256, 0, s>>>(c);
  ep_scan_dest_kernel<<<1, 32 * (p.world < 32 ? p.world : 32), 0, s>>>(
      p.cnt, const_cast<int*>(p.off), p.world, p.local_experts, p.cap, p.status);
  ep_p2p_pack_kernel<<<p.tokens > 0 ? p.tokens : 1, 256, 0, s>>>(p, x);
  return cudaGetLastError();
}

cudaError_t launch_ep_p2p_combine(const int32_t* ids, const float* weights, const int* pos,
                                  int tokens, int topk, const float* y_back, const float* y_shared,
                                  int has_shared, float* y, int hidden, const uint64_t* wait,
                                  int world, uint64_t epoch, uint32_t* status, cudaStream_t s) {
  ep_combine_kernel<<<tokens > 0 ? tokens : 1, 256, 0, s>>>(
      ids, weights, pos, topk, y_back, y_shared, has_shared, y, hidden, tokens, wait, world, epoch,
      status);
  return cudaGetLastError();
}

cudaError_t launch_ep_dispatch(const EpArgs& a, const float* x, uint8_t* send, cudaStream_t s) {
  const int n = a.tokens * a.topk;
  cudaError_t e = cudaMemsetAsync(a.cnt, 0, sizeof(int) * a.world * a.local_experts, s);
  if (e != cudaSuccess) return e;
  ep_count_kernel<<<(n + 255) / 256, 256, 0, s>>>(a);
  ep_scan_kernel<<<1, 32, 0, s>>>(a);
  ep_pack_kernel<<<a.tokens, 128, 0, s>>>(a, x, send);
  return cudaGetLastError();
}

// regroup the received rows expert-major, add the own tokens as shared-expert
// rows, build the grouped-GEMM units (GroupedPlanArgs.counts = a.totals)
cudaError_t launch_ep_prepare(const EpSortArgs& a, const GroupedPlanArgs& g, const float* x_local,
                              int hidden, int recv_rows, cudaStream_t s) {
  ep_totals_kernel<<<1, 1024, 0, s>>>(a);
  grouped_units_kernel<<<1, 1024, 0, s>>>(g);
  ep_permute_kernel<<<a.world * a.local_experts, 256, 0, s>>>(a);
  if (g.has_shared && g.tokens > 0) {
    const int* first = a.exp_off + a.local_experts;
    ep_pack_local_kernel<<<g.tokens, 128, 0, s>>>(x_local, hidden, a.sorted, a.row_bytes, first);
    ep_map_tail_kernel<<<(g.tokens + 255) / 256, 256, 0, s>>>(a.row_map, first, recv_rows,
                                                              g.tokens);
  }
  return cudaGetLastError();
}

cudaError_t launch_ep_combine(const int32_t* ids, const float* weights, const int* pos, int tokens,
                              int topk, const float* y_back, const float* y_shared, int has_shared,
                              float* y, int hidden, cudaStream_t s) {
  ep_combine_kernel<<<tokens, 256, 0, s>>>(ids, weights, pos, topk, y_back, y_shared, has_shared,
                                           y, hidden, tokens, nullptr, 0, 0, nullptr);
  return cudaGetLastError();
}

}  // namespace wh
