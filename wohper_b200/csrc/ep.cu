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
namespace wh {

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

// the rank's own tokens as rows first_row + t (shared expert input)
__global__ void __launch_bounds__(128) ep_pack_local_kernel(const float* x, int hidden,
                                                            uint8_t* base, int row_bytes,
                                                            int first_row) {
  const int t = blockIdx.x;
  __shared__ int rows[1];
  if (threadIdx.x == 0) rows[0] = first_row + t;
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
  int* totals;             // [local_experts] rows per local expert
  int* seg_off;            // [world * local_experts] first received row of each segment
  int* src_off;            // [world * local_experts] offset of the segment in its expert block
  const int* exp_off;      // [local_experts + 2] expert block starts (from grouped_units_kernel)
  const uint8_t* recv;     // received rows
  uint8_t* sorted;         // expert-major rows (+ the own tokens at the tail)
  int* row_map;            // [rows] received row of each sorted row
  int row_bytes;
};

__global__ void ep_totals_kernel(EpSortArgs a) {
  const int nseg = a.world * a.local_experts;
  if (threadIdx.x < 32) warp_exclusive_scan(a.recv_counts, a.seg_off, nseg, threadIdx.x);
  for (int l = threadIdx.x; l < a.local_experts; l += blockDim.x) {
    int acc = 0;
    for (int s = 0; s < a.world; ++s) {
      a.src_off[s * a.local_experts + l] = acc;
      acc += a.recv_counts[s * a.local_experts + l];
    }
    a.totals[l] = acc;
  }
}

__global__ void __launch_bounds__(256) ep_permute_kernel(EpSortArgs a) {
  const int s = blockIdx.x;  // segment (source, local expert)
  const int l = s % a.local_experts;
  const int n = a.recv_counts[s];
  const int src0 = a.seg_off[s], dst0 = a.exp_off[l] + a.src_off[s];
  const int chunks = a.row_bytes / 16;
  for (int i = threadIdx.x; i < n * chunks; i += blockDim.x) {
    const int r = i / chunks, c = i % chunks;
    reinterpret_cast<uint4*>(a.sorted + (long long)(dst0 + r) * a.row_bytes)[c] =
        reinterpret_cast<const uint4*>(a.recv + (long long)(src0 + r) * a.row_bytes)[c];
  }
  for (int r = threadIdx.x; r < n; r += blockDim.x) a.row_map[dst0 + r] = src0 + r;
}

__global__ void ep_map_tail_kernel(int* row_map, int first, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) row_map[first + i] = first + i;
}

// y[t] = y_shared[t] + sum over routes in ascending expert id of y_back[pos] * w/sum(w)
__global__ void __launch_bounds__(256) ep_combine_kernel(const int32_t* ids, const float* weights,
                                                         const int* pos, int topk,
                                                         const float* y_back,
                                                         const float* y_shared, int has_shared,
                                                         float* y, int hidden) {
  const int t = blockIdx.x;
  __shared__ int rows[33];
  __shared__ float ws[32];
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
    ep_pack_local_kernel<<<g.tokens, 128, 0, s>>>(x_local, hidden, a.sorted, a.row_bytes,
                                                  recv_rows);
    ep_map_tail_kernel<<<(g.tokens + 255) / 256, 256, 0, s>>>(a.row_map, recv_rows, g.tokens);
  }
  return cudaGetLastError();
}

cudaError_t launch_ep_combine(const int32_t* ids, const float* weights, const int* pos, int tokens,
                              int topk, const float* y_back, const float* y_shared, int has_shared,
                              float* y, int hidden, cudaStream_t s) {
  ep_combine_kernel<<<tokens, 256, 0, s>>>(ids, weights, pos, topk, y_back, y_shared, has_shared,
                                           y, hidden);
  return cudaGetLastError();
}

}  // namespace wh
