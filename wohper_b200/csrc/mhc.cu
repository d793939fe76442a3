// mhc.cu -- DeepSeek-V4's manifold-constrained hyper-connections (mHC) for sm_100a.
//
// Replaces hc_pre_into, hc_split_sinkhorn_scalar, hc_post_into and hc_head_pool
// (engine/zc_infer_core/src/compute.rs:4945-5132).  The residual stream is
// hc copies of the hidden vector (x [hc][hidden], flattened to hc_dim).
//   hc_pre   mixes_j = (fn_j . x) * inv_rms, inv_rms = 1 / sqrt(sum(x^2) / hc_dim
//            + eps); the split: pre = sigmoid(.) + eps, post = 2 sigmoid(.),
//            comb = softmax rows + eps, then Sinkhorn column/row
//            normalisations; y = sum_i pre_i x_i
//   hc_post  out_k = post_k y + sum_i comb[k][i] res_i
//   hc_head  the same pooling as hc_pre with sigmoid gates and no Sinkhorn
// The reference's sums run in index order with every product and sum rounded
// (no fused multiply-add), and its exp is the host libm's expf (libm_expf).
//
// The sum of squares and the fn-row dots are dependent chains of hc_dim
// additions (16384 for V4: about 33 us at 4 cycles an add), so one CTA per
// token runs them side by side, one thread per chain (chain 0 is x . x, so
// every chain lane runs the same instruction stream).  The chains consume
// 25 rows x 4 B per 4 cycles, about 50 GB/s for one SM: the columns of x and
// of the fn rows stream through a 3-stage cp.async ring of 512-column chunks
// that all 256 threads fill, so about 100 KB are in flight.  The Sinkhorn
// split runs on one thread; the pooled output, and hc_post, are elementwise
// over all threads.
#include "common.cuh"
#include "kernels.cuh"

namespace wh {

constexpr int kHcThreads = 256;
constexpr int kHcStages = 3;

__device__ __forceinline__ float hc_sigmoid(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, libm_expf(-x)));
}

__device__ __forceinline__ void hc_cp_async(float* smem, const float* gmem, bool vec16) {
  const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
  if (vec16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void hc_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void hc_cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Stage st of the ring: columns [st * chunk, +chunk) of x (row 0) and of the
// fn rows (rows 1 .. rows), copied by every thread of the CTA.
__device__ __forceinline__ void hc_issue_stage(const HcArgs& a, const float* x, float* slot,
                                               int st, int rows, int hc_dim) {
  const int chunk = a.chunk, ld = chunk + 4;
  const int c0 = st * chunk, ncol = min(chunk, hc_dim - c0);
  const int cw = a.vec4 ? 4 : 1;
  const int per_row = (ncol + cw - 1) / cw;
  for (int i = threadIdx.x; i < (rows + 1) * per_row; i += blockDim.x) {
    const int r = i / per_row, c = (i - r * per_row) * cw;
    const float* src = r == 0 ? x + c0 + c : a.fn + (long long)(r - 1) * hc_dim + c0 + c;
    hc_cp_async(slot + r * ld + c, src, a.vec4);
  }
}

// hc_pre (head == 0) or hc_head (head == 1) for token blockIdx.x
__global__ void __launch_bounds__(kHcThreads) hc_mix_kernel(HcArgs a) {
  extern __shared__ __align__(16) float hc_ring[];  // [kHcStages][rows + 1][chunk + 4]
  __shared__ float s_dot[1 + kHcMaxMix];
  __shared__ float s_pre[kHcMaxHc], s_post[kHcMaxHc], s_comb[kHcMaxHc * kHcMaxHc];
  const int t = blockIdx.x, tid = threadIdx.x;
  const int hc = a.hc, hidden = a.hidden, hc_dim = hc * hidden;
  const int rows = a.head ? hc : (2 + hc) * hc;
  const float* x = a.x + (long long)t * hc_dim;
  const int ld = a.chunk + 4, slot_floats = (rows + 1) * ld;
  const int nst = (hc_dim + a.chunk - 1) / a.chunk;
  pdl_wait_prior();
  // chain 0: sum of squares (x . x); chain 1 + j: fn_j . x; the columns stream
  // through a cp.async ring that every thread fills
#pragma unroll
  for (int st = 0; st < kHcStages - 1; ++st) {
    if (st < nst) hc_issue_stage(a, x, hc_ring + st * slot_floats, st, rows, hc_dim);
    hc_cp_commit();
  }
  const bool chain = tid <= rows;
  float acc = 0.0f;
  for (int st = 0; st < nst; ++st) {
    hc_cp_wait<kHcStages - 2>();
    __syncthreads();  // stage st landed for every thread; slot st - 1 is free
    const int nx = st + kHcStages - 1;
    if (nx < nst) hc_issue_stage(a, x, hc_ring + (nx % kHcStages) * slot_floats, nx, rows, hc_dim);
    hc_cp_commit();
    if (chain) {
      const float* slot = hc_ring + (st % kHcStages) * slot_floats;
      const float* xr = slot;             // row 0: x
      const float* wr = slot + tid * ld;  // this chain's row (x itself for chain 0)
      const int ncol = min(a.chunk, hc_dim - st * a.chunk);
      int i = 0;
#pragma unroll 4
      for (; i + 4 <= ncol; i += 4) {
        const float4 wv = *reinterpret_cast<const float4*>(wr + i);
        const float4 xv = *reinterpret_cast<const float4*>(xr + i);
        acc = __fadd_rn(acc, __fmul_rn(wv.x, xv.x));
        acc = __fadd_rn(acc, __fmul_rn(wv.y, xv.y));
        acc = __fadd_rn(acc, __fmul_rn(wv.z, xv.z));
        acc = __fadd_rn(acc, __fmul_rn(wv.w, xv.w));
      }
      for (; i < ncol; ++i) acc = __fadd_rn(acc, __fmul_rn(wr[i], xr[i]));
    }
  }
  hc_cp_wait<0>();
  if (chain) s_dot[tid] = acc;
  __syncthreads();
  if (tid == 0) {
    const float eps = a.eps;
    const float mean_square = __fdiv_rn(s_dot[0], (float)hc_dim);
    const float inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean_square, eps)));
    if (a.head) {
      for (int j = 0; j < hc; ++j) {
        const float mix = __fmul_rn(s_dot[1 + j], inv_rms);
        s_pre[j] =
            __fadd_rn(hc_sigmoid(__fadd_rn(__fmul_rn(mix, a.head_scale), a.base[j])), eps);
      }
    } else {
      float* mix = s_dot + 1;
      for (int j = 0; j < rows; ++j) mix[j] = __fmul_rn(mix[j], inv_rms);
      const float s0 = a.scale[0], s1 = a.scale[1], s2 = a.scale[2];
      for (int j = 0; j < hc; ++j) {
        s_pre[j] = __fadd_rn(hc_sigmoid(__fadd_rn(__fmul_rn(mix[j], s0), a.base[j])), eps);
        s_post[j] = __fmul_rn(
            2.0f, hc_sigmoid(__fadd_rn(__fmul_rn(mix[j + hc], s1), a.base[j + hc])));
      }
      float* comb = s_comb;
      for (int j = 0; j < hc * hc; ++j)
        comb[j] = __fadd_rn(__fmul_rn(mix[2 * hc + j], s2), a.base[2 * hc + j]);
      // comb = softmax(comb, rows) + eps
      for (int j = 0; j < hc; ++j) {
        float* row = comb + j * hc;
        float mx = -INFINITY;
        for (int k = 0; k < hc; ++k) mx = fmaxf(mx, row[k]);
        float sum = 0.0f;
        for (int k = 0; k < hc; ++k) {
          row[k] = libm_expf(__fsub_rn(row[k], mx));
          sum = __fadd_rn(sum, row[k]);
        }
        for (int k = 0; k < hc; ++k) row[k] = __fadd_rn(__fdiv_rn(row[k], sum), eps);
      }
      // the column normalisation, then (iters - 1) row/column rounds
      for (int it = 0; it < (a.iters > 1 ? a.iters : 1); ++it) {
        if (it > 0)
          for (int j = 0; j < hc; ++j) {
            float sum = 0.0f;
            for (int k = 0; k < hc; ++k) sum = __fadd_rn(sum, comb[j * hc + k]);
            const float den = __fadd_rn(sum, eps);
            for (int k = 0; k < hc; ++k) comb[j * hc + k] = __fdiv_rn(comb[j * hc + k], den);
          }
        for (int k = 0; k < hc; ++k) {
          float sum = 0.0f;
          for (int j = 0; j < hc; ++j) sum = __fadd_rn(sum, comb[j * hc + k]);
          const float den = __fadd_rn(sum, eps);
          for (int j = 0; j < hc; ++j) comb[j * hc + k] = __fdiv_rn(comb[j * hc + k], den);
        }
      }
      for (int j = 0; j < hc; ++j) a.post[(long long)t * hc + j] = s_post[j];
      for (int j = 0; j < hc * hc; ++j) a.comb[(long long)t * hc * hc + j] = comb[j];
    }
  }
  __syncthreads();
  for (int d = tid; d < hidden; d += blockDim.x) {
    float acc = 0.0f;
    for (int i = 0; i < hc; ++i) acc = __fadd_rn(acc, __fmul_rn(s_pre[i], x[i * hidden + d]));
    a.y[(long long)t * hidden + d] = acc;
  }
  pdl_launch_dependents();
}

// out[t][k][d] = post[t][k] y[t][d] + sum_i comb[t][k][i] res[t][i][d]
__global__ void __launch_bounds__(kHcThreads) hc_post_kernel(HcPostArgs a) {
  const int hc = a.hc, hidden = a.hidden, hc_dim = hc * hidden;
  const long long n = (long long)a.tokens * hc_dim;
  pdl_wait_prior();
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const long long t = e / hc_dim;
    const int r = (int)(e - t * hc_dim), k = r / hidden, d = r - k * hidden;
    const float* comb = a.comb + t * hc * hc + (long long)k * hc;
    const float* res = a.residual + t * hc_dim + d;
    float acc = __fmul_rn(a.post[t * hc + k], a.y[t * hidden + d]);
    for (int i = 0; i < hc; ++i) acc = __fadd_rn(acc, __fmul_rn(comb[i], res[(long long)i * hidden]));
    a.out[e] = acc;
  }
  pdl_launch_dependents();
}

// Columns per ring stage: the largest power of two up to 512 whose three
// stages of (rows + 1) padded rows fit 200 KB.
int hc_chunk(int rows) {
  int chunk = 512;
  while (chunk > 16 && (size_t)kHcStages * (rows + 1) * (chunk + 4) * sizeof(float) > 200 * 1024)
    chunk >>= 1;
  return chunk;
}

size_t hc_mix_smem(int rows, int chunk) {
  return (size_t)kHcStages * (rows + 1) * (chunk + 4) * sizeof(float);
}

cudaError_t launch_hc_mix(const HcArgs& a, cudaStream_t s) {
  const int rows = a.head ? a.hc : (2 + a.hc) * a.hc;
  const size_t smem = hc_mix_smem(rows, a.chunk);
  cudaError_t e = ensure_smem(hc_mix_kernel, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(a.tokens);
  cfg.blockDim = dim3(kHcThreads);
  cfg.dynamicSmemBytes = smem;
  return cudaLaunchKernelEx(&cfg, hc_mix_kernel, a);
}

cudaError_t launch_hc_post(const HcPostArgs& a, int num_sms, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const long long n = (long long)a.tokens * a.hc * a.hidden;
  cfg.gridDim = dim3((unsigned)std::min<long long>((n + kHcThreads - 1) / kHcThreads,
                                                   8LL * num_sms));
  cfg.blockDim = dim3(kHcThreads);
  return cudaLaunchKernelEx(&cfg, hc_post_kernel, a);
}

}  // namespace wh
