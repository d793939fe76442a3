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
// additions (16384 for V4: about 37 us at 4.4 cycles an add).  hc_dots_kernel
// runs each chain in a CTA of its own (25 CTAs per token for V4); the split
// kernel then runs the Sinkhorn (or the head gates) and the pooled output;
// hc_post is elementwise.
#include "common.cuh"
#include "kernels.cuh"

namespace wh {

constexpr int kHcThreads = 256;
constexpr int kHcChunk = 512;  // columns per ring stage
constexpr int kHcRing = 8;     // ring stages (32 KB of shared memory)

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

// One chain per CTA: CTA (c, t) computes chain c of token t -- c = 0 is x . x,
// c = 1 + j is fn_j . x -- with the columns of its row and of x streamed
// through a cp.async ring that the whole CTA fills (one 16-byte copy per
// thread per stage); thread 0 runs the chain.  One SM alone cannot keep enough
// plain loads in flight to feed 25 chains from HBM, so the chains are spread
// over 25 SMs, each needing about 4 GB/s.
__global__ void __launch_bounds__(kHcThreads) hc_dots_kernel(HcArgs a) {
  __shared__ __align__(16) float ring[kHcRing][2][kHcChunk];
  const int c = blockIdx.x, t = blockIdx.y, tid = threadIdx.x;
  const int hc_dim = a.hc * a.hidden;
  const int rows = a.head ? a.hc : (2 + a.hc) * a.hc;
  const float* x = a.x + (long long)t * hc_dim;
  const float* w = c == 0 ? x : a.fn + (long long)(c - 1) * hc_dim;
  const int nst = (hc_dim + kHcChunk - 1) / kHcChunk;
  pdl_wait_prior();
  auto issue = [&](int st) {
    const int c0 = st * kHcChunk, ncol = min(kHcChunk, hc_dim - c0);
    float* slot = &ring[st % kHcRing][0][0];
    if (a.vec4) {
      const int per_row = ncol / 4;
      for (int i = tid; i < 2 * per_row; i += blockDim.x) {
        const int r = i / per_row, col = (i - r * per_row) * 4;
        hc_cp_async(slot + r * kHcChunk + col, (r ? x : w) + c0 + col, true);
      }
    } else {
      for (int i = tid; i < 2 * ncol; i += blockDim.x) {
        const int r = i / ncol, col = i - r * ncol;
        hc_cp_async(slot + r * kHcChunk + col, (r ? x : w) + c0 + col, false);
      }
    }
  };
#pragma unroll 1
  for (int st = 0; st < kHcRing - 1; ++st) {
    if (st < nst) issue(st);
    hc_cp_commit();
  }
  float acc = 0.0f;
#pragma unroll 1
  for (int st = 0; st < nst; ++st) {
    hc_cp_wait<kHcRing - 2>();
    __syncthreads();  // stage st landed for every thread; slot st - 1 is free
    if (st + kHcRing - 1 < nst) issue(st + kHcRing - 1);
    hc_cp_commit();
    if (tid == 0) {
      const float* wr = &ring[st % kHcRing][0][0];
      const float* xr = &ring[st % kHcRing][1][0];
      const int ncol = min(kHcChunk, hc_dim - st * kHcChunk);
      int i = 0;
      if (ncol == kHcChunk) {
        // the products of 16 columns formed ahead of their additions
#pragma unroll 2
        for (; i < kHcChunk; i += 16) {
          float pr[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 wv = *reinterpret_cast<const float4*>(wr + i + 4 * q);
            const float4 xv = *reinterpret_cast<const float4*>(xr + i + 4 * q);
            pr[4 * q] = __fmul_rn(wv.x, xv.x);
            pr[4 * q + 1] = __fmul_rn(wv.y, xv.y);
            pr[4 * q + 2] = __fmul_rn(wv.z, xv.z);
            pr[4 * q + 3] = __fmul_rn(wv.w, xv.w);
          }
#pragma unroll
          for (int q = 0; q < 16; ++q) acc = __fadd_rn(acc, pr[q]);
        }
      }
      for (; i < ncol; ++i) acc = __fadd_rn(acc, __fmul_rn(wr[i], xr[i]));
    }
  }
  hc_cp_wait<0>();
  if (tid == 0) a.dots[(long long)t * (rows + 1) + c] = acc;
  pdl_launch_dependents();
}

// The split (hc_pre: Sinkhorn; hc_head: sigmoid gates) and the pooled output
// of token blockIdx.x from its chain results.  Elementwise steps run one thread
// per element; every sum (a softmax row, a Sinkhorn row or column) runs in the
// reference's order on one thread.  With hc * hc <= 32 the Sinkhorn runs in one
// warp, each lane gathering its row and column by shuffles; larger hc takes
// block barriers between the steps.
__global__ void __launch_bounds__(kHcThreads) hc_split_kernel(HcArgs a) {
  __shared__ float s_dot[1 + kHcMaxMix], s_base[kHcMaxMix];
  __shared__ float s_pre[kHcMaxHc], s_comb[kHcMaxHc * kHcMaxHc], s_sum[kHcMaxHc];
  __shared__ float s_scale[3], s_inv;
  const int t = blockIdx.x, tid = threadIdx.x;
  const int hc = a.hc, hidden = a.hidden, hc_dim = hc * hidden, hh = hc * hc;
  const int rows = a.head ? hc : (2 + hc) * hc;
  const float* x = a.x + (long long)t * hc_dim;
  const float eps = a.eps;
  pdl_wait_prior();
  for (int i = tid; i <= rows; i += blockDim.x) s_dot[i] = a.dots[(long long)t * (rows + 1) + i];
  for (int i = tid; i < rows; i += blockDim.x) s_base[i] = a.base[i];
  if (!a.head && tid < 3) s_scale[tid] = a.scale[tid];
  __syncthreads();
  if (tid == 0) {
    const float mean_square = __fdiv_rn(s_dot[0], (float)hc_dim);
    s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean_square, eps)));
  }
  __syncthreads();
  const float inv_rms = s_inv;
  if (a.head) {
    if (tid < hc) {
      const float mix = __fmul_rn(s_dot[1 + tid], inv_rms);
      s_pre[tid] =
          __fadd_rn(hc_sigmoid(__fadd_rn(__fmul_rn(mix, a.head_scale), s_base[tid])), eps);
    }
  } else {
    const float* mix = s_dot + 1;  // scaled by inv_rms where used
    if (tid < hc) {
      const int j = tid;
      s_pre[j] = __fadd_rn(
          hc_sigmoid(__fadd_rn(__fmul_rn(__fmul_rn(mix[j], inv_rms), s_scale[0]), s_base[j])),
          eps);
      a.post[(long long)t * hc + j] = __fmul_rn(
          2.0f, hc_sigmoid(__fadd_rn(__fmul_rn(__fmul_rn(mix[j + hc], inv_rms), s_scale[1]),
                                     s_base[j + hc])));
    }
    if (hh <= 32) {
      // one warp: lane = comb element (j, k); each lane forms its row's and its
      // column's sums itself, in the reference's order, from shuffles
      if (tid < 32) {
        const int lane = tid, j = lane / hc, k = lane % hc;
        const bool on = lane < hh;
        float v = on ? __fadd_rn(__fmul_rn(__fmul_rn(mix[2 * hc + lane], inv_rms), s_scale[2]),
                                 s_base[2 * hc + lane])
                     : 0.0f;
        float mx = -INFINITY;
        for (int kk = 0; kk < hc; ++kk)
          mx = fmaxf(mx, __shfl_sync(0xffffffffu, v, (j * hc + kk) & 31));
        v = on ? libm_expf(__fsub_rn(v, mx)) : 0.0f;
        float sum = 0.0f;
        for (int kk = 0; kk < hc; ++kk)
          sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, v, (j * hc + kk) & 31));
        v = __fadd_rn(__fdiv_rn(v, sum), eps);
        for (int it = 0; it < (a.iters > 1 ? a.iters : 1); ++it) {
          if (it > 0) {
            float rs = 0.0f;
            for (int kk = 0; kk < hc; ++kk)
              rs = __fadd_rn(rs, __shfl_sync(0xffffffffu, v, (j * hc + kk) & 31));
            v = __fdiv_rn(v, __fadd_rn(rs, eps));
          }
          float cs = 0.0f;
          for (int jj = 0; jj < hc; ++jj)
            cs = __fadd_rn(cs, __shfl_sync(0xffffffffu, v, (jj * hc + k) & 31));
          v = __fdiv_rn(v, __fadd_rn(cs, eps));
        }
        if (on) s_comb[lane] = v;
      }
      __syncthreads();
    } else {
      if (tid < hh)
        s_comb[tid] = __fadd_rn(__fmul_rn(__fmul_rn(mix[2 * hc + tid], inv_rms), s_scale[2]),
                                s_base[2 * hc + tid]);
      __syncthreads();
      // comb = softmax(comb, rows) + eps: the row max on the row's thread
      if (tid < hc) {
        float mx = -INFINITY;
        for (int k = 0; k < hc; ++k) mx = fmaxf(mx, s_comb[tid * hc + k]);
        s_sum[tid] = mx;
      }
      __syncthreads();
      if (tid < hh) s_comb[tid] = libm_expf(__fsub_rn(s_comb[tid], s_sum[tid / hc]));
      __syncthreads();
      if (tid < hc) {
        float sum = 0.0f;
        for (int k = 0; k < hc; ++k) sum = __fadd_rn(sum, s_comb[tid * hc + k]);
        s_sum[tid] = sum;
      }
      __syncthreads();
      if (tid < hh) s_comb[tid] = __fadd_rn(__fdiv_rn(s_comb[tid], s_sum[tid / hc]), eps);
      // the column normalisation, then (iters - 1) row/column rounds
      for (int it = 0; it < (a.iters > 1 ? a.iters : 1); ++it) {
        if (it > 0) {
          __syncthreads();
          if (tid < hc) {
            float sum = 0.0f;
            for (int k = 0; k < hc; ++k) sum = __fadd_rn(sum, s_comb[tid * hc + k]);
            s_sum[tid] = __fadd_rn(sum, eps);
          }
          __syncthreads();
          if (tid < hh) s_comb[tid] = __fdiv_rn(s_comb[tid], s_sum[tid / hc]);
        }
        __syncthreads();
        if (tid < hc) {
          float sum = 0.0f;
          for (int j = 0; j < hc; ++j) sum = __fadd_rn(sum, s_comb[j * hc + tid]);
          s_sum[tid] = __fadd_rn(sum, eps);
        }
        __syncthreads();
        if (tid < hh) s_comb[tid] = __fdiv_rn(s_comb[tid], s_sum[tid % hc]);
      }
    }
    if (tid < hh) a.comb[(long long)t * hh + tid] = s_comb[tid];
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

cudaError_t launch_hc_mix(const HcArgs& a, cudaStream_t s) {
  const int rows = a.head ? a.hc : (2 + a.hc) * a.hc;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(rows + 1, a.tokens);
  cfg.blockDim = dim3(kHcThreads);
  cudaError_t e = cudaLaunchKernelEx(&cfg, hc_dots_kernel, a);
  if (e != cudaSuccess) return e;
  cfg.gridDim = dim3(a.tokens);
  return cudaLaunchKernelEx(&cfg, hc_split_kernel, a);
}

size_t hc_dots_bytes(int tokens, int rows) {
  return sizeof(float) * (size_t)tokens * (rows + 1);
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
