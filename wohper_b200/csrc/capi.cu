// capi.cu -- the extern "C" boundary (include/wohper_b200.h): argument
// validation in the reference's error order, tensor-map construction, plan /
// context management and kernel dispatch.  Host code only.
#include <cudaTypedefs.h>
#include <math.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/wohper_b200.h"
#include "common.cuh"
#include "kernels.cuh"

namespace wh {
cudaError_t launch_router_ex(const RouterArgs& a, __half* xq, float* xq_mult, cudaStream_t s,
                             bool pdl);
cudaError_t launch_moe_up_ex(const MoeArgs& a, const __half* xq, const float* xq_mult, __half* hq,
                             float* hq_mult, cudaStream_t s, bool pdl);
cudaError_t launch_moe_down_ex(const MoeArgs& a, const __half* hq, const float* hq_mult,
                               cudaStream_t s, bool pdl);
cudaError_t launch_xq(const float* x, int n, int tokens, __half* xq, float* xq_mult,
                      cudaStream_t s);
cudaError_t launch_swiglu(float* gate, const float* up, int n, uint32_t* status, cudaStream_t s);
cudaError_t launch_stage_rows(const float* src, float* dst, size_t n, cudaStream_t s);
}  // namespace wh

using namespace wh;

namespace {

thread_local std::string g_detail;

wh_status fail(wh_status st, const std::string& why) {
  g_detail = why;
  return st;
}
wh_status cuda_fail(cudaError_t e, const char* where) {
  g_detail = std::string(where) + ": " + cudaGetErrorString(e);
  return WH_ERR_CUDA;
}
#define WH_CUDA(call)                                   \
  do {                                                  \
    cudaError_t e_ = (call);                            \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
  } while (0)

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// 0: device (or managed) memory; 1: pinned host memory the device reaches at
// the same address; -1: neither (pageable host memory, or not a valid pointer)
int device_reach(const void* p) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) return 0;
  if (at.type == cudaMemoryTypeHost) return at.devicePointer == p ? 1 : -1;
  return -1;
}

// ---------------------------------------------------------------------------
// Act-quant threshold table: ceilf(log2f(q)) == k for q = 2^k * (1 + m/2^23)
// exactly when m == 0 or m < thr[E] (E = k + 127); measured with the host
// libm log2f, which is what the reference engine calls.
// ---------------------------------------------------------------------------
ActQuantTable build_act_quant_table() {
  ActQuantTable t;
  for (int E = 0; E < 256; ++E) {
    t.thr[E] = 0;
    if (E == 0 || E == 255) continue;
    const int k = E - 127;
    auto ceil_is_k = [&](uint32_t m) {
      float q = u2f((uint32_t(E) << 23) | m);
      return ceilf(log2f(q)) == (float)k;
    };
    // smallest m in [1, 2^23) with ceil(log2f(q)) != k  (log2f is monotonic)
    uint32_t lo = 1, hi = 1u << 23;
    if (!ceil_is_k(1)) {
      t.thr[E] = 1;
      continue;
    }
    while (hi - lo > 1) {
      uint32_t mid = lo + (hi - lo) / 2;
      if (ceil_is_k(mid))
        lo = mid;
      else
        hi = mid;
    }
    t.thr[E] = hi;
  }
  return t;
}
const ActQuantTable& act_quant_table_host() {
  static ActQuantTable t = build_act_quant_table();
  return t;
}

// ---------------------------------------------------------------------------
// Tensor maps
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// u8 matrix [rows][row_bytes], box [box_rows][box_bytes]: 128-byte swizzle
// for 128-byte boxes (the layout the kernels read back), none otherwise.
wh_status make_u8_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes,
                      uint32_t box_rows, uint32_t box_bytes = 128) {
  auto fn = encode_fn();
  if (!fn) return fail(WH_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_bytes, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d) rows=%llu row_bytes=%llu",
             (int)r, (unsigned long long)rows, (unsigned long long)row_bytes);
    return fail(WH_ERR_CUDA, buf);
  }
  return WH_OK;
}

// f32 matrix [height][width], rows ld floats apart: box [16 rows][136 floats],
// no swizzle (the batched FP8 GEMV's input tiles; 136 = a 128-column group
// plus 8 floats that pad each row of the tile onto other banks).  Returns
// false, recording nothing, when the driver refuses the map (the caller then
// runs the generic kernel).
bool make_f32_xmap(CUtensorMap* map, const float* base, uint64_t width, uint64_t height,
                   uint64_t ld) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {width, height};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {136, 16};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// validate_fp4_matvec (src/deepseek_v4.rs:434-462)
wh_status validate_fp4(const wh_fp4_matvec_spec& s, size_t input_len, size_t output_len) {
  if (s.rows == 0 || s.cols == 0 || s.scale_cols == 0) return fail(WH_ERR_EMPTY_SHAPE, "empty shape");
  if (input_len < s.cols) return fail(WH_ERR_INPUT_TOO_SMALL, "input too small");
  if (output_len < s.rows) return fail(WH_ERR_OUTPUT_TOO_SMALL, "output too small");
  if (s.cols % s.scale_cols != 0) return fail(WH_ERR_INVALID_SHAPE, "cols % scale_cols != 0");
  const size_t row_bytes = (s.cols + 1) / 2;
  if (s.rows > SIZE_MAX / row_bytes) return fail(WH_ERR_INVALID_SHAPE, "weight size overflow");
  if (s.packed_len < s.rows * row_bytes)
    return fail(WH_ERR_PACKED_WEIGHT_TOO_SMALL, "packed weight too small");
  if (s.rows > SIZE_MAX / s.scale_cols) return fail(WH_ERR_INVALID_SHAPE, "scale size overflow");
  if (s.scales_len < s.rows * s.scale_cols) return fail(WH_ERR_SCALE_TOO_SMALL, "scales too small");
  if (!s.packed_weight || !s.ue8m0_scales) return fail(WH_ERR_INVALID_POINTER, "null weight");
  if (s.rows > 0x7fffffff || s.cols > 0x7fffffff) return fail(WH_ERR_UNSUPPORTED, "shape > 2^31");
  return WH_OK;
}

// Fast (TMA) path shape rule for an expert: 32-column groups, box-aligned rows.
bool expert_fast_ok(const wh_fp4_expert& e, size_t hidden, size_t inter) {
  auto ok = [](const wh_fp4_matvec_spec& s) {
    return s.cols % 32 == 0 && s.scale_cols == s.cols / 32 && aligned(s.packed_weight, 16) &&
           aligned(s.ue8m0_scales, 16);
  };
  return ok(e.w1) && ok(e.w3) && ok(e.w2) && hidden % 256 == 0 && inter % 256 == 0 &&
         hidden % 16 == 0 && hidden <= 16384 && inter <= 16384;
}

struct DevExpertSet {
  CUtensorMap* maps = nullptr;      // device [n][3]
  Fp4ExpertDev* experts = nullptr;  // device [n]
  CUtensorMap* gmaps = nullptr;     // device [n][3], grouped-GEMM boxes (nullable)
  CUtensorMap* dmaps = nullptr;     // device [n], w2 boxes [8 rows][128 B] (decode kernel)
  int n = 0;
};

wh_status build_expert_set(const wh_fp4_expert* list, int n, DevExpertSet* out) {
  std::vector<CUtensorMap> maps(size_t(n) * 3), dmaps(n);
  std::vector<Fp4ExpertDev> ex(n);
  for (int i = 0; i < n; ++i) {
    const wh_fp4_expert& e = list[i];
    wh_status st;
    if ((st = make_u8_map(&dmaps[i], e.w2.packed_weight, e.w2.rows, e.w2.cols / 2,
                          kDecDownRows)))
      return st;
    if ((st = make_u8_map(&maps[i * 3 + 0], e.w1.packed_weight, e.w1.rows, e.w1.cols / 2,
                          kMoeUpRows)))
      return st;
    if ((st = make_u8_map(&maps[i * 3 + 1], e.w3.packed_weight, e.w3.rows, e.w3.cols / 2,
                          kMoeUpRows)))
      return st;
    if ((st = make_u8_map(&maps[i * 3 + 2], e.w2.packed_weight, e.w2.rows, e.w2.cols / 2,
                          kMoeDownRows)))
      return st;
    ex[i] = Fp4ExpertDev{e.w1.ue8m0_scales, e.w3.ue8m0_scales, e.w2.ue8m0_scales,
                         e.w1.packed_weight, e.w3.packed_weight, e.w2.packed_weight};
  }
  WH_CUDA(cudaMalloc(&out->maps, maps.size() * sizeof(CUtensorMap)));
  WH_CUDA(cudaMalloc(&out->dmaps, dmaps.size() * sizeof(CUtensorMap)));
  WH_CUDA(cudaMalloc(&out->experts, ex.size() * sizeof(Fp4ExpertDev)));
  WH_CUDA(cudaMemcpy(out->maps, maps.data(), maps.size() * sizeof(CUtensorMap),
                     cudaMemcpyHostToDevice));
  WH_CUDA(cudaMemcpy(out->dmaps, dmaps.data(), dmaps.size() * sizeof(CUtensorMap),
                     cudaMemcpyHostToDevice));
  WH_CUDA(cudaMemcpy(out->experts, ex.data(), ex.size() * sizeof(Fp4ExpertDev),
                     cudaMemcpyHostToDevice));
  out->n = n;
  return WH_OK;
}
void free_expert_set(DevExpertSet& s) {
  if (s.maps) cudaFree(s.maps);
  if (s.experts) cudaFree(s.experts);
  if (s.gmaps) cudaFree(s.gmaps);
  if (s.dmaps) cudaFree(s.dmaps);
  s = DevExpertSet{};
}

// u8 matrix whose rows are `row_bytes` long but only the first `cols` bytes
// are loaded: box [box_rows][128 B], 128-byte swizzle.
wh_status make_u8_map_strided(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                              uint64_t row_bytes, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(WH_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(WH_ERR_CUDA, "cuTensorMapEncodeTiled (strided) failed");
  return WH_OK;
}

// Whether any expert scale byte is 0 or 255 (device scan of every matrix).
wh_status scan_scale_bytes(const Fp4ExpertDev* ex, int n, int hidden, int inter, int* bad) {
  uint32_t* flag = nullptr;
  WH_CUDA(cudaMalloc(&flag, sizeof(uint32_t)));
  uint32_t h = 1;
  cudaError_t e = cudaMemset(flag, 0, sizeof(uint32_t));
  if (e == cudaSuccess) e = launch_scale_check(ex, n, hidden, inter, flag, nullptr);
  if (e == cudaSuccess) e = cudaMemcpy(&h, flag, sizeof h, cudaMemcpyDeviceToHost);
  cudaFree(flag);
  if (e != cudaSuccess) return cuda_fail(e, "scale scan");
  *bad = h != 0;
  return WH_OK;
}

// Grouped-GEMM tensor maps: FP4 tiles of 128 rows x 128 K (64 B), unswizzled.
wh_status build_grouped_maps(const wh_fp4_expert* list, int n, DevExpertSet* out) {
  std::vector<CUtensorMap> maps(size_t(n) * 3);
  for (int i = 0; i < n; ++i) {
    const wh_fp4_matvec_spec* m[3] = {&list[i].w1, &list[i].w3, &list[i].w2};
    for (int j = 0; j < 3; ++j) {
      wh_status st = make_u8_map(&maps[i * 3 + j], m[j]->packed_weight, m[j]->rows,
                                 m[j]->cols / 2, 128, 64);
      if (st != WH_OK) return st;
    }
  }
  WH_CUDA(cudaMalloc(&out->gmaps, maps.size() * sizeof(CUtensorMap)));
  WH_CUDA(cudaMemcpy(out->gmaps, maps.data(), maps.size() * sizeof(CUtensorMap),
                     cudaMemcpyHostToDevice));
  return WH_OK;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

struct wh_ctx {
  int device = 0;
  int num_sms = 148;
  uint32_t* status = nullptr;    // device word: WH_DEV_* bits
  uint32_t* counters = nullptr;  // device, router last-CTA counters (zero at rest)
  int counters_len = 0;
  uint32_t* blk_counters = nullptr;  // device, moe_up act-quant block counters (zero at rest)
  int blk_counters_len = 0;
  void* work = nullptr;  // generic-path workspace
  size_t work_bytes = 0;
  std::map<std::tuple<const void*, int, int, int>, CUtensorMap> fp8_maps;
  // batched FP8 GEMV inputs: (x, width, batch, ldx) -> map of box [16][136] f32
  std::map<std::tuple<const void*, long long, int, int>, CUtensorMap> fp8_xmaps;
  std::map<std::tuple<const void*, const void*, const void*, size_t, size_t>, DevExpertSet> experts;
  bool profile = false;
  std::vector<cudaEvent_t> ev;  // 2 per phase
  int phases = 0;

  bool pdl() const { return !profile; }
  void prof_begin() { phases = 0; }
  wh_status prof_mark(cudaStream_t s) {  // call before the first and after every kernel
    if (!profile) return WH_OK;
    if ((int)ev.size() <= phases) {
      cudaEvent_t e;
      WH_CUDA(cudaEventCreate(&e));
      ev.push_back(e);
    }
    WH_CUDA(cudaEventRecord(ev[phases], s));
    ++phases;
    return WH_OK;
  }

  void* hc_work = nullptr;  // mHC chain results
  size_t hc_work_bytes = 0;
  wh_status ensure_hc_work(size_t bytes) {
    if (bytes <= hc_work_bytes) return WH_OK;
    if (hc_work) cudaFree(hc_work);
    hc_work = nullptr;
    hc_work_bytes = 0;
    WH_CUDA(cudaMalloc(&hc_work, bytes));
    hc_work_bytes = bytes;
    return WH_OK;
  }
  void* mla_work = nullptr;  // MLA scores and tile maxima
  size_t mla_work_bytes = 0;
  wh_status ensure_mla_work(size_t bytes) {
    if (bytes <= mla_work_bytes) return WH_OK;
    if (mla_work) cudaFree(mla_work);
    mla_work = nullptr;
    mla_work_bytes = 0;
    WH_CUDA(cudaMalloc(&mla_work, bytes));
    mla_work_bytes = bytes;
    return WH_OK;
  }
  wh_status ensure_work(size_t bytes) {
    if (bytes <= work_bytes) return WH_OK;
    if (work) cudaFree(work);
    work = nullptr;
    work_bytes = 0;
    WH_CUDA(cudaMalloc(&work, bytes));
    work_bytes = bytes;
    return WH_OK;
  }
  wh_status ensure_blk_counters(int n) {
    if (n <= blk_counters_len) return WH_OK;
    if (blk_counters) cudaFree(blk_counters);
    blk_counters = nullptr;
    blk_counters_len = 0;
    WH_CUDA(cudaMalloc(&blk_counters, sizeof(uint32_t) * n));
    WH_CUDA(cudaMemset(blk_counters, 0, sizeof(uint32_t) * n));
    blk_counters_len = n;
    return WH_OK;
  }
  wh_status ensure_counters(int n) {
    if (n <= counters_len) return WH_OK;
    if (counters) cudaFree(counters);
    counters = nullptr;
    counters_len = 0;
    WH_CUDA(cudaMalloc(&counters, sizeof(uint32_t) * n));
    WH_CUDA(cudaMemset(counters, 0, sizeof(uint32_t) * n));
    counters_len = n;
    return WH_OK;
  }
};

struct wh_moe_plan {
  wh_ctx* ctx = nullptr;
  wh_moe_desc d{};
  DevExpertSet set;  // routed experts, then the shared expert
  uint32_t* counters = nullptr;      // router: [max_tokens]
  uint32_t* blk_counters = nullptr;  // moe_up: [max_tokens][slots][inter/64]
  bool grouped = false;              // tensor-core path available (desc.exact == 0)
  uint32_t* dec_sync = nullptr;      // decode kernel's grid counters [4] (zero at rest)
  int decode_ok = -1;                // one-token persistent kernel: -1 not checked yet
  bool decode_on = false;            // wh_moe_plan_set_fused_decode (opt-in)
  bool has_sfp8 = false;             // an FP8 shared expert (run after the routed path)
  wh_fp8_expert sfp8{};
};

extern "C" {

int wh_version(void) { return 200; }

const char* wh_last_error_detail(void) { return g_detail.c_str(); }

wh_status wh_ctx_create(int device, wh_ctx** out) {
  if (!out) return fail(WH_ERR_INVALID_POINTER, "out is null");
  *out = nullptr;
  WH_CUDA(cudaSetDevice(device));
  int major = 0, minor = 0;
  WH_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  WH_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
  if (major != 10 || minor != 0)
    return fail(WH_ERR_UNSUPPORTED, "wohper_b200 kernels are built for sm_100a (B200)");
  wh_ctx* c = new wh_ctx();
  c->device = device;
  cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  cudaError_t e = cudaMalloc(&c->status, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(c->status, 0, sizeof(uint32_t));
  if (e != cudaSuccess) {
    delete c;
    return cuda_fail(e, "status word");
  }
  set_act_quant_table(act_quant_table_host(), nullptr);
  cudaError_t te = cudaSuccess;
  if (!install_expf_table(&te)) {
    cudaFree(c->status);
    delete c;
    return fail(WH_ERR_UNSUPPORTED, "host expf differs outside the device's midpoint gate");
  }
  e = te != cudaSuccess ? te : cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(c->status);
    delete c;
    return cuda_fail(e, "act quant table upload");
  }
  *out = c;
  return WH_OK;
}

void wh_ctx_destroy(wh_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  for (auto& kv : c->experts) free_expert_set(kv.second);
  for (auto e : c->ev) cudaEventDestroy(e);
  if (c->status) cudaFree(c->status);
  if (c->counters) cudaFree(c->counters);
  if (c->blk_counters) cudaFree(c->blk_counters);
  if (c->work) cudaFree(c->work);
  if (c->mla_work) cudaFree(c->mla_work);
  if (c->hc_work) cudaFree(c->hc_work);
  delete c;
}

wh_status wh_ctx_sync(wh_ctx* c, wh_stream_t stream) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "ctx is null");
  WH_CUDA(cudaStreamSynchronize(stream));
  uint32_t st = 0;
  WH_CUDA(cudaMemcpy(&st, c->status, sizeof st, cudaMemcpyDeviceToHost));
  if (st == 0) return WH_OK;
  WH_CUDA(cudaMemset(c->status, 0, sizeof st));
  if (st & WH_DEV_TIMEOUT) return fail(WH_ERR_TIMEOUT, "a device-side wait timed out");
  if (st & WH_DEV_BADARG) return fail(WH_ERR_DEVICE_ARG, "device-side index check failed");
  return fail(WH_ERR_NON_FINITE_OUTPUT, "non-finite output");
}

wh_status wh_ctx_set_profiling(wh_ctx* c, int on) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "ctx is null");
  c->profile = on != 0;
  c->phases = 0;
  return WH_OK;
}

int wh_ctx_phase_times(wh_ctx* c, float* ms, int max_phases) {
  if (!c || !c->profile || c->phases < 2) return 0;
  if (cudaEventSynchronize(c->ev[c->phases - 1]) != cudaSuccess) return 0;
  int n = 0;
  for (int i = 0; i + 1 < c->phases && n < max_phases; ++i, ++n)
    cudaEventElapsedTime(&ms[n], c->ev[i], c->ev[i + 1]);
  return n;
}

// ---------------------------------------------------------------------------
wh_status wh_act_quant_fp8(wh_ctx* c, float* v, size_t n, int block, wh_stream_t stream) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "ctx is null");
  if (block <= 0 || n == 0) return WH_OK;  // the reference returns early
  if (!v) return fail(WH_ERR_INVALID_POINTER, "values is null");
  WH_CUDA(launch_act_quant(v, (long long)n, block, c->status, c->num_sms, stream));
  return WH_OK;
}

}  // extern "C"

namespace {
// wh_fp8_gemv with an optional addend (laid out like y): y = gemv + addend
// x_group_rows > 0: row r reads the input at x + (r / x_group_rows) * x_group_off
wh_status fp8_gemv_impl(wh_ctx* c, const uint8_t* weight, const uint8_t* scale, int rows,
                        int cols, int scale_rows, int scale_cols, int row_start, int row_end,
                        const float* x, int batch, int ldx, float* y, int ldy,
                        int act_quant_block, const float* addend, wh_stream_t stream,
                        int x_group_rows = 0, long long x_group_off = 0) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "ctx is null");
  // src/compute.rs:6256-6289 validation order
  if (rows <= 0 || cols <= 0 || scale_rows <= 0 || scale_cols <= 0 || rows % scale_rows != 0 ||
      cols % scale_cols != 0)
    return fail(WH_ERR_INVALID_SHAPE, "DeepSeek FP8 scale shape");
  if (row_start < 0 || row_start >= row_end || row_end > rows)
    return fail(WH_ERR_INVALID_SHAPE, "DeepSeek FP8 row range");
  if (batch <= 0) return fail(WH_ERR_INVALID_SHAPE, "FP8 multi GEMV input/output count");
  if (ldx < cols) return fail(WH_ERR_INVALID_SHAPE, "DeepSeek FP8 GEMV input too small");
  if (ldy < row_end - row_start) return fail(WH_ERR_OUTPUT_TOO_SMALL, "output too small");
  if (act_quant_block < 0) return fail(WH_ERR_INVALID_SHAPE, "act_quant_block < 0");
  if (!weight || !scale || !x || !y) return fail(WH_ERR_INVALID_POINTER, "null pointer");

  Fp8GemvArgs a{};
  a.weight = weight;
  a.scale = scale;
  a.rows = rows;
  a.cols = cols;
  a.scale_rows = scale_rows;
  a.scale_cols = scale_cols;
  a.row_start = row_start;
  a.row_end = row_end;
  a.x = x;
  a.ldx = ldx;
  a.y = y;
  a.ldy = ldy;
  a.batch = batch;
  a.act_quant_block = act_quant_block;
  a.status = c->status;
  a.addend = addend;
  a.x_group_rows = x_group_rows;
  a.x_group_off = x_group_off;

  // the columns one input spans (grouped: every group's slice)
  const long long xspan =
      x_group_rows > 0 ? (long long)(rows / x_group_rows - 1) * x_group_off + cols : cols;
  // act quant ahead of the kernel: blocks never straddle inputs or groups
  const bool pre_aq_ok =
      act_quant_block == 0 || (xspan % act_quant_block == 0 && cols % act_quant_block == 0);
  bool fast = cols / scale_cols == 128 && aligned(weight, 16) && aligned(x, 16) &&
              ldx % 4 == 0 && x_group_off % 4 == 0 && cols <= 8192;
  bool in_kernel_aq = false;  // the one-input kernel quantises x itself
  // every CTA's rows must lie in one group: a box height dividing the group
  // and the start row
  auto fit_groups = [&](int box_rows) {
    if (x_group_rows > 0)
      while (box_rows > 1 && (x_group_rows % box_rows != 0 || row_start % box_rows != 0))
        --box_rows;
    return box_rows;
  };
  const CUtensorMap* xmap = nullptr;
  if (fast) {
    // one input: boxes of ceil(rows / SMs) rows, one per SM; the batched
    // kernel: boxes of 32 rows
    const int nrows = row_end - row_start;
    const int per = std::max(1, c->num_sms);
    a.box_rows = fit_groups(std::min(32, std::max(1, (nrows + per - 1) / per)));
    in_kernel_aq = batch == 1 && fp8_gemv_rowgroup_fits(a, c->num_sms);
    if (!in_kernel_aq) {
      a.box_rows = fit_groups(32);
      if (act_quant_block > 0 && !pre_aq_ok) fast = false;
    }
  }
  if (fast && !in_kernel_aq) {
    // the batched kernel's input tiles: x itself, or the act-quantised copy of
    // each input's span in the workspace
    const float* xsrc = x;
    int xld = ldx;
    if (act_quant_block > 0) {
      wh_status st = c->ensure_work(sizeof(float) * (size_t)batch * xspan);
      if (st != WH_OK) return st;
      xsrc = static_cast<const float*>(c->work);
      xld = (int)xspan;
    }
    auto xkey = std::make_tuple((const void*)xsrc, xspan, batch, xld);
    auto xit = c->fp8_xmaps.find(xkey);
    if (xit == c->fp8_xmaps.end()) {
      CUtensorMap m;
      if (xspan >= 136 && make_f32_xmap(&m, xsrc, xspan, batch, xld))
        xit = c->fp8_xmaps.emplace(xkey, m).first;
    }
    if (xit == c->fp8_xmaps.end())
      fast = false;  // no input map for this shape: the generic kernel
    else
      xmap = &xit->second;
  }
  if (fast) {
    const int box_rows = a.box_rows;
    auto key = std::make_tuple((const void*)weight, rows, cols, box_rows);
    auto it = c->fp8_maps.find(key);
    if (it == c->fp8_maps.end()) {
      CUtensorMap m;
      wh_status st = make_u8_map(&m, weight, rows, cols, box_rows);
      if (st != WH_OK) return st;
      it = c->fp8_maps.emplace(key, m).first;
    }
    if (act_quant_block > 0 && !in_kernel_aq) {
      // the batched kernel streams its inputs: quantise each input's span
      // beforehand (blocks never straddle inputs or groups)
      wh_status st = c->ensure_work(sizeof(float) * (size_t)batch * xspan);
      if (st != WH_OK) return st;
      float* xw = static_cast<float*>(c->work);
      WH_CUDA(cudaMemcpy2DAsync(xw, sizeof(float) * xspan, x, sizeof(float) * ldx,
                                sizeof(float) * xspan, batch, cudaMemcpyDeviceToDevice, stream));
      WH_CUDA(launch_act_quant(xw, (long long)batch * xspan, act_quant_block, c->status,
                               c->num_sms, stream));
      a.x = xw;
      a.ldx = (int)xspan;
      a.act_quant_block = 0;
    }
    // programmatic dependent launch, so that back-to-back GEMVs overlap one's
    // weight stream with the previous one's tail
    WH_CUDA(launch_fp8_gemv(&it->second, xmap, a, c->num_sms, stream, c->pdl()));
    return WH_OK;
  }
  // generic path
  if (act_quant_block > 0 && x_group_rows > 0)
    return fail(WH_ERR_UNSUPPORTED, "grouped FP8 GEMV with act quant needs the fast path's shapes");
  if (act_quant_block > 0) {
    wh_status st = c->ensure_work(sizeof(float) * (size_t)batch * cols);
    if (st != WH_OK) return st;
    float* xw = static_cast<float*>(c->work);
    WH_CUDA(cudaMemcpy2DAsync(xw, sizeof(float) * cols, x, sizeof(float) * ldx,
                              sizeof(float) * cols, batch, cudaMemcpyDeviceToDevice, stream));
    WH_CUDA(launch_act_quant(xw, (long long)batch * cols, act_quant_block, c->status, c->num_sms,
                             stream));
    // blocks must not straddle inputs: the reference quantises each input alone
    if (cols % act_quant_block != 0) {
      for (int b = 0; b < batch; ++b) {
        WH_CUDA(cudaMemcpyAsync(xw + (size_t)b * cols, x + (size_t)b * ldx, sizeof(float) * cols,
                                cudaMemcpyDeviceToDevice, stream));
        WH_CUDA(launch_act_quant(xw + (size_t)b * cols, cols, act_quant_block, c->status,
                                 c->num_sms, stream));
      }
    }
    a.x = xw;
    a.ldx = cols;
    a.act_quant_block = 0;
  }
  WH_CUDA(launch_fp8_gemv(nullptr, nullptr, a, c->num_sms, stream, false));
  return WH_OK;
}

// compute_deepseek_fp8_shared_expert_into_hidden (src/compute.rs:5545-5614) for
// `tokens` inputs: act quant (64) -> w1, w3 -> SwiGLU with the reference clamps
// -> act quant (64) -> w2, written to y (+ addend).  h1 / h3: [tokens][inter].
wh_status fp8_expert_run(wh_ctx* c, const wh_fp8_expert& e, const float* x, int tokens, int ldx,
                         float* y, int ldy, const float* addend, float* h1, float* h3,
                         wh_stream_t stream) {
  const int inter = e.w1.rows;
  wh_status st;
  if ((st = fp8_gemv_impl(c, e.w1.weight, e.w1.scale, e.w1.rows, e.w1.cols, e.w1.scale_rows,
                          e.w1.scale_cols, 0, e.w1.rows, x, tokens, ldx, h1, inter, 64, nullptr,
                          stream)) != WH_OK)
    return st;
  if ((st = fp8_gemv_impl(c, e.w3.weight, e.w3.scale, e.w3.rows, e.w3.cols, e.w3.scale_rows,
                          e.w3.scale_cols, 0, e.w3.rows, x, tokens, ldx, h3, inter, 64, nullptr,
                          stream)) != WH_OK)
    return st;
  WH_CUDA(launch_swiglu(h1, h3, tokens * inter, c->status, (cudaStream_t)stream));
  return fp8_gemv_impl(c, e.w2.weight, e.w2.scale, e.w2.rows, e.w2.cols, e.w2.scale_rows,
                       e.w2.scale_cols, 0, e.w2.rows, h1, tokens, inter, y, ldy, 64, addend,
                       stream);
}

// the shape checks of compute_deepseek_fp8_shared_expert_into_hidden
wh_status fp8_expert_check(const wh_fp8_expert& e, size_t hidden) {
  if ((size_t)e.w1.cols != hidden || (size_t)e.w3.cols != hidden)
    return fail(WH_ERR_INVALID_SHAPE, "DeepSeek shared expert input dim");
  if (e.w1.rows != e.w3.rows || e.w2.cols != e.w1.rows)
    return fail(WH_ERR_INVALID_SHAPE, "DeepSeek shared expert projection shape");
  return WH_OK;
}
}  // namespace

// The MLA attention core for `ntok` tokens in one set of launches (grid z =
// token): each token's own q, cache rows, position, compressed rows and out.
struct MlaToken {
  const float* q;
  const float* keys;
  int token_pos;
  const float* compressed;
  int compressed_count;
  float* out;
};

wh_status mla_attention_tokens(wh_ctx* c, int heads, int head_dim, int nope_dim, int key_stride,
                               int window, const float* sink, const float* inv_freqs,
                               const MlaToken* toks, int ntok, wh_stream_t stream) {
  if (heads < 1 || head_dim < 1 || nope_dim < 0 || nope_dim > head_dim ||
      (head_dim - nope_dim) % 2 != 0 || key_stride < head_dim || window < 1 || ntok < 1)
    return fail(WH_ERR_INVALID_SHAPE, "MLA attention shape");
  if (ntok > kMlaMaxTok) return fail(WH_ERR_UNSUPPORTED, "more than 32 tokens per call");
  const int pairs = (head_dim - nope_dim) / 2;
  if (pairs > 64 || (ntok > 1 && pairs > 64)) return fail(WH_ERR_UNSUPPORTED, "rope dim > 128");
  if (pairs > 0 && nope_dim % 2 != 0) return fail(WH_ERR_UNSUPPORTED, "odd nope_dim");
  if (pairs > 0 && !inv_freqs) return fail(WH_ERR_INVALID_POINTER, "null pointer");
  for (int t = 0; t < ntok; ++t) {
    const MlaToken& k = toks[t];
    if (k.token_pos < 0 || k.compressed_count < 0)
      return fail(WH_ERR_INVALID_SHAPE, "MLA attention shape");
    if (!k.q || !k.keys || !k.out || (k.compressed_count > 0 && !k.compressed))
      return fail(WH_ERR_INVALID_POINTER, "null pointer");
  }
  auto batch = std::make_unique<MlaBatch<kMlaMaxTok>>();
  auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  int widest = 0, pmax = -1;
  size_t work = 0;
  std::vector<size_t> woff(ntok);
  for (int t = 0; t < ntok; ++t) {
    const MlaToken& k = toks[t];
    MlaArgs& a = batch->t[t];
    a.q = k.q;
    a.keys = k.keys;
    a.compressed = k.compressed;
    a.sink = sink;
    a.out = k.out;
    a.heads = heads;
    a.head_dim = head_dim;
    a.nope_dim = nope_dim;
    a.key_stride = key_stride;
    const int context = k.token_pos + 1;
    a.window_start = context > window ? context - window : 0;  // saturating_sub
    a.window_len = context - a.window_start;
    a.compressed_count = k.compressed_count;
    a.vec4 = head_dim % 4 == 0 && key_stride % 4 == 0 && al16(k.q) && al16(k.keys) &&
             (k.compressed_count == 0 || al16(k.compressed));
    a.scale = powf((float)head_dim, -0.5f);  // (head_dim as f32).powf(-0.5)
    const float pos = (float)k.token_pos;
    for (int i = 0; i < pairs; ++i) {
      const float angle = pos * inv_freqs[i];
      a.rope_sin[i] = sinf(angle);
      a.rope_cos[i] = cosf(angle);
    }
    const int P = a.window_len + a.compressed_count;
    if (P > pmax) {
      pmax = P;
      widest = t;
    }
    woff[t] = work;
    work += align256(mla_scratch_bytes(heads, P));
  }
  size_t smem_scores = 0, smem_output = 0;
  if (!mla_plan(batch->t[widest], &smem_scores, &smem_output))
    return fail(WH_ERR_UNSUPPORTED, "heads, head_dim or visible rows do not fit shared memory");
  cudaSetDevice(c->device);
  if (wh_status st = c->ensure_mla_work(work)) return st;
  for (int t = 0; t < ntok; ++t) {
    MlaArgs& a = batch->t[t];
    a.smem_ld = batch->t[widest].smem_ld;
    a.head_group = batch->t[widest].head_group;
    a.stages = batch->t[widest].stages;
    const int P = a.window_len + a.compressed_count;
    a.scores = reinterpret_cast<float*>(static_cast<uint8_t*>(c->mla_work) + woff[t]);
    a.weights = a.scores + (size_t)P * heads;
    a.tile_max = a.weights + (size_t)P * heads;
    a.head_max = a.tile_max + mla_tile_count(P) * heads;
  }
  if (ntok == 1) {
    MlaBatch<1> one;
    one.t[0] = batch->t[0];
    WH_CUDA(launch_mla_attention<1>(one, 1, smem_scores, smem_output, (cudaStream_t)stream));
  } else {
    WH_CUDA(launch_mla_attention<kMlaMaxTok>(*batch, ntok, smem_scores, smem_output,
                                             (cudaStream_t)stream));
  }
  return WH_OK;
}

extern "C" {

wh_status wh_fp8_gemv(wh_ctx* c, const uint8_t* weight, const uint8_t* scale, int rows, int cols,
                      int scale_rows, int scale_cols, int row_start, int row_end, const float* x,
                      int batch, int ldx, float* y, int ldy, int act_quant_block,
                      wh_stream_t stream) {
  return fp8_gemv_impl(c, weight, scale, rows, cols, scale_rows, scale_cols, row_start, row_end,
                       x, batch, ldx, y, ldy, act_quant_block, nullptr, stream);
}

wh_status wh_fp8_gemv_grouped(wh_ctx* c, const uint8_t* weight, const uint8_t* scale, int rows,
                              int cols, int scale_rows, int scale_cols, int row_start,
                              int row_end, const float* x, int batch, int ldx, int group_rows,
                              long long group_offset, float* y, int ldy, int act_quant_block,
                              wh_stream_t stream) {
  if (group_rows < 1 || group_offset < 0 || rows % group_rows != 0)
    return fail(WH_ERR_INVALID_SHAPE, "DeepSeek FP8 grouped rows");
  // the reference quantises each group's input alone: blocks must not straddle groups
  if (act_quant_block > 0 && (cols % act_quant_block != 0 || group_offset % act_quant_block != 0))
    return fail(WH_ERR_INVALID_SHAPE, "act quant blocks straddle the groups' inputs");
  return fp8_gemv_impl(c, weight, scale, rows, cols, scale_rows, scale_cols, row_start, row_end,
                       x, batch, ldx, y, ldy, act_quant_block, nullptr, stream, group_rows,
                       group_offset);
}

size_t wh_fp8_expert_scratch_len(size_t hidden, size_t intermediate) {
  return hidden + 2 * intermediate;
}

wh_status wh_fp8_expert_forward(wh_ctx* c, const wh_fp8_expert* e, const float* input,
                                size_t input_len, float* output, size_t output_len,
                                float* scratch, size_t scratch_len, wh_stream_t stream) {
  if (!c || !e) return fail(WH_ERR_INVALID_POINTER, "null ctx/expert");
  wh_status st;
  if ((st = fp8_expert_check(*e, input_len)) != WH_OK) return st;
  if ((size_t)e->w2.rows > output_len)
    return fail(WH_ERR_OUTPUT_TOO_SMALL, "output too small: required=" +
                                             std::to_string(e->w2.rows) +
                                             ", actual=" + std::to_string(output_len));
  const size_t inter = (size_t)e->w1.rows;
  if (scratch_len < wh_fp8_expert_scratch_len(input_len, inter))
    return fail(WH_ERR_SCRATCH_TOO_SMALL, "scratch too small");
  if (!input || !output || !scratch) return fail(WH_ERR_INVALID_POINTER, "null buffer");
  return fp8_expert_run(c, *e, input, 1, (int)input_len, output, (int)output_len, nullptr,
                        scratch, scratch + inter, stream);
}

// ---------------------------------------------------------------------------
wh_status wh_fp4_matvec(wh_ctx* c, const wh_fp4_matvec_spec* s, const float* input,
                        size_t input_len, float* output, size_t output_len, wh_stream_t stream) {
  if (!c || !s) return fail(WH_ERR_INVALID_POINTER, "null ctx/spec");
  wh_status st = validate_fp4(*s, input_len, output_len);
  if (st != WH_OK) return st;
  if (!input || !output) return fail(WH_ERR_INVALID_POINTER, "null input/output");
  Fp4MatvecArgs a{s->packed_weight, s->ue8m0_scales, (int)s->rows, (int)s->cols,
                  (int)s->scale_cols, input, output, c->status};
  WH_CUDA(launch_fp4_matvec(a, c->num_sms, stream));
  return WH_OK;
}

size_t wh_fp4_expert_scratch_len(size_t intermediate) { return intermediate * 2; }

wh_status wh_fp4_expert_forward(wh_ctx* c, const wh_fp4_expert* e, const float* input,
                                size_t input_len, float* output, size_t output_len,
                                float* scratch, size_t scratch_len, wh_stream_t stream) {
  if (!c || !e) return fail(WH_ERR_INVALID_POINTER, "null ctx/expert");
  // src/deepseek_v4.rs:567-583
  if (e->w1.cols != input_len || e->w3.cols != input_len || e->w1.rows != e->w3.rows ||
      e->w2.cols != e->w1.rows)
    return fail(WH_ERR_INVALID_SHAPE, "expert shapes");
  if (output_len < e->w2.rows) return fail(WH_ERR_OUTPUT_TOO_SMALL, "output too small");
  const size_t inter = e->w1.rows, hidden = input_len;
  if (scratch_len < wh_fp4_expert_scratch_len(inter))
    return fail(WH_ERR_SCRATCH_TOO_SMALL, "scratch too small");
  wh_status st;
  if ((st = validate_fp4(e->w1, hidden, inter)) != WH_OK) return st;
  if ((st = validate_fp4(e->w3, hidden, inter)) != WH_OK) return st;
  if ((st = validate_fp4(e->w2, inter, output_len)) != WH_OK) return st;
  if (!input || !output || !scratch) return fail(WH_ERR_INVALID_POINTER, "null buffer");

  if (expert_fast_ok(*e, hidden, inter) && e->w2.rows == hidden) {
    auto key = std::make_tuple((const void*)e->w1.packed_weight, (const void*)e->w3.packed_weight,
                               (const void*)e->w2.packed_weight, hidden, inter);
    auto it = c->experts.find(key);
    if (it == c->experts.end()) {
      DevExpertSet set;
      if ((st = build_expert_set(e, 1, &set)) != WH_OK) return st;
      it = c->experts.emplace(key, set).first;
    }
    // scratch layout: xq f16[hidden] | xq_mult f32[hidden/64] | h f32[inter] |
    //                 hq f16[inter] | hq_mult f32[inter/64]
    const size_t o_xqm = align256(hidden * 2);
    const size_t o_h = o_xqm + align256(hidden / 16);
    const size_t o_hq = o_h + align256(inter * 4);
    const size_t o_hqm = o_hq + align256(inter * 2);
    const size_t need = o_hqm + align256(inter / 16);
    uint8_t* base = reinterpret_cast<uint8_t*>(scratch);
    if (need > scratch_len * sizeof(float) || !aligned(scratch, 256)) {
      if ((st = c->ensure_work(need)) != WH_OK) return st;
      base = static_cast<uint8_t*>(c->work);
    }
    if ((st = c->ensure_blk_counters((int)(inter / 64))) != WH_OK) return st;
    __half* xq = reinterpret_cast<__half*>(base);
    float* xqm = reinterpret_cast<float*>(base + o_xqm);
    float* hbuf = reinterpret_cast<float*>(base + o_h);
    __half* hq = reinterpret_cast<__half*>(base + o_hq);
    float* hqm = reinterpret_cast<float*>(base + o_hqm);
    MoeArgs a{};
    a.maps = it->second.maps;
    a.experts = it->second.experts;
    a.num_experts = 0;
    a.has_shared = 1;
    a.hidden = (int)hidden;
    a.inter = (int)inter;
    a.x = input;
    a.tokens = 1;
    a.topk = 0;
    a.h = hbuf;
    a.blk_counters = c->blk_counters;
    a.y = output;
    a.expert_out = output;
    a.combine = 0;
    a.status = c->status;
    c->prof_begin();
    if ((st = c->prof_mark(stream)) != WH_OK) return st;
    WH_CUDA(launch_xq(input, (int)hidden, 1, xq, xqm, stream));
    if ((st = c->prof_mark(stream)) != WH_OK) return st;
    WH_CUDA(launch_moe_up_ex(a, xq, xqm, hq, hqm, stream, c->pdl()));
    if ((st = c->prof_mark(stream)) != WH_OK) return st;
    WH_CUDA(launch_moe_down_ex(a, hq, hqm, stream, c->pdl()));
    return c->prof_mark(stream);
  }
  // generic exact path: act quant -> w1,w3 -> SwiGLU -> act quant -> w2
  if ((st = c->ensure_work(sizeof(float) * hidden)) != WH_OK) return st;
  float* xw = static_cast<float*>(c->work);
  WH_CUDA(cudaMemcpyAsync(xw, input, sizeof(float) * hidden, cudaMemcpyDeviceToDevice, stream));
  WH_CUDA(launch_act_quant(xw, (long long)hidden, 64, c->status, c->num_sms, stream));
  float* gate = scratch;
  float* up = scratch + inter;
  Fp4MatvecArgs m1{e->w1.packed_weight, e->w1.ue8m0_scales, (int)inter, (int)hidden,
                   (int)e->w1.scale_cols, xw, gate, c->status};
  Fp4MatvecArgs m3{e->w3.packed_weight, e->w3.ue8m0_scales, (int)inter, (int)hidden,
                   (int)e->w3.scale_cols, xw, up, c->status};
  WH_CUDA(launch_fp4_matvec(m1, c->num_sms, stream));
  WH_CUDA(launch_fp4_matvec(m3, c->num_sms, stream));
  WH_CUDA(launch_swiglu(gate, up, (int)inter, c->status, stream));
  WH_CUDA(launch_act_quant(gate, (long long)inter, 64, c->status, c->num_sms, stream));
  Fp4MatvecArgs m2{e->w2.packed_weight, e->w2.ue8m0_scales, (int)e->w2.rows, (int)inter,
                   (int)e->w2.scale_cols, gate, output, c->status};
  WH_CUDA(launch_fp4_matvec(m2, c->num_sms, stream));
  return WH_OK;
}

// ---------------------------------------------------------------------------
wh_status wh_router_topk(wh_ctx* c, const uint16_t* gate, int experts, int hidden,
                         const float* x, int tokens, int topk, int mode, const float* bias,
                         float route_scale, const int32_t* hash_ids, int32_t* ids,
                         float* weights, float* logits, wh_stream_t stream) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "ctx is null");
  if (experts <= 0 || hidden <= 0 || tokens <= 0 || topk <= 0)
    return fail(WH_ERR_INVALID_SHAPE, "router shape");
  if (experts > 1024 || topk > 32) return fail(WH_ERR_UNSUPPORTED, "experts > 1024 or topk > 32");
  if (mode != WH_ROUTER_RAW_LOGITS && mode != WH_ROUTER_SQRT_SOFTPLUS)
    return fail(WH_ERR_INVALID_SHAPE, "router mode");
  if (!gate || !x || !ids || !weights) return fail(WH_ERR_INVALID_POINTER, "null pointer");
  // the 16-column chunk loop reads bf16 pairs and float2s; below one chunk only
  // the scalar tail runs
  if (hidden >= 16 && (hidden % 2 != 0 || !aligned(gate, 4) || !aligned(x, 8)))
    return fail(WH_ERR_UNSUPPORTED, "router needs an even hidden size and aligned rows");
  wh_status st = c->ensure_counters(tokens);
  if (st != WH_OK) return st;
  float* lg = logits;
  if (!lg) {
    if ((st = c->ensure_work(sizeof(float) * (size_t)tokens * experts)) != WH_OK) return st;
    lg = static_cast<float*>(c->work);
  }
  RouterArgs a{};
  a.gate = gate;
  a.experts = experts;
  a.hidden = hidden;
  a.x = x;
  a.tokens = tokens;
  a.topk = topk;
  a.mode = mode;
  a.bias = bias;
  a.route_scale = route_scale;
  a.hash_ids = hash_ids;
  a.logits = lg;
  a.ids = ids;
  a.weights = weights;
  a.combine_w = nullptr;
  a.counters = c->counters;
  a.status = c->status;
  WH_CUDA(launch_router_ex(a, nullptr, nullptr, stream, false));
  return WH_OK;
}

// ---------------------------------------------------------------------------
// rope_inv_freqs (src/compute.rs:2591-2621), operation for operation in f32
void wh_rope_inv_freqs(int rope_dim, float theta, float yarn_factor, float yarn_beta_fast,
                       float yarn_beta_slow, uint64_t yarn_original_seq_len, float* inv_freqs) {
  if (!inv_freqs || rope_dim < 2) return;
  const int pairs = rope_dim / 2;
  for (int p = 0; p < pairs; ++p)
    inv_freqs[p] = powf(theta, -(float)(2 * p) / (float)rope_dim);
  if (yarn_factor <= 0.0f || yarn_original_seq_len == 0) return;
  const float dim = (float)rope_dim;
  const float base_ln = logf(theta);
  const float pi = 3.14159265358979323846f;
  auto correction_dim = [&](float rotations) {
    return dim * logf((float)yarn_original_seq_len / (rotations * 2.0f * pi)) /
           (2.0f * base_ln);
  };
  const float low = fmaxf(floorf(correction_dim(yarn_beta_fast)), 0.0f);
  float high = fminf(ceilf(correction_dim(yarn_beta_slow)), dim - 1.0f);
  if (fabsf(low - high) < 1.1920929e-07f) high = low + 0.001f;
  for (int p = 0; p < pairs; ++p) {
    float ramp = ((float)p - low) / (high - low);
    ramp = ramp < 0.0f ? 0.0f : (ramp > 1.0f ? 1.0f : ramp);
    const float smooth = 1.0f - ramp;
    inv_freqs[p] = inv_freqs[p] / yarn_factor * (1.0f - smooth) + inv_freqs[p] * smooth;
  }
}

wh_status wh_mla_attention(wh_ctx* c, const float* q, int heads, int head_dim, int nope_dim,
                           const float* keys, int key_stride, int token_pos, int window,
                           const float* compressed, int compressed_count, const float* sink,
                           const float* inv_freqs, float* out, wh_stream_t stream) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "ctx is null");
  MlaToken t{q, keys, token_pos, compressed, compressed_count, out};
  return mla_attention_tokens(c, heads, head_dim, nope_dim, key_stride, window, sink, inv_freqs,
                              &t, 1, stream);
}

// ---------------------------------------------------------------------------
// mHC hyper-connections (src/compute.rs:4945-5132)
static wh_status hc_common_check(wh_ctx* c, int tokens, int hc, int hidden) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "ctx is null");
  if (tokens < 1 || hc < 1 || hidden < 1) return fail(WH_ERR_INVALID_SHAPE, "hc sizes");
  if (hc > kHcMaxHc) return fail(WH_ERR_UNSUPPORTED, "hc_mult > 8");
  if ((long long)hc * hidden > (1LL << 30)) return fail(WH_ERR_INVALID_SHAPE, "hc_dim too large");
  return WH_OK;
}

static bool hc_al16(const void* p) { return ((uintptr_t)p & 15) == 0; }

wh_status wh_hc_pre(wh_ctx* c, const float* fn, const float* scale, const float* base,
                    const float* x, int tokens, int hc, int hidden, int sinkhorn_iters,
                    float eps, float* y, float* post, float* comb, wh_stream_t stream) {
  if (wh_status st = hc_common_check(c, tokens, hc, hidden)) return st;
  if (sinkhorn_iters < 0) return fail(WH_ERR_INVALID_SHAPE, "sinkhorn_iters < 0");
  if (!fn || !scale || !base || !x || !y || !post || !comb)
    return fail(WH_ERR_INVALID_POINTER, "null pointer");
  HcArgs a{};
  a.fn = fn;
  a.scale = scale;
  a.base = base;
  a.x = x;
  a.y = y;
  a.post = post;
  a.comb = comb;
  a.tokens = tokens;
  a.hc = hc;
  a.hidden = hidden;
  a.iters = sinkhorn_iters;
  a.eps = eps;
  a.head = 0;
  a.vec4 = (hc * hidden) % 4 == 0 && hc_al16(fn) && hc_al16(x);
  cudaSetDevice(c->device);
  if (wh_status st = c->ensure_hc_work(hc_dots_bytes(tokens, (2 + hc) * hc))) return st;
  a.dots = (float*)c->hc_work;
  WH_CUDA(launch_hc_mix(a, (cudaStream_t)stream));
  return WH_OK;
}

wh_status wh_hc_post(wh_ctx* c, const float* y, const float* residual, const float* post,
                     const float* comb, int tokens, int hc, int hidden, float* out,
                     wh_stream_t stream) {
  if (wh_status st = hc_common_check(c, tokens, hc, hidden)) return st;
  if (!y || !residual || !post || !comb || !out)
    return fail(WH_ERR_INVALID_POINTER, "null pointer");
  HcPostArgs a{y, residual, post, comb, out, tokens, hc, hidden};
  cudaSetDevice(c->device);
  WH_CUDA(launch_hc_post(a, c->num_sms, (cudaStream_t)stream));
  return WH_OK;
}

wh_status wh_hc_head(wh_ctx* c, const float* fn, float scale, const float* base, const float* x,
                     int tokens, int hc, int hidden, float eps, float* pooled,
                     wh_stream_t stream) {
  if (wh_status st = hc_common_check(c, tokens, hc, hidden)) return st;
  if (!fn || !base || !x || !pooled) return fail(WH_ERR_INVALID_POINTER, "null pointer");
  HcArgs a{};
  a.fn = fn;
  a.base = base;
  a.x = x;
  a.y = pooled;
  a.tokens = tokens;
  a.hc = hc;
  a.hidden = hidden;
  a.eps = eps;
  a.head = 1;
  a.head_scale = scale;
  a.vec4 = (hc * hidden) % 4 == 0 && hc_al16(fn) && hc_al16(x);
  cudaSetDevice(c->device);
  if (wh_status st = c->ensure_hc_work(hc_dots_bytes(tokens, hc))) return st;
  a.dots = (float*)c->hc_work;
  WH_CUDA(launch_hc_mix(a, (cudaStream_t)stream));
  return WH_OK;
}

// ---------------------------------------------------------------------------
size_t wh_lm_head_scratch_bytes(long long rows, int top_k) {
  return lm_head_scratch_bytes(rows < 1 ? 1 : rows, top_k < 1 ? 1 : top_k);
}

wh_status wh_lm_head_topk(wh_ctx* c, const uint16_t* weight, long long rows, int cols,
                          uint32_t row_base, const float* x, size_t x_len, int top_k,
                          uint32_t* out_tokens, float* out_logits, float* logits, void* scratch,
                          size_t scratch_bytes, wh_stream_t stream) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "ctx is null");
  top_k = top_k < 1 ? 1 : top_k;  // top_k.max(1) (src/compute.rs:2777)
  // src/compute.rs:2769-2797 and score_bf16_lm_head_topk's checks, in order
  if (!scratch || scratch_bytes == 0) return fail(WH_ERR_SCRATCH_TOO_SMALL, "scratch is empty");
  if (cols <= 0 || rows < 0) return fail(WH_ERR_INVALID_SHAPE, "LM-head shape");
  if (x_len < (size_t)cols) return fail(WH_ERR_INVALID_SHAPE, "LM-head input too small");
  if (rows == 0) return fail(WH_ERR_INVALID_SHAPE, "LM-head has no rows");
  if (!weight || !x || !out_tokens || !out_logits) return fail(WH_ERR_INVALID_POINTER, "null pointer");
  if (!lm_head_supported(rows, cols, top_k) || cols % 8 != 0 || !aligned(weight, 16))
    return fail(WH_ERR_UNSUPPORTED,
                "lm_head top-k needs cols % 8 == 0, cols <= 16384, a 16-byte aligned weight "
                "and top_k <= 511");
  if (scratch_bytes < lm_head_scratch_bytes(rows, top_k))
    return fail(WH_ERR_SCRATCH_TOO_SMALL, "lm_head scratch too small");
  uint8_t* p = static_cast<uint8_t*>(scratch);
  auto carve = [&](size_t bytes) {
    uint8_t* q = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 255) & ~uintptr_t(255));
    p = q + bytes;
    return q;
  };
  LmHeadArgs a{};
  a.weight = weight;
  a.x = x;
  a.rows = rows;
  a.cols = cols;
  a.top_k = top_k;
  a.row_base = row_base;
  float* lg = reinterpret_cast<float*>(carve(size_t(rows) * 4));
  a.logits = logits ? logits : lg;
  // flags, counter, candidate count and the histogram are zeroed by one memset
  a.flags = reinterpret_cast<uint32_t*>(carve(16 + 4096 * 4));
  a.counter = a.flags + 1;
  a.cand_count = a.flags + 2;
  a.hist = reinterpret_cast<int*>(a.flags + 4);
  a.cand = reinterpret_cast<uint64_t*>(carve(8192 * 8));
  a.out_tokens = out_tokens;
  a.out_logits = out_logits;
  a.tokens = 1;
  a.ldx = cols;
  cudaStream_t s = (cudaStream_t)stream;
  WH_CUDA(cudaMemsetAsync(a.flags, 0, 16 + 4096 * 4, s));
  wh_status st;
  c->prof_begin();
  if ((st = c->prof_mark(s)) != WH_OK) return st;
  for (int stage = 0; stage < 3; ++stage) {
    WH_CUDA(launch_lm_head_stage(a, stage, c->pdl(), s));
    if ((st = c->prof_mark(s)) != WH_OK) return st;
  }
  return WH_OK;
}

size_t wh_lm_head_batch_scratch_bytes(long long rows, int top_k, int tokens) {
  return tokens < 1 ? 0 : lm_head_batch_scratch_bytes(rows, top_k, tokens);
}

wh_status wh_lm_head_topk_batch(wh_ctx* c, const uint16_t* weight, long long rows, int cols,
                                uint32_t row_base, const float* x, int tokens, int ldx,
                                int top_k, uint32_t* out_tokens, float* out_logits,
                                float* logits, void* scratch, size_t scratch_bytes,
                                wh_stream_t stream) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "ctx is null");
  top_k = top_k < 1 ? 1 : top_k;  // top_k.max(1) (src/compute.rs:2777)
  if (tokens < 1) return fail(WH_ERR_EMPTY_SHAPE, "LM-head batch has no tokens");
  if (tokens > 65535) return fail(WH_ERR_UNSUPPORTED, "LM-head batch takes at most 65535 tokens");
  if (!scratch || scratch_bytes == 0) return fail(WH_ERR_SCRATCH_TOO_SMALL, "scratch is empty");
  if (cols <= 0 || rows < 0) return fail(WH_ERR_INVALID_SHAPE, "LM-head shape");
  if (ldx < cols) return fail(WH_ERR_INVALID_SHAPE, "LM-head input too small");
  if (rows == 0) return fail(WH_ERR_INVALID_SHAPE, "LM-head has no rows");
  if (!weight || !x || !out_tokens || !out_logits) return fail(WH_ERR_INVALID_POINTER, "null pointer");
  if (!lm_head_supported(rows, cols, top_k) || cols % 8 != 0 || !aligned(weight, 16))
    return fail(WH_ERR_UNSUPPORTED,
                "lm_head top-k needs cols % 8 == 0, cols <= 16384, a 16-byte aligned weight "
                "and top_k <= 511");
  if (scratch_bytes < lm_head_batch_scratch_bytes(rows, top_k, tokens))
    return fail(WH_ERR_SCRATCH_TOO_SMALL, "lm_head batch scratch too small");
  uint8_t* p = static_cast<uint8_t*>(scratch);
  auto carve = [&](size_t bytes) {
    uint8_t* q = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 255) & ~uintptr_t(255));
    p = q + bytes;
    return q;
  };
  LmHeadArgs a{};
  a.weight = weight;
  a.x = x;
  a.rows = rows;
  a.cols = cols;
  a.top_k = top_k;
  a.row_base = row_base;
  a.tokens = tokens;
  a.ldx = ldx;
  float* lg = reinterpret_cast<float*>(carve(size_t(tokens) * rows * 4));
  a.logits = logits ? logits : lg;
  // per token: flags, pass counter, candidate count, -, histogram; one memset
  const size_t words = size_t(tokens) * kLmTokWords;
  a.flags = reinterpret_cast<uint32_t*>(carve(words * 4));
  a.counter = a.flags + 1;
  a.cand_count = a.flags + 2;
  a.hist = reinterpret_cast<int*>(a.flags + 4);
  a.cand = reinterpret_cast<uint64_t*>(carve(size_t(tokens) * 8192 * 8));
  a.out_tokens = out_tokens;
  a.out_logits = out_logits;
  cudaStream_t s = (cudaStream_t)stream;
  WH_CUDA(cudaMemsetAsync(a.flags, 0, words * 4, s));
  WH_CUDA(launch_lm_head_batch(a, c->pdl(), s));
  return WH_OK;
}

// ---------------------------------------------------------------------------
wh_status wh_moe_plan_create(wh_ctx* c, const wh_moe_desc* d, wh_moe_plan** out) {
  if (!c || !d || !out) return fail(WH_ERR_INVALID_POINTER, "null argument");
  *out = nullptr;
  if (d->num_experts <= 0 || d->hidden <= 0 || d->inter <= 0 || d->topk <= 0 ||
      d->max_tokens <= 0)
    return fail(WH_ERR_EMPTY_SHAPE, "moe shape");
  if (d->topk > d->num_experts || d->topk > 7 || d->num_experts > 1024)
    return fail(WH_ERR_UNSUPPORTED, "topk must be <= 7 (8 slots with the shared expert)");
  if (!d->experts) return fail(WH_ERR_INVALID_POINTER, "experts");
  if (d->shared && d->shared_fp8)
    return fail(WH_ERR_INVALID_SHAPE, "at most one shared expert (FP4 or FP8)");
  if (d->shared_fp8) {
    wh_status sst = fp8_expert_check(*d->shared_fp8, (size_t)d->hidden);
    if (sst != WH_OK) return sst;
    if (d->shared_fp8->w2.rows != d->hidden)
      return fail(WH_ERR_INVALID_SHAPE, "FP8 shared expert output rows != hidden");
    if (!d->shared_fp8->w1.weight || !d->shared_fp8->w3.weight || !d->shared_fp8->w2.weight ||
        !d->shared_fp8->w1.scale || !d->shared_fp8->w3.scale || !d->shared_fp8->w2.scale)
      return fail(WH_ERR_INVALID_POINTER, "FP8 shared expert weights");
  }
  if (d->router_mode != WH_ROUTER_RAW_LOGITS && d->router_mode != WH_ROUTER_SQRT_SOFTPLUS)
    return fail(WH_ERR_INVALID_SHAPE, "router mode");
  const int n = d->num_experts + (d->shared ? 1 : 0);
  std::vector<wh_fp4_expert> all(d->experts, d->experts + d->num_experts);
  if (d->shared) all.push_back(*d->shared);
  for (const auto& e : all) {
    if (e.w1.cols != (size_t)d->hidden || e.w3.cols != (size_t)d->hidden ||
        e.w1.rows != (size_t)d->inter || e.w3.rows != (size_t)d->inter ||
        e.w2.cols != (size_t)d->inter || e.w2.rows != (size_t)d->hidden)
      return fail(WH_ERR_INVALID_SHAPE, "expert shape differs from the layer shape");
    wh_status st;
    if ((st = validate_fp4(e.w1, d->hidden, d->inter)) != WH_OK) return st;
    if ((st = validate_fp4(e.w3, d->hidden, d->inter)) != WH_OK) return st;
    if ((st = validate_fp4(e.w2, d->inter, d->hidden)) != WH_OK) return st;
    if (!expert_fast_ok(e, d->hidden, d->inter))
      return fail(WH_ERR_UNSUPPORTED,
                  "MoE layer needs 32-column scale groups, hidden/inter multiples of 256 and "
                  "16-byte aligned weights");
  }
  wh_moe_plan* p = new wh_moe_plan();
  p->ctx = c;
  p->d = *d;
  p->d.experts = nullptr;
  p->d.shared = nullptr;
  p->d.shared_fp8 = nullptr;
  if (d->shared_fp8) {
    p->has_sfp8 = true;
    p->sfp8 = *d->shared_fp8;
  }
  wh_status st = build_expert_set(all.data(), n, &p->set);
  if (st != WH_OK) {
    free_expert_set(p->set);
    delete p;
    return st;
  }
  p->d.shared = d->shared ? reinterpret_cast<const wh_fp4_expert*>(1) : nullptr;  // flag only
  if (d->exact != 1 && d->hidden % 512 == 0 && d->inter % 512 == 0) {
    // UE8M0 bytes 0 and 255 mean 0 and +inf in the reference but 2^-127 and NaN
    // to the tensor core: layers holding either stay on the per-token path
    int bad = 1;
    st = build_grouped_maps(all.data(), n, &p->set);
    if (st == WH_OK) st = scan_scale_bytes(p->set.experts, n, d->hidden, d->inter, &bad);
    if (st != WH_OK) {
      free_expert_set(p->set);
      delete p;
      return st;
    }
    p->grouped = bad == 0;
  }
  const size_t nblk = (size_t)d->max_tokens * (d->topk + 1) * (d->inter / 64);
  cudaError_t e = cudaMalloc(&p->counters, sizeof(uint32_t) * d->max_tokens);
  if (e == cudaSuccess) e = cudaMemset(p->counters, 0, sizeof(uint32_t) * d->max_tokens);
  if (e == cudaSuccess) e = cudaMalloc(&p->blk_counters, sizeof(uint32_t) * nblk);
  if (e == cudaSuccess) e = cudaMemset(p->blk_counters, 0, sizeof(uint32_t) * nblk);
  if (e == cudaSuccess) e = cudaMalloc(&p->dec_sync, sizeof(uint32_t) * 4);
  if (e == cudaSuccess) e = cudaMemset(p->dec_sync, 0, sizeof(uint32_t) * 4);
  if (e != cudaSuccess) {
    free_expert_set(p->set);
    delete p;
    return cuda_fail(e, "plan counters");
  }
  *out = p;
  return WH_OK;
}

void wh_moe_plan_destroy(wh_moe_plan* p) {
  if (!p) return;
  free_expert_set(p->set);
  if (p->counters) cudaFree(p->counters);
  if (p->blk_counters) cudaFree(p->blk_counters);
  if (p->dec_sync) cudaFree(p->dec_sync);
  delete p;
}

wh_status wh_moe_plan_set_fused_decode(wh_moe_plan* p, int on) {
  if (!p) return fail(WH_ERR_INVALID_POINTER, "null plan");
  p->decode_on = on != 0;
  return WH_OK;
}

namespace {
struct MoeScratch {
  float* logits;
  float* combine_w;
  int32_t* ids;
  float* weights;
  __half* xq;
  float* xq_mult;
  float* h;
  __half* hq;
  float* hq_mult;
  size_t bytes;
};
MoeScratch moe_scratch_layout(const wh_moe_plan* p, int T, uint8_t* base) {
  const auto& d = p->d;
  const int S = d.topk + (d.shared ? 1 : 0);
  MoeScratch s{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* q = base ? base + off : nullptr;
    off += align256(bytes);
    return q;
  };
  s.logits = reinterpret_cast<float*>(take(sizeof(float) * T * d.num_experts));
  s.combine_w = reinterpret_cast<float*>(take(sizeof(float) * T * d.topk));
  s.ids = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * T * d.topk));
  s.weights = reinterpret_cast<float*>(take(sizeof(float) * T * d.topk));
  s.xq = reinterpret_cast<__half*>(take(2 * (size_t)T * d.hidden));
  s.xq_mult = reinterpret_cast<float*>(take(sizeof(float) * T * (d.hidden / 64)));
  s.h = reinterpret_cast<float*>(take(4 * (size_t)T * S * d.inter));
  s.hq = reinterpret_cast<__half*>(take(2 * (size_t)T * S * d.inter));
  s.hq_mult = reinterpret_cast<float*>(take(sizeof(float) * T * S * (d.inter / 64)));
  s.bytes = off;
  return s;
}
}  // namespace

// 16-token tiles while the routed experts average at most 4 rows (decode-sized
// calls and batched decode: each expert's weights stream and convert once per
// tile, and a batch tile would carry mostly empty columns); kGN-token tiles
// beyond that.
int grouped_tile_n(const wh_moe_plan* p, int tokens) {
  return (tokens < kGroupedMinTokens || (long long)tokens * p->d.topk <= 4LL * p->d.num_experts)
             ? kGNSmall
             : kGN;
}

struct GroupedScratch {
  float* logits;
  float* combine_w;
  int32_t* ids;
  float* weights;
  int* slot;
  int* counts;
  int* offsets;
  int4* units_up;
  int4* units_down;
  int* n_units;
  uint8_t* xq;   // [rows][hidden] E4M3
  uint8_t* xsf;  // [rows][hidden/32]
  uint8_t* hq;   // [rows][inter] E4M3
  uint8_t* hsf;  // [rows][inter/32]
  float* yrows;  // [rows][hidden]
  int rows;
  size_t bytes;
};
GroupedScratch grouped_scratch_layout(const wh_moe_plan* p, int T, uint8_t* base) {
  const auto& d = p->d;
  const int ne = d.num_experts + (d.shared ? 1 : 0);
  const int R = T * d.topk + (d.shared ? T : 0);
  const size_t tiles = size_t(R) / grouped_tile_n(p, T) + 1 + ne;  // >= sum of ceil(rows/tile)
  GroupedScratch s{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* q = base ? base + off : nullptr;
    off += align256(bytes);
    return q;
  };
  s.logits = reinterpret_cast<float*>(take(sizeof(float) * T * d.num_experts));
  s.combine_w = reinterpret_cast<float*>(take(sizeof(float) * T * d.topk));
  s.ids = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * T * d.topk));
  s.weights = reinterpret_cast<float*>(take(sizeof(float) * T * d.topk));
  s.slot = reinterpret_cast<int*>(take(sizeof(int) * T * d.topk));
  s.counts = reinterpret_cast<int*>(take(sizeof(int) * (ne + 1)));
  s.offsets = reinterpret_cast<int*>(take(sizeof(int) * (ne + 2)));
  s.units_up = reinterpret_cast<int4*>(take(sizeof(int4) * tiles * (d.inter / 128)));
  s.units_down = reinterpret_cast<int4*>(take(sizeof(int4) * tiles * (d.hidden / 128)));
  s.n_units = reinterpret_cast<int*>(take(sizeof(int) * 2));
  s.xq = take((size_t)R * d.hidden);
  s.xsf = take((size_t)R * (d.hidden / 32));
  s.hq = take((size_t)R * d.inter);
  s.hsf = take((size_t)R * (d.inter / 32));
  s.yrows = reinterpret_cast<float*>(take(sizeof(float) * (size_t)R * d.hidden));
  s.rows = R;
  s.bytes = off;
  return s;
}
// exact 0 (auto): tensor cores from kGroupedMinTokens tokens on, the exact
// kernels below (they are faster for decode-sized calls); 2: tensor cores for
// every call; 1: never.
bool use_grouped(const wh_moe_plan* p, int tokens) {
  if (!p->grouped) return false;
  return p->d.exact == 2 ? tokens >= 1 : tokens >= kGroupedMinTokens;
}

// the path's scratch, then room to stage x when the caller passes it in host
// memory
size_t moe_path_scratch_bytes(const wh_moe_plan* p, int tokens) {
  return use_grouped(p, tokens) ? grouped_scratch_layout(p, tokens, nullptr).bytes
                                : moe_scratch_layout(p, tokens, nullptr).bytes;
}

wh_status wh_moe_scratch_field(const wh_moe_plan* p, int tokens, int field, size_t* offset,
                               size_t* bytes) {
  if (!p || !offset || !bytes) return fail(WH_ERR_INVALID_POINTER, "null plan/out");
  if (tokens <= 0) return fail(WH_ERR_EMPTY_SHAPE, "tokens");
  if (!use_grouped(p, tokens)) return fail(WH_ERR_UNSUPPORTED, "the call does not take the grouped path");
  // lay the scratch out at a stand-in base address and report offsets from it
  uint8_t* base = reinterpret_cast<uint8_t*>(uintptr_t(1) << 40);
  const GroupedScratch g = grouped_scratch_layout(p, tokens, base);
  const auto& d = p->d;
  const size_t T = tokens, k = d.topk, R = g.rows, ne = d.num_experts + (d.shared ? 1 : 0);
  const void* q = nullptr;
  size_t n = 0;
  switch (field) {
    case WH_MOE_FIELD_SLOT: q = g.slot; n = sizeof(int) * T * k; break;
    case WH_MOE_FIELD_OFFSETS: q = g.offsets; n = sizeof(int) * (ne + 1); break;
    case WH_MOE_FIELD_COMBINE_W: q = g.combine_w; n = sizeof(float) * T * k; break;
    case WH_MOE_FIELD_XQ: q = g.xq; n = R * d.hidden; break;
    case WH_MOE_FIELD_XSF: q = g.xsf; n = R * (d.hidden / 32); break;
    case WH_MOE_FIELD_HQ: q = g.hq; n = R * d.inter; break;
    case WH_MOE_FIELD_HSF: q = g.hsf; n = R * (d.inter / 32); break;
    case WH_MOE_FIELD_YROWS: q = g.yrows; n = sizeof(float) * R * d.hidden; break;
    default: return fail(WH_ERR_UNSUPPORTED, "unknown scratch field");
  }
  *offset = size_t(static_cast<const uint8_t*>(q) - base);
  *bytes = n;
  return WH_OK;
}

size_t wh_moe_scratch_bytes(const wh_moe_plan* p, int tokens) {
  if (!p || tokens <= 0) return 0;
  size_t n = align256(moe_path_scratch_bytes(p, tokens)) +
             align256(sizeof(float) * (size_t)tokens * p->d.hidden);
  if (p->has_sfp8) n += 2 * align256(sizeof(float) * (size_t)tokens * p->d.inter);
  return n;
}

// Batched path (tokens >= kGroupedMinTokens): router, routing bookkeeping and
// dispatch, grouped up/down GEMMs on the tensor cores, combine.
wh_status moe_ffn_grouped(wh_ctx* c, const wh_moe_plan* p, const float* x, int tokens,
                          const int32_t* hash_ids, float* y, int32_t* ids_out,
                          float* weights_out, void* scratch, size_t scratch_bytes,
                          wh_stream_t stream) {
  const auto& d = p->d;
  GroupedScratch g = grouped_scratch_layout(p, tokens, static_cast<uint8_t*>(scratch));
  if (scratch_bytes < g.bytes) return fail(WH_ERR_SCRATCH_TOO_SMALL, "moe scratch too small");
  const int has_shared = d.shared ? 1 : 0;
  RouterArgs r{};
  r.gate = d.gate;
  r.experts = d.num_experts;
  r.hidden = d.hidden;
  r.x = x;
  r.tokens = tokens;
  r.topk = d.topk;
  r.mode = d.router_mode;
  r.bias = d.gate_bias;
  r.route_scale = d.route_scale;
  r.hash_ids = hash_ids;
  r.logits = g.logits;
  r.ids = ids_out ? ids_out : g.ids;
  r.weights = weights_out ? weights_out : g.weights;
  r.combine_w = g.combine_w;
  r.counters = p->counters;
  r.status = c->status;
  GroupedPlanArgs pa{};
  pa.ids = r.ids;
  pa.tokens = tokens;
  pa.topk = d.topk;
  pa.num_experts = d.num_experts;
  pa.has_shared = has_shared;
  pa.counts = g.counts;
  pa.slot = g.slot;
  pa.offsets = g.offsets;
  pa.units_up = g.units_up;
  pa.units_down = g.units_down;
  pa.n_units = g.n_units;
  pa.mt_up = d.inter / 128;
  pa.mt_down = d.hidden / 128;
  pa.tile_n = grouped_tile_n(p, tokens);
  pa.route_order = tokens < kGroupedMinTokens;
  pa.status = c->status;
  CUtensorMap bup, bdown;
  wh_status st;
  if ((st = make_u8_map(&bup, g.xq, g.rows, d.hidden, pa.tile_n, 128)) != WH_OK) return st;
  if ((st = make_u8_map(&bdown, g.hq, g.rows, d.inter, pa.tile_n, 128)) != WH_OK) return st;
  GroupedArgs up{};
  up.amaps = p->set.gmaps;
  up.experts = p->set.experts;
  up.K = d.hidden;
  up.M = d.inter;
  up.bsf = g.xsf;
  up.bsf_stride = d.hidden / 32;
  up.rows_total = g.rows;
  up.units = g.units_up;
  up.n_units = g.n_units;
  up.hq = g.hq;
  up.hsf = g.hsf;
  up.status = c->status;
  GroupedArgs down = up;
  down.K = d.inter;
  down.M = d.hidden;
  down.bsf = g.hsf;
  down.bsf_stride = d.inter / 32;
  down.units = g.units_down;
  down.n_units = g.n_units + 1;
  down.hq = nullptr;
  down.hsf = nullptr;
  down.y = g.yrows;
  c->prof_begin();
  if ((st = c->prof_mark(stream)) != WH_OK) return st;
  WH_CUDA(cudaMemsetAsync(g.counts, 0, sizeof(int) * (d.num_experts + 1), stream));
  WH_CUDA(launch_router_ex(r, nullptr, nullptr, stream, false));
  if ((st = c->prof_mark(stream)) != WH_OK) return st;
  WH_CUDA(launch_grouped_route(pa, x, d.hidden, g.xq, g.xsf, stream));
  if ((st = c->prof_mark(stream)) != WH_OK) return st;
  WH_CUDA(launch_grouped_gemm(true, pa.tile_n, bup, up, c->num_sms, stream));
  if ((st = c->prof_mark(stream)) != WH_OK) return st;
  WH_CUDA(launch_grouped_gemm(false, pa.tile_n, bdown, down, c->num_sms, stream));
  if ((st = c->prof_mark(stream)) != WH_OK) return st;
  WH_CUDA(launch_grouped_combine(pa, g.yrows, g.combine_w, x, y, d.hidden, stream));
  return c->prof_mark(stream);
}

static wh_status moe_ffn_routed(wh_ctx* c, const wh_moe_plan* p, const float* x, int tokens,
                                const int32_t* hash_ids, float* y, int32_t* ids_out,
                                float* weights_out, void* scratch, size_t scratch_bytes,
                                wh_stream_t stream);

wh_status wh_moe_ffn(wh_ctx* c, const wh_moe_plan* p, const float* x, int tokens,
                     const int32_t* hash_ids, float* y, int32_t* ids_out, float* weights_out,
                     void* scratch, size_t scratch_bytes, wh_stream_t stream) {
  wh_status st = moe_ffn_routed(c, p, x, tokens, hash_ids, y, ids_out, weights_out, scratch,
                                scratch_bytes, stream);
  if (st != WH_OK || !p->has_sfp8) return st;
  // y = shared(x) + routed (src/compute.rs:1940-1944): the FP8 shared expert's
  // w2 GEMV adds the routed result in its epilogue
  uint8_t* base = static_cast<uint8_t*>(scratch) + align256(moe_path_scratch_bytes(p, tokens));
  const float* xd = device_reach(x) == 1 ? reinterpret_cast<const float*>(base) : x;
  base += align256(sizeof(float) * (size_t)tokens * p->d.hidden);
  float* h1 = reinterpret_cast<float*>(base);
  float* h3 = reinterpret_cast<float*>(base + align256(sizeof(float) * (size_t)tokens * p->d.inter));
  return fp8_expert_run(c, p->sfp8, xd, tokens, p->d.hidden, y, p->d.hidden, y, h1, h3, stream);
}

static wh_status moe_ffn_routed(wh_ctx* c, const wh_moe_plan* p, const float* x, int tokens,
                                const int32_t* hash_ids, float* y, int32_t* ids_out,
                                float* weights_out, void* scratch, size_t scratch_bytes,
                                wh_stream_t stream) {
  if (!c || !p) return fail(WH_ERR_INVALID_POINTER, "null ctx/plan");
  if (tokens <= 0) return fail(WH_ERR_EMPTY_SHAPE, "tokens <= 0");
  if (tokens > p->d.max_tokens) return fail(WH_ERR_INVALID_SHAPE, "tokens > plan max_tokens");
  if (!x || !y || !scratch) return fail(WH_ERR_INVALID_POINTER, "null buffer");
  if (!p->d.gate) return fail(WH_ERR_INVALID_POINTER, "plan has no router gate");
  if (!aligned(x, 16) || !aligned(scratch, 256))
    return fail(WH_ERR_INVALID_POINTER, "x must be 16-byte and scratch 256-byte aligned");
  if (scratch_bytes < wh_moe_scratch_bytes(p, tokens))
    return fail(WH_ERR_SCRATCH_TOO_SMALL, "moe scratch too small");
  // x and y may be device memory or pinned host memory the device can address
  // (the reference passes host slices): x is then pulled into the scratch by a
  // kernel and y is written straight to host memory by the last kernel, with no
  // copy-engine transfer on either side
  const int xk = device_reach(x), yk = device_reach(y);
  if (xk < 0 || yk < 0)
    return fail(WH_ERR_INVALID_POINTER,
                "x and y must be device memory or pinned, device-mapped host memory");
  if (xk == 1) {
    float* xs = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) +
                                         align256(moe_path_scratch_bytes(p, tokens)));
    WH_CUDA(launch_stage_rows(x, xs, (size_t)tokens * p->d.hidden, stream));
    x = xs;
  }
  if (use_grouped(p, tokens))
    return moe_ffn_grouped(c, p, x, tokens, hash_ids, y, ids_out, weights_out, scratch,
                           scratch_bytes, stream);
  MoeScratch s = moe_scratch_layout(p, tokens, static_cast<uint8_t*>(scratch));
  if (scratch_bytes < s.bytes) return fail(WH_ERR_SCRATCH_TOO_SMALL, "moe scratch too small");
  const auto& d = p->d;
  RouterArgs r{};
  r.gate = d.gate;
  r.experts = d.num_experts;
  r.hidden = d.hidden;
  r.x = x;
  r.tokens = tokens;
  r.topk = d.topk;
  r.mode = d.router_mode;
  r.bias = d.gate_bias;
  r.route_scale = d.route_scale;
  r.hash_ids = hash_ids;
  r.logits = s.logits;
  r.ids = ids_out ? ids_out : s.ids;
  r.weights = weights_out ? weights_out : s.weights;
  r.combine_w = s.combine_w;
  r.counters = p->counters;
  r.status = c->status;
  c->prof_begin();
  wh_status pst;
  if ((pst = c->prof_mark(stream)) != WH_OK) return pst;
  MoeArgs a{};
  a.maps = p->set.maps;
  a.experts = p->set.experts;
  a.num_experts = d.num_experts;
  a.has_shared = d.shared ? 1 : 0;
  a.hidden = d.hidden;
  a.inter = d.inter;
  a.x = x;
  a.tokens = tokens;
  a.topk = d.topk;
  a.ids = r.ids;
  a.combine_w = s.combine_w;
  a.h = s.h;
  a.blk_counters = p->blk_counters;
  a.y = y;
  a.expert_out = nullptr;
  a.combine = 1;
  a.status = c->status;
  wh_moe_plan* mp = const_cast<wh_moe_plan*>(p);
  if (tokens == 1 && p->decode_on) {
    if (mp->decode_ok < 0)
      mp->decode_ok = decode_supported(d.num_experts, d.hidden, d.inter, d.topk,
                                       d.shared ? 1 : 0, c->num_sms) ? 1 : 0;
    if (mp->decode_ok) {
      // the whole step as one persistent kernel (decode.cu)
      DecodeArgs da{};
      da.r = r;
      da.m = a;
      da.dmaps = p->set.dmaps;
      da.xq = s.xq;
      da.xq_mult = s.xq_mult;
      da.hq = s.hq;
      da.hq_mult = s.hq_mult;
      da.sync = p->dec_sync;
      WH_CUDA(launch_moe_decode(da, c->num_sms, stream));
      return c->prof_mark(stream);
    }
  }
  WH_CUDA(launch_router_ex(r, s.xq, s.xq_mult, stream, c->pdl()));
  if ((pst = c->prof_mark(stream)) != WH_OK) return pst;
  WH_CUDA(launch_moe_up_ex(a, s.xq, s.xq_mult, s.hq, s.hq_mult, stream, c->pdl()));
  if ((pst = c->prof_mark(stream)) != WH_OK) return pst;
  WH_CUDA(launch_moe_down_ex(a, s.hq, s.hq_mult, stream, c->pdl()));
  return c->prof_mark(stream);
}


void wh_debug_act_quant_table(uint32_t out[256]) {
  const ActQuantTable& t = act_quant_table_host();
  memcpy(out, t.thr, sizeof(t.thr));
}

float wh_debug_e4m3_round(float t) { return e4m3_nearest_ties_lower(t); }

void wh_debug_e4m3_round_n(const float* in, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = e4m3_nearest_ties_lower(in[i]);
}

int wh_debug_expf_table(const uint32_t** keys, const float** vals) {
  int n = 0;
  const bool ok = expf_table_host(keys, vals, &n);
  return ok ? n : -n;
}

double wh_debug_expf_near(void) { return expf_near_host(); }

wh_status wh_debug_ref_expf(wh_ctx* c, const float* x, float* y, size_t n, wh_stream_t stream) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "ctx is null");
  if (n > 0 && (!x || !y)) return fail(WH_ERR_INVALID_POINTER, "null pointer");
  cudaSetDevice(c->device);
  WH_CUDA(launch_ref_expf(x, y, (long long)n, (cudaStream_t)stream));
  return WH_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Expert parallelism (routed experts sharded over ranks, collectives between
// the calls).  The plan holds the rank's local experts (and the shared one).
// ---------------------------------------------------------------------------
namespace {
struct EpScratch {
  int* slot;
  int* off;
  int* seg_cnt;
  int* totals;
  int* seg_off;
  int* src_off;
  int* exp_off;
  int* row_map;
  int4* units_up;
  int4* units_down;
  int* n_units;
  uint8_t* sorted;
  uint8_t* hq;
  uint8_t* hsf;
  size_t bytes;
};
EpScratch ep_scratch_layout(const wh_moe_plan* p, int world, int tokens, int max_recv_rows,
                            uint8_t* base) {
  const auto& d = p->d;
  const int El = d.num_experts, nseg = world * El;
  const size_t rows = (size_t)max_recv_rows + tokens;
  const size_t tiles = rows / kGN + El + 2;
  const size_t rb = wh_ep_row_bytes(d.hidden);
  EpScratch s{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* q = base ? base + off : nullptr;
    off += align256(bytes);
    return q;
  };
  s.slot = reinterpret_cast<int*>(take(sizeof(int) * (size_t)tokens * d.topk));
  s.off = reinterpret_cast<int*>(take(sizeof(int) * nseg));
  s.seg_cnt = reinterpret_cast<int*>(take(sizeof(int) * nseg));
  s.totals = reinterpret_cast<int*>(take(sizeof(int) * (El + 1)));
  s.seg_off = reinterpret_cast<int*>(take(sizeof(int) * nseg));
  s.src_off = reinterpret_cast<int*>(take(sizeof(int) * nseg));
  s.exp_off = reinterpret_cast<int*>(take(sizeof(int) * (El + 2)));
  s.row_map = reinterpret_cast<int*>(take(sizeof(int) * rows));
  s.units_up = reinterpret_cast<int4*>(take(sizeof(int4) * tiles * (d.inter / 128)));
  s.units_down = reinterpret_cast<int4*>(take(sizeof(int4) * tiles * (d.hidden / 128)));
  s.n_units = reinterpret_cast<int*>(take(sizeof(int) * 2));
  s.sorted = take(rows * rb);
  s.hq = take(rows * d.inter);
  s.hsf = take(rows * (d.inter / 32));
  s.bytes = off;
  return s;
}
wh_status ep_check(const wh_moe_plan* p, int world) {
  if (!p) return fail(WH_ERR_INVALID_POINTER, "null plan");
  if (p->has_sfp8)
    return fail(WH_ERR_UNSUPPORTED, "expert parallelism takes an FP4 shared expert");
  if (world < 1 || world * p->d.num_experts > 1024)
    return fail(WH_ERR_UNSUPPORTED, "world * local experts must be in [1, 1024]");
  if (!p->grouped)
    return fail(WH_ERR_UNSUPPORTED,
                "expert parallelism runs on the tensor-core path: hidden and inter multiples "
                "of 512, desc.exact != 1, no UE8M0 scale byte 0 or 255");
  return WH_OK;
}
}  // namespace

extern "C" {

size_t wh_ep_row_bytes(int hidden) {
  return ((size_t)hidden + (size_t)hidden / 32 + 15) & ~size_t(15);
}

size_t wh_ep_scratch_bytes(const wh_moe_plan* p, int world, int tokens, int max_recv_rows) {
  if (!p || world < 1 || tokens < 0 || max_recv_rows < 0) return 0;
  return ep_scratch_layout(p, world, tokens, max_recv_rows, nullptr).bytes;
}

wh_status wh_ep_dispatch(wh_ctx* c, const wh_moe_plan* p, int world, const float* x, int tokens,
                         const int32_t* ids, uint8_t* send, int32_t* send_counts, int32_t* pos,
                         void* scratch, size_t scratch_bytes, wh_stream_t stream) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "null ctx");
  wh_status st;
  if ((st = ep_check(p, world)) != WH_OK) return st;
  if (tokens < 0) return fail(WH_ERR_INVALID_SHAPE, "tokens < 0");
  if (!send_counts || !scratch) return fail(WH_ERR_INVALID_POINTER, "null buffer");
  const auto& d = p->d;
  EpScratch s = ep_scratch_layout(p, world, tokens, 0, static_cast<uint8_t*>(scratch));
  if (scratch_bytes < s.bytes) return fail(WH_ERR_SCRATCH_TOO_SMALL, "ep scratch too small");
  if (tokens == 0) {
    WH_CUDA(cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * world * d.num_experts, stream));
    return WH_OK;
  }
  if (!x || !ids || !send || !pos) return fail(WH_ERR_INVALID_POINTER, "null buffer");
  if (!aligned(x, 16) || !aligned(send, 16)) return fail(WH_ERR_INVALID_POINTER, "alignment");
  EpArgs a{};
  a.world = world;
  a.local_experts = d.num_experts;
  a.topk = d.topk;
  a.hidden = d.hidden;
  a.row_bytes = (int)wh_ep_row_bytes(d.hidden);
  a.ids = ids;
  a.tokens = tokens;
  a.cnt = send_counts;
  a.slot = s.slot;
  a.off = s.off;
  a.pos = pos;
  a.status = c->status;
  WH_CUDA(launch_ep_dispatch(a, x, send, stream));
  return WH_OK;
}

wh_status wh_ep_expert_ffn(wh_ctx* c, const wh_moe_plan* p, int world, const uint8_t* recv,
                           const int32_t* recv_counts, int recv_rows, const float* x_local,
                           int tokens, float* y_rows, void* scratch, size_t scratch_bytes,
                           wh_stream_t stream) {
  if (!c) return fail(WH_ERR_INVALID_POINTER, "null ctx");
  wh_status st;
  if ((st = ep_check(p, world)) != WH_OK) return st;
  if (recv_rows < 0 || tokens < 0) return fail(WH_ERR_INVALID_SHAPE, "negative rows");
  const auto& d = p->d;
  const int has_shared = d.shared ? 1 : 0;
  const int rows = recv_rows + (has_shared ? tokens : 0);
  if (rows == 0) return WH_OK;
  if (!recv_counts || !y_rows || !scratch || (recv_rows > 0 && !recv) || (tokens > 0 && !x_local))
    return fail(WH_ERR_INVALID_POINTER, "null buffer");
  EpScratch s = ep_scratch_layout(p, world, tokens, recv_rows, static_cast<uint8_t*>(scratch));
  if (scratch_bytes < s.bytes) return fail(WH_ERR_SCRATCH_TOO_SMALL, "ep scratch too small");
  const int rb = (int)wh_ep_row_bytes(d.hidden);
  EpSortArgs so{};
  so.recv_counts = recv_counts;
  so.world = world;
  so.local_experts = d.num_experts;
  so.seg_stride = 0;
  so.max_rows = recv_rows;
  so.status = c->status;
  so.seg_cnt = s.seg_cnt;
  so.totals = s.totals;
  so.seg_off = s.seg_off;
  so.src_off = s.src_off;
  so.exp_off = s.exp_off;
  so.recv = recv;
  so.sorted = s.sorted;
  so.row_map = s.row_map;
  so.row_bytes = rb;
  GroupedPlanArgs g{};
  g.tokens = has_shared ? tokens : 0;
  g.num_experts = d.num_experts;
  g.has_shared = has_shared;
  g.counts = s.totals;
  g.offsets = s.exp_off;
  g.units_up = s.units_up;
  g.units_down = s.units_down;
  g.n_units = s.n_units;
  g.mt_up = d.inter / 128;
  g.mt_down = d.hidden / 128;
  g.tile_n = kGN;
  g.status = c->status;
  WH_CUDA(launch_ep_prepare(so, g, x_local, d.hidden, recv_rows, stream));
  // B operand: the sorted rows (E4M3 hidden bytes, then the exponents)
  CUtensorMap bup, bdown;
  if ((st = make_u8_map_strided(&bup, s.sorted, rows, d.hidden, rb, kGN)) != WH_OK) return st;
  if ((st = make_u8_map(&bdown, s.hq, rows, d.inter, kGN, 128)) != WH_OK) return st;
  GroupedArgs up{};
  up.amaps = p->set.gmaps;
  up.experts = p->set.experts;
  up.K = d.hidden;
  up.M = d.inter;
  up.bsf = s.sorted + d.hidden;
  up.bsf_stride = rb;
  up.rows_total = rows;
  up.units = s.units_up;
  up.n_units = s.n_units;
  up.hq = s.hq;
  up.hsf = s.hsf;
  up.status = c->status;
  GroupedArgs dn = up;
  dn.K = d.inter;
  dn.M = d.hidden;
  dn.bsf = s.hsf;
  dn.bsf_stride = d.inter / 32;
  dn.units = s.units_down;
  dn.n_units = s.n_units + 1;
  dn.hq = nullptr;
  dn.hsf = nullptr;
  dn.y = y_rows;
  dn.y_row_map = s.row_map;
  WH_CUDA(launch_grouped_gemm(true, kGN, bup, up, c->num_sms, stream));
  WH_CUDA(launch_grouped_gemm(false, kGN, bdown, dn, c->num_sms, stream));
  return WH_OK;
}

wh_status wh_ep_combine(wh_ctx* c, const wh_moe_plan* p, const int32_t* ids, const float* weights,
                        const int32_t* pos, int tokens, const float* y_back, const float* y_shared,
                        float* y, wh_stream_t stream) {
  if (!c || !p) return fail(WH_ERR_INVALID_POINTER, "null ctx/plan");
  if (tokens <= 0) return WH_OK;
  if (!ids || !weights || !pos || !y || (!y_back && p->d.topk > 0) || (p->d.shared && !y_shared))
    return fail(WH_ERR_INVALID_POINTER, "null buffer");
  WH_CUDA(launch_ep_combine(ids, weights, pos, tokens, p->d.topk, y_back, y_shared,
                            p->d.shared ? 1 : 0, y, p->d.hidden, stream));
  return WH_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Expert parallelism over peer memory (CUDA IPC windows, NVLink stores).
// ---------------------------------------------------------------------------
static_assert(sizeof(cudaIpcMemHandle_t) == WH_EP_IPC_HANDLE_BYTES, "IPC handle size");

struct wh_ep_window {
  wh_ctx* ctx = nullptr;
  const wh_moe_plan* plan = nullptr;
  int world = 0, rank = 0, max_tokens = 0, cap = 0, row_bytes = 0;
  // the exported window: [recv rows | counts | row flags, result flags | result rows]
  uint8_t* base = nullptr;
  size_t bytes = 0, o_recv = 0, o_counts = 0, o_flags = 0, o_yback = 0;
  // rank-private state
  uint8_t* local = nullptr;
  EpScratch sc{};
  int* cnt = nullptr;
  int* off = nullptr;
  uint32_t* done = nullptr;  // [2] arrival counters: dispatch, down GEMM
  EpPeer* peers = nullptr;   // [world]
  float** yback_peers = nullptr;        // [world] peer d's result rows
  uint64_t** res_flag_peers = nullptr;  // [world] &peer d's res_flag[rank]
  int32_t* pos = nullptr;    // [max_tokens * topk] result row of each route (wh_ep_moe_layer)
  float* y_shared = nullptr; // [max_tokens][hidden] shared-expert output (wh_ep_moe_layer)
  CUtensorMap bup{}, bdown{};
  std::vector<void*> opened;
  uint64_t epoch = 0;
  int stage = 0;  // 0 idle / after combine, 1 dispatched, 2 expert FFN issued
  bool connected = false;
};

namespace {
struct EpWindowLayout {
  size_t recv, counts, flags, yback, bytes;
};
EpWindowLayout ep_window_layout(const wh_moe_plan* p, int world, int cap) {
  const auto& d = p->d;
  EpWindowLayout w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += align256(bytes);
    return at;
  };
  w.recv = take((size_t)world * cap * wh_ep_row_bytes(d.hidden));
  w.counts = take(sizeof(int) * (size_t)world * d.num_experts);
  w.flags = take(sizeof(uint64_t) * 2 * (size_t)world);
  w.yback = take(sizeof(float) * (size_t)world * cap * d.hidden);
  w.bytes = off;
  return w;
}
wh_status ep_window_args(const wh_moe_plan* p, int world, int rank, int max_tokens) {
  wh_status st;
  if ((st = ep_check(p, world)) != WH_OK) return st;
  if (rank < 0 || rank >= world) return fail(WH_ERR_INVALID_SHAPE, "rank out of [0, world)");
  if (max_tokens < 1) return fail(WH_ERR_INVALID_SHAPE, "max_tokens < 1");
  if ((long long)world * max_tokens * p->d.topk + max_tokens > (1LL << 30))
    return fail(WH_ERR_INVALID_SHAPE, "world * max_tokens * topk too large");
  return WH_OK;
}
void ep_window_free(wh_ep_window* w) {
  for (void* q : w->opened) cudaIpcCloseMemHandle(q);
  if (w->base) cudaFree(w->base);
  if (w->local) cudaFree(w->local);
  delete w;
}
}  // namespace

extern "C" {

size_t wh_ep_window_bytes(const wh_moe_plan* p, int world, int max_tokens) {
  if (ep_window_args(p, world, 0, max_tokens) != WH_OK) return 0;
  return ep_window_layout(p, world, max_tokens * p->d.topk).bytes;
}

wh_status wh_ep_window_create(wh_ctx* c, const wh_moe_plan* p, int world, int rank,
                              int max_tokens, wh_ep_window** out, uint8_t* ipc_handle) {
  if (!c || !out || !ipc_handle) return fail(WH_ERR_INVALID_POINTER, "null ctx/out/handle");
  *out = nullptr;
  wh_status st;
  if ((st = ep_window_args(p, world, rank, max_tokens)) != WH_OK) return st;
  const auto& d = p->d;
  wh_ep_window* w = new wh_ep_window();
  w->ctx = c;
  w->plan = p;
  w->world = world;
  w->rank = rank;
  w->max_tokens = max_tokens;
  w->cap = max_tokens * d.topk;
  w->row_bytes = (int)wh_ep_row_bytes(d.hidden);
  const EpWindowLayout L = ep_window_layout(p, world, w->cap);
  w->bytes = L.bytes;
  w->o_recv = L.recv;
  w->o_counts = L.counts;
  w->o_flags = L.flags;
  w->o_yback = L.yback;
  const int nseg = world * d.num_experts;
  const size_t sc_bytes =
      ep_scratch_layout(p, world, max_tokens, world * w->cap, nullptr).bytes;
  const size_t tab = align256(sc_bytes) + 2 * align256(sizeof(int) * nseg) + 256 +
                     align256(sizeof(EpPeer) * world) + 2 * align256(sizeof(void*) * world) +
                     align256(sizeof(int32_t) * (size_t)w->cap) +
                     align256(sizeof(float) * (size_t)max_tokens * d.hidden);
  cudaError_t e = cudaMalloc(&w->base, w->bytes);
  if (e == cudaSuccess) e = cudaMemset(w->base, 0, w->bytes);
  if (e == cudaSuccess) e = cudaMalloc(&w->local, tab);
  if (e == cudaSuccess) e = cudaMemset(w->local, 0, tab);
  cudaIpcMemHandle_t h{};
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, w->base);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    ep_window_free(w);
    return cuda_fail(e, "expert-parallel window");
  }
  size_t o = 0;
  w->sc = ep_scratch_layout(p, world, max_tokens, world * w->cap, w->local);
  o += align256(sc_bytes);
  w->cnt = reinterpret_cast<int*>(w->local + o);
  o += align256(sizeof(int) * nseg);
  w->off = reinterpret_cast<int*>(w->local + o);
  o += align256(sizeof(int) * nseg);
  w->done = reinterpret_cast<uint32_t*>(w->local + o);
  o += 256;
  w->peers = reinterpret_cast<EpPeer*>(w->local + o);
  o += align256(sizeof(EpPeer) * world);
  w->yback_peers = reinterpret_cast<float**>(w->local + o);
  o += align256(sizeof(void*) * world);
  w->res_flag_peers = reinterpret_cast<uint64_t**>(w->local + o);
  o += align256(sizeof(void*) * world);
  w->pos = reinterpret_cast<int32_t*>(w->local + o);
  o += align256(sizeof(int32_t) * (size_t)w->cap);
  w->y_shared = reinterpret_cast<float*>(w->local + o);
  // B operand maps over the fixed sorted-row and h buffers
  const int rows = world * w->cap + max_tokens;
  if ((st = make_u8_map_strided(&w->bup, w->sc.sorted, rows, d.hidden, w->row_bytes, kGN)) !=
          WH_OK ||
      (st = make_u8_map(&w->bdown, w->sc.hq, rows, d.inter, kGN, 128)) != WH_OK) {
    ep_window_free(w);
    return st;
  }
  memcpy(ipc_handle, &h, WH_EP_IPC_HANDLE_BYTES);
  *out = w;
  return WH_OK;
}

wh_status wh_ep_window_connect(wh_ep_window* w, const uint8_t* handles) {
  if (!w || !handles) return fail(WH_ERR_INVALID_POINTER, "null window/handles");
  if (w->connected) return fail(WH_ERR_UNSUPPORTED, "window already connected");
  std::vector<EpPeer> peers(w->world);
  std::vector<float*> yb(w->world);
  std::vector<uint64_t*> rf(w->world);
  for (int d = 0; d < w->world; ++d) {
    uint8_t* b = w->base;
    if (d != w->rank) {
      cudaIpcMemHandle_t h;
      memcpy(&h, handles + (size_t)d * WH_EP_IPC_HANDLE_BYTES, WH_EP_IPC_HANDLE_BYTES);
      void* q = nullptr;
      WH_CUDA(cudaIpcOpenMemHandle(&q, h, cudaIpcMemLazyEnablePeerAccess));
      w->opened.push_back(q);
      b = static_cast<uint8_t*>(q);
    }
    peers[d].recv = b + w->o_recv;
    peers[d].counts = reinterpret_cast<int*>(b + w->o_counts);
    peers[d].row_flag = reinterpret_cast<uint64_t*>(b + w->o_flags);
    peers[d].res_flag = peers[d].row_flag + w->world;
    peers[d].yback = reinterpret_cast<float*>(b + w->o_yback);
    yb[d] = peers[d].yback;
    rf[d] = peers[d].res_flag + w->rank;
  }
  WH_CUDA(cudaMemcpy(w->peers, peers.data(), sizeof(EpPeer) * w->world, cudaMemcpyHostToDevice));
  WH_CUDA(cudaMemcpy(w->yback_peers, yb.data(), sizeof(void*) * w->world,
                     cudaMemcpyHostToDevice));
  WH_CUDA(cudaMemcpy(w->res_flag_peers, rf.data(), sizeof(void*) * w->world,
                     cudaMemcpyHostToDevice));
  w->connected = true;
  return WH_OK;
}

void wh_ep_window_destroy(wh_ep_window* w) {
  if (!w) return;
  cudaDeviceSynchronize();
  ep_window_free(w);
}

wh_status wh_ep_p2p_dispatch(wh_ctx* c, wh_ep_window* w, const float* x, int tokens,
                             const int32_t* ids, int32_t* pos, wh_stream_t stream) {
  if (!c || !w) return fail(WH_ERR_INVALID_POINTER, "null ctx/window");
  if (!w->connected) return fail(WH_ERR_UNSUPPORTED, "window not connected");
  if (w->stage != 0) return fail(WH_ERR_UNSUPPORTED, "dispatch before the previous combine");
  if (tokens < 0 || tokens > w->max_tokens)
    return fail(WH_ERR_INVALID_SHAPE, "tokens outside [0, max_tokens]");
  if (tokens > 0 && (!x || !ids || !pos)) return fail(WH_ERR_INVALID_POINTER, "null buffer");
  if (tokens > 0 && !aligned(x, 16)) return fail(WH_ERR_INVALID_POINTER, "alignment");
  const auto& d = w->plan->d;
  EpArgs a{};
  a.world = w->world;
  a.local_experts = d.num_experts;
  a.topk = d.topk;
  a.hidden = d.hidden;
  a.row_bytes = w->row_bytes;
  a.ids = ids;
  a.tokens = tokens;
  a.cnt = w->cnt;
  a.slot = w->sc.slot;
  a.status = c->status;
  EpP2pArgs q{};
  q.world = w->world;
  q.rank = w->rank;
  q.local_experts = d.num_experts;
  q.topk = d.topk;
  q.hidden = d.hidden;
  q.row_bytes = w->row_bytes;
  q.cap = w->cap;
  q.ids = ids;
  q.tokens = tokens;
  q.cnt = w->cnt;
  q.slot = w->sc.slot;
  q.off = w->off;
  q.pos = pos;
  q.peers = w->peers;
  q.done = w->done;
  q.epoch = w->epoch + 1;
  q.status = c->status;
  WH_CUDA(launch_ep_p2p_dispatch(q, a, x, stream));
  ++w->epoch;
  w->stage = 1;
  return WH_OK;
}

wh_status wh_ep_p2p_expert_ffn(wh_ctx* c, wh_ep_window* w, const float* x_local, int tokens,
                               float* y_shared, wh_stream_t stream) {
  if (!c || !w) return fail(WH_ERR_INVALID_POINTER, "null ctx/window");
  if (w->stage != 1) return fail(WH_ERR_UNSUPPORTED, "expert FFN without a dispatch");
  if (tokens < 0 || tokens > w->max_tokens)
    return fail(WH_ERR_INVALID_SHAPE, "tokens outside [0, max_tokens]");
  const auto& d = w->plan->d;
  const int has_shared = d.shared ? 1 : 0;
  if (has_shared && tokens > 0 && (!x_local || !y_shared))
    return fail(WH_ERR_INVALID_POINTER, "null buffer");
  if (has_shared && tokens > 0 && !aligned(x_local, 16))
    return fail(WH_ERR_INVALID_POINTER, "alignment");
  const int peer_rows = w->world * w->cap;
  const EpScratch& s = w->sc;
  EpSortArgs so{};
  so.recv_counts = reinterpret_cast<const int*>(w->base + w->o_counts);
  so.world = w->world;
  so.local_experts = d.num_experts;
  so.seg_stride = w->cap;
  so.max_rows = peer_rows;
  so.wait = reinterpret_cast<const uint64_t*>(w->base + w->o_flags);
  so.epoch = w->epoch;
  so.status = c->status;
  so.seg_cnt = s.seg_cnt;
  so.totals = s.totals;
  so.seg_off = s.seg_off;
  so.src_off = s.src_off;
  so.exp_off = s.exp_off;
  so.recv = w->base + w->o_recv;
  so.sorted = s.sorted;
  so.row_map = s.row_map;
  so.row_bytes = w->row_bytes;
  GroupedPlanArgs g{};
  g.tokens = has_shared ? tokens : 0;
  g.num_experts = d.num_experts;
  g.has_shared = has_shared;
  g.counts = s.totals;
  g.offsets = s.exp_off;
  g.units_up = s.units_up;
  g.units_down = s.units_down;
  g.n_units = s.n_units;
  g.mt_up = d.inter / 128;
  g.mt_down = d.hidden / 128;
  g.tile_n = kGN;
  g.status = c->status;
  WH_CUDA(launch_ep_prepare(so, g, x_local, d.hidden, peer_rows, stream));
  GroupedArgs up{};
  up.amaps = w->plan->set.gmaps;
  up.experts = w->plan->set.experts;
  up.K = d.hidden;
  up.M = d.inter;
  up.bsf = s.sorted + d.hidden;
  up.bsf_stride = w->row_bytes;
  up.rows_total = peer_rows + w->max_tokens;
  up.units = s.units_up;
  up.n_units = s.n_units;
  up.hq = s.hq;
  up.hsf = s.hsf;
  up.status = c->status;
  GroupedArgs dn = up;
  dn.K = d.inter;
  dn.M = d.hidden;
  dn.bsf = s.hsf;
  dn.bsf_stride = d.inter / 32;
  dn.units = s.units_down;
  dn.n_units = s.n_units + 1;
  dn.hq = nullptr;
  dn.hsf = nullptr;
  dn.y = y_shared;
  dn.y_row_map = s.row_map;
  dn.y_peers = w->yback_peers;
  dn.y_peer_rows = peer_rows;
  dn.y_cap = w->cap;
  dn.y_self_off = w->rank * w->cap;
  dn.sig_flags = w->res_flag_peers;
  dn.sig_done = w->done + 1;
  dn.sig_n = w->world;
  dn.sig_epoch = w->epoch;
  WH_CUDA(launch_grouped_gemm(true, kGN, w->bup, up, c->num_sms, stream));
  WH_CUDA(launch_grouped_gemm(false, kGN, w->bdown, dn, c->num_sms, stream));
  w->stage = 2;
  return WH_OK;
}

wh_status wh_ep_p2p_combine(wh_ctx* c, wh_ep_window* w, const int32_t* ids, const float* weights,
                            const int32_t* pos, int tokens, const float* y_shared, float* y,
                            wh_stream_t stream) {
  if (!c || !w) return fail(WH_ERR_INVALID_POINTER, "null ctx/window");
  if (w->stage != 2) return fail(WH_ERR_UNSUPPORTED, "combine without an expert FFN");
  if (tokens < 0 || tokens > w->max_tokens)
    return fail(WH_ERR_INVALID_SHAPE, "tokens outside [0, max_tokens]");
  const auto& d = w->plan->d;
  if (tokens > 0 && (!ids || !weights || !pos || !y || (d.shared && !y_shared)))
    return fail(WH_ERR_INVALID_POINTER, "null buffer");
  WH_CUDA(launch_ep_p2p_combine(
      ids, weights, pos, tokens, d.topk, reinterpret_cast<const float*>(w->base + w->o_yback),
      y_shared, d.shared ? 1 : 0, y, d.hidden,
      reinterpret_cast<const uint64_t*>(w->base + w->o_flags) + w->world, w->world, w->epoch,
      c->status, stream));
  w->stage = 0;
  return WH_OK;
}

wh_status wh_ep_moe_layer(wh_ctx* c, wh_ep_window* w, const float* x, int tokens,
                          const int32_t* ids, const float* weights, float* y,
                          wh_stream_t stream) {
  if (!c || !w) return fail(WH_ERR_INVALID_POINTER, "null ctx/window");
  if (tokens > w->max_tokens) return fail(WH_ERR_INVALID_SHAPE, "tokens > the window's max_tokens");
  wh_status st;
  if ((st = wh_ep_p2p_dispatch(c, w, x, tokens, ids, w->pos, stream)) != WH_OK) return st;
  if ((st = wh_ep_p2p_expert_ffn(c, w, x, tokens, w->y_shared, stream)) != WH_OK) return st;
  return wh_ep_p2p_combine(c, w, ids, weights, w->pos, tokens, w->y_shared, y, stream);
}

}  // extern "C"
