// noalloc.cu -- wh_fp4_expert_forward_noalloc: the FP4 expert forward with its
// scratch in a fixed, statically sized device array of this module instead of
// caller or context memory.  A call allocates no device memory (no cudaMalloc,
// no cudaFree, no allocating library) however many experts or shapes it sees.
//
// Scratch: the file-scope array g_expert_scratch below, kNoAllocScratchFloats
// floats (256 KiB).  One call uses hidden + 2 * inter floats of it:
//   [0, hidden)                  act-quantised copy of the input
//   [hidden, hidden + inter)     w1 output, then SwiGLU h, then act-quantised h
//   [hidden + inter, + inter)    w3 output
// Every word a call reads is written earlier in the same call, so nothing in
// the array has to start at zero or be cleared between calls.  Larger experts
// are rejected with WH_ERR_SCRATCH_TOO_SMALL before anything is launched.
//
// Set-up: the array's device address is looked up once per device context,
// with that device current, by cudaGetSymbolAddress (which may load the
// module on that device); host code passes only that looked-up pointer to the
// kernels.  Make the first call on each device before any stream capture
// begins.  The lookup is keyed by the driver's context id (cuCtxGetId, never
// reused): after cudaDeviceReset the primary context is created anew, the
// module is loaded again and the array may move, so the next call looks it up
// again instead of launching on the old address.  That call is again a first
// call and belongs before any stream capture.
//
// The array is one per device and process: calls that overlap in time on one
// device (two streams, two threads, two contexts) race on it.  Calls issued in
// order on one stream are safe.
//
// The kernels are the exact (reference-order) FP4 path: act quant of the
// input, w1 and w3 matvecs, SwiGLU, act quant of h, w2 matvec -- the path
// wh_fp4_expert_forward takes for shapes its TMA kernels do not cover.

namespace wh {
constexpr size_t kNoAllocScratchFloats = 65536;  // 256 KiB
}  // namespace wh

static __device__ __align__(256) float g_expert_scratch[wh::kNoAllocScratchFloats];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {};
unsigned long long g_noalloc_ctx_id[kMaxDevices] = {};

using PfnCtxGetCurrent = CUresult (*)(CUcontext*);
using PfnCtxGetId = CUresult (*)(CUcontext, unsigned long long*);

// Id of the current driver context (unique for the life of the process).
wh_status current_ctx_id(unsigned long long* id) {
  static PfnCtxGetCurrent get_current = nullptr;
  static PfnCtxGetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PfnCtxGetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PfnCtxGetId>(p);
  });
  if (!get_current || !get_id) return fail(WH_ERR_CUDA, "cuCtxGetCurrent/cuCtxGetId unavailable");
  CUcontext cx = nullptr;
  if (get_current(&cx) != CUDA_SUCCESS || !cx) return fail(WH_ERR_CUDA, "no current CUDA context");
  if (get_id(cx, id) != CUDA_SUCCESS) return fail(WH_ERR_CUDA, "cuCtxGetId failed");
  return WH_OK;
}

// Device address of g_expert_scratch in the current context of `device`,
// looked up once per context.
wh_status noalloc_scratch(int device, float** out) {
  if (device < 0 || device >= kMaxDevices) return fail(WH_ERR_UNSUPPORTED, "device ordinal >= 64");
  unsigned long long id = 0;
  wh_status st = current_ctx_id(&id);
  if (st != WH_OK) return st;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[device] || g_noalloc_ctx_id[device] != id) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_expert_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(expert scratch)");
    if (!p || !aligned(p, 256)) return fail(WH_ERR_CUDA, "expert scratch address not 256-aligned");
    g_noalloc_ptr[device] = static_cast<float*>(p);
    g_noalloc_ctx_id[device] = id;
  }
  *out = g_noalloc_ptr[device];
  return WH_OK;
}

}  // namespace

extern "C" wh_status wh_fp4_expert_forward_noalloc(wh_ctx* c, const wh_fp4_expert* e,
                                                   const float* input, size_t input_len,
                                                   float* output, size_t output_len,
                                                   wh_stream_t stream) {
  if (!c || !e) return fail(WH_ERR_INVALID_POINTER, "null ctx/expert");
  // the argument checks of wh_fp4_expert_forward (src/deepseek_v4.rs:567-583)
  if (e->w1.cols != input_len || e->w3.cols != input_len || e->w1.rows != e->w3.rows ||
      e->w2.cols != e->w1.rows)
    return fail(WH_ERR_INVALID_SHAPE, "expert shapes");
  if (output_len < e->w2.rows) return fail(WH_ERR_OUTPUT_TOO_SMALL, "output too small");
  const size_t inter = e->w1.rows, hidden = input_len;
  wh_status st;
  if ((st = validate_fp4(e->w1, hidden, inter)) != WH_OK) return st;
  if ((st = validate_fp4(e->w3, hidden, inter)) != WH_OK) return st;
  if ((st = validate_fp4(e->w2, inter, output_len)) != WH_OK) return st;
  if (!input || !output) return fail(WH_ERR_INVALID_POINTER, "null buffer");
  if (hidden > kNoAllocScratchFloats || inter > kNoAllocScratchFloats ||
      hidden + 2 * inter > kNoAllocScratchFloats) {
    char buf[160];
    snprintf(buf, sizeof buf,
             "static expert scratch holds %zu floats; hidden + 2 * inter = %zu + 2 * %zu exceeds it",
             kNoAllocScratchFloats, hidden, inter);
    return fail(WH_ERR_SCRATCH_TOO_SMALL, buf);
  }
  int cur = -1;
  WH_CUDA(cudaGetDevice(&cur));
  if (cur != c->device) return fail(WH_ERR_CUDA, "the context's device is not the current device");
  float* scratch = nullptr;
  if ((st = noalloc_scratch(cur, &scratch)) != WH_OK) return st;

  float* xw = scratch;
  float* gate = scratch + hidden;
  float* up = gate + inter;
  WH_CUDA(cudaMemcpyAsync(xw, input, sizeof(float) * hidden, cudaMemcpyDeviceToDevice, stream));
  WH_CUDA(launch_act_quant(xw, (long long)hidden, 64, c->status, c->num_sms, stream));
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
