// libm_exact.cu -- the host C library's expf on the device, bit for bit.
//
// The reference computes f32::exp with the host's libm (glibc expf).  A device
// exp evaluated in double and rounded once to float is the correctly rounded
// result; glibc's expf is not correctly rounded everywhere (its documented
// error bound is slightly above half an ulp), so the two differ on a small,
// fixed set of inputs: about 1.7e5 of the 2.2e9 floats in (-104, 89) for
// glibc 2.39.  Those inputs all lie where exp(x) is within 2^-30 (relative) of
// a float rounding midpoint.
//
// The table is measured, not derived: at the first wh_ctx_create the library
// calls the running process's expf on every float in (-104, 89) (all host
// threads, about 3 s of host time once per process) and records each x whose
// expf differs from the once-rounded double exp, plus every x whose exp lies
// within 2^-44 of a midpoint (there a one-ulp difference between the host's and
// the device's double exp could flip the rounding).  The table is installed
// once per device in constant memory (c_expf).  On the device, ref_expf rounds
// exp((double)x) once and looks x up only when the result is close to a
// midpoint: one load of x's bucket bounds (2^20 buckets by the top 20 bits of
// x), then a binary search over that bucket's keys (65 at most for glibc 2.39,
// a few cache lines).  "Close" is a band measured with the table: the smallest
// power of two at least twice the farthest relative distance from a midpoint
// of any input where the two differ (2^-33.2 for glibc 2.39, so 2^-32: about
// 0.14 % of inputs are looked up), and never below the 2^-44 band.  Outside
// (-104, 89) both sides saturate to 0 or inf.  Every exp of the reference's arithmetic on this path
// (SiLU, the router's softplus and softmax, the MLA softmax) goes through
// libm_expf.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace wh {

namespace {

struct ExpfHostTable {
  std::vector<uint32_t> keys;  // float bits of x, ascending as uint32
  std::vector<float> vals;     // the host expf(x)
  std::vector<uint32_t> bucket;  // first key index per (bits >> 12) bucket, plus n
  bool model_ok = true;          // every difference lies inside the device gate
  double near = 0x1p-30;         // the device's lookup band (ExpfTable::near)
};

inline float bits_to_float(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
inline uint32_t float_to_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

void scan_expf_range(uint32_t lo, uint32_t hi, std::vector<uint32_t>& keys,
                     std::vector<float>& vals, bool& ok, double& far) {
  for (uint32_t u = lo; u < hi; ++u) {
    const float x = bits_to_float(u);
    const float g = expf(x);
    const double yd = exp((double)x);
    const float c = (float)yd;
    const uint32_t cb = float_to_bits(c);
    const double dc = (double)c;
    const double other = (double)bits_to_float(yd > dc ? cb + 1u : cb - 1u);
    const double dist = fabs(yd - 0.5 * (dc + other));
    const bool differs = float_to_bits(g) != cb;
    if (differs || dist <= yd * 0x1p-44) {
      keys.push_back(u);
      vals.push_back(g);
      if (differs && !(dist <= yd * 0x1p-30)) ok = false;
      if (differs) far = std::max(far, dist / yd);
    }
  }
}

const ExpfHostTable& expf_host_table() {
  static ExpfHostTable table;
  static std::once_flag once;
  std::call_once(once, [] {
    // (-104, 89): non-negative floats [0, 89) then negative floats (-0 .. -104)
    const uint32_t pos_end = float_to_bits(89.0f);
    const uint32_t neg_end = float_to_bits(-104.0f);
    constexpr uint32_t kChunk = 1u << 22;
    std::vector<std::pair<uint32_t, uint32_t>> chunks;
    for (uint32_t u = 0; u < pos_end; u += std::min(kChunk, pos_end - u))
      chunks.push_back({u, std::min(u + kChunk, pos_end)});
    for (uint32_t u = 0x80000000u; u < neg_end; u += std::min(kChunk, neg_end - u))
      chunks.push_back({u, std::min(u + kChunk, neg_end)});
    std::vector<std::vector<uint32_t>> ck(chunks.size());
    std::vector<std::vector<float>> cv(chunks.size());
    std::vector<char> cok(chunks.size(), 1);
    std::vector<double> cfar(chunks.size(), 0.0);
    std::atomic<size_t> next{0};
    unsigned nt = std::max(1u, std::thread::hardware_concurrency());
    std::vector<std::thread> pool;
    for (unsigned t = 0; t < nt; ++t)
      pool.emplace_back([&] {
        for (size_t i = next++; i < chunks.size(); i = next++) {
          bool ok = true;
          scan_expf_range(chunks[i].first, chunks[i].second, ck[i], cv[i], ok, cfar[i]);
          cok[i] = ok;
        }
      });
    for (auto& th : pool) th.join();
    for (size_t i = 0; i < chunks.size(); ++i) {
      table.keys.insert(table.keys.end(), ck[i].begin(), ck[i].end());
      table.vals.insert(table.vals.end(), cv[i].begin(), cv[i].end());
      if (!cok[i]) table.model_ok = false;
    }
    // the lookup band: the smallest power of two >= twice the farthest
    // difference (the device's double exp may sit an ulp of a double away from
    // the host's), between 2^-44 (the band the table holds in full) and 2^-30
    const double far = *std::max_element(cfar.begin(), cfar.end());
    table.near = 0x1p-44;
    while (table.near < 2.0 * far && table.near < 0x1p-30) table.near *= 2.0;
    table.bucket.resize((size_t)kExpfBuckets + 1);
    size_t k = 0;
    for (uint64_t b = 0; b <= kExpfBuckets; ++b) {
      const uint64_t lo = b << kExpfBucketShift;
      while (k < table.keys.size() && table.keys[k] < lo) ++k;
      table.bucket[b] = (uint32_t)k;
    }
  });
  return table;
}

}  // namespace

// Builds (once per process) and returns the table on the host.
bool expf_table_host(const uint32_t** keys, const float** vals, int* n) {
  const ExpfHostTable& t = expf_host_table();
  *keys = t.keys.data();
  *vals = t.vals.data();
  *n = (int)t.keys.size();
  return t.model_ok;
}

bool expf_bucket_host(const uint32_t** bucket) {
  *bucket = expf_host_table().bucket.data();
  return expf_host_table().model_ok;
}

double expf_near_host() { return expf_host_table().near; }

bool install_expf_table(cudaError_t* err) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static void* dev_mem[kMaxDevices] = {};
  *err = cudaSuccess;
  const uint32_t* keys;
  const float* vals;
  const uint32_t* bucket;
  int n;
  if (!expf_table_host(&keys, &vals, &n) || !expf_bucket_host(&bucket)) return false;
  int device = 0;
  if ((*err = cudaGetDevice(&device)) != cudaSuccess) return true;
  if (device < 0 || device >= kMaxDevices) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (dev_mem[device]) return true;  // installed for the process's lifetime
  const size_t kb = sizeof(uint32_t) * (size_t)n, vb = sizeof(float) * (size_t)n;
  const size_t bb = sizeof(uint32_t) * ((size_t)kExpfBuckets + 1);
  void* mem = nullptr;
  if ((*err = cudaMalloc(&mem, kb + vb + bb)) != cudaSuccess) return true;
  const ExpfTable t{(const uint32_t*)mem, (const float*)((char*)mem + kb),
                    (const uint32_t*)((char*)mem + kb + vb), n, expf_near_host()};
  if ((*err = cudaMemcpy(mem, keys, kb, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (*err = cudaMemcpy((char*)mem + kb, vals, vb, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (*err = cudaMemcpy((char*)mem + kb + vb, bucket, bb, cudaMemcpyHostToDevice)) !=
          cudaSuccess ||
      (*err = cudaMemcpyToSymbol(c_expf, &t, sizeof(t))) != cudaSuccess) {
    cudaFree(mem);
    return true;
  }
  dev_mem[device] = mem;
  return true;
}

__global__ void ref_expf_kernel(const float* x, float* y, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = libm_expf(x[i]);
}

cudaError_t launch_ref_expf(const float* x, float* y, long long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const long long blocks = std::min<long long>((n + 255) / 256, 148 * 16);
  ref_expf_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, y, n);
  return cudaGetLastError();
}

}  // namespace wh
