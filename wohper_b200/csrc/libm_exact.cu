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
// The table is measured, not derived: at first use the library calls the
// running process's expf on every float in (-104, 89) (all host threads) and
// records each x whose expf differs from the once-rounded double exp, plus
// every x whose exp lies within 2^-44 of a midpoint (there a one-ulp
// difference between the host's and the device's double exp could flip the
// rounding).  On the device, ref_expf rounds exp((double)x) once and looks x up
// in the sorted table only when the result is within 2^-30 of a midpoint,
// about 0.6 % of inputs.  Outside (-104, 89) both sides saturate to 0 or inf.
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
  bool model_ok = true;        // every difference lies inside the device gate
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
                     std::vector<float>& vals, bool& ok) {
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
    std::atomic<size_t> next{0};
    unsigned nt = std::max(1u, std::thread::hardware_concurrency());
    std::vector<std::thread> pool;
    for (unsigned t = 0; t < nt; ++t)
      pool.emplace_back([&] {
        for (size_t i = next++; i < chunks.size(); i = next++) {
          bool ok = true;
          scan_expf_range(chunks[i].first, chunks[i].second, ck[i], cv[i], ok);
          cok[i] = ok;
        }
      });
    for (auto& th : pool) th.join();
    for (size_t i = 0; i < chunks.size(); ++i) {
      table.keys.insert(table.keys.end(), ck[i].begin(), ck[i].end());
      table.vals.insert(table.vals.end(), cv[i].begin(), cv[i].end());
      if (!cok[i]) table.model_ok = false;
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

__global__ void ref_expf_kernel(const float* x, float* y, long long n, ExpfTable t) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = ref_expf(x[i], t);
}

cudaError_t launch_ref_expf(const float* x, float* y, long long n, ExpfTable t, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const long long blocks = std::min<long long>((n + 255) / 256, 148 * 16);
  ref_expf_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, y, n, t);
  return cudaGetLastError();
}

}  // namespace wh
