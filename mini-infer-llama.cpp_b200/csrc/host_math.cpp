// Host-side math tables of the backend, evaluated with the host libm so the
// device reproduces the reference's libm calls bit for bit. Compiled with
// -ffp-contract=off.
#include <cmath>
#include <cstdint>
#include <thread>
#include <vector>

#include "mi_expf_core.h"
#include "mi_internal.h"

namespace mi {

// RoPE (cos, sin) per (position, pair), exactly as mi_compute_rope evaluates
// them (reference src/ops_cpu.cpp:286-292): freq = powf(base, -(float)(2p) /
// (float)n_dims); theta = (float)pos * freq; cosf / sinf of theta.
void build_rope_table(int32_t pos0, int32_t n_pos, int32_t n_dims, float freq_base, float* cs) {
  const int32_t half = n_dims / 2;
  std::vector<float> freq((size_t)half);
  for (int32_t p = 0; p < half; p++) {
    const float e = -(float)(2 * p) / (float)n_dims;
    freq[(size_t)p] = powf(freq_base, e);
  }
  for (int32_t t = 0; t < n_pos; t++) {
    const int64_t pos = (int64_t)pos0 + t;
    for (int32_t p = 0; p < half; p++) {
      const float theta = (float)pos * freq[(size_t)p];
      cs[((size_t)t * half + p) * 2] = cosf(theta);
      cs[((size_t)t * half + p) * 2 + 1] = sinf(theta);
    }
  }
}

void expf_fingerprints(uint32_t* core, uint32_t* libm) {
  uint32_t c = 0, l = 0;
  for (uint32_t i = 0; i < (1u << 20); i++) {
    const float x = mi_u2f(i * 65521u);
    if (x != x) continue;
    c = c * 31u + mi_f2u(mi_expf_core(x));
    l = l * 31u + mi_f2u(expf(x));
  }
  *core = c;
  *libm = l;
}

uint64_t expf_count_mismatch(uint64_t first, int64_t n, const float* y) {
  const unsigned nt = std::max(1u, std::thread::hardware_concurrency());
  std::vector<uint64_t> counts(nt, 0);
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; t++) {
    th.emplace_back([&, t]() {
      const int64_t b = n * (int64_t)t / (int64_t)nt, e = n * (int64_t)(t + 1) / (int64_t)nt;
      uint64_t c = 0;
      for (int64_t i = b; i < e; i++) {
        const float x = mi_u2f((uint32_t)(first + (uint64_t)i));
        const uint32_t want = mi_f2u(expf(x)), got = mi_f2u(y[i]);
        if (x != x) {
          if ((got & 0x7f800000u) != 0x7f800000u || (got & 0x7fffffu) == 0) c++;
        } else if (want != got) {
          c++;
        }
      }
      counts[t] = c;
    });
  }
  for (auto& t : th) t.join();
  uint64_t total = 0;
  for (uint64_t c : counts) total += c;
  return total;
}

}  // namespace mi
