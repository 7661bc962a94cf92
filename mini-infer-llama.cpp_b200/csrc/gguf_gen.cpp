// mi_gguf_gen: fills the tensor data of a random-init Qwen2 GGUF whose header
// (metadata, tensor infos, alignment padding) has already been written by
// mi_gguf.write_qwen2_gguf_fast. Multithreaded; the bytes depend only on the
// seed, never on the thread count.
//
//   mi_gguf_gen <file> <plan> <seed> <std> <threads>
//
// <plan> holds one line per tensor: "<index> <type> <ne0> <ne1> <offset> <ones>"
// with type 0 (F32) or 8 (Q8_0), the tensor's absolute file offset, and ones=1
// for norm weights (all 1.0). Every other value is N(0, std): row r of tensor t
// draws from its own splitmix64 stream keyed by (seed, t, r), Box-Muller in
// double precision, rounded to float. Q8_0 blocks follow the GGUF quantizer
// (ref src/quant.cpp:173-197 restated): d = amax / 127, q = round-to-nearest-even
// of x / d clamped to +-127, d stored as IEEE half (round to nearest even).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <string>
#include <thread>
#include <unistd.h>
#include <vector>

namespace {

struct Tensor {
  int index = 0, type = 0, ones = 0;
  int64_t ne0 = 0, ne1 = 0, offset = 0;
};

uint64_t splitmix(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Row stream: the state is a hash of (seed, tensor, row).
struct Stream {
  uint64_t s;
  bool have = false;
  double spare = 0.0;
  Stream(uint64_t seed, int t, int64_t row) {
    uint64_t h = seed;
    s = splitmix(h) ^ ((uint64_t)(uint32_t)t << 40) ^ (uint64_t)row;
    (void)splitmix(s);
  }
  double normal() {
    if (have) {
      have = false;
      return spare;
    }
    const double u1 = ((double)(splitmix(s) >> 11) + 1.0) * (1.0 / 9007199254740992.0);  // (0, 1]
    const double u2 = (double)(splitmix(s) >> 11) * (1.0 / 9007199254740992.0);          // [0, 1)
    const double r = std::sqrt(-2.0 * std::log(u1));
    const double a = 6.283185307179586 * u2;
    spare = r * std::sin(a);
    have = true;
    return r * std::cos(a);
  }
};

// float -> IEEE binary16, round to nearest even (finite inputs below 65520).
uint16_t to_half(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t mag = x & 0x7fffffffu;
  if (mag >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // overflow -> inf
  if (mag < 0x38800000u) {                                     // subnormal half
    // value = mag_float; half subnormal unit = 2^-24
    float a;
    std::memcpy(&a, &mag, 4);
    const float scaled = a * 16777216.0f;  // exact: power-of-two scale
    const uint32_t q = (uint32_t)std::nearbyint(scaled);
    return (uint16_t)(sign | q);
  }
  const uint32_t e = (mag >> 23) - 112u;  // rebias 127 -> 15
  uint32_t m = mag & 0x7fffffu;
  uint32_t h = (e << 10) | (m >> 13);
  const uint32_t rest = m & 0x1fffu;
  if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

void fill_rows(const Tensor& t, uint64_t seed, float stdv, int64_t r0, int64_t r1, int fd,
               std::string* err) {
  const int64_t K = t.ne0;
  std::vector<uint8_t> buf;
  std::vector<float> x((size_t)K);
  const size_t row_bytes = t.type == 0 ? (size_t)K * 4 : (size_t)(K / 32) * 34;
  const int64_t chunk = std::max<int64_t>(1, (int64_t)((4u << 20) / row_bytes));
  for (int64_t c0 = r0; c0 < r1; c0 += chunk) {
    const int64_t c1 = std::min(r1, c0 + chunk);
    buf.resize((size_t)(c1 - c0) * row_bytes);
    for (int64_t r = c0; r < c1; r++) {
      uint8_t* out = buf.data() + (size_t)(r - c0) * row_bytes;
      if (t.ones) {
        for (int64_t k = 0; k < K; k++) x[(size_t)k] = 1.0f;
      } else {
        Stream st(seed, t.index, r);
        for (int64_t k = 0; k < K; k++) x[(size_t)k] = (float)(st.normal() * (double)stdv);
      }
      if (t.type == 0) {
        std::memcpy(out, x.data(), (size_t)K * 4);
        continue;
      }
      for (int64_t b = 0; b < K / 32; b++) {
        const float* v = x.data() + b * 32;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = std::max(amax, std::fabs(v[i]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = to_half(d);
        uint8_t* blk = out + b * 34;
        std::memcpy(blk, &dh, 2);
        for (int i = 0; i < 32; i++) {
          float q = std::nearbyint(v[i] * id);
          q = q > 127.0f ? 127.0f : (q < -127.0f ? -127.0f : q);
          blk[2 + i] = (uint8_t)(int8_t)q;
        }
      }
    }
    const off_t off = (off_t)(t.offset + (int64_t)((size_t)(c0 - 0) * row_bytes));
    size_t done = 0;
    while (done < buf.size()) {
      const ssize_t w = pwrite(fd, buf.data() + done, buf.size() - done, off + (off_t)done);
      if (w <= 0) {
        *err = "write failed";
        return;
      }
      done += (size_t)w;
    }
  }
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 6) {
    std::fprintf(stderr, "usage: %s <file> <plan> <seed> <std> <threads>\n", argv[0]);
    return 2;
  }
  const uint64_t seed = std::strtoull(argv[3], nullptr, 10);
  const float stdv = std::strtof(argv[4], nullptr);
  const int n_threads = std::max(1, std::atoi(argv[5]));
  std::vector<Tensor> plan;
  FILE* pf = std::fopen(argv[2], "r");
  if (!pf) {
    std::perror("plan");
    return 1;
  }
  Tensor t;
  long long ne0, ne1, off;
  while (std::fscanf(pf, "%d %d %lld %lld %lld %d", &t.index, &t.type, &ne0, &ne1, &off, &t.ones) == 6) {
    t.ne0 = ne0;
    t.ne1 = ne1;
    t.offset = off;
    if ((t.type != 0 && t.type != 8) || (t.type == 8 && ne0 % 32)) {
      std::fprintf(stderr, "bad plan line for tensor %d\n", t.index);
      return 1;
    }
    plan.push_back(t);
  }
  std::fclose(pf);
  const int fd = open(argv[1], O_WRONLY);
  if (fd < 0) {
    std::perror("open");
    return 1;
  }
  // Work items: (tensor, row range) of about 16 MB each, handed out round-robin.
  struct Item {
    size_t t;
    int64_t r0, r1;
  };
  std::vector<Item> items;
  for (size_t i = 0; i < plan.size(); i++) {
    const Tensor& x = plan[i];
    const size_t row_bytes = x.type == 0 ? (size_t)x.ne0 * 4 : (size_t)(x.ne0 / 32) * 34;
    const int64_t step = std::max<int64_t>(1, (int64_t)((16u << 20) / row_bytes));
    for (int64_t r = 0; r < x.ne1; r += step) items.push_back({i, r, std::min(x.ne1, r + step)});
  }
  std::vector<std::string> errs((size_t)n_threads);
  std::vector<std::thread> th;
  for (int w = 0; w < n_threads; w++)
    th.emplace_back([&, w]() {
      for (size_t k = (size_t)w; k < items.size(); k += (size_t)n_threads) {
        fill_rows(plan[items[k].t], seed, stdv, items[k].r0, items[k].r1, fd, &errs[(size_t)w]);
        if (!errs[(size_t)w].empty()) return;
      }
    });
  for (auto& x : th) x.join();
  close(fd);
  for (auto& e : errs)
    if (!e.empty()) {
      std::fprintf(stderr, "%s\n", e.c_str());
      return 1;
    }
  return 0;
}
