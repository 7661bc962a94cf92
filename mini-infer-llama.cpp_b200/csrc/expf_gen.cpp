// mi_expf_gen: builds the expf exception table used by the device kernels.
//
//   mi_expf_gen <out.bin>
//
// Runs the host libm's expf and mi_expf_core over all 2^32 float inputs,
// collects every input where the two differ (about 171k of them with glibc
// 2.39 on x86-64), and stores them as a two-choice bucketed hash (4 slots per
// 32-byte bucket) whose buckets are sized for a low load so that insertion by
// eviction always succeeds. The header also records fingerprints of both
// functions over a fixed sample so the library can refuse a table made for a
// different libm.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "mi_expf_core.h"

namespace {

struct entry {
  uint32_t key, val;
};

void scan(uint32_t hi_begin, uint32_t hi_end, std::vector<entry>* out) {
  for (uint32_t hi = hi_begin; hi < hi_end; hi++) {
    for (uint32_t lo = 0; lo < 65536u; lo++) {
      uint32_t b = (hi << 16) | lo;
      float x = mi_u2f(b);
      if (x != x) continue;
      uint32_t want = mi_f2u(expf(x));
      uint32_t got = mi_f2u(mi_expf_core(x));
      if (want != got) out->push_back({b, want});
    }
  }
}

bool build_table(const std::vector<entry>& es, uint32_t log2b, uint32_t mul1, uint32_t mul2,
                 std::vector<uint32_t>* slots) {
  size_t nb = (size_t)1 << log2b;
  slots->assign(nb * MI_EXPF_SLOTS * 2, MI_EXPF_EMPTY);
  auto try_put = [&](uint32_t bucket, entry e) {
    uint32_t* s = slots->data() + (size_t)bucket * MI_EXPF_SLOTS * 2;
    for (int i = 0; i < MI_EXPF_SLOTS; i++)
      if (s[2 * i] == MI_EXPF_EMPTY) {
        s[2 * i] = e.key;
        s[2 * i + 1] = e.val;
        return true;
      }
    return false;
  };
  uint32_t rng = 12345u;
  for (const entry& e0 : es) {
    entry e = e0;
    bool placed = false;
    for (int kick = 0; kick < 500 && !placed; kick++) {
      uint32_t b1 = mi_expf_bucket(e.key, mul1, log2b), b2 = mi_expf_bucket(e.key, mul2, log2b);
      if (try_put(b1, e) || try_put(b2, e)) {
        placed = true;
        break;
      }
      rng = rng * 1664525u + 1013904223u;
      uint32_t b = (rng >> 16) & 1 ? b1 : b2;
      int victim = (int)((rng >> 8) % MI_EXPF_SLOTS);
      uint32_t* s = slots->data() + (size_t)b * MI_EXPF_SLOTS * 2 + 2 * victim;
      entry out{s[0], s[1]};
      s[0] = e.key;
      s[1] = e.val;
      e = out;
    }
    if (!placed) return false;
  }
  return true;
}

}  // namespace

// Fingerprints over inputs (i * 65521) mod 2^32, i < 2^20: a quick check that
// the libm and core functions at run time are the ones the table was made for.
extern "C" void mi_expf_fingerprints(uint32_t* core, uint32_t* libm) {
  uint32_t c = 0, l = 0;
  for (uint32_t i = 0; i < (1u << 20); i++) {
    float x = mi_u2f(i * 65521u);
    if (x != x) continue;
    c = c * 31u + mi_f2u(mi_expf_core(x));
    l = l * 31u + mi_f2u(expf(x));
  }
  *core = c;
  *libm = l;
}

int main(int argc, char** argv) {
  if (argc != 2) {
    std::fprintf(stderr, "usage: %s <out.bin>\n", argv[0]);
    return 2;
  }
  unsigned nt = std::max(1u, std::thread::hardware_concurrency());
  std::vector<std::vector<entry>> parts(nt);
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; t++) {
    uint32_t b = (uint32_t)((65536ull * t) / nt), e = (uint32_t)((65536ull * (t + 1)) / nt);
    th.emplace_back(scan, b, e, &parts[t]);
  }
  for (auto& t : th) t.join();
  std::vector<entry> all;
  for (auto& p : parts) all.insert(all.end(), p.begin(), p.end());
  std::sort(all.begin(), all.end(), [](const entry& a, const entry& b) { return a.key < b.key; });

  uint32_t log2b = 1;
  while (((size_t)1 << log2b) * MI_EXPF_SLOTS < all.size() * 3) log2b++;
  std::vector<uint32_t> slots;
  uint32_t mul1 = 0x9e3779b1u, mul2 = 0x85ebca77u;
  int attempt = 0;
  while (!build_table(all, log2b, mul1, mul2, &slots)) {
    if (++attempt > 64) {
      std::fprintf(stderr, "mi_expf_gen: could not place %zu entries\n", all.size());
      return 1;
    }
    mul1 = mul1 * 0x2545f491u + 2u;
    mul1 |= 1u;
    mul2 = mul2 * 0x6c8e9cf5u + 2u;
    mul2 |= 1u;
  }
  mi_expf_table_header h{};
  h.magic = MI_EXPF_MAGIC;
  h.log2_buckets = log2b;
  h.mul1 = mul1;
  h.mul2 = mul2;
  h.n_entries = (uint32_t)all.size();
  // The device may skip the table for results far from a rounding boundary
  // only if no exception lies far from one.
  size_t far = 0;
  for (const entry& e : all) {
    const float x = mi_u2f(e.key);
    if (!(x >= -110.0f && x <= 100.0f)) continue;  // these always probe
    if (!mi_expf_near_tie(mi_expf_core_wide(x), MI_EXPF_TIE_VERIFIED)) far++;
  }
  if (far == 0) h.flags |= MI_EXPF_FLAG_TIE_FILTER;
  mi_expf_fingerprints(&h.core_checksum, &h.libm_checksum);
  std::string tmp = std::string(argv[1]) + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) {
    std::perror("fopen");
    return 1;
  }
  bool ok = std::fwrite(&h, sizeof(h), 1, f) == 1 &&
            std::fwrite(slots.data(), 4, slots.size(), f) == slots.size();
  ok = (std::fclose(f) == 0) && ok;
  if (!ok || std::rename(tmp.c_str(), argv[1]) != 0) {
    std::fprintf(stderr, "mi_expf_gen: write failed\n");
    return 1;
  }
  std::printf("mi_expf_gen: %zu exceptions, 2^%u buckets, %zu far from a rounding boundary\n", all.size(), log2b,
              far);
  return 0;
}
