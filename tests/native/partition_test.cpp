// Host check of the stream-K work partition shared by host and device code
// (harp-q_b200/csrc/hqb_schedule.h): CTA ranges [unit_start(i), unit_start(i+1)) tile
// the units exactly and in order, and unit_owner() inverts unit_start() for every unit
// probed, on random unit and CTA counts.
#include <cstdint>
#include <cstdio>
#include <random>

#include "hqb_schedule.h"

int main() {
  std::mt19937_64 rng(12345);
  int checked = 0;
  for (int trial = 0; trial < 20000; ++trial) {
    const uint64_t total = 1 + rng() % 2000000;
    uint64_t ctas = 1 + rng() % 1200;
    if (ctas > total) ctas = total;
    if (hqb::unit_start(0, total, ctas) != 0 || hqb::unit_start(ctas, total, ctas) != total) {
      std::printf("FAIL bounds total=%llu ctas=%llu\n", (unsigned long long)total, (unsigned long long)ctas);
      return 1;
    }
    for (uint64_t i = 0; i < ctas; ++i) {
      if (hqb::unit_start(i + 1, total, ctas) <= hqb::unit_start(i, total, ctas)) {
        std::printf("FAIL empty or unordered range total=%llu ctas=%llu i=%llu\n", (unsigned long long)total,
                    (unsigned long long)ctas, (unsigned long long)i);
        return 1;
      }
    }
    for (int k = 0; k < 64; ++k) {
      const uint64_t u = k == 0 ? 0 : (k == 1 ? total - 1 : rng() % total);
      const uint32_t o = hqb::unit_owner(u, total, ctas);
      if (!(o < ctas && hqb::unit_start(o, total, ctas) <= u && u < hqb::unit_start(o + 1, total, ctas))) {
        std::printf("FAIL owner total=%llu ctas=%llu u=%llu o=%u\n", (unsigned long long)total,
                    (unsigned long long)ctas, (unsigned long long)u, o);
        return 1;
      }
      ++checked;
    }
  }
  std::printf("partition ok (%d units checked)\n", checked);
  return 0;
}
