// Checks FastDiv (dcnv2_b200/csrc/dcn_plan.h) against integer division: the
// multiply-high formula the kernels use, for every divisor the index
// arithmetic can see in a test-sized range and for large ones, at the ends of
// the numerator range and on random numerators below 2^31.
#include <cstdint>
#include <cstdio>
#include <random>

#include "dcn_plan.h"

static uint32_t umulhi(uint32_t a, uint32_t b) { return (uint32_t)(((uint64_t)a * b) >> 32); }
static uint32_t fdiv(uint32_t n, const dcn::FastDiv& f) { return f.d == 1 ? n : umulhi(n, f.m) >> f.sh; }

int main() {
  std::mt19937_64 rng(7);
  long bad = 0, n = 0;
  auto check = [&](uint32_t d, uint32_t x) {
    const dcn::FastDiv f = dcn::make_fastdiv(d);
    if (fdiv(x, f) != x / d) {
      if (bad < 5) std::printf("mismatch d=%u n=%u\n", d, x);
      ++bad;
    }
    ++n;
  };
  for (uint32_t d = 1; d <= 4096; ++d) {
    for (uint32_t k = 0; k < 64; ++k) check(d, k * d + (k % d)), check(d, k * d + d - 1);
    check(d, 0x7fffffffu);
    for (int k = 0; k < 64; ++k) check(d, (uint32_t)(rng() & 0x7fffffffu));
  }
  const uint32_t big[] = {16383u, 16384u, 65535u, 1000003u, 1u << 20, (1u << 30) + 1, 0x7fffffffu};
  for (uint32_t d : big)
    for (int k = 0; k < 200000; ++k) check(d, (uint32_t)(rng() & 0x7fffffffu));
  std::printf("checked %ld bad %ld\n", n, bad);
  return bad == 0 ? 0 : 1;
}
