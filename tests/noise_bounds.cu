// Exhaustive check of the FP32 Gumbel noise used by the row kernel's
// certified draws, over all 2^32 Philox words:
//
//   |noise32(w) - G(w)| <= NOISE_ERR * (1 + |G(w)|)   (the bound the draws assume)
//   noise_upper(w) >= G(w)                           (the pruning screen is an upper bound)
//   G(w) <= NOISE_MAX                                (the noise ceiling of the first screen)
//
// G(w) = -log(-log u), u = (w + 0.5) / 2^32, in FP64 with log1p above u = 1/2.
// Built with the library's flags (--fmad=false) by tests/noise_bounds.py;
// prints one JSON line and exits 0 iff every check holds.
#include <cstdio>
#include <vector>

#include "../exactsample_b200/csrc/es_device.cuh"

namespace {
constexpr int BLOCKS = 148 * 16, THREADS = 256;

struct Stats {
  double worst_ratio, min_margin, max_g, min_g;
  unsigned long long violations, screen_violations;
  unsigned worst_word;
};

__device__ double reference_noise(uint32_t w) {
  const double e = w < 0x80000000u ? -log((double(w) + 0.5) * 0x1p-32) : -log1p(-(double(~w) + 0.5) * 0x1p-32);
  return -log(e);
}

__global__ void check(Stats* out) {
  Stats s{0., 1e300, -1e300, 1e300, 0, 0, 0};
  const uint64_t stride = uint64_t(BLOCKS) * THREADS;
  for (uint64_t i = uint64_t(blockIdx.x) * THREADS + threadIdx.x; i < (1ull << 32); i += stride) {
    const uint32_t w = uint32_t(i);
    const double g = reference_noise(w);
    const double ratio = fabs(double(es::noise32(w)) - g) / (double(es::NOISE_ERR) * (1. + fabs(g)));
    if (ratio > s.worst_ratio) { s.worst_ratio = ratio; s.worst_word = w; }
    s.violations += ratio > 1.;
    const double margin = double(es::noise_upper(w)) - g;
    s.min_margin = fmin(s.min_margin, margin);
    s.screen_violations += margin < 0.;
    s.max_g = fmax(s.max_g, g);
    s.min_g = fmin(s.min_g, g);
  }
  out[blockIdx.x * THREADS + threadIdx.x] = s;
}
}  // namespace

int main() {
  const int n = BLOCKS * THREADS;
  Stats* device = nullptr;
  if (cudaMalloc(&device, n * sizeof(Stats)) != cudaSuccess) return 2;
  check<<<BLOCKS, THREADS>>>(device);
  if (cudaDeviceSynchronize() != cudaSuccess) return 2;
  std::vector<Stats> host(n);
  if (cudaMemcpy(host.data(), device, n * sizeof(Stats), cudaMemcpyDeviceToHost) != cudaSuccess) return 2;
  cudaFree(device);
  Stats t = host[0];
  t.violations = t.screen_violations = 0;
  for (const Stats& s : host) {
    if (s.worst_ratio > t.worst_ratio) { t.worst_ratio = s.worst_ratio; t.worst_word = s.worst_word; }
    t.min_margin = s.min_margin < t.min_margin ? s.min_margin : t.min_margin;
    t.max_g = s.max_g > t.max_g ? s.max_g : t.max_g;
    t.min_g = s.min_g < t.min_g ? s.min_g : t.min_g;
    t.violations += s.violations;
    t.screen_violations += s.screen_violations;
  }
  const bool pass = t.violations == 0 && t.screen_violations == 0 && t.max_g <= double(es::NOISE_MAX);
  std::printf("{\"words\": 4294967296, \"noise_err\": %.3g, \"worst_error_over_bound\": %.6f, \"worst_word\": %u, "
              "\"error_violations\": %llu, \"screen_min_margin\": %.9g, \"screen_violations\": %llu, "
              "\"max_noise\": %.9f, \"min_noise\": %.9f, \"noise_max\": %.6f, \"passed\": %s}\n",
              double(es::NOISE_ERR), t.worst_ratio, t.worst_word, t.violations, t.min_margin, t.screen_violations,
              t.max_g, t.min_g, double(es::NOISE_MAX), pass ? "true" : "false");
  return pass ? 0 : 1;
}
