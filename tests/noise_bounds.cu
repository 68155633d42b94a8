// Exhaustive check, on the GPU, of the three facts about the FP32 Gumbel
// noise that the row kernel's certified draws rest on. For every 32-bit
// Philox word w, with G(w) = -log(-log u), u = (w + 0.5) / 2^32, computed in
// FP64 (log1p of the exact complement for u >= 1/2):
//
//   (1) |noise32(w) - G(w)| <= NOISE_ERR * (1 + |G(w)|)
//   (2) noise_upper(w) >= G(w)
//   (3) G(w) <= NOISE_MAX
//
// Layout: the 2^32 words are cut into 2^16 pages of 2^16 words; blocks take
// pages in turn. Each thread keeps its findings in registers, each block
// folds them in shared memory, and one thread per block folds the block's
// summary into a single device record with atomics. The report is a
// histogram of the error as a fraction of its bound (eighths, last bucket
// above the bound), the worst word, the smallest screen margin and the
// noise range. Built with the library's flags (--fmad=false) by
// tests/noise_bounds.py; prints one JSON line, exit status 0 iff all three
// hold for every word.
#include <cstdio>
#include <cstring>

#include "../exactsample_b200/csrc/es_device.cuh"

namespace {

constexpr int PAGE_BITS = 16;
constexpr unsigned PAGES = 1u << (32 - PAGE_BITS);
constexpr int BLOCK = 512;
constexpr int BUCKETS = 9;  // error / bound in [k/8, (k+1)/8) for k < 8; bucket 8: above the bound

// Order-preserving 64-bit keys of doubles, so that atomicMax / atomicMin on
// integers track a maximum or minimum double.
__device__ unsigned long long up_key(double x) {
  const unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(x));
  return (b >> 63) ? ~b : (b | (1ull << 63));
}
double from_key(unsigned long long k) {
  const unsigned long long b = (k >> 63) ? (k & ~(1ull << 63)) : ~k;
  double x;
  std::memcpy(&x, &b, sizeof x);
  return x;
}

struct Record {
  unsigned long long bucket[BUCKETS];
  unsigned long long worst;       // (float bits of error/bound) << 32 | word: the largest ratio
  unsigned long long min_margin;  // up_key of the smallest noise_upper - G
  unsigned long long screen_failures;
  unsigned long long max_noise, min_noise;  // up_key of the noise range
};

__device__ double exact_noise(uint32_t w) {
  const double minus_log_u = w < 0x80000000u ? -log((double(w) + 0.5) * 0x1p-32)
                                             : -log1p(-(double(~w) + 0.5) * 0x1p-32);
  return -log(minus_log_u);
}

__global__ void __launch_bounds__(BLOCK) sweep(Record* out) {
  __shared__ unsigned long long s_bucket[BUCKETS];
  __shared__ unsigned long long s_worst, s_margin, s_screen, s_max, s_min;
  if (threadIdx.x < BUCKETS) s_bucket[threadIdx.x] = 0;
  if (threadIdx.x == 0) {
    s_worst = 0;
    s_margin = ~0ull;
    s_screen = 0;
    s_max = 0;
    s_min = ~0ull;
  }
  __syncthreads();
  unsigned long long bucket[BUCKETS] = {};
  unsigned long long worst = 0, margin = ~0ull, screen = 0, gmax = 0, gmin = ~0ull;
  for (unsigned page = blockIdx.x; page < PAGES; page += gridDim.x) {
    for (unsigned k = threadIdx.x; k < (1u << PAGE_BITS); k += BLOCK) {
      const uint32_t w = (page << PAGE_BITS) | k;
      const double g = exact_noise(w);
      const double ratio = fabs(double(es::noise32(w)) - g) / (double(es::NOISE_ERR) * (1.0 + fabs(g)));
      ++bucket[ratio > 1.0 ? BUCKETS - 1 : min(int(ratio * 8.0), BUCKETS - 2)];
      const unsigned long long tagged =
          (static_cast<unsigned long long>(__float_as_uint(float(ratio))) << 32) | w;
      worst = tagged > worst ? tagged : worst;
      const double gap = double(es::noise_upper(w)) - g;
      screen += gap < 0.0;
      const unsigned long long gk = up_key(gap), nk = up_key(g);
      margin = gk < margin ? gk : margin;
      gmax = nk > gmax ? nk : gmax;
      gmin = nk < gmin ? nk : gmin;
    }
  }
  for (int b = 0; b < BUCKETS; ++b)
    if (bucket[b]) atomicAdd(&s_bucket[b], bucket[b]);
  atomicMax(&s_worst, worst);
  atomicMin(&s_margin, margin);
  if (screen) atomicAdd(&s_screen, screen);
  atomicMax(&s_max, gmax);
  atomicMin(&s_min, gmin);
  __syncthreads();
  if (threadIdx.x < BUCKETS) atomicAdd(&out->bucket[threadIdx.x], s_bucket[threadIdx.x]);
  if (threadIdx.x == 0) {
    atomicMax(&out->worst, s_worst);
    atomicMin(&out->min_margin, s_margin);
    atomicAdd(&out->screen_failures, s_screen);
    atomicMax(&out->max_noise, s_max);
    atomicMin(&out->min_noise, s_min);
  }
}

}  // namespace

int main() {
  Record init{};
  init.min_margin = ~0ull;
  init.min_noise = ~0ull;
  Record* dev = nullptr;
  if (cudaMalloc(&dev, sizeof(Record)) != cudaSuccess) return 2;
  if (cudaMemcpy(dev, &init, sizeof init, cudaMemcpyHostToDevice) != cudaSuccess) return 2;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  sweep<<<4 * (sms > 0 ? sms : 148), BLOCK>>>(dev);
  Record r{};
  if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&r, dev, sizeof r, cudaMemcpyDeviceToHost) != cudaSuccess)
    return 2;
  cudaFree(dev);
  unsigned long long words = 0;
  for (unsigned long long b : r.bucket) words += b;
  const unsigned worst_bits = unsigned(r.worst >> 32);
  float worst_ratio;
  std::memcpy(&worst_ratio, &worst_bits, sizeof worst_ratio);
  const double max_noise = from_key(r.max_noise), min_noise = from_key(r.min_noise);
  const bool pass = words == (1ull << 32) && r.bucket[BUCKETS - 1] == 0 && r.screen_failures == 0 &&
                    max_noise <= double(es::NOISE_MAX);
  std::printf("{\"words\": %llu, \"noise_err\": %.3g, \"error_over_bound_eighths\": [", words, double(es::NOISE_ERR));
  for (int b = 0; b < BUCKETS; ++b) std::printf("%s%llu", b ? ", " : "", r.bucket[b]);
  std::printf("], \"error_violations\": %llu, \"worst_error_over_bound\": %.6f, \"worst_word\": %u, "
              "\"screen_violations\": %llu, \"screen_min_margin\": %.9g, \"max_noise\": %.9f, \"min_noise\": %.9f, "
              "\"noise_max\": %.6f, \"passed\": %s}\n",
              r.bucket[BUCKETS - 1], double(worst_ratio), unsigned(r.worst & 0xffffffffu), r.screen_failures,
              from_key(r.min_margin), max_noise, min_noise, double(es::NOISE_MAX), pass ? "true" : "false");
  return pass ? 0 : 1;
}
