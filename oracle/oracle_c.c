/*
 * TEST INFRASTRUCTURE ONLY - the CPU oracle's native helpers.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library. The product (exactsample_b200) never links it.
 *
 * These are plain-C restatements of the Python-level loops of the reference's
 * FP64 NumPy oracle, so that it runs at full-vocabulary sizes in seconds:
 *
 *   es_oracle_philox        python/exactsample/rng.py:22-43 (Random123 Philox4x32-10)
 *   es_oracle_word          python/exactsample/rng.py:46-56 (counter layout of docs/rng.md)
 *   es_oracle_sample        python/exactsample/reference.py:94-104 (Gumbel argmax,
 *                           strict '>' so the lowest token ID wins a tie)
 *   es_oracle_fsum          math.fsum, the correctly rounded sum used at
 *                           reference.py:73 and :84
 *   es_oracle_top_p_count   reference.py:74-83 (shortest prefix whose fsum
 *                           reaches the target), in O(n) instead of O(n^2)
 *
 * Arithmetic is IEEE binary64 with no contraction (built with
 * -ffp-contract=off); log() is the C library's, which is what CPython's
 * math.log calls, so the results are bit-identical to the Python oracle.
 */
#include <math.h>
#include <stdint.h>

static const uint32_t PHILOX_M0 = 0xD2511F53u, PHILOX_M1 = 0xCD9E8D57u;
static const uint32_t PHILOX_W0 = 0x9E3779B9u, PHILOX_W1 = 0xBB67AE85u;

void es_oracle_philox(const uint32_t counter[4], const uint32_t key[2], uint32_t out[4]) {
  uint32_t c0 = counter[0], c1 = counter[1], c2 = counter[2], c3 = counter[3];
  uint32_t k0 = key[0], k1 = key[1];
  for (int round = 0; round < 10; ++round) {
    const uint64_t p0 = (uint64_t)c0 * PHILOX_M0;
    const uint64_t p1 = (uint64_t)c2 * PHILOX_M1;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
    const uint32_t n1 = (uint32_t)p1;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    const uint32_t n3 = (uint32_t)p0;
    c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    k0 += PHILOX_W0;
    k1 += PHILOX_W1;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* The 32-bit word for (seed, stream, position, substream, token): counter
 * (stream, position, substream, token / 4), key (seed low, seed high), lane
 * token % 4. */
uint32_t es_oracle_word(uint64_t seed, uint32_t stream, uint32_t position, uint32_t substream,
                        uint64_t token) {
  const uint32_t counter[4] = {stream, position, substream, (uint32_t)(token / 4)};
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint32_t out[4];
  es_oracle_philox(counter, key, out);
  return out[token % 4];
}

/* Words for tokens [0, n) at one address, four per Philox call. */
void es_oracle_words(uint64_t seed, uint32_t stream, uint32_t position, uint32_t substream,
                     int64_t n, uint32_t* out) {
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  for (int64_t g = 0; 4 * g < n; ++g) {
    const uint32_t counter[4] = {stream, position, substream, (uint32_t)g};
    uint32_t w[4];
    es_oracle_philox(counter, key, w);
    for (int j = 0; j < 4 && 4 * g + j < n; ++j) out[4 * g + j] = w[j];
  }
}

static double uniform_of(uint32_t word) { return ((double)word + 0.5) / 4294967296.0; }

/* argmax over tokens with probs[t] > 0 of log(probs[t]) - log(-log(u_t)), the
 * first (lowest ID) maximum winning; -1 if no token has positive mass. */
int64_t es_oracle_sample(const double* probs, int64_t n, uint64_t seed, uint32_t stream,
                         uint32_t position, uint32_t substream) {
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  int64_t best_token = -1;
  double best_value = -INFINITY;
  for (int64_t g = 0; 4 * g < n; ++g) {
    int any = 0;
    for (int j = 0; j < 4 && 4 * g + j < n; ++j) any |= probs[4 * g + j] > 0;
    if (!any) continue;
    const uint32_t counter[4] = {stream, position, substream, (uint32_t)g};
    uint32_t w[4];
    es_oracle_philox(counter, key, w);
    for (int j = 0; j < 4 && 4 * g + j < n; ++j) {
      const double p = probs[4 * g + j];
      if (!(p > 0)) continue;
      const double gumbel = -log(-log(uniform_of(w[j])));
      const double score = log(p) + gumbel;
      if (score > best_value) { best_value = score; best_token = 4 * g + j; }
    }
  }
  return best_token;
}

/* Exact summation (Shewchuk's non-overlapping partials) with the final
 * correctly rounded, half-even result, as published for msum / math.fsum.
 * Inputs here are finite and nonnegative, so no special values arise. */
typedef struct { double p[64]; int m; } Partials;

static void partials_add(Partials* s, double x) {
  int i = 0;
  for (int j = 0; j < s->m; ++j) {
    double y = s->p[j];
    if (fabs(x) < fabs(y)) { const double t = x; x = y; y = t; }
    const double hi = x + y;
    const double lo = y - (hi - x);
    if (lo != 0.0) s->p[i++] = lo;
    x = hi;
  }
  s->p[i++] = x;
  s->m = i;
}

static double partials_round(const Partials* s) {
  int n = s->m;
  if (n == 0) return 0.0;
  double hi = s->p[--n], lo = 0.0;
  while (n > 0) {
    const double x = hi, y = s->p[--n];
    hi = x + y;
    lo = y - (hi - x);
    if (lo != 0.0) break;
  }
  /* Half-way case: the rest of the partials decide the direction. */
  if (n > 0 && ((lo < 0.0 && s->p[n - 1] < 0.0) || (lo > 0.0 && s->p[n - 1] > 0.0))) {
    const double y = lo * 2.0, x = hi + y;
    if (y == x - hi) hi = x;
  }
  return hi;
}

double es_oracle_fsum(const double* x, int64_t n) {
  Partials s = {{0}, 0};
  for (int64_t i = 0; i < n; ++i) partials_add(&s, x[i]);
  return partials_round(&s);
}

/* The count of the shortest prefix of w whose correctly rounded sum is at
 * least target; n if none is. */
int64_t es_oracle_top_p_count(const double* w, int64_t n, double target) {
  Partials s = {{0}, 0};
  for (int64_t i = 0; i < n; ++i) {
    partials_add(&s, w[i]);
    if (partials_round(&s) >= target) return i + 1;
  }
  return n;
}
