/*
 * division_check.c -- CPU checks of the two division routines the CUDA
 * kernels use in place of IEEE division (gdn-state-codec_b200/csrc/
 * codec_device.cuh), restated here with the same operation order and
 * compared bit for bit with IEEE single-precision division.  Built and run
 * by tests/test_division.py; test infrastructure only.
 *
 *   div127 <threads>
 *       a / 127 as fma(a, zh, RN(a * zl)) with zh = RN(1/127) and
 *       zl = RN(1/127 - zh) (Brisebarre, Muller and Raina, "Accelerating
 *       correctly rounded floating-point division when the divisor is known
 *       in advance", IEEE TC 53(8), 2004).  Checked for EVERY finite float
 *       with |a| >= 2^-112 (both signs), zero, the infinities and NaN.
 *
 *   markstein <threads> <samples per thread>
 *       a / c from y = RN(1/c): q0 = RN(a*y), then twice r = fma(-q, c, a),
 *       q = fma(r, y, q) (Markstein, "Computation of elementary functions on
 *       the IBM RISC System/6000 processor", IBM J. R&D 34(1), 1990).
 *       Checked on random operands over the kernels' fast-path ranges
 *       (c in [2^-14, 2^100], |a| >= 2^-102, normal quotient) and on
 *       operands built so that a / c lies within a few ulps of a rounding
 *       midpoint -- the hard cases of correctly rounded division.
 *
 * Prints one line "<mode> checked=<n> mismatches=<m>" and exits 0 when m is 0.
 * Compiled with -ffp-contract=off so that every operation rounds as written;
 * fmaf comes from libm (correctly rounded, hardware FMA where available).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float from_bits(uint32_t u) {
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}
static uint32_t to_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  return u;
}
static int same(float a, float b) {
  if (isnan(a) && isnan(b)) return 1;
  return to_bits(a) == to_bits(b);
}

/* ---- divide by 127 -------------------------------------------------------- */

static const float kZh = 0x1.020408p-7F;
static const float kZl = 0x1.020408p-35F;

static float div127(float a) { return fmaf(a, kZh, a * kZl); }

struct Range {
  uint32_t begin, end; /* bit patterns [begin, end) */
  uint64_t checked, mismatches;
  uint32_t first_bad;
};

static void* div127_worker(void* arg) {
  struct Range* r = (struct Range*)arg;
  for (uint32_t u = r->begin; u != r->end; ++u) {
    for (int sign = 0; sign < 2; ++sign) {
      const float a = from_bits(u | (sign ? 0x80000000u : 0u));
      const float want = a / 127.0F;
      const float got = div127(a);
      ++r->checked;
      if (!same(got, want)) {
        if (r->mismatches == 0) r->first_bad = to_bits(a);
        ++r->mismatches;
      }
    }
  }
  return NULL;
}

static int run_div127(int threads) {
  /* 2^-112 = 0x07800000; 0x7f800000 is +inf (excluded, checked below). */
  const uint32_t lo = 0x07800000u, hi = 0x7f800000u;
  struct Range* ranges = calloc((size_t)threads, sizeof *ranges);
  pthread_t* tid = calloc((size_t)threads, sizeof *tid);
  const uint32_t span = (hi - lo + (uint32_t)threads - 1) / (uint32_t)threads;
  for (int t = 0; t < threads; ++t) {
    ranges[t].begin = lo + (uint32_t)t * span;
    ranges[t].end = ranges[t].begin + span > hi ? hi : ranges[t].begin + span;
    pthread_create(&tid[t], NULL, div127_worker, &ranges[t]);
  }
  uint64_t checked = 0, bad = 0;
  uint32_t first_bad = 0;
  for (int t = 0; t < threads; ++t) {
    pthread_join(tid[t], NULL);
    checked += ranges[t].checked;
    if (ranges[t].mismatches && !bad) first_bad = ranges[t].first_bad;
    bad += ranges[t].mismatches;
  }
  const float specials[] = {0.0F, -0.0F, INFINITY, -INFINITY, NAN};
  for (size_t i = 0; i < sizeof specials / sizeof specials[0]; ++i) {
    ++checked;
    if (!same(div127(specials[i]), specials[i] / 127.0F)) ++bad;
  }
  printf("div127 checked=%llu mismatches=%llu", (unsigned long long)checked,
         (unsigned long long)bad);
  if (bad) printf(" first=0x%08x", first_bad);
  printf("\n");
  free(ranges);
  free(tid);
  return bad == 0 ? 0 : 1;
}

/* ---- Markstein quotient ----------------------------------------------------- */

static float div_markstein(float a, float c) {
  const float y = 1.0F / c;  /* RN(1/c), as __frcp_rn on the device */
  const float nc = -c;
  const float q0 = a * y;
  const float r0 = fmaf(q0, nc, a);
  const float q1 = fmaf(r0, y, q0);
  const float r1 = fmaf(q1, nc, a);
  return fmaf(r1, y, q1);
}

static uint64_t next(uint64_t* s) { /* SplitMix64 */
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* A float with a random mantissa and an exponent uniform in [emin, emax]. */
static float random_float(uint64_t* s, int emin, int emax) {
  const uint64_t r = next(s);
  const int e = emin + (int)(r % (uint64_t)(emax - emin + 1));
  const uint32_t mant = (uint32_t)(r >> 40) & 0x7FFFFFu;
  const uint32_t sign = (uint32_t)(r >> 39) & 1u;
  return from_bits((sign << 31) | ((uint32_t)(e + 127) << 23) | mant);
}

struct Sample {
  uint64_t seed, samples, checked, mismatches;
  float bad_a, bad_c;
};

static int in_range(float a, float c) {
  const float q = a / c;
  return fabsf(a) >= 0x1p-102F && fabsf(c) >= 0x1p-14F && fabsf(c) <= 0x1p100F &&
         isnormal(q) && isfinite(a);
}

static void check(struct Sample* s, float a, float c) {
  if (!in_range(a, c)) return;
  ++s->checked;
  if (!same(div_markstein(a, c), a / c)) {
    if (s->mismatches == 0) {
      s->bad_a = a;
      s->bad_c = c;
    }
    ++s->mismatches;
  }
}

static void* markstein_worker(void* arg) {
  struct Sample* s = (struct Sample*)arg;
  uint64_t state = s->seed;
  for (uint64_t i = 0; i < s->samples; ++i) {
    const float c = fabsf(random_float(&state, -14, 99));
    /* (1) random numerators across the range */
    check(s, random_float(&state, -102, 127), c);
    /* (2) numerators whose quotient lies next to a rounding midpoint: take a
     * float q, the midpoint m = q + ulp(q)/2 (exact in double), and
     * a = RN(m * c); then a / c = m (1 + d) with |d| <= 2^-24. */
    const float q = random_float(&state, -60, 60);
    const double ulp = ldexp(1.0, ilogb(q) - 23);
    const double m = (double)q + ulp * 0.5;
    const float a2 = (float)(m * (double)c);
    check(s, a2, c);
    check(s, nextafterf(a2, INFINITY), c);
    check(s, nextafterf(a2, -INFINITY), c);
    /* (3) exact quotients: a = q * c when representable */
    const float a3 = q * c;
    if ((double)a3 == (double)q * (double)c) check(s, a3, c);
  }
  return NULL;
}

static int run_markstein(int threads, uint64_t samples) {
  struct Sample* s = calloc((size_t)threads, sizeof *s);
  pthread_t* tid = calloc((size_t)threads, sizeof *tid);
  for (int t = 0; t < threads; ++t) {
    s[t].seed = 0x5EEDull + 7919ull * (uint64_t)t;
    s[t].samples = samples;
    pthread_create(&tid[t], NULL, markstein_worker, &s[t]);
  }
  uint64_t checked = 0, bad = 0;
  float bad_a = 0.0F, bad_c = 0.0F;
  for (int t = 0; t < threads; ++t) {
    pthread_join(tid[t], NULL);
    checked += s[t].checked;
    if (s[t].mismatches && !bad) {
      bad_a = s[t].bad_a;
      bad_c = s[t].bad_c;
    }
    bad += s[t].mismatches;
  }
  printf("markstein checked=%llu mismatches=%llu", (unsigned long long)checked,
         (unsigned long long)bad);
  if (bad) printf(" first=%a/%a", (double)bad_a, (double)bad_c);
  printf("\n");
  free(s);
  free(tid);
  return bad == 0 ? 0 : 1;
}

int main(int argc, char** argv) {
  if (argc >= 3 && strcmp(argv[1], "div127") == 0) return run_div127(atoi(argv[2]));
  if (argc >= 4 && strcmp(argv[1], "markstein") == 0) {
    return run_markstein(atoi(argv[2]), strtoull(argv[3], NULL, 10));
  }
  fprintf(stderr, "usage: %s div127 <threads> | markstein <threads> <samples>\n", argv[0]);
  return 2;
}
