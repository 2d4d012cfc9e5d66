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
 *       a / c from the two-term reciprocal y = RN(1/c), yl = RN((1 - c y) y):
 *       the faithful q0 = fma(a, y, RN(a yl)), then one correction
 *       r = fma(-q0, c, a), q = fma(r, y, q0) (Markstein, "Computation of
 *       elementary functions on the IBM RISC System/6000 processor", IBM
 *       J. R&D 34(1), 1990).  Checked on random operands over the kernels'
 *       fast-path ranges (c in [2^-14, 2^100], |a| >= 2^-102, quotient of
 *       magnitude >= 2^-125), on quotients at the bottom of that range, and
 *       on operands built so that a / c lies within a few ulps of a rounding
 *       midpoint -- the hard cases of correctly rounded division.
 *
 *   codes <threads> <samples per thread>
 *       the quantizer's code rule from one fma, u = fma(s, RN(127 / b), M)
 *       with M = 1.5 * 2^23, and its flag |fma(s, km, M - u)| > 0.5 - 3 * 2^-17:
 *       every unflagged code equals the reference's
 *       clamp(lround(RN(RN(s / b) * 127))), on random values and on values
 *       next to rounding boundaries.
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
  const float yl = fmaf(-c, y, 1.0F) * y;  /* second reciprocal term */
  const float nc = -c;
  const float q0 = fmaf(a, y, a * yl);  /* faithful */
  const float r = fmaf(q0, nc, a);
  return fmaf(r, y, q0);
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
         isfinite(q) && fabsf(q) >= 0x1p-125F && isfinite(a);
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
    /* (4) quotients at the bottom of the range, where RN(a yl) is tiny */
    const float cl = fabsf(random_float(&state, 60, 99));
    const float ql = random_float(&state, -125, -110);
    const float a4 = (float)((double)ql * (double)cl);
    check(s, a4, cl);
    check(s, nextafterf(a4, INFINITY), cl);
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

/* ---- codes from one fma ----------------------------------------------------- */

/* The quantizer's code rule: km = RN(127 / b), u = fma(s, km, M) with
 * M = 1.5 * 2^23, d = fma(s, km, M - u).  When |d| <= 0.5 - 3 * 2^-17 the code is
 * u - M; otherwise the element is flagged for the exact path.  An unflagged
 * code must equal the reference's clamp(lround(RN(RN(s / b) * 127))). */
struct CodeSample {
  uint64_t seed, samples, checked, flagged, mismatches, random_flagged;
  float bad_s, bad_b;
};

static int check_code(struct CodeSample* cs, float s, float b) {
  if (!(fabsf(s) <= b)) return 0;
  const float km = 127.0F / b;
  const float magic = 12582912.0F;
  const float u = fmaf(s, km, magic);
  const float d = fmaf(s, km, magic - u);
  ++cs->checked;
  if (!(fabsf(d) <= 0.5F - 0x1.8p-16F)) {
    ++cs->flagged;
    return 1;
  }
  long want = lroundf((s / b) * 127.0F);
  want = want < -127 ? -127 : (want > 127 ? 127 : want);
  if ((long)(u - magic) != want) {
    if (cs->mismatches == 0) {
      cs->bad_s = s;
      cs->bad_b = b;
    }
    ++cs->mismatches;
  }
  return 0;
}

static void* code_worker(void* arg) {
  struct CodeSample* cs = (struct CodeSample*)arg;
  uint64_t state = cs->seed;
  for (uint64_t i = 0; i < cs->samples; ++i) {
    const float b = fabsf(random_float(&state, -64, 99));
    /* (1) a random smoothed value in [-b, b] */
    const uint64_t r = next(&state);
    const float s = (float)(((double)(r >> 11) * 0x1p-53 * 2.0 - 1.0) * (double)b);
    cs->random_flagged += (uint64_t)check_code(cs, s, b);
    /* (2) values whose scaled code lies next to a rounding boundary n + 1/2 */
    const long n = (long)(next(&state) % 254u) - 127;
    const float t = (float)((double)n + 0.5);
    const float s2 = (float)((double)t * (double)b / 127.0);
    float v = s2;
    for (int k = 0; k < 4; ++k) v = nextafterf(v, -INFINITY);
    for (int k = 0; k < 9; ++k, v = nextafterf(v, INFINITY)) check_code(cs, v, b);
    /* (3) the maximum itself and its neighbours */
    check_code(cs, b, b);
    check_code(cs, -b, b);
    check_code(cs, nextafterf(b, 0.0F), b);
  }
  return NULL;
}

static int run_codes(int threads, uint64_t samples) {
  struct CodeSample* cs = calloc((size_t)threads, sizeof *cs);
  pthread_t* tid = calloc((size_t)threads, sizeof *tid);
  for (int t = 0; t < threads; ++t) {
    cs[t].seed = 0xC0DEull + 104729ull * (uint64_t)t;
    cs[t].samples = samples;
    pthread_create(&tid[t], NULL, code_worker, &cs[t]);
  }
  uint64_t checked = 0, flagged = 0, bad = 0, random_flagged = 0;
  float bad_s = 0.0F, bad_b = 0.0F;
  for (int t = 0; t < threads; ++t) {
    pthread_join(tid[t], NULL);
    checked += cs[t].checked;
    flagged += cs[t].flagged;
    random_flagged += cs[t].random_flagged;
    if (cs[t].mismatches && !bad) {
      bad_s = cs[t].bad_s;
      bad_b = cs[t].bad_b;
    }
    bad += cs[t].mismatches;
  }
  printf("codes checked=%llu flagged=%llu random=%llu random_flagged=%llu mismatches=%llu",
         (unsigned long long)checked, (unsigned long long)flagged,
         (unsigned long long)samples * (uint64_t)threads, (unsigned long long)random_flagged,
         (unsigned long long)bad);
  if (bad) printf(" first=%a/%a", (double)bad_s, (double)bad_b);
  printf("\n");
  free(cs);
  free(tid);
  return bad == 0 ? 0 : 1;
}

int main(int argc, char** argv) {
  if (argc >= 3 && strcmp(argv[1], "div127") == 0) return run_div127(atoi(argv[2]));
  if (argc >= 4 && strcmp(argv[1], "markstein") == 0) {
    return run_markstein(atoi(argv[2]), strtoull(argv[3], NULL, 10));
  }
  if (argc >= 4 && strcmp(argv[1], "codes") == 0) {
    return run_codes(atoi(argv[2]), strtoull(argv[3], NULL, 10));
  }
  fprintf(stderr, "usage: %s div127 <threads> | markstein|codes <threads> <samples>\n",
          argv[0]);
  return 2;
}
