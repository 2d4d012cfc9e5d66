/*
 * gdn_window_oracle.c -- CPU oracle for the windowed decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA window
 * kernels are compared against; it is never linked into, loaded by, or called
 * from the product library.  Only tests/, __graft_entry__.smoke() and the CPU
 * legs of bench.py may use it.
 *
 * It restates, in plain C and in the reference's operation order, the
 * portable codec's window (vLLM-HUST/gdn-state-codec,
 * native/src/gdn_state_codec_state_capsule.cpp):
 *
 *   window read   capsule.cpp:256-304   ReadWindowState: records newest to
 *                                       oldest (projection of the suffix-
 *                                       decayed read, then decay the suffix),
 *                                       then the INT8 boundary, then the
 *                                       rank-4 compensators
 *   token step    capsule.cpp:354-397   ApplyToken: correction = value -
 *                                       read(read); output = read(decay *
 *                                       query) + correction * (key . query);
 *                                       append {decay, key, correction}
 *   dense state   capsule.cpp:337-352   DenseState: dequantize, then every
 *                                       record oldest first: decay * S +
 *                                       key (x) correction
 *   boundary fit  capsule.cpp:130-225   QuantizeBoundary: rank-4 power
 *                                       iteration (sinf start vectors,
 *                                       `iterations` sweeps; the reference
 *                                       fixes 32) with deflation, then the
 *                                       INT8 stage
 *   dense step    native/ascendc/gdn_state_codec/kernel/
 *                 gdn_state_codec_fp32_gdn_step.cpp:10-16 (fp32 GDN step on a
 *                                       dense [key][value] state, the
 *                                       comparator the reference's window
 *                                       probe gates against)
 *
 * The device ABI stores the window records (keys, corrections) and the
 * compensators in binary16 (gdn_state_codec_windowed_gdn_kernel.h:5-6).  With
 * `round_storage` set, every value is rounded to binary16 (round to nearest,
 * ties to even) at the moment it is stored, exactly where the device stores
 * it; with it clear, storage is fp32 as in the portable library, which is how
 * tests pin this file against the reference library itself.
 *
 * One head is [128 key x 128 value].  The boundary codes are addressed with
 * the same geometry helper as gdn_codec_oracle.c: capsule [k][v] or provider
 * [v][k].  Compile with -ffp-contract=off (see Makefile): every product is
 * rounded before its sum, as in the reference build.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define W_KEYS 128
#define W_VALUES 128
#define W_RANK 4
#define W_WINDOW 16
#define W_ELEMENTS (W_KEYS * W_VALUES)

static const float kQMax = 127.0F;
static const float kFloor = 1.0e-8F;

static inline size_t w_at(int provider, uint32_t k, uint32_t v) {
  return provider ? (size_t)v * W_KEYS + k : (size_t)k * W_VALUES + v;
}

/* ---- binary16 / bfloat16 rounding (IEEE 754 round-to-nearest-even) ----- */

static inline uint32_t f32_bits(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  return b;
}
static inline float bits_f32(uint32_t b) {
  float x;
  memcpy(&x, &b, 4);
  return x;
}

/* float -> binary16 bits, round to nearest even, overflow to infinity. */
uint16_t oracle_f32_to_f16(float x) {
  const uint32_t b = f32_bits(x);
  const uint32_t sign = (b >> 16) & 0x8000u;
  const uint32_t exp = (b >> 23) & 0xFFu;
  uint32_t man = b & 0x7FFFFFu;
  if (exp == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
  /* unbiased exponent e: value = 1.man * 2^e (normal floats) */
  const int e = (int)exp - 127;
  if (e > 15) return (uint16_t)(sign | 0x7C00u);
  if (e >= -14) {
    /* normal half: 10 mantissa bits, drop 13 with RNE */
    uint32_t h = ((uint32_t)(e + 15) << 10) | (man >> 13);
    const uint32_t rest = man & 0x1FFFu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h; /* carry may reach inf */
    return (uint16_t)(sign | h);
  }
  if (exp == 0) return (uint16_t)sign; /* float subnormals are far below half's */
  /* subnormal half: value = m * 2^-24, m = significand * 2^(e + 1) */
  const int drop = -e - 1; /* 14..: low significand bits below 2^-24 */
  if (drop > 24) return (uint16_t)sign; /* below half of 2^-24: rounds to zero */
  man |= 0x800000u;
  uint32_t h = man >> drop;
  const uint32_t rest = man & ((1u << drop) - 1u);
  const uint32_t half = 1u << (drop - 1);
  if (rest > half || (rest == half && (h & 1u))) ++h;
  return (uint16_t)(sign | h);
}

float oracle_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  const uint32_t man = h & 0x3FFu;
  if (exp == 0x1Fu) return bits_f32(sign | 0x7F800000u | (man << 13));
  if (exp == 0) {
    /* subnormal: man * 2^-24, exact in float */
    const float m = (float)man * 5.9604644775390625e-08F;
    return sign ? -m : m;
  }
  return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

float oracle_round_f16(float x) { return oracle_f16_to_f32(oracle_f32_to_f16(x)); }

/* float -> bfloat16 bits, round to nearest even (finite inputs; NaN kept). */
uint16_t oracle_f32_to_bf16(float x) {
  const uint32_t b = f32_bits(x);
  if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x7FFFFFu)) return (uint16_t)((b >> 16) | 0x40u);
  return (uint16_t)((b + 0x7FFFu + ((b >> 16) & 1u)) >> 16);
}

float oracle_bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

static inline float store(float x, int round_storage) {
  return round_storage ? oracle_round_f16(x) : x;
}

/* ---- window read (capsule.cpp:256-304) ---------------------------------- */

/* out[v] = S^T x for the window: `records` buffered updates (record u has
 * scalar decay rdecay[u], key rkeys[u*128 + k], correction rcorr[u*128 + v])
 * over the boundary (codes in `provider` layout, smoothing c, scales b, and
 * compensators ck [k][4] / cv [v][4], or none when either is NULL). */
void oracle_window_read(int provider, const int8_t* codes, const float* c, const float* b,
                        const float* ck, const float* cv, uint32_t records,
                        const float* rdecay, const float* rkeys, const float* rcorr,
                        const float* x, float* out) {
  float suffix[W_KEYS];
  memcpy(suffix, x, sizeof(suffix));
  for (uint32_t v = 0; v < W_VALUES; ++v) out[v] = 0.0F;
  for (uint32_t u = records; u > 0; --u) {
    const float* key = rkeys + (size_t)(u - 1) * W_KEYS;
    const float* corr = rcorr + (size_t)(u - 1) * W_VALUES;
    float projection = 0.0F;
    for (uint32_t k = 0; k < W_KEYS; ++k) projection += key[k] * suffix[k];
    for (uint32_t v = 0; v < W_VALUES; ++v) out[v] += corr[v] * projection;
    for (uint32_t k = 0; k < W_KEYS; ++k) suffix[k] *= rdecay[u - 1];
  }
  for (uint32_t v = 0; v < W_VALUES; ++v) {
    float rp = 0.0F;
    for (uint32_t k = 0; k < W_KEYS; ++k) rp += (float)codes[w_at(provider, k, v)] * c[k] * suffix[k];
    out[v] += rp / kQMax * b[v];
  }
  if (ck != NULL && cv != NULL) {
    for (uint32_t r = 0; r < W_RANK; ++r) {
      float projection = 0.0F;
      for (uint32_t k = 0; k < W_KEYS; ++k) projection += ck[k * W_RANK + r] * suffix[k];
      for (uint32_t v = 0; v < W_VALUES; ++v) out[v] += cv[v * W_RANK + r] * projection;
    }
  }
}

/* ---- token step (capsule.cpp:354-397) ----------------------------------- */

/* One ApplyToken with a scalar decay: reads the window at position
 * *position (< 16), writes out[v], then appends record *position (stored
 * through binary16 when round_storage) and advances the position.  The
 * window fold at a full window is the separate oracle_window_fold. */
void oracle_window_step(int provider, const int8_t* codes, const float* c, const float* b,
                        const float* ck, const float* cv, float* rdecay, float* rkeys,
                        float* rcorr, uint32_t* position, float decay, const float* key,
                        const float* read, const float* query, const float* value,
                        int round_storage, float* out) {
  const uint32_t p = *position;
  float state_read[W_VALUES], decayed_query[W_KEYS], correction[W_VALUES];
  oracle_window_read(provider, codes, c, b, ck, cv, p, rdecay, rkeys, rcorr, read, state_read);
  for (uint32_t v = 0; v < W_VALUES; ++v) correction[v] = value[v] - state_read[v];
  float update_projection = 0.0F;
  for (uint32_t k = 0; k < W_KEYS; ++k) {
    decayed_query[k] = decay * query[k];
    update_projection += key[k] * query[k];
  }
  oracle_window_read(provider, codes, c, b, ck, cv, p, rdecay, rkeys, rcorr, decayed_query, out);
  for (uint32_t v = 0; v < W_VALUES; ++v) out[v] += correction[v] * update_projection;
  rdecay[p] = decay;
  for (uint32_t k = 0; k < W_KEYS; ++k) rkeys[(size_t)p * W_KEYS + k] = store(key[k], round_storage);
  for (uint32_t v = 0; v < W_VALUES; ++v) {
    rcorr[(size_t)p * W_VALUES + v] = store(correction[v], round_storage);
  }
  *position = p + 1;
}

/* ---- dense state (capsule.cpp:229-251, 337-352) ------------------------- */

/* dense[k][v] (capsule order) of the window: dequantized boundary plus the
 * compensators, then every record oldest first. */
void oracle_window_dense(int provider, const int8_t* codes, const float* c, const float* b,
                         const float* ck, const float* cv, uint32_t records,
                         const float* rdecay, const float* rkeys, const float* rcorr,
                         float* dense) {
  for (uint32_t k = 0; k < W_KEYS; ++k) {
    for (uint32_t v = 0; v < W_VALUES; ++v) {
      float value = c[k] * (float)codes[w_at(provider, k, v)] / kQMax * b[v];
      if (ck != NULL && cv != NULL) {
        for (uint32_t r = 0; r < W_RANK; ++r) value += ck[k * W_RANK + r] * cv[v * W_RANK + r];
      }
      dense[(size_t)k * W_VALUES + v] = value;
    }
  }
  for (uint32_t u = 0; u < records; ++u) {
    const float* key = rkeys + (size_t)u * W_KEYS;
    const float* corr = rcorr + (size_t)u * W_VALUES;
    for (uint32_t k = 0; k < W_KEYS; ++k) {
      for (uint32_t v = 0; v < W_VALUES; ++v) {
        float* s = dense + (size_t)k * W_VALUES + v;
        *s = rdecay[u] * *s + key[k] * corr[v];
      }
    }
  }
}

/* ---- boundary fit (capsule.cpp:47-65, 130-225) -------------------------- */

static float norm_of(const float* x, uint32_t n) {
  double sum = 0.0;
  for (uint32_t i = 0; i < n; ++i) sum += (double)x[i] * x[i];
  return (float)sqrt(sum);
}

static int normalize(float* x, uint32_t n) {
  const float norm = norm_of(x, n);
  if (!(norm > 1.1920928955078125e-07F)) return 0; /* FLT_EPSILON */
  for (uint32_t i = 0; i < n; ++i) x[i] /= norm;
  return 1;
}

/* QuantizeBoundary of a dense capsule-order head: with iterations > 0 the
 * rank-4 fit (start vectors sinf((r+1)(c+1)), `iterations` power sweeps,
 * deflation), then smoothing and INT8 codes of the residual.  Codes are
 * written in `provider` layout.  ck / cv receive the compensators (stored
 * through binary16 when round_storage; zeros when iterations == 0).
 * Returns 0, or 1 when the reference would reject the head (non-finite
 * input or singular value). */
int oracle_quantize_boundary(const float* dense_in, uint32_t iterations, int provider,
                             int round_storage, int8_t* codes, float* c, float* b, float* ck,
                             float* cv) {
  static _Thread_local float residual[W_ELEMENTS];
  static _Thread_local float smoothed[W_ELEMENTS];
  int status = 0;
  for (uint32_t i = 0; i < W_ELEMENTS; ++i) {
    residual[i] = dense_in[i];
    if (!isfinite(dense_in[i])) status = 1;
  }
  for (uint32_t i = 0; i < W_KEYS * W_RANK; ++i) ck[i] = 0.0F;
  for (uint32_t i = 0; i < W_VALUES * W_RANK; ++i) cv[i] = 0.0F;
  for (uint32_t rank = 0; iterations > 0 && rank < W_RANK; ++rank) {
    float right[W_VALUES], left[W_KEYS];
    for (uint32_t col = 0; col < W_VALUES; ++col) right[col] = sinf((float)((rank + 1) * (col + 1)));
    if (!normalize(right, W_VALUES)) right[0] = 1.0F;
    for (uint32_t it = 0; it < iterations; ++it) {
      for (uint32_t row = 0; row < W_KEYS; ++row) {
        left[row] = 0.0F;
        for (uint32_t col = 0; col < W_VALUES; ++col) {
          left[row] += residual[row * W_VALUES + col] * right[col];
        }
      }
      if (!normalize(left, W_KEYS)) break;
      for (uint32_t col = 0; col < W_VALUES; ++col) {
        right[col] = 0.0F;
        for (uint32_t row = 0; row < W_KEYS; ++row) {
          right[col] += residual[row * W_VALUES + col] * left[row];
        }
      }
      if (!normalize(right, W_VALUES)) break;
    }
    float sv = 0.0F;
    for (uint32_t row = 0; row < W_KEYS; ++row) {
      for (uint32_t col = 0; col < W_VALUES; ++col) {
        sv += left[row] * residual[row * W_VALUES + col] * right[col];
      }
    }
    if (!isfinite(sv)) status = 1;
    for (uint32_t row = 0; row < W_KEYS; ++row) {
      ck[row * W_RANK + rank] = store(left[row] * sv, round_storage);
    }
    for (uint32_t col = 0; col < W_VALUES; ++col) {
      cv[col * W_RANK + rank] = store(right[col], round_storage);
    }
    for (uint32_t row = 0; row < W_KEYS; ++row) {
      for (uint32_t col = 0; col < W_VALUES; ++col) {
        residual[row * W_VALUES + col] -= left[row] * sv * right[col];
      }
    }
  }
  for (uint32_t row = 0; row < W_KEYS; ++row) {
    double mean_absolute = 0.0;
    for (uint32_t col = 0; col < W_VALUES; ++col) mean_absolute += fabs((double)residual[row * W_VALUES + col]);
    mean_absolute /= (double)W_VALUES;
    const float m = (float)mean_absolute;
    c[row] = sqrtf(m < kFloor ? kFloor : m); /* std::max(m, floor) */
    for (uint32_t col = 0; col < W_VALUES; ++col) {
      smoothed[row * W_VALUES + col] = residual[row * W_VALUES + col] / c[row];
    }
  }
  for (uint32_t col = 0; col < W_VALUES; ++col) {
    float maximum = 0.0F;
    for (uint32_t row = 0; row < W_KEYS; ++row) {
      const float a = fabsf(smoothed[row * W_VALUES + col]);
      maximum = maximum < a ? a : maximum;
    }
    b[col] = maximum;
    for (uint32_t row = 0; row < W_KEYS; ++row) {
      const float scaled = maximum == 0.0F ? 0.0F : smoothed[row * W_VALUES + col] / maximum * kQMax;
      long q = lroundf(scaled);
      q = q < -127 ? -127 : (q > 127 ? 127 : q);
      codes[w_at(provider, row, col)] = (int8_t)q;
    }
  }
  return status;
}

/* Window fold (the refit at a window boundary): DenseState of the window,
 * QuantizeBoundary of it into the next boundary, records cleared (decay,
 * keys and corrections zero) and the position reset to 0. */
int oracle_window_fold(int provider, const int8_t* codes, const float* c, const float* b,
                       const float* ck, const float* cv, float* rdecay, float* rkeys,
                       float* rcorr, uint32_t* position, uint32_t iterations, int round_storage,
                       int8_t* next_codes, float* next_c, float* next_b, float* next_ck,
                       float* next_cv) {
  static _Thread_local float dense[W_ELEMENTS];
  oracle_window_dense(provider, codes, c, b, ck, cv, *position, rdecay, rkeys, rcorr, dense);
  const int status = oracle_quantize_boundary(dense, iterations, provider, round_storage,
                                              next_codes, next_c, next_b, next_ck, next_cv);
  for (uint32_t u = 0; u < W_WINDOW; ++u) rdecay[u] = 0.0F;
  memset(rkeys, 0, sizeof(float) * W_WINDOW * W_KEYS);
  memset(rcorr, 0, sizeof(float) * W_WINDOW * W_VALUES);
  *position = 0;
  return status;
}

/* ---- dense fp32 GDN step (fp32_gdn_step.cpp:10-16) ---------------------- */

/* In place on one dense capsule-order head: per value column v,
 * correction = value[v] - sum_k S[k][v] read[k]; S[k][v] = decay S[k][v] +
 * key[k] correction; out[v] = sum_k S_new[k][v] query[k] (k sequential). */
void oracle_dense_step(float* state, float decay, const float* key, const float* read,
                       const float* query, const float* value, float* out) {
  for (uint32_t v = 0; v < W_VALUES; ++v) {
    float projection = 0.0F;
    for (uint32_t k = 0; k < W_KEYS; ++k) projection += state[(size_t)k * W_VALUES + v] * read[k];
    const float correction = value[v] - projection;
    float o = 0.0F;
    for (uint32_t k = 0; k < W_KEYS; ++k) {
      float* s = state + (size_t)k * W_VALUES + v;
      const float next = decay * *s + key[k] * correction;
      *s = next;
      o += next * query[k];
    }
    out[v] = o;
  }
}
