/*
 * gdn_codec_oracle.c -- CPU oracle for the GDN state codec hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA kernels
 * are compared against; it is never linked into, loaded by, or called from
 * the product library.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may use it.
 *
 * It restates, in plain C, the arithmetic of the reference's portable C++
 * codec (vLLM-HUST/gdn-state-codec, native/src/gdn_state_codec_state_capsule.cpp):
 *
 *   smoothing   capsule.cpp:190-200   c_k = sqrtf(max((float)(sum_v |R_kv| in
 *                                     double, sequential v) / 128.0), 1e-8f))
 *   quantize    capsule.cpp:201-225   s = R/c; b_v = max_k |s_kv|;
 *                                     z = clamp(lround(s / b * 127), +-127)
 *   dequantize  capsule.cpp:236-248   ((c * z) / 127) * b  (+ sum_r K_kr V_vr)
 *   projection  capsule.cpp:281-304   o_v = 0 + (sum_k (z*c)*x, sequential k)
 *                                     / 127 * b  (+ sum_r V_vr (sum_k K_kr x_k))
 *   layout      gdn_state_codec_qwen38_gdn_adapter.cpp:21-57 (provider [v,k]
 *                                     <-> capsule [k,v] transpose)
 *
 * Every operation is written in the same order as the reference so that the
 * results are bit-identical when compiled as ISO C with -ffp-contract=off on
 * x86-64 (SSE arithmetic, no FMA contraction), which is how the reference's
 * own CMake build compiles (CMAKE_CXX_EXTENSIONS OFF, no -march flags).
 *
 * Parity is pinned against the real reference library: tests/golden holds
 * vectors produced by native/src compiled from the reference sources, and
 * tests/test_oracle_golden.py checks this file reproduces them bit for bit.
 *
 * Element (k, v) of one head lives at base[k * stride_k + v * stride_v]:
 *   capsule layout  [key, value]  stride_k = values, stride_v = 1
 *   provider layout [value, key]  stride_k = 1,      stride_v = keys
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>

#define ORACLE_RANK 4
static const float kQuantizedMaximum = 127.0F;
static const float kSmoothingFloor = 1.0e-8F;

typedef struct {
  uint32_t keys, values;
  size_t stride_k, stride_v; /* element strides inside one head */
} geometry_t;

static geometry_t make_geometry(uint32_t keys, uint32_t values, int provider) {
  geometry_t g;
  g.keys = keys;
  g.values = values;
  g.stride_k = provider ? 1 : values;
  g.stride_v = provider ? keys : 1;
  return g;
}

static inline size_t at(const geometry_t* g, uint32_t k, uint32_t v) {
  return (size_t)k * g->stride_k + (size_t)v * g->stride_v;
}

/* capsule.cpp:192-200: double accumulator, sequential over the value axis. */
static void smoothing_head(const geometry_t* g, const float* r, float* c) {
  for (uint32_t k = 0; k < g->keys; ++k) {
    double mean_absolute = 0.0;
    for (uint32_t v = 0; v < g->values; ++v) {
      mean_absolute += fabsf(r[at(g, k, v)]);
    }
    mean_absolute /= (double)g->values;
    const float mean = (float)mean_absolute;
    /* std::max(mean, floor) returns floor only when mean < floor. */
    c[k] = sqrtf(mean < kSmoothingFloor ? kSmoothingFloor : mean);
  }
}

/* capsule.cpp:201-225 given the per-key smoothing c (capsule.cpp:202-203
 * divides, :210-215 takes the column maximum, :216-224 rounds). */
static void quantize_head_given_smoothing(const geometry_t* g, const float* r,
                                          const float* c, int8_t* z, float* b) {
  for (uint32_t v = 0; v < g->values; ++v) {
    float maximum = 0.0F;
    for (uint32_t k = 0; k < g->keys; ++k) {
      const float smoothed = r[at(g, k, v)] / c[k];
      const float magnitude = fabsf(smoothed);
      /* std::max(maximum, magnitude) keeps maximum unless it is smaller. */
      if (maximum < magnitude) maximum = magnitude;
    }
    b[v] = maximum;
    for (uint32_t k = 0; k < g->keys; ++k) {
      const float smoothed = r[at(g, k, v)] / c[k];
      const float scaled =
          maximum == 0.0F ? 0.0F : smoothed / maximum * kQuantizedMaximum;
      long quantized = lroundf(scaled);
      if (quantized < -127L) quantized = -127L;
      if (quantized > 127L) quantized = 127L;
      z[at(g, k, v)] = (int8_t)quantized;
    }
  }
}

/* capsule.cpp:236-248. */
static void dequantize_head(const geometry_t* g, const int8_t* z, const float* c,
                            const float* b, const float* ck, const float* cv,
                            float* out) {
  for (uint32_t k = 0; k < g->keys; ++k) {
    for (uint32_t v = 0; v < g->values; ++v) {
      float value = c[k] * (float)z[at(g, k, v)] / kQuantizedMaximum * b[v];
      if (ck != NULL && cv != NULL) {
        for (uint32_t r = 0; r < ORACLE_RANK; ++r) {
          value += ck[k * ORACLE_RANK + r] * cv[v * ORACLE_RANK + r];
        }
      }
      out[at(g, k, v)] = value;
    }
  }
}

/* capsule.cpp:264 (output starts at zero), :281-290 (boundary readout),
 * :291-304 (rank-4 compensator readout). */
static void project_head(const geometry_t* g, const int8_t* z, const float* c,
                         const float* b, const float* ck, const float* cv,
                         const float* x, float* out) {
  for (uint32_t v = 0; v < g->values; ++v) {
    float residual_projection = 0.0F;
    for (uint32_t k = 0; k < g->keys; ++k) {
      residual_projection += (float)z[at(g, k, v)] * c[k] * x[k];
    }
    float output = 0.0F;
    output += residual_projection / kQuantizedMaximum * b[v];
    out[v] = output;
  }
  if (ck != NULL && cv != NULL) {
    for (uint32_t r = 0; r < ORACLE_RANK; ++r) {
      float projection = 0.0F;
      for (uint32_t k = 0; k < g->keys; ++k) {
        projection += ck[k * ORACLE_RANK + r] * x[k];
      }
      for (uint32_t v = 0; v < g->values; ++v) {
        out[v] += cv[v * ORACLE_RANK + r] * projection;
      }
    }
  }
}

/* ------------------------------------------------------------------------ */
/* Batched entry points (heads are contiguous; plain pointers, no globals).  */

void oracle_smoothing(const float* state, uint64_t heads, uint32_t keys,
                      uint32_t values, int provider, float* smoothing) {
  const geometry_t g = make_geometry(keys, values, provider);
  const size_t elements = (size_t)keys * values;
  for (uint64_t h = 0; h < heads; ++h) {
    smoothing_head(&g, state + h * elements, smoothing + h * keys);
  }
}

void oracle_quantize_given_smoothing(const float* state, const float* smoothing,
                                     uint64_t heads, uint32_t keys,
                                     uint32_t values, int provider,
                                     int8_t* codes, float* scales) {
  const geometry_t g = make_geometry(keys, values, provider);
  const size_t elements = (size_t)keys * values;
  for (uint64_t h = 0; h < heads; ++h) {
    quantize_head_given_smoothing(&g, state + h * elements, smoothing + h * keys,
                                  codes + h * elements, scales + h * values);
  }
}

/* Fused smoothing + quantize for one range of heads. */
static void quantize_range(const geometry_t* g, const float* state,
                           uint64_t first, uint64_t last, float* smoothing,
                           int8_t* codes, float* scales) {
  const size_t elements = (size_t)g->keys * g->values;
  for (uint64_t h = first; h < last; ++h) {
    smoothing_head(g, state + h * elements, smoothing + h * g->keys);
    quantize_head_given_smoothing(g, state + h * elements, smoothing + h * g->keys,
                                  codes + h * elements, scales + h * g->values);
  }
}

void oracle_quantize(const float* state, uint64_t heads, uint32_t keys,
                     uint32_t values, int provider, float* smoothing,
                     int8_t* codes, float* scales) {
  const geometry_t g = make_geometry(keys, values, provider);
  quantize_range(&g, state, 0, heads, smoothing, codes, scales);
}

void oracle_dequantize(const int8_t* codes, const float* smoothing,
                       const float* scales, const float* compensator_keys,
                       const float* compensator_values, uint64_t heads,
                       uint32_t keys, uint32_t values, int provider,
                       float* dense) {
  const geometry_t g = make_geometry(keys, values, provider);
  const size_t elements = (size_t)keys * values;
  for (uint64_t h = 0; h < heads; ++h) {
    dequantize_head(
        &g, codes + h * elements, smoothing + h * keys, scales + h * values,
        compensator_keys ? compensator_keys + h * keys * ORACLE_RANK : NULL,
        compensator_values ? compensator_values + h * values * ORACLE_RANK : NULL,
        dense + h * elements);
  }
}

void oracle_project(const int8_t* codes, const float* smoothing,
                    const float* scales, const float* compensator_keys,
                    const float* compensator_values, const float* queries,
                    uint64_t heads, uint32_t keys, uint32_t values, int provider,
                    float* outputs) {
  const geometry_t g = make_geometry(keys, values, provider);
  const size_t elements = (size_t)keys * values;
  for (uint64_t h = 0; h < heads; ++h) {
    project_head(
        &g, codes + h * elements, smoothing + h * keys, scales + h * values,
        compensator_keys ? compensator_keys + h * keys * ORACLE_RANK : NULL,
        compensator_values ? compensator_values + h * values * ORACLE_RANK : NULL,
        queries + h * keys, outputs + h * values);
  }
}

/* adapter.cpp:21-38 (provider -> capsule) and :40-57 (capsule -> provider). */
void oracle_provider_to_capsule(const float* provider, uint64_t heads,
                                uint32_t keys, uint32_t values, float* capsule) {
  const size_t elements = (size_t)keys * values;
  for (uint64_t h = 0; h < heads; ++h) {
    for (uint32_t v = 0; v < values; ++v) {
      for (uint32_t k = 0; k < keys; ++k) {
        capsule[h * elements + (size_t)k * values + v] =
            provider[h * elements + (size_t)v * keys + k];
      }
    }
  }
}

void oracle_capsule_to_provider(const float* capsule, uint64_t heads,
                                uint32_t keys, uint32_t values, float* provider) {
  const size_t elements = (size_t)keys * values;
  for (uint64_t h = 0; h < heads; ++h) {
    for (uint32_t k = 0; k < keys; ++k) {
      for (uint32_t v = 0; v < values; ++v) {
        provider[h * elements + (size_t)v * keys + k] =
            capsule[h * elements + (size_t)k * values + v];
      }
    }
  }
}

/* ------------------------------------------------------------------------ */
/* Multi-threaded drivers for the timed CPU baseline: one pthread per core   */
/* over independent heads (the codec has no shared mutable state).           */

typedef struct {
  int op; /* 0 quantize, 1 dequantize, 2 project */
  geometry_t g;
  uint64_t first, last;
  const float* state;
  float* smoothing;
  int8_t* codes;
  float* scales;
  const int8_t* in_codes;
  const float* in_smoothing;
  const float* in_scales;
  const float* queries;
  float* out;
} work_t;

static void* worker(void* arg) {
  work_t* w = (work_t*)arg;
  const size_t elements = (size_t)w->g.keys * w->g.values;
  if (w->op == 0) {
    quantize_range(&w->g, w->state, w->first, w->last, w->smoothing, w->codes,
                   w->scales);
  } else {
    for (uint64_t h = w->first; h < w->last; ++h) {
      if (w->op == 1) {
        dequantize_head(&w->g, w->in_codes + h * elements,
                        w->in_smoothing + h * w->g.keys,
                        w->in_scales + h * w->g.values, NULL, NULL,
                        w->out + h * elements);
      } else {
        project_head(&w->g, w->in_codes + h * elements,
                     w->in_smoothing + h * w->g.keys,
                     w->in_scales + h * w->g.values, NULL, NULL,
                     w->queries + h * w->g.keys, w->out + h * w->g.values);
      }
    }
  }
  return NULL;
}

static int run_threads(work_t* proto, uint64_t heads, int threads) {
  if (threads < 1) threads = 1;
  if ((uint64_t)threads > heads) threads = heads ? (int)heads : 1;
  pthread_t* ids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  work_t* items = (work_t*)calloc((size_t)threads, sizeof(work_t));
  if (!ids || !items) {
    free(ids);
    free(items);
    return -1;
  }
  int started = 0;
  for (int t = 0; t < threads; ++t) {
    items[t] = *proto;
    items[t].first = heads * (uint64_t)t / (uint64_t)threads;
    items[t].last = heads * (uint64_t)(t + 1) / (uint64_t)threads;
    if (pthread_create(&ids[t], NULL, worker, &items[t]) != 0) break;
    ++started;
  }
  for (int t = 0; t < started; ++t) pthread_join(ids[t], NULL);
  /* Any thread that failed to start: finish its range on this thread. */
  for (int t = started; t < threads; ++t) worker(&items[t]);
  free(ids);
  free(items);
  return threads;
}

int oracle_quantize_mt(const float* state, uint64_t heads, uint32_t keys,
                       uint32_t values, int provider, float* smoothing,
                       int8_t* codes, float* scales, int threads) {
  work_t w = {0};
  w.op = 0;
  w.g = make_geometry(keys, values, provider);
  w.state = state;
  w.smoothing = smoothing;
  w.codes = codes;
  w.scales = scales;
  return run_threads(&w, heads, threads);
}

int oracle_dequantize_mt(const int8_t* codes, const float* smoothing,
                         const float* scales, uint64_t heads, uint32_t keys,
                         uint32_t values, int provider, float* dense,
                         int threads) {
  work_t w = {0};
  w.op = 1;
  w.g = make_geometry(keys, values, provider);
  w.in_codes = codes;
  w.in_smoothing = smoothing;
  w.in_scales = scales;
  w.out = dense;
  return run_threads(&w, heads, threads);
}

int oracle_project_mt(const int8_t* codes, const float* smoothing,
                      const float* scales, const float* queries, uint64_t heads,
                      uint32_t keys, uint32_t values, int provider,
                      float* outputs, int threads) {
  work_t w = {0};
  w.op = 2;
  w.g = make_geometry(keys, values, provider);
  w.in_codes = codes;
  w.in_smoothing = smoothing;
  w.in_scales = scales;
  w.queries = queries;
  w.out = outputs;
  return run_threads(&w, heads, threads);
}
