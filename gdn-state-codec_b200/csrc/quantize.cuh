// quantize.cuh -- int8 encode of GDN recurrent state heads (sm_100a).
//
// Restates the reference's quant stage (native/src/gdn_state_codec_state_
// capsule.cpp:190-225; quant-only semantics as in the device probe
// native/ascendc/gdn_state_codec/host/gdn_state_codec_provider_quantize_probe
// .cpp:130-165) with bit-identical results:
//
//   c_k = sqrtf(max((float)(sum_v |R_kv| (double) / 128), 1e-8f))
//   s_kv = R_kv / c_k                         (IEEE fp32 division)
//   b_v = max_k |s_kv|
//   z_kv = clamp(lround(s_kv / b_v * 127), -127, 127), 0 when b_v == 0
//
// Design (HBM-bound: 64 KiB read + 17 KiB written per head):
//  * one persistent 512-thread CTA per SM with a ring of kStages 64 KiB
//    shared-memory landing buffers, each filled by one TMA bulk copy
//    (cp.async.bulk + mbarrier); while a head is computed from registers the
//    next kStages-1 heads stream in.
//  * warp w holds rows 8w..8w+7 of the head, lane l holds columns 4l..4l+3
//    (32 floats per thread, read with conflict-free 128-bit shared loads: a
//    warp reads one 512-byte row per instruction).
//  * smoothing sums run in double; the per-value maximum and the codes run in
//    fp32 from one multiply by RN(1/c) with a proven error bound, and the few
//    elements inside that bound of a decision point are recomputed with IEEE
//    division, so every output is exact.
//  * capsule layout: row sums by warp shuffles, column maxima through shared
//    memory; provider layout: column sums through shared memory, row maxima
//    by warp shuffles.
#pragma once

#include "codec_device.cuh"

namespace gdnsc {

constexpr int kQThreads = 512;
constexpr int kQWarps = kQThreads / 32;        // 16
constexpr int kRowsPerWarp = kKeys / kQWarps;  // 8
constexpr int kLanesPerRow = 32 / kRowsPerWarp;  // 4 lanes share a reduced row
constexpr int kStages = 2;

// Error bound of the reciprocal product: s' = RN(R * RN(1/c)) is within
// 1.5 * 2^-23 of RN(R / c) relative (two roundings of 2^-24 each plus the
// reciprocal's), so (a) the exact maximum can only come from an element whose
// s' is within 2^-20 of the approximate maximum m', and (b) the approximate
// scaled value t' = RN(s' * RN(127 / m')) is within 2^-13.7 of the exact
// RN(RN(s / m) * 127): a code is decided directly unless t' lies within
// 2^-12 of a rounding boundary n + 0.5.  Outside [2^-100, 2^100] (all-zero or
// denormal columns, non-finite data) the exact path is taken for the column.
constexpr float kCandidateFactor = 1.0F - 0x1p-20F;
constexpr float kAmbiguous = 0.5F - 0x1p-12F;
constexpr float kFastMin = 0x1p-100F;
constexpr float kFastMax = 0x1p100F;

enum QuantizeMode : int {
  kFused = 0,           // smoothing + quantize (initialize_launch_v3)
  kGivenSmoothing = 1,  // quantize with the caller's smoothing
  kSmoothingOnly = 2,   // smoothing only
};

struct QuantizeParams {
  const float* state;         // [heads][128][128] fp32
  const float* smoothing_in;  // kGivenSmoothing: [heads][128]
  float* smoothing;           // kFused / kSmoothingOnly output [heads][128]
  int8_t* codes;              // [heads][128][128]
  float* scales;              // [heads][128]
  uint64_t items;             // work items (heads, or entries * heads_per_slot)
  SlotMap map;
  uint32_t* status;           // optional caller status word
};

struct __align__(128) QuantizeShared {
  float stage[kStages][kElements];  // TMA landing buffers (64 KiB each)
  union {
    float col_part[kQWarps][kValues];  // capsule: per-warp column maxima
    double col_dsum[kQWarps][kKeys];   // provider: per-warp column sums
  };
  float key_c[kKeys];            // provider: smoothing per key
  float key_y[kKeys];            // provider: RN(1/c) per key
  float col_km[kValues];         // capsule: RN(127 / m') per column
  float col_thr[kValues];        // capsule: candidate threshold per column
  uint32_t col_exact[kValues];   // capsule: exact column maximum (bits)
  float colbuf[kKeys];           // provider: one column for a sequential re-sum
  float row_c[kQWarps][kRowsPerWarp];       // capsule: smoothing of my rows
  float row_y[kQWarps][kRowsPerWarp];       // capsule: RN(1/c) of my rows
  float row_km[kQWarps][kRowsPerWarp];      // provider: per-row km
  float row_thr[kQWarps][kRowsPerWarp];     // provider: per-row threshold
  uint32_t row_exact[kQWarps][kRowsPerWarp];  // provider: exact row maximum
  int col_flag[kKeys];
  uint64_t full[kStages];        // one mbarrier per landing buffer
};

// ---------------------------------------------------------------------------
// Small helpers.

__device__ __forceinline__ float4 mul4s(float4 a, float y) {
  const f2 yy = pack2(y, y);
  const f2 lo = mul2(pack2(a.x, a.y), yy);
  const f2 hi = mul2(pack2(a.z, a.w), yy);
  return make_float4(lo2(lo), hi2(lo), lo2(hi), hi2(hi));
}
__device__ __forceinline__ float4 mul4v(float4 a, float4 y) {
  const f2 lo = mul2(pack2(a.x, a.y), pack2(y.x, y.y));
  const f2 hi = mul2(pack2(a.z, a.w), pack2(y.z, y.w));
  return make_float4(lo2(lo), hi2(lo), lo2(hi), hi2(hi));
}
__device__ __forceinline__ float absmax4(float4 a) {
  return fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w)));
}
__device__ __forceinline__ float comp(const float4& a, int i) {
  return i == 0 ? a.x : (i == 1 ? a.y : (i == 2 ? a.z : a.w));
}

// Approximate codes for four elements: t = s * km rounded through the magic
// constant; returns the packed int8x4 word and flags elements within the
// ambiguity band of a rounding boundary.
__device__ __forceinline__ uint32_t approx_codes(float4 s, float4 km, bool* amb) {
  const f2 t01 = mul2(pack2(s.x, s.y), pack2(km.x, km.y));
  const f2 t23 = mul2(pack2(s.z, s.w), pack2(km.z, km.w));
  const f2 magic = pack2(kRoundMagic, kRoundMagic);
  const f2 u01 = add2(t01, magic);
  const f2 u23 = add2(t23, magic);
  const f2 d01 = sub2(t01, sub2(u01, magic));
  const f2 d23 = sub2(t23, sub2(u23, magic));
  const float worst = fmaxf(fmaxf(fabsf(lo2(d01)), fabsf(hi2(d01))),
                            fmaxf(fabsf(lo2(d23)), fabsf(hi2(d23))));
  *amb = *amb || !(worst <= kAmbiguous);
  const uint32_t w01 = __byte_perm(static_cast<uint32_t>(u01), static_cast<uint32_t>(u01 >> 32), 0x0040);
  const uint32_t w23 = __byte_perm(static_cast<uint32_t>(u23), static_cast<uint32_t>(u23 >> 32), 0x0040);
  return __byte_perm(w01, w23, 0x5410);
}

__device__ __forceinline__ bool approx_ambiguous(float s, float km) {
  const float t = __fmul_rn(s, km);
  const float u = __fadd_rn(t, kRoundMagic);
  const float d = __fsub_rn(t, __fsub_rn(u, kRoundMagic));
  return !(fabsf(d) <= kAmbiguous);
}

__device__ __forceinline__ float4 select_row(const float4 (&v)[kRowsPerWarp], int r) {
  float4 out = v[0];
#pragma unroll
  for (int j = 1; j < kRowsPerWarp; ++j) {
    if (j == r) out = v[j];
  }
  return out;
}

// Warp reduce-scatter of kRowsPerWarp per-row partials: afterwards the
// kLanesPerRow lanes with lane / kLanesPerRow == r hold the total of row r.
__device__ __forceinline__ double reduce_scatter_sum(double (&p)[kRowsPerWarp], int lane) {
  int offset = 16;
#pragma unroll
  for (int half = kRowsPerWarp / 2; half >= 1; half >>= 1, offset >>= 1) {
    const bool upper = (lane & offset) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const double send = upper ? p[i] : p[i + half];
      const double keep = upper ? p[i + half] : p[i];
      p[i] = keep + __shfl_xor_sync(0xffffffffu, send, offset);
    }
  }
  double total = p[0];
#pragma unroll
  for (int o = kLanesPerRow / 2; o >= 1; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
  return total;
}

__device__ __forceinline__ float reduce_scatter_max(float (&p)[kRowsPerWarp], int lane) {
  int offset = 16;
#pragma unroll
  for (int half = kRowsPerWarp / 2; half >= 1; half >>= 1, offset >>= 1) {
    const bool upper = (lane & offset) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = upper ? p[i] : p[i + half];
      const float keep = upper ? p[i + half] : p[i];
      p[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, offset));
    }
  }
  float total = p[0];
#pragma unroll
  for (int o = kLanesPerRow / 2; o >= 1; o >>= 1) {
    total = fmaxf(total, __shfl_xor_sync(0xffffffffu, total, o));
  }
  return total;
}

// Next work item at or after `item` (stride `step`) that names a real head.
__device__ __forceinline__ uint64_t next_item(const QuantizeParams& p, uint64_t item,
                                              uint64_t step, int64_t* head, bool report_bad) {
  while (item < p.items) {
    bool bad = false;
    const int64_t h = resolve_item(p.map, item, &bad);
    if (bad && report_bad) report(p.status, kStatusBadSlot);
    if (h >= 0) {
      *head = h;
      return item;
    }
    item += step;
  }
  *head = -1;
  return item;
}

__device__ __forceinline__ void issue_head(QuantizeShared& sh, const QuantizeParams& p, int stage,
                                           int64_t head) {
  fence_proxy_async();
  mbar_expect_tx(&sh.full[stage], kElements * sizeof(float));
  bulk_load(sh.stage[stage], p.state + static_cast<uint64_t>(head) * kElements,
            kElements * sizeof(float), &sh.full[stage], evict_first_policy());
}

// ---------------------------------------------------------------------------
// Capsule layout [key, value]: row k = key, column v = value.  Returns false
// when the block must stop (a bounded wait expired somewhere in the block).

template <int kMode>
__device__ __forceinline__ bool quantize_capsule_head(const QuantizeParams& p, QuantizeShared& sh,
                                                      const float4 (&v)[kRowsPerWarp],
                                                      int64_t head, int warp, int lane, int tid,
                                                      bool timed_out, int stage,
                                                      int64_t refill_head) {
  const int row0 = warp * kRowsPerWarp;
  // -- smoothing per row (warp-local) -----------------------------------------
  if (kMode == kGivenSmoothing) {
    if (lane < kRowsPerWarp) {
      const float c = __ldg(p.smoothing_in + head * kKeys + row0 + lane);
      sh.row_c[warp][lane] = c;
      sh.row_y[warp][lane] = __frcp_rn(c);
    }
  } else {
    double part[kRowsPerWarp];
#pragma unroll
    for (int j = 0; j < kRowsPerWarp; ++j) {
      part[j] = (static_cast<double>(fabsf(v[j].x)) + static_cast<double>(fabsf(v[j].y))) +
                (static_cast<double>(fabsf(v[j].z)) + static_cast<double>(fabsf(v[j].w)));
    }
    double sum = reduce_scatter_sum(part, lane);
    const int my_row = lane / kLanesPerRow;
    // Rows whose float mean could depend on the summation order are re-summed
    // in the reference's order (capsule.cpp:193-196): value 0..127.
    uint32_t flagged = __ballot_sync(0xffffffffu, near_float_midpoint(sum * (1.0 / 128.0))) &
                       0x11111111u;
    while (flagged != 0u) {
      const int owner = __ffs(flagged) - 1;
      flagged &= flagged - 1u;
      const float4 mine = select_row(v, owner / kLanesPerRow);
      double seq = 0.0;
      for (int src = 0; src < 32; ++src) {
        seq += fabsf(__shfl_sync(0xffffffffu, mine.x, src));
        seq += fabsf(__shfl_sync(0xffffffffu, mine.y, src));
        seq += fabsf(__shfl_sync(0xffffffffu, mine.z, src));
        seq += fabsf(__shfl_sync(0xffffffffu, mine.w, src));
      }
      if (my_row == owner / kLanesPerRow) sum = seq;
    }
    const float c = smoothing_from_sum(sum);
    if (lane % kLanesPerRow == 0) {
      sh.row_c[warp][my_row] = c;
      sh.row_y[warp][my_row] = __frcp_rn(c);
      p.smoothing[head * kKeys + row0 + my_row] = c;
    }
  }
  __syncwarp();
  if (kMode == kSmoothingOnly) {
    if (__syncthreads_or(timed_out) != 0) return false;
    if (tid == 0 && refill_head >= 0) issue_head(sh, p, stage, refill_head);
    return true;
  }

  // -- approximate column maxima -------------------------------------------
  float4 pm = make_float4(0.F, 0.F, 0.F, 0.F);
#pragma unroll
  for (int j = 0; j < kRowsPerWarp; ++j) {
    const float4 s = mul4s(v[j], sh.row_y[warp][j]);
    pm.x = fmaxf(pm.x, fabsf(s.x));
    pm.y = fmaxf(pm.y, fabsf(s.y));
    pm.z = fmaxf(pm.z, fabsf(s.z));
    pm.w = fmaxf(pm.w, fabsf(s.w));
  }
  reinterpret_cast<float4*>(sh.col_part[warp])[lane] = pm;
  // B1: every warp has read the landing buffer and published its maxima.
  if (__syncthreads_or(timed_out) != 0) return false;
  if (tid == 0 && refill_head >= 0) issue_head(sh, p, stage, refill_head);
  int slow = 0;
  if (tid < kValues) {
    float m = 0.0F;
#pragma unroll
    for (int w = 0; w < kQWarps; ++w) m = fmaxf(m, sh.col_part[w][tid]);
    slow = !(m >= kFastMin && m <= kFastMax);
    sh.col_km[tid] = slow ? 0.0F : __fdiv_rn(kQuantMax, m);
    sh.col_thr[tid] = slow ? -1.0F : __fmul_rn(m, kCandidateFactor);
    sh.col_exact[tid] = 0u;
  }
  const bool any_slow = __syncthreads_or(slow) != 0;  // B2

  // -- codes, and exact maxima from the candidates --------------------------
  const float4 km = reinterpret_cast<const float4*>(sh.col_km)[lane];
  const float4 thr = reinterpret_cast<const float4*>(sh.col_thr)[lane];
  uint32_t amb_rows = 0u;
  int8_t* codes = p.codes + static_cast<uint64_t>(head) * kElements;
#pragma unroll
  for (int j = 0; j < kRowsPerWarp; ++j) {
    const float4 s = mul4s(v[j], sh.row_y[warp][j]);
    const bool cand = (fabsf(s.x) >= thr.x) || (fabsf(s.y) >= thr.y) ||
                      (fabsf(s.z) >= thr.z) || (fabsf(s.w) >= thr.w);
    if (cand) {
      const float c = sh.row_c[warp][j];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float r = comp(v[j], i);
        if (fabsf(comp(s, i)) >= comp(thr, i) && r != 0.0F) {
          const float exact = fabsf(__fdiv_rn(r, c));
          atomicMax(&sh.col_exact[4 * lane + i], __float_as_uint(exact));
        }
      }
    }
    bool amb = false;
    const uint32_t word = approx_codes(s, km, &amb);
    st_cs_u32(codes + (row0 + j) * kValues + 4 * lane, word);
    amb_rows |= amb ? (1u << j) : 0u;
  }
  __syncthreads();  // B3: exact maxima complete
  if (tid < kValues) p.scales[head * kValues + tid] = __uint_as_float(sh.col_exact[tid]);
  // Elements inside the ambiguity band, and every element of a column outside
  // the fast range, take the exact computation with the exact maximum.
  const bool my_slow = any_slow && (thr.x < 0.F || thr.y < 0.F || thr.z < 0.F || thr.w < 0.F);
  if (amb_rows != 0u || my_slow) {
    for (int j = 0; j < kRowsPerWarp; ++j) {
      const bool row_amb = (amb_rows >> j) & 1u;
      if (!row_amb && !my_slow) continue;
      const float4 r4 = select_row(v, j);
      const float c = sh.row_c[warp][j];
      const float yy = sh.row_y[warp][j];
      for (int i = 0; i < 4; ++i) {
        const int col = 4 * lane + i;
        const float r = comp(r4, i);
        bool redo = comp(thr, i) < 0.F;
        if (!redo && row_amb) redo = approx_ambiguous(__fmul_rn(r, yy), comp(km, i));
        if (!redo) continue;
        const float m = __uint_as_float(sh.col_exact[col]);
        codes[(row0 + j) * kValues + col] = exact_code(__fdiv_rn(r, c), m);
      }
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// Provider layout [value, key]: row = value v, column = key k.

template <int kMode>
__device__ __forceinline__ bool quantize_provider_head(const QuantizeParams& p, QuantizeShared& sh,
                                                       const float4 (&v)[kRowsPerWarp],
                                                       int64_t head, int warp, int lane, int tid,
                                                       bool timed_out, int stage,
                                                       int64_t refill_head) {
  const int row0 = warp * kRowsPerWarp;
  // -- smoothing per key (column), across warps --------------------------------
  if (kMode != kGivenSmoothing) {
    double cs0 = 0.0, cs1 = 0.0, cs2 = 0.0, cs3 = 0.0;
#pragma unroll
    for (int j = 0; j < kRowsPerWarp; ++j) {
      cs0 += fabsf(v[j].x);
      cs1 += fabsf(v[j].y);
      cs2 += fabsf(v[j].z);
      cs3 += fabsf(v[j].w);
    }
    double* dst = &sh.col_dsum[warp][4 * lane];
    dst[0] = cs0;
    dst[1] = cs1;
    dst[2] = cs2;
    dst[3] = cs3;
  }
  // B1: every warp has read the landing buffer.
  if (__syncthreads_or(timed_out) != 0) return false;
  if (tid == 0 && refill_head >= 0) issue_head(sh, p, stage, refill_head);
  int flag = 0;
  if (tid < kKeys) {
    float c;
    if (kMode == kGivenSmoothing) {
      c = __ldg(p.smoothing_in + head * kKeys + tid);
    } else {
      double sum = 0.0;
#pragma unroll
      for (int w = 0; w < kQWarps; ++w) sum += sh.col_dsum[w][tid];
      flag = near_float_midpoint(sum * (1.0 / 128.0));
      c = smoothing_from_sum(sum);
      if (!flag) p.smoothing[head * kKeys + tid] = c;
    }
    sh.key_c[tid] = c;
    sh.key_y[tid] = __frcp_rn(c);
    sh.col_flag[tid] = flag;
  }
  if (__syncthreads_or(flag) != 0) {  // B2; the rare re-sum branch is block-uniform
    for (int k = 0; k < kKeys; ++k) {
      if (!sh.col_flag[k]) continue;
      if (lane == (k >> 2)) {
#pragma unroll
        for (int j = 0; j < kRowsPerWarp; ++j) sh.colbuf[row0 + j] = comp(v[j], k & 3);
      }
      __syncthreads();
      if (tid == 0) {
        double seq = 0.0;  // capsule.cpp:193-196 order: value 0..127
        for (int r = 0; r < kValues; ++r) seq += fabsf(sh.colbuf[r]);
        const float c = smoothing_from_sum(seq);
        sh.key_c[k] = c;
        sh.key_y[k] = __frcp_rn(c);
        p.smoothing[head * kKeys + k] = c;
      }
      __syncthreads();
    }
  }
  if (kMode == kSmoothingOnly) return true;

  const float4 y4 = reinterpret_cast<const float4*>(sh.key_y)[lane];
  // -- approximate row maxima (warp-local) ---------------------------------------
  float rm[kRowsPerWarp];
#pragma unroll
  for (int j = 0; j < kRowsPerWarp; ++j) rm[j] = absmax4(mul4v(v[j], y4));
  const float m = reduce_scatter_max(rm, lane);
  if (lane % kLanesPerRow == 0) {
    const int r = lane / kLanesPerRow;
    const bool slow = !(m >= kFastMin && m <= kFastMax);
    sh.row_km[warp][r] = slow ? 0.0F : __fdiv_rn(kQuantMax, m);
    sh.row_thr[warp][r] = slow ? -1.0F : __fmul_rn(m, kCandidateFactor);
    sh.row_exact[warp][r] = 0u;
  }
  __syncwarp();

  // -- codes, and exact maxima from the candidates ---------------------------------
  const float4 c4 = reinterpret_cast<const float4*>(sh.key_c)[lane];
  uint32_t amb_rows = 0u, slow_rows = 0u;
  int8_t* codes = p.codes + static_cast<uint64_t>(head) * kElements;
#pragma unroll
  for (int j = 0; j < kRowsPerWarp; ++j) {
    const float km = sh.row_km[warp][j];
    const float thr = sh.row_thr[warp][j];
    const float4 s = mul4v(v[j], y4);
    if (absmax4(s) >= thr) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float r = comp(v[j], i);
        if (fabsf(comp(s, i)) >= thr && r != 0.0F) {
          const float exact = fabsf(__fdiv_rn(r, comp(c4, i)));
          atomicMax(&sh.row_exact[warp][j], __float_as_uint(exact));
        }
      }
    }
    bool amb = false;
    const uint32_t word = approx_codes(s, make_float4(km, km, km, km), &amb);
    st_cs_u32(codes + (row0 + j) * kKeys + 4 * lane, word);
    amb_rows |= amb ? (1u << j) : 0u;
    slow_rows |= thr < 0.F ? (1u << j) : 0u;
  }
  __syncwarp();
  if (lane < kRowsPerWarp) {
    p.scales[head * kValues + row0 + lane] = __uint_as_float(sh.row_exact[warp][lane]);
  }
  const uint32_t redo_rows = amb_rows | slow_rows;
  if (redo_rows != 0u) {
    for (int j = 0; j < kRowsPerWarp; ++j) {
      if (!((redo_rows >> j) & 1u)) continue;
      const float4 r4 = select_row(v, j);
      const float km = sh.row_km[warp][j];
      const float mx = __uint_as_float(sh.row_exact[warp][j]);
      const bool row_slow = (slow_rows >> j) & 1u;
      for (int i = 0; i < 4; ++i) {
        const float r = comp(r4, i);
        const bool redo = row_slow || approx_ambiguous(__fmul_rn(r, comp(y4, i)), km);
        if (!redo) continue;
        codes[(row0 + j) * kKeys + 4 * lane + i] = exact_code(__fdiv_rn(r, comp(c4, i)), mx);
      }
    }
  }
  return true;
}

// ---------------------------------------------------------------------------

template <bool kProvider, int kMode>
__global__ void __launch_bounds__(kQThreads, 1) quantize_kernel(QuantizeParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  QuantizeShared& sh = *reinterpret_cast<QuantizeShared*>(smem_raw);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint64_t step = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&sh.full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // The producer (thread 0) runs kStages valid heads ahead of the consumers;
  // both walk the same deterministic item sequence.
  int64_t prod_head = -1;
  uint64_t prod_item = next_item(p, blockIdx.x, step, &prod_head, false);
  uint32_t issued = 0;  // loads issued so far (thread 0)
  if (tid == 0) {
    for (int s = 0; s < kStages && prod_head >= 0; ++s) {
      issue_head(sh, p, s, prod_head);
      ++issued;
      prod_item = next_item(p, prod_item + step, step, &prod_head, false);
    }
  }
  int64_t head = -1;
  uint64_t item = next_item(p, blockIdx.x, step, &head, tid == 0);
  uint32_t consumed = 0;
  while (head >= 0) {
    const int stage = static_cast<int>(consumed % kStages);
    const uint32_t parity = (consumed / kStages) & 1u;
    const bool timed_out = !mbar_wait_bounded(&sh.full[stage], parity);
    float4 v[kRowsPerWarp];
    const float4* src = reinterpret_cast<const float4*>(sh.stage[stage]);
#pragma unroll
    for (int j = 0; j < kRowsPerWarp; ++j) v[j] = src[(warp * kRowsPerWarp + j) * 32 + lane];
    ++consumed;

    // Head to stream into this landing buffer once every warp has read it.
    int64_t refill = -1;
    if (tid == 0) {
      refill = prod_head;
      if (prod_head >= 0) {
        ++issued;
        prod_item = next_item(p, prod_item + step, step, &prod_head, false);
      }
    }
    const bool keep_going =
        kProvider ? quantize_provider_head<kMode>(p, sh, v, head, warp, lane, tid, timed_out,
                                                  stage, refill)
                  : quantize_capsule_head<kMode>(p, sh, v, head, warp, lane, tid, timed_out,
                                                 stage, refill);
    if (!keep_going) {
      // A bounded wait expired somewhere in the block (the head functions stop
      // before issuing `refill`).  Report it, then wait, again bounded, for
      // every copy that may still be in flight -- load indices consumed-1 up
      // to the last one issued -- so none lands in this block's shared memory
      // after it exits.  Outputs of this launch are then unspecified.
      if (tid == 0) {
        report(p.status, kStatusWaitTimeout);
        const uint32_t issued_for_real = issued - (refill >= 0 ? 1u : 0u);
        for (uint32_t idx = consumed - 1u; idx < issued_for_real; ++idx) {
          (void)mbar_wait_bounded(&sh.full[idx % kStages], (idx / kStages) & 1u);
        }
      }
      return;
    }
    item = next_item(p, item + step, step, &head, tid == 0);
  }
}

// ---------------------------------------------------------------------------
// Host-side launch helpers.

template <bool kProvider, int kMode>
cudaError_t launch_quantize_t(const QuantizeParams& p, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = sizeof(QuantizeShared);
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, quantize_kernel<kProvider, kMode>, p);
}

template <bool kProvider, int kMode>
cudaError_t prepare_quantize_t(int* blocks_per_sm) {
  auto kernel = quantize_kernel<kProvider, kMode>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(sizeof(QuantizeShared)));
  if (err != cudaSuccess) return err;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kernel, kQThreads,
                                                       sizeof(QuantizeShared));
}

inline cudaError_t prepare_quantize(bool provider, int mode, int* blocks_per_sm) {
  if (provider) {
    if (mode == kFused) return prepare_quantize_t<true, kFused>(blocks_per_sm);
    if (mode == kGivenSmoothing) return prepare_quantize_t<true, kGivenSmoothing>(blocks_per_sm);
    return prepare_quantize_t<true, kSmoothingOnly>(blocks_per_sm);
  }
  if (mode == kFused) return prepare_quantize_t<false, kFused>(blocks_per_sm);
  if (mode == kGivenSmoothing) return prepare_quantize_t<false, kGivenSmoothing>(blocks_per_sm);
  return prepare_quantize_t<false, kSmoothingOnly>(blocks_per_sm);
}

inline cudaError_t launch_quantize(bool provider, int mode, const QuantizeParams& p, int grid,
                                   cudaStream_t stream) {
  if (provider) {
    if (mode == kFused) return launch_quantize_t<true, kFused>(p, grid, stream);
    if (mode == kGivenSmoothing) return launch_quantize_t<true, kGivenSmoothing>(p, grid, stream);
    return launch_quantize_t<true, kSmoothingOnly>(p, grid, stream);
  }
  if (mode == kFused) return launch_quantize_t<false, kFused>(p, grid, stream);
  if (mode == kGivenSmoothing) return launch_quantize_t<false, kGivenSmoothing>(p, grid, stream);
  return launch_quantize_t<false, kSmoothingOnly>(p, grid, stream);
}

}  // namespace gdnsc
