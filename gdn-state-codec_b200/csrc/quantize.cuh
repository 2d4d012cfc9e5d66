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
//    (cp.async.bulk + mbarrier).  A buffer stays valid while its head is
//    processed (the rare exact paths read it by run-time index) and is
//    refilled once every thread has moved on, so kStages - 1 heads are always
//    in flight behind the one being computed.
//  * the smoothing sums run in double (tree order, with a proof-backed check
//    that sends the rare order-sensitive rows to the reference's sequential
//    order); every smoothed value s = R / c is computed correctly rounded from
//    RN(1/c) by two packed fma corrections (div4_exact), so the per-value
//    maxima b are exact without any search; codes come from one multiply by
//    RN(127 / b) and the few elements within the proven error band of a
//    rounding boundary are recomputed with IEEE division.
//  * thread tiles keep the double-precision reduction mostly inside a thread:
//    capsule layout (row sums over values) uses 4 rows x 8 columns per thread,
//    provider layout (column sums over values) 8 rows x 4 columns; both read
//    the landing buffer without bank conflicts.
#pragma once

#include "codec_device.cuh"

namespace gdnsc {

constexpr int kQThreads = 512;
constexpr int kQWarps = kQThreads / 32;      // 16
constexpr int kWarpRows = kKeys / kQWarps;   // 8 rows of a head per warp
constexpr int kStages = 3;                   // TMA landing buffers per CTA

// Codes: t' = RN(s * RN(127 / b)) and the exact t = RN(RN(s / b) * 127) both
// lie within 2^-23 (relative, two roundings each) of s * 127 / b, so
// |t' - t| <= 127 * 2^-22 < 2^-15: a code is decided from t' unless t' lies
// within 2^-13 of a rounding boundary n + 0.5.
constexpr float kAmbiguous = 0.5F - 0x1p-13F;
// Fast-path ranges: a per-value maximum b in [2^-64, 2^100] and smoothing in
// [2^-14, 2^100] keep every element that can be a maximum or have a nonzero
// code (|s| >= b / 254) inside div4_exact's preconditions (|R| >= 2^-102,
// normal quotient).  Smoothing computed here is always >= sqrt(1e-8) = 1e-4.
// Values outside (all-zero or denormal columns, non-finite data, caller-given
// smoothing out of range) take the IEEE path for the affected columns.
constexpr float kFastMin = 0x1p-64F;
constexpr float kFastMax = 0x1p100F;
constexpr float kSmoothMin = 0x1p-14F;

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
  float key_c[kKeys];               // provider: smoothing per key
  float key_y[kKeys];               // provider: RN(1/c) per key
  float col_b[kValues];             // capsule: exact per-value maximum
  float col_km[kValues];            // capsule: RN(127 / b) (0 on the IEEE path)
  uint32_t col_exact[kValues];      // capsule IEEE path: maximum (bits)
  float colbuf[kKeys];              // provider: one column for a sequential re-sum
  float row_c[kQWarps][kWarpRows];  // capsule: smoothing of the warp's rows
  float row_y[kQWarps][kWarpRows];  // capsule: RN(1/c) of the warp's rows
  float row_b[kQWarps][kWarpRows];  // provider: exact per-value maximum
  float row_km[kQWarps][kWarpRows]; // provider: RN(127 / b) (0 on the IEEE path)
  int col_flag[kKeys];
  uint64_t full[kStages];           // one mbarrier per landing buffer
};

// ---------------------------------------------------------------------------
// Small helpers.

__device__ __forceinline__ float4 absmax4v(float4 m, float4 a) {
  return make_float4(fmaxf(m.x, fabsf(a.x)), fmaxf(m.y, fabsf(a.y)), fmaxf(m.z, fabsf(a.z)),
                     fmaxf(m.w, fabsf(a.w)));
}
__device__ __forceinline__ float absmax4(float4 a) {
  return fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w)));
}
__device__ __forceinline__ float comp(const float4& a, int i) {
  return i == 0 ? a.x : (i == 1 ? a.y : (i == 2 ? a.z : a.w));
}
__device__ __forceinline__ double abs_sum4(float4 a) {
  return (static_cast<double>(fabsf(a.x)) + static_cast<double>(fabsf(a.y))) +
         (static_cast<double>(fabsf(a.z)) + static_cast<double>(fabsf(a.w)));
}
__device__ __forceinline__ bool fast_max(float b) { return b >= kFastMin && b <= kFastMax; }
__device__ __forceinline__ bool fast_smoothing(float c) {
  return c >= kSmoothMin && c <= kFastMax;
}

// Approximate codes of four elements from exact s: t = s * km rounded through
// the magic constant; returns the packed int8x4 word and reports whether any
// element lies within the ambiguity band of a rounding boundary.
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
  *amb = !(worst <= kAmbiguous);
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

__device__ __forceinline__ void issue_head(const QuantizeParams& p, float* buffer, uint64_t* bar,
                                           int64_t head) {
  fence_proxy_async();
  mbar_expect_tx(bar, kElements * sizeof(float));
  bulk_load(buffer, p.state + static_cast<uint64_t>(head) * kElements, kElements * sizeof(float),
            bar, evict_first_policy());
}

// ---------------------------------------------------------------------------
// Capsule layout [key, value]: row k = key, column v = value.
//
// Thread tile: lane l = 16g + q (g = l/16, q = l%16) of warp w holds rows
// r_j = 8w + 2j + g (j = 0..3) and, in each row, two 4-column chunks c = 0, 1
// at columns 64c + 4q .. 64c + 4q + 3.  For a fixed (j, c) a half warp reads
// 256 contiguous bytes of one row: conflict-free.  A row is shared by the 16
// lanes of one g (row sums reduce over lane bits 0-3); a column by the two
// lanes of one q (column maxima reduce over lane bit 4, then across warps).

struct CapsuleTile {
  float4 v[4][2];  // [row j][chunk c]: R, then s = R / c
};

__device__ __forceinline__ void load_capsule_tile(const float* stage_f, CapsuleTile& t, int warp,
                                                  int lane) {
  const int g = lane >> 4, q = lane & 15;
  const float4* stage = reinterpret_cast<const float4*>(stage_f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int row = warp * kWarpRows + 2 * j + g;
#pragma unroll
    for (int c = 0; c < 2; ++c) t.v[j][c] = stage[row * 32 + 16 * c + q];
  }
}

template <int kMode>
__device__ __forceinline__ void quantize_capsule_head(const QuantizeParams& p, QuantizeShared& sh,
                                                      CapsuleTile& t, const float* stage,
                                                      int64_t head, int warp, int lane, int tid) {
  const int g = lane >> 4, q = lane & 15;
  const int row_base = warp * kWarpRows;
  // -- smoothing per row -----------------------------------------------------
  bool bad_smoothing = false;
  if (kMode == kGivenSmoothing) {
    if (lane < kWarpRows) {
      const float c = __ldg(p.smoothing_in + head * kKeys + row_base + lane);
      sh.row_c[warp][lane] = c;
      sh.row_y[warp][lane] = __frcp_rn(c);
      bad_smoothing = !fast_smoothing(c);
    }
  } else {
    double part[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) part[j] = abs_sum4(t.v[j][0]) + abs_sum4(t.v[j][1]);
    // Reduce-scatter over the 16 lanes of this g (lane bits 3, 2), then sum
    // over lane bits 1, 0: lanes 4i..4i+3 of the half warp hold row j = i.
    {
      const bool up = (lane & 8) != 0;
      const double s0 = up ? part[0] : part[2], s1 = up ? part[1] : part[3];
      const double k0 = up ? part[2] : part[0], k1 = up ? part[3] : part[1];
      part[0] = k0 + __shfl_xor_sync(0xffffffffu, s0, 8);
      part[1] = k1 + __shfl_xor_sync(0xffffffffu, s1, 8);
    }
    {
      const bool up = (lane & 4) != 0;
      const double s0 = up ? part[0] : part[1];
      const double k0 = up ? part[1] : part[0];
      part[0] = k0 + __shfl_xor_sync(0xffffffffu, s0, 4);
    }
    double sum = part[0] + __shfl_xor_sync(0xffffffffu, part[0], 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    const int my_j = (lane >> 2) & 3;  // this lane group's row r = 8w + 2*my_j + g
    // Rows whose float mean could depend on the summation order are re-summed
    // in the reference's order (capsule.cpp:193-196): value 0..127, read from
    // the landing buffer.  Rare.
    uint32_t flagged =
        __ballot_sync(0xffffffffu, near_float_midpoint(sum * (1.0 / 128.0))) & 0x11111111u;
    while (flagged != 0u) {
      const int owner = __ffs(flagged) - 1;
      flagged &= flagged - 1u;
      const int row = row_base + 2 * ((owner >> 2) & 3) + (owner >> 4);
      const float4 mine = reinterpret_cast<const float4*>(stage)[row * 32 + lane];
      double seq = 0.0;
      for (int src = 0; src < 32; ++src) {
        seq += fabsf(__shfl_sync(0xffffffffu, mine.x, src));
        seq += fabsf(__shfl_sync(0xffffffffu, mine.y, src));
        seq += fabsf(__shfl_sync(0xffffffffu, mine.z, src));
        seq += fabsf(__shfl_sync(0xffffffffu, mine.w, src));
      }
      if ((lane >> 2) == (owner >> 2)) sum = seq;
    }
    const float c = smoothing_from_sum(sum);
    if ((lane & 3) == 0) {
      const int r = 2 * my_j + g;
      sh.row_c[warp][r] = c;
      sh.row_y[warp][r] = __frcp_rn(c);
      p.smoothing[head * kKeys + row_base + r] = c;
    }
  }
  __syncwarp();
  if (kMode == kSmoothingOnly) return;

  // -- exact smoothed values and column maxima ------------------------------------
  float4 pm[2] = {make_float4(0.F, 0.F, 0.F, 0.F), make_float4(0.F, 0.F, 0.F, 0.F)};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float y = sh.row_y[warp][2 * j + g];
    const float nc = -sh.row_c[warp][2 * j + g];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      t.v[j][c] = div4_exact_s(t.v[j][c], y, nc);
      pm[c] = absmax4v(pm[c], t.v[j][c]);
    }
  }
  {
    // Exchange over lane bit 4: afterwards this lane holds the warp maximum
    // of chunk c = g (columns 64g + 4q ..).
    const bool up = (lane & 16) != 0;
    const float4 send = up ? pm[0] : pm[1];
    const float4 keep = up ? pm[1] : pm[0];
    const float4 m = make_float4(fmaxf(keep.x, __shfl_xor_sync(0xffffffffu, send.x, 16)),
                                 fmaxf(keep.y, __shfl_xor_sync(0xffffffffu, send.y, 16)),
                                 fmaxf(keep.z, __shfl_xor_sync(0xffffffffu, send.z, 16)),
                                 fmaxf(keep.w, __shfl_xor_sync(0xffffffffu, send.w, 16)));
    reinterpret_cast<float4*>(sh.col_part[warp])[16 * g + q] = m;
  }
  const bool head_slow = __syncthreads_or(bad_smoothing) != 0;  // B1
  int slow = 0;
  if (tid < kValues) {
    float b = 0.0F;
#pragma unroll
    for (int w = 0; w < kQWarps; ++w) b = fmaxf(b, sh.col_part[w][tid]);
    slow = head_slow || !fast_max(b);
    sh.col_b[tid] = b;
    sh.col_km[tid] = slow ? 0.0F : __fdiv_rn(kQuantMax, b);
    sh.col_exact[tid] = 0u;
    if (!slow) p.scales[head * kValues + tid] = b;
  }
  const bool any_slow = __syncthreads_or(slow) != 0;  // B2

  // -- codes ----------------------------------------------------------------------
  uint32_t amb_mask = 0u;  // bit 2j+c: chunk (j, c) holds an ambiguous element
  int8_t* codes = p.codes + static_cast<uint64_t>(head) * kElements;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const float4 km = reinterpret_cast<const float4*>(sh.col_km)[16 * c + q];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      bool amb;
      const uint32_t word = approx_codes(t.v[j][c], km, &amb);
      st_cs_u32(codes + (row_base + 2 * j + g) * kValues + 64 * c + 4 * q, word);
      amb_mask |= (amb ? 1u : 0u) << (2 * j + c);
    }
  }
  // Elements inside the ambiguity band take the exact code (IEEE division
  // from the landing buffer, exact maximum).
  while (amb_mask != 0u) {
    const int bit = __ffs(amb_mask) - 1;
    amb_mask &= amb_mask - 1u;
    const int r_local = 2 * (bit >> 1) + g, c = bit & 1;
    const float c_r = sh.row_c[warp][r_local];
    const float y_r = sh.row_y[warp][r_local];
    for (int e = 0; e < 4; ++e) {
      const int col = 64 * c + 4 * q + e;
      const float km = sh.col_km[col];
      if (km == 0.0F) continue;  // IEEE-path column, handled below
      const float r = stage[(row_base + r_local) * kValues + col];
      if (approx_ambiguous(div4_exact_s(make_float4(r, 0.F, 0.F, 0.F), y_r, -c_r).x, km)) {
        codes[(row_base + r_local) * kValues + col] = exact_code(__fdiv_rn(r, c_r), sh.col_b[col]);
      }
    }
  }
  if (any_slow) {
    // IEEE path for columns outside the fast ranges (rare; all-zero columns
    // included): exact quotients, an exact maximum across the block, codes.
    for (int j = 0; j < 4; ++j) {
      const int r_local = 2 * j + g;
      for (int c = 0; c < 2; ++c) {
        for (int e = 0; e < 4; ++e) {
          const int col = 64 * c + 4 * q + e;
          if (sh.col_km[col] != 0.0F) continue;
          const float r = stage[(row_base + r_local) * kValues + col];
          if (r != 0.0F) {
            atomicMax(&sh.col_exact[col],
                      __float_as_uint(fabsf(__fdiv_rn(r, sh.row_c[warp][r_local]))));
          }
        }
      }
    }
    __syncthreads();
    if (tid < kValues && sh.col_km[tid] == 0.0F) {
      p.scales[head * kValues + tid] = __uint_as_float(sh.col_exact[tid]);
    }
    for (int j = 0; j < 4; ++j) {
      const int r_local = 2 * j + g;
      for (int c = 0; c < 2; ++c) {
        for (int e = 0; e < 4; ++e) {
          const int col = 64 * c + 4 * q + e;
          if (sh.col_km[col] != 0.0F) continue;
          const float r = stage[(row_base + r_local) * kValues + col];
          codes[(row_base + r_local) * kValues + col] =
              exact_code(r == 0.0F ? 0.0F : __fdiv_rn(r, sh.row_c[warp][r_local]),
                         __uint_as_float(sh.col_exact[col]));
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Provider layout [value, key]: row = value v, column = key k.
// Thread tile: warp w holds rows 8w..8w+7, lane l columns 4l..4l+3 (a warp
// reads one 512-byte row per instruction: conflict-free).

template <int kMode>
__device__ __forceinline__ void quantize_provider_head(const QuantizeParams& p, QuantizeShared& sh,
                                                       float4 (&v)[kWarpRows], const float* stage,
                                                       int64_t head, int warp, int lane,
                                                       int tid) {
  const int row_base = warp * kWarpRows;
  // -- smoothing per key (column): thread-local over 8 rows, then across warps
  if (kMode != kGivenSmoothing) {
    double cs0 = 0.0, cs1 = 0.0, cs2 = 0.0, cs3 = 0.0;
#pragma unroll
    for (int j = 0; j < kWarpRows; ++j) {
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
  __syncthreads();  // B1: column partial sums published
  int flag = 0;
  bool bad_smoothing = false;
  if (tid < kKeys) {
    float c;
    if (kMode == kGivenSmoothing) {
      c = __ldg(p.smoothing_in + head * kKeys + tid);
      bad_smoothing = !fast_smoothing(c);
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
  // B2: smoothing ready; bit 0 = a column needs the sequential re-sum,
  // bit 1 = caller-given smoothing outside the fast range.
  const int b2 = __syncthreads_or(flag | (bad_smoothing ? 2 : 0));
  if (b2 & 1) {  // rare, block-uniform
    for (int k = 0; k < kKeys; ++k) {
      if (!sh.col_flag[k]) continue;
      if (tid < kValues) sh.colbuf[tid] = stage[tid * kKeys + k];
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
  if (kMode == kSmoothingOnly) return;
  const bool head_slow = (b2 & 2) != 0;

  // -- exact smoothed values and row maxima (warp-local) ------------------------------
  const float4 c4 = reinterpret_cast<const float4*>(sh.key_c)[lane];
  const float4 y4 = reinterpret_cast<const float4*>(sh.key_y)[lane];
  const float4 nc4 = make_float4(-c4.x, -c4.y, -c4.z, -c4.w);
  float rm[kWarpRows];
#pragma unroll
  for (int j = 0; j < kWarpRows; ++j) {
    v[j] = div4_exact(v[j], y4, nc4);
    rm[j] = absmax4(v[j]);
  }
  {
    int offset = 16;
#pragma unroll
    for (int half = kWarpRows / 2; half >= 1; half >>= 1, offset >>= 1) {
      const bool up = (lane & offset) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = up ? rm[i] : rm[i + half];
        const float keep = up ? rm[i + half] : rm[i];
        rm[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, offset));
      }
    }
  }
  float b = fmaxf(rm[0], __shfl_xor_sync(0xffffffffu, rm[0], 2));
  b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, 1));
  const int my_row = lane >> 2;  // lanes 4r..4r+3 hold row r
  const bool my_slow = head_slow || !fast_max(b);
  if ((lane & 3) == 0) {
    sh.row_b[warp][my_row] = b;
    sh.row_km[warp][my_row] = my_slow ? 0.0F : __fdiv_rn(kQuantMax, b);
    if (!my_slow) p.scales[head * kValues + row_base + my_row] = b;
  }
  const uint32_t slow_rows = __ballot_sync(0xffffffffu, my_slow && (lane & 3) == 0);
  __syncwarp();

  // -- codes ------------------------------------------------------------------------
  uint32_t amb_rows = 0u;
  int8_t* codes = p.codes + static_cast<uint64_t>(head) * kElements;
#pragma unroll
  for (int j = 0; j < kWarpRows; ++j) {
    const float km = sh.row_km[warp][j];
    bool amb;
    const uint32_t word = approx_codes(v[j], make_float4(km, km, km, km), &amb);
    st_cs_u32(codes + (row_base + j) * kKeys + 4 * lane, word);
    amb_rows |= (amb ? 1u : 0u) << j;
  }
  while (amb_rows != 0u) {
    const int j = __ffs(amb_rows) - 1;
    amb_rows &= amb_rows - 1u;
    const float km = sh.row_km[warp][j];
    if (km == 0.0F) continue;  // IEEE-path row, handled below
    const float4 r4 = reinterpret_cast<const float4*>(stage)[(row_base + j) * 32 + lane];
    const float4 s4 = div4_exact(r4, y4, nc4);
    for (int i = 0; i < 4; ++i) {
      if (approx_ambiguous(comp(s4, i), km)) {
        codes[(row_base + j) * kKeys + 4 * lane + i] =
            exact_code(__fdiv_rn(comp(r4, i), comp(c4, i)), sh.row_b[warp][j]);
      }
    }
  }
  // IEEE path for rows outside the fast ranges (rare; all-zero rows included).
  uint32_t slow_left = slow_rows;
  while (slow_left != 0u) {
    const int owner = __ffs(slow_left) - 1;
    slow_left &= slow_left - 1u;
    const int j = owner >> 2;
    const float4 r4 = reinterpret_cast<const float4*>(stage)[(row_base + j) * 32 + lane];
    float4 s4;
    s4.x = r4.x == 0.0F ? 0.0F : __fdiv_rn(r4.x, c4.x);
    s4.y = r4.y == 0.0F ? 0.0F : __fdiv_rn(r4.y, c4.y);
    s4.z = r4.z == 0.0F ? 0.0F : __fdiv_rn(r4.z, c4.z);
    s4.w = r4.w == 0.0F ? 0.0F : __fdiv_rn(r4.w, c4.w);
    float mx = absmax4(s4);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) p.scales[head * kValues + row_base + j] = mx;
    const uint32_t word = (static_cast<uint32_t>(static_cast<uint8_t>(exact_code(s4.x, mx)))) |
                          (static_cast<uint32_t>(static_cast<uint8_t>(exact_code(s4.y, mx))) << 8) |
                          (static_cast<uint32_t>(static_cast<uint8_t>(exact_code(s4.z, mx))) << 16) |
                          (static_cast<uint32_t>(static_cast<uint8_t>(exact_code(s4.w, mx))) << 24);
    st_cs_u32(codes + (row_base + j) * kKeys + 4 * lane, word);
  }
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
  // both walk the same deterministic item sequence.  Head number n lives in
  // landing buffer n % kStages, whose fill for it has parity (n / kStages) & 1.
  int64_t prod_head = -1;
  uint64_t prod_item = 0;
  uint32_t issued = 0;
  if (tid == 0) {
    prod_item = next_item(p, blockIdx.x, step, &prod_head, false);
    for (int s = 0; s < kStages && prod_head >= 0; ++s) {
      issue_head(p, sh.stage[s], &sh.full[s], prod_head);
      ++issued;
      prod_item = next_item(p, prod_item + step, step, &prod_head, false);
    }
  }
  int64_t head = -1;
  uint64_t item = next_item(p, blockIdx.x, step, &head, tid == 0);
  uint32_t consumed = 0;
  while (head >= 0) {
    const int stage = static_cast<int>(consumed % kStages);
    const bool timed_out = !mbar_wait_bounded(&sh.full[stage], (consumed / kStages) & 1u);
    CapsuleTile ct;
    float4 pv[kWarpRows];
    if (kProvider) {
      const float4* src = reinterpret_cast<const float4*>(sh.stage[stage]);
#pragma unroll
      for (int j = 0; j < kWarpRows; ++j) pv[j] = src[(warp * kWarpRows + j) * 32 + lane];
    } else {
      load_capsule_tile(sh.stage[stage], ct, warp, lane);
    }
    ++consumed;
    // B0: every warp holds its part of this head and has finished the previous
    // one, whose landing buffer now takes the head kStages - 1 ahead.
    if (__syncthreads_or(timed_out) != 0) {
      // A bounded wait expired: report it, then wait, again bounded, for every
      // copy that may still be in flight (fills consumed-1 .. issued-1) so that
      // none lands in this block's shared memory after it exits.  Outputs of
      // this launch are then unspecified.
      if (tid == 0) {
        report(p.status, kStatusWaitTimeout);
        for (uint32_t n = consumed - 1u; n < issued; ++n) {
          (void)mbar_wait_bounded(&sh.full[n % kStages], (n / kStages) & 1u);
        }
      }
      return;
    }
    if (tid == 0 && consumed >= 2 && prod_head >= 0) {
      const int prev = static_cast<int>((consumed - 2) % kStages);
      issue_head(p, sh.stage[prev], &sh.full[prev], prod_head);
      ++issued;
      prod_item = next_item(p, prod_item + step, step, &prod_head, false);
    }
    if (kProvider) {
      quantize_provider_head<kMode>(p, sh, pv, sh.stage[stage], head, warp, lane, tid);
    } else {
      quantize_capsule_head<kMode>(p, sh, ct, sh.stage[stage], head, warp, lane, tid);
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
