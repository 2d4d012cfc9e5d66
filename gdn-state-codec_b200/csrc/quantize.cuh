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
//  * persistent 256-thread CTAs, two per SM.  Each walks its own sequence of
//    heads with one 64 KiB shared-memory landing buffer filled by a single TMA
//    bulk copy (cp.async.bulk + mbarrier, normal L2 policy); as soon as the
//    CTA holds a head in registers the buffer takes its next head.  The two
//    CTAs of an SM drift out of phase, so one's barriers and reductions
//    overlap the other's arithmetic, and two heads are in flight per SM.
//  * the rare elements next to a rounding boundary owe exact codes, written
//    after the launch's last head (owed exact codes, below).
//  * the smoothing sums run in double (tree order, with a proof-backed check
//    that sends the rare order-sensitive rows to the reference's sequential
//    order); every smoothed value s = R / c is computed correctly rounded from
//    the two-term reciprocal of c by one packed fma correction (div4_exact),
//    so the per-value maxima b are exact without any search; codes come from
//    one fma of s and RN(127 / b) with the rounding constant, and the few
//    elements within the proven error band of a rounding boundary take the
//    exact code by IEEE division (out of line).
//  * thread tiles (64 elements per thread) keep the double-precision
//    reduction mostly inside a thread: capsule layout (row sums over values)
//    uses 4 rows x 16 columns, provider layout (column sums over values)
//    16 rows x 4 columns; both read the landing buffer without bank conflicts.
#pragma once

#include "codec_device.cuh"

namespace gdnsc {

constexpr int kQThreads = 256;
constexpr int kQBlocksPerSm = 2;                    // independent head streams per SM
constexpr int kGroupWarps = kQThreads / 32;         // 8
constexpr int kWarpRows = kKeys / kGroupWarps;      // 16 rows of a head per warp

// Codes: with km = RN(127 / b) = (127 / b)(1 + e1), the exact product
// s * km = T (1 + e1) and the reference's t = RN(RN(s / b) * 127) =
// T (1 + e3)(1 + e4) of T = 127 s / b, |T| <= 127, |e_i| <= u = 2^-24, differ
// by at most 127 (3u + u^2) < 381.01 u.  One fma forms u' = RN(s km + M) with
// M = 1.5 * 2^23, i.e. M + n for the integer n nearest to s km (the low byte
// of u' is n as int8), and a second gives d = RN(s km - n) within u / 4 of
// s km - n (M - u' = -n is exact).  If |d| <= 0.5 - 384 u, then
// |t - n| <= 0.5 - 384 u + u / 4 + 381.01 u < 0.5 and the reference's lround
// gives n as well; every other element (ties of t included) takes the exact
// code.  tests/division_check.c checks the rule on the CPU.
constexpr float kAmbiguous = 0.5F - 0x1.8p-16F;  // 0.5 - 384 * 2^-24
// Fast-path ranges: a per-value maximum b in [2^-64, 2^100] and smoothing in
// [2^-14, 2^100] keep every element that can be a maximum or have a nonzero
// code (|s| >= b / 254) inside div4_exact's preconditions (|R| >= 2^-102,
// normal quotient).  Smoothing computed here is always >= sqrt(1e-8) = 1e-4.
// Values outside (all-zero or denormal columns, non-finite data, caller-given
// smoothing out of range) take the IEEE path for the affected values.
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
  uint64_t wait_limit_ns = kWaitLimitNs;  // limit of every bounded wait
  // Test support (quantize_wait_selftest_v1): arm the landing barrier for
  // the first head's bytes but issue no copy at all, so the first wait runs
  // out with nothing in flight.
  uint32_t arm_only = 0u;
};

// Shared state of one CTA.
struct __align__(128) QuantizeGroupShared {
  float stage[kElements];  // TMA landing buffer (64 KiB)
  union {
    float col_part[kGroupWarps][kValues];  // capsule: per-warp column maxima
    double col_dsum[kGroupWarps][kKeys];   // provider: per-warp column sums
  };
  float key_c[kKeys];                  // smoothing per key
  float key_y[kKeys];                  // RN(1/c) per key
  float key_yl[kKeys];                 // RN((1 - c y) y): second reciprocal term
  float val_b[kValues];                // exact per-value maximum
  float val_km[kValues];               // RN(127 / b), 0 on the IEEE path
  uint32_t val_exact[kValues];         // IEEE path: maximum (bits)
  float colbuf[kKeys];                 // provider: one column for a sequential re-sum
  int col_flag[kKeys];
  uint64_t owed[kQThreads][2];         // per thread: owed (head, mask) pairs, 0 = free
  uint64_t full;                       // landing buffer holds the next head (TMA bytes)
  uint64_t empty;                      // provider: every warp has copied the head
  int readers;                         // capsule: warps that have copied the current head
};

// Block-wide barriers (the CTA is one head stream).
__device__ __forceinline__ void group_sync(int) { __syncthreads(); }
__device__ __forceinline__ bool group_sync_or(int, bool pred) { return __syncthreads_or(pred) != 0; }

// ---------------------------------------------------------------------------
// Small helpers.

__device__ __forceinline__ double abs_sum4(float4 a) {
  return (static_cast<double>(fabsf(a.x)) + static_cast<double>(fabsf(a.y))) +
         (static_cast<double>(fabsf(a.z)) + static_cast<double>(fabsf(a.w)));
}
__device__ __forceinline__ float4 absmax4x4(float4 a, float4 b, float4 c, float4 d) {
  return make_float4(fmaxf(fmaxf(fabsf(a.x), fabsf(b.x)), fmaxf(fabsf(c.x), fabsf(d.x))),
                     fmaxf(fmaxf(fabsf(a.y), fabsf(b.y)), fmaxf(fabsf(c.y), fabsf(d.y))),
                     fmaxf(fmaxf(fabsf(a.z), fabsf(b.z)), fmaxf(fabsf(c.z), fabsf(d.z))),
                     fmaxf(fmaxf(fabsf(a.w), fabsf(b.w)), fmaxf(fabsf(c.w), fabsf(d.w))));
}
__device__ __forceinline__ float absmax4(float4 a) {
  return fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w)));
}
__device__ __forceinline__ float4 fmax4(float4 a, float4 b) {
  return make_float4(fmaxf(a.x, b.x), fmaxf(a.y, b.y), fmaxf(a.z, b.z), fmaxf(a.w, b.w));
}
__device__ __forceinline__ float4 shfl_xor4(float4 v, int offset) {
  return make_float4(__shfl_xor_sync(0xffffffffu, v.x, offset),
                     __shfl_xor_sync(0xffffffffu, v.y, offset),
                     __shfl_xor_sync(0xffffffffu, v.z, offset),
                     __shfl_xor_sync(0xffffffffu, v.w, offset));
}
__device__ __forceinline__ bool fast_max(float b) { return b >= kFastMin && b <= kFastMax; }
__device__ __forceinline__ bool fast_smoothing(float c) {
  return c >= kSmoothMin && c <= kFastMax;
}

// Approximate codes of four elements from exact s: t = s * km rounded through
// the magic constant; returns the packed int8x4 word and reports whether any
// element lies within the ambiguity band of a rounding boundary.
__device__ __forceinline__ uint32_t approx_codes(float4 s, float4 km, bool* amb) {
  const f2 s01 = pack2(s.x, s.y), s23 = pack2(s.z, s.w);
  const f2 k01 = pack2(km.x, km.y), k23 = pack2(km.z, km.w);
  const f2 magic = pack2(kRoundMagic, kRoundMagic);
  const f2 u01 = fma2(s01, k01, magic);
  const f2 u23 = fma2(s23, k23, magic);
  const f2 d01 = fma2(s01, k01, sub2(magic, u01));
  const f2 d23 = fma2(s23, k23, sub2(magic, u23));
  const float worst = fmaxf(fmaxf(fabsf(lo2(d01)), fabsf(hi2(d01))),
                            fmaxf(fabsf(lo2(d23)), fabsf(hi2(d23))));
  *amb = !(worst <= kAmbiguous);
  const uint32_t w01 = __byte_perm(static_cast<uint32_t>(u01), static_cast<uint32_t>(u01 >> 32), 0x0040);
  const uint32_t w23 = __byte_perm(static_cast<uint32_t>(u23), static_cast<uint32_t>(u23 >> 32), 0x0040);
  return __byte_perm(w01, w23, 0x5410);
}

__device__ __forceinline__ bool approx_ambiguous(float s, float km) {
  const float u = __fmaf_rn(s, km, kRoundMagic);
  const float d = __fmaf_rn(s, km, __fsub_rn(kRoundMagic, u));
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

// The head's copy keeps the normal L2 policy, not evict-first: the rare
// exact-code and re-sum paths re-read a few rows of the head from global
// memory right after the head is consumed, and with evict-first those reads
// went to DRAM (0.850 -> 0.81-0.84 ms capsule, 0.900 -> 0.861 ms provider at
// 61,440 heads, same outputs).
__device__ __forceinline__ void issue_head(const QuantizeParams& p, QuantizeGroupShared& gs,
                                           int64_t head) {
  fence_proxy_async();
  if (p.arm_only != 0u) return;  // test support: only the first head is armed
  mbar_expect_tx(&gs.full, kElements * sizeof(float));
  bulk_load(gs.stage, p.state + static_cast<uint64_t>(head) * kElements, kElements * sizeof(float),
            &gs.full, evict_normal_policy());
}

__device__ __forceinline__ float state_at(const QuantizeParams& p, int64_t head, int row, int col) {
  return __ldg(p.state + static_cast<uint64_t>(head) * kElements + row * 128 + col);
}

// ---------------------------------------------------------------------------
// Cold paths, kept out of line so the hot per-head code stays compact (they
// run for a small fraction of heads and re-read their inputs from global
// memory instead of holding extra registers).

// Sequential re-sum, in the reference's order (capsule.cpp:193-196: value
// 0..127), of the capsule rows whose double mean lies near a float rounding
// midpoint.  `flagged` has one bit per owning lane pair (even lanes); lanes
// of a flagged pair get the sequential sum, the others keep `sum`.
__device__ __noinline__ double resum_capsule_rows(const float* head_state, int row_base,
                                                  int lane, uint32_t flagged, double sum) {
  while (flagged != 0u) {
    const int owner = __ffs(flagged) - 1;
    flagged &= flagged - 1u;
    const int row = row_base + 4 * ((owner >> 1) & 3) + (owner >> 3);
    const float4 mine = __ldg(reinterpret_cast<const float4*>(head_state + row * 128) + lane);
    double seq = 0.0;
    for (int src = 0; src < 32; ++src) {
      seq += fabsf(__shfl_sync(0xffffffffu, mine.x, src));
      seq += fabsf(__shfl_sync(0xffffffffu, mine.y, src));
      seq += fabsf(__shfl_sync(0xffffffffu, mine.z, src));
      seq += fabsf(__shfl_sync(0xffffffffu, mine.w, src));
    }
    if ((lane >> 1) == (owner >> 1)) sum = seq;
  }
  return sum;
}

// Exact codes for a capsule thread's 4-element chunks flagged in `mask` (bit
// 4c + j: row 16w + 4j + g, columns 32c + 4q ..): s = R / c by IEEE division
// (equal to the kernel's exact quotient), then the reference's code.  Values
// on the IEEE path (km == 0) are left to slow_capsule_values.
__device__ __noinline__ void patch_capsule_codes(const float* head_state, int8_t* codes,
                                                 const float* key_c, const float* val_b,
                                                 const float* val_km, int row_base, int g, int q,
                                                 uint32_t mask) {
  while (mask != 0u) {
    const int bit = __ffs(mask) - 1;
    mask &= mask - 1u;
    const int r = row_base + 4 * (bit & 3) + g;
    const float c = key_c[r];
    const int col0 = 32 * (bit >> 2) + 4 * q;
    const float4 r4 = __ldg(reinterpret_cast<const float4*>(head_state + r * 128 + col0));
    const float rv[4] = {r4.x, r4.y, r4.z, r4.w};
    for (int e = 0; e < 4; ++e) {
      const int col = col0 + e;
      const float km = val_km[col];
      if (km == 0.0F) continue;
      const float s = __fdiv_rn(rv[e], c);
      if (approx_ambiguous(s, km)) codes[r * kValues + col] = exact_code(s, val_b[col]);
    }
  }
}

// IEEE path of a capsule head for values outside the fast ranges: exact
// quotients from the input, exact maxima across the block, then codes and
// scales.  Called by every thread of the block (contains block barriers).
__device__ __noinline__ void slow_capsule_values(const float* head_state, int8_t* codes,
                                                 float* scales, const float* key_c,
                                                 const float* val_km, uint32_t* val_exact,
                                                 int row_base, int g, int q, int gtid) {
  for (int j = 0; j < 4; ++j) {
    const int r = row_base + 4 * j + g;
    for (int c = 0; c < 4; ++c) {
      for (int e = 0; e < 4; ++e) {
        const int col = 32 * c + 4 * q + e;
        if (val_km[col] != 0.0F) continue;
        const float x = __ldg(head_state + r * 128 + col);
        if (x != 0.0F) atomicMax(&val_exact[col], __float_as_uint(fabsf(__fdiv_rn(x, key_c[r]))));
      }
    }
  }
  __syncthreads();
  if (gtid < kValues && val_km[gtid] == 0.0F) scales[gtid] = __uint_as_float(val_exact[gtid]);
  for (int j = 0; j < 4; ++j) {
    const int r = row_base + 4 * j + g;
    for (int c = 0; c < 4; ++c) {
      for (int e = 0; e < 4; ++e) {
        const int col = 32 * c + 4 * q + e;
        if (val_km[col] != 0.0F) continue;
        const float x = __ldg(head_state + r * 128 + col);
        codes[r * kValues + col] =
            exact_code(x == 0.0F ? 0.0F : __fdiv_rn(x, key_c[r]), __uint_as_float(val_exact[col]));
      }
    }
  }
}

// Provider counterpart of patch_capsule_codes: rows v = row_base + j flagged
// in `mask`, this lane's keys 4l .. 4l + 3.
__device__ __noinline__ void patch_provider_codes(const float* head_state, int8_t* codes,
                                                  const float* key_c, const float* val_b,
                                                  const float* val_km, int row_base, int lane,
                                                  uint32_t mask) {
  while (mask != 0u) {
    const int j = __ffs(mask) - 1;
    mask &= mask - 1u;
    const int v = row_base + j;
    const float km = val_km[v];
    if (km == 0.0F) continue;
    const float4 r4 = __ldg(reinterpret_cast<const float4*>(head_state + v * 128) + lane);
    const float rv[4] = {r4.x, r4.y, r4.z, r4.w};
    for (int e = 0; e < 4; ++e) {
      const int k = 4 * lane + e;
      const float s = __fdiv_rn(rv[e], key_c[k]);
      if (approx_ambiguous(s, km)) codes[v * kKeys + k] = exact_code(s, val_b[v]);
    }
  }
}

// Provider IEEE path for the value rows in `slow_rows` (bit 2j: row
// row_base + j): exact quotients, the row maximum across the warp, codes.
__device__ __noinline__ void slow_provider_rows(const float* head_state, int8_t* codes,
                                                float* scales, float4 c4, int row_base, int lane,
                                                uint32_t slow_rows) {
  while (slow_rows != 0u) {
    const int owner = __ffs(slow_rows) - 1;
    slow_rows &= slow_rows - 1u;
    const int j = owner >> 1;
    const float4 r4 = __ldg(reinterpret_cast<const float4*>(head_state + (row_base + j) * 128) + lane);
    float4 s4;
    s4.x = r4.x == 0.0F ? 0.0F : __fdiv_rn(r4.x, c4.x);
    s4.y = r4.y == 0.0F ? 0.0F : __fdiv_rn(r4.y, c4.y);
    s4.z = r4.z == 0.0F ? 0.0F : __fdiv_rn(r4.z, c4.z);
    s4.w = r4.w == 0.0F ? 0.0F : __fdiv_rn(r4.w, c4.w);
    float mx = absmax4(s4);
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) scales[row_base + j] = mx;
    const uint32_t word = (static_cast<uint32_t>(static_cast<uint8_t>(exact_code(s4.x, mx)))) |
                          (static_cast<uint32_t>(static_cast<uint8_t>(exact_code(s4.y, mx))) << 8) |
                          (static_cast<uint32_t>(static_cast<uint8_t>(exact_code(s4.z, mx))) << 16) |
                          (static_cast<uint32_t>(static_cast<uint8_t>(exact_code(s4.w, mx))) << 24);
    st_cs_u32(codes + (row_base + j) * kKeys + 4 * lane, word);
  }
}

// ---------------------------------------------------------------------------
// Capsule layout [key, value]: row k = key, column v = value.
//
// Thread tile: lane l = 8g + q (g = l/8, q = l%8) of group warp w holds rows
// r_j = 16w + 4j + g (j = 0..3) and, in each row, four 4-column chunks
// c = 0..3 at columns 32c + 4q .. 32c + 4q + 3.  For a fixed (j, c) a quarter
// warp reads 128 contiguous bytes of one row: conflict-free.  A row is shared
// by the 8 lanes of one g (row sums reduce over lane bits 0-2); a column by
// the 4 lanes of one q (column maxima reduce over lane bits 3-4, then across
// the group's warps).

struct CapsuleTile {
  float4 v[4][4];  // [row j][chunk c]: R, then s = R / c
};

template <int kMode>
__device__ __forceinline__ bool quantize_capsule_head(const QuantizeParams& p,
                                                      QuantizeGroupShared& gs, CapsuleTile& t,
                                                      int64_t head, int group, int warp, int lane,
                                                      int gtid, bool timed_out,
                                                      uint32_t& amb_out) {
  const int g = lane >> 3, q = lane & 7;
  const int row_base = warp * kWarpRows;
  // -- smoothing per row -----------------------------------------------------
  if (kMode == kGivenSmoothing) {
    if (lane < kWarpRows) {
      const float c = __ldg(p.smoothing_in + head * kKeys + row_base + lane);
      gs.key_c[row_base + lane] = c;
      const float y = __frcp_rn(c);
      gs.key_y[row_base + lane] = y;
      gs.key_yl[row_base + lane] = recip_lo(c, y);
    }
  } else {
    double part[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      part[j] = (abs_sum4(t.v[j][0]) + abs_sum4(t.v[j][1])) +
                (abs_sum4(t.v[j][2]) + abs_sum4(t.v[j][3]));
    }
    // Reduce-scatter over the 8 lanes of this g (lane bits 2, 1), then sum
    // over lane bit 0: lanes 2i, 2i+1 of the group of 8 hold row j = i.
    {
      const bool up = (lane & 4) != 0;
      const double s0 = up ? part[0] : part[2], s1 = up ? part[1] : part[3];
      const double k0 = up ? part[2] : part[0], k1 = up ? part[3] : part[1];
      part[0] = k0 + __shfl_xor_sync(0xffffffffu, s0, 4);
      part[1] = k1 + __shfl_xor_sync(0xffffffffu, s1, 4);
    }
    {
      const bool up = (lane & 2) != 0;
      const double s0 = up ? part[0] : part[1];
      const double k0 = up ? part[1] : part[0];
      part[0] = k0 + __shfl_xor_sync(0xffffffffu, s0, 2);
    }
    double sum = part[0] + __shfl_xor_sync(0xffffffffu, part[0], 1);
    const int my_j = (lane >> 1) & 3;  // this lane pair's row r = 16w + 4*my_j + g
    // Rows whose float mean could depend on the summation order are re-summed
    // in the reference's order.  Rare.
    const uint32_t flagged =
        __ballot_sync(0xffffffffu, near_float_midpoint(sum * (1.0 / 128.0))) & 0x55555555u;
    if (flagged != 0u) {
      sum = resum_capsule_rows(p.state + static_cast<uint64_t>(head) * kElements, row_base, lane,
                               flagged, sum);
    }
    const float c = smoothing_from_sum(sum);
    if ((lane & 1) == 0) {
      const int r = row_base + 4 * my_j + g;
      gs.key_c[r] = c;
      const float y = __frcp_rn(c);
      gs.key_y[r] = y;
      gs.key_yl[r] = recip_lo(c, y);
      p.smoothing[head * kKeys + r] = c;
    }
  }
  __syncwarp();
  if (kMode == kSmoothingOnly) return group_sync_or(group, timed_out);

  // -- exact smoothed values and column maxima ------------------------------------
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = row_base + 4 * j + g;
    const float y = gs.key_y[r];
    const float yl = gs.key_yl[r];
    const float nc = -gs.key_c[r];
#pragma unroll
    for (int c = 0; c < 4; ++c) t.v[j][c] = div4_exact_s(t.v[j][c], y, yl, nc);
  }
  float4 pm[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) pm[c] = absmax4x4(t.v[0][c], t.v[1][c], t.v[2][c], t.v[3][c]);
  // Reduce-scatter over lane bits 4, 3: afterwards this lane holds the warp
  // maximum of chunk c = g (columns 32g + 4q ..).
  float4 red[2];
  {
    const bool up = (lane & 16) != 0;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float4 send = up ? pm[i] : pm[i + 2];
      const float4 keep = up ? pm[i + 2] : pm[i];
      red[i] = fmax4(keep, shfl_xor4(send, 16));
    }
  }
  {
    const bool up = (lane & 8) != 0;
    const float4 send = up ? red[0] : red[1];
    const float4 keep = up ? red[1] : red[0];
    reinterpret_cast<float4*>(gs.col_part[warp])[8 * g + q] = fmax4(keep, shfl_xor4(send, 8));
  }
  // B1: column partial maxima and smoothing published; a bounded wait that
  // expired anywhere in the block ends the launch (uniform result).
  if (group_sync_or(group, timed_out)) return true;
  bool slow = false;
  if (gtid < kValues) {
    // Caller-given smoothing out of the fast range sends the whole head to
    // the IEEE path; each of these warps checks all 128 keys itself, so no
    // barrier result has to stay live into this branch.
    bool head_slow = false;
    if (kMode == kGivenSmoothing) {
      const float4 c4 = reinterpret_cast<const float4*>(gs.key_c)[lane];
      head_slow = __any_sync(0xffffffffu, !(fast_smoothing(c4.x) && fast_smoothing(c4.y) &&
                                            fast_smoothing(c4.z) && fast_smoothing(c4.w)));
    }
    float b = 0.0F;
#pragma unroll
    for (int w = 0; w < kGroupWarps; ++w) b = fmaxf(b, gs.col_part[w][gtid]);
    slow = head_slow || !fast_max(b);
    gs.val_b[gtid] = b;
    gs.val_km[gtid] = slow ? 0.0F : __fdiv_rn(kQuantMax, b);
    gs.val_exact[gtid] = 0u;
    if (!slow) p.scales[head * kValues + gtid] = b;
  }
  const bool any_slow = group_sync_or(group, slow);  // B2

  // -- codes ----------------------------------------------------------------------
  int8_t* codes = p.codes + static_cast<uint64_t>(head) * kElements;
  uint32_t amb_mask = 0u;  // bit 4c + j: chunk (j, c) holds an element near a boundary
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 km = reinterpret_cast<const float4*>(gs.val_km)[8 * c + q];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      bool amb;
      const uint32_t word = approx_codes(t.v[j][c], km, &amb);
      st_cs_u32(codes + (row_base + 4 * j + g) * kValues + 32 * c + 4 * q, word);
      amb_mask |= (amb ? 1u : 0u) << (4 * c + j);
    }
  }
  const float* head_state = p.state + static_cast<uint64_t>(head) * kElements;
  // Rare: chunks near a rounding boundary owe exact codes; quantize_kernel
  // writes them after its last head (pay_late), off this head's critical path.
  amb_out = amb_mask;
  if (any_slow) {  // rare and block-uniform: values outside the fast ranges
    slow_capsule_values(head_state, codes, p.scales + head * kValues, gs.key_c, gs.val_km,
                        gs.val_exact, row_base, g, q, gtid);
  }
  return false;
}

// ---------------------------------------------------------------------------
// Provider layout [value, key]: row = value v, column = key k.
// Thread tile: group warp w holds rows 16w..16w+15, lane l columns 4l..4l+3
// (a warp reads one 512-byte row per instruction: conflict-free).

template <int kMode>
__device__ __forceinline__ bool quantize_provider_head(const QuantizeParams& p,
                                                       QuantizeGroupShared& gs,
                                                       float4 (&v)[kWarpRows], int64_t head,
                                                       int group, int warp, int lane, int gtid,
                                                       bool timed_out, uint32_t& amb_out) {
  const int row_base = warp * kWarpRows;
  // -- smoothing per key (column): thread-local over 16 rows, then across warps
  if (kMode != kGivenSmoothing) {
    double cs0 = 0.0, cs1 = 0.0, cs2 = 0.0, cs3 = 0.0;
#pragma unroll
    for (int j = 0; j < kWarpRows; ++j) {
      cs0 += fabsf(v[j].x);
      cs1 += fabsf(v[j].y);
      cs2 += fabsf(v[j].z);
      cs3 += fabsf(v[j].w);
    }
    double* dst = &gs.col_dsum[warp][4 * lane];
    dst[0] = cs0;
    dst[1] = cs1;
    dst[2] = cs2;
    dst[3] = cs3;
  }
  // B1: column partial sums published; a bounded wait that expired anywhere
  // in the block ends the launch (uniform result).
  if (group_sync_or(group, timed_out)) return true;
  int flag = 0;
  bool bad_smoothing = false;
  if (gtid < kKeys) {
    float c;
    if (kMode == kGivenSmoothing) {
      c = __ldg(p.smoothing_in + head * kKeys + gtid);
      bad_smoothing = !fast_smoothing(c);
    } else {
      double sum = 0.0;
#pragma unroll
      for (int w = 0; w < kGroupWarps; ++w) sum += gs.col_dsum[w][gtid];
      flag = near_float_midpoint(sum * (1.0 / 128.0));
      c = smoothing_from_sum(sum);
      if (!flag) p.smoothing[head * kKeys + gtid] = c;
    }
    gs.key_c[gtid] = c;
    const float y = __frcp_rn(c);
    gs.key_y[gtid] = y;
    gs.key_yl[gtid] = recip_lo(c, y);
    gs.col_flag[gtid] = flag;
  }
  // B2: smoothing ready.  With computed smoothing it also tells whether a
  // column needs the sequential re-sum; with caller-given smoothing, whether a
  // value left the fast range.
  const bool b2 = group_sync_or(group, kMode == kGivenSmoothing ? bad_smoothing : flag != 0);
  const bool any_flag = kMode != kGivenSmoothing && b2;
  const bool head_slow = kMode == kGivenSmoothing && b2;
  if (any_flag) {  // rare, group-uniform
    for (int k = 0; k < kKeys; ++k) {
      if (!gs.col_flag[k]) continue;
      if (gtid < kValues) gs.colbuf[gtid] = state_at(p, head, gtid, k);
      group_sync(group);
      if (gtid == 0) {
        double seq = 0.0;  // capsule.cpp:193-196 order: value 0..127
        for (int r = 0; r < kValues; ++r) seq += fabsf(gs.colbuf[r]);
        const float c = smoothing_from_sum(seq);
        gs.key_c[k] = c;
        const float y = __frcp_rn(c);
        gs.key_y[k] = y;
        gs.key_yl[k] = recip_lo(c, y);
        p.smoothing[head * kKeys + k] = c;
      }
      group_sync(group);
    }
  }
  if (kMode == kSmoothingOnly) return false;

  // -- exact smoothed values and row maxima (warp-local) ------------------------------
  const float4 c4 = reinterpret_cast<const float4*>(gs.key_c)[lane];
  const float4 y4 = reinterpret_cast<const float4*>(gs.key_y)[lane];
  const float4 yl4 = reinterpret_cast<const float4*>(gs.key_yl)[lane];
  const float4 nc4 = make_float4(-c4.x, -c4.y, -c4.z, -c4.w);
  float rm[kWarpRows];
#pragma unroll
  for (int j = 0; j < kWarpRows; ++j) {
    v[j] = div4_exact(v[j], y4, yl4, nc4);
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
  const float b = fmaxf(rm[0], __shfl_xor_sync(0xffffffffu, rm[0], 1));
  const int my_row = lane >> 1;  // lanes 2r, 2r+1 hold row r
  const bool my_slow = head_slow || !fast_max(b);
  const int vrow = row_base + my_row;
  if ((lane & 1) == 0) {
    gs.val_b[vrow] = b;
    gs.val_km[vrow] = my_slow ? 0.0F : __fdiv_rn(kQuantMax, b);
    if (!my_slow) p.scales[head * kValues + vrow] = b;
  }
  const uint32_t slow_rows = __ballot_sync(0xffffffffu, my_slow && (lane & 1) == 0);
  __syncwarp();

  // -- codes ------------------------------------------------------------------------
  int8_t* codes = p.codes + static_cast<uint64_t>(head) * kElements;
  uint32_t amb_rows = 0u;
#pragma unroll
  for (int j = 0; j < kWarpRows; ++j) {
    const float km = gs.val_km[row_base + j];
    bool amb;
    const uint32_t word = approx_codes(v[j], make_float4(km, km, km, km), &amb);
    st_cs_u32(codes + (row_base + j) * kKeys + 4 * lane, word);
    amb_rows |= (amb ? 1u : 0u) << j;
  }
  const float* head_state = p.state + static_cast<uint64_t>(head) * kElements;
  // Rare: rows near a rounding boundary owe exact codes; quantize_kernel
  // writes them after its last head (pay_late), off this head's critical path.
  amb_out = amb_rows;
  // IEEE path for rows outside the fast ranges (rare; all-zero rows included).
  if (slow_rows != 0u) {
    slow_provider_rows(head_state, codes, p.scales + head * kValues, c4, row_base, lane,
                       slow_rows);
  }
  return false;
}

// ---------------------------------------------------------------------------
// Owed exact codes.  A thread that flags a chunk (capsule) or row (provider)
// near a rounding boundary records (head, mask) and writes the exact codes
// after the launch's last head, so the IEEE divisions and the re-read of the
// rows no longer hold its warp back from the next head's block barriers
// (0.812 -> 0.762 ms at 61,440 capsule heads, 0.863 -> 0.814 ms provider).
// The late pass (pay_late) uses global memory only: the input rows, and the
// smoothing and scales this launch wrote (or the caller's smoothing), visible
// after the kernel's final block barrier.  It writes the reference's exact
// code, clamp(lround(RN(RN(R / c) / b) * 127)), which equals the code already
// stored for every element that is not ambiguous and is the IEEE path's own
// formula, so it rewrites whole chunks without testing them again.  A thread
// with more than two flagged heads patches the extra ones at once from the
// head's shared arrays (pay_now, patch_*_codes).

__device__ __noinline__ void late_capsule_codes(const float* head_state, const float* smoothing,
                                                const float* scales, int8_t* codes, int row_base,
                                                int g, int q, uint32_t mask) {
  while (mask != 0u) {
    const int bit = __ffs(mask) - 1;
    mask &= mask - 1u;
    const int r = row_base + 4 * (bit & 3) + g;
    const float c = smoothing[r];
    const int col0 = 32 * (bit >> 2) + 4 * q;
    const float4 r4 = __ldg(reinterpret_cast<const float4*>(head_state + r * 128 + col0));
    const float rv[4] = {r4.x, r4.y, r4.z, r4.w};
    for (int e = 0; e < 4; ++e) {
      const float s = rv[e] == 0.0F ? 0.0F : __fdiv_rn(rv[e], c);
      codes[r * kValues + col0 + e] = exact_code(s, scales[col0 + e]);
    }
  }
}

__device__ __noinline__ void late_provider_codes(const float* head_state, const float* smoothing,
                                                 const float* scales, int8_t* codes, int row_base,
                                                 int lane, uint32_t mask) {
  const float4 c4 = *reinterpret_cast<const float4*>(smoothing + 4 * lane);
  const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
  while (mask != 0u) {
    const int j = __ffs(mask) - 1;
    mask &= mask - 1u;
    const int v = row_base + j;
    const float b = scales[v];
    const float4 r4 = __ldg(reinterpret_cast<const float4*>(head_state + v * 128) + lane);
    const float rv[4] = {r4.x, r4.y, r4.z, r4.w};
    for (int e = 0; e < 4; ++e) {
      const float s = rv[e] == 0.0F ? 0.0F : __fdiv_rn(rv[e], cv[e]);
      codes[v * kKeys + 4 * lane + e] = exact_code(s, b);
    }
  }
}

template <bool kProvider, int kMode>
__device__ __forceinline__ void pay_late(const QuantizeParams& p, int64_t head, int warp,
                                         int lane, uint32_t mask) {
  const uint64_t h = static_cast<uint64_t>(head);
  const float* smoothing = (kMode == kGivenSmoothing ? p.smoothing_in : p.smoothing) + h * kKeys;
  if (kProvider) {
    late_provider_codes(p.state + h * kElements, smoothing, p.scales + h * kValues,
                        p.codes + h * kElements, warp * kWarpRows, lane, mask);
  } else {
    late_capsule_codes(p.state + h * kElements, smoothing, p.scales + h * kValues,
                       p.codes + h * kElements, warp * kWarpRows, lane >> 3, lane & 7, mask);
  }
}

template <bool kProvider>
__device__ __forceinline__ void pay_now(const QuantizeParams& p, const QuantizeGroupShared& gs,
                                        int64_t head, int warp, int lane, uint32_t mask) {
  const float* head_state = p.state + static_cast<uint64_t>(head) * kElements;
  int8_t* codes = p.codes + static_cast<uint64_t>(head) * kElements;
  if (kProvider) {
    patch_provider_codes(head_state, codes, gs.key_c, gs.val_b, gs.val_km, warp * kWarpRows,
                         lane, mask);
  } else {
    patch_capsule_codes(head_state, codes, gs.key_c, gs.val_b, gs.val_km, warp * kWarpRows,
                        lane >> 3, lane & 7, mask);
  }
}

template <bool kProvider, int kMode>
__global__ void __launch_bounds__(kQThreads, kQBlocksPerSm) quantize_kernel(QuantizeParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  QuantizeGroupShared& gs = *reinterpret_cast<QuantizeGroupShared*>(smem_raw);
  const int group = 0;
  const int gtid = threadIdx.x;
  const int warp = gtid >> 5;
  const int lane = gtid & 31;
  // Block b takes items b, b + G, b + 2G, ... (G = gridDim.x).
  const uint64_t step = gridDim.x;
  const uint64_t first = blockIdx.x;

  if (gtid == 0) {
    mbar_init(&gs.full, 1);
    mbar_init(&gs.empty, kGroupWarps);
    gs.readers = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // The landing buffer cycles full -> (every warp copies it) -> refill, and
  // warps never wait for one another there.  Two release schemes, chosen per
  // layout by measurement: the provider kernel has every warp arrive on the
  // `empty` mbarrier and thread 0 wait on it before issuing the next head;
  // the capsule kernel counts copies in shared memory and the last warp to
  // finish issues the next head itself (the count is reset before that
  // warp's arrive.expect_tx, whose release the other warps acquire through
  // the `full` barrier before they count again).  The block barriers inside
  // the head (B1, B2) order every other shared array between heads.
  int64_t head = -1;
  uint64_t item = next_item(p, first, step, &head, gtid == 0);
  if (gtid == 0 && head >= 0) {
    if (p.arm_only != 0u) {
      // Test support: the first head's barrier expects bytes that never
      // come, so the first wait runs out; no further arrival is made on it.
      mbar_expect_tx(&gs.full, kElements * sizeof(float));
    } else {
      issue_head(p, gs, head);
    }
  }
  uint32_t parity = 0;
  // Up to two owed (head, mask) pairs per thread, each packed as
  // mask << 32 | head in shared memory (registers are at the kernel's limit;
  // a head index above 32 bits, 256 TiB of state, is patched at once).
  uint64_t* owed = gs.owed[gtid];
  owed[0] = 0u;
  owed[1] = 0u;
  while (head >= 0) {
    bool timed_out = !mbar_wait_bounded(&gs.full, parity, p.wait_limit_ns);
    CapsuleTile ct;
    float4 pv[kWarpRows];
    if (kProvider) {
      const float4* src = reinterpret_cast<const float4*>(gs.stage);
#pragma unroll
      for (int j = 0; j < kWarpRows; ++j) pv[j] = src[(warp * kWarpRows + j) * 32 + lane];
    } else {
      const int g = lane >> 3, q = lane & 7;
      const float4* src = reinterpret_cast<const float4*>(gs.stage);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int row = warp * kWarpRows + 4 * j + g;
#pragma unroll
        for (int c = 0; c < 4; ++c) ct.v[j][c] = src[row * 32 + 8 * c + q];
      }
    }
    __syncwarp();
    int64_t next_head = -1;
    const uint64_t next = next_item(p, item + step, step, &next_head, gtid == 0);
    bool issued = false;
    if (kProvider) {
      // Every warp arrives on `empty`; thread 0 waits for all of them, then
      // issues the next head.
      if (lane == 0) mbar_arrive(&gs.empty);
      if (gtid == 0 && next_head >= 0) {
        if (mbar_wait_bounded(&gs.empty, parity, p.wait_limit_ns)) {
          issue_head(p, gs, next_head);
          issued = true;
        } else {
          timed_out = true;
        }
      }
    } else {
      // The last warp to finish copying issues the next head; nobody waits.
      int last = 0;
      if (lane == 0) {
        __threadfence_block();  // this warp's reads of the buffer precede its count
        last = atomicAdd(&gs.readers, 1) == kGroupWarps - 1;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last && lane == 0) {
        gs.readers = 0;
        if (next_head >= 0) {
          issue_head(p, gs, next_head);
          issued = true;
        }
      }
    }
    parity ^= 1u;
    // The head functions fold `timed_out` into their first block barrier and
    // return the block-wide result.
    uint32_t amb = 0u;
    const bool abort =
        kProvider ? quantize_provider_head<kMode>(p, gs, pv, head, group, warp, lane, gtid,
                                                  timed_out, amb)
                  : quantize_capsule_head<kMode>(p, gs, ct, head, group, warp, lane, gtid,
                                                 timed_out, amb);
    if (abort) {
      // A bounded wait expired somewhere in the block: report it, let a copy
      // still in flight land (again bounded) so that no bulk copy targets this
      // block after it exits, and stop.  Outputs of this launch are then
      // unspecified.
      if (gtid == 0) {
        report(p.status, kStatusWaitTimeout);
        if (issued) (void)mbar_wait_bounded(&gs.full, parity, p.wait_limit_ns);
      }
      return;
    }
    if (amb != 0u) {  // rare
      const uint64_t entry = static_cast<uint64_t>(amb) << 32 | static_cast<uint32_t>(head);
      const bool fits = (static_cast<uint64_t>(head) >> 32) == 0u;
      if (fits && owed[0] == 0u) {
        owed[0] = entry;
      } else if (fits && owed[1] == 0u) {
        owed[1] = entry;
      } else {
        pay_now<kProvider>(p, gs, head, warp, lane, amb);
      }
    }
    item = next;
    head = next_head;
  }
  // Every thread of the block leaves the loop together; the barrier makes the
  // last head's scales (the IEEE path writes them after its own barriers)
  // visible to the late pass.
  __syncthreads();
#pragma unroll 1
  for (int i = 0; i < 2; ++i) {
    const uint64_t entry = owed[i];
    if (entry != 0u) {
      pay_late<kProvider, kMode>(p, static_cast<uint32_t>(entry), warp, lane,
                                 static_cast<uint32_t>(entry >> 32));
    }
  }
}

// ---------------------------------------------------------------------------
// Host-side launch helpers.

template <bool kProvider, int kMode>
cudaError_t launch_quantize_t(const QuantizeParams& p, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = sizeof(QuantizeGroupShared);
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, quantize_kernel<kProvider, kMode>, p);
}

template <bool kProvider, int kMode>
cudaError_t prepare_quantize_t(int* blocks_per_sm) {
  auto kernel = quantize_kernel<kProvider, kMode>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(sizeof(QuantizeGroupShared)));
  if (err != cudaSuccess) return err;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kernel, kQThreads,
                                                       sizeof(QuantizeGroupShared));
}

// Work units of a launch are heads; one head is processed per block at a time.
inline int quantize_units_per_block() { return 1; }

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
