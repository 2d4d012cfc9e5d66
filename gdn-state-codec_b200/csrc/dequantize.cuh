// dequantize.cuh -- fp32 reconstruction of encoded GDN state heads (sm_100a).
//
// Restates DequantizeBoundary (native/src/gdn_state_codec_state_capsule.cpp:
// 229-251) bit for bit:
//
//   dense_kv = ((c_k * (float)z_kv) / 127) * b_v
//   dense_kv += K_kr * V_vr   for r = 0..3 in order (only when compensators
//                             are given; the quant-only format has none)
//
// Streaming kernel (17 KiB read, 64 KiB written per head): warp w handles
// rows 16w..16w+15 of a head, lane l handles columns 4l..4l+3, so each code
// load is one coalesced 128-byte row per warp and each store one coalesced
// 512-byte row per warp.  Division by 127 uses the exhaustively verified
// two-term reciprocal (codec_device.cuh); keys with |c| < 2^-112 fall back to
// IEEE division.  Products run as packed fp32x2.
#pragma once

#include "codec_device.cuh"

namespace gdnsc {

constexpr int kDThreads = 256;
constexpr int kDWarps = kDThreads / 32;
constexpr int kDRows = kKeys / kDWarps;  // 16 rows per warp

struct DequantizeParams {
  const int8_t* codes;               // [heads][128][128]
  const float* smoothing;            // [heads][128]  (per key)
  const float* scales;               // [heads][128]  (per value)
  const float* compensator_keys;     // [heads][128][4] or nullptr
  const float* compensator_values;   // [heads][128][4] or nullptr
  float* dense;                      // [heads][128][128]
  uint64_t items;
  SlotMap map;
  uint32_t* status;
};

__device__ __forceinline__ bool key_needs_ieee(float c) {
  return !(fabsf(c) >= kDiv127Safe || c == 0.0F);
}

// Four elements: key factors ck (per element), value factors bv (per element).
__device__ __forceinline__ float4 dequant4(uint32_t word, f2 c01, f2 c23, f2 b01, f2 b23,
                                           bool ieee) {
  f2 z01, z23;
  unpack_codes(word, z01, z23);
  const f2 t01 = mul2(c01, z01);  // c * (float)z
  const f2 t23 = mul2(c23, z23);
  f2 q01, q23;
  if (!ieee) {
    q01 = div127x2(t01);
    q23 = div127x2(t23);
  } else {
    q01 = pack2(__fdiv_rn(lo2(t01), kQuantMax), __fdiv_rn(hi2(t01), kQuantMax));
    q23 = pack2(__fdiv_rn(lo2(t23), kQuantMax), __fdiv_rn(hi2(t23), kQuantMax));
  }
  const f2 o01 = mul2(q01, b01);
  const f2 o23 = mul2(q23, b23);
  return make_float4(lo2(o01), hi2(o01), lo2(o23), hi2(o23));
}

// value += K[k][r] * V[v][r], r = 0..3 in order (capsule.cpp:241-246).  The
// running value may be -0 for arbitrary caller data, so this (full-codec,
// off the quant-only hot path) sum uses scalar .rn operations, which are never
// contracted, rather than the packed +0-addend product of mul2_for_add.
__device__ __forceinline__ float4 add_compensation(float4 d, const float4 kr[4], const float4 vr[4]) {
  float out[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
  for (int r = 0; r < kRank; ++r) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float k = reinterpret_cast<const float*>(&kr[i])[r];
      const float v = reinterpret_cast<const float*>(&vr[i])[r];
      out[i] = __fadd_rn(out[i], __fmul_rn(k, v));
    }
  }
  return make_float4(out[0], out[1], out[2], out[3]);
}

template <bool kProvider, bool kCompensated>
__global__ void __launch_bounds__(kDThreads) dequantize_kernel(DequantizeParams p) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = warp * kDRows;
  for (uint64_t item = blockIdx.x; item < p.items; item += gridDim.x) {
    bool bad = false;
    const int64_t head = resolve_item(p.map, item, &bad);
    if (bad && threadIdx.x == 0) report(p.status, kStatusBadSlot);
    if (head < 0) continue;
    const uint64_t base = static_cast<uint64_t>(head) * kElements;
    const int8_t* codes = p.codes + base;
    float* dense = p.dense + base;
    // Issue every code load of this warp's 16 rows before any math.
    uint32_t words[kDRows];
#pragma unroll
    for (int j = 0; j < kDRows; ++j) words[j] = ld_cs_u32(codes + (row0 + j) * 128 + 4 * lane);
    // Per-lane column factors and per-row factors.
    const float4 col = __ldg(reinterpret_cast<const float4*>(
                                 (kProvider ? p.smoothing : p.scales) + head * 128) + lane);
    const float* row_factor = (kProvider ? p.scales : p.smoothing) + head * 128 + row0;
    float4 col_comp[4];
    if (kCompensated) {
      // Compensators are [heads][128][4]: one float4 of rank entries per
      // key / value; this lane's four columns are entries 4l..4l+3.
      const float4* comp_base = reinterpret_cast<const float4*>(
          (kProvider ? p.compensator_keys : p.compensator_values)) +
          static_cast<uint64_t>(head) * 128;
#pragma unroll
      for (int i = 0; i < 4; ++i) col_comp[i] = __ldg(comp_base + 4 * lane + i);
    }
    const f2 col01 = pack2(col.x, col.y), col23 = pack2(col.z, col.w);
    bool col_ieee = false;
    if (kProvider) {
      col_ieee = key_needs_ieee(col.x) || key_needs_ieee(col.y) || key_needs_ieee(col.z) ||
                 key_needs_ieee(col.w);
    }
#pragma unroll
    for (int j = 0; j < kDRows; ++j) {
      const float rf = __ldg(row_factor + j);
      const f2 rf2 = pack2(rf, rf);
      float4 out;
      if (kProvider) {
        // provider element (v, k): key factor per column, value factor per row.
        out = dequant4(words[j], col01, col23, rf2, rf2, col_ieee);
      } else {
        out = dequant4(words[j], rf2, rf2, col01, col23, key_needs_ieee(rf));
      }
      if (kCompensated) {
        float4 row_comp[4];
        const float4 rc = __ldg(reinterpret_cast<const float4*>(
                                    (kProvider ? p.compensator_values : p.compensator_keys)) +
                                static_cast<uint64_t>(head) * 128 + row0 + j);
        // The row's four rank entries apply to all four elements.
        row_comp[0] = rc;
        row_comp[1] = rc;
        row_comp[2] = rc;
        row_comp[3] = rc;
        if (kProvider) {
          out = add_compensation(out, col_comp, row_comp);  // K per column, V per row
        } else {
          out = add_compensation(out, row_comp, col_comp);  // K per row, V per column
        }
      }
      st_cs_v4(dense + (row0 + j) * 128 + 4 * lane, out);
    }
  }
}

cudaError_t launch_dequantize(bool provider, const DequantizeParams& p, int grid,
                              cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kDThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  const bool comp = p.compensator_keys != nullptr && p.compensator_values != nullptr;
  if (provider) {
    return comp ? cudaLaunchKernelEx(&cfg, dequantize_kernel<true, true>, p)
                : cudaLaunchKernelEx(&cfg, dequantize_kernel<true, false>, p);
  }
  return comp ? cudaLaunchKernelEx(&cfg, dequantize_kernel<false, true>, p)
              : cudaLaunchKernelEx(&cfg, dequantize_kernel<false, false>, p);
}

cudaError_t prepare_dequantize(bool provider, bool comp, int* blocks_per_sm) {
  if (provider) {
    return comp ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, dequantize_kernel<true, true>, kDThreads, 0)
                : cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, dequantize_kernel<true, false>, kDThreads, 0);
  }
  return comp ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, dequantize_kernel<false, true>, kDThreads, 0)
              : cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, dequantize_kernel<false, false>, kDThreads, 0);
}

}  // namespace gdnsc
