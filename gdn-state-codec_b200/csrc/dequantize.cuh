// dequantize.cuh -- fp32 reconstruction of encoded GDN state heads (sm_100a).
//
// Restates DequantizeBoundary (native/src/gdn_state_codec_state_capsule.cpp:
// 229-251) bit for bit:
//
//   dense_kv = ((c_k * (float)z_kv) / 127) * b_v
//   dense_kv += K_kr * V_vr   for r = 0..3 in order (only when compensators
//                             are given; the quant-only format has none)
//
// Streaming kernel (17 KiB read, 64 KiB written per head), write-bound:
// persistent 256-thread CTAs, four per SM (three with compensators).  A head is produced in four
// chunks of 32 rows; warp w computes rows 4w..4w+3 of a chunk, lane l columns
// 4l..4l+3 (one coalesced 128-byte code row per warp and load).  Each chunk
// is assembled in one of two 16 KiB shared-memory buffers and written by a
// single bulk store (cp.async.bulk, shared -> global), which reaches a higher
// write bandwidth than per-thread stores.  Division by 127 uses the
// exhaustively verified two-term reciprocal (codec_device.cuh); keys with
// |c| < 2^-112 fall back to IEEE division.  Products run as packed fp32x2.
#pragma once

#include "codec_device.cuh"

namespace gdnsc {

constexpr int kDThreads = 256;
constexpr int kDWarps = kDThreads / 32;
constexpr int kDBlocksPerSm = 4;
constexpr int kDChunkRows = 32;                     // rows per bulk store (16 KiB)
constexpr int kDChunks = kKeys / kDChunkRows;       // 4 per head
constexpr int kDWarpRows = kDChunkRows / kDWarps;   // 4 rows per warp and chunk
constexpr int kDStages = 2;                         // chunk buffers in rotation

struct __align__(128) DequantizeShared {
  float stage[kDStages][kDChunkRows * kValues];
};

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
__global__ void __launch_bounds__(kDThreads, kCompensated ? kDBlocksPerSm - 1 : kDBlocksPerSm)
    dequantize_kernel(DequantizeParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  DequantizeShared& sh = *reinterpret_cast<DequantizeShared*>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int stage = 0;
  for (uint64_t item = blockIdx.x; item < p.items; item += gridDim.x) {
    bool bad = false;
    const int64_t head = resolve_item(p.map, item, &bad);
    if (bad && threadIdx.x == 0) report(p.status, kStatusBadSlot);
    if (head < 0) continue;  // block-uniform
    const uint64_t base = static_cast<uint64_t>(head) * kElements;
    const int8_t* codes = p.codes + base;
    float* dense = p.dense + base;
    // Issue every code load of this thread (4 chunks x 4 rows) before any math.
    uint32_t words[kDChunks][kDWarpRows];
#pragma unroll
    for (int ch = 0; ch < kDChunks; ++ch) {
#pragma unroll
      for (int j = 0; j < kDWarpRows; ++j) {
        words[ch][j] = ld_cs_u32(codes + (kDChunkRows * ch + kDWarpRows * warp + j) * 128 + 4 * lane);
      }
    }
    // Per-lane column factors and per-row factors.
    const float4 col = __ldg(reinterpret_cast<const float4*>(
                                 (kProvider ? p.smoothing : p.scales) + head * 128) + lane);
    const float* row_factor = (kProvider ? p.scales : p.smoothing) + head * 128;
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
    for (int ch = 0; ch < kDChunks; ++ch) {
      float4 out[kDWarpRows];
#pragma unroll
      for (int j = 0; j < kDWarpRows; ++j) {
        const int row = kDChunkRows * ch + kDWarpRows * warp + j;
        const float rf = __ldg(row_factor + row);
        const f2 rf2 = pack2(rf, rf);
        if (kProvider) {
          // provider element (v, k): key factor per column, value factor per row.
          out[j] = dequant4(words[ch][j], col01, col23, rf2, rf2, col_ieee);
        } else {
          out[j] = dequant4(words[ch][j], rf2, rf2, col01, col23, key_needs_ieee(rf));
        }
        if (kCompensated) {
          float4 row_comp[4];
          const float4 rc = __ldg(reinterpret_cast<const float4*>(
                                      (kProvider ? p.compensator_values : p.compensator_keys)) +
                                  static_cast<uint64_t>(head) * 128 + row);
          // The row's four rank entries apply to all four elements.
          row_comp[0] = rc;
          row_comp[1] = rc;
          row_comp[2] = rc;
          row_comp[3] = rc;
          if (kProvider) {
            out[j] = add_compensation(out[j], col_comp, row_comp);  // K per column, V per row
          } else {
            out[j] = add_compensation(out[j], row_comp, col_comp);  // K per row, V per column
          }
        }
      }
      // The buffer is free once the store issued kDStages chunks ago has read it.
      if (threadIdx.x == 0) bulk_wait_read<kDStages - 1>();
      __syncthreads();
      float* buf = sh.stage[stage];
#pragma unroll
      for (int j = 0; j < kDWarpRows; ++j) {
        reinterpret_cast<float4*>(buf + (kDWarpRows * warp + j) * kValues)[lane] = out[j];
      }
      fence_proxy_async();  // these generic-proxy writes precede the bulk store's reads
      __syncthreads();
      if (threadIdx.x == 0) {
        bulk_store(dense + kDChunkRows * ch * kValues, buf, kDChunkRows * kValues * sizeof(float));
        bulk_commit();
      }
      stage ^= 1;
    }
  }
  if (threadIdx.x == 0) bulk_wait_all();  // shared memory stays valid until the stores read it
}

cudaError_t launch_dequantize(bool provider, const DequantizeParams& p, int grid,
                              cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kDThreads);
  cfg.dynamicSmemBytes = sizeof(DequantizeShared);
  cfg.stream = stream;
  const bool comp = p.compensator_keys != nullptr && p.compensator_values != nullptr;
  if (provider) {
    return comp ? cudaLaunchKernelEx(&cfg, dequantize_kernel<true, true>, p)
                : cudaLaunchKernelEx(&cfg, dequantize_kernel<true, false>, p);
  }
  return comp ? cudaLaunchKernelEx(&cfg, dequantize_kernel<false, true>, p)
              : cudaLaunchKernelEx(&cfg, dequantize_kernel<false, false>, p);
}

template <bool kProvider, bool kCompensated>
cudaError_t prepare_dequantize_t(int* blocks_per_sm) {
  const auto kernel = dequantize_kernel<kProvider, kCompensated>;
  const cudaError_t err = cudaFuncSetAttribute(
      kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sizeof(DequantizeShared)));
  if (err != cudaSuccess) return err;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kernel, kDThreads,
                                                       sizeof(DequantizeShared));
}

cudaError_t prepare_dequantize(bool provider, bool comp, int* blocks_per_sm) {
  if (provider) {
    return comp ? prepare_dequantize_t<true, true>(blocks_per_sm)
                : prepare_dequantize_t<true, false>(blocks_per_sm);
  }
  return comp ? prepare_dequantize_t<false, true>(blocks_per_sm)
              : prepare_dequantize_t<false, false>(blocks_per_sm);
}

}  // namespace gdnsc
