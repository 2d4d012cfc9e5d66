// projection.cuh -- encoded projection o = dequant(S)^T q straight from the
// int8 codes (sm_100a).  The fp32 state is never materialised.
//
// Restates the boundary readout of ReadWindowState (native/src/
// gdn_state_codec_state_capsule.cpp:264, 281-304) with an empty update
// window, bit for bit:
//
//   rp_v  = sum_k ((float)z_kv * c_k) * x_k        fp32, k = 0..127 in order
//   o_v   = 0 + (rp_v / 127) * b_v
//   p_r   = sum_k K_kr * x_k                        fp32, k in order
//   o_v  += V_vr * p_r                              r = 0..3 in order
//
// x is the bf16 query widened to fp32 (exact).  Each warp owns one head and
// each lane four outputs v = 4l..4l+3, so the sequential k-sum is four
// independent fp32 chains per lane (two packed fp32x2 chains).
//  * capsule codes [k][v]: at step k a warp reads one 128-byte code row;
//    the loads of the next batch of 8 rows are in flight while the current
//    batch is accumulated (software pipelining).
//  * provider codes [v][k]: a lane's four outputs are four code rows, so the
//    warp loads its 16 KiB head with coalesced 128-bit loads, stores it to
//    shared memory with an XOR swizzle on 16-byte chunks and reads its rows
//    back conflict-free.
#pragma once

#include "codec_device.cuh"

namespace gdnsc {

constexpr int kPThreads = 128;
constexpr int kPWarps = kPThreads / 32;
constexpr int kPBatch = 8;   // capsule code rows per pipelined batch

struct ProjectParams {
  const int8_t* codes;              // [heads][128][128]
  const float* smoothing;           // [heads][128]
  const float* scales;              // [heads][128]
  const float* compensator_keys;    // [heads][128][4] or nullptr
  const float* compensator_values;  // [heads][128][4] or nullptr
  const uint16_t* queries;          // bf16 [items][128]
  float* outputs;                   // [items][128]
  uint64_t items;
  SlotMap map;
  uint32_t* status;
};

struct ProjectShared {
  float2 cx[kPWarps][kKeys];        // (c_k, x_k) per warp
  float4 kr[kPWarps][kKeys];        // compensator keys per warp (full format only)
};

// Provider codes are streamed through shared memory in key slabs: slab s of a
// head holds keys 32s .. 32s + 31 of all 128 value rows (4 KiB).  Each warp
// owns a ring of kSlabStages slabs filled by cp.async, so the copies of the
// next slabs (of this head or the next) overlap the current slab's arithmetic.
// Within a slab, the 32 bytes of rows 4L .. 4L + 3 form line L (128 bytes,
// eight 16-byte chunks c = 2 * (row % 4) + half) and chunk c is stored at
// position c ^ (L % 8), so a lane reading its own four rows hits eight
// distinct bank groups per quarter warp.
constexpr int kSlabKeys = 32;
constexpr int kSlabsPerHead = kKeys / kSlabKeys;           // 4
constexpr int kSlabStages = 3;
constexpr int kSlabChunks = kValues * kSlabKeys / 16;      // 256 x 16 bytes
struct ProviderProjectShared {
  uint4 slab[kPWarps][kSlabStages][kSlabChunks];
  float4 cx[kPWarps][kKeys / 2];    // (c_k, x_k, c_k+1, x_k+1) per warp
  float4 kr[kPWarps][kKeys];        // compensator keys per warp (full format only)
};

__device__ __forceinline__ float4 bf16x4_to_float4(uint2 w) {
  return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xFFFF0000u),
                     __uint_as_float(w.y << 16), __uint_as_float(w.y & 0xFFFF0000u));
}

// One k step for four outputs whose codes are given as magic floats.
__device__ __forceinline__ void accumulate(f2& a01, f2& a23, f2 z01, f2 z23, float c, float x) {
  const f2 cc = pack2(c, c), xx = pack2(x, x);
  a01 = add2(a01, mul2_for_add(mul2(z01, cc), xx));
  a23 = add2(a23, mul2_for_add(mul2(z23, cc), xx));
}

__device__ __forceinline__ float4 finish_outputs(f2 a01, f2 a23, float4 b4, bool comp,
                                                 f2 kp01, f2 kp23, const float* vbase) {
  float rp[4] = {lo2(a01), hi2(a01), lo2(a23), hi2(a23)};
  float q[4];
  const bool fast = (fabsf(rp[0]) >= kDiv127Safe || rp[0] == 0.F) &&
                    (fabsf(rp[1]) >= kDiv127Safe || rp[1] == 0.F) &&
                    (fabsf(rp[2]) >= kDiv127Safe || rp[2] == 0.F) &&
                    (fabsf(rp[3]) >= kDiv127Safe || rp[3] == 0.F);
  if (fast) {
    const f2 q01 = div127x2(a01), q23 = div127x2(a23);
    q[0] = lo2(q01); q[1] = hi2(q01); q[2] = lo2(q23); q[3] = hi2(q23);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = div127_any(rp[i]);
  }
  // output = 0 + (rp / 127) * b (capsule.cpp:264, 288-289)
  const f2 zero = pack2(0.F, 0.F);
  f2 o01 = add2(zero, mul2_for_add(pack2(q[0], q[1]), pack2(b4.x, b4.y)));
  f2 o23 = add2(zero, mul2_for_add(pack2(q[2], q[3]), pack2(b4.z, b4.w)));
  if (comp) {
    const float p[4] = {lo2(kp01), hi2(kp01), lo2(kp23), hi2(kp23)};
    const float4 v0 = __ldg(reinterpret_cast<const float4*>(vbase) + 0);
    const float4 v1 = __ldg(reinterpret_cast<const float4*>(vbase) + 1);
    const float4 v2 = __ldg(reinterpret_cast<const float4*>(vbase) + 2);
    const float4 v3 = __ldg(reinterpret_cast<const float4*>(vbase) + 3);
#pragma unroll
    for (int r = 0; r < kRank; ++r) {
      const f2 pp = pack2(p[r], p[r]);
      const float e0 = reinterpret_cast<const float*>(&v0)[r];
      const float e1 = reinterpret_cast<const float*>(&v1)[r];
      const float e2 = reinterpret_cast<const float*>(&v2)[r];
      const float e3 = reinterpret_cast<const float*>(&v3)[r];
      o01 = add2(o01, mul2_for_add(pack2(e0, e1), pp));
      o23 = add2(o23, mul2_for_add(pack2(e2, e3), pp));
    }
  }
  return make_float4(lo2(o01), hi2(o01), lo2(o23), hi2(o23));
}

// Capsule codes [k][v].
template <bool kCompensated>
__global__ void __launch_bounds__(kPThreads) project_kernel(ProjectParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  ProjectShared& sh = *reinterpret_cast<ProjectShared*>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kPWarps;
  for (uint64_t item = static_cast<uint64_t>(blockIdx.x) * kPWarps + warp; item < p.items;
       item += stride) {
    bool bad = false;
    const int64_t head = resolve_item(p.map, item, &bad);
    float* out = p.outputs + item * kValues + 4 * lane;
    if (head < 0) {
      if (bad && lane == 0) report(p.status, kStatusBadSlot);
      *reinterpret_cast<float4*>(out) = make_float4(0.F, 0.F, 0.F, 0.F);
      continue;
    }
    const uint64_t hbase = static_cast<uint64_t>(head);
    const int8_t* codes = p.codes + hbase * kElements;
    // (c_k, x_k) and compensator keys for this head into this warp's slots.
    const float4 c4 = __ldg(reinterpret_cast<const float4*>(p.smoothing + hbase * kKeys) + lane);
    const float4 x4 = bf16x4_to_float4(
        __ldg(reinterpret_cast<const uint2*>(p.queries + item * kKeys) + lane));
    __syncwarp();  // previous head's readers are done with this warp's slots
    reinterpret_cast<float4*>(sh.cx[warp])[2 * lane] = make_float4(c4.x, x4.x, c4.y, x4.y);
    reinterpret_cast<float4*>(sh.cx[warp])[2 * lane + 1] = make_float4(c4.z, x4.z, c4.w, x4.w);
    if (kCompensated) {
      const float4* kp = reinterpret_cast<const float4*>(p.compensator_keys) + hbase * kKeys;
#pragma unroll
      for (int i = 0; i < 4; ++i) sh.kr[warp][4 * lane + i] = __ldg(kp + 4 * lane + i);
    }
    __syncwarp();

    f2 a01 = pack2(0.F, 0.F), a23 = pack2(0.F, 0.F);
    f2 kp01 = pack2(0.F, 0.F), kp23 = pack2(0.F, 0.F);
    {
      // Software-pipelined over batches of kPBatch code rows: the loads of the
      // next batch are in flight while this batch is accumulated.
      const uint32_t* cw = reinterpret_cast<const uint32_t*>(codes) + lane;
      const float4* cx2 = reinterpret_cast<const float4*>(sh.cx[warp]);  // rows k, k + 1
      auto rows = [&](const uint32_t (&w)[kPBatch], int k) {
#pragma unroll
        for (int i = 0; i < kPBatch; i += 2) {
          const float4 cc = cx2[(k + i) >> 1];
          f2 z01, z23;
          unpack_codes(w[i], z01, z23);
          accumulate(a01, a23, z01, z23, cc.x, cc.y);
          unpack_codes(w[i + 1], z01, z23);
          accumulate(a01, a23, z01, z23, cc.z, cc.w);
          if (kCompensated) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const float4 kk = sh.kr[warp][k + i + h];
              const float x = h == 0 ? cc.y : cc.w;
              const f2 xx = pack2(x, x);
              kp01 = add2(kp01, mul2_for_add(pack2(kk.x, kk.y), xx));
              kp23 = add2(kp23, mul2_for_add(pack2(kk.z, kk.w), xx));
            }
          }
        }
      };
      uint32_t wa[kPBatch], wb[kPBatch];
#pragma unroll
      for (int i = 0; i < kPBatch; ++i) wa[i] = ld_cs_u32(cw + i * 32);
#pragma unroll 1
      for (int k0 = 0; k0 < kKeys; k0 += 2 * kPBatch) {
#pragma unroll
        for (int i = 0; i < kPBatch; ++i) wb[i] = ld_cs_u32(cw + (k0 + kPBatch + i) * 32);
        rows(wa, k0);
        if (k0 + 2 * kPBatch < kKeys) {
#pragma unroll
          for (int i = 0; i < kPBatch; ++i) wa[i] = ld_cs_u32(cw + (k0 + 2 * kPBatch + i) * 32);
        }
        rows(wb, k0 + kPBatch);
      }
    }
    const float4 b4 = __ldg(reinterpret_cast<const float4*>(p.scales + hbase * kValues) + lane);
    // Every lane holds all four rank projections p_r (identical chains).
    const float* vbase = kCompensated
                             ? p.compensator_values + (hbase * kValues + 4 * lane) * kRank
                             : nullptr;
    const float4 o = finish_outputs(a01, a23, b4, kCompensated, kp01, kp23, vbase);
    __stcs(reinterpret_cast<float4*>(out), o);
  }
}

// Provider codes [v][k]: lane l owns outputs v = 4l .. 4l + 3 (rows of the
// code matrix) and accumulates them over k = 0..127 in order, slab by slab.
template <bool kCompensated>
__global__ void __launch_bounds__(kPThreads) project_provider_kernel(ProjectParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  ProviderProjectShared& sh = *reinterpret_cast<ProviderProjectShared*>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kPWarps;
  const uint64_t first = static_cast<uint64_t>(blockIdx.x) * kPWarps + warp;
  uint4* ring = sh.slab[warp][0];

  // The warp streams (item, slab) positions in order; a position's slab sits
  // in ring stage (position % kSlabStages).  Copies run kSlabStages - 1
  // positions ahead of the arithmetic.
  auto head_of = [&](uint64_t item) -> int64_t {
    bool bad = false;
    return item < p.items ? resolve_item(p.map, item, &bad) : -1;
  };
  // Lane-constant parts of the slab copy: piece lane + 32i is row
  // 16i + lane/2, half lane%2, stored in line 4i + lane/8 at chunk
  // (lane%8) ^ ((4i + lane/8) % 8) = (lane%8) ^ g ^ 4(i%2), g = lane/8.
  const int g = lane >> 3;
  const int src_lane = (lane >> 1) * 128 + 16 * (lane & 1);
  const int dst_even = 8 * g + ((lane & 7) ^ g);
  const int dst_odd = 8 * g + ((lane & 7) ^ g ^ 4);
  auto issue = [&](int slab, int stage, int64_t head) {
    if (head >= 0) {
      const int8_t* src = p.codes + static_cast<uint64_t>(head) * kElements + kSlabKeys * slab + src_lane;
      uint4* dst = ring + stage * kSlabChunks;
#pragma unroll
      for (int i = 0; i < 8; ++i) cp_async16(dst + 32 * i + ((i & 1) ? dst_odd : dst_even), src + 2048 * i);
    }
    cp_async_commit();  // one group per position, empty ones included
  };

  // Per-head inputs of the next item, fetched one head ahead.
  float4 c_next = make_float4(0.F, 0.F, 0.F, 0.F), b_next = c_next;
  uint2 q_next = make_uint2(0u, 0u);
  auto fetch = [&](uint64_t item, int64_t head) {
    if (head < 0) return;
    c_next = __ldg(reinterpret_cast<const float4*>(p.smoothing + static_cast<uint64_t>(head) * kKeys) + lane);
    b_next = __ldg(reinterpret_cast<const float4*>(p.scales + static_cast<uint64_t>(head) * kValues) + lane);
    q_next = __ldg(reinterpret_cast<const uint2*>(p.queries + item * kKeys) + lane);
  };
  int64_t next_head = head_of(first);  // head of the item after the current one
  fetch(first, next_head);
  // Prologue: the first kSlabStages - 1 positions (slabs of the first item).
#pragma unroll
  for (int t = 0; t < kSlabStages - 1; ++t) issue(t, t, next_head);

  const f2 magic = pack2(kCodeMagic, kCodeMagic);
  const int swz = lane & 7;
  int stage = 0;                              // ring stage of the current position
  int ahead = kSlabStages - 1;                // ring stage of the position being issued
  for (uint64_t item = first; item < p.items; item += stride) {
    bool bad = false;
    (void)resolve_item(p.map, item, &bad);
    if (bad && lane == 0) report(p.status, kStatusBadSlot);
    const int64_t head = next_head;
    next_head = head_of(item + stride);
    // (c_k, x_k) of this head into the warp's slots; the previous head's
    // readers finished at the end of its last slab.
    const float4 x4 = bf16x4_to_float4(q_next);
    sh.cx[warp][2 * lane] = make_float4(c_next.x, x4.x, c_next.y, x4.y);
    sh.cx[warp][2 * lane + 1] = make_float4(c_next.z, x4.z, c_next.w, x4.w);
    if (kCompensated && head >= 0) {
      const float4* kp = reinterpret_cast<const float4*>(p.compensator_keys) +
                         static_cast<uint64_t>(head) * kKeys;
#pragma unroll
      for (int i = 0; i < 4; ++i) sh.kr[warp][4 * lane + i] = __ldg(kp + 4 * lane + i);
    }
    const float4 b4 = b_next;
    fetch(item + stride, next_head);
    f2 a01 = pack2(0.F, 0.F), a23 = a01, kp01 = a01, kp23 = a01;
#pragma unroll 1
    for (int s = 0; s < kSlabsPerHead; ++s) {
      // Issue the position kSlabStages - 1 ahead: slab s + 2 of this item or
      // slab s - 2 of the next one.
      const int ahead_slab = s + kSlabStages - 1;
      if (ahead_slab < kSlabsPerHead) {
        issue(ahead_slab, ahead, head);
      } else {
        issue(ahead_slab - kSlabsPerHead, ahead, next_head);
      }
      ahead = ahead + 1 == kSlabStages ? 0 : ahead + 1;
      cp_async_wait<kSlabStages - 1>();  // this position's slab has landed (own copies)
      __syncwarp();                      // ... and every lane's copies are visible
      if (head >= 0) {
        const uint4* buf = ring + stage * kSlabChunks + lane * 8;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint4 r[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) r[j] = buf[(2 * j + half) ^ swz];
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const uint32_t b0 = reinterpret_cast<const uint32_t*>(&r[0])[wi] ^ kCodeBias;
            const uint32_t b1 = reinterpret_cast<const uint32_t*>(&r[1])[wi] ^ kCodeBias;
            const uint32_t b2 = reinterpret_cast<const uint32_t*>(&r[2])[wi] ^ kCodeBias;
            const uint32_t b3 = reinterpret_cast<const uint32_t*>(&r[3])[wi] ^ kCodeBias;
            const int k0 = kSlabKeys * s + 16 * half + 4 * wi;
#pragma unroll
            for (int pair = 0; pair < 2; ++pair) {
              const float4 cc = sh.cx[warp][(k0 >> 1) + pair];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int byte = 2 * pair + e;
                const float c = e == 0 ? cc.x : cc.z, x = e == 0 ? cc.y : cc.w;
                const f2 z01 = sub2(pack2(code_magic(b0, byte), code_magic(b1, byte)), magic);
                const f2 z23 = sub2(pack2(code_magic(b2, byte), code_magic(b3, byte)), magic);
                accumulate(a01, a23, z01, z23, c, x);
                if (kCompensated) {
                  const float4 kk = sh.kr[warp][k0 + byte];
                  const f2 xx = pack2(x, x);
                  kp01 = add2(kp01, mul2_for_add(pack2(kk.x, kk.y), xx));
                  kp23 = add2(kp23, mul2_for_add(pack2(kk.z, kk.w), xx));
                }
              }
            }
          }
        }
      }
      __syncwarp();  // this slab (and after the last one, the head's slots) free again
      stage = stage + 1 == kSlabStages ? 0 : stage + 1;
    }
    float* out = p.outputs + item * kValues + 4 * lane;
    if (head < 0) {
      *reinterpret_cast<float4*>(out) = make_float4(0.F, 0.F, 0.F, 0.F);
    } else {
      const float* vbase = kCompensated
                               ? p.compensator_values +
                                     (static_cast<uint64_t>(head) * kValues + 4 * lane) * kRank
                               : nullptr;
      __stcs(reinterpret_cast<float4*>(out),
             finish_outputs(a01, a23, b4, kCompensated, kp01, kp23, vbase));
    }
  }
  cp_async_wait<0>();  // no copy may still target this block's memory at exit
}

size_t project_smem_bytes(bool provider, bool compensated) {
  if (provider) {
    return compensated ? sizeof(ProviderProjectShared) : offsetof(ProviderProjectShared, kr);
  }
  return compensated ? sizeof(ProjectShared) : offsetof(ProjectShared, kr);
}

template <bool kProvider, bool kCompensated>
constexpr auto project_kernel_for() {
  if constexpr (kProvider) {
    return project_provider_kernel<kCompensated>;
  } else {
    return project_kernel<kCompensated>;
  }
}

template <bool kProvider, bool kCompensated>
cudaError_t launch_project_t(const ProjectParams& p, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = project_smem_bytes(kProvider, kCompensated);
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, project_kernel_for<kProvider, kCompensated>(), p);
}

template <bool kProvider, bool kCompensated>
cudaError_t prepare_project_t(int* blocks_per_sm) {
  auto kernel = project_kernel_for<kProvider, kCompensated>();
  const size_t bytes = project_smem_bytes(kProvider, kCompensated);
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(bytes));
  if (err != cudaSuccess) return err;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kernel, kPThreads, bytes);
}

cudaError_t prepare_project(bool provider, bool comp, int* blocks_per_sm) {
  if (provider) return comp ? prepare_project_t<true, true>(blocks_per_sm)
                            : prepare_project_t<true, false>(blocks_per_sm);
  return comp ? prepare_project_t<false, true>(blocks_per_sm)
              : prepare_project_t<false, false>(blocks_per_sm);
}

cudaError_t launch_project(bool provider, const ProjectParams& p, int grid, cudaStream_t stream) {
  const bool comp = p.compensator_keys != nullptr && p.compensator_values != nullptr;
  if (provider) return comp ? launch_project_t<true, true>(p, grid, stream)
                            : launch_project_t<true, false>(p, grid, stream);
  return comp ? launch_project_t<false, true>(p, grid, stream)
              : launch_project_t<false, false>(p, grid, stream);
}

}  // namespace gdnsc
