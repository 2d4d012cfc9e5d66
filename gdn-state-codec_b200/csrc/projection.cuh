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
  float4 kr[kPWarps][kKeys];        // compensator keys per warp
  uint4 codes[kPWarps][kElements / 16];  // provider: staged head (swizzled)
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

template <bool kProvider, bool kCompensated>
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
    // Provider codes: issue the first half of the head's coalesced loads.
    uint4 staged[kProvider ? 16 : 1];
    if (kProvider) {
#pragma unroll
      for (int i = 0; i < 16; ++i) staged[i] = ld_cs_v4u(codes + i * 512 + 16 * lane);
    }
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
    if (kProvider) {
      // Load i covers row r = 4i + lane/8, chunk lane%8; it is stored at the
      // swizzled chunk (lane%8) ^ (r/4 % 8) so that a lane reading its own
      // rows (r/4 == lane) hits eight distinct bank groups per quarter warp.
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        if (half == 1) {
#pragma unroll
          for (int i = 0; i < 16; ++i) staged[i] = ld_cs_v4u(codes + (16 + i) * 512 + 16 * lane);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int li = 16 * half + i;
          const int row = 4 * li + (lane >> 3);
          const int chunk = (lane & 7) ^ (li & 7);
          sh.codes[warp][row * 8 + chunk] = staged[i];
        }
      }
    }
    __syncwarp();

    f2 a01 = pack2(0.F, 0.F), a23 = pack2(0.F, 0.F);
    f2 kp01 = pack2(0.F, 0.F), kp23 = pack2(0.F, 0.F);
    const f2 magic = pack2(kCodeMagic, kCodeMagic);
    if (!kProvider) {
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
    } else {
      // Lane owns rows v = 4l + j; rows j = 0,1 form pair 01, rows 2,3 pair 23.
      const int swz = lane & 7;  // (row >> 2) & 7 for all four rows
#pragma unroll 1
      for (int chunk = 0; chunk < 8; ++chunk) {
        uint4 r[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) r[j] = sh.codes[warp][(4 * lane + j) * 8 + (chunk ^ swz)];
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          const uint32_t b0 = reinterpret_cast<const uint32_t*>(&r[0])[wi] ^ kCodeBias;
          const uint32_t b1 = reinterpret_cast<const uint32_t*>(&r[1])[wi] ^ kCodeBias;
          const uint32_t b2 = reinterpret_cast<const uint32_t*>(&r[2])[wi] ^ kCodeBias;
          const uint32_t b3 = reinterpret_cast<const uint32_t*>(&r[3])[wi] ^ kCodeBias;
#pragma unroll
          for (int byte = 0; byte < 4; ++byte) {
            const int k = chunk * 16 + wi * 4 + byte;
            const float2 cx = sh.cx[warp][k];
            const f2 z01 = sub2(pack2(code_magic(b0, byte), code_magic(b1, byte)), magic);
            const f2 z23 = sub2(pack2(code_magic(b2, byte), code_magic(b3, byte)), magic);
            accumulate(a01, a23, z01, z23, cx.x, cx.y);
            if (kCompensated) {
              const float4 kk = sh.kr[warp][k];
              const f2 xx = pack2(cx.y, cx.y);
              kp01 = add2(kp01, mul2_for_add(pack2(kk.x, kk.y), xx));
              kp23 = add2(kp23, mul2_for_add(pack2(kk.z, kk.w), xx));
            }
          }
        }
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

size_t project_smem_bytes(bool provider) {
  return provider ? sizeof(ProjectShared)
                  : offsetof(ProjectShared, codes);
}

template <bool kProvider, bool kCompensated>
cudaError_t launch_project_t(const ProjectParams& p, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = project_smem_bytes(kProvider);
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, project_kernel<kProvider, kCompensated>, p);
}

template <bool kProvider, bool kCompensated>
cudaError_t prepare_project_t(int* blocks_per_sm) {
  auto kernel = project_kernel<kProvider, kCompensated>;
  const size_t bytes = project_smem_bytes(kProvider);
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
