// fit.cuh -- rank-4 compensator fit of the full GDN state codec (sm_100a).
//
// Restates QuantizeBoundary's low-rank stage (native/src/gdn_state_codec_
// state_capsule.cpp:140-188) bit for bit, for [128 key x 128 value] heads:
//
//   for rank r = 0..3:
//     right[c] = sinf((r + 1) (c + 1)); Normalize(right) or right[0] = 1
//     32 times: left  = R right   (fp32, sequential over c), Normalize or stop
//               right = R^T left  (fp32, sequential over rows), Normalize or stop
//     sv = sum over rows, then columns, of (left[k] R[k][c]) right[c]  (fp32)
//     K[k][r] = left[k] sv;  V[c][r] = right[c];  R[k][c] -= (left[k] sv) right[c]
//
// where Normalize(x) divides by (float) sqrt(sum x_i^2) (squares summed in
// double, capsule.cpp:47-65) unless that norm is <= FLT_EPSILON.  Every fp32
// product is rounded before its add (the reference is built without FMA
// contraction), so the kernel uses explicitly rounded __fmul_rn / __fadd_rn.
//
// Design: one 128-thread CTA per head, persistent over heads, three CTAs per
// SM.  The residual lives in shared memory with rows padded to 132 floats, so
// the row sweep (thread = row, float4 loads) and the column sweep (thread =
// column) are both conflict-free.  Each matrix-vector product keeps the
// reference's sequential order per output.  Norms sum the exact double
// squares in a tree and fall back to the reference's sequential order when
// the square root lies near a float rounding midpoint (the same proof as the
// smoothing sums).  The singular value is one sequential 16,384-term chain:
// all threads form its products four rows at a time and one thread adds
// them in order; the other CTAs of the SM overlap the chain.  The residual the
// int8 stage encodes is written to a caller-provided workspace.
#pragma once

#include <cmath>

#include <cuda_fp16.h>

#include "codec_device.cuh"

namespace gdnsc {

constexpr int kFitThreads = 128;
constexpr int kFitStride = 132;            // padded row of the shared residual
constexpr int kFitIterations = 32;         // capsule.cpp:146

// sinf((r + 1) (c + 1)) of the reference, computed on the host with the same
// C library function (capsule.cpp:141-143) and uploaded once per device.
__constant__ float c_fit_sines[kRank][kValues];

struct FitParams {
  const float* dense;       // [heads][128][128] capsule [k][v] or provider [v][k]
  float* residual;          // [heads][128][128] same layout as dense
  float* compensator_keys;  // [heads][128][4]
  float* compensator_values;  // [heads][128][4]
  uint64_t heads;
  uint32_t* status;
  int provider;
};

constexpr int kSvRows = 4;  // rows of singular-value products formed per step

struct __align__(16) FitShared {
  float r[kKeys][kFitStride];  // residual [key][value]
  float left[kKeys];
  float right[kValues];
  float prod[kSvRows][kValues];  // singular-value products of kSvRows rows
  double part[kFitThreads / 32];
  float norm;               // broadcast of a norm or of the singular value
};

// Normalize(vec) for the vector whose element t is held by thread t (and
// mirrored in `vec` in shared memory).  Returns the block-uniform result of
// norm > FLT_EPSILON; on success every element is divided by the norm.
__device__ __forceinline__ bool fit_normalize(FitShared& sh, float* vec, float& v, int t) {
  double sq = static_cast<double>(v) * static_cast<double>(v);  // exact
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) sq = __dadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, off));
  if ((t & 31) == 0) sh.part[t >> 5] = sq;
  __syncthreads();
  // Every thread forms the same norm from the same partials (no broadcast).
  const double tree = __dadd_rn(__dadd_rn(sh.part[0], sh.part[1]), __dadd_rn(sh.part[2], sh.part[3]));
  double root = __dsqrt_rn(tree);
  if (near_float_midpoint(root)) {  // block-uniform
    // The float norm could depend on the summation order: redo the sum in
    // the reference's order (element 0..127).
    double seq = 0.0;
    for (int i = 0; i < kKeys; ++i) {
      seq = __dadd_rn(seq, static_cast<double>(vec[i]) * static_cast<double>(vec[i]));
    }
    root = __dsqrt_rn(seq);
    __syncthreads();  // every thread has read vec before any thread rescales it
  }
  const float norm = __double2float_rn(root);
  if (!(norm > 1.1920928955078125e-07F)) return false;  // FLT_EPSILON
  v = __fdiv_rn(v, norm);
  vec[t] = v;
  return true;
}

// The rank loop of QuantizeBoundary on the residual in shared memory:
// `iterations` power sweeps per rank (the reference fixes 32), then the
// compensators and the deflation.  Compensator keys / values of `head` go to
// ck_out [heads][128][4] / cv_out as fp32, or rounded to binary16 when
// kHalfOut (the window ABI's storage).  Called by all kFitThreads threads.
template <bool kHalfOut>
__device__ __forceinline__ void fit_ranks(FitShared& sh, int t, int iterations, uint64_t head,
                                          void* ck_out, void* cv_out, uint32_t* status) {
  for (int rank = 0; rank < kRank; ++rank) {
    // -- start vector (capsule.cpp:140-144) --------------------------------
    float rv = c_fit_sines[rank][t];
    sh.right[t] = rv;
    if (!fit_normalize(sh, sh.right, rv, t)) {
      __syncthreads();
      if (t == 0) sh.right[0] = 1.0F;
      rv = t == 0 ? 1.0F : rv;
    }
    __syncthreads();
    float lv = 0.0F;
    for (int it = 0; it < iterations; ++it) {
      // left[t] = sum_c R[t][c] * right[c], c = 0..127 in order.
      {
        float acc = 0.0F;
        const float4* row = reinterpret_cast<const float4*>(sh.r[t]);
        const float4* rgt = reinterpret_cast<const float4*>(sh.right);
#pragma unroll 8
        for (int c4 = 0; c4 < kValues / 4; ++c4) {
          const float4 a = row[c4], b = rgt[c4];
          acc = __fadd_rn(acc, __fmul_rn(a.x, b.x));
          acc = __fadd_rn(acc, __fmul_rn(a.y, b.y));
          acc = __fadd_rn(acc, __fmul_rn(a.z, b.z));
          acc = __fadd_rn(acc, __fmul_rn(a.w, b.w));
        }
        lv = acc;
        sh.left[t] = lv;
      }
      if (!fit_normalize(sh, sh.left, lv, t)) break;
      __syncthreads();
      // right[t] = sum_k R[k][t] * left[k], k = 0..127 in order.
      {
        float acc = 0.0F;
        const float4* lft = reinterpret_cast<const float4*>(sh.left);
#pragma unroll 4
        for (int k4 = 0; k4 < kKeys / 4; ++k4) {
          const float4 l = lft[k4];
          acc = __fadd_rn(acc, __fmul_rn(sh.r[4 * k4][t], l.x));
          acc = __fadd_rn(acc, __fmul_rn(sh.r[4 * k4 + 1][t], l.y));
          acc = __fadd_rn(acc, __fmul_rn(sh.r[4 * k4 + 2][t], l.z));
          acc = __fadd_rn(acc, __fmul_rn(sh.r[4 * k4 + 3][t], l.w));
        }
        rv = acc;
        sh.right[t] = rv;  // right[] is not read by this sweep
      }
      if (!fit_normalize(sh, sh.right, rv, t)) break;
      __syncthreads();
    }
    __syncthreads();
    // -- singular value: one sequential chain in row-major order -----------
    // All threads form the products (left[k] R[k][c]) right[c] of kSvRows
    // rows at a time (thread t: column t); thread 0 adds them in order.
    {
      float sv = 0.0F;  // thread 0's running sum
      const float rt = sh.right[t];
      for (int k0 = 0; k0 < kKeys; k0 += kSvRows) {
#pragma unroll
        for (int j = 0; j < kSvRows; ++j) {
          sh.prod[j][t] = __fmul_rn(__fmul_rn(sh.left[k0 + j], sh.r[k0 + j][t]), rt);
        }
        __syncthreads();
        if (t == 0) {
          const float4* pr = reinterpret_cast<const float4*>(&sh.prod[0][0]);
#pragma unroll 8
          for (int i = 0; i < kSvRows * kValues / 4; ++i) {
            const float4 q = pr[i];
            sv = __fadd_rn(sv, q.x);
            sv = __fadd_rn(sv, q.y);
            sv = __fadd_rn(sv, q.z);
            sv = __fadd_rn(sv, q.w);
          }
        }
        __syncthreads();
      }
      if (t == 0) {
        if (!isfinite(sv)) report(status, kStatusFitNonFinite);
        sh.norm = sv;
      }
    }
    __syncthreads();
    const float sv = sh.norm;
    // -- compensators and deflation (capsule.cpp:175-187) ------------------
    const float kl = __fmul_rn(sh.left[t], sv);
    const uint64_t kidx = (head * kKeys + t) * kRank + rank;
    const uint64_t vidx = (head * kValues + t) * kRank + rank;
    if constexpr (kHalfOut) {
      static_cast<uint16_t*>(ck_out)[kidx] = __half_as_ushort(__float2half_rn(kl));
      static_cast<uint16_t*>(cv_out)[vidx] = __half_as_ushort(__float2half_rn(sh.right[t]));
    } else {
      static_cast<float*>(ck_out)[kidx] = kl;
      static_cast<float*>(cv_out)[vidx] = sh.right[t];
    }
    {
      float4* row = reinterpret_cast<float4*>(sh.r[t]);
      const float4* rgt = reinterpret_cast<const float4*>(sh.right);
#pragma unroll 8
      for (int c4 = 0; c4 < kValues / 4; ++c4) {
        float4 a = row[c4];
        const float4 b = rgt[c4];
        a.x = __fsub_rn(a.x, __fmul_rn(kl, b.x));
        a.y = __fsub_rn(a.y, __fmul_rn(kl, b.y));
        a.z = __fsub_rn(a.z, __fmul_rn(kl, b.z));
        a.w = __fsub_rn(a.w, __fmul_rn(kl, b.w));
        row[c4] = a;
      }
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kFitThreads) fit_kernel(FitParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  FitShared& sh = *reinterpret_cast<FitShared*>(smem_raw);
  const int t = threadIdx.x;
  for (uint64_t head = blockIdx.x; head < p.heads; head += gridDim.x) {
    const float* dense = p.dense + head * kElements;
    // -- residual <- dense (capsule order [k][v] in shared memory) -----------
    bool finite = true;
    if (!p.provider) {
#pragma unroll 4
      for (int i = 0; i < kElements / 4 / kFitThreads; ++i) {
        const int piece = t + kFitThreads * i;   // 16-byte piece: row piece/32
        const int row = piece >> 5, col = 4 * (piece & 31);
        const float4 x = __ldcs(reinterpret_cast<const float4*>(dense + row * 128 + col));
        finite = finite && isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w);
        *reinterpret_cast<float4*>(&sh.r[row][col]) = x;
      }
    } else {
      // provider [v][k]: read rows of values, store transposed.
#pragma unroll 4
      for (int v = 0; v < kValues; ++v) {
        const float x = __ldcs(dense + v * 128 + t);
        finite = finite && isfinite(x);
        sh.r[t][v] = x;
      }
    }
    if (__syncthreads_or(!finite) != 0 && t == 0) report(p.status, kStatusFitNonFinite);

    fit_ranks<false>(sh, t, kFitIterations, head, p.compensator_keys, p.compensator_values,
                     p.status);
    // -- residual out, in the input's layout ---------------------------------
    float* out = p.residual + head * kElements;
    if (!p.provider) {
      for (int k = 0; k < kKeys; ++k) __stcs(out + k * 128 + t, sh.r[k][t]);
    } else {
      for (int v = 0; v < kValues; ++v) __stcs(out + v * 128 + t, sh.r[t][v]);
    }
    __syncthreads();  // the next head overwrites the shared residual
  }
}

inline size_t fit_smem_bytes() { return sizeof(FitShared); }

// Host: upload sinf((r + 1)(c + 1)) computed with the C library, as the
// reference computes its start vectors.
inline cudaError_t prepare_fit(int* blocks_per_sm) {
  float sines[kRank][kValues];
  for (int r = 0; r < kRank; ++r) {
    for (int c = 0; c < kValues; ++c) {
      sines[r][c] = std::sin(static_cast<float>((r + 1) * (c + 1)));
    }
  }
  cudaError_t err = cudaMemcpyToSymbol(c_fit_sines, sines, sizeof(sines));
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(fit_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(fit_smem_bytes()));
  if (err != cudaSuccess) return err;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, fit_kernel, kFitThreads,
                                                       fit_smem_bytes());
}

inline cudaError_t launch_fit(const FitParams& p, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kFitThreads);
  cfg.dynamicSmemBytes = fit_smem_bytes();
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, fit_kernel, p);
}

}  // namespace gdnsc
