// window.cuh -- the p = 16 windowed decode step, its boundary refit and the
// dense fp32 GDN step (sm_100a).
//
// A head's decode state is the INT8 boundary (codes, smoothing c, scales b,
// binary16 rank-4 compensators) plus up to 16 buffered rank-one records
// {decay, key, correction} (record_decay fp32 [16], record_keys /
// record_corrections binary16 [16][128], position u32 at [head][8]), the
// buffers of gdn_state_codec_windowed_gdn_kernel.h:5-6.
//
// Step (capsule.cpp:354-397, ApplyToken, with the read of :256-304):
//   state_read = Read(read);  correction = value - state_read
//   output     = Read(decay * query) + correction * (key . query)
//   append {decay, key, correction}; position += 1
// where Read(x)[v] walks the records newest first (projection of the
// suffix-decayed x onto the record key, times the record correction, then
// x *= record decay), then adds the boundary readout
// (sum_k (z[k][v] c_k) x_k, k in order) / 127 * b_v and the compensators
// V[v][r] (sum_k K[k][r] x_k).  Every sum keeps the reference's sequential
// order and every product is rounded before its add (__fmul_rn / __fadd_rn),
// so outputs and records are bit-identical to the portable library's
// arithmetic with the ABI's binary16 record storage.
//
// Qwen3.5 form (the vLLM plugin's decode, runtime.py:750-845): decay =
// exp(log decay), key = beta k, read = decay k, query = 128^-0.5 q, with q / k
// of head h taken from head h / 2 (two value heads per query/key head) and a
// bf16 output; boundary codes in the provider layout [v][k].  Generic form
// (windowed_gdn_step_launch_v1): decay, write key, read, query and value
// given directly (binary16), fp32 output, capsule-layout codes [k][v].
//
// Design: one 128-thread CTA per head, persistent over heads.  Thread t owns
// key t for the vector work and value column t for the readout.  The suffix-
// decayed read vectors live in shared memory (rows padded to 132 floats so
// the per-record projections, one thread per (record, read), read four keys
// per conflict-free vector load); those projections and the compensator /
// update projections run on the first warps while every thread sums its
// column's boundary readout for both reads at once, two consecutive keys per
// packed fp32x2 product.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "codec_device.cuh"
#include "fit.cuh"

namespace gdnsc {

constexpr int kWindow = 16;                 // capsule.h:14, p = 16
constexpr int kPositionStride = 8;          // positions [head][8]
constexpr int kWinThreads = 128;
constexpr float kQueryScale = 0.08838834764831845F;  // 128^-0.5 (windowed_gdn_step.cpp:297)

struct WindowBuffers {
  const int8_t* codes;             // [heads][128][128]
  const float* smoothing;          // [heads][128]
  const float* scales;             // [heads][128]
  const uint16_t* ck;              // binary16 [heads][128][4] or nullptr (none)
  const uint16_t* cv;              // binary16 [heads][128][4] or nullptr
  float* record_decay;             // [heads][16]
  uint16_t* record_keys;           // binary16 [heads][16][128]
  uint16_t* record_corrections;    // binary16 [heads][16][128]
  uint32_t* positions;             // [heads][8], position at [head][0]
};

struct StepParams {
  WindowBuffers w;
  const float* decay;        // Qwen: log decay [heads]; generic: decay [heads]
  const uint16_t* beta;      // Qwen: bf16 [heads]
  const uint16_t* keys;      // Qwen: bf16 [heads/2][128]; generic: binary16 write keys [heads][128]
  const uint16_t* reads;     // generic: binary16 [heads][128]
  const uint16_t* queries;   // Qwen: bf16 [heads/2][128]; generic: binary16 [heads][128]
  const uint16_t* values;    // Qwen: bf16 [heads][128]; generic: binary16 [heads][128]
  void* outputs;             // Qwen: bf16 [heads][128]; generic: fp32 [heads][128]
  uint64_t heads;
};

constexpr int kRowPad = kKeys + 4;  // 16-byte rows; 8 rows at one key hit 32 banks

struct __align__(16) StepShared {
  float suffix[2][kWindow][kRowPad];    // suffix-decayed read / query before record p-1-j
  float rkey[kWindow][kRowPad];         // record keys (fp32)
  float4 sq[kKeys / 2];                  // suffix after every record, per key pair j:
                                        // (read 2j, read 2j+1, query 2j, query 2j+1)
  float4 ck[kKeys];                     // compensator keys
  float c[kKeys];                       // smoothing
  float key[kKeys];                     // write key of this token
  float query[kKeys];                   // query of this token (undecayed)
  float proj[2][kWindow];               // record projections per read
  float cproj[2][kRank];                // compensator projections per read
  float rdecay[kWindow];                // record decays
  float up;                             // key . query
};

struct __align__(16) StepSharedCapsule {
  StepShared s;
  int8_t codes[kElements];  // capsule-layout codes staged for column reads
};

__device__ __forceinline__ float half_to_float(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ float bf16_to_float(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}
__device__ __forceinline__ uint16_t float_to_half_bits(float x) {
  return __half_as_ushort(__float2half_rn(x));
}

// One sequential dot product sum_k a[k] * b[k], k = 0..127, of two
// contiguous, 16-byte aligned vectors, four keys per load.
__device__ __forceinline__ float chain_dot4(const float* a, const float* b) {
  const float4* a4 = reinterpret_cast<const float4*>(a);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  float acc = 0.0F;
#pragma unroll 8
  for (int k4 = 0; k4 < kKeys / 4; ++k4) {
    const float4 x = a4[k4], y = b4[k4];
    acc = __fadd_rn(acc, __fmul_rn(x.x, y.x));
    acc = __fadd_rn(acc, __fmul_rn(x.y, y.y));
    acc = __fadd_rn(acc, __fmul_rn(x.z, y.z));
    acc = __fadd_rn(acc, __fmul_rn(x.w, y.w));
  }
  return acc;
}

template <bool kQwen, bool kComp>
__global__ void __launch_bounds__(kWinThreads, 6) window_step_kernel(StepParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  StepShared& sh = *reinterpret_cast<StepShared*>(smem_raw);
  const int t = threadIdx.x;
  for (uint64_t head = blockIdx.x; head < p.heads; head += gridDim.x) {
    // Every load that does not depend on the window position is issued
    // before the position is first used, so their latencies overlap.
    const uint32_t pos = __ldcg(p.w.positions + head * kPositionStride);
    const uint64_t rbase = head * kWindow;
    // ---- codes of column t (provider: one 128-byte row per value) ---------
    uint4 zrow[8];
    if constexpr (kQwen) {
      const uint4* src = reinterpret_cast<const uint4*>(p.w.codes + head * kElements + t * kKeys);
#pragma unroll
      for (int i = 0; i < 8; ++i) zrow[i] = __ldcs(src + i);
    } else {
      int8_t* staged = reinterpret_cast<StepSharedCapsule*>(smem_raw)->codes;
      const uint4* src = reinterpret_cast<const uint4*>(p.w.codes + head * kElements);
#pragma unroll
      for (int i = 0; i < kElements / 16 / kWinThreads; ++i) {
        reinterpret_cast<uint4*>(staged)[t + kWinThreads * i] = __ldcs(src + t + kWinThreads * i);
      }
    }
    // ---- token inputs (thread t: key t and value t) -----------------------
    float alpha, key_t, read_t, query_t, value_t;
    if constexpr (kQwen) {
      alpha = expf(__ldg(p.decay + head));
      const float beta = bf16_to_float(__ldg(p.beta + head));
      const uint64_t qk = (head >> 1) * kKeys + t;
      const float k = bf16_to_float(__ldg(p.keys + qk));
      key_t = __fmul_rn(beta, k);
      read_t = __fmul_rn(alpha, k);
      query_t = __fmul_rn(kQueryScale, bf16_to_float(__ldg(p.queries + qk)));
      value_t = bf16_to_float(__ldg(p.values + head * kValues + t));
    } else {
      alpha = __ldg(p.decay + head);
      key_t = half_to_float(__ldg(p.keys + head * kKeys + t));
      read_t = half_to_float(__ldg(p.reads + head * kKeys + t));
      query_t = half_to_float(__ldg(p.queries + head * kKeys + t));
      value_t = half_to_float(__ldg(p.values + head * kValues + t));
    }
    sh.key[t] = key_t;
    sh.query[t] = query_t;
    sh.c[t] = __ldg(p.w.smoothing + head * kKeys + t);
    const float b_t = __ldg(p.w.scales + head * kValues + t);
    float cv_t[kRank] = {0.F, 0.F, 0.F, 0.F};
    if constexpr (kComp) {
      const uint2 kw = __ldg(reinterpret_cast<const uint2*>(p.w.ck + (head * kKeys + t) * kRank));
      sh.ck[t] = make_float4(half_to_float(kw.x & 0xFFFFu), half_to_float(kw.x >> 16),
                             half_to_float(kw.y & 0xFFFFu), half_to_float(kw.y >> 16));
      const uint2 vw = __ldg(reinterpret_cast<const uint2*>(p.w.cv + (head * kValues + t) * kRank));
      cv_t[0] = half_to_float(vw.x & 0xFFFFu);
      cv_t[1] = half_to_float(vw.x >> 16);
      cv_t[2] = half_to_float(vw.y & 0xFFFFu);
      cv_t[3] = half_to_float(vw.y >> 16);
    }
    if (t < kWindow) sh.rdecay[t] = __ldcg(p.w.record_decay + rbase + t);
    // ---- records: keys to shared memory, corrections of column t ----------
    // All 16 slots are read before the position is known, so a head costs one
    // memory round trip; slots at or past the position are never used.
    float rc[kWindow];
#pragma unroll
    for (int u = 0; u < kWindow; ++u) {
      sh.rkey[u][t] = half_to_float(__ldcg(p.w.record_keys + (rbase + u) * kKeys + t));
      rc[u] = half_to_float(__ldcg(p.w.record_corrections + (rbase + u) * kValues + t));
    }
    if (pos >= kWindow) {  // block-uniform: every thread read the same word
      if (t == 0) report(nullptr, kStatusWindowFull);
      continue;
    }
    const int np = static_cast<int>(pos);
    __syncthreads();  // record keys and decays in shared memory
    // ---- suffix-decayed read and query (thread t = key t) -----------------
    {
      float s0 = read_t, s1 = __fmul_rn(alpha, query_t);
#pragma unroll
      for (int u = kWindow - 1; u >= 0; --u) {  // record u is read with suffix np-1-u
        if (u < np) {
          sh.suffix[0][np - 1 - u][t] = s0;
          sh.suffix[1][np - 1 - u][t] = s1;
          const float d = sh.rdecay[u];
          s0 = __fmul_rn(s0, d);
          s1 = __fmul_rn(s1, d);
        }
      }
      float* sq = reinterpret_cast<float*>(sh.sq) + 4 * (t >> 1) + (t & 1);
      sq[0] = s0;
      sq[2] = s1;
    }
    __syncthreads();
    // ---- sequential projections: records, compensators, update -----------
    const int chains = 2 * np + (kComp ? 2 * kRank : 0) + 1;
    if (kComp && t >= 2 * np && t < 2 * np + 2 * kRank) {
      const int i = t - 2 * np;
      const int r = i / kRank, m = i % kRank;
      const float* ck = reinterpret_cast<const float*>(sh.ck) + m;
      const float* sq = reinterpret_cast<const float*>(sh.sq) + 2 * r;
      float acc = 0.0F;
#pragma unroll 8
      for (int k = 0; k < kKeys; ++k) {
        acc = __fadd_rn(acc, __fmul_rn(ck[4 * k], sq[4 * (k >> 1) + (k & 1)]));
      }
      sh.cproj[r][m] = acc;
    } else if (t < chains) {
      const float* a = sh.key;
      const float* b = sh.query;
      float* dst = &sh.up;
      if (t < 2 * np) {
        const int r = t / np == 0 ? 0 : 1;
        const int u = t - r * np;
        a = &sh.rkey[u][0];
        b = &sh.suffix[r][np - 1 - u][0];
        dst = &sh.proj[r][u];
      }
      *dst = chain_dot4(a, b);
    }
    // ---- boundary readout of column t for both reads ----------------------
    // Products of two consecutive keys are formed as one packed pair per
    // read; the sums take them in key order.
    float acc0 = 0.0F, acc1 = 0.0F;
    if constexpr (kQwen) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t words[4] = {zrow[i].x, zrow[i].y, zrow[i].z, zrow[i].w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int k0 = 16 * i + 4 * w;
          f2 z01, z23;
          unpack_codes(words[w], z01, z23);
          const float4 c4 = *reinterpret_cast<const float4*>(&sh.c[k0]);
          const f2 zc01 = mul2(z01, pack2(c4.x, c4.y));
          const f2 zc23 = mul2(z23, pack2(c4.z, c4.w));
          const float4 sa = sh.sq[k0 >> 1], sb = sh.sq[(k0 >> 1) + 1];
          f2 p0 = mul2_for_add(zc01, pack2(sa.x, sa.y));
          f2 p1 = mul2_for_add(zc01, pack2(sa.z, sa.w));
          acc0 = __fadd_rn(__fadd_rn(acc0, lo2(p0)), hi2(p0));
          acc1 = __fadd_rn(__fadd_rn(acc1, lo2(p1)), hi2(p1));
          p0 = mul2_for_add(zc23, pack2(sb.x, sb.y));
          p1 = mul2_for_add(zc23, pack2(sb.z, sb.w));
          acc0 = __fadd_rn(__fadd_rn(acc0, lo2(p0)), hi2(p0));
          acc1 = __fadd_rn(__fadd_rn(acc1, lo2(p1)), hi2(p1));
        }
      }
    } else {
      const int8_t* staged = reinterpret_cast<StepSharedCapsule*>(smem_raw)->codes;
      const float* sq = reinterpret_cast<const float*>(sh.sq);
#pragma unroll 8
      for (int k = 0; k < kKeys; ++k) {
        const float zc = __fmul_rn(static_cast<float>(staged[k * kValues + t]), sh.c[k]);
        const int j = 4 * (k >> 1) + (k & 1);
        acc0 = __fadd_rn(acc0, __fmul_rn(zc, sq[j]));
        acc1 = __fadd_rn(acc1, __fmul_rn(zc, sq[j + 2]));
      }
    }
    __syncthreads();
    // ---- column t: records newest first, boundary, compensators -----------
    float out0 = 0.0F, out1 = 0.0F;
#pragma unroll
    for (int u = kWindow - 1; u >= 0; --u) {
      if (u < np) {
        out0 = __fadd_rn(out0, __fmul_rn(rc[u], sh.proj[0][u]));
        out1 = __fadd_rn(out1, __fmul_rn(rc[u], sh.proj[1][u]));
      }
    }
    out0 = __fadd_rn(out0, __fmul_rn(div127_any(acc0), b_t));
    out1 = __fadd_rn(out1, __fmul_rn(div127_any(acc1), b_t));
    if constexpr (kComp) {
#pragma unroll
      for (int m = 0; m < kRank; ++m) {
        out0 = __fadd_rn(out0, __fmul_rn(cv_t[m], sh.cproj[0][m]));
        out1 = __fadd_rn(out1, __fmul_rn(cv_t[m], sh.cproj[1][m]));
      }
    }
    const float correction = __fsub_rn(value_t, out0);
    const float output = __fadd_rn(out1, __fmul_rn(correction, sh.up));
    if constexpr (kQwen) {
      static_cast<uint16_t*>(p.outputs)[head * kValues + t] =
          __bfloat16_as_ushort(__float2bfloat16_rn(output));
    } else {
      static_cast<float*>(p.outputs)[head * kValues + t] = output;
    }
    if (!isfinite(output)) report(nullptr, kStatusWindowNonFinite);
    // ---- append the record -------------------------------------------------
    p.w.record_keys[(rbase + np) * kKeys + t] = float_to_half_bits(key_t);
    p.w.record_corrections[(rbase + np) * kValues + t] = float_to_half_bits(correction);
    if (t == 0) {
      p.w.record_decay[rbase + np] = alpha;
      p.w.positions[head * kPositionStride] = pos + 1u;
    }
    __syncthreads();  // shared memory is reused by the next head
  }
}

template <bool kQwen>
inline size_t window_step_smem_bytes() {
  return kQwen ? sizeof(StepShared) : sizeof(StepSharedCapsule);
}

// ---------------------------------------------------------------------------
// Boundary refit (window_boundary_launch_v1): DenseState of the window
// (capsule.cpp:337-352, dequantized boundary then every record oldest first)
// into shared memory, QuantizeBoundary's rank loop with `iterations` power
// sweeps (none: quant-only refit, zero compensators), the residual written to
// the caller's workspace in the provider layout for the INT8 stage that
// follows, and the window cleared (records zero, position 0).

struct FoldParams {
  WindowBuffers w;           // current boundary and records (records cleared)
  uint16_t* next_ck;         // binary16 [heads][128][4]
  uint16_t* next_cv;         // binary16 [heads][128][4]
  float* workspace;          // [heads][128][128] residual, provider layout
  uint64_t heads;
  int iterations;            // 0..32
};

struct __align__(16) FoldExtra {
  float rc[kWindow][kValues];   // record corrections
  float4 cv[kValues];           // compensator values
  float b[kValues];             // scales
};

__global__ void __launch_bounds__(kFitThreads) window_fold_kernel(FoldParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  FitShared& sh = *reinterpret_cast<FitShared*>(smem_raw);
  FoldExtra& ex = *reinterpret_cast<FoldExtra*>(smem_raw + ((sizeof(FitShared) + 15) & ~size_t{15}));
  const int t = threadIdx.x;
  const bool comp = p.w.ck != nullptr;
  for (uint64_t head = blockIdx.x; head < p.heads; head += gridDim.x) {
    const uint32_t pos_raw = __ldcg(p.w.positions + head * kPositionStride);
    const int np = pos_raw < static_cast<uint32_t>(kWindow) ? static_cast<int>(pos_raw) : kWindow;
    const uint64_t rbase = head * kWindow;
    // ---- gather the window (thread t: key t, value t) ----------------------
    ex.b[t] = __ldg(p.w.scales + head * kValues + t);
    float4 ck_t = make_float4(0.F, 0.F, 0.F, 0.F);
    if (comp) {
      const uint2 kw = __ldg(reinterpret_cast<const uint2*>(p.w.ck + (head * kKeys + t) * kRank));
      ck_t = make_float4(half_to_float(kw.x & 0xFFFFu), half_to_float(kw.x >> 16),
                         half_to_float(kw.y & 0xFFFFu), half_to_float(kw.y >> 16));
      const uint2 vw = __ldg(reinterpret_cast<const uint2*>(p.w.cv + (head * kValues + t) * kRank));
      ex.cv[t] = make_float4(half_to_float(vw.x & 0xFFFFu), half_to_float(vw.x >> 16),
                             half_to_float(vw.y & 0xFFFFu), half_to_float(vw.y >> 16));
    }
    float rk[kWindow], rd[kWindow];
#pragma unroll
    for (int u = 0; u < kWindow; ++u) {
      rk[u] = 0.0F;
      rd[u] = 0.0F;
      if (u < np) {
        rk[u] = half_to_float(__ldcg(p.w.record_keys + (rbase + u) * kKeys + t));
        rd[u] = __ldcg(p.w.record_decay + rbase + u);
        ex.rc[u][t] = half_to_float(__ldcg(p.w.record_corrections + (rbase + u) * kValues + t));
      }
    }
    const float c_t = __ldg(p.w.smoothing + head * kKeys + t);
    __syncthreads();
    // ---- dense[t][v]: boundary, compensators, records oldest first ---------
    bool finite = true;
    const int8_t* codes = p.w.codes + head * kElements;
    for (int v = 0; v < kValues; ++v) {
      const float z = static_cast<float>(__ldg(codes + v * kKeys + t));  // provider [v][k]
      float value = __fmul_rn(div127_any(__fmul_rn(c_t, z)), ex.b[v]);
      if (comp) {
        const float4 cvv = ex.cv[v];
        value = __fadd_rn(value, __fmul_rn(ck_t.x, cvv.x));
        value = __fadd_rn(value, __fmul_rn(ck_t.y, cvv.y));
        value = __fadd_rn(value, __fmul_rn(ck_t.z, cvv.z));
        value = __fadd_rn(value, __fmul_rn(ck_t.w, cvv.w));
      }
#pragma unroll
      for (int u = 0; u < kWindow; ++u) {
        if (u < np) value = __fadd_rn(__fmul_rn(rd[u], value), __fmul_rn(rk[u], ex.rc[u][v]));
      }
      finite = finite && isfinite(value);
      sh.r[t][v] = value;
    }
    if (__syncthreads_or(!finite) != 0 && t == 0) report(nullptr, kStatusWindowNonFinite);
    // ---- the window is folded: clear it (every read of it is done) ---------
#pragma unroll 4
    for (int u = 0; u < kWindow; ++u) {
      p.w.record_keys[(rbase + u) * kKeys + t] = 0;
      p.w.record_corrections[(rbase + u) * kValues + t] = 0;
    }
    if (t < kWindow) p.w.record_decay[rbase + t] = 0.0F;
    if (t == 0) p.w.positions[head * kPositionStride] = 0u;
    // ---- rank-4 fit, or zero compensators for the quant-only refit ---------
    if (p.iterations > 0) {
      fit_ranks<true>(sh, t, p.iterations, head, p.next_ck, p.next_cv, nullptr);
    } else {
      reinterpret_cast<uint2*>(p.next_ck + (head * kKeys + t) * kRank)[0] = make_uint2(0u, 0u);
      reinterpret_cast<uint2*>(p.next_cv + (head * kValues + t) * kRank)[0] = make_uint2(0u, 0u);
    }
    // ---- residual to the workspace, provider layout [v][k] -----------------
    float* out = p.workspace + head * kElements;
    for (int v = 0; v < kValues; ++v) __stcg(out + v * kKeys + t, sh.r[t][v]);
    __syncthreads();  // the next head overwrites shared memory
  }
}

// Quant-only refit (no power iterations): the window's DenseState streamed
// straight to the workspace, one 256-thread CTA per head.  Thread t owns the
// key pair (2 (t mod 64), 2 (t mod 64) + 1) of rows v = t / 64 + 4 i, so an
// element pair is adjacent in the provider layout [v][k]: its two codes are
// one 16-bit word, its smoothing, record keys and compensator keys are natural
// register pairs, and it is written with one 8-byte store.  The per-row
// factors (scale, compensator values, record corrections) are the same for
// both elements and for the whole warp (a warp holds one row), so shared
// memory keeps them duplicated, (x, x), and one broadcast load yields the
// packed operand.  Every element follows the reference order (dequantize,
// compensators by rank, records oldest first) in packed fp32x2 arithmetic,
// each product rounded before its add.
constexpr int kDenseThreads = 256;
constexpr int kDensePairs = kKeys / 2;                    // threads per row
constexpr int kDenseRowGroups = kDenseThreads / kDensePairs;  // rows in flight per CTA

struct __align__(16) WindowDenseShared {
  int8_t codes[kElements];              // the head's codes, provider [v][k]
  float4 rc[kWindow / 2][kValues];      // (rc_u, rc_u, rc_u+1, rc_u+1) per row, u even
  float4 cv[2][kValues];                // (V0, V0, V1, V1), (V2, V2, V3, V3) per row
  f2 b[kValues];                        // (b, b) per row
  float4 dd[kWindow / 2];               // (d_u, d_u, d_u+1, d_u+1), u even
};

// a / 127 for both lanes, exact for every float (the two-term reciprocal
// below 2^-112 is replaced by the IEEE division, as in div127_any).
__device__ __forceinline__ f2 div127x2_any(f2 a) {
  const float lo = lo2(a), hi = hi2(a);
  const bool ok = (fabsf(lo) >= kDiv127Safe || lo == 0.0F) &&
                  (fabsf(hi) >= kDiv127Safe || hi == 0.0F);
  return ok ? div127x2(a) : pack2(div127_any(lo), div127_any(hi));
}

__device__ __forceinline__ f2 lo_pair(float4 v) { return pack2(v.x, v.y); }
__device__ __forceinline__ f2 hi_pair(float4 v) { return pack2(v.z, v.w); }

// The workspace rows of one thread (rows row0 + 4 i, keys 2 kp, 2 kp + 1).
// Returns an accumulator that stays +0 while every element is finite and
// becomes NaN otherwise (x * 0 is NaN exactly for infinite or NaN x).
template <bool kComp>
__device__ __forceinline__ f2 dense_rows(const WindowDenseShared& sh, f2 cc, bool c_safe,
                                         const f2 (&rk)[kWindow], const f2 (&ck)[kRank],
                                         int row0, int kp, float* workspace) {
  const uint16_t* codes = reinterpret_cast<const uint16_t*>(sh.codes) + kp;  // [v][pair]
  f2* out = reinterpret_cast<f2*>(workspace) + kp;
  const f2 magic = pack2(kCodeMagic, kCodeMagic);
  const f2 zero = pack2(0.0F, 0.0F);
  f2 flags = zero;
#pragma unroll 2
  for (int i = 0; i < kValues / kDenseRowGroups; ++i) {
    const int v = row0 + kDenseRowGroups * i;
    const uint32_t biased = static_cast<uint32_t>(codes[v * kDensePairs]) ^ kCodeBias;
    const f2 z = sub2(pack2(code_magic(biased, 0), code_magic(biased, 1)), magic);
    const f2 cz = mul2(cc, z);
    f2 q = div127x2(cz);
    if (!c_safe) q = div127x2_any(cz);  // a smoothing below 2^-112 in magnitude
    // Rounded before the compensator adds: a single-use mul.f32x2 feeding an
    // add.f32x2 would be contracted into one fma.  The +0 addend can turn a
    // -0 product into +0, which the INT8 stage encodes identically.
    f2 val = mul2_for_add(q, sh.b[v]);
    if constexpr (kComp) {
      const float4 c01 = sh.cv[0][v], c23 = sh.cv[1][v];
      val = add2(val, mul2_for_add(ck[0], lo_pair(c01)));
      val = add2(val, mul2_for_add(ck[1], hi_pair(c01)));
      val = add2(val, mul2_for_add(ck[2], lo_pair(c23)));
      val = add2(val, mul2_for_add(ck[3], hi_pair(c23)));
    }
#pragma unroll
    for (int j = 0; j < kWindow / 2; ++j) {
      const float4 d = sh.dd[j], r = sh.rc[j][v];
      val = add2(mul2_for_add(lo_pair(d), val), mul2_for_add(rk[2 * j], lo_pair(r)));
      val = add2(mul2_for_add(hi_pair(d), val), mul2_for_add(rk[2 * j + 1], hi_pair(r)));
    }
    flags = fma2(val, zero, flags);
    __stcg(reinterpret_cast<unsigned long long*>(out + v * kDensePairs), val);
  }
  return flags;
}

template <bool kComp>
__global__ void __launch_bounds__(kDenseThreads, 3) window_dense_kernel(FoldParams p) {
  __shared__ WindowDenseShared sh;
  const int t = threadIdx.x;
  const int kp = t % kDensePairs;          // keys 2 kp, 2 kp + 1
  const int row0 = t / kDensePairs;        // rows row0 + 4 i
  for (uint64_t head = blockIdx.x; head < p.heads; head += gridDim.x) {
    const uint32_t pos_raw = __ldcg(p.w.positions + head * kPositionStride);
    const int np = pos_raw < static_cast<uint32_t>(kWindow) ? static_cast<int>(pos_raw) : kWindow;
    const uint64_t rbase = head * kWindow;
    // ---- gather: codes, records, scales, compensators ------------------------
    {
      const uint4* src = reinterpret_cast<const uint4*>(p.w.codes + head * kElements);
#pragma unroll
      for (int i = 0; i < kElements / 16 / kDenseThreads; ++i) {
        reinterpret_cast<uint4*>(sh.codes)[t + kDenseThreads * i] = __ldcs(src + t + kDenseThreads * i);
      }
    }
    // Records past the position are identity records (decay 1, zero key and
    // correction): v -> RN(1 v) + RN(0 0) = v, except that a -0 may become +0,
    // which the INT8 stage maps to the same codes, smoothing and scales.  The
    // record loop below is then free of position tests.
    for (int i = t; i < (kWindow / 2) * kValues; i += kDenseThreads) {
      const int u = 2 * (i / kValues), v = i % kValues;
      const uint16_t* rcs = p.w.record_corrections + rbase * kValues + v;
      const float a = u < np ? half_to_float(__ldcg(rcs + u * kValues)) : 0.0F;
      const float c = u + 1 < np ? half_to_float(__ldcg(rcs + (u + 1) * kValues)) : 0.0F;
      sh.rc[u / 2][v] = make_float4(a, a, c, c);
    }
    if (t < kValues) {
      const float b = __ldg(p.w.scales + head * kValues + t);
      sh.b[t] = pack2(b, b);
      if constexpr (kComp) {
        const uint2 vw = __ldg(reinterpret_cast<const uint2*>(p.w.cv + (head * kValues + t) * kRank));
        const float v0 = half_to_float(vw.x & 0xFFFFu), v1 = half_to_float(vw.x >> 16);
        const float v2 = half_to_float(vw.y & 0xFFFFu), v3 = half_to_float(vw.y >> 16);
        sh.cv[0][t] = make_float4(v0, v0, v1, v1);
        sh.cv[1][t] = make_float4(v2, v2, v3, v3);
      }
    }
    if (t < kWindow / 2) {
      const float d0 = 2 * t < np ? __ldcg(p.w.record_decay + rbase + 2 * t) : 1.0F;
      const float d1 = 2 * t + 1 < np ? __ldcg(p.w.record_decay + rbase + 2 * t + 1) : 1.0F;
      sh.dd[t] = make_float4(d0, d0, d1, d1);
    }
    f2 rk[kWindow];  // (key 2 kp, key 2 kp + 1) of every record
#pragma unroll
    for (int u = 0; u < kWindow; ++u) {
      uint32_t w = 0u;
      if (u < np) w = __ldcg(reinterpret_cast<const uint32_t*>(p.w.record_keys + (rbase + u) * kKeys) + kp);
      rk[u] = pack2(half_to_float(w & 0xFFFFu), half_to_float(w >> 16));
    }
    f2 ck[kRank] = {0ull, 0ull, 0ull, 0ull};
    if constexpr (kComp) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(p.w.ck + head * kKeys * kRank) + kp);
      // keys 2 kp (ranks 0..3 in w.x, w.y) and 2 kp + 1 (w.z, w.w)
      ck[0] = pack2(half_to_float(w.x & 0xFFFFu), half_to_float(w.z & 0xFFFFu));
      ck[1] = pack2(half_to_float(w.x >> 16), half_to_float(w.z >> 16));
      ck[2] = pack2(half_to_float(w.y & 0xFFFFu), half_to_float(w.w & 0xFFFFu));
      ck[3] = pack2(half_to_float(w.y >> 16), half_to_float(w.w >> 16));
    }
    const f2 cc = *reinterpret_cast<const f2*>(p.w.smoothing + head * kKeys + 2 * kp);
    __syncthreads();
    // ---- the window is about to be folded: clear it --------------------------
    for (int i = t; i < kWindow * kKeys; i += kDenseThreads) {
      p.w.record_keys[rbase * kKeys + i] = 0;
      p.w.record_corrections[rbase * kValues + i] = 0;
    }
    if (t < kWindow) p.w.record_decay[rbase + t] = 0.0F;
    if (t == 0) p.w.positions[head * kPositionStride] = 0u;
    if (t < kKeys) {
      reinterpret_cast<uint2*>(p.next_ck + (head * kKeys + t) * kRank)[0] = make_uint2(0u, 0u);
      reinterpret_cast<uint2*>(p.next_cv + (head * kValues + t) * kRank)[0] = make_uint2(0u, 0u);
    }
    // ---- dense rows ----------------------------------------------------------
    // With this thread's smoothing pair at least 2^-112 in magnitude, zero or
    // not finite, every product c z is zero or at least 2^-112 in magnitude
    // (codes are integers), where the two-term reciprocal division is exact;
    // otherwise each product is checked.
    const float c0 = lo2(cc), c1 = hi2(cc);
    const bool c_safe = (fabsf(c0) >= kDiv127Safe || c0 == 0.0F || c0 != c0) &&
                        (fabsf(c1) >= kDiv127Safe || c1 == 0.0F || c1 != c1);
    float* rows = p.workspace + head * kElements;
    const f2 flags = dense_rows<kComp>(sh, cc, c_safe, rk, ck, row0, kp, rows);
    const bool finite = lo2(flags) == 0.0F && hi2(flags) == 0.0F;
    if (__syncthreads_or(!finite) != 0 && t == 0) report(nullptr, kStatusWindowNonFinite);
  }
}

inline size_t window_fold_smem_bytes() {
  return ((sizeof(FitShared) + 15) & ~size_t{15}) + sizeof(FoldExtra);
}

// ---------------------------------------------------------------------------
// Dense fp32 GDN step (fp32_gdn_step_launch_v1; reference kernel
// native/ascendc/gdn_state_codec/kernel/gdn_state_codec_fp32_gdn_step.cpp:
// 10-16), in place on capsule-layout [k][v] states: per value column v,
// correction = value[v] - sum_k S[k][v] read[k]; S[k][v] = decay S[k][v] +
// key[k] correction; out[v] = sum_k S_new[k][v] query[k] (k in order).
//
// HBM-bound (64 KiB read + 64 KiB written per head).  Persistent 128-thread
// CTAs, three per SM, each with one 64 KiB landing buffer filled by a single
// bulk copy: both column passes read the head from shared memory, so each
// state element crosses HBM once each way.  Thread t owns value column t;
// the updated rows go straight to global memory, 512 contiguous bytes per key.

struct DenseStepParams {
  float* state;              // [heads][128][128] capsule layout, updated in place
  const float* decay;        // [heads]
  const uint16_t* keys;      // binary16 [heads][128]
  const uint16_t* reads;
  const uint16_t* queries;
  const uint16_t* values;
  float* outputs;            // [heads][128]
  uint64_t heads;
  uint64_t wait_limit_ns = kWaitLimitNs;  // limit of every bounded wait
  // Test support (fp32_gdn_step_wait_selftest_v1): the first head's barrier
  // is armed for bytes that are never copied, so the first wait runs out with
  // nothing in flight and the block returns before it writes anything.
  uint32_t arm_only = 0u;
};

constexpr int kDenseStepBlocksPerSm = 3;

struct __align__(128) DenseStepShared {
  float stage[kElements];    // the head's state, [k][v]
  float4 key[kKeys / 4];     // token vectors, four keys per entry
  float4 read[kKeys / 4];
  float4 query[kKeys / 4];
  uint64_t full;             // the stage holds the current head
};

__device__ __forceinline__ void dense_step_issue(const DenseStepParams& p, DenseStepShared& sh,
                                                 uint64_t head) {
  fence_proxy_async();
  mbar_expect_tx(&sh.full, kElements * sizeof(float));
  bulk_load(sh.stage, p.state + head * kElements, kElements * sizeof(float), &sh.full,
            evict_first_policy());
}

__global__ void __launch_bounds__(kWinThreads, kDenseStepBlocksPerSm)
    dense_step_kernel(DenseStepParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  DenseStepShared& sh = *reinterpret_cast<DenseStepShared*>(smem_raw);
  const int t = threadIdx.x;
  if (t == 0) {
    mbar_init(&sh.full, 1);
    fence_mbar_init();
    if (p.arm_only != 0u) {
      mbar_expect_tx(&sh.full, kElements * sizeof(float));  // test support: nothing lands
    } else {
      dense_step_issue(p, sh, blockIdx.x);  // the grid never exceeds the head count
    }
  }
  __syncthreads();
  uint32_t parity = 0;
  for (uint64_t head = blockIdx.x; head < p.heads; head += gridDim.x) {
    // Token inputs while the state lands.
    reinterpret_cast<float*>(sh.key)[t] = half_to_float(__ldg(p.keys + head * kKeys + t));
    reinterpret_cast<float*>(sh.read)[t] = half_to_float(__ldg(p.reads + head * kKeys + t));
    reinterpret_cast<float*>(sh.query)[t] = half_to_float(__ldg(p.queries + head * kKeys + t));
    const float value = half_to_float(__ldg(p.values + head * kValues + t));
    const float decay = __ldg(p.decay + head);
    const uint32_t phase = parity;
    parity ^= 1u;
    const bool landed = mbar_wait_bounded(&sh.full, phase, p.wait_limit_ns);
    if (__syncthreads_or(!landed)) {  // token vectors published; uniform result
      // A bounded wait expired: report it, let the copy land (again bounded)
      // so that it no longer targets this block, and stop.
      if (t == 0) {
        report(nullptr, kStatusWaitTimeout);
        (void)mbar_wait_bounded(&sh.full, phase, p.wait_limit_ns);
      }
      return;
    }
    const float* s = sh.stage + t;
    float projection = 0.0F;
#pragma unroll 4
    for (int k4 = 0; k4 < kKeys / 4; ++k4) {
      const float4 r = sh.read[k4];
      const float* col = s + 4 * k4 * kValues;
      projection = __fadd_rn(projection, __fmul_rn(col[0], r.x));
      projection = __fadd_rn(projection, __fmul_rn(col[kValues], r.y));
      projection = __fadd_rn(projection, __fmul_rn(col[2 * kValues], r.z));
      projection = __fadd_rn(projection, __fmul_rn(col[3 * kValues], r.w));
    }
    const float correction = __fsub_rn(value, projection);
    float* dst = p.state + head * kElements + t;
    float out = 0.0F;
#pragma unroll 2
    for (int k4 = 0; k4 < kKeys / 4; ++k4) {
      const float4 kk = sh.key[k4], qq = sh.query[k4];
      const float kv[4] = {kk.x, kk.y, kk.z, kk.w};
      const float qv[4] = {qq.x, qq.y, qq.z, qq.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = 4 * k4 + i;
        const float next = __fadd_rn(__fmul_rn(decay, s[k * kValues]),
                                     __fmul_rn(kv[i], correction));
        dst[k * kValues] = next;
        out = __fadd_rn(out, __fmul_rn(next, qv[i]));
      }
    }
    p.outputs[head * kValues + t] = out;
    __syncthreads();  // every thread is done with the stage and the token vectors
    const uint64_t next_head = head + gridDim.x;
    if (t == 0 && next_head < p.heads) dense_step_issue(p, sh, next_head);
  }
}

// ---------------------------------------------------------------------------
// Host set-up and launches.

struct WindowBlocks {
  int step[2][2] = {};  // [qwen][comp] blocks per SM
  int fold = 0;
  int window_dense = 0;
  int dense = 0;
};

template <bool kQwen, bool kComp>
inline cudaError_t prepare_step_variant(int* blocks) {
  const auto kernel = window_step_kernel<kQwen, kComp>;
  const size_t smem = window_step_smem_bytes<kQwen>();
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, kernel, kWinThreads, smem);
}

inline cudaError_t prepare_window(WindowBlocks* b) {
  cudaError_t err;
  if ((err = prepare_step_variant<true, true>(&b->step[1][1])) != cudaSuccess) return err;
  if ((err = prepare_step_variant<true, false>(&b->step[1][0])) != cudaSuccess) return err;
  if ((err = prepare_step_variant<false, true>(&b->step[0][1])) != cudaSuccess) return err;
  if ((err = prepare_step_variant<false, false>(&b->step[0][0])) != cudaSuccess) return err;
  err = cudaFuncSetAttribute(window_fold_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(window_fold_smem_bytes()));
  if (err != cudaSuccess) return err;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b->fold, window_fold_kernel, kFitThreads,
                                                      window_fold_smem_bytes());
  if (err != cudaSuccess) return err;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b->window_dense, window_dense_kernel<true>,
                                                      kDenseThreads, 0);
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(dense_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(DenseStepShared)));
  if (err != cudaSuccess) return err;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b->dense, dense_step_kernel, kWinThreads,
                                                       sizeof(DenseStepShared));
}

inline cudaError_t launch_window_step(bool qwen, bool comp, const StepParams& p, int grid,
                                      cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWinThreads);
  cfg.stream = stream;
  if (qwen) {
    cfg.dynamicSmemBytes = window_step_smem_bytes<true>();
    return comp ? cudaLaunchKernelEx(&cfg, window_step_kernel<true, true>, p)
                : cudaLaunchKernelEx(&cfg, window_step_kernel<true, false>, p);
  }
  cfg.dynamicSmemBytes = window_step_smem_bytes<false>();
  return comp ? cudaLaunchKernelEx(&cfg, window_step_kernel<false, true>, p)
              : cudaLaunchKernelEx(&cfg, window_step_kernel<false, false>, p);
}

inline cudaError_t launch_window_fold(const FoldParams& p, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kFitThreads);
  cfg.dynamicSmemBytes = window_fold_smem_bytes();
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, window_fold_kernel, p);
}

inline cudaError_t launch_window_dense(const FoldParams& p, int grid, cudaStream_t stream) {
  if (p.w.ck != nullptr) {
    window_dense_kernel<true><<<grid, kDenseThreads, 0, stream>>>(p);
  } else {
    window_dense_kernel<false><<<grid, kDenseThreads, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

inline cudaError_t launch_dense_step(const DenseStepParams& p, int grid, cudaStream_t stream) {
  dense_step_kernel<<<grid, kWinThreads, sizeof(DenseStepShared), stream>>>(p);
  return cudaGetLastError();
}

}  // namespace gdnsc
