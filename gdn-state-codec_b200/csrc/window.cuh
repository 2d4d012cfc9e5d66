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
#include <type_traits>
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

struct __align__(128) StepSharedCapsule {
  StepShared s;
  // Capsule-layout codes staged for column reads; 128-byte aligned so that a
  // warp's 32-byte piece of a 128-byte key row never straddles two lines.
  alignas(128) int8_t codes[kElements];
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
// Qwen3.5 steps with the next head's inputs staged a head ahead.  The same
// arithmetic as window_step_kernel<true, comp>; every per-head global read
// (codes, records, position, smoothing, scales, compensators and the token's
// log decay, beta, key, query and value) is a cp.async into one stage that
// the CTA consumes at the start of the head -- codes into registers, records
// converted into the chain rows -- and then refills for its next head while
// this head's suffix, chains and readout run.  Needs 16-byte aligned key,
// query and value rows and a 4-byte aligned beta (the host checks and
// otherwise launches window_step_kernel).
//   window_step_staged_kernel (quant-only boundary): four warps, the
//     sequential projections on the first lanes before their readout, as in
//     window_step_kernel; 55 KB of shared memory, four CTAs per SM.
//   window_step_staged_comp_kernel (rank-4 boundary, whose 41 projections
//     would spill onto a second warp): a fifth warp runs every projection,
//     two per lane in one packed add, beside the four readout warps.

// 128-byte aligned: the code rows' swizzle makes a column read conflict-free
// only when each 128-byte row starts a shared-memory line (measured: 0.49
// against 0.55-0.59 ms per step when the stage sat 48 or 80 bytes past one).
struct __align__(128) StepStage {
  uint4 codes[kValues][8];          // provider row v, 16-byte chunk j at j ^ (v & 7)
  uint16_t rkeys[kWindow][kKeys];   // records (binary16)
  uint16_t rcorr[kWindow][kValues];
  float rdecay[kWindow];
  uint32_t position[4];             // positions[head][0..3]
  float c[kKeys];                   // smoothing
  float b[kValues];                 // scales
  uint16_t key[kKeys];              // bf16 token inputs of the head
  uint16_t query[kKeys];
  uint16_t value[kValues];
  float log_decay;
  uint32_t beta_pair;               // beta[head & ~1], beta[head | 1]
  uint32_t pad[2];
};

struct __align__(16) StagedComp {
  uint2 stage_ck[kKeys];            // staged binary16 compensators
  uint2 stage_cv[kValues];
};

// Quant-only step: the working set of window_step_kernel and the stage.
struct __align__(128) StagedStepShared {
  float suffix[2][kWindow][kRowPad];
  float rkey[kWindow][kRowPad];
  float4 sq[kKeys / 2];
  float c[kKeys];
  float key[kKeys];
  float query[kKeys];
  float proj[2][kWindow];
  float rdecay[kWindow];
  float up;
  StepStage stage;
};

// Compensated step.  Chain operand rows: rkey rows 0..15 are the records,
// row 16 the write key, rows 17..20 the compensator keys by rank; suffix
// rows 0..15 hold (read, query) decayed by the j newest records, row 16
// (q, q) for the update chain, row 17 the final pair for the compensator
// chains.
constexpr int kStagedCompThreads = kKeys + 32;
constexpr int kUpdateRow = kWindow;
constexpr int kCompRow = kWindow + 1;
constexpr int kFinalRow = kWindow + 1;
constexpr int kPairRowPad = kKeys + 2;  // f2: 16-byte rows, 8 rows at one key hit 32 banks

struct __align__(128) StagedCompShared {
  f2 suffix[kWindow + 2][kPairRowPad];
  float rkey[kWindow + 1 + kRank][kRowPad];
  float4 sq[kKeys / 2];
  float c[kKeys];
  float proj[2][kWindow];
  float cproj[2][kRank];
  float rdecay[kWindow];
  float up;
  StepStage stage;
  StagedComp comp;
};

// Two sequential dot products at once, sum_k a[k] * (b0[k], b1[k]) for
// k = 0..127, with a one fp32 row and b a row of pairs (both 16-byte
// aligned): each key's two products in one packed fma (+0 addend, so that
// the product is rounded before the add) and one packed add.
__device__ __forceinline__ f2 chain_dot2(const float* a, const f2* b) {
  const float4* a4 = reinterpret_cast<const float4*>(a);
  const ulonglong2* b2 = reinterpret_cast<const ulonglong2*>(b);
  f2 acc = pack2(0.0F, 0.0F);
#pragma unroll 8
  for (int k4 = 0; k4 < kKeys / 4; ++k4) {
    const float4 x = a4[k4];
    const ulonglong2 y01 = b2[2 * k4], y23 = b2[2 * k4 + 1];
    acc = add2(acc, mul2_for_add(pack2(x.x, x.x), y01.x));
    acc = add2(acc, mul2_for_add(pack2(x.y, x.y), y01.y));
    acc = add2(acc, mul2_for_add(pack2(x.z, x.z), y23.x));
    acc = add2(acc, mul2_for_add(pack2(x.w, x.w), y23.y));
  }
  return acc;
}

// This thread's share of head h's stage (threads 0..127 issue; one commit).
template <bool kComp, class Shared>
__device__ __forceinline__ void step_stage_issue(const StepParams& p, Shared& sh, uint64_t h,
                                                 int t) {
  StepStage& st = sh.stage;
  const uint4* codes = reinterpret_cast<const uint4*>(p.w.codes + h * kElements);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int i = t + kWinThreads * m;  // chunk j of row v, read coalesced
    const int v = i >> 3, j = i & 7;
    cp_async16(&st.codes[v][j ^ (v & 7)], codes + i);
  }
  // records: 2 x 4 KiB = 512 chunks, 4 per thread
  cp_async16(reinterpret_cast<uint4*>(&st.rkeys[0][0]) + t,
             reinterpret_cast<const uint4*>(p.w.record_keys + h * kWindow * kKeys) + t);
  cp_async16(reinterpret_cast<uint4*>(&st.rkeys[0][0]) + t + kWinThreads,
             reinterpret_cast<const uint4*>(p.w.record_keys + h * kWindow * kKeys) + t + kWinThreads);
  cp_async16(reinterpret_cast<uint4*>(&st.rcorr[0][0]) + t,
             reinterpret_cast<const uint4*>(p.w.record_corrections + h * kWindow * kValues) + t);
  cp_async16(reinterpret_cast<uint4*>(&st.rcorr[0][0]) + t + kWinThreads,
             reinterpret_cast<const uint4*>(p.w.record_corrections + h * kWindow * kValues) + t +
                 kWinThreads);
  if (t < 4) {
    cp_async16(reinterpret_cast<uint4*>(st.rdecay) + t,
               reinterpret_cast<const uint4*>(p.w.record_decay + h * kWindow) + t);
  } else if (t == 4) {
    cp_async16(st.position, p.w.positions + h * kPositionStride);
  } else if (t == 5) {
    cp_async4(&st.log_decay, p.decay + h);
  } else if (t == 6) {
    cp_async4(&st.beta_pair, p.beta + (h & ~uint64_t{1}));
  } else if (t >= 32 && t < 64) {
    const int i = t - 32;
    cp_async16(reinterpret_cast<uint4*>(st.c) + i,
               reinterpret_cast<const uint4*>(p.w.smoothing + h * kKeys) + i);
  } else if (t >= 64 && t < 96) {
    const int i = t - 64;
    cp_async16(reinterpret_cast<uint4*>(st.b) + i,
               reinterpret_cast<const uint4*>(p.w.scales + h * kValues) + i);
  } else if (t >= 96) {
    const int i = t - 96;  // 32 threads: key, query (16 chunks each)
    const uint4* kq = reinterpret_cast<const uint4*>(i < 16 ? p.keys : p.queries) +
                      (h >> 1) * (kKeys / 8);
    cp_async16(reinterpret_cast<uint4*>(i < 16 ? st.key : st.query) + (i & 15), kq + (i & 15));
  }
  if (t >= 7 && t < 7 + 16) {
    const int i = t - 7;
    cp_async16(reinterpret_cast<uint4*>(st.value) + i,
               reinterpret_cast<const uint4*>(p.values + h * kValues) + i);
  }
  if constexpr (kComp) {
    // 2 x 1 KiB = 128 chunks, one per thread
    if (t < 64) {
      cp_async16(reinterpret_cast<uint4*>(sh.comp.stage_ck) + t,
                 reinterpret_cast<const uint4*>(p.w.ck + h * kKeys * kRank) + t);
    } else {
      cp_async16(reinterpret_cast<uint4*>(sh.comp.stage_cv) + (t - 64),
                 reinterpret_cast<const uint4*>(p.w.cv + h * kValues * kRank) + (t - 64));
    }
  }
  cp_async_commit();
}

__global__ void __launch_bounds__(kWinThreads, 4) window_step_staged_kernel(StepParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  StagedStepShared& sh = *reinterpret_cast<StagedStepShared*>(smem_raw);
  StepStage& st = sh.stage;
  const int t = threadIdx.x;
  uint64_t head = blockIdx.x;
  if (head < p.heads) step_stage_issue<false>(p, sh, head, t);
  for (; head < p.heads; head += gridDim.x) {
    const uint64_t next = head + gridDim.x;
    cp_async_wait<0>();
    __syncthreads();  // this head's stage has landed; the previous head is done
    const uint32_t pos = st.position[0];
    const uint64_t rbase = head * kWindow;
    if (pos >= kWindow) {  // block-uniform: every thread read the same word
      if (t == 0) report(nullptr, kStatusWindowFull);
      __syncthreads();  // every thread has read the stage
      if (next < p.heads) step_stage_issue<false>(p, sh, next, t);
      continue;
    }
    const int np = static_cast<int>(pos);
    // ---- consume the stage: codes row t to registers, records, inputs -------
    uint4 zrow[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) zrow[j] = st.codes[t][j ^ (t & 7)];
    const float alpha = expf(st.log_decay);
    const float beta = bf16_to_float(static_cast<uint16_t>(st.beta_pair >> (16 * (head & 1))));
    const float k = bf16_to_float(st.key[t]);
    const float key_t = __fmul_rn(beta, k);
    const float read_t = __fmul_rn(alpha, k);
    const float query_t = __fmul_rn(kQueryScale, bf16_to_float(st.query[t]));
    const float value_t = bf16_to_float(st.value[t]);
    sh.key[t] = key_t;
    sh.query[t] = query_t;
    sh.c[t] = st.c[t];
    const float b_t = st.b[t];
    if (t < kWindow) sh.rdecay[t] = st.rdecay[t];
    float rc[kWindow];
#pragma unroll
    for (int u = 0; u < kWindow; ++u) {
      sh.rkey[u][t] = half_to_float(st.rkeys[u][t]);
      rc[u] = half_to_float(st.rcorr[u][t]);
    }
    __syncthreads();  // the stage is consumed: refill it with the next head
    if (next < p.heads) step_stage_issue<false>(p, sh, next, t);
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
    const int chains = 2 * np + 1;
    if (t < chains) {
      const float* a = sh.key;
      const float* bq = sh.query;
      float* dst = &sh.up;
      if (t < 2 * np) {
        const int r = t / np == 0 ? 0 : 1;
        const int u = t - r * np;
        a = &sh.rkey[u][0];
        bq = &sh.suffix[r][np - 1 - u][0];
        dst = &sh.proj[r][u];
      }
      *dst = chain_dot4(a, bq);
    }
    // ---- boundary readout of column t for both reads ----------------------
    float acc0 = 0.0F, acc1 = 0.0F;
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
    const float correction = __fsub_rn(value_t, out0);
    const float output = __fadd_rn(out1, __fmul_rn(correction, sh.up));
    static_cast<uint16_t*>(p.outputs)[head * kValues + t] =
        __bfloat16_as_ushort(__float2bfloat16_rn(output));
    if (!isfinite(output)) report(nullptr, kStatusWindowNonFinite);
    // ---- append the record -------------------------------------------------
    p.w.record_keys[(rbase + np) * kKeys + t] = float_to_half_bits(key_t);
    p.w.record_corrections[(rbase + np) * kValues + t] = float_to_half_bits(correction);
    if (t == 0) {
      p.w.record_decay[rbase + np] = alpha;
      p.w.positions[head * kPositionStride] = pos + 1u;
    }
    // The barrier at the top of the next head orders these shared-memory
    // reads before the next head's writes.
  }
}

__global__ void __launch_bounds__(kStagedCompThreads, 3)
    window_step_staged_comp_kernel(StepParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  StagedCompShared& sh = *reinterpret_cast<StagedCompShared*>(smem_raw);
  StepStage& st = sh.stage;
  const int t = threadIdx.x;
  const bool reader = t < kKeys;
  uint64_t head = blockIdx.x;
  if (reader && head < p.heads) step_stage_issue<true>(p, sh, head, t);
  for (; head < p.heads; head += gridDim.x) {
    const uint64_t next = head + gridDim.x;
    cp_async_wait<0>();
    __syncthreads();  // this head's stage has landed; the previous head is done
    const uint32_t pos = st.position[0];
    const uint64_t rbase = head * kWindow;
    if (pos >= kWindow) {  // block-uniform: every thread read the same word
      if (t == 0) report(nullptr, kStatusWindowFull);
      __syncthreads();  // every thread has read the stage
      if (reader && next < p.heads) step_stage_issue<true>(p, sh, next, t);
      continue;
    }
    const int np = static_cast<int>(pos);
    uint4 zrow[8];
    float alpha = 0.0F, key_t = 0.0F, read_t = 0.0F, query_t = 0.0F, value_t = 0.0F, b_t = 0.0F;
    float rc[kWindow];
    float cv_t[kRank] = {0.F, 0.F, 0.F, 0.F};
    if (reader) {
      // ---- consume the stage: codes row t to registers, records, inputs -----
#pragma unroll
      for (int j = 0; j < 8; ++j) zrow[j] = st.codes[t][j ^ (t & 7)];
      alpha = expf(st.log_decay);
      const float beta = bf16_to_float(static_cast<uint16_t>(st.beta_pair >> (16 * (head & 1))));
      const float k = bf16_to_float(st.key[t]);
      key_t = __fmul_rn(beta, k);
      read_t = __fmul_rn(alpha, k);
      query_t = __fmul_rn(kQueryScale, bf16_to_float(st.query[t]));
      value_t = bf16_to_float(st.value[t]);
      sh.rkey[kUpdateRow][t] = key_t;
      sh.suffix[kUpdateRow][t] = pack2(query_t, query_t);
      sh.c[t] = st.c[t];
      b_t = st.b[t];
      {
        const uint2 kw = sh.comp.stage_ck[t];
        sh.rkey[kCompRow + 0][t] = half_to_float(kw.x & 0xFFFFu);
        sh.rkey[kCompRow + 1][t] = half_to_float(kw.x >> 16);
        sh.rkey[kCompRow + 2][t] = half_to_float(kw.y & 0xFFFFu);
        sh.rkey[kCompRow + 3][t] = half_to_float(kw.y >> 16);
        const uint2 vw = sh.comp.stage_cv[t];
        cv_t[0] = half_to_float(vw.x & 0xFFFFu);
        cv_t[1] = half_to_float(vw.x >> 16);
        cv_t[2] = half_to_float(vw.y & 0xFFFFu);
        cv_t[3] = half_to_float(vw.y >> 16);
      }
      if (t < kWindow) sh.rdecay[t] = st.rdecay[t];
#pragma unroll
      for (int u = 0; u < kWindow; ++u) {
        sh.rkey[u][t] = half_to_float(st.rkeys[u][t]);
        rc[u] = half_to_float(st.rcorr[u][t]);
      }
    }
    __syncthreads();  // the stage is consumed: refill it with the next head
    if (reader) {
      if (next < p.heads) step_stage_issue<true>(p, sh, next, t);
      // ---- suffix-decayed read and query (thread t = key t) ---------------
      float s0 = read_t, s1 = __fmul_rn(alpha, query_t);
#pragma unroll
      for (int u = kWindow - 1; u >= 0; --u) {  // record u is read with suffix np-1-u
        if (u < np) {
          sh.suffix[np - 1 - u][t] = pack2(s0, s1);
          const float d = sh.rdecay[u];
          s0 = __fmul_rn(s0, d);
          s1 = __fmul_rn(s1, d);
        }
      }
      float* sq = reinterpret_cast<float*>(sh.sq) + 4 * (t >> 1) + (t & 1);
      sq[0] = s0;
      sq[2] = s1;
      sh.suffix[kFinalRow][t] = pack2(s0, s1);
    }
    __syncthreads();
    float acc0 = 0.0F, acc1 = 0.0F;
    if (!reader) {
      // ---- chain warp: two sequential projections per lane -----------------
      // lane u < np: record u against both reads (suffix row np-1-u); lane
      // np: the write key against the query; lanes np+1..np+4 (with
      // compensators): compensator key m against the final suffix pair.
      const int lane = t - kKeys;
      const int chains = np + 1 + kRank;
      if (lane < chains) {
        int arow = kUpdateRow, brow = kUpdateRow;
        float* dst0 = &sh.up;
        float* dst1 = nullptr;
        if (lane < np) {
          arow = lane;
          brow = np - 1 - lane;
          dst0 = &sh.proj[0][lane];
          dst1 = &sh.proj[1][lane];
        } else if (lane > np) {
          const int m = lane - np - 1;
          arow = kCompRow + m;
          brow = kFinalRow;
          dst0 = &sh.cproj[0][m];
          dst1 = &sh.cproj[1][m];
        }
        const f2 acc = chain_dot2(&sh.rkey[arow][0], &sh.suffix[brow][0]);
        *dst0 = lo2(acc);
        if (dst1 != nullptr) *dst1 = hi2(acc);
      }
    } else {
      // ---- boundary readout of column t for both reads --------------------
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
    }
    __syncthreads();
    if (reader) {
      // ---- column t: records newest first, boundary, compensators ---------
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
      {
#pragma unroll
        for (int m = 0; m < kRank; ++m) {
          out0 = __fadd_rn(out0, __fmul_rn(cv_t[m], sh.cproj[0][m]));
          out1 = __fadd_rn(out1, __fmul_rn(cv_t[m], sh.cproj[1][m]));
        }
      }
      const float correction = __fsub_rn(value_t, out0);
      const float output = __fadd_rn(out1, __fmul_rn(correction, sh.up));
      static_cast<uint16_t*>(p.outputs)[head * kValues + t] =
          __bfloat16_as_ushort(__float2bfloat16_rn(output));
      if (!isfinite(output)) report(nullptr, kStatusWindowNonFinite);
      // ---- append the record -------------------------------------------------
      p.w.record_keys[(rbase + np) * kKeys + t] = float_to_half_bits(key_t);
      p.w.record_corrections[(rbase + np) * kValues + t] = float_to_half_bits(correction);
      if (t == 0) {
        p.w.record_decay[rbase + np] = alpha;
        p.w.positions[head * kPositionStride] = pos + 1u;
      }
    }
    // The barrier at the top of the next head orders these shared-memory
    // reads before the next head's writes.
  }
}

template <bool kComp>
inline size_t window_step_staged_smem_bytes() {
  return kComp ? sizeof(StagedCompShared) : sizeof(StagedStepShared);
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
      // Compensator and record products multiply two binary16 values, exact
      // in fp32, so RN(x + RN(a b)) is fma(a, b, x).
      if (comp) {
        const float4 cvv = ex.cv[v];
        value = __fmaf_rn(ck_t.x, cvv.x, value);
        value = __fmaf_rn(ck_t.y, cvv.y, value);
        value = __fmaf_rn(ck_t.z, cvv.z, value);
        value = __fmaf_rn(ck_t.w, cvv.w, value);
      }
#pragma unroll
      for (int u = 0; u < kWindow; ++u) {
        if (u < np) value = __fmaf_rn(rk[u], ex.rc[u][v], __fmul_rn(rd[u], value));
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
// straight to the workspace, one 256-thread CTA per head in two passes of 64
// rows.  Lane l = t mod 16 owns keys 4l..4l+3 and 64+4l..64+4l+3, and thread
// t owns rows 4 (t / 16) + i (i < 4) of each pass: 32 elements, held in
// registers as 16 adjacent key pairs of the provider layout [v][k] while the
// whole window is applied.  Records are the outer loop, so each record's
// decay, key quads and row corrections are one broadcast load per use and
// serve 16 element pairs.  The reference's update RN(RN(d S) + RN(k c)) is
// one rounded product and one fma per element in packed fp32x2 arithmetic,
// because k c (two binary16 values) is exact in fp32.  Every element follows
// the reference order (dequantize, compensators by rank, records oldest
// first); the 16-lane row segments keep both the shared-memory key loads and
// the 16-byte workspace stores contiguous.
constexpr int kDenseThreads = 256;
constexpr int kDenseLanes = 16;                                             // threads across a row
constexpr int kDenseRows = 4;                                               // rows per thread per pass
constexpr int kDenseRowsPerPass = kDenseThreads / kDenseLanes * kDenseRows;  // 64
constexpr int kDensePasses = kValues / kDenseRowsPerPass;                   // 2
static_assert(kDenseLanes * 8 == kKeys && kDensePasses * kDenseRowsPerPass == kValues,
              "dense refit tile");
static_assert(kWindow * kDenseLanes == kDenseThreads, "one thread per record chunk of 8");

struct __align__(16) WindowDenseShared {
  float rk[kWindow][kKeys];      // record keys (fp32), u < position only
  float rc[kWindow][kValues];    // record corrections (fp32), u < position only
  f2 d[kWindow];                 // (decay, decay), u < position only
  float ck[kRank][kKeys];        // compensator keys, rank-major (compensated boundary)
  f2 cv[kRank][kValues];         // (V, V) per rank and row
  // Stage filled by cp.async one pass ahead of its use.
  int8_t codes[kElements];                     // [v][k]: rows 0..63 pass 0, 64..127 pass 1
  uint16_t raw_keys[kWindow][kKeys];           // next head's records (binary16)
  uint16_t raw_corrections[kWindow][kValues];
  float raw_decay[kWindow];
  uint32_t raw_position[4];                    // positions[head][0..3]
  float c[2][kKeys];                           // smoothing, by head parity
  float b[2][kValues];                         // scales, by head parity
};

// This thread's share of head h's records, decays, position, smoothing and
// scales (into parity slot `par`); one commit group per call site.
__device__ __forceinline__ void dense_stage_head(const FoldParams& p, WindowDenseShared& sh,
                                                 uint64_t h, int par, int t) {
  cp_async16(reinterpret_cast<uint4*>(&sh.raw_keys[0][0]) + t,
             reinterpret_cast<const uint4*>(p.w.record_keys + h * kWindow * kKeys) + t);
  cp_async16(reinterpret_cast<uint4*>(&sh.raw_corrections[0][0]) + t,
             reinterpret_cast<const uint4*>(p.w.record_corrections + h * kWindow * kValues) + t);
  if (t < kWindow / 4) {
    cp_async16(reinterpret_cast<float4*>(sh.raw_decay) + t,
               reinterpret_cast<const float4*>(p.w.record_decay + h * kWindow) + t);
  } else if (t == kWindow / 4) {
    cp_async16(sh.raw_position, p.w.positions + h * kPositionStride);
  } else if (t >= 32 && t < 32 + kKeys / 4) {
    cp_async16(reinterpret_cast<float4*>(sh.c[par]) + (t - 32),
               reinterpret_cast<const float4*>(p.w.smoothing + h * kKeys) + (t - 32));
  } else if (t >= 64 && t < 64 + kValues / 4) {
    cp_async16(reinterpret_cast<float4*>(sh.b[par]) + (t - 64),
               reinterpret_cast<const float4*>(p.w.scales + h * kValues) + (t - 64));
  }
}
// This thread's share of head h's codes for one pass (64 rows, 8 KiB).
__device__ __forceinline__ void dense_stage_codes(const FoldParams& p, WindowDenseShared& sh,
                                                  uint64_t h, int pass, int t) {
  const uint4* src = reinterpret_cast<const uint4*>(p.w.codes + h * kElements) +
                     pass * (kElements / 2 / 16);
  uint4* dst = reinterpret_cast<uint4*>(sh.codes) + pass * (kElements / 2 / 16);
  cp_async16(dst + t, src + t);
  cp_async16(dst + t + kDenseThreads, src + t + kDenseThreads);
}
static_assert(kElements / 2 / 16 == 2 * kDenseThreads, "two 16-byte code chunks per thread");
static_assert(kWindow * kKeys * 2 / 16 == kDenseThreads, "one 16-byte record chunk per thread");

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

// The dequantized boundary of one row segment of four keys, before any
// compensator: codes word `zw`, smoothing pairs (c0, c1), (c2, c3) in `c`,
// scale pair `bb`.  Every later use of the result is an fma addend or
// multiplicand, which no contraction can merge with this product.
__device__ __forceinline__ void dense_boundary(uint32_t zw, float4 c, bool c_safe, f2 bb,
                                               f2& s01, f2& s23) {
  f2 z01, z23;
  unpack_codes(zw, z01, z23);
  const f2 cz01 = mul2(lo_pair(c), z01), cz23 = mul2(hi_pair(c), z23);
  f2 q01 = div127x2(cz01), q23 = div127x2(cz23);
  if (!c_safe) {  // a smoothing below 2^-112 in magnitude
    q01 = div127x2_any(cz01);
    q23 = div127x2_any(cz23);
  }
  s01 = mul2(q01, bb);
  s23 = mul2(q23, bb);
}

// One pass (64 rows) of this thread's tile: dequantize, compensators,
// records, store; returns the finiteness accumulator.
template <bool kComp>
__device__ __forceinline__ f2 dense_pass(const WindowDenseShared& sh, int pass, int par, int np,
                                         bool c_safe, int ka, int kb, int row0, float* rows,
                                         f2 flags) {
  const int v0 = pass * kDenseRowsPerPass + row0;
  uint32_t za[kDenseRows], zb[kDenseRows];
#pragma unroll
  for (int i = 0; i < kDenseRows; ++i) {
    za[i] = *reinterpret_cast<const uint32_t*>(&sh.codes[(v0 + i) * kKeys + ka]);
    zb[i] = *reinterpret_cast<const uint32_t*>(&sh.codes[(v0 + i) * kKeys + kb]);
  }
  const float4 ca = *reinterpret_cast<const float4*>(&sh.c[par][ka]);
  const float4 cb = *reinterpret_cast<const float4*>(&sh.c[par][kb]);
  const float4 b4 = *reinterpret_cast<const float4*>(&sh.b[par][v0]);
  const float bs[kDenseRows] = {b4.x, b4.y, b4.z, b4.w};
  f2 s[kDenseRows][4];  // row i: keys (ka, ka+1), (ka+2, ka+3), (kb, kb+1), (kb+2, kb+3)
#pragma unroll
  for (int i = 0; i < kDenseRows; ++i) {
    const f2 bb = pack2(bs[i], bs[i]);
    dense_boundary(za[i], ca, c_safe, bb, s[i][0], s[i][1]);
    dense_boundary(zb[i], cb, c_safe, bb, s[i][2], s[i][3]);
  }
  if constexpr (kComp) {  // compensators by rank: S = RN(S + RN(K[k][m] V[v][m]))
#pragma unroll
    for (int m = 0; m < kRank; ++m) {
      const float4 k4a = *reinterpret_cast<const float4*>(&sh.ck[m][ka]);
      const float4 k4b = *reinterpret_cast<const float4*>(&sh.ck[m][kb]);
      const float4 v01 = *reinterpret_cast<const float4*>(&sh.cv[m][v0]);
      const float4 v23 = *reinterpret_cast<const float4*>(&sh.cv[m][v0 + 2]);
      const f2 kk[4] = {lo_pair(k4a), hi_pair(k4a), lo_pair(k4b), hi_pair(k4b)};
      const f2 vv[kDenseRows] = {lo_pair(v01), hi_pair(v01), lo_pair(v23), hi_pair(v23)};
      // K and V are binary16 too: the product is exact, so the add is one fma.
#pragma unroll
      for (int i = 0; i < kDenseRows; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fma2(kk[j], vv[i], s[i][j]);
      }
    }
  }
  // Records oldest first: S = RN(RN(d S) + RN(key correction)).  Key and
  // correction are binary16 values (11-bit significands, magnitudes in
  // [2^-24, 65504]), so their product has at most 22 significant bits and
  // lies in fp32's normal range: RN(key correction) = key correction, and the
  // update is exactly fma(key, correction, RN(d S)) -- two operations per
  // element instead of three, for every input including zeros of either
  // sign, infinities and NaN.
#pragma unroll 8
  for (int u = 0; u < np; ++u) {
    const f2 d = sh.d[u];
    const float4 k4a = *reinterpret_cast<const float4*>(&sh.rk[u][ka]);
    const float4 k4b = *reinterpret_cast<const float4*>(&sh.rk[u][kb]);
    const float4 r4 = *reinterpret_cast<const float4*>(&sh.rc[u][v0]);
    const f2 kk[4] = {lo_pair(k4a), hi_pair(k4a), lo_pair(k4b), hi_pair(k4b)};
    const f2 rr[kDenseRows] = {pack2(r4.x, r4.x), pack2(r4.y, r4.y), pack2(r4.z, r4.z),
                               pack2(r4.w, r4.w)};
#pragma unroll
    for (int i = 0; i < kDenseRows; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = fma2(kk[j], rr[i], mul2(d, s[i][j]));
    }
  }
  const f2 zero = pack2(0.0F, 0.0F);
#pragma unroll
  for (int i = 0; i < kDenseRows; ++i) {
    float* row = rows + (v0 + i) * kKeys;
    __stcg(reinterpret_cast<float4*>(row + ka),
           make_float4(lo2(s[i][0]), hi2(s[i][0]), lo2(s[i][1]), hi2(s[i][1])));
    __stcg(reinterpret_cast<float4*>(row + kb),
           make_float4(lo2(s[i][2]), hi2(s[i][2]), lo2(s[i][3]), hi2(s[i][3])));
#pragma unroll
    for (int j = 0; j < 4; ++j) flags = fma2(s[i][j], zero, flags);
  }
  return flags;
}

// Four CTAs per SM (64 registers) for the quant-only boundary; the
// compensated one keeps three so that its rank loop does not spill.
//
// Software pipeline per CTA (cp.async, 16-byte copies, each thread waiting
// on its own commit groups, a block barrier publishing them): the next
// head's records, position, smoothing and scales are staged while this
// head's first pass runs, and each pass's 64 code rows one pass ahead.  The
// commit groups stay in issue order: [head h + pass-0 codes], [pass-1 codes],
// then per head [next head], [next pass-0 codes], [next pass-1 codes]
// (empty groups past the last head keep the count uniform).
template <bool kComp>
__global__ void __launch_bounds__(kDenseThreads, kComp ? 3 : 4)
    window_dense_kernel(FoldParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  WindowDenseShared& sh = *reinterpret_cast<WindowDenseShared*>(smem_raw);
  const int t = threadIdx.x;
  const int lane = t % kDenseLanes;
  const int ka = 4 * lane, kb = kKeys / 2 + 4 * lane;
  const int row0 = kDenseRows * (t / kDenseLanes);
  uint64_t head = blockIdx.x;
  if (head < p.heads) {
    dense_stage_head(p, sh, head, 0, t);
    dense_stage_codes(p, sh, head, 0, t);
    cp_async_commit();
    dense_stage_codes(p, sh, head, 1, t);
    cp_async_commit();
  }
  for (int par = 0; head < p.heads; head += gridDim.x, par ^= 1) {
    const uint64_t next = head + gridDim.x;
    const bool has_next = next < p.heads;
    cp_async_wait<1>();  // this head's records and pass-0 codes (pass-1 codes may be in flight)
    __syncthreads();
    const uint32_t pos_raw = sh.raw_position[0];
    const int np = pos_raw < static_cast<uint32_t>(kWindow) ? static_cast<int>(pos_raw) : kWindow;
    const uint64_t rbase = head * kWindow;
    // ---- records (u < position) to fp32: 8 keys and 8 corrections a thread --
    {
      const int u = t / kDenseLanes, k8 = 8 * (t % kDenseLanes);
      if (u < np) {
        const uint4 kw = *reinterpret_cast<const uint4*>(&sh.raw_keys[u][k8]);
        const uint4 cw = *reinterpret_cast<const uint4*>(&sh.raw_corrections[u][k8]);
        const uint32_t kws[4] = {kw.x, kw.y, kw.z, kw.w};
        const uint32_t cws[4] = {cw.x, cw.y, cw.z, cw.w};
        float4* rk = reinterpret_cast<float4*>(&sh.rk[u][k8]);
        float4* rc = reinterpret_cast<float4*>(&sh.rc[u][k8]);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          rk[j] = make_float4(half_to_float(kws[2 * j] & 0xFFFFu), half_to_float(kws[2 * j] >> 16),
                              half_to_float(kws[2 * j + 1] & 0xFFFFu),
                              half_to_float(kws[2 * j + 1] >> 16));
          rc[j] = make_float4(half_to_float(cws[2 * j] & 0xFFFFu), half_to_float(cws[2 * j] >> 16),
                              half_to_float(cws[2 * j + 1] & 0xFFFFu),
                              half_to_float(cws[2 * j + 1] >> 16));
        }
      }
      if (t < np) sh.d[t] = pack2(sh.raw_decay[t], sh.raw_decay[t]);
    }
    if constexpr (kComp) {
      if (t < kKeys) {
        const uint2 kw = __ldg(reinterpret_cast<const uint2*>(p.w.ck + (head * kKeys + t) * kRank));
        sh.ck[0][t] = half_to_float(kw.x & 0xFFFFu);
        sh.ck[1][t] = half_to_float(kw.x >> 16);
        sh.ck[2][t] = half_to_float(kw.y & 0xFFFFu);
        sh.ck[3][t] = half_to_float(kw.y >> 16);
      } else {
        const int v = t - kKeys;
        const uint2 vw = __ldg(reinterpret_cast<const uint2*>(p.w.cv + (head * kValues + v) * kRank));
        const float vm[kRank] = {half_to_float(vw.x & 0xFFFFu), half_to_float(vw.x >> 16),
                                 half_to_float(vw.y & 0xFFFFu), half_to_float(vw.y >> 16)};
#pragma unroll
        for (int m = 0; m < kRank; ++m) sh.cv[m][v] = pack2(vm[m], vm[m]);
      }
    }
    __syncthreads();  // converted records visible; the record stage is free
    if (has_next) dense_stage_head(p, sh, next, par ^ 1, t);
    cp_async_commit();
    // ---- the window is about to be folded: clear it ------------------------
    {
      const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
      reinterpret_cast<uint4*>(p.w.record_keys + rbase * kKeys)[t] = z4;
      reinterpret_cast<uint4*>(p.w.record_corrections + rbase * kValues)[t] = z4;
      if (t < kWindow) p.w.record_decay[rbase + t] = 0.0F;
      if (t == 0) p.w.positions[head * kPositionStride] = 0u;
      if (t < kKeys) {
        reinterpret_cast<uint2*>(p.next_ck + (head * kKeys + t) * kRank)[0] = make_uint2(0u, 0u);
      } else {
        reinterpret_cast<uint2*>(p.next_cv + (head * kValues + t - kKeys) * kRank)[0] =
            make_uint2(0u, 0u);
      }
    }
    // With this thread's smoothing at least 2^-112 in magnitude, zero or not
    // finite, every product c z is zero or at least 2^-112 in magnitude (codes
    // are integers), where the two-term reciprocal division is exact;
    // otherwise each product is checked.
    bool c_safe = true;
    {
      const float4 ca = *reinterpret_cast<const float4*>(&sh.c[par][ka]);
      const float4 cb = *reinterpret_cast<const float4*>(&sh.c[par][kb]);
      const float cs[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c_safe = c_safe && (fabsf(cs[j]) >= kDiv127Safe || cs[j] == 0.0F || cs[j] != cs[j]);
      }
    }
    // x * 0 + flags stays +0 while every element is finite and becomes NaN
    // otherwise (x * 0 is NaN exactly for infinite or NaN x).
    float* rows = p.workspace + head * kElements;
    f2 flags = dense_pass<kComp>(sh, 0, par, np, c_safe, ka, kb, row0, rows, pack2(0.0F, 0.0F));
    cp_async_wait<1>();  // this head's pass-1 codes (the next head's records may be in flight)
    __syncthreads();     // pass 0 done everywhere: its code rows are free
    if (has_next) dense_stage_codes(p, sh, next, 0, t);
    cp_async_commit();
    flags = dense_pass<kComp>(sh, 1, par, np, c_safe, ka, kb, row0, rows, flags);
    const bool finite = lo2(flags) == 0.0F && hi2(flags) == 0.0F;
    // Also the barrier before pass-1 code rows and shared memory are reused.
    if (__syncthreads_or(!finite) != 0 && t == 0) report(nullptr, kStatusWindowNonFinite);
    if (has_next) dense_stage_codes(p, sh, next, 1, t);
    cp_async_commit();
  }
}

inline size_t window_dense_smem_bytes() { return sizeof(WindowDenseShared); }

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
  int step_staged[2] = {};  // [comp]
  int fold = 0;
  int window_dense[2] = {};  // [compensated]
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

template <bool kComp>
inline cudaError_t prepare_staged_variant(int* blocks) {
  const auto kernel = kComp ? window_step_staged_comp_kernel : window_step_staged_kernel;
  const int threads = kComp ? kStagedCompThreads : kWinThreads;
  const size_t smem = window_step_staged_smem_bytes<kComp>();
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, kernel, threads, smem);
}

inline cudaError_t prepare_window(WindowBlocks* b) {
  cudaError_t err;
  if ((err = prepare_staged_variant<false>(&b->step_staged[0])) != cudaSuccess) return err;
  if ((err = prepare_staged_variant<true>(&b->step_staged[1])) != cudaSuccess) return err;
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
  const int dense_smem = static_cast<int>(window_dense_smem_bytes());
  err = cudaFuncSetAttribute(window_dense_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             dense_smem);
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(window_dense_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             dense_smem);
  if (err != cudaSuccess) return err;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b->window_dense[0], window_dense_kernel<false>,
                                                      kDenseThreads, dense_smem);
  if (err != cudaSuccess) return err;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b->window_dense[1], window_dense_kernel<true>,
                                                      kDenseThreads, dense_smem);
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(dense_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(DenseStepShared)));
  if (err != cudaSuccess) return err;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b->dense, dense_step_kernel, kWinThreads,
                                                       sizeof(DenseStepShared));
}

inline cudaError_t launch_window_step_staged(bool comp, const StepParams& p, int grid,
                                             cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.stream = stream;
  if (comp) {
    cfg.blockDim = dim3(kStagedCompThreads);
    cfg.dynamicSmemBytes = window_step_staged_smem_bytes<true>();
    return cudaLaunchKernelEx(&cfg, window_step_staged_comp_kernel, p);
  }
  cfg.blockDim = dim3(kWinThreads);
  cfg.dynamicSmemBytes = window_step_staged_smem_bytes<false>();
  return cudaLaunchKernelEx(&cfg, window_step_staged_kernel, p);
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
  const size_t smem = window_dense_smem_bytes();
  if (p.w.ck != nullptr) {
    window_dense_kernel<true><<<grid, kDenseThreads, smem, stream>>>(p);
  } else {
    window_dense_kernel<false><<<grid, kDenseThreads, smem, stream>>>(p);
  }
  return cudaGetLastError();
}

inline cudaError_t launch_dense_step(const DenseStepParams& p, int grid, cudaStream_t stream) {
  dense_step_kernel<<<grid, kWinThreads, sizeof(DenseStepShared), stream>>>(p);
  return cudaGetLastError();
}

}  // namespace gdnsc
