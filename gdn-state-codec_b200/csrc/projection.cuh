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
//  * capsule codes [k][v]: every warp streams its heads' codes through its own
//    two-stage shared-memory ring, 64 code rows (8 KiB) per stage, each stage
//    filled by one bulk copy (cp.async.bulk, mbarrier completion, this GPU's
//    own memory, no multicast).  While one half of a head is accumulated the
//    other half is in flight, and the smoothing, query and scales of the next
//    head are fetched one head ahead, so a warp never waits on a global load
//    inside a head.  A lane reads its four codes of row k with one
//    conflict-free 32-bit shared load.
//  * provider codes [v][k]: a lane's four outputs are four code rows, so the
//    warp loads its 16 KiB head with coalesced 128-bit loads, stores it to
//    shared memory with an XOR swizzle on 16-byte chunks and reads its rows
//    back conflict-free.
#pragma once

#include "codec_device.cuh"

namespace gdnsc {

constexpr int kPThreads = 128;
constexpr int kPWarps = kPThreads / 32;

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
  uint64_t wait_limit_ns = kWaitLimitNs;  // limit of every bounded wait
  // Test support (encoded_projection_wait_selftest_v1, capsule codes): arm
  // each ring stage with its bytes but issue no copy, so every wait runs out
  // with nothing in flight.
  uint32_t arm_only = 0u;
};

// Capsule codes: per-warp ring of kRingStages stages of kRingRows code rows.
// A warp's positions t = 0, 1, 2, ... are (its item number t / kRingPerHead,
// rows (t % kRingPerHead) * kRingRows ..); position t uses stage
// t % kRingStages, whose mbarrier completes once per use (phase parity
// (t / kRingStages) & 1).  Sized by A/B timing on B200 (61,440 heads):
// 64 rows x 2 stages beat 32 x 2, 32 x 3, 64 x 3 and 128 x 2.
constexpr int kRingRows = 64;
constexpr int kRingStages = 2;
constexpr int kRingPerHead = kKeys / kRingRows;
constexpr uint32_t kRingBytes = kRingRows * kValues;  // int8 codes per stage
// With as many stages as parts per head, position t + kRingStages is the same
// part of the warp's next item, whose head the warp has already resolved.
static_assert(kRingStages == kRingPerHead, "the ring holds exactly one head");
struct __align__(128) ProjectWarpShared {
  uint32_t ring[kRingStages][kRingBytes / 4];
  float2 cx[kKeys];                 // (c_k, x_k) of the current head
  uint64_t bar[kRingStages];
};
struct ProjectShared {
  ProjectWarpShared warp[kPWarps];
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
  ProjectWarpShared& ws = sh.warp[warp];
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kPWarps;
  const uint64_t first = static_cast<uint64_t>(blockIdx.x) * kPWarps + warp;
  if (lane == 0) {
    for (int s = 0; s < kRingStages; ++s) mbar_init(&ws.bar[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  const uint64_t policy = evict_first_policy();
  // Head of an item (-1: padding, an invalid id (*bad) or past the end).
  auto resolve = [&](uint64_t item, bool* bad) -> int64_t {
    *bad = false;
    return item < p.items ? resolve_item(p.map, item, bad) : -1;
  };
  auto item_of = [&](uint64_t t) { return first + (t / kRingPerHead) * stride; };
  // Lane 0 issues position t of head `head` (see ProjectWarpShared).  A
  // skipped head (PAD or invalid id) arrives with zero bytes, so its stage
  // completes the same phase without a copy and the consumer waits
  // uniformly; positions past the last item are not issued.
  auto issue = [&](uint64_t t, int64_t head) {
    if (item_of(t) >= p.items) return;
    const int stage = static_cast<int>(t % kRingStages);
    fence_proxy_async();  // the stage's previous reads precede the copy
    if (head < 0) {
      mbar_expect_tx(&ws.bar[stage], 0);
    } else {
      mbar_expect_tx(&ws.bar[stage], kRingBytes);
      if (p.arm_only == 0u) bulk_load(ws.ring[stage],
                p.codes + static_cast<uint64_t>(head) * kElements +
                    static_cast<uint64_t>(t % kRingPerHead) * kRingBytes,
                kRingBytes, &ws.bar[stage], policy);
    }
  };
  bool next_bad = false;
  int64_t next_head = resolve(first, &next_bad);
  if (lane == 0) {
    for (int t = 0; t < kRingStages; ++t) issue(t, next_head);
  }
  uint64_t pos = 0;  // next position to consume
  // A lane whose bounded wait expires stops computing and issuing; the warp
  // agrees on the failure once per head (lanes stay converged until then).
  bool failed = false;
  int fail_part = kRingPerHead;  // first part of the head whose wait expired
  // Smoothing, query and scales of the next item, fetched one head ahead.
  float4 c_next = make_float4(0.F, 0.F, 0.F, 0.F), b_next = c_next;
  uint2 q_next = make_uint2(0u, 0u);
  auto fetch = [&](uint64_t item, int64_t head) {
    if (head < 0) return;
    c_next = __ldg(reinterpret_cast<const float4*>(p.smoothing + static_cast<uint64_t>(head) * kKeys) + lane);
    b_next = __ldg(reinterpret_cast<const float4*>(p.scales + static_cast<uint64_t>(head) * kValues) + lane);
    q_next = __ldg(reinterpret_cast<const uint2*>(p.queries + item * kKeys) + lane);
  };
  fetch(first, next_head);
  for (uint64_t item = first; item < p.items; item += stride) {
    const int64_t head = next_head;
    const bool bad = next_bad;
    next_head = resolve(item + stride, &next_bad);
    // The output address is formed here, ahead of the ring loop: forming it
    // after the loop measured 12 % slower on B200.
    float* out = p.outputs + item * kValues + 4 * lane;
    const float4 c4 = c_next;
    const float4 x4 = bf16x4_to_float4(q_next);
    const float4 b4 = b_next;
    fetch(item + stride, next_head);
    __syncwarp();  // the previous head's readers are done with cx / kr
    reinterpret_cast<float4*>(ws.cx)[2 * lane] = make_float4(c4.x, x4.x, c4.y, x4.y);
    reinterpret_cast<float4*>(ws.cx)[2 * lane + 1] = make_float4(c4.z, x4.z, c4.w, x4.w);
    if (kCompensated && head >= 0) {
      const float4* kp = reinterpret_cast<const float4*>(p.compensator_keys) +
                         static_cast<uint64_t>(head) * kKeys;
#pragma unroll
      for (int i = 0; i < 4; ++i) sh.kr[warp][4 * lane + i] = __ldg(kp + 4 * lane + i);
    }
    __syncwarp();
    f2 a01 = pack2(0.F, 0.F), a23 = a01, kp01 = a01, kp23 = a01;
    const float4* cx2 = reinterpret_cast<const float4*>(ws.cx);  // rows k, k + 1
#pragma unroll 1
    for (int part = 0; part < kRingPerHead; ++part, ++pos) {
      const int stage = static_cast<int>(pos % kRingStages);
      const uint32_t parity = static_cast<uint32_t>((pos / kRingStages) & 1u);
      if (!failed && !mbar_wait_bounded(&ws.bar[stage], parity, p.wait_limit_ns)) {
        failed = true;
        fail_part = part;
      }
      if (head >= 0 && !failed) {
        const uint32_t* rows = ws.ring[stage] + lane;
#pragma unroll
        for (int r0 = 0; r0 < kRingRows; r0 += 8) {
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = rows[(r0 + i) * 32];
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            const int k = part * kRingRows + r0 + i;
            const float4 cc = cx2[k >> 1];
            f2 z01, z23;
            unpack_codes(w[i], z01, z23);
            accumulate(a01, a23, z01, z23, cc.x, cc.y);
            unpack_codes(w[i + 1], z01, z23);
            accumulate(a01, a23, z01, z23, cc.z, cc.w);
            if (kCompensated) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const float4 kk = sh.kr[warp][k + h];
                const float x = h == 0 ? cc.y : cc.w;
                const f2 xx = pack2(x, x);
                kp01 = add2(kp01, mul2_for_add(pack2(kk.x, kk.y), xx));
                kp23 = add2(kp23, mul2_for_add(pack2(kk.z, kk.w), xx));
              }
            }
          }
        }
      }
      __syncwarp();  // every lane is done with this stage
      if (lane == 0 && !failed) issue(pos + kRingStages, next_head);
    }
    if (__any_sync(0xffffffffu, failed)) {
      // A bounded wait expired.  Lane 0 reports it and lets every copy that
      // may still be in flight land (again bounded) before the warp leaves,
      // so that no bulk copy targets the block's shared memory after it
      // exits: positions from the first one any lane gave up on up to those
      // lane 0 issued.  Outputs of this launch are then unspecified.
      const uint64_t head_pos = pos - kRingPerHead;
      const uint64_t from = head_pos + static_cast<uint32_t>(
                                           __reduce_min_sync(0xffffffffu, static_cast<uint32_t>(fail_part)));
      if (lane == 0) {
        report(p.status, kStatusWaitTimeout);
        const uint64_t to = (failed ? head_pos + fail_part : pos) + kRingStages;
        for (uint64_t t = from; t < to; ++t) {
          if (item_of(t) >= p.items) break;
          (void)mbar_wait_bounded(&ws.bar[t % kRingStages], static_cast<uint32_t>((t / kRingStages) & 1u),
                                 p.wait_limit_ns);
        }
      }
      return;
    }
    if (head < 0) {
      if (bad && lane == 0) report(p.status, kStatusBadSlot);
      *reinterpret_cast<float4*>(out) = make_float4(0.F, 0.F, 0.F, 0.F);
      continue;
    }
    // Every lane holds all four rank projections p_r (identical chains).
    const float* vbase = kCompensated
                             ? p.compensator_values + (static_cast<uint64_t>(head) * kValues + 4 * lane) * kRank
                             : nullptr;
    __stcs(reinterpret_cast<float4*>(out), finish_outputs(a01, a23, b4, kCompensated, kp01, kp23, vbase));
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
  return compensated ? sizeof(ProjectShared) : offsetof(ProjectShared, kr);  // kr last
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
