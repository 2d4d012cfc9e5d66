// codec_device.cuh -- device-side building blocks shared by the GDN state
// codec kernels (sm_100a only).
//
// One "head" is one GDN recurrent-state matrix with d_k = d_v = 128 stored as
// fp32 (64 KiB).  Its encoded form is int8 codes [128 x 128] (16 KiB) plus a
// per-key smoothing vector c[128] and a per-value scale vector b[128] (fp32).
// Two element orders exist for the same matrix:
//   capsule  [key, value] -- native/src capsule layout (capsule.cpp:190-251)
//   provider [value, key] -- vLLM ssm_state layout (runtime.py:460-547)
//
// Arithmetic contract: every value the kernels produce is bit-identical to
// the reference's portable C++ codec (native/src/gdn_state_codec_state_capsule
// .cpp).  The library is compiled with -fmad=false so that nvcc never fuses
// a multiply and an add on its own; the only FMAs are the explicit ones in
// this file, each used inside an error-free or proven-exact construction.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace gdnsc {

constexpr int kKeys = 128;
constexpr int kValues = 128;
constexpr int kElements = kKeys * kValues;  // 16384 per head
constexpr int kRank = 4;                    // compensator rank (capsule.h:15)
constexpr float kQuantMax = 127.0F;         // capsule.cpp:20
constexpr float kSmoothingFloor = 1.0e-8F;  // capsule.h:17

// Status bits a kernel ORs into the caller's status word (when one is given)
// and into the library's sticky per-device error word.  Each condition has
// its own bit.
constexpr uint32_t kStatusBadSlot = 1u;          // bit 0: slot id outside [-1, num_slots)
constexpr uint32_t kStatusWaitTimeout = 2u;      // bit 1: a bounded wait gave up
constexpr uint32_t kStatusFitNonFinite = 4u;     // bit 2: full-codec fit saw non-finite data
constexpr uint32_t kStatusWindowFull = 8u;       // bit 3: a decode step found a full window
constexpr uint32_t kStatusWindowNonFinite = 16u; // bit 4: non-finite decode output or refit state

// --------------------------------------------------------------------------
// Packed fp32x2 arithmetic (PTX ISA 8.6, sm_100a): two IEEE round-to-nearest
// operations per instruction, same results as the scalar .rn forms.
using f2 = unsigned long long;

__device__ __forceinline__ f2 pack2(float lo, float hi) {
  f2 d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ float lo2(f2 v) {
  return __uint_as_float(static_cast<uint32_t>(v));
}
__device__ __forceinline__ float hi2(f2 v) {
  return __uint_as_float(static_cast<uint32_t>(v >> 32));
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Separately rounded product destined for an add.  ptxas (CUDA 12.9) turns a
// single-use mul.rn.f32x2 whose result feeds add.rn.f32x2 into one fused
// multiply-add, despite the explicit rounding modifier and -fmad=false (found
// by a GPU rounding check: every element where fma != mul-then-add followed
// the fma).  An fma with a +0 addend is not contracted further and equals
// RN(a * b), except that a -0 product comes out as +0.  Adding +0 instead of
// -0 changes a sum only when the running sum is -0, and a round-to-nearest sum
// that starts at +0 is never -0 (x + y = -0 needs x = y = -0), so every
// accumulation below that starts at +0 is bit-identical to the reference's.
__device__ __forceinline__ f2 mul2_for_add(f2 a, f2 b) {
  return fma2(a, b, pack2(0.0F, 0.0F));
}

// --------------------------------------------------------------------------
// int8 code <-> float without the conversion pipe.  For a word holding four
// int8 codes, xor 0x80 turns each into the biased byte z + 128; placing that
// byte under the exponent of 2^23 gives the float 2^23 + z + 128 exactly, and
// subtracting 2^23 + 128 recovers z exactly.
constexpr uint32_t kCodeBias = 0x80808080u;
constexpr float kCodeMagic = 8388736.0F;  // 2^23 + 128

__device__ __forceinline__ float code_magic(uint32_t biased_word, int byte) {
  return __uint_as_float(__byte_perm(biased_word, 0x4B000000u, 0x7540u | byte));
}
// Four codes -> two packed pairs (z0, z1), (z2, z3).
__device__ __forceinline__ void unpack_codes(uint32_t word, f2& z01, f2& z23) {
  const uint32_t biased = word ^ kCodeBias;
  const f2 magic = pack2(kCodeMagic, kCodeMagic);
  z01 = sub2(pack2(code_magic(biased, 0), code_magic(biased, 1)), magic);
  z23 = sub2(pack2(code_magic(biased, 2), code_magic(biased, 3)), magic);
}

// Round-to-nearest integer through the 1.5 * 2^23 magic constant: for
// |t| < 2^22, t + 1.5*2^23 rounds t to an integer n (ties to even) and the low
// byte of the sum's bit pattern is n as two's complement int8.
constexpr float kRoundMagic = 12582912.0F;  // 1.5 * 2^23

// --------------------------------------------------------------------------
// Exact division by the constant 127 with a two-term reciprocal
// (Brisebarre, Muller, Raina, "Accelerating correctly rounded floating-point
// division when the divisor is known in advance", IEEE Trans. Computers 53(8),
// 2004): q = fma(a, zh, a * zl) with zh = RN(1/127), zl = RN(1/127 - zh).
// Checked exhaustively over every float: it equals the IEEE quotient a / 127
// for all |a| >= 2^-112, zero, infinities and NaN (tests/test_division.py
// re-runs the sweep on the CPU; the GPU parity tests compare against the
// oracle's IEEE division).  Callers guard the |a| < 2^-112 range.
constexpr float kInv127Hi = 0x1.020408p-7F;
constexpr float kInv127Lo = 0x1.020408p-35F;
constexpr float kDiv127Safe = 0x1p-112F;

__device__ __forceinline__ float div127(float a) {
  return __fmaf_rn(a, kInv127Hi, __fmul_rn(a, kInv127Lo));
}
__device__ __forceinline__ f2 div127x2(f2 a) {
  return fma2(a, pack2(kInv127Hi, kInv127Hi),
              mul2(a, pack2(kInv127Lo, kInv127Lo)));
}
// a / 127 exactly for every float a.
__device__ __forceinline__ float div127_any(float a) {
  return (fabsf(a) >= kDiv127Safe || a == 0.0F) ? div127(a) : __fdiv_rn(a, 127.0F);
}

// --------------------------------------------------------------------------
// Correctly rounded quotients a / c for many a and one divisor c, from a
// two-term reciprocal y = RN(1/c), yl = RN((1 - c y) y) and nc = -c, with one
// fused-multiply-add correction:
//   q0 = RN(a y + RN(a yl))   faithful (within 1 ulp of a / c)
//   q  = RN(q0 + (a - q0 c) y) = RN(a / c)
// y + yl equals 1/c within about 2^-47 relative: 1 - c y is exact (the
// remainder of the faithful reciprocal y), and (1 - c y) y = (1/c - y)(c y)
// with |1 - c y| <= 2^-24.  So a y + RN(a yl) lies within 2^-46 |a / c| of
// a / c and its one rounding stays below one ulp.  The remainder a - q0 c of
// a faithful quotient is exactly representable and the last fma then rounds
// correctly because y = RN(1/c) (Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1),
// 1990; Muller et al., "Handbook of Floating-Point Arithmetic", 2nd ed.,
// 2018, sec. 4.7 and 5.3).  Four operations where RN(a y) and two
// corrections take five.  Preconditions: c and 1/c normal, |a| >= 2^-102 (no
// remainder underflows) and |a / c| >= 2^-125, or a == 0.  Callers check
// the ranges per row / column and fall back to IEEE division outside them;
// tests/test_gpu_division.py compares the routine with IEEE division on the
// device.
__device__ __forceinline__ float recip_lo(float c, float y) {
  return __fmul_rn(__fmaf_rn(-c, y, 1.0F), y);
}
__device__ __forceinline__ f2 div2_exact(f2 a, f2 y, f2 yl, f2 nc) {
  const f2 q0 = fma2(a, y, mul2(a, yl));
  const f2 r = fma2(q0, nc, a);
  return fma2(r, y, q0);
}
__device__ __forceinline__ float4 div4_exact(float4 a, float4 y, float4 yl, float4 nc) {
  const f2 lo = div2_exact(pack2(a.x, a.y), pack2(y.x, y.y), pack2(yl.x, yl.y),
                           pack2(nc.x, nc.y));
  const f2 hi = div2_exact(pack2(a.z, a.w), pack2(y.z, y.w), pack2(yl.z, yl.w),
                           pack2(nc.z, nc.w));
  return make_float4(lo2(lo), hi2(lo), lo2(hi), hi2(hi));
}
__device__ __forceinline__ float4 div4_exact_s(float4 a, float y, float yl, float nc) {
  const f2 yy = pack2(y, y), ll = pack2(yl, yl), cc = pack2(nc, nc);
  const f2 lo = div2_exact(pack2(a.x, a.y), yy, ll, cc);
  const f2 hi = div2_exact(pack2(a.z, a.w), yy, ll, cc);
  return make_float4(lo2(lo), hi2(lo), lo2(hi), hi2(hi));
}

// --------------------------------------------------------------------------
// Smoothing from a row sum.  The reference accumulates |R_kv| in double,
// sequentially over v, then rounds mean = sum / 128 to float
// (capsule.cpp:193-199).  The kernels sum the same doubles in a tree order.
// For n = 128 non-negative terms any two summation orders differ by at most
// 2 * 127 * 2^-53 relative (Higham, "Accuracy and Stability of Numerical
// Algorithms", 2nd ed., eq. 4.4), under 2^-45.  The float rounding of the mean
// can only differ between orders when the double mean lies within that
// distance of a float rounding midpoint: the 29 discarded mantissa bits are
// then within 2^9 of 2^28 (one ulp of float = 2^29 units).  Such rows are
// flagged and re-summed in the reference's exact sequential order.
__device__ __forceinline__ bool near_float_midpoint(double mean) {
  const uint32_t low = static_cast<uint32_t>(__double2loint(mean)) & 0x1FFFFFFFu;
  const int32_t distance = static_cast<int32_t>(low) - (1 << 28);
  return distance <= 512 && distance >= -512;
}

__device__ __forceinline__ float smoothing_from_sum(double sum) {
  const float mean = __double2float_rn(sum * (1.0 / 128.0));  // exact scaling
  return __fsqrt_rn(mean < kSmoothingFloor ? kSmoothingFloor : mean);
}

// The reference quantizer's code for one element (capsule.cpp:216-223) from
// the exact smoothed value s = RN(R / c) and the exact column maximum m.
__device__ __forceinline__ int8_t exact_code(float smoothed, float maximum) {
  if (maximum == 0.0F) return 0;
  const float scaled = __fmul_rn(__fdiv_rn(smoothed, maximum), kQuantMax);
  long q = lroundf(scaled);
  q = q < -127 ? -127 : (q > 127 ? 127 : q);
  return static_cast<int8_t>(q);
}

// --------------------------------------------------------------------------
// Bulk asynchronous copies (TMA engine, no tensor map, no multicast) with
// mbarrier completion.  Only this GPU's own global memory is ever the source.
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Orders this thread's earlier generic-proxy shared-memory accesses (made
// block-wide by a preceding barrier) before a following bulk copy writes.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
      "r"(bytes)
      : "memory");
}
// Plain arrival (count 1) on an mbarrier, release semantics at CTA scope.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: gives up after `limit_ns` (2 s unless a test-support launch
// asks for less) and returns false.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - start > limit_ns) return false;
  }
  return true;
}
// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned), completing on `bar`; evict-first L2 policy because every
// state byte is read exactly once.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src,
                                          uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
// Shared -> global bulk store of `bytes` (multiple of 16, both addresses
// 16-byte aligned), tracked by the issuing thread's bulk groups.  Before the
// source buffer is written again, that thread waits with bulk_wait_read<N>
// until at most N of its committed groups still read shared memory; before
// the block exits, bulk_wait_all.
__device__ __forceinline__ void bulk_store(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
               "r"(smem_addr(smem_src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}
__device__ __forceinline__ uint64_t evict_normal_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// Streaming (evict-first) 32-bit global store and load.
__device__ __forceinline__ void st_cs_u32(void* p, uint32_t v) { __stcs(reinterpret_cast<unsigned int*>(p), v); }
__device__ __forceinline__ uint32_t ld_cs_u32(const void* p) {
  return __ldcs(reinterpret_cast<const unsigned int*>(p));
}

// Asynchronous 16-byte global -> shared copies (cp.async, cached in L2 only),
// grouped per thread with commit / wait_group.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// Wait until at most N of this thread's committed groups are still pending.
// Asynchronous 4-byte global -> shared copy (cp.async, cached in L1 and L2).
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// --------------------------------------------------------------------------
// Slot-indexed work lists.  A work item is (batch entry, head within slot).
// slot_ids == nullptr means item i is head i of a dense batch.
struct SlotMap {
  const int32_t* slot_ids;  // [count] or nullptr
  uint32_t heads_per_slot;  // heads addressed by one slot id
  uint32_t num_slots;       // valid ids are [0, num_slots); -1 is padding
};

// Returns the global head index for item, or -1 to skip it (padding or an
// invalid id; invalid ids are reported through *bad).
__device__ __forceinline__ int64_t resolve_item(const SlotMap& map, uint64_t item,
                                                bool* bad) {
  if (map.slot_ids == nullptr) return static_cast<int64_t>(item);
  const uint64_t entry = item / map.heads_per_slot;
  const int32_t slot = __ldg(map.slot_ids + entry);
  if (slot == -1) return -1;
  if (slot < 0 || static_cast<uint32_t>(slot) >= map.num_slots) {
    *bad = true;
    return -1;
  }
  return static_cast<int64_t>(slot) * map.heads_per_slot + item % map.heads_per_slot;
}

// Sticky per-device error word (read and cleared through the C ABI).  The
// library is one translation unit (gdn_state_codec.cu), so this header is
// included exactly once and the definition lives here.
__device__ uint32_t g_device_error = 0u;

__device__ __forceinline__ void report(uint32_t* status, uint32_t bits) {
  if (status != nullptr) atomicOr(status, bits);
  atomicOr(&g_device_error, bits);
}

}  // namespace gdnsc
