// capsule.cuh -- the reference's capsule wire format on the device (sm_100a).
//
// Serialize (native/src/gdn_state_codec_state_capsule.cpp:446-475) and
// Restore (capsule.cpp:477-578) of boundary capsules -- a 128 x 128 head,
// rank-4 compensators, window position 0 -- for a batch of heads, byte for
// byte as the portable C++ codec writes and checks them:
//
//   "LQCAPS01" | u32 schema 1 | u32 window 16 | u32 rank 4 | u32 bits 8 |
//   f32 smoothing floor 1e-8 | u64 generation | u64 epoch | u32 keys 128 |
//   u32 values 128 | u32 updates 0 | 64-char geometry digest |
//   int8 codes [key][value] | f32 smoothing [128] | f32 scales [128] |
//   f32 K [128][4] | f32 V [128][4] | 64-char lowercase hex SHA-256 of all
//   preceding bytes
//
// (little-endian integers and floats; 21,688 bytes per capsule).  Capsules
// sit back to back in the output, so capsule h starts at h * 21,688, an
// 8-byte boundary.  Serialize is two kernels: a warp per head assembles the
// capsule with coalesced 8-byte stores, then a thread per head hashes it
// (SHA-256 is sequential within a message and independent across heads).
// Restore checks each capsule in the reference's order and reports the first
// failing check per head: a thread per head checks the header and the
// SHA-256 digest, then a CTA per head whose header passed checks the payload
// and the finiteness of the dense state it encodes, and writes the boundary
// only when every check passed.
//
// SHA-256 follows FIPS 180-4 (sections 4.1.2, 5.1.1, 6.2.2).  Its constants
// are derived on the host from their definition -- the first 32 fractional
// bits of the cube roots (K) and square roots (H0) of the first primes -- by
// exact integer roots, and uploaded once per device.
#pragma once

#include <cstring>

#include "codec_device.cuh"

namespace gdnsc {

constexpr int kCapsuleHeader = 120;
constexpr int kCapsulePayload = kElements + 4 * (kKeys + kValues + kRank * (kKeys + kValues));
constexpr int kCapsuleContent = kCapsuleHeader + kCapsulePayload;  // bytes hashed
constexpr int kCapsuleBytes = kCapsuleContent + 64;                // 21,688
constexpr int kCapsuleThreads = 128;

// Per-head restore status: 0 restored, else the first failing check of
// capsule.cpp:477-578, in the reference's order.
enum CapsuleStatus : int32_t {
  kCapsuleOk = 0,
  kCapsuleMagic = 1,         // "capsule magic differs"
  kCapsuleDigestFormat = 2,  // "checksum encoding is invalid"
  kCapsuleDigest = 3,        // "checksum differs"
  kCapsuleParameters = 4,    // "quantization parameters differ"
  kCapsuleIdentity = 5,      // "identity or geometry differs"
  kCapsuleWindow = 6,        // "window position is invalid" / "window phase differs"
  kCapsuleCode = 7,          // "INT8 residual contains -128"
  kCapsulePayloadBad = 8,    // "boundary payload is invalid"
  kCapsuleDense = 9,         // "restored state is non-finite"
};

struct CapsuleIdentity {
  char geometry[64];  // lowercase hex digest of the model geometry
  uint64_t generation;
  uint64_t epoch;
};

// ---------------------------------------------------------------------------
// SHA-256 (FIPS 180-4), usable on the host (test support) and the device.

__constant__ uint32_t c_sha256_k[64];
__constant__ uint32_t c_sha256_h0[8];

struct Sha256Constants {
  uint32_t k[64];
  uint32_t h0[8];
};

// Exact integer k-th root (k = 2 or 3) of n < 2^110.
inline unsigned __int128 integer_root(unsigned __int128 n, int k) {
  unsigned __int128 lo = 0, hi = static_cast<unsigned __int128>(1) << 37;
  while (lo < hi) {
    const unsigned __int128 mid = (lo + hi + 1) / 2;
    const unsigned __int128 power = k == 2 ? mid * mid : mid * mid * mid;
    if (power <= n) {
      lo = mid;
    } else {
      hi = mid - 1;
    }
  }
  return lo;
}

// K[t] = first 32 fractional bits of cbrt(p_t), H0[i] = of sqrt(p_i).
inline const Sha256Constants& sha256_constants() {
  static const Sha256Constants constants = [] {
    Sha256Constants c{};
    int found = 0;
    for (uint32_t p = 2; found < 64; ++p) {
      bool prime = true;
      for (uint32_t d = 2; d * d <= p; ++d) prime = prime && (p % d != 0);
      if (!prime) continue;
      const unsigned __int128 cube = integer_root(static_cast<unsigned __int128>(p) << 96, 3);
      c.k[found] = static_cast<uint32_t>(cube);  // low 32 bits = fractional part
      if (found < 8) {
        const unsigned __int128 square = integer_root(static_cast<unsigned __int128>(p) << 64, 2);
        c.h0[found] = static_cast<uint32_t>(square);
      }
      ++found;
    }
    return c;
  }();
  return constants;
}

__host__ __device__ __forceinline__ uint32_t rotr32(uint32_t x, int n) {
  return (x >> n) | (x << (32 - n));
}

__host__ __device__ __forceinline__ uint32_t sha256_k(int t) {
#ifdef __CUDA_ARCH__
  return c_sha256_k[t];
#else
  return sha256_constants().k[t];
#endif
}

__host__ __device__ __forceinline__ void sha256_init(uint32_t h[8]) {
  for (int i = 0; i < 8; ++i) {
#ifdef __CUDA_ARCH__
    h[i] = c_sha256_h0[i];
#else
    h[i] = sha256_constants().h0[i];
#endif
  }
}

// One 512-bit block given as 16 big-endian words.
__host__ __device__ __forceinline__ void sha256_block(uint32_t h[8], const uint32_t block[16]) {
  uint32_t w[16];
  for (int i = 0; i < 16; ++i) w[i] = block[i];
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
#ifdef __CUDA_ARCH__
#pragma unroll
#endif
  for (int t = 0; t < 64; ++t) {
    uint32_t wt;
    if (t < 16) {
      wt = w[t];
    } else {
      const uint32_t w15 = w[(t - 15) & 15], w2 = w[(t - 2) & 15];
      const uint32_t s0 = rotr32(w15, 7) ^ rotr32(w15, 18) ^ (w15 >> 3);
      const uint32_t s1 = rotr32(w2, 17) ^ rotr32(w2, 19) ^ (w2 >> 10);
      wt = w[t & 15] + s0 + w[(t - 7) & 15] + s1;
      w[t & 15] = wt;
    }
    const uint32_t big1 = rotr32(e, 6) ^ rotr32(e, 11) ^ rotr32(e, 25);
    const uint32_t ch = (e & f) ^ (~e & g);
    const uint32_t t1 = hh + big1 + ch + sha256_k(t) + wt;
    const uint32_t big0 = rotr32(a, 2) ^ rotr32(a, 13) ^ rotr32(a, 22);
    const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
    const uint32_t t2 = big0 + maj;
    hh = g;
    g = f;
    f = e;
    e = d + t1;
    d = c;
    c = b;
    b = a;
    a = t1 + t2;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d;
  h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

// Device compression with the 32-bit adds issued as multiply-adds by a
// runtime 1 (c_fma_one, set by prepare_capsule, so the compiler cannot fold
// it back into an add): the adds then run on the FMA pipe beside the rotates
// and logic operations, which alone fill the integer ALU pipe.
__constant__ uint32_t c_fma_one;

__device__ __forceinline__ uint32_t add_on_fma(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(c_fma_one), "r"(b));
  return d;
}

__device__ __forceinline__ void sha256_block_dev(uint32_t h[8], const uint32_t block[16]) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = block[i];
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
#pragma unroll
  for (int t = 0; t < 64; ++t) {
    uint32_t wt;
    if (t < 16) {
      wt = w[t];
    } else {
      const uint32_t w15 = w[(t - 15) & 15], w2 = w[(t - 2) & 15];
      const uint32_t s0 = rotr32(w15, 7) ^ rotr32(w15, 18) ^ (w15 >> 3);
      const uint32_t s1 = rotr32(w2, 17) ^ rotr32(w2, 19) ^ (w2 >> 10);
      wt = add_on_fma(add_on_fma(add_on_fma(w[t & 15], s0), w[(t - 7) & 15]), s1);
      w[t & 15] = wt;
    }
    const uint32_t big1 = rotr32(e, 6) ^ rotr32(e, 11) ^ rotr32(e, 25);
    const uint32_t ch = (e & f) ^ (~e & g);
    // The terms known early (h, K, W) first, the ones that wait on e last.
    const uint32_t t1 =
        add_on_fma(add_on_fma(add_on_fma(add_on_fma(hh, sha256_k(t)), wt), ch), big1);
    const uint32_t big0 = rotr32(a, 2) ^ rotr32(a, 13) ^ rotr32(a, 22);
    const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
    hh = g;
    g = f;
    f = e;
    e = add_on_fma(d, t1);
    d = c;
    c = b;
    b = a;
    a = add_on_fma(add_on_fma(t1, maj), big0);
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d;
  h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

__host__ __device__ __forceinline__ uint32_t load_be32(const uint8_t* p) {
  return (static_cast<uint32_t>(p[0]) << 24) | (static_cast<uint32_t>(p[1]) << 16) |
         (static_cast<uint32_t>(p[2]) << 8) | static_cast<uint32_t>(p[3]);
}

// Digest of `size` bytes at `data` (padding of FIPS 180-4 section 5.1.1).
__host__ __device__ inline void sha256(const uint8_t* data, uint64_t size, uint32_t h[8]) {
  sha256_init(h);
  uint32_t block[16];
  uint64_t done = 0;
  for (; done + 64 <= size; done += 64) {
    for (int i = 0; i < 16; ++i) block[i] = load_be32(data + done + 4 * i);
    sha256_block(h, block);
  }
  uint8_t tail[128];
  const int rest = static_cast<int>(size - done);
  for (int i = 0; i < rest; ++i) tail[i] = data[done + i];
  tail[rest] = 0x80;
  const int blocks = rest + 1 + 8 <= 64 ? 1 : 2;
  for (int i = rest + 1; i < 64 * blocks - 8; ++i) tail[i] = 0;
  const uint64_t bits = size * 8;
  for (int i = 0; i < 8; ++i) tail[64 * blocks - 1 - i] = static_cast<uint8_t>(bits >> (8 * i));
  for (int b = 0; b < blocks; ++b) {
    for (int i = 0; i < 16; ++i) block[i] = load_be32(tail + 64 * b + 4 * i);
    sha256_block(h, block);
  }
}

// Device digest of `size` bytes at an 8-byte aligned `data`: whole blocks
// are read as eight 8-byte words and byte-swapped to big-endian words.  The
// next block's words are loaded while the current block is compressed, so
// the load latency overlaps the 64 rounds.
__device__ inline void sha256_aligned8(const uint8_t* data, uint64_t size, uint32_t h[8]) {
  sha256_init(h);
  uint32_t block[16];
  uint64_t done = 0;
  uint2 next[8];
  if (size >= 64) {
    const uint2* words = reinterpret_cast<const uint2*>(data);
#pragma unroll
    for (int i = 0; i < 8; ++i) next[i] = words[i];
  }
  for (; done + 64 <= size; done += 64) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      block[2 * i] = __byte_perm(next[i].x, 0u, 0x0123);
      block[2 * i + 1] = __byte_perm(next[i].y, 0u, 0x0123);
    }
    if (done + 128 <= size) {
      const uint2* words = reinterpret_cast<const uint2*>(data + done + 64);
#pragma unroll
      for (int i = 0; i < 8; ++i) next[i] = words[i];
    }
    sha256_block_dev(h, block);
  }
  uint8_t tail[128];
  const int rest = static_cast<int>(size - done);
  for (int i = 0; i < rest; ++i) tail[i] = data[done + i];
  tail[rest] = 0x80;
  const int blocks = rest + 1 + 8 <= 64 ? 1 : 2;
  for (int i = rest + 1; i < 64 * blocks - 8; ++i) tail[i] = 0;
  const uint64_t bits = size * 8;
  for (int i = 0; i < 8; ++i) tail[64 * blocks - 1 - i] = static_cast<uint8_t>(bits >> (8 * i));
  for (int b = 0; b < blocks; ++b) {
    for (int i = 0; i < 16; ++i) block[i] = load_be32(tail + 64 * b + 4 * i);
    sha256_block_dev(h, block);
  }
}

__host__ __device__ __forceinline__ char hex_digit(uint32_t v) {
  return static_cast<char>(v < 10 ? '0' + v : 'a' + (v - 10));
}

__host__ __device__ inline void sha256_hex(const uint32_t h[8], char out[64]) {
  for (int i = 0; i < 8; ++i) {
    for (int n = 0; n < 8; ++n) out[8 * i + n] = hex_digit((h[i] >> (28 - 4 * n)) & 15u);
  }
}

// ---------------------------------------------------------------------------
// Serialize.

struct SerializeParams {
  const int8_t* codes;       // [heads][128][128], capsule or provider layout
  const float* smoothing;    // [heads][128]
  const float* scales;       // [heads][128]
  const float* compensator_keys;    // [heads][128][4] or nullptr (zeros)
  const float* compensator_values;  // [heads][128][4] or nullptr (zeros)
  uint8_t* capsules;         // [heads][kCapsuleBytes]
  uint64_t heads;
  int provider;
  CapsuleIdentity id;
};

__device__ __forceinline__ void put_u32(uint8_t* p, uint32_t v) {
  for (int i = 0; i < 4; ++i) p[i] = static_cast<uint8_t>(v >> (8 * i));
}
__device__ __forceinline__ void put_u64(uint8_t* p, uint64_t v) {
  for (int i = 0; i < 8; ++i) p[i] = static_cast<uint8_t>(v >> (8 * i));
}

// The 120-byte header (capsule.cpp:446-460).
__device__ inline void write_header(uint8_t* p, const CapsuleIdentity& id) {
  const char magic[8] = {'L', 'Q', 'C', 'A', 'P', 'S', '0', '1'};
  for (int i = 0; i < 8; ++i) p[i] = static_cast<uint8_t>(magic[i]);
  put_u32(p + 8, 1u);                                   // schema_version
  put_u32(p + 12, 16u);                                 // window_size
  put_u32(p + 16, static_cast<uint32_t>(kRank));        // compensator_rank
  put_u32(p + 20, 8u);                                  // quant_bits
  put_u32(p + 24, __float_as_uint(kSmoothingFloor));    // smoothing_floor
  put_u64(p + 28, id.generation);
  put_u64(p + 36, id.epoch);
  put_u32(p + 44, static_cast<uint32_t>(kKeys));
  put_u32(p + 48, static_cast<uint32_t>(kValues));
  put_u32(p + 52, 0u);                                  // buffered updates
  for (int i = 0; i < 64; ++i) p[56 + i] = static_cast<uint8_t>(id.geometry[i]);
}

// Warp per head: header, codes (capsule order), then the float planes.
__global__ void __launch_bounds__(kCapsuleThreads) capsule_assemble_kernel(SerializeParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * (kCapsuleThreads / 32);
  for (uint64_t head = static_cast<uint64_t>(blockIdx.x) * (kCapsuleThreads / 32) + warp;
       head < p.heads; head += stride) {
    uint8_t* out = p.capsules + head * kCapsuleBytes;
    if (lane == 0) write_header(out, p.id);
    const int8_t* codes = p.codes + head * kElements;
    uint2* dst = reinterpret_cast<uint2*>(out + kCapsuleHeader);
    if (!p.provider) {
      const uint2* src = reinterpret_cast<const uint2*>(codes);
      for (int i = lane; i < kElements / 8; i += 32) dst[i] = src[i];
    } else {
      // provider codes [v][k] -> capsule order [k][v]: 8 values of one key per store
      for (int i = lane; i < kElements / 8; i += 32) {
        const int k = i >> 4, v0 = 8 * (i & 15);
        uint32_t lo = 0, hi = 0;
        for (int e = 0; e < 4; ++e) {
          lo |= static_cast<uint32_t>(static_cast<uint8_t>(codes[(v0 + e) * kKeys + k])) << (8 * e);
          hi |= static_cast<uint32_t>(static_cast<uint8_t>(codes[(v0 + 4 + e) * kKeys + k])) << (8 * e);
        }
        dst[i] = make_uint2(lo, hi);
      }
    }
    // Float planes: smoothing, scales, K, V (capsule.cpp:465-468).
    uint32_t* fdst = reinterpret_cast<uint32_t*>(out + kCapsuleHeader + kElements);
    const uint32_t* sm = reinterpret_cast<const uint32_t*>(p.smoothing + head * kKeys);
    const uint32_t* sc = reinterpret_cast<const uint32_t*>(p.scales + head * kValues);
    for (int i = lane; i < kKeys; i += 32) fdst[i] = sm[i];
    for (int i = lane; i < kValues; i += 32) fdst[kKeys + i] = sc[i];
    uint32_t* kdst = fdst + kKeys + kValues;
    uint32_t* vdst = kdst + kKeys * kRank;
    for (int i = lane; i < kKeys * kRank; i += 32) {
      kdst[i] = p.compensator_keys
                    ? __float_as_uint(p.compensator_keys[head * kKeys * kRank + i]) : 0u;
      vdst[i] = p.compensator_values
                    ? __float_as_uint(p.compensator_values[head * kValues * kRank + i]) : 0u;
    }
  }
}

// Thread per head: the SHA-256 digest of the content, as lowercase hex.
__global__ void __launch_bounds__(kCapsuleThreads) capsule_digest_kernel(uint8_t* capsules,
                                                                         uint64_t heads) {
  const uint64_t head = static_cast<uint64_t>(blockIdx.x) * kCapsuleThreads + threadIdx.x;
  if (head >= heads) return;
  uint8_t* capsule = capsules + head * kCapsuleBytes;
  uint32_t h[8];
  sha256_aligned8(capsule, kCapsuleContent, h);
  char hex[64];
  sha256_hex(h, hex);
  for (int i = 0; i < 64; ++i) capsule[kCapsuleContent + i] = static_cast<uint8_t>(hex[i]);
}

// ---------------------------------------------------------------------------
// Restore.

struct RestoreParams {
  const uint8_t* capsules;   // [heads][kCapsuleBytes]
  int8_t* codes;             // [heads][128][128], capsule or provider layout
  float* smoothing;
  float* scales;
  float* compensator_keys;   // [heads][128][4]
  float* compensator_values; // [heads][128][4]
  int32_t* head_status;      // [heads]
  uint64_t heads;
  int provider;
  CapsuleIdentity id;
};

__device__ __forceinline__ uint32_t get_u32(const uint8_t* p) {
  uint32_t v = 0;
  for (int i = 0; i < 4; ++i) v |= static_cast<uint32_t>(p[i]) << (8 * i);
  return v;
}
__device__ __forceinline__ uint64_t get_u64(const uint8_t* p) {
  uint64_t v = 0;
  for (int i = 0; i < 8; ++i) v |= static_cast<uint64_t>(p[i]) << (8 * i);
  return v;
}

// Restore, part 1 (thread per capsule): the header checks and the SHA-256
// digest, which is sequential within a capsule -- checks 1 to 6 of
// capsule.cpp:477-578 in the reference's order.  Returns the first failing
// one, or kCapsuleOk when the payload checks may proceed.
__device__ int32_t restore_header_check(const uint8_t* c, const CapsuleIdentity& id) {
  const char magic[8] = {'L', 'Q', 'C', 'A', 'P', 'S', '0', '1'};
  for (int i = 0; i < 8; ++i) {
    if (c[i] != static_cast<uint8_t>(magic[i])) return kCapsuleMagic;
  }
  const uint8_t* recorded = c + kCapsuleContent;
  for (int i = 0; i < 64; ++i) {
    const uint8_t ch = recorded[i];
    if (!((ch >= '0' && ch <= '9') || (ch >= 'a' && ch <= 'f'))) return kCapsuleDigestFormat;
  }
  uint32_t h[8];
  sha256_aligned8(c, kCapsuleContent, h);
  char hex[64];
  sha256_hex(h, hex);
  for (int i = 0; i < 64; ++i) {
    if (recorded[i] != static_cast<uint8_t>(hex[i])) return kCapsuleDigest;
  }
  if (get_u32(c + 8) != 1u || get_u32(c + 12) != 16u || get_u32(c + 16) != kRank ||
      get_u32(c + 20) != 8u || get_u32(c + 24) != __float_as_uint(kSmoothingFloor)) {
    return kCapsuleParameters;
  }
  bool same = get_u64(c + 28) == id.generation && get_u64(c + 36) == id.epoch &&
              get_u32(c + 44) == kKeys && get_u32(c + 48) == kValues;
  for (int i = 0; i < 64; ++i) same = same && c[56 + i] == static_cast<uint8_t>(id.geometry[i]);
  if (!same) return kCapsuleIdentity;
  if (get_u32(c + 52) != 0u) return kCapsuleWindow;  // this format has no update records
  return kCapsuleOk;
}

constexpr int kVerifyThreads = 64;

__global__ void __launch_bounds__(kVerifyThreads) capsule_verify_kernel(RestoreParams p) {
  const uint64_t head = static_cast<uint64_t>(blockIdx.x) * kVerifyThreads + threadIdx.x;
  if (head >= p.heads) return;
  p.head_status[head] = restore_header_check(p.capsules + head * kCapsuleBytes, p.id);
}

// Restore, part 2 (a 128-thread CTA per capsule whose header checks passed):
// checks 7 to 9 -- no code is -128; smoothing finite and positive, scales
// finite and non-negative, compensators finite; the dense state the capsule
// encodes (((c z) / 127) b + sum_r K V, the reference's order) finite --
// reported in that order, and only when all pass are the codes and planes
// written (fail closed).  Thread t scans codes row t (key t) and owns plane
// entry t.
struct __align__(16) RestoreShared {
  int8_t codes[kElements];   // [key][value] as in the capsule
  float b[kValues];          // scales
  float4 v[kValues];         // compensator values
  float4 bound[kCapsuleThreads / 32];  // per-warp max |c|, |b|, |K|, |V|
};

__global__ void __launch_bounds__(kCapsuleThreads) capsule_payload_kernel(RestoreParams p) {
  __shared__ RestoreShared sh;
  const int t = threadIdx.x;
  for (uint64_t head = blockIdx.x; head < p.heads; head += gridDim.x) {
    if (__ldcg(p.head_status + head) != kCapsuleOk) continue;  // block-uniform
    const uint8_t* c = p.capsules + head * kCapsuleBytes;
    const uint8_t* codes = c + kCapsuleHeader;      // 8-byte aligned
    const uint8_t* planes = codes + kElements;      // 8-byte aligned
    // -- codes to shared memory, checking for -128 ----------------------------
    bool bad_code = false;
#pragma unroll 4
    for (int i = t; i < kElements / 8; i += kCapsuleThreads) {
      const uint2 w = __ldcs(reinterpret_cast<const uint2*>(codes) + i);
      bad_code = bad_code || (__vcmpeq4(w.x, 0x80808080u) | __vcmpeq4(w.y, 0x80808080u)) != 0u;
      reinterpret_cast<uint2*>(sh.codes)[i] = w;
    }
    // -- planes of entry t ----------------------------------------------------
    const float* f = reinterpret_cast<const float*>(planes);  // 4-byte aligned
    const float smooth = f[t];
    const float scale = f[kKeys + t];
    const float* kp = f + kKeys + kValues;
    const float* vp = kp + kKeys * kRank;
    const float4 kr = make_float4(kp[4 * t], kp[4 * t + 1], kp[4 * t + 2], kp[4 * t + 3]);
    const float4 vr = make_float4(vp[4 * t], vp[4 * t + 1], vp[4 * t + 2], vp[4 * t + 3]);
    const bool bad_payload =
        !isfinite(smooth) || !(smooth > 0.0F) || !isfinite(scale) || !(scale >= 0.0F) ||
        !isfinite(kr.x) || !isfinite(kr.y) || !isfinite(kr.z) || !isfinite(kr.w) ||
        !isfinite(vr.x) || !isfinite(vr.y) || !isfinite(vr.z) || !isfinite(vr.w);
    sh.b[t] = scale;
    sh.v[t] = vr;
    const bool any_code = __syncthreads_or(bad_code) != 0;
    const bool any_payload = __syncthreads_or(bad_payload) != 0;
    // -- DenseState finite (capsule.cpp:574-576) --------------------------------
    // With finite planes every element is at most (max|c| max|b| + 4 max|K|
    // max|V|) times the growth of its eight roundings, far below FLT_MAX when
    // that bound is below 1e38; only a larger bound needs the element check
    // (row t per thread, in the reference's order).
    bool any_dense = false;
    if (!any_code && !any_payload) {
      float mc = fabsf(smooth), mb = fabsf(scale);
      float mk = fmaxf(fmaxf(fabsf(kr.x), fabsf(kr.y)), fmaxf(fabsf(kr.z), fabsf(kr.w)));
      float mv = fmaxf(fmaxf(fabsf(vr.x), fabsf(vr.y)), fmaxf(fabsf(vr.z), fabsf(vr.w)));
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, off));
        mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
        mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, off));
        mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, off));
      }
      if ((t & 31) == 0) sh.bound[t >> 5] = make_float4(mc, mb, mk, mv);
      __syncthreads();
      float4 m = sh.bound[0];
#pragma unroll
      for (int w = 1; w < kCapsuleThreads / 32; ++w) {
        const float4 o = sh.bound[w];
        m = make_float4(fmaxf(m.x, o.x), fmaxf(m.y, o.y), fmaxf(m.z, o.z), fmaxf(m.w, o.w));
      }
      const double bound = static_cast<double>(m.x) * m.y + 4.0 * static_cast<double>(m.z) * m.w;
      if (!(bound < 1.0e38)) {  // block-uniform
        bool bad_dense = false;
        for (int v = 0; v < kValues; ++v) {
          const float z = static_cast<float>(sh.codes[t * kValues + v]);
          float value = __fmul_rn(div127_any(__fmul_rn(smooth, z)), sh.b[v]);
          const float4 vv = sh.v[v];
          value = __fadd_rn(value, __fmul_rn(kr.x, vv.x));
          value = __fadd_rn(value, __fmul_rn(kr.y, vv.y));
          value = __fadd_rn(value, __fmul_rn(kr.z, vv.z));
          value = __fadd_rn(value, __fmul_rn(kr.w, vv.w));
          bad_dense = bad_dense || !isfinite(value);
        }
        any_dense = __syncthreads_or(bad_dense) != 0;
      }
    }
    const int32_t status = any_code      ? kCapsuleCode
                           : any_payload ? kCapsulePayloadBad
                           : any_dense   ? kCapsuleDense
                                         : kCapsuleOk;
    if (t == 0) p.head_status[head] = status;
    if (status == kCapsuleOk) {
      // -- write the boundary -------------------------------------------------
      int8_t* out = p.codes + head * kElements;
      if (!p.provider) {
#pragma unroll 4
        for (int i = t; i < kElements / 16; i += kCapsuleThreads) {
          reinterpret_cast<uint4*>(out)[i] = reinterpret_cast<const uint4*>(sh.codes)[i];
        }
      } else {
        // row v = t of the provider layout: codes [k][t] for k = 0..127
        for (int k0 = 0; k0 < kKeys; k0 += 16) {
          uint32_t w[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t word = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              word |= static_cast<uint32_t>(static_cast<uint8_t>(
                          sh.codes[(k0 + 4 * j + b) * kValues + t])) << (8 * b);
            }
            w[j] = word;
          }
          reinterpret_cast<uint4*>(out + t * kKeys + k0)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      p.smoothing[head * kKeys + t] = smooth;
      p.scales[head * kValues + t] = scale;
      reinterpret_cast<float4*>(p.compensator_keys)[head * kKeys + t] = kr;
      reinterpret_cast<float4*>(p.compensator_values)[head * kValues + t] = vr;
    }
    __syncthreads();  // shared memory is reused by the next capsule
  }
}

// ---------------------------------------------------------------------------
// Host helpers.

inline cudaError_t prepare_capsule() {
  const Sha256Constants& c = sha256_constants();
  cudaError_t err = cudaMemcpyToSymbol(c_sha256_k, c.k, sizeof(c.k));
  if (err != cudaSuccess) return err;
  const uint32_t one = 1u;
  err = cudaMemcpyToSymbol(c_fma_one, &one, sizeof(one));
  if (err != cudaSuccess) return err;
  return cudaMemcpyToSymbol(c_sha256_h0, c.h0, sizeof(c.h0));
}

inline bool lowercase_hex64(const char* s) {
  for (int i = 0; i < 64; ++i) {
    const char ch = s[i];
    if (!((ch >= '0' && ch <= '9') || (ch >= 'a' && ch <= 'f'))) return false;
  }
  return true;
}

}  // namespace gdnsc
