// synth.cuh -- seeded synthetic GDN state and query generators (benchmark and
// test support; not part of the reference ABI).
//
// Distribution (the benchmark configurations' stand-in for real Qwen3.5 GDN
// state): per head, x ~ N(0,1) times a per-head factor 10^(-3u), u ~ U[0,1)
// (log-uniform in [1e-3, 1]), then 1% of entries set to exactly 0.  Queries
// are N(0,1), L2-normalised per head, rounded to bf16.
//
// Every value is a pure function of (seed, slot, layer, head, element): a
// counter-based generator built on the SplitMix64 finaliser (Steele, Lea,
// Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014), so a
// shard of slots generated on any GPU equals the same slots generated on one.
// Normals use the Box-Muller transform with the CUDA math library.
#include <cuda_bf16.h>

#pragma once

#include "codec_device.cuh"

namespace gdnsc {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t head_key(uint64_t seed, uint64_t slot, uint64_t layer,
                                             uint64_t head) {
  return mix64(mix64(mix64(seed ^ 0x6764'6e5f'7374'6174ull) ^ slot) ^ (layer << 20 | head));
}

// Uniform in (0, 1) from 32 bits.
__device__ __forceinline__ float unit(uint32_t bits) {
  return (static_cast<float>(bits >> 8) + 0.5F) * 0x1p-24F;
}

__device__ __forceinline__ float normal_from(uint64_t r) {
  const float u1 = unit(static_cast<uint32_t>(r >> 32));
  const float u2 = unit(static_cast<uint32_t>(r));
  return sqrtf(-2.0F * logf(u1)) * cospif(2.0F * u2);
}

struct SynthParams {
  void* out;
  uint64_t heads;      // slots * layers * heads_per_layer
  uint64_t seed;
  uint32_t slot_base;  // global slot id of the first slot in `out`
  uint32_t layers;
  uint32_t heads_per_layer;
  uint32_t provider;   // element order of the state output
};

__device__ __forceinline__ void decompose(const SynthParams& p, uint64_t h, uint64_t* slot,
                                          uint64_t* layer, uint64_t* head) {
  const uint64_t per_slot = static_cast<uint64_t>(p.layers) * p.heads_per_layer;
  *slot = p.slot_base + h / per_slot;
  *layer = (h / p.heads_per_layer) % p.layers;
  *head = h % p.heads_per_layer;
}

// One thread per (head, key k, 4 consecutive values v): logical element
// (k, v) is written at [k][v] (capsule) or [v][k] (provider).
__global__ void synth_state_kernel(SynthParams p) {
  float* out = static_cast<float*>(p.out);
  const uint64_t total = p.heads * (kElements / 4);
  for (uint64_t t = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t h = t / (kElements / 4);
    const int quad = static_cast<int>(t % (kElements / 4));
    const int k = quad / 32;
    const int v0 = (quad % 32) * 4;
    uint64_t slot, layer, head;
    decompose(p, h, &slot, &layer, &head);
    const uint64_t key = head_key(p.seed, slot, layer, head);
    const float scale = exp10f(-3.0F * unit(static_cast<uint32_t>(mix64(key ^ 0x5CA1Eull) >> 32)));
    float vals[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint64_t e = static_cast<uint64_t>(k) * kValues + v0 + i;
      const uint64_t r = mix64(key + 2 * e + 1);
      const uint64_t zero_draw = mix64(key + 2 * e + 2);
      const bool zero = (zero_draw >> 40) < (uint64_t{1} << 24) / 100;  // 1%
      vals[i] = zero ? 0.0F : normal_from(r) * scale;
    }
    float* base = out + h * kElements;
    if (p.provider) {
#pragma unroll
      for (int i = 0; i < 4; ++i) base[(v0 + i) * kKeys + k] = vals[i];
    } else {
      *reinterpret_cast<float4*>(base + k * kValues + v0) =
          make_float4(vals[0], vals[1], vals[2], vals[3]);
    }
  }
}

// One warp per head: 128 normals, L2-normalised, rounded to bf16.
__global__ void synth_query_kernel(SynthParams p) {
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
  const int lane = threadIdx.x & 31;
  const uint64_t warps = static_cast<uint64_t>(gridDim.x) * (blockDim.x / 32);
  for (uint64_t h = blockIdx.x * static_cast<uint64_t>(blockDim.x / 32) + threadIdx.x / 32;
       h < p.heads; h += warps) {
    uint64_t slot, layer, head;
    decompose(p, h, &slot, &layer, &head);
    const uint64_t key = head_key(p.seed ^ 0x7175657279ull, slot, layer, head);
    float q[4];
    float ss = 0.0F;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q[i] = normal_from(mix64(key + 4 * lane + i));
      ss += q[i] * q[i];
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = rsqrtf(ss);
#pragma unroll
    for (int i = 0; i < 4; ++i) out[h * kKeys + 4 * lane + i] = __float2bfloat16_rn(q[i] * inv);
  }
}

cudaError_t launch_synth_states(const SynthParams& p, int sms, cudaStream_t stream) {
  synth_state_kernel<<<sms * 8, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_synth_queries(const SynthParams& p, int sms, cudaStream_t stream) {
  synth_query_kernel<<<sms * 4, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace gdnsc
