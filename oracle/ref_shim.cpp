// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A C-ABI wrapper over the reference's own portable codec library
// (native/src of vLLM-HUST/gdn-state-codec, compiled unmodified from the
// reference source tree by oracle/Makefile into oracle/_ref/).  Python tests
// load it with ctypes to (a) pin the C oracle in gdn_codec_oracle.c against
// the real library and (b) generate the golden vectors in tests/golden.
// Nothing in the product links or loads this file.
//
// Public reference API used (native/include/statecentric/
// gdn_state_codec_state_capsule.h:56-69):
//   GdnStateCodecCapsule::FromDenseBoundary  (capsule.cpp:318-335)
//   GdnStateCodecCapsule::Serialize          (capsule.cpp:446-475)
//   GdnStateCodecCapsule::DenseState         (capsule.cpp:337-352)
//   GdnStateCodecCapsule::ApplyToken         (capsule.cpp:354-397)
// and the Qwen layout adapter (gdn_state_codec_qwen38_gdn_adapter.h:10-17).
#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <span>
#include <string>
#include <vector>

#include "statecentric/gdn_state_codec_qwen38_gdn_adapter.h"
#include "statecentric/gdn_state_codec_state_capsule.h"

namespace {

using statecentric::GdnStateCodecCapsule;
using statecentric::GdnStateCodecIdentity;
using statecentric::GdnStateCodecParameters;
using statecentric::GdnStateCodecTokenInput;

constexpr std::size_t kRank = 4;
// Serialized header: magic(8) + 4 x u32 + f32 + 2 x u64 + 3 x u32 + 64-char
// geometry digest = 120 bytes (reference test capsule_test.cpp:321 pins the
// INT8 residual at offset 120).
constexpr std::size_t kResidualOffset = 120;

GdnStateCodecIdentity Identity(std::uint32_t keys, std::uint32_t values) {
  return {std::string(64, 'a'), 7, 11, keys, values};
}

float ReadF32(const std::vector<std::uint8_t>& bytes, std::size_t offset) {
  std::uint32_t bits = 0;
  for (std::size_t i = 0; i < 4; ++i) {
    bits |= static_cast<std::uint32_t>(bytes[offset + i]) << (8U * i);
  }
  float value;
  std::memcpy(&value, &bits, sizeof(value));
  return value;
}

}  // namespace

// Encode one dense capsule-layout [keys, values] head with the reference's
// full codec (rank-4 compensator fit + INT8 boundary), then read back the
// boundary planes from the serialized capsule, the reconstructed dense state,
// and the encoded readout S^T q (ApplyToken with decay=1, key=read=value=0,
// which leaves the query unchanged and adds an exactly-zero update term).
// Any null output pointer is skipped.  Returns 0 on success, 1 when the
// reference rejects the input (it throws std::invalid_argument).
extern "C" int ref_codec_head(const float* dense, std::uint32_t keys,
                              std::uint32_t values, const float* query,
                              std::int8_t* codes, float* smoothing,
                              float* scales, float* compensator_keys,
                              float* compensator_values, float* dense_out,
                              float* projection_out) {
  try {
    const std::size_t elements = static_cast<std::size_t>(keys) * values;
    std::vector<float> state(dense, dense + elements);
    auto capsule = GdnStateCodecCapsule::FromDenseBoundary(
        state, Identity(keys, values), GdnStateCodecParameters{});
    const auto bytes = capsule.Serialize();
    std::size_t offset = kResidualOffset;
    for (std::size_t i = 0; i < elements; ++i, ++offset) {
      if (codes) codes[i] = static_cast<std::int8_t>(bytes[offset]);
    }
    for (std::uint32_t k = 0; k < keys; ++k, offset += 4) {
      if (smoothing) smoothing[k] = ReadF32(bytes, offset);
    }
    for (std::uint32_t v = 0; v < values; ++v, offset += 4) {
      if (scales) scales[v] = ReadF32(bytes, offset);
    }
    for (std::size_t i = 0; i < keys * kRank; ++i, offset += 4) {
      if (compensator_keys) compensator_keys[i] = ReadF32(bytes, offset);
    }
    for (std::size_t i = 0; i < values * kRank; ++i, offset += 4) {
      if (compensator_values) compensator_values[i] = ReadF32(bytes, offset);
    }
    if (dense_out) {
      const auto reconstructed = capsule.DenseState();
      std::memcpy(dense_out, reconstructed.data(), elements * sizeof(float));
    }
    if (projection_out && query) {
      GdnStateCodecTokenInput token;
      token.decay.assign(keys, 1.0F);
      token.key.assign(keys, 0.0F);
      token.read.assign(keys, 0.0F);
      token.value.assign(values, 0.0F);
      token.query.assign(query, query + keys);
      const auto result = capsule.ApplyToken(token);
      std::memcpy(projection_out, result.output.data(), values * sizeof(float));
    }
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}

// Size in bytes of the reference's serialized capsule for this geometry
// with no buffered updates (header + payload + 64-char digest).
extern "C" std::uint64_t ref_capsule_bytes(std::uint32_t keys,
                                           std::uint32_t values) {
  return kResidualOffset + static_cast<std::uint64_t>(keys) * values +
         4ULL * (keys + values + kRank * (keys + values)) + 64ULL;
}

// Reference adapter, provider [value,key] -> capsule [key,value].
extern "C" int ref_provider_to_capsule(const float* provider, std::uint32_t keys,
                                       std::uint32_t values, float* capsule) {
  try {
    const std::size_t elements = static_cast<std::size_t>(keys) * values;
    const auto out = statecentric::Qwen38ProviderStateToGdnStateCodec(
        std::vector<float>(provider, provider + elements), keys, values);
    std::memcpy(capsule, out.data(), elements * sizeof(float));
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}

// The reference's memory accounting for one head (capsule_test.cpp:392-403).
extern "C" int ref_head_bytes(std::uint32_t keys, std::uint32_t values,
                              std::uint64_t* fp32_bytes,
                              std::uint64_t* boundary_bytes) {
  try {
    const std::vector<float> state(static_cast<std::size_t>(keys) * values, 0.0F);
    const auto capsule = GdnStateCodecCapsule::FromDenseBoundary(
        state, Identity(keys, values), GdnStateCodecParameters{});
    *fp32_bytes = capsule.fp32_state_bytes();
    *boundary_bytes = capsule.compressed_boundary_bytes();
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}

namespace {

GdnStateCodecIdentity IdentityOf(const char* geometry64, std::uint64_t generation,
                                 std::uint64_t epoch, std::uint32_t keys, std::uint32_t values) {
  return {std::string(geometry64, 64), generation, epoch, keys, values};
}

}  // namespace

// The reference's serialized capsule (Serialize, capsule.cpp:446-475) of
// FromDenseBoundary(dense) under the given identity, written to `out`.
// Returns the byte count, or 0 when the reference rejects the input or the
// buffer is too small.
extern "C" std::uint64_t ref_serialize_head(const float* dense, std::uint32_t keys,
                                            std::uint32_t values, const char* geometry64,
                                            std::uint64_t generation, std::uint64_t epoch,
                                            std::uint8_t* out, std::uint64_t capacity) {
  try {
    const std::size_t elements = static_cast<std::size_t>(keys) * values;
    std::vector<float> state(dense, dense + elements);
    const auto capsule = GdnStateCodecCapsule::FromDenseBoundary(
        state, IdentityOf(geometry64, generation, epoch, keys, values), GdnStateCodecParameters{});
    const auto bytes = capsule.Serialize();
    if (bytes.size() > capacity) return 0;
    std::memcpy(out, bytes.data(), bytes.size());
    return bytes.size();
  } catch (const std::exception&) {
    return 0;
  }
}

// The reference's Restore (capsule.cpp:477-578) of `bytes` with the expected
// identity, default parameters and window position 0.  Returns 0 when it
// accepts, 1 when it rejects; the rejection message goes to `message`.
extern "C" int ref_restore_capsule(const std::uint8_t* bytes, std::uint64_t size,
                                   const char* geometry64, std::uint64_t generation,
                                   std::uint64_t epoch, std::uint32_t keys, std::uint32_t values,
                                   char* message, std::uint64_t message_capacity) {
  try {
    (void)GdnStateCodecCapsule::Restore(
        std::span<const std::uint8_t>(bytes, size),
        IdentityOf(geometry64, generation, epoch, keys, values), GdnStateCodecParameters{}, 0);
    if (message && message_capacity) message[0] = '\0';
    return 0;
  } catch (const std::exception& error) {
    if (message && message_capacity) {
      std::strncpy(message, error.what(), message_capacity - 1);
      message[message_capacity - 1] = '\0';
    }
    return 1;
  }
}

// FromDenseBoundary(dense) followed by `tokens` ApplyToken calls
// (capsule.cpp:354-397) with a scalar decay per token broadcast over the
// keys.  Token t reads decay[t], key/read/query [t][keys] and value
// [t][values]; its output goes to outputs[t][values] and crossed[t] is 1 when
// the token completed a window (the library refit its boundary).  The final
// DenseState (capsule.cpp:337-352) goes to dense_out when it is not null.
// Returns 0, or 1 when the reference rejects an input.
extern "C" int ref_apply_tokens(const float* dense, std::uint32_t keys, std::uint32_t values,
                                std::uint32_t tokens, const float* decay, const float* key,
                                const float* read, const float* query, const float* value,
                                float* outputs, std::uint8_t* crossed, float* dense_out,
                                std::uint32_t* window_position) {
  try {
    const std::size_t elements = static_cast<std::size_t>(keys) * values;
    std::vector<float> state(dense, dense + elements);
    auto capsule = GdnStateCodecCapsule::FromDenseBoundary(
        state, Identity(keys, values), GdnStateCodecParameters{});
    for (std::uint32_t t = 0; t < tokens; ++t) {
      GdnStateCodecTokenInput token;
      token.decay.assign(keys, decay[t]);
      token.key.assign(key + static_cast<std::size_t>(t) * keys,
                       key + static_cast<std::size_t>(t + 1) * keys);
      token.read.assign(read + static_cast<std::size_t>(t) * keys,
                        read + static_cast<std::size_t>(t + 1) * keys);
      token.query.assign(query + static_cast<std::size_t>(t) * keys,
                         query + static_cast<std::size_t>(t + 1) * keys);
      token.value.assign(value + static_cast<std::size_t>(t) * values,
                         value + static_cast<std::size_t>(t + 1) * values);
      const auto result = capsule.ApplyToken(token);
      std::memcpy(outputs + static_cast<std::size_t>(t) * values, result.output.data(),
                  values * sizeof(float));
      if (crossed) crossed[t] = result.crossed_window_boundary ? 1 : 0;
    }
    if (dense_out) {
      const auto reconstructed = capsule.DenseState();
      std::memcpy(dense_out, reconstructed.data(), elements * sizeof(float));
    }
    if (window_position) *window_position = static_cast<std::uint32_t>(capsule.window_position());
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}

// Seconds spent inside `tokens` ApplyToken calls (capsule.cpp:354-397) on a
// capsule made by FromDenseBoundary(dense), timed with a steady clock around
// the token loop only (the boundary fit before it is not timed).  Token t
// uses the scalar decay decay[t] broadcast over the keys.  Returns a negative
// value when the reference rejects an input.  Used as the CPU baseline of the
// decode step.
extern "C" double ref_time_apply_tokens(const float* dense, std::uint32_t keys,
                                        std::uint32_t values, std::uint32_t tokens,
                                        const float* decay, const float* key, const float* read,
                                        const float* query, const float* value) {
  try {
    const std::size_t elements = static_cast<std::size_t>(keys) * values;
    std::vector<float> state(dense, dense + elements);
    auto capsule = GdnStateCodecCapsule::FromDenseBoundary(
        state, Identity(keys, values), GdnStateCodecParameters{});
    std::vector<GdnStateCodecTokenInput> inputs(tokens);
    for (std::uint32_t t = 0; t < tokens; ++t) {
      auto& token = inputs[t];
      token.decay.assign(keys, decay[t]);
      token.key.assign(key + static_cast<std::size_t>(t) * keys,
                       key + static_cast<std::size_t>(t + 1) * keys);
      token.read.assign(read + static_cast<std::size_t>(t) * keys,
                        read + static_cast<std::size_t>(t + 1) * keys);
      token.query.assign(query + static_cast<std::size_t>(t) * keys,
                         query + static_cast<std::size_t>(t + 1) * keys);
      token.value.assign(value + static_cast<std::size_t>(t) * values,
                         value + static_cast<std::size_t>(t + 1) * values);
    }
    const auto begin = std::chrono::steady_clock::now();
    for (std::uint32_t t = 0; t < tokens; ++t) (void)capsule.ApplyToken(inputs[t]);
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - begin).count();
  } catch (const std::exception&) {
    return -1.0;
  }
}

// Seconds spent in `reps` Serialize calls (capsule.cpp:446-475) and in `reps`
// Restore calls (:477-578) of the capsule FromDenseBoundary(dense) makes (the
// fit itself is not timed), each timed with a steady clock.  Returns 0, or 1
// when the reference rejects an input.  Used as the CPU baseline of the
// capsule wire format.
extern "C" int ref_time_capsule(const float* dense, std::uint32_t keys, std::uint32_t values,
                                std::uint32_t reps, double* serialize_seconds,
                                double* restore_seconds) {
  try {
    const std::size_t elements = static_cast<std::size_t>(keys) * values;
    std::vector<float> state(dense, dense + elements);
    const auto identity = Identity(keys, values);
    const auto capsule =
        GdnStateCodecCapsule::FromDenseBoundary(state, identity, GdnStateCodecParameters{});
    std::vector<std::uint8_t> bytes;
    auto begin = std::chrono::steady_clock::now();
    for (std::uint32_t r = 0; r < reps; ++r) bytes = capsule.Serialize();
    *serialize_seconds =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - begin).count();
    begin = std::chrono::steady_clock::now();
    for (std::uint32_t r = 0; r < reps; ++r) {
      (void)GdnStateCodecCapsule::Restore(std::span<const std::uint8_t>(bytes), identity,
                                          GdnStateCodecParameters{}, 0);
    }
    *restore_seconds =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - begin).count();
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}
