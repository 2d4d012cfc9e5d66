// ref_quant_shim.cpp -- TEST AND BASELINE INFRASTRUCTURE ONLY.
//
// The reference's own quant-only codec, callable from C.  The reference
// library (native/src of vLLM-HUST/gdn-state-codec) keeps its quantizer,
// dequantizer and boundary readout in an anonymous namespace
// (gdn_state_codec_state_capsule.cpp:127-308) and exposes them only through
// the full rank-4 codec.  This file compiles that source file, unmodified and
// from where it lies in the reference tree (oracle/Makefile passes its
// directory), into the same translation unit and calls:
//
//   QuantizeBoundary    capsule.cpp:129-225   with compensator_rank = 0: the
//                       rank-4 power-iteration loop runs zero times, leaving
//                       the smoothing + INT8 stage on the dense input -- the
//                       plugin's quant_only initializer
//                       (manifests/vllm-hust-extension-v0.3.json:64-70);
//   DequantizeBoundary  capsule.cpp:229-251   rank 0 (no compensator terms);
//   ReadWindowState     capsule.cpp:256-305   rank 0, no update records: the
//                       encoded projection S^T x from the boundary; and, in
//                       ref_window_read, with buffered update records and an
//                       optional rank-4 boundary: the window read of the
//                       decode step.
//
// The batch entry points split heads across std::threads; the reference
// library has no shared mutable state.  Used by tests (to pin the C oracle
// and the kernels on quant-only heads) and by bench.py's CPU baseline and
// reference arm.  Nothing in the product links or loads this file.
#include "gdn_state_codec_state_capsule.cpp"  // NOLINT: the reference source itself

#include <algorithm>
#include <cstdint>
#include <exception>
#include <thread>
#include <vector>

namespace {

using statecentric::GdnStateCodecCapsule;
using statecentric::GdnStateCodecIdentity;
using statecentric::GdnStateCodecParameters;

GdnStateCodecParameters QuantOnly() {
  GdnStateCodecParameters parameters;
  parameters.compensator_rank = 0;
  return parameters;
}

GdnStateCodecIdentity Geometry(std::uint32_t keys, std::uint32_t values) {
  GdnStateCodecIdentity identity;
  identity.key_dimension = keys;
  identity.value_dimension = values;
  return identity;
}

// Runs body(h) for h in [0, heads) on `threads` threads; false if any threw.
template <typename Body>
bool ForHeads(std::uint64_t heads, int threads, Body body) {
  threads = std::max(1, std::min<int>(threads, static_cast<int>(std::min<std::uint64_t>(heads, 1024))));
  std::vector<std::thread> pool;
  std::vector<int> failed(static_cast<std::size_t>(threads), 0);
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([&, t] {
      try {
        for (std::uint64_t h = static_cast<std::uint64_t>(t); h < heads;
             h += static_cast<std::uint64_t>(threads)) {
          body(h);
        }
      } catch (const std::exception&) {
        failed[static_cast<std::size_t>(t)] = 1;
      }
    });
  }
  for (auto& thread : pool) thread.join();
  return std::none_of(failed.begin(), failed.end(), [](int f) { return f != 0; });
}

}  // namespace

extern "C" {

// Quant-only encode of `heads` capsule-layout [keys, values] heads:
// codes [heads][keys][values], smoothing [heads][keys], scales [heads][values].
// Returns 0 on success, 1 on bad arguments or a reference exception.
int ref_quant_only_encode(const float* dense, std::uint64_t heads, std::uint32_t keys,
                          std::uint32_t values, int threads, std::int8_t* codes,
                          float* smoothing, float* scales) {
  if (dense == nullptr || codes == nullptr || smoothing == nullptr || scales == nullptr ||
      heads == 0 || keys == 0 || values == 0) {
    return 1;
  }
  const auto identity = Geometry(keys, values);
  const auto parameters = QuantOnly();
  const std::size_t elements = static_cast<std::size_t>(keys) * values;
  const bool ok = ForHeads(heads, threads, [&](std::uint64_t h) {
    const auto boundary = statecentric::QuantizeBoundary(
        std::span<const float>(dense + h * elements, elements), identity, parameters);
    std::copy(boundary->residual.begin(), boundary->residual.end(), codes + h * elements);
    std::copy(boundary->smoothing.begin(), boundary->smoothing.end(), smoothing + h * keys);
    std::copy(boundary->value_scales.begin(), boundary->value_scales.end(),
              scales + h * values);
  });
  return ok ? 0 : 1;
}

// Quant-only dense reconstruction of `heads` boundaries (capsule layout).
int ref_quant_only_decode(const std::int8_t* codes, const float* smoothing, const float* scales,
                          std::uint64_t heads, std::uint32_t keys, std::uint32_t values,
                          int threads, float* dense) {
  if (codes == nullptr || smoothing == nullptr || scales == nullptr || dense == nullptr ||
      heads == 0 || keys == 0 || values == 0) {
    return 1;
  }
  const auto identity = Geometry(keys, values);
  const auto parameters = QuantOnly();
  const std::size_t elements = static_cast<std::size_t>(keys) * values;
  const bool ok = ForHeads(heads, threads, [&](std::uint64_t h) {
    GdnStateCodecCapsule::Boundary boundary;
    boundary.residual.assign(codes + h * elements, codes + (h + 1) * elements);
    boundary.smoothing.assign(smoothing + h * keys, smoothing + (h + 1) * keys);
    boundary.value_scales.assign(scales + h * values, scales + (h + 1) * values);
    const auto out = statecentric::DequantizeBoundary(boundary, identity, parameters);
    std::copy(out.begin(), out.end(), dense + h * elements);
  });
  return ok ? 0 : 1;
}

// Encoded projection outputs[h] = S_h^T queries[h] from quant-only
// boundaries (capsule layout), queries fp32 [heads][keys].
int ref_quant_only_project(const std::int8_t* codes, const float* smoothing,
                           const float* scales, const float* queries, std::uint64_t heads,
                           std::uint32_t keys, std::uint32_t values, int threads,
                           float* outputs) {
  if (codes == nullptr || smoothing == nullptr || scales == nullptr || queries == nullptr ||
      outputs == nullptr || heads == 0 || keys == 0 || values == 0) {
    return 1;
  }
  const auto identity = Geometry(keys, values);
  const auto parameters = QuantOnly();
  const std::size_t elements = static_cast<std::size_t>(keys) * values;
  const bool ok = ForHeads(heads, threads, [&](std::uint64_t h) {
    GdnStateCodecCapsule::Boundary boundary;
    boundary.residual.assign(codes + h * elements, codes + (h + 1) * elements);
    boundary.smoothing.assign(smoothing + h * keys, smoothing + (h + 1) * keys);
    boundary.value_scales.assign(scales + h * values, scales + (h + 1) * values);
    const auto out = statecentric::ReadWindowState(
        boundary, std::span<const GdnStateCodecCapsule::UpdateRecord>(),
        std::span<const float>(queries + h * keys, keys), identity, parameters);
    std::copy(out.begin(), out.end(), outputs + h * values);
  });
  return ok ? 0 : 1;
}

// ReadWindowState (capsule.cpp:256-304) of one capsule-layout head with
// `records` buffered updates: record u has the scalar decay decay[u]
// (broadcast over the keys), key keys[u][keys] and correction
// corrections[u][values].  With compensator_keys / compensator_values
// ([keys][4] / [values][4]) the boundary has rank 4, else rank 0.  out gets
// S^T read.  Returns 0, or 1 on bad arguments or a reference exception.
int ref_window_read(const std::int8_t* codes, const float* smoothing, const float* scales,
                    const float* compensator_keys, const float* compensator_values,
                    std::uint32_t keys, std::uint32_t values, std::uint32_t records,
                    const float* decay, const float* record_keys,
                    const float* record_corrections, const float* read, float* out) {
  if (codes == nullptr || smoothing == nullptr || scales == nullptr || read == nullptr ||
      out == nullptr || keys == 0 || values == 0 ||
      (compensator_keys == nullptr) != (compensator_values == nullptr) ||
      (records > 0 && (decay == nullptr || record_keys == nullptr ||
                       record_corrections == nullptr))) {
    return 1;
  }
  try {
    const auto identity = Geometry(keys, values);
    auto parameters = QuantOnly();
    const std::size_t elements = static_cast<std::size_t>(keys) * values;
    GdnStateCodecCapsule::Boundary boundary;
    boundary.residual.assign(codes, codes + elements);
    boundary.smoothing.assign(smoothing, smoothing + keys);
    boundary.value_scales.assign(scales, scales + values);
    if (compensator_keys != nullptr) {
      parameters.compensator_rank = 4;
      boundary.compensator_keys.assign(compensator_keys, compensator_keys + keys * 4);
      boundary.compensator_values.assign(compensator_values, compensator_values + values * 4);
    }
    std::vector<GdnStateCodecCapsule::UpdateRecord> updates(records);
    for (std::uint32_t u = 0; u < records; ++u) {
      updates[u].decay.assign(keys, decay[u]);
      updates[u].key.assign(record_keys + static_cast<std::size_t>(u) * keys,
                            record_keys + static_cast<std::size_t>(u + 1) * keys);
      updates[u].correction.assign(record_corrections + static_cast<std::size_t>(u) * values,
                                   record_corrections + static_cast<std::size_t>(u + 1) * values);
    }
    const auto result = statecentric::ReadWindowState(
        boundary, updates, std::span<const float>(read, keys), identity, parameters);
    std::copy(result.begin(), result.end(), out);
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}

}  // extern "C"
