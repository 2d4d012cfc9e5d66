// gdn_state_codec.cu -- the single translation unit of the B200 GDN state
// codec library: the kernels (quantize.cuh, dequantize.cuh, projection.cuh,
// synth.cuh) and the C ABI of include/statecentric/gdn_state_codec_kernel.h
// over them: argument validation, per-device launch set-up and the launches.
// The ABI allocates nothing and never synchronises the host.
#include <cstdint>
#include <mutex>

#include "capsule.cuh"
#include "codec_device.cuh"
#include "dequantize.cuh"
#include "fit.cuh"
#include "projection.cuh"
#include "quantize.cuh"
#include "synth.cuh"
#include "window.cuh"
#include "statecentric/gdn_state_codec_kernel.h"
#include "statecentric/gdn_state_codec_windowed_gdn_kernel.h"

namespace gdnsc {

// Test support: the quantizer's exact-division routine (div4_exact) applied
// elementwise, so tests can compare it with IEEE division on the device.
__global__ void division_selftest_kernel(const float* a, const float* c, float* out, uint64_t n) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const float ci = c[i];
    const float y = __frcp_rn(ci);
    out[i] = div4_exact_s(make_float4(a[i], 0.F, 0.F, 0.F), y, recip_lo(ci, y), -ci).x;
  }
}

namespace {

constexpr int32_t kOk = 0;
constexpr int32_t kBadArgs = 1;
constexpr int32_t kLaunchFailed = 2;
constexpr int32_t kSetupFailed = 3;
constexpr int kMaxDevices = 64;

struct DeviceSetup {
  bool ready = false;
  int sms = 0;
  int quantize_blocks[2][3] = {};  // [provider][mode] blocks per SM
  int dequantize_blocks[2][2] = {};
  int project_blocks[2][2] = {};
  int fit_blocks = 0;
  WindowBlocks window;
};

std::mutex g_setup_mutex;
DeviceSetup g_setup[kMaxDevices];

// Per-device one-time set-up (shared-memory opt-in and occupancy); guarded by
// a mutex so concurrent host threads on one device are safe.
const DeviceSetup* device_setup() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  DeviceSetup& s = g_setup[device];
  if (s.ready) return &s;
  if (cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      s.sms <= 0) {
    return nullptr;
  }
  for (int prov = 0; prov < 2; ++prov) {
    for (int mode = 0; mode < 3; ++mode) {
      if (prepare_quantize(prov != 0, mode, &s.quantize_blocks[prov][mode]) != cudaSuccess ||
          s.quantize_blocks[prov][mode] < 1) {
        return nullptr;
      }
    }
    for (int comp = 0; comp < 2; ++comp) {
      if (prepare_dequantize(prov != 0, comp != 0, &s.dequantize_blocks[prov][comp]) !=
              cudaSuccess ||
          s.dequantize_blocks[prov][comp] < 1) {
        return nullptr;
      }
      if (prepare_project(prov != 0, comp != 0, &s.project_blocks[prov][comp]) != cudaSuccess ||
          s.project_blocks[prov][comp] < 1) {
        return nullptr;
      }
    }
  }
  if (prepare_fit(&s.fit_blocks) != cudaSuccess || s.fit_blocks < 1) return nullptr;
  if (prepare_capsule() != cudaSuccess) return nullptr;
  if (prepare_window(&s.window) != cudaSuccess || s.window.fold < 1 || s.window.dense < 1 ||
      s.window.window_dense[0] < 1 || s.window.window_dense[1] < 1 ||
      s.window.step[0][0] < 1 || s.window.step[0][1] < 1 || s.window.step[1][0] < 1 ||
      s.window.step[1][1] < 1 || s.window.step_staged[0] < 1 || s.window.step_staged[1] < 1) {
    return nullptr;
  }
  s.ready = true;
  return &s;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

int grid_for(uint64_t work_units, int sms, int blocks_per_sm) {
  const uint64_t resident = static_cast<uint64_t>(sms) * static_cast<uint64_t>(blocks_per_sm);
  return static_cast<int>(work_units < resident ? work_units : resident);
}

int32_t run_quantize(void* stream, bool provider, int mode, const float* state,
                     const float* smoothing_in, float* smoothing, int8_t* codes, float* scales,
                     uint64_t items, SlotMap map, uint32_t* status,
                     uint64_t wait_limit_ns = kWaitLimitNs, uint32_t arm_only = 0u) {
  const DeviceSetup* s = device_setup();
  if (s == nullptr) return kSetupFailed;
  QuantizeParams p{state, smoothing_in, smoothing, codes, scales, items, map, status};
  p.wait_limit_ns = wait_limit_ns;
  p.arm_only = arm_only;
  const uint64_t units = (items + quantize_units_per_block() - 1) / quantize_units_per_block();
  const int grid = grid_for(units, s->sms, s->quantize_blocks[provider][mode]);
  return launch_quantize(provider, mode, p, grid, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? kOk
             : kLaunchFailed;
}

int32_t run_dequantize(void* stream, bool provider, const int8_t* codes, const float* smoothing,
                       const float* scales, const float* ck, const float* cv, float* dense,
                       uint64_t items, SlotMap map, uint32_t* status) {
  const DeviceSetup* s = device_setup();
  if (s == nullptr) return kSetupFailed;
  const bool comp = ck != nullptr;
  DequantizeParams p{codes, smoothing, scales, ck, cv, dense, items, map, status};
  const int grid = grid_for(items, s->sms, s->dequantize_blocks[provider][comp]);
  return launch_dequantize(provider, p, grid, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? kOk
             : kLaunchFailed;
}

int32_t run_project(void* stream, bool provider, const int8_t* codes, const float* smoothing,
                    const float* scales, const float* ck, const float* cv,
                    const uint16_t* queries, float* outputs, uint64_t items, SlotMap map,
                    uint32_t* status, uint64_t wait_limit_ns = kWaitLimitNs,
                    uint32_t arm_only = 0u) {
  const DeviceSetup* s = device_setup();
  if (s == nullptr) return kSetupFailed;
  const bool comp = ck != nullptr;
  ProjectParams p{codes, smoothing, scales, ck, cv, queries, outputs, items, map, status};
  p.wait_limit_ns = wait_limit_ns;
  p.arm_only = arm_only;
  const uint64_t blocks = (items + 3) / 4;  // four warps (heads) per block
  const int grid = grid_for(blocks, s->sms, s->project_blocks[provider][comp]);
  return launch_project(provider, p, grid, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? kOk
             : kLaunchFailed;
}

int32_t run_full(void* stream, bool provider, const float* dense, float* residual,
                 float* smoothing, int8_t* codes, float* scales, float* ck, float* cv,
                 uint64_t heads, uint32_t* status) {
  const DeviceSetup* s = device_setup();
  if (s == nullptr) return kSetupFailed;
  FitParams f{dense, residual, ck, cv, heads, status, provider ? 1 : 0};
  const int grid = grid_for(heads, s->sms, s->fit_blocks);
  if (launch_fit(f, grid, static_cast<cudaStream_t>(stream)) != cudaSuccess) return kLaunchFailed;
  return run_quantize(stream, provider, kFused, residual, nullptr, smoothing, codes, scales, heads,
                      SlotMap{nullptr, 1, 1}, status);
}

bool compensators_ok(const float* ck, const float* cv) {
  if ((ck == nullptr) != (cv == nullptr)) return false;
  return ck == nullptr || (aligned16(ck) && aligned16(cv));
}

bool indexed_ok(uint32_t layout, const int32_t* slot_ids, uint32_t count,
                uint32_t heads_per_slot, uint32_t num_slots) {
  return layout <= 1u && slot_ids != nullptr && count != 0u && heads_per_slot != 0u &&
         num_slots != 0u && (reinterpret_cast<uintptr_t>(slot_ids) & 3u) == 0;
}

}  // namespace
}  // namespace gdnsc

using gdnsc::SlotMap;
using gdnsc::aligned16;
using gdnsc::aligned8;

extern "C" {

// ---- Reference entry points -------------------------------------------------

int32_t statecentric_gdn_state_codec_smoothing_launch_v1(void* stream, const float* residual,
                                                         float* smoothing) {
  if (residual == nullptr || smoothing == nullptr || !aligned16(residual) ||
      !aligned16(smoothing)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_quantize(stream, false, gdnsc::kSmoothingOnly, residual, nullptr, smoothing,
                             nullptr, nullptr, 1, SlotMap{nullptr, 1, 1}, nullptr);
}

int32_t statecentric_gdn_state_codec_provider_smoothing_launch_v2(void* stream,
                                                                  const float* provider_state,
                                                                  float* smoothing,
                                                                  uint32_t states) {
  if (provider_state == nullptr || smoothing == nullptr || states == 0u ||
      !aligned16(provider_state) || !aligned16(smoothing)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_quantize(stream, true, gdnsc::kSmoothingOnly, provider_state, nullptr,
                             smoothing, nullptr, nullptr, states, SlotMap{nullptr, 1, 1},
                             nullptr);
}

int32_t statecentric_gdn_state_codec_quantize_launch_v1(void* stream, const float* residual,
                                                        const float* smoothing,
                                                        int8_t* quantized, float* value_scales) {
  if (residual == nullptr || smoothing == nullptr || quantized == nullptr ||
      value_scales == nullptr || !aligned16(residual) || !aligned16(smoothing) ||
      !aligned16(quantized) || !aligned16(value_scales)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_quantize(stream, false, gdnsc::kGivenSmoothing, residual, smoothing, nullptr,
                             quantized, value_scales, 1, SlotMap{nullptr, 1, 1}, nullptr);
}

int32_t statecentric_gdn_state_codec_provider_quantize_launch_v2(
    void* stream, const float* provider_state, const float* smoothing, int8_t* quantized,
    float* value_scales, uint32_t states) {
  if (provider_state == nullptr || smoothing == nullptr || quantized == nullptr ||
      value_scales == nullptr || states == 0u || !aligned16(provider_state) ||
      !aligned16(smoothing) || !aligned16(quantized) || !aligned16(value_scales)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_quantize(stream, true, gdnsc::kGivenSmoothing, provider_state, smoothing,
                             nullptr, quantized, value_scales, states, SlotMap{nullptr, 1, 1},
                             nullptr);
}

int32_t statecentric_gdn_state_codec_provider_initialize_launch_v3(
    void* stream, const float* provider_state, float* smoothing, int8_t* quantized,
    float* value_scales, uint32_t states) {
  if (provider_state == nullptr || smoothing == nullptr || quantized == nullptr ||
      value_scales == nullptr || states == 0u || !aligned16(provider_state) ||
      !aligned16(smoothing) || !aligned16(quantized) || !aligned16(value_scales)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_quantize(stream, true, gdnsc::kFused, provider_state, nullptr, smoothing,
                             quantized, value_scales, states, SlotMap{nullptr, 1, 1}, nullptr);
}

int32_t statecentric_gdn_state_codec_dequantize_launch_v1(
    void* stream, const int8_t* quantized, const float* smoothing, const float* value_scales,
    const float* compensator_keys, const float* compensator_values, float* dense) {
  // The reference's single-head launcher requires both compensators.
  if (quantized == nullptr || smoothing == nullptr || value_scales == nullptr ||
      compensator_keys == nullptr || compensator_values == nullptr || dense == nullptr ||
      !aligned16(quantized) || !aligned16(smoothing) || !aligned16(value_scales) ||
      !aligned16(dense) || !gdnsc::compensators_ok(compensator_keys, compensator_values)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_dequantize(stream, false, quantized, smoothing, value_scales,
                               compensator_keys, compensator_values, dense, 1,
                               SlotMap{nullptr, 1, 1}, nullptr);
}

// ---- Batched extensions -------------------------------------------------------

int32_t statecentric_gdn_state_codec_initialize_launch_v3(void* stream, const float* residual,
                                                          float* smoothing, int8_t* quantized,
                                                          float* value_scales, uint32_t states) {
  if (residual == nullptr || smoothing == nullptr || quantized == nullptr ||
      value_scales == nullptr || states == 0u || !aligned16(residual) || !aligned16(smoothing) ||
      !aligned16(quantized) || !aligned16(value_scales)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_quantize(stream, false, gdnsc::kFused, residual, nullptr, smoothing,
                             quantized, value_scales, states, SlotMap{nullptr, 1, 1}, nullptr);
}

static int32_t dequantize_batched(void* stream, bool provider, const int8_t* quantized,
                                  const float* smoothing, const float* value_scales,
                                  const float* ck, const float* cv, float* dense,
                                  uint32_t states) {
  if (quantized == nullptr || smoothing == nullptr || value_scales == nullptr ||
      dense == nullptr || states == 0u || !aligned16(quantized) || !aligned16(smoothing) ||
      !aligned16(value_scales) || !aligned16(dense) || !gdnsc::compensators_ok(ck, cv)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_dequantize(stream, provider, quantized, smoothing, value_scales, ck, cv,
                               dense, states, SlotMap{nullptr, 1, 1}, nullptr);
}

int32_t statecentric_gdn_state_codec_dequantize_launch_v2(
    void* stream, const int8_t* quantized, const float* smoothing, const float* value_scales,
    const float* compensator_keys, const float* compensator_values, float* dense,
    uint32_t states) {
  return dequantize_batched(stream, false, quantized, smoothing, value_scales, compensator_keys,
                            compensator_values, dense, states);
}

int32_t statecentric_gdn_state_codec_provider_dequantize_launch_v2(
    void* stream, const int8_t* quantized, const float* smoothing, const float* value_scales,
    const float* compensator_keys, const float* compensator_values, float* dense,
    uint32_t states) {
  return dequantize_batched(stream, true, quantized, smoothing, value_scales, compensator_keys,
                            compensator_values, dense, states);
}

static int32_t project_batched(void* stream, bool provider, const int8_t* residual,
                               const float* smoothing, const float* scales, const float* ck,
                               const float* cv, const uint16_t* queries, float* outputs,
                               uint32_t states) {
  if (residual == nullptr || smoothing == nullptr || scales == nullptr || queries == nullptr ||
      outputs == nullptr || states == 0u || !aligned16(residual) || !aligned16(smoothing) ||
      !aligned16(scales) || !aligned8(queries) || !aligned16(outputs) ||
      !gdnsc::compensators_ok(ck, cv)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_project(stream, provider, residual, smoothing, scales, ck, cv, queries,
                            outputs, states, SlotMap{nullptr, 1, 1}, nullptr);
}

int32_t statecentric_gdn_state_codec_encoded_projection_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing, const float* scales,
    const float* compensator_keys, const float* compensator_values, const uint16_t* queries_bf16,
    float* outputs, uint32_t states) {
  return project_batched(stream, false, residual, smoothing, scales, compensator_keys,
                         compensator_values, queries_bf16, outputs, states);
}

int32_t statecentric_gdn_state_codec_provider_encoded_projection_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing, const float* scales,
    const float* compensator_keys, const float* compensator_values, const uint16_t* queries_bf16,
    float* outputs, uint32_t states) {
  return project_batched(stream, true, residual, smoothing, scales, compensator_keys,
                         compensator_values, queries_bf16, outputs, states);
}

// ---- Slot-indexed extensions ----------------------------------------------------

int32_t statecentric_gdn_state_codec_initialize_indexed_launch_v1(
    void* stream, uint32_t layout, const float* state_cache, float* smoothing_cache,
    int8_t* codes_cache, float* scales_cache, const int32_t* slot_ids, uint32_t count,
    uint32_t heads_per_slot, uint32_t num_slots, uint32_t* status) {
  if (!gdnsc::indexed_ok(layout, slot_ids, count, heads_per_slot, num_slots) ||
      state_cache == nullptr || smoothing_cache == nullptr || codes_cache == nullptr ||
      scales_cache == nullptr || !aligned16(state_cache) || !aligned16(smoothing_cache) ||
      !aligned16(codes_cache) || !aligned16(scales_cache)) {
    return gdnsc::kBadArgs;
  }
  const uint64_t items = static_cast<uint64_t>(count) * heads_per_slot;
  return gdnsc::run_quantize(stream, layout == 1u, gdnsc::kFused, state_cache, nullptr,
                             smoothing_cache, codes_cache, scales_cache, items,
                             SlotMap{slot_ids, heads_per_slot, num_slots}, status);
}

int32_t statecentric_gdn_state_codec_dequantize_indexed_launch_v1(
    void* stream, uint32_t layout, const int8_t* codes_cache, const float* smoothing_cache,
    const float* scales_cache, const float* compensator_keys_cache,
    const float* compensator_values_cache, float* state_cache, const int32_t* slot_ids,
    uint32_t count, uint32_t heads_per_slot, uint32_t num_slots, uint32_t* status) {
  if (!gdnsc::indexed_ok(layout, slot_ids, count, heads_per_slot, num_slots) ||
      codes_cache == nullptr || smoothing_cache == nullptr || scales_cache == nullptr ||
      state_cache == nullptr || !aligned16(codes_cache) || !aligned16(smoothing_cache) ||
      !aligned16(scales_cache) || !aligned16(state_cache) ||
      !gdnsc::compensators_ok(compensator_keys_cache, compensator_values_cache)) {
    return gdnsc::kBadArgs;
  }
  const uint64_t items = static_cast<uint64_t>(count) * heads_per_slot;
  return gdnsc::run_dequantize(stream, layout == 1u, codes_cache, smoothing_cache, scales_cache,
                               compensator_keys_cache, compensator_values_cache, state_cache,
                               items, SlotMap{slot_ids, heads_per_slot, num_slots}, status);
}

int32_t statecentric_gdn_state_codec_encoded_projection_indexed_launch_v1(
    void* stream, uint32_t layout, const int8_t* codes_cache, const float* smoothing_cache,
    const float* scales_cache, const float* compensator_keys_cache,
    const float* compensator_values_cache, const uint16_t* queries_bf16, float* outputs,
    const int32_t* slot_ids, uint32_t count, uint32_t heads_per_slot, uint32_t num_slots,
    uint32_t* status) {
  if (!gdnsc::indexed_ok(layout, slot_ids, count, heads_per_slot, num_slots) ||
      codes_cache == nullptr || smoothing_cache == nullptr || scales_cache == nullptr ||
      queries_bf16 == nullptr || outputs == nullptr || !aligned16(codes_cache) ||
      !aligned16(smoothing_cache) || !aligned16(scales_cache) || !aligned8(queries_bf16) ||
      !aligned16(outputs) ||
      !gdnsc::compensators_ok(compensator_keys_cache, compensator_values_cache)) {
    return gdnsc::kBadArgs;
  }
  const uint64_t items = static_cast<uint64_t>(count) * heads_per_slot;
  return gdnsc::run_project(stream, layout == 1u, codes_cache, smoothing_cache, scales_cache,
                            compensator_keys_cache, compensator_values_cache, queries_bf16,
                            outputs, items, SlotMap{slot_ids, heads_per_slot, num_slots}, status);
}

// ---- Full codec ------------------------------------------------------------------

int32_t statecentric_gdn_state_codec_full_initialize_launch_v1(
    void* stream, uint32_t layout, const float* dense, float* residual_workspace,
    float* smoothing, int8_t* quantized, float* value_scales, float* compensator_keys,
    float* compensator_values, uint32_t states, uint32_t* status) {
  if (layout > 1u || dense == nullptr || residual_workspace == nullptr || smoothing == nullptr ||
      quantized == nullptr || value_scales == nullptr || compensator_keys == nullptr ||
      compensator_values == nullptr || states == 0u || !aligned16(dense) ||
      !aligned16(residual_workspace) || !aligned16(smoothing) || !aligned16(quantized) ||
      !aligned16(value_scales) || !aligned16(compensator_keys) || !aligned16(compensator_values)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_full(stream, layout == 1u, dense, residual_workspace, smoothing, quantized,
                         value_scales, compensator_keys, compensator_values, states, status);
}

// ---- Capsule wire format ------------------------------------------------------------

namespace gdnsc {
namespace {

bool identity_ok(const char* geometry, uint64_t generation, uint64_t epoch) {
  return geometry != nullptr && lowercase_hex64(geometry) && generation > 0 && epoch > 0;
}

CapsuleIdentity make_identity(const char* geometry, uint64_t generation, uint64_t epoch) {
  CapsuleIdentity id{};
  std::memcpy(id.geometry, geometry, sizeof(id.geometry));
  id.generation = generation;
  id.epoch = epoch;
  return id;
}

}  // namespace
}  // namespace gdnsc

int32_t statecentric_gdn_state_codec_capsule_serialize_launch_v1(
    void* stream, uint32_t layout, const int8_t* codes, const float* smoothing,
    const float* scales, const float* compensator_keys, const float* compensator_values,
    const char* model_geometry_sha256, uint64_t generation, uint64_t epoch, uint8_t* capsules,
    uint32_t states) {
  if (layout > 1u || codes == nullptr || smoothing == nullptr || scales == nullptr ||
      capsules == nullptr || states == 0u || !aligned16(codes) || !aligned16(smoothing) ||
      !aligned16(scales) || !aligned8(capsules) ||
      !gdnsc::compensators_ok(compensator_keys, compensator_values) ||
      !gdnsc::identity_ok(model_geometry_sha256, generation, epoch)) {
    return gdnsc::kBadArgs;
  }
  const gdnsc::DeviceSetup* s = gdnsc::device_setup();
  if (s == nullptr) return gdnsc::kSetupFailed;
  gdnsc::SerializeParams p{codes, smoothing, scales, compensator_keys, compensator_values,
                           capsules, states, static_cast<int>(layout),
                           gdnsc::make_identity(model_geometry_sha256, generation, epoch)};
  const auto st = static_cast<cudaStream_t>(stream);
  constexpr int kWarps = gdnsc::kCapsuleThreads / 32;
  const int assemble_grid = gdnsc::grid_for((states + kWarps - 1) / kWarps, s->sms, 16);
  gdnsc::capsule_assemble_kernel<<<assemble_grid, gdnsc::kCapsuleThreads, 0, st>>>(p);
  if (cudaGetLastError() != cudaSuccess) return gdnsc::kLaunchFailed;
  const unsigned digest_grid = (states + gdnsc::kCapsuleThreads - 1) / gdnsc::kCapsuleThreads;
  gdnsc::capsule_digest_kernel<<<digest_grid, gdnsc::kCapsuleThreads, 0, st>>>(capsules, states);
  return cudaGetLastError() == cudaSuccess ? gdnsc::kOk : gdnsc::kLaunchFailed;
}

int32_t statecentric_gdn_state_codec_capsule_restore_launch_v1(
    void* stream, uint32_t layout, const uint8_t* capsules, const char* model_geometry_sha256,
    uint64_t generation, uint64_t epoch, int8_t* codes, float* smoothing, float* scales,
    float* compensator_keys, float* compensator_values, int32_t* head_status, uint32_t states) {
  if (layout > 1u || capsules == nullptr || codes == nullptr || smoothing == nullptr ||
      scales == nullptr || compensator_keys == nullptr || compensator_values == nullptr ||
      head_status == nullptr || states == 0u || !aligned8(capsules) || !aligned16(codes) ||
      !aligned16(smoothing) || !aligned16(scales) || !aligned16(compensator_keys) ||
      !aligned16(compensator_values) || (reinterpret_cast<uintptr_t>(head_status) & 3u) != 0 ||
      !gdnsc::identity_ok(model_geometry_sha256, generation, epoch)) {
    return gdnsc::kBadArgs;
  }
  const gdnsc::DeviceSetup* s = gdnsc::device_setup();
  if (s == nullptr) return gdnsc::kSetupFailed;
  gdnsc::RestoreParams p{capsules, codes, smoothing, scales, compensator_keys,
                         compensator_values, head_status, states, static_cast<int>(layout),
                         gdnsc::make_identity(model_geometry_sha256, generation, epoch)};
  const auto st = static_cast<cudaStream_t>(stream);
  const unsigned verify_grid = (states + gdnsc::kVerifyThreads - 1) / gdnsc::kVerifyThreads;
  gdnsc::capsule_verify_kernel<<<verify_grid, gdnsc::kVerifyThreads, 0, st>>>(p);
  if (cudaGetLastError() != cudaSuccess) return gdnsc::kLaunchFailed;
  gdnsc::capsule_payload_kernel<<<gdnsc::grid_for(states, s->sms, 8), gdnsc::kCapsuleThreads, 0,
                                  st>>>(p);
  return cudaGetLastError() == cudaSuccess ? gdnsc::kOk : gdnsc::kLaunchFailed;
}

int32_t statecentric_gdn_state_codec_sha256_v1(const uint8_t* data, uint64_t size,
                                               char* hex64) {
  if ((data == nullptr && size != 0) || hex64 == nullptr) return gdnsc::kBadArgs;
  uint32_t h[8];
  gdnsc::sha256(data, size, h);
  gdnsc::sha256_hex(h, hex64);
  return gdnsc::kOk;
}

// ---- Full codec without a caller workspace ----------------------------------------
//
// Some callers cannot allocate device memory on the call path: a serving
// engine that has already handed nearly all of the GPU's memory to its state
// and KV cache pools after profiling, or a host process that owns every
// device allocation; cudaMalloc would also synchronize the device.  For them
// the full encode can keep the residual between its two stages in a static
// device array instead of a caller workspace.  The array is loaded with the
// library and held by every GPU that loads it until the process exits.

namespace gdnsc {
namespace {

constexpr uint32_t kStaticFullMaxStates = 64;  // 64 heads x 64 KiB = 4 MiB
static __device__ __align__(256) float g_full_residual_scratch[kStaticFullMaxStates * kElements];

std::mutex g_scratch_mutex;
float* g_scratch_address[kMaxDevices] = {};

// Device address of the static array on the current device, looked up once
// per device (the array's host-side name is not a device address).
float* static_full_scratch() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[device] == nullptr) {
    void* address = nullptr;
    if (cudaGetSymbolAddress(&address, g_full_residual_scratch) != cudaSuccess) return nullptr;
    g_scratch_address[device] = static_cast<float*>(address);
  }
  return g_scratch_address[device];
}

}  // namespace
}  // namespace gdnsc

int32_t statecentric_gdn_state_codec_full_initialize_static_launch_v1(
    void* stream, uint32_t layout, const float* dense, float* smoothing, int8_t* quantized,
    float* value_scales, float* compensator_keys, float* compensator_values, uint32_t states,
    uint32_t* status) {
  if (states > gdnsc::kStaticFullMaxStates) return gdnsc::kBadArgs;  // over the array's size
  if (layout > 1u || dense == nullptr || smoothing == nullptr || quantized == nullptr ||
      value_scales == nullptr || compensator_keys == nullptr || compensator_values == nullptr ||
      states == 0u || !aligned16(dense) || !aligned16(smoothing) || !aligned16(quantized) ||
      !aligned16(value_scales) || !aligned16(compensator_keys) || !aligned16(compensator_values)) {
    return gdnsc::kBadArgs;
  }
  float* scratch = gdnsc::static_full_scratch();
  if (scratch == nullptr) return gdnsc::kSetupFailed;
  // The fit overwrites every element of the scratch it uses before the int8
  // stage reads it, so nothing left by an earlier call needs clearing.
  return gdnsc::run_full(stream, layout == 1u, dense, scratch, smoothing, quantized,
                         value_scales, compensator_keys, compensator_values, states, status);
}

// ---- Status and synthetic inputs --------------------------------------------------

int32_t statecentric_gdn_state_codec_device_error_v1(uint32_t* bits, int32_t clear) {
  if (bits == nullptr) return gdnsc::kBadArgs;
  if (cudaMemcpyFromSymbol(bits, gdnsc::g_device_error, sizeof(uint32_t)) != cudaSuccess) {
    return gdnsc::kLaunchFailed;
  }
  if (clear != 0) {
    const uint32_t zero = 0u;
    if (cudaMemcpyToSymbol(gdnsc::g_device_error, &zero, sizeof(uint32_t)) != cudaSuccess) {
      return gdnsc::kLaunchFailed;
    }
  }
  return gdnsc::kOk;
}

int32_t statecentric_gdn_state_codec_synthesize_states_v1(void* stream, float* out,
                                                          uint32_t layout, uint64_t seed,
                                                          uint32_t slot_base, uint32_t slots,
                                                          uint32_t layers,
                                                          uint32_t heads_per_layer) {
  if (out == nullptr || layout > 1u || slots == 0u || layers == 0u || heads_per_layer == 0u ||
      !aligned16(out)) {
    return gdnsc::kBadArgs;
  }
  const gdnsc::DeviceSetup* s = gdnsc::device_setup();
  if (s == nullptr) return gdnsc::kSetupFailed;
  gdnsc::SynthParams p{out, static_cast<uint64_t>(slots) * layers * heads_per_layer, seed,
                       slot_base, layers, heads_per_layer, layout};
  return gdnsc::launch_synth_states(p, s->sms, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? gdnsc::kOk
             : gdnsc::kLaunchFailed;
}

int32_t statecentric_gdn_state_codec_synthesize_queries_v1(void* stream, uint16_t* out,
                                                           uint64_t seed, uint32_t slot_base,
                                                           uint32_t slots, uint32_t layers,
                                                           uint32_t heads_per_layer) {
  if (out == nullptr || slots == 0u || layers == 0u || heads_per_layer == 0u || !aligned8(out)) {
    return gdnsc::kBadArgs;
  }
  const gdnsc::DeviceSetup* s = gdnsc::device_setup();
  if (s == nullptr) return gdnsc::kSetupFailed;
  gdnsc::SynthParams p{out, static_cast<uint64_t>(slots) * layers * heads_per_layer, seed,
                       slot_base, layers, heads_per_layer, 0u};
  return gdnsc::launch_synth_queries(p, s->sms, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? gdnsc::kOk
             : gdnsc::kLaunchFailed;
}

int32_t statecentric_gdn_state_codec_division_selftest_v1(void* stream, const float* numerators,
                                                          const float* divisors, float* quotients,
                                                          uint64_t count) {
  if (numerators == nullptr || divisors == nullptr || quotients == nullptr || count == 0u) {
    return gdnsc::kBadArgs;
  }
  const gdnsc::DeviceSetup* s = gdnsc::device_setup();
  if (s == nullptr) return gdnsc::kSetupFailed;
  gdnsc::division_selftest_kernel<<<s->sms * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      numerators, divisors, quotients, count);
  return cudaGetLastError() == cudaSuccess ? gdnsc::kOk : gdnsc::kLaunchFailed;
}

// Test support: the capsule quantize and encoded projection with every
// bounded wait made to run out (barriers armed, no copy issued).
int32_t statecentric_gdn_state_codec_quantize_wait_selftest_v1(
    void* stream, const float* residual, float* smoothing, int8_t* quantized, float* value_scales,
    uint32_t states, uint64_t limit_ns, uint32_t* status) {
  if (residual == nullptr || smoothing == nullptr || quantized == nullptr ||
      value_scales == nullptr || status == nullptr || states == 0u || limit_ns == 0u ||
      limit_ns > gdnsc::kWaitLimitNs || !aligned16(residual) || !aligned16(smoothing) ||
      !aligned16(quantized) || !aligned16(value_scales)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_quantize(stream, false, gdnsc::kFused, residual, nullptr, smoothing,
                             quantized, value_scales, states, SlotMap{nullptr, 1, 1}, status,
                             limit_ns, 1u);
}

int32_t statecentric_gdn_state_codec_encoded_projection_wait_selftest_v1(
    void* stream, const int8_t* residual, const float* smoothing, const float* scales,
    const uint16_t* queries_bf16, float* outputs, uint32_t states, uint64_t limit_ns,
    uint32_t* status) {
  if (residual == nullptr || smoothing == nullptr || scales == nullptr ||
      queries_bf16 == nullptr || outputs == nullptr || status == nullptr || states == 0u ||
      limit_ns == 0u || limit_ns > gdnsc::kWaitLimitNs || !aligned16(residual) ||
      !aligned16(smoothing) || !aligned16(scales) || !aligned16(outputs) ||
      !gdnsc::aligned8(queries_bf16)) {
    return gdnsc::kBadArgs;
  }
  return gdnsc::run_project(stream, false, residual, smoothing, scales, nullptr, nullptr,
                            queries_bf16, outputs, states, SlotMap{nullptr, 1, 1}, status,
                            limit_ns, 1u);
}

// ---- Windowed decode: step, boundary refit, dense fp32 step -------------------

namespace gdnsc {
namespace {

bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }
bool aligned2(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 1u) == 0; }

// The window buffers every step / refit reads: all 16-byte aligned (the
// kernels load codes, smoothing pairs, compensator rows and record-key pairs
// as vectors).
bool window_ok(const WindowBuffers& w, bool need_compensators) {
  if (w.codes == nullptr || w.smoothing == nullptr || w.scales == nullptr ||
      w.record_decay == nullptr || w.record_keys == nullptr || w.record_corrections == nullptr ||
      w.positions == nullptr) {
    return false;
  }
  if ((w.ck == nullptr) != (w.cv == nullptr)) return false;
  if (need_compensators && w.ck == nullptr) return false;
  if (w.ck != nullptr && (!aligned16(w.ck) || !aligned16(w.cv))) return false;
  return aligned16(w.codes) && aligned16(w.smoothing) && aligned16(w.scales) &&
         aligned16(w.record_decay) && aligned16(w.record_keys) &&
         aligned16(w.record_corrections) && aligned16(w.positions);
}

int32_t run_window_step(void* stream, bool qwen, bool comp, const StepParams& p) {
  const DeviceSetup* s = device_setup();
  if (s == nullptr) return kSetupFailed;
  // The staged Qwen step copies key, query and value rows and the beta pair
  // with cp.async: 16-byte aligned rows and a 4-byte aligned beta.
  if (qwen && aligned16(p.keys) && aligned16(p.queries) && aligned16(p.values) &&
      aligned4(p.beta)) {
    const int grid = grid_for(p.heads, s->sms, s->window.step_staged[comp]);
    return launch_window_step_staged(comp, p, grid, static_cast<cudaStream_t>(stream)) ==
                   cudaSuccess
               ? kOk
               : kLaunchFailed;
  }
  const int grid = grid_for(p.heads, s->sms, s->window.step[qwen][comp]);
  return launch_window_step(qwen, comp, p, grid, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? kOk
             : kLaunchFailed;
}

}  // namespace
}  // namespace gdnsc

int32_t statecentric_gdn_state_codec_windowed_gdn_step_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing, const float* scales,
    const uint16_t* compensator_keys, const uint16_t* compensator_values, float* record_decay,
    uint16_t* record_keys, uint16_t* record_corrections, uint32_t* positions, const float* decay,
    const uint16_t* write_keys, const uint16_t* reads, const uint16_t* queries,
    const uint16_t* values, float* outputs, uint32_t states) {
  const gdnsc::WindowBuffers w{residual, smoothing, scales, compensator_keys, compensator_values,
                               record_decay, record_keys, record_corrections, positions};
  if (!gdnsc::window_ok(w, true) || decay == nullptr || write_keys == nullptr ||
      reads == nullptr || queries == nullptr || values == nullptr || outputs == nullptr ||
      states == 0u || !gdnsc::aligned4(decay) || !gdnsc::aligned2(write_keys) ||
      !gdnsc::aligned2(reads) || !gdnsc::aligned2(queries) || !gdnsc::aligned2(values) ||
      !gdnsc::aligned4(outputs)) {
    return gdnsc::kBadArgs;
  }
  const gdnsc::StepParams p{w, decay, nullptr, write_keys, reads, queries, values, outputs,
                            states};
  return gdnsc::run_window_step(stream, false, true, p);
}

namespace {

int32_t window_step_bf16(void* stream, bool comp, const int8_t* residual, const float* smoothing,
                         const float* scales, const uint16_t* compensator_keys,
                         const uint16_t* compensator_values, float* record_decay,
                         uint16_t* record_keys, uint16_t* record_corrections,
                         uint32_t* positions, const float* decay, const uint16_t* beta,
                         const uint16_t* keys, const uint16_t* queries, const uint16_t* values,
                         uint16_t* outputs, uint32_t states) {
  const gdnsc::WindowBuffers w{residual,     smoothing,   scales,
                               comp ? compensator_keys : nullptr,
                               comp ? compensator_values : nullptr,
                               record_decay, record_keys, record_corrections, positions};
  if ((compensator_keys == nullptr) != (compensator_values == nullptr) ||
      !gdnsc::window_ok(w, comp) || decay == nullptr || beta == nullptr || keys == nullptr ||
      queries == nullptr || values == nullptr || outputs == nullptr || states == 0u ||
      states % 2u != 0u || !gdnsc::aligned4(decay) || !gdnsc::aligned2(beta) ||
      !gdnsc::aligned2(keys) || !gdnsc::aligned2(queries) || !gdnsc::aligned2(values) ||
      !gdnsc::aligned2(outputs)) {
    return gdnsc::kBadArgs;
  }
  const gdnsc::StepParams p{w, decay, beta, keys, nullptr, queries, values, outputs, states};
  return gdnsc::run_window_step(stream, true, comp, p);
}

}  // namespace

int32_t statecentric_gdn_state_codec_windowed_gdn_step_bf16_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing, const float* scales,
    const uint16_t* compensator_keys, const uint16_t* compensator_values, float* record_decay,
    uint16_t* record_keys, uint16_t* record_corrections, uint32_t* positions, const float* decay,
    const uint16_t* beta, const uint16_t* keys, const uint16_t* queries, const uint16_t* values,
    uint16_t* outputs, uint32_t states) {
  return window_step_bf16(stream, true, residual, smoothing, scales, compensator_keys,
                          compensator_values, record_decay, record_keys, record_corrections,
                          positions, decay, beta, keys, queries, values, outputs, states);
}

int32_t statecentric_gdn_state_codec_windowed_gdn_step_bf16_quant_only_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing, const float* scales,
    const uint16_t* compensator_keys, const uint16_t* compensator_values, float* record_decay,
    uint16_t* record_keys, uint16_t* record_corrections, uint32_t* positions, const float* decay,
    const uint16_t* beta, const uint16_t* keys, const uint16_t* queries, const uint16_t* values,
    uint16_t* outputs, uint32_t states) {
  return window_step_bf16(stream, false, residual, smoothing, scales, compensator_keys,
                          compensator_values, record_decay, record_keys, record_corrections,
                          positions, decay, beta, keys, queries, values, outputs, states);
}

int32_t statecentric_gdn_state_codec_window_boundary_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing, const float* scales,
    const uint16_t* compensator_keys, const uint16_t* compensator_values, float* record_decay,
    uint16_t* record_keys, uint16_t* record_corrections, uint32_t* positions,
    int8_t* next_residual, float* next_smoothing, float* next_scales,
    uint16_t* next_compensator_keys, uint16_t* next_compensator_values, float* residual_workspace,
    uint32_t states, uint32_t power_iterations) {
  const gdnsc::WindowBuffers w{residual, smoothing, scales, compensator_keys, compensator_values,
                               record_decay, record_keys, record_corrections, positions};
  if (!gdnsc::window_ok(w, false) || next_residual == nullptr || next_smoothing == nullptr ||
      next_scales == nullptr || next_compensator_keys == nullptr ||
      next_compensator_values == nullptr || residual_workspace == nullptr || states == 0u ||
      power_iterations > 32u || !aligned16(next_residual) || !aligned16(next_smoothing) ||
      !aligned16(next_scales) || !aligned16(next_compensator_keys) ||
      !aligned16(next_compensator_values) || !aligned16(residual_workspace)) {
    return gdnsc::kBadArgs;
  }
  const gdnsc::DeviceSetup* s = gdnsc::device_setup();
  if (s == nullptr) return gdnsc::kSetupFailed;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const gdnsc::FoldParams fp{w, next_compensator_keys, next_compensator_values,
                             residual_workspace, states, static_cast<int>(power_iterations)};
  // The quant-only refit streams the window's dense state; with power
  // iterations the fit kernel folds and fits each head in shared memory.
  const cudaError_t err =
      power_iterations == 0u
          ? gdnsc::launch_window_dense(
                fp, gdnsc::grid_for(states, s->sms, s->window.window_dense[w.ck != nullptr]), st)
          : gdnsc::launch_window_fold(fp, gdnsc::grid_for(states, s->sms, s->window.fold), st);
  if (err != cudaSuccess) return gdnsc::kLaunchFailed;
  return gdnsc::run_quantize(stream, true, gdnsc::kFused, residual_workspace, nullptr,
                             next_smoothing, next_residual, next_scales, states,
                             SlotMap{nullptr, 1, 1}, nullptr);
}

int32_t statecentric_gdn_state_codec_fp32_gdn_step_launch_v1(
    void* stream, float* dense_state, const float* decay, const uint16_t* key,
    const uint16_t* read, const uint16_t* query, const uint16_t* value, float* output,
    uint32_t states) {
  if (dense_state == nullptr || decay == nullptr || key == nullptr || read == nullptr ||
      query == nullptr || value == nullptr || output == nullptr || states == 0u ||
      !gdnsc::aligned16(dense_state) || !gdnsc::aligned4(decay) || !gdnsc::aligned2(key) ||
      !gdnsc::aligned2(read) || !gdnsc::aligned2(query) || !gdnsc::aligned2(value) ||
      !gdnsc::aligned4(output)) {
    return gdnsc::kBadArgs;
  }
  const gdnsc::DeviceSetup* s = gdnsc::device_setup();
  if (s == nullptr) return gdnsc::kSetupFailed;
  const gdnsc::DenseStepParams p{dense_state, decay, key, read, query, value, output, states};
  return gdnsc::launch_dense_step(p, gdnsc::grid_for(states, s->sms, s->window.dense),
                                  static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? gdnsc::kOk
             : gdnsc::kLaunchFailed;
}

// Test support: the dense fp32 step with its first bounded wait made to run
// out (barrier armed, no copy issued).
int32_t statecentric_gdn_state_codec_fp32_gdn_step_wait_selftest_v1(
    void* stream, float* dense_state, const float* decay, const uint16_t* key,
    const uint16_t* read, const uint16_t* query, const uint16_t* value, float* output,
    uint32_t states, uint64_t limit_ns) {
  if (dense_state == nullptr || decay == nullptr || key == nullptr || read == nullptr ||
      query == nullptr || value == nullptr || output == nullptr || states == 0u ||
      limit_ns == 0u || limit_ns > gdnsc::kWaitLimitNs || !gdnsc::aligned16(dense_state) ||
      !gdnsc::aligned4(decay) || !gdnsc::aligned2(key) || !gdnsc::aligned2(read) ||
      !gdnsc::aligned2(query) || !gdnsc::aligned2(value) || !gdnsc::aligned4(output)) {
    return gdnsc::kBadArgs;
  }
  const gdnsc::DeviceSetup* s = gdnsc::device_setup();
  if (s == nullptr) return gdnsc::kSetupFailed;
  gdnsc::DenseStepParams p{dense_state, decay, key, read, query, value, output, states};
  p.wait_limit_ns = limit_ns;
  p.arm_only = 1u;
  return gdnsc::launch_dense_step(p, gdnsc::grid_for(states, s->sms, s->window.dense),
                                  static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? gdnsc::kOk
             : gdnsc::kLaunchFailed;
}

}  // extern "C"
