/*
 * gdn_state_codec_kernel.h -- C ABI of the B200 (sm_100a) GDN state codec.
 *
 * Drop-in boundary for the quant-only hot path of vLLM-HUST/gdn-state-codec:
 * every entry point the reference declares in native/include/statecentric/
 * gdn_state_codec_kernel.h is kept with the same name, argument order,
 * argument meaning and return convention; the library files that carry them
 * keep the reference's names (libstatecentric_gdn_state_codec_*.so, loaded
 * by src/gdn_state_codec/runtime.py:55-237).
 *
 * Conventions shared by every entry point:
 *  - `stream` is a cudaStream_t.  NULL means the legacy default stream (the
 *    reference rejected a NULL aclrtStream; CUDA's NULL stream is valid).
 *  - All pointers are device pointers owned by the caller; launches allocate
 *    and free nothing and never synchronise the host.  Buffers of 4-byte or
 *    wider elements must be 16-byte aligned (torch allocations are).
 *  - One state ("head") is one [128 x 128] fp32 matrix.  Capsule layout is
 *    [key, value] (reference capsule order, [heads, d_k, d_v]); provider
 *    layout is [value, key] (vLLM ssm_state order).  Codes use the same
 *    layout as the fp32 state they encode; smoothing is per key [128],
 *    value scales are per value [128], compensators are [128][4] fp32.
 *  - Return values: 0 = enqueued; 1 = rejected arguments (null pointer,
 *    zero count, misalignment, bad layout flag); 2 = the CUDA launch failed;
 *    3 = device query or kernel set-up failed.
 *  - `states` may be any value >= 1 (the reference's Ascend launchers
 *    capped it at 64 per launch; this is a documented superset).
 *  - Results are bit-identical to the reference's portable C++ codec
 *    (native/src/gdn_state_codec_state_capsule.cpp) for finite inputs and
 *    positive finite smoothing; non-finite inputs give unspecified codes.
 */
#ifndef STATECENTRIC_GDN_STATE_CODEC_KERNEL_H_
#define STATECENTRIC_GDN_STATE_CODEC_KERNEL_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Reference entry points (gdn_state_codec_kernel.h:5-36) ------------- */

/* One capsule-layout head: c[k] = sqrtf(max(mean_v |R[k][v]|, 1e-8)).
 * Replaces gdn_state_codec_kernel.h:5-6 (libstatecentric_gdn_state_codec_
 * smoothing_kernel.so). */
int32_t statecentric_gdn_state_codec_smoothing_launch_v1(
    void* stream, const float* residual, float* smoothing);

/* `states` provider-layout heads [state][value][key] -> smoothing
 * [state][key].  Replaces gdn_state_codec_kernel.h:11-14. */
int32_t statecentric_gdn_state_codec_provider_smoothing_launch_v2(
    void* stream, const float* provider_state, float* smoothing,
    uint32_t states);

/* One capsule-layout head quantized with the caller's smoothing: codes
 * [key][value], value_scales [value].  Replaces gdn_state_codec_kernel.h:
 * 16-18 (libstatecentric_gdn_state_codec_quantize_kernel.so). */
int32_t statecentric_gdn_state_codec_quantize_launch_v1(
    void* stream, const float* residual, const float* smoothing,
    int8_t* quantized, float* value_scales);

/* Provider-layout heads quantized with the caller's smoothing; codes keep
 * the [state][value][key] order.  Replaces gdn_state_codec_kernel.h:20-23. */
int32_t statecentric_gdn_state_codec_provider_quantize_launch_v2(
    void* stream, const float* provider_state, const float* smoothing,
    int8_t* quantized, float* value_scales, uint32_t states);

/* Fused smoothing + quantize of provider-layout heads: the entry point the
 * vLLM plugin calls (runtime.py:505-517).  One kernel instead of the
 * reference's two (host/gdn_state_codec_provider_runtime.cpp:3-15).
 * Replaces gdn_state_codec_kernel.h:28-31
 * (libstatecentric_gdn_state_codec_provider_runtime.so). */
int32_t statecentric_gdn_state_codec_provider_initialize_launch_v3(
    void* stream, const float* provider_state, float* smoothing,
    int8_t* quantized, float* value_scales, uint32_t states);

/* One capsule-layout head: dense = ((c*z)/127)*b + sum_r K[k][r] V[v][r].
 * compensator_keys / compensator_values are [128][4] fp32.  Replaces
 * gdn_state_codec_kernel.h:33-36
 * (libstatecentric_gdn_state_codec_dequantize_kernel.so). */
int32_t statecentric_gdn_state_codec_dequantize_launch_v1(
    void* stream, const int8_t* quantized, const float* smoothing,
    const float* value_scales, const float* compensator_keys,
    const float* compensator_values, float* dense);

/* ---- Batched and slot-indexed extensions -------------------------------- */
/* The reference exports these only in single-head or Ascend-window forms;
 * the batched forms below follow the same conventions. */

/* Fused smoothing + quantize of `states` capsule-layout heads
 * [state][key][value] (capsule counterpart of provider_initialize_launch_v3,
 * capsule.cpp:190-225 per head). */
int32_t statecentric_gdn_state_codec_initialize_launch_v3(
    void* stream, const float* residual, float* smoothing, int8_t* quantized,
    float* value_scales, uint32_t states);

/* Batched dequantize, capsule layout.  Compensators may both be NULL (the
 * quant-only format, the plugin's default `quant_only` initializer); if one
 * is non-NULL both must be.  Batched form of dequantize_launch_v1. */
int32_t statecentric_gdn_state_codec_dequantize_launch_v2(
    void* stream, const int8_t* quantized, const float* smoothing,
    const float* value_scales, const float* compensator_keys,
    const float* compensator_values, float* dense, uint32_t states);

/* Batched dequantize, provider layout: codes [state][value][key] -> dense
 * [state][value][key] (runtime.py:550-561 `reconstruct`). */
int32_t statecentric_gdn_state_codec_provider_dequantize_launch_v2(
    void* stream, const int8_t* quantized, const float* smoothing,
    const float* value_scales, const float* compensator_keys,
    const float* compensator_values, float* dense, uint32_t states);

/* Encoded projection from capsule-layout codes: outputs[s][v] =
 * (dequant(S_s)^T q_s)[v] computed from the codes without materialising the
 * fp32 state (ReadWindowState boundary term, capsule.cpp:281-304).  queries
 * are bf16 [state][128]; outputs fp32 [state][128].  Compensators nullable
 * as above.  Added to libstatecentric_gdn_state_codec_encoded_projection_
 * kernel.so (native/ascendc/gdn_state_codec/CMakeLists.txt:60-61), whose
 * reference exports are the Ascend window/Cube pieces
 * (gdn_state_codec_windowed_gdn_kernel.h:113-169). */
int32_t statecentric_gdn_state_codec_encoded_projection_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing,
    const float* scales, const float* compensator_keys,
    const float* compensator_values, const uint16_t* queries_bf16,
    float* outputs, uint32_t states);

/* Encoded projection from provider-layout codes [state][value][key] (the
 * plugin's encoded residual order, runtime.py:406-409). */
int32_t statecentric_gdn_state_codec_provider_encoded_projection_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing,
    const float* scales, const float* compensator_keys,
    const float* compensator_values, const uint16_t* queries_bf16,
    float* outputs, uint32_t states);

/* Slot-indexed forms.  The caches hold `num_slots` slots of
 * `heads_per_slot` heads each (slot-major: head index slot*heads_per_slot+h).
 * `slot_ids` is a device array of `count` int32 ids (any order, may repeat
 * only for read-only use); id -1 (PAD_SLOT_ID) is skipped; ids outside
 * [-1, num_slots) are skipped and set bit 0 (value 1) in *status (device
 * uint32, optional) and in the library's sticky error word.  `layout` is 0 for
 * capsule, 1 for provider.  The vLLM runtime range-checks its cache index on
 * the host (runtime.py:607-608); these kernels check on the device instead. */

/* state_cache -> (smoothing, codes, scales) caches at the listed slots. */
int32_t statecentric_gdn_state_codec_initialize_indexed_launch_v1(
    void* stream, uint32_t layout, const float* state_cache,
    float* smoothing_cache, int8_t* codes_cache, float* scales_cache,
    const int32_t* slot_ids, uint32_t count, uint32_t heads_per_slot,
    uint32_t num_slots, uint32_t* status);

/* (codes, smoothing, scales[, compensators]) caches -> state_cache at the
 * listed slots. */
int32_t statecentric_gdn_state_codec_dequantize_indexed_launch_v1(
    void* stream, uint32_t layout, const int8_t* codes_cache,
    const float* smoothing_cache, const float* scales_cache,
    const float* compensator_keys_cache, const float* compensator_values_cache,
    float* state_cache, const int32_t* slot_ids, uint32_t count,
    uint32_t heads_per_slot, uint32_t num_slots, uint32_t* status);

/* Encoded projection gathered by slot: queries_bf16 and outputs are compact
 * [count][heads_per_slot][128]; padded or invalid entries output zeros. */
int32_t statecentric_gdn_state_codec_encoded_projection_indexed_launch_v1(
    void* stream, uint32_t layout, const int8_t* codes_cache,
    const float* smoothing_cache, const float* scales_cache,
    const float* compensator_keys_cache, const float* compensator_values_cache,
    const uint16_t* queries_bf16, float* outputs, const int32_t* slot_ids,
    uint32_t count, uint32_t heads_per_slot, uint32_t num_slots,
    uint32_t* status);

/* ---- Full codec ------------------------------------------------------------ */

/* The reference's full encode (FromDenseBoundary's QuantizeBoundary,
 * capsule.cpp:129-225) of `states` heads: the rank-4 compensator fit (32 power
 * iterations per rank, deflation) bit-identical to the portable C++ codec,
 * then smoothing + int8 quantize of the residual.  `layout` 0: dense is
 * capsule [state][key][value]; 1: provider [state][value][key] (the fit runs
 * on the [key][value] matrix either way).  Outputs: residual_workspace (the
 * fp32 residual the int8 stage encodes, in the input's layout), smoothing
 * [state][128], quantized codes (input's layout), value_scales [state][128],
 * compensator_keys [state][128 keys][4] and compensator_values [state][128
 * values][4] fp32 -- the planes of the reference's serialized boundary.
 * Heads with non-finite input or singular value (which the reference rejects)
 * set bit 2 (value 4) of *status (optional) and of the sticky error word;
 * their outputs are unspecified. */
int32_t statecentric_gdn_state_codec_full_initialize_launch_v1(
    void* stream, uint32_t layout, const float* dense, float* residual_workspace,
    float* smoothing, int8_t* quantized, float* value_scales, float* compensator_keys,
    float* compensator_values, uint32_t states, uint32_t* status);

/* ---- Capsule wire format ---------------------------------------------------- */

/* Bytes of one serialized boundary capsule: 128 x 128 head, rank-4
 * compensators, window position 0 (120-byte header + 21,504-byte payload +
 * 64-character digest). */
#define STATECENTRIC_GDN_STATE_CODEC_CAPSULE_BYTES 21688u

/* The reference's Serialize (capsule.cpp:446-475) of `states` encoded heads,
 * byte for byte: capsule h is written at capsules + h * 21688 (8-byte
 * aligned).  Codes in `layout` 0 (capsule [key][value]) or 1 (provider
 * [value][key]); compensators [state][128][4] fp32, or both NULL for the
 * quant-only format (serialized as zeros).  The identity (64 lowercase hex
 * characters, HOST pointer; generation > 0; epoch > 0) is the same for every
 * capsule.  Runs on the stream; the SHA-256 digests are computed on the
 * device. */
int32_t statecentric_gdn_state_codec_capsule_serialize_launch_v1(
    void* stream, uint32_t layout, const int8_t* codes, const float* smoothing,
    const float* scales, const float* compensator_keys, const float* compensator_values,
    const char* model_geometry_sha256, uint64_t generation, uint64_t epoch,
    uint8_t* capsules, uint32_t states);

/* The reference's Restore (capsule.cpp:477-578) of `states` capsules under
 * the expected identity, default parameters and window position 0, fail-closed
 * per head: head_status[h] (device int32) = 0 when restored, else the first
 * failing check in the reference's order -- 1 magic, 2 checksum encoding,
 * 3 checksum, 4 parameters, 5 identity or geometry, 6 window position,
 * 7 a -128 code, 8 invalid boundary payload, 9 non-finite dense state.
 * Nothing is written for a rejected head. */
int32_t statecentric_gdn_state_codec_capsule_restore_launch_v1(
    void* stream, uint32_t layout, const uint8_t* capsules, const char* model_geometry_sha256,
    uint64_t generation, uint64_t epoch, int8_t* codes, float* smoothing, float* scales,
    float* compensator_keys, float* compensator_values, int32_t* head_status, uint32_t states);

/* Test support: SHA-256 (FIPS 180-4) of `size` HOST bytes as 64 lowercase hex
 * characters (not terminated), computed on the host by the same code the
 * capsule kernels run.  Synchronous. */
int32_t statecentric_gdn_state_codec_sha256_v1(const uint8_t* data, uint64_t size, char* hex64);

/* full_initialize_launch_v1 without a residual workspace, for callers that
 * cannot allocate device memory on the call path (a serving engine whose
 * memory is already handed to its cache pools, a host that owns every device
 * allocation; cudaMalloc would also synchronize the device).  No counterpart
 * in the reference.  The residual between the fit and the int8 stage lives in
 * a static device array of 64 heads (4 MiB) that every GPU loading the
 * library holds until exit; `states` above 64 is rejected with 1.  The first
 * call on a device looks up the array's device address (make it before any
 * stream capture on that device).  All calls on a device share its array,
 * which keeps the last call's contents: calls that can overlap on that GPU
 * (for example on different streams) race and must be serialized by the
 * caller.  Allocates nothing. */
int32_t statecentric_gdn_state_codec_full_initialize_static_launch_v1(
    void* stream, uint32_t layout, const float* dense, float* smoothing, int8_t* quantized,
    float* value_scales, float* compensator_keys, float* compensator_values, uint32_t states,
    uint32_t* status);

/* ---- Library status and benchmark support ------------------------------- */

/* Read (and with clear != 0 reset) the sticky per-device error word of the
 * current device, one bit per condition: bit 0 (value 1) = an invalid slot id
 * was seen, bit 1 (value 2) = a bounded device wait expired, bit 2 (value 4)
 * = non-finite data in a full-codec fit, bit 3 (value 8) = a decode step found
 * a head's window full, bit 4 (value 16) = a decode output or refit state was
 * non-finite.
 * Synchronous. */
int32_t statecentric_gdn_state_codec_device_error_v1(uint32_t* bits, int32_t clear);

/* Seeded synthetic inputs (benchmark and test support): `slots` slots of
 * `layers` x `heads_per_layer` heads starting at global slot `slot_base`.
 * States follow x ~ N(0,1) * 10^(-3u), u ~ U[0,1) per head, 1% zeros, in
 * `layout` order; queries are N(0,1), L2-normalised per head, bf16. */
int32_t statecentric_gdn_state_codec_synthesize_states_v1(
    void* stream, float* out, uint32_t layout, uint64_t seed,
    uint32_t slot_base, uint32_t slots, uint32_t layers,
    uint32_t heads_per_layer);
int32_t statecentric_gdn_state_codec_synthesize_queries_v1(
    void* stream, uint16_t* out, uint64_t seed, uint32_t slot_base,
    uint32_t slots, uint32_t layers, uint32_t heads_per_layer);

/* Test support: quotients[i] = numerators[i] / divisors[i] computed with the
 * quantizer's exact-division routine (RN(1/c) plus two fma corrections), for
 * comparison with IEEE division.  Valid where that routine's preconditions
 * hold (normal divisor and reciprocal, |numerator| >= 2^-102, normal
 * quotient). */
int32_t statecentric_gdn_state_codec_division_selftest_v1(
    void* stream, const float* numerators, const float* divisors, float* quotients,
    uint64_t count);

/* Test support for the failure path (no counterpart in the reference, which
 * has no bounded device waits): the batched capsule-layout quantize
 * (initialize_launch_v3) and encoded projection (encoded_projection_launch_v1,
 * quant-only format) launched with their mbarriers armed for the bytes of a
 * bulk copy that is never issued.  Every bounded wait therefore runs out after
 * `limit_ns` nanoseconds (0 < limit_ns <= 2e9); the kernels OR bit 1 (value 2,
 * "a bounded device wait expired") into *status (required) and into the sticky
 * error word, and return.  No copy is in flight when they exit, so the CUDA
 * context stays usable.  Outputs are unspecified. */
int32_t statecentric_gdn_state_codec_quantize_wait_selftest_v1(
    void* stream, const float* residual, float* smoothing, int8_t* quantized,
    float* value_scales, uint32_t states, uint64_t limit_ns, uint32_t* status);
int32_t statecentric_gdn_state_codec_encoded_projection_wait_selftest_v1(
    void* stream, const int8_t* residual, const float* smoothing,
    const float* scales, const uint16_t* queries_bf16, float* outputs,
    uint32_t states, uint64_t limit_ns, uint32_t* status);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* STATECENTRIC_GDN_STATE_CODEC_KERNEL_H_ */
