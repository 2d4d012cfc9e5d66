/*
 * gdn_state_codec_windowed_gdn_kernel.h -- the p = 16 windowed decode path.
 *
 * Entry points of the reference's window libraries
 * (native/include/statecentric/gdn_state_codec_windowed_gdn_kernel.h), with
 * their names and arguments, implemented for CUDA.  The vLLM plugin binds
 * them at load (src/gdn_state_codec/runtime.py:71-125) and calls the bf16
 * step per decode token and the boundary refit every 16 tokens
 * (runtime.py:627-845).
 *
 * One state is one GDN head with d_k = d_v = 128.  Per head the window is:
 *   residual [128][128] int8, smoothing [128] fp32, scales [128] fp32 (the
 *   INT8 boundary); compensator_keys / compensator_values [128][4] binary16;
 *   record_decay [16] fp32, record_keys [16][128] binary16, record_corrections
 *   [16][128] binary16 (the buffered rank-one updates); positions [8] uint32
 *   with the window position (0..16) in element 0.
 *
 * Semantics: each step is the portable library's ApplyToken
 * (native/src/gdn_state_codec_state_capsule.cpp:354-397) with a scalar decay
 * per head, reading the window in ReadWindowState's order (:256-304), every
 * sum sequential and every product rounded before its add; the record it
 * appends is stored in binary16 (round to nearest even).  The refit is
 * DenseState (:337-352) followed by QuantizeBoundary (:130-225) with
 * `power_iterations` sweeps per rank (the library fixes 32; 0 gives the
 * quant-only boundary with zero compensators), compensators stored in
 * binary16.  Outputs are therefore bit-identical to that arithmetic, which
 * the CPU oracle restates.
 *
 * Layouts: the bf16 steps and the refit read the boundary codes as
 * [value][key] (the plugin's provider layout, as the reference's bf16 step
 * and boundary kernels index them); windowed_gdn_step_launch_v1 reads them as
 * [key][value] (as the reference's generic step kernel does).
 *
 * Common rules: stream is a cudaStream_t (NULL: default stream); every
 * pointer is a device pointer owned by the caller; launches are
 * asynchronous; nothing is allocated.  Return 0 enqueued, 1 bad arguments
 * (a null required pointer, states == 0, a window or boundary buffer not
 * 16-byte aligned, a token vector not naturally aligned), 2 launch failed,
 * 3 device set-up failed.  `states` may be any value >= 1 (the Ascend launchers capped it at
 * 16384).  A step on a head whose window is already full (position 16)
 * leaves that head untouched and sets bit 3 (value 8) of the sticky device
 * error word (statecentric_gdn_state_codec_device_error_v1); a non-finite
 * decode output or refit state sets bit 4 (value 16).
 */
#ifndef STATECENTRIC_GDN_STATE_CODEC_WINDOWED_GDN_KERNEL_H_
#define STATECENTRIC_GDN_STATE_CODEC_WINDOWED_GDN_KERNEL_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Generic step (reference header :8-16): decay [states] fp32, write_keys /
 * reads / queries / values [states][128] binary16, outputs [states][128]
 * fp32; codes [key][value]; compensators required. */
int32_t statecentric_gdn_state_codec_windowed_gdn_step_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing,
    const float* scales, const uint16_t* compensator_keys,
    const uint16_t* compensator_values, float* record_decay,
    uint16_t* record_keys, uint16_t* record_corrections, uint32_t* positions,
    const float* decay, const uint16_t* write_keys, const uint16_t* reads,
    const uint16_t* queries, const uint16_t* values, float* outputs,
    uint32_t states);

/* Qwen3.5 decode step (reference header :18-28): decay is the log decay
 * [states] fp32 (the step uses exp of it), beta [states] bf16, keys / queries
 * [states/2][128] bf16 (value heads 2j and 2j+1 share query/key head j),
 * values [states][128] bf16, outputs [states][128] bf16.  key = beta k,
 * read = exp(decay) k, query = 128^-0.5 q.  states must be even; codes
 * [value][key]; compensators required.  Key, query and value rows that are
 * 16-byte aligned and a 4-byte aligned beta take the kernel that stages each
 * head's inputs one head ahead; other alignments (2 bytes suffice) take a
 * kernel that loads them directly, with identical results. */
int32_t statecentric_gdn_state_codec_windowed_gdn_step_bf16_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing,
    const float* scales, const uint16_t* compensator_keys,
    const uint16_t* compensator_values, float* record_decay,
    uint16_t* record_keys, uint16_t* record_corrections, uint32_t* positions,
    const float* decay, const uint16_t* beta, const uint16_t* keys,
    const uint16_t* queries, const uint16_t* values, uint16_t* outputs,
    uint32_t states);

/* The same step for quant-only boundaries (reference header :30-40): the
 * compensators are not read (they may be NULL). */
int32_t statecentric_gdn_state_codec_windowed_gdn_step_bf16_quant_only_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing,
    const float* scales, const uint16_t* compensator_keys,
    const uint16_t* compensator_values, float* record_decay,
    uint16_t* record_keys, uint16_t* record_corrections, uint32_t* positions,
    const float* decay, const uint16_t* beta, const uint16_t* keys,
    const uint16_t* queries, const uint16_t* values, uint16_t* outputs,
    uint32_t states);

/* Dense fp32 GDN step (reference header :42-46), in place on [states][128]
 * [128] fp32 states in [key][value] order: correction = value - S^T read;
 * S = decay S + key (x) correction; output = S^T query.  key / read / query /
 * value binary16, decay fp32 [states], outputs fp32.  dense_state must be
 * 16-byte aligned (each head is staged by one bulk copy); returns 1 otherwise. */
int32_t statecentric_gdn_state_codec_fp32_gdn_step_launch_v1(
    void* stream, float* dense_state, const float* decay, const uint16_t* key,
    const uint16_t* read, const uint16_t* query, const uint16_t* value,
    float* output, uint32_t states);

/* Test support for the failure path (no counterpart in the reference, which
 * has no bounded device waits): fp32_gdn_step_launch_v1 launched with every
 * block's first landing barrier armed for a copy that is never issued.  Each
 * block's bounded wait runs out after `limit_ns` nanoseconds (0 < limit_ns <=
 * 2e9), bit 1 (value 2) of the sticky error word is set, and the blocks return
 * before writing any state or output.  No copy is in flight, so the CUDA
 * context stays usable. */
int32_t statecentric_gdn_state_codec_fp32_gdn_step_wait_selftest_v1(
    void* stream, float* dense_state, const float* decay, const uint16_t* key,
    const uint16_t* read, const uint16_t* query, const uint16_t* value,
    float* output, uint32_t states, uint64_t limit_ns);

/* Boundary refit (reference header :48-60): folds each head's window (its
 * `position` records, normally 16) into a new INT8 boundary plus binary16
 * compensators in the next_* buffers, then clears the records (decay, keys
 * and corrections zero) and sets the position to 0.  Codes [value][key],
 * residual_workspace [states][128][128] fp32, power_iterations <= 32.  Input and output boundary buffers must
 * not alias.  Compensators of the current boundary may be NULL (quant-only
 * boundary). */
int32_t statecentric_gdn_state_codec_window_boundary_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing,
    const float* scales, const uint16_t* compensator_keys,
    const uint16_t* compensator_values, float* record_decay,
    uint16_t* record_keys, uint16_t* record_corrections, uint32_t* positions,
    int8_t* next_residual, float* next_smoothing, float* next_scales,
    uint16_t* next_compensator_keys, uint16_t* next_compensator_values,
    float* residual_workspace, uint32_t states, uint32_t power_iterations);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* STATECENTRIC_GDN_STATE_CODEC_WINDOWED_GDN_KERNEL_H_ */
