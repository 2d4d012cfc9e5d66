/*
 * gdn_state_codec_windowed_gdn_kernel.h -- loader-compatibility entry points.
 *
 * The vLLM plugin (src/gdn_state_codec/runtime.py:71-115) binds two symbols
 * unconditionally when it loads the window libraries.  The p=16 windowed
 * decode step and the window-boundary refit are outside the quant-only hot
 * path this backend implements, so these are present only so the plugin's
 * loader succeeds; both return 5 ("not implemented by this backend") and
 * enqueue nothing.  The encoded readout that the decode step consumes is
 * statecentric_gdn_state_codec_encoded_projection_launch_v1
 * (gdn_state_codec_kernel.h).
 */
#ifndef STATECENTRIC_GDN_STATE_CODEC_WINDOWED_GDN_KERNEL_H_
#define STATECENTRIC_GDN_STATE_CODEC_WINDOWED_GDN_KERNEL_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Signature of gdn_state_codec_windowed_gdn_kernel.h:8-16 (reference). */
int32_t statecentric_gdn_state_codec_windowed_gdn_step_launch_v1(
    void* stream, const int8_t* residual, const float* smoothing,
    const float* scales, const uint16_t* compensator_keys,
    const uint16_t* compensator_values, float* record_decay,
    uint16_t* record_keys, uint16_t* record_corrections, uint32_t* positions,
    const float* decay, const uint16_t* write_keys, const uint16_t* reads,
    const uint16_t* queries, const uint16_t* values, float* outputs,
    uint32_t states);

/* Signature of gdn_state_codec_windowed_gdn_kernel.h:50-60 (reference). */
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
