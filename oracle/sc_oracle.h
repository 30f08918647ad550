/*
 * sc_oracle.h -- CPU restatement of mosure/bevy_synth's sparse submanifold
 * convolution path (crate burn_flex_gmm + the decoder block math of
 * burn_trellis), used ONLY as test infrastructure: the parity checker for the
 * CUDA library and the timed CPU baseline of bench.py.  Nothing in the
 * product path links or calls this library.
 *
 * Parity status: the reference is Rust and cannot be built in this
 * environment (no cargo/rustc), so no reference-produced output vectors
 * exist.  The restatement is pinned to the reference's own known-answer
 * tests (burn_trellis/src/runtime_model/sparse_decoder_tests.rs:189-292) and
 * to its flex==legacy property tests driven by the reference LCG
 * (burn_flex_gmm/src/lib.rs:764-972); see tests/test_oracle.py.
 *
 * Conventions follow the reference exactly:
 *   coords   [N,4] u32  (batch, x, y, z)
 *   weight   [Cout, KD, KH, KW, Cin/groups] f32 (PyTorch channels-last)
 *   packed   [groups][K*Cin/g][Cout/g] f32           (pack_flex_weight)
 *   neighbor [N,K] i32, -1 = invalid
 */
#ifndef SC_ORACLE_H
#define SC_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct oc_conv_config {
    int64_t in_channels, out_channels;
    int64_t kernel_d, kernel_h, kernel_w;
    int64_t in_channels_per_group, out_channels_per_group, groups;
    int32_t axis_order[3];
    int32_t axis_sign[3];
} oc_conv_config;

/* Duplicate-coordinate rule.  The CPU reference inserts into a HashMap, so
 * the LAST row with a coordinate wins (lib.rs:83-86); every device builder
 * keeps the LOWEST row (neighbor_kernels.rs:37-39, 249-256). */
enum { OC_DUP_LAST = 0, OC_DUP_LOWEST = 1 };

/* Returns 0 on success, negative on error; message via oc_last_error. */
const char* oc_last_error(void);

int oc_validate_config(const oc_conv_config* cfg);
int oc_kernel_rows(const oc_conv_config* cfg, int64_t* rows);
int oc_kernel_offsets(const oc_conv_config* cfg, int32_t* offsets /* [K*3] */);

int oc_build_neighbor_rows(const oc_conv_config* cfg, const uint32_t* coords, int64_t n_rows,
                           int dup_rule, int32_t* out /* [N*K] */);
/* Query coordinates q_coords against the table built from in_coords
 * (build == query when both are the same array). */
int oc_build_neighbor_rows_query(const oc_conv_config* cfg, const uint32_t* in_coords,
                                 int64_t n_in, const uint32_t* q_coords, int64_t n_q,
                                 int dup_rule, int32_t* out /* [n_q*K] */);

int oc_pack_flex_weight(const oc_conv_config* cfg, const float* weight, float* packed);

int oc_subm_conv_flex_precomputed(const oc_conv_config* cfg, const float* weight,
                                  const float* bias, const float* input, int64_t input_rows,
                                  const int32_t* neighbor_rows, int64_t rows,
                                  const float* packed /* nullable */, int n_threads,
                                  float* out /* [rows*Cout] */);

int oc_subm_conv_legacy(const oc_conv_config* cfg, const float* weight, const float* bias,
                        const uint32_t* coords, int64_t n_rows, const float* input,
                        float* out);

int oc_layer_norm_inplace(float* data, int64_t rows, int64_t channels, const float* gamma,
                          const float* beta, float eps);
void oc_silu_inplace(float* data, int64_t n);
void oc_bf16_round_inplace(float* data, int64_t n);
void oc_f16_round_inplace(float* data, int64_t n);

int oc_channel2spatial(const uint32_t* coords, int64_t rows, const float* feats,
                       int64_t in_channels, const uint8_t* mask /* [rows*8] */,
                       uint32_t* out_coords, float* out_feats, int64_t* out_rows);
int oc_repeat_interleave_channels(const float* feats, int64_t rows, int64_t in_channels,
                                  int64_t repeat, float* out);

#ifdef __cplusplus
}
#endif
#endif
