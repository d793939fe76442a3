/*
 * wohper_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference engine's (Twenytwo/wohper, crate
 * engine/zc_infer_core) dequant-matmul kernels, written in C++ with the same
 * AVX2 intrinsics in the same association order as the Rust code, so that its
 * outputs are bit-identical to what the Rust engine produces on an AVX2+FMA
 * host (libm calls -- expf, log1pf, log2f, exp2f -- resolve to glibc on both
 * sides).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load this library, and only as the checker or as the timed CPU
 * baseline.  The product library (wohper_b200/libwohper_b200.so) never links
 * or calls it.
 *
 * Parity is pinned by the reference's own known-answer tests, restated in
 * tests/golden/ (see tests/golden/make_kats.py) and checked by
 * tests/test_oracle_kats.py.
 */
#ifndef WOHPER_ORACLE_H
#define WOHPER_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: same numbering as wohper_b200.h (WH_*), which mirrors
 * DeepSeekV4KernelError (src/deepseek_v4.rs:398-408) in declaration order. */
enum {
  ORC_OK = 0,
  ORC_ERR_EMPTY_SHAPE = 1,
  ORC_ERR_INVALID_SHAPE = 2,
  ORC_ERR_PACKED_WEIGHT_TOO_SMALL = 3,
  ORC_ERR_SCALE_TOO_SMALL = 4,
  ORC_ERR_INPUT_TOO_SMALL = 5,
  ORC_ERR_OUTPUT_TOO_SMALL = 6,
  ORC_ERR_SCRATCH_TOO_SMALL = 7,
  ORC_ERR_NON_FINITE_OUTPUT = 8,
};

/* Mirrors Fp4Matvec (src/deepseek_v4.rs:410-417); lengths are in bytes. */
typedef struct {
  const uint8_t* packed_weight;
  size_t packed_len;
  const uint8_t* ue8m0_scales;
  size_t scales_len;
  size_t rows, cols, scale_cols;
} orc_fp4_spec;

/* Mirrors DeepSeekV4Fp4Expert (src/deepseek_v4.rs:419-428). */
typedef struct {
  orc_fp4_spec w1, w3, w2;
} orc_fp4_expert;

/* Thread count used by the row-parallel helpers; 0 = reference default
 * (ZC_COMPUTE_THREADS or nproc-2, min 1; src/deepseek_v4.rs:206-221). */
void orc_set_threads(int threads);
int orc_get_threads(void);

/* a1: decoders and LUTs (src/deepseek_v4.rs:151-204, 358-372). */
float orc_decode_fp8_e4m3(uint8_t byte, float scale);
float orc_decode_ue8m0_scale(uint8_t byte);
float orc_decode_fp4_e2m1(uint8_t nibble, float scale);
void orc_fp8_e4m3_base_lut(float out[256]);
void orc_ue8m0_scale_lut(float out[256]);
void orc_fp4_e2m1_base_lut(float out[16]);
void orc_fp8_e4m3_sorted_lut(float out[256]);

/* a2: one FP8 row dot (AVX2 path src/compute.rs:5977-6018 when avx2!=0,
 * scalar path src/compute.rs:5936-5960 otherwise). */
float orc_fp8_dot_row(const uint8_t* weight_row, const uint8_t* scale_row, size_t scale_cols,
                      size_t col_group, const float* input, int avx2);

/* a3/a4: FP8 E4M3 + UE8M0 GEMV over rows [row_start,row_end)
 * (src/compute.rs:6174-6321).  output[r-row_start] for each row. */
int orc_fp8_gemv_rows(const uint8_t* weight, size_t weight_len, size_t rows, size_t cols,
                      const uint8_t* scale, size_t scale_len, size_t scale_rows, size_t scale_cols,
                      size_t row_start, size_t row_end, const float* input, size_t input_len,
                      float* output, size_t output_len);

/* a5: batched FP8 GEMV (src/compute.rs:6384-6577); inputs is count x ldx,
 * outputs is count x ldy (outputs[i*ldy + r-row_start]). */
int orc_fp8_gemv_rows_multi(const uint8_t* weight, size_t weight_len, size_t rows, size_t cols,
                            const uint8_t* scale, size_t scale_len, size_t scale_rows,
                            size_t scale_cols, size_t row_start, size_t row_end,
                            const float* inputs, size_t count, size_t ldx, float* outputs,
                            size_t ldy);

/* a7: act quant-dequant in place (src/compute.rs:2504-2545). */
void orc_fp8_act_quant_dequant_in_place(float* values, size_t n, size_t block_size);

/* BF16 dot / GEMV (src/compute.rs:6115-6172, 2910-2944). avx2 selects the path. */
float orc_bf16_dot_row(const uint16_t* row, const float* input, size_t n, int avx2);
int orc_bf16_gemv(const uint16_t* weight, size_t rows, size_t cols, const float* input,
                  float* output);

/* a9/a10: FP4 matvec (src/deepseek_v4.rs:434-549).  path: 0 = reference
 * dispatch (AVX2 when shapes allow), 1 = force group-hoisted scalar,
 * 2 = force per-element. */
int orc_fp4_matvec(const orc_fp4_spec* spec, const float* input, size_t input_len,
                   float* output, size_t output_len, int path);

/* a11: FP4 expert forward (src/deepseek_v4.rs:561-601). */
int orc_fp4_expert_forward(const orc_fp4_expert* expert, const float* input, size_t input_len,
                           float* output, size_t output_len, float* scratch, size_t scratch_len);
size_t orc_fp4_expert_scratch_len(size_t intermediate);

/* FP8 shared expert (src/compute.rs:5545-5614): w1/w3/w2 FP8 with
 * 128x128-block UE8M0 scales. */
typedef struct {
  const uint8_t* weight;
  const uint8_t* scale;
  size_t rows, cols, scale_rows, scale_cols;
} orc_fp8_matrix;
typedef struct {
  orc_fp8_matrix w1, w3, w2;
} orc_fp8_expert;
int orc_fp8_expert_forward(const orc_fp8_expert* expert, const float* input, size_t hidden,
                           float* output);

/* a15: router.  mode 0 = RawLogits (legacy: top-k by raw logit, then softmax
 * over the selected, src/server/generation.rs:3152-3180), mode 1 = DeepSeek
 * sqrt-softplus + selection bias + route_scale (src/compute.rs:2129-2268).
 * hash_ids (nullable, topk entries) replaces score top-k by a tid2eid row.
 * Writes topk ids and the final per-route weights (after the mode's
 * normalisation; before the combine's w/sum). logits_out (nullable, E). */
int orc_router(const uint16_t* gate_bf16, size_t experts, size_t hidden, const float* x,
               size_t topk, int mode, const float* bias, float route_scale,
               const int32_t* hash_ids, int32_t* ids_out, float* weights_out, float* logits_out);

/* deepseek_sqrtsoftplus_route (src/deepseek_v4.rs:618-652), the crate's
 * standalone helper (its own softplus and partial_cmp sort). */
size_t orc_deepseek_sqrtsoftplus_route(const float* logits, size_t n, const float* bias,
                                       size_t topk, float route_scale, int32_t* ids_out,
                                       float* weights_out);

/* a12/a13: one-token MoE FFN: routed experts combined with w_i/sum(w)
 * (src/compute.rs:1948-2030), plus the shared expert (src/compute.rs:1872-1946).
 * shared_fp4 / shared_fp8: at most one non-null. */
int orc_moe_combine_token(const orc_fp4_expert* experts, const int32_t* ids, const float* weights,
                          size_t topk, const orc_fp4_expert* shared_fp4,
                          const orc_fp8_expert* shared_fp8, const float* x, size_t hidden,
                          float* y);

/* a14: expert-major batched MoE (src/compute.rs:1779-1810 +
 * src/server/generation.rs:2487-2606), union in ascending expert id. */
int orc_moe_batched(const orc_fp4_expert* experts, size_t num_experts, const int32_t* ids,
                    const float* weights, size_t tokens, size_t topk,
                    const orc_fp4_expert* shared_fp4, const float* x, size_t hidden, float* y);

#ifdef __cplusplus
}
#endif
#endif
