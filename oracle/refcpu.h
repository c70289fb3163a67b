/*
 * refcpu.h -- CPU restatement of the M=1 decode hot path (TEST INFRASTRUCTURE).
 *
 * This library is the parity oracle and the timed CPU baseline.  It is never
 * linked into, loaded by or called from the product library
 * (libb200_decode.so); only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline / reference arm may load it.
 *
 * What it restates, and from where:
 *   - ggml block formats Q4_0 / Q8_0 and their reference quantisers
 *     (ggml-quants.c quantize_row_q{4,8}_0_ref at llama.cpp 37b3a9e0; pinned
 *     in this repository against gguf-py 0.19.0 gguf/quants.py:220-252 and
 *     378-401 by tests/golden/make_golden.py fixtures).
 *   - ggml-cpu MUL_MAT semantics at M=1 (src1 converted to the weight's
 *     vec_dot_type: F16 for F16 weights, Q8_0 for Q4_0/Q8_0 weights; integer
 *     per-block dots; fp32 result).  ggml-cpu itself is not in this container,
 *     so the dot-product accumulation order is NOT pinned; the integer parts
 *     (Q8_0 activation bytes/scales, per-block int32 dots) are exact.
 *   - FLASH_ATTN_EXT decode with additive f16 mask, scale before mask
 *     (reference attention_step_custom.cpp:160-184), online softmax rescale
 *     (attention_step_custom.cpp:220-223, 269), kv_len truncation
 *     (attention_step_custom.cpp:110-113), q cast to f16 before the dot
 *     (patch P:1403).
 *   - The reference add-on's own A8W8 variant: per-token activation int8
 *     quantiser (w8a8_quantize_custom_vector.cpp:35-64), per-output-column
 *     weight transform into int8 NZ 16x32 order (patch P:1674-1695), int32
 *     matmul (matmul_w8a8_i32_custom.cpp:15-48) and dequant.
 *   - The reference's W4A16 probe packing and its f16 sequential golden
 *     (experiments/w4a16-gemv/source/gen_data.py:17-39).
 *   - Llama-architecture decode step (RMSNorm, RoPE NORM mode, SwiGLU,
 *     residual, GET_ROWS, argmax) used for whole-model teacher-forced logits.
 */
#ifndef REFCPU_H
#define REFCPU_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define REF_QK 32

typedef struct { uint16_t d; uint8_t qs[16]; } ref_block_q4_0; /* 18 bytes */
typedef struct { uint16_t d; int8_t  qs[32]; } ref_block_q8_0; /* 34 bytes */

/* ---- fp16 ---- */
float    ref_f16_to_f32(uint16_t h);
uint16_t ref_f32_to_f16(float f);                 /* round to nearest even */
void     ref_f32_to_f16_row(const float *x, uint16_t *y, int64_t n);
void     ref_f16_to_f32_row(const uint16_t *x, float *y, int64_t n);

/* ---- ggml block quantisers ---- */
void ref_quantize_q8_0(const float *x, ref_block_q8_0 *y, int64_t k);
void ref_quantize_q4_0(const float *x, ref_block_q4_0 *y, int64_t k);
void ref_dequantize_q8_0(const ref_block_q8_0 *x, float *y, int64_t k);
void ref_dequantize_q4_0(const ref_block_q4_0 *x, float *y, int64_t k);

int32_t ref_dot_block_q4_0_q8_0(const ref_block_q4_0 *w, const ref_block_q8_0 *x);
int32_t ref_dot_block_q8_0_q8_0(const ref_block_q8_0 *w, const ref_block_q8_0 *x);

/* 0: fp64 block-sum accumulator (default); 1: fp32 sequential. */
void ref_set_accum_mode(int mode);

/* ---- MUL_MAT, M = 1: W rows n contiguous along K; y[n] = sum_k W[n,k] x[k] ---- */
void ref_mul_mat_f16(const uint16_t *w, const float *x, float *y, int64_t n, int64_t k, int nthreads);
/* mode 0: ggml-cpu semantics (x -> Q8_0, integer block dots)
 * mode 1: true W4A16 (x -> f16, dequantised weights, fp accumulation) */
void ref_mul_mat_q4_0(const void *w, const float *x, float *y, int64_t n, int64_t k, int mode, int nthreads);
void ref_mul_mat_q4_0_xq(const void *w, const void *xq, float *y, int64_t n, int64_t k, int nthreads);
void ref_block_dots_q4_0_xq(const void *w, const void *xq, int32_t *dots, int64_t n, int64_t k);
void ref_mul_mat_q8_0(const void *w, const float *x, float *y, int64_t n, int64_t k, int nthreads);
/* per-(row, block) int32 dots for exactness checks; dots is [n][k/32] */
void ref_block_dots_q4_0(const void *w, const float *x, int32_t *dots, int64_t n, int64_t k);
void ref_block_dots_q8_0(const void *w, const float *x, int32_t *dots, int64_t n, int64_t k);

/* ---- FLASH_ATTN_EXT, one query token ----
 * q   f32 [Hq][D] (ggml q [D,1,Hq,1]); out f32 [Hq][D]
 * k,v f16, element (t, h, d) at k[t*k_row + h*k_head + d] (strides in elements)
 * mask f16 [n_kv] or NULL; kv_len int32 [1] or NULL (used when 0 < kv_len < n_kv)
 * mode 0: fp64 two-pass truth; mode 1: ggml-cpu online softmax with the V
 * accumulator rounded to f16 after every update; mode 2: the reference
 * AttentionStepCustom (fp32 online softmax over 240-row tiles, output rounded
 * to f16 with round-to-nearest-even). */
void ref_flash_attn_ext_decode(const float *q, const uint16_t *k, const uint16_t *v,
                               const uint16_t *mask, const int32_t *kv_len, float *out,
                               int D, int Hq, int Hkv, int n_kv,
                               int64_t k_row, int64_t k_head, int64_t v_row, int64_t v_head,
                               float scale, int mode);
/* llama-graph.cpp set_input_kv_lengths_impl (patch P:2900-2916): 1 + index of
 * the last finite mask entry, at least 1.  mask f16 [n_rows][n_kv]. */
void ref_kv_lengths_from_mask_f16(const uint16_t *mask, int64_t n_kv, int64_t n_rows, int32_t *out);

/* ---- reference add-on A8W8 (per-token x, per-column w) ---- */
void ref_a8w8_quantize_token(const uint16_t *x_f16, int8_t *xq, uint16_t *scale_f16, int64_t k);
void ref_a8w8_transform_weight(const uint16_t *w_f16, int8_t *q_nz, uint16_t *scales, int64_t k, int64_t n);
void ref_a8w8_matmul_i32(const int8_t *xq, const int8_t *w_nz, int32_t *acc, int64_t k, int64_t n);
void ref_a8w8_dequant(const int32_t *acc, uint16_t x_scale, const uint16_t *w_scales, uint16_t *out, int64_t n);

/* ---- reference W4A16 probe (own packing, tile 448, group 32) ---- */
void ref_w4a16_probe(const uint16_t *x_f16, const uint8_t *packed, const uint16_t *scale_layout,
                     uint16_t *y_f16, int64_t k, int64_t n, int64_t tile);

/* ---- deterministic synthetic data (counter-based; same stream as the device generator) ---- */
float ref_synth_normal(uint64_t seed, uint64_t index);   /* N(0,1) */
/* Q4_0 rows of N(0, sigma^2): rows [row0, row0+nrows) of a matrix with k columns */
void  ref_synth_q4_0(uint64_t seed, float sigma, int64_t row0, int64_t nrows, int64_t k, ref_block_q4_0 *out, int nthreads);
void  ref_synth_rows_f16(uint64_t seed, uint64_t base, int64_t nrows, int64_t rl, int64_t rg, int64_t col0,
                         uint16_t *out, int nthreads);

/* ---- Llama-architecture decode ---- */
typedef struct {
    int n_layer, d_model, n_head, n_kv_head, head_dim, d_ff, vocab, kv_size;
    float rope_theta, eps;
} ref_llama_cfg;

typedef struct {
    ref_llama_cfg cfg;
    const ref_block_q4_0 *tok_embd;          /* [vocab][d_model] */
    const ref_block_q4_0 *const *wq, *const *wk, *const *wv, *const *wo;   /* per layer */
    const ref_block_q4_0 *const *wgate, *const *wup, *const *wdown;
    const float *const *attn_norm, *const *ffn_norm;                        /* per layer [d_model] */
    const float *out_norm;                                                  /* [d_model] */
    const ref_block_q4_0 *lm_head;           /* [vocab][d_model] */
    uint16_t *const *k_cache, *const *v_cache; /* per layer [kv_size][n_kv_head*head_dim] f16 */
} ref_llama;

/* One decode step at position pos for layers [l0, l1); when do_head, the final
 * norm + lm_head run and logits (f32 [vocab]) are written.  x is the f32
 * residual stream [d_model]; when l0 == 0 it is initialised from the token's
 * embedding row.  Returns argmax (when do_head) or -1. */
int64_t ref_llama_step(const ref_llama *m, int32_t token, int32_t pos, float *x, float *logits,
                       int l0, int l1, int do_head, int nthreads);

void ref_rms_norm_mul(const float *x, const float *w, float *y, int64_t n, float eps);
void ref_rope_norm(float *x, int n_heads, int head_dim, int pos, float theta_base);
int64_t ref_argmax(const float *x, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
