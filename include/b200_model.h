/*
 * b200_model.h -- C ABI of the native whole-model batch-1 decode driver
 * (Llama architecture, Q4_0 weights, fp16 KV cache, tensor parallel over the
 * GPUs of one node with NCCL).
 *
 * This is the B200 counterpart of running llama.cpp's decode graph with the
 * reference add-on's CANN backend: one token per call through
 * ggml_backend_sched -> graph_compute (patch:1884-1923) with the MUL_MAT,
 * FLASH_ATTN_EXT and neighbour ops of every layer.  Here the whole step is a
 * single captured CUDA graph of fused kernels: per layer RMSNorm+Q8_0+QKV
 * GEMV+RoPE+KV write, split-KV attention, O GEMV+residual, RMSNorm+gate/up
 * GEMV+SwiGLU, down GEMV+residual; then the lm_head GEMV with argmax.
 * Tensor parallelism shards Q/K/V/gate/up by output rows (whole KV heads),
 * O/down by input columns, and the lm_head by vocabulary rows; NCCL
 * all-reduces follow O and down, and an all-reduce(max) picks the argmax.
 */
#ifndef B200_MODEL_H
#define B200_MODEL_H

#include <stddef.h>
#include <stdint.h>

#include "b200_decode.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b200_model b200_model;

typedef struct {
    int n_layer;
    int d_model;
    int n_head;
    int n_head_kv;
    int head_dim;
    int d_ff;
    int vocab;
    int kv_size; /* KV cache rows (maximum context) */
    float rope_theta;
    float rms_eps;
} b200_llama_config;

/* Weight ids for b200_model_export_weight. */
#define B200_W_TOK_EMBD 0
#define B200_W_Q 1
#define B200_W_K 2
#define B200_W_V 3
#define B200_W_O 4
#define B200_W_GATE 5
#define B200_W_UP 6
#define B200_W_DOWN 7
#define B200_W_LM_HEAD 8

/* 128-byte NCCL unique id, made on one rank and shared with the others. */
int b200_nccl_unique_id(void *out128);

/* Creates the model on `device` (made current).  tp_world == 1 needs no id. */
int b200_model_create(const b200_llama_config *cfg, int device, int tp_rank, int tp_world, const void *nccl_id128,
                      b200_model **out);
void b200_model_destroy(b200_model *m);

/* Random-init weights: every Q4_0 matrix from N(0, sigma^2) samples quantised
 * with ggml's Q4_0 rule, norms = 1.  A rank generates exactly the rows or
 * columns of its shard of the unsharded tensors. */
int b200_model_init_synthetic(b200_model *m, uint64_t seed, float sigma);
/* KV cache rows [0, n_pos) of every layer ~ N(0, 1) in f16. */
int b200_model_fill_kv_synthetic(b200_model *m, uint64_t seed, int n_pos);

/* This rank's shard of a weight in ggml layout (Q4_0 blocks), regenerated on
 * the device and copied to host memory of `bytes` (query with host == NULL). */
int b200_model_export_weight(b200_model *m, int layer, int which, void *host, size_t *bytes);

/* This rank's KV cache rows [0, n_pos) of one layer (which: 0 = K, 1 = V) as
 * f16 [n_pos][n_head_kv_local * head_dim], copied to host memory. */
int b200_model_export_kv(b200_model *m, int layer, int which, int n_pos, void *host);

/* Captures one decode step into a CUDA graph (call once, after init). */
int b200_model_capture(b200_model *m);

/* Sets the device step state (async on the model stream): the next step
 * decodes `token` at `pos`; when advance != 0 each step feeds its argmax back
 * as the next token and increments pos. */
int b200_model_set_state(b200_model *m, int token, int pos, int advance);
/* One captured step, asynchronous on the model stream. */
int b200_model_launch(b200_model *m);
/* End to end: host token in, host next token out (and the local logits shard
 * when logits_host != NULL).  Copies in and out are inside the call. */
int b200_model_decode(b200_model *m, int token, int pos, int *next_token, float *logits_host);
/* Copies the logits of the last step: this rank's rows [offset, offset+count). */
int b200_model_logits(b200_model *m, float *host, int64_t *offset, int64_t *count);
b200_stream_t b200_model_stream(b200_model *m);
/* Layer dump (the decode-path analogue of the reference's LLAMA_LAYER_DUMP
 * eval callback, patch:825-892): one eager step at (token, pos) that copies
 * the residual stream after the embedding and after every layer into
 * x_host [(n_layer + 1) * d_model], and, when q_host / att_host are not NULL,
 * the roped q and the attention output of every layer
 * ([n_layer][n_head_local * head_dim] each).  Logits land as after a decode. */
int b200_model_debug_step(b200_model *m, int token, int pos, float *x_host, float *q_host, float *att_host);
/* Full layer dump of one eager step at (token, pos): every stage's output
 * and every quantised activation the step's GEMVs consume, so that a test
 * can check each stage against a CPU oracle fed the GPU's own stage input
 * (stage-level teacher forcing).  Any pointer may be NULL (not dumped).
 * Shapes are this rank's: hq = n_head / tp_world heads, hkv = n_head_kv /
 * tp_world, ff = d_ff / tp_world, qkv_rows = (hq + 2 hkv) head_dim.  Q8_0
 * activations are ggml block_q8_0 rows (k / 32 blocks of 34 bytes): for
 * QKV, gate/up and the lm_head the bytes the GEMV's own prologue quantised
 * (its first CTA's copy), for O and down the image the producing kernel
 * (attention, the SwiGLU epilogue) wrote and the GEMV copies.  dots_* are
 * the int32 dot of every (packed weight row, 32-block) from the same GEMV
 * launch (its export variant): QKV rows are q, then k, then v rows; gate/up
 * rows alternate gate i, up i. */
typedef struct {
    float *x;          /* [n_layer + 1][d_model] residual after the embedding and after every layer */
    float *x_mid;      /* [n_layer][d_model] residual after the O projection (summed over ranks) */
    float *q;          /* [n_layer][hq * head_dim] roped q */
    uint16_t *k_row;   /* [n_layer][hkv * head_dim] f16 K row written at pos */
    uint16_t *v_row;   /* [n_layer][hkv * head_dim] f16 V row written at pos */
    float *att;        /* [n_layer][hq * head_dim] attention output */
    float *h;          /* [n_layer][ff] SwiGLU output */
    float *logits;     /* [vocab / tp_world] */
    uint8_t *xq_qkv;   /* [n_layer][d_model / 32 * 34] */
    uint8_t *xq_o;     /* [n_layer][hq * head_dim / 32 * 34] */
    uint8_t *xq_gu;    /* [n_layer][d_model / 32 * 34] */
    uint8_t *xq_down;  /* [n_layer][ff / 32 * 34] */
    uint8_t *xq_head;  /* [d_model / 32 * 34] */
    int32_t *dots_qkv; /* [n_layer][qkv_rows][d_model / 32] */
    int32_t *dots_o;   /* [n_layer][d_model][hq * head_dim / 32] */
    int32_t *dots_gu;  /* [n_layer][2 ff][d_model / 32] */
    int32_t *dots_down;/* [n_layer][d_model][ff / 32] */
    int32_t *dots_head;/* [vocab / tp_world][d_model / 32] */
} b200_step_dump;
int b200_model_debug_step_ex(b200_model *m, int token, int pos, const b200_step_dump *dump);

/* Algorithmic HBM bytes one decode step reads on this rank at context ctx. */
int b200_model_step_bytes(b200_model *m, int ctx, uint64_t *bytes);
/* Runs `iters` eager (not captured) steps with CUDA events around every
 * kernel and returns the mean duration in microseconds per kernel class:
 * [0] embed, [1] QKV GEMV, [2] attention, [3] O GEMV, [4] gate/up GEMV,
 * [5] down GEMV, [6] lm_head GEMV, [7] all-reduces (0 at tp_world 1).
 * Leaves the step state where the last step put it. */
int b200_model_profile(b200_model *m, int iters, float *us_per_class8);

/* Where one captured step's time goes, measured inside the step: a second
 * CUDA graph of the step whose kernels record the device clock (globaltimer)
 * at their first CTA's return from the wait on the previous kernel and at
 * their last CTA's exit.  Kernel classes as in b200_model_profile:
 *   out[c]      time by which the step's end moved while class c ran
 *               (exit of a kernel minus the latest earlier exit), summed
 *               over the step; out[1..7] add up to out[16];
 *   out[8 + c]  mean span of one kernel of class c (exit minus the end of
 *               its wait), in microseconds;
 *   out[16]     the step, from the first QKV GEMV's start to the lm_head's
 *               end.
 * Runs one real decode step (the state advances as after b200_model_launch);
 * call between steps.  The embedding and bookkeeping kernels are not
 * stamped. */
int b200_model_timeline(b200_model *m, float *out17);

/* Phases inside the kernels of the last b200_model_timeline step, per kernel
 * class c (as above), means over the step's kernels of that class, in
 * microseconds from the class's return from the wait on the previous kernel
 * (w = the earliest CTA's return):
 *   out[8c + 0]  w minus the earliest CTA's entry (how early the kernel was
 *                resident under programmatic launch);
 *   out[8c + 1..3]  the LATEST CTA at: input ready (GEMV: activation in shared
 *                memory; attention: q loaded; all-reduce: every rank
 *                announced), first streamed chunk landed, main loop done;
 *   out[8c + 4]  the latest CTA's exit (the span of out17[8 + c]);
 *   out[8c + 5..7]  the EARLIEST CTA at the three marks.
 * A mark a class does not have reads 0.  B200_EINVAL before the first
 * b200_model_timeline call. */
int b200_model_timeline_phases(b200_model *m, float *out64);

/* The gate/up GEMV alone: one CUDA graph of the n_layer gate/up launches of
 * the step (each layer's own weights, chained as in the step), replayed
 * `iters` times between CUDA events on the model's stream; *us_per_launch is
 * the elapsed time over iters x n_layer launches.  Overwrites the SwiGLU
 * output and its image (scratch of the step); call between steps. */
int b200_model_time_gate_up(b200_model *m, int iters, float *us_per_launch);

#ifdef __cplusplus
}
#endif
#endif /* B200_MODEL_H */
