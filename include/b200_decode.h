/*
 * b200_decode.h -- C ABI of the B200 (sm_100a) single-token decode hot path.
 *
 * Plain C: device pointers, element counts, byte strides, a CUDA stream, and
 * an int status (0 = ok, negative = B200_E*).  No ggml or torch types.  Every
 * kernel entry point is asynchronous on the given stream; "device pointer"
 * means memory of the device that is current on the calling thread.
 *
 * Each entry point names the reference interface it replaces.  References
 * use the path inside the reference project; "patch:N" is line N of
 * patches/ascend310b4-llama-cpp.patch, a diff against llama.cpp 37b3a9e0.
 */
#ifndef B200_DECODE_H
#define B200_DECODE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; NULL means the legacy default stream. */
typedef struct CUstream_st *b200_stream_t;

/* Status codes. */
#define B200_OK 0
#define B200_EINVAL (-1)       /* bad pointer, shape or stride */
#define B200_ECUDA (-2)        /* a CUDA runtime call failed */
#define B200_EUNSUPPORTED (-3) /* valid ggml op variant that this backend does not implement */
#define B200_ENOMEM (-4)
#define B200_ENCCL (-5)
#define B200_ESTATE (-6)       /* call out of order (not initialised, wrong phase) */

/* Bits of the device status word (b200_device_status). */
#define B200_DEVSTATUS_TIMEOUT 1u /* a bounded device-side wait expired */
#define B200_DEVSTATUS_BOUNDS 2u  /* a device-side range check failed; the access was skipped */

/* Weight type ids: the values of ggml's enum ggml_type. */
#define B200_TYPE_F32 0
#define B200_TYPE_F16 1
#define B200_TYPE_Q4_0 2
#define B200_TYPE_Q8_0 8
/* This library's int8 layout for the reference's A8W8 scheme (per-row weight
 * scale, per-token activation scale); not a ggml type id. */
#define B200_TYPE_A8W8 100

/* Q4_0 GEMV arithmetic. */
#define B200_Q4_MODE_GGML 0  /* ggml-cpu semantics: x -> Q8_0 blocks, integer block dots */
#define B200_Q4_MODE_W4A16 1 /* x -> f16, fp32 multiply-accumulate of dequantised weights */

const char *b200_version(void);
const char *b200_strerror(int code);

/* Reads (and optionally clears) the status word of the current device.
 * Synchronises the device.  Once a bounded wait has expired (TIMEOUT set),
 * every later wait that depends on another CTA, kernel or rank gives up at
 * once, so a dead peer costs one limit, not one per collective; clearing the
 * word re-arms them. */
int b200_device_status(unsigned int *status, int reset);

/* Limit of every bounded device-side wait on the current device, in
 * nanoseconds (0 restores the default, 2 s).  Synchronous; call between
 * steps (it changes kernels launched after it). */
int b200_set_wait_timeout(uint64_t ns);

/* ------------------------------------------------------------------------
 * One-shot all-reduce (sum) of n floats over peer-mapped memory: the
 * collective after the row-split O and down projections of tensor
 * parallelism.  The reference has no multi-device code; this replaces the
 * ncclAllReduce(sum) a tensor-parallel llama.cpp backend issues there.  On
 * every rank of `world`:
 *   parts[r]      rank r's partial [n] (device pointers; peers' through
 *                 CUDA IPC or another peer mapping), 16-byte aligned;
 *   flags         this rank's flag array [world] (device; zero at start);
 *   peer_flags[r] &flags_of_rank_r[rank];
 *   seq           collective number, > every earlier one on these flags.
 * The kernel stores seq into every peer_flags[r] (release, system scope),
 * waits until flags[r] >= seq for every r (bounded; B200_DEVSTATUS_TIMEOUT
 * when a rank never arrives) and writes x = sum of parts in rank order 0,
 * 1, ... (bit-identical on every rank).  A rank may overwrite its partial
 * for collective seq + 2 only; alternate two partial buffers. */
int b200_tp_allreduce_f32(float *x, const float *const *parts, int world, int rank, int64_t n,
                          unsigned long long *flags, unsigned long long *const *peer_flags, uint64_t seq,
                          b200_stream_t stream);

/* ------------------------------------------------------------------------
 * Weight pre-layout.  Replaces the FRACTAL_NZ dual layout of the reference
 * (ggml_cann_310b_nz_offset/size patch:1551-1562, set_tensor NZ branch
 * patch:1768-1806, get_alloc_size patch:1810-1846, aclnnTransMatmulWeight).
 *
 * Packed rows are contiguous (row r at r * row_stride).  Inside a row, with
 * U = K/32 blocks (Q4_0, Q8_0) or U = K/8 units of 8 halves (F16):
 *   F16 : K halves, identical to the ggml row           row_stride = 2K
 *   Q4_0: nibbles qs[U][16], then scales d[U] (f16)      row_stride = 16U + pad16(2U)
 *   Q8_0: quant bytes 0..15 [U][16], bytes 16..31
 *         [U][16], then d[U] (f16)                       row_stride = 32U + pad16(2U)
 * Scale planes are zero-padded to 16 bytes.  Each plane of a row chunk is one
 * 16-byte-aligned bulk copy, and 32 lanes reading 32 consecutive blocks issue
 * conflict-free 16-byte shared-memory loads.
 * ---------------------------------------------------------------------- */
int64_t b200_packed_row_stride(int type, int64_t n, int64_t k); /* 0 when unsupported */
size_t b200_packed_size(int type, int64_t n, int64_t k);        /* 0 when unsupported */
/* src: ggml rows (n rows of k elements, row stride = ggml_row_size) on the device. */
int b200_repack(int type, const void *src, void *dst, int64_t n, int64_t k, b200_stream_t stream);
/* Packs 2*n_each rows: packed row 2i is src_even row i, 2i+1 is src_odd row i
 * (gate/up pairs for the fused SwiGLU GEMV). */
int b200_repack_interleave2(int type, const void *src_even, const void *src_odd, void *dst, int64_t n_each,
                            int64_t k, b200_stream_t stream);

/* ------------------------------------------------------------------------
 * MUL_MAT at M = 1 (ggml mul_mat(W[K,N], x[K,1]) -> y f32 [N]).
 * Replaces ggml_cann_mat_mul_fp (patch:1188-1355): the F16 NZ decode branch
 * (cast, aclnnMatmul, cast: patch:1286-1313) and the A8W8 chain (cast,
 * W8a8QuantizeCustom, MatmulW8a8I32Custom, W8a8DequantCustom, cast:
 * patch:1223-1282) -- here one kernel launch each.
 * w_packed is b200_repack output; x f32 [k]; y f32 [n]. */
int b200_gemv_f16(const void *w_packed, const float *x, float *y, int64_t n, int64_t k, b200_stream_t stream);
/* Small-M F16 matmul (decode batches and speculative tokens): y[j][r] =
 * sum_i w[r][i] * f16(x[j][i]) for j < m <= 8 (fp32 accumulation), the weight
 * streamed once for all m columns on tensor cores.  Replaces the FRACTAL_NZ
 * branch of ggml_cann_mat_mul_fp that the reference takes for up to 8 src1
 * columns (patch:1290-1300).  w: the ggml F16 weight [n rows][k] (k % 8 ==
 * 0, 16-byte aligned); x: f32 [m][ldx]; y: f32 [m][ldy].  m == 1 is
 * b200_gemv_f16.  When m columns of k halves do not fit in shared memory
 * beside the weight ring, the weight streams once per group of columns. */
int b200_mul_mat_f16(const void *w, const float *x, float *y, int64_t n, int64_t k, int m, int64_t ldx, int64_t ldy,
                     b200_stream_t stream);
/* Prefill MUL_MAT with an F16 weight, any number of columns (tokens):
 * y[j][r] = sum_i w[r][i] * f16(x[j][i]) for j < m, on the 5th-generation
 * tensor cores (tcgen05.mma, fp32 accumulator in tensor memory, operands
 * staged by TMA in the 128-byte swizzle).  The reference sends M >= 16 to
 * CANN's own matmul on the ND copy (patch:1200-1204); its NZ kernels serve
 * M <= 8 only.  w: the ggml F16 weight [n rows][k] (k % 8 == 0, 16-byte
 * aligned); x: f32 [m][ldx]; y: f32 [m][ldy]; workspace: device memory of
 * b200_mul_mat_f16_tc_workspace_size(m, k) bytes (16-byte aligned) that
 * receives f16(x) first. */
size_t b200_mul_mat_f16_tc_workspace_size(int64_t m, int64_t k);
int b200_mul_mat_f16_tc(const void *w, const float *x, float *y, int64_t n, int64_t k, int64_t m, int64_t ldx,
                        int64_t ldy, void *workspace, size_t workspace_size, b200_stream_t stream);
int b200_gemv_q4_0(const void *w_packed, const float *x, float *y, int64_t n, int64_t k, int mode,
                   b200_stream_t stream);
int b200_gemv_q8_0_q8_0(const void *w_packed, const float *x, float *y, int64_t n, int64_t k,
                        b200_stream_t stream);

/* The reference add-on's own A8W8 scheme (per-output-column int8 weights,
 * per-token int8 activation, int32 accumulation), as opposed to ggml's
 * Q8_0 x Q8_0 above.
 * b200_a8w8_transform replaces ggml_backend_cann_transform_f16_a8w8
 * (patch:1674-1695): w_f16 holds the ggml F16 weight (n rows of k) on the
 * device; dst (b200_packed_size(B200_TYPE_A8W8, n, k) bytes) receives per
 * row s = max(amax / 127, 1e-8) as f16 and q = clamp(roundf(w / s), +-127).
 * b200_gemv_a8w8 replaces the dispatch chain cast -> W8a8QuantizeCustom ->
 * MatmulW8a8I32Custom -> W8a8DequantCustom -> cast (patch:1223-1282) with one
 * launch: x f32 [k] -> f16 -> int8 with one scale amax / 127 (round half to
 * even), exact int32 dot per row, y[r] = f16(acc * s_x * s_w[r]) as f32. */
int b200_a8w8_transform(const void *w_f16, void *dst, int64_t n, int64_t k, b200_stream_t stream);
int b200_gemv_a8w8(const void *w_packed, const float *x, float *y, int64_t n, int64_t k, b200_stream_t stream);

/* Which weights the reference's A8W8 scheme takes (host only; replaces
 * ggml_cann_310b_is_a8w8_weight and ggml_cann_310b_a8w8_layer_disabled,
 * patch:1481-1533): an F16 weight with ne[2] == ne[3] == 1 that is an FFN
 * gate/up/down weight ("ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"
 * in its ggml name) of a layer "blk.N." not listed in disable_layers, or, with
 * tied_output set, "token_embd.weight" of shape [1536, 151936].
 * disable_layers is the GGML_CANN_A8W8_DISABLE_LAYERS value: comma-separated
 * layers and inclusive ranges ("0-3, 27"); NULL or "" disables none.
 * Returns 1 (selected), 0 (not), or B200_EINVAL for a NULL name or a list item
 * that is not a number or a range of numbers (where the reference throws). */
int b200_a8w8_selects_weight(const char *name, int type, const int64_t ne[4], const char *disable_layers,
                             int tied_output);

/* Exactness exports.  b200_quantize_q8_0 runs the activation quantiser that
 * the Q4_0/Q8_0 GEMVs fuse (replaces W8a8QuantizeCustom,
 * w8a8_quantize_custom_vector.cpp:97-106, with ggml's per-32 Q8_0 rule) and
 * writes ggml block_q8_0 bytes (k/32 * 34).  b200_gemv_block_dots runs the
 * GEMV kernel itself in its export mode: it writes the int32 dot of every
 * (row, 32-block) to dots[n][k/32] and, when xq_blocks != NULL, the Q8_0
 * blocks its prologue quantised x into (k/32 * 34 bytes). */
int b200_quantize_q8_0(const float *x, void *blocks, int64_t k, b200_stream_t stream);
int b200_gemv_block_dots(int type, const void *w_packed, const float *x, int32_t *dots, void *xq_blocks, int64_t n,
                         int64_t k, b200_stream_t stream);

/* ------------------------------------------------------------------------
 * FLASH_ATTN_EXT, one query token (GQA, online softmax, split-KV).
 * Replaces ggml_cann_flash_attn_ext's custom branch (patch:1370-1432) and
 * aclnnAttentionStepCustom (attention_step_custom.cpp:599-622).
 *   q    f32 [n_head][head_dim] (ggml q [D,1,Hq,1], contiguous)
 *   k, v f16; element (t, h, d) at byte t*nb1 + h*nb2 + 2*d (ggml view
 *        [D, n_kv, Hkv] with nb1 = Hkv*D*2 for the llama cache)
 *   mask f16 [n_kv] additive (may be NULL); kv_len int32 [1] (may be NULL):
 *        only the first kv_len[0] positions are read when 0 < kv_len[0] < n_kv
 *        (attention_step_custom.cpp:110-113; src[5] of patch:2009-2023)
 *   out  f32 [n_head][head_dim]
 * q must be 8-byte and out 16-byte aligned.
 * s = scale * (f16(q) . k) + mask; positions whose mask is -inf are skipped.
 * The workspace (b200_fa_workspace_size bytes) must be zero-filled before its
 * first use; every call leaves its counters zero again.  Calls that share a
 * workspace must not overlap on the GPU. */
size_t b200_fa_workspace_size(int head_dim, int n_head, int n_head_kv, int n_kv);
int b200_fa_decode(const float *q, const void *k, const void *v, const void *mask, const int32_t *kv_len,
                   float *out, int head_dim, int n_head, int n_head_kv, int n_kv, int64_t k_nb1, int64_t k_nb2,
                   int64_t v_nb1, int64_t v_nb2, float scale, void *workspace, size_t workspace_size,
                   b200_stream_t stream);

/* Allocation-free FLASH_ATTN_EXT (no counterpart in the reference: the
 * reference's attention always takes its scratch from the CANN memory pool).
 *
 * For callers that cannot allocate device memory when attention runs: a
 * plugin inside an engine whose pool owns every byte of the GPU and must not
 * see foreign allocations, code that runs between another component's
 * allocations and must not shift them, and hosts that link only the kernels
 * and have no buffer to lend.  Arguments and results are those of
 * b200_fa_decode, minus the workspace; the split-KV partials go to a fixed
 * B200_FA_STATIC_SCRATCH_BYTES array inside the library's device image, which
 * every GPU that loads the library holds until the process exits.
 *   - Calls whose b200_fa_workspace_size exceeds that size return
 *     B200_ESCRATCH and launch nothing.
 *   - The first call on a device looks up the array's device address (no
 *     allocation); make that first call before any stream capture.
 *   - One array per device is shared by every call on that device: calls that
 *     overlap on the GPU (other streams, other threads) race and corrupt each
 *     other's results.  Calls in one stream are ordered and safe; each call
 *     clears its own counters first, so an earlier call's leftovers do not
 *     matter.
 * Every head_dim (64, 128, 256) uses the CUDA-core split-KV kernel. */
#define B200_ESCRATCH (-7) /* request larger than a fixed static scratch array */
#define B200_FA_STATIC_SCRATCH_BYTES ((size_t)4 << 20)
int b200_fa_decode_static_scratch(const float *q, const void *k, const void *v, const void *mask,
                                  const int32_t *kv_len, float *out, int head_dim, int n_head, int n_head_kv,
                                  int n_kv, int64_t k_nb1, int64_t k_nb2, int64_t v_nb1, int64_t v_nb2, float scale,
                                  b200_stream_t stream);

/* ------------------------------------------------------------------------
 * Neighbour ops of the decode step, for a backend that runs the graph op by
 * op (the whole-model driver fuses them into the GEMVs).  The reference
 * patches these for the 310B: RMS_NORM decomposed into mul/mean/add/sqrt/div
 * (patch:1133-1170) and enabled in supports_op (patch:1942-1951), SET_ROWS
 * through IndexPut (patch:1179-1184), ROPE through its fallback
 * (patch:1360-1363).  Out-of-range row indices are skipped and set
 * B200_DEVSTATUS_BOUNDS.
 *   rms_norm : rows x n f32; y = x / sqrt(mean(x^2) + eps) (sum in double), then
 *              * w when w != NULL (RMS_NORM followed by MUL)
 *   rope_norm: x, y f32 [n_tokens][n_heads][head_dim]; pos int32 [n_tokens]
 *              (ggml ROPE, mode 0: adjacent pairs)
 *   set_rows : src f32 [nrows][n] -> f16 rows idx[r] of dst (byte stride)
 *   get_rows : Q4_0 table [vocab][n] -> dst f32 [nidx][n]
 *   swiglu   : y = g / (1 + exp(-g)) * u;  add: y = a + b
 *   argmax   : out[0] = index of the first maximum of x[n] */
int b200_rms_norm_f32(const float *x, const float *w, float *y, int64_t n, int64_t rows, float eps,
                      b200_stream_t stream);
int b200_rope_norm_f32(const float *x, float *y, const int32_t *pos, int64_t n_tokens, int n_heads, int head_dim,
                       float freq_base, b200_stream_t stream);
int b200_set_rows_f16(const float *src, const int64_t *rows_idx, void *dst, int64_t n, int64_t nrows,
                      int64_t dst_row_stride, int64_t dst_rows, b200_stream_t stream);
int b200_get_rows_q4_0(const void *table, const int32_t *idx, float *dst, int64_t n, int64_t nidx, int64_t vocab,
                       b200_stream_t stream);
/* GET_ROWS from the packed Q4_0 copy (b200_repack output): a tied token
 * embedding / output matrix then needs one device copy, where the reference
 * keeps an ND and an NZ copy (patch:1451-1468). */
int b200_get_rows_q4_0_packed(const void *table_packed, const int32_t *idx, float *dst, int64_t n, int64_t nidx,
                              int64_t vocab, b200_stream_t stream);
int b200_swiglu_f32(const float *g, const float *u, float *y, int64_t n, b200_stream_t stream);
int b200_add_f32(const float *a, const float *b, float *y, int64_t n, b200_stream_t stream);
/* y = a * b (ggml MUL): b has n elements, or nb elements broadcast over the
 * n / nb rows of a (a norm weight). */
int b200_mul_f32(const float *a, const float *b, float *y, int64_t n, int64_t nb, b200_stream_t stream);
int b200_argmax_f32(const float *x, int64_t n, int32_t *out, b200_stream_t stream);

/* ------------------------------------------------------------------------
 * Weight upload in chunks.  Replaces the reference's TensorSetTracker and the
 * NZ branch of set_tensor (patch:1745-1807): the model loader may call
 * set_tensor for a tensor in pieces and from several threads, and the layout
 * transform can only run once every byte has arrived.
 *   begin: one ggml weight (type, n rows of k) whose packed copy is dst_packed
 *          (b200_packed_size bytes, device); allocates a device staging buffer
 *          of the ggml size on the current device.
 *   write: bytes [offset, offset + size) of the ggml-layout tensor from host
 *          memory; returns once the host memory has been read.  Thread safe.
 *          Covered ranges are tracked exactly (repeats and overlaps count
 *          once); the write that completes the tensor repacks it into
 *          dst_packed and returns with *complete = 1 once that is done.
 *   end:   releases the staging buffer; B200_ESTATE if the tensor never
 *          became complete. */
typedef struct b200_upload b200_upload;
int b200_upload_begin(int type, int64_t n, int64_t k, void *dst_packed, b200_upload **out);
int b200_upload_write(b200_upload *u, size_t offset, const void *host, size_t size, int *complete);
int b200_upload_end(b200_upload *u);

/* Host helper mirroring llama-graph.cpp set_input_kv_lengths_impl
 * (patch:2900-2916): out[r] = 1 + index of the last finite entry of mask row
 * r (at least 1).  mask f16 host array [n_rows][n_kv]. */
int b200_kv_lengths_from_mask_f16(const uint16_t *mask, int64_t n_kv, int64_t n_rows, int32_t *out);

#ifdef __cplusplus
}
#endif
#endif /* B200_DECODE_H */
