/*
 * b200_graph.h -- the ggml-backend core of the B200 decode path: tensor
 * descriptors, buffers, supports_op, get_alloc_size and graph_compute over
 * the kernels of b200_decode.h.  Plain C, no ggml headers: a ggml backend
 * adapter (ggml-b200/ggml-b200.cpp, built against upstream ggml) copies the
 * fields of each struct ggml_tensor into a b200_tensor and forwards the
 * vtable calls here; tests drive the same functions directly.
 *
 * Counterparts in the reference (patches/ascend310b4-llama-cpp.patch, a diff
 * against llama.cpp 37b3a9e0, "patch:N" = line N):
 *   b200_buffer_* (alloc, init/set/get/memset tensor, clear)  -> CANN buffer
 *       interface, set_tensor with the NZ transform (patch:1700-1807)
 *   b200_alloc_size                                           -> get_alloc_size
 *       (patch:1810-1846)
 *   b200_backend_synchronize / free                           -> patch:1862-1881
 *   b200_graph_compute (+ GGML_B200_TRACE_SYNC)               -> graph_compute and
 *       its GGML_CANN_TRACE_NODE_SYNC loop (patch:1884-1923)
 *   b200_supports_op                                          -> supports_op,
 *       with the FLASH_ATTN_EXT gate of patch:1925-1986 (patch:1964-1983)
 */
#ifndef B200_GRAPH_H
#define B200_GRAPH_H

#include <stddef.h>
#include <stdint.h>

#include "b200_decode.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Tensor element types: the values of ggml's enum ggml_type. */
#define B200_TYPE_I32 26
#define B200_TYPE_I64 27

/* Operations (the adapter maps ggml_op to these). */
enum b200_op {
    B200_OP_NONE = 0,        /* leaf: weights, inputs, caches */
    B200_OP_VIEW,            /* VIEW, RESHAPE, PERMUTE, TRANSPOSE: no work, data already set */
    B200_OP_GET_ROWS,        /* src0 Q4_0 [n, vocab] (ggml layout), src1 I32 [m] -> F32 [n, m] */
    B200_OP_RMS_NORM,        /* op_params[0] = eps (f32 bits); F32 rows */
    B200_OP_MUL,             /* F32 * F32, src1 the same shape or one row broadcast over rows */
    B200_OP_ADD,             /* F32 + F32, same shape */
    B200_OP_MUL_MAT,         /* src0 weight F16 / Q4_0 / Q8_0 [K, N], src1 F32 [K, M] -> F32 [N, M] */
    B200_OP_ROPE,            /* ggml ROPE op_params layout; NORM mode only */
    B200_OP_SET_ROWS,        /* src0 F32 [n, r], src1 I64 [r] -> rows of dst F16 [n, rows] */
    B200_OP_FLASH_ATTN_EXT,  /* q, k, v, mask, (sinks), kv_lengths; op_params scale, max_bias, softcap */
    B200_OP_GLU,             /* op_params[0] = glu op (2 = SWIGLU), [1] = swapped; split form (src1 set) */
    B200_OP_ARGMAX,          /* F32 [n, rows] -> I32 [rows] */
    B200_OP_CPY,             /* F32 -> F32 of the same number of elements, both contiguous */
    B200_OP_COUNT
};

#define B200_GLU_SWIGLU 2 /* ggml's GGML_GLU_OP_SWIGLU */
#define B200_MAX_SRC 10
#define B200_MAX_OP_PARAMS 16 /* int32 words, as ggml's 64 bytes */

/* Flags. */
#define B200_TENSOR_WEIGHT 1u /* a matmul weight: its buffer keeps a packed copy (set by b200_buffer_init_tensor) */

/* The fields of struct ggml_tensor the backend reads.  ne / nb as in ggml:
 * ne[0] is the innermost (contiguous) dimension, nb[i] byte strides. */
typedef struct b200_tensor {
    int type;
    int op;
    int64_t ne[4];
    size_t nb[4];
    int32_t op_params[B200_MAX_OP_PARAMS];
    struct b200_tensor *src[B200_MAX_SRC];
    void *data;      /* device address of the tensor in ggml layout */
    void *extra;     /* matmul weights: device address of the packed copy */
    const char *name;
    unsigned flags;
} b200_tensor;

/* ggml_nbytes of the descriptor (0 for an unknown type). */
size_t b200_nbytes(const b200_tensor *t);

/* Environment registry, read once at first use (and again by
 * b200_config_reload):
 *   GGML_B200_DISABLE_F16 / _Q4_0 / _Q8_0 / _FA = 1: supports_op refuses
 *       MUL_MAT with that weight type / FLASH_ATTN_EXT, so the scheduler
 *       places the node on another backend (the oracle comparison switch);
 *   GGML_B200_TRACE_SYNC = 1 or a comma list of op names (MUL_MAT,
 *       FLASH_ATTN_EXT, ...): graph_compute logs each such node's begin and
 *       end on stderr and synchronises the stream after it, reporting the
 *       first failing node (the reference's GGML_CANN_TRACE_NODE_SYNC and
 *       _SYNC_MUL_MAT / _SYNC_SET_ROWS / _SYNC_ROPE, patch:1888-1921);
 *   GGML_B200_NVTX = 1: an NVTX range per node (name and op) for nsys.
 * b200_config_flags returns the parsed switches as bits below. */
#define B200_CFG_DISABLE_F16 1u
#define B200_CFG_DISABLE_Q4_0 2u
#define B200_CFG_DISABLE_Q8_0 4u
#define B200_CFG_DISABLE_FA 8u
#define B200_CFG_TRACE_SYNC 16u
#define B200_CFG_NVTX 32u
unsigned b200_config_flags(void);
void b200_config_reload(void);
/* 1 when GGML_B200_TRACE_SYNC selects nodes of this op. */
int b200_config_traces_op(int op);
const char *b200_op_name(int op);

/* 1: the op can run here; 0: it cannot (the scheduler falls back). */
int b200_supports_op(const b200_tensor *op);

/* Is this tensor a matmul weight whose buffer keeps a packed copy?  Weight
 * buffers only (weights_buffer != 0), F16 / Q4_0 / Q8_0, two-dimensional,
 * rows that the packed layout supports, and -- when the descriptor carries
 * a name -- a ggml name ending in ".weight" (the reference's
 * is_matmul_weight, patch:1451-1468), so a 2-D F16 KV cache is not packed. */
int b200_is_matmul_weight(const b200_tensor *t, int weights_buffer);
/* Bytes a tensor takes in a buffer: ggml_nbytes, and for a matmul weight
 * the ggml bytes rounded up to 256 plus the packed copy, which lives at
 * data + b200_packed_offset (tensor->data stays the ggml-layout slot, as in
 * the reference's dual layout). */
size_t b200_alloc_size(const b200_tensor *t, int weights_buffer);
size_t b200_packed_offset(const b200_tensor *t);

/* ------------------------------------------------------------------ buffer */
typedef struct b200_buffer b200_buffer;
/* size bytes of device memory on `device`, 256-byte aligned. */
int b200_buffer_alloc(int device, size_t size, int weights_buffer, b200_buffer **out);
void b200_buffer_free(b200_buffer *b);
void *b200_buffer_base(b200_buffer *b);
size_t b200_buffer_size(b200_buffer *b);
/* Marks matmul weights (flags, extra = packed copy). */
int b200_buffer_init_tensor(b200_buffer *b, b200_tensor *t);
/* ggml bytes [offset, offset + size) from host memory; for a weight the
 * write that completes the tensor (byte coverage tracked exactly, chunks in
 * any order and from several threads) also builds the packed copy. */
int b200_buffer_set_tensor(b200_buffer *b, b200_tensor *t, const void *host, size_t offset, size_t size);
/* ggml bytes (the original-layout slot) to host memory. */
int b200_buffer_get_tensor(b200_buffer *b, const b200_tensor *t, void *host, size_t offset, size_t size);
int b200_buffer_memset_tensor(b200_buffer *b, b200_tensor *t, uint8_t value, size_t offset, size_t size);
int b200_buffer_clear(b200_buffer *b, uint8_t value);

/* ----------------------------------------------------------------- backend */
typedef struct b200_backend b200_backend;
int b200_backend_create(int device, b200_backend **out);
void b200_backend_free(b200_backend *be);
b200_stream_t b200_backend_stream(b200_backend *be);
int b200_backend_synchronize(b200_backend *be);
/* Runs the nodes in order on the backend's stream (asynchronous unless
 * tracing).  RMS_NORM followed by a MUL of its only consumer with a
 * broadcast row is fused into one kernel.  Returns B200_OK, the failing
 * node's error, or B200_EUNSUPPORTED for a node supports_op refuses. */
int b200_graph_compute(b200_backend *be, b200_tensor *const *nodes, int n_nodes);
/* Index of the node that failed in the last b200_graph_compute, or -1. */
int b200_graph_failed_node(b200_backend *be);

#ifdef __cplusplus
}
#endif
#endif /* B200_GRAPH_H */
