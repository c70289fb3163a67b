// graph.cpp -- the ggml-backend core (include/b200_graph.h): buffers with
// the dual ggml + packed weight layout, supports_op, get_alloc_size and an
// op-by-op graph_compute over the kernels of the C ABI.
//
// Each node runs the kernel of its op on the backend's stream.  MUL_MAT
// weights are read from their packed copy (tensor->extra), filled once when
// set_tensor completes the tensor; everything else is read where ggml put
// it.  The reference's CANN backend has the same shape (patch:1700-1986):
// buffer type + buffer with the NZ transform in set_tensor, an op loop in
// graph_compute with optional per-node synchronisation, and supports_op.
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/b200_graph.h"

namespace {

#define CR(x)                           \
    do {                                \
        const int r_ = (x);             \
        if (r_ != B200_OK) return r_;   \
    } while (0)

int ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        fprintf(stderr, "b200_graph: %s: %s\n", what, cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? B200_ENOMEM : B200_ECUDA;
    }
    return B200_OK;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// ggml block size and bytes per block of the types this backend reads.
bool type_traits(int type, int64_t* blck, size_t* bytes) {
    switch (type) {
        case B200_TYPE_F32: *blck = 1; *bytes = 4; return true;
        case B200_TYPE_F16: *blck = 1; *bytes = 2; return true;
        case B200_TYPE_Q4_0: *blck = 32; *bytes = 18; return true;
        case B200_TYPE_Q8_0: *blck = 32; *bytes = 34; return true;
        case B200_TYPE_I32: *blck = 1; *bytes = 4; return true;
        case B200_TYPE_I64: *blck = 1; *bytes = 8; return true;
        default: return false;
    }
}

int64_t nelements(const b200_tensor* t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

// Rows of ne[0] elements stored back to back (ggml_is_contiguous).
bool contiguous(const b200_tensor* t) {
    int64_t blck;
    size_t bytes;
    if (!type_traits(t->type, &blck, &bytes)) return false;
    if (t->nb[0] != bytes) return false;
    size_t want = (size_t)(t->ne[0] / blck) * bytes;
    for (int i = 1; i < 4; ++i) {
        if (t->ne[i] != 1 && t->nb[i] != want) return false;
        want *= (size_t)t->ne[i];
    }
    return true;
}

float op_f32(const b200_tensor* t, int i) {
    float v;
    std::memcpy(&v, &t->op_params[i], 4);
    return v;
}

// ------------------------------------------------------------------ config

struct Config {
    unsigned flags = 0;
    bool trace_op[B200_OP_COUNT] = {};
};

const char* const kOpNames[B200_OP_COUNT] = {"NONE",    "VIEW", "GET_ROWS",       "RMS_NORM", "MUL",
                                             "ADD",     "MUL_MAT", "ROPE",        "SET_ROWS", "FLASH_ATTN_EXT",
                                             "GLU",     "ARGMAX",  "CPY"};

bool env_on(const char* name) {
    const char* e = getenv(name);
    return e != nullptr && e[0] != '\0' && std::strcmp(e, "0") != 0;
}

Config read_config() {
    Config c;
    if (env_on("GGML_B200_DISABLE_F16")) c.flags |= B200_CFG_DISABLE_F16;
    if (env_on("GGML_B200_DISABLE_Q4_0")) c.flags |= B200_CFG_DISABLE_Q4_0;
    if (env_on("GGML_B200_DISABLE_Q8_0")) c.flags |= B200_CFG_DISABLE_Q8_0;
    if (env_on("GGML_B200_DISABLE_FA")) c.flags |= B200_CFG_DISABLE_FA;
    if (env_on("GGML_B200_NVTX")) c.flags |= B200_CFG_NVTX;
    if (const char* e = getenv("GGML_B200_TRACE_SYNC")) {
        const std::string v(e);
        if (v == "1" || v == "all" || v == "ALL") {
            c.flags |= B200_CFG_TRACE_SYNC;
            for (bool& b : c.trace_op) b = true;
        } else if (!v.empty() && v != "0") {
            size_t p = 0;
            while (p <= v.size()) {
                const size_t q = std::min(v.find(',', p), v.size());
                const std::string name = v.substr(p, q - p);
                for (int op = 0; op < B200_OP_COUNT; ++op)
                    if (name == kOpNames[op]) {
                        c.trace_op[op] = true;
                        c.flags |= B200_CFG_TRACE_SYNC;
                    }
                p = q + 1;
            }
        }
    }
    return c;
}

std::mutex g_cfg_mu;
Config g_cfg;
bool g_cfg_read = false;

Config config() {
    std::lock_guard<std::mutex> lk(g_cfg_mu);
    if (!g_cfg_read) {
        g_cfg = read_config();
        g_cfg_read = true;
    }
    return g_cfg;
}

// --------------------------------------------------------------- op checks

bool is_weight_type(int type) {
    return type == B200_TYPE_F16 || type == B200_TYPE_Q4_0 || type == B200_TYPE_Q8_0;
}

bool f32_rows(const b200_tensor* t) { return t != nullptr && t->type == B200_TYPE_F32 && contiguous(t); }

// A named tensor is a weight only when its ggml name ends in ".weight" (the
// loader's naming: "blk.0.ffn_up.weight", "token_embd.weight"), so that an
// F16 KV cache ("cache_k_l0") in the same buffer is never packed.
bool weight_name(const b200_tensor* t) {
    if (t->name == nullptr) return true;
    const size_t n = std::strlen(t->name);
    return n >= 7 && std::strcmp(t->name + n - 7, ".weight") == 0;
}

bool supports_mul_mat(const b200_tensor* op, const Config& c) {
    const b200_tensor* w = op->src[0];
    const b200_tensor* x = op->src[1];
    if (!w || !x || !is_weight_type(w->type) || w->ne[2] != 1 || w->ne[3] != 1) return false;
    if ((w->type == B200_TYPE_F16 && (c.flags & B200_CFG_DISABLE_F16)) ||
        (w->type == B200_TYPE_Q4_0 && (c.flags & B200_CFG_DISABLE_Q4_0)) ||
        (w->type == B200_TYPE_Q8_0 && (c.flags & B200_CFG_DISABLE_Q8_0)))
        return false;
    if (!f32_rows(x) || op->type != B200_TYPE_F32 || !contiguous(op)) return false;
    if (x->ne[0] != w->ne[0] || x->ne[2] != 1 || x->ne[3] != 1) return false;
    if (op->ne[0] != w->ne[1] || op->ne[1] != x->ne[1]) return false;
    return b200_packed_size(w->type, w->ne[1], w->ne[0]) != 0;
}

// The reference's FLASH_ATTN_EXT gate (patch:1964-1983): one query token,
// f16 K/V with the cache's token-major stride pattern, f16 mask, no ALiBi,
// no softcap; widened here from head dim 64 to 64 / 128 / 256 and any GQA
// ratio.
bool supports_fa(const b200_tensor* op, const Config& c) {
    if (c.flags & B200_CFG_DISABLE_FA) return false;
    const b200_tensor *q = op->src[0], *k = op->src[1], *v = op->src[2], *mask = op->src[3];
    if (!q || !k || !v) return false;
    if (op->src[4] != nullptr) return false;  // attention sinks
    if (q->type != B200_TYPE_F32 || k->type != B200_TYPE_F16 || v->type != B200_TYPE_F16) return false;
    const int64_t D = q->ne[0];
    if (D != 64 && D != 128 && D != 256) return false;
    if (q->ne[1] != 1 || q->ne[3] != 1 || k->ne[3] != 1 || v->ne[3] != 1) return false;
    if (k->ne[0] != D || v->ne[0] != D || k->ne[1] != v->ne[1] || k->ne[2] != v->ne[2]) return false;
    const int64_t hq = q->ne[2], hkv = k->ne[2];
    if (hkv <= 0 || hq % hkv || k->ne[1] <= 0 || k->ne[1] > INT32_MAX) return false;
    if (q->nb[0] != 4 || (hq > 1 && q->nb[2] != (size_t)D * 4)) return false;
    if (k->nb[0] != 2 || v->nb[0] != 2 || (k->nb[1] & 15) || (k->nb[2] & 15) || (v->nb[1] & 15) || (v->nb[2] & 15))
        return false;
    if (mask != nullptr && (mask->type != B200_TYPE_F16 || mask->ne[0] < k->ne[1] || mask->nb[0] != 2)) return false;
    if (op_f32(op, 1) != 0.0f || op_f32(op, 2) != 0.0f) return false;  // max_bias, logit_softcap
    const b200_tensor* kvl = op->src[5];
    if (kvl != nullptr && (kvl->type != B200_TYPE_I32 || !contiguous(kvl))) return false;
    if (op->type != B200_TYPE_F32 || !contiguous(op) || op->ne[0] != D || op->ne[1] != hq) return false;
    return true;
}

bool supports_rope(const b200_tensor* op) {
    const b200_tensor *x = op->src[0], *pos = op->src[1];
    if (!f32_rows(x) || !pos || pos->type != B200_TYPE_I32 || !contiguous(pos) || op->src[2] != nullptr) return false;
    const int n_dims = op->op_params[1], mode = op->op_params[2];
    if (mode != 0 || n_dims != x->ne[0] || (x->ne[0] & 1) || x->ne[3] != 1 || pos->ne[0] != x->ne[2]) return false;
    // freq_scale 1, ext_factor 0, attn_factor 1: plain NORM-mode rotation
    if (op_f32(op, 6) != 1.0f || op_f32(op, 7) != 0.0f || op_f32(op, 8) != 1.0f) return false;
    return op->type == B200_TYPE_F32 && contiguous(op);
}

b200_buffer* buffer_of(const b200_tensor* t);

}  // namespace

// ------------------------------------------------------------------ buffer

struct b200_buffer {
    int device = 0;
    bool weights = false;
    uint8_t* base = nullptr;
    size_t size = 0;
    cudaStream_t stream = nullptr;
    std::mutex mu;
    // per weight tensor (by data address): covered ggml byte ranges
    struct Track {
        std::map<size_t, size_t> covered;
        size_t bytes = 0;
        bool packed = false;
    };
    std::map<const void*, Track> track;
};

struct b200_backend {
    int device = 0;
    cudaStream_t stream = nullptr;
    void* fa_ws = nullptr;
    size_t fa_ws_bytes = 0;
    void* tc_ws = nullptr;
    size_t tc_ws_bytes = 0;
    int failed = -1;
};

namespace {

// Adds [a, b) to an interval set; returns the newly covered bytes.
size_t cover(std::map<size_t, size_t>& m, size_t a, size_t b) {
    size_t added = b - a;
    auto it = m.upper_bound(a);
    if (it != m.begin()) {
        auto pv = std::prev(it);
        if (pv->second >= a) {
            if (pv->second >= b) return 0;
            added -= pv->second - a;
            a = pv->first;
            it = m.erase(pv);
        }
    }
    while (it != m.end() && it->first <= b) {
        const size_t s = it->first, e = it->second;
        added -= (e < b ? e : b) - s;
        if (e > b) b = e;
        it = m.erase(it);
    }
    m[a] = b;
    return added;
}

// FA workspace of the backend, grown when a larger one is needed (zero
// filled; every call leaves its counters zero again).
int fa_workspace(b200_backend* be, size_t need, void** out) {
    if (need > be->fa_ws_bytes) {
        CR(ck(cudaStreamSynchronize(be->stream), "synchronize"));
        if (be->fa_ws) cudaFree(be->fa_ws);
        be->fa_ws = nullptr;
        be->fa_ws_bytes = 0;
        CR(ck(cudaMalloc(&be->fa_ws, need), "FA workspace"));
        CR(ck(cudaMemsetAsync(be->fa_ws, 0, need, be->stream), "FA workspace fill"));
        be->fa_ws_bytes = need;
    }
    *out = be->fa_ws;
    return B200_OK;
}

// Workspace of the prefill GEMM (the f16 copy of the activation), grown on demand.
int tc_workspace(b200_backend* be, size_t need, void** out) {
    if (need > be->tc_ws_bytes) {
        CR(ck(cudaStreamSynchronize(be->stream), "synchronize"));
        if (be->tc_ws) cudaFree(be->tc_ws);
        be->tc_ws = nullptr;
        be->tc_ws_bytes = 0;
        CR(ck(cudaMalloc(&be->tc_ws, need), "GEMM workspace"));
        be->tc_ws_bytes = need;
    }
    *out = be->tc_ws;
    return B200_OK;
}

b200_stream_t S(b200_backend* be) { return (b200_stream_t)be->stream; }

int run_mul_mat(b200_backend* be, b200_tensor* op) {
    const b200_tensor* w = op->src[0];
    const b200_tensor* x = op->src[1];
    const int64_t k = w->ne[0], n = w->ne[1], m = x->ne[1];
    if (w->extra == nullptr) return B200_ESTATE;  // the weight was never uploaded through a b200 weight buffer
    const float* xp = static_cast<const float*>(x->data);
    float* y = static_cast<float*>(op->data);
    const int64_t ldx = (int64_t)(x->nb[1] / 4);
    if (w->type == B200_TYPE_F16 && m > 8) {
        // prefill: the tcgen05 GEMM on the ggml-layout weight
        const size_t need = b200_mul_mat_f16_tc_workspace_size(m, k);
        void* ws = nullptr;
        CR(tc_workspace(be, need, &ws));
        return b200_mul_mat_f16_tc(w->data, xp, y, n, k, m, ldx, n, ws, need, S(be));
    }
    if (w->type == B200_TYPE_F16 && m > 1)  // the reference's small-M (M <= 8) branch
        return b200_mul_mat_f16(w->data, xp, y, n, k, (int)m, ldx, n, S(be));
    for (int64_t j = 0; j < m; ++j) {
        const float* xj = xp + j * (int64_t)(x->nb[1] / 4);
        float* yj = y + j * n;
        switch (w->type) {
            case B200_TYPE_F16: CR(b200_gemv_f16(w->extra, xj, yj, n, k, S(be))); break;
            case B200_TYPE_Q4_0: CR(b200_gemv_q4_0(w->extra, xj, yj, n, k, B200_Q4_MODE_GGML, S(be))); break;
            case B200_TYPE_Q8_0: CR(b200_gemv_q8_0_q8_0(w->extra, xj, yj, n, k, S(be))); break;
            default: return B200_EUNSUPPORTED;
        }
    }
    return B200_OK;
}

int run_fa(b200_backend* be, b200_tensor* op) {
    const b200_tensor *q = op->src[0], *k = op->src[1], *v = op->src[2], *mask = op->src[3], *kvl = op->src[5];
    const int D = (int)q->ne[0], hq = (int)q->ne[2], hkv = (int)k->ne[2], n_kv = (int)k->ne[1];
    const size_t need = b200_fa_workspace_size(D, hq, hkv, n_kv);
    if (need == 0) return B200_EINVAL;
    void* ws = nullptr;
    CR(fa_workspace(be, need, &ws));
    return b200_fa_decode(static_cast<const float*>(q->data), k->data, v->data, mask ? mask->data : nullptr,
                          kvl ? static_cast<const int32_t*>(kvl->data) : nullptr, static_cast<float*>(op->data), D,
                          hq, hkv, n_kv, (int64_t)k->nb[1], (int64_t)k->nb[2], (int64_t)v->nb[1], (int64_t)v->nb[2],
                          op_f32(op, 0), ws, be->fa_ws_bytes, S(be));
}

// How many source slots of the graph's nodes name each tensor.
using Readers = std::unordered_map<const b200_tensor*, int>;

Readers count_readers(b200_tensor* const* nodes, int n) {
    Readers r;
    r.reserve((size_t)n * 2);
    for (int j = 0; j < n; ++j)
        for (int s = 0; s < B200_MAX_SRC; ++s)
            if (nodes[j]->src[s] != nullptr) ++r[nodes[j]->src[s]];
    return r;
}

int run_node(b200_backend* be, b200_tensor* const* nodes, int n, int i, int* skip, const Readers& readers) {
    b200_tensor* op = nodes[i];
    const b200_tensor* a = op->src[0];
    const b200_tensor* b = op->src[1];
    switch (op->op) {
        case B200_OP_NONE:
        case B200_OP_VIEW: return B200_OK;
        case B200_OP_GET_ROWS:
            return b200_get_rows_q4_0(a->data, static_cast<const int32_t*>(b->data), static_cast<float*>(op->data),
                                      a->ne[0], b->ne[0], a->ne[1], S(be));
        case B200_OP_RMS_NORM: {
            const float eps = op_f32(op, 0);
            const int64_t cols = a->ne[0], rows = nelements(a) / cols;
            // RMS_NORM -> MUL by a broadcast weight row, the MUL the only reader: one kernel
            if (i + 1 < n) {
                b200_tensor* nx = nodes[i + 1];
                const b200_tensor* wv = nx->src[1];
                const auto it = readers.find(op);
                if (nx->op == B200_OP_MUL && nx->src[0] == op && f32_rows(wv) && nelements(wv) == cols &&
                    f32_rows(nx) && wv != op && it != readers.end() && it->second == 1) {
                    *skip = 1;
                    return b200_rms_norm_f32(static_cast<const float*>(a->data), static_cast<const float*>(wv->data),
                                             static_cast<float*>(nx->data), cols, rows, eps, S(be));
                }
            }
            return b200_rms_norm_f32(static_cast<const float*>(a->data), nullptr, static_cast<float*>(op->data), cols,
                                     rows, eps, S(be));
        }
        case B200_OP_MUL:
            return b200_mul_f32(static_cast<const float*>(a->data), static_cast<const float*>(b->data),
                                static_cast<float*>(op->data), nelements(a), nelements(b), S(be));
        case B200_OP_ADD:
            return b200_add_f32(static_cast<const float*>(a->data), static_cast<const float*>(b->data),
                                static_cast<float*>(op->data), nelements(a), S(be));
        case B200_OP_MUL_MAT: return run_mul_mat(be, op);
        case B200_OP_ROPE:
            return b200_rope_norm_f32(static_cast<const float*>(a->data), static_cast<float*>(op->data),
                                      static_cast<const int32_t*>(b->data), a->ne[2], (int)a->ne[1], (int)a->ne[0],
                                      op_f32(op, 5), S(be));
        case B200_OP_SET_ROWS:
            return b200_set_rows_f16(static_cast<const float*>(a->data), static_cast<const int64_t*>(b->data),
                                     op->data, a->ne[0], a->ne[1], (int64_t)op->nb[1], op->ne[1], S(be));
        case B200_OP_FLASH_ATTN_EXT: return run_fa(be, op);
        case B200_OP_GLU: {
            const bool swapped = op->op_params[1] != 0;
            const b200_tensor* g = swapped ? b : a;
            const b200_tensor* u = swapped ? a : b;
            return b200_swiglu_f32(static_cast<const float*>(g->data), static_cast<const float*>(u->data),
                                   static_cast<float*>(op->data), nelements(op), S(be));
        }
        case B200_OP_ARGMAX: {
            const int64_t cols = a->ne[0], rows = nelements(a) / cols;
            for (int64_t r = 0; r < rows; ++r)
                CR(b200_argmax_f32(static_cast<const float*>(a->data) + r * cols, cols,
                                   static_cast<int32_t*>(op->data) + r, S(be)));
            return B200_OK;
        }
        case B200_OP_CPY:
            return ck(cudaMemcpyAsync(op->data, a->data, (size_t)nelements(a) * 4, cudaMemcpyDeviceToDevice,
                                      be->stream),
                      "CPY");
        default: return B200_EUNSUPPORTED;
    }
}

}  // namespace

extern "C" {

size_t b200_nbytes(const b200_tensor* t) {
    int64_t blck;
    size_t bytes;
    if (!t || !type_traits(t->type, &blck, &bytes)) return 0;
    for (int i = 0; i < 4; ++i)
        if (t->ne[i] <= 0) return 0;
    size_t nb;
    if (blck == 1) {
        nb = bytes;
        for (int i = 0; i < 4; ++i) nb += (size_t)(t->ne[i] - 1) * t->nb[i];
    } else {
        nb = (size_t)(t->ne[0] / blck) * bytes;
        for (int i = 1; i < 4; ++i) nb += (size_t)(t->ne[i] - 1) * t->nb[i];
    }
    return nb;
}

unsigned b200_config_flags(void) { return config().flags; }

void b200_config_reload(void) {
    std::lock_guard<std::mutex> lk(g_cfg_mu);
    g_cfg = read_config();
    g_cfg_read = true;
}

int b200_config_traces_op(int op) {
    if (op < 0 || op >= B200_OP_COUNT) return 0;
    return config().trace_op[op] ? 1 : 0;
}

const char* b200_op_name(int op) { return op >= 0 && op < B200_OP_COUNT ? kOpNames[op] : "?"; }

int b200_supports_op(const b200_tensor* op) {
    if (!op) return 0;
    const Config c = config();
    const b200_tensor *a = op->src[0], *b = op->src[1];
    switch (op->op) {
        case B200_OP_NONE:
        case B200_OP_VIEW: return 1;
        case B200_OP_GET_ROWS:
            return a && b && a->type == B200_TYPE_Q4_0 && contiguous(a) && b->type == B200_TYPE_I32 &&
                   contiguous(b) && a->ne[2] == 1 && a->ne[3] == 1 && b->ne[1] == 1 && f32_rows(op) &&
                   op->ne[0] == a->ne[0] && op->ne[1] == b->ne[0];
        case B200_OP_RMS_NORM:
            return f32_rows(a) && f32_rows(op) && nelements(op) == nelements(a);
        case B200_OP_MUL:
            return f32_rows(a) && f32_rows(b) && f32_rows(op) && nelements(op) == nelements(a) &&
                   (nelements(b) == nelements(a) || (b->ne[0] == a->ne[0] && nelements(b) == a->ne[0]));
        case B200_OP_ADD:
            return f32_rows(a) && f32_rows(b) && f32_rows(op) && nelements(b) == nelements(a) &&
                   nelements(op) == nelements(a);
        case B200_OP_MUL_MAT: return supports_mul_mat(op, c);
        case B200_OP_ROPE: return supports_rope(op);
        case B200_OP_SET_ROWS:
            return f32_rows(a) && b && b->type == B200_TYPE_I64 && contiguous(b) && b->ne[0] == a->ne[1] &&
                   op->type == B200_TYPE_F16 && op->nb[0] == 2 && op->ne[0] == a->ne[0] && a->ne[2] == 1 &&
                   a->ne[3] == 1;
        case B200_OP_FLASH_ATTN_EXT: return supports_fa(op, c);
        case B200_OP_GLU:
            return op->op_params[0] == B200_GLU_SWIGLU && f32_rows(a) && f32_rows(b) && f32_rows(op) &&
                   nelements(a) == nelements(op) && nelements(b) == nelements(op);
        case B200_OP_ARGMAX:
            return f32_rows(a) && op->type == B200_TYPE_I32 && contiguous(op) && a->ne[0] <= INT32_MAX;
        case B200_OP_CPY: return f32_rows(a) && f32_rows(op) && nelements(a) == nelements(op);
        default: return 0;
    }
}

int b200_is_matmul_weight(const b200_tensor* t, int weights_buffer) {
    if (!t || !weights_buffer || !is_weight_type(t->type) || t->ne[2] != 1 || t->ne[3] != 1) return 0;
    if (!weight_name(t)) return 0;
    if (!contiguous(t)) return 0;
    return b200_packed_size(t->type, t->ne[1], t->ne[0]) != 0 ? 1 : 0;
}

size_t b200_packed_offset(const b200_tensor* t) { return align256(b200_nbytes(t)); }

size_t b200_alloc_size(const b200_tensor* t, int weights_buffer) {
    const size_t nb = b200_nbytes(t);
    if (!b200_is_matmul_weight(t, weights_buffer)) return nb;
    return align256(nb) + b200_packed_size(t->type, t->ne[1], t->ne[0]);
}

int b200_buffer_alloc(int device, size_t size, int weights_buffer, b200_buffer** out) {
    if (!out) return B200_EINVAL;
    *out = nullptr;
    CR(ck(cudaSetDevice(device), "set device"));
    b200_buffer* b = new b200_buffer();
    b->device = device;
    b->weights = weights_buffer != 0;
    b->size = size;
    int rc = ck(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking), "stream");
    if (rc == B200_OK) rc = ck(cudaMalloc(reinterpret_cast<void**>(&b->base), std::max<size_t>(size, 256)), "alloc");
    if (rc != B200_OK) {
        b200_buffer_free(b);
        return rc;
    }
    *out = b;
    return B200_OK;
}

void b200_buffer_free(b200_buffer* b) {
    if (!b) return;
    cudaSetDevice(b->device);
    if (b->stream) cudaStreamSynchronize(b->stream);
    if (b->base) cudaFree(b->base);
    if (b->stream) cudaStreamDestroy(b->stream);
    delete b;
}

void* b200_buffer_base(b200_buffer* b) { return b ? b->base : nullptr; }
size_t b200_buffer_size(b200_buffer* b) { return b ? b->size : 0; }

int b200_buffer_init_tensor(b200_buffer* b, b200_tensor* t) {
    if (!b || !t || !t->data) return B200_EINVAL;
    const uint8_t* p = static_cast<const uint8_t*>(t->data);
    if (p < b->base || p + b200_alloc_size(t, b->weights) > b->base + b->size) return B200_EINVAL;
    if (b200_is_matmul_weight(t, b->weights)) {
        t->flags |= B200_TENSOR_WEIGHT;
        t->extra = static_cast<uint8_t*>(t->data) + b200_packed_offset(t);
        std::lock_guard<std::mutex> lk(b->mu);
        b->track[t->data] = b200_buffer::Track();
    }
    return B200_OK;
}

int b200_buffer_set_tensor(b200_buffer* b, b200_tensor* t, const void* host, size_t offset, size_t size) {
    if (!b || !t || !host || !t->data) return B200_EINVAL;
    const size_t nb = b200_nbytes(t);
    if (offset > nb || size > nb - offset) return B200_EINVAL;
    if (size == 0) return B200_OK;
    CR(ck(cudaSetDevice(b->device), "set device"));
    // set_tensor's contract: the host memory may be reused once this returns
    CR(ck(cudaMemcpyAsync(static_cast<uint8_t*>(t->data) + offset, host, size, cudaMemcpyHostToDevice, b->stream),
          "set_tensor copy"));
    CR(ck(cudaStreamSynchronize(b->stream), "set_tensor sync"));
    if (!(t->flags & B200_TENSOR_WEIGHT)) return B200_OK;
    std::lock_guard<std::mutex> lk(b->mu);
    auto it = b->track.find(t->data);
    if (it == b->track.end()) return B200_ESTATE;  // not initialised through b200_buffer_init_tensor
    b200_buffer::Track& tr = it->second;
    tr.bytes += cover(tr.covered, offset, offset + size);
    if (tr.bytes == nb) {
        // every byte is here: (re)build the packed copy (a tensor written again is packed again)
        CR(b200_repack(t->type, t->data, t->extra, t->ne[1], t->ne[0], (b200_stream_t)b->stream));
        CR(ck(cudaStreamSynchronize(b->stream), "repack sync"));
        tr.packed = true;
        tr.covered.clear();
        tr.bytes = 0;
    }
    return B200_OK;
}

int b200_buffer_get_tensor(b200_buffer* b, const b200_tensor* t, void* host, size_t offset, size_t size) {
    if (!b || !t || !host || !t->data) return B200_EINVAL;
    const size_t nb = b200_nbytes(t);
    if (offset > nb || size > nb - offset) return B200_EINVAL;
    if (size == 0) return B200_OK;
    CR(ck(cudaSetDevice(b->device), "set device"));
    CR(ck(cudaMemcpyAsync(host, static_cast<const uint8_t*>(t->data) + offset, size, cudaMemcpyDeviceToHost,
                          b->stream),
          "get_tensor copy"));
    return ck(cudaStreamSynchronize(b->stream), "get_tensor sync");
}

int b200_buffer_memset_tensor(b200_buffer* b, b200_tensor* t, uint8_t value, size_t offset, size_t size) {
    if (!b || !t || !t->data) return B200_EINVAL;
    const size_t nb = b200_nbytes(t);
    if (offset > nb || size > nb - offset) return B200_EINVAL;
    CR(ck(cudaSetDevice(b->device), "set device"));
    CR(ck(cudaMemsetAsync(static_cast<uint8_t*>(t->data) + offset, value, size, b->stream), "memset"));
    CR(ck(cudaStreamSynchronize(b->stream), "memset sync"));
    if (t->flags & B200_TENSOR_WEIGHT) {  // a weight filled in place: its packed copy follows
        CR(b200_repack(t->type, t->data, t->extra, t->ne[1], t->ne[0], (b200_stream_t)b->stream));
        CR(ck(cudaStreamSynchronize(b->stream), "repack sync"));
    }
    return B200_OK;
}

int b200_buffer_clear(b200_buffer* b, uint8_t value) {
    if (!b) return B200_EINVAL;
    CR(ck(cudaSetDevice(b->device), "set device"));
    CR(ck(cudaMemsetAsync(b->base, value, b->size, b->stream), "clear"));
    return ck(cudaStreamSynchronize(b->stream), "clear sync");
}

int b200_backend_create(int device, b200_backend** out) {
    if (!out) return B200_EINVAL;
    *out = nullptr;
    CR(ck(cudaSetDevice(device), "set device"));
    b200_backend* be = new b200_backend();
    be->device = device;
    const int rc = ck(cudaStreamCreateWithFlags(&be->stream, cudaStreamNonBlocking), "stream");
    if (rc != B200_OK) {
        delete be;
        return rc;
    }
    *out = be;
    return B200_OK;
}

void b200_backend_free(b200_backend* be) {
    if (!be) return;
    cudaSetDevice(be->device);
    if (be->stream) cudaStreamSynchronize(be->stream);
    if (be->fa_ws) cudaFree(be->fa_ws);
    if (be->tc_ws) cudaFree(be->tc_ws);
    if (be->stream) cudaStreamDestroy(be->stream);
    delete be;
}

b200_stream_t b200_backend_stream(b200_backend* be) { return be ? (b200_stream_t)be->stream : nullptr; }

int b200_backend_synchronize(b200_backend* be) {
    if (!be) return B200_EINVAL;
    CR(ck(cudaSetDevice(be->device), "set device"));
    return ck(cudaStreamSynchronize(be->stream), "synchronize");
}

int b200_graph_failed_node(b200_backend* be) { return be ? be->failed : -1; }

int b200_graph_compute(b200_backend* be, b200_tensor* const* nodes, int n_nodes) {
    if (!be || (!nodes && n_nodes > 0) || n_nodes < 0) return B200_EINVAL;
    be->failed = -1;
    CR(ck(cudaSetDevice(be->device), "set device"));
    const Config c = config();
    for (int i = 0; i < n_nodes; ++i)
        if (nodes[i] == nullptr) return B200_EINVAL;
    const Readers readers = count_readers(nodes, n_nodes);
    for (int i = 0; i < n_nodes; ++i) {
        b200_tensor* op = nodes[i];
        if (!b200_supports_op(op)) {
            be->failed = i;
            fprintf(stderr, "b200_graph: node %d (%s, %s) is not supported\n", i, op ? b200_op_name(op->op) : "?",
                    op && op->name ? op->name : "");
            return B200_EUNSUPPORTED;
        }
        const bool trace = (c.flags & B200_CFG_TRACE_SYNC) && op->op < B200_OP_COUNT && c.trace_op[op->op];
        if (trace) fprintf(stderr, "[b200] node %d %s %s: begin\n", i, b200_op_name(op->op), op->name ? op->name : "");
        if (c.flags & B200_CFG_NVTX) {
            char label[160];
            snprintf(label, sizeof(label), "%s %s", b200_op_name(op->op), op->name ? op->name : "");
            nvtxRangePushA(label);
        }
        int skip = 0;
        int rc = run_node(be, nodes, n_nodes, i, &skip, readers);
        if (rc == B200_OK && trace) rc = ck(cudaStreamSynchronize(be->stream), "node synchronize");
        if (c.flags & B200_CFG_NVTX) nvtxRangePop();
        if (rc != B200_OK) {
            be->failed = i;
            fprintf(stderr, "[b200] node %d %s %s failed: %s\n", i, b200_op_name(op->op), op->name ? op->name : "",
                    b200_strerror(rc));
            return rc;
        }
        if (trace) fprintf(stderr, "[b200] node %d %s %s: end\n", i, b200_op_name(op->op), op->name ? op->name : "");
        i += skip;
    }
    return B200_OK;
}

}  // extern "C"
