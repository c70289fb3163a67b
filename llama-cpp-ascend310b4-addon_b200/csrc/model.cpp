// model.cpp -- native batch-1 decode driver (see include/b200_model.h).
//
// Device memory per rank: packed Q4_0 weights of its shard, f32 norms, the
// f16 KV cache of its KV heads ([kv_size][n_head_kv_local * head_dim] per
// layer, the ggml cache layout), a few activation vectors and the step state.
// One decode step = embed, n_layer x (QKV, attention, O [+all-reduce],
// gate/up, down [+all-reduce]), lm_head [+all-reduce max], finish; captured
// once into a CUDA graph and replayed.
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../../include/b200_model.h"
#include "internal.h"

using namespace b200;

#define CK(x)                                                                                         \
    do {                                                                                              \
        cudaError_t e_ = (x);                                                                         \
        if (e_ != cudaSuccess) {                                                                      \
            fprintf(stderr, "b200_model: %s (%s:%d)\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
            return B200_ECUDA;                                                                        \
        }                                                                                             \
    } while (0)
#define CR(x)                           \
    do {                                \
        const int r_ = (x);             \
        if (r_ != B200_OK) return r_;   \
    } while (0)
#define NK(x)                                                                                  \
    do {                                                                                       \
        ncclResult_t n_ = (x);                                                                 \
        if (n_ != ncclSuccess) {                                                               \
            fprintf(stderr, "b200_model: NCCL %s (%s:%d)\n", ncclGetErrorString(n_), __FILE__, \
                    __LINE__);                                                                 \
            return B200_ENCCL;                                                                 \
        }                                                                                      \
    } while (0)

namespace {

struct Layer {
    uint8_t *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr;
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    uint16_t *kc = nullptr, *vc = nullptr;
};

constexpr int64_t kQ4Block = 18;

int64_t q4_bytes(int64_t rows, int64_t cols) { return rows * (cols / 32) * kQ4Block; }

// Seed of one weight tensor's counter stream: distinct per (tensor, layer).
uint64_t tensor_seed(uint64_t seed, int layer, int which) {
    return seed * 0x9E3779B97F4A7C15ull + (uint64_t)(layer + 2) * 0x100ull + (uint64_t)which;
}

// Profiling: event pairs around every launch, accumulated per kernel class.
struct Prof {
    std::vector<cudaEvent_t> ev;
    std::vector<int> cls;
    size_t used = 0;
    int begin(cudaStream_t s, int c) {
        if (used + 2 > ev.size()) {
            for (int i = 0; i < 64; ++i) {
                cudaEvent_t e;
                CK(cudaEventCreate(&e));
                ev.push_back(e);
            }
        }
        CK(cudaEventRecord(ev[used], s));
        cls.push_back(c);
        return B200_OK;
    }
    int end(cudaStream_t s) {
        CK(cudaEventRecord(ev[used + 1], s));
        used += 2;
        return B200_OK;
    }
    ~Prof() {
        for (auto e : ev) cudaEventDestroy(e);
    }
};

}  // namespace

struct b200_model {
    b200_llama_config c{};
    int device = 0, rank = 0, world = 1;
    ncclComm_t comm = nullptr;
    int hq = 0, hkv = 0, ff = 0, voc = 0;
    int64_t qkv_rows = 0;
    std::vector<Layer> L;
    uint8_t* tok_embd = nullptr;
    float* out_norm = nullptr;
    uint8_t* lm_head = nullptr;
    float *x = nullptr, *q = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr;
    StepState* st = nullptr;
    StepState* h_st = nullptr;
    int* h_next = nullptr;
    void* fa_ws = nullptr;
    size_t fa_ws_bytes = 0;
    uint8_t* staging = nullptr;
    size_t staging_bytes = 0;
    cudaStream_t stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    std::vector<void*> allocs;
    uint64_t seed = 0;
    float sigma = 0.f;
    FaLayout fa{};
    // Programmatic dependent launch between the step's kernels (on unless
    // B200_PDL=0): each GEMV starts streaming its weights while the previous
    // kernel drains.
    bool pdl = true;
    // Producers quantise the next GEMV's activation (on unless
    // B200_XQ_FUSED=0): the gate/up epilogue writes the down projection's
    // Q8_0 image (img_h, with per-block tickets), the attention merge writes
    // the o projection's (img_att); those GEMVs copy the image instead of
    // quantising in every CTA.
    bool xq_fused = true;
    // Weight and KV streams of the step are read with the evict_first L2
    // policy (on unless B200_L2_EF=0).
    int l2_ef = 1;
    uint8_t* img_h = nullptr;
    uint8_t* img_att = nullptr;
    int gu_grid = 0;  // CTAs of the gate/up GEMV (the down projection's image fix-up)
    // The O GEMV follows attention, whose fa_ctas CTAs hold as many SMs: its
    // last fa_ctas CTAs start late and get o_late_pct % of an even row share
    // (GemvArgs::late_ctas; B200_O_SKEW, 100 = even).
    int fa_ctas = 0;
    int o_late_pct = 65;
    // Tensor parallel: the O / down partials go to an IPC-shared region
    // (two partial buffers, then the per-rank flags) summed by the
    // peer-memory all-reduce; B200_TP_ALLREDUCE=nccl selects ncclAllReduce.
    bool peer_ar = true;
    // B200_TP_ALLREDUCE=fused: no all-reduce kernel; the O / down epilogue
    // pushes its rows to every rank's receive slots and releases a per-CTA
    // flag, the next GEMV's prologue waits for the flags and sums the slots
    // in rank order (GemvArgs::ar_*).  Layer-dump and profiling steps keep
    // the all-reduce kernel (ar_now is the current step's choice).
    bool ar_fused = false, ar_now = false;
    size_t recv_off = 0, fflags_off = 0;
    int ar_grid_o = 0, ar_grid_down = 0;
    uint8_t* comm_region = nullptr;
    void* peer_region[kMaxRanks] = {};
    size_t part_stride = 0, flags_off = 0;
    // b200_model_timeline: a second captured step whose kernels fold
    // globaltimer stamps into tl_stamps ([3][tl_n]), classes in tl_cls
    unsigned long long* tl_stamps = nullptr;
    std::vector<unsigned long long> tl_host;  // the last timeline step's stamps, [9][tl_n]
    int tl_n = 0;
    std::vector<int> tl_cls;
    cudaGraph_t tl_graph = nullptr;
    cudaGraphExec_t tl_exec = nullptr;
};

namespace {

// Host-side fault injection for failure-detection tests (no GPU fault is
// ever made): B200_INJECT_FAULT=nccl_init makes the communicator set-up
// report an NCCL failure instead of calling NCCL; =alloc:N makes the N-th
// device allocation of b200_model_create report cudaErrorMemoryAllocation.
// Read once per b200_model_create.
struct FaultPlan {
    bool nccl_init = false;
    long alloc_at = -1;  // 1-based index of the allocation that fails
    long allocs = 0;
};

FaultPlan fault_plan() {
    FaultPlan f;
    if (const char* e = getenv("B200_INJECT_FAULT")) {
        if (std::strcmp(e, "nccl_init") == 0) f.nccl_init = true;
        if (std::strncmp(e, "alloc:", 6) == 0) f.alloc_at = atol(e + 6);
    }
    return f;
}

thread_local FaultPlan* t_fault = nullptr;

int dalloc(b200_model* m, void** p, size_t bytes) {
    if (bytes == 0) bytes = 16;
    cudaError_t e;
    if (t_fault != nullptr && ++t_fault->allocs == t_fault->alloc_at) {
        e = cudaErrorMemoryAllocation;
        *p = nullptr;
    } else {
        e = cudaMalloc(p, bytes);
    }
    if (e != cudaSuccess) {
        cudaGetLastError();  // a failed allocation is reported here, not by the next launch check
        fprintf(stderr, "b200_model: cudaMalloc(%zu) failed: %s\n", bytes, cudaGetErrorString(e));
        return B200_ENOMEM;
    }
    m->allocs.push_back(*p);
    return B200_OK;
}

template <class T>
int dalloc_t(b200_model* m, T** p, size_t bytes) {
    void* v = nullptr;
    CR(dalloc(m, &v, bytes));
    *p = static_cast<T*>(v);
    return B200_OK;
}

// Shard geometry of one weight on this rank: rows [r0, r0+nr) and columns
// [c0, c0+nc) of the unsharded [rows][kg] tensor.
int weight_shard(const b200_model* m, int which, int64_t* r0, int64_t* nr, int64_t* c0, int64_t* nc, int64_t* kg) {
    const b200_llama_config& c = m->c;
    const int D = c.head_dim;
    *r0 = 0;
    *c0 = 0;
    switch (which) {
        case B200_W_TOK_EMBD: *nr = c.vocab; *nc = *kg = c.d_model; break;
        case B200_W_Q: *r0 = (int64_t)m->rank * m->hq * D; *nr = (int64_t)m->hq * D; *nc = *kg = c.d_model; break;
        case B200_W_K:
        case B200_W_V: *r0 = (int64_t)m->rank * m->hkv * D; *nr = (int64_t)m->hkv * D; *nc = *kg = c.d_model; break;
        case B200_W_O:
            *nr = c.d_model; *c0 = (int64_t)m->rank * m->hq * D; *nc = (int64_t)m->hq * D; *kg = (int64_t)c.n_head * D;
            break;
        case B200_W_GATE:
        case B200_W_UP: *r0 = (int64_t)m->rank * m->ff; *nr = m->ff; *nc = *kg = c.d_model; break;
        case B200_W_DOWN: *nr = c.d_model; *c0 = (int64_t)m->rank * m->ff; *nc = m->ff; *kg = c.d_ff; break;
        case B200_W_LM_HEAD: *r0 = (int64_t)m->rank * m->voc; *nr = m->voc; *nc = *kg = c.d_model; break;
        default: return B200_EINVAL;
    }
    return B200_OK;
}

// Regenerates one weight shard of this rank in ggml layout at `dst`, which
// holds `cap` bytes; returns its row count and column count through
// rows/cols.  Refuses (EINVAL, nothing launched) when the shard does not fit.
int gen_weight(b200_model* m, int layer, int which, uint8_t* dst, size_t cap, int64_t* rows, int64_t* cols) {
    int64_t r0, nr, c0, nc, kg;
    CR(weight_shard(m, which, &r0, &nr, &c0, &nc, &kg));
    if ((size_t)q4_bytes(nr, nc) > cap) return B200_EINVAL;
    *rows = nr;
    *cols = nc;
    return b200i_synth_q4_0(tensor_seed(m->seed, layer, which), m->sigma, r0, nr, c0, nc, kg, dst, m->stream);
}

float* part_buf(b200_model* m, int which) { return reinterpret_cast<float*>(m->comm_region + which * m->part_stride); }

// x = sum over ranks of partial buffer `which` (0: O projection, 1: down),
// collective `idx` of the step.
// Timeline stamps of one step (b200_model_timeline): kernel i of the step
// folds its entry / post-wait / exit times into base[i], base[n + i],
// base[2n + i] and its phase marks into base[(3..8)n + i]; cls[i] is its
// kernel class (PROFILE classes of b200_model.h).
struct Stamps {
    unsigned long long* base = nullptr;
    int n = 0, next = 0;
    std::vector<int> cls;
    template <class A>
    void assign(A& a, int c) {
        if (next >= n) return;  // more kernels than slots: the rest go unstamped
        a.stamp = base + next;
        a.stamp_stride = n;
        cls.push_back(c);
        ++next;
    }
};

int allreduce_sum(b200_model* m, int which, int idx, cudaStream_t s, bool pdl, Stamps* stamps = nullptr) {
    if (!m->peer_ar) {
        NK(ncclAllReduce(part_buf(m, which), m->x, m->c.d_model, ncclFloat32, ncclSum, m->comm, s));
        return B200_OK;
    }
    ArArgs a;
    std::memset(&a, 0, sizeof(a));
    a.world = m->world;
    a.rank = m->rank;
    a.n = m->c.d_model;
    a.idx = idx;
    a.per_step = 2 * m->c.n_layer;
    a.st = m->st;
    a.x = m->x;
    for (int r = 0; r < m->world; ++r) {
        uint8_t* base = static_cast<uint8_t*>(m->peer_region[r]);
        a.part[r] = reinterpret_cast<const float*>(base + which * m->part_stride);
        a.peer_flag[r] = reinterpret_cast<unsigned long long*>(base + m->flags_off) + m->rank;
    }
    a.flags = reinterpret_cast<unsigned long long*>(m->comm_region + m->flags_off);
    if (stamps) stamps->assign(a, 7);
    return b200i_tp_allreduce(a, s, pdl);
}

// Device buffers of a layer dump (b200_step_dump, same shapes); any may be
// null.  Q8_0 images are ggml block_q8_0 rows.
struct Dump {
    float* x = nullptr;      // [(n_layer + 1) * d]
    float* x_mid = nullptr;  // [n_layer * d]
    float* q = nullptr;      // [n_layer * hq * D]
    uint16_t* k_row = nullptr;
    uint16_t* v_row = nullptr;  // [n_layer * hkv * D]
    float* att = nullptr;    // [n_layer * hq * D]
    float* h = nullptr;      // [n_layer * ff]
    uint8_t *xq_qkv = nullptr, *xq_o = nullptr, *xq_gu = nullptr, *xq_down = nullptr, *xq_head = nullptr;
    int32_t *dots_qkv = nullptr, *dots_o = nullptr, *dots_gu = nullptr, *dots_down = nullptr, *dots_head = nullptr;
    int pos = 0;
};

// Producer-side quantisation (see b200_model::xq_fused): the SwiGLU
// epilogue writes the image only on the split-row path (d_model >= 2048),
// the attention merge only in the tensor-core kernel (head dim 64 / 128).
bool fused_down(const b200_model* m) { return m->xq_fused && m->c.d_model / 32 >= 64 && m->ff % 32 == 0; }
bool fused_o(const b200_model* m) { return m->xq_fused && (m->c.head_dim == 64 || m->c.head_dim == 128); }

// Fused all-reduce (see b200_model::ar_fused).  Producer: collective idx
// (2 l for O, 2 l + 1 for down) lands in slot [which][rank] of every rank.
void set_push(const b200_model* m, GemvArgs& a, int idx, int which) {
    for (int r = 0; r < m->world; ++r) {
        uint8_t* base = static_cast<uint8_t*>(m->peer_region[r]);
        a.ar_dst[r] = reinterpret_cast<float*>(base + m->recv_off + ((size_t)which * m->world + m->rank) * m->part_stride);
        a.ar_flag_dst[r] = reinterpret_cast<unsigned long long*>(base + m->fflags_off) + (size_t)m->rank * kArMaxCtas;
    }
    a.ar_world = m->world;
    a.ar_idx = idx;
    a.ar_per_step = 2 * m->c.n_layer;
    a.ar_st = m->st;
}

// Consumer of collective idx (slots `which`, produced by a grid of `grid`).
void set_ar_consumer(const b200_model* m, GemvArgs& a, int idx, int which, int grid) {
    a.ar_src = reinterpret_cast<const float*>(m->comm_region + m->recv_off + (size_t)which * m->world * m->part_stride);
    a.ar_stride = (int64_t)(m->part_stride / sizeof(float));
    a.ar_flags = reinterpret_cast<unsigned long long*>(m->comm_region + m->fflags_off);
    a.ar_x_out = m->x;
    a.ar_world = m->world;
    a.ar_grid = grid;
    a.ar_idx = idx;
    a.ar_per_step = 2 * m->c.n_layer;
    a.ar_st = m->st;
}

// Argument blocks of the step's kernels (layer l).
GemvArgs qkv_args(const b200_model* m, int l) {
    const b200_llama_config& c = m->c;
    const int D = c.head_dim;
    const Layer& Ly = m->L[l];
    GemvArgs a;
    std::memset(&a, 0, sizeof(a));
    a.w = Ly.wqkv;
    a.n = m->qkv_rows;
    a.k = c.d_model;
    a.x = m->x;
    a.norm_w = Ly.attn_norm;
    a.eps = c.rms_eps;
    a.pro = PRO_RMSNORM;
    a.epi = EPI_QKV;
    a.y = m->q;
    a.nq = m->hq * D;
    a.nkv = m->hkv * D;
    a.head_dim = D;
    a.pos = &m->st->pos;
    a.theta_scale = powf(c.rope_theta, -2.0f / (float)D);
    a.kc = Ly.kc;
    a.vc = Ly.vc;
    if (m->ar_now && l > 0) set_ar_consumer(m, a, 2 * (l - 1) + 1, 1, m->ar_grid_down);
    return a;
}

FaArgs fa_args(const b200_model* m, int l) {
    const b200_llama_config& c = m->c;
    const int D = c.head_dim;
    const Layer& Ly = m->L[l];
    FaArgs f;
    std::memset(&f, 0, sizeof(f));
    f.q = m->q;
    f.k = reinterpret_cast<const uint8_t*>(Ly.kc);
    f.v = reinterpret_cast<const uint8_t*>(Ly.vc);
    f.mask = nullptr;
    f.kv_len = &m->st->ctx;
    f.out = m->att;
    f.Hq = m->hq;
    f.Hkv = m->hkv;
    f.G = m->hq / m->hkv;
    f.gchunks = m->fa.gchunks;
    f.n_kv = c.kv_size;
    f.n_splits = m->fa.n_splits;
    f.chunks_per_split = m->fa.chunks_per_split;
    f.k_nb1 = f.v_nb1 = (int64_t)m->hkv * D * 2;
    f.k_nb2 = f.v_nb2 = (int64_t)D * 2;
    f.scale = 1.0f / sqrtf((float)D);
    uint8_t* ws = static_cast<uint8_t*>(m->fa_ws);
    f.part_o = reinterpret_cast<float*>(ws + m->fa.off_o);
    f.part_ml = reinterpret_cast<float*>(ws + m->fa.off_ml);
    f.tickets = reinterpret_cast<unsigned int*>(ws + m->fa.off_tickets);
    if (fused_o(m)) {
        f.xq_img = m->img_att;
        f.xq_U = m->hq * D / 32;
    }
    return f;
}

// Row-split projection (O: which 0, down: which 1) adding into the residual
// stream; with tensor parallelism rank 0 adds the residual into its partial
// and the others store theirs, for the all-reduce.
GemvArgs proj_args(b200_model* m, int l, int which) {
    const b200_llama_config& c = m->c;
    const Layer& Ly = m->L[l];
    GemvArgs a;
    std::memset(&a, 0, sizeof(a));
    a.w = which == 0 ? Ly.wo : Ly.wdown;
    a.n = c.d_model;
    a.k = which == 0 ? (int64_t)m->hq * c.head_dim : m->ff;
    a.x = which == 0 ? m->att : m->h;
    if (which == 0 && fused_o(m)) a.xq_in = m->img_att;
    if (which == 0) {
        a.late_ctas = m->fa_ctas;
        a.late_pct = m->o_late_pct;
    }
    if (which == 1 && fused_down(m)) {
        a.xq_in = m->img_h;
        a.xq_fix_h = m->h;
        a.xq_fix_out = m->img_h;
        a.xq_fix_items = m->ff;
        a.xq_fix_grid = m->gu_grid;
    }
    a.pro = PRO_PLAIN;
    a.res = m->x;
    if (m->world == 1) {
        a.epi = EPI_ADD;
        a.y = m->x;
    } else if (m->ar_now) {
        a.epi = EPI_PUSH;  // rank 0's partial carries the residual
        a.res = m->rank == 0 ? m->x : nullptr;
        set_push(m, a, 2 * l + which, which);
    } else {
        a.epi = m->rank == 0 ? EPI_ADD : EPI_STORE;
        a.y = part_buf(m, which);
    }
    return a;
}

GemvArgs gate_up_args(const b200_model* m, int l) {
    const b200_llama_config& c = m->c;
    GemvArgs a;
    std::memset(&a, 0, sizeof(a));
    a.w = m->L[l].wgu;
    a.n = 2 * (int64_t)m->ff;
    a.k = c.d_model;
    a.x = m->x;
    a.norm_w = m->L[l].ffn_norm;
    a.eps = c.rms_eps;
    a.pro = PRO_RMSNORM;
    a.epi = EPI_SWIGLU;
    a.y = m->h;
    if (fused_down(m)) a.xq_img = m->img_h;
    if (m->ar_now) set_ar_consumer(m, a, 2 * l, 0, m->ar_grid_o);
    return a;
}

GemvArgs head_args(const b200_model* m) {
    const b200_llama_config& c = m->c;
    GemvArgs a;
    std::memset(&a, 0, sizeof(a));
    a.w = m->lm_head;
    a.n = m->voc;
    a.k = c.d_model;
    a.x = m->x;
    a.norm_w = m->out_norm;
    a.eps = c.rms_eps;
    a.pro = PRO_RMSNORM;
    a.epi = EPI_ARGMAX;
    a.y = m->logits;
    a.amax = &m->st->amax;
    a.row_offset = (int64_t)m->rank * m->voc;
    if (m->ar_now) set_ar_consumer(m, a, 2 * m->c.n_layer - 1, 1, m->ar_grid_down);
    return a;
}

int enqueue_step(b200_model* m, cudaStream_t s, Prof* prof, const Dump* dump = nullptr, Stamps* stamps = nullptr) {
    const b200_llama_config& c = m->c;
    const int D = c.head_dim;
    auto B = [&](int cls) { return prof ? prof->begin(s, cls) : B200_OK; };
    auto E = [&]() { return prof ? prof->end(s) : B200_OK; };
    // events and dump copies between the kernels would serialise them anyway
    const bool pdl = m->pdl && !prof && !dump;
    m->ar_now = m->world > 1 && m->ar_fused && !prof && !dump;

    CR(B(0));
    CR(b200i_embed(m->tok_embd, c.d_model, c.vocab, m->st, m->x, s));
    CR(E());

    const size_t qbytes = (size_t)m->hq * D * sizeof(float);
    const int64_t qd = (int64_t)m->hq * D, kvd = (int64_t)m->hkv * D, d = c.d_model;
    // Layer-dump hooks: the GEMV's own prologue image (CTA 0) and its
    // per-block dots (the export variant of the same kernel), or a copy of
    // the producer-written image the GEMV reads.
    auto dcopy = [&](void* dst, const void* src, size_t bytes) {
        return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s);
    };
    auto hook = [&](GemvArgs& a, uint8_t* xq, int32_t* dots) {
        if (xq != nullptr && a.xq_in == nullptr) a.xq_out = xq;
        if (dots != nullptr) a.dots = dots;
        return dots != nullptr;
    };
    auto image_out = [&](const uint8_t* img, uint8_t* xq, int64_t k) -> int {
        return b200i_image_to_q8_0(img, k / 32, xq, s);
    };
    if (dump && dump->x) CK(dcopy(dump->x, m->x, d * sizeof(float)));
    auto l2 = [&](GemvArgs& a) { a.l2_ef = m->l2_ef; };
    for (int l = 0; l < c.n_layer; ++l) {
        CR(B(1));
        {
            GemvArgs a = qkv_args(m, l);
            l2(a);
            bool dbg = false;
            if (dump)
                dbg = hook(a, dump->xq_qkv ? dump->xq_qkv + (size_t)l * (d / 32) * 34 : nullptr,
                           dump->dots_qkv ? dump->dots_qkv + (size_t)l * m->qkv_rows * (d / 32) : nullptr);
            if (stamps) stamps->assign(a, 1);
            CR(b200i_gemv(FMT_Q4, a, dbg, s, pdl));
        }
        CR(E());
        if (dump) {
            if (dump->q) CK(dcopy(dump->q + (size_t)l * qd, m->q, qbytes));
            const size_t off = (size_t)dump->pos * kvd;
            if (dump->k_row) CK(dcopy(dump->k_row + (size_t)l * kvd, m->L[l].kc + off, kvd * 2));
            if (dump->v_row) CK(dcopy(dump->v_row + (size_t)l * kvd, m->L[l].vc + off, kvd * 2));
        }
        CR(B(2));
        {
            FaArgs f = fa_args(m, l);
            f.l2_ef = m->l2_ef;
            if (stamps) stamps->assign(f, 2);
            CR(b200i_fa(f, D, s, pdl));
        }
        CR(E());
        if (dump && dump->att) CK(dcopy(dump->att + (size_t)l * qd, m->att, qbytes));
        CR(B(3));
        {
            GemvArgs a = proj_args(m, l, 0);
            l2(a);
            bool dbg = false;
            if (dump) {
                uint8_t* xq = dump->xq_o ? dump->xq_o + (size_t)l * (qd / 32) * 34 : nullptr;
                if (xq && a.xq_in) CR(image_out(a.xq_in, xq, qd));
                dbg = hook(a, xq, dump->dots_o ? dump->dots_o + (size_t)l * d * (qd / 32) : nullptr);
            }
            if (stamps) stamps->assign(a, 3);
            CR(b200i_gemv(FMT_Q4, a, dbg, s, pdl));
        }
        CR(E());
        if (m->world > 1 && !m->ar_now) {
            CR(B(7));
            CR(allreduce_sum(m, 0, 2 * l, s, pdl, stamps));
            CR(E());
        }
        if (dump && dump->x_mid) CK(dcopy(dump->x_mid + (size_t)l * d, m->x, d * sizeof(float)));
        CR(B(4));
        {
            GemvArgs a = gate_up_args(m, l);
            l2(a);
            bool dbg = false;
            if (dump)
                dbg = hook(a, dump->xq_gu ? dump->xq_gu + (size_t)l * (d / 32) * 34 : nullptr,
                           dump->dots_gu ? dump->dots_gu + (size_t)l * 2 * m->ff * (d / 32) : nullptr);
            if (stamps) stamps->assign(a, 4);
            CR(b200i_gemv(FMT_Q4, a, dbg, s, pdl));
        }
        CR(E());
        if (dump && dump->h) CK(dcopy(dump->h + (size_t)l * m->ff, m->h, (size_t)m->ff * sizeof(float)));
        CR(B(5));
        {
            GemvArgs a = proj_args(m, l, 1);
            l2(a);
            bool dbg = false;
            uint8_t* xq = nullptr;
            if (dump) {
                xq = dump->xq_down ? dump->xq_down + (size_t)l * (m->ff / 32) * 34 : nullptr;
                dbg = hook(a, xq, dump->dots_down ? dump->dots_down + (size_t)l * d * (m->ff / 32) : nullptr);
            }
            if (stamps) stamps->assign(a, 5);
            CR(b200i_gemv(FMT_Q4, a, dbg, s, pdl));
            // the image is complete once this GEMV has quantised the blocks
            // its producer's CTAs share (written back by its CTA 0)
            if (xq && a.xq_in) CR(image_out(a.xq_in, xq, m->ff));
        }
        CR(E());
        if (m->world > 1 && !m->ar_now) {
            CR(B(7));
            CR(allreduce_sum(m, 1, 2 * l + 1, s, pdl, stamps));
            CR(E());
        }
        if (dump && dump->x) CK(dcopy(dump->x + (size_t)(l + 1) * d, m->x, d * sizeof(float)));
    }
    CR(B(6));
    {
        GemvArgs a = head_args(m);
        l2(a);
        bool dbg = false;
        if (dump) dbg = hook(a, dump->xq_head, dump->dots_head);
        if (stamps) stamps->assign(a, 6);
        CR(b200i_gemv(FMT_Q4, a, dbg, s, pdl));
    }
    CR(E());
    if (m->world > 1) {
        CR(B(7));
        NK(ncclAllReduce(&m->st->amax, &m->st->amax, 1, ncclUint64, ncclMax, m->comm, s));
        CR(E());
    }
    CR(b200i_finish(m->st, s));
    return B200_OK;
}

// Partial buffers (and, for the peer all-reduce, the flags) of tensor
// parallelism.  With the peer all-reduce the region is shared: every rank
// maps every peer's region through CUDA IPC, the handles travelling through
// one ncclAllGather.
int setup_comm_region(b200_model* m) {
    if (m->world == 1) return B200_OK;
    m->part_stride = (size_t)align256((size_t)m->c.d_model * sizeof(float));
    m->flags_off = 2 * m->part_stride;
    m->recv_off = m->flags_off + 256;  // fused all-reduce: receive slots [2][world][d], flags [kMaxRanks][kArMaxCtas]
    m->fflags_off = m->recv_off + 2 * (size_t)m->world * m->part_stride;
    const size_t bytes = m->fflags_off + (size_t)kMaxRanks * kArMaxCtas * sizeof(unsigned long long);
    if (cudaMalloc(reinterpret_cast<void**>(&m->comm_region), bytes) != cudaSuccess) {
        cudaGetLastError();
        return B200_ENOMEM;
    }
    CK(cudaMemset(m->comm_region, 0, bytes));
    if (!m->peer_ar) return B200_OK;
    cudaIpcMemHandle_t mine;
    CK(cudaIpcGetMemHandle(&mine, m->comm_region));
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    uint8_t* d = nullptr;
    CK(cudaMalloc(reinterpret_cast<void**>(&d), 64 * (size_t)(m->world + 1)));
    std::vector<cudaIpcMemHandle_t> all(m->world);
    int rc = B200_OK;
    if (cudaMemcpy(d, &mine, 64, cudaMemcpyHostToDevice) != cudaSuccess) rc = B200_ECUDA;
    if (rc == B200_OK && ncclAllGather(d, d + 64, 64, ncclUint8, m->comm, m->stream) != ncclSuccess) rc = B200_ENCCL;
    if (rc == B200_OK && cudaStreamSynchronize(m->stream) != cudaSuccess) rc = B200_ECUDA;
    if (rc == B200_OK && cudaMemcpy(all.data(), d + 64, 64 * (size_t)m->world, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = B200_ECUDA;
    cudaFree(d);
    if (rc) return rc;
    for (int r = 0; r < m->world; ++r) {
        if (r == m->rank) {
            m->peer_region[r] = m->comm_region;
            continue;
        }
        CK(cudaIpcOpenMemHandle(&m->peer_region[r], all[r], cudaIpcMemLazyEnablePeerAccess));
    }
    return B200_OK;
}

int validate(const b200_llama_config& c, int world) {
    if (c.n_layer <= 0 || c.d_model <= 0 || c.n_head <= 0 || c.n_head_kv <= 0 || c.head_dim <= 0 || c.d_ff <= 0 ||
        c.vocab <= 0 || c.kv_size <= 0 || world <= 0)
        return B200_EINVAL;
    if (c.n_head % c.n_head_kv || c.n_head_kv % world || c.d_ff % (32 * world) || c.vocab % world)
        return B200_EINVAL;
    if (c.d_model % 256 || c.head_dim % 2 || ((c.n_head / world) * c.head_dim) % 32) return B200_EINVAL;
    if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256) return B200_EUNSUPPORTED;
    return B200_OK;
}

}  // namespace

extern "C" {

int b200_nccl_unique_id(void* out128) {
    if (!out128) return B200_EINVAL;
    ncclUniqueId id;
    NK(ncclGetUniqueId(&id));
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
    std::memcpy(out128, &id, sizeof(id));
    return B200_OK;
}

int b200_model_create(const b200_llama_config* cfg, int device, int tp_rank, int tp_world, const void* nccl_id128,
                      b200_model** out) {
    if (!cfg || !out) return B200_EINVAL;
    *out = nullptr;
    CR(validate(*cfg, tp_world));
    if (tp_rank < 0 || tp_rank >= tp_world || (tp_world > 1 && !nccl_id128)) return B200_EINVAL;
    CK(cudaSetDevice(device));
    b200_model* m = new b200_model();
    m->c = *cfg;
    m->device = device;
    if (const char* e = getenv("B200_PDL")) m->pdl = atoi(e) != 0;
    if (const char* e = getenv("B200_XQ_FUSED")) m->xq_fused = atoi(e) != 0;
    if (const char* e = getenv("B200_L2_EF")) m->l2_ef = atoi(e) != 0;

    m->rank = tp_rank;
    m->world = tp_world;
    const b200_llama_config& c = m->c;
    const int D = c.head_dim;
    m->hq = c.n_head / tp_world;
    m->hkv = c.n_head_kv / tp_world;
    m->ff = c.d_ff / tp_world;
    m->voc = c.vocab / tp_world;
    m->qkv_rows = (int64_t)(m->hq + 2 * m->hkv) * D;
    int rc = B200_OK;
    auto fail = [&](int r) {
        b200_model_destroy(m);
        return r;
    };
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(B200_ECUDA);
    FaultPlan fp = fault_plan();
    t_fault = &fp;
    struct Reset {
        ~Reset() { t_fault = nullptr; }
    } reset_fault;
    if (tp_world > 1) {
        ncclUniqueId id;
        std::memcpy(&id, nccl_id128, sizeof(id));
        const ncclResult_t nr = fp.nccl_init ? ncclSystemError : ncclCommInitRank(&m->comm, tp_world, id, tp_rank);
        if (nr != ncclSuccess) {
            fprintf(stderr, "b200_model: NCCL communicator set-up failed: %s\n", ncclGetErrorString(nr));
            m->comm = nullptr;
            return fail(B200_ENCCL);
        }
    }
    if (const char* e = getenv("B200_TP_ALLREDUCE")) {
        m->peer_ar = std::strcmp(e, "nccl") != 0;
        m->ar_fused = std::strcmp(e, "fused") == 0;
    }
    if (tp_world > kMaxRanks) m->peer_ar = m->ar_fused = false;
    if ((rc = setup_comm_region(m))) return fail(rc);
    if (m->ar_fused) {
        m->ar_grid_o = b200i_gemv_grid(FMT_Q4, c.d_model, (int64_t)m->hq * D, EPI_PUSH);
        m->ar_grid_down = b200i_gemv_grid(FMT_Q4, c.d_model, m->ff, EPI_PUSH);
        if (m->ar_grid_o <= 0 || m->ar_grid_o > kArMaxCtas || m->ar_grid_down <= 0 || m->ar_grid_down > kArMaxCtas)
            m->ar_fused = false;
    }
    const size_t p_qkv = b200_packed_size(B200_TYPE_Q4_0, m->qkv_rows, c.d_model);
    const size_t p_o = b200_packed_size(B200_TYPE_Q4_0, c.d_model, (int64_t)m->hq * D);
    const size_t p_gu = b200_packed_size(B200_TYPE_Q4_0, 2 * (int64_t)m->ff, c.d_model);
    const size_t p_down = b200_packed_size(B200_TYPE_Q4_0, c.d_model, m->ff);
    const size_t p_head = b200_packed_size(B200_TYPE_Q4_0, m->voc, c.d_model);
    if (!p_qkv || !p_o || !p_gu || !p_down || !p_head) return fail(B200_EUNSUPPORTED);
    const size_t kv_bytes = (size_t)c.kv_size * m->hkv * D * 2;
    m->L.resize(c.n_layer);
    for (auto& Ly : m->L) {
        if ((rc = dalloc_t(m, &Ly.wqkv, p_qkv)) || (rc = dalloc_t(m, &Ly.wo, p_o)) ||
            (rc = dalloc_t(m, &Ly.wgu, p_gu)) || (rc = dalloc_t(m, &Ly.wdown, p_down)) ||
            (rc = dalloc_t(m, &Ly.attn_norm, c.d_model * 4)) || (rc = dalloc_t(m, &Ly.ffn_norm, c.d_model * 4)) ||
            (rc = dalloc_t(m, &Ly.kc, kv_bytes)) || (rc = dalloc_t(m, &Ly.vc, kv_bytes)))
            return fail(rc);
    }
    m->staging_bytes = (size_t)std::max<int64_t>(
        std::max<int64_t>(q4_bytes(m->qkv_rows, c.d_model), q4_bytes(c.d_model, (int64_t)m->hq * D)),
        std::max<int64_t>(std::max<int64_t>(2 * q4_bytes(m->ff, c.d_model), q4_bytes(c.d_model, m->ff)),
                          q4_bytes(m->voc, c.d_model)));
    m->fa = fa_layout(D, m->hq, m->hkv, c.kv_size);
    m->fa_ws_bytes = m->fa.total;
    if ((rc = dalloc_t(m, &m->tok_embd, q4_bytes(c.vocab, c.d_model))) || (rc = dalloc_t(m, &m->lm_head, p_head)) ||
        (rc = dalloc_t(m, &m->out_norm, c.d_model * 4)) || (rc = dalloc_t(m, &m->x, c.d_model * 4)) ||
        (rc = dalloc_t(m, &m->q, (size_t)m->hq * D * 4)) || (rc = dalloc_t(m, &m->att, (size_t)m->hq * D * 4)) ||
        (rc = dalloc_t(m, &m->h, (size_t)m->ff * 4)) ||
        (rc = dalloc_t(m, &m->logits, (size_t)m->voc * 4)) || (rc = dalloc_t(m, &m->st, sizeof(StepState))) ||
        (rc = dalloc(m, &m->fa_ws, m->fa_ws_bytes)) || (rc = dalloc_t(m, &m->staging, m->staging_bytes)))
        return fail(rc);
    if ((rc = dalloc_t(m, &m->img_h, (size_t)(40 * (m->ff / 32)))) ||
        (rc = dalloc_t(m, &m->img_att, (size_t)(40 * ((int64_t)m->hq * D / 32)))))
        return fail(rc);
    m->fa_ctas = b200i_fa_ctas(fa_args(m, 0), D);
    if (const char* e = getenv("B200_O_SKEW")) m->o_late_pct = std::max(1, std::min(100, atoi(e)));
    m->gu_grid = b200i_gemv_grid(FMT_Q4, 2 * (int64_t)m->ff, c.d_model, EPI_SWIGLU);
    if (m->gu_grid <= 0 || 2 * (m->gu_grid - 1) > kGemvThreads) return fail(B200_EUNSUPPORTED);  // one fix-up round
    if (cudaMemset(m->fa_ws, 0, m->fa_ws_bytes) != cudaSuccess) return fail(B200_ECUDA);
    if (cudaMallocHost(reinterpret_cast<void**>(&m->h_st), sizeof(StepState)) != cudaSuccess) return fail(B200_ENOMEM);
    if (cudaMallocHost(reinterpret_cast<void**>(&m->h_next), sizeof(int)) != cudaSuccess) return fail(B200_ENOMEM);
    std::memset(m->h_st, 0, sizeof(StepState));
    m->h_st->ctx = 1;
    if (cudaMemcpy(m->st, m->h_st, sizeof(StepState), cudaMemcpyHostToDevice) != cudaSuccess) return fail(B200_ECUDA);
    *out = m;
    return B200_OK;
}

void b200_model_destroy(b200_model* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    // Graphs that hold NCCL work are released before the communicator.
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    if (m->tl_exec) cudaGraphExecDestroy(m->tl_exec);
    if (m->tl_graph) cudaGraphDestroy(m->tl_graph);
    if (m->tl_stamps) cudaFree(m->tl_stamps);
    if (m->comm && m->comm_region && m->x) {
        // no peer may still read this rank's region when it is unmapped and freed
        ncclAllReduce(m->x, m->x, 1, ncclFloat32, ncclSum, m->comm, m->stream);
        cudaStreamSynchronize(m->stream);
    }
    for (int r = 0; r < kMaxRanks; ++r)
        if (m->peer_region[r] && r != m->rank) cudaIpcCloseMemHandle(m->peer_region[r]);
    if (m->comm_region) cudaFree(m->comm_region);
    if (m->comm) ncclCommDestroy(m->comm);
    for (void* p : m->allocs) cudaFree(p);
    if (m->h_st) cudaFreeHost(m->h_st);
    if (m->h_next) cudaFreeHost(m->h_next);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

int b200_model_init_synthetic(b200_model* m, uint64_t seed, float sigma) {
    if (!m) return B200_EINVAL;
    CK(cudaSetDevice(m->device));
    m->seed = seed;
    m->sigma = sigma;
    const b200_llama_config& c = m->c;
    const cudaStream_t s = m->stream;
    int64_t r, k;
    CR(gen_weight(m, -1, B200_W_TOK_EMBD, m->tok_embd, (size_t)q4_bytes(c.vocab, c.d_model), &r, &k));
    CR(gen_weight(m, -1, B200_W_LM_HEAD, m->staging, m->staging_bytes, &r, &k));
    CR(b200_repack(B200_TYPE_Q4_0, m->staging, m->lm_head, r, k, (b200_stream_t)s));
    CR(b200i_fill_f32(m->out_norm, c.d_model, 1.0f, s));
    for (int l = 0; l < c.n_layer; ++l) {
        Layer& Ly = m->L[l];
        int64_t rq, rk, rv;
        CR(gen_weight(m, l, B200_W_Q, m->staging, m->staging_bytes, &rq, &k));
        CR(gen_weight(m, l, B200_W_K, m->staging + q4_bytes(rq, k), m->staging_bytes - q4_bytes(rq, k), &rk, &k));
        CR(gen_weight(m, l, B200_W_V, m->staging + q4_bytes(rq + rk, k), m->staging_bytes - q4_bytes(rq + rk, k),
                       &rv, &k));
        CR(b200_repack(B200_TYPE_Q4_0, m->staging, Ly.wqkv, rq + rk + rv, k, (b200_stream_t)s));
        CR(gen_weight(m, l, B200_W_O, m->staging, m->staging_bytes, &r, &k));
        CR(b200_repack(B200_TYPE_Q4_0, m->staging, Ly.wo, r, k, (b200_stream_t)s));
        int64_t rg, ru;
        CR(gen_weight(m, l, B200_W_GATE, m->staging, m->staging_bytes, &rg, &k));
        CR(gen_weight(m, l, B200_W_UP, m->staging + q4_bytes(rg, k), m->staging_bytes - q4_bytes(rg, k), &ru, &k));
        CR(b200_repack_interleave2(B200_TYPE_Q4_0, m->staging, m->staging + q4_bytes(rg, k), Ly.wgu, rg, k,
                                   (b200_stream_t)s));
        CR(gen_weight(m, l, B200_W_DOWN, m->staging, m->staging_bytes, &r, &k));
        CR(b200_repack(B200_TYPE_Q4_0, m->staging, Ly.wdown, r, k, (b200_stream_t)s));
        CR(b200i_fill_f32(Ly.attn_norm, c.d_model, 1.0f, s));
        CR(b200i_fill_f32(Ly.ffn_norm, c.d_model, 1.0f, s));
    }
    CK(cudaStreamSynchronize(s));
    return B200_OK;
}

int b200_model_fill_kv_synthetic(b200_model* m, uint64_t seed, int n_pos) {
    if (!m || n_pos < 0 || n_pos > m->c.kv_size) return B200_EINVAL;
    CK(cudaSetDevice(m->device));
    const b200_llama_config& c = m->c;
    const int64_t rl = (int64_t)m->hkv * c.head_dim, rg = (int64_t)c.n_head_kv * c.head_dim;
    const int64_t col0 = (int64_t)m->rank * rl;
    for (int l = 0; l < c.n_layer; ++l) {
        for (int w = 0; w < 2; ++w) {
            const uint64_t base = ((uint64_t)(2 * l + w)) << 40;
            CR(b200i_synth_rows_f16(seed, base, n_pos, rl, rg, col0, w ? (void*)m->L[l].vc : (void*)m->L[l].kc,
                                    m->stream));
        }
    }
    CK(cudaStreamSynchronize(m->stream));
    return B200_OK;
}

int b200_model_export_weight(b200_model* m, int layer, int which, void* host, size_t* bytes) {
    if (!m || !bytes) return B200_EINVAL;
    if (which != B200_W_TOK_EMBD && which != B200_W_LM_HEAD && (layer < 0 || layer >= m->c.n_layer))
        return B200_EINVAL;
    CK(cudaSetDevice(m->device));
    int64_t r0, nr, c0, nc, kg;
    CR(weight_shard(m, which, &r0, &nr, &c0, &nc, &kg));
    const size_t need = (size_t)q4_bytes(nr, nc);
    if (!host) {
        *bytes = need;
        return B200_OK;
    }
    if (*bytes < need) return B200_EINVAL;
    const uint8_t* src = m->tok_embd;  // the embedding table is resident in ggml layout on every rank
    if (which != B200_W_TOK_EMBD) {
        int64_t r, k;
        CR(gen_weight(m, which == B200_W_LM_HEAD ? -1 : layer, which, m->staging, m->staging_bytes, &r, &k));
        src = m->staging;
    }
    CK(cudaMemcpyAsync(host, src, need, cudaMemcpyDeviceToHost, m->stream));
    CK(cudaStreamSynchronize(m->stream));
    *bytes = need;
    return B200_OK;
}

int b200_model_export_kv(b200_model* m, int layer, int which, int n_pos, void* host) {
    if (!m || !host || layer < 0 || layer >= m->c.n_layer || which < 0 || which > 1 || n_pos < 0 ||
        n_pos > m->c.kv_size)
        return B200_EINVAL;
    CK(cudaSetDevice(m->device));
    const size_t bytes = (size_t)n_pos * m->hkv * m->c.head_dim * 2;
    CK(cudaMemcpyAsync(host, which ? (void*)m->L[layer].vc : (void*)m->L[layer].kc, bytes, cudaMemcpyDeviceToHost,
                       m->stream));
    CK(cudaStreamSynchronize(m->stream));
    return B200_OK;
}

int b200_model_capture(b200_model* m) {
    if (!m) return B200_EINVAL;
    CK(cudaSetDevice(m->device));
    if (m->exec) return B200_OK;
    CR(b200i_prepare_device());
    CK(cudaStreamSynchronize(m->stream));
    CK(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue_step(m, m->stream, nullptr);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (rc != B200_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    CK(e);
    m->graph = g;
    CK(cudaGraphInstantiate(&m->exec, m->graph, 0));
    return B200_OK;
}

int b200_model_set_state(b200_model* m, int token, int pos, int advance) {
    if (!m || pos < 0 || pos >= m->c.kv_size || token < 0 || token >= m->c.vocab) return B200_EINVAL;
    CK(cudaSetDevice(m->device));
    CK(cudaStreamSynchronize(m->stream));
    m->h_st->token = token;
    m->h_st->pos = pos;
    m->h_st->ctx = pos + 1;
    m->h_st->advance = advance ? 1 : 0;
    CK(cudaMemcpyAsync(m->st, m->h_st, 4 * sizeof(int), cudaMemcpyHostToDevice, m->stream));
    return B200_OK;
}

int b200_model_launch(b200_model* m) {
    if (!m) return B200_EINVAL;
    if (!m->exec) CR(b200_model_capture(m));
    CK(cudaGraphLaunch(m->exec, m->stream));
    return B200_OK;
}

int b200_model_decode(b200_model* m, int token, int pos, int* next_token, float* logits_host) {
    if (!m || pos < 0 || pos >= m->c.kv_size || token < 0 || token >= m->c.vocab) return B200_EINVAL;
    CK(cudaSetDevice(m->device));
    if (!m->exec) CR(b200_model_capture(m));
    m->h_st->token = token;
    m->h_st->pos = pos;
    m->h_st->ctx = pos + 1;
    m->h_st->advance = 0;
    CK(cudaMemcpyAsync(m->st, m->h_st, 4 * sizeof(int), cudaMemcpyHostToDevice, m->stream));
    CK(cudaGraphLaunch(m->exec, m->stream));
    CK(cudaMemcpyAsync(m->h_next, &m->st->next, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    if (logits_host)
        CK(cudaMemcpyAsync(logits_host, m->logits, (size_t)m->voc * 4, cudaMemcpyDeviceToHost, m->stream));
    CK(cudaStreamSynchronize(m->stream));
    if (next_token) *next_token = *m->h_next;
    return B200_OK;
}

int b200_model_logits(b200_model* m, float* host, int64_t* offset, int64_t* count) {
    if (!m) return B200_EINVAL;
    if (offset) *offset = (int64_t)m->rank * m->voc;
    if (count) *count = m->voc;
    if (!host) return B200_OK;
    CK(cudaSetDevice(m->device));
    CK(cudaMemcpyAsync(host, m->logits, (size_t)m->voc * 4, cudaMemcpyDeviceToHost, m->stream));
    CK(cudaStreamSynchronize(m->stream));
    return B200_OK;
}

b200_stream_t b200_model_stream(b200_model* m) { return m ? (b200_stream_t)m->stream : nullptr; }

int b200_model_step_bytes(b200_model* m, int ctx, uint64_t* bytes) {
    if (!m || !bytes) return B200_EINVAL;
    const b200_llama_config& c = m->c;
    const int64_t D = c.head_dim;
    uint64_t b = 0;
    const uint64_t per_layer = (uint64_t)q4_bytes(m->qkv_rows, c.d_model) + q4_bytes(c.d_model, m->hq * D) +
                               2 * (uint64_t)q4_bytes(m->ff, c.d_model) + q4_bytes(c.d_model, m->ff) +
                               2ull * c.d_model * 4 + 2ull * (uint64_t)ctx * m->hkv * D * 2;
    b += per_layer * c.n_layer;
    b += (uint64_t)q4_bytes(m->voc, c.d_model) + (uint64_t)c.d_model * 4 + (uint64_t)(c.d_model / 32) * 18;
    *bytes = b;
    return B200_OK;
}

int b200_model_debug_step_ex(b200_model* m, int token, int pos, const b200_step_dump* hd) {
    if (!m || !hd || pos < 0 || pos >= m->c.kv_size || token < 0 || token >= m->c.vocab) return B200_EINVAL;
    CK(cudaSetDevice(m->device));
    CR(b200i_prepare_device());
    const b200_llama_config& c = m->c;
    const size_t L = (size_t)c.n_layer, d = (size_t)c.d_model, qd = (size_t)m->hq * c.head_dim,
                 kvd = (size_t)m->hkv * c.head_dim, ff = (size_t)m->ff;
    // (host pointer, device pointer slot, bytes) of every requested part
    struct Part {
        void* host;
        void** dev;
        size_t bytes;
    };
    Dump dd;
    dd.pos = pos;
    const Part parts[] = {
        {hd->x, (void**)&dd.x, (L + 1) * d * 4},
        {hd->x_mid, (void**)&dd.x_mid, L * d * 4},
        {hd->q, (void**)&dd.q, L * qd * 4},
        {hd->k_row, (void**)&dd.k_row, L * kvd * 2},
        {hd->v_row, (void**)&dd.v_row, L * kvd * 2},
        {hd->att, (void**)&dd.att, L * qd * 4},
        {hd->h, (void**)&dd.h, L * ff * 4},
        {hd->xq_qkv, (void**)&dd.xq_qkv, L * (d / 32) * 34},
        {hd->xq_o, (void**)&dd.xq_o, L * (qd / 32) * 34},
        {hd->xq_gu, (void**)&dd.xq_gu, L * (d / 32) * 34},
        {hd->xq_down, (void**)&dd.xq_down, L * (ff / 32) * 34},
        {hd->xq_head, (void**)&dd.xq_head, (d / 32) * 34},
        {hd->dots_qkv, (void**)&dd.dots_qkv, L * (size_t)m->qkv_rows * (d / 32) * 4},
        {hd->dots_o, (void**)&dd.dots_o, L * d * (qd / 32) * 4},
        {hd->dots_gu, (void**)&dd.dots_gu, L * 2 * ff * (d / 32) * 4},
        {hd->dots_down, (void**)&dd.dots_down, L * d * (ff / 32) * 4},
        {hd->dots_head, (void**)&dd.dots_head, (size_t)m->voc * (d / 32) * 4},
    };
    int rc = B200_OK;
    for (const Part& p : parts)
        if (rc == B200_OK && p.host != nullptr && cudaMalloc(p.dev, p.bytes) != cudaSuccess) {
            cudaGetLastError();
            rc = B200_ENOMEM;
        }
    if (rc == B200_OK) {
        m->h_st->token = token;
        m->h_st->pos = pos;
        m->h_st->ctx = pos + 1;
        m->h_st->advance = 0;
        if (cudaMemcpyAsync(m->st, m->h_st, 4 * sizeof(int), cudaMemcpyHostToDevice, m->stream) != cudaSuccess)
            rc = B200_ECUDA;
    }
    if (rc == B200_OK) rc = enqueue_step(m, m->stream, nullptr, &dd);
    if (rc == B200_OK && cudaStreamSynchronize(m->stream) != cudaSuccess) rc = B200_ECUDA;
    for (const Part& p : parts)
        if (rc == B200_OK && p.host != nullptr &&
            cudaMemcpy(p.host, *p.dev, p.bytes, cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = B200_ECUDA;
    if (rc == B200_OK && hd->logits != nullptr &&
        cudaMemcpy(hd->logits, m->logits, (size_t)m->voc * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = B200_ECUDA;
    for (const Part& p : parts)
        if (*p.dev != nullptr) cudaFree(*p.dev);
    return rc;
}

int b200_model_debug_step(b200_model* m, int token, int pos, float* x_host, float* q_host, float* att_host) {
    if (!x_host) return B200_EINVAL;
    b200_step_dump d;
    std::memset(&d, 0, sizeof(d));
    d.x = x_host;
    d.q = q_host;
    d.att = att_host;
    return b200_model_debug_step_ex(m, token, pos, &d);
}

int b200_model_profile(b200_model* m, int iters, float* us) {
    if (!m || !us || iters <= 0) return B200_EINVAL;
    CK(cudaSetDevice(m->device));
    CR(b200i_prepare_device());
    double acc[8] = {0};
    int cnt[8] = {0};
    for (int it = 0; it < iters; ++it) {
        Prof p;
        CR(enqueue_step(m, m->stream, &p));
        CK(cudaStreamSynchronize(m->stream));
        for (size_t i = 0; i < p.cls.size(); ++i) {
            float ms = 0.f;
            CK(cudaEventElapsedTime(&ms, p.ev[2 * i], p.ev[2 * i + 1]));
            acc[p.cls[i]] += ms * 1000.0;
            cnt[p.cls[i]] += 1;
        }
    }
    for (int i = 0; i < 8; ++i) us[i] = cnt[i] ? (float)(acc[i] / cnt[i]) : 0.f;
    return B200_OK;
}

int b200_model_timeline(b200_model* m, float* out17) {
    if (!m || !out17) return B200_EINVAL;
    CK(cudaSetDevice(m->device));
    CR(b200i_prepare_device());
    CK(cudaStreamSynchronize(m->stream));
    if (!m->tl_exec) {
        // every stamped kernel of a step: 5 per layer, 2 all-reduces per layer, the lm_head
        m->tl_n = 7 * m->c.n_layer + 1;
        if (cudaMalloc(reinterpret_cast<void**>(&m->tl_stamps), (size_t)9 * m->tl_n * sizeof(unsigned long long)) !=
            cudaSuccess) {
            cudaGetLastError();
            m->tl_stamps = nullptr;
            return B200_ENOMEM;
        }
        Stamps st;
        st.base = m->tl_stamps;
        st.n = m->tl_n;
        CK(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
        const int rc = enqueue_step(m, m->stream, nullptr, nullptr, &st);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(m->stream, &g);
        if (rc != B200_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        CK(e);
        m->tl_graph = g;
        CK(cudaGraphInstantiate(&m->tl_exec, g, 0));
        m->tl_cls = st.cls;
    }
    const int n = m->tl_n, used = (int)m->tl_cls.size();
    // min slots (entry, post-wait, earliest phase marks) start at ~0, max slots at 0
    CK(cudaMemsetAsync(m->tl_stamps, 0xFF, (size_t)2 * n * sizeof(unsigned long long), m->stream));
    CK(cudaMemsetAsync(m->tl_stamps + 2 * n, 0, (size_t)4 * n * sizeof(unsigned long long), m->stream));
    CK(cudaMemsetAsync(m->tl_stamps + 6 * n, 0xFF, (size_t)3 * n * sizeof(unsigned long long), m->stream));
    CK(cudaGraphLaunch(m->tl_exec, m->stream));
    std::vector<unsigned long long>& h = m->tl_host;
    h.assign((size_t)9 * n, 0);
    CK(cudaMemcpyAsync(h.data(), m->tl_stamps, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                       m->stream));
    CK(cudaStreamSynchronize(m->stream));
    double inc[8] = {0}, own[8] = {0};
    int cnt[8] = {0};
    unsigned long long prev = 0, first = 0;
    for (int i = 0; i < used; ++i) {
        const unsigned long long e = h[i], w = h[n + i], x = h[2 * n + i];
        if (x == 0 || w == ~0ull) continue;  // a kernel that stamped nothing
        if (prev == 0) prev = first = w;     // the step starts when the first stamped kernel may run
        const int c = m->tl_cls[i];
        inc[c] += (double)(x > prev ? x - prev : 0) * 1e-3;
        own[c] += (double)(x > w ? x - w : 0) * 1e-3;
        cnt[c] += 1;
        prev = x > prev ? x : prev;
        (void)e;
    }
    for (int c = 0; c < 8; ++c) {
        out17[c] = (float)inc[c];
        out17[8 + c] = cnt[c] ? (float)(own[c] / cnt[c]) : 0.f;
    }
    out17[16] = (float)((double)(prev - first) * 1e-3);
    return B200_OK;
}

int b200_model_timeline_phases(b200_model* m, float* out64) {
    if (!m || !out64) return B200_EINVAL;
    const int n = m->tl_n, used = (int)m->tl_cls.size();
    if (m->tl_host.size() != (size_t)9 * n || n == 0) return B200_EINVAL;  // no timeline step yet
    const std::vector<unsigned long long>& h = m->tl_host;
    double sum[8][8] = {};
    int cnt[8][8] = {};
    for (int i = 0; i < used; ++i) {
        const unsigned long long e = h[i], w = h[n + i], x = h[2 * n + i];
        if (x == 0 || w == ~0ull || e == ~0ull) continue;
        const int c = m->tl_cls[i];
        auto add = [&](int j, unsigned long long t, unsigned long long from, bool valid) {
            if (!valid) return;
            sum[c][j] += (double)((long long)t - (long long)from) * 1e-3;
            cnt[c][j] += 1;
        };
        add(0, w, e, true);
        for (int k = 0; k < 3; ++k) {
            const unsigned long long hi = h[(size_t)(3 + k) * n + i], lo = h[(size_t)(6 + k) * n + i];
            add(1 + k, hi, w, hi != 0);
            add(5 + k, lo, w, lo != ~0ull);
        }
        add(4, x, w, true);
    }
    for (int c = 0; c < 8; ++c)
        for (int j = 0; j < 8; ++j) out64[c * 8 + j] = cnt[c][j] ? (float)(sum[c][j] / cnt[c][j]) : 0.f;
    return B200_OK;
}

int b200_model_time_gate_up(b200_model* m, int iters, float* us_per_launch) {
    if (!m || !us_per_launch || iters <= 0) return B200_EINVAL;
    CK(cudaSetDevice(m->device));
    CR(b200i_prepare_device());
    CK(cudaStreamSynchronize(m->stream));
    m->ar_now = false;  // the launches read x as it is
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int rc = B200_OK;
    for (int l = 0; l < m->c.n_layer && rc == B200_OK; ++l)
        rc = b200i_gemv(FMT_Q4, gate_up_args(m, l), false, m->stream, m->pdl);
    const cudaError_t ec = cudaStreamEndCapture(m->stream, &g);
    if (rc != B200_OK || ec != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return rc != B200_OK ? rc : B200_ECUDA;
    }
    cudaGraphExec_t ge = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    for (int w = 0; w < 2 && e == cudaSuccess; ++w) e = cudaGraphLaunch(ge, m->stream);  // warm-up
    if (e == cudaSuccess) e = cudaEventRecord(e0, m->stream);
    for (int i = 0; i < iters && e == cudaSuccess; ++i) e = cudaGraphLaunch(ge, m->stream);
    if (e == cudaSuccess) e = cudaEventRecord(e1, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (ge) cudaGraphExecDestroy(ge);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return B200_ECUDA;
    *us_per_launch = ms * 1000.f / (float)(iters * m->c.n_layer);
    return B200_OK;
}

}  // extern "C"
