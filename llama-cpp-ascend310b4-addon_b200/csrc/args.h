// args.h -- kernel argument blocks and launch plans shared by the device
// code (kernels.cu) and the host-side runtime (graph runner, decode driver).
// No device code here, so any translation unit may include it.
#pragma once

#include <cuda.h>  // CUtensorMap (a plain 128-byte descriptor type)
#include <stddef.h>
#include <stdint.h>

#include "../../include/b200_decode.h"

#if defined(__CUDACC__)
#define B200_HD __host__ __device__
#else
#define B200_HD
#endif

namespace b200 {

enum GemvFmt { FMT_F16 = 0, FMT_Q4 = 1, FMT_Q4W = 2, FMT_Q8 = 3, FMT_A8 = 4 };
enum GemvPro { PRO_PLAIN = 0, PRO_RMSNORM = 1 };
enum GemvEpi { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_QKV = 3, EPI_ARGMAX = 4, EPI_PUSH = 5 };

constexpr int kMaxRanks = 8;      // tensor-parallel ranks of one node
constexpr int kArMaxCtas = 256;   // flag slots per source rank of the fused all-reduce
struct StepState;

constexpr int kGemvWarps = 16;              // warps per CTA; each runs its own copy ring
constexpr int kGemvThreads = 32 * kGemvWarps;
constexpr int kGemvStagesMax = 4;           // copy-ring depth per warp
constexpr int64_t kGemvSmemBudget = 200 * 1024;

// Packed layout: rows are contiguous, row r at r * rs.  Inside a row:
//   F16 : K halves                                       rs = 2K
//   Q4_0: qs[U][16 bytes], then d[U] f16 padded to 16     rs = 16U + pad16(2U)
//   Q8_0: qs bytes 0..15 [U][16], bytes 16..31 [U][16],
//         then d[U] f16 padded to 16                      rs = 32U + pad16(2U)
//   A8W8: int8 bytes 0..15 [U][16], bytes 16..31 [U][16]  rs = 32U, then one f16
//         scale per row after all n rows (padded to 16)
// (U = K/8 units of 8 halves for F16, K/32 blocks for Q4_0/Q8_0.)  Planes
// are split so that 32 lanes reading consecutive units issue conflict-free
// 16-byte shared-memory loads, and every plane start is 16-byte aligned for
// the bulk copies.
//
// A warp streams its rows in chunks: a chunk is either units [u0, u0+kc) of
// one row (rpc == 1; one bulk copy per plane) or rpc whole consecutive rows
// when rows are short (one bulk copy).  Inside a staged chunk, unit i of a
// row sits at 16 i in plane 0, 16 pw + 16 i in plane 1 (Q8_0), and the scale
// at (Q8_0: 32 pw, Q4_0: 16 pw) + 2 i, where pw = kc (rpc == 1) or U.
struct GemvPlan {
    int type;
    int64_t n, k;
    int U;              // units per row
    int ub;             // bytes per unit (16, 18, 34)
    int64_t rs;         // packed row stride
    int rpc;            // rows per chunk
    int kc;             // units per chunk row (== U when rpc > 1)
    int nchunk;         // chunks per row (1 when rpc > 1)
    int tpr;            // lanes per row (32 / rpc)
    int tpr_log2;
    int upl;            // units per lane per chunk row
    int full_upl;       // units per lane of a full chunk (rpc == 1 and kc % 32 == 0), else 0
    int64_t stage_bytes;
};

B200_HD inline int64_t pad16(int64_t v) { return (v + 15) & ~int64_t(15); }

B200_HD inline int64_t gemv_stage_bytes_rpc1(int type, int kc) {
    if (type == B200_TYPE_F16) return 16 * (int64_t)kc;
    if (type == B200_TYPE_A8W8) return 32 * (int64_t)kc;
    if (type == B200_TYPE_Q4_0) return 16 * (int64_t)kc + pad16(2 * (int64_t)kc);
    return 32 * (int64_t)kc + pad16(2 * (int64_t)kc);
}

B200_HD inline bool make_plan(int type, int64_t n, int64_t k, GemvPlan* p) {
    if (n <= 0 || k <= 0) return false;
    p->type = type;
    p->n = n;
    p->k = k;
    int kc_max;
    if (type == B200_TYPE_F16) {
        if (k % 8) return false;
        p->U = (int)(k / 8);
        p->ub = 16;
        p->rs = 2 * k;
        kc_max = 256;
    } else if (type == B200_TYPE_Q4_0) {
        if (k % 32) return false;
        p->U = (int)(k / 32);
        p->ub = 18;
        p->rs = 16 * (int64_t)p->U + pad16(2 * (int64_t)p->U);
        kc_max = 256;
    } else if (type == B200_TYPE_Q8_0) {
        if (k % 32) return false;
        p->U = (int)(k / 32);
        p->ub = 34;
        p->rs = 32 * (int64_t)p->U + pad16(2 * (int64_t)p->U);
        kc_max = 128;
    } else if (type == B200_TYPE_A8W8) {
        if (k % 32 || k > 131072) return false;  // |int32 row sum| <= k * 127^2
        p->U = (int)(k / 32);
        p->ub = 32;
        p->rs = 32 * (int64_t)p->U;  // int8 bytes 0..15 [U][16], bytes 16..31 [U][16]; row scales after all rows
        kc_max = 128;
    } else {
        return false;
    }
    if (k > (int64_t)1 << 24) return false;
    const int U = p->U;
    if (U >= 64) {
        p->rpc = 1;
        p->tpr = 32;
        p->tpr_log2 = 5;
        // Chunk width: a multiple of 32 (every full chunk gives each lane the
        // same number of units; the scale plane stays 16-byte aligned);
        // prefer the widest one that divides the row, so that no row ends in
        // a partial chunk.  Otherwise: the row in equal chunks, rounded up to
        // a multiple of 64.
        int kc = 0;
        for (int c = kc_max; c >= 64; c -= 32)
            if (U % c == 0) {
                kc = c;
                break;
            }
        if (kc == 0) {
            const int nch = (U + kc_max - 1) / kc_max;
            kc = (((U + nch - 1) / nch) + 63) & ~63;
            if (kc > kc_max) kc = kc_max;
        }
        p->kc = kc;
        p->nchunk = (U + kc - 1) / kc;
        p->upl = (kc + 31) / 32;
        p->full_upl = (kc % 32 == 0) ? kc / 32 : 0;
        p->stage_bytes = gemv_stage_bytes_rpc1(type, kc);
    } else {
        int rpc = 32;
        while (rpc > 1 && rpc * U > 128) rpc >>= 1;
        p->rpc = rpc;
        p->tpr = 32 / rpc;
        p->tpr_log2 = 0;
        while ((1 << p->tpr_log2) < p->tpr) ++p->tpr_log2;
        p->kc = U;
        p->nchunk = 1;
        p->upl = (U + p->tpr - 1) / p->tpr;
        p->full_upl = 0;
        p->stage_bytes = rpc * p->rs;
    }
    return true;
}

B200_HD inline int64_t gemv_packed_bytes(const GemvPlan& p) {
    return p.n * p.rs + (p.type == B200_TYPE_A8W8 ? pad16(2 * p.n) : 0);
}

struct GemvArgs {
    const uint8_t* w;
    GemvPlan p;
    int stages;
    int64_t n, k;
    // prologue
    const float* x;
    const float* norm_w;
    float eps;
    int pro;
    // epilogue
    int epi;
    float* y;
    const float* res;
    int nq, nkv, head_dim;        // EPI_QKV: rows [0,nq) q, [nq,nq+nkv) k, then v
    const int* pos;               // EPI_QKV: device position
    float theta_scale;            // EPI_QKV: powf(theta_base, -2/head_dim)
    uint16_t* kc;                 // EPI_QKV: K cache row 0 ([kv_size][nkv] f16)
    uint16_t* vc;
    unsigned long long* amax;     // EPI_ARGMAX: packed (value, index) maximum
    int64_t row_offset;           // EPI_ARGMAX: global index of local row 0
    // exactness exports
    int32_t* dots;                // [n][U] int32 block dots (Q formats, DEBUG kernels)
    uint8_t* xq_out;              // Q8_0 blocks of the quantised activation (CTA 0)
    // Quantised-activation images (Q4_0 / Q8_0 weights).  An image holds the
    // Q8_0 activation in the prologue's shared-memory layout, 40 U bytes:
    // words [U][4] of q bytes 0..15, words [U][4] of bytes 16..31, then
    // {d as f32, sum of q}[U].
    const uint8_t* xq_in;         // set: the prologue copies this image instead of quantising x
    uint8_t* xq_img;              // EPI_SWIGLU (rpc == 1): also quantise the output into this image
                                  // (the 32-blocks each CTA owns whole; see xq_fix_*)
    // With xq_in: the image's blocks that span two CTAs of its SwiGLU
    // producer (a grid of xq_fix_grid CTAs over xq_fix_items outputs) are
    // quantised in this prologue from the producer's f32 output xq_fix_h;
    // CTA 0 writes them to xq_fix_out (the image) as well.
    const float* xq_fix_h;
    uint8_t* xq_fix_out;
    int64_t xq_fix_items;
    int xq_fix_grid;
    // Fused tensor-parallel all-reduce of a row-split projection's partial
    // (collective number seq = step x ar_per_step + ar_idx + 1).
    //   EPI_PUSH (producer): row n's partial (+ res[n] when res is set) goes
    //   to ar_dst[r][n] on every rank r; then every CTA releases seq into
    //   ar_flag_dst[r][blockIdx.x] on every rank.
    //   Prologue (consumer, ar_src set): waits until ar_flags[r][c] >= seq
    //   for every rank r and producer CTA c < ar_grid, sums the ranks'
    //   partials ar_src + r ar_stride in rank order as x, and CTA 0 writes
    //   that sum to ar_x_out.
    float* ar_dst[kMaxRanks];
    unsigned long long* ar_flag_dst[kMaxRanks];
    const float* ar_src;
    unsigned long long* ar_flags;  // [kMaxRanks][kArMaxCtas]
    float* ar_x_out;
    int64_t ar_stride;             // floats between two ranks' slots
    int ar_world, ar_grid, ar_idx, ar_per_step;
    const StepState* ar_st;
    // Timeline stamps (globaltimer ns), when set: [0] earliest CTA entry,
    // [n] earliest return from griddepcontrol.wait, [2n] latest CTA exit,
    // [3n..5n] latest and [6n..8n] earliest CTA at the phase marks (input
    // ready, first chunk landed, main loop done), n = stamp_stride
    // (atomicMin / atomicMax by one thread per CTA).
    unsigned long long* stamp;
    int stamp_stride;
    // The weight stream is read with the evict_first L2 policy when set
    // (weights are read once per step).
    int l2_ef;
    // Uneven rows (rpc == 1): the last late_ctas CTAs of the grid get
    // late_pct % of an even share, the others the rest.  For a GEMV that
    // follows a kernel holding late_ctas SMs: under programmatic launch the
    // low-numbered CTAs become resident on the free SMs first and start
    // streaming as soon as the wait ends, the last ones only once the
    // previous kernel's CTAs have left their SMs (gemv_cta_start).
    int late_ctas;
    int late_pct;
};

// First item of CTA c of `grid` over `items` (see GemvArgs::late_ctas);
// an even split when late is 0 or not below grid.
B200_HD inline int64_t gemv_cta_start(int64_t c, int64_t grid, int64_t items, int64_t late, int64_t pct) {
    if (late <= 0 || late >= grid || pct <= 0 || pct >= 100) return c * items / grid;
    const int64_t early = grid - late;
    const int64_t total = 100 * early + pct * late;
    const int64_t w = c <= early ? 100 * c : 100 * early + pct * (c - early);
    return w * items / total;
}

constexpr int kFaThreads = 128;
constexpr int kFaChunk = 64;    // positions per inner step
constexpr int kFaMaxG = 8;      // query heads per CTA
constexpr int kFaTargetCtas = 296;

struct FaArgs {
    const float* q;
    const uint8_t* k;
    const uint8_t* v;
    const uint16_t* mask;
    const int32_t* kv_len;
    float* out;
    int Hq, Hkv, G, gchunks, n_kv, n_splits, chunks_per_split;
    int64_t k_nb1, k_nb2, v_nb1, v_nb2;
    float scale;
    float* part_o;          // [n_splits][Hq][D]
    float* part_ml;         // [n_splits][Hq][2]
    unsigned int* tickets;  // [Hkv][gchunks]
    // Tensor-core kernel: when set, the output is also quantised (Q8_0 over
    // blocks of 32 of the flat [Hq][D] vector) into this activation image of
    // xq_U = Hq D / 32 blocks, the layout of GemvArgs::xq_in.
    uint8_t* xq_img;
    int xq_U;
    // TMA descriptors of K and V ([head_dim, Hkv, n_kv], 64 x 1 x 64 boxes,
    // 128-byte swizzle), filled by the launcher of the tensor-core kernel.
    CUtensorMap tmk, tmv;
    unsigned long long* stamp;  // timeline stamps as GemvArgs::stamp
    int stamp_stride;
    // Tensor-core kernel: K and V are read with the evict_first L2 policy
    // when set (as GemvArgs::l2_ef).
    int l2_ef;
};

// Small-M F16 matmul (gemm_small.cuh).
struct SmallMArgs {
    CUtensorMap tmw;      // weight [n rows][k halves]: 64 x 16 boxes, 128-byte swizzle
    const float* x;       // [m][ldx] f32
    float* y;             // [m][ldy] f32
    int64_t n, k, ldx, ldy;
    int64_t xstride;      // halves per activation row in shared memory
    int m, stages;
    int xvec;             // x rows 16-byte aligned: load them as float4
};

struct FaLayout {
    int n_splits, chunks_per_split, gchunks;
    size_t off_o, off_ml, off_tickets, total;
};

B200_HD inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

B200_HD inline FaLayout fa_layout(int D, int Hq, int Hkv, int n_kv) {
    FaLayout L;
    const int G = Hq / Hkv;
    L.gchunks = (G + kFaMaxG - 1) / kFaMaxG;
    const int nchunks = (n_kv + kFaChunk - 1) / kFaChunk;
    int want = (kFaTargetCtas + Hkv * L.gchunks - 1) / (Hkv * L.gchunks);
    if (want < 1) want = 1;
    if (want > nchunks) want = nchunks;
    L.chunks_per_split = (nchunks + want - 1) / want;
    L.n_splits = (nchunks + L.chunks_per_split - 1) / L.chunks_per_split;
    L.off_o = 0;
    L.off_ml = align256((size_t)L.n_splits * Hq * D * sizeof(float));
    L.off_tickets = L.off_ml + align256((size_t)L.n_splits * Hq * 2 * sizeof(float));
    L.total = L.off_tickets + align256((size_t)Hkv * L.gchunks * sizeof(unsigned int));
    return L;
}


// Per-step device state of the captured decode graph.
struct StepState {
    int token;                // input token of this step
    int pos;                  // its position
    int ctx;                  // pos + 1: number of valid KV rows (attention kv_len)
    int advance;              // 1: the step feeds its argmax back and pos += 1
    int next;                 // argmax token of this step
    int pad_;
    unsigned long long amax;  // packed (value, index) argmax of the logits
    unsigned long long step;  // steps run so far (set by the embedding kernel; numbers the collectives)
};

// Tensor-parallel all-reduce over peer memory (one-shot): every rank sums
// all ranks' partial vectors for collective `idx` of the current step.
struct ArArgs {
    int world, rank, n;        // ranks, this rank, floats per vector (multiple of 4)
    int idx, per_step;         // collective index within the step, collectives per step
    const StepState* st;       // null: the collective's number is `seq`
    unsigned long long seq;
    float* x;                  // result [n] on this rank
    const float* part[kMaxRanks];                  // rank r's partial [n] (peer mapped)
    unsigned long long* flags;                      // this rank's flags [kMaxRanks]: flags[r] = last seq rank r announced
    unsigned long long* peer_flag[kMaxRanks];       // &flags of rank r [this rank]
    unsigned long long* stamp;                      // timeline stamps as GemvArgs::stamp
    int stamp_stride;
};

}  // namespace b200
