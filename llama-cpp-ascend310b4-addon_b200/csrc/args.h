// args.h -- kernel argument blocks and launch plans shared by the device
// code (kernels.cu) and the host-side runtime (graph runner, decode driver).
// No device code here, so any translation unit may include it.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "../../include/b200_decode.h"

#if defined(__CUDACC__)
#define B200_HD __host__ __device__
#else
#define B200_HD
#endif

namespace b200 {

enum GemvFmt { FMT_F16 = 0, FMT_Q4 = 1, FMT_Q4W = 2, FMT_Q8 = 3 };
enum GemvPro { PRO_PLAIN = 0, PRO_RMSNORM = 1 };
enum GemvEpi { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_QKV = 3, EPI_ARGMAX = 4 };

constexpr int kGemvThreads = 256;
constexpr int64_t kTileTarget = 32768;  // preferred tile bytes
constexpr int64_t kTileMax = 65536;     // largest tile one stage may hold
constexpr int kMaxR = 32;
constexpr int kMaxSlots = 8;            // kGemvThreads / 32

struct GemvPlan {
    int type;
    int64_t n, k;
    int U;             // units per row: 8 halves (F16) or one 32-block (Q4_0/Q8_0)
    int64_t rowbytes;  // packed bytes per row
    int R;             // rows per tile
    int64_t tile_bytes;
    int64_t ntiles;
};

B200_HD inline int64_t pad16(int64_t v) { return (v + 15) & ~int64_t(15); }

B200_HD inline bool make_plan(int type, int64_t n, int64_t k, GemvPlan* p) {
    if (n <= 0 || k <= 0) return false;
    p->type = type;
    p->n = n;
    p->k = k;
    if (type == B200_TYPE_F16) {
        if (k % 8) return false;
        p->U = (int)(k / 8);
        p->rowbytes = 2 * k;
    } else if (type == B200_TYPE_Q4_0) {
        if (k % 32) return false;
        p->U = (int)(k / 32);
        p->rowbytes = k / 2 + k / 16;
    } else if (type == B200_TYPE_Q8_0) {
        if (k % 32) return false;
        p->U = (int)(k / 32);
        p->rowbytes = k + k / 16;
    } else {
        return false;
    }
    int R = kMaxR;
    while (R > 1 && R * p->rowbytes > kTileTarget) R >>= 1;
    p->R = R;
    p->tile_bytes = pad16(R * p->rowbytes);
    if (p->tile_bytes > kTileMax) return false;
    p->ntiles = (n + R - 1) / R;
    return true;
}

struct GemvArgs {
    const uint8_t* w;
    int64_t tile_bytes, ntiles;
    int R, RG, U, stages;
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
};

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
};

}  // namespace b200
