// fa_mma.cuh -- single-token GQA flash-decoding on tensor cores (head_dim 64
// and 128).
//
// Grid (split, kv head, q-head chunk), G = 2 or 3 groups of 4 warps.  mma.sync
// m16n8k16 with the positions as the 16-row A side and the query heads of one
// GQA group (up to 8) as the n = 8 side, so every row of every mma is used and
// each K/V tile is read from HBM once for the whole group:
//   S^T = K Q^T : A = 16 positions x 16 dims of K by ldmatrix from an
//                 XOR-swizzled shared-memory stage, B = f16(q) (registers for
//                 the whole split);
//   O^T += V^T P^T : A = V^T by ldmatrix.trans, B = P^T, moved from the S^T
//                 accumulator layout by movmatrix.  P is split into an f16
//                 high part and an f16 residual so the product keeps ~22 bits.
// Each thread keeps the online-softmax state (max, sum) of two heads over its
// warp's 16 positions.  K/V chunks of 64 positions arrive by TMA (a 3-D tensor
// map over [head_dim, kv head, position]; boxes of 64 positions x 64 dims with
// the 128-byte swizzle) into per-group mbarrier rings; V rows past the context
// are zeroed in shared memory.  The groups walk every G-th chunk of the split,
// each with its own ring and named barrier (3 groups x 2 stages when a CTA has
// 6 or more chunks, else 2 x 3), so G independent load/mma/softmax chains run
// per SM; the warps are combined in shared memory.  The splits of one (kv
// head, head chunk) form one thread-block cluster: every CTA stores its
// partial of each slice of the outputs into the shared memory of the CTA that
// owns the slice (distributed shared memory), and after one cluster barrier
// the owners merge locally, so partials never leave the SMs.
#pragma once

#include <cooperative_groups.h>

#include "args.h"
#include "common.cuh"

namespace b200 {

namespace cgx = cooperative_groups;

// Warp groups per CTA (each walks every G-th chunk of the split with its own
// ring) and ring stages per group: 3 x 2 when a CTA has at least 6 chunks,
// else 2 x 3 (both 6 stages of shared memory).
B200_HD constexpr int fm_stages(int groups) { return groups == 3 ? 2 : 3; }
B200_HD constexpr int fm_threads(int groups) { return 128 * groups; }
constexpr int kFmMaxThreads = fm_threads(3);

// Barrier of one 128-thread warp group (ids 1.. ; 0 is __syncthreads).
__device__ __forceinline__ void group_sync(int grp) { asm volatile("bar.sync %0, 128;" ::"r"(grp + 1) : "memory"); }

__device__ __forceinline__ void mma_16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t r[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t r[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// 3-D tiled TMA load of one box into this CTA's shared memory; completion
// is counted on `bar`; `pol` is the L2 policy (l2_policy).  x (the head_dim
// coordinate) is a multiple of 64 halves, so its byte offset is 16-byte
// aligned.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int x, int y, int z, uint64_t* bar,
                                            uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%2, %3, %4}], [%5], %6;" ::"r"(dst),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// Transpose of an 8 x 8 b16 matrix held one row pair per lane (lane g*4+t
// holds row g, columns 2t, 2t+1) into the same layout.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Shared memory of fa_mma_kernel<D, G>: per warp group fm_stages(G) x (K tile + V
// tile) of kFaChunk rows x D halves, sized for the six stage slots that both
// variants hold (3 x 2, 2 x 3); reused after the loop for the warp combine
// (at most 12 warps x kFaMaxG rows of D + 8 floats, a bound on the padded
// rows used, plus the CTA partial, kFaMaxG x D floats).
constexpr int kFmMaxCluster = 16;
B200_HD inline size_t fa_mma_smem_bytes(int D) {
    const size_t ring = (size_t)6 * 2 * kFaChunk * D * 2 + 1024;  // groups x stages = 6; + alignment of the TMA boxes
    const size_t merge = ((size_t)4 * 3 * kFaMaxG * (D + 8) + (size_t)kFaMaxG * D) * sizeof(float);
    return ring > merge ? ring : merge;
}

template <int D, int G>
__global__ void __launch_bounds__(fm_threads(G)) fa_mma_kernel(const __grid_constant__ FaArgs a) {
    constexpr int kFmGroups = G;
    constexpr int kFmStages = fm_stages(G);
    constexpr int kFmThreads = fm_threads(G);
    constexpr int KT = D / 16;       // k tiles of the QK^T product
    constexpr int GR = D / 8;        // 16-byte granules per K/V row
    constexpr int BOXB = kFaChunk * 128;  // one TMA box: 64 positions x 64 halves
    constexpr int NB = D / 64;            // boxes per K (or V) tile
    constexpr int TILE = NB * BOXB;       // K (or V) tile of one chunk
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NW = 4 * kFmGroups;  // warps per CTA
    __shared__ float wm[NW][kFaMaxG], wl[NW][kFaMaxG];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = warp >> 2, gw = warp & 3, gtid = tid & 127;  // warp group, warp and thread in it
    if (tid == 0) stamp_point(a.stamp, a.stamp_stride, 0);
    const int g = lane >> 2, t = lane & 3;
    const int split = blockIdx.x, hk = blockIdx.y, gc = blockIdx.z;
    const int h0 = hk * a.G + gc * kFaMaxG;
    const int hn = min(kFaMaxG, a.G - gc * kFaMaxG);

    // The context length and every K/V row but the newest (position
    // ctx - 1, written by this step's QKV projection) come from earlier
    // steps, so under a programmatic launch the first copies of chunks
    // before the newest row start ahead of griddep_wait; q, the newest row
    // and the mask are read after it.
    int ctx = a.n_kv;
    if (a.kv_len != nullptr) {
        const int kl = a.kv_len[0];
        if (kl > 0 && kl < a.n_kv) ctx = kl;
    }
    const int nchunks_ctx = (ctx + kFaChunk - 1) / kFaChunk;
    const int c_begin = split * a.chunks_per_split;
    const int c_end = min(c_begin + a.chunks_per_split, nchunks_ctx);
    const bool active = c_begin < c_end;
    const uint32_t sbase = (smem_u32(smem) + 1023u) & ~1023u;  // TMA 128-byte swizzle: 1 KiB aligned boxes
    __shared__ __align__(8) uint64_t fbar[kFmGroups][kFmStages];
    __shared__ int fabort[kFmGroups];

    // online-softmax state of heads 2t and 2t + 1 over this warp's positions
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    constexpr int MT = D / 16;  // 16-dim tiles of the output
    float o[MT][4];             // O^T tile mt: (dim 16 mt + g, heads 2t, 2t+1), (dim + 8, same heads)
#pragma unroll
    for (int n = 0; n < MT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

    // this group's chunks: c_begin + grp + kFmGroups * i, i < ncg
    const int ncg = active ? (c_end - c_begin - grp + kFmGroups - 1) / kFmGroups : 0;
    const uint64_t pol = l2_policy(a.l2_ef != 0);
    if (ncg <= 0) {
        griddep_wait();
        griddep_launch_dependents();
        if (gtid == 0) stamp_point(a.stamp, a.stamp_stride, 1);
    }
    if (ncg > 0) {
        const uint32_t gbase = sbase + (uint32_t)(grp * kFmStages * 2 * TILE);
        uint64_t* bars = fbar[grp];
        const int cfirst = c_begin + grp;
        // chunk ci of this group -> stage ci % kFmStages; one thread issues
        auto issue = [&](int ci) {
            const int st = ci % kFmStages;
            const int p0 = (cfirst + kFmGroups * ci) * kFaChunk;
            const uint32_t kdst = gbase + (uint32_t)(st * 2 * TILE);
            mbar_arrive_expect_tx(&bars[st], 2 * TILE);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                tma_load_3d(kdst + b * BOXB, &a.tmk, 64 * b, hk, p0, &bars[st], pol);
                tma_load_3d(kdst + TILE + b * BOXB, &a.tmv, 64 * b, hk, p0, &bars[st], pol);
            }
        };
        const int c_new = (ctx - 1) / kFaChunk;  // the chunk holding the newest row
        if (gtid == 0) {
            for (int st = 0; st < kFmStages; ++st) mbar_init(&bars[st], 1);
            mbar_fence_init();
            fabort[grp] = 0;
            int ci = 0;
            for (; ci < ncg && ci < kFmStages && cfirst + kFmGroups * ci < c_new; ++ci) issue(ci);
            griddep_wait();
            for (; ci < ncg && ci < kFmStages; ++ci) issue(ci);
        }
        griddep_wait();
        griddep_launch_dependents();
        if (gtid == 0) stamp_point(a.stamp, a.stamp_stride, 1);

        // Q fragments (the B operand: k = dims, n = heads; heads past the
        // group are zero), loaded while the first K/V copies are in flight
        uint32_t qa[KT][2];
        {
            const bool hv = g < hn;
            const float* qr = a.q + (int64_t)(h0 + (hv ? g : 0)) * D;
#pragma unroll
            for (int kt = 0; kt < KT; ++kt) {
                const float2 x0 = *reinterpret_cast<const float2*>(qr + 16 * kt + 2 * t);
                const float2 x1 = *reinterpret_cast<const float2*>(qr + 16 * kt + 2 * t + 8);
                qa[kt][0] = hv ? pack_half2(x0.x, x0.y) : 0u;
                qa[kt][1] = hv ? pack_half2(x1.x, x1.y) : 0u;
            }
        }
        group_sync(grp);  // barrier init visible to the group
        if (tid == 0) stamp_point(a.stamp, a.stamp_stride, 3);

        int ci = 0;
        for (; ci < ncg; ++ci) {
            const int c = cfirst + kFmGroups * ci;
            const int stage = ci % kFmStages;
            if (!mbar_wait_bounded(&bars[stage], (uint32_t)((ci / kFmStages) & 1))) fabort[grp] = 1;
            if (ci == 0 && tid == 0) stamp_point(a.stamp, a.stamp_stride, 4);
            // V rows at or past the context hold no cache data: zero them
            const int valid = ctx - c * kFaChunk;
            if (valid < kFaChunk) {
                const uint32_t vz = gbase + (uint32_t)(stage * 2 * TILE + TILE);
                const int r0 = valid > 0 ? valid : 0;
                for (int u = gtid; u < (kFaChunk - r0) * NB * 8; u += 128) {
                    const int row = r0 + u / (NB * 8), rem = u - (u / (NB * 8)) * (NB * 8);
                    const uint32_t addr = vz + (uint32_t)((rem >> 3) * BOXB + row * 128 + ((rem & 7) << 4));
                    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u) : "memory");
                }
            }
            group_sync(grp);  // chunk c is in shared memory for every warp of the group
            if (fabort[grp]) break;

            const uint32_t kst = gbase + (uint32_t)(stage * 2 * TILE);
            const uint32_t vst = kst + TILE;
            const int pw = 16 * gw;  // this warp's 16 positions in the chunk
            // ---- S^T = K Q^T: A = 16 positions x 16 dims of K, B = Q^T ----
            float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};  // even / odd k tiles
            {
                const int mi = lane >> 3, ri = lane & 7;
                const int j = mi >> 1, hh = mi & 1;
                const int r = pw + 8 * j + ri;
#pragma unroll
                for (int kt = 0; kt < KT; ++kt) {
                    uint32_t b[4];  // (pos 0-7, k 0-7), (pos 0-7, k 8-15), (pos 8-15, k 0-7), (pos 8-15, k 8-15)
                    const int gk = 2 * kt + hh;  // 16-byte granule of the row
                    ldsm_x4(b, kst + (uint32_t)((gk >> 3) * BOXB + r * 128 + (((gk & 7) ^ ri) << 4)));
                    const uint32_t af[4] = {b[0], b[2], b[1], b[3]};
                    mma_16816((kt & 1) ? sb : sa, af, qa[kt][0], qa[kt][1]);
                }
            }
            // ---- scale, mask, online softmax; this thread: positions g and g + 8
            // of its warp, heads 2t (values 0, 2) and 2t + 1 (values 1, 3) ----
            const int pbase = c * kFaChunk + pw;
            float sv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int p = pbase + g + (e >= 2 ? 8 : 0);
                float mv = 0.f;
                if (a.mask != nullptr && p < ctx) mv = h2f(a.mask[p]);
                const float sc = sa[e] + sb[e];
                sv[e] = (p < ctx && mv != -INFINITY) ? __fadd_rn(__fmul_rn(sc, a.scale), mv) : -INFINITY;
            }
            float pv[4];
            float alpha[2];
#pragma unroll
            for (int hh2 = 0; hh2 < 2; ++hh2) {
                float cmax = fmaxf(sv[hh2], sv[hh2 + 2]);
                cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 4));
                cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 8));
                cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 16));
                const float m_new = fmaxf(m_run[hh2], cmax);
                alpha[hh2] = 1.f;
                if (m_new == -INFINITY) {
                    pv[hh2] = pv[hh2 + 2] = 0.f;
                } else {
                    alpha[hh2] = m_run[hh2] == -INFINITY ? 0.f : expf(m_run[hh2] - m_new);
                    pv[hh2] = sv[hh2] == -INFINITY ? 0.f : expf(sv[hh2] - m_new);
                    pv[hh2 + 2] = sv[hh2 + 2] == -INFINITY ? 0.f : expf(sv[hh2 + 2] - m_new);
                }
                float psum = pv[hh2] + pv[hh2 + 2];
                psum += __shfl_xor_sync(0xffffffffu, psum, 4);
                psum += __shfl_xor_sync(0xffffffffu, psum, 8);
                psum += __shfl_xor_sync(0xffffffffu, psum, 16);
                l_run[hh2] = l_run[hh2] * alpha[hh2] + psum;
                m_run[hh2] = m_new;
            }
#pragma unroll
            for (int n = 0; n < MT; ++n) {
                o[n][0] *= alpha[0];
                o[n][1] *= alpha[1];
                o[n][2] *= alpha[0];
                o[n][3] *= alpha[1];
            }
            // ---- O^T += V^T P^T, P = P_hi + P_lo in f16; P^T's B fragments by
            // movmatrix from the S^T accumulator layout ----
            const uint32_t hi0 = pack_half2(pv[0], pv[1]), hi1 = pack_half2(pv[2], pv[3]);
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&hi0));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&hi1));
            const uint32_t lo0 = pack_half2(pv[0] - f0.x, pv[1] - f0.y), lo1 = pack_half2(pv[2] - f1.x, pv[3] - f1.y);
            const uint32_t bh0 = movmatrix_trans(hi0), bh1 = movmatrix_trans(hi1);
            const uint32_t bl0 = movmatrix_trans(lo0), bl1 = movmatrix_trans(lo1);
            {
                const int mi = lane >> 3, ri = lane & 7;
                const int ph = mi & 1, jn = mi >> 1;
                const int r = pw + 8 * ph + ri;
#pragma unroll
                for (int jj = 0; jj < MT; ++jj) {
                    uint32_t b[4];  // transposed: (d 0-7, p 0-7), (d 0-7, p 8-15), (d 8-15, p 0-7), (d 8-15, p 8-15)
                    const int gv = 2 * jj + jn;
                    ldsm_x4_trans(b, vst + (uint32_t)((gv >> 3) * BOXB + r * 128 + (((gv & 7) ^ ri) << 4)));
                    const uint32_t av[4] = {b[0], b[2], b[1], b[3]};
                    mma_16816(o[jj], av, bh0, bh1);
                    mma_16816(o[jj], av, bl0, bl1);
                }
            }
            group_sync(grp);  // every warp is done with this stage
            if (gtid == 0 && ci + kFmStages < ncg) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue(ci + kFmStages);
            }
        }
        if (ci < ncg && gtid == 0) {
            // a wait expired: let the copies still in flight land before the
            // shared memory is reused or the CTA exits
            for (int cj = ci; cj < ncg && cj < ci + kFmStages; ++cj)
                mbar_wait_drain(&bars[cj % kFmStages], (uint32_t)((cj / kFmStages) & 1));
        }
    }

    // ---- combine the NW warps into this CTA's partial (shared memory re-used) ----
    // Per (warp, head) weights exp(m_warp - M) are computed once; every warp
    // scales its output by its weight and the scaled outputs are summed in
    // warp order.  Rows are padded by 8 floats so the float2 stores of a
    // warp do not collide in shared-memory banks.
    constexpr int WS = D + 4;                                 // padded row stride (floats)
    float* wo = reinterpret_cast<float*>(smem);             // [NW][kFaMaxG][WS] scaled warp outputs
    float* co = wo + NW * kFaMaxG * WS;                       // [kFaMaxG][D]  this CTA's partial
    __shared__ float cm[kFaMaxG], cl[kFaMaxG], ew[NW][kFaMaxG];
    __syncthreads();  // the rings are no longer read
    if (tid == 0) stamp_point(a.stamp, a.stamp_stride, 5);
    if (g == 0) {
        wm[warp][2 * t] = m_run[0];
        wm[warp][2 * t + 1] = m_run[1];
        wl[warp][2 * t] = l_run[0];
        wl[warp][2 * t + 1] = l_run[1];
    }
    __syncthreads();
    static_assert(NW <= 16 && 16 * kFaMaxG <= kFmThreads, "the warp combine reduces over groups of 16 lanes");
    if (tid < 16 * kFaMaxG) {
        // thread (h, w) = (tid / 16, tid % 16): max and weighted sum over the
        // 16 lanes of head h (warps w >= NW hold nothing), a fixed shuffle tree
        const int h = tid >> 4, w = tid & 15;
        const bool live = active && h < hn && w < NW;
        const float mw = live ? wm[w][h] : -INFINITY;
        float M = mw;
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o, 16));
        const float e = (M == -INFINITY || mw == -INFINITY) ? 0.f : expf(mw - M);
        if (w < NW) ew[w][h] = e;
        float L = live ? wl[w][h] * e : 0.f;
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) L += __shfl_xor_sync(0xffffffffu, L, o, 16);
        if (w == 0) {
            cm[h] = M;
            cl[h] = L;
        }
    }
    __syncthreads();
    {
        const float e0 = ew[warp][2 * t], e1 = ew[warp][2 * t + 1];
        float* r0 = wo + (warp * kFaMaxG + 2 * t) * WS + g;
        float* r1 = r0 + WS;
#pragma unroll
        for (int n = 0; n < MT; ++n) {
            r0[16 * n] = o[n][0] * e0;
            r1[16 * n] = o[n][1] * e1;
            r0[16 * n + 8] = o[n][2] * e0;
            r1[16 * n + 8] = o[n][3] * e1;
        }
    }
    __syncthreads();
    for (int i4 = tid; i4 < kFaMaxG * D / 4; i4 += kFmThreads) {
        const int h = (4 * i4) / D, d = 4 * i4 - h * D;
        float4 acc = *reinterpret_cast<const float4*>(wo + h * WS + d);
#pragma unroll
        for (int w = 1; w < NW; ++w) {
            const float4 v = *reinterpret_cast<const float4*>(wo + (w * kFaMaxG + h) * WS + d);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        reinterpret_cast<float4*>(co)[i4] = acc;
    }
    __syncthreads();

    // ---- cluster merge over the splits (distributed shared memory, push) ----
    // The outputs (float4 units) form tb blocks of 8 units (32 values); CTA k
    // of the cluster owns units [8 (k tb / S), 8 ((k+1) tb / S)), whole
    // blocks, so that it can also quantise them.  Every CTA stores its
    // partial of each owner's slice, and its (max, sum) per head, straight
    // into the owner's shared memory; after one cluster barrier every owner
    // merges from local shared memory, and no CTA touches a peer's shared
    // memory again.
    constexpr int kTot4Max = kFaMaxG * D / 4;
    __shared__ __align__(16) float4 rcv[kTot4Max + 8 * kFmMaxCluster];  // [S][slice4]
    __shared__ float rml[kFmMaxCluster][kFaMaxG][2];
    __shared__ float wr[kFaMaxG][kFmMaxCluster];
    cgx::cluster_group cluster = cgx::this_cluster();
    const int S = (int)cluster.num_blocks();
    const int rank = (int)cluster.block_rank();
    const int tot4 = hn * D / 4;
    const int tb = tot4 / 8;                       // D is a multiple of 32
    const int slice4 = 8 * ((tb + S - 1) / S);
    for (int i4 = tid; i4 < tot4; i4 += kFmThreads) {
        const int bi = i4 >> 3;
        int k = (int)(((int64_t)bi * S + S - 1) / tb);  // owner: k tb / S <= bi < (k+1) tb / S
        while (k > 0 && k * tb / S > bi) --k;
        while (k + 1 < S && (k + 1) * tb / S <= bi) ++k;
        float4* dst = cluster.map_shared_rank(rcv, k);
        dst[rank * slice4 + (i4 - 8 * (k * tb / S))] = reinterpret_cast<const float4*>(co)[i4];
    }
    if (tid < S * kFaMaxG) {
        const int k = tid / kFaMaxG, h = tid - (tid / kFaMaxG) * kFaMaxG;
        float* dst = &cluster.map_shared_rank(&rml[0][0][0], k)[(rank * kFaMaxG + h) * 2];
        dst[0] = cm[h];
        dst[1] = cl[h];
    }
    cluster.sync();  // every push has landed
    static_assert(kFmMaxCluster == 16 && kFaMaxG * kFmMaxCluster <= kFmThreads, "merge lanes");
    {
        // thread (h, r) = (tid / 16, tid % 16): max, weighted sum and
        // weights over the 16 lanes of head h (ranks r >= S hold nothing)
        const int h = tid >> 4, r = tid & 15;
        const bool live = h < hn && r < S;
        const float mr = live ? rml[r][h][0] : -INFINITY;
        float M = mr;
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o, 16));
        const float e = (mr == -INFINITY) ? 0.f : expf(mr - M);
        float L = live ? rml[r][h][1] * e : 0.f;
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) L += __shfl_xor_sync(0xffffffffu, L, o, 16);
        const float inv = L > 0.f ? 1.0f / L : 0.f;
        if (live) wr[h][r] = e * inv;
    }
    __syncthreads();
    const int o0 = 8 * (rank * tb / S), o1 = 8 * ((rank + 1) * tb / S);
    // Whole warps walk the slice together (o0 and o1 are multiples of 8, so
    // each 8-lane group is one block, all in or all out of the slice).
    for (int base = o0; base < o1; base += kFmThreads) {
        const int i4 = base + tid;
        const bool valid = i4 < o1;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (valid) {
            const int h = (4 * i4) / D, d = 4 * i4 - h * D;
            for (int r = 0; r < S; ++r) {
                const float w = wr[h][r];
                const float4 v = rcv[r * slice4 + (i4 - o0)];
                acc.x = fmaf(v.x, w, acc.x);
                acc.y = fmaf(v.y, w, acc.y);
                acc.z = fmaf(v.z, w, acc.z);
                acc.w = fmaf(v.w, w, acc.w);
            }
            *reinterpret_cast<float4*>(a.out + (int64_t)(h0 + h) * D + d) = acc;
        }
        if (a.xq_img != nullptr && base + (tid & ~31) < o1) {
            // the o projection's Q8_0 activation, quantised here once
            float4 v[1] = {acc};
            int word[1], qs[1];
            uint16_t dh[1];
            q8_units<1>(v, word, dh, qs);
            if (valid) q8_image_store(a.xq_img, a.xq_U, (int64_t)h0 * D / 4 + i4, word[0], dh[0], qs[0]);
        }
    }
    if (a.stamp != nullptr) {  // uniform over the grid
        __syncthreads();
        if (tid == 0) stamp_point(a.stamp, a.stamp_stride, 2);
    }
}

}  // namespace b200
