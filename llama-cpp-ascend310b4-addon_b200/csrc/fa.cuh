// fa.cuh -- single-token GQA flash-decoding (split-KV) for FLASH_ATTN_EXT.
//
// Grid (split, kv head, q-head chunk).  A CTA keeps up to 8 query heads of
// one GQA group (all that share the KV head) and walks its share of the KV
// sequence in 64-position chunks with an online softmax, so each K/V row is
// read from HBM once per group, not once per query head.  Every CTA writes an
// unnormalised partial (o, m, l); the last CTA of a (kv head, chunk) -- found
// with an atomic ticket, no spinning -- merges the partials in split order and
// resets its ticket, so results do not depend on CTA timing.
#pragma once

#include "args.h"
#include "common.cuh"

namespace b200 {

template <int D>
__global__ void __launch_bounds__(kFaThreads) fa_decode_kernel(const FaArgs a) {
    constexpr int DL = D / 32;  // dims per lane in the PV step
    constexpr int NW = kFaThreads / 32;
    __shared__ __align__(16) float qs[kFaMaxG][D];
    __shared__ float sc[kFaMaxG][kFaChunk];
    // Cross-warp reduction buffer [NW][kFaMaxG][D]; reused by the merging CTA
    // for the split weights [kFaMaxG][kFaTargetCtas].
    constexpr int kRed = NW * kFaMaxG * D > kFaMaxG * kFaTargetCtas ? NW * kFaMaxG * D : kFaMaxG * kFaTargetCtas;
    __shared__ float redbuf[kRed];
    auto red = reinterpret_cast<float (*)[kFaMaxG][D]>(redbuf);
    auto wts = reinterpret_cast<float (*)[kFaTargetCtas]>(redbuf);
    __shared__ float m_run[kFaMaxG], l_run[kFaMaxG], alpha[kFaMaxG];
    __shared__ int is_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x, hk = blockIdx.y, gc = blockIdx.z;
    const int h0 = hk * a.G + gc * kFaMaxG;
    const int hn = min(kFaMaxG, a.G - gc * kFaMaxG);

    int ctx = a.n_kv;
    if (a.kv_len != nullptr) {
        const int kl = a.kv_len[0];
        if (kl > 0 && kl < a.n_kv) ctx = kl;
    }
    const int nchunks_ctx = (ctx + kFaChunk - 1) / kFaChunk;
    const int c_begin = split * a.chunks_per_split;
    const int c_end = min(c_begin + a.chunks_per_split, nchunks_ctx);
    const bool active = c_begin < c_end;

    if (active) {
        for (int idx = tid; idx < kFaMaxG * D; idx += kFaThreads) {
            const int h = idx / D, d = idx - (idx / D) * D;
            qs[h][d] = h < hn ? round_f16(a.q[(int64_t)(h0 + h) * D + d]) : 0.f;
        }
        if (tid < kFaMaxG) {
            m_run[tid] = -INFINITY;
            l_run[tid] = 0.f;
        }
        float acc[kFaMaxG][DL];
#pragma unroll
        for (int h = 0; h < kFaMaxG; ++h)
#pragma unroll
            for (int e = 0; e < DL; ++e) acc[h][e] = 0.f;
        __syncthreads();

        for (int c = c_begin; c < c_end; ++c) {
            const int p0 = c * kFaChunk;
            // ---- scores: two threads per position, each half of the head dim ----
            {
                const int t = tid >> 1, half = tid & 1;
                const int p = p0 + t;
                float s[kFaMaxG];
#pragma unroll
                for (int h = 0; h < kFaMaxG; ++h) s[h] = 0.f;
                float mv = 0.f;
                const bool inb = p < ctx;
                if (inb && a.mask != nullptr) mv = h2f(a.mask[p]);
                const bool live = inb && mv != -INFINITY;
                if (live) {
                    const uint8_t* kr = a.k + (int64_t)p * a.k_nb1 + (int64_t)hk * a.k_nb2 + half * D;
#pragma unroll 4
                    for (int d0 = 0; d0 < D / 2; d0 += 8) {
                        const uint4 kv = *reinterpret_cast<const uint4*>(kr + d0 * 2);
                        const __half2* kh = reinterpret_cast<const __half2*>(&kv);
                        float kf[8];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = __half22float2(kh[e]);
                            kf[2 * e] = f.x;
                            kf[2 * e + 1] = f.y;
                        }
#pragma unroll
                        for (int h = 0; h < kFaMaxG; ++h) {
                            const float4 qa = *reinterpret_cast<const float4*>(&qs[h][half * (D / 2) + d0]);
                            const float4 qb = *reinterpret_cast<const float4*>(&qs[h][half * (D / 2) + d0 + 4]);
                            s[h] = fmaf(qa.x, kf[0], s[h]);
                            s[h] = fmaf(qa.y, kf[1], s[h]);
                            s[h] = fmaf(qa.z, kf[2], s[h]);
                            s[h] = fmaf(qa.w, kf[3], s[h]);
                            s[h] = fmaf(qb.x, kf[4], s[h]);
                            s[h] = fmaf(qb.y, kf[5], s[h]);
                            s[h] = fmaf(qb.z, kf[6], s[h]);
                            s[h] = fmaf(qb.w, kf[7], s[h]);
                        }
                    }
                }
#pragma unroll
                for (int h = 0; h < kFaMaxG; ++h) s[h] += __shfl_xor_sync(0xffffffffu, s[h], 1);
                if (half == 0) {
#pragma unroll
                    for (int h = 0; h < kFaMaxG; ++h)
                        sc[h][t] = live ? __fadd_rn(__fmul_rn(s[h], a.scale), mv) : -INFINITY;
                }
            }
            __syncthreads();
            // ---- online softmax update: warp w owns heads w, w + NW ----
            for (int h = warp; h < kFaMaxG; h += NW) {
                const float s0 = sc[h][lane], s1 = sc[h][lane + 32];
                const float cm = warp_max(fmaxf(s0, s1));
                const float mo = m_run[h];
                const float mn = fmaxf(mo, cm);
                const float p0v = s0 == -INFINITY ? 0.f : expf(s0 - mn);
                const float p1v = s1 == -INFINITY ? 0.f : expf(s1 - mn);
                const float ps = warp_sum(p0v + p1v);
                sc[h][lane] = p0v;
                sc[h][lane + 32] = p1v;
                __syncwarp();
                if (lane == 0) {
                    const float al = mo == -INFINITY ? 0.f : expf(mo - mn);
                    alpha[h] = mn == -INFINITY ? 1.f : al;
                    l_run[h] = l_run[h] * alpha[h] + ps;
                    m_run[h] = mn;
                }
            }
            __syncthreads();
            // ---- P.V: warp w takes positions w, w+4, ...; lanes split the head dim ----
#pragma unroll
            for (int h = 0; h < kFaMaxG; ++h) {
                const float al = alpha[h];
#pragma unroll
                for (int e = 0; e < DL; ++e) acc[h][e] *= al;
            }
            const int tmax = min(kFaChunk, ctx - p0);
            for (int t = warp; t < tmax; t += NW) {
                const int p = p0 + t;
                const uint8_t* vr = a.v + (int64_t)p * a.v_nb1 + (int64_t)hk * a.v_nb2 + lane * DL * 2;
                float vf[DL];
                if constexpr (DL == 4) {
                    const uint2 vv = *reinterpret_cast<const uint2*>(vr);
                    const __half2* vh = reinterpret_cast<const __half2*>(&vv);
                    const float2 f0 = __half22float2(vh[0]), f1 = __half22float2(vh[1]);
                    vf[0] = f0.x; vf[1] = f0.y; vf[2] = f1.x; vf[3] = f1.y;
                } else if constexpr (DL == 2) {
                    const __half2 vh = *reinterpret_cast<const __half2*>(vr);
                    const float2 f0 = __half22float2(vh);
                    vf[0] = f0.x; vf[1] = f0.y;
                } else {
#pragma unroll
                    for (int e = 0; e < DL; e += 2) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(vr + e * 2));
                        vf[e] = f.x;
                        vf[e + 1] = f.y;
                    }
                }
#pragma unroll
                for (int h = 0; h < kFaMaxG; ++h) {
                    const float pw = sc[h][t];
#pragma unroll
                    for (int e = 0; e < DL; ++e) acc[h][e] = fmaf(pw, vf[e], acc[h][e]);
                }
            }
            __syncthreads();  // sc is rewritten by the next chunk
        }
        // ---- cross-warp reduction of the partial output ----
#pragma unroll
        for (int h = 0; h < kFaMaxG; ++h)
#pragma unroll
            for (int e = 0; e < DL; ++e) red[warp][h][lane * DL + e] = acc[h][e];
        __syncthreads();
        for (int idx = tid; idx < hn * D; idx += kFaThreads) {
            const int h = idx / D, d = idx - (idx / D) * D;
            float o = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) o += red[w][h][d];
            a.part_o[((int64_t)split * a.Hq + h0 + h) * D + d] = o;
        }
        if (tid < hn) {
            a.part_ml[((int64_t)split * a.Hq + h0 + tid) * 2 + 0] = m_run[tid];
            a.part_ml[((int64_t)split * a.Hq + h0 + tid) * 2 + 1] = l_run[tid];
        }
    }

    // ---- ticket: the last CTA of this (kv head, chunk) merges ----
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned int* tk = a.tickets + hk * a.gchunks + gc;
        const unsigned int old = atomicAdd(tk, 1u);
        is_last = old == (unsigned int)(a.n_splits - 1);
        if (is_last) *tk = 0u;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();

    const int n_act = (nchunks_ctx + a.chunks_per_split - 1) / a.chunks_per_split;
    // Merge: w[h][s] = exp(m_s - M_h) / L_h computed once into shared memory,
    // then every (head, dim) output is an unrolled dot over the splits.
    for (int h = warp; h < hn; h += NW) {
        float M = -INFINITY;
        for (int s = lane; s < n_act; s += 32) M = fmaxf(M, __ldcg(&a.part_ml[((int64_t)s * a.Hq + h0 + h) * 2]));
        M = warp_max(M);
        float L = 0.f;
        for (int s = lane; s < n_act; s += 32) {
            const float ms = __ldcg(&a.part_ml[((int64_t)s * a.Hq + h0 + h) * 2]);
            const float ls = __ldcg(&a.part_ml[((int64_t)s * a.Hq + h0 + h) * 2 + 1]);
            const float e = (ms == -INFINITY) ? 0.f : expf(ms - M);
            wts[h][s] = e;
            L += ls * e;
        }
        L = warp_sum(L);
        const float inv = (L > 0.f) ? 1.0f / L : 0.f;
        __syncwarp();
        for (int s = lane; s < n_act; s += 32) wts[h][s] *= inv;
    }
    __syncthreads();
    for (int idx = tid; idx < hn * D; idx += kFaThreads) {
        const int h = idx / D, d = idx - (idx / D) * D;
        const float* po = a.part_o + (int64_t)(h0 + h) * D + d;
        const int64_t stride = (int64_t)a.Hq * D;
        float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
        int s = 0;
        for (; s + 4 <= n_act; s += 4) {
            o0 = fmaf(__ldcg(po + (int64_t)(s + 0) * stride), wts[h][s + 0], o0);
            o1 = fmaf(__ldcg(po + (int64_t)(s + 1) * stride), wts[h][s + 1], o1);
            o2 = fmaf(__ldcg(po + (int64_t)(s + 2) * stride), wts[h][s + 2], o2);
            o3 = fmaf(__ldcg(po + (int64_t)(s + 3) * stride), wts[h][s + 3], o3);
        }
        for (; s < n_act; ++s) o0 = fmaf(__ldcg(po + (int64_t)s * stride), wts[h][s], o0);
        a.out[(int64_t)(h0 + h) * D + d] = (o0 + o1) + (o2 + o3);
    }
}

}  // namespace b200
