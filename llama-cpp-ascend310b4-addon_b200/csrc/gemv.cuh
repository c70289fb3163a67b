// gemv.cuh -- M=1 matrix-vector kernels streamed from the packed tile layout.
//
// One persistent CTA per SM owns a contiguous range of tiles (R rows x K).
// Thread 0 keeps `stages` tiles in flight with cp.async.bulk into a shared
// memory ring (one mbarrier per stage, bounded waits); the 256 threads hold
// their slice of the activation in registers for the whole kernel, so every
// byte of weight is read from HBM once and from shared memory once.
//
// Activation handling follows ggml-cpu's MUL_MAT vec_dot_type conversion:
//   F16  : x -> f16, fp32 FMA over f16 products
//   Q4_0 : x -> Q8_0 blocks (quantize_row_q8_0_ref rule), dp4a integer block
//          dots, fp32 sum of d_w * d_x * dot (ggml mode), or x -> f16 and an
//          fp32 FMA over dequantised nibbles (W4A16 mode)
//   Q8_0 : x -> Q8_0 blocks, dp4a block dots
// Prologues fuse RMSNorm * weight; epilogues fuse the residual add, SwiGLU,
// RoPE + KV-cache write, and argmax (the decode neighbours of MUL_MAT).
#pragma once

#include "args.h"
#include "common.cuh"

namespace b200 {

// Order-preserving key of a float for unsigned max.
__device__ __forceinline__ unsigned int float_key(float f) {
    const unsigned int b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ unsigned long long pack_argmax(float v, int64_t idx) {
    return ((unsigned long long)float_key(v) << 32) | (unsigned long long)(0xffffffffu - (unsigned int)idx);
}

// ggml quantize_row_q8_0_ref on one block of 32 values: d = amax/127,
// q = roundf(x * (1/d)) (half away from zero), d stored as f16.  `load(e)`
// returns values 4e..4e+3; it is called twice so only four values are live.
template <class Load>
__device__ __forceinline__ void quantize_block32(Load load, int q[8], float& d_out, uint16_t& d_h, int& qsum) {
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float4 v = load(e);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.f ? __frcp_rn(d) : 0.f;
    int s = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float4 v = load(e);
        const int q0 = round_half_away(__fmul_rn(v.x, id));
        const int q1 = round_half_away(__fmul_rn(v.y, id));
        const int q2 = round_half_away(__fmul_rn(v.z, id));
        const int q3 = round_half_away(__fmul_rn(v.w, id));
        s += q0 + q1 + q2 + q3;
        q[e] = (int)((unsigned)(q0 & 0xff) | ((unsigned)(q1 & 0xff) << 8) | ((unsigned)(q2 & 0xff) << 16) |
                     ((unsigned)(q3 & 0xff) << 24));
    }
    d_h = f2h(d);
    d_out = h2f(d_h);
    qsum = s;
}

// Writes one ggml block_q8_0 (f16 d, 32 x int8) as 17 aligned 16-bit stores.
__device__ __forceinline__ void store_block_q8_0(uint8_t* dst, uint16_t dh, const int q[8]) {
    uint16_t* p = reinterpret_cast<uint16_t*>(dst);
    p[0] = dh;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        p[1 + 2 * w] = (uint16_t)((unsigned)q[w] & 0xffffu);
        p[2 + 2 * w] = (uint16_t)((unsigned)q[w] >> 16);
    }
}

template <int FMT>
struct MaxNU {
    static constexpr int value = FMT == FMT_Q4W ? 2 : 8;
};

// Chooses the number of row groups for a launch: the largest power of two
// that divides R and keeps every thread at <= MAXNU units.
inline int choose_row_groups(const GemvPlan& p, int maxnu) {
    for (int rg = 32; rg >= 1; rg >>= 1) {
        if (rg > p.R || p.R % rg) continue;
        const int tpr = kGemvThreads / rg;
        if ((p.U + tpr - 1) / tpr <= maxnu) return rg;
    }
    return 0;
}

template <int FMT, int MAXNU, bool DEBUG>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = a.stages;
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (int64_t)S * a.tile_bytes);
    float* part = reinterpret_cast<float*>(full + S);  // [2][kMaxR][kMaxSlots]
    float* red = part + 2 * kMaxR * kMaxSlots;         // [32]

    const int tid = threadIdx.x;
    const int TPR = kGemvThreads / a.RG;
    const int g = tid / TPR;
    const int j = tid - g * TPR;
    const int nslot = TPR > 32 ? TPR / 32 : 1;
    const int slot = TPR > 32 ? (j >> 5) : 0;
    const int R = a.R, U = a.U;

    const int64_t G = gridDim.x;
    const int64_t t0 = (int64_t)blockIdx.x * a.ntiles / G;
    const int64_t t1 = (int64_t)(blockIdx.x + 1) * a.ntiles / G;
    const int nt = (int)(t1 - t0);
    const uint32_t tb = (uint32_t)a.tile_bytes;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
        mbar_fence_init();
        for (int s = 0; s < S && s < nt; ++s) {
            mbar_arrive_expect_tx(&full[s], tb);
            bulk_g2s(ring + (int64_t)s * tb, a.w + (t0 + s) * a.tile_bytes, tb, &full[s]);
        }
    }

    // ---- prologue: RMSNorm scale (optional) ----
    float nscale = 1.f;
    if (a.pro == PRO_RMSNORM) {
        float ss = 0.f;
        const float4* x4 = reinterpret_cast<const float4*>(a.x);
        for (int64_t i = tid; i < a.k / 4; i += kGemvThreads) {
            const float4 v = x4[i];
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
    }
    __syncthreads();  // barrier init visible; norm partials ready
    if (a.pro == PRO_RMSNORM) {
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kGemvThreads / 32; ++w) tot += red[w];
        const float mean = __fdiv_rn(tot, (float)a.k);
        nscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
    }

    // ---- activation slice into registers ----
    float xf[(FMT == FMT_F16) ? MAXNU * 8 : (FMT == FMT_Q4W ? MAXNU * 32 : 1)];
    int xq[(FMT == FMT_Q4 || FMT == FMT_Q8) ? MAXNU * 8 : 1];
    float xd[(FMT == FMT_Q4 || FMT == FMT_Q8) ? MAXNU : 1];
    int xs[(FMT == FMT_Q4) ? MAXNU : 1];
#pragma unroll
    for (int i = 0; i < MAXNU; ++i) {
        const int u = j + TPR * i;
        const bool valid = u < U;
        if constexpr (FMT == FMT_F16) {
#pragma unroll
            for (int e = 0; e < 8; ++e) xf[i * 8 + e] = 0.f;
            if (valid) {
                const float4* src = reinterpret_cast<const float4*>(a.x + (int64_t)u * 8);
                float v[8];
                *reinterpret_cast<float4*>(&v[0]) = src[0];
                *reinterpret_cast<float4*>(&v[4]) = src[1];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    float t = v[e];
                    if (a.pro == PRO_RMSNORM) t = __fmul_rn(__fmul_rn(t, nscale), a.norm_w[(int64_t)u * 8 + e]);
                    xf[i * 8 + e] = round_f16(t);
                }
            }
        } else if constexpr (FMT == FMT_Q4W) {
#pragma unroll
            for (int e = 0; e < 32; ++e) xf[i * 32 + e] = 0.f;
            if (valid) {
                const float4* src = reinterpret_cast<const float4*>(a.x + (int64_t)u * 32);
                const float4* wn = reinterpret_cast<const float4*>(a.norm_w + (int64_t)u * 32);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    float4 v = src[e];
                    if (a.pro == PRO_RMSNORM) {
                        const float4 w4 = wn[e];
                        v.x = __fmul_rn(__fmul_rn(v.x, nscale), w4.x);
                        v.y = __fmul_rn(__fmul_rn(v.y, nscale), w4.y);
                        v.z = __fmul_rn(__fmul_rn(v.z, nscale), w4.z);
                        v.w = __fmul_rn(__fmul_rn(v.w, nscale), w4.w);
                    }
                    xf[i * 32 + 4 * e + 0] = round_f16(v.x);
                    xf[i * 32 + 4 * e + 1] = round_f16(v.y);
                    xf[i * 32 + 4 * e + 2] = round_f16(v.z);
                    xf[i * 32 + 4 * e + 3] = round_f16(v.w);
                }
            }
        } else {
            const float4* src = reinterpret_cast<const float4*>(a.x + (int64_t)(valid ? u : 0) * 32);
            const float4* wn = reinterpret_cast<const float4*>(a.norm_w + (int64_t)(valid ? u : 0) * 32);
            const bool norm = a.pro == PRO_RMSNORM;
            auto load = [&](int e) -> float4 {
                if (!valid) return make_float4(0.f, 0.f, 0.f, 0.f);
                float4 v = src[e];
                if (norm) {
                    const float4 w4 = wn[e];
                    v.x = __fmul_rn(__fmul_rn(v.x, nscale), w4.x);
                    v.y = __fmul_rn(__fmul_rn(v.y, nscale), w4.y);
                    v.z = __fmul_rn(__fmul_rn(v.z, nscale), w4.z);
                    v.w = __fmul_rn(__fmul_rn(v.w, nscale), w4.w);
                }
                return v;
            };
            int q[8];
            float d;
            uint16_t dh;
            int qs;
            quantize_block32(load, q, d, dh, qs);
#pragma unroll
            for (int e = 0; e < 8; ++e) xq[i * 8 + e] = q[e];
            xd[i] = d;
            if constexpr (FMT == FMT_Q4) xs[i] = qs;
            if (a.xq_out != nullptr && blockIdx.x == 0 && g == 0 && valid)
                store_block_q8_0(a.xq_out + (int64_t)u * 34, dh, q);
        }
    }

    // ---- stream the tiles ----
    for (int it = 0; it < nt; ++it) {
        const int s = it % S;
        const uint32_t parity = (uint32_t)((it / S) & 1);
        const bool ok = mbar_wait_bounded(&full[s], parity);
        const uint8_t* tile = ring + (int64_t)s * tb;
        const int64_t tglob = t0 + it;
        float* pbuf = part + (it & 1) * kMaxR * kMaxSlots;
        if (ok) {
            for (int r = g; r < R; r += a.RG) {
                float acc = 0.f;
#pragma unroll
                for (int i = 0; i < MAXNU; ++i) {
                    const int u = j + TPR * i;
                    if (u < U) {
                        if constexpr (FMT == FMT_F16) {
                            const uint4 wv = *reinterpret_cast<const uint4*>(tile + ((int64_t)r * a.k + (int64_t)u * 8) * 2);
                            const __half2* h = reinterpret_cast<const __half2*>(&wv);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float2 f = __half22float2(h[e]);
                                acc = fmaf(f.x, xf[i * 8 + 2 * e], acc);
                                acc = fmaf(f.y, xf[i * 8 + 2 * e + 1], acc);
                            }
                        } else if constexpr (FMT == FMT_Q4 || FMT == FMT_Q4W) {
                            const int64_t bi = (int64_t)r * U + u;
                            const uint4 qv = *reinterpret_cast<const uint4*>(tile + bi * 16);
                            const float dw = h2f(*reinterpret_cast<const uint16_t*>(tile + (int64_t)R * U * 16 + bi * 2));
                            const unsigned int wq[4] = {qv.x, qv.y, qv.z, qv.w};
                            if constexpr (FMT == FMT_Q4) {
                                int sumi = 0;
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    sumi = dp4a((int)(wq[e] & 0x0f0f0f0fu), xq[i * 8 + e], sumi);
                                    sumi = dp4a((int)((wq[e] >> 4) & 0x0f0f0f0fu), xq[i * 8 + 4 + e], sumi);
                                }
                                sumi -= 8 * xs[i];
                                if constexpr (DEBUG) {
                                    const int64_t nrow = tglob * R + r;
                                    if (nrow < a.n) a.dots[nrow * U + u] = sumi;
                                }
                                acc = fmaf(dw * xd[i], (float)sumi, acc);
                            } else {
                                float p = 0.f;
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
#pragma unroll
                                    for (int b = 0; b < 4; ++b) {
                                        const int lo = (int)((wq[e] >> (8 * b)) & 0xfu) - 8;
                                        const int hi = (int)((wq[e] >> (8 * b + 4)) & 0xfu) - 8;
                                        p = fmaf((float)lo, xf[i * 32 + 4 * e + b], p);
                                        p = fmaf((float)hi, xf[i * 32 + 16 + 4 * e + b], p);
                                    }
                                }
                                acc = fmaf(dw, p, acc);
                            }
                        } else {  // FMT_Q8
                            const int64_t bi = (int64_t)r * U + u;
                            const uint4 lo = *reinterpret_cast<const uint4*>(tile + bi * 16);
                            const uint4 hi = *reinterpret_cast<const uint4*>(tile + (int64_t)R * U * 16 + bi * 16);
                            const float dw = h2f(*reinterpret_cast<const uint16_t*>(tile + (int64_t)R * U * 32 + bi * 2));
                            int sumi = 0;
                            sumi = dp4a((int)lo.x, xq[i * 8 + 0], sumi);
                            sumi = dp4a((int)lo.y, xq[i * 8 + 1], sumi);
                            sumi = dp4a((int)lo.z, xq[i * 8 + 2], sumi);
                            sumi = dp4a((int)lo.w, xq[i * 8 + 3], sumi);
                            sumi = dp4a((int)hi.x, xq[i * 8 + 4], sumi);
                            sumi = dp4a((int)hi.y, xq[i * 8 + 5], sumi);
                            sumi = dp4a((int)hi.z, xq[i * 8 + 6], sumi);
                            sumi = dp4a((int)hi.w, xq[i * 8 + 7], sumi);
                            if constexpr (DEBUG) {
                                const int64_t nrow = tglob * R + r;
                                if (nrow < a.n) a.dots[nrow * U + u] = sumi;
                            }
                            acc = fmaf(dw * xd[i], (float)sumi, acc);
                        }
                    }
                }
                acc = group_sum(acc, TPR < 32 ? TPR : 32);
                if ((j & 31) == 0) pbuf[r * kMaxSlots + slot] = acc;
            }
        }
        // Stage s is free once every thread passed this barrier.
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                // Drain the copies still in flight (bounded), then leave.
                for (int k2 = it + 1; k2 < nt && k2 < it + S; ++k2)
                    mbar_wait_bounded(&full[k2 % S], (uint32_t)((k2 / S) & 1));
            }
            return;
        }
        if (tid == 0 && it + S < nt) {
            mbar_arrive_expect_tx(&full[s], tb);
            bulk_g2s(ring + (int64_t)s * tb, a.w + (t0 + it + S) * a.tile_bytes, tb, &full[s]);
        }

        // ---- finalize the tile's rows (warp 0) ----
        if (tid < 32) {
            const int64_t nbase = tglob * R;
            auto rowsum = [&](int r) {
                float v = 0.f;
                for (int q = 0; q < nslot; ++q) v += pbuf[r * kMaxSlots + q];
                return v;
            };
            if (a.epi == EPI_STORE || a.epi == EPI_ADD) {
                if (tid < R) {
                    const int64_t n = nbase + tid;
                    if (n < a.n) {
                        float v = rowsum(tid);
                        if (a.epi == EPI_ADD) v = __fadd_rn(v, a.res[n]);
                        a.y[n] = v;
                    }
                }
            } else if (a.epi == EPI_SWIGLU) {
                if (2 * tid < R) {
                    const int64_t n = nbase + 2 * tid;
                    if (n < a.n) {
                        const float gt = rowsum(2 * tid), up = rowsum(2 * tid + 1);
                        const float sg = __fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt)));
                        a.y[n / 2] = __fmul_rn(sg, up);
                    }
                }
            } else if (a.epi == EPI_QKV) {
                if (2 * tid < R) {
                    const int64_t n = nbase + 2 * tid;
                    if (n < a.n) {
                        const float v0 = rowsum(2 * tid), v1 = rowsum(2 * tid + 1);
                        const int pos = *a.pos;
                        if (n < a.nq + a.nkv) {
                            const int local = (int)(n < a.nq ? n : n - a.nq);
                            const int i0 = local % a.head_dim;
                            float theta = (float)pos;
                            for (int t = 0; t < i0 / 2; ++t) theta = __fmul_rn(theta, a.theta_scale);
                            float sn, cs;
                            sincosf(theta, &sn, &cs);
                            const float r0 = __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn));
                            const float r1 = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, cs));
                            if (n < a.nq) {
                                a.y[n] = r0;
                                a.y[n + 1] = r1;
                            } else {
                                uint16_t* kr = a.kc + (int64_t)pos * a.nkv + local;
                                kr[0] = f2h(r0);
                                kr[1] = f2h(r1);
                            }
                        } else {
                            const int local = (int)(n - a.nq - a.nkv);
                            uint16_t* vr = a.vc + (int64_t)pos * a.nkv + local;
                            vr[0] = f2h(v0);
                            vr[1] = f2h(v1);
                        }
                    }
                }
            } else if (a.epi == EPI_ARGMAX) {
                unsigned long long best = 0ull;
                if (tid < R) {
                    const int64_t n = nbase + tid;
                    if (n < a.n) {
                        const float v = rowsum(tid);
                        a.y[n] = v;
                        best = pack_argmax(v, n + a.row_offset);
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                    best = other > best ? other : best;
                }
                if (tid == 0 && best != 0ull) atomicMax(a.amax, best);
            }
        }
    }
}

}  // namespace b200
