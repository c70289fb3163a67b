// gemv.cuh -- M=1 matrix-vector kernels streamed from the packed row layout.
//
// Structure (one CTA per SM, 16 warps):
//   * prologue: the CTA turns x into the form the dot needs, once, in shared
//     memory -- Q8_0 blocks (ggml quantize_row_q8_0_ref rule) for Q4_0/Q8_0
//     weights, f16-rounded values for F16 weights and the W4A16 mode --
//     optionally fusing RMSNorm * weight;
//   * main loop: every warp owns a contiguous range of rows and streams them
//     through its own ring of shared-memory stages with cp.async.bulk
//     (lane 0 issues, an mbarrier per stage, bounded waits).  Warps never
//     synchronise with each other after the prologue, so the memory system
//     always has ~16 x stages x chunk bytes in flight per SM;
//   * lanes split a row's units; a row's sum is a warp (or lane-group)
//     reduction, and the epilogue (store, residual add, SwiGLU pair,
//     RoPE + KV-cache write, argmax) runs on the lane that holds it.
//
// Arithmetic follows ggml-cpu's MUL_MAT with src1 converted to the weight's
// vec_dot_type: F16 -> fp32 FMA over f16 products; Q4_0/Q8_0 -> integer
// dp4a block dots, fp32 sum of d_w * d_x * dot; W4A16 -> fp32 FMA over
// dequantised nibbles and f16-rounded x.
#pragma once

#include <type_traits>

#include "args.h"
#include "allreduce.cuh"
#include "common.cuh"

namespace b200 {

// Order-preserving key of a float for unsigned max.
__device__ __forceinline__ unsigned int float_key(float f) {
    const unsigned int b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// (value, index) packed so that a larger value wins and, on ties, the
// smaller index wins (ggml_argmax returns the first maximum).
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
        q[e] = pack_q4(q0, q1, q2, q3);
        s = __dp4a(q[e], 0x01010101, s);
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

// Exact int -> float for |v| < 2^22 on the integer/FMA pipes (the int->float
// conversion instruction runs on the narrow transcendental pipe): the bits of
// 1.5 * 2^23 + v, minus 1.5 * 2^23.
__device__ __forceinline__ float small_int_to_float(int v) {
    return __int_as_float(0x4B400000 + v) - 12582912.0f;
}

// Bytes of the activation region at the start of shared memory.
B200_HD inline int64_t gemv_x_bytes(int fmt, const GemvPlan& p) {
    if (fmt == FMT_Q4 || fmt == FMT_Q8 || fmt == FMT_A8)
        return pad16(40 * (int64_t)p.U);  // xq planes 2 x [U][16] + {d, sum}[U] (A8W8: the token scale)
    return pad16(2 * p.k);                                                // f16 x[K]
}

// ------------------------------------------------------------- epilogues

template <bool AR = false>
__device__ __forceinline__ void epi_row(const GemvArgs& a, int64_t n, float v, unsigned long long& best) {
    if (a.epi == EPI_STORE) {
        a.y[n] = v;
    } else if (a.epi == EPI_ADD) {
        a.y[n] = __fadd_rn(v, a.res[n]);
    } else if (AR && a.epi == EPI_PUSH) {
        const float o = a.res != nullptr ? __fadd_rn(v, a.res[n]) : v;
        for (int r = 0; r < a.ar_world; ++r) a.ar_dst[r][n] = o;
    } else if (a.epi == EPI_ARGMAX) {
        a.y[n] = v;
        const unsigned long long k = pack_argmax(v, n + a.row_offset);
        best = k > best ? k : best;
    }
}

// ggml swiglu of a (gate, up) pair: silu(g) * u with silu(g) = g / (1 + exp(-g)).
__device__ __forceinline__ float swiglu(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// Rows n (even) and n + 1.
__device__ __forceinline__ void epi_pair(const GemvArgs& a, int64_t n, float v0, float v1) {
    if (a.epi == EPI_SWIGLU) {
        a.y[n / 2] = swiglu(v0, v1);
    } else if (a.epi == EPI_QKV) {
        const int pos = *a.pos;
        if (n < a.nq + a.nkv) {
            // ggml rope, NORM mode: theta_i = pos * theta_scale^i, built by
            // repeated fp32 multiplication as ggml_rope_cache_init does.
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

// ------------------------------------------------------------ unit dots

template <int FMT>
struct GemvTraits {
    // units per lane per chunk row, upper bound (plan: kc <= 128 for Q8_0 / A8W8, 256 otherwise)
    static constexpr int kMaxUpl = (FMT == FMT_Q8 || FMT == FMT_A8) ? 4 : 8;
    // A8W8 rows are exact int32 sums (one scale per row and token); the
    // other formats scale every block and accumulate in fp32
    using Acc = std::conditional_t<FMT == FMT_A8, int, float>;
};

// Sum over the lanes of a warp, in the accumulator type.
__device__ __forceinline__ float warp_sum_acc(float v) { return warp_sum(v); }
__device__ __forceinline__ int warp_sum_acc(int v) { return __reduce_add_sync(0xffffffffu, v); }
__device__ __forceinline__ int group_sum(int v, int width) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        if (o < width) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// A8W8 output: y = f16(f32(acc) * s_x * s_w) as an f32 (the reference's
// W8a8DequantCustom writes f16, then the op casts back to f32).
__device__ __forceinline__ float a8w8_dequant(int acc, float xs, uint16_t ws) {
    return round_f16(__fmul_rn(__fmul_rn(__int2float_rn(acc), xs), h2f(ws)));
}

// Sum of one staged chunk row for this lane: units i = i0 + step*j (j < upl,
// i < nu) of a row whose planes are `pw` units wide; `u0` is the row offset of
// unit 0 of the chunk.  All loads of the row are issued before the math.
template <int FMT, bool DEBUG>
__device__ __forceinline__ typename GemvTraits<FMT>::Acc unit_dot(const uint8_t* row, int pw, int i, int u,
                                                                  const uint8_t* xr, int U, int32_t* dots,
                                                                  int64_t nrow) {
    if constexpr (FMT == FMT_A8) {
        const int4 xa = reinterpret_cast<const int4*>(xr)[u];
        const int4 xb = reinterpret_cast<const int4*>(xr + 16 * (int64_t)U)[u];
        const uint4 lo = *reinterpret_cast<const uint4*>(row + 16 * i);
        const uint4 hi = *reinterpret_cast<const uint4*>(row + 16 * pw + 16 * i);
        int s0 = dp4a((int)lo.x, xa.x, 0), s1 = dp4a((int)hi.x, xb.x, 0);
        s0 = dp4a((int)lo.y, xa.y, s0);
        s1 = dp4a((int)hi.y, xb.y, s1);
        s0 = dp4a((int)lo.z, xa.z, s0);
        s1 = dp4a((int)hi.z, xb.z, s1);
        s0 = dp4a((int)lo.w, xa.w, s0);
        s1 = dp4a((int)hi.w, xb.w, s1);
        return s0 + s1;
    } else if constexpr (FMT == FMT_F16) {
        const uint4 wv = *reinterpret_cast<const uint4*>(row + 16 * i);
        const uint4 xv = *reinterpret_cast<const uint4*>(xr + 16 * u);
        const __half2* wh = reinterpret_cast<const __half2*>(&wv);
        const __half2* xh = reinterpret_cast<const __half2*>(&xv);
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 wf = __half22float2(wh[e]);
            const float2 xf = __half22float2(xh[e]);
            acc = fmaf(wf.x, xf.x, acc);
            acc = fmaf(wf.y, xf.y, acc);
        }
        return acc;
    } else if constexpr (FMT == FMT_Q4W) {
        const uint4 qv = *reinterpret_cast<const uint4*>(row + 16 * i);
        const float dw = h2f(*reinterpret_cast<const uint16_t*>(row + 16 * pw + 2 * i));
        const uint4* x4 = reinterpret_cast<const uint4*>(xr + 64 * u);
        const unsigned int wq[4] = {qv.x, qv.y, qv.z, qv.w};
        float p = 0.f;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {  // elements 0..15 (low nibbles), then 16..31 (high nibbles)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const uint4 xv = x4[hf * 2 + e];
                const __half2* xh = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float2 xf = __half22float2(xh[t]);
                    const int jj = e * 8 + t * 2;  // element index within the half
                    const unsigned int w = wq[jj >> 2];
                    const int sh = 8 * (jj & 3) + 4 * hf;
                    // nibble - 8 as a float without an int->float conversion:
                    // the bits 2^23 + nibble, minus (2^23 + 8)
                    const float q0 = __uint_as_float(0x4B000000u | ((w >> sh) & 0xfu)) - 8388616.0f;
                    const float q1 = __uint_as_float(0x4B000000u | ((w >> (sh + 8)) & 0xfu)) - 8388616.0f;
                    p = fmaf(q0, xf.x, p);
                    p = fmaf(q1, xf.y, p);
                }
            }
        }
        return dw * p;
    } else {
        const int4 xa = reinterpret_cast<const int4*>(xr)[u];
        const int4 xb = reinterpret_cast<const int4*>(xr + 16 * (int64_t)U)[u];
        const int2 ds = reinterpret_cast<const int2*>(xr + 32 * (int64_t)U)[u];
        int s0, s1;
        float dw;
        if constexpr (FMT == FMT_Q4) {
            const uint4 qv = *reinterpret_cast<const uint4*>(row + 16 * i);
            dw = h2f(*reinterpret_cast<const uint16_t*>(row + 16 * pw + 2 * i));
            s0 = dp4a((int)(qv.x & 0x0f0f0f0fu), xa.x, 0);
            s1 = dp4a((int)((qv.x >> 4) & 0x0f0f0f0fu), xb.x, 0);
            s0 = dp4a((int)(qv.y & 0x0f0f0f0fu), xa.y, s0);
            s1 = dp4a((int)((qv.y >> 4) & 0x0f0f0f0fu), xb.y, s1);
            s0 = dp4a((int)(qv.z & 0x0f0f0f0fu), xa.z, s0);
            s1 = dp4a((int)((qv.z >> 4) & 0x0f0f0f0fu), xb.z, s1);
            s0 = dp4a((int)(qv.w & 0x0f0f0f0fu), xa.w, s0);
            s1 = dp4a((int)((qv.w >> 4) & 0x0f0f0f0fu), xb.w, s1);
            s0 -= 8 * ds.y;  // nibbles are stored +8
        } else {
            const uint4 lo = *reinterpret_cast<const uint4*>(row + 16 * i);
            const uint4 hi = *reinterpret_cast<const uint4*>(row + 16 * pw + 16 * i);
            dw = h2f(*reinterpret_cast<const uint16_t*>(row + 32 * pw + 2 * i));
            s0 = dp4a((int)lo.x, xa.x, 0);
            s1 = dp4a((int)hi.x, xb.x, 0);
            s0 = dp4a((int)lo.y, xa.y, s0);
            s1 = dp4a((int)hi.y, xb.y, s1);
            s0 = dp4a((int)lo.z, xa.z, s0);
            s1 = dp4a((int)hi.z, xb.z, s1);
            s0 = dp4a((int)lo.w, xa.w, s0);
            s1 = dp4a((int)hi.w, xb.w, s1);
        }
        const int sumi = s0 + s1;
        if constexpr (DEBUG) dots[nrow * U + u] = sumi;
        return (dw * __int_as_float(ds.x)) * small_int_to_float(sumi);
    }
}

// Generic chunk row (tails, short rows): units i = i0 + step*j, j < upl, i < nu.
template <int FMT, bool DEBUG>
__device__ __forceinline__ typename GemvTraits<FMT>::Acc chunk_row_dot(const uint8_t* row, int pw, int i0, int step,
                                                                       int upl, int nu, int u0, const uint8_t* xr,
                                                                       int U, int32_t* dots, int64_t nrow) {
    typename GemvTraits<FMT>::Acc acc = 0;
    for (int j = 0; j < upl; ++j) {
        const int i = i0 + step * j;
        if (i < nu) acc += unit_dot<FMT, DEBUG>(row, pw, i, u0 + i, xr, U, dots, nrow);
    }
    return acc;
}

// Full chunk on the one-row path: exactly UPL units per lane at compile-time
// offsets (unit j of this lane is chunk unit lane + 32 j), no predicates.
template <int FMT, bool DEBUG, int UPL>
__device__ __forceinline__ typename GemvTraits<FMT>::Acc chunk_full_dot(const uint8_t* st, int kc, int lane, int u0,
                                                                        const uint8_t* xr, int U, int32_t* dots,
                                                                        int64_t nrow) {
    if constexpr (FMT == FMT_A8) {
        const uint8_t* wl = st + 16 * lane;
        const uint8_t* wh = st + 16 * kc + 16 * lane;
        const int4* xpa = reinterpret_cast<const int4*>(xr) + u0 + lane;
        const int4* xpb = reinterpret_cast<const int4*>(xr + 16 * (int64_t)U) + u0 + lane;
        int s0 = 0, s1 = 0;
#pragma unroll
        for (int j = 0; j < UPL; ++j) {
            const uint4 lo = *reinterpret_cast<const uint4*>(wl + 512 * j);
            const uint4 hi = *reinterpret_cast<const uint4*>(wh + 512 * j);
            const int4 xa = xpa[32 * j], xb = xpb[32 * j];
            s0 = dp4a((int)lo.x, xa.x, s0);
            s1 = dp4a((int)hi.x, xb.x, s1);
            s0 = dp4a((int)lo.y, xa.y, s0);
            s1 = dp4a((int)hi.y, xb.y, s1);
            s0 = dp4a((int)lo.z, xa.z, s0);
            s1 = dp4a((int)hi.z, xb.z, s1);
            s0 = dp4a((int)lo.w, xa.w, s0);
            s1 = dp4a((int)hi.w, xb.w, s1);
        }
        return s0 + s1;
    }
    float acc = 0.f;
    if constexpr (FMT == FMT_Q4 || FMT == FMT_Q8) {
        const uint8_t* wq = st + 16 * lane;
        const uint8_t* wh = st + 16 * kc + 16 * lane;                           // Q8_0 bytes 16..31
        const uint8_t* wd = st + (FMT == FMT_Q8 ? 32 : 16) * kc + 2 * lane;     // scales
        const int4* xpa = reinterpret_cast<const int4*>(xr) + u0 + lane;
        const int4* xpb = reinterpret_cast<const int4*>(xr + 16 * (int64_t)U) + u0 + lane;
        const int2* xpd = reinterpret_cast<const int2*>(xr + 32 * (int64_t)U) + u0 + lane;
#pragma unroll
        for (int j0 = 0; j0 < UPL; j0 += 2) {
            constexpr int Bt = 2;
            uint4 wa[Bt], wb[Bt];
            int4 xa[Bt], xb[Bt];
            int2 ds[Bt];
            uint16_t dwh[Bt];
#pragma unroll
            for (int b = 0; b < Bt; ++b) {
                const int j = j0 + b;
                if (j < UPL) {
                    wa[b] = *reinterpret_cast<const uint4*>(wq + 512 * j);
                    if constexpr (FMT == FMT_Q8) wb[b] = *reinterpret_cast<const uint4*>(wh + 512 * j);
                    dwh[b] = *reinterpret_cast<const uint16_t*>(wd + 64 * j);
                    xa[b] = xpa[32 * j];
                    xb[b] = xpb[32 * j];
                    ds[b] = xpd[32 * j];
                }
            }
#pragma unroll
            for (int b = 0; b < Bt; ++b) {
                const int j = j0 + b;
                if (j < UPL) {
                    int s0, s1;
                    if constexpr (FMT == FMT_Q4) {
                        const uint4 qv = wa[b];
                        s0 = dp4a((int)(qv.x & 0x0f0f0f0fu), xa[b].x, 0);
                        s1 = dp4a((int)((qv.x >> 4) & 0x0f0f0f0fu), xb[b].x, 0);
                        s0 = dp4a((int)(qv.y & 0x0f0f0f0fu), xa[b].y, s0);
                        s1 = dp4a((int)((qv.y >> 4) & 0x0f0f0f0fu), xb[b].y, s1);
                        s0 = dp4a((int)(qv.z & 0x0f0f0f0fu), xa[b].z, s0);
                        s1 = dp4a((int)((qv.z >> 4) & 0x0f0f0f0fu), xb[b].z, s1);
                        s0 = dp4a((int)(qv.w & 0x0f0f0f0fu), xa[b].w, s0);
                        s1 = dp4a((int)((qv.w >> 4) & 0x0f0f0f0fu), xb[b].w, s1);
                        s0 -= 8 * ds[b].y;  // nibbles are stored +8
                    } else {
                        s0 = dp4a((int)wa[b].x, xa[b].x, 0);
                        s1 = dp4a((int)wb[b].x, xb[b].x, 0);
                        s0 = dp4a((int)wa[b].y, xa[b].y, s0);
                        s1 = dp4a((int)wb[b].y, xb[b].y, s1);
                        s0 = dp4a((int)wa[b].z, xa[b].z, s0);
                        s1 = dp4a((int)wb[b].z, xb[b].z, s1);
                        s0 = dp4a((int)wa[b].w, xa[b].w, s0);
                        s1 = dp4a((int)wb[b].w, xb[b].w, s1);
                    }
                    const int sumi = s0 + s1;
                    if constexpr (DEBUG) dots[nrow * U + u0 + lane + 32 * j] = sumi;
                    acc = fmaf(h2f(dwh[b]) * __int_as_float(ds[b].x), small_int_to_float(sumi), acc);
                }
            }
        }
        return acc;
    } else if constexpr (FMT == FMT_F16) {
        const uint8_t* wp = st + 16 * lane;
        const uint8_t* xp = xr + 16 * (int64_t)(u0 + lane);
#pragma unroll
        for (int j0 = 0; j0 < UPL; j0 += 2) {
            uint4 wv[2], xv[2];
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                wv[b] = *reinterpret_cast<const uint4*>(wp + 512 * (j0 + b));
                xv[b] = *reinterpret_cast<const uint4*>(xp + 512 * (j0 + b));
            }
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const __half2* wh = reinterpret_cast<const __half2*>(&wv[b]);
                const __half2* xh = reinterpret_cast<const __half2*>(&xv[b]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 wf = __half22float2(wh[e]);
                    const float2 xf = __half22float2(xh[e]);
                    acc = fmaf(wf.x, xf.x, acc);
                    acc = fmaf(wf.y, xf.y, acc);
                }
            }
        }
        return acc;
    } else {
        return chunk_row_dot<FMT, DEBUG>(st, kc, lane, 32, UPL, kc, u0, xr, U, dots, nrow);
    }
}

// ------------------------------------------------------------ activation

// ggml rms_norm's sum of squares: every square rounded to f32 (x * x), the
// sum kept in double (ggml_float); here a per-thread double sum, then warp
// and CTA sums in double.  Rounded to f32 only as mean = sum / n, as ggml
// does, so the scale matches ggml-cpu's bit for bit unless the two double
// sums (different orders, each within ~n * 2^-53 of the exact value)
// straddle an f32 rounding boundary of the mean.
__device__ __forceinline__ double sumsq4(float4 v) {
    return ((double)__fmul_rn(v.x, v.x) + (double)__fmul_rn(v.y, v.y)) +
           ((double)__fmul_rn(v.z, v.z) + (double)__fmul_rn(v.w, v.w));
}

// CTA-wide: 1 / sqrtf(mean + eps) with mean = f32(sum / n).  `red` holds
// kGemvWarps doubles.  Ends with every thread holding the scale.
__device__ __forceinline__ float rms_scale(double ss, int64_t n, float eps, float* red, int lane, int warp) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    double* rd = reinterpret_cast<double*>(red);
    if (lane == 0) rd[warp] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < kGemvWarps; ++w) tot += rd[w];
    const float mean = __double2float_rn(__ddiv_rn(tot, (double)n));
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

__device__ __forceinline__ float4 norm_unit(float4 v, float4 w, float nscale) {
    v.x = __fmul_rn(__fmul_rn(v.x, nscale), w.x);
    v.y = __fmul_rn(__fmul_rn(v.y, nscale), w.y);
    v.z = __fmul_rn(__fmul_rn(v.z, nscale), w.z);
    v.w = __fmul_rn(__fmul_rn(v.w, nscale), w.w);
    return v;
}

// x -> Q8_0 activation planes in shared memory (optionally RMSNorm * w first).
// Two lanes per 32-block (q8_halves): thread t takes half-blocks t, t + T, ...
// (T threads), four float4 each, with the next half-block's loads in flight
// while the current one is quantised; every lane runs every round (loads
// clamped to the last half-block, stores only for real ones).  The sum of
// squares runs over each thread's values in order.  `after_issue` runs once
// the first loads are in flight (the caller issues its remaining weight
// copies there).  `wpre`: this thread's norm weights of round 0, loaded by
// the caller before its wait on the previous kernel (norm_w is constant).
// Ends with __syncthreads.
template <bool AR, class AfterIssue>
__device__ __forceinline__ void activation_q8(const GemvArgs& a, const GemvPlan& P, uint8_t* xr, float* red, int tid,
                                              int lane, int warp, const float4 (&wpre)[4], AfterIssue after_issue) {
    const bool norm = a.pro == PRO_RMSNORM;
    const int nh = 2 * P.U;  // half-blocks of x
    const int rounds = (nh + kGemvThreads - 1) / kGemvThreads;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    const float4* w4 = reinterpret_cast<const float4*>(a.norm_w);
    // Fused all-reduce: x is the rank-ordered sum of the ranks' partials,
    // once every producer CTA of every rank has released this collective.
    const bool ar = AR && a.ar_src != nullptr;
    if (ar) {
        const unsigned long long seq =
            a.ar_st->step * (unsigned long long)a.ar_per_step + (unsigned long long)a.ar_idx + 1ull;
        const int nf = a.ar_world * a.ar_grid;
        bool ok = true;
        for (int i = tid; i < nf && ok; i += kGemvThreads)
            ok = wait_flag_geq(a.ar_flags + (int64_t)(i / a.ar_grid) * kArMaxCtas + (i % a.ar_grid), seq);
        // a flag that never came: the sums below would read partials that
        // are not there; the quantised image is still written (from
        // whatever the slots hold) so the kernel's shape of work is kept,
        // and the status word tells the host that the step is void
        __syncthreads();
    }
    auto ldx = [&](int u) -> float4 {
        if (!ar) return x4[u];
        const float4* s4 = reinterpret_cast<const float4*>(a.ar_src);
        float4 acc = __ldcg(s4 + u);
        for (int r = 1; r < a.ar_world; ++r) {
            const float4 v = __ldcg(s4 + (int64_t)r * (a.ar_stride / 4) + u);
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        if (blockIdx.x == 0) reinterpret_cast<float4*>(a.ar_x_out)[u] = acc;  // the residual stream
        return acc;
    };
    float4 xv[4], wv[4];
    auto load = [&](int r) {
        const int h = min(r * kGemvThreads + tid, nh - 1);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            xv[j] = ldx(4 * h + j);
            if (norm) wv[j] = r == 0 ? wpre[j] : w4[4 * h + j];
        }
    };
    load(0);
    after_issue();
    float nscale = 1.f;
    if (norm) {
        double ss = 0.0;
        for (int r = 0; r < rounds; ++r) {
            float4 t[4];
            const int h = r * kGemvThreads + tid;
#pragma unroll
            for (int j = 0; j < 4; ++j) t[j] = r == 0 ? xv[j] : ldx(4 * min(h, nh - 1) + j);
            if (h < nh) {
#pragma unroll
                for (int j = 0; j < 4; ++j) ss += sumsq4(t[j]);
            }
        }
        nscale = rms_scale(ss, a.k, a.eps, red, lane, warp);
    }
    uint8_t* xq_out = blockIdx.x == 0 ? a.xq_out : nullptr;
    for (int r = 0; r < rounds; ++r) {
        const int h = r * kGemvThreads + tid;
        float4 v[1][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[0][j] = norm ? norm_unit(xv[j], wv[j], nscale) : xv[j];
        if (r + 1 < rounds) load(r + 1);
        int4 w[1];
        uint16_t dh[1];
        int qs[1];
        q8_halves<1>(v, w, dh, qs);
        if (h < nh) {  // both lanes of a pair together (nh and T are even)
            q8_image_store_half(xr, P.U, h, w[0], dh[0], qs[0]);
            if (xq_out != nullptr) {
                // ggml block_q8_0: f16 d, then 32 int8 (2-byte aligned)
                uint16_t* o = reinterpret_cast<uint16_t*>(xq_out + (int64_t)(h >> 1) * 34);
                const int p = h & 1;
                if (p == 0) o[0] = dh[0];
                const int wds[4] = {w[0].x, w[0].y, w[0].z, w[0].w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    o[1 + 8 * p + 2 * k] = (uint16_t)((unsigned)wds[k] & 0xffffu);
                    o[2 + 8 * p + 2 * k] = (uint16_t)((unsigned)wds[k] >> 16);
                }
            }
        }
    }
    __syncthreads();
}

// x -> the reference's per-token int8 activation (W8a8QuantizeCustom,
// w8a8_quantize_custom_vector.cpp:35-64): x cast to f16, one scale
// amax / 127 (amax at least 1.27e-6) kept as f16, q = rint(x * 127 / amax)
// (round half to even).  Same planes as activation_q8; the token scale (the
// f16 value as f32) goes where the per-block scales would be.  Ends with
// __syncthreads.
template <class AfterIssue>
__device__ __forceinline__ void activation_a8(const GemvArgs& a, const GemvPlan& P, uint8_t* xr, float* red, int tid,
                                              int lane, int warp, AfterIssue after_issue) {
    constexpr int R = 8;
    const int nu = P.U * 8;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    float4 xv[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const int u = tid + i * kGemvThreads;
        if (u < nu) xv[i] = x4[u];
    }
    after_issue();
    float amax = 0.f;
    for (int base = 0; base < nu; base += R * kGemvThreads) {
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const int u = base + tid + i * kGemvThreads;
            if (u >= nu) continue;
            const float4 v = base == 0 ? xv[i] : x4[u];
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(round_f16(v.x)), fabsf(round_f16(v.y))),
                                     fmaxf(fabsf(round_f16(v.z)), fabsf(round_f16(v.w)))));
        }
    }
    amax = warp_max(amax);
    if (lane == 0) red[warp] = amax;
    __syncthreads();
    amax = 0.f;
#pragma unroll
    for (int w = 0; w < kGemvWarps; ++w) amax = fmaxf(amax, red[w]);
    amax = fmaxf(amax, 0.00000127f);
    const float inv = __fdiv_rn(127.0f, amax);
    if (tid == 0) *reinterpret_cast<float*>(xr + 32 * (int64_t)P.U) = round_f16(__fdiv_rn(amax, 127.0f));
    int* xw = reinterpret_cast<int*>(xr);
    const int wd = lane & 7;
    for (int base = 0; base < nu; base += R * kGemvThreads) {
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const int u = base + tid + i * kGemvThreads;
            if (u >= nu) continue;
            const float4 v = base == 0 ? xv[i] : x4[u];
            const int q0 = __float2int_rn(__fmul_rn(round_f16(v.x), inv));
            const int q1 = __float2int_rn(__fmul_rn(round_f16(v.y), inv));
            const int q2 = __float2int_rn(__fmul_rn(round_f16(v.z), inv));
            const int q3 = __float2int_rn(__fmul_rn(round_f16(v.w), inv));
            const int word = (int)((unsigned)(q0 & 0xff) | ((unsigned)(q1 & 0xff) << 8) |
                                   ((unsigned)(q2 & 0xff) << 16) | ((unsigned)(q3 & 0xff) << 24));
            xw[(wd < 4 ? 0 : 4 * P.U) + 4 * (u >> 3) + (wd & 3)] = word;
        }
    }
    __syncthreads();
}

// ------------------------------------------------------------ the kernel

// UPL: units per lane of this plan's full chunks (P.full_upl), or 0 when the
// plan has none; fixed at compile time so those chunks run fully unrolled.
// SwiGLU outputs [j0, j1) of this CTA, held in shared memory at hs[j - jb]
// (jb = j0 rounded down to a block, so blocks start 16-byte aligned), into
// the Q8_0 image a.xq_img that the down projection reads: the 32-blocks this
// CTA owns whole.  A block that spans two CTAs is left to the
// down projection's prologue, which quantises it from h (GemvArgs::xq_fix_*)
// -- no cross-CTA fence or counter on this kernel's tail.
__device__ __forceinline__ void swiglu_quantise(const GemvArgs& a, int64_t j0, int64_t j1, int tid, const float* hs) {
    const int64_t nout = a.n / 2;
    const int64_t b0 = (j0 + 31) / 32, b1 = j1 / 32;  // whole blocks [b0, b1)
    const int nh = b1 > b0 ? (int)(2 * (b1 - b0)) : 0;  // half-blocks
    const int lane = tid & 31;
    // 2 lanes per block, 16 values each; whole warps run q8_halves
    for (int g0 = (tid >> 5) * 32; g0 < nh; g0 += kGemvThreads) {
        const int hi = g0 + lane;
        const bool valid = hi < nh;
        const float4* src = reinterpret_cast<const float4*>(hs + (32 * b0 - (j0 & ~31LL)) + 16 * (int64_t)(valid ? hi : 0));
        float4 v[1][4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[0][k] = src[k];
        int4 w[1];
        uint16_t dh[1];
        int qs[1];
        q8_halves<1>(v, w, dh, qs);
        if (valid) q8_image_store_half(a.xq_img, nout / 32, 2 * b0 + hi, w[0], dh[0], qs[0]);
    }
}

// The blocks of an image that span two CTAs of its producer (the SwiGLU
// epilogue above leaves them), quantised here from the producer's f32
// output a.xq_fix_h into this CTA's shared-memory image: the producer's CTA
// c (1 <= c < xq_fix_grid) starts at output c * xq_fix_items / xq_fix_grid;
// a start inside a block marks that block, two half-blocks (lanes) each.
// Thread t takes half-block t (2 (grid - 1) <= 2 * 255 < kGemvThreads, so
// one round); fix_load issues its loads (with the image copy's), fix_store
// quantises whole warps and replaces the block in the copied image; CTA 0
// also writes it to the global image (a.xq_fix_out), so the image in HBM is
// complete after this kernel.
struct ImageFix {
    float4 v[1][4];
    int64_t half;
    bool valid, run;  // run: this warp takes part (q8_halves needs whole warps)
};

__device__ __forceinline__ ImageFix fix_load(const GemvArgs& a, int tid) {
    ImageFix f;
    const int nfix = 2 * (a.xq_fix_grid - 1);
    f.run = (tid & ~31) < nfix;
    const int hi = tid < nfix ? tid : 0;
    const int c = 1 + hi / 2;
    const int64_t jc = (int64_t)c * a.xq_fix_items / a.xq_fix_grid;
    f.valid = tid < nfix && (jc & 31) != 0;
    f.half = 2 * (jc / 32) + (hi & 1);
    if (f.run) {
        const float4* src = reinterpret_cast<const float4*>(a.xq_fix_h) + 4 * f.half;
#pragma unroll
        for (int k = 0; k < 4; ++k) f.v[0][k] = src[k];
    }
    return f;
}

__device__ __forceinline__ void fix_store(const GemvArgs& a, const GemvPlan& P, uint8_t* xr, const ImageFix& f) {
    if (!f.run) return;  // uniform over the warp
    int4 w[1];
    uint16_t dh[1];
    int qs[1];
    q8_halves<1>(f.v, w, dh, qs);
    if (f.valid) {
        q8_image_store_half(xr, P.U, f.half, w[0], dh[0], qs[0]);
        if (blockIdx.x == 0 && a.xq_fix_out != nullptr) q8_image_store_half(a.xq_fix_out, P.U, f.half, w[0], dh[0], qs[0]);
    }
}

// AR: the fused tensor-parallel all-reduce variant (EPI_PUSH epilogue,
// summing prologue), instantiated apart so that the other kernels keep
// their register allocation.
template <int FMT, bool DEBUG, int UPL, bool AR = false>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvPlan& P = a.p;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) stamp_point(a.stamp, a.stamp_stride, 0);
    const int S = a.stages;
    const int64_t xbytes = gemv_x_bytes(FMT, P);
    uint8_t* xr = smem;
    uint8_t* rings = smem + xbytes;
    uint8_t* ring = rings + (int64_t)warp * S * P.stage_bytes;
    uint64_t* bars_all = reinterpret_cast<uint64_t*>(rings + (int64_t)kGemvWarps * S * P.stage_bytes);
    uint64_t* bars = bars_all + warp * S;
    float* red = reinterpret_cast<float*>(bars_all + kGemvWarps * S);  // [kGemvWarps] doubles (8-byte aligned)

    // ---- work distribution ----
    // rpc > 1 (short rows): every warp owns a contiguous range of row groups
    // and runs the epilogue itself.  rpc == 1: every CTA owns a contiguous,
    // balanced range of rows [cr0, cr1); its chunk sequence (row-major) is
    // split evenly over the 16 warps, row partials meet in shared memory and
    // the epilogue runs at the end over the CTA's rows.
    const bool pair = a.epi == EPI_SWIGLU || a.epi == EPI_QKV;
    int64_t row_begin, row_end, nq, q_begin = 0;
    int64_t cr0 = 0, cr1 = 0;
    if (P.rpc > 1) {
        const int64_t items = (P.n + P.rpc - 1) / P.rpc;
        const int64_t gw = (int64_t)blockIdx.x * kGemvWarps + warp, ngw = (int64_t)gridDim.x * kGemvWarps;
        const int64_t it0 = gw * items / ngw, it1 = (gw + 1) * items / ngw;
        row_begin = it0 * P.rpc;
        row_end = min(it1 * P.rpc, P.n);
        nq = it1 - it0;
    } else {
        const int64_t item_rows = pair ? 2 : 1;
        const int64_t items = (P.n + item_rows - 1) / item_rows;
        cr0 = gemv_cta_start(blockIdx.x, gridDim.x, items, a.late_ctas, a.late_pct) * item_rows;
        cr1 = min(gemv_cta_start(blockIdx.x + 1, gridDim.x, items, a.late_ctas, a.late_pct) * item_rows, P.n);
        const int64_t R = cr1 - cr0;
        int64_t q_end;
        if (R >= kGemvWarps) {
            // >= nchunk chunks per warp: a row meets at most two warps
            const int64_t total = R * P.nchunk;
            q_begin = (int64_t)warp * total / kGemvWarps;
            q_end = (int64_t)(warp + 1) * total / kGemvWarps;
        } else {
            // few rows: whole rows per warp
            q_begin = ((int64_t)warp * R / kGemvWarps) * P.nchunk;
            q_end = ((int64_t)(warp + 1) * R / kGemvWarps) * P.nchunk;
        }
        nq = q_end - q_begin;
        row_begin = cr0 + q_begin / P.nchunk;
        row_end = cr1;
    }
    // Row partials of this CTA (rpc == 1): part0 gets the partial of the warp
    // that holds the row's first chunk, part1 the rest (at most two warps
    // share a row; see the launcher), summed in that order.
    float* part0 = red + 2 * kGemvWarps;  // red: kGemvWarps doubles
    float* part1 = part0 + (P.rpc > 1 ? 0 : (cr1 - cr0));

    // Lane 0 only: stage the next chunk into ring slot s.  The issue cursor
    // (row offset, chunk in row) advances by one chunk per call; the loop
    // below keeps the same order, so no division is needed on the hot path.
    int64_t irow = 0;
    int ic = P.rpc > 1 ? 0 : (int)(q_begin % P.nchunk);
    const uint64_t pol = l2_policy(a.l2_ef != 0);
    auto issue = [&](int s) {
        uint8_t* dst = ring + (int64_t)s * P.stage_bytes;
        uint64_t* bar = &bars[s];
        if (P.rpc > 1) {
            const int64_t r0 = row_begin + irow;
            const int64_t nr = min((int64_t)P.rpc, P.n - r0);
            const uint32_t bytes = (uint32_t)(nr * P.rs);
            mbar_arrive_expect_tx(bar, bytes);
            bulk_g2s_pol(dst, a.w + r0 * P.rs, bytes, bar, pol);
            irow += P.rpc;
        } else {
            const int64_t row = row_begin + irow;
            const int u0 = ic * P.kc;
            const int nu = min(P.kc, P.U - u0);
            const uint8_t* base = a.w + row * P.rs;
            const uint32_t b0 = (uint32_t)(16 * nu);
            if constexpr (FMT == FMT_F16) {
                mbar_arrive_expect_tx(bar, b0);
                bulk_g2s_pol(dst, base + 16 * (int64_t)u0, b0, bar, pol);
            } else if constexpr (FMT == FMT_Q8) {
                const uint32_t b1 = (uint32_t)pad16(2 * nu);
                mbar_arrive_expect_tx(bar, 2 * b0 + b1);
                bulk_g2s_pol(dst, base + 16 * (int64_t)u0, b0, bar, pol);
                bulk_g2s_pol(dst + 16 * P.kc, base + 16 * (int64_t)P.U + 16 * (int64_t)u0, b0, bar, pol);
                bulk_g2s_pol(dst + 32 * P.kc, base + 32 * (int64_t)P.U + 2 * (int64_t)u0, b1, bar, pol);
            } else if constexpr (FMT == FMT_A8) {
                mbar_arrive_expect_tx(bar, 2 * b0);
                bulk_g2s_pol(dst, base + 16 * (int64_t)u0, b0, bar, pol);
                bulk_g2s_pol(dst + 16 * P.kc, base + 16 * (int64_t)P.U + 16 * (int64_t)u0, b0, bar, pol);
            } else {
                const uint32_t b1 = (uint32_t)pad16(2 * nu);
                mbar_arrive_expect_tx(bar, b0 + b1);
                bulk_g2s_pol(dst, base + 16 * (int64_t)u0, b0, bar, pol);
                bulk_g2s_pol(dst + 16 * P.kc, base + 16 * (int64_t)P.U + 2 * (int64_t)u0, b1, bar, pol);
            }
            if (++ic == P.nchunk) {
                ic = 0;
                ++irow;
            }
        }
    };

    // Lane 0: the rest of the ring's first S stages (stage 0 goes before the
    // wait on the previous kernel).
    auto issue_rest = [&]() {
        for (int s = 1; s < S && s < nq; ++s) issue(s);
    };
    // The norm weights are constant: round 0 of them is loaded before the
    // first weight copies and the wait on the previous kernel, so that after
    // the wait the prologue waits only for x (an L2 hit), not for an HBM
    // read queued behind every SM's copies.
    float4 wpre[4] = {};
    if constexpr (FMT == FMT_Q4 || FMT == FMT_Q8) {
        if (a.pro == PRO_RMSNORM && a.xq_in == nullptr) {
            const int h = min(tid, 2 * P.U - 1);
#pragma unroll
            for (int j = 0; j < 4; ++j) wpre[j] = reinterpret_cast<const float4*>(a.norm_w)[4 * h + j];
        }
    }
    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        mbar_fence_init();
        if (nq > 0) issue(0);
    }
    // row partials zeroed (shared memory only; published by the prologue's
    // closing barrier)
    if (P.rpc == 1)
        for (int64_t r = tid; r < 2 * (cr1 - cr0); r += kGemvThreads) part0[r] = 0.f;
    // The first stage of every ring reads only constant data, so under a
    // programmatic launch it overlaps the previous kernel's tail; the
    // activation, residual and outputs are touched only after this wait.
    griddep_wait();
    griddep_launch_dependents();
    if (tid == 0) stamp_point(a.stamp, a.stamp_stride, 1);

    // ---- prologue: the activation, once per CTA, into shared memory ----
    // Q8_0 activations: every thread's first loads of x (and of the norm
    // weights) are issued BEFORE the rest of the weight ring, so these
    // latency-critical loads do not queue behind megabytes of weight copies.
    const bool norm = a.pro == PRO_RMSNORM;
    if constexpr (FMT == FMT_Q4 || FMT == FMT_Q8) {
        if (a.xq_in != nullptr) {
            // the producer already quantised the activation: copy its image
            // (loads first, then the rest of the weight ring)
            const int64_t n16 = 40 * (int64_t)P.U / 16;
            const int4* src = reinterpret_cast<const int4*>(a.xq_in);
            int4* dst = reinterpret_cast<int4*>(xr);
            const bool fix = a.xq_fix_h != nullptr;
            ImageFix fx;
            if (fix) fx = fix_load(a, tid);
            constexpr int RC = 8;
            int4 t[RC];
            for (int64_t base = 0; base < n16; base += RC * kGemvThreads) {
#pragma unroll
                for (int i = 0; i < RC; ++i)
                    if (base + tid + i * kGemvThreads < n16) t[i] = src[base + tid + i * kGemvThreads];
                if (base == 0 && lane == 0) issue_rest();
#pragma unroll
                for (int i = 0; i < RC; ++i)
                    if (base + tid + i * kGemvThreads < n16) dst[base + tid + i * kGemvThreads] = t[i];
            }
            if (tid == 0 && (P.U & 1))  // 40 U is a multiple of 8 only: the last 8 bytes
                reinterpret_cast<int2*>(xr)[5 * (int64_t)P.U - 1] = reinterpret_cast<const int2*>(a.xq_in)[5 * (int64_t)P.U - 1];
            if (fix) {
                __syncthreads();  // the copied image, before its boundary blocks are replaced
                fix_store(a, P, xr, fx);
            }
        } else {
            activation_q8<AR>(a, P, xr, red, tid, lane, warp, wpre, [&] {
                if (lane == 0) issue_rest();
            });
        }
    } else if constexpr (FMT == FMT_A8) {
        activation_a8(a, P, xr, red, tid, lane, warp, [&] {
            if (lane == 0) issue_rest();
        });
    } else {
        if (lane == 0) issue_rest();
        float nscale = 1.f;
        if (norm) {
            double ss = 0.0;
            const float4* x4 = reinterpret_cast<const float4*>(a.x);
            for (int64_t i = tid; i < a.k / 4; i += kGemvThreads) ss += sumsq4(x4[i]);
            nscale = rms_scale(ss, a.k, a.eps, red, lane, warp);
        }
        uint4* xh = reinterpret_cast<uint4*>(xr);
        for (int64_t i = tid; i < a.k / 8; i += kGemvThreads) {
            const float4* src = reinterpret_cast<const float4*>(a.x + i * 8);
            float v[8];
            *reinterpret_cast<float4*>(&v[0]) = src[0];
            *reinterpret_cast<float4*>(&v[4]) = src[1];
            if (norm) {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], nscale), a.norm_w[i * 8 + e]);
            }
            uint4 o;
            __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e) oh[e] = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
            xh[i] = o;
        }
    }
    __syncthreads();  // activation ready; also publishes every warp's barrier init
    if (tid == 0) stamp_point(a.stamp, a.stamp_stride, 3);

    // ---- stream this warp's chunks ----
    using Acc = typename GemvTraits<FMT>::Acc;
    Acc acc = 0;
    unsigned long long best = 0ull;
    // A8W8: the token scale (activation_a8) and the per-row weight scales
    const float a8_xs = FMT == FMT_A8 ? *reinterpret_cast<const float*>(xr + 32 * (int64_t)P.U) : 0.f;
    const uint16_t* a8_ws = reinterpret_cast<const uint16_t*>(a.w + P.n * P.rs);
    Acc* pacc0 = reinterpret_cast<Acc*>(part0);
    Acc* pacc1 = reinterpret_cast<Acc*>(part1);
    int s = 0;
    uint32_t parity = 0;
    int64_t crow = 0;                                             // rows consumed (offset from row_begin)
    int cc = P.rpc > 1 ? 0 : (int)(q_begin % P.nchunk);           // chunk within the row
    bool first_part = cc == 0;                                    // this warp holds the row's first chunk
    const int rr = lane >> P.tpr_log2, li = lane & (P.tpr - 1);
    for (int64_t q = 0; q < nq; ++q) {
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bars[s], parity));
        if (!ok) {
            if (lane == 0) {
                // let every copy this warp issued (stages q .. q + S - 1) land
                // before the shared memory is reused or the CTA exits
                int s2 = s;
                uint32_t p2 = parity;
                for (int64_t q2 = q; q2 < nq && q2 < q + S; ++q2) {
                    mbar_wait_drain(&bars[s2], p2);
                    if (++s2 == S) {
                        s2 = 0;
                        p2 ^= 1u;
                    }
                }
            }
            break;  // the status word records the timeout; still meet the CTA barrier below
        }
        if (q == 0 && tid == 0) stamp_point(a.stamp, a.stamp_stride, 4);
        const uint8_t* st = ring + (int64_t)s * P.stage_bytes;
        if (P.rpc > 1) {
            const int64_t r0 = row_begin + crow;
            const int nr = (int)min((int64_t)P.rpc, P.n - r0);
            Acc v = 0;
            if (rr < nr)
                v = chunk_row_dot<FMT, DEBUG>(st + (int64_t)rr * P.rs, P.U, li, P.tpr, P.upl, P.U, 0, xr, P.U,
                                              a.dots, r0 + rr);
            v = group_sum(v, P.tpr);
            const Acc vn = __shfl_down_sync(0xffffffffu, v, P.tpr < 32 ? P.tpr : 0);
            if (li == 0 && rr < nr) {
                if constexpr (FMT == FMT_A8) {
                    a.y[r0 + rr] = a8w8_dequant(v, a8_xs, a8_ws[r0 + rr]);
                } else if (pair) {
                    if ((rr & 1) == 0) epi_pair(a, r0 + rr, v, vn);
                } else {
                    epi_row<AR>(a, r0 + rr, v, best);
                }
            }
            crow += P.rpc;
        } else {
            const int u0 = cc * P.kc;
            const int nu = min(P.kc, P.U - u0);
            const int64_t row = row_begin + crow;
            if (UPL > 0 && nu == P.kc)
                acc += chunk_full_dot<FMT, DEBUG, (UPL > 0 ? UPL : 2)>(st, P.kc, lane, u0, xr, P.U, a.dots, row);
            else
                acc += chunk_row_dot<FMT, DEBUG>(st, P.kc, lane, 32, P.upl, nu, u0, xr, P.U, a.dots, row);
            const bool row_done = ++cc == P.nchunk;
            if (row_done || q == nq - 1) {
                const Acc v = warp_sum_acc(acc);
                acc = 0;
                if (lane == 0) (first_part ? pacc0 : pacc1)[row - cr0] = v;
                if (row_done) {
                    cc = 0;
                    ++crow;
                    first_part = true;
                }
            }
        }
        __syncwarp();  // every lane is done reading stage s
        if (lane == 0 && q + S < nq) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(s);
        }
        if (++s == S) {
            s = 0;
            parity ^= 1u;
        }
    }
    if (P.rpc == 1) {
        __syncthreads();  // all row partials of the CTA are in shared memory
        if (tid == 0) stamp_point(a.stamp, a.stamp_stride, 5);
        const int64_t nrows = cr1 - cr0;
        if constexpr (FMT == FMT_A8) {
            for (int64_t r = tid; r < nrows; r += kGemvThreads)
                a.y[cr0 + r] = a8w8_dequant(pacc0[r] + pacc1[r], a8_xs, a8_ws[cr0 + r]);
        } else if (a.epi == EPI_SWIGLU && a.xq_img != nullptr) {
            // the outputs also go to shared memory (the rings: every copy has
            // landed and been read) for the image of the down projection
            float* hs = reinterpret_cast<float*>(rings);
            const int64_t jb = (cr0 / 2) & ~31LL;
            for (int64_t r = 2 * (int64_t)tid; r < nrows; r += 2 * kGemvThreads) {
                const float v = swiglu(part0[r] + part1[r], part0[r + 1] + part1[r + 1]);
                a.y[(cr0 + r) / 2] = v;
                hs[(cr0 + r) / 2 - jb] = v;
            }
            __syncthreads();
            swiglu_quantise(a, cr0 / 2, cr1 / 2, tid, hs);
        } else if (pair) {
            for (int64_t r = 2 * (int64_t)tid; r < nrows; r += 2 * kGemvThreads)
                epi_pair(a, cr0 + r, part0[r] + part1[r], part0[r + 1] + part1[r + 1]);
        } else {
            for (int64_t r = tid; r < nrows; r += kGemvThreads) epi_row<AR>(a, cr0 + r, part0[r] + part1[r], best);
        }
    }
    if (a.epi == EPI_ARGMAX) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0 && best != 0ull) atomicMax(a.amax, best);
    }
    if (AR && a.epi == EPI_PUSH) {
        // every row of this CTA is on every rank: release the collective
        __threadfence_system();
        __syncthreads();
        if (tid < a.ar_world) {
            const unsigned long long seq =
                a.ar_st->step * (unsigned long long)a.ar_per_step + (unsigned long long)a.ar_idx + 1ull;
            st_release_sys_u64(a.ar_flag_dst[tid] + blockIdx.x, seq);
        }
    }
    if (a.stamp != nullptr) {  // uniform over the grid
        __syncthreads();
        if (tid == 0) stamp_point(a.stamp, a.stamp_stride, 2);
    }
}


}  // namespace b200
