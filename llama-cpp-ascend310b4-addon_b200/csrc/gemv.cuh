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

#include "args.h"
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

// Bytes of the activation region at the start of shared memory.
B200_HD inline int64_t gemv_x_bytes(int fmt, const GemvPlan& p) {
    if (fmt == FMT_Q4 || fmt == FMT_Q8) return pad16(40 * (int64_t)p.U);  // xq[U][32] + {d, sum}[U]
    return pad16(2 * p.k);                                                // f16 x[K]
}

// ------------------------------------------------------------- epilogues

__device__ __forceinline__ void epi_row(const GemvArgs& a, int64_t n, float v, unsigned long long& best) {
    if (a.epi == EPI_STORE) {
        a.y[n] = v;
    } else if (a.epi == EPI_ADD) {
        a.y[n] = __fadd_rn(v, a.res[n]);
    } else if (a.epi == EPI_ARGMAX) {
        a.y[n] = v;
        const unsigned long long k = pack_argmax(v, n + a.row_offset);
        best = k > best ? k : best;
    }
}

// Rows n (even) and n + 1.
__device__ __forceinline__ void epi_pair(const GemvArgs& a, int64_t n, float v0, float v1) {
    if (a.epi == EPI_SWIGLU) {
        // ggml swiglu: silu(g) * u with silu(g) = g / (1 + exp(-g))
        const float sg = __fdiv_rn(v0, __fadd_rn(1.0f, expf(-v0)));
        a.y[n / 2] = __fmul_rn(sg, v1);
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

// Contribution of one unit: `row` is the staged chunk row, `pw` its plane
// width, `i` the unit's index in the chunk row, `u` its index in the full row.
template <int FMT, bool DEBUG>
__device__ __forceinline__ float unit_dot(const uint8_t* row, int pw, int i, int u, const uint8_t* xr,
                                          int32_t* dots, int64_t nrow, int U) {
    if constexpr (FMT == FMT_F16) {
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
                    const int j = e * 8 + t * 2;  // element index within the half
                    const unsigned int w = wq[j >> 2];
                    const int sh = 8 * (j & 3) + 4 * hf;
                    const int q0 = (int)((w >> sh) & 0xfu) - 8;
                    const int q1 = (int)((w >> (sh + 8)) & 0xfu) - 8;
                    p = fmaf((float)q0, xf.x, p);
                    p = fmaf((float)q1, xf.y, p);
                }
            }
        }
        return dw * p;
    } else {
        const int4* xq = reinterpret_cast<const int4*>(xr + 32 * u);
        const int4 xa = xq[0], xb = xq[1];
        const int2 ds = reinterpret_cast<const int2*>(xr + 32 * U)[u];
        const float xd = __int_as_float(ds.x);
        int sumi = 0;
        float dw;
        if constexpr (FMT == FMT_Q4) {
            const uint4 qv = *reinterpret_cast<const uint4*>(row + 16 * i);
            dw = h2f(*reinterpret_cast<const uint16_t*>(row + 16 * pw + 2 * i));
            sumi = dp4a((int)(qv.x & 0x0f0f0f0fu), xa.x, sumi);
            sumi = dp4a((int)(qv.y & 0x0f0f0f0fu), xa.y, sumi);
            sumi = dp4a((int)(qv.z & 0x0f0f0f0fu), xa.z, sumi);
            sumi = dp4a((int)(qv.w & 0x0f0f0f0fu), xa.w, sumi);
            sumi = dp4a((int)((qv.x >> 4) & 0x0f0f0f0fu), xb.x, sumi);
            sumi = dp4a((int)((qv.y >> 4) & 0x0f0f0f0fu), xb.y, sumi);
            sumi = dp4a((int)((qv.z >> 4) & 0x0f0f0f0fu), xb.z, sumi);
            sumi = dp4a((int)((qv.w >> 4) & 0x0f0f0f0fu), xb.w, sumi);
            sumi -= 8 * ds.y;  // nibbles are stored +8
        } else {
            const uint4 lo = *reinterpret_cast<const uint4*>(row + 16 * i);
            const uint4 hi = *reinterpret_cast<const uint4*>(row + 16 * pw + 16 * i);
            dw = h2f(*reinterpret_cast<const uint16_t*>(row + 32 * pw + 2 * i));
            sumi = dp4a((int)lo.x, xa.x, sumi);
            sumi = dp4a((int)lo.y, xa.y, sumi);
            sumi = dp4a((int)lo.z, xa.z, sumi);
            sumi = dp4a((int)lo.w, xa.w, sumi);
            sumi = dp4a((int)hi.x, xb.x, sumi);
            sumi = dp4a((int)hi.y, xb.y, sumi);
            sumi = dp4a((int)hi.z, xb.z, sumi);
            sumi = dp4a((int)hi.w, xb.w, sumi);
        }
        if constexpr (DEBUG) dots[nrow * U + u] = sumi;
        return (dw * xd) * (float)sumi;
    }
}

// ------------------------------------------------------------ the kernel

template <int FMT, bool DEBUG>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvPlan& P = a.p;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = a.stages;
    const int64_t xbytes = gemv_x_bytes(FMT, P);
    uint8_t* xr = smem;
    uint8_t* rings = smem + xbytes;
    uint8_t* ring = rings + (int64_t)warp * S * P.stage_bytes;
    uint64_t* bars_all = reinterpret_cast<uint64_t*>(rings + (int64_t)kGemvWarps * S * P.stage_bytes);
    uint64_t* bars = bars_all + warp * S;
    float* red = reinterpret_cast<float*>(bars_all + kGemvWarps * S);  // [kGemvWarps]

    // ---- this warp's rows ----
    const bool pair = a.epi == EPI_SWIGLU || a.epi == EPI_QKV;
    const int64_t item_rows = P.rpc > 1 ? P.rpc : (pair ? 2 : 1);
    const int64_t items = (P.n + item_rows - 1) / item_rows;
    const int64_t gw = (int64_t)blockIdx.x * kGemvWarps + warp, ngw = (int64_t)gridDim.x * kGemvWarps;
    const int64_t it0 = gw * items / ngw, it1 = (gw + 1) * items / ngw;
    const int64_t row_begin = it0 * item_rows;
    const int64_t row_end = min(it1 * item_rows, P.n);
    const int64_t nq = P.rpc > 1 ? (it1 - it0) : (row_end - row_begin) * P.nchunk;

    // Lane 0 only: stage chunk q into ring slot s.
    auto issue = [&](int64_t q, int s) {
        uint8_t* dst = ring + (int64_t)s * P.stage_bytes;
        uint64_t* bar = &bars[s];
        if (P.rpc > 1) {
            const int64_t r0 = row_begin + q * P.rpc;
            const int64_t nr = min((int64_t)P.rpc, P.n - r0);
            const uint32_t bytes = (uint32_t)(nr * P.rs);
            mbar_arrive_expect_tx(bar, bytes);
            bulk_g2s(dst, a.w + r0 * P.rs, bytes, bar);
        } else {
            const int64_t row = row_begin + q / P.nchunk;
            const int u0 = (int)(q % P.nchunk) * P.kc;
            const int nu = min(P.kc, P.U - u0);
            const uint8_t* base = a.w + row * P.rs;
            const uint32_t b0 = (uint32_t)(16 * nu);
            if constexpr (FMT == FMT_F16) {
                mbar_arrive_expect_tx(bar, b0);
                bulk_g2s(dst, base + 16 * (int64_t)u0, b0, bar);
            } else if constexpr (FMT == FMT_Q8) {
                const uint32_t b1 = (uint32_t)pad16(2 * nu);
                mbar_arrive_expect_tx(bar, 2 * b0 + b1);
                bulk_g2s(dst, base + 16 * (int64_t)u0, b0, bar);
                bulk_g2s(dst + 16 * P.kc, base + 16 * (int64_t)P.U + 16 * (int64_t)u0, b0, bar);
                bulk_g2s(dst + 32 * P.kc, base + 32 * (int64_t)P.U + 2 * (int64_t)u0, b1, bar);
            } else {
                const uint32_t b1 = (uint32_t)pad16(2 * nu);
                mbar_arrive_expect_tx(bar, b0 + b1);
                bulk_g2s(dst, base + 16 * (int64_t)u0, b0, bar);
                bulk_g2s(dst + 16 * P.kc, base + 16 * (int64_t)P.U + 2 * (int64_t)u0, b1, bar);
            }
        }
    };

    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        mbar_fence_init();
        for (int s = 0; s < S && s < nq; ++s) issue(s, s);
    }

    // ---- prologue: the activation, once per CTA, into shared memory ----
    float nscale = 1.f;
    const bool norm = a.pro == PRO_RMSNORM;
    if (norm) {
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
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) tot += red[w];
        const float mean = __fdiv_rn(tot, (float)a.k);
        nscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
    }
    if constexpr (FMT == FMT_Q4 || FMT == FMT_Q8) {
        int4* xq = reinterpret_cast<int4*>(xr);
        int2* xds = reinterpret_cast<int2*>(xr + 32 * (int64_t)P.U);
        for (int b = tid; b < P.U; b += kGemvThreads) {
            const float4* src = reinterpret_cast<const float4*>(a.x + (int64_t)b * 32);
            const float4* wn = reinterpret_cast<const float4*>(a.norm_w + (int64_t)b * 32);
            auto load = [&](int e) -> float4 {
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
            xq[2 * b] = make_int4(q[0], q[1], q[2], q[3]);
            xq[2 * b + 1] = make_int4(q[4], q[5], q[6], q[7]);
            xds[b] = make_int2(__float_as_int(d), qs);
            if (a.xq_out != nullptr && blockIdx.x == 0) store_block_q8_0(a.xq_out + (int64_t)b * 34, dh, q);
        }
    } else {
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

    // ---- stream this warp's chunks ----
    float acc = 0.f, pend = 0.f;
    unsigned long long best = 0ull;
    for (int64_t q = 0; q < nq; ++q) {
        const int s = (int)(q % S);
        const uint32_t parity = (uint32_t)((q / S) & 1);
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bars[s], parity));
        if (!ok) {
            if (lane == 0)
                for (int64_t q2 = q + 1; q2 < nq && q2 < q + S; ++q2)
                    mbar_wait_bounded(&bars[q2 % S], (uint32_t)((q2 / S) & 1));
            return;
        }
        const uint8_t* st = ring + (int64_t)s * P.stage_bytes;
        if (P.rpc > 1) {
            const int64_t r0 = row_begin + q * P.rpc;
            const int rr = lane / P.tpr, li = lane - rr * P.tpr;
            const int nr = (int)min((int64_t)P.rpc, P.n - r0);
            float v = 0.f;
            if (rr < nr) {
                const uint8_t* row = st + (int64_t)rr * P.rs;
                for (int j = 0; j < P.upl; ++j) {
                    const int u = li + P.tpr * j;
                    if (u < P.U) v += unit_dot<FMT, DEBUG>(row, P.U, u, u, xr, a.dots, r0 + rr, P.U);
                }
            }
            v = group_sum(v, P.tpr);
            const float vn = __shfl_down_sync(0xffffffffu, v, P.tpr < 32 ? P.tpr : 0);
            if (li == 0 && rr < nr) {
                if (pair) {
                    if ((rr & 1) == 0) epi_pair(a, r0 + rr, v, vn);
                } else {
                    epi_row(a, r0 + rr, v, best);
                }
            }
        } else {
            const int c = (int)(q % P.nchunk);
            const int u0 = c * P.kc;
            const int nu = min(P.kc, P.U - u0);
            const int64_t row = row_begin + q / P.nchunk;
            for (int j = 0; j < P.upl; ++j) {
                const int i = lane + 32 * j;
                if (i < nu) acc += unit_dot<FMT, DEBUG>(st, P.kc, i, u0 + i, xr, a.dots, row, P.U);
            }
            if (c == P.nchunk - 1) {
                const float v = warp_sum(acc);
                acc = 0.f;
                if (lane == 0) {
                    if (pair) {
                        if (((row - row_begin) & 1) == 0)
                            pend = v;
                        else
                            epi_pair(a, row - 1, pend, v);
                    } else {
                        epi_row(a, row, v, best);
                    }
                }
            }
        }
        __syncwarp();  // every lane is done reading stage s
        if (lane == 0 && q + S < nq) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(q + S, s);
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
}

}  // namespace b200
