// model_ops.cuh -- small kernels around the decode step: synthetic weight and
// KV generation, embedding lookup (GET_ROWS of a Q4_0 table), the step's
// device state (token, position, argmax) and fills.
#pragma once

#include "args.h"
#include "common.cuh"

namespace b200 {

__host__ __device__ inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// ln(u) for a normal float u > 0: u = m 2^e with m in [sqrt(1/2), sqrt(2)),
// ln m = 2 atanh(s) = 2 s (1 + s^2/3 + ... + s^10/11) with s = (m-1)/(m+1),
// |s| < 0.1716 (series truncation < 1e-10).  Only correctly rounded f32
// operations (add, mul, div, fma), so a host restatement with the same
// steps gives the same bits.
__device__ __forceinline__ float synth_ln(float u) {
    const unsigned b = __float_as_uint(u);
    int e = (int)((b >> 23) & 0xffu) - 127;
    float m = __uint_as_float((b & 0x7fffffu) | 0x3f800000u);
    if (m > 1.41421356f) {
        m = __fmul_rn(m, 0.5f);
        e += 1;
    }
    const float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
    const float s2 = __fmul_rn(s, s);
    float p = __fmaf_rn(s2, 0.0909090909f, 0.111111111f);
    p = __fmaf_rn(s2, p, 0.142857143f);
    p = __fmaf_rn(s2, p, 0.2f);
    p = __fmaf_rn(s2, p, 0.333333333f);
    p = __fmaf_rn(s2, p, 1.0f);
    return __fmaf_rn((float)e, 0.693147181f, __fmul_rn(__fmul_rn(2.0f, s), p));
}

// cos(2 pi t) for t in [0, 1): folded to a in [0, 1/4] (cos is even and
// cos(2 pi (1/2 - a)) = -cos(2 pi a); each fold is exact in f32), then the
// Taylor series of cos(x), x = 2 pi a <= pi/2, through x^16 (error < 1e-12).
__device__ __forceinline__ float synth_cos2pi(float t) {
    float a = t > 0.5f ? __fsub_rn(1.0f, t) : t;
    const bool flip = a > 0.25f;
    if (flip) a = __fsub_rn(0.5f, a);
    const float x = __fmul_rn(a, 6.28318531f);
    const float x2 = __fmul_rn(x, x);
    float p = __fmaf_rn(x2, 4.77947733e-14f, -1.14707456e-11f);
    p = __fmaf_rn(x2, p, 2.08767570e-9f);
    p = __fmaf_rn(x2, p, -2.75573192e-7f);
    p = __fmaf_rn(x2, p, 2.48015873e-5f);
    p = __fmaf_rn(x2, p, -1.38888889e-3f);
    p = __fmaf_rn(x2, p, 4.16666667e-2f);
    p = __fmaf_rn(x2, p, -0.5f);
    p = __fmaf_rn(x2, p, 1.0f);
    return flip ? -p : p;
}

// N(0, 1) by Box-Muller on two 24-bit uniforms drawn from
// splitmix64(seed_mixed ^ index * odd constant): r = sqrt(-2 ln u1),
// value r cos(2 pi u2).  Bit-identical to the CPU oracle's ref_synth_normal
// (same operations, all correctly rounded), so a host can regenerate the
// device's synthetic weights and KV cache exactly.
__device__ __forceinline__ float synth_normal(uint64_t seed_mixed, uint64_t index) {
    const uint64_t h = splitmix64(seed_mixed ^ (index * 0xD1B54A32D192ED03ull));
    const float u1 = __fmul_rn(__fadd_rn((float)(uint32_t)(h >> 40), 0.5f), 1.0f / 16777216.0f);
    const float u2 = __fmul_rn((float)(uint32_t)(h & 0xFFFFFFu), 1.0f / 16777216.0f);
    const float r = __fsqrt_rn(__fmul_rn(-2.0f, synth_ln(u1)));
    return __fmul_rn(r, synth_cos2pi(u2));
}

// ggml Q4_0 blocks of N(0, sigma^2) samples: local rows [0, nrows) are global
// rows row0 + r; local columns [0, ncols) are global columns col0 + c of a
// matrix with kglob columns.  One thread per block, ggml block layout out.
__global__ void synth_q4_0_kernel(uint64_t seed, float sigma, int64_t row0, int64_t nrows, int64_t col0,
                                  int64_t ncols, int64_t kglob, uint8_t* out) {
    const int64_t nb = ncols / 32;
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nrows * nb) return;
    const int64_t r = b / nb, cb = b - r * nb;
    const uint64_t sm = splitmix64(seed);
    const uint64_t base = (uint64_t)(row0 + r) * (uint64_t)kglob + (uint64_t)(col0 + cb * 32);
    float v[32];
    float amax = 0.f, mx = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        v[j] = __fmul_rn(sigma, synth_normal(sm, base + j));
        if (amax < fabsf(v[j])) {
            amax = fabsf(v[j]);
            mx = v[j];
        }
    }
    // quantize_row_q4_0_ref: d = max / -8, q = min(15, (int8)(x*id + 8.5f))
    const float d = __fdiv_rn(mx, -8.0f);
    const float id = d != 0.f ? __frcp_rn(d) : 0.f;
    // the block as nine 16-bit words (blocks are 18 bytes, so 2-byte aligned)
    uint16_t* blk = reinterpret_cast<uint16_t*>(out + b * 18);
    blk[0] = f2h(d);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
        unsigned pair = 0;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            // x * id + 8.5 lies in [0.5, 16.5]: truncation is the (int8_t) cast of the reference rule
            const int q0 = min((int)__fadd_rn(__fmul_rn(v[j + e], id), 8.5f), 15);
            const int q1 = min((int)__fadd_rn(__fmul_rn(v[16 + j + e], id), 8.5f), 15);
            pair |= (unsigned)(q0 | (q1 << 4)) << (8 * e);
        }
        blk[1 + j / 2] = (uint16_t)pair;
    }
}

// f16 N(0,1) rows: local element (r, c) of rows of `rl` elements takes the
// stream index base + r * rg + col0 + c (rg = global row length), so a
// tensor-parallel shard holds exactly the values of the unsharded tensor.
__global__ void synth_rows_f16_kernel(uint64_t seed, uint64_t base, int64_t nrows, int64_t rl, int64_t rg,
                                      int64_t col0, uint16_t* out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nrows * rl) return;
    const int64_t r = i / rl, c = i - r * rl;
    out[i] = f2h(synth_normal(splitmix64(seed), base + (uint64_t)(r * rg + col0 + c)));
}

__global__ void fill_f32_kernel(float* p, int64_t n, float v) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

// GET_ROWS of a Q4_0 table (ggml dequantize_row_q4_0: d * (q - 8)), plus the
// step bookkeeping that must precede the layers.
__global__ void embed_kernel(const uint8_t* table, int64_t d_model, int64_t vocab, StepState* st, float* x) {
    int tok = st->token;
    if (tok < 0 || tok >= vocab) {  // bad token id: record it and read row 0 instead
        if (blockIdx.x == 0 && threadIdx.x == 0) record_status(B200_DEVSTATUS_BOUNDS);
        tok = 0;
    }
    const int64_t nb = d_model / 32;
    const uint8_t* row = table + (int64_t)tok * nb * 18;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < d_model; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / 32, j = i % 32;
        const uint8_t* blk = row + b * 18;
        const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
        const int q = j < 16 ? (blk[2 + j] & 0x0f) : (blk[2 + j - 16] >> 4);
        x[i] = (float)(q - 8) * d;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        st->ctx = st->pos + 1;
        st->amax = 0ull;
        st->step += 1;
    }
}

// Image -> ggml block_q8_0: block b's q bytes 0..15 from plane 0, 16..31
// from plane 1, its scale from the f32 copy of the f16 value (exact).
__global__ void image_to_q8_0_kernel(const uint8_t* img, int64_t U, uint8_t* out) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= U) return;
    const float d = __int_as_float(reinterpret_cast<const int2*>(img + 32 * U)[b].x);
    // 17 16-bit words per block (34 bytes, so 2-byte aligned); the planes
    // hold the q bytes of each half-block as four 32-bit words
    uint16_t* o = reinterpret_cast<uint16_t*>(out + b * 34);
    o[0] = f2h(d);
    const int4 lo = reinterpret_cast<const int4*>(img)[b];
    const int4 hi = reinterpret_cast<const int4*>(img + 16 * U)[b];
    const int w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        o[1 + 2 * i] = (uint16_t)((unsigned)w[i] & 0xffffu);
        o[2 + 2 * i] = (uint16_t)((unsigned)w[i] >> 16);
    }
}

__global__ void finish_step_kernel(StepState* st) {
    const unsigned long long a = st->amax;
    const int idx = (int)(0xffffffffu - (unsigned int)(a & 0xffffffffull));
    st->next = idx;
    if (st->advance) {
        st->token = idx;
        st->pos = st->pos + 1;
    }
}

}  // namespace b200
