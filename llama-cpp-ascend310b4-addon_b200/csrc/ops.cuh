// ops.cuh -- the decode step's neighbour ops as standalone kernels, for a
// backend that runs a ggml graph op by op (the model driver fuses all of them
// into the GEMV prologues and epilogues).  Semantics follow ggml-cpu:
//   RMS_NORM  y = x / sqrt(mean(x^2) + eps), the sum of squares in double
//             (then MUL by the norm weight, fused when w != NULL)
//   ROPE      NORM mode (adjacent pairs), theta_i = pos * base^(-2i/D) built
//             by repeated fp32 multiplication
//   SET_ROWS  f32 rows -> f16 rows at int64 indices (the KV-cache write)
//   GET_ROWS  Q4_0 rows -> f32 (d * (q - 8)) at int32 indices (embedding)
//   SWIGLU    silu(g) * u with silu(g) = g / (1 + exp(-g))
//   ADD, ARGMAX (first maximum)
// Out-of-range indices are skipped (the output row is zero-filled for
// GET_ROWS) and recorded as B200_DEVSTATUS_BOUNDS.
#pragma once

#include "args.h"
#include "common.cuh"

namespace b200 {

constexpr int kOpThreads = 256;

// One CTA per row.
__global__ void __launch_bounds__(kOpThreads) rms_norm_kernel(const float* x, const float* w, float* y, int64_t n,
                                                              float eps) {
    const float* xr = x + (int64_t)blockIdx.x * n;
    float* yr = y + (int64_t)blockIdx.x * n;
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += kOpThreads) {
        const float v = xr[i];
        s += (double)__fmul_rn(v, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __shared__ double part[kOpThreads / 32];
    __shared__ float scale_s;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) part[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int i = 0; i < kOpThreads / 32; ++i) t += part[i];
        const float mean = (float)(t / (double)n);
        scale_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }
    __syncthreads();
    const float scale = scale_s;
    for (int64_t i = threadIdx.x; i < n; i += kOpThreads) {
        float v = __fmul_rn(xr[i], scale);
        if (w != nullptr) v = __fmul_rn(v, w[i]);
        yr[i] = v;
    }
}

// One thread per (token, head, pair).
__global__ void rope_norm_kernel(const float* x, float* y, const int32_t* pos, int64_t n_tokens, int n_heads,
                                 int head_dim, float theta_scale) {
    const int64_t pairs = (int64_t)n_heads * (head_dim / 2);
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_tokens * pairs) return;
    const int64_t t = i / pairs;
    const int j = (int)(i - t * pairs) % (head_dim / 2);  // pair within the head
    float theta = (float)pos[t];
    for (int k = 0; k < j; ++k) theta = __fmul_rn(theta, theta_scale);
    float sn, cs;
    sincosf(theta, &sn, &cs);
    const int64_t e = 2 * i;
    const float x0 = x[e], x1 = x[e + 1];
    y[e] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
    y[e + 1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
}

__global__ void set_rows_f16_kernel(const float* src, const int64_t* idx, uint8_t* dst, int64_t n, int64_t nrows,
                                    int64_t dst_stride, int64_t dst_rows) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * nrows) return;
    const int64_t r = i / n, c = i - r * n;
    const int64_t d = idx[r];
    if (d < 0 || d >= dst_rows) {
        if (c == 0) record_status(B200_DEVSTATUS_BOUNDS);
        return;
    }
    reinterpret_cast<uint16_t*>(dst + d * dst_stride)[c] = f2h(src[i]);
}

__global__ void get_rows_q4_0_kernel(const uint8_t* table, const int32_t* idx, float* dst, int64_t n, int64_t nidx,
                                     int64_t vocab) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * nidx) return;
    const int64_t r = i / n, c = i - r * n;
    const int64_t row = idx[r];
    if (row < 0 || row >= vocab) {
        if (c == 0) record_status(B200_DEVSTATUS_BOUNDS);
        dst[i] = 0.f;
        return;
    }
    const uint8_t* blk = table + (row * (n / 32) + c / 32) * 18;
    const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
    const int j = (int)(c & 31);
    const int q = j < 16 ? (blk[2 + j] & 0x0f) : (blk[2 + j - 16] >> 4);
    dst[i] = __fmul_rn((float)(q - 8), d);
}

// GET_ROWS from the packed Q4_0 layout (the table is also the lm_head's
// GEMV operand, so a tied embedding needs one copy): row r at r * rs,
// nibbles qs[U][16] then the scales d[U].
__global__ void get_rows_q4_0_packed_kernel(const uint8_t* table, const int32_t* idx, float* dst, int64_t n,
                                            int64_t nidx, int64_t vocab, int64_t rs) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * nidx) return;
    const int64_t r = i / n, c = i - r * n;
    const int64_t row = idx[r];
    if (row < 0 || row >= vocab) {
        if (c == 0) record_status(B200_DEVSTATUS_BOUNDS);
        dst[i] = 0.f;
        return;
    }
    const int64_t U = n / 32, b = c / 32;
    const uint8_t* base = table + row * rs;
    const float d = h2f((uint16_t)(base[16 * U + 2 * b] | (base[16 * U + 2 * b + 1] << 8)));
    const int j = (int)(c & 31);
    const int q = j < 16 ? (base[16 * b + j] & 0x0f) : (base[16 * b + j - 16] >> 4);
    dst[i] = __fmul_rn((float)(q - 8), d);
}

__global__ void swiglu_kernel(const float* g, const float* u, float* y, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = g[i];
    y[i] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u[i]);
}

__global__ void add_kernel(const float* a, const float* b, float* y, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fadd_rn(a[i], b[i]);
}

// ggml MUL with src1 the same shape (nb == n) or one row broadcast over
// the rows of src0 (n % nb == 0).
__global__ void mul_kernel(const float* a, const float* b, float* y, int64_t n, int64_t nb) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fmul_rn(a[i], b[nb == n ? i : i % nb]);
}

// One CTA: packed (value, ~index) keys, so the first maximum wins.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* x, int64_t n, int32_t* out) {
    unsigned long long best = 0ull;
    for (int64_t i = threadIdx.x; i < n; i += 1024) {
        const unsigned int b = __float_as_uint(x[i]);
        const unsigned int key = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
        const unsigned long long k = ((unsigned long long)key << 32) | (0xffffffffu - (unsigned int)i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    __shared__ unsigned long long wb[32];
    if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < 32; ++i) best = wb[i] > best ? wb[i] : best;
        best = wb[0] > best ? wb[0] : best;
        out[0] = (int32_t)(0xffffffffu - (unsigned int)(best & 0xffffffffull));
    }
}

}  // namespace b200
