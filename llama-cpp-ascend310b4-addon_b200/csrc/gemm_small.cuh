// gemm_small.cuh -- small-M F16 matmul for decode batches of up to 8 tokens:
// y[m][n] = sum_k w[n][k] * f16(x[m][k]) with fp32 accumulation (ggml-cpu's
// F16 mul_mat: src1 rounded to f16, f32 dot).  The reference serves M <= 8
// from its FRACTAL_NZ weight copy (ggml_cann_mat_mul_fp, patch:1290-1300);
// here the weight streams once from HBM for all M columns.
//
// Tensor cores, mma.sync m16n8k16 with the weight as A (16 rows x 16 k) and
// the M <= 8 activation rows as B (n = 8; columns past M are zero), so one
// 16-row weight tile meets every token in one instruction.  4 warps per CTA;
// warp w of the grid owns a contiguous range of 16-row tiles and streams each
// tile's K in chunks of 256 halves through its own ring: a chunk is 4 TMA
// boxes of 64 halves x 16 rows (2-D tensor map over [n][k], 128-byte
// swizzle, out-of-range rows and columns zero-filled), read back with
// ldmatrix at the swizzled addresses.  The activation sits in shared memory
// as f16 rows padded to 64 k + 8 halves (conflict-free B fragments).  Each
// chunk's 256-k partial comes from two fresh mma accumulators (even and odd
// k steps, two independent chains) and is added to the tile's fp32 sum in
// registers: the tensor core's internal accumulation is not IEEE fp32 over
// long k.  Work is HBM-bound: 8 columns of 16-bit weights are at most 8 FLOP
// per byte.
#pragma once

#include "args.h"
#include "common.cuh"
#include "fa_mma.cuh"

namespace b200 {

constexpr int kSmWarps = 4;
constexpr int kSmThreads = 32 * kSmWarps;
constexpr int kSmChunk = 256;                   // halves of K per ring stage
constexpr int kSmBoxes = kSmChunk / 64;         // TMA boxes per stage
constexpr int kSmBoxBytes = 64 * 16 * 2;        // one TMA box: 64 halves x 16 rows
constexpr int kSmStageBytes = kSmBoxes * kSmBoxBytes;
constexpr int kSmStagesMax = 4;

// 2-D tiled TMA load of one box (x: the k coordinate, a multiple of 64
// halves; y: the row).  Completion is counted on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

B200_HD inline int64_t small_m_xstride(int64_t k) { return ((k + 63) / 64) * 64 + 8; }

// Shared memory: 1 KiB of alignment slack, the rings, the activation rows,
// the ring barriers.
B200_HD inline size_t small_m_smem_bytes(int64_t k, int m, int stages) {
    return 1024 + (size_t)kSmWarps * stages * kSmStageBytes + (size_t)m * small_m_xstride(k) * 2 +
           (size_t)kSmWarps * stages * sizeof(uint64_t);
}

__global__ void __launch_bounds__(kSmThreads) gemm_small_m_kernel(const __grid_constant__ SmallMArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sbase = (smem_u32(smem) + 1023u) & ~1023u;  // 128-byte swizzle: 1 KiB aligned boxes
    uint8_t* sp = smem + (sbase - smem_u32(smem));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = a.stages;
    __half* xs = reinterpret_cast<__half*>(sp + (size_t)kSmWarps * S * kSmStageBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(xs + (size_t)a.m * a.xstride) + warp * S;
    const uint32_t ring = sbase + (uint32_t)(warp * S * kSmStageBytes);

    // this warp's tiles [t0, t1) and their chunks, tile-major
    const int64_t T = (a.n + 15) / 16;
    const int64_t gw = (int64_t)blockIdx.x * kSmWarps + warp, ngw = (int64_t)gridDim.x * kSmWarps;
    const int64_t t0 = gw * T / ngw, t1 = (gw + 1) * T / ngw;
    const int nck = (int)((a.k + kSmChunk - 1) / kSmChunk);
    const int64_t nq = (t1 - t0) * nck;

    auto issue = [&](int64_t q, int s) {  // lane 0
        const int64_t tile = t0 + q / nck;
        const int c = (int)(q % nck);
        mbar_arrive_expect_tx(&bars[s], kSmStageBytes);
        const uint32_t dst = ring + (uint32_t)(s * kSmStageBytes);
#pragma unroll
        for (int b = 0; b < kSmBoxes; ++b)
            tma_load_2d(dst + b * kSmBoxBytes, &a.tmw, c * kSmChunk + 64 * b, (int)(tile * 16), &bars[s]);
    };
    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        mbar_fence_init();
        for (int s = 0; s < S && s < nq; ++s) issue(s, s);
    }
    // activation rows -> f16 (zero past k), while the first copies fly.  Each
    // thread issues a batch of independent loads before converting any (16-byte
    // loads when the rows allow), so the fill costs a few load latencies, not
    // one per element.
    const int xw = (int)a.xstride;
    if (a.xvec) {
        const int q4 = xw / 4;  // float4 units per padded row (xstride is a multiple of 8)
        const int total = a.m * q4;
        constexpr int RB = 8;
        for (int base = 0; base < total; base += RB * kSmThreads) {
            float4 v[RB];
#pragma unroll
            for (int i = 0; i < RB; ++i) {
                const int u = base + tid + i * kSmThreads;
                const int r = u / q4, c4 = u - r * q4;
                v[i] = (u < total && 4 * c4 < a.k)
                           ? *reinterpret_cast<const float4*>(a.x + (int64_t)r * a.ldx + 4 * c4)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < RB; ++i) {
                const int u = base + tid + i * kSmThreads;
                if (u < total) {
                    const int r = u / q4, c4 = u - r * q4;
                    __half2* d = reinterpret_cast<__half2*>(xs + (int64_t)r * xw + 4 * c4);
                    d[0] = __floats2half2_rn(v[i].x, v[i].y);
                    d[1] = __floats2half2_rn(v[i].z, v[i].w);
                }
            }
        }
    } else {
        const int total = a.m * xw;
        constexpr int RB = 16;
        for (int base = 0; base < total; base += RB * kSmThreads) {
            float v[RB];
#pragma unroll
            for (int i = 0; i < RB; ++i) {
                const int u = base + tid + i * kSmThreads;
                const int r = u / xw, c = u - r * xw;
                v[i] = (u < total && c < a.k) ? a.x[(int64_t)r * a.ldx + c] : 0.f;
            }
#pragma unroll
            for (int i = 0; i < RB; ++i) {
                const int u = base + tid + i * kSmThreads;
                if (u < total) xs[u] = __float2half_rn(v[i]);
            }
        }
    }
    __syncthreads();

    const int g = lane >> 2, t = lane & 3;    // mma fragment coordinates
    const int mi = lane >> 3, ri = lane & 7;  // ldmatrix address lanes
    const int ar = ri + 8 * (mi & 1);         // A tile row this lane addresses
    const __half* xg = xs + (size_t)(g < a.m ? g : 0) * xw + 2 * t;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    int s = 0;
    uint32_t parity = 0;
    for (int64_t q = 0; q < nq; ++q) {
        const int64_t tile = t0 + q / nck;
        const int ch = (int)(q % nck);
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[s], parity))) {
            if (lane == 0) {  // let the copies in flight (stages q .. q + S - 1) land before the CTA exits
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
            break;
        }
        const uint32_t st = ring + (uint32_t)(s * kSmStageBytes);
        float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int b = 0; b < kSmBoxes; ++b) {
            const int kb = ch * kSmChunk + 64 * b;
            if (kb >= a.k) break;  // boxes past k are zero: skip them
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                uint32_t af[4];
                const int gk = 2 * ks + (mi >> 1);  // 16-byte granule of the row
                ldsm_x4(af, st + (uint32_t)(b * kSmBoxBytes + ar * 128 + ((gk ^ (ar & 7)) << 4)));
                uint32_t b0 = 0u, b1 = 0u;
                if (g < a.m) {
                    const __half* xr = xg + kb + 16 * ks;
                    b0 = *reinterpret_cast<const uint32_t*>(xr);
                    b1 = *reinterpret_cast<const uint32_t*>(xr + 8);
                }
                mma_16816((ks & 1) ? c1 : c0, af, b0, b1);
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) c[e] += c0[e] + c1[e];
        __syncwarp();  // every lane is done reading stage s
        if (lane == 0 && q + S < nq) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(q + S, s);
        }
        if (++s == S) {
            s = 0;
            parity ^= 1u;
        }
        if (ch == nck - 1) {
            // c: (row g, column 2t), (row g, 2t + 1), (row g + 8, 2t), (row g + 8, 2t + 1)
            const int64_t r0 = tile * 16 + g, r1 = r0 + 8;
            const int m0 = 2 * t, m1 = 2 * t + 1;
            if (m0 < a.m) {
                if (r0 < a.n) a.y[m0 * a.ldy + r0] = c[0];
                if (r1 < a.n) a.y[m0 * a.ldy + r1] = c[2];
            }
            if (m1 < a.m) {
                if (r0 < a.n) a.y[m1 * a.ldy + r0] = c[1];
                if (r1 < a.n) a.y[m1 * a.ldy + r1] = c[3];
            }
            c[0] = c[1] = c[2] = c[3] = 0.f;
        }
    }
}

}  // namespace b200
