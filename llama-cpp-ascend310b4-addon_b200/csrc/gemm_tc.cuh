// gemm_tc.cuh -- prefill MUL_MAT with an F16 weight (many activation
// columns) on the 5th-generation tensor cores: tcgen05.mma with the
// accumulator in tensor memory, operands staged by TMA.
//
//   Y[j][r] = sum_i W[r][i] * X16[j][i]     r < n (weight rows), j < m (tokens)
//
// One CTA computes a 128 x BN tile: 128 weight rows (the MMA's M side) by BN
// tokens (its N side, 64 / 128 / 256), in two BN-column tensor-memory
// accumulators of the 128 lanes.  K runs in stages of 64 halves (one
// 128-byte swizzle row): thread 0 issues the two TMA boxes of a stage (W 64
// x 128, X 64 x BN, both K-major with the 128-byte swizzle) into a 4-stage
// mbarrier ring; thread 32 issues the stage's four K = 16 MMAs and commits
// them to the stage's "empty" barrier, which hands the slot back to thread
// 0.  Every 8 stages (a segment) the MMAs switch accumulator and the
// finished one is committed to the eight epilogue warps, which add it into
// fp32 registers with tcgen05.ld (two warps per 32-lane quarter, half the
// columns each) and hand it back; at the end each thread stores its row's
// sums (a warp writes 32 consecutive weight rows of one token: 128-byte
// stores).  Every wait is bounded; a CTA that gives up lets its copies
// land, drains the MMAs it issued and frees its tensor memory.
// X16 is the activation converted to f16 first (ggml-cpu converts src1 to
// the F16 weight's vec_dot_type the same way).
#pragma once

#include "args.h"
#include "common.cuh"
#include "gemm_small.cuh"  // tma_load_2d

namespace b200 {

constexpr int kTcBM = 128;       // weight rows per CTA (MMA M)
constexpr int kTcBK = 64;        // halves of K per stage: one 128-byte swizzle row
constexpr int kTcStages = 4;

struct TcArgs {
    CUtensorMap tmw;  // W [n][k] f16, boxes 64 x 128, 128-byte swizzle
    CUtensorMap tmx;  // X16 [m][k] f16, boxes 64 x BN, 128-byte swizzle
    float* y;         // [m][ldy] f32
    int64_t n, m, k, ldy;
};

B200_HD constexpr uint32_t tc_stage_bytes(int bn) { return (uint32_t)(kTcBM + bn) * 128u; }
B200_HD constexpr size_t tc_smem_bytes(int bn) { return (size_t)kTcStages * tc_stage_bytes(bn) + 1024; }

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte
// swizzle layout: rows of 128 bytes, 8-row groups 1024 bytes apart (stride
// byte offset), start address 1024-aligned (base offset 0), descriptor
// version 1 (bits 46-47), layout 2 = 128-byte swizzle (bits 61-63).  The
// leading byte offset is unused for this layout (one swizzle row spans the
// stage's K).  Advancing K by 16 halves within the row adds 32 bytes to the
// start address (2 in its 16-byte units).
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: D f32 (bits 4-5 = 1), A and B f16
// (bits 7-9, 10-12 = 0), both K-major (bits 15, 16 = 0), N >> 3 in bits
// 17-22, M >> 4 in bits 24-28.
template <int BN>
__device__ __forceinline__ constexpr uint32_t tc_idesc_f16() {
    return (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kTcBM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t idesc, int acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(da), "l"(db), "r"(idesc), "r"(acc));
}

// Arrives on `bar` once every tcgen05 operation this thread issued before
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive 32-bit columns of this warp's 32 lanes (lane = thread).
__device__ __forceinline__ void tc_ld_x16(uint32_t (&r)[16], uint32_t taddr) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// K runs in segments of kTcSegKb k-blocks (512 halves).  A segment's MMAs
// accumulate in one of two tensor-memory accumulators (segments alternate),
// and the epilogue warps drain each finished segment into fp32 registers
// while the next one is computed.  The tensor core's own accumulation is not
// IEEE-exact over thousands of products; with chains of 32 MMAs and the
// segments summed in fp32, outputs stay within 1e-3 of an fp32 reference
// (elementwise, with the 1e-3 max floor) at K = 8192 -- the same promotion
// of partial sums to CUDA-core accumulators that FP8 GEMMs use.
constexpr int kTcSegKb = 8;
constexpr int kTcEpiWarps = 8;                        // two warps per 32-lane quarter of tensor memory
constexpr int kTcThreads2 = 64 + 32 * kTcEpiWarps;    // producer warp, MMA warp, epilogue warps

template <int BN>
__global__ void __launch_bounds__(kTcThreads2, 1) gemm_f16_tc_kernel(const __grid_constant__ TcArgs a) {
    static_assert(BN == 64 || BN == 128 || BN == 256, "tile width");
    constexpr uint32_t A_BYTES = kTcBM * 128u;
    constexpr uint32_t STAGE = tc_stage_bytes(BN);
    constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators; a power of two <= 512
    constexpr int HALF = BN / 2;            // columns per epilogue thread
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], accf[2], acce[2], done;
    __shared__ uint32_t tmem_base;
    __shared__ int issued, consumed, aborted;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
    const int64_t n0 = (int64_t)blockIdx.y * kTcBM, m0 = (int64_t)blockIdx.x * BN;
    const int kb_total = (int)((a.k + kTcBK - 1) / kTcBK);
    const int nseg = (kb_total + kTcSegKb - 1) / kTcSegKb;

    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int q = 0; q < 2; ++q) {
            mbar_init(&accf[q], 1);
            mbar_init(&acce[q], kTcEpiWarps);  // one arrival per epilogue warp
        }
        mbar_init(&done, 1);
        issued = consumed = aborted = 0;
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    float acc[HALF];
#pragma unroll
    for (int j = 0; j < HALF; ++j) acc[j] = 0.f;

    if (tid == 0) {
        // producer: a stage's slot is reused once the MMAs that read it committed
        int kb = 0;
        for (; kb < kb_total; ++kb) {
            const int s = kb % kTcStages;
            if (kb >= kTcStages && !mbar_wait_bounded(&empty[s], (uint32_t)(((kb / kTcStages) - 1) & 1))) {
                aborted = 1;
                break;
            }
            const uint32_t st = sbase + (uint32_t)s * STAGE;
            mbar_arrive_expect_tx(&full[s], STAGE);
            tma_load_2d(st, &a.tmw, kb * kTcBK, (int)n0, &full[s]);
            tma_load_2d(st + A_BYTES, &a.tmx, kb * kTcBK, (int)m0, &full[s]);
        }
        issued = kb;
    } else if (tid == 32) {
        // MMA issuer: segment g into accumulator g % 2, once the epilogue
        // has drained that accumulator's previous segment
        constexpr uint32_t idesc = tc_idesc_f16<BN>();
        int kb = 0;
        for (int g = 0; g < nseg && !aborted; ++g) {
            const int q = g & 1;
            if (g >= 2 && !mbar_wait_bounded(&acce[q], (uint32_t)(((g >> 1) - 1) & 1))) {
                aborted = 1;
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)(q * BN);
            const int kb_end = min(kb_total, (g + 1) * kTcSegKb);
            for (; kb < kb_end; ++kb) {
                const int s = kb % kTcStages;
                if (!mbar_wait_bounded(&full[s], (uint32_t)((kb / kTcStages) & 1))) {
                    aborted = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t st = sbase + (uint32_t)s * STAGE;
                const uint64_t da = tc_desc_sw128(st), db = tc_desc_sw128(st + A_BYTES);
#pragma unroll
                for (int kk = 0; kk < kTcBK / 16; ++kk)
                    tc_mma_f16(d, da + (uint64_t)(2 * kk), db + (uint64_t)(2 * kk), idesc,
                               (kb > g * kTcSegKb || kk > 0) ? 1 : 0);
                tc_commit(&empty[s]);
            }
            if (aborted) break;
            tc_commit(&accf[q]);  // the segment's sum is complete in accumulator q
        }
        consumed = kb;
    } else if (warp >= 2) {
        // epilogue warps: drain every segment into fp32 registers
        const int e = warp - 2;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;  // this warp's tensor-memory lanes
        const uint32_t col0 = (uint32_t)((e >> 2) * HALF);              // this warp's half of the columns
        for (int g = 0; g < nseg; ++g) {
            const int q = g & 1;
            if (!mbar_wait_bounded(&accf[q], (uint32_t)((g >> 1) & 1))) {
                aborted = 1;
                break;
            }
            tc_fence_after();
            const uint32_t taddr = tmem + lane_base + (uint32_t)(q * BN) + col0;
#pragma unroll
            for (int c = 0; c < HALF; c += 16) {
                uint32_t v[16];
                tc_ld_x16(v, taddr + (uint32_t)c);
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[c + j] = __fadd_rn(acc[c + j], __uint_as_float(v[j]));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acce[q])) : "memory");
        }
    }
    __syncthreads();  // every loop is over
    if (tid == 32) {
        if (aborted) {
            // copies issued but never consumed must land before the CTA exits
            for (int kb = consumed; kb < issued; ++kb)
                mbar_wait_drain(&full[kb % kTcStages], (uint32_t)((kb / kTcStages) & 1));
        }
        tc_commit(&done);  // every MMA issued above has completed
    }
    mbar_wait_drain(&done, 0);
    tc_fence_after();
    if (!aborted && warp >= 2) {
        const int e = warp - 2;
        const int64_t r = n0 + (warp & 3) * 32 + lane;
        const int64_t t0 = m0 + (e >> 2) * HALF;
        if (r < a.n) {
#pragma unroll
            for (int j = 0; j < HALF; ++j) {
                const int64_t t = t0 + j;
                if (t < a.m) a.y[t * a.ldy + r] = acc[j];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// x f32 [m][ldx] -> X16 [m][k] f16 (round to nearest even), 8 values per thread.
__global__ void f32_to_f16_rows_kernel(const float* x, int64_t ldx, uint16_t* out, int64_t m, int64_t k) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t per_row = k / 8;
    if (i >= m * per_row) return;
    const int64_t r = i / per_row, c = (i - r * per_row) * 8;
    const float* src = x + r * ldx + c;
    uint4 o;
    __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) oh[e] = __floats2half2_rn(src[2 * e], src[2 * e + 1]);
    *reinterpret_cast<uint4*>(out + r * k + c) = o;
}

}  // namespace b200
