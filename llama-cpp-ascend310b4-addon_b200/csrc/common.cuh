// common.cuh -- shared device helpers for the sm_100a decode kernels.
//
// Bulk-async copies (cp.async.bulk, one CTA each) into shared memory signalled
// through mbarriers, bounded waits that report a status word instead of
// hanging, f16 helpers and warp reductions.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200_decode.h"

namespace b200 {

// Device status word: kernels OR a B200_DEVSTATUS_* bit in when a bounded wait
// expires or a runtime bound check fails.  Read with b200_device_status().
__device__ unsigned int g_status;

// Limit of one bounded wait in nanoseconds (2 s unless b200_set_wait_timeout
// changed it for this device).
__device__ unsigned long long g_wait_timeout_ns = 2000000000ull;

// True once any bounded wait on this device has expired (the status word's
// TIMEOUT bit, read without caching).  Waits that depend on another kernel,
// CTA or rank then give up at once instead of spinning their full limit
// again: after a peer dies every later collective of the step returns in
// microseconds.  Cleared by b200_device_status(..., reset = 1).
__device__ __forceinline__ bool waits_abandoned() {
    return (*reinterpret_cast<volatile unsigned int*>(&g_status) & B200_DEVSTATUS_TIMEOUT) != 0u;
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the mbarrier phase with the given parity.  Gives up after
// g_wait_timeout_ns, records B200_DEVSTATUS_TIMEOUT and returns false; gives
// up at once (false, nothing recorded) when an earlier wait already expired.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    if (waits_abandoned()) return false;
    const unsigned long long t0 = globaltimer(), limit = g_wait_timeout_ns;
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (waits_abandoned()) return false;
            if (globaltimer() - t0 > limit) {
                atomicOr(&g_status, (unsigned int)B200_DEVSTATUS_TIMEOUT);
                return false;
            }
        }
    }
}

// For a CTA that gave up: waits (time-bounded only, never abandoned early)
// for a bulk copy it issued, so that no copy is still writing into shared
// memory when the CTA reuses it or exits.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return;
    const unsigned long long t0 = globaltimer(), limit = g_wait_timeout_ns;
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return;
        if ((it & 255u) == 0 && globaltimer() - t0 > limit) {
            atomicOr(&g_status, (unsigned int)B200_DEVSTATUS_TIMEOUT);
            return;
        }
    }
}

// Global -> shared bulk copy; completion is counted on `bar` (transaction
// bytes).  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// L2 eviction policy for a copy: evict_first for data read once per step,
// evict_normal otherwise.
__device__ __forceinline__ uint64_t l2_policy(bool evict_first) {
    uint64_t p;
    if (evict_first)
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    else
        asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// bulk_g2s with an L2 cache policy.
__device__ __forceinline__ void bulk_g2s_pol(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void record_status(unsigned int bit) { atomicOr(&g_status, bit); }

// Kernel timeline (b200_model_timeline): one thread per CTA folds the
// globaltimer into slot s[which * stride] -- which 0: entry (min), 1: return
// from griddepcontrol.wait (min), 2: exit (max); 3, 4, 5: phase marks inside
// the kernel (input ready, first streamed data landed, main loop done), each
// folded as a max into s[which * stride] and as a min into
// s[(which + 3) * stride].  No-ops when s is null.
__device__ __forceinline__ void stamp_point(unsigned long long* s, int stride, int which) {
    if (s == nullptr) return;
    const unsigned long long t = globaltimer();
    if (which < 2) {
        atomicMin(s + (int64_t)which * stride, t);
    } else {
        atomicMax(s + (int64_t)which * stride, t);
        if (which > 2) atomicMin(s + (int64_t)(which + 3) * stride, t);
    }
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialisation may start while the previous kernel in the stream is still
// finishing; griddep_wait() returns once that kernel has completed and its
// writes are visible.  Everything before it may read only data no earlier
// kernel writes (weights) and write only shared memory.  In a normal launch
// both are no-ops.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum over aligned groups of `width` lanes (width a power of two <= 32).
__device__ __forceinline__ float group_sum(float v, int width) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        if (o < width) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
// f32 -> f16 (round to nearest even) -> f32: ggml-cpu converts src1 to F16
// before an F16 dot and q to F16 before the attention dot.
__device__ __forceinline__ float round_f16(float f) { return __half2float(__float2half_rn(f)); }

// Round half away from zero (C roundf semantics) for |x| < 2^31, in three
// instructions: add h = 0.5 - 2^-25 (the largest float below one half) with
// x's sign, round to nearest even, truncate.  For x >= 0 (the sign is
// symmetric): an exact half k + 0.5 gives k + 1 - 2^-25, which rounds to
// k + 1 (for k = 0 it is the midpoint of 1 - 2^-24 and 1 and the tie goes
// to the even 1; above, floats are at least 2^-23 apart and k + 1 is
// nearest); x at most one spacing below k + 0.5 gives a sum below k + 1
// that rounds to a float below k + 1 (same binade as the sum's rounding
// neighbours, and at k = 0 exactly 1 - 2^-24 at most); from 2^23 on, x is an
// integer and adding less than half its spacing rounds back to x.
// tests/test_oracle_golden.py checks the identity on every float in
// [0.25, 256) and on samples below.
__device__ __forceinline__ int round_half_away(float x) {
    return __float2int_rz(__fadd_rn(x, copysignf(0.49999997f, x)));
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Low bytes of q0..q3 (each in [-127, 127]) packed into one word, q0 lowest.
__device__ __forceinline__ int pack_q4(int q0, int q1, int q2, int q3) {
    return (int)__byte_perm(__byte_perm(q0, q1, 0x0040), __byte_perm(q2, q3, 0x0040), 0x5410);
}

// Sum of the four signed bytes of a packed word.
__device__ __forceinline__ int sum_q4(int w) { return __dp4a(w, 0x01010101, 0); }

// R float4 units per lane, each an eighth of a 32-block: the 8 units of a
// block sit in 8 consecutive lanes (lane & 7 = the unit's index in the
// block), quantised with quantize_row_q8_0_ref's rule: d = amax / 127,
// q = roundf(x / d) (x times the reciprocal, as ggml does).  The block max
// and the sum of q are 8-lane shuffle reductions (order free).  The R units
// are independent chains written phase by phase, so they interleave; all 32
// lanes must execute this (full-warp shuffles).  Out: this lane's 4 bytes of
// q packed in a word, and the block's f16 scale and sum of q (every lane of
// the group).
template <int R>
__device__ __forceinline__ void q8_units(const float4 (&v)[R], int (&word)[R], uint16_t (&dh)[R], int (&qs)[R]) {
    float amax[R], id[R];
#pragma unroll
    for (int i = 0; i < R; ++i)
        amax[i] = fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w)));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int i = 0; i < R; ++i) amax[i] = fmaxf(amax[i], __shfl_xor_sync(0xffffffffu, amax[i], o, 8));
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const float d = __fdiv_rn(amax[i], 127.0f);
        id[i] = d != 0.f ? __frcp_rn(d) : 0.f;
        dh[i] = f2h(d);
    }
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const int q0 = round_half_away(__fmul_rn(v[i].x, id[i]));
        const int q1 = round_half_away(__fmul_rn(v[i].y, id[i]));
        const int q2 = round_half_away(__fmul_rn(v[i].z, id[i]));
        const int q3 = round_half_away(__fmul_rn(v[i].w, id[i]));
        word[i] = pack_q4(q0, q1, q2, q3);
        qs[i] = sum_q4(word[i]);
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int i = 0; i < R; ++i) qs[i] += __shfl_xor_sync(0xffffffffu, qs[i], o, 8);
}

// R half-blocks per lane: lanes 2k and 2k + 1 hold values 0..15 and 16..31
// of one 32-block, four float4 each, quantised with quantize_row_q8_0_ref's
// rule (d = amax / 127, q = roundf(x / d) as x times the reciprocal).  The
// block max and the sum of q meet over the lane pair (order free).  Out: this
// lane's 16 q bytes as four words, the block's f16 scale and sum of q (both
// lanes).  Every lane of the warp must run it (full-warp shuffles).
template <int R>
__device__ __forceinline__ void q8_halves(const float4 (&v)[R][4], int4 (&w)[R], uint16_t (&dh)[R], int (&qs)[R]) {
    float amax[R], id[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
        float m[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) m[j] = fmaxf(fmaxf(fabsf(v[i][j].x), fabsf(v[i][j].y)), fmaxf(fabsf(v[i][j].z), fabsf(v[i][j].w)));
        amax[i] = fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
    }
#pragma unroll
    for (int i = 0; i < R; ++i) amax[i] = fmaxf(amax[i], __shfl_xor_sync(0xffffffffu, amax[i], 1));
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const float d = __fdiv_rn(amax[i], 127.0f);
        id[i] = d != 0.f ? __frcp_rn(d) : 0.f;
        dh[i] = f2h(d);
    }
#pragma unroll
    for (int i = 0; i < R; ++i) {
        int wd[4], s = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int q0 = round_half_away(__fmul_rn(v[i][j].x, id[i]));
            const int q1 = round_half_away(__fmul_rn(v[i][j].y, id[i]));
            const int q2 = round_half_away(__fmul_rn(v[i][j].z, id[i]));
            const int q3 = round_half_away(__fmul_rn(v[i][j].w, id[i]));
            wd[j] = pack_q4(q0, q1, q2, q3);
            s = __dp4a(wd[j], 0x01010101, s);
        }
        w[i] = make_int4(wd[0], wd[1], wd[2], wd[3]);
        qs[i] = s;
    }
#pragma unroll
    for (int i = 0; i < R; ++i) qs[i] += __shfl_xor_sync(0xffffffffu, qs[i], 1);
}

// Half-block `half` (block half / 2; values 0..15 or 16..31) into a
// quantised-activation image of U blocks: its 16 q bytes are words 0..3 of
// the block in plane 0 or plane 1; the first half also stores {d, sum}.
__device__ __forceinline__ void q8_image_store_half(uint8_t* img, int64_t U, int64_t half, int4 w, uint16_t dh,
                                                    int qs) {
    const int64_t b = half >> 1;
    const int p = (int)(half & 1);
    reinterpret_cast<int4*>(img)[(p ? U : 0) + b] = w;
    if (p == 0) reinterpret_cast<int2*>(img + 32 * U)[b] = make_int2(__float_as_int(h2f(dh)), qs);
}

// Unit `unit` of the flat activation (4 values; block unit / 8, word
// unit % 8 of the block) into a quantised-activation image of U blocks
// (words [U][4] of q bytes 0..15, words [U][4] of bytes 16..31, then
// {d as f32, sum of q}[U]); the block's {d, sum} from its word-0 lane.
__device__ __forceinline__ void q8_image_store(uint8_t* img, int64_t U, int64_t unit, int word, uint16_t dh, int qs) {
    const int64_t b = unit >> 3;
    const int wd = (int)(unit & 7);
    reinterpret_cast<int*>(img)[(wd < 4 ? 0 : 4 * U) + 4 * b + (wd & 3)] = word;
    if (wd == 0) reinterpret_cast<int2*>(img + 32 * U)[b] = make_int2(__float_as_int(h2f(dh)), qs);
}

}  // namespace b200
