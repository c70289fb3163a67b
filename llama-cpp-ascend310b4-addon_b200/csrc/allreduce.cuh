// allreduce.cuh -- tensor-parallel all-reduce of one activation vector over
// NVLink peer memory, for the partial sums of the row-split O and down
// projections (the reference decomposes nothing; this replaces an
// ncclAllReduce(sum) of d_model floats per call).
//
// Every rank's producing GEMV has written its partial into its own buffer
// (mapped into every peer through CUDA IPC).  This kernel, on every rank:
//   1. announces "partial of collective seq is complete" by storing seq into
//      each rank's flag slot for this rank (release, system scope);
//   2. waits until every rank's announcement for seq has arrived in its own
//      flags (acquire, system scope; bounded: 2 s, then a status bit);
//   3. sums the partials of ranks 0..world-1 in that order, reading the peers'
//      buffers directly over NVLink, and writes the full vector locally.
// The order is fixed, so every rank gets bit-identical results.  seq grows
// with the device step counter, so a captured graph replays correctly.
// Buffer reuse is safe with two partial buffers used alternately: a rank
// overwrites a buffer two collectives later, after every peer has announced
// the collective in between, which each does only after finishing this one.
#pragma once

#include "args.h"
#include "common.cuh"

namespace b200 {

constexpr int kArThreads = 256;

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// 16-byte load of a peer's (or this rank's) partial, bypassing L1 (no stale
// copy from an earlier collective); ordered after the acquire of the flags.
// A plain cached-at-L2 load rather than a volatile one, so that the loads of
// all ranks are in flight together.
__device__ __forceinline__ float4 ld_sys_f4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// Spins until *flag >= want (flags only grow).  Gives up after
// g_wait_timeout_ns, records B200_DEVSTATUS_TIMEOUT and returns false; gives
// up at once when an earlier wait on this device already expired (a dead
// peer then costs one limit per step, not one per collective).
__device__ __forceinline__ bool wait_flag_geq(const unsigned long long* flag, unsigned long long want) {
    if (ld_acquire_sys_u64(flag) >= want) return true;
    if (waits_abandoned()) return false;
    const unsigned long long t0 = globaltimer(), limit = g_wait_timeout_ns;
    for (uint32_t it = 1;; ++it) {
        if (ld_acquire_sys_u64(flag) >= want) return true;
        if ((it & 63u) == 0) {
            if (waits_abandoned()) return false;
            if (globaltimer() - t0 > limit) {
                record_status(B200_DEVSTATUS_TIMEOUT);
                return false;
            }
        }
    }
}

__global__ void __launch_bounds__(kArThreads) tp_allreduce_kernel(const ArArgs a) {
    if (threadIdx.x == 0) stamp_point(a.stamp, a.stamp_stride, 0);
    griddep_wait();  // this rank's partial is complete
    griddep_launch_dependents();
    if (threadIdx.x == 0) stamp_point(a.stamp, a.stamp_stride, 1);
    const unsigned long long seq =
        a.st != nullptr ? a.st->step * (unsigned long long)a.per_step + (unsigned long long)a.idx + 1ull : a.seq;
    if (blockIdx.x == 0 && threadIdx.x < a.world) {
        __threadfence_system();
        st_release_sys_u64(a.peer_flag[threadIdx.x], seq);
    }
    // thread r of each CTA waits for rank r's announcement (the ranks in
    // parallel, one poller per flag and CTA), then the CTA meets
    bool ok = true;
    if (threadIdx.x < a.world) ok = wait_flag_geq(&a.flags[threadIdx.x], seq);
    ok = __syncthreads_and(ok) != 0;
    if (threadIdx.x == 0) stamp_point(a.stamp, a.stamp_stride, 3);  // every rank's partial is announced
    if (!ok) {
        if (threadIdx.x == 0) stamp_point(a.stamp, a.stamp_stride, 2);
        return;
    }
    const int n4 = a.n >> 2;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        // every rank's load in flight before the first add (a warp issues in
        // order: an add between two loads would make them one NVLink round
        // trip each), then the sum in rank order
        float4 v[kMaxRanks];
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
            if (r < a.world) v[r] = ld_sys_f4(a.part[r] + 4 * i);
        float4 acc = v[0];
#pragma unroll
        for (int r = 1; r < kMaxRanks; ++r) {
            if (r < a.world) {
                acc.x = __fadd_rn(acc.x, v[r].x);
                acc.y = __fadd_rn(acc.y, v[r].y);
                acc.z = __fadd_rn(acc.z, v[r].z);
                acc.w = __fadd_rn(acc.w, v[r].w);
            }
        }
        reinterpret_cast<float4*>(a.x)[i] = acc;
    }
    if (threadIdx.x == 0) stamp_point(a.stamp, a.stamp_stride, 2);  // thread 0's exit (no barrier: ok may differ per thread)
}

}  // namespace b200
