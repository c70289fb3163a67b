// kernels.cu -- device code translation unit and the kernel half of the C ABI.
//
// All device code is compiled in this one unit (the .cuh files are included
// here) so the device status word and helpers need no relocatable device
// code.  Host-side code elsewhere (graph runner, backend, decode driver)
// reaches the kernels through include/b200_decode.h and internal.h.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "allreduce.cuh"
#include "common.cuh"
#include "fa.cuh"
#include "fa_mma.cuh"
#include "gemm_small.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "model_ops.cuh"
#include "ops.cuh"

using namespace b200;

namespace {

constexpr int kMaxDevices = 64;
constexpr size_t kSmemBudget = 200 * 1024;

int g_sms[kMaxDevices];
std::mutex g_attr_mu;
bool g_attr_done[kMaxDevices][5][2][9][2];

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

int sm_count(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return 148;
    if (g_sms[dev] == 0) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        g_sms[dev] = v > 0 ? v : 148;
    }
    return g_sms[dev];
}

// B200_GEMV_STAGES caps the bulk-copy pipeline depth (tuning sweeps); unset
// or 0 means as many stages as the shared-memory budget holds.
int stage_cap() {
    static const int cap = [] {
        const char* s = getenv("B200_GEMV_STAGES");
        return s ? atoi(s) : 0;
    }();
    return cap;
}

int cuda_status(cudaError_t e) {
    if (e != cudaSuccess) {
        fprintf(stderr, "b200_decode: CUDA error %s (%s)\n", cudaGetErrorName(e), cudaGetErrorString(e));
        return B200_ECUDA;
    }
    return B200_OK;
}

#define CR_(x)                        \
    do {                              \
        const int r_ = (x);           \
        if (r_ != B200_OK) return r_; \
    } while (0)

// Opts a GEMV instantiation into large dynamic shared memory, once per device.
// Done before any stream capture (b200i_prepare_device) so that capturing a
// decode step never calls it.
template <int FMT, bool DEBUG, int UPL, bool AR = false>
int set_gemv_attr(int dev) {
    std::lock_guard<std::mutex> lk(g_attr_mu);
    const int slot = UPL;
    if (dev < 0 || dev >= kMaxDevices || g_attr_done[dev][FMT][DEBUG ? 1 : 0][slot][AR ? 1 : 0]) return B200_OK;
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<FMT, DEBUG, UPL, AR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return cuda_status(e);
    g_attr_done[dev][FMT][DEBUG ? 1 : 0][slot][AR ? 1 : 0] = true;
    return B200_OK;
}

template <int FMT, bool DEBUG>
int set_gemv_attrs(int dev) {
    CR_((set_gemv_attr<FMT, DEBUG, 0>(dev)));
    CR_((set_gemv_attr<FMT, DEBUG, 2>(dev)));
    CR_((set_gemv_attr<FMT, DEBUG, 4>(dev)));
    CR_((set_gemv_attr<FMT, DEBUG, 3>(dev)));
    if constexpr (FMT != FMT_Q8 && FMT != FMT_A8) {
        CR_((set_gemv_attr<FMT, DEBUG, 5>(dev)));
        CR_((set_gemv_attr<FMT, DEBUG, 6>(dev)));
        CR_((set_gemv_attr<FMT, DEBUG, 7>(dev)));
        CR_((set_gemv_attr<FMT, DEBUG, 8>(dev)));
    }
    if constexpr (FMT == FMT_Q4 && !DEBUG) {  // the fused all-reduce variants of the model's GEMVs
        CR_((set_gemv_attr<FMT, DEBUG, 0, true>(dev)));
        CR_((set_gemv_attr<FMT, DEBUG, 2, true>(dev)));
        CR_((set_gemv_attr<FMT, DEBUG, 3, true>(dev)));
        CR_((set_gemv_attr<FMT, DEBUG, 4, true>(dev)));
        CR_((set_gemv_attr<FMT, DEBUG, 5, true>(dev)));
        CR_((set_gemv_attr<FMT, DEBUG, 6, true>(dev)));
        CR_((set_gemv_attr<FMT, DEBUG, 7, true>(dev)));
        CR_((set_gemv_attr<FMT, DEBUG, 8, true>(dev)));
    }
    return B200_OK;
}

// Shared memory of one GEMV launch: activation region, kGemvWarps rings of
// `stages` chunks, their barriers, and a small reduction scratch.
size_t gemv_smem_bytes(int fmt, const GemvPlan& p, int stages, int64_t rows_per_cta) {
    return (size_t)gemv_x_bytes(fmt, p) + (size_t)kGemvWarps * stages * (size_t)p.stage_bytes +
           (size_t)kGemvWarps * stages * sizeof(uint64_t) + kGemvWarps * sizeof(double) +
           (p.rpc > 1 ? 0 : (size_t)(2 * rows_per_cta) * sizeof(float));
}

// Launch attribute for programmatic dependent launch (see b200i_gemv).
cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute at;
    at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at.val.programmaticStreamSerializationAllowed = 1;
    return at;
}

template <int FMT, bool DEBUG, int UPL>
int launch_gemv_u(GemvArgs a, const GemvPlan& p, cudaStream_t st, bool pdl) {
    const int dev = current_device();
    // the fused all-reduce variant only where it is asked for (model Q4_0 GEMVs)
    bool ar = a.ar_src != nullptr || a.epi == EPI_PUSH;
    if constexpr (FMT != FMT_Q4 || DEBUG) {
        if (ar) return B200_EUNSUPPORTED;
    }
    if (ar) {
        CR_((set_gemv_attr<FMT, DEBUG, UPL, true>(dev)));
    } else {
        CR_((set_gemv_attr<FMT, DEBUG, UPL>(dev)));
    }
    const bool pair = a.epi == EPI_SWIGLU || a.epi == EPI_QKV;
    if (pair && (p.n & 1)) return B200_EINVAL;
    const int64_t item_rows = p.rpc > 1 ? p.rpc : (pair ? 2 : 1);
    const int64_t items = (p.n + item_rows - 1) / item_rows;
    const int64_t grid64 = p.rpc > 1 ? std::min<int64_t>(sm_count(dev), (items + kGemvWarps - 1) / kGemvWarps)
                                     : std::min<int64_t>(sm_count(dev), items);
    const int grid = (int)std::max<int64_t>(1, grid64);
    int64_t rows_per_cta = ((items + grid - 1) / grid) * item_rows;
    if (p.rpc == 1 && a.late_ctas > 0) {  // uneven shares: the largest
        rows_per_cta = 0;
        for (int c = 0; c < grid; ++c)
            rows_per_cta = std::max(rows_per_cta, (gemv_cta_start(c + 1, grid, items, a.late_ctas, a.late_pct) -
                                                   gemv_cta_start(c, grid, items, a.late_ctas, a.late_pct)) *
                                                      item_rows);
    }
    int S = kGemvStagesMax;
    const int cap = stage_cap();
    if (cap > 0) S = std::min(S, cap);
    while (S > 1 && gemv_smem_bytes(FMT, p, S, rows_per_cta) > (size_t)kGemvSmemBudget) --S;
    const size_t smem = gemv_smem_bytes(FMT, p, S, rows_per_cta);
    if (smem > 227 * 1024) return B200_EUNSUPPORTED;
    a.p = p;
    a.n = p.n;
    a.k = p.k;
    a.stages = S;
    if (pdl) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid, 1, 1);
        cfg.blockDim = dim3(kGemvThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute at = pdl_attr();
        cfg.attrs = &at;
        cfg.numAttrs = 1;
        if (ar) return cuda_status(cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, DEBUG, UPL, FMT == FMT_Q4 && !DEBUG>, a));
        return cuda_status(cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, DEBUG, UPL>, a));
    }
    if (ar)
        gemv_kernel<FMT, DEBUG, UPL, FMT == FMT_Q4 && !DEBUG><<<grid, kGemvThreads, smem, st>>>(a);
    else
        gemv_kernel<FMT, DEBUG, UPL><<<grid, kGemvThreads, smem, st>>>(a);
    return cuda_status(cudaGetLastError());
}

template <int FMT, bool DEBUG>
int launch_gemv_t(GemvArgs a, const GemvPlan& p, cudaStream_t st, bool pdl) {
    switch (p.full_upl) {
        case 2: return launch_gemv_u<FMT, DEBUG, 2>(a, p, st, pdl);
        case 3: return launch_gemv_u<FMT, DEBUG, 3>(a, p, st, pdl);
        case 4: return launch_gemv_u<FMT, DEBUG, 4>(a, p, st, pdl);
        case 5:
            if constexpr (FMT != FMT_Q8 && FMT != FMT_A8) return launch_gemv_u<FMT, DEBUG, 5>(a, p, st, pdl);
            break;
        case 6:
            if constexpr (FMT != FMT_Q8 && FMT != FMT_A8) return launch_gemv_u<FMT, DEBUG, 6>(a, p, st, pdl);
            break;
        case 7:
            if constexpr (FMT != FMT_Q8 && FMT != FMT_A8) return launch_gemv_u<FMT, DEBUG, 7>(a, p, st, pdl);
            break;
        case 8:
            if constexpr (FMT != FMT_Q8 && FMT != FMT_A8) return launch_gemv_u<FMT, DEBUG, 8>(a, p, st, pdl);
            break;
        default: break;
    }
    return launch_gemv_u<FMT, DEBUG, 0>(a, p, st, pdl);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ggml rows -> packed rows (layout in args.h).  One thread per (row, unit).
__global__ void repack_kernel(int type, const uint8_t* src0, const uint8_t* src1, int interleave, uint8_t* dst,
                              int64_t n, int U, int64_t rs, int64_t total) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const int64_t p = idx / U;
    const int u = (int)(idx - p * U);
    if (p >= n) return;
    const uint8_t* src = src0;
    int64_t sr = p;
    if (interleave) {
        src = (p & 1) ? src1 : src0;
        sr = p >> 1;
    }
    uint8_t* row = dst + p * rs;
    if (type == B200_TYPE_F16) {
        const uint8_t* s = src + sr * (16 * (int64_t)U) + (int64_t)u * 16;
        uint8_t* d = row + (int64_t)u * 16;
        for (int i = 0; i < 16; ++i) d[i] = s[i];
    } else if (type == B200_TYPE_Q4_0) {
        const uint8_t* s = src + (sr * U + u) * 18;
        uint8_t* q = row + (int64_t)u * 16;
        uint8_t* dd = row + 16 * (int64_t)U + 2 * (int64_t)u;
        dd[0] = s[0];
        dd[1] = s[1];
        for (int i = 0; i < 16; ++i) q[i] = s[2 + i];
    } else {
        const uint8_t* s = src + (sr * U + u) * 34;
        uint8_t* lo = row + (int64_t)u * 16;
        uint8_t* hi = row + 16 * (int64_t)U + (int64_t)u * 16;
        uint8_t* dd = row + 32 * (int64_t)U + 2 * (int64_t)u;
        dd[0] = s[0];
        dd[1] = s[1];
        for (int i = 0; i < 16; ++i) {
            lo[i] = s[2 + i];
            hi[i] = s[18 + i];
        }
    }
}

__global__ void quantize_q8_0_kernel(const float* x, uint8_t* out, int64_t nb) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nb) return;
    const float4* src = reinterpret_cast<const float4*>(x + b * 32);
    int q[8];
    float d;
    uint16_t dh;
    int qs;
    quantize_block32([&](int e) { return src[e]; }, q, d, dh, qs);
    store_block_q8_0(out + b * 34, dh, q);
}

int gemv_common(int fmt, const void* w, const float* x, float* y, int64_t n, int64_t k, int32_t* dots,
                cudaStream_t st) {
    const int type = fmt == FMT_F16  ? B200_TYPE_F16
                     : fmt == FMT_Q8 ? B200_TYPE_Q8_0
                     : fmt == FMT_A8 ? B200_TYPE_A8W8
                                     : B200_TYPE_Q4_0;
    GemvPlan p;
    if (!make_plan(type, n, k, &p)) return B200_EUNSUPPORTED;
    if (!w || !x || !y || !aligned16(w) || !aligned16(x)) return B200_EINVAL;
    GemvArgs a;
    memset(&a, 0, sizeof(a));
    a.w = static_cast<const uint8_t*>(w);
    a.x = x;
    a.pro = PRO_PLAIN;
    a.epi = EPI_STORE;
    a.y = y;
    a.dots = dots;
    a.n = n;
    a.k = k;
    return b200i_gemv(fmt, a, dots != nullptr, st);
}

}  // namespace

// ------------------------------------------------------------------ internal

int b200i_gemv(int fmt, GemvArgs a, bool debug, cudaStream_t st, bool pdl) {
    const int type = fmt == FMT_F16  ? B200_TYPE_F16
                     : fmt == FMT_Q8 ? B200_TYPE_Q8_0
                     : fmt == FMT_A8 ? B200_TYPE_A8W8
                                     : B200_TYPE_Q4_0;
    GemvPlan p;
    if (!make_plan(type, a.n, a.k, &p)) return B200_EUNSUPPORTED;
    if (debug) {
        if (fmt == FMT_Q4) return launch_gemv_t<FMT_Q4, true>(a, p, st, pdl);
        if (fmt == FMT_Q8) return launch_gemv_t<FMT_Q8, true>(a, p, st, pdl);
        return B200_EINVAL;
    }
    switch (fmt) {
        case FMT_F16: return launch_gemv_t<FMT_F16, false>(a, p, st, pdl);
        case FMT_Q4: return launch_gemv_t<FMT_Q4, false>(a, p, st, pdl);
        case FMT_Q4W: return launch_gemv_t<FMT_Q4W, false>(a, p, st, pdl);
        case FMT_Q8: return launch_gemv_t<FMT_Q8, false>(a, p, st, pdl);
        case FMT_A8: return launch_gemv_t<FMT_A8, false>(a, p, st, pdl);
        default: return B200_EINVAL;
    }
}

// How many clusters of each size (16, 8, 4, 2 CTAs) of the tensor-core
// attention kernel can be resident at once, per head dim; set once per device.
int g_fa_active[kMaxDevices][2][kFmMaxCluster + 1];  // [dev][head dim 64 / 128][cluster size]
bool g_small_m_attr[kMaxDevices];
bool g_tc_attr[kMaxDevices][3];
bool g_fa_ready[kMaxDevices][2];

template <int D>
int fa_cluster_probe(int dev) {
    const int slot = D == 64 ? 0 : 1;
    if (g_fa_ready[dev][slot]) return B200_OK;
    cudaError_t e = cudaFuncSetAttribute(fa_mma_kernel<D, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)fa_mma_smem_bytes(D));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fa_mma_kernel<D, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)fa_mma_smem_bytes(D));
    if (e != cudaSuccess) return cuda_status(e);
    const bool nonportable =
        cudaFuncSetAttribute(fa_mma_kernel<D, 2>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess &&
        cudaFuncSetAttribute(fa_mma_kernel<D, 3>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
    for (int cs = 1; cs <= kFmMaxCluster; ++cs) {
        g_fa_active[dev][slot][cs] = 0;
        if (cs > 8 && !nonportable) continue;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(cs, 1, 1);
        cfg.blockDim = dim3(kFmMaxThreads, 1, 1);  // the larger variant; both hold the same shared memory
        cfg.dynamicSmemBytes = fa_mma_smem_bytes(D);
        cudaLaunchAttribute at;
        at.id = cudaLaunchAttributeClusterDimension;
        at.val.clusterDim.x = cs;
        at.val.clusterDim.y = 1;
        at.val.clusterDim.z = 1;
        cfg.attrs = &at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, fa_mma_kernel<D, 3>, &cfg) == cudaSuccess) g_fa_active[dev][slot][cs] = n;
    }
    cudaGetLastError();
    if (g_fa_active[dev][slot][1] <= 0) g_fa_active[dev][slot][1] = 1;
    g_fa_ready[dev][slot] = true;
    return B200_OK;
}

// Cluster size for `needed` clusters over `nchunks` chunks: the largest size
// (any of 1..16, not only powers of two: a GPC that cannot host a cluster of
// 16 may host one of 12) whose clusters all fit on the device at once, else
// the one that keeps the most CTAs resident.  B200_FA_CLUSTER forces a size
// (tuning sweeps).
int fa_cluster_override() {
    static const int v = [] {
        const char* s = getenv("B200_FA_CLUSTER");
        const int c = s ? atoi(s) : 0;
        return c >= 1 && c <= kFmMaxCluster ? c : 0;
    }();
    return v;
}

template <int D>
int fa_pick_cluster(int dev, int needed, int nchunks) {
    const int slot = D == 64 ? 0 : 1;
    if (const int f = fa_cluster_override()) return std::max(1, std::min(f, nchunks));
    int best = 1, best_ctas = 0;
    // powers of two only: on the Llama-3-70B shape 10 CTAs per cluster ran no
    // faster than 8 (10.2 vs 10.0 us) and 12-16 ran in two waves (15.6-17.3 us)
    for (int cs = kFmMaxCluster; cs >= 1; cs >>= 1) {
        const int act = g_fa_active[dev][slot][cs];
        if (act <= 0) continue;
        const int use = std::min(cs, nchunks);
        if (act >= needed) return std::max(1, use);
        const int ctas = act * use;
        if (ctas > best_ctas) {
            best_ctas = ctas;
            best = use;
        }
    }
    return std::max(1, best);
}

int set_fa_attrs() {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return B200_EINVAL;
    std::lock_guard<std::mutex> lk(g_attr_mu);
    CR_(fa_cluster_probe<64>(dev));
    return fa_cluster_probe<128>(dev);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// K or V cache view [D, Hkv, n_kv] (byte strides nb2 per head, nb1 per
// position) as a TMA descriptor with 64 x 1 x 64 boxes and the 128-byte
// swizzle that the tensor-core kernel's ldmatrix addressing expects.
int encode_kv_map(CUtensorMap* m, const void* base, int D, int Hkv, int n_kv, int64_t nb1, int64_t nb2) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return B200_ECUDA;
    const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)Hkv, (cuuint64_t)n_kv};
    const cuuint64_t strides[2] = {(cuuint64_t)nb2, (cuuint64_t)nb1};
    const cuuint32_t box[3] = {64, 1, (cuuint32_t)kFaChunk};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        fprintf(stderr, "b200_decode: cuTensorMapEncodeTiled failed (%d)\n", (int)r);
        return B200_EUNSUPPORTED;
    }
    return B200_OK;
}

template <int D>
int launch_fa_mma(FaArgs a, cudaStream_t st, bool pdl) {
    const int dev = current_device();
    CR_(encode_kv_map(&a.tmk, a.k, D, a.Hkv, a.n_kv, a.k_nb1, a.k_nb2));
    CR_(encode_kv_map(&a.tmv, a.v, D, a.Hkv, a.n_kv, a.v_nb1, a.v_nb2));
    CR_(set_fa_attrs());
    const int nchunks = (a.n_kv + kFaChunk - 1) / kFaChunk;
    const int S = fa_pick_cluster<D>(dev, a.Hkv * a.gchunks, nchunks);
    a.n_splits = S;
    a.chunks_per_split = (nchunks + S - 1) / S;
    // three warp groups (2 stages each) once a CTA has 6 or more chunks
    const int groups = a.chunks_per_split >= 6 ? 3 : 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, a.Hkv, a.gchunks);
    cfg.blockDim = dim3(fm_threads(groups), 1, 1);
    cfg.dynamicSmemBytes = fa_mma_smem_bytes(D);
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = S;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1] = pdl_attr();
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 2 : 1;
    return cuda_status(groups == 3 ? cudaLaunchKernelEx(&cfg, fa_mma_kernel<D, 3>, a)
                                   : cudaLaunchKernelEx(&cfg, fa_mma_kernel<D, 2>, a));
}

// head_dim 64 / 128: tensor-core cluster kernel (fa_mma.cuh); 256: CUDA-core
// kernel with global partials (fa.cuh).
int b200i_fa(const FaArgs& in, int D, cudaStream_t st, bool pdl) {
    FaArgs a = in;
    switch (D) {
        case 64: return launch_fa_mma<64>(a, st, pdl);
        case 128: return launch_fa_mma<128>(a, st, pdl);
        case 256: {
            dim3 grid(a.n_splits, a.Hkv, a.gchunks);
            fa_decode_kernel<256><<<grid, kFaThreads, 0, st>>>(a);
            return cuda_status(cudaGetLastError());
        }
        default: return B200_EUNSUPPORTED;
    }
}

// CTAs (one per SM) of the tensor-core attention launch for these arguments
// (head dim 64 / 128; the same choice as launch_fa_mma); 0 for head dim 256,
// whose kernel shares SMs.
int b200i_fa_ctas(const FaArgs& a, int D) {
    if (D != 64 && D != 128) return 0;
    if (set_fa_attrs() != B200_OK) return 0;
    const int dev = current_device();
    const int nchunks = (a.n_kv + kFaChunk - 1) / kFaChunk;
    const int S = D == 64 ? fa_pick_cluster<64>(dev, a.Hkv * a.gchunks, nchunks)
                          : fa_pick_cluster<128>(dev, a.Hkv * a.gchunks, nchunks);
    return S * a.Hkv * a.gchunks;
}

int b200i_tp_allreduce(const ArArgs& a, cudaStream_t st, bool pdl) {
    if (a.world < 1 || a.world > kMaxRanks || a.n <= 0 || (a.n & 3)) return B200_EINVAL;
    const int grid = std::max(1, std::min(16, (a.n / 4 + kArThreads - 1) / kArThreads));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kArThreads, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute at = pdl_attr();
    cfg.attrs = &at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cuda_status(cudaLaunchKernelEx(&cfg, tp_allreduce_kernel, a));
}

int b200i_sm_count() { return sm_count(current_device()); }

// The grid b200i_gemv launches for a GEMV of this shape (the same rule as
// launch_gemv_u); 0 for an unsupported shape.
int b200i_gemv_grid(int fmt, int64_t n, int64_t k, int epi) {
    const int type = fmt == FMT_F16  ? B200_TYPE_F16
                     : fmt == FMT_Q8 ? B200_TYPE_Q8_0
                     : fmt == FMT_A8 ? B200_TYPE_A8W8
                                     : B200_TYPE_Q4_0;
    GemvPlan p;
    if (!make_plan(type, n, k, &p)) return 0;
    const bool pair = epi == EPI_SWIGLU || epi == EPI_QKV;
    const int64_t item_rows = p.rpc > 1 ? p.rpc : (pair ? 2 : 1);
    const int64_t items = (p.n + item_rows - 1) / item_rows;
    const int sm = sm_count(current_device());
    const int64_t grid64 = p.rpc > 1 ? std::min<int64_t>(sm, (items + kGemvWarps - 1) / kGemvWarps)
                                     : std::min<int64_t>(sm, items);
    return (int)std::max<int64_t>(1, grid64);
}

int set_fa_attrs();

int b200i_prepare_device() {
    const int dev = current_device();
    sm_count(dev);
    CR_((set_gemv_attrs<FMT_F16, false>(dev)));
    CR_((set_gemv_attrs<FMT_Q4, false>(dev)));
    CR_((set_gemv_attrs<FMT_Q4W, false>(dev)));
    CR_((set_gemv_attrs<FMT_Q8, false>(dev)));
    CR_((set_gemv_attrs<FMT_A8, false>(dev)));
    CR_((set_gemv_attrs<FMT_Q4, true>(dev)));
    CR_((set_gemv_attrs<FMT_Q8, true>(dev)));
    CR_(set_fa_attrs());
    return B200_OK;
}

static unsigned grid_for(int64_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

int b200i_synth_q4_0(uint64_t seed, float sigma, int64_t row0, int64_t nrows, int64_t col0, int64_t ncols,
                     int64_t kglob, void* out, cudaStream_t st) {
    if (ncols % 32 || nrows <= 0) return B200_EINVAL;
    synth_q4_0_kernel<<<grid_for(nrows * (ncols / 32), 128), 128, 0, st>>>(seed, sigma, row0, nrows, col0, ncols,
                                                                          kglob, static_cast<uint8_t*>(out));
    return cuda_status(cudaGetLastError());
}

int b200i_synth_rows_f16(uint64_t seed, uint64_t base, int64_t nrows, int64_t rl, int64_t rg, int64_t col0,
                         void* out, cudaStream_t st) {
    if (nrows <= 0 || rl <= 0) return B200_OK;
    synth_rows_f16_kernel<<<grid_for(nrows * rl, 256), 256, 0, st>>>(seed, base, nrows, rl, rg, col0,
                                                                     static_cast<uint16_t*>(out));
    return cuda_status(cudaGetLastError());
}

int b200i_fill_f32(float* p, int64_t n, float v, cudaStream_t st) {
    fill_f32_kernel<<<grid_for(n, 256), 256, 0, st>>>(p, n, v);
    return cuda_status(cudaGetLastError());
}

int b200i_embed(const void* table, int64_t d_model, int64_t vocab, StepState* state, float* x, cudaStream_t st) {
    embed_kernel<<<grid_for(d_model, 256) < 64 ? grid_for(d_model, 256) : 64, 256, 0, st>>>(
        static_cast<const uint8_t*>(table), d_model, vocab, state, x);
    return cuda_status(cudaGetLastError());
}

int b200i_image_to_q8_0(const uint8_t* img, int64_t U, uint8_t* out, cudaStream_t st) {
    if (U <= 0) return B200_OK;
    image_to_q8_0_kernel<<<grid_for(U, 128), 128, 0, st>>>(img, U, out);
    return cuda_status(cudaGetLastError());
}

int b200i_finish(StepState* state, cudaStream_t st) {
    finish_step_kernel<<<1, 1, 0, st>>>(state);
    return cuda_status(cudaGetLastError());
}

// ------------------------------------------------------------------- C ABI

extern "C" {

const char* b200_version(void) { return "b200_decode 0.1 (sm_100a)"; }

const char* b200_strerror(int code) {
    switch (code) {
        case B200_OK: return "ok";
        case B200_EINVAL: return "invalid argument";
        case B200_ECUDA: return "CUDA runtime error";
        case B200_EUNSUPPORTED: return "unsupported op variant";
        case B200_ENOMEM: return "out of memory";
        case B200_ENCCL: return "NCCL error";
        case B200_ESTATE: return "invalid state";
        case B200_ESCRATCH: return "request exceeds the fixed static scratch (B200_FA_STATIC_SCRATCH_BYTES)";
        default: return "unknown status";
    }
}

int b200_set_wait_timeout(uint64_t ns) {
    const unsigned long long v = ns == 0 ? 2000000000ull : (unsigned long long)ns;
    return cuda_status(cudaMemcpyToSymbol(g_wait_timeout_ns, &v, sizeof(v)));
}

int b200_tp_allreduce_f32(float* x, const float* const* parts, int world, int rank, int64_t n,
                          unsigned long long* flags, unsigned long long* const* peer_flags, uint64_t seq,
                          b200_stream_t stream) {
    if (!x || !parts || !flags || !peer_flags || world < 1 || world > kMaxRanks || rank < 0 || rank >= world ||
        n <= 0 || (n & 3) || n > (int64_t)1 << 30 || seq == 0)
        return B200_EINVAL;
    if (!aligned16(x)) return B200_EINVAL;
    ArArgs a;
    memset(&a, 0, sizeof(a));
    a.world = world;
    a.rank = rank;
    a.n = (int)n;
    a.st = nullptr;
    a.seq = (unsigned long long)seq;
    a.x = x;
    a.flags = flags;
    for (int r = 0; r < world; ++r) {
        if (!parts[r] || !peer_flags[r] || !aligned16(parts[r])) return B200_EINVAL;
        a.part[r] = parts[r];
        a.peer_flag[r] = peer_flags[r];
    }
    return b200i_tp_allreduce(a, (cudaStream_t)stream, false);
}

int b200_device_status(unsigned int* status, int reset) {
    if (!status) return B200_EINVAL;
    int rc = cuda_status(cudaDeviceSynchronize());
    if (rc) return rc;
    rc = cuda_status(cudaMemcpyFromSymbol(status, g_status, sizeof(unsigned int)));
    if (rc) return rc;
    if (reset) {
        const unsigned int z = 0;
        rc = cuda_status(cudaMemcpyToSymbol(g_status, &z, sizeof(unsigned int)));
    }
    return rc;
}

int64_t b200_packed_row_stride(int type, int64_t n, int64_t k) {
    GemvPlan p;
    return make_plan(type, n, k, &p) ? p.rs : 0;
}

size_t b200_packed_size(int type, int64_t n, int64_t k) {
    GemvPlan p;
    return make_plan(type, n, k, &p) ? (size_t)gemv_packed_bytes(p) : 0;
}

// The reference's host transform ggml_backend_cann_transform_f16_a8w8
// (patch:1674-1695) on the device: per weight row (an output column of the
// ggml matmul) s = max(amax / 127, 1e-8) kept as f16, q = clamp(roundf(w / s),
// +-127) with the f32 s.  One CTA per row; q into the two int8 planes of the
// A8W8 layout, s after all rows.
__global__ void __launch_bounds__(256) a8w8_transform_kernel(const uint16_t* w, uint8_t* dst, int64_t n, int64_t k) {
    const int64_t r = blockIdx.x;
    const uint16_t* wr = w + r * k;
    float amax = 0.f;
    for (int64_t i = threadIdx.x; i < k; i += 256) amax = fmaxf(amax, fabsf(h2f(wr[i])));
    amax = warp_max(amax);
    __shared__ float wm[8];
    if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = 0.f;
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, wm[i]);
    float scale = __fdiv_rn(amax, 127.0f);
    if (scale < 1.0e-8f) scale = 1.0e-8f;
    const int64_t U = k / 32;
    uint8_t* row = dst + r * 32 * U;
    for (int64_t i = threadIdx.x; i < k; i += 256) {
        float q = roundf(__fdiv_rn(h2f(wr[i]), scale));
        q = fminf(fmaxf(q, -127.0f), 127.0f);
        const int64_t b = i / 32, j = i - b * 32;
        row[(j < 16 ? 0 : 16 * U) + 16 * b + (j & 15)] = (uint8_t)(int8_t)q;
    }
    if (threadIdx.x == 0) reinterpret_cast<uint16_t*>(dst + n * 32 * U)[r] = f2h(scale);
}

static int repack_impl(int type, const void* s0, const void* s1, int interleave, void* dst, int64_t n,
                       int64_t k, cudaStream_t st) {
    GemvPlan p;
    if (!make_plan(type, n, k, &p)) return B200_EUNSUPPORTED;
    if (!s0 || !dst || (interleave && !s1) || !aligned16(dst)) return B200_EINVAL;
    int rc = cuda_status(cudaMemsetAsync(dst, 0, (size_t)gemv_packed_bytes(p), st));
    if (rc) return rc;
    const int64_t total = p.n * p.U;
    const int threads = 256;
    const int64_t blocks = (total + threads - 1) / threads;
    repack_kernel<<<(unsigned)blocks, threads, 0, st>>>(type, static_cast<const uint8_t*>(s0),
                                                        static_cast<const uint8_t*>(s1), interleave,
                                                        static_cast<uint8_t*>(dst), n, p.U, p.rs, total);
    return cuda_status(cudaGetLastError());
}

int b200_repack(int type, const void* src, void* dst, int64_t n, int64_t k, b200_stream_t stream) {
    return repack_impl(type, src, nullptr, 0, dst, n, k, (cudaStream_t)stream);
}

int b200_repack_interleave2(int type, const void* src_even, const void* src_odd, void* dst, int64_t n_each,
                            int64_t k, b200_stream_t stream) {
    return repack_impl(type, src_even, src_odd, 1, dst, 2 * n_each, k, (cudaStream_t)stream);
}

int b200_gemv_f16(const void* w, const float* x, float* y, int64_t n, int64_t k, b200_stream_t stream) {
    return gemv_common(FMT_F16, w, x, y, n, k, nullptr, (cudaStream_t)stream);
}

size_t b200_mul_mat_f16_tc_workspace_size(int64_t m, int64_t k) {
    if (m <= 0 || k <= 0) return 0;
    return align256((size_t)m * (size_t)k * 2);
}

int b200_mul_mat_f16_tc(const void* w, const float* x, float* y, int64_t n, int64_t k, int64_t m, int64_t ldx,
                        int64_t ldy, void* workspace, size_t workspace_size, b200_stream_t stream) {
    if (!w || !x || !y || !workspace || n <= 0 || k <= 0 || m <= 0 || ldx < k || ldy < n) return B200_EINVAL;
    if (k % 8 || !aligned16(w) || !aligned16(workspace)) return B200_EINVAL;
    if (workspace_size < b200_mul_mat_f16_tc_workspace_size(m, k)) return B200_EINVAL;
    if (n > INT32_MAX || m > INT32_MAX || k > INT32_MAX) return B200_EUNSUPPORTED;  // TMA coordinates are int32
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return B200_EINVAL;
    const cudaStream_t st = (cudaStream_t)stream;
    // tile width: the fewest token tiles (each re-reads the weight tile)
    const int bn = m <= 64 ? 64 : m <= 128 ? 128 : 256;
    const int slot = bn == 64 ? 0 : bn == 128 ? 1 : 2;
    {
        std::lock_guard<std::mutex> lk(g_attr_mu);
        if (!g_tc_attr[dev][slot]) {
            const void* fn = bn == 64    ? (const void*)gemm_f16_tc_kernel<64>
                             : bn == 128 ? (const void*)gemm_f16_tc_kernel<128>
                                         : (const void*)gemm_f16_tc_kernel<256>;
            CR_(cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)tc_smem_bytes(bn))));
            g_tc_attr[dev][slot] = true;
        }
    }
    // X16 = f16(x), K-contiguous rows
    uint16_t* x16 = static_cast<uint16_t*>(workspace);
    const int64_t units = m * (k / 8);
    f32_to_f16_rows_kernel<<<(unsigned)((units + 255) / 256), 256, 0, st>>>(x, ldx, x16, m, k);
    CR_(cuda_status(cudaGetLastError()));
    TcArgs a;
    std::memset(&a, 0, sizeof(a));
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return B200_ECUDA;
    const cuuint32_t estr[2] = {1, 1};
    {
        const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)n};
        const cuuint64_t strides[1] = {(cuuint64_t)(2 * k)};
        const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)kTcBM};
        if (enc(&a.tmw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(w), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return B200_EUNSUPPORTED;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
        const cuuint64_t strides[1] = {(cuuint64_t)(2 * k)};
        const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)bn};
        if (enc(&a.tmx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x16, dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return B200_EUNSUPPORTED;
    }
    a.y = y;
    a.n = n;
    a.m = m;
    a.k = k;
    a.ldy = ldy;
    // x = token tile (fastest), y = weight-row tile: CTAs that run together
    // share a weight tile, so its re-reads for the other token tiles hit L2
    const dim3 grid((unsigned)((m + bn - 1) / bn), (unsigned)((n + kTcBM - 1) / kTcBM), 1);
    const size_t smem = tc_smem_bytes(bn);
    switch (bn) {
        case 64: gemm_f16_tc_kernel<64><<<grid, kTcThreads2, smem, st>>>(a); break;
        case 128: gemm_f16_tc_kernel<128><<<grid, kTcThreads2, smem, st>>>(a); break;
        default: gemm_f16_tc_kernel<256><<<grid, kTcThreads2, smem, st>>>(a); break;
    }
    return cuda_status(cudaGetLastError());
}

int b200_mul_mat_f16(const void* w, const float* x, float* y, int64_t n, int64_t k, int m, int64_t ldx, int64_t ldy,
                     b200_stream_t stream) {
    if (!w || !x || !y || n <= 0 || k <= 0 || m < 1 || m > 8 || ldx < k || ldy < n) return B200_EINVAL;
    if (k % 8 || !aligned16(w)) return B200_EINVAL;
    if (m == 1) return b200_gemv_f16(w, x, y, n, k, stream);
    if (n > (int64_t)1 << 30 || k > (int64_t)1 << 30) return B200_EUNSUPPORTED;  // TMA coordinates are int32
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return B200_EINVAL;
    {
        std::lock_guard<std::mutex> lk(g_attr_mu);
        if (!g_small_m_attr[dev]) {
            CR_(cuda_status(cudaFuncSetAttribute(gemm_small_m_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 227 * 1024)));
            g_small_m_attr[dev] = true;
        }
    }
    SmallMArgs a;
    std::memset(&a, 0, sizeof(a));
    {
        PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
        if (!enc) return B200_ECUDA;
        const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)n};
        const cuuint64_t strides[1] = {(cuuint64_t)(2 * k)};
        const cuuint32_t box[2] = {64, 16};
        const cuuint32_t estr[2] = {1, 1};
        const CUresult r = enc(&a.tmw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(w), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return B200_EUNSUPPORTED;
    }
    // columns per launch and ring depth within the shared-memory budget: all
    // m columns in one pass with the deepest ring that fits (down to 2
    // stages); otherwise 2 stages and the weight streamed once per group
    int mg = m, S = kSmStagesMax;
    while (S > 2 && small_m_smem_bytes(k, mg, S) > (size_t)kGemvSmemBudget) --S;
    while (mg > 1 && small_m_smem_bytes(k, mg, S) > (size_t)kGemvSmemBudget) --mg;
    if (small_m_smem_bytes(k, mg, S) > 227 * 1024) return B200_EUNSUPPORTED;
    const int64_t tiles = (n + 15) / 16;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(sm_count(dev), (tiles + kSmWarps - 1) / kSmWarps));
    a.n = n;
    a.k = k;
    a.ldx = ldx;
    a.ldy = ldy;
    a.xstride = small_m_xstride(k);
    a.stages = S;
    a.xvec = aligned16(x) && ldx % 4 == 0 ? 1 : 0;
    for (int m0 = 0; m0 < m; m0 += mg) {
        a.x = x + (int64_t)m0 * ldx;
        a.y = y + (int64_t)m0 * ldy;
        a.m = std::min(mg, m - m0);
        gemm_small_m_kernel<<<grid, kSmThreads, small_m_smem_bytes(k, a.m, S), (cudaStream_t)stream>>>(a);
        CR_(cuda_status(cudaGetLastError()));
    }
    return B200_OK;
}

int b200_gemv_q4_0(const void* w, const float* x, float* y, int64_t n, int64_t k, int mode,
                   b200_stream_t stream) {
    if (mode != B200_Q4_MODE_GGML && mode != B200_Q4_MODE_W4A16) return B200_EINVAL;
    return gemv_common(mode == B200_Q4_MODE_GGML ? FMT_Q4 : FMT_Q4W, w, x, y, n, k, nullptr,
                       (cudaStream_t)stream);
}

int b200_gemv_q8_0_q8_0(const void* w, const float* x, float* y, int64_t n, int64_t k, b200_stream_t stream) {
    return gemv_common(FMT_Q8, w, x, y, n, k, nullptr, (cudaStream_t)stream);
}

int b200_quantize_q8_0(const float* x, void* blocks, int64_t k, b200_stream_t stream) {
    if (!x || !blocks || k <= 0 || k % 32 || !aligned16(x)) return B200_EINVAL;
    const int64_t nb = k / 32;
    quantize_q8_0_kernel<<<(unsigned)((nb + 127) / 128), 128, 0, (cudaStream_t)stream>>>(
        x, static_cast<uint8_t*>(blocks), nb);
    return cuda_status(cudaGetLastError());
}

int b200_gemv_block_dots(int type, const void* w, const float* x, int32_t* dots, void* xq_blocks, int64_t n,
                         int64_t k, b200_stream_t stream) {
    if (!dots) return B200_EINVAL;
    if (type != B200_TYPE_Q4_0 && type != B200_TYPE_Q8_0) return B200_EUNSUPPORTED;
    GemvPlan p;
    if (!make_plan(type, n, k, &p)) return B200_EUNSUPPORTED;
    GemvArgs a;
    memset(&a, 0, sizeof(a));
    a.w = static_cast<const uint8_t*>(w);
    a.x = x;
    a.pro = PRO_PLAIN;
    a.epi = -1;  // no epilogue: only the block dots are exported
    a.y = nullptr;
    a.dots = dots;
    a.xq_out = static_cast<uint8_t*>(xq_blocks);
    a.n = n;
    a.k = k;
    if (!w || !x || !aligned16(w) || !aligned16(x)) return B200_EINVAL;
    return b200i_gemv(type == B200_TYPE_Q4_0 ? FMT_Q4 : FMT_Q8, a, true, (cudaStream_t)stream);
}

int b200_a8w8_transform(const void* w_f16, void* dst, int64_t n, int64_t k, b200_stream_t stream) {
    GemvPlan p;
    if (!w_f16 || !dst || !aligned16(dst)) return B200_EINVAL;
    if (!make_plan(B200_TYPE_A8W8, n, k, &p) || n > INT32_MAX) return B200_EUNSUPPORTED;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t tail = pad16(2 * n) - 2 * n;  // zero the scale plane's padding
    if (tail) CR_(cuda_status(cudaMemsetAsync(static_cast<uint8_t*>(dst) + n * p.rs + 2 * n, 0, tail, st)));
    a8w8_transform_kernel<<<(unsigned)n, 256, 0, st>>>(static_cast<const uint16_t*>(w_f16), static_cast<uint8_t*>(dst),
                                                      n, k);
    return cuda_status(cudaGetLastError());
}

int b200_gemv_a8w8(const void* w_packed, const float* x, float* y, int64_t n, int64_t k, b200_stream_t stream) {
    return gemv_common(FMT_A8, w_packed, x, y, n, k, nullptr, (cudaStream_t)stream);
}

// ---- neighbour ops (ops.cuh) ----

int b200_rms_norm_f32(const float* x, const float* w, float* y, int64_t n, int64_t rows, float eps,
                      b200_stream_t stream) {
    if (!x || !y || n <= 0 || rows <= 0 || rows > INT32_MAX) return B200_EINVAL;
    rms_norm_kernel<<<(unsigned)rows, kOpThreads, 0, (cudaStream_t)stream>>>(x, w, y, n, eps);
    return cuda_status(cudaGetLastError());
}

int b200_rope_norm_f32(const float* x, float* y, const int32_t* pos, int64_t n_tokens, int n_heads, int head_dim,
                       float freq_base, b200_stream_t stream) {
    if (!x || !y || !pos || n_tokens <= 0 || n_heads <= 0 || head_dim <= 0 || (head_dim & 1)) return B200_EINVAL;
    const int64_t total = n_tokens * n_heads * (head_dim / 2);
    const float theta_scale = powf(freq_base, -2.0f / (float)head_dim);
    rope_norm_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(x, y, pos, n_tokens, n_heads,
                                                                                       head_dim, theta_scale);
    return cuda_status(cudaGetLastError());
}

int b200_set_rows_f16(const float* src, const int64_t* rows_idx, void* dst, int64_t n, int64_t nrows,
                      int64_t dst_row_stride, int64_t dst_rows, b200_stream_t stream) {
    if (!src || !rows_idx || !dst || n <= 0 || nrows <= 0 || dst_rows <= 0 || dst_row_stride < 2 * n ||
        (dst_row_stride & 1) || (reinterpret_cast<uintptr_t>(dst) & 1))
        return B200_EINVAL;
    const int64_t total = n * nrows;
    set_rows_f16_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        src, rows_idx, static_cast<uint8_t*>(dst), n, nrows, dst_row_stride, dst_rows);
    return cuda_status(cudaGetLastError());
}

int b200_get_rows_q4_0(const void* table, const int32_t* idx, float* dst, int64_t n, int64_t nidx, int64_t vocab,
                       b200_stream_t stream) {
    if (!table || !idx || !dst || n <= 0 || (n % 32) || nidx <= 0 || vocab <= 0) return B200_EINVAL;
    const int64_t total = n * nidx;
    get_rows_q4_0_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        static_cast<const uint8_t*>(table), idx, dst, n, nidx, vocab);
    return cuda_status(cudaGetLastError());
}

int b200_get_rows_q4_0_packed(const void* table_packed, const int32_t* idx, float* dst, int64_t n, int64_t nidx,
                              int64_t vocab, b200_stream_t stream) {
    if (!table_packed || !idx || !dst || n <= 0 || (n % 32) || nidx <= 0 || vocab <= 0) return B200_EINVAL;
    const int64_t rs = b200_packed_row_stride(B200_TYPE_Q4_0, vocab, n);
    if (rs <= 0) return B200_EUNSUPPORTED;
    const int64_t total = n * nidx;
    get_rows_q4_0_packed_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        static_cast<const uint8_t*>(table_packed), idx, dst, n, nidx, vocab, rs);
    return cuda_status(cudaGetLastError());
}

int b200_swiglu_f32(const float* g, const float* u, float* y, int64_t n, b200_stream_t stream) {
    if (!g || !u || !y || n <= 0) return B200_EINVAL;
    swiglu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(g, u, y, n);
    return cuda_status(cudaGetLastError());
}

int b200_add_f32(const float* a, const float* b, float* y, int64_t n, b200_stream_t stream) {
    if (!a || !b || !y || n <= 0) return B200_EINVAL;
    add_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a, b, y, n);
    return cuda_status(cudaGetLastError());
}

int b200_mul_f32(const float* a, const float* b, float* y, int64_t n, int64_t nb, b200_stream_t stream) {
    if (!a || !b || !y || n <= 0 || nb <= 0 || n % nb) return B200_EINVAL;
    mul_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a, b, y, n, nb);
    return cuda_status(cudaGetLastError());
}

int b200_argmax_f32(const float* x, int64_t n, int32_t* out, b200_stream_t stream) {
    if (!x || !out || n <= 0 || n > INT32_MAX) return B200_EINVAL;
    argmax_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(x, n, out);
    return cuda_status(cudaGetLastError());
}

size_t b200_fa_workspace_size(int head_dim, int n_head, int n_head_kv, int n_kv) {
    if (head_dim <= 0 || n_head <= 0 || n_head_kv <= 0 || n_kv <= 0 || n_head % n_head_kv) return 0;
    return fa_layout(head_dim, n_head, n_head_kv, n_kv).total;
}

int b200_fa_decode(const float* q, const void* k, const void* v, const void* mask, const int32_t* kv_len,
                   float* out, int head_dim, int n_head, int n_head_kv, int n_kv, int64_t k_nb1, int64_t k_nb2,
                   int64_t v_nb1, int64_t v_nb2, float scale, void* workspace, size_t workspace_size,
                   b200_stream_t stream) {
    if (!q || !k || !v || !out || !workspace) return B200_EINVAL;
    if (!aligned16(out) || (reinterpret_cast<uintptr_t>(q) & 7)) return B200_EINVAL;
    if (n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv || n_kv <= 0) return B200_EINVAL;
    if (head_dim != 64 && head_dim != 128 && head_dim != 256) return B200_EUNSUPPORTED;
    if (!aligned16(k) || !aligned16(v) || (k_nb1 & 15) || (k_nb2 & 15) || (v_nb1 & 15) || (v_nb2 & 15))
        return B200_EINVAL;
    const FaLayout L = fa_layout(head_dim, n_head, n_head_kv, n_kv);
    if (workspace_size < L.total) return B200_EINVAL;
    FaArgs a;
    memset(&a, 0, sizeof(a));
    a.q = q;
    a.k = static_cast<const uint8_t*>(k);
    a.v = static_cast<const uint8_t*>(v);
    a.mask = static_cast<const uint16_t*>(mask);
    a.kv_len = kv_len;
    a.out = out;
    a.Hq = n_head;
    a.Hkv = n_head_kv;
    a.G = n_head / n_head_kv;
    a.gchunks = L.gchunks;
    a.n_kv = n_kv;
    a.n_splits = L.n_splits;
    a.chunks_per_split = L.chunks_per_split;
    a.k_nb1 = k_nb1;
    a.k_nb2 = k_nb2;
    a.v_nb1 = v_nb1;
    a.v_nb2 = v_nb2;
    a.scale = scale;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    a.part_o = reinterpret_cast<float*>(ws + L.off_o);
    a.part_ml = reinterpret_cast<float*>(ws + L.off_ml);
    a.tickets = reinterpret_cast<unsigned int*>(ws + L.off_tickets);
    return b200i_fa(a, head_dim, (cudaStream_t)stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free attention for callers that may not allocate device memory
// (an engine's pool owns the GPU; the caller runs between another
// component's allocations; the host links only the kernels).  The split-KV
// partials and merge tickets live in this fixed array of the module's device
// image: each GPU that loads the library holds its own copy until exit.
// In host code `g_fa_static_scratch` is only a handle for the runtime; the
// device address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) unsigned char g_fa_static_scratch[B200_FA_STATIC_SCRATCH_BYTES];

namespace {

std::mutex g_static_scratch_mu;
unsigned char* g_static_scratch_dev[kMaxDevices];
CUcontext g_static_scratch_ctx[kMaxDevices];

// The calling thread's current CUDA context (driver entry point through the
// runtime, so the library needs no link against the driver library).
CUcontext current_context() {
    using Fn = CUresult (*)(CUcontext*);
    static const Fn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<Fn>(p);
    }();
    CUcontext c = nullptr;
    if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

// Device address of g_fa_static_scratch on the current device, looked up on
// the first call there (with that device current) and cached with the
// context it belongs to: after a cudaDeviceReset the device's next primary
// context loads the module again, so a call in a different context than
// the cached one looks the address up again.
int static_scratch(unsigned char** out) {
    int dev = -1;
    CR_(cuda_status(cudaGetDevice(&dev)));
    if (dev < 0 || dev >= kMaxDevices) return B200_EINVAL;
    CUcontext ctx = current_context();
    if (ctx == nullptr) {
        // no context yet on this thread: cudaFree(NULL) makes the device's
        // primary context current and allocates nothing (not allowed while
        // a stream captures, hence only here, on a first call)
        CR_(cuda_status(cudaFree(nullptr)));
        ctx = current_context();
    }
    std::lock_guard<std::mutex> lk(g_static_scratch_mu);
    if (g_static_scratch_dev[dev] == nullptr || ctx == nullptr || g_static_scratch_ctx[dev] != ctx) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_fa_static_scratch);
        if (e != cudaSuccess || p == nullptr) return e != cudaSuccess ? cuda_status(e) : B200_ECUDA;
        g_static_scratch_dev[dev] = static_cast<unsigned char*>(p);
        g_static_scratch_ctx[dev] = ctx;
    }
    *out = g_static_scratch_dev[dev];
    return B200_OK;
}

}  // namespace

extern "C" int b200_fa_decode_static_scratch(const float* q, const void* k, const void* v, const void* mask,
                                             const int32_t* kv_len, float* out, int head_dim, int n_head,
                                             int n_head_kv, int n_kv, int64_t k_nb1, int64_t k_nb2, int64_t v_nb1,
                                             int64_t v_nb2, float scale, b200_stream_t stream) {
    if (!q || !k || !v || !out) return B200_EINVAL;
    if (n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv || n_kv <= 0) return B200_EINVAL;
    if (head_dim != 64 && head_dim != 128 && head_dim != 256) return B200_EUNSUPPORTED;
    if (!aligned16(k) || !aligned16(v) || (k_nb1 & 15) || (k_nb2 & 15) || (v_nb1 & 15) || (v_nb2 & 15))
        return B200_EINVAL;
    const FaLayout L = fa_layout(head_dim, n_head, n_head_kv, n_kv);
    if (L.total > B200_FA_STATIC_SCRATCH_BYTES) return B200_ESCRATCH;
    unsigned char* ws = nullptr;
    CR_(static_scratch(&ws));
    const cudaStream_t st = (cudaStream_t)stream;
    // The merge tickets must start at zero; the partials are written before
    // they are read.
    CR_(cuda_status(cudaMemsetAsync(ws + L.off_tickets, 0, (size_t)n_head_kv * L.gchunks * sizeof(unsigned int), st)));
    FaArgs a;
    memset(&a, 0, sizeof(a));
    a.q = q;
    a.k = static_cast<const uint8_t*>(k);
    a.v = static_cast<const uint8_t*>(v);
    a.mask = static_cast<const uint16_t*>(mask);
    a.kv_len = kv_len;
    a.out = out;
    a.Hq = n_head;
    a.Hkv = n_head_kv;
    a.G = n_head / n_head_kv;
    a.gchunks = L.gchunks;
    a.n_kv = n_kv;
    a.n_splits = L.n_splits;
    a.chunks_per_split = L.chunks_per_split;
    a.k_nb1 = k_nb1;
    a.k_nb2 = k_nb2;
    a.v_nb1 = v_nb1;
    a.v_nb2 = v_nb2;
    a.scale = scale;
    a.part_o = reinterpret_cast<float*>(ws + L.off_o);
    a.part_ml = reinterpret_cast<float*>(ws + L.off_ml);
    a.tickets = reinterpret_cast<unsigned int*>(ws + L.off_tickets);
    const dim3 grid(L.n_splits, n_head_kv, L.gchunks);
    switch (head_dim) {
        case 64: fa_decode_kernel<64><<<grid, kFaThreads, 0, st>>>(a); break;
        case 128: fa_decode_kernel<128><<<grid, kFaThreads, 0, st>>>(a); break;
        default: fa_decode_kernel<256><<<grid, kFaThreads, 0, st>>>(a); break;
    }
    return cuda_status(cudaGetLastError());
}
