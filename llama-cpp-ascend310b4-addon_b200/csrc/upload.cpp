// upload.cpp -- chunked, possibly concurrent upload of one ggml weight tensor
// into its packed layout (the B200 counterpart of the reference's
// TensorSetTracker + set_tensor NZ branch, patch:1745-1807).
//
// The reference counts the bytes written to a tensor and transforms it once
// the count reaches the tensor size.  Here the covered byte ranges are kept
// as merged intervals, so a range written twice or overlapping chunks cannot
// fake completion.  Chunks go host -> a device staging buffer in ggml layout
// on the upload's own stream; each write returns after its copy has consumed
// the host memory (set_tensor's contract).  The write that completes the
// coverage repacks the staging buffer into the packed destination and waits
// for it, so the destination is ready when that call returns.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <map>
#include <mutex>

#include "../../include/b200_decode.h"

struct b200_upload {
    int device = 0;
    int type = 0;
    int64_t n = 0, k = 0;
    void* dst = nullptr;
    uint8_t* staging = nullptr;
    size_t total = 0;
    cudaStream_t stream = nullptr;
    std::mutex mu;
    std::map<size_t, size_t> covered;  // start -> end, disjoint and non-adjacent
    size_t covered_bytes = 0;
    bool repacked = false;
};

namespace {

int ck(cudaError_t e) {
    if (e != cudaSuccess) {
        fprintf(stderr, "b200_upload: CUDA error %s\n", cudaGetErrorString(e));
        return B200_ECUDA;
    }
    return B200_OK;
}

int64_t ggml_row_bytes(int type, int64_t k) {
    if (type == B200_TYPE_F16) return 2 * k;
    if (type == B200_TYPE_Q4_0) return k / 32 * 18;
    if (type == B200_TYPE_Q8_0) return k / 32 * 34;
    return 0;
}

// Adds [a, b) to the interval set and returns the bytes newly covered.
size_t cover(std::map<size_t, size_t>& m, size_t a, size_t b) {
    size_t added = b - a;
    auto it = m.upper_bound(a);
    if (it != m.begin()) {
        auto pv = std::prev(it);
        if (pv->second >= a) {  // overlaps or touches the previous interval
            if (pv->second >= b) return 0;
            added -= pv->second - a;
            a = pv->first;
            it = m.erase(pv);
        }
    }
    while (it != m.end() && it->first <= b) {  // swallow the following intervals
        const size_t s = it->first, e = it->second;
        added -= (e < b ? e : b) - s;
        if (e > b) b = e;
        it = m.erase(it);
    }
    m[a] = b;
    return added;
}

}  // namespace

extern "C" {

int b200_upload_begin(int type, int64_t n, int64_t k, void* dst_packed, b200_upload** out) {
    if (!out || !dst_packed || n <= 0 || k <= 0) return B200_EINVAL;
    *out = nullptr;
    const int64_t rb = ggml_row_bytes(type, k);
    if (rb <= 0 || b200_packed_size(type, n, k) == 0) return B200_EUNSUPPORTED;
    b200_upload* u = new b200_upload();
    u->type = type;
    u->n = n;
    u->k = k;
    u->dst = dst_packed;
    u->total = (size_t)(rb * n);
    int rc = ck(cudaGetDevice(&u->device));
    if (rc == B200_OK) rc = ck(cudaStreamCreateWithFlags(&u->stream, cudaStreamNonBlocking));
    if (rc == B200_OK && cudaMalloc(reinterpret_cast<void**>(&u->staging), u->total) != cudaSuccess) rc = B200_ENOMEM;
    if (rc != B200_OK) {
        b200_upload_end(u);
        return rc;
    }
    *out = u;
    return B200_OK;
}

int b200_upload_write(b200_upload* u, size_t offset, const void* host, size_t size, int* complete) {
    if (!u || !host || size == 0 || offset > u->total || size > u->total - offset) return B200_EINVAL;
    int rc = ck(cudaSetDevice(u->device));
    if (rc) return rc;
    // The copy runs outside the lock: chunks of one tensor never share bytes
    // that matter (a byte written twice carries the same value).
    rc = ck(cudaMemcpyAsync(u->staging + offset, host, size, cudaMemcpyHostToDevice, u->stream));
    if (rc == B200_OK) rc = ck(cudaStreamSynchronize(u->stream));
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(u->mu);
    u->covered_bytes += cover(u->covered, offset, offset + size);
    const bool full = u->covered_bytes == u->total;
    if (full && !u->repacked) {
        rc = b200_repack(u->type, u->staging, u->dst, u->n, u->k, (b200_stream_t)u->stream);
        if (rc == B200_OK) rc = ck(cudaStreamSynchronize(u->stream));
        if (rc) return rc;
        u->repacked = true;
    }
    if (complete) *complete = u->repacked ? 1 : 0;
    return B200_OK;
}

int b200_upload_end(b200_upload* u) {
    if (!u) return B200_EINVAL;
    const bool done = u->repacked;
    cudaSetDevice(u->device);
    if (u->stream) cudaStreamSynchronize(u->stream);
    if (u->staging) cudaFree(u->staging);
    if (u->stream) cudaStreamDestroy(u->stream);
    delete u;
    return done ? B200_OK : B200_ESTATE;
}

}  // extern "C"
