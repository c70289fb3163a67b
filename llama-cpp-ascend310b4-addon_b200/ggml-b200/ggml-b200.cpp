// ggml-b200.cpp -- the ggml backend of the B200 decode path, for llama.cpp
// at 37b3a9e0 (the commit the reference add-on patches).  Registered through
// ggml_backend_reg / ggml_backend_dev like any ggml backend and loadable with
// ggml_backend_load (GGML_BACKEND_DL_IMPL below); every vtable entry
// converts the ggml tensors it is given into b200_tensor descriptors and
// calls the core in include/b200_graph.h, which runs the sm_100a kernels of
// libb200_decode.so.
//
// This file needs upstream ggml's headers (ggml.h, ggml-backend.h and the
// internal ggml-backend-impl.h) and is built only when they are given:
//     python llama-cpp-ascend310b4-addon_b200/build.py --ggml-dir <llama.cpp>/ggml
// or as ggml/src/ggml-b200 inside a llama.cpp tree (CMakeLists.txt beside
// this file).  The same calls, minus the ggml structs, are exercised by the
// tests through the C ABI (tests/test_graph_*.py).
//
// Counterparts in the reference (patches/ascend310b4-llama-cpp.patch):
//   buffer type / buffer with the NZ transform in set_tensor  patch:1700-1846
//   synchronize / free                                        patch:1862-1881
//   graph_compute with per-node trace synchronisation         patch:1884-1923
//   supports_op (FLASH_ATTN_EXT gate patch:1964-1983)         patch:1925-1986
// Ownership follows the reference: tensor->data is the ggml-layout slot and
// the packed copy of a matmul weight sits after it in the same allocation
// (tensor->extra points at it), so get_tensor returns ggml bytes and
// GET_ROWS of a tied embedding reads the same tensor as the lm_head.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "ggml-backend-impl.h"
#include "ggml-backend.h"
#include "ggml.h"

#include "b200_graph.h"

namespace {

constexpr size_t kAlign = 256;

int map_op(enum ggml_op op) {
    switch (op) {
        case GGML_OP_NONE: return B200_OP_NONE;
        case GGML_OP_VIEW:
        case GGML_OP_RESHAPE:
        case GGML_OP_PERMUTE:
        case GGML_OP_TRANSPOSE: return B200_OP_VIEW;
        case GGML_OP_GET_ROWS: return B200_OP_GET_ROWS;
        case GGML_OP_RMS_NORM: return B200_OP_RMS_NORM;
        case GGML_OP_MUL: return B200_OP_MUL;
        case GGML_OP_ADD: return B200_OP_ADD;
        case GGML_OP_MUL_MAT: return B200_OP_MUL_MAT;
        case GGML_OP_ROPE: return B200_OP_ROPE;
        case GGML_OP_SET_ROWS: return B200_OP_SET_ROWS;
        case GGML_OP_FLASH_ATTN_EXT: return B200_OP_FLASH_ATTN_EXT;
        case GGML_OP_GLU: return B200_OP_GLU;
        case GGML_OP_ARGMAX: return B200_OP_ARGMAX;
        case GGML_OP_CPY:
        case GGML_OP_CONT: return B200_OP_CPY;
        default: return -1;
    }
}

// ggml_tensor -> b200_tensor, sources converted recursively (memoised per
// graph so that shared sources stay shared).
struct Converter {
    std::unordered_map<const ggml_tensor*, b200_tensor*> map;
    std::vector<b200_tensor*> owned;
    bool ok = true;

    ~Converter() {
        for (b200_tensor* t : owned) delete t;
    }

    b200_tensor* get(const ggml_tensor* g) {
        if (g == nullptr) return nullptr;
        auto it = map.find(g);
        if (it != map.end()) return it->second;
        b200_tensor* t = new b200_tensor();
        std::memset(t, 0, sizeof(*t));
        owned.push_back(t);
        map[g] = t;
        t->type = (int)g->type;
        const int op = map_op(g->op);
        if (op < 0) ok = false;
        t->op = op < 0 ? B200_OP_COUNT : op;
        for (int i = 0; i < 4; ++i) {
            t->ne[i] = g->ne[i];
            t->nb[i] = g->nb[i];
        }
        static_assert(sizeof(g->op_params) >= sizeof(t->op_params), "op_params size");
        std::memcpy(t->op_params, g->op_params, sizeof(t->op_params));
        t->data = g->data;
        t->extra = g->extra;
        t->name = g->name;
        for (int s = 0; s < GGML_MAX_SRC && s < B200_MAX_SRC; ++s) t->src[s] = get(g->src[s]);
        if (g->extra != nullptr) t->flags |= B200_TENSOR_WEIGHT;
        return t;
    }
};

// ------------------------------------------------------------ buffer type

struct BuftCtx {
    int device;
    std::string name;
};

struct BufCtx {
    b200_buffer* buf = nullptr;
    int device = 0;
};

b200_tensor describe_one(const ggml_tensor* g) {
    b200_tensor t;
    std::memset(&t, 0, sizeof(t));
    t.type = (int)g->type;
    for (int i = 0; i < 4; ++i) {
        t.ne[i] = g->ne[i];
        t.nb[i] = g->nb[i];
    }
    t.data = g->data;
    t.name = g->name;
    return t;
}

void buffer_free(ggml_backend_buffer_t buffer) {
    BufCtx* c = static_cast<BufCtx*>(buffer->context);
    b200_buffer_free(c->buf);
    delete c;
}

void* buffer_get_base(ggml_backend_buffer_t buffer) {
    return b200_buffer_base(static_cast<BufCtx*>(buffer->context)->buf);
}

enum ggml_status buffer_init_tensor(ggml_backend_buffer_t buffer, ggml_tensor* tensor) {
    if (tensor->view_src != nullptr) return GGML_STATUS_SUCCESS;  // views share their source's data and extra
    b200_tensor t = describe_one(tensor);
    if (b200_buffer_init_tensor(static_cast<BufCtx*>(buffer->context)->buf, &t) != B200_OK)
        return GGML_STATUS_FAILED;
    tensor->extra = t.extra;  // packed copy of a matmul weight, else NULL
    return GGML_STATUS_SUCCESS;
}

void buffer_memset_tensor(ggml_backend_buffer_t buffer, ggml_tensor* tensor, uint8_t value, size_t offset,
                          size_t size) {
    b200_tensor t = describe_one(tensor);
    t.extra = tensor->extra;
    if (t.extra) t.flags |= B200_TENSOR_WEIGHT;
    GGML_ASSERT(b200_buffer_memset_tensor(static_cast<BufCtx*>(buffer->context)->buf, &t, value, offset, size) ==
                B200_OK);
}

void buffer_set_tensor(ggml_backend_buffer_t buffer, ggml_tensor* tensor, const void* data, size_t offset,
                       size_t size) {
    b200_tensor t = describe_one(tensor);
    t.extra = tensor->extra;
    if (t.extra) t.flags |= B200_TENSOR_WEIGHT;
    GGML_ASSERT(b200_buffer_set_tensor(static_cast<BufCtx*>(buffer->context)->buf, &t, data, offset, size) ==
                B200_OK);
}

void buffer_get_tensor(ggml_backend_buffer_t buffer, const ggml_tensor* tensor, void* data, size_t offset,
                       size_t size) {
    b200_tensor t = describe_one(tensor);
    GGML_ASSERT(b200_buffer_get_tensor(static_cast<BufCtx*>(buffer->context)->buf, &t, data, offset, size) ==
                B200_OK);
}

void buffer_clear(ggml_backend_buffer_t buffer, uint8_t value) {
    GGML_ASSERT(b200_buffer_clear(static_cast<BufCtx*>(buffer->context)->buf, value) == B200_OK);
}

const char* buft_get_name(ggml_backend_buffer_type_t buft) {
    return static_cast<BuftCtx*>(buft->context)->name.c_str();
}

ggml_backend_buffer_t buft_alloc_buffer(ggml_backend_buffer_type_t buft, size_t size) {
    BuftCtx* bc = static_cast<BuftCtx*>(buft->context);
    BufCtx* c = new BufCtx();
    c->device = bc->device;
    if (b200_buffer_alloc(bc->device, size, /*weights_buffer=*/1, &c->buf) != B200_OK) {
        delete c;
        return nullptr;  // the allocator reports GGML_STATUS_ALLOC_FAILED
    }
    ggml_backend_buffer_i iface = {};
    iface.free_buffer = buffer_free;
    iface.get_base = buffer_get_base;
    iface.init_tensor = buffer_init_tensor;
    iface.memset_tensor = buffer_memset_tensor;
    iface.set_tensor = buffer_set_tensor;
    iface.get_tensor = buffer_get_tensor;
    iface.cpy_tensor = nullptr;
    iface.clear = buffer_clear;
    return ggml_backend_buffer_init(buft, iface, c, size);
}

size_t buft_get_alignment(ggml_backend_buffer_type_t) { return kAlign; }

size_t buft_get_alloc_size(ggml_backend_buffer_type_t, const ggml_tensor* tensor) {
    b200_tensor t = describe_one(tensor);
    // weights are recognised by name (".weight"), as the reference does
    return b200_alloc_size(&t, 1);
}

bool buft_is_host(ggml_backend_buffer_type_t) { return false; }

// ---------------------------------------------------------------- backend

struct BackendCtx {
    b200_backend* be = nullptr;
    int device = 0;
    std::string name;
};

const char* backend_get_name(ggml_backend_t backend) { return static_cast<BackendCtx*>(backend->context)->name.c_str(); }

void backend_free(ggml_backend_t backend) {
    BackendCtx* c = static_cast<BackendCtx*>(backend->context);
    b200_backend_free(c->be);
    delete c;
    delete backend;
}

void backend_synchronize(ggml_backend_t backend) {
    GGML_ASSERT(b200_backend_synchronize(static_cast<BackendCtx*>(backend->context)->be) == B200_OK);
}

enum ggml_status backend_graph_compute(ggml_backend_t backend, ggml_cgraph* cgraph) {
    BackendCtx* c = static_cast<BackendCtx*>(backend->context);
    Converter cv;
    const int n = ggml_graph_n_nodes(cgraph);
    std::vector<b200_tensor*> nodes;
    nodes.reserve(n);
    for (int i = 0; i < n; ++i) nodes.push_back(cv.get(ggml_graph_node(cgraph, i)));
    if (!cv.ok) return GGML_STATUS_FAILED;
    const int rc = b200_graph_compute(c->be, nodes.data(), n);
    return rc == B200_OK ? GGML_STATUS_SUCCESS : GGML_STATUS_FAILED;
}

ggml_guid_t backend_guid() {
    static ggml_guid guid = {0xb2, 0x00, 0x5a, 0x1d, 0x3c, 0x4e, 0x11, 0xf0,
                             0x8a, 0x6b, 0x2d, 0x19, 0x7e, 0x41, 0x0c, 0x55};
    return &guid;
}

// ----------------------------------------------------------------- device

struct DevCtx {
    int device;
    std::string name, description;
    ggml_backend_buffer_type buft;
    BuftCtx buft_ctx;
};

const char* dev_get_name(ggml_backend_dev_t dev) { return static_cast<DevCtx*>(dev->context)->name.c_str(); }
const char* dev_get_description(ggml_backend_dev_t dev) {
    return static_cast<DevCtx*>(dev->context)->description.c_str();
}

void dev_get_memory(ggml_backend_dev_t dev, size_t* free, size_t* total) {
    cudaSetDevice(static_cast<DevCtx*>(dev->context)->device);
    if (cudaMemGetInfo(free, total) != cudaSuccess) *free = *total = 0;
}

enum ggml_backend_dev_type dev_get_type(ggml_backend_dev_t) { return GGML_BACKEND_DEVICE_TYPE_GPU; }

void dev_get_props(ggml_backend_dev_t dev, ggml_backend_dev_props* props) {
    props->name = dev_get_name(dev);
    props->description = dev_get_description(dev);
    props->type = dev_get_type(dev);
    dev_get_memory(dev, &props->memory_free, &props->memory_total);
    props->caps.async = false;
    props->caps.host_buffer = false;
    props->caps.buffer_from_host_ptr = false;
    props->caps.events = false;
}

ggml_backend_t dev_init_backend(ggml_backend_dev_t dev, const char*) {
    DevCtx* d = static_cast<DevCtx*>(dev->context);
    BackendCtx* c = new BackendCtx();
    c->device = d->device;
    c->name = d->name;
    if (b200_backend_create(d->device, &c->be) != B200_OK) {
        delete c;
        return nullptr;
    }
    ggml_backend_i iface = {};
    iface.get_name = backend_get_name;
    iface.free = backend_free;
    iface.synchronize = backend_synchronize;
    iface.graph_compute = backend_graph_compute;
    return new ggml_backend{backend_guid(), iface, dev, c};
}

ggml_backend_buffer_type_t dev_get_buffer_type(ggml_backend_dev_t dev) {
    return &static_cast<DevCtx*>(dev->context)->buft;
}

bool dev_supports_op(ggml_backend_dev_t, const ggml_tensor* op) {
    Converter cv;
    b200_tensor* t = cv.get(op);
    return cv.ok && b200_supports_op(t) == 1;
}

bool dev_supports_buft(ggml_backend_dev_t dev, ggml_backend_buffer_type_t buft) {
    return buft == &static_cast<DevCtx*>(dev->context)->buft;
}

bool dev_offload_op(ggml_backend_dev_t, const ggml_tensor*) { return false; }

// --------------------------------------------------------------- registry

struct RegCtx {
    std::vector<ggml_backend_device> devices;
    std::vector<DevCtx*> ctxs;
};

const char* reg_get_name(ggml_backend_reg_t) { return "B200"; }
size_t reg_get_device_count(ggml_backend_reg_t reg) { return static_cast<RegCtx*>(reg->context)->devices.size(); }
ggml_backend_dev_t reg_get_device(ggml_backend_reg_t reg, size_t index) {
    RegCtx* c = static_cast<RegCtx*>(reg->context);
    GGML_ASSERT(index < c->devices.size());
    return &c->devices[index];
}
void* reg_get_proc_address(ggml_backend_reg_t, const char*) { return nullptr; }

}  // namespace

extern "C" ggml_backend_reg_t ggml_backend_b200_reg(void) {
    static ggml_backend_reg reg;
    static std::once_flag once;
    std::call_once(once, [] {
        RegCtx* rc = new RegCtx();
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
        rc->devices.resize(n);
        for (int i = 0; i < n; ++i) {
            cudaDeviceProp prop;
            cudaGetDeviceProperties(&prop, i);
            DevCtx* d = new DevCtx();
            d->device = i;
            d->name = "B200" + std::to_string(i);
            d->description = prop.name;
            d->buft_ctx.device = i;
            d->buft_ctx.name = d->name;
            ggml_backend_buffer_type_i bi = {};
            bi.get_name = buft_get_name;
            bi.alloc_buffer = buft_alloc_buffer;
            bi.get_alignment = buft_get_alignment;
            bi.get_alloc_size = buft_get_alloc_size;
            bi.is_host = buft_is_host;
            d->buft.iface = bi;
            d->buft.device = &rc->devices[i];
            d->buft.context = &d->buft_ctx;
            ggml_backend_device_i di = {};
            di.get_name = dev_get_name;
            di.get_description = dev_get_description;
            di.get_memory = dev_get_memory;
            di.get_type = dev_get_type;
            di.get_props = dev_get_props;
            di.init_backend = dev_init_backend;
            di.get_buffer_type = dev_get_buffer_type;
            di.supports_op = dev_supports_op;
            di.supports_buft = dev_supports_buft;
            di.offload_op = dev_offload_op;
            rc->devices[i].iface = di;
            rc->devices[i].reg = &reg;
            rc->devices[i].context = d;
            rc->ctxs.push_back(d);
        }
        ggml_backend_reg_i ri = {};
        ri.get_name = reg_get_name;
        ri.get_device_count = reg_get_device_count;
        ri.get_device = reg_get_device;
        ri.get_proc_address = reg_get_proc_address;
        reg.api_version = GGML_BACKEND_API_VERSION;
        reg.iface = ri;
        reg.context = rc;
    });
    return &reg;
}

GGML_BACKEND_DL_IMPL(ggml_backend_b200_reg)
