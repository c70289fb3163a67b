// host.cpp -- host-only helpers of the C ABI.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>

#include "../../include/b200_decode.h"

namespace {

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = -1;
            do {
                mant <<= 1;
                ++e;
            } while ((mant & 0x400u) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mant & 0x3ffu) << 13);
        }
    } else {
        bits = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

}  // namespace

extern "C" int b200_kv_lengths_from_mask_f16(const uint16_t* mask, int64_t n_kv, int64_t n_rows, int32_t* out) {
    if (!mask || !out || n_kv <= 0 || n_rows < 0) return B200_EINVAL;
    for (int64_t r = 0; r < n_rows; ++r) {
        int64_t len = n_kv;
        while (len > 0 && !std::isfinite(half_to_float(mask[r * n_kv + len - 1]))) --len;
        out[r] = (int32_t)(len > 1 ? len : 1);
    }
    return B200_OK;
}

namespace {

// Leading spaces, then one or more decimal digits; the rest of the text is
// ignored (as std::stoi does).  False when there is no digit.
bool parse_layer_number(const char* p, const char* end, long* out) {
    while (p < end && *p == ' ') ++p;
    if (p >= end || *p < '0' || *p > '9') return false;
    long v = 0;
    while (p < end && *p >= '0' && *p <= '9' && v < 100000000) v = v * 10 + (*p++ - '0');
    *out = v;
    return true;
}

// 1: layer is in the list, 0: not, B200_EINVAL: malformed item.
int layer_listed(long layer, const char* list) {
    if (!list) return 0;
    const char* p = list;
    const char* end = list + std::strlen(list);
    while (p < end) {
        while (p < end && (*p == ',' || *p == ' ')) ++p;
        const char* e = p;
        while (e < end && *e != ',') ++e;
        if (e > p) {
            const char* dash = p;
            while (dash < e && *dash != '-') ++dash;
            long lo = 0, hi = 0;
            if (!parse_layer_number(p, dash, &lo)) return B200_EINVAL;
            if (dash < e) {
                if (!parse_layer_number(dash + 1, e, &hi)) return B200_EINVAL;
            } else {
                hi = lo;
            }
            if (layer >= lo && layer <= hi) return 1;
        }
        p = e + 1;
    }
    return 0;
}

}  // namespace

extern "C" int b200_a8w8_selects_weight(const char* name, int type, const int64_t ne[4], const char* disable_layers,
                                        int tied_output) {
    if (!name || !ne) return B200_EINVAL;
    if (type != B200_TYPE_F16 || ne[2] != 1 || ne[3] != 1) return 0;
    const std::string nm(name);
    if (tied_output && nm == "token_embd.weight" && ne[0] == 1536 && ne[1] == 151936) return 1;
    const bool ffn = nm.find("ffn_gate.weight") != std::string::npos || nm.find("ffn_up.weight") != std::string::npos ||
                     nm.find("ffn_down.weight") != std::string::npos;
    if (!ffn) return 0;
    const size_t at = nm.find("blk.");
    if (at == std::string::npos) return 1;
    long layer = 0;
    const char* digits = nm.c_str() + at + 4;
    if (!parse_layer_number(digits, nm.c_str() + nm.size(), &layer) || *digits == ' ') return 1;
    const int listed = layer_listed(layer, disable_layers);
    if (listed < 0) return listed;
    return listed ? 0 : 1;
}
