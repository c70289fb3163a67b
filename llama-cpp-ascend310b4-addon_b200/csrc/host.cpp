// host.cpp -- host-only helpers of the C ABI.
#include <cmath>
#include <cstdint>
#include <cstring>

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
