// IEEE binary16 <-> binary32 on the host (round to nearest even), from the format definition.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

inline float srhpm_host_fp16_to_fp32(uint16_t h) {
    const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
    float          v;
    if (e == 0) {
        v = std::ldexp((float) m, -24);
    } else if (e == 31) {
        v = m ? NAN : INFINITY;
    } else {
        v = std::ldexp((float) (m | 1024), (int) e - 25);
    }
    return s ? -v : v;
}

inline uint16_t srhpm_host_fp32_to_fp16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t) ((x >> 16) & 0x8000);
    const uint32_t ax   = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return sign | (ax > 0x7f800000u ? 0x7e00 : 0x7c00);
    if (ax >= 0x477ff000u) return sign | 0x7c00;  // >= 65520 rounds to infinity
    if (ax < 0x38800000u) {                      // binary16 subnormal: round(|f| * 2^24) units of 2^-24
        float af;
        std::memcpy(&af, &ax, 4);
        return sign | (uint16_t) std::nearbyint(af * 16777216.0f);
    }
    const uint32_t mant = ax & 0x7fffffu;
    uint32_t       h    = ((((ax >> 23) - 127 + 15) & 0x1f) << 10) | (mant >> 13);
    const uint32_t rem  = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
    return sign | (uint16_t) h;
}
