// quant_device.cuh — element-wise dequantization of packed GGML blocks.
#pragma once

#include "brew_common.cuh"

namespace brew {

__device__ __forceinline__ float ld_half(const uint8_t* p) {
    return half_bits_to_float((uint16_t)(p[0] | (p[1] << 8)));
}

// Dequantizes element e of a packed tensor.  Formulas and operation order
// follow gguf-py 0.19.0 (Q4_0, Q4_K, Q6_K) and QuantizedWeights.dequantizeRow
// (gguf/QuantizedWeights.java:76-85, Q8_0); products are rounded separately.
__device__ __forceinline__ float dequant_elem(int type, const uint8_t* w, int64_t e) {
    switch (type) {
        case BREW_TYPE_Q8_0: {
            const uint8_t* b = w + (e / 32) * 34;
            return __fmul_rn((float)(int8_t)b[2 + (e % 32)], ld_half(b));
        }
        case BREW_TYPE_Q4_0: {
            const uint8_t* b = w + (e / 32) * 18;
            const int i = (int)(e % 32);
            const int q = i < 16 ? (b[2 + i] & 15) : (b[2 + i - 16] >> 4);
            return __fmul_rn(ld_half(b), (float)(q - 8));
        }
        case BREW_TYPE_Q4_K: {
            const uint8_t* b = w + (e / 256) * 144;
            const int r = (int)(e % 256), s = r / 32, i = r % 32;
            const uint8_t* sb = b + 4;
            int sc, m;
            if (s < 4) {
                sc = sb[s] & 63;
                m = sb[s + 4] & 63;
            } else {
                sc = (sb[s + 4] & 0xF) | ((sb[s - 4] >> 6) << 4);
                m = (sb[s + 4] >> 4) | ((sb[s] >> 6) << 4);
            }
            const uint8_t qb = b[16 + 32 * (s / 2) + i];
            const int q = (s & 1) ? (qb >> 4) : (qb & 15);
            const float t = __fmul_rn(ld_half(b), (float)sc);
            const float u = __fmul_rn(ld_half(b + 2), (float)m);
            return __fsub_rn(__fmul_rn(t, (float)q), u);
        }
        case BREW_TYPE_Q6_K: {
            const uint8_t* b = w + (e / 256) * 210;
            const int r = (int)(e % 256), h = r / 128, rr = r % 128, grp = rr / 32, l = rr % 32;
            const int lq = b[64 * h + (grp & 1) * 32 + l];
            const int low = grp < 2 ? (lq & 15) : (lq >> 4);
            const int high = (b[128 + 32 * h + l] >> (2 * grp)) & 3;
            const int q = (low | (high << 4)) - 32;
            const float t = __fmul_rn(ld_half(b + 208), (float)(int8_t)b[192 + r / 16]);
            return __fmul_rn(t, (float)q);
        }
        case BREW_TYPE_F32:
            return reinterpret_cast<const float*>(w)[e];
        case BREW_TYPE_F16:
            return ld_half(w + 2 * e);
    }
    return 0.0f;
}

}  // namespace brew
