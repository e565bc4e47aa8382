// dequant.cuh - per-element GGUF dequantization, bit-exact with the engine.
//
// Each branch restates nya_llm_tensor_value (backend/core/llm_quant.c:91-142)
// including its evaluation order: the engine is built as ISO C17, so no
// multiply-add is contracted. The explicit __fmul_rn/__fsub_rn keep nvcc from
// fusing them either, which is what makes the values bit-identical.
#pragma once
#include "common.cuh"

namespace fyb {

template <unsigned TYPE>
FYB_DEV float dequant_at(const unsigned char *base, unsigned long long i)
{
    if constexpr (TYPE == T_F32) {
        return __ldg(reinterpret_cast<const float *>(base) + i);
    } else if constexpr (TYPE == T_F16) {
        return half_at(base + i * 2);
    } else if constexpr (TYPE == T_BF16) {
        const unsigned char *p = base + i * 2;
        return __uint_as_float(((unsigned)p[0] | ((unsigned)p[1] << 8)) << 16);
    } else if constexpr (TYPE == T_Q8_0) {
        const unsigned char *b = base + (i / 32) * 34;
        return __fmul_rn(half_at(b), (float)(signed char)b[2 + i % 32]);
    } else if constexpr (TYPE == T_Q4_0) {
        const unsigned char *b = base + (i / 32) * 18;
        unsigned o = (unsigned)(i % 32);
        unsigned char packed = b[2 + o % 16];
        int q = o < 16 ? (packed & 15) : (packed >> 4);
        return __fmul_rn(half_at(b), (float)(q - 8));
    } else if constexpr (TYPE == T_Q4_K) {
        const unsigned char *b = base + (i / 256) * 144;
        unsigned j = (unsigned)(i % 256), g = j / 32;
        const unsigned char *s = b + 4;
        unsigned sc = g < 4 ? s[g] & 63u : (s[g + 4] & 15u) | ((unsigned)(s[g - 4] >> 6) << 4);
        unsigned mn = g < 4 ? s[g + 4] & 63u : (s[g + 4] >> 4) | ((unsigned)(s[g] >> 6) << 4);
        unsigned q = (b[16 + g / 2 * 32 + j % 32] >> (g % 2 * 4)) & 15u;
        return __fsub_rn(__fmul_rn(__fmul_rn(half_at(b), (float)sc), (float)q),
                         __fmul_rn(half_at(b + 2), (float)mn));
    } else {  // T_Q6_K
        const unsigned char *b = base + (i / 256) * 210;
        unsigned j = (unsigned)(i % 256), half = j / 128, quarter = j % 128 / 32, lane = j % 32;
        unsigned lo = b[half * 64 + quarter % 2 * 32 + lane], hi = b[128 + half * 32 + lane];
        int q = (int)(((lo >> (quarter / 2 * 4)) & 15u) | (((hi >> (quarter * 2)) & 3u) << 4)) - 32;
        int sc = (signed char)b[192 + half * 8 + quarter * 2 + lane / 16];
        return __fmul_rn(__fmul_rn(half_at(b + 208), (float)sc), (float)q);
    }
}

// Runtime-dispatched form for code that is not on a hot loop.
FYB_DEV float dequant_any(const unsigned char *base, unsigned long long i, unsigned type)
{
    switch (type) {
    case T_F32: return dequant_at<T_F32>(base, i);
    case T_F16: return dequant_at<T_F16>(base, i);
    case T_BF16: return dequant_at<T_BF16>(base, i);
    case T_Q8_0: return dequant_at<T_Q8_0>(base, i);
    case T_Q4_0: return dequant_at<T_Q4_0>(base, i);
    case T_Q4_K: return dequant_at<T_Q4_K>(base, i);
    default: return dequant_at<T_Q6_K>(base, i);
    }
}

}  // namespace fyb
