// generic.cu - type-generic kernels: bit-exact dequantization, a warp-per-row
// matmul for every storage type and shape the engine can pass, and the
// embedding-row gather. These cover the engine contract everywhere the
// tensor-core GEMV (qgemv.cu) does not apply; they are not on the 8B decode
// hot path except for the one-row gather.
#include "common.cuh"
#include "dequant.cuh"
#include "kernels.h"

namespace fyb {

template <unsigned TYPE>
__global__ void dequant_kernel(const unsigned char *w, unsigned long long count, float *out)
{
    unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
    unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
    for (; i < count; i += stride) out[i] = dequant_at<TYPE>(w, i);
}

// y[b][r] = sum_k W[r][k] * x[b][k] for b < NB. One warp per row; lanes stride
// over columns; the 32 lane partials meet in a butterfly reduction.
template <unsigned TYPE, int NB>
__global__ void __launch_bounds__(256) generic_matmul_kernel(const unsigned char *w, unsigned long long row_bytes,
    unsigned long long rows, unsigned long long cols, const float *x, unsigned long long x_stride,
    float *y, unsigned long long y_stride, int nb)
{
    unsigned lane = threadIdx.x & 31;
    unsigned long long row = (unsigned long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const unsigned char *wr = w + row * row_bytes;
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
    for (unsigned long long k = lane; k < cols; k += 32) {
        float v = dequant_at<TYPE>(wr, k);
#pragma unroll
        for (int b = 0; b < NB; ++b)
            if (b < nb) acc[b] = fmaf(v, __ldg(x + b * x_stride + k), acc[b]);
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        float s = warp_sum(acc[b]);
        if (lane == 0 && b < nb) y[b * y_stride + row] = s;
    }
}

// One embedding row (token from the device request word when present).
template <unsigned TYPE>
__global__ void gather_kernel(const unsigned char *w, unsigned long long row_bytes, unsigned long long n,
    const unsigned *token_ptr, unsigned token, float *out)
{
    pdl_wait();
    if (token_ptr) token = *token_ptr;
    const unsigned char *wr = w + (unsigned long long)token * row_bytes;
    for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (unsigned long long)gridDim.x * blockDim.x)
        out[i] = dequant_at<TYPE>(wr, i);
    pdl_launch_dependents();
}

// Batch of embedding rows for prefill: out[t][i] = dequant(row tokens[t]).
template <unsigned TYPE>
__global__ void gather_batch_kernel(const unsigned char *w, unsigned long long row_bytes, unsigned long long n,
    const unsigned *tokens, unsigned count, float *out)
{
    unsigned long long total = n * count;
    for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (unsigned long long)gridDim.x * blockDim.x) {
        unsigned t = (unsigned)(i / n);
        out[i] = dequant_at<TYPE>(w + (unsigned long long)tokens[t] * row_bytes, i % n);
    }
}

#define FYB_TYPE_SWITCH(type, ...)                                   \
    switch (type) {                                                  \
    case T_F32: { constexpr unsigned TT = T_F32; __VA_ARGS__; } break;  \
    case T_F16: { constexpr unsigned TT = T_F16; __VA_ARGS__; } break;  \
    case T_BF16: { constexpr unsigned TT = T_BF16; __VA_ARGS__; } break; \
    case T_Q8_0: { constexpr unsigned TT = T_Q8_0; __VA_ARGS__; } break; \
    case T_Q4_0: { constexpr unsigned TT = T_Q4_0; __VA_ARGS__; } break; \
    case T_Q4_K: { constexpr unsigned TT = T_Q4_K; __VA_ARGS__; } break; \
    case T_Q6_K: { constexpr unsigned TT = T_Q6_K; __VA_ARGS__; } break; \
    default: return -1;                                              \
    }

int launch_dequant(const void *w, unsigned type, size_t count, float *out, cudaStream_t s)
{
    if (count == 0) return 0;
    unsigned blocks = (unsigned)std::min<size_t>((count + 255) / 256, 148 * 16);
    FYB_TYPE_SWITCH(type, dequant_kernel<TT><<<blocks, 256, 0, s>>>((const unsigned char *)w, count, out));
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int launch_generic_matmul(const void *w, size_t row_bytes, size_t rows, size_t cols, unsigned type,
    const float *x, size_t x_stride, float *y, size_t y_stride, size_t batch, cudaStream_t s)
{
    if (rows == 0 || batch == 0) return 0;
    unsigned blocks = (unsigned)((rows + 7) / 8);
    for (size_t b0 = 0; b0 < batch; b0 += 8) {
        int nb = (int)std::min<size_t>(8, batch - b0);
        const float *xb = x + b0 * x_stride;
        float *yb = y + b0 * y_stride;
#define FYB_GM(NBV) generic_matmul_kernel<TT, NBV><<<blocks, 256, 0, s>>>((const unsigned char *)w, row_bytes, rows, cols, xb, x_stride, yb, y_stride, nb)
        if (nb == 1) { FYB_TYPE_SWITCH(type, FYB_GM(1)); }
        else if (nb <= 2) { FYB_TYPE_SWITCH(type, FYB_GM(2)); }
        else if (nb <= 4) { FYB_TYPE_SWITCH(type, FYB_GM(4)); }
        else { FYB_TYPE_SWITCH(type, FYB_GM(8)); }
#undef FYB_GM
        if (cudaGetLastError() != cudaSuccess) return -2;
    }
    return 0;
}

int launch_gather(const void *w, size_t row_bytes, unsigned type, size_t n, const unsigned *token_ptr,
    unsigned token, float *out, cudaStream_t s, bool pdl)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((n + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaErrorInvalidValue;
    FYB_TYPE_SWITCH(type, e = cudaLaunchKernelEx(&cfg, gather_kernel<TT>, (const unsigned char *)w,
        (unsigned long long)row_bytes, (unsigned long long)n, token_ptr, token, out));
    return e == cudaSuccess ? 0 : -2;
}

int launch_gather_batch(const void *w, size_t row_bytes, unsigned type, size_t n, const unsigned *tokens,
    unsigned count, float *out, cudaStream_t s)
{
    size_t total = n * count;
    unsigned blocks = (unsigned)std::min<size_t>((total + 255) / 256, 148 * 16);
    FYB_TYPE_SWITCH(type, gather_batch_kernel<TT><<<blocks, 256, 0, s>>>((const unsigned char *)w,
        (unsigned long long)row_bytes, (unsigned long long)n, tokens, count, out));
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace fyb
