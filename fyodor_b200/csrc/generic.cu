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

// Q8_0 rows (34-byte blocks: fp16 d, 32 int8) staged in shared memory by one
// bulk copy per CTA: a CTA takes R consecutive rows (contiguous bytes, a
// multiple of 16 when cols % 256 == 0; R <= 8 so that they fit
// Q8_SMEM_MAX). Warp w takes the blocks [nblk w / 8, nblk (w + 1) / 8) of all
// R rows, each half-warp one block at a time: lane l holds values
// 2 (l % 16), +1 of x for NB vectors (loaded once per warp, coalesced) and
// accumulates (d q) x in fp32 for every row (d * q is exact). The warps'
// sums meet in shared memory and add in warp order. The weights cross HBM
// once however many vectors there are.
constexpr unsigned Q8_WARPS = 8;
constexpr unsigned Q8_SMEM_MAX = 100 * 1024;

template <int NB>
__global__ void __launch_bounds__(Q8_WARPS * 32) q8_0_matmul_kernel(const unsigned char *w, unsigned rows,
    unsigned cols, unsigned rpc, const float *x, unsigned long long x_stride, float *y,
    unsigned long long y_stride, int nb)
{
    extern __shared__ __align__(128) unsigned char q8s[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ float red[Q8_WARPS][Q8_WARPS][NB];  // [warp][row][vector]
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5, hl = lane & 15;
    const unsigned row0 = blockIdx.x * rpc, here = min(rpc, rows - row0);
    const unsigned nblk = cols / 32, rb = nblk * 34;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        mbar_expect_tx(&bar, here * rb);
        bulk_copy_g2s(q8s, w + (size_t)row0 * rb, here * rb, &bar);
    }
    const bool landed = mbar_wait_bounded(&bar, 0);  // a copy that never lands yields NaN rows
    float acc[Q8_WARPS][NB];
#pragma unroll
    for (int r = 0; r < (int)Q8_WARPS; ++r)
#pragma unroll
        for (int v = 0; v < NB; ++v) acc[r][v] = landed ? 0.f : __int_as_float(0x7fc00000);
    if (landed) {
        // U block pairs per step: their x loads are all issued before any is
        // used, so a warp waits on one round trip per step
        constexpr int U = NB == 1 ? 8 : NB <= 4 ? 2 : 1;
        const unsigned b0 = nblk * warp / Q8_WARPS, b1 = nblk * (warp + 1) / Q8_WARPS;
        for (unsigned bs = b0 + (lane >> 4); bs < b1; bs += 2 * U) {
            float2 xv[U][NB];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int v = 0; v < NB; ++v) {
                    const unsigned b = bs + 2 * u;
                    xv[u][v] = v < nb && b < b1
                                   ? __ldg(reinterpret_cast<const float2 *>(x + v * x_stride + (size_t)b * 32 + 2 * hl))
                                   : make_float2(0.f, 0.f);
                }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const unsigned b = bs + 2 * u;
                if (b >= b1) break;
#pragma unroll
                for (int r = 0; r < (int)Q8_WARPS; ++r) {
                    if ((unsigned)r < here) {
                        const unsigned char *blk = q8s + (size_t)r * rb + b * 34;
                        const float d = half_bits_to_float(*reinterpret_cast<const unsigned short *>(blk));
                        const unsigned short h = *reinterpret_cast<const unsigned short *>(blk + 2 + 2 * hl);
                        const float q0 = d * (float)(signed char)(h & 0xff), q1 = d * (float)(signed char)(h >> 8);
#pragma unroll
                        for (int v = 0; v < NB; ++v) {
                            acc[r][v] = fmaf(q0, xv[u][v].x, acc[r][v]);
                            acc[r][v] = fmaf(q1, xv[u][v].y, acc[r][v]);
                        }
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < (int)Q8_WARPS; ++r)
#pragma unroll
        for (int v = 0; v < NB; ++v) {
            const float t = warp_sum(acc[r][v]);
            if (lane == 0) red[warp][r][v] = t;
        }
    __syncthreads();
    for (unsigned t = threadIdx.x; t < here * (unsigned)nb; t += blockDim.x) {
        const unsigned r = t / nb, v = t % nb;
        float sum = 0.f;
        for (unsigned w2 = 0; w2 < Q8_WARPS; ++w2) sum += red[w2][r][v];
        y[v * y_stride + row0 + r] = sum;
    }
}

// Rows per CTA (a power of two up to 8) so that they fit Q8_SMEM_MAX bytes;
// 0 if one row alone does not.
static unsigned q8_rows_per_cta(size_t cols)
{
    const size_t rb = cols / 32 * 34;
    for (unsigned r = Q8_WARPS; r >= 1; r /= 2)
        if ((size_t)r * rb <= Q8_SMEM_MAX) return r;
    return 0;
}

static int launch_q8_0_matmul(const void *w, size_t rows, size_t cols, const float *x, size_t x_stride, float *y,
    size_t y_stride, size_t batch, cudaStream_t s)
{
    const unsigned rpc = q8_rows_per_cta(cols);
    const size_t smem = (size_t)rpc * (cols / 32 * 34);
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(q8_0_matmul_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, Q8_SMEM_MAX) ||
            cudaFuncSetAttribute(q8_0_matmul_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, Q8_SMEM_MAX) ||
            cudaFuncSetAttribute(q8_0_matmul_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, Q8_SMEM_MAX))
            return -2;
        attr_set[dev] = true;
    }
    const unsigned blocks = (unsigned)((rows + rpc - 1) / rpc);
    for (size_t b0 = 0; b0 < batch; b0 += 8) {
        const int nb = (int)std::min<size_t>(8, batch - b0);
        const float *xb = x + b0 * x_stride;
        float *yb = y + b0 * y_stride;
        if (nb == 1)
            q8_0_matmul_kernel<1><<<blocks, Q8_WARPS * 32, smem, s>>>((const unsigned char *)w, (unsigned)rows,
                (unsigned)cols, rpc, xb, x_stride, yb, y_stride, nb);
        else if (nb <= 4)
            q8_0_matmul_kernel<4><<<blocks, Q8_WARPS * 32, smem, s>>>((const unsigned char *)w, (unsigned)rows,
                (unsigned)cols, rpc, xb, x_stride, yb, y_stride, nb);
        else
            q8_0_matmul_kernel<8><<<blocks, Q8_WARPS * 32, smem, s>>>((const unsigned char *)w, (unsigned)rows,
                (unsigned)cols, rpc, xb, x_stride, yb, y_stride, nb);
        if (cudaGetLastError() != cudaSuccess) return -2;
    }
    return 0;
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
    if (type == T_Q8_0 && cols % 256 == 0 && q8_rows_per_cta(cols) && rows <= 0x7fffffffu && x_stride % 4 == 0 &&
        (reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0)
        return launch_q8_0_matmul(w, rows, cols, x, x_stride, y, y_stride, batch, s);
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
