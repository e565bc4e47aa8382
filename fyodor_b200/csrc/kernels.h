// kernels.h - host-side launch interface of the provider's CUDA kernels.
#pragma once
#include <cstddef>
#include <cstdint>
#include <algorithm>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace fyb {

// ---------------------------------------------------------------- generic.cu
int launch_dequant(const void *w, unsigned type, size_t count, float *out, cudaStream_t s);
int launch_generic_matmul(const void *w, size_t row_bytes, size_t rows, size_t cols, unsigned type,
    const float *x, size_t x_stride, float *y, size_t y_stride, size_t batch, cudaStream_t s);
int launch_gather(const void *w, size_t row_bytes, unsigned type, size_t n, const unsigned *token_ptr,
    unsigned token, float *out, cudaStream_t s, bool pdl);
int launch_gather_batch(const void *w, size_t row_bytes, unsigned type, size_t n, const unsigned *tokens,
    unsigned count, float *out, cudaStream_t s);

// ---------------------------------------------------------------- qgemv.cu
// Device layout of a K-quant matrix used by the tensor-core GEMV.
//   Q4_K: the GGUF bytes unchanged (rows x nblk x 144 B).
//   Q6_K: repacked by repack_q6k(): three regions
//         bits  rows x nblk x 192 B   (ql 128 + qh 64 per block; inside every
//                                       32-byte run the bytes are interleaved
//                                       [0-3,16-19,4-7,20-23,8-11,24-27,12-15,28-31])
//         scale rows x nblk x 16 B    (the int8 sub-block scales)
//         d     rows x nblk x 4 B     (the fp16 super-block scale widened to f32)
struct QMatrix {
    const unsigned char *bits = nullptr;
    const signed char *scales = nullptr;
    const float *d = nullptr;
    unsigned rows = 0;
    unsigned cols = 0;
    unsigned type = 0;
};
size_t q6k_repacked_bytes(size_t rows, size_t cols);
int repack_q6k(const void *raw, size_t rows, size_t cols, void *dst, QMatrix *out, cudaStream_t s);
QMatrix q4k_matrix(const void *raw, size_t rows, size_t cols);

enum QgEpilogue { EPI_STORE = 0, EPI_QKV = 1, EPI_SWIGLU = 2, EPI_LOGITS = 3 };

// One fused GEMV launch. Up to three matrices ("segments") share the input
// vector and are tiled independently (EPI_SWIGLU pairs segment 0 and 1 row
// for row instead).
struct QgemvLaunch {
    int epilogue = EPI_STORE;
    int nseg = 1;
    QMatrix seg[3];
    float *out[3] = {nullptr, nullptr, nullptr};   // STORE/LOGITS/SWIGLU: out[0]; QKV: q
    __half *kcache = nullptr, *vcache = nullptr;   // QKV: this layer's [kv_heads][capacity][hd]
    size_t out_stride = 0;                          // per-vector output stride (floats)
    int nvec = 1;                                   // 1 or 2 input vectors
    // input vector preparation
    const float *x = nullptr;       // [nvec][K]
    const float *delta = nullptr;   // optional: x + delta is the residual stream
    float *x_out = nullptr;         // optional: where x + delta is written back
    const float *norm_w = nullptr;  // optional RMSNorm weight (F32)
    float eps = 1e-5f;
    // RoPE / KV append (QKV)
    const float *rope_cos = nullptr, *rope_sin = nullptr;  // [capacity][hd/2]
    const unsigned *request = nullptr;                      // device {token, position}
    unsigned position = 0;
    unsigned head_dim = 128;
    unsigned capacity = 0;
    // greedy argmax (LOGITS)
    unsigned long long *argmax_key = nullptr;  // [nvec]
    unsigned *argmax_token = nullptr;          // [nvec] result token
    unsigned *tiles_done = nullptr;
    // scratch for the stream-K fix-up (see qgemv_workspace_bytes)
    void *workspace = nullptr;
    size_t workspace_bytes = 0;
    unsigned *error = nullptr;
    int grid = 0;       // CTAs (0: one per SM)
    bool pdl = false;   // programmatic dependent launch
};
size_t qgemv_workspace_bytes(const QgemvLaunch &L, int grid);
int qgemv_supported(unsigned type, size_t cols, size_t nvec);
int launch_qgemv(const QgemvLaunch &L, cudaStream_t s);

// ---------------------------------------------------------------- attention.cu
struct AttentionLaunch {
    const float *q = nullptr;       // [nseq][heads][hd]
    const __half *k = nullptr;      // per sequence: [kv_heads][capacity][hd]
    const __half *v = nullptr;
    size_t seq_stride = 0;          // elements between sequences' caches (0: one sequence)
    const unsigned *lengths = nullptr;  // device: attended length per sequence (or null)
    const unsigned *request = nullptr;  // device {token, position}: length = position + 1
    unsigned length = 0;            // host length when both pointers are null
    unsigned nseq = 1, heads = 32, kv_heads = 8, head_dim = 128, capacity = 0;
    float scale = 0.f;
    float *out = nullptr;           // [nseq][heads][hd]
    unsigned splits = 0;            // partitions of the context per (seq, kv head)
    void *workspace = nullptr;
    size_t workspace_bytes = 0;
    bool pdl = false;
};
size_t attention_workspace_bytes(const AttentionLaunch &L);
int launch_attention(const AttentionLaunch &L, cudaStream_t s);

}  // namespace fyb
