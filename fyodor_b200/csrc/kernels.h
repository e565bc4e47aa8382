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
// Tensor-core GEMV weights: Q4_K / Q6_K matrices repacked into units of
// 16 rows x 256 columns, unit (tile t, block b) at units + (t*nblk + b)*unit,
// unit = 2304 B (Q4_K) or 3360 B (Q6_K). A fused matrix stacks the tiles of
// several tensors (REPACK_QKV puts rows 2i and 2i+1 of every 16-row tile in
// the same lane; REPACK_GATEUP interleaves 8 gate rows with 8 up rows).
enum RepackMode { REPACK_PLAIN = 0, REPACK_QKV = 1, REPACK_GATEUP = 2 };
struct QWeights {
    const unsigned char *units = nullptr;
    unsigned type = 0, cols = 0, tiles = 0;
};
size_t qunits_bytes(unsigned type, size_t tiles, size_t cols);
// Repack `tiles` tiles of a raw GGUF matrix (rows x cols, device memory) into
// dst_units; REPACK_GATEUP reads the up rows from src1.
int repack_units(const void *src0, const void *src1, size_t rows, size_t cols, unsigned type, int mode,
    void *dst_units, size_t tiles, cudaStream_t s);

enum QgEpilogue { EPI_STORE = 0, EPI_QKV = 1, EPI_SWIGLU = 2, EPI_LOGITS = 3 };

// One fused GEMV launch over a repacked matrix whose tiles belong to up to
// three output segments (QKV: q, k, v; SWIGLU: gate and up rows paired).
struct QgemvLaunch {
    int epilogue = EPI_STORE;
    QWeights w;
    int nseg = 1;
    unsigned seg_rows[3] = {0, 0, 0};
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
    // stream-K scratch: per-tile counters (zero before the first launch;
    // launches leave them zero) and partial sums
    unsigned *counters = nullptr;
    size_t counters_capacity = 0;  // entries
    float *partials = nullptr;
    size_t partials_bytes = 0;
    unsigned *error = nullptr;
    int grid = 0;       // CTAs (0: one per SM)
    bool pdl = false;   // programmatic dependent launch
};
unsigned qgemv_tiles(const QgemvLaunch &L);
size_t qgemv_partials_bytes(const QgemvLaunch &L, int grid);
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
