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

// ---------------------------------------------------------------- qgemm.cu
// Small-batch GEMM (3..16 vectors) reading every weight unit once: x [nv][cols],
// y [nv][out_stride]. Workspace: qgemm_workspace_bytes (zero before the first
// launch; launches leave it so).
size_t qgemm_workspace_bytes(unsigned type, size_t rows, size_t cols, size_t nv, int sms);
int launch_qgemm(const QWeights &w, unsigned rows, const float *x, float *y, size_t out_stride, unsigned nv,
    void *workspace, size_t workspace_bytes, unsigned *error, int sms, cudaStream_t s);

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
    unsigned queries = 1;           // query rows per sequence; q and out then [nseq][queries][heads][hd]
    float scale = 0.f;
    float *out = nullptr;           // [nseq][heads][hd]
    unsigned splits = 0;            // partitions of the context per (seq, kv head)
    void *workspace = nullptr;
    size_t workspace_bytes = 0;
    bool pdl = false;
};
size_t attention_workspace_bytes(const AttentionLaunch &L);
int launch_attention(const AttentionLaunch &L, cudaStream_t s);

// ---------------------------------------------------------------- decode.cu
// Tensor-parallel exchange region of a plan (byte offsets). Every rank has
// one; rank j writes its partial O and down rows as tagged 8-byte words into
// [xo|xd] + j*d words of every rank's region, its vocabulary slice of the
// logits into `logits`, its best argmax key into keys[j]; counters: keys at
// 2 nl, the shared abort word at 2 nl + 1.
struct XchgLayout {
    size_t xo = 0, xd = 0, logits = 0, keys = 0, ctr = 0, bytes = 0;
};
inline XchgLayout xchg_layout(unsigned tp, unsigned d, unsigned V, unsigned nl)
{
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    XchgLayout x;
    size_t o = 0;
    x.xo = o; o += up((size_t)tp * d * 8);
    x.xd = o; o += up((size_t)tp * d * 8);
    x.logits = o; o += up((size_t)V * 4);
    x.keys = o; o += up((size_t)tp * 8);
    x.ctr = o; o += up(((size_t)2 * nl + 4) * 4);
    x.bytes = o;
    return x;
}

// One decode step of a dense LLaMA model as one persistent kernel.
struct DecodeLayer {
    QWeights qkv, o, gateup, down;  // repacked as for the stand-alone GEMV
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
};
struct DecodeGeometry {
    unsigned nl = 0, d = 0, H = 0, Hkv = 0, hd = 0, ffn = 0, V = 0, capacity = 0;
};
// Vectors handed from phase to phase as tagged 8-byte words {float, tag}
// (zero at plan creation; decode_kernel.cuh describes the tags).
struct DecodeLL {
    unsigned long long *xa = nullptr;     // [d] x after down (tp > 1: the exchange base before O)
    unsigned long long *xm = nullptr;     // [d] x after O (tp > 1: the exchange base before down)
    unsigned long long *q = nullptr;      // [H * hd] q after RoPE
    unsigned long long *kvnew = nullptr;  // [2][Hkv * hd] this position's K (after RoPE) and V, fp16-rounded
    unsigned long long *attn = nullptr;   // [H * hd] attention output
    unsigned long long *h = nullptr;      // [ffn] SwiGLU output
};
inline size_t decode_ll_words(const DecodeGeometry &g)
{
    return (size_t)2 * g.d + (size_t)2 * g.H * g.hd + (size_t)2 * g.Hkv * g.hd + g.ffn;
}
// Device-side synchronization words of a plan (all zero at creation; the
// kernel keeps them consistent from step to step).
struct DecodeSync {
    unsigned *exit_count = nullptr, *abort_flag = nullptr;
    unsigned *logit_tiles = nullptr;
};
struct DecodeLaunch {
    DecodeGeometry g;
    const DecodeLayer *layers = nullptr;  // device array [nl]
    QWeights out_head;
    const float *out_norm = nullptr;
    const unsigned char *embd = nullptr;
    size_t embd_row_bytes = 0;
    unsigned embd_type = 0;
    float eps = 1e-5f, attn_scale = 0.f;
    const float *rope_cos = nullptr, *rope_sin = nullptr;
    unsigned *request = nullptr;  // {token, position, tokens logged, steps, steps with logits}
    DecodeLL ll;
    float *logits = nullptr;
    DecodeSync sync;
    float *attn_partials = nullptr;  // decode_attn_partials_floats()
    unsigned attn_splits = 1;
    unsigned long long *argmax_key = nullptr;
    unsigned *argmax_token = nullptr, *tokens_log = nullptr;
    unsigned *error = nullptr;
    int logits_mode = 1;  // 0 none, 1 logits + argmax, 2 logits + greedy advance
    int grid = 0;
    unsigned long long *trace = nullptr;  // profiling: [decode_trace_points()][grid] globaltimer ns
    unsigned trace_slots = 0;
    unsigned long long *dtrace = nullptr;  // profiling: [grid][16 warps][decode_dtrace_points()] of layer nl / 2
    unsigned ring_bytes = 0;  // per-warp weight ring (0: as much as shared memory allows)
    // tensor parallelism (tp > 1): g holds this rank's heads, FFN rows and
    // vocabulary rows (g.V), the d-row phases exchange partial sums
    unsigned tp = 1, tp_rank = 0, vocab0 = 0;
    unsigned char *const *peers = nullptr;  // device array [tp] of exchange regions
    XchgLayout xl;
    // K and V caches of all layers, layer l at l*kv_heads*capacity*head_dim
    __half *kcache = nullptr, *vcache = nullptr;
};
// Trace points per CTA of one step: start, per layer the ends of QKV,
// attention, O, gate/up and down, the end of the logits, exit.
inline unsigned decode_trace_points(unsigned layers) { return 1 + 5 * layers + 1 + 1; }
inline unsigned decode_dtrace_points() { return 32; }
inline size_t decode_dtrace_words(int grid) { return (size_t)grid * 16 * decode_dtrace_points(); }  // 16 warps per CTA
// Attention partition results: kv_heads x 16 partitions x G x (hd + 2)
// tagged 8-byte words (two floats each).
inline size_t decode_attn_partials_floats(const DecodeGeometry &g)
{
    return (size_t)2 * g.Hkv * 16 * (g.H / g.Hkv) * (g.hd + 2);
}
int decode_supported(const DecodeGeometry &g, unsigned type_out);
int decode_grid(int sms, const DecodeGeometry &g);
int launch_decode(const DecodeLaunch &L, cudaStream_t s);

// ---------------------------------------------------------------- batch.cu
// Elementwise kernels of the batched decode step (B <= BATCH_MAX sequences).
// req on the device: [B] tokens | [B] positions | [B] attended lengths | step.
constexpr unsigned BATCH_MAX = 16;
struct BatchRequest {
    unsigned token[BATCH_MAX], position[BATCH_MAX];
};
int launch_bt_add_norm(float *x, const float *delta, const float *w, float *xn, unsigned d, float eps, unsigned nseq,
    cudaStream_t s);
int launch_bt_rope_kv(const float *y, unsigned qkv_rows, unsigned H, unsigned Hkv, unsigned hd,
    const unsigned *positions, const float *rope_cos, const float *rope_sin, float *q, __half *kc, __half *vc,
    unsigned capacity, unsigned nseq, unsigned slot_div, cudaStream_t s);
int launch_bt_swiglu(const float *y, unsigned ffn, float *h, unsigned nseq, cudaStream_t s);
int launch_bt_argmax(const float *logits, unsigned V, unsigned *req, unsigned nseq, unsigned *tokens_out, unsigned *log,
    bool advance, unsigned *error, cudaStream_t s);
int launch_bt_set(const BatchRequest &r, unsigned *req, unsigned nseq, cudaStream_t s);

}  // namespace fyb
