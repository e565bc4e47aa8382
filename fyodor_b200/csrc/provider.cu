// provider.cu - the engine-facing provider: nya_backend_interface for B200.
//
// Context (create/destroy/active/matvec/matmul) follows CUDA/cuda.c:179-456:
// a weight cache keyed by the borrowed host pointer (cuda.c:23,382-395), a
// memory budget of free - max(10%, 256 MiB) overridable by
// NYA_CUDA_MEMORY_MIB (cuda.c:314-328), argument validation before any write
// (cuda.c:366-378) and poisoning on a driver failure (cuda.c:430-433).
// Plans (plan_create/free/token/prefill/stats/read_kv) follow
// CUDA/resident.inc: whole-plan admission (:109-308), single-token decode as a
// captured CUDA graph replayed per token (:434-580), logits download with the
// finiteness check and suppression list (:563-570), KV snapshot (:601-630)
// and the fault-injection switches NYA_CUDA_FAIL_AFTER /
// NYA_CUDA_FAIL_ALLOCATION_AFTER (:184-198, :100-107).
//
// What differs is below the vtable: one fused kernel per projection group
// (QKV+RoPE+KV append, O, gate/up+SwiGLU, down, logits+argmax) on the
// integer tensor cores, an fp16 KV cache, split-K attention, and graph nodes
// chained with programmatic dependent launch.
#include "fyodor_b200.h"
#include "common.cuh"
#include "kernels.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

// the batched step (defined after the plan): also the plan's prompt chunker
namespace fyb { struct Plan; }
struct Batch;
static void batch_free(Batch *bt);
static Batch *batch_create(fyb::Plan *p, unsigned batch, bool chunk);
static int prefill_chunks(fyb::Plan *p, Batch *bt, const uint32_t *tokens, size_t count, size_t position, float *out);

namespace fyb {

static bool debug_enabled() { return std::getenv("NYA_CUDA_DEBUG") != nullptr; }
static void debug(const char *what, cudaError_t e)
{
    if (debug_enabled()) std::fprintf(stderr, "fyodor_b200: %s: %s\n", what, cudaGetErrorString(e));
}

static bool env_size(const char *name, size_t *out)
{
    const char *s = std::getenv(name);
    if (!s || s[0] < '0' || s[0] > '9') return false;
    char *end;
    unsigned long long v = std::strtoull(s, &end, 10);
    if (*end) return false;
    *out = (size_t)v;
    return true;
}

static bool type_geometry(unsigned type, size_t *block, size_t *bytes)
{
    switch (type) {
    case T_F32: *block = 1; *bytes = 4; return true;
    case T_F16: case T_BF16: *block = 1; *bytes = 2; return true;
    case T_Q4_0: *block = 32; *bytes = 18; return true;
    case T_Q8_0: *block = 32; *bytes = 34; return true;
    case T_Q4_K: *block = 256; *bytes = 144; return true;
    case T_Q6_K: *block = 256; *bytes = 210; return true;
    default: return false;
    }
}

// Scoped device selection: the caller's current device is restored on exit
// (the runtime-API form of the push/pop etiquette in cuda.c:179-204).
struct DeviceScope {
    int previous = -1;
    bool ok = false;
    explicit DeviceScope(int device)
    {
        if (cudaGetDevice(&previous) != cudaSuccess) previous = -1;
        ok = cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceScope()
    {
        if (previous >= 0) cudaSetDevice(previous);
    }
};

// ======================================================================
// Context
// ======================================================================
struct CachedWeight {
    const void *source = nullptr;
    size_t rows = 0, cols = 0, bytes = 0;
    unsigned type = 0;
    void *dev = nullptr;  // GGUF bytes (generic types) or tensor-core units (K-quants)
    QWeights qw;
};

struct Context {
    int device = 0;
    cudaStream_t stream = nullptr;
    size_t cache_limit = 0, cached_bytes = 0;
    std::vector<CachedWeight> weights;
    bool failed = false;
    float *dx = nullptr, *dy = nullptr;
    size_t dx_bytes = 0, dy_bytes = 0;
    unsigned *counters = nullptr;  // stream-K tile counters, kept zero between launches
    size_t counters_bytes = 0;
    float *partials = nullptr;
    size_t partials_bytes = 0;
    void *gemm = nullptr;  // small-batch GEMM workspace, kept zero between launches
    size_t gemm_bytes = 0;
    int sms = 148;
};

constexpr size_t WEIGHT_LIMIT = 2048;

static void context_free(Context *c)
{
    if (!c) return;
    {
        DeviceScope scope(c->device);
        if (c->stream) cudaStreamSynchronize(c->stream);
        for (auto &w : c->weights) cudaFree(w.dev);
        cudaFree(c->dx); cudaFree(c->dy); cudaFree(c->counters); cudaFree(c->partials); cudaFree(c->gemm);
        if (c->stream) cudaStreamDestroy(c->stream);
    }
    delete c;
}

static Context *context_create()
{
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
        cudaGetLastError();
        if (debug_enabled()) std::fprintf(stderr, "fyodor_b200: no CUDA device; CPU fallback selected\n");
        return nullptr;
    }
    size_t dev = 0;
    env_size("NYA_CUDA_DEVICE", &dev);
    if ((int)dev >= count) return nullptr;
    Context *c = new Context();
    c->device = (int)dev;
    DeviceScope scope(c->device);
    if (!scope.ok) { delete c; return nullptr; }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, c->device) != cudaSuccess || prop.major < 10) {
        // sm_100a code only: anything else declines and keeps the CPU path
        if (debug_enabled()) std::fprintf(stderr, "fyodor_b200: device is not sm_100; declining\n");
        delete c;
        return nullptr;
    }
    c->sms = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) { delete c; return nullptr; }
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) { context_free(c); return nullptr; }
    size_t reserve = std::max<size_t>(free_b / 10, (size_t)256 << 20);
    c->cache_limit = free_b > reserve ? free_b - reserve : 0;
    size_t mib;
    if (env_size("NYA_CUDA_MEMORY_MIB", &mib) && mib * ((size_t)1 << 20) < c->cache_limit) c->cache_limit = mib << 20;
    return c;
}

static int grow(void **p, size_t *cap, size_t bytes, bool zero)
{
    if (*cap >= bytes) return 0;
    void *n = nullptr;
    if (cudaMalloc(&n, bytes) != cudaSuccess) { cudaGetLastError(); return -1; }
    if (zero && (cudaMemset(n, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)) { cudaFree(n); return -1; }
    if (*p) cudaFree(*p);
    *p = n;
    *cap = bytes;
    return 0;
}

// Tensor-core units of a raw device matrix (freed by the caller).
static int repack_plain(const void *raw, size_t rows, size_t cols, unsigned type, void **units, QWeights *qw,
    cudaStream_t s)
{
    const size_t tiles = (rows + 15) / 16;
    if (cudaMalloc(units, qunits_bytes(type, tiles, cols)) != cudaSuccess) { cudaGetLastError(); return -1; }
    if (repack_units(raw, nullptr, rows, cols, type, REPACK_PLAIN, *units, tiles, s) ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        cudaFree(*units); *units = nullptr; return -1;
    }
    qw->units = (const unsigned char *)*units; qw->type = type; qw->cols = (unsigned)cols; qw->tiles = (unsigned)tiles;
    return 0;
}

// Host-to-device copy ordered on `s`. A plain cudaMemcpy from pageable memory
// may return before its DMA lands and is ordered only on the legacy stream,
// which the provider's non-blocking stream does not wait for (the reference
// documents the same hazard in CUDA/cuda.c:399-403).
static bool upload(void *dst, const void *src, size_t bytes, cudaStream_t s)
{
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s) == cudaSuccess;
}

static CachedWeight *cached_weight(Context *c, const void *w, size_t rows, size_t cols, unsigned type, size_t bytes)
{
    for (auto &e : c->weights)
        if (e.source == w && e.rows == rows && e.cols == cols && e.type == type) return &e;
    if (c->weights.size() >= WEIGHT_LIMIT) return nullptr;
    const bool tc = qgemv_supported(type, cols, 1);
    const size_t resident = tc ? qunits_bytes(type, (rows + 15) / 16, cols) : bytes;
    if (resident > c->cache_limit - std::min(c->cache_limit, c->cached_bytes)) return nullptr;
    CachedWeight e;
    e.source = w; e.rows = rows; e.cols = cols; e.type = type; e.bytes = resident;
    void *raw = nullptr;
    if (cudaMalloc(&raw, bytes) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    if (!upload(raw, w, bytes, c->stream)) { cudaFree(raw); return nullptr; }
    if (tc) {
        const int r = repack_plain(raw, rows, cols, type, &e.dev, &e.qw, c->stream);
        cudaFree(raw);
        if (r) return nullptr;
    } else {
        e.dev = raw;
    }
    c->cached_bytes += e.bytes;
    c->weights.push_back(e);
    return &c->weights.back();
}

struct Scratch {
    unsigned **counters;
    size_t *counters_bytes;
    float **partials;
    size_t *partials_bytes;
    void **gemm;          // small-batch GEMM workspace (zero between launches)
    size_t *gemm_bytes;
};

// Y[b] = W X[b] on resident data. K-quants: batches of 3 or more run the
// weight-reusing small-batch GEMM in groups of up to 16 vectors (each weight
// read once per group); one or two vectors (and a remainder of one or two)
// run the tensor-core GEMV. Every other type runs the generic kernel.
static int device_matmul(const QWeights *qw, const void *raw, size_t row_bytes, size_t rows, size_t cols,
    unsigned type, const float *x, float *y, size_t batch, const Scratch &sc, cudaStream_t s, int sms)
{
    if (qw && qw->units) {
        for (size_t b0 = 0; b0 < batch;) {
            const size_t left = batch - b0;
            if (left >= 3) {
                const unsigned nv = (unsigned)std::min<size_t>(16, left);
                const size_t need = qgemm_workspace_bytes(type, rows, cols, nv, sms);
                if (!need || grow(sc.gemm, sc.gemm_bytes, need, true)) return -2;
                const int r = launch_qgemm(*qw, (unsigned)rows, x + b0 * cols, y + b0 * rows, rows, nv, *sc.gemm,
                                           *sc.gemm_bytes, nullptr, sms, s);
                if (r) return r;
                b0 += nv;
                continue;
            }
            const int nvec = (int)std::min<size_t>(2, left);
            if (!qgemv_supported(type, cols, nvec)) return -1;
            QgemvLaunch L;
            L.epilogue = EPI_STORE;
            L.w = *qw;
            L.seg_rows[0] = (unsigned)rows;
            L.nvec = nvec;
            L.x = x + b0 * cols;
            L.out[0] = y + b0 * rows;
            L.out_stride = rows;
            L.grid = sms;
            if (grow((void **)sc.counters, sc.counters_bytes, (size_t)qw->tiles * 4, true) ||
                grow((void **)sc.partials, sc.partials_bytes, qgemv_partials_bytes(L, sms), false))
                return -2;
            L.counters = *sc.counters; L.counters_capacity = *sc.counters_bytes / 4;
            L.partials = *sc.partials; L.partials_bytes = *sc.partials_bytes;
            const int r = launch_qgemv(L, s);
            if (r) return r;
            b0 += (size_t)nvec;
        }
        return 0;
    }
    return launch_generic_matmul(raw, row_bytes, rows, cols, type, x, cols, y, rows, batch, s);
}

static int context_matmul(Context *c, const void *w, size_t rows, size_t cols, unsigned type, const float *x,
    float *y, size_t batch)
{
    size_t block, bbytes;
    if (!c || c->failed || !w || !x || !y || rows == 0 || cols == 0 || batch == 0 || batch > 512 ||
        cols > SIZE_MAX / sizeof(float) / batch || rows > SIZE_MAX / sizeof(float) / batch ||
        !type_geometry(type, &block, &bbytes) || cols % block != 0 || cols / block > SIZE_MAX / bbytes)
        return -1;
    const size_t row_bytes = cols / block * bbytes;
    if (rows > SIZE_MAX / row_bytes || rows > 0x7fffffffu) return -1;
    DeviceScope scope(c->device);
    if (!scope.ok) { c->failed = true; return -1; }
    CachedWeight *e = cached_weight(c, w, rows, cols, type, rows * row_bytes);
    if (!e) return -1;  // cache full or over budget: the engine runs its CPU kernel
    int result = -1;
    do {
        if (grow((void **)&c->dx, &c->dx_bytes, cols * batch * sizeof(float), false) ||
            grow((void **)&c->dy, &c->dy_bytes, rows * batch * sizeof(float), false))
            break;
        if (cudaMemcpyAsync(c->dx, x, cols * batch * sizeof(float), cudaMemcpyHostToDevice, c->stream) != cudaSuccess) break;
        const Scratch sc{&c->counters, &c->counters_bytes, &c->partials, &c->partials_bytes, &c->gemm, &c->gemm_bytes};
        if (device_matmul(e->qw.units ? &e->qw : nullptr, e->dev, row_bytes, rows, cols, type, c->dx, c->dy, batch,
                          sc, c->stream, c->sms) != 0)
            break;
        if (cudaMemcpyAsync(y, c->dy, rows * batch * sizeof(float), cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) break;
        if (cudaStreamSynchronize(c->stream) != cudaSuccess) break;
        result = 0;
    } while (0);
    if (result) {
        debug("matmul failed", cudaGetLastError());
        c->failed = true;
    }
    return result;
}

// ======================================================================
// Resident plan
// ======================================================================
struct LayerW {
    QWeights qkv, o, gateup, down;
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
};

enum StepMode { STEP_LOGITS = 0, STEP_NO_LOGITS = 1, STEP_GREEDY = 2 };
enum KernelClass { KC_MATRIX = 0, KC_ATTENTION = 1, KC_OTHER = 2 };

struct Plan {
    Context *ctx = nullptr;
    const nya_llm_context *m = nullptr;
    size_t capacity = 0;
    unsigned d = 0, H = 0, Hkv = 0, hd = 0, ffn = 0, V = 0, nl = 0;
    float eps = 1e-5f;
    std::vector<void *> allocations;
    std::vector<LayerW> layers;
    QWeights out_head;
    const void *embd = nullptr;
    size_t embd_row_bytes = 0;
    unsigned embd_type = 0;
    const float *out_norm = nullptr;
    __half *kcache = nullptr, *vcache = nullptr;
    float *x[2] = {nullptr, nullptr};
    float *delta = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr, *logits = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    unsigned *request = nullptr;  // {token, position, step, 0}
    unsigned long long *argmax_key = nullptr;
    unsigned *argmax_token = nullptr, *tiles_done = nullptr, *tokens_log = nullptr;
    unsigned *counters = nullptr;   // stream-K tile counters shared by every GEMV of the step
    size_t counters_capacity = 0;
    float *partials = nullptr;
    size_t partials_bytes = 0;
    void *attn_ws = nullptr;
    size_t attn_ws_bytes = 0;
    unsigned attn_splits = 1;
    unsigned *err_host = nullptr, *err_dev = nullptr;
    cudaGraphExec_t graphs[3] = {nullptr, nullptr, nullptr};
    unsigned long long graph_kernels[3] = {0, 0, 0};
    bool use_graphs = true, failed = false;
    size_t valid = 0;
    size_t fail_after = SIZE_MAX, allocation_count = 0, fail_allocation_after = SIZE_MAX;
    nya_compute_stats stats;
    unsigned long long launches = 0;  // counted while enqueuing
    std::vector<uint16_t> kv_stage;
    // profiling: when set, an event is recorded after every launch (second:
    // kernel class | projection << 4)
    std::vector<std::pair<cudaEvent_t, int>> *marks = nullptr;
    // NYA_CUDA_PROFILE=1: every step runs the per-operation kernels without
    // graphs, timed per kernel class and per projection, printed at plan_free
    bool profile = false;
    double prof_ms[4] = {0, 0, 0, 0};     // matrix, attention, other, prefill chunks
    double prof_proj_ms[5] = {0, 0, 0, 0, 0};
    unsigned long long prof_proj_calls[5] = {0, 0, 0, 0, 0}, prof_steps = 0;
    // persistent decode kernel (decode.cu); dec_grid == 0: per-kernel launches
    int dec_grid = 0;
    DecodeLayer *dec_layers = nullptr;
    DecodeSync dec_sync;
    DecodeLL dec_ll;
    float *dec_attn = nullptr;
    unsigned dec_splits = 1;
    size_t dec_bytes = 0;
    unsigned dec_ring_bytes = 0;  // per-warp weight ring; NYA_CUDA_RING_BYTES (0 = as much as fits)
    // tensor parallelism: this plan holds rank tp_rank's shard of tp_size
    // (H, Hkv and ffn above are this rank's; V is the whole vocabulary)
    unsigned tp_size = 1, tp_rank = 0, vocab_rows = 0, vocab0 = 0;
    unsigned char *xchg = nullptr;     // exchange region peers write into (tp_size > 1)
    size_t xchg_bytes = 0;
    XchgLayout xl;
    unsigned char **peers_dev = nullptr;  // [tp_size] device pointers to every rank's region
    std::vector<unsigned char *> peers;   // host copy; peers opened through IPC are closed on free
    bool connected = false;
    // chunked prefill: prompt chunks of up to BATCH_MAX tokens through the
    // batched step, writing this plan's own KV cache (created on first use)
    ::Batch *prefill = nullptr;
    bool prefill_tried = false;
};

static void *plan_alloc(Plan *p, size_t bytes)
{
    if (p->allocation_count >= p->fail_allocation_after) return nullptr;
    void *d = nullptr;
    if (cudaMalloc(&d, bytes ? bytes : 256) != cudaSuccess) {
        cudaGetLastError();
        std::fprintf(stderr, "fyodor_b200: resident allocation of %zu bytes failed\n", bytes);
        return nullptr;
    }
    ++p->allocation_count;
    p->allocations.push_back(d);
    return d;
}

static void plan_free(void *opaque)
{
    Plan *p = (Plan *)opaque;
    if (!p) return;
    if (p->profile) {
        std::fprintf(stderr,
                     "fyodor_b200 profile: steps=%llu kernel GPU milliseconds: matrix=%.3f attention=%.3f other=%.3f "
                     "prefill_chunks=%.3f (per-operation kernels, graphs off)\n",
                     p->prof_steps, p->prof_ms[0], p->prof_ms[1], p->prof_ms[2], p->prof_ms[3]);
        static const char *names[5] = {"qkv", "o", "gateup", "down", "logits"};
        const QWeights *w[5] = {p->layers.empty() ? nullptr : &p->layers[0].qkv,
                                p->layers.empty() ? nullptr : &p->layers[0].o,
                                p->layers.empty() ? nullptr : &p->layers[0].gateup,
                                p->layers.empty() ? nullptr : &p->layers[0].down, &p->out_head};
        for (int k = 0; k < 5; ++k)
            if (p->prof_proj_calls[k] && w[k])
                std::fprintf(stderr, "fyodor_b200 matrix profile: projection=%s type=%u rows=%u columns=%u calls=%llu "
                             "milliseconds=%.6f\n", names[k], w[k]->type, w[k]->tiles * 16, w[k]->cols,
                             p->prof_proj_calls[k], p->prof_proj_ms[k]);
    }
    if (p->prefill) ::batch_free(p->prefill);
    {
        DeviceScope scope(p->ctx->device);
        cudaStreamSynchronize(p->ctx->stream);
        for (auto &g : p->graphs) if (g) cudaGraphExecDestroy(g);
        for (unsigned j = 0; j < p->peers.size(); ++j)
            if (j != p->tp_rank && p->peers[j]) cudaIpcCloseMemHandle(p->peers[j]);
        for (void *a : p->allocations) cudaFree(a);
        if (p->err_host) cudaFreeHost(p->err_host);
    }
    delete p;
}

static void *plan_decline(const char *why)
{
    if (debug_enabled()) std::fprintf(stderr, "fyodor_b200: resident plan declined: %s; CPU reference selected\n", why);
    return nullptr;
}

__global__ void set_request_kernel(unsigned *req, unsigned token, unsigned position)
{
    req[0] = token; req[1] = position; req[2] = 0;
}
__global__ void advance_kernel(unsigned *req, const unsigned *argmax_token, unsigned *log)
{
    pdl_wait();
    const unsigned t = argmax_token[0];
    log[req[2]] = t;
    req[0] = t;
    req[1] += 1;
    req[2] += 1;
}

static int launch_advance(Plan *p, bool pdl)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1);
    cfg.stream = p->ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, advance_kernel, p->request, (const unsigned *)p->argmax_token, p->tokens_log) ==
           cudaSuccess ? 0 : -2;
}

// ---- launch descriptions of the fused kernels of one layer ----------------
static QgemvLaunch gemv_base(const Plan *p)
{
    QgemvLaunch L;
    L.counters = p->counters; L.counters_capacity = p->counters_capacity;
    L.partials = p->partials; L.partials_bytes = p->partials_bytes;
    L.error = p->err_dev;
    L.grid = p->ctx->sms;
    L.eps = p->eps;
    return L;
}

static QgemvLaunch qkv_launch(const Plan *p, unsigned l)
{
    QgemvLaunch L = gemv_base(p);
    L.epilogue = EPI_QKV;
    L.w = p->layers[l].qkv;
    L.nseg = 3;
    L.seg_rows[0] = p->H * p->hd; L.seg_rows[1] = p->Hkv * p->hd; L.seg_rows[2] = p->Hkv * p->hd;
    L.out[0] = p->q;
    L.kcache = p->kcache + (size_t)l * p->Hkv * p->capacity * p->hd;
    L.vcache = p->vcache + (size_t)l * p->Hkv * p->capacity * p->hd;
    L.norm_w = p->layers[l].attn_norm;
    L.rope_cos = p->rope_cos; L.rope_sin = p->rope_sin;
    L.request = p->request;
    L.head_dim = p->hd;
    L.capacity = (unsigned)p->capacity;
    return L;
}

static QgemvLaunch o_launch(const Plan *p, unsigned l)
{
    QgemvLaunch L = gemv_base(p);
    L.w = p->layers[l].o;
    L.seg_rows[0] = p->d;
    L.out[0] = p->delta;
    L.x = p->attn;
    return L;
}

static QgemvLaunch gateup_launch(const Plan *p, unsigned l)
{
    QgemvLaunch L = gemv_base(p);
    L.epilogue = EPI_SWIGLU;
    L.w = p->layers[l].gateup;
    L.nseg = 2;
    L.seg_rows[0] = p->ffn; L.seg_rows[1] = p->ffn;
    L.out[0] = p->h;
    L.norm_w = p->layers[l].ffn_norm;
    return L;
}

static QgemvLaunch down_launch(const Plan *p, unsigned l)
{
    QgemvLaunch L = gemv_base(p);
    L.w = p->layers[l].down;
    L.seg_rows[0] = p->d;
    L.out[0] = p->delta;
    L.x = p->h;
    return L;
}

static QgemvLaunch logits_launch(const Plan *p)
{
    QgemvLaunch L = gemv_base(p);
    L.epilogue = EPI_LOGITS;
    L.w = p->out_head;
    L.seg_rows[0] = p->vocab_rows;
    L.out[0] = p->logits;
    L.norm_w = p->out_norm;
    L.argmax_key = p->argmax_key; L.argmax_token = p->argmax_token; L.tiles_done = p->tiles_done;
    return L;
}

static AttentionLaunch attention_launch(const Plan *p, unsigned l)
{
    AttentionLaunch A;
    A.q = p->q;
    A.k = p->kcache + (size_t)l * p->Hkv * p->capacity * p->hd;
    A.v = p->vcache + (size_t)l * p->Hkv * p->capacity * p->hd;
    A.request = p->request;
    A.nseq = 1; A.heads = p->H; A.kv_heads = p->Hkv; A.head_dim = p->hd;
    A.capacity = (unsigned)p->capacity;
    A.scale = 1.0f / std::sqrt((float)p->hd);
    A.out = p->attn;
    A.splits = p->attn_splits;
    A.workspace = p->attn_ws; A.workspace_bytes = p->attn_ws_bytes;
    return A;
}

// Enqueue one decode step reading {token, position} from p->request.
// Residual stream: x[cur] holds the stream, `delta` the last branch output
// not yet added; the kernel that adds it writes the sum to x[cur ^ 1].
static DecodeLaunch persistent_launch(const Plan *p, StepMode mode)
{
    DecodeLaunch L;
    L.g.nl = p->nl; L.g.d = p->d; L.g.H = p->H; L.g.Hkv = p->Hkv; L.g.hd = p->hd; L.g.ffn = p->ffn;
    L.g.V = p->vocab_rows;
    L.g.capacity = (unsigned)p->capacity;
    L.layers = p->dec_layers;
    L.out_head = p->out_head; L.out_norm = p->out_norm;
    L.embd = (const unsigned char *)p->embd; L.embd_row_bytes = p->embd_row_bytes; L.embd_type = p->embd_type;
    L.eps = p->eps; L.attn_scale = 1.0f / std::sqrt((float)p->hd);
    L.rope_cos = p->rope_cos; L.rope_sin = p->rope_sin;
    L.request = p->request;
    L.ll = p->dec_ll;
    L.logits = p->logits;
    L.sync = p->dec_sync;
    L.attn_partials = p->dec_attn; L.attn_splits = p->dec_splits;
    L.argmax_key = p->argmax_key; L.argmax_token = p->argmax_token; L.tokens_log = p->tokens_log;
    L.error = p->err_dev;
    L.logits_mode = mode == STEP_NO_LOGITS ? 0 : mode == STEP_GREEDY ? 2 : 1;
    L.grid = p->dec_grid;
    L.ring_bytes = p->dec_ring_bytes;
    L.kcache = p->kcache; L.vcache = p->vcache;
    if (p->tp_size > 1) {  // partial sums and logits go through the ranks' exchange regions
        L.tp = p->tp_size; L.tp_rank = p->tp_rank; L.vocab0 = p->vocab0;
        L.peers = p->peers_dev; L.xl = p->xl;
        L.logits = nullptr;
        L.sync.abort_flag = reinterpret_cast<unsigned *>(p->xchg + p->xl.ctr) + 2 * p->nl + 1;
    }
    return L;
}

static int enqueue_persistent(Plan *p, StepMode mode)
{
    p->launches = 1;
    return launch_decode(persistent_launch(p, mode), p->ctx->stream);
}

static int enqueue_step(Plan *p, StepMode mode)
{
    if (p->dec_grid && !p->marks) return enqueue_persistent(p, mode);
    cudaStream_t s = p->ctx->stream;
    const bool pdl = true;
    p->launches = 0;
    int kc = KC_OTHER, proj = 0;  // proj: 1 QKV, 2 O, 3 gate/up, 4 down, 5 logits (matrix launches)
#define RUN(expr) do { int r_ = (expr); ++p->launches; if (r_) return r_; \
        if (p->marks) { cudaEvent_t ev; cudaEventCreate(&ev); cudaEventRecord(ev, s); \
                        p->marks->push_back({ev, kc | (kc == KC_MATRIX ? proj << 4 : 0)}); } } while (0)
    RUN(launch_gather(p->embd, p->embd_row_bytes, p->embd_type, p->d, p->request, 0, p->x[0], s, false));
    int cur = 0;
    bool pending = false;
    for (unsigned l = 0; l < p->nl; ++l) {
        kc = KC_MATRIX;
        QgemvLaunch L = qkv_launch(p, l);
        L.x = p->x[cur];
        if (pending) { L.delta = p->delta; L.x_out = p->x[cur ^ 1]; }
        L.pdl = pdl;
        proj = 1;
        RUN(launch_qgemv(L, s));
        if (pending) cur ^= 1;

        kc = KC_ATTENTION;
        AttentionLaunch A = attention_launch(p, l);
        A.pdl = pdl;
        RUN(launch_attention(A, s));

        kc = KC_MATRIX;
        QgemvLaunch O = o_launch(p, l);
        O.pdl = pdl;
        proj = 2;
        RUN(launch_qgemv(O, s));

        QgemvLaunch G = gateup_launch(p, l);
        G.x = p->x[cur]; G.delta = p->delta; G.x_out = p->x[cur ^ 1];
        G.pdl = pdl;
        proj = 3;
        RUN(launch_qgemv(G, s));
        cur ^= 1;

        QgemvLaunch D = down_launch(p, l);
        D.pdl = pdl;
        proj = 4;
        RUN(launch_qgemv(D, s));
        pending = true;
    }
    if (mode == STEP_NO_LOGITS) return 0;  // the KV cache is what the next step reads
    kc = KC_MATRIX;
    QgemvLaunch Lg = logits_launch(p);
    Lg.x = p->x[cur];
    Lg.delta = pending ? p->delta : nullptr;
    Lg.pdl = pdl;
    proj = 5;
    RUN(launch_qgemv(Lg, s));
    kc = KC_OTHER;
    if (mode == STEP_GREEDY) RUN(launch_advance(p, pdl));
#undef RUN
    return 0;
}

// A step under NYA_CUDA_PROFILE: the per-operation kernels with an event after
// each, their times added per kernel class and per projection.
static int run_step_profiled(Plan *p, StepMode mode)
{
    cudaStream_t s = p->ctx->stream;
    std::vector<std::pair<cudaEvent_t, int>> marks;
    p->marks = &marks;
    cudaEvent_t start;
    cudaEventCreate(&start);
    cudaEventRecord(start, s);
    int r = enqueue_step(p, mode);
    p->marks = nullptr;
    p->stats.kernel_launches += p->launches;
    if (cudaStreamSynchronize(s) != cudaSuccess) r = -2;
    cudaEvent_t prev = start;
    for (auto &m : marks) {
        float ms = 0.f;
        if (!r && cudaEventElapsedTime(&ms, prev, m.first) == cudaSuccess) {
            p->prof_ms[m.second & 15] += ms;
            const int proj = m.second >> 4;
            if (proj >= 1 && proj <= 5) { p->prof_proj_ms[proj - 1] += ms; ++p->prof_proj_calls[proj - 1]; }
        }
        prev = m.first;
    }
    for (auto &m : marks) cudaEventDestroy(m.first);
    cudaEventDestroy(start);
    ++p->prof_steps;
    return r;
}

static int run_step(Plan *p, StepMode mode)
{
    if (p->profile) return run_step_profiled(p, mode);
    cudaStream_t s = p->ctx->stream;
    if (!p->use_graphs || p->marks) {
        const int r = enqueue_step(p, mode);
        p->stats.kernel_launches += p->launches;
        return r;
    }
    if (!p->graphs[mode]) {
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return -2;
        const int r = enqueue_step(p, mode);
        cudaError_t e = cudaStreamEndCapture(s, &g);
        if (r || e != cudaSuccess) { if (g) cudaGraphDestroy(g); debug("graph capture", e); return -2; }
        e = cudaGraphInstantiateWithFlags(&p->graphs[mode], g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) { p->graphs[mode] = nullptr; debug("graph instantiate", e); return -2; }
        p->graph_kernels[mode] = p->launches;
        ++p->stats.graph_captures;
    }
    if (cudaGraphLaunch(p->graphs[mode], s) != cudaSuccess) return -2;
    ++p->stats.graph_replays;
    p->stats.kernel_launches += p->graph_kernels[mode];
    return 0;
}

static int set_request(Plan *p, unsigned token, unsigned position)
{
    set_request_kernel<<<1, 1, 0, p->ctx->stream>>>(p->request, token, position);
    ++p->stats.kernel_launches;
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// A K-quant matrix of the expected shape. The persistent decode kernel takes
// any multiple of 256 columns; the per-operation step's GEMV has its own
// limit (qgemv_supported), checked when a plan runs that step.
static bool supported_matrix(const nya_llm_tensor *t, size_t cols, size_t rows)
{
    return t && (t->type == T_Q4_K || t->type == T_Q6_K) && t->dimension_count == 2 && t->dimensions[0] == cols &&
           t->dimensions[1] == rows && cols % 256 == 0;
}

// Upload the raw GGUF bytes of up to three tensors and repack them, tile
// after tile, into one fused unit array.
// A rank's part of a weight matrix: rows [r0, r0 + nr) and column blocks
// [cb0, cb0 + ncb) (256-value K-quant blocks); null slice = all of it.
struct Slice {
    size_t r0, nr, cb0, ncb;
};

static int upload_fused(Plan *p, const nya_llm_tensor *const *t, int n, int mode, QWeights *out,
    const Slice *slices = nullptr)
{
    const unsigned type = t[0]->type;
    size_t block = 256, bb = 0;
    type_geometry(type, &block, &bb);
    const size_t full_cols = (size_t)t[0]->dimensions[0], full_row = full_cols / block * bb;
    Slice sl[3];
    for (int i = 0; i < n; ++i)
        sl[i] = slices ? slices[i] : Slice{0, (size_t)t[i]->dimensions[1], 0, full_cols / block};
    const size_t cols = sl[0].ncb * block, row_bytes = sl[0].ncb * bb;
    size_t tiles[3] = {0, 0, 0}, total = 0;
    if (mode == REPACK_GATEUP) { tiles[0] = (sl[0].nr + 7) / 8; total = tiles[0]; }
    else for (int i = 0; i < n; ++i) { tiles[i] = (sl[i].nr + 15) / 16; total += tiles[i]; }
    unsigned char *units = (unsigned char *)plan_alloc(p, qunits_bytes(type, total, cols));
    if (!units) return -1;
    void *raw[3] = {nullptr, nullptr, nullptr};
    int r = 0;
    for (int i = 0; i < n && !r; ++i) {
        const unsigned char *src = (const unsigned char *)t[i]->data + sl[i].r0 * full_row + sl[i].cb0 * bb;
        if (cudaMalloc(&raw[i], sl[i].nr * row_bytes) != cudaSuccess) { r = -1; break; }
        if (row_bytes == full_row) r = upload(raw[i], src, sl[i].nr * row_bytes, p->ctx->stream) ? 0 : -1;
        else r = cudaMemcpy2DAsync(raw[i], row_bytes, src, full_row, row_bytes, sl[i].nr, cudaMemcpyHostToDevice,
                                   p->ctx->stream) == cudaSuccess ? 0 : -1;
    }
    size_t at = 0;
    if (!r && mode == REPACK_GATEUP)
        r = repack_units(raw[0], raw[1], sl[0].nr, cols, type, mode, units, total, p->ctx->stream);
    for (int i = 0; !r && mode != REPACK_GATEUP && i < n; ++i) {
        r = repack_units(raw[i], nullptr, sl[i].nr, cols, type, mode, units + qunits_bytes(type, at, cols), tiles[i],
                         p->ctx->stream);
        at += tiles[i];
    }
    if (cudaStreamSynchronize(p->ctx->stream) != cudaSuccess) r = -1;  // raw buffers are read until here
    for (int i = 0; i < n; ++i) cudaFree(raw[i]);
    cudaGetLastError();
    if (r) return -1;
    out->units = units; out->type = type; out->cols = (unsigned)cols; out->tiles = (unsigned)total;
    return 0;
}

// Buffers of the persistent decode kernel. Returns false only on an
// allocation or copy failure; an unsupported geometry leaves dec_grid 0 and
// the plan runs the per-kernel step.
static bool setup_persistent(Plan *p)
{
    const char *env = std::getenv("NYA_CUDA_PERSISTENT");
    if (env && !std::strcmp(env, "0")) return true;
    size_t v;
    if (env_size("NYA_CUDA_RING_BYTES", &v)) p->dec_ring_bytes = (unsigned)std::min<size_t>(v, 1u << 20);
    DecodeGeometry g;
    g.nl = p->nl; g.d = p->d; g.H = p->H; g.Hkv = p->Hkv; g.hd = p->hd; g.ffn = p->ffn; g.V = p->vocab_rows;
    g.capacity = (unsigned)p->capacity;
    if (!decode_supported(g, p->out_head.type)) return true;
    const int grid = decode_grid(p->ctx->sms, g);
    if (grid <= 0) return true;
    cudaStream_t s = p->ctx->stream;
    bool ok = true;
    auto A = [&](size_t bytes) -> void * {
        void *x = ok ? plan_alloc(p, bytes) : nullptr;
        if (!x) ok = false;
        p->dec_bytes += bytes;
        return x;
    };
    const size_t words = 3;
    unsigned *w = (unsigned *)A(words * 4);
    std::vector<DecodeLayer> layers(p->nl);
    for (unsigned l = 0; l < p->nl; ++l) {
        DecodeLayer &L = layers[l];
        L.qkv = p->layers[l].qkv; L.o = p->layers[l].o; L.gateup = p->layers[l].gateup; L.down = p->layers[l].down;
        L.attn_norm = p->layers[l].attn_norm; L.ffn_norm = p->layers[l].ffn_norm;
    }
    p->dec_layers = (DecodeLayer *)A(layers.size() * sizeof(DecodeLayer));
    const size_t llw = decode_ll_words(g);
    unsigned long long *ll = (unsigned long long *)A(llw * 8);
    p->dec_splits = (unsigned)std::max(1, std::min(16, grid / (int)p->Hkv));  // decode_kernel.cuh ATT_MAX_PARTS
    p->dec_attn = (float *)A(decode_attn_partials_floats(g) * 4);
    if (!ok) return false;
    DecodeSync &y = p->dec_sync;
    y.exit_count = w++; y.abort_flag = w++; y.logit_tiles = w++;
    DecodeLL &b = p->dec_ll;
    b.xa = ll; ll += p->d;
    b.xm = ll; ll += p->d;
    b.q = ll; ll += (size_t)p->H * p->hd;
    b.kvnew = ll; ll += (size_t)2 * p->Hkv * p->hd;
    b.attn = ll; ll += (size_t)p->H * p->hd;
    b.h = ll;
    if (cudaMemsetAsync(y.exit_count, 0, words * 4, s) != cudaSuccess ||
        cudaMemsetAsync(p->dec_ll.xa, 0, llw * 8, s) != cudaSuccess ||
        cudaMemsetAsync(p->dec_attn, 0, decode_attn_partials_floats(g) * 4, s) != cudaSuccess ||
        !upload(p->dec_layers, layers.data(), layers.size() * sizeof(DecodeLayer), s) ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return false;
    p->dec_grid = grid;
    return true;
}

static void *plan_create(void *opaque, const nya_llm_context *m, size_t capacity)
{
    Context *c = (Context *)opaque;
    if (!c || c->failed || !m) return nullptr;
    if (m->is_assistant || m->expert_count || m->per_layer_embedding_length || m->is_gemma)
        return plan_decline("only dense LLaMA graphs are lowered");
    if (capacity == 0 || capacity > m->context_length || capacity > UINT32_MAX || m->block_count == 0)
        return nullptr;
    const unsigned d = m->embedding_length, nl = m->block_count, V = m->tokenizer.vocabulary_size;
    const nya_llm_layer &l0 = m->layers[0];
    const unsigned H = l0.head_count, Hkv = l0.kv_head_count, hd = l0.head_dimension, ffn = l0.hidden_length;
    if (!H || !Hkv || H % Hkv || (hd != 64 && hd != 128) || H / Hkv > 8 || H * hd != d || (Hkv * hd) % 16)
        return plan_decline("head geometry");
    for (unsigned i = 0; i < nl; ++i) {
        const nya_llm_layer &w = m->layers[i];
        if (w.head_count != H || w.kv_head_count != Hkv || w.head_dimension != hd || w.hidden_length != ffn ||
            w.sliding_window || w.kv_source != i || w.rope_factors || w.output_scale ||
            w.cache_offset != (size_t)i * Hkv * hd)
            return plan_decline("non-uniform or non-LLaMA layer");
        if (!supported_matrix(w.query, d, H * hd) || !supported_matrix(w.key, d, Hkv * hd) ||
            !supported_matrix(w.value, d, Hkv * hd) || !supported_matrix(w.attention_output, H * hd, d) ||
            !supported_matrix(w.feed_forward_gate, d, ffn) || !supported_matrix(w.feed_forward_up, d, ffn) ||
            !supported_matrix(w.feed_forward_down, ffn, d))
            return plan_decline("projection storage type (Q4_K/Q6_K required)");
        if (!w.attention_norm || w.attention_norm->type != T_F32 || !w.feed_forward_norm ||
            w.feed_forward_norm->type != T_F32)
            return plan_decline("norm storage type");
        if (w.query->type != w.key->type || w.key->type != w.value->type || w.feed_forward_gate->type != w.feed_forward_up->type)
            return plan_decline("mixed projection types in one fused group");
    }
    if (!supported_matrix(m->output, d, V) || !m->output_norm || m->output_norm->type != T_F32 ||
        !m->token_embedding || m->final_logit_softcap > 0.f)
        return plan_decline("output head");
    size_t eblock, ebytes;
    if (!type_geometry(m->token_embedding->type, &eblock, &ebytes) || d % eblock) return plan_decline("embedding type");

    // tensor parallelism: this process holds rank tp_rank of tp_size shards
    size_t tp = 1, tp_rank = 0;
    env_size("NYA_CUDA_TP_SIZE", &tp);
    env_size("NYA_CUDA_TP_RANK", &tp_rank);
    if (tp == 0 || tp > 8 || tp_rank >= tp) return plan_decline("NYA_CUDA_TP_SIZE / NYA_CUDA_TP_RANK");
    if (tp > 1 && (H % tp || Hkv % tp || (H * hd / tp) % 256 || (ffn / tp) % 256 || ffn % tp || V % tp))
        return plan_decline("model does not shard evenly over NYA_CUDA_TP_SIZE ranks");
    if (tp > 1 && d > 8192) return plan_decline("tensor parallelism supports d <= 8192");
    const unsigned Hs = H / (unsigned)tp, Hkvs = Hkv / (unsigned)tp, ffns = ffn / (unsigned)tp;
    const unsigned Vs = V / (unsigned)tp, r = (unsigned)tp_rank;

    // admission: weights + KV + scratch against the budget (resident.inc:155-168)
    size_t weights = 0;
    for (size_t i = 0; i < m->tensor_count; ++i) weights += m->tensors[i].data_size;
    if (m->output == m->token_embedding) weights += m->output->data_size;  // gather copy + units
    weights = weights / tp + (tp > 1 ? m->token_embedding->data_size : 0);  // shards + the replicated embedding
    const size_t kv_bytes = (size_t)nl * Hkvs * capacity * hd * sizeof(__half) * 2;
    const size_t act = ((size_t)d * 3 + (size_t)H * hd * 2 + ffn + V) * sizeof(float) + 2 * capacity * (hd / 2) * sizeof(float);
    if (weights + kv_bytes + act > c->cache_limit) return plan_decline("weights plus KV/scratch exceed the memory budget");

    Plan *p = new Plan();
    p->ctx = c; p->m = m; p->capacity = capacity;
    p->d = d; p->H = Hs; p->Hkv = Hkvs; p->hd = hd; p->ffn = ffns; p->V = V; p->nl = nl;
    p->tp_size = (unsigned)tp; p->tp_rank = r; p->vocab_rows = Vs; p->vocab0 = r * Vs;
    p->connected = tp == 1;
    p->eps = m->norm_epsilon;
    std::memset(&p->stats, 0, sizeof(p->stats));
    const char *graphs = std::getenv("NYA_CUDA_GRAPHS");
    p->use_graphs = !(graphs && !std::strcmp(graphs, "0"));
    size_t at;
    if (env_size("NYA_CUDA_FAIL_AFTER", &at)) p->fail_after = at;
    if (env_size("NYA_CUDA_FAIL_ALLOCATION_AFTER", &at)) p->fail_allocation_after = at;

    DeviceScope scope(c->device);
    bool ok = scope.ok;
    auto A = [&](size_t bytes) -> void * { void *x = ok ? plan_alloc(p, bytes) : nullptr; if (!x) ok = false; return x; };
    // KV and scratch before weights, so a plan is admitted as a whole
    p->kcache = (__half *)A(kv_bytes / 2);
    p->vcache = (__half *)A(kv_bytes / 2);
    p->x[0] = (float *)A(d * 4); p->x[1] = (float *)A(d * 4); p->delta = (float *)A(d * 4);
    p->q = (float *)A((size_t)H * hd * 4); p->attn = (float *)A((size_t)H * hd * 4);
    p->h = (float *)A((size_t)ffn * 4); p->logits = (float *)A((size_t)V * 4);
    p->rope_cos = (float *)A(capacity * (hd / 2) * 4); p->rope_sin = (float *)A(capacity * (hd / 2) * 4);
    p->request = (unsigned *)A(64);
    p->argmax_key = (unsigned long long *)A(64);
    p->argmax_token = (unsigned *)A(64);
    p->tiles_done = (unsigned *)A(64);
    p->tokens_log = (unsigned *)A(capacity * 4 + 64);
    if (ok && cudaHostAlloc((void **)&p->err_host, 64, cudaHostAllocMapped) != cudaSuccess) { cudaGetLastError(); ok = false; }
    if (ok) { std::memset(p->err_host, 0, 64); ok = cudaHostGetDevicePointer((void **)&p->err_dev, p->err_host, 0) == cudaSuccess; }
    if (ok) ok = cudaMemsetAsync(p->argmax_key, 0, 64, c->stream) == cudaSuccess &&
                 cudaMemsetAsync(p->tiles_done, 0, 64, c->stream) == cudaSuccess &&
                 cudaMemsetAsync(p->request, 0, 64, c->stream) == cudaSuccess;

    // weights, repacked into fused tensor-core matrices
    p->layers.resize(nl);
    for (unsigned i = 0; ok && i < nl; ++i) {
        const nya_llm_layer &w = m->layers[i];
        LayerW &L = p->layers[i];
        const nya_llm_tensor *qkv[3] = {w.query, w.key, w.value};
        const nya_llm_tensor *o[1] = {w.attention_output};
        const nya_llm_tensor *gu[2] = {w.feed_forward_gate, w.feed_forward_up};
        const nya_llm_tensor *dn[1] = {w.feed_forward_down};
        // this rank's heads (rows of q/k/v, columns of O) and FFN rows (gate/up
        // rows, down columns); the whole matrices when tp == 1
        const Slice s_qkv[3] = {{(size_t)r * Hs * hd, (size_t)Hs * hd, 0, d / 256},
                                {(size_t)r * Hkvs * hd, (size_t)Hkvs * hd, 0, d / 256},
                                {(size_t)r * Hkvs * hd, (size_t)Hkvs * hd, 0, d / 256}};
        const Slice s_o[1] = {{0, d, (size_t)r * Hs * hd / 256, (size_t)Hs * hd / 256}};
        const Slice s_gu[2] = {{(size_t)r * ffns, ffns, 0, d / 256}, {(size_t)r * ffns, ffns, 0, d / 256}};
        const Slice s_dn[1] = {{0, d, (size_t)r * ffns / 256, ffns / 256}};
        ok = upload_fused(p, qkv, 3, REPACK_QKV, &L.qkv, s_qkv) == 0 && upload_fused(p, o, 1, REPACK_PLAIN, &L.o, s_o) == 0 &&
             upload_fused(p, gu, 2, REPACK_GATEUP, &L.gateup, s_gu) == 0 &&
             upload_fused(p, dn, 1, REPACK_PLAIN, &L.down, s_dn) == 0;
        if (!ok) break;
        float *an = (float *)A(d * 4), *fn = (float *)A(d * 4);
        ok = ok && upload(an, w.attention_norm->data, d * 4, c->stream) && upload(fn, w.feed_forward_norm->data, d * 4, c->stream);
        L.attn_norm = an; L.ffn_norm = fn;
    }
    if (ok) {
        const nya_llm_tensor *out[1] = {m->output};
        const Slice s_out[1] = {{(size_t)p->vocab0, Vs, 0, d / 256}};  // this rank's vocabulary rows
        ok = upload_fused(p, out, 1, REPACK_PLAIN, &p->out_head, s_out) == 0;
    }
    if (ok) {
        void *e = A(m->token_embedding->data_size);
        ok = ok && upload(e, m->token_embedding->data, m->token_embedding->data_size, c->stream);
        p->embd = e;
        p->embd_type = m->token_embedding->type;
        p->embd_row_bytes = d / eblock * ebytes;
        float *on = (float *)A(d * 4);
        ok = ok && upload(on, m->output_norm->data, d * 4, c->stream);
        p->out_norm = on;
    }
    // RoPE tables with the engine's own host formula (llm_cpu.c:216-229, :428-432)
    if (ok) {
        const unsigned pairs = hd / 2;
        std::vector<float> freq(pairs), co(capacity * pairs), si(capacity * pairs);
        for (unsigned j = 0; j < pairs; ++j) freq[j] = powf(m->rope_frequency_base, -(float)j / (float)pairs) / 1.0f;
        for (size_t t = 0; t < capacity; ++t)
            for (unsigned j = 0; j < pairs; ++j) {
                const float angle = (float)t * freq[j];
                co[t * pairs + j] = cosf(angle);
                si[t * pairs + j] = sinf(angle);
            }
        ok = upload(p->rope_cos, co.data(), co.size() * 4, c->stream) && upload(p->rope_sin, si.data(), si.size() * 4, c->stream) &&
             cudaStreamSynchronize(c->stream) == cudaSuccess;
    }
    // stream-K scratch for the largest GEMV of the step; attention partials
    if (ok) {
        const QgemvLaunch all[5] = {qkv_launch(p, 0), o_launch(p, 0), gateup_launch(p, 0), down_launch(p, 0), logits_launch(p)};
        size_t tiles = 0, partial = 0;
        for (const auto &L : all) {
            tiles = std::max<size_t>(tiles, qgemv_tiles(L));
            partial = std::max(partial, qgemv_partials_bytes(L, c->sms));
        }
        p->counters_capacity = tiles;
        p->counters = (unsigned *)A(tiles * 4);
        p->partials_bytes = partial;
        p->partials = (float *)A(partial);
        // one partition per ~128 positions of the context, at most 32
        p->attn_splits = (unsigned)std::min<size_t>(32, std::max<size_t>(1, (capacity + 127) / 128));
        AttentionLaunch al; al.nseq = 1; al.heads = H; al.kv_heads = Hkv; al.head_dim = hd; al.splits = p->attn_splits;
        p->attn_ws_bytes = attention_workspace_bytes(al);
        p->attn_ws = A(p->attn_ws_bytes);
        if (ok) ok = cudaMemsetAsync(p->counters, 0, tiles * 4, c->stream) == cudaSuccess &&
                     cudaMemsetAsync(p->attn_ws, 0, p->attn_ws_bytes, c->stream) == cudaSuccess;
    }
    if (ok) ok = setup_persistent(p);
    bool per_op = true;  // the per-operation step: every projection within the GEMV's limits
    {
        const size_t ks[3] = {d, (size_t)H * hd, ffn};
        for (size_t k : ks)
            if (!qgemv_supported(m->layers[0].query->type, k, 1) || !qgemv_supported(m->output->type, d, 1) ||
                !qgemv_supported(m->layers[0].feed_forward_down->type, k, 1))
                per_op = false;
    }
    if (ok && !p->dec_grid && !per_op) {
        plan_free(p);
        return plan_decline("geometry beyond the per-operation step's GEMV");
    }
    // NYA_CUDA_PROFILE=1 (resident.inc:176-183): every step runs the
    // per-operation kernels without graphs, timed per class and projection
    if (const char *prof = std::getenv("NYA_CUDA_PROFILE"))
        p->profile = !std::strcmp(prof, "1") && per_op && p->tp_size == 1;
    if (ok && p->tp_size > 1) {
        if (!p->dec_grid) {  // only the persistent kernel exchanges partial sums
            debug("tensor parallelism needs the persistent decode kernel", cudaSuccess);
            plan_free(p);
            return plan_decline("tensor parallelism needs the persistent decode kernel");
        }
        p->xl = xchg_layout(p->tp_size, d, V, nl);
        p->xchg_bytes = p->xl.bytes;
        p->xchg = (unsigned char *)A(p->xchg_bytes);
        p->peers_dev = (unsigned char **)A(p->tp_size * sizeof(void *));
        if (ok) ok = cudaMemsetAsync(p->xchg, 0, p->xchg_bytes, c->stream) == cudaSuccess;
    }
    if (ok) ok = cudaStreamSynchronize(c->stream) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
    if (!ok) {
        debug("resident plan setup failed; rolling back", cudaGetLastError());
        plan_free(p);
        return nullptr;
    }
    p->stats.weights_bytes = weights;
    p->stats.kv_bytes = kv_bytes;
    p->stats.scratch_bytes = act + p->counters_capacity * 4 + p->partials_bytes + p->attn_ws_bytes + p->dec_bytes;
    p->stats.prefill_batch = 1;
    return p;
}

static int plan_fail(Plan *p, size_t position)
{
    std::fprintf(stderr, "fyodor_b200: resident execution failed at token position %zu; CPU prefix replay required\n", position);
    cudaStreamSynchronize(p->ctx->stream);
    cudaGetLastError();
    p->failed = true;
    return -1;
}

static int finish_logits(Plan *p, float *out)
{
    cudaStream_t s = p->ctx->stream;
    ++p->stats.downloads;
    const void *src = p->tp_size > 1 ? (const void *)(p->xchg + p->xl.logits) : (const void *)p->logits;
    if (cudaMemcpyAsync(out, src, (size_t)p->V * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess) return -2;
    ++p->stats.synchronizations;
    if (cudaStreamSynchronize(s) != cudaSuccess) return -2;
    if (*(volatile unsigned *)p->err_host) return -2;
    for (size_t i = 0; i < p->V; ++i) if (!std::isfinite(out[i])) return -2;
    const nya_llm_tokenizer &tk = p->m->tokenizer;
    for (size_t i = 0; i < tk.suppressed_count; ++i) out[tk.suppressed_tokens[i]] = -INFINITY;
    return 0;
}

static int plan_token(void *opaque, uint32_t token, size_t position, int logits, float *out)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->failed || !p->connected || position >= p->capacity || (position != 0 && position > p->valid) ||
        (logits && !out) || token >= p->V)
        return -1;
    if (position >= p->fail_after) { p->failed = true; return -1; }
    DeviceScope scope(p->ctx->device);
    if (!scope.ok || set_request(p, token, (unsigned)position) || run_step(p, logits ? STEP_LOGITS : STEP_NO_LOGITS))
        return plan_fail(p, position);
    if (logits && finish_logits(p, out)) return plan_fail(p, position);
    p->valid = position + 1;
    return 0;
}

// Prefill in chunks of up to BATCH_MAX prompt tokens: every weight read
// once per chunk, causal attention inside the chunk. 1 when the plan has no
// chunker (tensor-parallel shards, NYA_CUDA_CHUNKED_PREFILL=0, a geometry the
// batched step does not take): the caller steps token by token.
static ::Batch *plan_chunker(Plan *p)
{
    if (!p->prefill && !p->prefill_tried) {
        p->prefill_tried = true;
        const char *env = std::getenv("NYA_CUDA_CHUNKED_PREFILL");
        if (!(env && !std::strcmp(env, "0")) && p->tp_size == 1) p->prefill = ::batch_create(p, BATCH_MAX, true);
        if (p->prefill) p->stats.prefill_batch = BATCH_MAX;
    }
    return p->prefill;
}

static int prefill_chunked(Plan *p, const uint32_t *tokens, size_t count, size_t position, float *out)
{
    ::Batch *bt = plan_chunker(p);
    if (!bt) return 1;
    return ::prefill_chunks(p, bt, tokens, count, position, out);
}

static int plan_prefill(void *opaque, const uint32_t *tokens, size_t count, size_t position, float *out)
{
    Plan *p = (Plan *)opaque;
    if (!p || !tokens || count == 0 || position > p->capacity || count > p->capacity - position) return -1;
    if (p->failed || !p->connected || (position != 0 && position > p->valid) || !out) return -1;
    for (size_t i = 0; i < count; ++i) if (tokens[i] >= p->V) return -1;
    if (position + count > p->fail_after) { p->failed = true; return -1; }
    DeviceScope scope(p->ctx->device);
    if (!scope.ok) return plan_fail(p, position);
    if (count > 1) {  // prompt chunks through the batched step (resident.inc:585-595 chunks prefill too)
        const int r = prefill_chunked(p, tokens, count, position, out);
        if (r == 0) {
            p->valid = position + count;
            return 0;
        }
        if (r != 1) return plan_fail(p, position);
    }  // r == 1: no chunker for this plan; one decode step per token
    for (size_t i = 0; i < count; ++i) {
        const bool last = i + 1 == count;
        if (set_request(p, tokens[i], (unsigned)(position + i)) || run_step(p, last ? STEP_LOGITS : STEP_NO_LOGITS))
            return plan_fail(p, position + i);
    }
    if (finish_logits(p, out)) return plan_fail(p, position + count - 1);
    p->valid = position + count;
    return 0;
}

static void plan_stats(const void *opaque, nya_compute_stats *stats)
{
    const Plan *p = (const Plan *)opaque;
    if (p && stats) *stats = p->stats;
}

static int plan_read_kv(void *opaque, size_t layer, size_t position, size_t count, float *keys, float *values,
    size_t elements)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->failed || p->tp_size > 1 || !keys || !values || !count || layer >= p->nl || position > p->valid ||
        count > p->valid - position)
        return -1;  // a tensor-parallel rank holds only its own KV heads
    const size_t width = (size_t)p->hd * p->Hkv;
    if (count > SIZE_MAX / width || elements != count * width) return -1;
    DeviceScope scope(p->ctx->device);
    ++p->stats.synchronizations;
    if (cudaStreamSynchronize(p->ctx->stream) != cudaSuccess) return -1;
    p->kv_stage.resize(count * p->hd);
    for (int which = 0; which < 2; ++which) {
        const __half *base = (which ? p->vcache : p->kcache) + (size_t)layer * p->Hkv * p->capacity * p->hd;
        float *dst = which ? values : keys;
        for (unsigned h = 0; h < p->Hkv; ++h) {
            if (cudaMemcpy(p->kv_stage.data(), base + ((size_t)h * p->capacity + position) * p->hd,
                           count * p->hd * 2, cudaMemcpyDeviceToHost) != cudaSuccess)
                return -1;
            for (size_t t = 0; t < count; ++t)
                for (unsigned e = 0; e < p->hd; ++e) {
                    __half_raw r; r.x = p->kv_stage[t * p->hd + e];
                    dst[t * width + (size_t)h * p->hd + e] = __half2float(__half(r));
                }
        }
        ++p->stats.downloads;
    }
    return 0;
}

// ======================================================================
// vtable
// ======================================================================
static void *backend_create() { return context_create(); }
static void backend_destroy(void *c) { context_free((Context *)c); }
static int backend_active(const void *c) { return c && !((const Context *)c)->failed; }
static int backend_matvec(void *c, const void *w, size_t r, size_t k, unsigned t, const float *x, float *y)
{
    return context_matmul((Context *)c, w, r, k, t, x, y, 1);
}
static int backend_matmul(void *c, const void *w, size_t r, size_t k, unsigned t, const float *x, float *y, size_t b)
{
    return context_matmul((Context *)c, w, r, k, t, x, y, b);
}

}  // namespace fyb

using namespace fyb;

extern "C" const nya_backend_interface *nya_cuda_backend(void)
{
    static const nya_backend_interface api = {
        NYA_BACKEND_CUDA, "cuda",
        NYA_COMPUTE_MATVEC | NYA_COMPUTE_QUANTIZED | NYA_COMPUTE_RESIDENT | NYA_COMPUTE_MATMUL,
        backend_create, backend_destroy, backend_active, backend_matvec,
        fyb::plan_create, fyb::plan_free, fyb::plan_token, fyb::plan_prefill, fyb::plan_stats,
        backend_matmul, nullptr, fyb::plan_read_kv, nullptr};
    return &api;
}

// ======================================================================
// Batched decode: B sequences (1..16) of one resident plan's model, each at
// its own position with its own KV cache, decoded together. Every
// projection is one small-batch GEMM over the plan's repacked weights
// (GEMV for one or two sequences, the mma.sync GEMM for 3..8, tcgen05 for
// 9..16: each weight unit read once per step for all sequences); attention
// is the ragged-batch kernel over the sequences' caches; norms, RoPE + KV
// append, SwiGLU and the greedy argmax are the kernels of batch.cu. A step is
// captured in a CUDA graph after its first (eager) run has sized the GEMM
// scratch; tokens, positions and attended lengths live on the device, so the
// graph serves every step.
// ======================================================================
struct Batch {
    Plan *p = nullptr;
    unsigned B = 0;
    unsigned rows = 0;    // rows of the step being enqueued (B for a batch of sequences)
    unsigned ws_rows = 0; // query rows the attention workspace's counters were last laid out for
    bool chunk = false;   // rows are consecutive positions of one sequence in the plan's own cache
    bool all_logits = false;  // chunk: logits of every row (verification), not only the last
    size_t capacity = 0;
    std::vector<void *> allocations;
    __half *kc = nullptr, *vc = nullptr;  // [layer][seq][kv head][capacity][hd] (chunk: the plan's cache)
    float *x = nullptr, *xn = nullptr, *delta = nullptr, *y = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr;
    float *logits = nullptr;             // [B][V]
    unsigned *req = nullptr;             // [B] tokens | [B] positions | [B] lengths | step
    unsigned *tokens = nullptr;          // [B] argmax of the last step
    unsigned *log = nullptr;             // [steps][B] greedy tokens
    size_t log_bytes = 0;
    void *attn_ws = nullptr;
    size_t attn_ws_bytes = 0;
    unsigned splits = 1;
    unsigned *counters = nullptr;
    size_t counters_bytes = 0;
    float *partials = nullptr;
    size_t partials_bytes = 0;
    void *gemm = nullptr;
    size_t gemm_bytes = 0;
    cudaGraphExec_t graphs[2] = {nullptr, nullptr};  // logits step, greedy step
    bool sized[2] = {false, false};
    unsigned long long launches = 0;
};

static void batch_free(Batch *bt)
{
    if (!bt) return;
    DeviceScope scope(bt->p->ctx->device);
    cudaStreamSynchronize(bt->p->ctx->stream);
    for (auto &g : bt->graphs) if (g) cudaGraphExecDestroy(g);
    for (void *a : bt->allocations) cudaFree(a);  // the attention workspace among them
    for (void *a : {(void *)bt->log, (void *)bt->counters, (void *)bt->partials, (void *)bt->gemm})  // grown buffers
        if (a) cudaFree(a);
    cudaGetLastError();
    delete bt;
}

static AttentionLaunch batch_attention(const Batch *bt, unsigned l)
{
    const Plan *p = bt->p;
    const size_t per_seq = (size_t)p->Hkv * bt->capacity * p->hd;
    const unsigned slots = bt->chunk ? 1u : bt->B;
    AttentionLaunch A;
    A.q = bt->q;
    A.k = bt->kc + (size_t)l * slots * per_seq;
    A.v = bt->vc + (size_t)l * slots * per_seq;
    A.seq_stride = per_seq;
    if (bt->chunk) {  // one sequence, the chunk's rows as causal queries; length of the last row
        A.nseq = 1; A.queries = std::max(1u, bt->rows);
        A.lengths = bt->req + 2 * bt->B + A.queries - 1;
    } else {
        A.nseq = bt->B;
        A.lengths = bt->req + 2 * bt->B;
    }
    A.heads = p->H; A.kv_heads = p->Hkv; A.head_dim = p->hd;
    A.capacity = (unsigned)bt->capacity;
    A.scale = 1.0f / std::sqrt((float)p->hd);
    A.out = bt->attn;
    A.splits = bt->splits;
    A.workspace = bt->attn_ws; A.workspace_bytes = bt->attn_ws_bytes;
    return A;
}

// One batched step reading tokens and positions from bt->req; greedy steps
// advance every sequence to its argmax token at the next position.
static int batch_enqueue(Batch *bt, bool greedy, bool logits = true)
{
    Plan *p = bt->p;
    cudaStream_t s = p->ctx->stream;
    const int sms = p->ctx->sms;
    const unsigned B = bt->B, R = bt->chunk ? bt->rows : B, slots = bt->chunk ? 1u : B;
    const Scratch sc{&bt->counters, &bt->counters_bytes, &bt->partials, &bt->partials_bytes, &bt->gemm,
                     &bt->gemm_bytes};
    const size_t per_seq = (size_t)p->Hkv * bt->capacity * p->hd;
    bt->launches = 0;
#define BRUN(expr) do { const int r_ = (expr); ++bt->launches; if (r_) return r_; } while (0)
    BRUN(launch_gather_batch(p->embd, p->embd_row_bytes, p->embd_type, p->d, bt->req, R, bt->x, s));
    for (unsigned l = 0; l < p->nl; ++l) {
        const LayerW &L = p->layers[l];
        const size_t qkv_rows = (size_t)L.qkv.tiles * 16, gu_rows = (size_t)L.gateup.tiles * 16;
        BRUN(launch_bt_add_norm(bt->x, l ? bt->delta : nullptr, L.attn_norm, bt->xn, p->d, p->eps, R, s));
        BRUN(device_matmul(&L.qkv, nullptr, 0, qkv_rows, p->d, L.qkv.type, bt->xn, bt->y, R, sc, s, sms));
        BRUN(launch_bt_rope_kv(bt->y, (unsigned)qkv_rows, p->H, p->Hkv, p->hd, bt->req + B, p->rope_cos, p->rope_sin,
                               bt->q, bt->kc + (size_t)l * slots * per_seq, bt->vc + (size_t)l * slots * per_seq,
                               (unsigned)bt->capacity, R, bt->chunk ? R : 1u, s));
        BRUN(launch_attention(batch_attention(bt, l), s));
        BRUN(device_matmul(&L.o, nullptr, 0, p->d, (size_t)p->H * p->hd, L.o.type, bt->attn, bt->delta, R, sc, s, sms));
        BRUN(launch_bt_add_norm(bt->x, bt->delta, L.ffn_norm, bt->xn, p->d, p->eps, R, s));
        BRUN(device_matmul(&L.gateup, nullptr, 0, gu_rows, p->d, L.gateup.type, bt->xn, bt->y, R, sc, s, sms));
        BRUN(launch_bt_swiglu(bt->y, p->ffn, bt->h, R, s));
        BRUN(device_matmul(&L.down, nullptr, 0, p->d, p->ffn, L.down.type, bt->h, bt->delta, R, sc, s, sms));
    }
    if (!logits) return 0;  // a prompt chunk before the last: only the KV cache matters
    BRUN(launch_bt_add_norm(bt->x, bt->delta, p->out_norm, bt->xn, p->d, p->eps, R, s));
    if (bt->chunk) {  // the logits of the chunk's last token, or of every row when verifying a draft
        const unsigned n = bt->all_logits ? R : 1u;
        BRUN(device_matmul(&p->out_head, nullptr, 0, p->V, p->d, p->out_head.type, bt->xn + (size_t)(R - n) * p->d,
                           bt->logits, n, sc, s, sms));
        return 0;
    }
    BRUN(device_matmul(&p->out_head, nullptr, 0, p->V, p->d, p->out_head.type, bt->xn, bt->logits, B, sc, s, sms));
    BRUN(launch_bt_argmax(bt->logits, p->V, bt->req, B, bt->tokens, bt->log, greedy, p->err_dev, s));
#undef BRUN
    return 0;
}

// The first step of a mode runs eagerly (the GEMM scratch grows to its
// size); later steps replay one captured graph.
static int batch_run(Batch *bt, bool greedy)
{
    cudaStream_t s = bt->p->ctx->stream;
    const int m = greedy ? 1 : 0;
    if (!bt->sized[m]) {
        const int r = batch_enqueue(bt, greedy);
        if (r) return r;
        if (cudaStreamSynchronize(s) != cudaSuccess) return -2;
        bt->sized[m] = true;
        return 0;
    }
    if (!bt->graphs[m]) {
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return -2;
        const int r = batch_enqueue(bt, greedy);
        cudaError_t e = cudaStreamEndCapture(s, &g);
        if (r || e != cudaSuccess) { if (g) cudaGraphDestroy(g); cudaGetLastError(); return -2; }
        e = cudaGraphInstantiateWithFlags(&bt->graphs[m], g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) { bt->graphs[m] = nullptr; cudaGetLastError(); return -2; }
    }
    return cudaGraphLaunch(bt->graphs[m], s) == cudaSuccess ? 0 : -2;
}

static int batch_set(Batch *bt, const uint32_t *tokens, const uint32_t *positions, size_t steps)
{
    BatchRequest r = {};
    for (unsigned b = 0; b < bt->B; ++b) {
        if (tokens[b] >= bt->p->V || (size_t)positions[b] + steps > bt->capacity) return -1;
        r.token[b] = tokens[b];
        r.position[b] = positions[b];
    }
    return launch_bt_set(r, bt->req, bt->B, bt->p->ctx->stream);
}

// A batch of `batch` sequences with their own caches, or (chunk) a prompt
// chunker of up to `batch` consecutive positions of the plan's own sequence.
static Batch *batch_create(Plan *p, unsigned batch, bool chunk)
{
    if (!p || p->failed || batch < 1 || batch > BATCH_MAX || p->tp_size != 1 || p->hd % 16 || p->ffn % 8 ||
        p->d % 4)
        return nullptr;
    DeviceScope scope(p->ctx->device);
    if (!scope.ok) return nullptr;
    Batch *bt = new Batch;
    bt->p = p;
    bt->B = batch;
    bt->rows = batch;
    bt->chunk = chunk;
    bt->capacity = p->capacity;
    const size_t kv = chunk ? 0 : (size_t)p->nl * batch * p->Hkv * bt->capacity * p->hd;
    const size_t qkv_rows = (size_t)p->layers[0].qkv.tiles * 16;
    const size_t ywidth = std::max<size_t>(qkv_rows, (size_t)p->layers[0].gateup.tiles * 16);
    bool ok = true;
    auto A = [&](size_t bytes) -> void * {
        void *d = nullptr;
        if (!ok || cudaMalloc(&d, bytes ? bytes : 256) != cudaSuccess) { cudaGetLastError(); ok = false; return nullptr; }
        bt->allocations.push_back(d);
        return d;
    };
    if (chunk) {
        bt->kc = p->kcache; bt->vc = p->vcache;
    } else {
        bt->kc = (__half *)A(kv * 2); bt->vc = (__half *)A(kv * 2);
    }
    bt->x = (float *)A((size_t)batch * p->d * 4); bt->xn = (float *)A((size_t)batch * p->d * 4);
    bt->delta = (float *)A((size_t)batch * p->d * 4);
    bt->y = (float *)A((size_t)batch * ywidth * 4);
    bt->q = (float *)A((size_t)batch * p->H * p->hd * 4); bt->attn = (float *)A((size_t)batch * p->H * p->hd * 4);
    bt->h = (float *)A((size_t)batch * p->ffn * 4);
    bt->logits = (float *)A((size_t)batch * p->V * 4);
    bt->req = (unsigned *)A((3 * BATCH_MAX + 1) * 4); bt->tokens = (unsigned *)A(BATCH_MAX * 4);
    // partitions of each (sequence, KV head): about four waves of the SMs, 4..16
    const size_t seqs = chunk ? 1 : batch;
    bt->splits = (unsigned)std::max<size_t>(4, std::min<size_t>(16, ((size_t)4 * p->ctx->sms + seqs * p->Hkv - 1) /
                                                                        (seqs * p->Hkv)));
    if (ok) {
        AttentionLaunch L = batch_attention(bt, 0);
        bt->attn_ws_bytes = attention_workspace_bytes(L);
        bt->attn_ws = A(bt->attn_ws_bytes);
    }
    if (ok) ok = (chunk || (cudaMemset(bt->kc, 0, kv * 2) == cudaSuccess && cudaMemset(bt->vc, 0, kv * 2) == cudaSuccess)) &&
                 cudaMemset(bt->attn_ws, 0, bt->attn_ws_bytes) == cudaSuccess &&
                 cudaMemset(bt->req, 0, (3 * BATCH_MAX + 1) * 4) == cudaSuccess &&
                 grow((void **)&bt->log, &bt->log_bytes, (size_t)BATCH_MAX * 4, true) == 0 &&
                 cudaDeviceSynchronize() == cudaSuccess;
    if (!ok) {
        batch_free(bt);
        return nullptr;
    }
    return bt;
}

extern "C" void *fyb_batch_create(void *plan, unsigned batch) { return batch_create((Plan *)plan, batch, false); }

// Prompt chunks into the plan's cache; out receives the logits of the last
// token, or with bt->all_logits (one chunk, a draft to verify) [count][V].
static int prefill_chunks(Plan *p, Batch *bt, const uint32_t *tokens, size_t count, size_t position, float *out)
{
    cudaStream_t s = p->ctx->stream;
    if (bt->all_logits && count > bt->B) return -1;
    cudaEvent_t t0 = nullptr, t1 = nullptr;  // NYA_CUDA_PROFILE: the chunks' time as one class
    if (p->profile && cudaEventCreate(&t0) == cudaSuccess && cudaEventCreate(&t1) == cudaSuccess)
        cudaEventRecord(t0, s);
    for (size_t c0 = 0; c0 < count; c0 += bt->B) {
        const unsigned R = (unsigned)std::min<size_t>(bt->B, count - c0);
        BatchRequest r = {};
        for (unsigned i = 0; i < R; ++i) {
            r.token[i] = tokens[c0 + i];
            r.position[i] = (unsigned)(position + c0 + i);
        }
        bt->rows = R;
        // the attention workspace keeps its counters after the partials, at an
        // offset set by the query rows: a chunk of another size starts from zero
        if (R != bt->ws_rows && cudaMemsetAsync(bt->attn_ws, 0, bt->attn_ws_bytes, s) != cudaSuccess) return -2;
        bt->ws_rows = R;
        if (launch_bt_set(r, bt->req, bt->B, s)) return -2;
        const int e = batch_enqueue(bt, false, c0 + R == count);
        p->stats.kernel_launches += bt->launches + 1;
        if (e) return -2;
    }
    ++p->stats.downloads;
    ++p->stats.synchronizations;
    const size_t rows = bt->all_logits ? count : 1;
    if (t1) cudaEventRecord(t1, s);
    if (cudaMemcpyAsync(out, bt->logits, rows * p->V * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess || *(volatile unsigned *)p->err_host)
        return -2;
    if (t1) {
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, t0, t1) == cudaSuccess) p->prof_ms[3] += ms;
        cudaEventDestroy(t0);
        cudaEventDestroy(t1);
    }
    for (size_t i = 0; i < rows * p->V; ++i) if (!std::isfinite(out[i])) return -2;
    const nya_llm_tokenizer &tk = p->m->tokenizer;
    for (size_t r = 0; r < rows; ++r)
        for (size_t i = 0; i < tk.suppressed_count; ++i) out[r * p->V + tk.suppressed_tokens[i]] = -INFINITY;
    return 0;
}

// Speculative verification: the count (1..16) draft tokens at positions
// [position, position + count) of the plan's sequence in one chunk, every
// row's logits to out [count][V] (suppressed ids -inf), the draft's K/V rows
// written to the cache (the caller continues from the accepted prefix and
// rewrites the rest, as the engine's session does).
extern "C" int fyb_plan_verify(void *opaque, const uint32_t *tokens, size_t count, size_t position, float *out)
{
    Plan *p = (Plan *)opaque;
    if (!p || !tokens || !out || count == 0 || count > BATCH_MAX || p->failed || !p->connected ||
        position > p->capacity || count > p->capacity - position || (position != 0 && position > p->valid))
        return -1;
    for (size_t i = 0; i < count; ++i) if (tokens[i] >= p->V) return -1;
    DeviceScope scope(p->ctx->device);
    if (!scope.ok) return -1;
    Batch *bt = plan_chunker(p);
    if (!bt) return -1;  // no chunker for this plan (tensor-parallel shard, or chunking switched off)
    bt->all_logits = true;
    const int r = prefill_chunks(p, bt, tokens, count, position, out);
    bt->all_logits = false;
    if (r) return plan_fail(p, position);
    p->valid = position + count;
    return 0;
}

extern "C" void fyb_batch_free(void *batch) { batch_free((Batch *)batch); }

extern "C" int fyb_batch_step(void *batch, const uint32_t *tokens, const uint32_t *positions, float *logits,
    uint32_t *argmax)
{
    Batch *bt = (Batch *)batch;
    if (!bt || !tokens || !positions || bt->p->failed) return -1;
    DeviceScope scope(bt->p->ctx->device);
    if (!scope.ok) return -1;
    cudaStream_t s = bt->p->ctx->stream;
    int r = batch_set(bt, tokens, positions, 1);
    if (r) return r;
    if ((r = batch_run(bt, false)) != 0) return r;
    if (logits && cudaMemcpyAsync(logits, bt->logits, (size_t)bt->B * bt->p->V * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return -2;
    if (argmax && cudaMemcpyAsync(argmax, bt->tokens, (size_t)bt->B * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return -2;
    if (cudaStreamSynchronize(s) != cudaSuccess || *(volatile unsigned *)bt->p->err_host) return -2;
    return 0;
}

// `steps` greedy steps from tokens / positions on the device; out[step][b].
extern "C" int fyb_batch_decode_greedy(void *batch, const uint32_t *tokens, const uint32_t *positions, size_t steps,
    uint32_t *out)
{
    Batch *bt = (Batch *)batch;
    if (!bt || !tokens || !positions || !out || steps == 0 || bt->p->failed) return -1;
    DeviceScope scope(bt->p->ctx->device);
    if (!scope.ok) return -1;
    cudaStream_t s = bt->p->ctx->stream;
    if (grow((void **)&bt->log, &bt->log_bytes, steps * bt->B * 4, true)) return -2;
    int r = batch_set(bt, tokens, positions, steps);
    for (size_t i = 0; i < steps && !r; ++i) r = batch_run(bt, true);
    if (r) return r;
    if (cudaMemcpyAsync(out, bt->log, steps * bt->B * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess || *(volatile unsigned *)bt->p->err_host)
        return -2;
    return 0;
}

// Milliseconds per greedy step of `steps` graph replays (CUDA events on the
// plan's stream), after two untimed steps from the same tokens and positions
// (the first sizes the scratch, the second captures the graph); < 0 on error.
extern "C" double fyb_batch_time_greedy(void *batch, const uint32_t *tokens, const uint32_t *positions, size_t steps)
{
    Batch *bt = (Batch *)batch;
    if (!bt || !tokens || !positions || steps == 0) return -1.0;
    DeviceScope scope(bt->p->ctx->device);
    cudaStream_t s = bt->p->ctx->stream;
    if (grow((void **)&bt->log, &bt->log_bytes, steps * bt->B * 4, true)) return -1.0;
    if (batch_set(bt, tokens, positions, steps)) return -1.0;
    for (int w = 0; w < 2; ++w) if (batch_run(bt, true)) return -1.0;  // sizes, then captures
    // the timed steps start again from the given tokens and positions
    if (batch_set(bt, tokens, positions, steps)) return -1.0;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0); cudaEventCreate(&e1);
    cudaEventRecord(e0, s);
    int r = 0;
    for (size_t i = 0; i < steps && !r; ++i) r = batch_run(bt, true);
    cudaEventRecord(e1, s);
    float ms = -1.f;
    if (!r && cudaEventSynchronize(e1) == cudaSuccess) cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0); cudaEventDestroy(e1);
    if (r || *(volatile unsigned *)bt->p->err_host) return -1.0;
    return ms / (double)steps;
}

extern "C" unsigned long long fyb_batch_launches_per_step(const void *batch)
{
    return batch ? ((const Batch *)batch)->launches : 0;
}

extern "C" const char *fyb_version(void) { return "fyodor_b200 0.1 (sm_100a)"; }

extern "C" int fyb_device_count(void)
{
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n;
}

extern "C" int fyb_dequantize(const void *w, size_t count, unsigned type, float *out, void *stream)
{
    size_t block, bytes;
    if (!w || !out || !type_geometry(type, &block, &bytes) || count % block) return -1;
    return launch_dequant(w, type, count, out, (cudaStream_t)stream);
}

// Workspace of fyb_quant_matmul for one shape: [tile counters][partials][units].
// Workspace of fyb_quant_matmul*: [stream-K counters][GEMV partials][units]
// [small-batch GEMM scratch for `batch` vectors, at most 16 per group].
static void qm_layout(size_t rows, size_t cols, unsigned type, int sms, size_t batch, size_t *counters,
    size_t *partials, size_t *units, size_t *gemm)
{
    QgemvLaunch L;
    L.w.type = type; L.w.cols = (unsigned)cols; L.w.tiles = (unsigned)((rows + 15) / 16);
    L.seg_rows[0] = (unsigned)rows;
    *counters = ((size_t)L.w.tiles * 4 + 255) / 256 * 256;
    *partials = (qgemv_partials_bytes(L, sms) + 255) / 256 * 256;
    *units = (qunits_bytes(type, L.w.tiles, cols) + 255) / 256 * 256;
    *gemm = 0;
    for (size_t nv = 3; nv <= std::min<size_t>(batch, 16); ++nv)
        *gemm = std::max(*gemm, qgemm_workspace_bytes(type, rows, cols, nv, sms));
}

static int current_sms()
{
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaGetLastError();
    return sms > 0 ? sms : 148;
}

extern "C" size_t fyb_quant_matmul_workspace(size_t rows, size_t cols, unsigned type, size_t batch)
{
    if (!qgemv_supported(type, cols, 1) || rows == 0) return 0;
    size_t a, b, u, g;
    qm_layout(rows, cols, type, current_sms(), batch, &a, &b, &u, &g);
    return a + b + u + g;
}

extern "C" int fyb_quant_matmul(const void *w, size_t rows, size_t cols, unsigned type, const float *x, float *y,
    size_t batch, void *workspace, size_t workspace_bytes, void *stream)
{
    size_t block, bbytes;
    if (!w || !x || !y || !rows || !cols || !batch || rows > 0x7fffffffu || !type_geometry(type, &block, &bbytes) ||
        cols % block)
        return -1;
    cudaStream_t s = (cudaStream_t)stream;
    const int sms = current_sms();
    const size_t row_bytes = cols / block * bbytes;
    if (!qgemv_supported(type, cols, 1))
        return launch_generic_matmul(w, row_bytes, rows, cols, type, x, cols, y, rows, batch, s);
    size_t cb, pb, ub, gb;
    qm_layout(rows, cols, type, sms, batch, &cb, &pb, &ub, &gb);
    if (!workspace || workspace_bytes < cb + pb + ub + gb) return -1;
    unsigned char *ws = (unsigned char *)workspace;
    QWeights qw;
    qw.units = ws + cb + pb; qw.type = type; qw.cols = (unsigned)cols; qw.tiles = (unsigned)((rows + 15) / 16);
    if (repack_units(w, nullptr, rows, cols, type, REPACK_PLAIN, ws + cb + pb, qw.tiles, s)) return -2;
    unsigned *counters = (unsigned *)ws;
    float *partials = (float *)(ws + cb);
    void *gemm = ws + cb + pb + ub;
    size_t cbytes = cb, pbytes = pb, gbytes = gb;
    const Scratch sc{&counters, &cbytes, &partials, &pbytes, &gemm, &gbytes};
    return device_matmul(&qw, w, row_bytes, rows, cols, type, x, y, batch, sc, s, sms) ? -2 : 0;
}

// fyb_quant_matmul in two halves: the repack into the workspace's units
// (once per weight matrix), then any number of products from them.
extern "C" int fyb_quant_repack(const void *w, size_t rows, size_t cols, unsigned type, void *workspace,
    size_t workspace_bytes, void *stream)
{
    size_t block, bbytes;
    if (!w || !rows || !cols || rows > 0x7fffffffu || !type_geometry(type, &block, &bbytes) || cols % block ||
        !qgemv_supported(type, cols, 1) || !workspace)
        return -1;
    size_t cb, pb, ub, gb;
    qm_layout(rows, cols, type, current_sms(), 1, &cb, &pb, &ub, &gb);
    if (workspace_bytes < cb + pb + ub) return -1;
    unsigned char *ws = (unsigned char *)workspace;
    return repack_units(w, nullptr, rows, cols, type, REPACK_PLAIN, ws + cb + pb, (unsigned)((rows + 15) / 16),
                        (cudaStream_t)stream) ? -2 : 0;
}

extern "C" int fyb_quant_matmul_prepared(size_t rows, size_t cols, unsigned type, const float *x, float *y,
    size_t batch, void *workspace, size_t workspace_bytes, void *stream)
{
    if (!x || !y || !rows || !cols || !batch || rows > 0x7fffffffu || !qgemv_supported(type, cols, 1) || !workspace)
        return -1;
    const int sms = current_sms();
    size_t cb, pb, ub, gb;
    qm_layout(rows, cols, type, sms, batch, &cb, &pb, &ub, &gb);
    if (workspace_bytes < cb + pb + ub + gb) return -1;
    unsigned char *ws = (unsigned char *)workspace;
    QWeights qw;
    qw.units = ws + cb + pb; qw.type = type; qw.cols = (unsigned)cols; qw.tiles = (unsigned)((rows + 15) / 16);
    unsigned *counters = (unsigned *)ws;
    float *partials = (float *)(ws + cb);
    void *gemm = ws + cb + pb + ub;
    size_t cbytes = cb, pbytes = pb, gbytes = gb;
    const Scratch sc{&counters, &cbytes, &partials, &pbytes, &gemm, &gbytes};
    return device_matmul(&qw, nullptr, 0, rows, cols, type, x, y, batch, sc, (cudaStream_t)stream, sms) ? -2 : 0;
}

extern "C" size_t fyb_attention_workspace(unsigned nseq, unsigned heads, unsigned kv_heads, unsigned head_dim, unsigned splits)
{
    if (!kv_heads || !nseq) return 0;
    AttentionLaunch L;
    L.nseq = nseq; L.heads = heads; L.kv_heads = kv_heads; L.head_dim = head_dim;
    L.splits = splits ? splits : 8;
    return attention_workspace_bytes(L);
}

extern "C" int fyb_attention_decode(const float *q, const void *k, const void *v, size_t seq_stride,
    const unsigned *lengths, unsigned nseq, unsigned heads, unsigned kv_heads, unsigned head_dim, unsigned capacity,
    float scale, float *out, unsigned splits, void *workspace, size_t workspace_bytes, void *stream)
{
    AttentionLaunch L;
    L.q = q; L.k = (const __half *)k; L.v = (const __half *)v;
    L.seq_stride = seq_stride; L.lengths = lengths;
    L.nseq = nseq; L.heads = heads; L.kv_heads = kv_heads; L.head_dim = head_dim; L.capacity = capacity;
    L.scale = scale; L.out = out; L.splits = splits ? splits : 8;
    L.workspace = workspace; L.workspace_bytes = workspace_bytes;
    if (!lengths) return -1;
    return launch_attention(L, (cudaStream_t)stream);
}

extern "C" int fyb_attention_verify(const float *q, const void *k, const void *v, size_t seq_stride,
    const unsigned *lengths, unsigned nseq, unsigned queries, unsigned heads, unsigned kv_heads, unsigned head_dim,
    unsigned capacity, float scale, float *out, unsigned splits, void *workspace, size_t workspace_bytes, void *stream)
{
    AttentionLaunch L;
    L.q = q; L.k = (const __half *)k; L.v = (const __half *)v;
    L.seq_stride = seq_stride; L.lengths = lengths;
    L.nseq = nseq; L.queries = queries; L.heads = heads; L.kv_heads = kv_heads; L.head_dim = head_dim;
    L.capacity = capacity; L.scale = scale; L.out = out; L.splits = splits ? splits : 8;
    L.workspace = workspace; L.workspace_bytes = workspace_bytes;
    if (!lengths) return -1;
    return launch_attention(L, (cudaStream_t)stream);
}

extern "C" int fyb_plan_decode_greedy(void *opaque, uint32_t token, size_t position, size_t steps, uint32_t *tokens_out)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->failed || !p->connected || !tokens_out || token >= p->V || position > p->valid || steps == 0 ||
        steps > p->capacity - position)
        return -1;
    DeviceScope scope(p->ctx->device);
    if (set_request(p, token, (unsigned)position)) return plan_fail(p, position);
    for (size_t i = 0; i < steps; ++i)
        if (run_step(p, STEP_GREEDY)) return plan_fail(p, position + i);
    if (cudaMemcpyAsync(tokens_out, p->tokens_log, steps * 4, cudaMemcpyDeviceToHost, p->ctx->stream) != cudaSuccess ||
        cudaStreamSynchronize(p->ctx->stream) != cudaSuccess || *(volatile unsigned *)p->err_host)
        return plan_fail(p, position);
    p->valid = position + steps;
    return 0;
}

extern "C" double fyb_plan_time_greedy(void *opaque, uint32_t token, size_t position, size_t steps)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->failed || !p->connected || token >= p->V || position > p->valid || steps == 0 ||
        steps > p->capacity - position)
        return -1.0;
    DeviceScope scope(p->ctx->device);
    cudaEvent_t a, b;
    cudaEventCreate(&a); cudaEventCreate(&b);
    set_request(p, token, (unsigned)position);
    cudaEventRecord(a, p->ctx->stream);
    for (size_t i = 0; i < steps; ++i)
        if (run_step(p, STEP_GREEDY)) { cudaEventDestroy(a); cudaEventDestroy(b); plan_fail(p, position + i); return -1.0; }
    cudaEventRecord(b, p->ctx->stream);
    float ms = -1.f;
    if (cudaEventSynchronize(b) != cudaSuccess || cudaEventElapsedTime(&ms, a, b) != cudaSuccess || *(volatile unsigned *)p->err_host)
        ms = -1.f;
    cudaEventDestroy(a); cudaEventDestroy(b);
    if (ms >= 0) p->valid = std::max(p->valid, position + steps);
    return ms;
}

extern "C" unsigned long long fyb_plan_launches_per_token(const void *opaque)
{
    const Plan *p = (const Plan *)opaque;
    if (!p) return 0;
    if (p->dec_grid) return 2;  // request + the persistent decode kernel
    // request (1) + gather (1) + 5 per layer + logits (1)
    return 3ull + 5ull * p->nl;
}

extern "C" int fyb_plan_decode_form(const void *opaque)
{
    const Plan *p = (const Plan *)opaque;
    if (!p) return -1;
    return !p->dec_grid ? 0 : 1;
}

extern "C" int fyb_plan_tp_info(const void *opaque, unsigned *rank, unsigned *size)
{
    const Plan *p = (const Plan *)opaque;
    if (!p) return -1;
    if (rank) *rank = p->tp_rank;
    if (size) *size = p->tp_size;
    return 0;
}

extern "C" int fyb_plan_tp_handle(void *opaque, void *handle, size_t bytes)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->tp_size < 2 || !handle || bytes < sizeof(cudaIpcMemHandle_t)) return -1;
    DeviceScope scope(p->ctx->device);
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p->xchg) != cudaSuccess) { cudaGetLastError(); return -2; }
    std::memcpy(handle, &h, sizeof(h));
    return 0;
}

extern "C" int fyb_plan_tp_connect(void *opaque, const void *handles, size_t count)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->tp_size < 2 || p->connected || !handles || count != p->tp_size) return -1;
    DeviceScope scope(p->ctx->device);
    p->peers.assign(p->tp_size, nullptr);
    p->peers[p->tp_rank] = p->xchg;
    for (unsigned j = 0; j < p->tp_size; ++j) {
        if (j == p->tp_rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, (const unsigned char *)handles + (size_t)j * sizeof(h), sizeof(h));
        void *ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            debug("opening a peer's exchange region", cudaErrorInvalidValue);
            return -2;
        }
        p->peers[j] = (unsigned char *)ptr;
    }
    if (!upload(p->peers_dev, p->peers.data(), p->tp_size * sizeof(void *), p->ctx->stream) ||
        cudaStreamSynchronize(p->ctx->stream) != cudaSuccess)
        return -2;
    p->connected = true;
    return 0;
}

extern "C" int fyb_plan_tp_connect_local(void *opaque, void *const *plans, size_t count)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->tp_size < 2 || p->connected || !plans || count != p->tp_size || plans[p->tp_rank] != opaque)
        return -1;
    for (unsigned j = 0; j < p->tp_size; ++j) {
        const Plan *q = (const Plan *)plans[j];
        if (!q || q->tp_size != p->tp_size || q->tp_rank != j || !q->xchg || q->xchg_bytes != p->xchg_bytes)
            return -1;
    }
    DeviceScope scope(p->ctx->device);
    for (unsigned j = 0; j < p->tp_size; ++j) {
        const int dev = ((const Plan *)plans[j])->ctx->device;
        if (dev == p->ctx->device) continue;
        int can = 0;
        if (cudaDeviceCanAccessPeer(&can, p->ctx->device, dev) != cudaSuccess || !can) { cudaGetLastError(); return -2; }
        const cudaError_t e = cudaDeviceEnablePeerAccess(dev, 0);
        if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) { cudaGetLastError(); return -2; }
        cudaGetLastError();
    }
    std::vector<unsigned char *> peers(p->tp_size);
    for (unsigned j = 0; j < p->tp_size; ++j) peers[j] = ((const Plan *)plans[j])->xchg;
    if (!upload(p->peers_dev, peers.data(), p->tp_size * sizeof(void *), p->ctx->stream) ||
        cudaStreamSynchronize(p->ctx->stream) != cudaSuccess)
        return -2;
    // the regions belong to the other plans: nothing to close on free
    p->peers.assign(p->tp_size, nullptr);
    p->peers[p->tp_rank] = p->xchg;
    p->connected = true;
    return 0;
}

extern "C" int fyb_plan_error(const void *opaque)
{
    const Plan *p = (const Plan *)opaque;
    if (!p) return -1;
    return p->err_host ? (int)*(volatile const unsigned *)p->err_host : 0;
}

extern "C" int fyb_plan_tp_disconnect(void *opaque)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->tp_size < 2) return -1;
    p->connected = false;  // plan_token and the greedy loop now decline without launching
    return 0;
}

extern "C" long fyb_plan_trace(void *opaque, uint32_t token, size_t position, unsigned long long *out,
    size_t out_count, unsigned *grid_out, unsigned long long *warp_out, size_t warp_count)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->failed || !p->connected || !p->dec_grid || token >= p->V || position >= p->capacity ||
        position > p->valid || !out)
        return -1;
    const unsigned points = decode_trace_points(p->nl);
    const size_t n = (size_t)points * p->dec_grid;
    if (out_count < n) return -1;
    const size_t wn = decode_dtrace_words(p->dec_grid);
    if (warp_out && warp_count < wn) return -1;
    DeviceScope scope(p->ctx->device);
    cudaStream_t s = p->ctx->stream;
    unsigned long long *buf = nullptr, *wbuf = nullptr;
    if (cudaMalloc(&buf, n * 8) != cudaSuccess) { cudaGetLastError(); return -1; }
    if (warp_out && cudaMalloc(&wbuf, wn * 8) != cudaSuccess) { cudaGetLastError(); cudaFree(buf); return -1; }
    DecodeLaunch L = persistent_launch(p, STEP_LOGITS);
    L.trace = buf; L.trace_slots = points; L.dtrace = wbuf;
    int r = cudaMemsetAsync(buf, 0, n * 8, s) == cudaSuccess &&
            (!wbuf || cudaMemsetAsync(wbuf, 0, wn * 8, s) == cudaSuccess) &&
            set_request(p, token, (unsigned)position) == 0 &&
            launch_decode(L, s) == 0 && cudaMemcpyAsync(out, buf, n * 8, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
            (!wbuf || cudaMemcpyAsync(warp_out, wbuf, wn * 8, cudaMemcpyDeviceToHost, s) == cudaSuccess) &&
            cudaStreamSynchronize(s) == cudaSuccess && !*(volatile unsigned *)p->err_host ? 0 : -1;
    if (wbuf) cudaFree(wbuf);
    cudaFree(buf);
    if (r) return plan_fail(p, position);
    p->valid = std::max(p->valid, position + 1);
    if (grid_out) *grid_out = (unsigned)p->dec_grid;
    return points;
}

extern "C" int fyb_plan_profile(void *opaque, uint32_t token, size_t position, size_t steps, double *out)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->failed || p->tp_size > 1 || !out || token >= p->V || position > p->valid || steps == 0 ||
        steps > p->capacity - position)
        return -1;
    DeviceScope scope(p->ctx->device);
    out[0] = out[1] = out[2] = 0.0;
    std::vector<std::pair<cudaEvent_t, int>> marks;
    p->marks = &marks;
    int r = 0;
    for (size_t i = 0; i < steps && !r; ++i) {
        cudaEvent_t start;
        cudaEventCreate(&start);
        set_request(p, token, (unsigned)(position + i));
        cudaEventRecord(start, p->ctx->stream);
        marks.clear();
        r = enqueue_step(p, STEP_LOGITS);
        if (cudaStreamSynchronize(p->ctx->stream) != cudaSuccess) r = -2;
        cudaEvent_t prev = start;
        for (auto &m : marks) {
            float ms = 0.f;
            if (!r && cudaEventElapsedTime(&ms, prev, m.first) == cudaSuccess) out[m.second & 15] += ms;
            prev = m.first;
        }
        for (auto &m : marks) cudaEventDestroy(m.first);
        cudaEventDestroy(start);
    }
    p->marks = nullptr;
    if (r) return plan_fail(p, position);
    for (int k = 0; k < 3; ++k) out[k] /= (double)steps;
    p->valid = std::max(p->valid, position + steps);
    return 0;
}

// Times `reps` stand-alone launches of one fused projection kernel of a
// layer (which: 0 QKV, 1 O, 2 gate/up, 3 down, 4 logits) with CUDA events on
// the plan's stream; *bytes receives its algorithmic bytes per launch
// (weights + input vector + norm weights + outputs).
extern "C" double fyb_plan_time_projection(void *opaque, unsigned layer, unsigned which, unsigned reps, size_t *bytes)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->failed || layer >= p->nl || which > 4 || reps == 0) return -1.0;
    DeviceScope scope(p->ctx->device);
    size_t in_bytes = (size_t)p->d * 4, out_bytes = 0, norm_bytes = 0;
    // launch i reads layer (layer + i) % layers, so back-to-back launches do
    // not find the previous launch's weights in L2 (unless the model is small)
    auto make = [&](unsigned l) {
        QgemvLaunch L;
        switch (which) {
        case 0:
            L = qkv_launch(p, l); L.x = p->x[0];
            norm_bytes = (size_t)p->d * 4;
            out_bytes = (size_t)p->H * p->hd * 4 + (size_t)2 * p->Hkv * p->hd * 2;
            break;
        case 1:
            L = o_launch(p, l);
            out_bytes = (size_t)p->d * 4; in_bytes = (size_t)p->H * p->hd * 4;
            break;
        case 2:
            L = gateup_launch(p, l); L.x = p->x[0];
            norm_bytes = (size_t)p->d * 4; out_bytes = (size_t)p->ffn * 4;
            break;
        case 3:
            L = down_launch(p, l);
            in_bytes = (size_t)p->ffn * 4; out_bytes = (size_t)p->d * 4;
            break;
        default:
            L = logits_launch(p); L.x = p->x[0];
            norm_bytes = (size_t)p->d * 4; out_bytes = (size_t)p->V * 4;
            break;
        }
        return L;
    };
    QgemvLaunch L = make(layer);
    // GGUF bytes of the weights (the repacked units have the same size)
    const size_t weight_bytes = qunits_bytes(L.w.type, L.w.tiles, L.w.cols);
    if (bytes) *bytes = weight_bytes + in_bytes + norm_bytes + out_bytes;
    cudaEvent_t a, b;
    cudaEventCreate(&a); cudaEventCreate(&b);
    if (launch_qgemv(L, p->ctx->stream)) { cudaEventDestroy(a); cudaEventDestroy(b); return -1.0; }  // warm-up
    cudaEventRecord(a, p->ctx->stream);
    int r = 0;
    for (unsigned i = 0; i < reps && !r; ++i) r = launch_qgemv(make((layer + 1 + i) % p->nl), p->ctx->stream);
    cudaEventRecord(b, p->ctx->stream);
    float ms = -1.f;
    if (r || cudaEventSynchronize(b) != cudaSuccess || cudaEventElapsedTime(&ms, a, b) != cudaSuccess) ms = -1.f;
    cudaEventDestroy(a); cudaEventDestroy(b);
    return ms < 0 ? -1.0 : (double)ms / reps;
}
