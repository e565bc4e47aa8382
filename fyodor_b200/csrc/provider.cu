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
    void *dev = nullptr;       // GGUF bytes
    void *repacked = nullptr;  // Q6_K tensor-core layout
    QMatrix qm;
};

struct Context {
    int device = 0;
    cudaStream_t stream = nullptr;
    size_t cache_limit = 0, cached_bytes = 0;
    std::vector<CachedWeight> weights;
    bool failed = false;
    float *dx = nullptr, *dy = nullptr;
    size_t dx_bytes = 0, dy_bytes = 0;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    int sms = 148;
};

constexpr size_t WEIGHT_LIMIT = 2048;

static void context_free(Context *c)
{
    if (!c) return;
    {
        DeviceScope scope(c->device);
        if (c->stream) cudaStreamSynchronize(c->stream);
        for (auto &w : c->weights) { cudaFree(w.dev); cudaFree(w.repacked); }
        cudaFree(c->dx); cudaFree(c->dy); cudaFree(c->ws);
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
    if (zero && cudaMemset(n, 0, bytes) != cudaSuccess) { cudaFree(n); return -1; }
    if (*p) cudaFree(*p);
    *p = n;
    *cap = bytes;
    return 0;
}

static CachedWeight *cached_weight(Context *c, const void *w, size_t rows, size_t cols, unsigned type, size_t bytes)
{
    for (auto &e : c->weights)
        if (e.source == w && e.rows == rows && e.cols == cols && e.type == type) return &e;
    if (c->weights.size() >= WEIGHT_LIMIT) return nullptr;
    size_t extra = type == T_Q6_K ? q6k_repacked_bytes(rows, cols) : 0;
    if (bytes + extra > c->cache_limit - std::min(c->cache_limit, c->cached_bytes)) return nullptr;
    CachedWeight e;
    e.source = w; e.rows = rows; e.cols = cols; e.type = type; e.bytes = bytes + extra;
    if (cudaMalloc(&e.dev, bytes) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    if (cudaMemcpy(e.dev, w, bytes, cudaMemcpyHostToDevice) != cudaSuccess) { cudaFree(e.dev); return nullptr; }
    if (type == T_Q4_K) e.qm = q4k_matrix(e.dev, rows, cols);
    if (type == T_Q6_K && cols % 256 == 0) {
        if (cudaMalloc(&e.repacked, extra) != cudaSuccess ||
            repack_q6k(e.dev, rows, cols, e.repacked, &e.qm, c->stream) != 0) {
            cudaGetLastError(); cudaFree(e.dev); cudaFree(e.repacked); return nullptr;
        }
    }
    c->cached_bytes += e.bytes;
    c->weights.push_back(e);
    return &c->weights.back();
}

// Shared device-side matmul on already-resident data.
static int device_matmul(const QMatrix *qm, const void *raw, size_t row_bytes, size_t rows, size_t cols,
    unsigned type, const float *x, float *y, size_t batch, void **ws, size_t *ws_bytes, cudaStream_t s, int sms)
{
    if (qm && qm->bits && qgemv_supported(type, cols, 1)) {
        for (size_t b0 = 0; b0 < batch; b0 += 2) {
            QgemvLaunch L;
            L.epilogue = EPI_STORE;
            L.nseg = 1;
            L.seg[0] = *qm;
            L.nvec = (int)std::min<size_t>(2, batch - b0);
            L.x = x + b0 * cols;
            L.out[0] = y + b0 * rows;
            L.out_stride = rows;
            L.grid = sms;
            size_t need = qgemv_workspace_bytes(L, sms);
            if (ws_bytes && grow(ws, ws_bytes, need, true) != 0) return -2;
            L.workspace = *ws;
            L.workspace_bytes = ws_bytes ? *ws_bytes : need;
            int r = launch_qgemv(L, s);
            if (r) return r;
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
        if (device_matmul(e->qm.bits ? &e->qm : nullptr, e->dev, row_bytes, rows, cols, type, c->dx, c->dy, batch,
                          &c->ws, &c->ws_bytes, c->stream, c->sms) != 0)
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
    QMatrix q, k, v, o, gate, up, down;
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
};

enum StepMode { STEP_LOGITS = 0, STEP_NO_LOGITS = 1, STEP_GREEDY = 2 };

struct Plan {
    Context *ctx = nullptr;
    const nya_llm_context *m = nullptr;
    size_t capacity = 0;
    unsigned d = 0, H = 0, Hkv = 0, hd = 0, ffn = 0, V = 0, nl = 0;
    float eps = 1e-5f;
    std::vector<void *> allocations;
    std::vector<LayerW> layers;
    QMatrix out_head;
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
    void *gemv_ws = nullptr;
    size_t gemv_ws_bytes = 0;
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
    // profiling: when set, an event is recorded after every launch
    std::vector<std::pair<cudaEvent_t, int>> *marks = nullptr;
};

enum KernelClass { KC_MATRIX = 0, KC_ATTENTION = 1, KC_OTHER = 2 };

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
    {
        DeviceScope scope(p->ctx->device);
        cudaStreamSynchronize(p->ctx->stream);
        for (auto &g : p->graphs) if (g) cudaGraphExecDestroy(g);
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

static int launch_plain(Plan *p, void (*k)(unsigned *, const unsigned *, unsigned *), bool pdl)
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
    return cudaLaunchKernelEx(&cfg, k, p->request, (const unsigned *)p->argmax_token, p->tokens_log) == cudaSuccess ? 0 : -2;
}

// Enqueue one decode step reading {token, position} from p->request.
static int enqueue_step(Plan *p, StepMode mode)
{
    cudaStream_t s = p->ctx->stream;
    const bool pdl = true;
    const int grid = p->ctx->sms;
    p->launches = 0;
    int kc = KC_OTHER;
#define RUN(expr) do { int r_ = (expr); ++p->launches; if (r_) return r_; \
        if (p->marks) { cudaEvent_t ev; cudaEventCreate(&ev); cudaEventRecord(ev, s); p->marks->push_back({ev, kc}); } } while (0)
    kc = KC_OTHER;
    RUN(launch_gather(p->embd, p->embd_row_bytes, p->embd_type, p->d, p->request, 0, p->x[0], s, false));
    int cur = 0;
    bool pending = false;  // delta holds an unadded branch output
    for (unsigned l = 0; l < p->nl; ++l) {
        const LayerW &w = p->layers[l];
        QgemvLaunch L;
        L.epilogue = EPI_QKV;
        L.nseg = 3;
        L.seg[0] = w.q; L.seg[1] = w.k; L.seg[2] = w.v;
        L.out[0] = p->q;
        L.kcache = p->kcache + (size_t)l * p->Hkv * p->capacity * p->hd;
        L.vcache = p->vcache + (size_t)l * p->Hkv * p->capacity * p->hd;
        L.x = p->x[cur];
        if (pending) { L.delta = p->delta; L.x_out = p->x[cur ^ 1]; }
        L.norm_w = w.attn_norm;
        L.eps = p->eps;
        L.rope_cos = p->rope_cos; L.rope_sin = p->rope_sin;
        L.request = p->request;
        L.head_dim = p->hd;
        L.capacity = (unsigned)p->capacity;
        L.workspace = p->gemv_ws; L.workspace_bytes = p->gemv_ws_bytes;
        L.error = p->err_dev;
        L.grid = grid; L.pdl = pdl;
        kc = KC_MATRIX;
        RUN(launch_qgemv(L, s));
        if (pending) cur ^= 1;

        AttentionLaunch A;
        A.q = p->q;
        A.k = L.kcache; A.v = L.vcache;
        A.request = p->request;
        A.nseq = 1; A.heads = p->H; A.kv_heads = p->Hkv; A.head_dim = p->hd;
        A.capacity = (unsigned)p->capacity;
        A.scale = 1.0f / std::sqrt((float)p->hd);
        A.out = p->attn;
        A.splits = p->attn_splits;
        A.workspace = p->attn_ws; A.workspace_bytes = p->attn_ws_bytes;
        A.pdl = pdl;
        kc = KC_ATTENTION;
        RUN(launch_attention(A, s));
        kc = KC_MATRIX;

        QgemvLaunch O;
        O.epilogue = EPI_STORE;
        O.seg[0] = w.o;
        O.out[0] = p->delta;
        O.x = p->attn;
        O.workspace = p->gemv_ws; O.workspace_bytes = p->gemv_ws_bytes;
        O.error = p->err_dev;
        O.grid = grid; O.pdl = pdl;
        RUN(launch_qgemv(O, s));

        QgemvLaunch G;
        G.epilogue = EPI_SWIGLU;
        G.nseg = 2;
        G.seg[0] = w.gate; G.seg[1] = w.up;
        G.out[0] = p->h;
        G.x = p->x[cur]; G.delta = p->delta; G.x_out = p->x[cur ^ 1];
        G.norm_w = w.ffn_norm; G.eps = p->eps;
        G.workspace = p->gemv_ws; G.workspace_bytes = p->gemv_ws_bytes;
        G.error = p->err_dev;
        G.grid = grid; G.pdl = pdl;
        RUN(launch_qgemv(G, s));
        cur ^= 1;

        QgemvLaunch D;
        D.epilogue = EPI_STORE;
        D.seg[0] = w.down;
        D.out[0] = p->delta;
        D.x = p->h;
        D.workspace = p->gemv_ws; D.workspace_bytes = p->gemv_ws_bytes;
        D.error = p->err_dev;
        D.grid = grid; D.pdl = pdl;
        RUN(launch_qgemv(D, s));
        pending = true;
    }
    if (mode == STEP_NO_LOGITS) {
        // the residual stream is complete in x[cur] + delta; nothing reads it
        return 0;
    }
    QgemvLaunch Lg;
    Lg.epilogue = EPI_LOGITS;
    Lg.seg[0] = p->out_head;
    Lg.out[0] = p->logits;
    Lg.x = p->x[cur];
    Lg.delta = pending ? p->delta : nullptr;
    Lg.norm_w = p->out_norm; Lg.eps = p->eps;
    Lg.argmax_key = p->argmax_key; Lg.argmax_token = p->argmax_token; Lg.tiles_done = p->tiles_done;
    Lg.workspace = p->gemv_ws; Lg.workspace_bytes = p->gemv_ws_bytes;
    Lg.error = p->err_dev;
    Lg.grid = grid; Lg.pdl = pdl;
    kc = KC_MATRIX;
    RUN(launch_qgemv(Lg, s));
    kc = KC_OTHER;
    if (mode == STEP_GREEDY) RUN(launch_plain(p, advance_kernel, pdl));
#undef RUN
    return 0;
}

static int run_step(Plan *p, StepMode mode)
{
    cudaStream_t s = p->ctx->stream;
    if (!p->use_graphs) {
        int r = enqueue_step(p, mode);
        p->stats.kernel_launches += p->launches;
        return r;
    }
    if (!p->graphs[mode]) {
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return -2;
        int r = enqueue_step(p, mode);
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

static bool supported_matrix(const nya_llm_tensor *t, size_t cols, size_t rows)
{
    return t && (t->type == T_Q4_K || t->type == T_Q6_K) && t->dimension_count == 2 && t->dimensions[0] == cols &&
           t->dimensions[1] == rows && qgemv_supported(t->type, cols, 1);
}

// Device copy of one matrix in the tensor-core layout.
static int upload_matrix(Plan *p, const nya_llm_tensor *t, QMatrix *out)
{
    const size_t cols = (size_t)t->dimensions[0], rows = (size_t)t->dimensions[1];
    if (t->type == T_Q4_K) {
        void *d = plan_alloc(p, t->data_size);
        if (!d || cudaMemcpy(d, t->data, t->data_size, cudaMemcpyHostToDevice) != cudaSuccess) return -1;
        *out = q4k_matrix(d, rows, cols);
        return 0;
    }
    void *raw = nullptr;
    if (cudaMalloc(&raw, t->data_size) != cudaSuccess) { cudaGetLastError(); return -1; }
    void *d = plan_alloc(p, q6k_repacked_bytes(rows, cols));
    int r = -1;
    if (d && cudaMemcpy(raw, t->data, t->data_size, cudaMemcpyHostToDevice) == cudaSuccess &&
        repack_q6k(raw, rows, cols, d, out, p->ctx->stream) == 0 && cudaStreamSynchronize(p->ctx->stream) == cudaSuccess)
        r = 0;
    cudaFree(raw);
    return r;
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

    // admission: weights + KV + scratch against the budget (resident.inc:155-168)
    size_t weights = 0;
    for (size_t i = 0; i < m->tensor_count; ++i) {
        const nya_llm_tensor &t = m->tensors[i];
        weights += t.type == T_Q6_K && t.dimension_count == 2 && &t != m->token_embedding
                       ? q6k_repacked_bytes((size_t)t.dimensions[1], (size_t)t.dimensions[0]) : t.data_size;
    }
    const size_t kv_bytes = (size_t)nl * Hkv * capacity * hd * sizeof(__half) * 2;
    const size_t act = ((size_t)d * 3 + (size_t)H * hd * 2 + ffn + V) * sizeof(float) + 2 * capacity * (hd / 2) * sizeof(float);
    if (weights + kv_bytes + act > c->cache_limit) return plan_decline("weights plus KV/scratch exceed the memory budget");

    Plan *p = new Plan();
    p->ctx = c; p->m = m; p->capacity = capacity;
    p->d = d; p->H = H; p->Hkv = Hkv; p->hd = hd; p->ffn = ffn; p->V = V; p->nl = nl;
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
    if (ok) ok = cudaMemset(p->argmax_key, 0, 64) == cudaSuccess && cudaMemset(p->tiles_done, 0, 64) == cudaSuccess &&
                 cudaMemset(p->request, 0, 64) == cudaSuccess;

    // weights
    p->layers.resize(nl);
    for (unsigned i = 0; ok && i < nl; ++i) {
        const nya_llm_layer &w = m->layers[i];
        LayerW &L = p->layers[i];
        ok = upload_matrix(p, w.query, &L.q) == 0 && upload_matrix(p, w.key, &L.k) == 0 &&
             upload_matrix(p, w.value, &L.v) == 0 && upload_matrix(p, w.attention_output, &L.o) == 0 &&
             upload_matrix(p, w.feed_forward_gate, &L.gate) == 0 && upload_matrix(p, w.feed_forward_up, &L.up) == 0 &&
             upload_matrix(p, w.feed_forward_down, &L.down) == 0;
        if (!ok) break;
        float *an = (float *)A(d * 4), *fn = (float *)A(d * 4);
        ok = ok && cudaMemcpy(an, w.attention_norm->data, d * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(fn, w.feed_forward_norm->data, d * 4, cudaMemcpyHostToDevice) == cudaSuccess;
        L.attn_norm = an; L.ffn_norm = fn;
    }
    if (ok) ok = upload_matrix(p, m->output, &p->out_head) == 0;
    if (ok) {
        void *e = A(m->token_embedding->data_size);
        ok = ok && cudaMemcpy(e, m->token_embedding->data, m->token_embedding->data_size, cudaMemcpyHostToDevice) == cudaSuccess;
        p->embd = e;
        p->embd_type = m->token_embedding->type;
        p->embd_row_bytes = d / eblock * ebytes;
        float *on = (float *)A(d * 4);
        ok = ok && cudaMemcpy(on, m->output_norm->data, d * 4, cudaMemcpyHostToDevice) == cudaSuccess;
        p->out_norm = on;
    }
    // RoPE tables with the engine's own host formula (llm_cpu.c:216-229, :428-432)
    if (ok) {
        const unsigned pairs = hd / 2;
        std::vector<float> freq(pairs), co(capacity * pairs), si(capacity * pairs);
        for (unsigned j = 0; j < pairs; ++j) freq[j] = powf(m->rope_frequency_base, -(float)j / (float)pairs) / 1.0f;
        for (size_t t = 0; t < capacity; ++t)
            for (unsigned j = 0; j < pairs; ++j) {
                float angle = (float)t * freq[j];
                co[t * pairs + j] = cosf(angle);
                si[t * pairs + j] = sinf(angle);
            }
        ok = cudaMemcpy(p->rope_cos, co.data(), co.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(p->rope_sin, si.data(), si.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
    }
    // workspaces: the largest GEMV of the step, and the attention partials
    if (ok) {
        size_t need = 0;
        const LayerW &L = p->layers[0];
        QgemvLaunch q3; q3.epilogue = EPI_QKV; q3.nseg = 3; q3.seg[0] = L.q; q3.seg[1] = L.k; q3.seg[2] = L.v;
        need = std::max(need, qgemv_workspace_bytes(q3, c->sms));
        QgemvLaunch o; o.seg[0] = L.o; need = std::max(need, qgemv_workspace_bytes(o, c->sms));
        QgemvLaunch g; g.epilogue = EPI_SWIGLU; g.nseg = 2; g.seg[0] = L.gate; g.seg[1] = L.up;
        need = std::max(need, qgemv_workspace_bytes(g, c->sms));
        QgemvLaunch dn; dn.seg[0] = L.down; need = std::max(need, qgemv_workspace_bytes(dn, c->sms));
        QgemvLaunch lg; lg.epilogue = EPI_LOGITS; lg.seg[0] = p->out_head; need = std::max(need, qgemv_workspace_bytes(lg, c->sms));
        p->gemv_ws = A(need); p->gemv_ws_bytes = need;
        // split the context so (kv heads x splits) covers about two CTAs per SM
        p->attn_splits = std::max(1u, (unsigned)(2 * c->sms) / Hkv);
        AttentionLaunch al; al.nseq = 1; al.heads = H; al.kv_heads = Hkv; al.head_dim = hd; al.splits = p->attn_splits;
        p->attn_ws_bytes = attention_workspace_bytes(al);
        p->attn_ws = A(p->attn_ws_bytes);
        if (ok) ok = cudaMemset(p->gemv_ws, 0, need) == cudaSuccess && cudaMemset(p->attn_ws, 0, p->attn_ws_bytes) == cudaSuccess;
    }
    if (ok) ok = cudaDeviceSynchronize() == cudaSuccess;
    if (!ok) {
        debug("resident plan setup failed; rolling back", cudaGetLastError());
        plan_free(p);
        return nullptr;
    }
    p->stats.weights_bytes = weights;
    p->stats.kv_bytes = kv_bytes;
    size_t scratch = act + p->gemv_ws_bytes + p->attn_ws_bytes;
    p->stats.scratch_bytes = scratch;
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
    if (cudaMemcpyAsync(out, p->logits, (size_t)p->V * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess) return -2;
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
    if (!p || p->failed || position >= p->capacity || (position != 0 && position > p->valid) || (logits && !out) ||
        token >= p->V)
        return -1;
    if (position >= p->fail_after) { p->failed = true; return -1; }
    DeviceScope scope(p->ctx->device);
    if (!scope.ok || set_request(p, token, (unsigned)position) || run_step(p, logits ? STEP_LOGITS : STEP_NO_LOGITS))
        return plan_fail(p, position);
    if (logits && finish_logits(p, out)) return plan_fail(p, position);
    p->valid = position + 1;
    return 0;
}

static int plan_prefill(void *opaque, const uint32_t *tokens, size_t count, size_t position, float *out)
{
    Plan *p = (Plan *)opaque;
    if (!p || !tokens || count == 0 || position > p->capacity || count > p->capacity - position) return -1;
    if (p->failed || (position != 0 && position > p->valid) || !out) return -1;
    for (size_t i = 0; i < count; ++i) if (tokens[i] >= p->V) return -1;
    if (position + count > p->fail_after) { p->failed = true; return -1; }
    DeviceScope scope(p->ctx->device);
    if (!scope.ok) return plan_fail(p, position);
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
    if (!p || p->failed || !keys || !values || !count || layer >= p->nl || position > p->valid ||
        count > p->valid - position)
        return -1;
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

extern "C" size_t fyb_quant_matmul_workspace(size_t rows, size_t cols, unsigned type, size_t batch)
{
    (void)batch;
    if ((type != T_Q4_K && type != T_Q6_K) || !qgemv_supported(type, cols, 1)) return 0;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaGetLastError();
    QgemvLaunch L;
    L.seg[0].rows = (unsigned)rows; L.seg[0].cols = (unsigned)cols; L.seg[0].type = type;
    size_t ws = qgemv_workspace_bytes(L, sms);
    if (type == T_Q6_K) ws += q6k_repacked_bytes(rows, cols);
    return ws;
}

extern "C" int fyb_quant_matmul(const void *w, size_t rows, size_t cols, unsigned type, const float *x, float *y,
    size_t batch, void *workspace, size_t workspace_bytes, void *stream)
{
    size_t block, bbytes;
    if (!w || !x || !y || !rows || !cols || !batch || !type_geometry(type, &block, &bbytes) || cols % block) return -1;
    cudaStream_t s = (cudaStream_t)stream;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t row_bytes = cols / block * bbytes;
    if ((type == T_Q4_K || type == T_Q6_K) && qgemv_supported(type, cols, 1)) {
        size_t need = fyb_quant_matmul_workspace(rows, cols, type, batch);
        if (!workspace || workspace_bytes < need) return -1;
        QMatrix qm = q4k_matrix(w, rows, cols);
        size_t gemv_bytes = need;
        if (type == T_Q6_K) {
            gemv_bytes = need - q6k_repacked_bytes(rows, cols);
            void *tail = (unsigned char *)workspace + gemv_bytes;
            if (repack_q6k(w, rows, cols, tail, &qm, s)) return -2;
        }
        return device_matmul(&qm, w, row_bytes, rows, cols, type, x, y, batch, &workspace, nullptr, s, sms) ? -2 : 0;
    }
    return launch_generic_matmul(w, row_bytes, rows, cols, type, x, cols, y, rows, batch, s);
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

extern "C" int fyb_plan_decode_greedy(void *opaque, uint32_t token, size_t position, size_t steps, uint32_t *tokens_out)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->failed || !tokens_out || token >= p->V || position > p->valid || steps == 0 ||
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
    if (!p || p->failed || token >= p->V || position > p->valid || steps == 0 || steps > p->capacity - position)
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
    // request (1) + gather (1) + 5 per layer + logits (1)
    return 3ull + 5ull * p->nl;
}

extern "C" int fyb_plan_profile(void *opaque, uint32_t token, size_t position, size_t steps, double *out)
{
    Plan *p = (Plan *)opaque;
    if (!p || p->failed || !out || token >= p->V || position > p->valid || steps == 0 || steps > p->capacity - position)
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
            if (!r && cudaEventElapsedTime(&ms, prev, m.first) == cudaSuccess) out[m.second] += ms;
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
    const LayerW &w = p->layers[layer];
    QgemvLaunch L;
    L.workspace = p->gemv_ws; L.workspace_bytes = p->gemv_ws_bytes;
    L.error = p->err_dev;
    L.grid = p->ctx->sms;
    L.eps = p->eps;
    size_t weight_bytes = 0, in_bytes = (size_t)p->d * 4, out_bytes = 0, norm_bytes = 0;
    auto wbytes = [](const QMatrix &m) {
        return m.type == T_Q4_K ? (size_t)m.rows * (m.cols / 256) * 144 : (size_t)m.rows * (m.cols / 256) * 210;
    };
    switch (which) {
    case 0:
        L.epilogue = EPI_QKV; L.nseg = 3; L.seg[0] = w.q; L.seg[1] = w.k; L.seg[2] = w.v;
        L.out[0] = p->q; L.kcache = p->kcache; L.vcache = p->vcache; L.x = p->x[0]; L.norm_w = w.attn_norm;
        L.rope_cos = p->rope_cos; L.rope_sin = p->rope_sin; L.request = p->request; L.head_dim = p->hd;
        L.capacity = (unsigned)p->capacity;
        weight_bytes = wbytes(w.q) + wbytes(w.k) + wbytes(w.v);
        norm_bytes = (size_t)p->d * 4;
        out_bytes = (size_t)p->H * p->hd * 4 + (size_t)2 * p->Hkv * p->hd * 2;
        break;
    case 1:
        L.seg[0] = w.o; L.out[0] = p->delta; L.x = p->attn;
        weight_bytes = wbytes(w.o); out_bytes = (size_t)p->d * 4; in_bytes = (size_t)p->H * p->hd * 4;
        break;
    case 2:
        L.epilogue = EPI_SWIGLU; L.nseg = 2; L.seg[0] = w.gate; L.seg[1] = w.up; L.out[0] = p->h;
        L.x = p->x[0]; L.norm_w = w.ffn_norm;
        weight_bytes = wbytes(w.gate) + wbytes(w.up); norm_bytes = (size_t)p->d * 4; out_bytes = (size_t)p->ffn * 4;
        break;
    case 3:
        L.seg[0] = w.down; L.out[0] = p->delta; L.x = p->h;
        weight_bytes = wbytes(w.down); in_bytes = (size_t)p->ffn * 4; out_bytes = (size_t)p->d * 4;
        break;
    default:
        L.epilogue = EPI_LOGITS; L.seg[0] = p->out_head; L.out[0] = p->logits; L.x = p->x[0]; L.norm_w = p->out_norm;
        L.argmax_key = p->argmax_key; L.argmax_token = p->argmax_token; L.tiles_done = p->tiles_done;
        weight_bytes = wbytes(p->out_head); norm_bytes = (size_t)p->d * 4; out_bytes = (size_t)p->V * 4;
        break;
    }
    if (bytes) *bytes = weight_bytes + in_bytes + norm_bytes + out_bytes;
    cudaEvent_t a, b;
    cudaEventCreate(&a); cudaEventCreate(&b);
    if (launch_qgemv(L, p->ctx->stream)) { cudaEventDestroy(a); cudaEventDestroy(b); return -1.0; }  // warm-up
    cudaEventRecord(a, p->ctx->stream);
    int r = 0;
    for (unsigned i = 0; i < reps && !r; ++i) r = launch_qgemv(L, p->ctx->stream);
    cudaEventRecord(b, p->ctx->stream);
    float ms = -1.f;
    if (r || cudaEventSynchronize(b) != cudaSuccess || cudaEventElapsedTime(&ms, a, b) != cudaSuccess) ms = -1.f;
    cudaEventDestroy(a); cudaEventDestroy(b);
    return ms < 0 ? -1.0 : (double)ms / reps;
}
