// attention.cu - split-K GQA decode attention over the fp16 KV cache.
//
// For every sequence s, KV head kh and its G = heads/kv_heads query heads:
//   out[h] = sum_t softmax_t(q_h . k_t * scale) v_t   over t in [0, L_s)
// (reference: the engine's scalar loop, backend/core/llm_cpu.c:510-535, and
// nya_attention_split/_combine, CUDA/resident.cu:175-269, which keep F32 KV
// and materialize the score row in global memory).
//
// Here the context of each (s, kh) is cut into `splits` partitions, one CTA
// each. A CTA streams its partition of K and V once, keeps an online softmax
// (running max, running sum, unnormalized output) per query head in
// registers, and writes {m, l, o[hd]} per head to a scratch slot. The CTA
// that finishes last for (s, kh) - an atomic counter, no waiting - merges the
// slots in partition order and writes the normalized output, so the result
// does not depend on scheduling. Nothing of size L is materialized.
//
// Inside a CTA each warp takes 32 positions at a time: lane j computes the
// full 128-wide dot products of position j with all G query heads (K row read
// as 16-byte vectors, query broadcast from shared memory), the warp updates
// the online softmax, then the lanes switch to 4 output dimensions each and
// accumulate p * v over the 32 positions.
#include "common.cuh"
#include "fyodor_b200.h"
#include "kernels.h"
#include <cfloat>
#include <mutex>

namespace fyb {

constexpr int AT_WARPS = 4;
constexpr int AT_THREADS = AT_WARPS * 32;

struct AtParams {
    const float *q;
    const __half *k, *v;
    unsigned long long seq_stride;
    const unsigned *lengths, *request;
    unsigned length, heads, kv_heads, capacity, splits;
    unsigned queries;  // query rows per KV sequence (speculative verification: the draft tokens)
    float scale;
    float *out;
    float *partials;
    unsigned *counters;
};

template <int HD, int G>
__global__ void __launch_bounds__(AT_THREADS) attention_kernel(const AtParams p)
{
    constexpr int DPL = HD / 32;  // output dims per lane
    __shared__ __align__(16) float qs[G][HD];
    __shared__ __align__(16) float pbuf[AT_WARPS][32][G];
    __shared__ float wm[AT_WARPS][G], wl[AT_WARPS][G];
    __shared__ __align__(16) float wo[AT_WARPS][G][HD];
    __shared__ unsigned last_flag;

    const unsigned sp = blockIdx.x, kh = blockIdx.y, seq = blockIdx.z;
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    pdl_launch_dependents();
    pdl_wait();
    // row `seq` is query j = seq % queries of KV sequence seq / queries; with
    // several queries, query j sits queries-1-j positions before the last one
    // and attends only up to itself (causal within the draft)
    const unsigned kvs = seq / p.queries, j = seq - kvs * p.queries;
    unsigned L = p.length;
    if (p.lengths) L = p.lengths[kvs];
    else if (p.request) L = p.request[1] + 1;
    if (p.queries > 1) L = L > p.queries - 1 - j ? L - (p.queries - 1 - j) : 1u;
    const unsigned chunk = (L + p.splits - 1) / p.splits;
    const unsigned c0 = min(L, sp * chunk), c1 = min(L, c0 + chunk);

    const __half *K = p.k + kvs * p.seq_stride + (size_t)kh * p.capacity * HD;
    const __half *V = p.v + kvs * p.seq_stride + (size_t)kh * p.capacity * HD;
    const float *qg = p.q + ((size_t)seq * p.heads + (size_t)kh * G) * HD;
    for (unsigned i = threadIdx.x; i < G * HD; i += AT_THREADS) qs[i / HD][i % HD] = qg[i];
    __syncthreads();

    float m[G], l[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[g][e] = 0.f;
    }

    for (unsigned base = c0 + warp * 32; base < c1; base += AT_WARPS * 32) {
        const unsigned t = base + lane;
        const bool valid = t < c1;
        float s[G];
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.f;
        if (valid) {
            // the whole K row in two batches of loads, then the dot products
            const uint4 *krow = reinterpret_cast<const uint4 *>(K + (size_t)t * HD);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint4 kk[HD / 16];
#pragma unroll
                for (int c = 0; c < HD / 16; ++c) kk[c] = __ldg(krow + half * (HD / 16) + c);
#pragma unroll
                for (int c = 0; c < HD / 16; ++c) {
                    const __half2 *h2 = reinterpret_cast<const __half2 *>(&kk[c]);
                    float kf[8];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f2 = __half22float2(h2[e]);
                        kf[2 * e] = f2.x; kf[2 * e + 1] = f2.y;
                    }
                    const int col = 8 * (half * (HD / 16) + c);
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float4 qa = *reinterpret_cast<const float4 *>(&qs[g][col]);
                        const float4 qb = *reinterpret_cast<const float4 *>(&qs[g][col + 4]);
                        float acc = s[g];
                        acc = fmaf(qa.x, kf[0], acc); acc = fmaf(qa.y, kf[1], acc);
                        acc = fmaf(qa.z, kf[2], acc); acc = fmaf(qa.w, kf[3], acc);
                        acc = fmaf(qb.x, kf[4], acc); acc = fmaf(qb.y, kf[5], acc);
                        acc = fmaf(qb.z, kf[6], acc); acc = fmaf(qb.w, kf[7], acc);
                        s[g] = acc;
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float sv = valid ? s[g] * p.scale : -INFINITY;
            const float mt = warp_max(sv);
            const float mn = fmaxf(m[g], mt);
            const float alpha = mn == -INFINITY ? 1.f : expf(m[g] - mn);
            const float pv = valid ? expf(sv - mn) : 0.f;
            l[g] = l[g] * alpha + warp_sum(pv);
            m[g] = mn;
#pragma unroll
            for (int e = 0; e < DPL; ++e) o[g][e] *= alpha;
            pbuf[warp][lane][g] = pv;
        }
        __syncwarp();
        const unsigned n = min(32u, c1 - base);
        // V rows of the tile: all loads first (8 at a time), then the FMAs
#pragma unroll
        for (unsigned j0 = 0; j0 < 32; j0 += 8) {
            if (j0 >= n) break;
            float vf[8][DPL];
#pragma unroll
            for (unsigned jj = 0; jj < 8; ++jj) {
                const unsigned j = j0 + jj < n ? j0 + jj : n - 1;
                const __half *vrow = V + (size_t)(base + j) * HD + lane * DPL;
                if constexpr (DPL == 4) {
                    uint2 vv = __ldg(reinterpret_cast<const uint2 *>(vrow));
                    const float2 a = __half22float2(*reinterpret_cast<__half2 *>(&vv.x));
                    const float2 b = __half22float2(*reinterpret_cast<__half2 *>(&vv.y));
                    vf[jj][0] = a.x; vf[jj][1] = a.y; vf[jj][2] = b.x; vf[jj][3] = b.y;
                } else {
                    unsigned vv = __ldg(reinterpret_cast<const unsigned *>(vrow));
                    const float2 a = __half22float2(*reinterpret_cast<__half2 *>(&vv));
                    vf[jj][0] = a.x; vf[jj][1] = a.y;
                }
            }
#pragma unroll
            for (unsigned jj = 0; jj < 8; ++jj) {
                if (j0 + jj >= n) break;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float pj = pbuf[warp][j0 + jj][g];
#pragma unroll
                    for (int e = 0; e < DPL; ++e) o[g][e] = fmaf(pj, vf[jj][e], o[g][e]);
                }
            }
        }
        __syncwarp();
    }

    // merge the warps of this CTA
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (lane == 0) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
#pragma unroll
        for (int e = 0; e < DPL; ++e) wo[warp][g][lane * DPL + e] = o[g][e];
    }
    __syncthreads();
    const size_t pair = (size_t)seq * p.kv_heads + kh;
    float *slot = p.partials + (pair * p.splits + sp) * (size_t)(G * (HD + 2));
    for (unsigned i = threadIdx.x; i < G * HD; i += AT_THREADS) {
        const unsigned g = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int w = 0; w < AT_WARPS; ++w) M = fmaxf(M, wm[w][g]);
        float acc = 0.f, den = 0.f;
        for (int w = 0; w < AT_WARPS; ++w) {
            const float f = wm[w][g] == -INFINITY ? 0.f : expf(wm[w][g] - M);
            acc += wo[w][g][d] * f;
            den += wl[w][g] * f;
        }
        slot[g * (HD + 2) + d] = acc;
        if (d == 0) { slot[g * (HD + 2) + HD] = M; slot[g * (HD + 2) + HD + 1] = den; }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned old = atomicAdd(p.counters + pair, 1u);
        last_flag = old == p.splits - 1;
    }
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    const float *all = p.partials + pair * p.splits * (size_t)(G * (HD + 2));
    for (unsigned i = threadIdx.x; i < G * HD; i += AT_THREADS) {
        const unsigned g = i / HD, d = i % HD;
        float M = -INFINITY;
        for (unsigned s2 = 0; s2 < p.splits; ++s2) M = fmaxf(M, __ldcg(all + s2 * (G * (HD + 2)) + g * (HD + 2) + HD));
        float acc = 0.f, den = 0.f;
        for (unsigned s2 = 0; s2 < p.splits; ++s2) {
            const float *sl = all + s2 * (G * (HD + 2)) + g * (HD + 2);
            const float ms = __ldcg(sl + HD);
            const float f = ms == -INFINITY ? 0.f : expf(ms - M);
            acc += __ldcg(sl + d) * f;
            den += __ldcg(sl + HD + 1) * f;
        }
        p.out[((size_t)seq * p.heads + (size_t)kh * G + g) * HD + d] = acc / den;
    }
    if (threadIdx.x == 0) p.counters[pair] = 0;
}

size_t attention_workspace_bytes(const AttentionLaunch &L)
{
    const unsigned G = L.heads / L.kv_heads;
    size_t pairs = (size_t)L.nseq * L.queries * L.kv_heads;
    size_t partial = pairs * L.splits * G * (L.head_dim + 2) * sizeof(float);
    return (partial + 255) / 256 * 256 + (pairs * sizeof(unsigned) + 255) / 256 * 256;
}

template <int HD, int G>
static cudaError_t launch_at(const AtParams &p, dim3 grid, cudaStream_t s, bool pdl)
{
    cudaFuncSetAttribute(attention_kernel<HD, G>, cudaFuncAttributePreferredSharedMemoryCarveout,
                         cudaSharedmemCarveoutMaxShared);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(AT_THREADS);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attention_kernel<HD, G>, p);
}

int launch_attention(const AttentionLaunch &L, cudaStream_t s)
{
    if (!L.q || !L.k || !L.v || !L.out || L.kv_heads == 0 || L.heads % L.kv_heads || L.splits == 0 ||
        L.capacity == 0 || L.nseq == 0 || L.queries == 0 || L.queries > L.capacity ||
        (size_t)L.nseq * L.queries > 65535)
        return -1;
    const unsigned G = L.heads / L.kv_heads;
    if (!L.workspace || L.workspace_bytes < attention_workspace_bytes(L)) return -1;
    AtParams p;
    p.q = L.q; p.k = L.k; p.v = L.v;
    p.seq_stride = L.seq_stride;
    p.lengths = L.lengths; p.request = L.request; p.length = L.length;
    p.heads = L.heads; p.kv_heads = L.kv_heads; p.capacity = L.capacity; p.splits = L.splits;
    p.queries = L.queries;
    p.scale = L.scale;
    p.out = L.out;
    const unsigned rows = L.nseq * L.queries;  // query rows (grid z)
    size_t pairs = (size_t)rows * L.kv_heads;
    size_t partial = (pairs * L.splits * G * (L.head_dim + 2) * sizeof(float) + 255) / 256 * 256;
    p.partials = (float *)L.workspace;
    p.counters = (unsigned *)((unsigned char *)L.workspace + partial);
    dim3 grid(L.splits, L.kv_heads, rows);
    cudaError_t e = cudaErrorInvalidValue;
#define FYB_AT(HDV, GV) if (L.head_dim == HDV && G == GV) e = launch_at<HDV, GV>(p, grid, s, L.pdl);
    FYB_AT(128, 1) FYB_AT(128, 2) FYB_AT(128, 4) FYB_AT(128, 8)
    FYB_AT(64, 1) FYB_AT(64, 2) FYB_AT(64, 4) FYB_AT(64, 8)
#undef FYB_AT
    if (e == cudaErrorInvalidValue) return -1;
    return e == cudaSuccess ? 0 : -2;
}

}  // namespace fyb

// ---------------------------------------------------------------------------
// fyb_attention_decode_static: the same kernel with its scratch (split
// partials + per-(sequence, KV head) counters) in a fixed device array of
// this module instead of a caller workspace. It is for callers that cannot
// allocate device memory at the point of the call: a host hook that runs
// under a device-memory budget it has already spent (the engine caps the
// provider with NYA_CUDA_MEMORY_MIB), or a caller on a latency-critical path
// that must not pay the implicit device synchronization of cudaFree. The
// entry point itself allocates nothing: no cudaMalloc, no cudaFree, no
// library allocator.
//
// Set-up: the first call on a device (with that device current) looks up the
// array's device address with cudaGetSymbolAddress and keeps it; that first
// call should therefore come before any stream capture on the device. Every
// call clears the counters it will use (the only part that must start at
// zero) with cudaMemsetAsync on the caller's stream, then launches.
// Problems whose scratch exceeds FYB_ATTENTION_STATIC_SCRATCH_BYTES are
// rejected with -3 before anything is launched. There is one array per
// device, so calls that overlap in time on the same device (other streams or
// threads) race on it; callers must serialize them.
namespace {

constexpr size_t kStaticScratchBytes = 4u << 20;
static_assert(kStaticScratchBytes == FYB_ATTENTION_STATIC_SCRATCH_BYTES, "header and module disagree");
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_attention_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void *g_scratch_ptr[kMaxDevices];

// Device address of this device's array, looked up once per device.
void *static_scratch(int device)
{
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_ptr[device]) {
        void *ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_attention_scratch) != cudaSuccess || !ptr) return nullptr;
        g_scratch_ptr[device] = ptr;
    }
    return g_scratch_ptr[device];
}

}  // namespace

extern "C" int fyb_attention_decode_static(const float *q, const void *k, const void *v, size_t seq_stride,
    const unsigned *lengths, unsigned nseq, unsigned heads, unsigned kv_heads, unsigned head_dim, unsigned capacity,
    float scale, float *out, unsigned splits, void *stream)
{
    using namespace fyb;
    AttentionLaunch L;
    L.q = q; L.k = (const __half *)k; L.v = (const __half *)v;
    L.seq_stride = seq_stride; L.lengths = lengths;
    L.nseq = nseq; L.heads = heads; L.kv_heads = kv_heads; L.head_dim = head_dim; L.capacity = capacity;
    L.scale = scale; L.out = out; L.splits = splits ? splits : 8;
    if (!lengths || !kv_heads || !nseq || heads % kv_heads) return -1;
    const size_t need = attention_workspace_bytes(L);
    if (need > kStaticScratchBytes) return -3;
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return -2;
    unsigned char *scratch = (unsigned char *)static_scratch(device);
    if (!scratch) return -2;
    // counters follow the 256-byte-rounded partials (attention_workspace_bytes' layout)
    const unsigned G = heads / kv_heads;
    const size_t pairs = (size_t)nseq * kv_heads;
    const size_t counters = (pairs * L.splits * G * (head_dim + 2) * sizeof(float) + 255) / 256 * 256;
    if (cudaMemsetAsync(scratch + counters, 0, pairs * sizeof(unsigned), (cudaStream_t)stream) != cudaSuccess)
        return -2;
    L.workspace = scratch;
    L.workspace_bytes = need;
    return launch_attention(L, (cudaStream_t)stream);
}
