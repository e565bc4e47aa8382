// batch.cu - the elementwise kernels of a batched decode step: B sequences
// (up to 16), each at its own position with its own KV cache, decoded
// together so that every projection is one small-batch GEMM that reads each
// weight once for all B rows (the engine's per-token step,
// CUDA/resident.inc:470-552, and its CPU definition,
// backend/core/llm_cpu.c:424-578, applied to every sequence of the batch).
//
// The projections run on the fused, repacked weights of a resident plan:
// the QKV GEMM returns its rows in the REPACK_QKV order (unit row r of tile
// t is source row 16t + 2r for r < 8, 16t + 2(r - 8) + 1 above: a RoPE pair
// sits in rows j and j + 8 of a tile) and the gate/up GEMM in the
// REPACK_GATEUP order (rows 0..7 of tile t are gate rows 8t..8t+7, rows
// 8..15 the up rows). The kernels here undo those orders while they apply
// RoPE, write the fp16 KV rows and form SwiGLU.
#include "common.cuh"
#include "kernels.h"
#include <cmath>

namespace fyb {

// x[b] += delta[b] (when delta is given, written back), then
// xn[b] = x[b] * (1 / sqrt(mean(x^2) + eps)) * w with the sum of squares in
// double (llm_cpu.c:83-103). One CTA of 1024 threads per sequence, four
// consecutive values per thread and pass (d a multiple of 4).
constexpr unsigned BT_NORM_THREADS = 1024;
__global__ void __launch_bounds__(BT_NORM_THREADS) bt_add_norm_kernel(float *x, const float *delta, const float *w,
    float *xn, unsigned d, float eps)
{
    const unsigned b = blockIdx.x;
    float4 *xr = reinterpret_cast<float4 *>(x + (size_t)b * d);
    const float4 *dr = delta ? reinterpret_cast<const float4 *>(delta + (size_t)b * d) : nullptr;
    __shared__ double part[BT_NORM_THREADS / 32];
    __shared__ float scale_s;
    double ss = 0.0;
    for (unsigned i = threadIdx.x; i < d / 4; i += BT_NORM_THREADS) {
        float4 v = xr[i];
        if (dr) {
            const float4 e = dr[i];
            v.x = __fadd_rn(v.x, e.x); v.y = __fadd_rn(v.y, e.y); v.z = __fadd_rn(v.z, e.z); v.w = __fadd_rn(v.w, e.w);
            xr[i] = v;
        }
        ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = part[threadIdx.x];
#pragma unroll
        for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) scale_s = (float)(1.0 / sqrt(t / (double)d + (double)eps));
    }
    __syncthreads();
    const float scale = scale_s;
    float4 *out = reinterpret_cast<float4 *>(xn + (size_t)b * d);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    for (unsigned i = threadIdx.x; i < d / 4; i += BT_NORM_THREADS) {
        const float4 v = xr[i], g = w ? w4[i] : make_float4(1.f, 1.f, 1.f, 1.f);
        out[i] = make_float4(__fmul_rn(__fmul_rn(v.x, scale), g.x), __fmul_rn(__fmul_rn(v.y, scale), g.y),
                             __fmul_rn(__fmul_rn(v.z, scale), g.z), __fmul_rn(__fmul_rn(v.w, scale), g.w));
    }
}

// RoPE and KV append from the fused QKV rows y[b][qkv_rows]: thread (b, t, j)
// owns rows j and j + 8 of tile t, the pair (2i, 2i + 1) of one head
// (llm_cpu.c:298-327; q and K rotated, V copied). q goes to q[b][H * hd] in
// natural order; K and V are rounded to fp16 into sequence b's cache row
// positions[b] (per layer: [seq][kv head][capacity][hd]). Row b writes the
// cache of sequence b / slot_div: slot_div 1 for a batch of sequences, the
// row count when the rows are consecutive positions of one sequence.
__global__ void bt_rope_kv_kernel(const float *y, unsigned qkv_rows, unsigned H, unsigned Hkv, unsigned hd,
    const unsigned *positions, const float *rope_cos, const float *rope_sin, float *q, __half *kc, __half *vc,
    unsigned capacity, unsigned nseq, unsigned slot_div)
{
    const unsigned tiles = qkv_rows / 16, tq = H * hd / 16, tk = Hkv * hd / 16;
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nseq * tiles * 8) return;
    const unsigned b = i / (tiles * 8), t = (i / 8) % tiles, j = i % 8;
    const float *yr = y + (size_t)b * qkv_rows;
    const float yA = yr[16 * t + j], yB = yr[16 * t + j + 8];
    const unsigned seg = t < tq ? 0 : t < tq + tk ? 1 : 2;
    const unsigned lt = t - (seg == 0 ? 0 : seg == 1 ? tq : tq + tk);
    const unsigned rowA = lt * 16 + 2 * j, pair = (rowA % hd) >> 1;
    const unsigned pos = positions[b];
    float a = yA, c2 = yB;
    if (seg <= 1) {
        const float c = rope_cos[(size_t)pos * (hd >> 1) + pair];
        const float s = rope_sin[(size_t)pos * (hd >> 1) + pair];
        a = __fsub_rn(__fmul_rn(yA, c), __fmul_rn(yB, s));
        c2 = __fadd_rn(__fmul_rn(yA, s), __fmul_rn(yB, c));
    }
    if (seg == 0) {
        q[(size_t)b * H * hd + rowA] = a;
        q[(size_t)b * H * hd + rowA + 1] = c2;
        return;
    }
    const unsigned kvh = rowA / hd, dd = rowA % hd;
    __half *dst = (seg == 1 ? kc : vc) + (((size_t)(b / slot_div) * Hkv + kvh) * capacity + pos) * hd + dd;
    *reinterpret_cast<__half2 *>(dst) = __halves2half2(__float2half_rn(a), __float2half_rn(c2));
}

// h[b][8t + j] = gate / (1 + expf(-gate)) * up (llm_cpu.c:336-342) from the
// fused gate/up rows y[b][2 ffn].
__global__ void bt_swiglu_kernel(const float *y, unsigned ffn, float *h, unsigned nseq)
{
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nseq * ffn) return;
    const unsigned b = i / ffn, f = i % ffn, t = f / 8, j = f % 8;
    const float *yr = y + (size_t)b * 2 * ffn;
    const float g = yr[16 * t + j], u = yr[16 * t + 8 + j];
    h[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// Greedy argmax of every sequence's logits (the first index of the maximum,
// llm_cpu.c:896-905). With advance set, the result becomes the sequence's
// next token at the next position and is logged at step request[2B].
// Layout of req: [B] tokens | [B] positions | [B] attended lengths | step.
__global__ void __launch_bounds__(1024) bt_argmax_kernel(const float *logits, unsigned V, unsigned *req, unsigned nseq,
    unsigned *tokens_out, unsigned *log, int advance, unsigned *error)
{
    const unsigned b = blockIdx.x;
    const float *lg = logits + (size_t)b * V;
    unsigned long long best = 0ull;
    bool bad = false;
    for (unsigned i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = lg[i];
        bad = bad || !isfinite(v);
        const unsigned long long k = ((unsigned long long)float_order_key(v) << 32) | (0xffffffffu - i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    __shared__ unsigned long long part[32];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = best;
    if (bad && error) atomicCAS(error, 0u, (unsigned)ERR_NONFINITE);
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (unsigned k = 0; k < blockDim.x / 32; ++k) best = part[k] > best ? part[k] : best;
    const unsigned tok = 0xffffffffu - (unsigned)(best & 0xffffffffu);
    tokens_out[b] = tok;
    if (advance) {
        const unsigned step = req[3 * nseq];
        log[(size_t)step * nseq + b] = tok;
        req[b] = tok;
        req[nseq + b] += 1;
        req[2 * nseq + b] += 1;
    }
}

// The last CTA of an advancing argmax bumps the step counter: a separate
// one-thread kernel keeps the argmax CTAs independent.
__global__ void bt_step_kernel(unsigned *req, unsigned nseq) { req[3 * nseq] += 1; }

// Tokens and positions of a step from the host (passed by value).
__global__ void bt_set_kernel(BatchRequest r, unsigned *req, unsigned nseq)
{
    const unsigned b = threadIdx.x;
    if (b < nseq) {
        req[b] = r.token[b];
        req[nseq + b] = r.position[b];
        req[2 * nseq + b] = r.position[b] + 1;
    }
    if (b == 0) req[3 * nseq] = 0;
}

int launch_bt_add_norm(float *x, const float *delta, const float *w, float *xn, unsigned d, float eps, unsigned nseq,
    cudaStream_t s)
{
    if (d % 4) return -1;
    bt_add_norm_kernel<<<nseq, BT_NORM_THREADS, 0, s>>>(x, delta, w, xn, d, eps);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int launch_bt_rope_kv(const float *y, unsigned qkv_rows, unsigned H, unsigned Hkv, unsigned hd,
    const unsigned *positions, const float *rope_cos, const float *rope_sin, float *q, __half *kc, __half *vc,
    unsigned capacity, unsigned nseq, unsigned slot_div, cudaStream_t s)
{
    if (qkv_rows % 16 || hd % 16 || slot_div == 0) return -1;
    const unsigned n = nseq * (qkv_rows / 16) * 8;
    bt_rope_kv_kernel<<<(n + 255) / 256, 256, 0, s>>>(y, qkv_rows, H, Hkv, hd, positions, rope_cos, rope_sin, q, kc,
                                                        vc, capacity, nseq, slot_div);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int launch_bt_swiglu(const float *y, unsigned ffn, float *h, unsigned nseq, cudaStream_t s)
{
    if (ffn % 8) return -1;
    const unsigned n = nseq * ffn;
    bt_swiglu_kernel<<<(n + 255) / 256, 256, 0, s>>>(y, ffn, h, nseq);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int launch_bt_argmax(const float *logits, unsigned V, unsigned *req, unsigned nseq, unsigned *tokens_out, unsigned *log,
    bool advance, unsigned *error, cudaStream_t s)
{
    bt_argmax_kernel<<<nseq, 1024, 0, s>>>(logits, V, req, nseq, tokens_out, log, advance ? 1 : 0, error);
    if (advance && cudaGetLastError() == cudaSuccess) bt_step_kernel<<<1, 1, 0, s>>>(req, nseq);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int launch_bt_set(const BatchRequest &r, unsigned *req, unsigned nseq, cudaStream_t s)
{
    if (nseq > BATCH_MAX) return -1;
    bt_set_kernel<<<1, 32, 0, s>>>(r, req, nseq);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace fyb
