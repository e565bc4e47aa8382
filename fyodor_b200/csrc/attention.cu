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
// The kernel below is the per-row form (G = 1 decode, drafts of more than
// 64 query rows per KV head); the tensor-core kernel further down takes the
// rest. Inside a CTA (two warps: with 32 KB of stages per warp, three CTAs
// share an SM, which measured faster than one CTA of four warps or six of one) each
// warp takes tiles of 32 positions (warp w: tiles w, w + 2, ...),
// double-buffered in shared memory: while it computes one tile, the
// K and V rows of its next tile stream in through cp.async (16-byte chunks,
// coalesced). Lane j computes the full dot products of position j with all G
// query heads (K row read from its swizzled stage, query broadcast from
// shared memory), the warp updates the online softmax, then the lanes switch
// to DPL output dimensions each and accumulate p * v over the tile.
#include "common.cuh"
#include "fyodor_b200.h"
#include "kernels.h"
#include <cfloat>
#include <mutex>

namespace fyb {

constexpr int AT_WARPS = 2;
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

constexpr int AT_TILE = 32;    // positions per warp tile
constexpr int AT_STAGES = 2;   // tiles per warp in shared memory (one streams in while one is used)

FYB_DEV void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(dst)), "l"(src) : "memory");
}
FYB_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
FYB_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// Copy the K and V rows of positions [base, min(base + AT_TILE, end)) into a
// warp's stage: 16-byte chunks, consecutive lanes on consecutive chunks
// (coalesced). K chunk c of row r goes to chunk c ^ (r % (HD/8)) of its row,
// so the lane-per-row dot products read shared memory without bank
// conflicts; V keeps its layout (lanes read along a row).
template <int HD>
FYB_DEV void at_stage_tile(__half *Ks, __half *Vs, const __half *K, const __half *V, unsigned base, unsigned end,
    unsigned lane)
{
    constexpr int CH = HD / 8;  // chunks per row
    const unsigned rows = end > base ? min((unsigned)AT_TILE, end - base) : 0u;
#pragma unroll 4
    for (unsigned q = lane; q < rows * CH; q += 32) {
        const unsigned r = q / CH, c = q % CH;
        cp_async16(Ks + r * HD + ((c ^ (r % CH)) * 8), K + (size_t)(base + r) * HD + c * 8);
        cp_async16(Vs + r * HD + c * 8, V + (size_t)(base + r) * HD + c * 8);
    }
}

// Dynamic shared memory of attention_kernel<HD, *>: AT_STAGES stages of K
// and V tiles per warp.
constexpr size_t at_stage_bytes(int hd) { return (size_t)AT_WARPS * AT_STAGES * 2 * AT_TILE * hd * sizeof(__half); }

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

    // this warp's stages of (K tile, V tile): AT_TILE positions each
    extern __shared__ __align__(128) unsigned char at_stage[];
    __half *stage = reinterpret_cast<__half *>(at_stage) + (size_t)warp * AT_STAGES * 2 * AT_TILE * HD;
    const unsigned ntiles = c1 > c0 ? (c1 - c0 + AT_TILE - 1) / AT_TILE : 0;
    auto issue = [&](unsigned tile) {  // tile-th tile of this warp: positions c0 + (warp + AT_WARPS tile) * AT_TILE ...
        const unsigned base = c0 + (warp + AT_WARPS * tile) * AT_TILE;
        __half *Ks = stage + (size_t)(tile % AT_STAGES) * 2 * AT_TILE * HD, *Vs = Ks + AT_TILE * HD;
        at_stage_tile<HD>(Ks, Vs, K, V, base, c1, lane);
        cp_async_commit();
    };
    const unsigned mine = ntiles > warp ? (ntiles - warp + AT_WARPS - 1) / AT_WARPS : 0;  // tiles of this warp
    for (unsigned t0 = 0; t0 + 1 < AT_STAGES && t0 < mine; ++t0) issue(t0);
    for (unsigned it = 0; it < mine; ++it) {
        // the stage of tile it + AT_STAGES - 1 held tile it - 1, done with at the end of the last pass
        if (it + AT_STAGES - 1 < mine) issue(it + AT_STAGES - 1);
        const unsigned ahead = min(mine - 1 - it, (unsigned)AT_STAGES - 1);  // groups that may stay in flight
        if (ahead >= 2) cp_async_wait<2>();
        else if (ahead == 1) cp_async_wait<1>();
        else cp_async_wait<0>();
        __syncwarp();
        const unsigned base = c0 + (warp + AT_WARPS * it) * AT_TILE;
        const __half *Ks = stage + (size_t)(it % AT_STAGES) * 2 * AT_TILE * HD, *Vs = Ks + AT_TILE * HD;
        const unsigned t = base + lane;
        const bool valid = t < c1;
        float s[G];
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.f;
        if (valid) {
            // row `lane` of the K tile, chunk c stored at chunk c ^ (lane % CH) (no bank conflicts)
            constexpr int CH = HD / 8;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const uint4 kk = *reinterpret_cast<const uint4 *>(Ks + lane * HD + ((c ^ (lane % CH)) * 8));
                const __half2 *h2 = reinterpret_cast<const __half2 *>(&kk);
                float kf[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f2 = __half22float2(h2[e]);
                    kf[2 * e] = f2.x; kf[2 * e + 1] = f2.y;
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float4 qa = *reinterpret_cast<const float4 *>(&qs[g][8 * c]);
                    const float4 qb = *reinterpret_cast<const float4 *>(&qs[g][8 * c + 4]);
                    float acc = s[g];
                    acc = fmaf(qa.x, kf[0], acc); acc = fmaf(qa.y, kf[1], acc);
                    acc = fmaf(qa.z, kf[2], acc); acc = fmaf(qa.w, kf[3], acc);
                    acc = fmaf(qb.x, kf[4], acc); acc = fmaf(qb.y, kf[5], acc);
                    acc = fmaf(qb.z, kf[6], acc); acc = fmaf(qb.w, kf[7], acc);
                    s[g] = acc;
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
        const unsigned n = min((unsigned)AT_TILE, c1 - base);
        // lanes own DPL output dimensions; V rows are read straight from the stage
        for (unsigned j = 0; j < n; ++j) {
            const __half *vrow = Vs + j * HD + lane * DPL;
            float vf[DPL];
            if constexpr (DPL == 4) {
                const uint2 vv = *reinterpret_cast<const uint2 *>(vrow);
                const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&vv.x));
                const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&vv.y));
                vf[0] = a.x; vf[1] = a.y; vf[2] = b.x; vf[3] = b.y;
            } else {
                const unsigned vv = *reinterpret_cast<const unsigned *>(vrow);
                const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&vv));
                vf[0] = a.x; vf[1] = a.y;
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float pj = pbuf[warp][j][g];
#pragma unroll
                for (int e = 0; e < DPL; ++e) o[g][e] = fmaf(pj, vf[e], o[g][e]);
            }
        }
        __syncwarp();  // the stage and pbuf are reused
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

// ---------------------------------------------------------------------------
// Decode and speculative verification on tensor cores (every shape with
// 2 <= queries x G <= 64; the kernel above keeps G = 1 decode and larger
// drafts). One CTA per (partition, KV head, KV sequence) takes all
// M = queries x G query rows of that KV head (row r = j * G + g: draft query
// j, head g of the group), so each K/V tile crosses HBM once for all of them
// (the per-row kernel above reads it once per row). Warps (r, h): row group
// r owns rows 16r..16r+15, half h the positions 16h..16h+15 of every
// 32-position tile; the two halves of a row group merge their softmax
// states at the end. Tiles are staged in shared memory through a three-stage
// cp.async ring shared by all warps:
//   S = Q K^T   (mma.sync m16n8k16, fp16 operands, fp32 accumulation; the
//                fp32 query is split into q_hi = fp16(q) and
//                q_lo = fp16(q - q_hi), two MMAs, so the products keep about
//                22 bits of the query)
//   online softmax per row (rows of a thread: gid and gid + 8 of the
//                fragment; row max / sum over the quad with shuffles)
//   O += P V    (P split into fp16 hi + lo the same way; V through ldmatrix.trans)
// Causality inside the draft: row j attends positions [0, L - (Q-1-j)).
// Tiles in shared memory are XOR-swizzled in 16-byte chunks (chunk c of row
// r at c ^ (r % 8)), so every ldmatrix reads eight distinct bank groups.
// The partials go to the same slots as the per-row kernel's and the last CTA
// of a (KV sequence, KV head) merges them in partition order.
constexpr int VT_TILE = 32;    // positions per tile
constexpr int VT_STAGES = 2;  // measured: 494 us for C4 decode against 605 with three (more CTAs per SM)
constexpr unsigned VT_MAX_ROWS = 64;  // queries x G handled by this kernel

// Dynamic shared memory: the query rows (hi, lo) and, in the same region
// after the last tile, the stages or the half-merge area (per thread of a
// row group: HD / 2 output values, two maxima, two sums), whichever is larger.
template <int HD>
constexpr size_t vt_stage_area(int rw)
{
    return (size_t)VT_STAGES * 2 * VT_TILE * HD * sizeof(__half) > (size_t)rw * 32 * (HD / 2 + 4) * sizeof(float)
               ? (size_t)VT_STAGES * 2 * VT_TILE * HD * sizeof(__half)
               : (size_t)rw * 32 * (HD / 2 + 4) * sizeof(float);
}
template <int HD>
constexpr size_t vt_smem_bytes(int rw)
{
    return (size_t)rw * 16 * HD * 2 * sizeof(__half) + vt_stage_area<HD>(rw);
}

template <int HD>
FYB_DEV unsigned vt_swz(unsigned r, unsigned d)  // half index of element (r, d), d % 8 == 0 for chunk starts
{
    return r * HD + ((((d >> 3) ^ (r & 7))) << 3) + (d & 7);
}

FYB_DEV void ldmatrix_x4_trans(unsigned (&r)[4], const void *p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}

// D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col)
FYB_DEV void mma_f16_k16(float (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

FYB_DEV void split_pack(float x0, float x1, unsigned &hi, unsigned &lo)
{
    const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
    const __half l0 = __float2half_rn(x0 - __half2float(h0)), l1 = __float2half_rn(x1 - __half2float(h1));
    const __half2 H = __halves2half2(h0, h1), Lo = __halves2half2(l0, l1);
    hi = *reinterpret_cast<const unsigned *>(&H);
    lo = *reinterpret_cast<const unsigned *>(&Lo);
}

// K and V rows of positions [base, base + VT_TILE) into a stage (rows at or
// past `end` are zero, so masked positions multiply zeros in P V).
template <int HD, int NT>
FYB_DEV void vt_stage_tile(__half *Ks, __half *Vs, const __half *K, const __half *V, unsigned base, unsigned end)
{
    constexpr int CH = HD / 8;
    const unsigned rows = end > base ? min((unsigned)VT_TILE, end - base) : 0u;
    for (unsigned q = threadIdx.x; q < VT_TILE * CH; q += NT) {
        const unsigned r = q / CH, c = q % CH;
        __half *kd = Ks + vt_swz<HD>(r, c * 8), *vd = Vs + vt_swz<HD>(r, c * 8);
        if (r < rows) {
            cp_async16(kd, K + (size_t)(base + r) * HD + c * 8);
            cp_async16(vd, V + (size_t)(base + r) * HD + c * 8);
        } else {
            *reinterpret_cast<uint4 *>(kd) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4 *>(vd) = make_uint4(0, 0, 0, 0);
        }
    }
}

template <int HD, int RW>
__global__ void __launch_bounds__(RW * 64) verify_mma_kernel(const AtParams p)
{
    constexpr int NT = RW * 64, NB = HD / 8;  // threads; 8-wide dimension blocks of the output
    extern __shared__ __align__(128) unsigned char vt_smem[];
    __half *qh = reinterpret_cast<__half *>(vt_smem);
    __half *ql = qh + RW * 16 * HD;
    __half *stages = ql + RW * 16 * HD;
    __shared__ unsigned last_flag;

    const unsigned sp = blockIdx.x, kh = blockIdx.y, kvs = blockIdx.z;
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, tig = lane & 3;
    const unsigned rw = warp % RW, ph = warp / RW;  // row group; half of each tile's positions
    const unsigned G = p.heads / p.kv_heads, Q = p.queries, M = G * Q;

    pdl_launch_dependents();
    pdl_wait();
    unsigned L = p.length;
    if (p.lengths) L = p.lengths[kvs];
    else if (p.request) L = p.request[1] + 1;
    const unsigned chunk = (L + p.splits - 1) / p.splits;
    const unsigned c0 = min(L, sp * chunk), c1 = min(L, c0 + chunk);

    const __half *K = p.k + kvs * p.seq_stride + (size_t)kh * p.capacity * HD;
    const __half *V = p.v + kvs * p.seq_stride + (size_t)kh * p.capacity * HD;
    const unsigned ntiles = c1 > c0 ? (c1 - c0 + VT_TILE - 1) / VT_TILE : 0;
    auto stage = [&](unsigned t) { return stages + (size_t)(t % VT_STAGES) * 2 * VT_TILE * HD; };
    auto issue = [&](unsigned t) {
        __half *Ks = stage(t);
        vt_stage_tile<HD, NT>(Ks, Ks + VT_TILE * HD, K, V, c0 + t * VT_TILE, c1);
        cp_async_commit();
    };
    for (unsigned t = 0; t + 1 < VT_STAGES && t < ntiles; ++t) issue(t);

    // query rows as fp16 hi + lo (rows past M are zero)
    for (unsigned i = threadIdx.x; i < RW * 16 * HD; i += NT) {
        const unsigned r = i / HD, d = i % HD;
        float x = 0.f;
        if (r < M) {
            const unsigned j = r / G, g = r - j * G;
            x = p.q[(((size_t)kvs * Q + j) * p.heads + (size_t)kh * G + g) * HD + d];
        }
        const __half h = __float2half_rn(x);
        qh[vt_swz<HD>(r, d)] = h;
        ql[vt_swz<HD>(r, d)] = __float2half_rn(x - __half2float(h));
    }

    // the two rows of this thread and the positions they attend
    const unsigned rA = rw * 16 + gid, rB = rA + 8;
    auto row_end = [&](unsigned r) -> unsigned {
        if (r >= M) return 0u;
        const unsigned back = Q - 1 - r / G;
        return min(c1, L > back ? L - back : 1u);
    };
    const unsigned eA = row_end(rA), eB = row_end(rB);
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
    float o[NB][4];
#pragma unroll
    for (int b = 0; b < NB; ++b) o[b][0] = o[b][1] = o[b][2] = o[b][3] = 0.f;

    static_assert(VT_STAGES == 2 || VT_STAGES == 3, "the waits below cover two or three stages");
    for (unsigned it = 0; it < ntiles; ++it) {
        // tiles it + 1 .. it + VT_STAGES - 2 (those issued) may stay in flight
        if (VT_STAGES == 3 && it + 1 < ntiles) cp_async_wait<1>();
        else cp_async_wait<0>();
        __syncthreads();  // tile `it` visible to all warps; the stage of tile it - 1 is free
        if (it + VT_STAGES - 1 < ntiles) issue(it + VT_STAGES - 1);
        const __half *Ks = stage(it), *Vs = Ks + VT_TILE * HD;
        const unsigned base = c0 + it * VT_TILE + 16 * ph;  // this warp's 16 positions

        // the q_hi and q_lo products accumulate separately (four independent
        // MMA chains instead of two), then add
        float s[2][4], sl[2][4];
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) s[n][i] = sl[n][i] = 0.f;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
            unsigned ah[4], al[4], b[4];
            const unsigned qr = rw * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), qc = ks * 16 + 8 * (lane >> 4);
            ldmatrix_x4(ah, qh + vt_swz<HD>(qr, qc));
            ldmatrix_x4(al, ql + vt_swz<HD>(qr, qc));
            const unsigned mi = lane >> 3;
            ldmatrix_x4(b, Ks + vt_swz<HD>(16 * ph + (lane & 7) + 8 * (mi >> 1), ks * 16 + 8 * (mi & 1)));
            mma_f16_k16(s[0], ah, b[0], b[1]);
            mma_f16_k16(s[1], ah, b[2], b[3]);
            mma_f16_k16(sl[0], al, b[0], b[1]);
            mma_f16_k16(sl[1], al, b[2], b[3]);
        }
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) s[n][i] += sl[n][i];
        // mask, scale, online softmax (rows A = gid, B = gid + 8)
        float tmA = -INFINITY, tmB = -INFINITY;
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const unsigned t = base + 8 * n + 2 * tig + e;
                s[n][e] = t < eA ? s[n][e] * p.scale : -INFINITY;
                s[n][2 + e] = t < eB ? s[n][2 + e] * p.scale : -INFINITY;
                tmA = fmaxf(tmA, s[n][e]);
                tmB = fmaxf(tmB, s[n][2 + e]);
            }
#pragma unroll
        for (int x = 1; x <= 2; x <<= 1) {
            tmA = fmaxf(tmA, __shfl_xor_sync(0xffffffffu, tmA, x));
            tmB = fmaxf(tmB, __shfl_xor_sync(0xffffffffu, tmB, x));
        }
        const float nA = fmaxf(mA, tmA), nB = fmaxf(mB, tmB);
        const float alA = nA == -INFINITY ? 1.f : expf(mA - nA), alB = nB == -INFINITY ? 1.f : expf(mB - nB);
        float sumA = 0.f, sumB = 0.f;
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                s[n][e] = s[n][e] == -INFINITY ? 0.f : expf(s[n][e] - nA);
                s[n][2 + e] = s[n][2 + e] == -INFINITY ? 0.f : expf(s[n][2 + e] - nB);
                sumA += s[n][e];
                sumB += s[n][2 + e];
            }
#pragma unroll
        for (int x = 1; x <= 2; x <<= 1) {
            sumA += __shfl_xor_sync(0xffffffffu, sumA, x);
            sumB += __shfl_xor_sync(0xffffffffu, sumB, x);
        }
        lA = lA * alA + sumA;
        lB = lB * alB + sumB;
        mA = nA;
        mB = nB;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            o[b][0] *= alA; o[b][1] *= alA;
            o[b][2] *= alB; o[b][3] *= alB;
        }
        // O += P V over this warp's 16 positions, P as the A operand straight
        // from the S fragments
        unsigned ph4[4], pl4[4];
        split_pack(s[0][0], s[0][1], ph4[0], pl4[0]);
        split_pack(s[0][2], s[0][3], ph4[1], pl4[1]);
        split_pack(s[1][0], s[1][1], ph4[2], pl4[2]);
        split_pack(s[1][2], s[1][3], ph4[3], pl4[3]);
#pragma unroll
        for (int d2 = 0; d2 < NB / 2; ++d2) {
            unsigned b[4];
            const unsigned mi = lane >> 3;
            ldmatrix_x4_trans(b, Vs + vt_swz<HD>(16 * ph + (lane & 7) + 8 * (mi & 1), 16 * d2 + 8 * (mi >> 1)));
            mma_f16_k16(o[2 * d2], ph4, b[0], b[1]);
            mma_f16_k16(o[2 * d2 + 1], ph4, b[2], b[3]);
            mma_f16_k16(o[2 * d2], pl4, b[0], b[1]);
            mma_f16_k16(o[2 * d2 + 1], pl4, b[2], b[3]);
        }
    }

    // the two position halves of each row group meet in shared memory (the
    // stages are free): half 1 leaves (m, l, o) in fragment order, half 0
    // rescales both to the common maximum and adds
    __syncthreads();
    float *xo = reinterpret_cast<float *>(stages) + ((size_t)rw * 32 + lane) * (NB * 4 + 4);
    if (ph == 1) {
#pragma unroll
        for (int b = 0; b < NB; ++b)
#pragma unroll
            for (int c = 0; c < 4; ++c) xo[b * 4 + c] = o[b][c];
        xo[NB * 4] = mA; xo[NB * 4 + 1] = mB; xo[NB * 4 + 2] = lA; xo[NB * 4 + 3] = lB;
    }
    __syncthreads();
    if (ph == 0) {
        const float m1A = xo[NB * 4], m1B = xo[NB * 4 + 1];
        const float MA = fmaxf(mA, m1A), MB = fmaxf(mB, m1B);
        const float f0A = mA == -INFINITY ? 0.f : expf(mA - MA), f1A = m1A == -INFINITY ? 0.f : expf(m1A - MA);
        const float f0B = mB == -INFINITY ? 0.f : expf(mB - MB), f1B = m1B == -INFINITY ? 0.f : expf(m1B - MB);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            o[b][0] = o[b][0] * f0A + xo[b * 4] * f1A;
            o[b][1] = o[b][1] * f0A + xo[b * 4 + 1] * f1A;
            o[b][2] = o[b][2] * f0B + xo[b * 4 + 2] * f1B;
            o[b][3] = o[b][3] * f0B + xo[b * 4 + 3] * f1B;
        }
        lA = lA * f0A + xo[NB * 4 + 2] * f1A;
        lB = lB * f0B + xo[NB * 4 + 3] * f1B;
        mA = MA;
        mB = MB;
        // partial slots {o[hd], m, l} of each row, the per-row kernel's layout
        auto slot_of = [&](unsigned r) {
            const unsigned j = r / G, g = r - j * G;
            const size_t pair = ((size_t)kvs * Q + j) * p.kv_heads + kh;
            return p.partials + (pair * p.splits + sp) * (size_t)(G * (HD + 2)) + (size_t)g * (HD + 2);
        };
        if (rA < M) {
            float *sl = slot_of(rA);
#pragma unroll
            for (int b = 0; b < NB; ++b) { sl[8 * b + 2 * tig] = o[b][0]; sl[8 * b + 2 * tig + 1] = o[b][1]; }
            if (tig == 0) { sl[HD] = mA; sl[HD + 1] = lA; }
        }
        if (rB < M) {
            float *sl = slot_of(rB);
#pragma unroll
            for (int b = 0; b < NB; ++b) { sl[8 * b + 2 * tig] = o[b][2]; sl[8 * b + 2 * tig + 1] = o[b][3]; }
            if (tig == 0) { sl[HD] = mB; sl[HD + 1] = lB; }
        }
    }
    __threadfence();
    __syncthreads();
    unsigned *counter = p.counters + (size_t)kvs * p.kv_heads + kh;
    if (threadIdx.x == 0) last_flag = atomicAdd(counter, 1u) == p.splits - 1;
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    for (unsigned i = threadIdx.x; i < M * HD; i += NT) {
        const unsigned r = i / HD, d = i % HD, j = r / G, g = r - j * G;
        const size_t pair = ((size_t)kvs * Q + j) * p.kv_heads + kh;
        const float *all = p.partials + pair * p.splits * (size_t)(G * (HD + 2)) + (size_t)g * (HD + 2);
        float Mx = -INFINITY;
        for (unsigned s2 = 0; s2 < p.splits; ++s2) Mx = fmaxf(Mx, __ldcg(all + (size_t)s2 * G * (HD + 2) + HD));
        float acc = 0.f, den = 0.f;
        for (unsigned s2 = 0; s2 < p.splits; ++s2) {
            const float *sl = all + (size_t)s2 * G * (HD + 2);
            const float ms = __ldcg(sl + HD);
            const float f = ms == -INFINITY ? 0.f : expf(ms - Mx);
            acc += __ldcg(sl + d) * f;
            den += __ldcg(sl + HD + 1) * f;
        }
        p.out[(((size_t)kvs * Q + j) * p.heads + (size_t)kh * G + g) * HD + d] = acc / den;
    }
    if (threadIdx.x == 0) *counter = 0;
}

template <int HD, int RW>
static cudaError_t launch_vt(const AtParams &p, dim3 grid, cudaStream_t s)
{
    const size_t smem = vt_smem_bytes<HD>(RW);
    if (cudaFuncSetAttribute(verify_mma_kernel<HD, RW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return cudaErrorInvalidConfiguration;
    verify_mma_kernel<HD, RW><<<grid, RW * 64, smem, s>>>(p);
    return cudaGetLastError();
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
    if (cudaFuncSetAttribute(attention_kernel<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)at_stage_bytes(HD)) != cudaSuccess)
        return cudaErrorInvalidConfiguration;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(AT_THREADS);
    cfg.dynamicSmemBytes = at_stage_bytes(HD);
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
    cudaError_t e = cudaErrorInvalidValue;
    if (G * L.queries >= 2 && G * L.queries <= VT_MAX_ROWS && (L.head_dim == 64 || L.head_dim == 128)) {
        // all query rows of a KV head (its G heads, every draft token) in one
        // CTA on tensor cores: K/V read once for all of them
        const dim3 vgrid(L.splits, L.kv_heads, L.nseq);
        const int rw = (int)((G * L.queries + 15) / 16);
#define FYB_VT(HDV, RWV) if (L.head_dim == HDV && rw == RWV) e = launch_vt<HDV, RWV>(p, vgrid, s);
        FYB_VT(128, 1) FYB_VT(128, 2) FYB_VT(128, 3) FYB_VT(128, 4)
        FYB_VT(64, 1) FYB_VT(64, 2) FYB_VT(64, 3) FYB_VT(64, 4)
#undef FYB_VT
        return e == cudaSuccess ? 0 : -2;
    }
    dim3 grid(L.splits, L.kv_heads, rows);
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
// call should therefore come before any stream capture on the device. The
// kept address assumes the device's primary context lives until the process
// exits (the provider never resets a device); after a reset it would be stale.
// The array takes 4 MiB on every device that loads this library, whether or
// not the entry point is called, outside any NYA_CUDA_MEMORY_MIB budget. Every
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
    // every argument launch_attention checks, checked before the stream is touched
    if (!q || !k || !v || !out || !lengths || !kv_heads || !nseq || !capacity || heads % kv_heads ||
        nseq > 65535 || (head_dim != 64 && head_dim != 128))
        return -1;
    const unsigned groups = heads / kv_heads;
    if (groups != 1 && groups != 2 && groups != 4 && groups != 8) return -1;
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
