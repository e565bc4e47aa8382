// qgemv.cu - dequant-fused K-quant GEMV on the integer tensor cores.
//
// y[r] = sum_k W[r][k] * x[k] for Q4_K / Q6_K weights, one or two input
// vectors (the engine's decode step; reference: nya_row_dot in
// CUDA/matvec.cu:69-111 and the scalar nya_llm_matvec, llm_quant.c:236-276).
//
// Why tensor cores at batch 1: a Q4_K value is half a byte, so at ~6.5 TB/s an
// SM must retire ~40 weights per clock. Unpacking each nibble to a float and
// multiplying on the FP32 pipe costs >3 instructions per weight, which would
// make the kernel ALU-bound well below the HBM roofline. Instead:
//   * the activation vector is split into four signed 8-bit limbs per value,
//     x ~= 2^(E-6) * (X0 + X1/128 + X2/128^2 + X3/128^3), with one power-of-two
//     exponent E per 256-value block (28 bits of mantissa; exact for any value
//     within 2^-4 of the block maximum, and below fp32 rounding otherwise);
//   * the packed nibbles go straight into the A operand of
//     mma.m16n8k32.u8.s8 after one AND (low nibbles) or shift+AND (high);
//   * the four limbs are four columns of the B operand, so one MMA computes
//     the exact integer dot product of 16 rows x 32 values against all limbs;
//   * each 32-value group's 6-bit scale is applied with an integer multiply
//     on the s32 accumulators, and only once per 256-value block are the
//     limb sums converted to float and scaled by d * 2^(E-6-7l).
// The Q4_K minimum term dmin*m_g*sum(x_g) uses the fp32 group sums of x.
// Q6_K runs the same scheme with m16n8k16 (its scales cover 16 values) and
// signed 6-bit quants.
//
// Work split: "units" are (16-row tile, 256-column block) pairs in tile-major
// order; every warp of the grid takes one contiguous range of units
// (stream-K). Rows a warp finishes completely go straight to the epilogue;
// a tile shared by several warps is reduced through a scratch slot per warp,
// and the warp that completes the tile (atomic unit count) sums the slots in
// column order - so results do not depend on timing - and runs the epilogue.
// Fused epilogues: plain store, RoPE + fp16 KV append (Q/K/V projections),
// SiLU(gate)*up, and logits with a greedy argmax.
#include "common.cuh"
#include "kernels.h"
#include <cmath>

namespace fyb {

constexpr int QG_WARPS = 8;
constexpr int QG_THREADS = QG_WARPS * 32;
constexpr int QG_XPAD = 32;  // limb-row padding: row stride = 32 (mod 128) bytes

struct QgSeg {
    const unsigned char *bits;
    const signed char *scales;
    const float *d;
    unsigned rows, tiles, tile_begin;
    float *out;
};

struct QgParams {
    QgSeg seg[3];
    int nseg, epilogue, nvec;
    unsigned tiles_total, nblk, K;
    unsigned long long units, row_bytes;
    unsigned long long out_stride;
    const float *x, *delta;
    float *x_out;
    const float *norm_w;
    float eps;
    __half *kcache, *vcache;
    const float *rope_cos, *rope_sin;
    const unsigned *request;
    unsigned position, head_dim, capacity;
    unsigned long long *argmax_key;
    unsigned *argmax_token, *tiles_done;
    float *partials;
    unsigned *counters;
    unsigned slots;
    unsigned *error;
};

// ------------------------------------------------------------ tile mapping
struct RowPair {
    int segA, segB;
    unsigned rowA, rowB;
    bool okA, okB;
};

FYB_DEV RowPair tile_rows(const QgParams &p, unsigned tile, unsigned gid)
{
    RowPair r;
    if (p.epilogue == EPI_SWIGLU) {
        r.segA = 0; r.segB = 1;
        r.rowA = tile * 8 + gid; r.rowB = r.rowA;
    } else {
        int s = 0;
        if (p.nseg > 1 && tile >= p.seg[1].tile_begin) s = 1;
        if (p.nseg > 2 && tile >= p.seg[2].tile_begin) s = 2;
        unsigned lt = tile - p.seg[s].tile_begin;
        r.segA = r.segB = s;
        if (p.epilogue == EPI_QKV) { r.rowA = lt * 16 + 2 * gid; r.rowB = r.rowA + 1; }
        else { r.rowA = lt * 16 + gid; r.rowB = r.rowA + 8; }
    }
    r.okA = r.rowA < p.seg[r.segA].rows;
    r.okB = r.rowB < p.seg[r.segB].rows;
    return r;
}

// ------------------------------------------------------------ weight buffers
struct Q4Buf { uint4 hA, hB; uint2 qA[4], qB[4]; };
struct Q6Buf { uint2 lA[4], lB[4], hA[2], hB[2]; uint4 sA, sB; float dA, dB; };

template <unsigned TYPE> struct BufOf;
template <> struct BufOf<T_Q4_K> { using T = Q4Buf; };
template <> struct BufOf<T_Q6_K> { using T = Q6Buf; };

struct RowPtrs {
    const unsigned char *a, *b;           // start of the row's bits
    const signed char *sa, *sb;           // Q6_K scales row
    const float *da, *db;                 // Q6_K d row
};

FYB_DEV RowPtrs row_ptrs(const QgParams &p, const RowPair &rp)
{
    const QgSeg &A = p.seg[rp.segA], &B = p.seg[rp.segB];
    unsigned ra = rp.okA ? rp.rowA : A.rows - 1, rb = rp.okB ? rp.rowB : B.rows - 1;
    RowPtrs q;
    q.a = A.bits + (unsigned long long)ra * p.row_bytes;
    q.b = B.bits + (unsigned long long)rb * p.row_bytes;
    q.sa = A.scales ? A.scales + (unsigned long long)ra * p.nblk * 16 : nullptr;
    q.sb = B.scales ? B.scales + (unsigned long long)rb * p.nblk * 16 : nullptr;
    q.da = A.d ? A.d + (unsigned long long)ra * p.nblk : nullptr;
    q.db = B.d ? B.d + (unsigned long long)rb * p.nblk : nullptr;
    return q;
}

FYB_DEV void load_unit(Q4Buf &f, const RowPtrs &r, unsigned blk, unsigned tig)
{
    const unsigned char *a = r.a + blk * 144u, *b = r.b + blk * 144u;
    f.hA = ldg_stream_u4(a);
    f.hB = ldg_stream_u4(b);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        f.qA[p] = ldg_stream_u2(a + 16 + 32 * p + 8 * tig);
        f.qB[p] = ldg_stream_u2(b + 16 + 32 * p + 8 * tig);
    }
}

FYB_DEV void load_unit(Q6Buf &f, const RowPtrs &r, unsigned blk, unsigned tig)
{
    const unsigned char *a = r.a + blk * 192u, *b = r.b + blk * 192u;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        f.lA[c] = ldg_stream_u2(a + 32 * c + 8 * tig);
        f.lB[c] = ldg_stream_u2(b + 32 * c + 8 * tig);
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        f.hA[c] = ldg_stream_u2(a + 128 + 32 * c + 8 * tig);
        f.hB[c] = ldg_stream_u2(b + 128 + 32 * c + 8 * tig);
    }
    f.sA = ldg_stream_u4(r.sa + blk * 16u);
    f.sB = ldg_stream_u4(r.sb + blk * 16u);
    f.dA = __uint_as_float(ldg_stream_u1(r.da + blk));
    f.dB = __uint_as_float(ldg_stream_u1(r.db + blk));
}

FYB_DEV void prefetch_unit(const QgParams &p, unsigned type, const RowPtrs &r, unsigned blk, unsigned lane)
{
    // Lanes 0-15 touch the first line of a row's block, 16-31 the last one.
    unsigned row = lane & 15;
    const unsigned char *base = row < 8 ? r.a : r.b;
    (void)row;
    unsigned bb = type == T_Q4_K ? 144u : 192u;
    const unsigned char *q = base + blk * bb + (lane >= 16 ? bb - 1 : 0);
    prefetch_l2(q);
    (void)p;
}

// ------------------------------------------------------------ byte helpers
FYB_DEV int ubyte(unsigned w, int i) { return (int)((w >> (8 * i)) & 0xffu); }
FYB_DEV int sbyte(unsigned w, int i) { return (int)(signed char)((w >> (8 * i)) & 0xffu); }

FYB_DEV float pow2f(int e)  // 2^e; zero below the normal range
{
    return e < -126 ? 0.0f : __int_as_float((e + 127) << 23);
}

// Signed Q6_K quants (q - 32) of four packed values: low nibble source ql
// (already shifted), two high bits from qh at bit 2*Q of every byte.
template <int Q>
FYB_DEV unsigned q6_signed(unsigned ql, unsigned qh)
{
    unsigned lo = (Q >> 1) ? (ql >> 4) : ql;
    unsigned hi;
    if (Q == 0) hi = qh << 4;
    else if (Q == 1) hi = qh << 2;
    else if (Q == 2) hi = qh;
    else hi = qh >> 2;
    unsigned v = (lo & 0x0F0F0F0Fu) | ((hi & 0x30303030u) ^ 0x20202020u);
    unsigned s = v & 0x20202020u;
    return v + 6u * s;  // sign-extend bit 5 into bits 6 and 7 of every byte
}

// ------------------------------------------------------------ per-unit math
// Accumulates one 256-column block of the warp's 16 rows into accA/accB.
// Lane (gid, tig) holds rows gid (A) and gid+8 (B), matrix columns
// 2*tig, 2*tig+1 = vector tig/2, limbs 2*(tig&1), 2*(tig&1)+1.
template <unsigned TYPE>
FYB_DEV void compute_unit(const typename BufOf<TYPE>::T &f, unsigned blk, const signed char *xl,
    unsigned xrow_stride, bool brow_ok, const int *exps_blk, unsigned nblk, const float *gs_blk,
    unsigned ngroups, int nvec, unsigned gid, unsigned tig, float &accA, float &accB)
{
    const unsigned vec = tig >> 1;
    const int l0 = 2 * (tig & 1);
    const signed char *xrow = xl + (size_t)(brow_ok ? gid : 0) * xrow_stride + blk * 256u;
    int T0 = 0, T1 = 0, T2 = 0, T3 = 0;
    if constexpr (TYPE == T_Q4_K) {
        const unsigned scA0 = f.hA.y & 0x3F3F3F3Fu, mnA0 = f.hA.z & 0x3F3F3F3Fu;
        const unsigned scA1 = (f.hA.w & 0x0F0F0F0Fu) | ((f.hA.y >> 2) & 0x30303030u);
        const unsigned mnA1 = ((f.hA.w >> 4) & 0x0F0F0F0Fu) | ((f.hA.z >> 2) & 0x30303030u);
        const unsigned scB0 = f.hB.y & 0x3F3F3F3Fu, mnB0 = f.hB.z & 0x3F3F3F3Fu;
        const unsigned scB1 = (f.hB.w & 0x0F0F0F0Fu) | ((f.hB.y >> 2) & 0x30303030u);
        const unsigned mnB1 = ((f.hB.w >> 4) & 0x0F0F0F0Fu) | ((f.hB.z >> 2) & 0x30303030u);
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            uint2 blo = make_uint2(0, 0), bhi = make_uint2(0, 0);
            if (brow_ok) {
                blo = *reinterpret_cast<const uint2 *>(xrow + 64 * pr + 8 * tig);
                bhi = *reinterpret_cast<const uint2 *>(xrow + 64 * pr + 32 + 8 * tig);
            }
            unsigned alo[4] = {f.qA[pr].x & 0x0F0F0F0Fu, f.qB[pr].x & 0x0F0F0F0Fu,
                               f.qA[pr].y & 0x0F0F0F0Fu, f.qB[pr].y & 0x0F0F0F0Fu};
            unsigned ahi[4] = {(f.qA[pr].x >> 4) & 0x0F0F0F0Fu, (f.qB[pr].x >> 4) & 0x0F0F0F0Fu,
                               (f.qA[pr].y >> 4) & 0x0F0F0F0Fu, (f.qB[pr].y >> 4) & 0x0F0F0F0Fu};
            int dlo[4] = {0, 0, 0, 0}, dhi[4] = {0, 0, 0, 0};
            mma_u8s8_k32(dlo, alo, blo.x, blo.y);
            mma_u8s8_k32(dhi, ahi, bhi.x, bhi.y);
            const int g0 = 2 * pr, g1 = 2 * pr + 1;
            const int sA0 = ubyte(g0 < 4 ? scA0 : scA1, g0 & 3), sA1 = ubyte(g1 < 4 ? scA0 : scA1, g1 & 3);
            const int sB0 = ubyte(g0 < 4 ? scB0 : scB1, g0 & 3), sB1 = ubyte(g1 < 4 ? scB0 : scB1, g1 & 3);
            T0 += sA0 * dlo[0] + sA1 * dhi[0];
            T1 += sA0 * dlo[1] + sA1 * dhi[1];
            T2 += sB0 * dlo[2] + sB1 * dhi[2];
            T3 += sB0 * dlo[3] + sB1 * dhi[3];
        }
        const float dA = half_bits_to_float((unsigned short)(f.hA.x & 0xffffu));
        const float mA = half_bits_to_float((unsigned short)(f.hA.x >> 16));
        const float dB = half_bits_to_float((unsigned short)(f.hB.x & 0xffffu));
        const float mB = half_bits_to_float((unsigned short)(f.hB.x >> 16));
        const int E = vec < (unsigned)nvec ? exps_blk[vec * nblk] : 0;
        const float f0 = pow2f(E - 6 - 7 * l0), f1 = pow2f(E - 6 - 7 * (l0 + 1));
        accA = fmaf(dA, fmaf((float)T0, f0, (float)T1 * f1), accA);
        accB = fmaf(dB, fmaf((float)T2, f0, (float)T3 * f1), accB);
        if ((tig & 1) == 0 && vec < (unsigned)nvec) {
            const float *gsum = gs_blk + (size_t)vec * ngroups;  // 8 group sums of this block
            const float4 s0 = *reinterpret_cast<const float4 *>(gsum);
            const float4 s1 = *reinterpret_cast<const float4 *>(gsum + 4);
            const float sx[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
            float bA = 0.f, bB = 0.f;
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                bA = fmaf((float)ubyte(g < 4 ? mnA0 : mnA1, g & 3), sx[g], bA);
                bB = fmaf((float)ubyte(g < 4 ? mnB0 : mnB1, g & 3), sx[g], bB);
            }
            accA = fmaf(-mA, bA, accA);
            accB = fmaf(-mB, bB, accB);
        }
    } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int Q = 0; Q < 4; ++Q) {
                const int c = 2 * h + (Q & 1);
                unsigned ax, ay, bx, by;
#define FYB_Q6(QQ)                                                            \
    ax = q6_signed<QQ>(f.lA[c].x, f.hA[h].x); ay = q6_signed<QQ>(f.lA[c].y, f.hA[h].y); \
    bx = q6_signed<QQ>(f.lB[c].x, f.hB[h].x); by = q6_signed<QQ>(f.lB[c].y, f.hB[h].y);
                if (Q == 0) { FYB_Q6(0) } else if (Q == 1) { FYB_Q6(1) } else if (Q == 2) { FYB_Q6(2) } else { FYB_Q6(3) }
#undef FYB_Q6
                unsigned b1 = 0, b2 = 0;
                if (brow_ok) {
                    b1 = *reinterpret_cast<const unsigned *>(xrow + h * 128 + Q * 32 + 4 * tig);
                    b2 = *reinterpret_cast<const unsigned *>(xrow + h * 128 + Q * 32 + 16 + 4 * tig);
                }
                int d1[4] = {0, 0, 0, 0}, d2[4] = {0, 0, 0, 0};
                asm volatile(
                    "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                    : "+r"(d1[0]), "+r"(d1[1]), "+r"(d1[2]), "+r"(d1[3]) : "r"(ax), "r"(bx), "r"(b1));
                asm volatile(
                    "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                    : "+r"(d2[0]), "+r"(d2[1]), "+r"(d2[2]), "+r"(d2[3]) : "r"(ay), "r"(by), "r"(b2));
                const int g = h * 8 + Q * 2;  // first of the two 16-value groups
                const unsigned wA = (&f.sA.x)[g >> 2], wB = (&f.sB.x)[g >> 2];
                const int s1A = sbyte(wA, g & 3), s2A = sbyte(wA, (g & 3) + 1);
                const int s1B = sbyte(wB, g & 3), s2B = sbyte(wB, (g & 3) + 1);
                T0 += s1A * d1[0] + s2A * d2[0];
                T1 += s1A * d1[1] + s2A * d2[1];
                T2 += s1B * d1[2] + s2B * d2[2];
                T3 += s1B * d1[3] + s2B * d2[3];
            }
        }
        const int E = vec < (unsigned)nvec ? exps_blk[vec * nblk] : 0;
        const float f0 = pow2f(E - 6 - 7 * l0), f1 = pow2f(E - 6 - 7 * (l0 + 1));
        accA = fmaf(f.dA, fmaf((float)T0, f0, (float)T1 * f1), accA);
        accB = fmaf(f.dB, fmaf((float)T2, f0, (float)T3 * f1), accB);
        (void)gs_blk; (void)ngroups;
    }
}

// ------------------------------------------------------------ epilogue
FYB_DEV void epilogue(const QgParams &p, unsigned tile, const RowPair &rp, float yA, float yB,
    unsigned gid, unsigned tig, unsigned lane)
{
    const unsigned vec = tig >> 1;
    const bool mine = (tig & 1) == 0 && vec < (unsigned)p.nvec;
    if (p.epilogue == EPI_STORE || p.epilogue == EPI_LOGITS) {
        if (mine) {
            if (rp.okA) p.seg[rp.segA].out[vec * p.out_stride + rp.rowA] = yA;
            if (rp.okB) p.seg[rp.segB].out[vec * p.out_stride + rp.rowB] = yB;
        }
        if (p.epilogue == EPI_LOGITS) {
            unsigned long long key[2] = {0ull, 0ull};
            if (mine) {
                unsigned long long kA = 0, kB = 0;
                if (rp.okA) kA = ((unsigned long long)float_order_key(yA) << 32) | (0xffffffffu - rp.rowA);
                if (rp.okB) kB = ((unsigned long long)float_order_key(yB) << 32) | (0xffffffffu - rp.rowB);
                if ((rp.okA && !isfinite(yA)) || (rp.okB && !isfinite(yB))) {
                    if (p.error) *(volatile unsigned *)p.error = ERR_NONFINITE;
                }
                key[vec] = kA > kB ? kA : kB;
            }
#pragma unroll
            for (int v = 0; v < 2; ++v) {
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    unsigned long long other = __shfl_xor_sync(0xffffffffu, key[v], o);
                    key[v] = other > key[v] ? other : key[v];
                }
            }
            if (lane == 0) {
                for (int v = 0; v < p.nvec; ++v) atomicMax(p.argmax_key + v, key[v]);
                __threadfence();
                unsigned done = atomicAdd(p.tiles_done, 1u);
                if (done == p.tiles_total - 1) {
                    __threadfence();
                    for (int v = 0; v < p.nvec; ++v) {
                        unsigned long long k = atomicExch(p.argmax_key + v, 0ull);
                        p.argmax_token[v] = 0xffffffffu - (unsigned)(k & 0xffffffffu);
                    }
                    atomicExch(p.tiles_done, 0u);
                }
            }
        }
        return;
    }
    if (!mine) return;
    if (p.epilogue == EPI_SWIGLU) {
        // llm_cpu.c:336-342: gate = gate / (1 + expf(-gate)) * up
        if (rp.okA) {
            float g = __fdiv_rn(yA, __fadd_rn(1.0f, expf(-yA)));
            p.seg[0].out[vec * p.out_stride + rp.rowA] = __fmul_rn(g, yB);
        }
        return;
    }
    // EPI_QKV: rows rowA (even) and rowB = rowA + 1 form one RoPE pair
    // (llm_cpu.c:298-327); the key and value rows go to the fp16 cache.
    if (!rp.okA) return;
    const unsigned pos = p.request ? p.request[1] : p.position;
    const unsigned hd = p.head_dim, pair = (rp.rowA % hd) >> 1;
    float a = yA, b = yB;
    if (rp.segA <= 1) {
        const float c = p.rope_cos[(size_t)pos * (hd >> 1) + pair];
        const float s = p.rope_sin[(size_t)pos * (hd >> 1) + pair];
        a = __fsub_rn(__fmul_rn(yA, c), __fmul_rn(yB, s));
        b = __fadd_rn(__fmul_rn(yA, s), __fmul_rn(yB, c));
    }
    if (rp.segA == 0) {
        p.seg[0].out[rp.rowA] = a;
        p.seg[0].out[rp.rowB] = b;
    } else {
        const unsigned kvh = rp.rowA / hd, dd = rp.rowA % hd;
        __half *cache = rp.segA == 1 ? p.kcache : p.vcache;
        __half2 v2 = __halves2half2(__float2half_rn(a), __float2half_rn(b));
        *reinterpret_cast<__half2 *>(cache + ((size_t)kvh * p.capacity + pos) * hd + dd) = v2;
    }
}

// ------------------------------------------------------------ x preparation
// Residual add, RMSNorm (llm_cpu.c:83-103: sum of squares in double, then
// x*scale*w in float), then the limb split. Every CTA prepares the whole
// vector; its slice of the residual stream is written back by one CTA.
template <int NT>
FYB_DEV double block_sum_double(double v, double *red)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = 0;
    for (int w = 0; w < NT / 32; ++w) t += red[w];
    return t;
}

FYB_DEV void load16(const float *src, float (&v)[16])
{
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float4 t = __ldcg(s4 + i);
        v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
}

FYB_DEV void prepare_x(const QgParams &p, signed char *xl, unsigned xstride, int *exps, float *gsums, double *red)
{
    const unsigned tid = threadIdx.x, K = p.K, nslot = K / 16, total = nslot * (unsigned)p.nvec;
    float scale[2] = {1.f, 1.f};
    if (p.norm_w) {
        for (int v = 0; v < p.nvec; ++v) {
            double ss = 0.0;
            for (unsigned s = tid; s < nslot; s += QG_THREADS) {
                float x[16];
                load16(p.x + (size_t)v * K + 16 * s, x);
                if (p.delta) {
                    float dl[16];
                    load16(p.delta + (size_t)v * K + 16 * s, dl);
#pragma unroll
                    for (int j = 0; j < 16; ++j) x[j] = __fadd_rn(x[j], dl[j]);
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) ss += (double)x[j] * (double)x[j];
            }
            ss = block_sum_double<QG_THREADS>(ss, red);
            scale[v] = (float)(1.0 / sqrt(ss / (double)K + (double)p.eps));
        }
    }
    const unsigned iters = (total + QG_THREADS - 1) / QG_THREADS;
    for (unsigned it = 0; it < iters; ++it) {
        const unsigned s = it * QG_THREADS + tid;
        const bool ok = s < total;
        const unsigned v = ok ? s / nslot : 0, sl = ok ? s % nslot : 0;
        float x[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] = 0.f;
        if (ok) {
            load16(p.x + (size_t)v * K + 16 * sl, x);
            if (p.delta) {
                float dl[16];
                load16(p.delta + (size_t)v * K + 16 * sl, dl);
#pragma unroll
                for (int j = 0; j < 16; ++j) x[j] = __fadd_rn(x[j], dl[j]);
            }
            if (p.x_out && (sl % gridDim.x) == blockIdx.x) {
                float4 *o4 = reinterpret_cast<float4 *>(p.x_out + (size_t)v * K + 16 * sl);
#pragma unroll
                for (int i = 0; i < 4; ++i) o4[i] = make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
            }
            if (p.norm_w) {
                float w[16];
                load16(p.norm_w + 16 * sl, w);
#pragma unroll
                for (int j = 0; j < 16; ++j) x[j] = __fmul_rn(__fmul_rn(x[j], scale[v]), w[j]);
            }
        }
        // 32-value group sums (fp32, sequential within the group)
        float gs = 0.f, mx = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) { gs = __fadd_rn(gs, x[j]); mx = fmaxf(mx, fabsf(x[j])); }
        const float other = __shfl_xor_sync(0xffffffffu, gs, 1);
        if (ok && (sl & 1) == 0) gsums[v * (K / 32) + sl / 2] = __fadd_rn(gs, other);
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        int E = 0;
        bool bad = !(mx <= 3.0e38f);  // inf or NaN in the block
        if (!bad && mx > 0.f) {
            frexpf(mx, &E);
            if (E < -120) E = -120;  // below 2^-121: limbs round to zero anyway
        }
        if (ok && (sl & 15) == 0) exps[v * p.nblk + sl / 16] = E;
        if (bad && p.error) *(volatile unsigned *)p.error = ERR_NONFINITE;
        const float sc = pow2f(6 - E);
        unsigned words[4][4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            unsigned t[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float r = bad ? 0.f : __fmul_rn(x[4 * q + i], sc);
#pragma unroll
                for (int l = 0; l < 4; ++l) {
                    const float m = __fadd_rn(r, 12582912.0f);  // rint via the 1.5*2^23 magic
                    const float X = __fsub_rn(m, 12582912.0f);
                    t[l][i] = __float_as_uint(m);
                    r = __fmul_rn(__fsub_rn(r, X), 128.0f);
                }
            }
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const unsigned lo = __byte_perm(t[l][0], t[l][1], 0x0040);
                const unsigned hi = __byte_perm(t[l][2], t[l][3], 0x0040);
                words[l][q] = __byte_perm(lo, hi, 0x5410);
            }
        }
        if (ok) {
#pragma unroll
            for (int l = 0; l < 4; ++l)
                *reinterpret_cast<uint4 *>(xl + (size_t)(v * 4 + l) * xstride + 16 * sl) =
                    make_uint4(words[l][0], words[l][1], words[l][2], words[l][3]);
        }
    }
}

// ------------------------------------------------------------ one unit step
struct WarpState {
    unsigned long long u, u_end;
    unsigned tile, tile_units;
    RowPair rp;
    RowPtrs ptr;
    float accA, accB;
};
struct Smem {
    const signed char *xl;
    unsigned xstride;
    const int *exps;
    const float *gsums;
};

// Consume unit st.u from `cur` after issuing the loads of unit st.u+1 into
// `nxt`; finish the tile (directly or through the fix-up) when it ends here.
template <unsigned TYPE, class Buf>
FYB_DEV bool step(const QgParams &p, WarpState &st, const Smem &sm, Buf &cur, Buf &nxt,
    unsigned long long NW, unsigned long long gw, unsigned lane)
{
    const unsigned nblk = p.nblk, gid = lane >> 2, tig = lane & 3;
    const unsigned blk = (unsigned)(st.u % nblk);
    const unsigned long long un = st.u + 1;
    RowPair rpn = st.rp;
    RowPtrs ptrn = st.ptr;
    unsigned tilen = st.tile;
    if (un < st.u_end) {
        tilen = (unsigned)(un / nblk);
        if (tilen != st.tile) { rpn = tile_rows(p, tilen, gid); ptrn = row_ptrs(p, rpn); }
        load_unit(nxt, ptrn, (unsigned)(un % nblk), tig);
        const unsigned long long up = st.u + 4;
        if (up < st.u_end) {
            unsigned t2 = (unsigned)(up / nblk);
            RowPtrs p2 = row_ptrs(p, tile_rows(p, t2, lane & 7));
            prefetch_unit(p, TYPE, p2, (unsigned)(up % nblk), lane);
        }
    }
    const bool brow_ok = gid < (unsigned)(4 * p.nvec);
    compute_unit<TYPE>(cur, blk, sm.xl, sm.xstride, brow_ok, sm.exps + blk, nblk,
                       sm.gsums + (size_t)blk * 8, p.K / 32, p.nvec, gid, tig, st.accA, st.accB);
    ++st.tile_units;
    if (blk + 1 == nblk || un == st.u_end) {
        // combine the two limb halves of every vector
        float yA = st.accA + __shfl_xor_sync(0xffffffffu, st.accA, 1);
        float yB = st.accB + __shfl_xor_sync(0xffffffffu, st.accB, 1);
        bool run_epilogue = true;
        if (st.tile_units != nblk) {
            // stream-K fix-up through the scratch slots of this tile
            const unsigned long long U = p.units;
            const unsigned long long t0 = (unsigned long long)st.tile * nblk;
            const unsigned long long owner0 = ((t0 + 1) * NW - 1) / U;
            const unsigned long long ownerN = ((t0 + nblk) * NW - 1) / U;
            const unsigned slot = (unsigned)(gw - owner0);
            const unsigned nslots = (unsigned)(ownerN - owner0 + 1);
            float *base = p.partials + ((size_t)st.tile * p.slots) * 32;
            const unsigned v = tig >> 1;
            if ((tig & 1) == 0) {
                base[slot * 32 + gid * 2 + v] = yA;
                base[slot * 32 + (gid + 8) * 2 + v] = yB;
            }
            __threadfence();
            __syncwarp();
            unsigned old = 0;
            if (lane == 0) old = atomicAdd(p.counters + st.tile, st.tile_units);
            old = __shfl_sync(0xffffffffu, old, 0);
            run_epilogue = old + st.tile_units == nblk;
            if (run_epilogue) {
                __threadfence();
                yA = 0.f; yB = 0.f;
                // sum, in column order, the slots of the warps whose unit
                // ranges intersect this tile (warps without units own none)
                for (unsigned s = 0; s < nslots; ++s) {
                    const unsigned long long g = owner0 + s;
                    const unsigned long long ub = g * U / NW, ue = (g + 1) * U / NW;
                    if (ue <= ub || ub >= t0 + nblk || ue <= t0) continue;
                    yA += __ldcg(base + s * 32 + gid * 2 + v);
                    yB += __ldcg(base + s * 32 + (gid + 8) * 2 + v);
                }
                if (lane == 0) p.counters[st.tile] = 0;
            }
        }
        if (run_epilogue) epilogue(p, st.tile, st.rp, yA, yB, gid, tig, lane);
        st.accA = 0.f; st.accB = 0.f;
        st.tile_units = 0;
    }
    st.u = un;
    st.tile = tilen; st.rp = rpn; st.ptr = ptrn;
    return st.u < st.u_end;
}

// ------------------------------------------------------------ the kernel
template <unsigned TYPE>
__global__ void __launch_bounds__(QG_THREADS, 1) qgemv_kernel(const QgParams p)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const unsigned K = p.K, nblk = p.nblk;
    const unsigned xstride = K + QG_XPAD;
    signed char *xl = reinterpret_cast<signed char *>(smem);
    size_t off = (size_t)p.nvec * 4 * xstride;
    int *exps = reinterpret_cast<int *>(smem + off);
    off += ((size_t)p.nvec * nblk * 4 + 15) / 16 * 16;
    float *gsums = reinterpret_cast<float *>(smem + off);
    off += ((size_t)p.nvec * (K / 32) * 4 + 15) / 16 * 16;
    double *red = reinterpret_cast<double *>(smem + off);

    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned gid = lane >> 2, tig = lane & 3;
    const unsigned long long NW = (unsigned long long)gridDim.x * QG_WARPS;
    const unsigned long long gw = (unsigned long long)blockIdx.x * QG_WARPS + warp;
    const unsigned long long U = p.units;
    unsigned long long u = gw * U / NW;
    const unsigned long long u_end = (gw + 1) * U / NW;

    using Buf = typename BufOf<TYPE>::T;
    Buf b0, b1;
    WarpState st;
    st.u = u; st.u_end = u_end; st.tile = 0; st.tile_units = 0; st.accA = 0.f; st.accB = 0.f;
    if (u < u_end) {
        st.tile = (unsigned)(u / nblk);
        st.rp = tile_rows(p, st.tile, gid);
        st.ptr = row_ptrs(p, st.rp);
        load_unit(b0, st.ptr, (unsigned)(u % nblk), tig);
        // warm L2 with the next units of this warp's range
        for (unsigned long long w = u + 1; w < u_end && w < u + 4; ++w) {
            unsigned t2 = (unsigned)(w / nblk);
            RowPtrs p2 = row_ptrs(p, tile_rows(p, t2, lane & 7));
            prefetch_unit(p, TYPE, p2, (unsigned)(w % nblk), lane);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    prepare_x(p, xl, xstride, exps, gsums, red);
    __syncthreads();

    const Smem sm{xl, xstride, exps, gsums};
    while (st.u < st.u_end) {
        if (!step<TYPE>(p, st, sm, b0, b1, NW, gw, lane)) break;
        if (!step<TYPE>(p, st, sm, b1, b0, NW, gw, lane)) break;
    }
}

// ------------------------------------------------------------ Q6_K repack
__global__ void repack_q6k_kernel(const unsigned char *raw, unsigned long long nblocks_total, unsigned char *bits,
    signed char *scales, float *d)
{
    unsigned long long b = (unsigned long long)blockIdx.x * blockDim.y + threadIdx.y;
    if (b >= nblocks_total) return;
    const unsigned char *src = raw + b * 210;
    unsigned char *dst = bits + b * 192;
    // 192 bit bytes as six 32-byte runs; lane t writes bytes 8(t%4)..+7 of run t/4
    for (unsigned i = threadIdx.x; i < 192; i += 32) {
        unsigned run = i / 32, k = i % 32;          // destination position
        unsigned tg = k / 8, part = (k % 8) / 4, e = k % 4;
        unsigned srcpos = run * 32 + part * 16 + tg * 4 + e;
        dst[i] = src[srcpos];
    }
    if (threadIdx.x < 16) scales[b * 16 + threadIdx.x] = (signed char)src[192 + threadIdx.x];
    if (threadIdx.x == 0) d[b] = half_at(src + 208);
}

size_t q6k_repacked_bytes(size_t rows, size_t cols)
{
    size_t nb = rows * (cols / 256);
    return nb * 192 + nb * 16 + nb * 4 + 256;
}

int repack_q6k(const void *raw, size_t rows, size_t cols, void *dst, QMatrix *out, cudaStream_t s)
{
    size_t nb = rows * (cols / 256);
    unsigned char *bits = (unsigned char *)dst;
    signed char *scales = (signed char *)(bits + nb * 192);
    float *d = (float *)(bits + nb * 192 + nb * 16);
    dim3 block(32, 8);
    unsigned grid = (unsigned)((nb + 7) / 8);
    if (nb) repack_q6k_kernel<<<grid, block, 0, s>>>((const unsigned char *)raw, nb, bits, scales, d);
    if (cudaGetLastError() != cudaSuccess) return -2;
    out->bits = bits; out->scales = scales; out->d = d;
    out->rows = (unsigned)rows; out->cols = (unsigned)cols; out->type = T_Q6_K;
    return 0;
}

QMatrix q4k_matrix(const void *raw, size_t rows, size_t cols)
{
    QMatrix m;
    m.bits = (const unsigned char *)raw;
    m.rows = (unsigned)rows; m.cols = (unsigned)cols; m.type = T_Q4_K;
    return m;
}

// ------------------------------------------------------------ host side
static int sm_count()
{
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

int qgemv_supported(unsigned type, size_t cols, size_t nvec)
{
    return (type == T_Q4_K || type == T_Q6_K) && cols % 256 == 0 && cols >= 256 && cols <= 16384 &&
           nvec >= 1 && nvec <= 2;
}

static size_t qgemv_smem(unsigned K, int nvec)
{
    size_t off = (size_t)nvec * 4 * (K + QG_XPAD);
    off += ((size_t)nvec * (K / 256) * 4 + 15) / 16 * 16;
    off += ((size_t)nvec * (K / 32) * 4 + 15) / 16 * 16;
    return off + QG_WARPS * sizeof(double) + 64;
}

static void build_params(const QgemvLaunch &L, int grid, QgParams &p, unsigned long long &units)
{
    p = QgParams{};
    const QMatrix &m0 = L.seg[0];
    p.K = m0.cols;
    p.nblk = m0.cols / 256;
    p.row_bytes = m0.type == T_Q4_K ? (unsigned long long)p.nblk * 144 : (unsigned long long)p.nblk * 192;
    p.nseg = L.nseg;
    p.epilogue = L.epilogue;
    p.nvec = L.nvec;
    unsigned tiles = 0;
    for (int s = 0; s < L.nseg; ++s) {
        QgSeg &g = p.seg[s];
        g.bits = L.seg[s].bits; g.scales = L.seg[s].scales; g.d = L.seg[s].d;
        g.rows = L.seg[s].rows;
        g.out = L.out[s];
        g.tile_begin = tiles;
        g.tiles = L.epilogue == EPI_SWIGLU ? (g.rows + 7) / 8 : (g.rows + 15) / 16;
        if (L.epilogue != EPI_SWIGLU) tiles += g.tiles;
    }
    if (L.epilogue == EPI_SWIGLU) tiles = p.seg[0].tiles;
    p.tiles_total = tiles;
    units = (unsigned long long)tiles * p.nblk;
    p.units = units;
    p.out_stride = L.out_stride;
    p.x = L.x; p.delta = L.delta; p.x_out = L.x_out; p.norm_w = L.norm_w; p.eps = L.eps;
    p.kcache = L.kcache; p.vcache = L.vcache;
    p.rope_cos = L.rope_cos; p.rope_sin = L.rope_sin;
    p.request = L.request; p.position = L.position; p.head_dim = L.head_dim; p.capacity = L.capacity;
    p.argmax_key = L.argmax_key; p.argmax_token = L.argmax_token; p.tiles_done = L.tiles_done;
    p.error = L.error;
    // slots: warp indices owner(t*nblk) .. owner(t*nblk + nblk - 1) of a tile
    // span at most ceil(nblk * NW / U) + 1 values
    unsigned long long NW = (unsigned long long)grid * QG_WARPS;
    p.slots = units ? (unsigned)((p.nblk * NW + units - 1) / units + 2) : 1;
}

// CTAs for a launch: one per SM, fewer when the problem gives a warp less
// than two units, so small matrices do not pay for idle CTAs' preparation.
static int qgemv_grid(const QgemvLaunch &L, int grid)
{
    if (grid <= 0) grid = sm_count();
    QgParams p;
    unsigned long long units;
    build_params(L, grid, p, units);
    unsigned long long want = (units + 2ull * QG_WARPS - 1) / (2ull * QG_WARPS);
    if (want < 1) want = 1;
    return (int)std::min<unsigned long long>((unsigned long long)grid, want);
}

size_t qgemv_workspace_bytes(const QgemvLaunch &L, int grid)
{
    grid = qgemv_grid(L, grid);
    QgParams p;
    unsigned long long units;
    build_params(L, grid, p, units);
    size_t partial = (size_t)p.tiles_total * p.slots * 32 * sizeof(float);
    size_t counters = (size_t)p.tiles_total * sizeof(unsigned);
    return (partial + 255) / 256 * 256 + (counters + 255) / 256 * 256;
}

int launch_qgemv(const QgemvLaunch &L, cudaStream_t s)
{
    const QMatrix &m0 = L.seg[0];
    if (!qgemv_supported(m0.type, m0.cols, (size_t)L.nvec) || L.nseg < 1 || L.nseg > 3) return -1;
    for (int i = 1; i < L.nseg; ++i)
        if (L.seg[i].type != m0.type || L.seg[i].cols != m0.cols) return -1;
    if ((L.epilogue == EPI_QKV || L.epilogue == EPI_SWIGLU) && L.nvec != 1) return -1;
    if (L.epilogue == EPI_SWIGLU && (L.nseg != 2 || L.seg[0].rows != L.seg[1].rows)) return -1;
    int grid = qgemv_grid(L, L.grid);
    QgParams p;
    unsigned long long units;
    build_params(L, grid, p, units);
    if (units == 0) return 0;
    size_t need = qgemv_workspace_bytes(L, L.grid);
    if (!L.workspace || L.workspace_bytes < need) return -1;
    size_t partial = ((size_t)p.tiles_total * p.slots * 32 * sizeof(float) + 255) / 256 * 256;
    p.partials = (float *)L.workspace;
    p.counters = (unsigned *)((unsigned char *)L.workspace + partial);
    size_t smem = qgemv_smem(p.K, p.nvec);
    auto kern = m0.type == T_Q4_K ? qgemv_kernel<T_Q4_K> : qgemv_kernel<T_Q6_K>;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return -2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(QG_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = L.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p) == cudaSuccess ? 0 : -2;
}

}  // namespace fyb
