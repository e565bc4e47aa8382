// qgemv_core.cuh - device building blocks of the K-quant tensor-core GEMV,
// shared by the stand-alone GEMV kernel (qgemv.cu) and the persistent
// decode kernel (decode.cu). The scheme is described in qgemv.cu.
#pragma once
#include "common.cuh"
#include "kernels.h"
#include <cmath>

namespace fyb {

#ifndef FYB_QG_WARPS
#define FYB_QG_WARPS 16
#endif
#ifndef FYB_QG_STAGES
#define FYB_QG_STAGES 2
#endif
constexpr int QG_WARPS = FYB_QG_WARPS;   // warps per CTA, one CTA per SM
constexpr int QG_THREADS = QG_WARPS * 32;
constexpr int QG_STAGES = FYB_QG_STAGES; // bulk-copy stages per warp
constexpr int QG_XPAD = 64;  // limb-row stride = 64 (mod 128) bytes: conflict-free B fragments

constexpr unsigned Q4_UNIT = 2304;  // qs [p4][h2][r16][16] | hdr [r16][16]
constexpr unsigned Q6_UNIT = 3360;  // ql [c4][h2][r16][16] | qh [c2][h2][r16][16] | sc [r16][16] | d [r16] f16
__host__ __device__ constexpr unsigned unit_bytes(unsigned type) { return type == T_Q4_K ? Q4_UNIT : Q6_UNIT; }

// ------------------------------------------------------------ byte helpers
FYB_DEV int ubyte(unsigned w, int i) { return (int)((w >> (8 * i)) & 0xffu); }
FYB_DEV int sbyte(unsigned w, int i) { return (int)(signed char)((w >> (8 * i)) & 0xffu); }
FYB_DEV float pow2f(int e) { return e < -126 ? 0.0f : __int_as_float((e + 127) << 23); }

// Signed Q6_K quants (q - 32) of four packed values: low nibbles from ql
// (high nibble for quarters 2 and 3), two high bits from qh at bit 2*Q.
template <int Q>
FYB_DEV unsigned q6_signed(unsigned ql, unsigned qh)
{
    const unsigned lo = (Q >> 1) ? (ql >> 4) : ql;
    unsigned hi;
    if (Q == 0) hi = qh << 4;
    else if (Q == 1) hi = qh << 2;
    else if (Q == 2) hi = qh;
    else hi = qh >> 2;
    const unsigned v = (lo & 0x0F0F0F0Fu) | ((hi & 0x30303030u) ^ 0x20202020u);
    const unsigned s = v & 0x20202020u;
    return v + 6u * s;  // sign-extend bit 5 into bits 6 and 7 of every byte
}

// ldmatrix.x4 of a [h2][r16][16 B] block: lane i addresses row (i&7)+8*((i>>3)&1),
// half (i>>4). Result regs: (r gid, bytes 4t..), (r gid+8, 4t..), (r gid, 16+4t..), (r gid+8, 16+4t..)
FYB_DEV void load_frag(unsigned (&r)[4], const unsigned char *base, unsigned lane)
{
    const unsigned row = (lane & 7) + 8 * ((lane >> 3) & 1), half = lane >> 4;
    ldmatrix_x4(r, base + half * 256 + row * 16);
}

// ------------------------------------------------------------ per-unit math
// x limbs in shared memory: four rows per vector (limb 0..3), row stride
// K + QG_XPAD bytes. Within every 64-byte chunk the 4-byte words are stored
// lane-major: word 4j + t of the natural order sits at position 4t + j, so
// the B fragments a lane needs from one chunk (natural words t, 4+t, 8+t,
// 12+t for lane t) are one 16-byte load, and the Q6_K pairs one 8-byte load.
// A row stride of 64 (mod 128) bytes keeps those loads free of bank conflicts.
FYB_HOST_DEV unsigned limb_pos(unsigned byte)  // natural byte offset -> stored offset
{
    const unsigned chunk = byte & ~63u, w = (byte & 63u) >> 2;
    return chunk + ((w & 3u) * 4u + (w >> 2)) * 4u + (byte & 3u);
}

// Accumulates one unit (16 rows x 256 columns, from shared memory) into
// accA (row gid) / accB (row gid+8) of lane (gid, tig). The MMA result
// columns of a lane are limbs 2*(tig&1), 2*(tig&1)+1 of vector tig>>1; with
// NV == 1, lanes tig 2 and 3 see zero B columns. The Q4_K minimum term is
// split over the lanes that share a vector (all four with NV == 1, two with
// NV == 2), so a tile's value is the sum of accA over those lanes.
template <unsigned TYPE, int NV>
FYB_DEV void compute_unit(const unsigned char *u, unsigned blk, const signed char *xl, unsigned xstride,
    const int *exps, unsigned nblk, const float *gsums, unsigned ngroups, unsigned lane, float &accA, float &accB)
{
    const unsigned gid = lane >> 2, tig = lane & 3, vec = tig >> 1;
    const bool brow_ok = gid < 4u * NV;
    const int l0 = 2 * (tig & 1);
    const signed char *xrow = xl + (size_t)(brow_ok ? gid : 0) * xstride + blk * 256u + tig * 16u;
    int T0 = 0, T1 = 0, T2 = 0, T3 = 0;
    if constexpr (TYPE == T_Q4_K) {
        const uint4 hA = *reinterpret_cast<const uint4 *>(u + 2048 + gid * 16);
        const uint4 hB = *reinterpret_cast<const uint4 *>(u + 2048 + (gid + 8) * 16);
        // six-bit scales (llm_quant.c:249): groups 0-3 in .y, 4-7 in .w/.y
        const unsigned scA0 = hA.y & 0x3F3F3F3Fu, scA1 = (hA.w & 0x0F0F0F0Fu) | ((hA.y >> 2) & 0x30303030u);
        const unsigned scB0 = hB.y & 0x3F3F3F3Fu, scB1 = (hB.w & 0x0F0F0F0Fu) | ((hB.y >> 2) & 0x30303030u);
        int U0 = 0, U1 = 0, U2 = 0, U3 = 0;  // high-nibble groups, 16x (the nibbles stay in place)
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            unsigned q[4];
            load_frag(q, u + pr * 512, lane);
            uint4 bw = make_uint4(0u, 0u, 0u, 0u);
            if (brow_ok) bw = *reinterpret_cast<const uint4 *>(xrow + 64 * pr);
            const unsigned alo[4] = {q[0] & 0x0F0F0F0Fu, q[1] & 0x0F0F0F0Fu, q[2] & 0x0F0F0F0Fu, q[3] & 0x0F0F0F0Fu};
            const unsigned ahi[4] = {q[0] & 0xF0F0F0F0u, q[1] & 0xF0F0F0F0u, q[2] & 0xF0F0F0F0u, q[3] & 0xF0F0F0F0u};
            int dlo[4] = {0, 0, 0, 0}, dhi[4] = {0, 0, 0, 0};
            mma_u8s8_k32(dlo, alo, bw.x, bw.y);
            mma_u8s8_k32(dhi, ahi, bw.z, bw.w);
            const unsigned wA = pr < 2 ? scA0 : scA1, wB = pr < 2 ? scB0 : scB1;
            const int b0 = (2 * pr) & 3, b1 = b0 + 1;
            const int sAl = (int)__byte_perm(wA, 0u, 0x4440 + b0), sAh = (int)__byte_perm(wA, 0u, 0x4440 + b1);
            const int sBl = (int)__byte_perm(wB, 0u, 0x4440 + b0), sBh = (int)__byte_perm(wB, 0u, 0x4440 + b1);
            T0 += sAl * dlo[0]; U0 += sAh * dhi[0];
            T1 += sAl * dlo[1]; U1 += sAh * dhi[1];
            T2 += sBl * dlo[2]; U2 += sBh * dhi[2];
            T3 += sBl * dlo[3]; U3 += sBh * dhi[3];
        }
        T0 += U0 >> 4; T1 += U1 >> 4; T2 += U2 >> 4; T3 += U3 >> 4;  // exact: U is a multiple of 16
        const float dA = half_bits_to_float((unsigned short)(hA.x & 0xffffu));
        const float dB = half_bits_to_float((unsigned short)(hB.x & 0xffffu));
        const int E = vec < (unsigned)NV ? exps[vec * nblk + blk] : 0;
        const float f0 = pow2f(E - 6 - 7 * l0), f1 = pow2f(E - 6 - 7 * (l0 + 1));
        accA = fmaf(dA, fmaf((float)T0, f0, (float)T1 * f1), accA);
        accB = fmaf(dB, fmaf((float)T2, f0, (float)T3 * f1), accB);
        // minimum term -dmin * sum_g m_g * sum(x_g) of both rows; with NV == 1
        // lane tig takes groups 2tig, 2tig+1, with NV == 2 groups 4(tig&1)..+3
        if (NV == 1 || vec < (unsigned)NV) {  // with one vector all four lanes take a share
            const unsigned mA0 = hA.z & 0x3F3F3F3Fu, mA1 = ((hA.w >> 4) & 0x0F0F0F0Fu) | ((hA.z >> 2) & 0x30303030u);
            const unsigned mB0 = hB.z & 0x3F3F3F3Fu, mB1 = ((hB.w >> 4) & 0x0F0F0F0Fu) | ((hB.z >> 2) & 0x30303030u);
            const float *gs = gsums + (size_t)(NV == 1 ? 0u : vec) * ngroups + blk * 8;  // the block's 8 group sums
            const float dmA = half_bits_to_float((unsigned short)(hA.x >> 16));
            const float dmB = half_bits_to_float((unsigned short)(hB.x >> 16));
            float bA = 0.f, bB = 0.f;
            if constexpr (NV == 1) {
                const float2 g2 = *reinterpret_cast<const float2 *>(gs + 2 * tig);
                const unsigned wA = tig < 2 ? mA0 : mA1, wB = tig < 2 ? mB0 : mB1;
                const unsigned o = (2 * tig) & 3;
                bA = fmaf((float)__byte_perm(wA, 0u, 0x4440 + o + 1), g2.y, (float)__byte_perm(wA, 0u, 0x4440 + o) * g2.x);
                bB = fmaf((float)__byte_perm(wB, 0u, 0x4440 + o + 1), g2.y, (float)__byte_perm(wB, 0u, 0x4440 + o) * g2.x);
            } else {
                const float4 g4 = *reinterpret_cast<const float4 *>(gs + 4 * (tig & 1));
                const unsigned wA = (tig & 1) ? mA1 : mA0, wB = (tig & 1) ? mB1 : mB0;
                bA = (float)__byte_perm(wA, 0u, 0x4440) * g4.x;
                bA = fmaf((float)__byte_perm(wA, 0u, 0x4441), g4.y, bA);
                bA = fmaf((float)__byte_perm(wA, 0u, 0x4442), g4.z, bA);
                bA = fmaf((float)__byte_perm(wA, 0u, 0x4443), g4.w, bA);
                bB = (float)__byte_perm(wB, 0u, 0x4440) * g4.x;
                bB = fmaf((float)__byte_perm(wB, 0u, 0x4441), g4.y, bB);
                bB = fmaf((float)__byte_perm(wB, 0u, 0x4442), g4.z, bB);
                bB = fmaf((float)__byte_perm(wB, 0u, 0x4443), g4.w, bB);
            }
            accA = fmaf(-dmA, bA, accA);
            accB = fmaf(-dmB, bB, accB);
        }
    } else {
        const uint4 sA = *reinterpret_cast<const uint4 *>(u + 3072 + gid * 16);
        const uint4 sB = *reinterpret_cast<const uint4 *>(u + 3072 + (gid + 8) * 16);
        const float dA = half_bits_to_float(*reinterpret_cast<const unsigned short *>(u + 3328 + gid * 2));
        const float dB = half_bits_to_float(*reinterpret_cast<const unsigned short *>(u + 3328 + (gid + 8) * 2));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            unsigned qh[4];
            load_frag(qh, u + 2048 + h * 512, lane);
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
                unsigned ql[4];
                load_frag(ql, u + (2 * h + c2) * 512, lane);
#pragma unroll
                for (int hiq = 0; hiq < 2; ++hiq) {
                    const int Q = c2 + 2 * hiq;  // quarter: ql chunk c2, nibble hiq
                    unsigned a[4];
#define FYB_Q6(QQ) for (int i = 0; i < 4; ++i) a[i] = q6_signed<QQ>(ql[i], qh[i]);
                    if (Q == 0) { FYB_Q6(0) } else if (Q == 1) { FYB_Q6(1) } else if (Q == 2) { FYB_Q6(2) } else { FYB_Q6(3) }
#undef FYB_Q6
                    uint2 bw = make_uint2(0u, 0u);
                    if (brow_ok) bw = *reinterpret_cast<const uint2 *>(xrow + (2 * h + (Q >> 1)) * 64 + 8 * (Q & 1));
                    int d1[4] = {0, 0, 0, 0}, d2[4] = {0, 0, 0, 0};
                    asm volatile(
                        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                        : "+r"(d1[0]), "+r"(d1[1]), "+r"(d1[2]), "+r"(d1[3]) : "r"(a[0]), "r"(a[1]), "r"(bw.x));
                    asm volatile(
                        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                        : "+r"(d2[0]), "+r"(d2[1]), "+r"(d2[2]), "+r"(d2[3]) : "r"(a[2]), "r"(a[3]), "r"(bw.y));
                    const int g = h * 8 + Q * 2;  // first of the two 16-value scale groups
                    const unsigned wA = (&sA.x)[g >> 2], wB = (&sB.x)[g >> 2];
                    const int s1A = sbyte(wA, g & 3), s2A = sbyte(wA, (g & 3) + 1);
                    const int s1B = sbyte(wB, g & 3), s2B = sbyte(wB, (g & 3) + 1);
                    T0 += s1A * d1[0] + s2A * d2[0];
                    T1 += s1A * d1[1] + s2A * d2[1];
                    T2 += s1B * d1[2] + s2B * d2[2];
                    T3 += s1B * d1[3] + s2B * d2[3];
                }
            }
        }
        const int E = vec < (unsigned)NV ? exps[vec * nblk + blk] : 0;
        const float f0 = pow2f(E - 6 - 7 * l0), f1 = pow2f(E - 6 - 7 * (l0 + 1));
        accA = fmaf(dA, fmaf((float)T0, f0, (float)T1 * f1), accA);
        accB = fmaf(dB, fmaf((float)T2, f0, (float)T3 * f1), accB);
        (void)gsums; (void)ngroups;
    }
}

// NT units of the same 256-column block (one input vector): the x-limb
// fragments and the block's exponent and group sums are loaded once and
// reused for every unit, and the units' MMA chains are independent, so a
// warp keeps NT chains in flight. acc[n][0] / acc[n][1] are unit n's row gid
// / gid + 8 partial sums as in compute_unit<TYPE, 1>.
// The per-lane constants of one prepared block: the limb weights of the
// lane's two MMA columns and (Q4_K) the lane's two group sums.
struct BlockConst {
    float f0, f1;
    float2 g2;
};
FYB_DEV BlockConst block_const(const int *exps, const float *gsums, unsigned lane)
{
    const unsigned tig = lane & 3;
    const int l0 = 2 * (tig & 1);
    const int E = tig < 2 ? exps[0] : 0;
    BlockConst c;
    c.f0 = pow2f(E - 6 - 7 * l0);
    c.f1 = pow2f(E - 6 - 7 * (l0 + 1));
    c.g2 = *reinterpret_cast<const float2 *>(gsums + 2 * tig);
    return c;
}

template <unsigned TYPE, int NT>
FYB_DEV void compute_units(const unsigned char *const (&u)[NT], const signed char *xl, unsigned xstride,
    const BlockConst &bc, unsigned lane, float (&acc)[NT][2])
{
    const unsigned gid = lane >> 2, tig = lane & 3;
    const bool brow_ok = gid < 4u;
    const signed char *xrow = xl + (size_t)(brow_ok ? gid : 0) * xstride + tig * 16u;
    const float f0 = bc.f0, f1 = bc.f1;
    if constexpr (TYPE == T_Q4_K) {
        int T[NT][4], Uh[NT][4];
        unsigned sc[NT][4];  // scales of rows A (groups 0-3, 4-7) and B (0-3, 4-7)
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const uint4 hA = *reinterpret_cast<const uint4 *>(u[n] + 2048 + gid * 16);
            const uint4 hB = *reinterpret_cast<const uint4 *>(u[n] + 2048 + (gid + 8) * 16);
            sc[n][0] = hA.y & 0x3F3F3F3Fu; sc[n][1] = (hA.w & 0x0F0F0F0Fu) | ((hA.y >> 2) & 0x30303030u);
            sc[n][2] = hB.y & 0x3F3F3F3Fu; sc[n][3] = (hB.w & 0x0F0F0F0Fu) | ((hB.y >> 2) & 0x30303030u);
#pragma unroll
            for (int i = 0; i < 4; ++i) { T[n][i] = 0; Uh[n][i] = 0; }
        }
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            uint4 bw = make_uint4(0u, 0u, 0u, 0u);
            if (brow_ok) bw = *reinterpret_cast<const uint4 *>(xrow + 64 * pr);
            const int b0 = (2 * pr) & 3, b1 = b0 + 1;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                unsigned q[4];
                load_frag(q, u[n] + pr * 512, lane);
                const unsigned alo[4] = {q[0] & 0x0F0F0F0Fu, q[1] & 0x0F0F0F0Fu, q[2] & 0x0F0F0F0Fu, q[3] & 0x0F0F0F0Fu};
                const unsigned ahi[4] = {q[0] & 0xF0F0F0F0u, q[1] & 0xF0F0F0F0u, q[2] & 0xF0F0F0F0u, q[3] & 0xF0F0F0F0u};
                int dlo[4] = {0, 0, 0, 0}, dhi[4] = {0, 0, 0, 0};
                mma_u8s8_k32(dlo, alo, bw.x, bw.y);
                mma_u8s8_k32(dhi, ahi, bw.z, bw.w);
                const unsigned wA = pr < 2 ? sc[n][0] : sc[n][1], wB = pr < 2 ? sc[n][2] : sc[n][3];
                const int sAl = (int)__byte_perm(wA, 0u, 0x4440 + b0), sAh = (int)__byte_perm(wA, 0u, 0x4440 + b1);
                const int sBl = (int)__byte_perm(wB, 0u, 0x4440 + b0), sBh = (int)__byte_perm(wB, 0u, 0x4440 + b1);
                T[n][0] += sAl * dlo[0]; Uh[n][0] += sAh * dhi[0];
                T[n][1] += sAl * dlo[1]; Uh[n][1] += sAh * dhi[1];
                T[n][2] += sBl * dlo[2]; Uh[n][2] += sBh * dhi[2];
                T[n][3] += sBl * dlo[3]; Uh[n][3] += sBh * dhi[3];
            }
        }
        const float2 g2 = bc.g2;
        const unsigned o = (2 * tig) & 3;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const uint4 hA = *reinterpret_cast<const uint4 *>(u[n] + 2048 + gid * 16);
            const uint4 hB = *reinterpret_cast<const uint4 *>(u[n] + 2048 + (gid + 8) * 16);
#pragma unroll
            for (int i = 0; i < 4; ++i) T[n][i] += Uh[n][i] >> 4;  // exact: Uh is a multiple of 16
            const float dA = half_bits_to_float((unsigned short)(hA.x & 0xffffu));
            const float dB = half_bits_to_float((unsigned short)(hB.x & 0xffffu));
            float aA = dA * fmaf((float)T[n][0], f0, (float)T[n][1] * f1);
            float aB = dB * fmaf((float)T[n][2], f0, (float)T[n][3] * f1);
            // minimum term -dmin * sum_g m_g * sum(x_g): lane tig takes groups 2tig, 2tig+1
            const unsigned mA0 = hA.z & 0x3F3F3F3Fu, mA1 = ((hA.w >> 4) & 0x0F0F0F0Fu) | ((hA.z >> 2) & 0x30303030u);
            const unsigned mB0 = hB.z & 0x3F3F3F3Fu, mB1 = ((hB.w >> 4) & 0x0F0F0F0Fu) | ((hB.z >> 2) & 0x30303030u);
            const float dmA = half_bits_to_float((unsigned short)(hA.x >> 16));
            const float dmB = half_bits_to_float((unsigned short)(hB.x >> 16));
            const unsigned wA = tig < 2 ? mA0 : mA1, wB = tig < 2 ? mB0 : mB1;
            const float bA = fmaf((float)__byte_perm(wA, 0u, 0x4440 + o + 1), g2.y, (float)__byte_perm(wA, 0u, 0x4440 + o) * g2.x);
            const float bB = fmaf((float)__byte_perm(wB, 0u, 0x4440 + o + 1), g2.y, (float)__byte_perm(wB, 0u, 0x4440 + o) * g2.x);
            acc[n][0] = fmaf(-dmA, bA, aA);
            acc[n][1] = fmaf(-dmB, bB, aB);
        }
    } else {
        int T[NT][4];
        uint4 sA[NT], sB[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            sA[n] = *reinterpret_cast<const uint4 *>(u[n] + 3072 + gid * 16);
            sB[n] = *reinterpret_cast<const uint4 *>(u[n] + 3072 + (gid + 8) * 16);
#pragma unroll
            for (int i = 0; i < 4; ++i) T[n][i] = 0;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            unsigned qh[NT][4];
#pragma unroll
            for (int n = 0; n < NT; ++n) load_frag(qh[n], u[n] + 2048 + h * 512, lane);
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
                unsigned ql[NT][4];
#pragma unroll
                for (int n = 0; n < NT; ++n) load_frag(ql[n], u[n] + (2 * h + c2) * 512, lane);
#pragma unroll
                for (int hiq = 0; hiq < 2; ++hiq) {
                    const int Q = c2 + 2 * hiq;  // quarter: ql chunk c2, nibble hiq
                    uint2 bw = make_uint2(0u, 0u);
                    if (brow_ok) bw = *reinterpret_cast<const uint2 *>(xrow + (2 * h + (Q >> 1)) * 64 + 8 * (Q & 1));
                    const int g = h * 8 + Q * 2;  // first of the two 16-value scale groups
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        unsigned a[4];
#define FYB_Q6(QQ) for (int i = 0; i < 4; ++i) a[i] = q6_signed<QQ>(ql[n][i], qh[n][i]);
                        if (Q == 0) { FYB_Q6(0) } else if (Q == 1) { FYB_Q6(1) } else if (Q == 2) { FYB_Q6(2) } else { FYB_Q6(3) }
#undef FYB_Q6
                        int d1[4] = {0, 0, 0, 0}, d2[4] = {0, 0, 0, 0};
                        asm volatile(
                            "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                            : "+r"(d1[0]), "+r"(d1[1]), "+r"(d1[2]), "+r"(d1[3]) : "r"(a[0]), "r"(a[1]), "r"(bw.x));
                        asm volatile(
                            "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                            : "+r"(d2[0]), "+r"(d2[1]), "+r"(d2[2]), "+r"(d2[3]) : "r"(a[2]), "r"(a[3]), "r"(bw.y));
                        const unsigned wA = (&sA[n].x)[g >> 2], wB = (&sB[n].x)[g >> 2];
                        const int s1A = sbyte(wA, g & 3), s2A = sbyte(wA, (g & 3) + 1);
                        const int s1B = sbyte(wB, g & 3), s2B = sbyte(wB, (g & 3) + 1);
                        T[n][0] += s1A * d1[0] + s2A * d2[0];
                        T[n][1] += s1A * d1[1] + s2A * d2[1];
                        T[n][2] += s1B * d1[2] + s2B * d2[2];
                        T[n][3] += s1B * d1[3] + s2B * d2[3];
                    }
                }
            }
        }
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const float dA = half_bits_to_float(*reinterpret_cast<const unsigned short *>(u[n] + 3328 + gid * 2));
            const float dB = half_bits_to_float(*reinterpret_cast<const unsigned short *>(u[n] + 3328 + (gid + 8) * 2));
            acc[n][0] = dA * fmaf((float)T[n][0], f0, (float)T[n][1] * f1);
            acc[n][1] = dB * fmaf((float)T[n][2], f0, (float)T[n][3] * f1);
        }
    }
}

// One unit against NPP vector pairs (vectors 2pp, 2pp + 1 of pair pp; their
// limb rows are pair * 8 + limb of xl, as compute_unit<TYPE, 2> reads one
// pair): the weight fragments, masks and scale bytes are formed once per
// 32-column chunk and used by every pair's MMAs. Pair pp's exponents and
// group sums are at exps + pp * 2 * nblk and gsums + pp * 2 * ngroups.
// acc[pp][0] / acc[pp][1] accumulate as compute_unit<TYPE, 2>'s accA / accB.
template <unsigned TYPE, int NPP>
FYB_DEV void compute_pairs(const unsigned char *u, unsigned blk, const signed char *xl, unsigned xstride,
    const int *exps, unsigned nblk, const float *gsums, unsigned ngroups, unsigned lane, float (&acc)[NPP][2])
{
    const unsigned gid = lane >> 2, tig = lane & 3, vec = tig >> 1;
    const int l0 = 2 * (tig & 1);
    const signed char *xrow = xl + (size_t)gid * xstride + blk * 256u + tig * 16u;
    int T[NPP][4];
#pragma unroll
    for (int n = 0; n < NPP; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) T[n][i] = 0;
    if constexpr (TYPE == T_Q4_K) {
        const uint4 hA = *reinterpret_cast<const uint4 *>(u + 2048 + gid * 16);
        const uint4 hB = *reinterpret_cast<const uint4 *>(u + 2048 + (gid + 8) * 16);
        const unsigned scA0 = hA.y & 0x3F3F3F3Fu, scA1 = (hA.w & 0x0F0F0F0Fu) | ((hA.y >> 2) & 0x30303030u);
        const unsigned scB0 = hB.y & 0x3F3F3F3Fu, scB1 = (hB.w & 0x0F0F0F0Fu) | ((hB.y >> 2) & 0x30303030u);
        int Uh[NPP][4];
#pragma unroll
        for (int n = 0; n < NPP; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) Uh[n][i] = 0;
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            unsigned q[4];
            load_frag(q, u + pr * 512, lane);
            const unsigned alo[4] = {q[0] & 0x0F0F0F0Fu, q[1] & 0x0F0F0F0Fu, q[2] & 0x0F0F0F0Fu, q[3] & 0x0F0F0F0Fu};
            const unsigned ahi[4] = {q[0] & 0xF0F0F0F0u, q[1] & 0xF0F0F0F0u, q[2] & 0xF0F0F0F0u, q[3] & 0xF0F0F0F0u};
            const unsigned wA = pr < 2 ? scA0 : scA1, wB = pr < 2 ? scB0 : scB1;
            const int b0 = (2 * pr) & 3, b1 = b0 + 1;
            const int sAl = (int)__byte_perm(wA, 0u, 0x4440 + b0), sAh = (int)__byte_perm(wA, 0u, 0x4440 + b1);
            const int sBl = (int)__byte_perm(wB, 0u, 0x4440 + b0), sBh = (int)__byte_perm(wB, 0u, 0x4440 + b1);
#pragma unroll
            for (int n = 0; n < NPP; ++n) {
                const uint4 bw = *reinterpret_cast<const uint4 *>(xrow + (size_t)n * 8 * xstride + 64 * pr);
                int dlo[4] = {0, 0, 0, 0}, dhi[4] = {0, 0, 0, 0};
                mma_u8s8_k32(dlo, alo, bw.x, bw.y);
                mma_u8s8_k32(dhi, ahi, bw.z, bw.w);
                T[n][0] += sAl * dlo[0]; Uh[n][0] += sAh * dhi[0];
                T[n][1] += sAl * dlo[1]; Uh[n][1] += sAh * dhi[1];
                T[n][2] += sBl * dlo[2]; Uh[n][2] += sBh * dhi[2];
                T[n][3] += sBl * dlo[3]; Uh[n][3] += sBh * dhi[3];
            }
        }
        const float dA = half_bits_to_float((unsigned short)(hA.x & 0xffffu));
        const float dB = half_bits_to_float((unsigned short)(hB.x & 0xffffu));
        const float dmA = half_bits_to_float((unsigned short)(hA.x >> 16));
        const float dmB = half_bits_to_float((unsigned short)(hB.x >> 16));
        const unsigned mA0 = hA.z & 0x3F3F3F3Fu, mA1 = ((hA.w >> 4) & 0x0F0F0F0Fu) | ((hA.z >> 2) & 0x30303030u);
        const unsigned mB0 = hB.z & 0x3F3F3F3Fu, mB1 = ((hB.w >> 4) & 0x0F0F0F0Fu) | ((hB.z >> 2) & 0x30303030u);
        const unsigned wmA = (tig & 1) ? mA1 : mA0, wmB = (tig & 1) ? mB1 : mB0;
        const float mA[4] = {(float)__byte_perm(wmA, 0u, 0x4440), (float)__byte_perm(wmA, 0u, 0x4441),
                             (float)__byte_perm(wmA, 0u, 0x4442), (float)__byte_perm(wmA, 0u, 0x4443)};
        const float mB[4] = {(float)__byte_perm(wmB, 0u, 0x4440), (float)__byte_perm(wmB, 0u, 0x4441),
                             (float)__byte_perm(wmB, 0u, 0x4442), (float)__byte_perm(wmB, 0u, 0x4443)};
#pragma unroll
        for (int n = 0; n < NPP; ++n) {
#pragma unroll
            for (int i = 0; i < 4; ++i) T[n][i] += Uh[n][i] >> 4;  // exact: Uh is a multiple of 16
            const int E = exps[n * 2 * nblk + vec * nblk + blk];
            const float f0 = pow2f(E - 6 - 7 * l0), f1 = pow2f(E - 6 - 7 * (l0 + 1));
            acc[n][0] = fmaf(dA, fmaf((float)T[n][0], f0, (float)T[n][1] * f1), acc[n][0]);
            acc[n][1] = fmaf(dB, fmaf((float)T[n][2], f0, (float)T[n][3] * f1), acc[n][1]);
            // minimum term: the two lanes of a vector take groups 4(tig&1)..+3
            const float4 g4 = *reinterpret_cast<const float4 *>(gsums + (size_t)n * 2 * ngroups + vec * ngroups +
                                                                 blk * 8 + 4 * (tig & 1));
            float bA = mA[0] * g4.x, bB = mB[0] * g4.x;
            bA = fmaf(mA[1], g4.y, bA); bB = fmaf(mB[1], g4.y, bB);
            bA = fmaf(mA[2], g4.z, bA); bB = fmaf(mB[2], g4.z, bB);
            bA = fmaf(mA[3], g4.w, bA); bB = fmaf(mB[3], g4.w, bB);
            acc[n][0] = fmaf(-dmA, bA, acc[n][0]);
            acc[n][1] = fmaf(-dmB, bB, acc[n][1]);
        }
    } else {
        const uint4 sA = *reinterpret_cast<const uint4 *>(u + 3072 + gid * 16);
        const uint4 sB = *reinterpret_cast<const uint4 *>(u + 3072 + (gid + 8) * 16);
        const float dA = half_bits_to_float(*reinterpret_cast<const unsigned short *>(u + 3328 + gid * 2));
        const float dB = half_bits_to_float(*reinterpret_cast<const unsigned short *>(u + 3328 + (gid + 8) * 2));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            unsigned qh[4];
            load_frag(qh, u + 2048 + h * 512, lane);
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
                unsigned ql[4];
                load_frag(ql, u + (2 * h + c2) * 512, lane);
#pragma unroll
                for (int hiq = 0; hiq < 2; ++hiq) {
                    const int Q = c2 + 2 * hiq;
                    unsigned a[4];
#define FYB_Q6(QQ) for (int i = 0; i < 4; ++i) a[i] = q6_signed<QQ>(ql[i], qh[i]);
                    if (Q == 0) { FYB_Q6(0) } else if (Q == 1) { FYB_Q6(1) } else if (Q == 2) { FYB_Q6(2) } else { FYB_Q6(3) }
#undef FYB_Q6
                    const int g = h * 8 + Q * 2;
                    const unsigned wA = (&sA.x)[g >> 2], wB = (&sB.x)[g >> 2];
                    const int s1A = sbyte(wA, g & 3), s2A = sbyte(wA, (g & 3) + 1);
                    const int s1B = sbyte(wB, g & 3), s2B = sbyte(wB, (g & 3) + 1);
#pragma unroll
                    for (int n = 0; n < NPP; ++n) {
                        const uint2 bw = *reinterpret_cast<const uint2 *>(xrow + (size_t)n * 8 * xstride +
                                                                          (2 * h + (Q >> 1)) * 64 + 8 * (Q & 1));
                        int d1[4] = {0, 0, 0, 0}, d2[4] = {0, 0, 0, 0};
                        asm volatile(
                            "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                            : "+r"(d1[0]), "+r"(d1[1]), "+r"(d1[2]), "+r"(d1[3]) : "r"(a[0]), "r"(a[1]), "r"(bw.x));
                        asm volatile(
                            "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                            : "+r"(d2[0]), "+r"(d2[1]), "+r"(d2[2]), "+r"(d2[3]) : "r"(a[2]), "r"(a[3]), "r"(bw.y));
                        T[n][0] += s1A * d1[0] + s2A * d2[0];
                        T[n][1] += s1A * d1[1] + s2A * d2[1];
                        T[n][2] += s1B * d1[2] + s2B * d2[2];
                        T[n][3] += s1B * d1[3] + s2B * d2[3];
                    }
                }
            }
        }
#pragma unroll
        for (int n = 0; n < NPP; ++n) {
            const int E = exps[n * 2 * nblk + vec * nblk + blk];
            const float f0 = pow2f(E - 6 - 7 * l0), f1 = pow2f(E - 6 - 7 * (l0 + 1));
            acc[n][0] = fmaf(dA, fmaf((float)T[n][0], f0, (float)T[n][1] * f1), acc[n][0]);
            acc[n][1] = fmaf(dB, fmaf((float)T[n][2], f0, (float)T[n][3] * f1), acc[n][1]);
        }
        (void)gsums; (void)ngroups;
    }
}

// Sum of a lane's tile accumulator over the lanes that share its vector.
template <int NV>
FYB_DEV float lane_total(float acc)
{
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    if constexpr (NV == 1) acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    return acc;
}

FYB_DEV double block_sum_double(double v, double *red)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = 0;
    for (int w = 0; w < QG_WARPS; ++w) t += red[w];
    return t;
}

// Sum of the partial slots of the warps that share a stream-K tile. The
// `ways` lanes that need the same values split the slots (slot s goes to the
// lane with part == s % ways) and keep four slots' loads in flight at once;
// has_units(s) tells whether the warp of slot s wrote it. The caller adds the
// `ways` partial sums with shuffles, so the order is fixed by the geometry.
template <class HasUnits>
FYB_DEV void sum_slots(const float *base, unsigned slot_floats, unsigned offA, unsigned offB, unsigned nslots,
    unsigned part, unsigned ways, HasUnits has_units, float &yA, float &yB)
{
    float a = 0.f, b = 0.f;
    for (unsigned s0 = part; s0 < nslots; s0 += 4 * ways) {
        float va[4], vb[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const unsigned s = s0 + j * ways;
            const bool ok = s < nslots && has_units(s);
            va[j] = ok ? __ldcg(base + (size_t)s * slot_floats + offA) : 0.f;
            vb[j] = ok ? __ldcg(base + (size_t)s * slot_floats + offB) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) { a += va[j]; b += vb[j]; }
    }
    yA = a;
    yB = b;
}

FYB_DEV void load16(const float *src, float (&v)[16])
{
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 t = __ldcg(s4 + i);
        v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
}

// Limb split of one 16-value slot `sl` of vector `v` (x already residual-
// added and normalized): fp32 group sums (pairs of slots, adjacent lanes),
// the block exponent (16 slots = 16 adjacent lanes) and four signed limbs.
// Every lane of the warp must call it (shuffles); `ok` marks real slots.
FYB_DEV void prep_slot(float (&x)[16], bool ok, unsigned v, unsigned sl, unsigned K, unsigned nblk, signed char *xl,
    unsigned xstride, int *exps, float *gsums, unsigned *error)
{
        float gs = 0.f, mx = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) { gs = __fadd_rn(gs, x[j]); mx = fmaxf(mx, fabsf(x[j])); }
        const float other = __shfl_xor_sync(0xffffffffu, gs, 1);
        if (ok && (sl & 1) == 0) gsums[v * (K / 32) + sl / 2] = __fadd_rn(gs, other);
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        int E = 0;
        const bool bad = !(mx <= 3.0e38f);  // inf or NaN in the block
        if (!bad && mx > 0.f) {
            frexpf(mx, &E);
            if (E < -120) E = -120;  // below 2^-121 the limbs round to zero anyway
        }
        if (ok && (sl & 15) == 0) exps[v * nblk + sl / 16] = E;
        if (ok && bad && error) *(volatile unsigned *)error = ERR_NONFINITE;
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
            // slot sl = natural words 4a..4a+3 of its chunk (a = sl % 4): stored at 4t + a
            const unsigned chunk = (sl >> 2) * 64u, a4 = (sl & 3u) * 4u;
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                signed char *row = xl + (size_t)(v * 4 + l) * xstride + chunk + a4;
#pragma unroll
                for (int t = 0; t < 4; ++t) *reinterpret_cast<unsigned *>(row + 16 * t) = words[l][t];
            }
        }
}

}  // namespace fyb
