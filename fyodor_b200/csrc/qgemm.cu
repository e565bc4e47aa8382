// qgemm.cu - weight-reusing small-batch GEMM on the integer tensor cores:
// Y[v][r] = sum_k W[r][k] X[v][k] for 3..16 input vectors (the engine's
// matmul, backend/include/compute.h:80-83; its reference small-batch path
// keeps one weight pass per batch, CUDA/gemm.cu:53-95). Two kernels, both
// reading every weight unit from HBM once per call: qgemm_kernel (legacy
// mma.sync integer MMAs, below) for the smaller batches and qgemm_tc_kernel
// (tcgen05 with the operand in tensor memory, further down) from
// tc_min_nv(type) vectors on; launch_qgemm picks between them.
//
// qgemm_kernel: every weight unit (16 rows x 256 columns, repacked as for the GEMV) is
// read from HBM once per call and multiplied against all vectors while it
// sits in shared memory: the x limbs of all vectors are B operands next to
// each other (two vectors x four limbs per m16n8 MMA), so one unit feeds
// ceil(v / 2) MMA column groups. The same unit math as the GEMV keeps the
// results exact to fp32 rounding (compute_unit<TYPE, 2> per vector pair).
//
// Shared memory cannot hold the limbs of 16 vectors over the whole K, so K
// is cut into slices of `nbs` 256-column blocks: CTA c works on slice
// c % KS for tile group c / KS (the same tile ranges in every slice). A CTA
// splits the limbs of its slice once, then its warps stream contiguous
// ranges of (tile, block) units in tile-major order through per-warp
// bulk-copy rings; a tile split between warps meets in shared-memory slots
// and is summed in warp order. With more than one slice the CTA writes its
// partial rows to a scratch area and the last CTA of a tile group (atomic
// count) adds the slices in slice order, so results do not depend on timing.
#include "qgemv_core.cuh"
#include <cstdio>
#include <cstdlib>

namespace fyb {

constexpr unsigned QM_MAX_PAIRS = 8;  // 16 vectors
constexpr unsigned QM_RING = 2 * Q6_UNIT;  // per-warp ring: two units of either type

struct QmParams {
    const unsigned char *units;
    unsigned rows, K, nblk, tiles, nv, np;  // np: vector pairs (ceil(nv / 2))
    unsigned nbs, KS, G;                    // blocks per slice, slices, tile groups
    const float *x;                         // [nv][K]
    float *y;                               // [nv][out_stride]
    unsigned long long out_stride;
    float *scratch;                         // [KS][tiles * 16][np * 2] when KS > 1
    unsigned *counters;                     // [G], zero between launches
    unsigned *error;
};

struct QmSmem {
    size_t xl, exps, gsums, slots, rings, bars, stile, misc, total;
    unsigned xstride;
};

FYB_HOST_DEV QmSmem qm_smem(unsigned np, unsigned nbs)
{
    QmSmem s;
    s.xstride = nbs * 256 + QG_XPAD;
    s.xl = 0;
    s.exps = s.xl + (size_t)np * 8 * s.xstride;
    s.gsums = s.exps + ((size_t)np * 2 * nbs * 4 + 15) / 16 * 16;
    s.slots = s.gsums + ((size_t)np * 2 * nbs * 8 * 4 + 15) / 16 * 16;
    s.rings = s.slots + (size_t)QG_WARPS * 2 * 16 * np * 2 * 4;
    s.bars = s.rings + (size_t)QG_WARPS * QM_RING;
    s.stile = s.bars + (size_t)QG_WARPS * 2 * 8;
    s.misc = s.stile + (size_t)QG_WARPS * 2 * 4;
    s.total = s.misc + 16;
    return s;
}

// Slice size: the most 256-column blocks whose limbs fit next to the rings
// and slots, then the fewest slices that cover K.
static unsigned qm_blocks_per_slice(unsigned np, unsigned nblk)
{
    unsigned nbs = nblk;
    while (nbs > 1 && qm_smem(np, nbs).total > 227 * 1024) --nbs;
    return nbs;
}

template <unsigned TYPE>
__global__ void __launch_bounds__(QG_THREADS, 1) qgemm_kernel(const QmParams p)
{
    extern __shared__ __align__(1024) unsigned char smem[];
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, tig = lane & 3;
    const unsigned s = blockIdx.x % p.KS, j = blockIdx.x / p.KS;
    if (j >= p.G) return;
    const QmSmem L = qm_smem(p.np, p.nbs);
    signed char *xl = reinterpret_cast<signed char *>(smem + L.xl);
    int *exps = reinterpret_cast<int *>(smem + L.exps);
    float *gsums = reinterpret_cast<float *>(smem + L.gsums);
    float *slots = reinterpret_cast<float *>(smem + L.slots);  // [warp][2][16 rows][np * 2]
    unsigned char *ring = smem + L.rings + (size_t)warp * QM_RING;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars) + warp * 2;
    unsigned *flag = reinterpret_cast<unsigned *>(smem + L.misc);
    unsigned *stile = reinterpret_cast<unsigned *>(smem + L.stile);  // [warp][2] tile held by each slot
    const unsigned b0 = s * p.nbs, nb = min(p.nbs, p.nblk - b0);
    const unsigned tb = (unsigned)((unsigned long long)p.tiles * j / p.G);
    const unsigned te = (unsigned)((unsigned long long)p.tiles * (j + 1) / p.G);
    const unsigned U = (te - tb) * nb;
    const unsigned ua = U * warp / QG_WARPS, n = U * (warp + 1) / QG_WARPS - ua;
    const unsigned ub = unit_bytes(TYPE), S = QM_RING / ub;

    // the warp's first units are requested before the limbs are split
    if (lane == 0) {
        for (unsigned k = 0; k < 2; ++k) mbar_init(bars + k, 1);
        fence_barrier_init();
        stile[warp * 2] = stile[warp * 2 + 1] = ~0u;
    }
    __syncwarp();
    auto unit_src = [&](unsigned k) {
        const unsigned u = ua + k, t = tb + u / nb, bl = u % nb;
        return p.units + ((unsigned long long)t * p.nblk + b0 + bl) * ub;
    };
    unsigned issued = 0, consumed = 0, par = 0;
    for (; issued < n && issued < S; ++issued)
        if (lane == 0) {
            mbar_expect_tx(bars + issued, ub);
            bulk_copy_g2s(ring + issued * ub, unit_src(issued), ub, bars + issued);
        }

    // limbs of the slice: vector v (zero past nv), 16-value slot sl
    const unsigned nslot = nb * 16, vtot = p.np * 2, Ks = nb * 256;
    for (unsigned s0 = 0; s0 < vtot * nslot; s0 += QG_THREADS) {
        const unsigned i = s0 + threadIdx.x;
        const bool ok = i < vtot * nslot;
        const unsigned v = ok ? i / nslot : 0, sl = ok ? i % nslot : 0;
        float x[16];
        if (ok && v < p.nv) load16(p.x + (size_t)v * p.K + (size_t)b0 * 256 + 16 * sl, x);
        else {
#pragma unroll
            for (int q = 0; q < 16; ++q) x[q] = 0.f;
        }
        prep_slot(x, ok, v, sl, Ks, nb, xl, L.xstride, exps, gsums, p.error);
    }
    __syncthreads();

    // units, tile-major; a tile's value builds up in the lane's accumulators
    float acc[QM_MAX_PAIRS][2];
#pragma unroll
    for (unsigned pp = 0; pp < QM_MAX_PAIRS; ++pp) acc[pp][0] = acc[pp][1] = 0.f;
    float *myslot = slots + (size_t)warp * 2 * 16 * p.np * 2;
    unsigned nslots_used = 0;
    unsigned tile = tb + ua / nb, bl = ua % nb, tile_units = 0;
    bool ok = true;
    auto emit = [&](unsigned t, bool whole) {
        // lanes tig 0 and 2 hold vectors 2pp and 2pp + 1 (their pair partner tig ^ 1 is added)
#pragma unroll
        for (unsigned pp = 0; pp < QM_MAX_PAIRS; ++pp) {
            if (pp >= p.np) break;
            const float yA = acc[pp][0] + __shfl_xor_sync(0xffffffffu, acc[pp][0], 1);
            const float yB = acc[pp][1] + __shfl_xor_sync(0xffffffffu, acc[pp][1], 1);
            const unsigned v = 2 * pp + (tig >> 1);
            if ((tig & 1) == 0) {
                if (whole) {
                    const unsigned rA = t * 16 + gid, rB = rA + 8;
                    if (p.KS == 1) {
                        if (v < p.nv && rA < p.rows) p.y[v * p.out_stride + rA] = yA;
                        if (v < p.nv && rB < p.rows) p.y[v * p.out_stride + rB] = yB;
                    } else {
                        float *sc = p.scratch + ((size_t)s * p.tiles * 16) * vtot;
                        sc[(size_t)rA * vtot + v] = yA;
                        sc[(size_t)rB * vtot + v] = yB;
                    }
                } else {
                    float *sl = myslot + (size_t)nslots_used * 16 * vtot;
                    sl[gid * vtot + v] = yA;
                    sl[(gid + 8) * vtot + v] = yB;
                }
            }
            acc[pp][0] = acc[pp][1] = 0.f;
        }
    };
    unsigned slot_tile[2] = {~0u, ~0u}, slot_last[2] = {0, 0};
    for (unsigned k = 0; k < n; ++k) {
        const unsigned sidx = consumed % S;
        const bool landed = mbar_wait_bounded(bars + sidx, (par >> sidx) & 1u);
        if (!__all_sync(0xffffffffu, landed)) {
            if (lane == 0 && p.error) atomicCAS(p.error, 0u, (unsigned)ERR_TIMEOUT);
            ok = false;
            break;
        }
        par ^= 1u << sidx;
        ++consumed;
        const unsigned char *u = ring + sidx * ub;
        // vector pairs two at a time: the unit's weight fragments are formed
        // once per two pairs
#pragma unroll
        for (unsigned g2 = 0; g2 < QM_MAX_PAIRS; g2 += 2) {
            if (g2 >= p.np) break;
            if (p.np - g2 >= 2) {
                float a2[2][2] = {{acc[g2][0], acc[g2][1]}, {acc[g2 + 1][0], acc[g2 + 1][1]}};
                compute_pairs<TYPE, 2>(u, bl, xl + (size_t)g2 * 8 * L.xstride, L.xstride, exps + g2 * 2 * nb, nb,
                                       gsums + g2 * 2 * nb * 8, nb * 8, lane, a2);
                acc[g2][0] = a2[0][0]; acc[g2][1] = a2[0][1];
                acc[g2 + 1][0] = a2[1][0]; acc[g2 + 1][1] = a2[1][1];
            } else {
                compute_unit<TYPE, 2>(u, bl, xl + (size_t)g2 * 8 * L.xstride, L.xstride, exps + g2 * 2 * nb, nb,
                                      gsums + g2 * 2 * nb * 8, nb * 8, lane, acc[g2][0], acc[g2][1]);
            }
        }
        __syncwarp();
        if (issued < n) {
            const unsigned s2 = issued % S;
            if (lane == 0) {
                mbar_expect_tx(bars + s2, ub);
                bulk_copy_g2s(ring + s2 * ub, unit_src(issued), ub, bars + s2);
            }
            ++issued;
        }
        ++tile_units;
        const bool tile_end = bl + 1 == nb;
        bl = tile_end ? 0 : bl + 1;
        if (!tile_end && k + 1 != n) continue;
        if (tile_units == nb) {
            emit(tile, true);
        } else if (nslots_used < 2) {  // only the first and the last tile of a range can be shared
            slot_tile[nslots_used] = tile;
            slot_last[nslots_used] = tile_end ? 1u : 0u;
            if (lane == 0) stile[warp * 2 + nslots_used] = tile;
            emit(tile, false);
            ++nslots_used;
        }
        tile_units = 0;
        if (tile_end) ++tile;
    }
    // let copies still in flight land before leaving (bounded)
    while (consumed != issued) {
        const unsigned sidx = consumed % S;
        if (!mbar_wait_bounded(bars + sidx, (par >> sidx) & 1u)) break;
        par ^= 1u << sidx;
        ++consumed;
    }
    __syncthreads();
    // shared tiles: the warp holding a tile's last unit adds every warp's part in warp order
    for (unsigned q2 = 0; q2 < 2 && ok; ++q2) {
        if (slot_tile[q2] == ~0u || !slot_last[q2]) continue;
        const unsigned t = slot_tile[q2];
        for (unsigned i = lane; i < 16 * vtot; i += 32) {
            const unsigned row = i / vtot, v = i % vtot;
            float y = 0.f;
            for (unsigned w = 0; w <= warp; ++w)
                for (unsigned sq = 0; sq < 2; ++sq)
                    if (stile[w * 2 + sq] == t) y += slots[((size_t)w * 2 + sq) * 16 * vtot + row * vtot + v];
            const unsigned r = t * 16 + row;
            if (p.KS == 1) {
                if (v < p.nv && r < p.rows) p.y[v * p.out_stride + r] = y;
            } else {
                p.scratch[((size_t)s * p.tiles * 16 + r) * vtot + v] = y;
            }
        }
    }
    if (p.KS == 1) return;
    // slices: the last CTA of the tile group adds them in slice order
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *flag = atomicAdd(p.counters + j, 1u) == p.KS - 1;
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    const unsigned r0 = tb * 16, r1 = min(te * 16, p.rows);
    for (unsigned i = threadIdx.x; i < (r1 - r0) * p.nv; i += QG_THREADS) {
        const unsigned r = r0 + i / p.nv, v = i % p.nv;
        float y = 0.f;
        for (unsigned q = 0; q < p.KS; ++q) y += __ldcg(p.scratch + ((size_t)q * p.tiles * 16 + r) * vtot + v);
        p.y[v * p.out_stride + r] = y;
    }
    if (threadIdx.x == 0) p.counters[j] = 0;  // read again only by the next launch
}

// Layout of a launch: slices, groups and the scratch bytes (0 with one slice).
static QmParams qm_plan(unsigned type, unsigned rows, unsigned cols, unsigned nv, int sms, size_t *scratch_bytes,
    size_t *counters)
{
    QmParams p = {};
    p.rows = rows; p.K = cols; p.nblk = cols / 256; p.tiles = (rows + 15) / 16;
    p.nv = nv; p.np = (nv + 1) / 2;
    p.nbs = qm_blocks_per_slice(p.np, p.nblk);
    p.KS = (p.nblk + p.nbs - 1) / p.nbs;
    p.G = std::max(1u, std::min((unsigned)sms / p.KS, p.tiles));
    if (p.KS > (unsigned)sms) p.G = 0;
    *scratch_bytes = p.KS > 1 ? (size_t)p.KS * p.tiles * 16 * p.np * 2 * sizeof(float) : 0;
    *counters = p.G;
    (void)type;
    return p;
}

// Workspace: [tile-group counters at a fixed offset][slice scratch]. The
// counters sit first so that calls with other vector counts (other slice
// layouts) never find scratch values where they keep their counts.
constexpr size_t QM_COUNTER_BYTES = 4096;  // up to 1024 tile groups

// ===========================================================================
// The same product on the 5th-generation tensor cores (tcgen05), for
// tc_min_nv(type)..16 vectors. A first small kernel (tc_limbs_kernel) splits the
// vectors once into the B operand of every 256-column block: four signed
// 7-bit limbs per value (the split of the mma.sync path), stored as
// canonical K-major core matrices, followed by the block's x constants
// (limb scales, 32-value group sums, limb sums). The GEMM kernel then runs one
// CTA per SM as a warp-specialized pipeline over items; an item is one
// M-tile of 128 weight rows (8 unit tiles) times one block of the CTA's K
// slice:
//  - producer (warp 0, one thread): bulk-copies the item's 8 units into a
//    unit ring stage, freed as soon as staging has read it, and the block's
//    B operand with its x constants into a B ring stage, freed once the MMAs
//    that read it and the epilogue are done (full / empty mbarriers per
//    stage; the two rings advance independently). With programmatic
//    dependent launch it starts streaming weights while the limb kernel
//    still runs and waits for that kernel only before the first B copy;
//  - staging (warps 2-9, two threads per row, each four of the eight
//    groups): form the scaled weights A' = s q of the row as two byte planes
//    in one of four operand half-buffers in tensor memory (tcgen05.st;
//    two halves of 128 columns per item), so neither the staging nor the MMA
//    moves the 2-byte-per-weight operand through shared memory. Q4_K: s = 8 s_hi + s_lo with 3-bit parts, plane p = s_p q <= 105,
//    one integer multiply per four packed nibbles (no carries between
//    bytes); Q6_K: s (q - 32) + 8192 in 16-bit lanes split into its two
//    bytes. They also copy the row's block constants (d, dmin, minimums) to a
//    small buffer for the epilogue, so the unit stage is free as soon as the
//    item is staged;
//  - MMA (warp 1, one thread): tcgen05.mma kind::i8 (u8 A from TMEM x s8 B
//    from shared memory, M 128,
//    N = 4 limbs x padded vectors, K 32) per 32-value group and plane into
//    one of four TMEM accumulators (the eight groups of a block accumulate in
//    TMEM, so the group scales cost no epilogue work); tcgen05.commit frees
//    the operand buffer and hands the accumulator to the epilogue;
//  - epilogue (warps 10-17: a row and half of the vectors per thread; warp
//    w reads TMEM lanes 32 (w % 4)..+31): tcgen05.ld of its row, planes and
//    limbs combined in integer (Q4_K: T = lo + 8 hi, then 128 T0 + T1 and
//    128 T2 + T3, which stay below 2^31), d 2^(E - 6 - 7 limb) and the Q4_K
//    minimum term applied in fp32, the row accumulated over the blocks of
//    the slice in registers.
// Every wait is bounded and polls a shared abort word, so a timeout in one
// role ends the others; the CTA lets its copies and MMAs in flight finish
// before it frees TMEM and leaves. K slices (used when the rows give fewer
// M-tiles than SMs) meet as in qgemm_kernel: partial rows in a scratch area,
// the last CTA of a group adds them in slice order.
constexpr unsigned TC_THREADS = 576;              // 18 warps
constexpr unsigned TC_STAGE0 = 2, TC_NSTAGE = 8;  // staging warps 2..9
constexpr unsigned TC_EPI0 = 10, TC_NEPI = 8;     // epilogue warps 10..17
// Fewest vectors that run on tcgen05; below it the mma.sync kernel is
// faster (measured: Q4_K up to 8 vectors, Q6_K up to 4).
FYB_HOST_DEV unsigned tc_min_nv(unsigned type) { return type == T_Q6_K ? 5u : 9u; }
#ifndef FYB_TC_SLEEP_NS
#define FYB_TC_SLEEP_NS 64
#endif
constexpr unsigned TC_CST = 2048;                 // per item: 128 rows x 16 B

FYB_HOST_DEV unsigned tc_n(unsigned nv) { return nv <= 4 ? 16u : nv <= 8 ? 32u : 64u; }  // 4 limbs x padded vectors
// B block: the MMA's operand [8 groups][N/8 core rows][2 K halves][8][16] s8
// limbs | limb scales [N/4][4] (2^(E - 6 - 7 l) of the block exponent E) |
// group sums [N/4][8] | limb sums [N]
FYB_HOST_DEV constexpr unsigned tc_bop(unsigned N) { return 8 * N * 32; }
FYB_HOST_DEV constexpr unsigned tc_bblk(unsigned N) { return tc_bop(N) + (N / 4) * 16 + (N / 4) * 32 + N * 4; }

struct TcSmem {
    size_t a, ring, bring, cst, bars, misc, total;
};

// rs unit ring stages (8 units each), rb B stages, dc constant buffers,
// barriers for da operand half-buffers and dc accumulators (both in TMEM).
FYB_HOST_DEV TcSmem tc_smem(unsigned type, unsigned N, unsigned rs, unsigned rb, unsigned da, unsigned dc)
{
    TcSmem s;
    s.a = 0;
    s.ring = 0;                                               // [rs][8 units]
    s.bring = s.ring + (size_t)rs * 8 * unit_bytes(type);     // [rb][B block]
    s.cst = s.bring + (size_t)rb * tc_bblk(N);                // [dc][TC_CST]
    s.bars = s.cst + (size_t)dc * TC_CST;
    s.misc = s.bars + (2 * rs + 2 * rb + 2 * da + 4 * dc + 1) * 8;
    s.total = s.misc + 16;
    return s;
}

// TMEM columns (512, one CTA per SM): dc accumulators of 2N columns (two
// planes), then da operand half-buffers of 64 columns (2 planes x 4 groups x
// 32 bytes per row). Four half-buffers; four accumulators, two at N = 64.
// Shared memory: the most unit stages (up to 8), then B stages (up to 4).
struct TcDepth {
    unsigned rs, rb, da, dc;
};
static TcDepth tc_depth(unsigned type, unsigned N)
{
    constexpr size_t cap = 227 * 1024;
    const unsigned da = 4, dc = N == 64 ? 2 : 4;
    for (unsigned rb = 4; rb >= 2; --rb)
        for (unsigned rs = 8; rs >= 3; --rs)
            if (tc_smem(type, N, rs, rb, da, dc).total <= cap && (rs >= 6 || rb == 2)) return {rs, rb, da, dc};
    return {0, 0, 0, 0};
}

struct TcParams {
    const unsigned char *units;
    unsigned rows, K, nblk, tiles, mtiles, nv, N;
    unsigned nbs, KS, G, rs, rb, da, dc;
    const float *x;
    float *y;
    unsigned long long out_stride;
    const unsigned char *bops;  // [nblk][tc_bblk(N)] (tc_limbs_kernel)
    float *scratch;             // [KS][mtiles * 128][N / 4] when KS > 1
    unsigned *counters;         // [G]
    unsigned *error;
};

// Offset of row R, K half kc within one group's 128 x 32 (or N x 32) operand.
FYB_HOST_DEV unsigned tc_core(unsigned R, unsigned kc) { return (R >> 3) * 256 + kc * 128 + (R & 7) * 16; }

// The B block of block blockIdx.x: thread i takes the 16-value slot i % 16
// of vector i / 16 (zero past nv).
template <unsigned N>
__global__ void __launch_bounds__(N * 4) tc_limbs_kernel(const float *x, unsigned K, unsigned nv, unsigned char *bops,
    unsigned *error)
{
    const unsigned bl = blockIdx.x, v = threadIdx.x >> 4, k16 = threadIdx.x & 15;
    unsigned char *out = bops + (size_t)bl * tc_bblk(N);
    float *scl = reinterpret_cast<float *>(out + tc_bop(N));
    float *gsums = reinterpret_cast<float *>(out + tc_bop(N) + (N / 4) * 16);
    int *lsum = reinterpret_cast<int *>(out + tc_bop(N) + (N / 4) * 48);
    float xv[16];
    if (v < nv) load16(x + (size_t)v * K + (size_t)bl * 256 + 16 * k16, xv);
    else {
#pragma unroll
        for (int q = 0; q < 16; ++q) xv[q] = 0.f;
    }
    pdl_launch_dependents();
    float gs = 0.f, mx = 0.f;
#pragma unroll
    for (int q = 0; q < 16; ++q) { gs = __fadd_rn(gs, xv[q]); mx = fmaxf(mx, fabsf(xv[q])); }
    const float other = __shfl_xor_sync(0xffffffffu, gs, 1);
    if ((k16 & 1) == 0) gsums[v * 8 + k16 / 2] = __fadd_rn(gs, other);
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int E = 0;
    const bool bad = !(mx <= 3.0e38f);  // inf or NaN in the block
    if (!bad && mx > 0.f) {
        frexpf(mx, &E);
        if (E < -120) E = -120;  // below 2^-121 the limbs round to zero anyway
    }
    if (k16 < 4) scl[v * 4 + k16] = pow2f(E - 6 - 7 * (int)k16);
    if (bad && error) *(volatile unsigned *)error = ERR_NONFINITE;
    const float sc = pow2f(6 - E);
    unsigned words[4][4];
    int ls[4] = {0, 0, 0, 0};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        unsigned t[4][4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float r = bad ? 0.f : __fmul_rn(xv[4 * q + e], sc);
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const float m = __fadd_rn(r, 12582912.0f);  // rint via the 1.5*2^23 magic
                const float X = __fsub_rn(m, 12582912.0f);
                t[l][e] = __float_as_uint(m);
                ls[l] += (int)X;
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
#pragma unroll
    for (int l = 0; l < 4; ++l)
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) ls[l] += __shfl_xor_sync(0xffffffffu, ls[l], o);
    const unsigned g = k16 / 2, kc = k16 & 1;
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        const unsigned n = 4 * v + l;
        *reinterpret_cast<uint4 *>(out + (size_t)g * N * 32 + tc_core(n, kc)) =
            make_uint4(words[l][0], words[l][1], words[l][2], words[l][3]);
        if (k16 == 0) lsum[n] = ls[l];
    }
}

// K-major canonical operand descriptor: core matrices of 8 rows x 16 bytes,
// the two 16-byte K halves 128 bytes apart (leading offset), 8-row groups
// 256 bytes apart (stride offset), no swizzle, descriptor version 1.
FYB_DEV uint64_t tc_desc(const void *p)
{
    return ((uint64_t)(smem_u32(p) >> 4) & 0x3FFFull) | (8ull << 16) | (16ull << 32) | (1ull << 46);
}
// kind::i8 instruction descriptor: s32 accumulator, A u8, B s8, both
// K-major, N, M = 128.
FYB_HOST_DEV constexpr uint32_t tc_idesc(unsigned N)
{
    return (2u << 4) | (0u << 7) | (1u << 10) | ((N >> 3) << 17) | ((128u >> 4) << 24);
}
FYB_DEV void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate)
{
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n"
                 :: "r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
}
FYB_DEV void tc_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}
FYB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
FYB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// eight consecutive 32-bit columns of this warp's 32 TMEM lanes
FYB_DEV void tc_ld8(uint32_t taddr, int *r)
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr) : "memory");
}
FYB_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// sixteen consecutive 32-bit columns of this thread's TMEM lane
FYB_DEV void tc_st16(uint32_t taddr, const unsigned (&v)[16])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                 "%14, %15, %16};"
                 :: "r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
                    "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
                 : "memory");
}
FYB_DEV void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// D (TMEM) (+)= A (TMEM: row m in lane m, 32 int8 K values in 8 consecutive columns) x B (shared memory)
FYB_DEV void tc_mma_ta(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t accumulate)
{
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}\n"
                 :: "r"(d), "r"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
}
FYB_DEV void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}
FYB_DEV bool mbar_test_wait(uint64_t *bar, unsigned parity)  // non-blocking
{
    unsigned ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait that also gives up when another role raised the abort word.
// After a few polls it sleeps between polls, so waiting warps leave the
// issue slots to the warps that stage operands.
FYB_DEV bool tc_wait(uint64_t *bar, unsigned parity, const volatile unsigned *abort)
{
    for (unsigned i = 0; i < (1u << 22); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && *abort) return false;
        if (i >= 4) __nanosleep(FYB_TC_SLEEP_NS);
    }
    return false;
}

// The same for every lane of a warp (the warp then runs .sync.aligned
// tcgen05 instructions together).
FYB_DEV bool tc_wait_warp(uint64_t *bar, unsigned parity, const volatile unsigned *abort)
{
    return __all_sync(0xffffffffu, tc_wait(bar, parity, abort));
}

// A' = (s - m) q + bias of four packed byte values q < 64 in 16-bit lanes
// (s <= 255; every lane stays in [0, 2^16) before and after the
// subtraction, so no lane borrows from its neighbour), split into its low
// and high bytes.
FYB_DEV void tc_scale4(unsigned q, unsigned s, unsigned bias2, unsigned m, unsigned &lo, unsigned &hi)
{
    const unsigned a = __byte_perm(q, 0u, 0x4140), b = __byte_perm(q, 0u, 0x4342);  // 16-bit lanes
    const unsigned pa = a * s + bias2 - a * m, pb = b * s + bias2 - b * m;
    lo = __byte_perm(pa, pb, 0x6420);
    hi = __byte_perm(pa, pb, 0x7531);
}

template <unsigned TYPE, unsigned N>
__global__ void __launch_bounds__(TC_THREADS, 1) qgemm_tc_kernel(const TcParams p)
{
    constexpr unsigned NV4 = N / 4;        // vector slots
    constexpr unsigned EV = N / 8;         // vectors per epilogue thread
    constexpr unsigned BBLK = tc_bblk(N);
    constexpr unsigned BOP = tc_bop(N);
    constexpr unsigned UB = unit_bytes(TYPE);
    constexpr unsigned NCOLS = 512;         // accumulators and operand buffers
    extern __shared__ __align__(1024) unsigned char smem[];
    const unsigned rs = p.rs, rb = p.rb, da = p.da, dc = p.dc;
    const TcSmem L = tc_smem(TYPE, N, rs, rb, da, dc);
    unsigned char *ring = smem + L.ring;
    unsigned char *bring = smem + L.bring;
    unsigned char *cst = smem + L.cst;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *u_full = bars, *u_empty = u_full + rs, *b_full = u_empty + rs, *b_empty = b_full + rb;
    uint64_t *a_full = b_empty + rb, *a_empty = a_full + da;
    uint64_t *acc_full = a_empty + da, *acc_empty = acc_full + dc, *cst_full = acc_empty + dc, *cst_empty = cst_full + dc;
    uint64_t *drain = cst_empty + dc;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.misc);
    unsigned *flag = reinterpret_cast<unsigned *>(smem + L.misc + 4);
    volatile unsigned *abort = reinterpret_cast<volatile unsigned *>(smem + L.misc + 8);

    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned s = blockIdx.x % p.KS, j = blockIdx.x / p.KS;
    if (j >= p.G) return;
    const unsigned b0 = s * p.nbs, nb = min(p.nbs, p.nblk - b0);
    const unsigned mb = (unsigned)((unsigned long long)p.mtiles * j / p.G);
    const unsigned me = (unsigned)((unsigned long long)p.mtiles * (j + 1) / p.G);
    const unsigned items = (me - mb) * nb;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(NCOLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 32) {
        for (unsigned k = 0; k < rs; ++k) { mbar_init(u_full + k, 1); mbar_init(u_empty + k, TC_NSTAGE); }
        for (unsigned k = 0; k < rb; ++k) { mbar_init(b_full + k, 1); mbar_init(b_empty + k, 1 + TC_NEPI); }
        for (unsigned k = 0; k < da; ++k) {
            mbar_init(a_full + k, TC_NSTAGE);
            mbar_init(a_empty + k, 1);
        }
        for (unsigned k = 0; k < dc; ++k) {
            mbar_init(acc_full + k, 1);
            mbar_init(acc_empty + k, TC_NEPI);
            mbar_init(cst_full + k, TC_NSTAGE);
            mbar_init(cst_empty + k, TC_NEPI);
        }
        mbar_init(drain, 1);
        *abort = 0u;
        fence_barrier_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t acols = dc * 2 * N;  // first TMEM column of the operand half-buffers
    auto fail = [&]() {
        *abort = 1u;
        if (p.error) atomicCAS(p.error, 0u, (unsigned)ERR_TIMEOUT);
    };

    if (warp == 0) {
        // ---------------------------------------------------------- producer
        // two rings served independently: units (freed by staging) and B
        // blocks (freed by the MMAs that read them and the epilogue)
        if (lane == 0) {
            unsigned iu = 0, ib = 0, idle = 0;
            while ((iu < items || ib < items) && !*abort) {
                bool moved = false;
                if (iu < items && (iu < rs || mbar_test_wait(u_empty + iu % rs, (iu / rs - 1) & 1u))) {
                    const unsigned st = iu % rs, mt = mb + iu / nb, bl = iu % nb;
                    const unsigned t0 = mt * 8, nt = min(8u, p.tiles - t0);
                    unsigned char *dst = ring + (size_t)st * 8 * UB;
                    mbar_expect_tx(u_full + st, nt * UB);
                    for (unsigned i = 0; i < nt; ++i)
                        bulk_copy_g2s(dst + i * UB, p.units + ((unsigned long long)(t0 + i) * p.nblk + b0 + bl) * UB, UB,
                                      u_full + st);
                    ++iu;
                    moved = true;
                }
                if (ib < items && (ib < rb || mbar_test_wait(b_empty + ib % rb, (ib / rb - 1) & 1u))) {
                    const unsigned st = ib % rb, bl = ib % nb;
                    if (ib == 0) pdl_wait();  // the limb kernel's output is complete and visible
                    mbar_expect_tx(b_full + st, BBLK);
                    bulk_copy_g2s(bring + (size_t)st * BBLK, p.bops + (size_t)(b0 + bl) * BBLK, BBLK, b_full + st);
                    ++ib;
                    moved = true;
                }
                if (moved) idle = 0;
                else if (++idle > (1u << 24)) { fail(); break; }
                else __nanosleep(32);
            }
            // every issued copy lands before the CTA leaves (bounded)
            for (unsigned st = 0; st < rs && st < iu; ++st) mbar_wait_bounded(u_full + st, ((iu - st - 1) / rs) & 1u);
            for (unsigned st = 0; st < rb && st < ib; ++st) mbar_wait_bounded(b_full + st, ((ib - st - 1) / rb) & 1u);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issue
        if (lane == 0) {
            constexpr uint32_t idesc = tc_idesc(N);
            for (unsigned it = 0; it < items; ++it) {
                const unsigned t = it % dc, sb = it % rb;
                if (it >= dc && !tc_wait(acc_empty + t, (it / dc - 1) & 1u, abort)) { fail(); break; }
                if (!tc_wait(b_full + sb, (it / rb) & 1u, abort)) { fail(); break; }
                tc_fence_after();
                const uint32_t dacc = tmem + t * 2 * N;
                const unsigned char *bb = bring + (size_t)sb * BBLK;
                bool ok = true;
                for (unsigned h = 0; h < 2; ++h) {
                    const unsigned hh = 2 * it + h, ab = hh % da;
                    if (!tc_wait(a_full + ab, (hh / da) & 1u, abort)) { fail(); ok = false; break; }
                    tc_fence_after();
                    const uint32_t ah = tmem + acols + ab * 64;  // plane p, group gl at column 32 p + 8 gl
#pragma unroll
                    for (unsigned gl = 0; gl < 4; ++gl) {
                        const uint64_t bd = tc_desc(bb + (size_t)(4 * h + gl) * N * 32);
                        const uint32_t acc_in = (h | gl) ? 1u : 0u;
                        tc_mma_ta(dacc, ah + gl * 8, bd, idesc, acc_in);
                        tc_mma_ta(dacc + N, ah + 32 + gl * 8, bd, idesc, acc_in);
                    }
                    tc_commit(a_empty + ab);
                }
                if (!ok) break;
                tc_commit(b_empty + sb);
                tc_commit(acc_full + t);
            }
            // every MMA issued has completed before TMEM is freed (bounded)
            tc_commit(drain);
            mbar_wait_bounded(drain, 0);
        }
    } else if (warp < TC_EPI0) {
        // ---------------------------------------------------------- staging
        // warp w writes TMEM lanes 32 (w % 4)..+31: row R, half vh of the groups
        const unsigned q4 = warp & 3u, vh = (warp - TC_STAGE0) >> 2;
        const unsigned R = 32 * q4 + lane, tile = R >> 4, r = R & 15;
        const uint32_t tA = tmem + ((32u * q4) << 16) + acols;
        for (unsigned it = 0; it < items; ++it) {
            const unsigned st = it % rs, mt = mb + it / nb, cb = it % dc;
            if (!tc_wait_warp(u_full + st, (it / rs) & 1u, abort)) { fail(); break; }
            const bool have = mt * 8 + tile < p.tiles;
            const unsigned char *u = ring + (size_t)st * 8 * UB + tile * UB;
            // the row's block constants for the epilogue
            if (it >= dc && !tc_wait_warp(cst_empty + cb, (it / dc - 1) & 1u, abort)) { fail(); break; }
            unsigned char *cb_base = cst + cb * TC_CST;
            uint4 hd = make_uint4(0u, 0u, 0u, 0u);
            if constexpr (TYPE == T_Q4_K) {
                if (have) hd = *reinterpret_cast<const uint4 *>(u + 2048 + r * 16);
                if (vh == 0) {
                    const float d = half_bits_to_float((unsigned short)(hd.x & 0xffffu));
                    const float dmin = half_bits_to_float((unsigned short)(hd.x >> 16));
                    const unsigned m0 = hd.z & 0x3F3F3F3Fu, m1 = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
                    *reinterpret_cast<uint4 *>(cb_base + R * 16) =
                        make_uint4(__float_as_uint(d), __float_as_uint(dmin), m0, m1);
                }
            } else {
                if (vh == 0) {
                    const float d = have ? half_bits_to_float(*reinterpret_cast<const unsigned short *>(u + 3328 + r * 2))
                                         : 0.f;
                    *reinterpret_cast<uint4 *>(cb_base + R * 16) = make_uint4(__float_as_uint(d), 0u, 0u, 0u);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(cst_full + cb);
            bool ok = true;
            for (unsigned h = 0; h < 2; ++h) {
                const unsigned hh = 2 * it + h, ab = hh % da;
                if (hh >= da && !tc_wait_warp(a_empty + ab, (hh / da - 1) & 1u, abort)) { fail(); ok = false; break; }
                unsigned v0[16], v1[16];  // planes 0 and 1: groups 2 vh, 2 vh + 1 of the half (K order)
#pragma unroll
                for (unsigned gi = 0; gi < 2; ++gi) {
                    const unsigned g = 4 * h + 2 * vh + gi, gl = 2 * vh + gi;
#pragma unroll
                    for (unsigned kc = 0; kc < 2; ++kc) {
                        uint4 lo4 = make_uint4(0u, 0u, 0u, 0u), hi4 = make_uint4(0u, 0u, 0u, 0u);
                        if (have) {
                            unsigned lo[4], hi[4];
                            if constexpr (TYPE == T_Q4_K) {
                                const unsigned sw = h ? ((hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u))
                                                      : (hd.y & 0x3F3F3F3Fu);
                                const unsigned sg = __byte_perm(sw, 0u, 0x4440 + gl);
                                const unsigned slo = sg & 7u, shi = sg >> 3;
                                const uint4 q = *reinterpret_cast<const uint4 *>(u + ((g >> 1) * 32 + kc * 16 + r) * 16);
                                const unsigned qa[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const unsigned w = (gi ? (qa[e] >> 4) : qa[e]) & 0x0F0F0F0Fu;
                                    lo[e] = w * slo;  // every byte <= 105: no carry into the next
                                    hi[e] = w * shi;
                                }
                            } else {
                                // value l = 16 kc + e of group g = 4 n2 + qq: ql chunk (2 n2 + (qq & 1), kc),
                                // qh chunk (n2, kc), scale byte 8 n2 + 2 qq + kc
                                const unsigned n2 = h, qq = gl;
                                const uint4 ql = *reinterpret_cast<const uint4 *>(u + ((2 * n2 + (qq & 1)) * 32 + kc * 16 + r) * 16);
                                const uint4 qh = *reinterpret_cast<const uint4 *>(u + 2048 + (n2 * 32 + kc * 16 + r) * 16);
                                const int sgn = (int)(signed char)u[3072 + r * 16 + 8 * n2 + 2 * qq + kc];
                                const unsigned sp = (unsigned)(sgn + 128);         // 0..255
                                const unsigned bias = (unsigned)(8192 - 32 * sgn);  // s (q - 32) + 8192 > 0
                                const unsigned bias2 = bias | (bias << 16);
                                const unsigned qsh = (qq >= 2) ? 4u : 0u, hsh = 2 * qq;
                                const unsigned lq[4] = {ql.x, ql.y, ql.z, ql.w}, hq[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const unsigned w = ((lq[e] >> qsh) & 0x0F0F0F0Fu) | (((hq[e] >> hsh) & 0x03030303u) << 4);
                                    // (s + 128) q - 128 q + 8192 - 32 s = s (q - 32) + 8192
                                    tc_scale4(w, sp, bias2, 128u, lo[e], hi[e]);
                                }
                            }
                            lo4 = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                            hi4 = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        }
                        const unsigned o = gi * 8 + kc * 4;
                        v0[o] = lo4.x; v0[o + 1] = lo4.y; v0[o + 2] = lo4.z; v0[o + 3] = lo4.w;
                        v1[o] = hi4.x; v1[o + 1] = hi4.y; v1[o + 2] = hi4.z; v1[o + 3] = hi4.w;
                    }
                }
                tc_st16(tA + ab * 64 + 16 * vh, v0);
                tc_st16(tA + ab * 64 + 32 + 16 * vh, v1);
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(a_full + ab);
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(u_empty + st);  // the unit stage is read
        }
    } else {
        // ---------------------------------------------------------- epilogue
        const unsigned q4 = warp & 3u, vh = (warp - TC_EPI0) >> 2;
        const unsigned R = 32 * q4 + lane;
        const uint32_t trow = tmem + ((32u * q4) << 16);
        float acc[EV];
#pragma unroll
        for (unsigned q = 0; q < EV; ++q) acc[q] = 0.f;
        for (unsigned it = 0; it < items; ++it) {
            const unsigned t = it % dc, mt = mb + it / nb, bl = it % nb, sb = it % rb;
            // b_full is complete already; waiting on it orders the B block's bytes for these threads
            if (!tc_wait_warp(acc_full + t, (it / dc) & 1u, abort) || !tc_wait_warp(cst_full + t, (it / dc) & 1u, abort) ||
                !tc_wait_warp(b_full + sb, (it / rb) & 1u, abort)) {
                fail();
                break;
            }
            tc_fence_after();
            const unsigned char *cb_base = cst + t * TC_CST;
            const uint4 c = *reinterpret_cast<const uint4 *>(cb_base + R * 16);
            const unsigned char *xcon = bring + (size_t)sb * BBLK + BOP;  // the block's x constants
            const float4 *scl = reinterpret_cast<const float4 *>(xcon);
            const float *gsums = reinterpret_cast<const float *>(xcon + NV4 * 16);
            const int *lsum = reinterpret_cast<const int *>(xcon + NV4 * 48);
            const float d = __uint_as_float(c.x), dmin = __uint_as_float(c.y);
            float mins[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) mins[g] = (float)__byte_perm(g < 4 ? c.z : c.w, 0u, 0x4440 + (g & 3));
            const uint32_t tacc = trow + t * 2 * N + vh * 4 * EV;
#pragma unroll
            for (unsigned c8 = 0; c8 < 4 * EV; c8 += 8) {
                int lo[8], hi[8];
                tc_ld8(tacc + c8, lo);
                tc_ld8(tacc + N + c8, hi);
                tc_wait_ld();
#pragma unroll
                for (unsigned k = 0; k < 2; ++k) {
                    const unsigned qv = c8 / 4 + k, v = vh * EV + qv;
                    const float4 fs = scl[v];  // 2^(E - 6), 2^(E - 13), 2^(E - 20), 2^(E - 27)
                    if constexpr (TYPE == T_Q4_K) {
                        const int T0 = lo[4 * k] + 8 * hi[4 * k], T1 = lo[4 * k + 1] + 8 * hi[4 * k + 1];
                        const int T2 = lo[4 * k + 2] + 8 * hi[4 * k + 2], T3 = lo[4 * k + 3] + 8 * hi[4 * k + 3];
                        const int P01 = T0 * 128 + T1, P23 = T2 * 128 + T3;  // |T| <= 945 * 64 * 256: below 2^31
                        const float sum = fmaf((float)P01, fs.y, (float)P23 * fs.w);
                        acc[qv] = fmaf(d, sum, acc[qv]);
                        const float *gsv = gsums + v * 8;
                        float mt_ = 0.f;
#pragma unroll
                        for (int g = 0; g < 8; ++g) mt_ = fmaf(mins[g], gsv[g], mt_);
                        acc[qv] = fmaf(-dmin, mt_, acc[qv]);
                    } else {
                        const float f[4] = {fs.x, fs.y, fs.z, fs.w};
                        float sum = 0.f;
#pragma unroll
                        for (unsigned l = 0; l < 4; ++l) {
                            const int T = lo[4 * k + l] + (hi[4 * k + l] << 8) - 8192 * lsum[4 * v + l];
                            sum = fmaf((float)T, f[l], sum);
                        }
                        acc[qv] = fmaf(d, sum, acc[qv]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(acc_empty + t);
                mbar_arrive(cst_empty + t);
                mbar_arrive(b_empty + sb);
            }
            if (bl + 1 == nb) {  // the M-tile's last block of this slice: write the rows
                const unsigned row = mt * 128 + R;
#pragma unroll
                for (unsigned q = 0; q < EV; ++q) {
                    const unsigned v = vh * EV + q;
                    if (p.KS == 1) {
                        if (v < p.nv && row < p.rows) p.y[v * p.out_stride + row] = acc[q];
                    } else {
                        p.scratch[((size_t)s * p.mtiles * 128 + row) * NV4 + v] = acc[q];
                    }
                    acc[q] = 0.f;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(NCOLS) : "memory");
    }
    if (p.KS == 1 || *abort) return;
    // slices: the last CTA of the M-tile group adds them in slice order
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *flag = atomicAdd(p.counters + j, 1u) == p.KS - 1;
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    const unsigned r0 = mb * 128, r1 = min(me * 128, p.rows);
    for (unsigned i = threadIdx.x; i < (r1 - r0) * p.nv; i += TC_THREADS) {
        const unsigned row = r0 + i / p.nv, v = i % p.nv;
        float y = 0.f;
        for (unsigned q = 0; q < p.KS; ++q) y += __ldcg(p.scratch + ((size_t)q * p.mtiles * 128 + row) * NV4 + v);
        p.y[v * p.out_stride + row] = y;
    }
    if (threadIdx.x == 0) p.counters[j] = 0;
}

// Layout of a launch: K slices and M-tile groups chosen for the least time
// of the busiest CTA (its items at about one SM's share of HBM time each,
// plus the slice sum by the last CTA of a group); G = 0 if the shape does
// not fit.
static TcParams tc_plan(unsigned type, unsigned rows, unsigned cols, unsigned nv, int sms, size_t *scratch_bytes)
{
    TcParams p = {};
    p.rows = rows; p.K = cols; p.nblk = cols / 256; p.tiles = (rows + 15) / 16; p.mtiles = (p.tiles + 7) / 8;
    p.nv = nv; p.N = tc_n(nv);
    const TcDepth dp = tc_depth(type, p.N);
    p.rs = dp.rs; p.rb = dp.rb; p.da = dp.da; p.dc = dp.dc;
    // tuning override "operand buffers,unit stages,B stages" (FYB_TC_DEPTH), taken when it fits
    if (const char *env = std::getenv("FYB_TC_DEPTH")) {
        unsigned a = 0, r = 0, b = 0;
        if (std::sscanf(env, "%u,%u,%u", &a, &r, &b) == 3 && a >= 2 && a <= 8 && r >= 2 && r <= 16 && b >= 2 &&
            b <= 16 && tc_smem(type, p.N, r, b, a, 4).total <= 227 * 1024) {
            p.da = a; p.rs = r; p.rb = b;
        }
    }
    *scratch_bytes = 0;
    if (!p.rs || sms < 1 || p.nblk == 0) return p;
    const double item_us = unit_bytes(type) * 8 / 43.0e3;
    double best = 1e30;
    for (unsigned nbs = p.nblk; nbs >= 1; --nbs) {
        const unsigned ks = (p.nblk + nbs - 1) / nbs;
        if ((p.nblk + ks - 1) / ks != nbs || ks > (unsigned)sms) continue;  // the same slices with fewer blocks
        const unsigned g = std::max(1u, std::min((unsigned)sms / ks, p.mtiles));
        const unsigned mt = (p.mtiles + g - 1) / g;
        double cost = (double)mt * nbs * item_us;
        if (ks > 1) cost += 1.0 + (double)ks * mt * 128 * nv * 4 / 150.0e3;  // slice sum (us)
        if (cost < best) { best = cost; p.nbs = nbs; p.KS = ks; p.G = g; }
    }
    *scratch_bytes = p.KS > 1 ? (size_t)p.KS * p.mtiles * 128 * (p.N / 4) * sizeof(float) : 0;
    return p;
}

// Workspace: [counters][B blocks (tcgen05 path)][slice scratch of either kernel].
static size_t tc_bops_bytes(unsigned N, unsigned nblk) { return ((size_t)nblk * tc_bblk(N) + 255) / 256 * 256; }

size_t qgemm_workspace_bytes(unsigned type, size_t rows, size_t cols, size_t nv, int sms)
{
    if (nv < 3 || nv > 2 * QM_MAX_PAIRS || cols % 256 || sms > 1024) return 0;
    size_t sb, cn, tb = 0, bb = 0;
    qm_plan(type, (unsigned)rows, (unsigned)cols, (unsigned)nv, sms, &sb, &cn);
    if (nv >= tc_min_nv(type)) {
        tc_plan(type, (unsigned)rows, (unsigned)cols, (unsigned)nv, sms, &tb);
        bb = tc_bops_bytes(tc_n((unsigned)nv), (unsigned)(cols / 256));
    }
    return QM_COUNTER_BYTES + bb + (std::max(sb, tb) + 255) / 256 * 256;
}

template <unsigned TYPE, unsigned N>
static cudaError_t launch_tc_n(const TcParams &p, cudaStream_t st)
{
    cudaError_t e = cudaSuccess;
    tc_limbs_kernel<N><<<p.nblk, N * 4, 0, st>>>(p.x, p.K, p.nv, const_cast<unsigned char *>(p.bops), p.error);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // at least half of the SM's shared memory, so one CTA holds an SM and
    // its TMEM allocation never waits for another CTA's
    const size_t smem = std::max(tc_smem(TYPE, N, p.rs, p.rb, p.da, p.dc).total, (size_t)116 * 1024);
    if ((e = cudaFuncSetAttribute(qgemm_tc_kernel<TYPE, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) !=
        cudaSuccess)
        return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.G * p.KS);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, qgemm_tc_kernel<TYPE, N>, p);
}

template <unsigned TYPE>
static cudaError_t launch_tc(const TcParams &p, cudaStream_t st)
{
    if (p.N == 16) return launch_tc_n<TYPE, 16>(p, st);
    if (p.N == 32) return launch_tc_n<TYPE, 32>(p, st);
    return launch_tc_n<TYPE, 64>(p, st);
}

int launch_qgemm(const QWeights &w, unsigned rows, const float *x, float *y, size_t out_stride, unsigned nv,
    void *workspace, size_t workspace_bytes, unsigned *error, int sms, cudaStream_t st)
{
    if (!w.units || (w.type != T_Q4_K && w.type != T_Q6_K) || w.cols % 256 || nv < 3 || nv > 2 * QM_MAX_PAIRS ||
        !x || !y || rows == 0 || (rows + 15) / 16 != w.tiles || !workspace || sms > 1024)
        return -1;
    if (workspace_bytes < qgemm_workspace_bytes(w.type, rows, w.cols, nv, sms)) return -1;
    unsigned char *ws = reinterpret_cast<unsigned char *>(workspace);
    if (nv >= tc_min_nv(w.type)) {
        size_t tb;
        TcParams p = tc_plan(w.type, rows, w.cols, nv, sms, &tb);
        if (p.G) {
            p.units = w.units;
            p.x = x; p.y = y; p.out_stride = out_stride;
            p.counters = reinterpret_cast<unsigned *>(ws);
            p.bops = ws + QM_COUNTER_BYTES;
            p.scratch = tb ? reinterpret_cast<float *>(ws + QM_COUNTER_BYTES + tc_bops_bytes(p.N, p.nblk)) : nullptr;
            p.error = error;
            const cudaError_t e = w.type == T_Q4_K ? launch_tc<T_Q4_K>(p, st) : launch_tc<T_Q6_K>(p, st);
            return e == cudaSuccess ? 0 : -2;
        }
    }
    size_t sb, cn;
    QmParams p = qm_plan(w.type, rows, w.cols, nv, sms, &sb, &cn);
    if (p.G == 0) return -1;
    p.units = w.units;
    p.x = x; p.y = y; p.out_stride = out_stride;
    p.counters = reinterpret_cast<unsigned *>(ws);
    p.scratch = sb ? reinterpret_cast<float *>(ws + QM_COUNTER_BYTES) : nullptr;
    p.error = error;
    const size_t smem = qm_smem(p.np, p.nbs).total;
    auto kern = w.type == T_Q4_K ? qgemm_kernel<T_Q4_K> : qgemm_kernel<T_Q6_K>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return -2;
    kern<<<p.G * p.KS, QG_THREADS, smem, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace fyb
