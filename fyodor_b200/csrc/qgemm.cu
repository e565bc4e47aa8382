// qgemm.cu - weight-reusing small-batch GEMM on the integer tensor cores:
// Y[v][r] = sum_k W[r][k] X[v][k] for 3..16 input vectors (the engine's
// matmul, backend/include/compute.h:80-83; its reference small-batch path
// keeps one weight pass per batch, CUDA/gemm.cu:53-95).
//
// Every weight unit (16 rows x 256 columns, repacked as for the GEMV) is
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
    extern __shared__ __align__(128) unsigned char smem[];
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
// The same product on the 5th-generation tensor cores (tcgen05, for
// TC_MIN_NV..16 vectors). A CTA of 256 threads takes M-tiles of 128 weight
// rows (8 unit tiles) over a K slice. Per 256-column block:
//  - the 8 units arrive by bulk copy (two-stage ring of whole blocks);
//  - every thread owns one row and half of its groups: it scales the row's
//    4- or 6-bit values by their group scale in integer and writes the
//    product A' as two byte planes (A' = lo + 256 hi; Q6_K adds 8192 so
//    both planes are unsigned) into shared memory in the canonical K-major
//    layout (8-row x 16-byte core matrices, no swizzle);
//  - one thread issues tcgen05.mma kind::i8 (u8 A x s8 B, M 128, N = 4 limbs
//    x vectors, K 32) for each group and plane; the products of all 8 groups
//    accumulate in TMEM (one fp32-exact int32 column set per plane), so the
//    group scales cost no epilogue work;
//  - tcgen05.commit signals an mbarrier; the threads read their row from
//    TMEM (tcgen05.ld 32x32b), form T = lo + 256 hi per limb (minus the
//    Q6_K bias times the block's limb sums) and apply d 2^(E - 6 - 7 limb)
//    and the Q4_K minimum term in fp32.
// The x limbs of the slice are split once per CTA into the B operand (same
// split as the mma.sync path); K slices meet as in qgemm_kernel.
constexpr unsigned TC_THREADS = 256;
constexpr unsigned TC_MIN_NV = 4;
constexpr unsigned TC_RING = 2;  // stages of 8 units

FYB_HOST_DEV unsigned tc_n(unsigned nv) { return nv <= 4 ? 16u : nv <= 8 ? 32u : 64u; }  // 4 limbs x padded vectors

struct TcSmem {
    size_t b, exps, gsums, lsum, a, ring, bars, misc, total;
};

FYB_HOST_DEV TcSmem tc_smem(unsigned type, unsigned N, unsigned nbs)
{
    TcSmem s;
    s.b = 0;                                                   // [nbs][8 groups][N/8][2][8][16] s8 limbs
    s.exps = s.b + (size_t)nbs * 8 * N * 32;                   // [nbs][N/4] int
    s.gsums = s.exps + (size_t)nbs * (N / 4) * 4;              // [nbs][N/4][8] float
    s.lsum = s.gsums + (size_t)nbs * (N / 4) * 8 * 4;          // [nbs][N] int
    s.a = (s.lsum + (size_t)nbs * N * 4 + 1023) / 1024 * 1024; // [2 halves][2 planes][4 groups][16][2][8][16]
    s.ring = s.a + 2 * 2 * 4 * 4096;                           // [TC_RING][8 units]
    s.bars = s.ring + (size_t)TC_RING * 8 * unit_bytes(type);
    s.misc = s.bars + (TC_RING + 1) * 8;
    s.total = s.misc + 16;
    return s;
}

static unsigned tc_blocks_per_slice(unsigned type, unsigned N, unsigned nblk)
{
    unsigned nbs = nblk;
    while (nbs > 1 && tc_smem(type, N, nbs).total > 227 * 1024) --nbs;
    return tc_smem(type, N, nbs).total <= 227 * 1024 ? nbs : 0;
}

struct TcParams {
    const unsigned char *units;
    unsigned rows, K, nblk, tiles, mtiles, nv, N;
    unsigned nbs, KS, G;
    const float *x;
    float *y;
    unsigned long long out_stride;
    float *scratch;      // [KS][mtiles * 128][N / 4] when KS > 1
    unsigned *counters;  // [G]
    unsigned *error;
};

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

// Offset of row R, K half kc within one group's 128 x 32 operand.
FYB_DEV unsigned tc_core(unsigned R, unsigned kc) { return (R >> 3) * 256 + kc * 128 + (R & 7) * 16; }

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

template <unsigned TYPE, unsigned NH>
__global__ void __launch_bounds__(TC_THREADS, 1) qgemm_tc_kernel(const TcParams p)
{
    constexpr unsigned N = 2 * NH, NVH = NH / 4;  // columns per plane; vectors per thread
    extern __shared__ __align__(1024) unsigned char smem[];
    const TcSmem L = tc_smem(TYPE, N, p.nbs);
    signed char *bsm = reinterpret_cast<signed char *>(smem + L.b);
    int *exps = reinterpret_cast<int *>(smem + L.exps);
    float *gsums = reinterpret_cast<float *>(smem + L.gsums);
    int *lsum = reinterpret_cast<int *>(smem + L.lsum);
    unsigned char *asm_ = smem + L.a;
    unsigned char *ring = smem + L.ring;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);  // [TC_RING] units, [TC_RING] MMAs done
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.misc);
    unsigned *flag = reinterpret_cast<unsigned *>(smem + L.misc + 4);

    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned s = blockIdx.x % p.KS, j = blockIdx.x / p.KS;
    if (j >= p.G) return;
    const unsigned b0 = s * p.nbs, nb = min(p.nbs, p.nblk - b0);
    const unsigned mb = (unsigned)((unsigned long long)p.mtiles * j / p.G);
    const unsigned me = (unsigned)((unsigned long long)p.mtiles * (j + 1) / p.G);
    const unsigned items = (me - mb) * nb;
    const unsigned ub = unit_bytes(TYPE);
    const unsigned ncols = N * 2 <= 32 ? 32u : N * 2;  // TMEM columns: the two planes

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(ncols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        for (unsigned k = 0; k < TC_RING + 1; ++k) mbar_init(bars + k, 1);
        fence_barrier_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto issue = [&](unsigned it) {  // the 8 units of item `it` into ring stage it % TC_RING
        const unsigned mt = mb + it / nb, bl = it % nb, st = it % TC_RING;
        const unsigned t0 = mt * 8, nt = min(8u, p.tiles - t0);
        mbar_expect_tx(bars + st, nt * ub);
        for (unsigned i = 0; i < nt; ++i)
            bulk_copy_g2s(ring + ((size_t)st * 8 + i) * ub,
                          p.units + ((unsigned long long)(t0 + i) * p.nblk + b0 + bl) * ub, ub, bars + st);
    };
    if (threadIdx.x == 0)
        for (unsigned it = 0; it < items && it < TC_RING; ++it) issue(it);

    // B: the slice's x limbs, vector v (zero past nv) in rows 4v..4v+3
    {
        const unsigned nslot = nb * 16, vtot = N / 4;
        for (unsigned s0 = 0; s0 < vtot * nslot; s0 += TC_THREADS) {
            const unsigned i = s0 + threadIdx.x;
            const bool ok = i < vtot * nslot;
            const unsigned v = ok ? i / nslot : 0, sl = ok ? i % nslot : 0, bl = sl / 16, k16 = sl % 16;
            float x[16];
            if (ok && v < p.nv) load16(p.x + (size_t)v * p.K + (size_t)b0 * 256 + 16 * sl, x);
            else {
#pragma unroll
                for (int q = 0; q < 16; ++q) x[q] = 0.f;
            }
            float gs = 0.f, mx = 0.f;
#pragma unroll
            for (int q = 0; q < 16; ++q) { gs = __fadd_rn(gs, x[q]); mx = fmaxf(mx, fabsf(x[q])); }
            const float other = __shfl_xor_sync(0xffffffffu, gs, 1);
            if (ok && (k16 & 1) == 0) gsums[(bl * vtot + v) * 8 + k16 / 2] = __fadd_rn(gs, other);
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            int E = 0;
            const bool bad = !(mx <= 3.0e38f);
            if (!bad && mx > 0.f) {
                frexpf(mx, &E);
                if (E < -120) E = -120;
            }
            if (ok && k16 == 0) exps[bl * vtot + v] = E;
            if (ok && bad && p.error) *(volatile unsigned *)p.error = ERR_NONFINITE;
            const float sc = pow2f(6 - E);
            unsigned words[4][4];
            int ls[4] = {0, 0, 0, 0};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                unsigned t[4][4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float r = bad ? 0.f : __fmul_rn(x[4 * q + e], sc);
#pragma unroll
                    for (int l = 0; l < 4; ++l) {
                        const float m = __fadd_rn(r, 12582912.0f);
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
            if (ok) {
                const unsigned g = k16 / 2, kc = k16 & 1;
#pragma unroll
                for (int l = 0; l < 4; ++l) {
                    const unsigned n = 4 * v + l;
                    *reinterpret_cast<uint4 *>(bsm + ((size_t)(bl * 8 + g) * (N / 8)) * 256 + tc_core(n, kc)) =
                        make_uint4(words[l][0], words[l][1], words[l][2], words[l][3]);
                    if (k16 == 0) lsum[bl * N + n] = ls[l];
                }
            }
        }
    }
    fence_proxy_async();
    __syncthreads();

    // rows: thread t owns row R = t % 128 of the M-tile; its half vh = t / 128
    // of the groups (staging) and of the vectors (epilogue); warp w reads TMEM
    // lanes 32 (w % 4) .. + 31, which are exactly rows R
    const unsigned R = threadIdx.x & 127, vh = threadIdx.x >> 7;
    const uint32_t idesc = tc_idesc(N);
    const uint32_t trow = tmem + ((32u * (warp & 3)) << 16);
    float acc[NVH];
#pragma unroll
    for (unsigned q = 0; q < NVH; ++q) acc[q] = 0.f;
    unsigned rpar = 0;
    bool ok = true;
    for (unsigned it = 0; it < items && ok; ++it) {
        const unsigned mt = mb + it / nb, bl = it % nb, st = it % TC_RING;
        const bool landed = mbar_wait_bounded(bars + st, (rpar >> st) & 1u);
        if (__syncthreads_or(!landed)) {
            if (threadIdx.x == 0 && p.error) atomicCAS(p.error, 0u, (unsigned)ERR_TIMEOUT);
            ok = false;
            break;
        }
        rpar ^= 1u << st;
        const unsigned tile = R >> 4, r = R & 15;
        const bool have = mt * 8 + tile < p.tiles;
        const unsigned char *u = ring + ((size_t)st * 8 + tile) * ub;
        // this row's block constants, read before the ring stage is refilled
        float d = 0.f, dmin = 0.f, mins[8];
        unsigned scq[8];
        if constexpr (TYPE == T_Q4_K) {
            const uint4 hd = have ? *reinterpret_cast<const uint4 *>(u + 2048 + r * 16) : make_uint4(0, 0, 0, 0);
            d = half_bits_to_float((unsigned short)(hd.x & 0xffffu));
            dmin = half_bits_to_float((unsigned short)(hd.x >> 16));
            const unsigned sc0 = hd.y & 0x3F3F3F3Fu, sc1 = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
            const unsigned m0 = hd.z & 0x3F3F3F3Fu, m1 = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                scq[g] = __byte_perm(g < 4 ? sc0 : sc1, 0u, 0x4440 + (g & 3));
                mins[g] = (float)__byte_perm(g < 4 ? m0 : m1, 0u, 0x4440 + (g & 3));
            }
        } else {
            d = have ? half_bits_to_float(*reinterpret_cast<const unsigned short *>(u + 3328 + r * 2)) : 0.f;
#pragma unroll
            for (int g = 0; g < 8; ++g) { scq[g] = 0; mins[g] = 0.f; }
        }
        for (unsigned h = 0; h < 2; ++h) {
            // groups 4h + 2vh, +1 of row R into the half-h operand buffer
            unsigned char *ah = asm_ + (size_t)h * 2 * 4 * 4096;
#pragma unroll
            for (unsigned gi = 0; gi < 2; ++gi) {
                const unsigned g = 4 * h + 2 * vh + gi, gl = g & 3;
#pragma unroll
                for (unsigned kc = 0; kc < 2; ++kc) {
                    uint4 lo4 = make_uint4(0, 0, 0, 0), hi4 = make_uint4(0, 0, 0, 0);
                    if (have) {
                        unsigned w[4], lo[4], hi[4];
                        if constexpr (TYPE == T_Q4_K) {
                            const uint4 q = *reinterpret_cast<const uint4 *>(u + ((g >> 1) * 32 + kc * 16 + r) * 16);
                            const unsigned sh = (g & 1) * 4;
                            w[0] = (q.x >> sh) & 0x0F0F0F0Fu; w[1] = (q.y >> sh) & 0x0F0F0F0Fu;
                            w[2] = (q.z >> sh) & 0x0F0F0F0Fu; w[3] = (q.w >> sh) & 0x0F0F0F0Fu;
                            const unsigned sg = vh ? scq[4 * h + 2 + gi] : scq[4 * h + gi];  // g, without a runtime index
#pragma unroll
                            for (int e = 0; e < 4; ++e) tc_scale4(w[e], sg, 0u, 0u, lo[e], hi[e]);  // A' = s q
                        } else {
                            // value l = 16 kc + e of group g = 4 n2 + qq: ql chunk (2 n2 + (qq & 1), kc),
                            // qh chunk (n2, kc), scale byte 8 n2 + 2 qq + kc
                            const unsigned n2 = g >> 2, qq = g & 3;
                            const uint4 ql = *reinterpret_cast<const uint4 *>(u + ((2 * n2 + (qq & 1)) * 32 + kc * 16 + r) * 16);
                            const uint4 qh = *reinterpret_cast<const uint4 *>(u + 2048 + (n2 * 32 + kc * 16 + r) * 16);
                            const int sgn = (int)(signed char)u[3072 + r * 16 + 8 * n2 + 2 * qq + kc];
                            const unsigned sp = (unsigned)(sgn + 128);                 // 0..255
                            const unsigned bias = (unsigned)(8192 - 32 * sgn);          // s (q - 32) + 8192 > 0
                            const unsigned bias2 = bias | (bias << 16);
                            const unsigned qsh = (qq >= 2) ? 4u : 0u, hsh = 2 * qq;
                            const unsigned lq[4] = {ql.x, ql.y, ql.z, ql.w}, hq[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                w[e] = ((lq[e] >> qsh) & 0x0F0F0F0Fu) | (((hq[e] >> hsh) & 0x03030303u) << 4);
                                // (s + 128) q - 128 q + 8192 - 32 s = s (q - 32) + 8192
                                tc_scale4(w[e], sp, bias2, 128u, lo[e], hi[e]);
                            }
                        }
                        lo4 = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        hi4 = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    }
                    *reinterpret_cast<uint4 *>(ah + (0 * 4 + gl) * 4096 + tc_core(R, kc)) = lo4;
                    *reinterpret_cast<uint4 *>(ah + (1 * 4 + gl) * 4096 + tc_core(R, kc)) = hi4;
                }
            }
            fence_proxy_async();
            __syncthreads();
            if (threadIdx.x == 0) {
                tc_fence_after();
                const signed char *bb = bsm + (size_t)bl * 8 * (N / 8) * 256;
#pragma unroll
                for (unsigned gl = 0; gl < 4; ++gl) {
                    const uint64_t bd = tc_desc(bb + (size_t)(4 * h + gl) * (N / 8) * 256);
                    const uint32_t acc_in = (h | gl) ? 1u : 0u;
                    tc_mma(tmem, tc_desc(ah + (0 * 4 + gl) * 4096), bd, idesc, acc_in);
                    tc_mma(tmem + N, tc_desc(ah + (1 * 4 + gl) * 4096), bd, idesc, acc_in);
                }
                if (h == 1) {
                    tc_commit(bars + TC_RING);  // every MMA of the item: the planes are complete
                    if (it + TC_RING < items) issue(it + TC_RING);  // the stage has been read by all threads
                }
            }
        }
        // epilogue: this row's planes for the vector half vh
        if (!mbar_wait_bounded(bars + TC_RING, it & 1u)) {
            if (p.error) atomicCAS(p.error, 0u, (unsigned)ERR_TIMEOUT);
            ok = false;
        }
        if (__syncthreads_or(!ok)) { ok = false; break; }
        tc_fence_after();
        int lo[NH], hi[NH];
#pragma unroll
        for (unsigned c = 0; c < NH; c += 8) {
            tc_ld8(trow + vh * NH + c, lo + c);
            tc_ld8(trow + N + vh * NH + c, hi + c);
        }
        tc_wait_ld();
        tc_fence_before();
#pragma unroll
        for (unsigned q = 0; q < NVH; ++q) {
            const unsigned v = vh * NVH + q;
            const int E = exps[bl * (N / 4) + v];
            float sum = 0.f;
#pragma unroll
            for (unsigned l = 0; l < 4; ++l) {
                int T = lo[4 * q + l] + (hi[4 * q + l] << 8);
                if constexpr (TYPE == T_Q6_K) T -= 8192 * lsum[bl * N + 4 * v + l];
                sum = fmaf((float)T, pow2f(E - 6 - 7 * (int)l), sum);
            }
            acc[q] = fmaf(d, sum, acc[q]);
            if constexpr (TYPE == T_Q4_K) {
                const float *gsv = gsums + (bl * (N / 4) + v) * 8;
                float mt_ = 0.f;
#pragma unroll
                for (int g = 0; g < 8; ++g) mt_ = fmaf(mins[g], gsv[g], mt_);
                acc[q] = fmaf(-dmin, mt_, acc[q]);
            }
        }
        if (bl + 1 == nb) {  // the M-tile's last block of this slice: write the rows
            const unsigned row = mt * 128 + R;
#pragma unroll
            for (unsigned q = 0; q < NVH; ++q) {
                const unsigned v = vh * NVH + q;
                if (p.KS == 1) {
                    if (v < p.nv && row < p.rows) p.y[v * p.out_stride + row] = acc[q];
                } else {
                    p.scratch[((size_t)s * p.mtiles * 128 + row) * (N / 4) + v] = acc[q];
                }
                acc[q] = 0.f;
            }
        }
    }
    // copies still in flight land before the CTA leaves (bounded)
    if (threadIdx.x == 0 && !ok)
        for (unsigned it2 = 0; it2 < TC_RING; ++it2) mbar_wait_bounded(bars + it2, (rpar >> it2) & 1u);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(ncols) : "memory");
    }
    if (p.KS == 1 || !ok) return;
    // slices: the last CTA of the M-tile group adds them in slice order
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *flag = atomicAdd(p.counters + j, 1u) == p.KS - 1;
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    const unsigned r0 = mb * 128, r1 = min(me * 128, p.rows), vt = N / 4;
    for (unsigned i = threadIdx.x; i < (r1 - r0) * p.nv; i += TC_THREADS) {
        const unsigned row = r0 + i / p.nv, v = i % p.nv;
        float y = 0.f;
        for (unsigned q = 0; q < p.KS; ++q) y += __ldcg(p.scratch + ((size_t)q * p.mtiles * 128 + row) * vt + v);
        p.y[v * p.out_stride + row] = y;
    }
    if (threadIdx.x == 0) p.counters[j] = 0;
}

static TcParams tc_plan(unsigned type, unsigned rows, unsigned cols, unsigned nv, int sms, size_t *scratch_bytes)
{
    TcParams p = {};
    p.rows = rows; p.K = cols; p.nblk = cols / 256; p.tiles = (rows + 15) / 16; p.mtiles = (p.tiles + 7) / 8;
    p.nv = nv; p.N = tc_n(nv);
    p.nbs = tc_blocks_per_slice(type, p.N, p.nblk);
    p.KS = p.nbs ? (p.nblk + p.nbs - 1) / p.nbs : 0;
    p.G = p.KS && p.KS <= (unsigned)sms ? std::max(1u, std::min((unsigned)sms / p.KS, p.mtiles)) : 0;
    *scratch_bytes = p.KS > 1 ? (size_t)p.KS * p.mtiles * 128 * (p.N / 4) * sizeof(float) : 0;
    return p;
}

// Workspace of either kernel: the larger of the two needs.
size_t qgemm_workspace_bytes(unsigned type, size_t rows, size_t cols, size_t nv, int sms)
{
    if (nv < 3 || nv > 2 * QM_MAX_PAIRS || cols % 256 || sms > 1024) return 0;
    size_t sb, cn, tb = 0;
    qm_plan(type, (unsigned)rows, (unsigned)cols, (unsigned)nv, sms, &sb, &cn);
    if (nv >= TC_MIN_NV) tc_plan(type, (unsigned)rows, (unsigned)cols, (unsigned)nv, sms, &tb);
    return QM_COUNTER_BYTES + (std::max(sb, tb) + 255) / 256 * 256;
}

template <unsigned TYPE>
static cudaError_t launch_tc(const TcParams &p, cudaStream_t st)
{
    // at least half of the SM's shared memory, so one CTA holds an SM and
    // its TMEM allocation never waits for another CTA's
    const size_t smem = std::max(tc_smem(TYPE, p.N, p.nbs).total, (size_t)116 * 1024);
    cudaError_t e = cudaSuccess;
#define FYB_TC(NHV)                                                                                               \
    if (p.N == 2 * NHV) {                                                                                         \
        e = cudaFuncSetAttribute(qgemm_tc_kernel<TYPE, NHV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        if (e == cudaSuccess) qgemm_tc_kernel<TYPE, NHV><<<p.G * p.KS, TC_THREADS, smem, st>>>(p);               \
    }
    FYB_TC(8) FYB_TC(16) FYB_TC(32)
#undef FYB_TC
    return e != cudaSuccess ? e : cudaGetLastError();
}

int launch_qgemm(const QWeights &w, unsigned rows, const float *x, float *y, size_t out_stride, unsigned nv,
    void *workspace, size_t workspace_bytes, unsigned *error, int sms, cudaStream_t st)
{
    if (!w.units || (w.type != T_Q4_K && w.type != T_Q6_K) || w.cols % 256 || nv < 3 || nv > 2 * QM_MAX_PAIRS ||
        !x || !y || rows == 0 || (rows + 15) / 16 != w.tiles || !workspace || sms > 1024)
        return -1;
    if (workspace_bytes < qgemm_workspace_bytes(w.type, rows, w.cols, nv, sms)) return -1;
    if (nv >= TC_MIN_NV) {
        size_t tb;
        TcParams p = tc_plan(w.type, rows, w.cols, nv, sms, &tb);
        if (p.G) {
            p.units = w.units;
            p.x = x; p.y = y; p.out_stride = out_stride;
            p.counters = reinterpret_cast<unsigned *>(workspace);
            p.scratch = tb ? reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(workspace) + QM_COUNTER_BYTES)
                           : nullptr;
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
    p.counters = reinterpret_cast<unsigned *>(workspace);
    p.scratch = sb ? reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(workspace) + QM_COUNTER_BYTES) : nullptr;
    p.error = error;
    const size_t smem = qm_smem(p.np, p.nbs).total;
    auto kern = w.type == T_Q4_K ? qgemm_kernel<T_Q4_K> : qgemm_kernel<T_Q6_K>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return -2;
    kern<<<p.G * p.KS, QG_THREADS, smem, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace fyb
