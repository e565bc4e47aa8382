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

size_t qgemm_workspace_bytes(unsigned type, size_t rows, size_t cols, size_t nv, int sms)
{
    if (nv < 3 || nv > 2 * QM_MAX_PAIRS || cols % 256 || sms > 1024) return 0;
    size_t sb, cn;
    qm_plan(type, (unsigned)rows, (unsigned)cols, (unsigned)nv, sms, &sb, &cn);
    return QM_COUNTER_BYTES + (sb + 255) / 256 * 256;
}

int launch_qgemm(const QWeights &w, unsigned rows, const float *x, float *y, size_t out_stride, unsigned nv,
    void *workspace, size_t workspace_bytes, unsigned *error, int sms, cudaStream_t st)
{
    if (!w.units || (w.type != T_Q4_K && w.type != T_Q6_K) || w.cols % 256 || nv < 3 || nv > 2 * QM_MAX_PAIRS ||
        !x || !y || rows == 0 || (rows + 15) / 16 != w.tiles || !workspace || sms > 1024)
        return -1;
    size_t sb, cn;
    QmParams p = qm_plan(w.type, rows, w.cols, nv, sms, &sb, &cn);
    if (p.G == 0) return -1;
    if (workspace_bytes < QM_COUNTER_BYTES + (sb + 255) / 256 * 256) return -1;
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
