// qgemv.cu - dequant-fused K-quant GEMV on the integer tensor cores.
//
// y[r] = sum_k W[r][k] * x[k] for Q4_K / Q6_K weights and one or two input
// vectors: the engine's decode projections (reference: nya_row_dot,
// CUDA/matvec.cu:69-111; scalar semantics nya_llm_matvec,
// backend/core/llm_quant.c:236-276).
//
// Why tensor cores at batch 1: a Q4_K value is half a byte, so at ~6.5 TB/s an
// SM must retire ~40 weights per clock. Unpacking each nibble to a float and
// multiplying on the FP32 pipe costs >3 instructions per weight, which would
// make the kernel ALU-bound below the HBM roofline. Instead:
//   * the activation vector is split into four signed 8-bit limbs per value,
//     x ~= 2^(E-6) * (X0 + X1/128 + X2/128^2 + X3/128^3), one power-of-two
//     exponent E per 256-value block (28 bits of mantissa: exact for values
//     within 2^-4 of the block maximum, below fp32 rounding otherwise);
//   * the packed nibbles go straight into the A operand of
//     mma.m16n8k32.u8.s8 after one AND (low nibbles) or shift+AND (high);
//   * the limbs are columns of the B operand, so one MMA computes the exact
//     integer dot product of 16 rows x 32 values against all limbs;
//   * each 32-value group's 6-bit scale multiplies the s32 accumulators, and
//     once per 256-value block the limb sums become float, scaled by
//     d * 2^(E-6-7l). The Q4_K minimum term dmin*m_g*sum(x_g) uses fp32
//     group sums of x. Q6_K runs the same scheme with m16n8k16 (its scales
//     cover 16 values) and signed quants.
//
// Weights are repacked once (repack_units) into "units": 16 rows x 256
// columns stored contiguously (2304 B Q4_K, 3360 B Q6_K, the GGUF byte count),
// laid out for conflict-free ldmatrix. A fused matrix may interleave rows of
// several tensors (QKV with RoPE pairs side by side, gate/up pairs), so an
// epilogue finds everything it needs in one warp.
//
// Work split: units are taken in tile-major order and every warp of the grid
// owns one contiguous range (stream-K). Each warp streams its units with
// cp.async.bulk into a private shared-memory ring (mbarrier per
// stage, bounded waits) - the first stages are issued before the
// programmatic-dependent-launch wait, as weights never depend on the
// previous kernel. A tile finished by one warp goes straight to the
// epilogue; a tile shared by several warps meets in a scratch slot per warp,
// and the warp completing it (atomic unit count) sums the slots in column
// order, so results do not depend on timing.
#include "qgemv_core.cuh"

namespace fyb {

struct QgSeg {
    unsigned rows, tile_begin;
    float *out;
};

struct QgParams {
    const unsigned char *units;
    QgSeg seg[3];
    int nseg, epilogue, nvec;
    unsigned tiles_total, nblk, K, unit;
    unsigned long long total_units;
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
        const unsigned lt = tile - p.seg[s].tile_begin;
        r.segA = r.segB = s;
        if (p.epilogue == EPI_QKV) { r.rowA = lt * 16 + 2 * gid; r.rowB = r.rowA + 1; }
        else { r.rowA = lt * 16 + gid; r.rowB = r.rowA + 8; }
    }
    r.okA = r.rowA < p.seg[r.segA].rows;
    r.okB = r.rowB < p.seg[r.segB].rows;
    return r;
}

// ------------------------------------------------------------ epilogue
FYB_DEV void epilogue(const QgParams &p, const RowPair &rp, float yA, float yB, unsigned lane)
{
    const unsigned tig = lane & 3, vec = tig >> 1;
    const bool mine = (tig & 1) == 0 && vec < (unsigned)p.nvec;
    if (p.epilogue == EPI_STORE || p.epilogue == EPI_LOGITS) {
        if (mine) {
            if (rp.okA) p.seg[rp.segA].out[vec * p.out_stride + rp.rowA] = yA;
            if (rp.okB) p.seg[rp.segB].out[vec * p.out_stride + rp.rowB] = yB;
        }
        if (p.epilogue == EPI_LOGITS) {
            unsigned long long k0 = 0ull, k1 = 0ull;
            if (mine) {
                unsigned long long kA = 0, kB = 0;
                if (rp.okA) kA = ((unsigned long long)float_order_key(yA) << 32) | (0xffffffffu - rp.rowA);
                if (rp.okB) kB = ((unsigned long long)float_order_key(yB) << 32) | (0xffffffffu - rp.rowB);
                if (((rp.okA && !isfinite(yA)) || (rp.okB && !isfinite(yB))) && p.error)
                    *(volatile unsigned *)p.error = ERR_NONFINITE;
                const unsigned long long k = kA > kB ? kA : kB;
                if (vec == 0) k0 = k; else k1 = k;
            }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long a = __shfl_xor_sync(0xffffffffu, k0, o);
                const unsigned long long b = __shfl_xor_sync(0xffffffffu, k1, o);
                k0 = a > k0 ? a : k0;
                k1 = b > k1 ? b : k1;
            }
            if (lane == 0) {
                atomicMax(p.argmax_key, k0);
                if (p.nvec > 1) atomicMax(p.argmax_key + 1, k1);
                __threadfence();
                const unsigned done = atomicAdd(p.tiles_done, 1u);
                if (done == p.tiles_total - 1) {
                    __threadfence();
                    for (int v = 0; v < p.nvec; ++v) {
                        const unsigned long long k = atomicExch(p.argmax_key + v, 0ull);
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
            const float g = __fdiv_rn(yA, __fadd_rn(1.0f, expf(-yA)));
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
        const __half2 v2 = __halves2half2(__float2half_rn(a), __float2half_rn(b));
        *reinterpret_cast<__half2 *>(cache + ((size_t)kvh * p.capacity + pos) * hd + dd) = v2;
    }
}

// ------------------------------------------------------------ x preparation
// Residual add, RMSNorm (llm_cpu.c:83-103: sum of squares in double, then
// x*scale*w in float) and the limb split. Every CTA prepares the whole
// vector; one CTA per 16-value slot writes the residual stream back.
FYB_DEV void prepare_x(const QgParams &p, signed char *xl, unsigned xstride, int *exps, float *gsums, double *red)
{
    const unsigned tid = threadIdx.x, K = p.K, nslot = K / 16, total = nslot * (unsigned)p.nvec;
    float scale0 = 1.f, scale1 = 1.f;
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
            ss = block_sum_double(ss, red);
            const float sc = (float)(1.0 / sqrt(ss / (double)K + (double)p.eps));
            if (v == 0) scale0 = sc; else scale1 = sc;
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
                const float sc = v == 0 ? scale0 : scale1;
#pragma unroll
                for (int j = 0; j < 16; ++j) x[j] = __fmul_rn(__fmul_rn(x[j], sc), w[j]);
            }
        }
        prep_slot(x, ok, v, sl, K, p.nblk, xl, xstride, exps, gsums, p.error);
    }
}

// ------------------------------------------------------------ tile completion
template <int NV>
FYB_DEV void finish_tile(const QgParams &p, unsigned tile, unsigned tile_units, const RowPair &rp, float accA,
    float accB, unsigned long long NW, unsigned long long gw, unsigned lane)
{
    const unsigned nblk = p.nblk, gid = lane >> 2, tig = lane & 3, v = tig >> 1;
    float yA = lane_total<NV>(accA);  // the limb halves (and the split minimum term)
    float yB = lane_total<NV>(accB);
    if (tile_units != nblk) {
        const unsigned long long U = p.total_units;
        const unsigned long long t0 = (unsigned long long)tile * nblk;
        const unsigned long long owner0 = ((t0 + 1) * NW - 1) / U;
        const unsigned long long ownerN = ((t0 + nblk) * NW - 1) / U;
        const unsigned slot = (unsigned)(gw - owner0);
        const unsigned nslots = (unsigned)(ownerN - owner0 + 1);
        float *base = p.partials + (size_t)tile * p.slots * 32;
        if ((tig & 1) == 0) {
            base[slot * 32 + gid * 2 + v] = yA;
            base[slot * 32 + (gid + 8) * 2 + v] = yB;
        }
        __threadfence();
        __syncwarp();
        unsigned old = 0;
        if (lane == 0) old = atomicAdd(p.counters + tile, tile_units);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old + tile_units != nblk) return;
        __threadfence();
        // the slots of the warps whose unit ranges intersect this tile (warps
        // without units own no slot); lanes tig and tig ^ 1 split them
        auto has_units = [&](unsigned s) {
            const unsigned long long g = owner0 + s;
            const unsigned long long ub = g * U / NW, ue = (g + 1) * U / NW;
            return !(ue <= ub || ub >= t0 + nblk || ue <= t0);
        };
        sum_slots(base, 32, gid * 2 + v, (gid + 8) * 2 + v, nslots, tig & 1, 2, has_units, yA, yB);
        yA += __shfl_xor_sync(0xffffffffu, yA, 1);
        yB += __shfl_xor_sync(0xffffffffu, yB, 1);
        if (lane == 0) p.counters[tile] = 0;
    }
    epilogue(p, rp, yA, yB, lane);
}

// ------------------------------------------------------------ the kernel
template <unsigned TYPE, int NV>
__global__ void __launch_bounds__(QG_THREADS, 1) qgemv_kernel(const QgParams p)
{
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr unsigned UB = unit_bytes(TYPE);
    const unsigned K = p.K, nblk = p.nblk;
    const unsigned xstride = K + QG_XPAD;
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    // shared memory: [stages of all warps][mbarriers][x limbs][exps][group sums][reduction]
    unsigned char *stages = smem + (size_t)warp * QG_STAGES * UB;
    size_t off = (size_t)QG_WARPS * QG_STAGES * UB;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + off) + warp * QG_STAGES;
    off += QG_WARPS * QG_STAGES * sizeof(uint64_t);
    signed char *xl = reinterpret_cast<signed char *>(smem + off);
    off += (size_t)p.nvec * 4 * xstride;
    int *exps = reinterpret_cast<int *>(smem + off);
    off += ((size_t)p.nvec * nblk * 4 + 15) / 16 * 16;
    float *gsums = reinterpret_cast<float *>(smem + off);
    off += ((size_t)p.nvec * (K / 32) * 4 + 15) / 16 * 16;
    double *red = reinterpret_cast<double *>(smem + off);

    const unsigned long long NW = (unsigned long long)gridDim.x * QG_WARPS;
    const unsigned long long gw = (unsigned long long)blockIdx.x * QG_WARPS + warp;
    const unsigned long long U = p.total_units;
    const unsigned long long u0 = gw * U / NW, u1 = (gw + 1) * U / NW;
    const unsigned n = (unsigned)(u1 - u0);

    if (lane == 0) {
        for (int s = 0; s < QG_STAGES; ++s) mbar_init(bars + s, 1);
        fence_barrier_init();
    }
    __syncwarp();
    // weights never depend on the previous kernel: start streaming now
    if (lane == 0) {
        for (unsigned i = 0; i < n && i < (unsigned)QG_STAGES; ++i) {
            mbar_expect_tx(bars + i, UB);
            bulk_copy_g2s(stages + i * UB, p.units + (u0 + i) * UB, UB, bars + i);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    prepare_x(p, xl, xstride, exps, gsums, red);
    __syncthreads();

    float accA = 0.f, accB = 0.f;
    unsigned tile = (unsigned)(u0 / nblk), tile_units = 0;
    unsigned blk = (unsigned)(u0 - (unsigned long long)tile * nblk);  // advanced per unit, no division
    RowPair rp = tile_rows(p, tile, lane >> 2);
    for (unsigned i = 0; i < n; ++i) {
        const unsigned long long u = u0 + i;
        const unsigned s = i % QG_STAGES, phase = (i / QG_STAGES) & 1;
        if (!mbar_wait_bounded(bars + s, phase)) {
            if (p.error) *(volatile unsigned *)p.error = ERR_TIMEOUT;
            return;
        }
        compute_unit<TYPE, NV>(stages + s * UB, blk, xl, xstride, exps, nblk, gsums, K / 32, lane, accA, accB);
        __syncwarp();
        if (lane == 0 && i + QG_STAGES < n) {
            fence_proxy_async();
            mbar_expect_tx(bars + s, UB);
            bulk_copy_g2s(stages + s * UB, p.units + (u + QG_STAGES) * UB, UB, bars + s);
        }
        ++tile_units;
        if (blk + 1 == nblk || i + 1 == n) {
            finish_tile<NV>(p, tile, tile_units, rp, accA, accB, NW, gw, lane);
            accA = 0.f; accB = 0.f;
            tile_units = 0;
            if (i + 1 < n) {
                ++tile;
                rp = tile_rows(p, tile, lane >> 2);
            }
        }
        blk = blk + 1 == nblk ? 0 : blk + 1;
    }
}

// ------------------------------------------------------------ repacking
// One thread per 16-byte chunk of the output units. The source block of unit
// row r comes from the mode's row map; rows past a source's end are zeros.
__global__ void repack_kernel(const unsigned char *src0, const unsigned char *src1, unsigned rows, unsigned nblk,
    unsigned type, int mode, unsigned tiles, unsigned char *dst)
{
    const unsigned UB = type == T_Q4_K ? Q4_UNIT : Q6_UNIT, BB = type == T_Q4_K ? 144u : 210u;
    const unsigned chunks = UB / 16;
    const unsigned long long idx = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned long long total = (unsigned long long)tiles * nblk * chunks;
    if (idx >= total) return;
    const unsigned j = (unsigned)(idx % chunks);
    const unsigned long long unit = idx / chunks;
    const unsigned blk = (unsigned)(unit % nblk), t = (unsigned)(unit / nblk);
    unsigned char out[16];
    auto source = [&](unsigned r, const unsigned char **blkp) -> bool {
        unsigned row;
        const unsigned char *base = src0;
        if (mode == REPACK_QKV) row = 16 * t + (r < 8 ? 2 * r : 2 * (r - 8) + 1);
        else if (mode == REPACK_GATEUP) { row = 8 * t + (r & 7); if (r >= 8) base = src1; }
        else row = 16 * t + r;
        if (row >= rows) return false;
        *blkp = base + ((unsigned long long)row * nblk + blk) * BB;
        return true;
    };
    const unsigned char *b = nullptr;
    if (type == T_Q4_K) {
        if (j < 128) {  // qs [p][h][r]
            const unsigned pr = j / 32, h = (j / 16) % 2, r = j % 16;
            const bool ok = source(r, &b);
            for (int e = 0; e < 16; ++e) out[e] = ok ? b[16 + pr * 32 + h * 16 + e] : 0;
        } else {        // header [r]
            const unsigned r = j - 128;
            const bool ok = source(r, &b);
            for (int e = 0; e < 16; ++e) out[e] = ok ? b[e] : 0;
        }
    } else {
        if (j < 128) {          // ql [c][h][r]
            const unsigned c = j / 32, h = (j / 16) % 2, r = j % 16;
            const bool ok = source(r, &b);
            for (int e = 0; e < 16; ++e) out[e] = ok ? b[c * 32 + h * 16 + e] : 0;
        } else if (j < 192) {   // qh [c][h][r]
            const unsigned jj = j - 128, c = jj / 32, h = (jj / 16) % 2, r = jj % 16;
            const bool ok = source(r, &b);
            for (int e = 0; e < 16; ++e) out[e] = ok ? b[128 + c * 32 + h * 16 + e] : 0;
        } else if (j < 208) {   // scales [r]
            const unsigned r = j - 192;
            const bool ok = source(r, &b);
            for (int e = 0; e < 16; ++e) out[e] = ok ? b[192 + e] : 0;
        } else {                // d [r] as fp16, rows 8*(j-208) .. +7
            for (int k = 0; k < 8; ++k) {
                const unsigned r = 8 * (j - 208) + k;
                const bool ok = source(r, &b);
                out[2 * k] = ok ? b[208] : 0;
                out[2 * k + 1] = ok ? b[209] : 0;
            }
        }
    }
    uint4 w;
    memcpy(&w, out, 16);
    *reinterpret_cast<uint4 *>(dst + unit * UB + j * 16) = w;
}

size_t qunits_bytes(unsigned type, size_t tiles, size_t cols)
{
    return tiles * (cols / 256) * unit_bytes(type);
}

int repack_units(const void *src0, const void *src1, size_t rows, size_t cols, unsigned type, int mode,
    void *dst_units, size_t tiles, cudaStream_t s)
{
    if ((type != T_Q4_K && type != T_Q6_K) || cols % 256 || !src0 || !dst_units) return -1;
    if (mode == REPACK_GATEUP && !src1) return -1;
    const unsigned chunks = unit_bytes(type) / 16;
    const unsigned long long total = (unsigned long long)tiles * (cols / 256) * chunks;
    if (total == 0) return 0;
    const unsigned blocks = (unsigned)((total + 255) / 256);
    repack_kernel<<<blocks, 256, 0, s>>>((const unsigned char *)src0, (const unsigned char *)src1, (unsigned)rows,
                                         (unsigned)(cols / 256), type, mode, (unsigned)tiles, (unsigned char *)dst_units);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
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

static size_t qgemv_smem(unsigned type, unsigned K, int nvec);

int qgemv_supported(unsigned type, size_t cols, size_t nvec)
{
    return (type == T_Q4_K || type == T_Q6_K) && cols % 256 == 0 && cols >= 256 && cols <= 16384 &&
           nvec >= 1 && nvec <= 2 && qgemv_smem(type, (unsigned)cols, (int)nvec) <= 227 * 1024;
}

static size_t qgemv_smem(unsigned type, unsigned K, int nvec)
{
    size_t off = (size_t)QG_WARPS * QG_STAGES * unit_bytes(type) + QG_WARPS * QG_STAGES * 8;
    off += (size_t)nvec * 4 * (K + QG_XPAD);
    off += ((size_t)nvec * (K / 256) * 4 + 15) / 16 * 16;
    off += ((size_t)nvec * (K / 32) * 4 + 15) / 16 * 16;
    return off + QG_WARPS * sizeof(double) + 64;
}

static unsigned tiles_of(const QgemvLaunch &L, unsigned *tile_begin)
{
    unsigned tiles = 0;
    for (int s = 0; s < L.nseg; ++s) {
        if (tile_begin) tile_begin[s] = tiles;
        if (L.epilogue == EPI_SWIGLU) { tiles = (L.seg_rows[0] + 7) / 8; break; }
        tiles += (L.seg_rows[s] + 15) / 16;
    }
    return tiles;
}

unsigned qgemv_tiles(const QgemvLaunch &L) { return tiles_of(L, nullptr); }

// CTAs for a launch: one per SM, fewer when the problem gives a warp less
// than two units, so small matrices do not pay for idle CTAs' preparation.
static int qgemv_grid(const QgemvLaunch &L, int grid)
{
    if (grid <= 0) grid = sm_count();
    const unsigned long long units = (unsigned long long)tiles_of(L, nullptr) * (L.w.cols / 256);
    unsigned long long want = (units + 2ull * QG_WARPS - 1) / (2ull * QG_WARPS);
    if (want < 1) want = 1;
    return (int)std::min<unsigned long long>((unsigned long long)grid, want);
}

static unsigned qgemv_slots(const QgemvLaunch &L, int grid)
{
    const unsigned long long units = (unsigned long long)tiles_of(L, nullptr) * (L.w.cols / 256);
    const unsigned long long NW = (unsigned long long)grid * QG_WARPS;
    return units ? (unsigned)(((L.w.cols / 256) * NW + units - 1) / units + 2) : 1;
}

size_t qgemv_partials_bytes(const QgemvLaunch &L, int grid)
{
    grid = qgemv_grid(L, grid);
    return (size_t)tiles_of(L, nullptr) * qgemv_slots(L, grid) * 32 * sizeof(float);
}

int launch_qgemv(const QgemvLaunch &L, cudaStream_t s)
{
    const QWeights &w = L.w;
    if (!qgemv_supported(w.type, w.cols, (size_t)L.nvec) || L.nseg < 1 || L.nseg > 3 || !w.units) return -1;
    if ((L.epilogue == EPI_QKV || L.epilogue == EPI_SWIGLU) && L.nvec != 1) return -1;
    if (L.epilogue == EPI_SWIGLU && (L.nseg != 2 || L.seg_rows[0] != L.seg_rows[1])) return -1;
    const int grid = qgemv_grid(L, L.grid);
    QgParams p = {};
    unsigned tb[3] = {0, 0, 0};
    p.tiles_total = tiles_of(L, tb);
    if (p.tiles_total != w.tiles) return -1;
    p.units = w.units;
    p.nseg = L.nseg;
    p.epilogue = L.epilogue;
    p.nvec = L.nvec;
    for (int i = 0; i < L.nseg; ++i) { p.seg[i].rows = L.seg_rows[i]; p.seg[i].tile_begin = tb[i]; p.seg[i].out = L.out[i]; }
    p.K = w.cols;
    p.nblk = w.cols / 256;
    p.unit = unit_bytes(w.type);
    p.total_units = (unsigned long long)p.tiles_total * p.nblk;
    p.out_stride = L.out_stride;
    p.x = L.x; p.delta = L.delta; p.x_out = L.x_out; p.norm_w = L.norm_w; p.eps = L.eps;
    p.kcache = L.kcache; p.vcache = L.vcache;
    p.rope_cos = L.rope_cos; p.rope_sin = L.rope_sin;
    p.request = L.request; p.position = L.position; p.head_dim = L.head_dim; p.capacity = L.capacity;
    p.argmax_key = L.argmax_key; p.argmax_token = L.argmax_token; p.tiles_done = L.tiles_done;
    p.error = L.error;
    p.slots = qgemv_slots(L, grid);
    if (p.total_units == 0) return 0;
    if (!L.counters || L.counters_capacity < p.tiles_total || !L.partials ||
        L.partials_bytes < (size_t)p.tiles_total * p.slots * 32 * sizeof(float))
        return -1;
    p.partials = L.partials;
    p.counters = L.counters;
    const size_t smem = qgemv_smem(w.type, p.K, p.nvec);
    auto kern = w.type == T_Q4_K ? (p.nvec == 1 ? qgemv_kernel<T_Q4_K, 1> : qgemv_kernel<T_Q4_K, 2>)
                                 : (p.nvec == 1 ? qgemv_kernel<T_Q6_K, 1> : qgemv_kernel<T_Q6_K, 2>);
    // The max-shared carveout lets the next kernel's CTAs (programmatic
    // dependent launch) sit next to this one and start their weight streams.
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) != cudaSuccess)
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
