// decode_df.cuh - the dataflow form of the persistent decode kernel (shares
// the unit math, attention and helpers of decode_kernel.cuh).
#pragma once
#include "decode_kernel.cuh"

namespace fyb {

//
// The barrier form makes every CTA wait for the whole input vector of a
// phase, prepare all of it, and meet its warps at the end of the phase. Here
// each GEMV unit (16-row tile, 256-column block b) waits only for block b of
// its input: producers count finished tiles per 256-row block (O, down) or
// per 256-row block of h (gate/up), and attention per KV head. On entering a
// phase every half-warp of the CTA claims one block (shared-memory state
// word), waits until its producers are done, splits its 256 values into
// limbs in the CTA's buffer for the phase and marks it ready, so the blocks
// are prepared in parallel as they become ready; a unit whose block is not
// ready yet waits for it or, if nobody claimed it, prepares it. Consecutive
// GEMV phases use two limb buffers (A: d-column phases, B: O and down), and a
// warp may start the next phase while its siblings finish the current one.
//
// RMSNorm: the limbs hold x * w and the tile outputs multiply by the scale
// 1/sqrt(mean(x^2) + eps) (a scalar, so W (x * scale * w) = scale * W (x * w)),
// which the CTA forms from the per-block sums of squares of the blocks it
// prepared; every CTA prepares every block, and all of a tile's blocks are
// ready before its output, so no global reduction is needed.
//
// Tiles a warp covers completely produce their output at once; tiles shared
// by warps of a CTA meet in shared-memory slots, and the warp whose units
// complete the tile adds the slots in warp order. A tile's output is followed
// by the warp's fence and one counter update; no CTA barrier inside a GEMV
// phase. The attention phase stays CTA-wide.

constexpr unsigned DF_TILES_PER_CTA = 64;  // shared-tile counters per CTA (tiles a CTA owns in one phase)

struct DfBuf {           // one limb buffer (shared memory)
    signed char *xl;
    unsigned xstride;
    int *exps;
    float *gsums;
    unsigned *state;     // per block: 2 seq + 1 claimed, 2 seq + 2 ready (phase seq)
    double *bss;         // per block: sum of x^2 (norm phases)
};

struct DfShared {
    DfBuf a, b;          // limb buffers: a for QKV, gate/up, logits; b for O, down
    PartSlot *slots;     // [2 parities][warps][2]: a warp's first (0) and last (1) tile
    unsigned *tcount;    // [2][DF_TILES_PER_CTA] units done per shared tile
    unsigned *exits;     // [2] warps that left a phase using buffer A / B
    unsigned long long *cta_key;  // logits: the CTA's best key
    unsigned *cta_logit_warps;    // logits: warps of the CTA done
};

using DfSync = DecodeDfSync;

FYB_DEV bool spin_smem_eq(const DecodeParams &p, const volatile unsigned *w, unsigned value)
{
    for (unsigned i = 0; i < WAIT_LIMIT; ++i) {
        if (*w == value) return true;
        if (aborted(p)) return false;
        __nanosleep(20);
    }
    raise_abort(p, ERR_TIMEOUT);
    return false;
}

FYB_DEV bool spin_smem_geq(const DecodeParams &p, const volatile unsigned *w, unsigned value)
{
    for (unsigned i = 0; i < WAIT_LIMIT; ++i) {
        if (reached(*w, value)) return true;
        if (aborted(p)) return false;
        __nanosleep(20);
    }
    raise_abort(p, ERR_TIMEOUT);
    return false;
}

// One lane polls a global counter (acquire) until it reached target.
FYB_DEV bool lane_wait(const DecodeParams &p, const unsigned *ctr, unsigned target)
{
    for (unsigned i = 0; i < WAIT_LIMIT; ++i) {
        if (reached(ld_acquire(ctr), target)) return true;
        if (aborted(p)) return false;
        __nanosleep(32);
    }
    raise_abort(p, ERR_TIMEOUT);
    return false;
}

// Global readiness of input block b of phase ph at this step (one lane).
FYB_DEV bool df_block_ready(const DecodeParams &p, const DfSync &ds, const Phase &ph, unsigned b, unsigned step)
{
    const unsigned l = ph.layer, nbd = p.d / 256;
    switch (ph.kind) {
    case PH_QKV:
        return l == 0 || lane_wait(p, ds.bdn + (l - 1) * nbd + b, 16 * step);
    case PH_O: {  // the KV heads whose query heads the block's 256 rows belong to
        const unsigned G = p.H / p.Hkv, k0 = (b * 256 / p.hd) / G, k1 = ((b * 256 + 255) / p.hd) / G;
        for (unsigned kvh = k0; kvh <= k1; ++kvh)
            if (!lane_wait(p, ds.attn_kv + l * p.Hkv + kvh, step)) return false;
        return true;
    }
    case PH_GATEUP:
        return lane_wait(p, ds.bo + l * nbd + b, 16 * step);
    case PH_DOWN:
        return lane_wait(p, ds.bgu + l * (p.ffn / 256) + b, 32 * step);
    default:  // PH_LOGITS
        return lane_wait(p, ds.bdn + (p.nl - 1) * nbd + b, 16 * step);
    }
}

// Split block b (one per half-warp; `ok` for this half) of the phase's input
// into limbs. Every lane calls it: prep_slot shuffles within half-warps.
FYB_DEV void df_prep_half(const DecodeParams &p, const Phase &ph, const DfBuf &bf, unsigned b, bool ok,
    unsigned lane)
{
    const unsigned K = ph.K, nblk = ph.nblk;
    const unsigned sl = ok ? 16 * b + (lane & 15) : 0;
    const bool norm = ph.kind == PH_QKV || ph.kind == PH_GATEUP || ph.kind == PH_LOGITS;
    float x[16], w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) { x[j] = 0.f; w[j] = 1.f; }
    if (ok) {
        const float *nw = ph.kind == PH_QKV ? p.layers[ph.layer].attn_norm
                        : ph.kind == PH_GATEUP ? p.layers[ph.layer].ffn_norm : p.out_norm;
        if (norm) load16(nw + 16 * sl, w);
        if (ph.kind == PH_QKV && ph.layer == 0) {
            const unsigned char *erow = p.embd + (unsigned long long)__ldcg(p.request) * p.embd_row_bytes;
#pragma unroll
            for (int j = 0; j < 16; ++j) x[j] = dequant_any(erow, 16ull * sl + j, p.embd_type);
        } else {
            const float *src = ph.kind == PH_O ? p.attn : ph.kind == PH_GATEUP ? p.xm : ph.kind == PH_DOWN ? p.h : p.xa;
            load16(src + 16 * sl, x);
        }
    }
    if (norm) {
        double sq = 0.0;
#pragma unroll
        for (int j = 0; j < 16; ++j) sq += (double)x[j] * (double)x[j];
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (ok && (lane & 15) == 0) bf.bss[b] = sq;
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] = __fmul_rn(x[j], w[j]);
    }
    prep_slot(x, ok, 0, sl, K, nblk, bf.xl, bf.xstride, bf.exps, bf.gsums, p.error);
}

// Phase entry: half-warp h of warp w claims block 2w + h (+ 32k), waits for
// its producers and prepares it, so all blocks get prepared in parallel.
FYB_DEV bool df_eager_blocks(const DecodeParams &p, const DfSync &ds, const Phase &ph, const DfBuf &bf,
    unsigned seq, unsigned step, unsigned lane)
{
    const unsigned warp = threadIdx.x >> 5, half = lane >> 4, leader = lane & 16;
    const unsigned claimed = 2 * seq + 1, ready = 2 * seq + 2;
    for (unsigned base = 2 * warp; base < ph.nblk; base += 2 * QG_WARPS) {
        const unsigned b = base + half;
        unsigned mine = 0;
        if ((lane & 15) == 0 && b < ph.nblk) {
            volatile unsigned *st = bf.state + b;
            const unsigned s = *st;
            if (s != claimed && s != ready) mine = atomicCAS(const_cast<unsigned *>(st), s, claimed) == s;
            if (mine && !df_block_ready(p, ds, ph, b, step)) mine = 2;  // abort while waiting
        }
        mine = __shfl_sync(0xffffffffu, mine, leader);
        const unsigned other = __shfl_xor_sync(0xffffffffu, mine, 16);
        if (mine == 2 || other == 2) return false;
        if (!mine && !other) continue;
        df_prep_half(p, ph, bf, b, mine == 1, lane);
        __threadfence_block();
        __syncwarp();
        if (mine == 1 && (lane & 15) == 0) *(volatile unsigned *)(bf.state + b) = ready;
    }
    return true;
}

// Make block b of the phase's buffer ready (claim and prepare it, or wait
// for the warp that claimed it). Warp-uniform; false on abort.
FYB_DEV bool df_ensure_block(const DecodeParams &p, const DfSync &ds, const Phase &ph, const DfBuf &bf, unsigned b,
    unsigned seq, unsigned step, unsigned lane)
{
    volatile unsigned *st = bf.state + b;
    const unsigned claimed = 2 * seq + 1, ready = 2 * seq + 2;
    for (unsigned i = 0; i < WAIT_LIMIT; ++i) {
        unsigned s = lane == 0 ? *st : 0;
        s = __shfl_sync(0xffffffffu, s, 0);
        if (s == ready) {
            __threadfence_block();
            return true;
        }
        if (s == claimed) {
            bool okw = true;
            if (lane == 0) okw = spin_smem_eq(p, st, ready);
            okw = __shfl_sync(0xffffffffu, okw ? 1 : 0, 0) != 0;
            if (!okw) return false;
            __threadfence_block();
            return true;
        }
        unsigned won = 0;
        if (lane == 0) won = atomicCAS(const_cast<unsigned *>(st), s, claimed) == s;
        won = __shfl_sync(0xffffffffu, won, 0);
        if (!won) continue;
        bool okr = true;
        if (lane == 0) okr = df_block_ready(p, ds, ph, b, step);
        okr = __shfl_sync(0xffffffffu, okr ? 1 : 0, 0) != 0;
        if (!okr) return false;
        df_prep_half(p, ph, bf, b, lane < 16, lane);
        __threadfence_block();
        __syncwarp();
        if (lane == 0) *st = ready;
        return true;
    }
    raise_abort(p, ERR_TIMEOUT);
    return false;
}

// The RMSNorm scale from the CTA's per-block sums (all blocks are ready).
FYB_DEV float df_scale(const DecodeParams &p, const DfBuf &bf, unsigned nblk, unsigned lane)
{
    double s = 0.0;
    for (unsigned b = lane; b < nblk; b += 32) s += bf.bss[b];
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return (float)(1.0 / sqrt(s / (double)(nblk * 256) + (double)p.eps));
}

// Output of one complete tile and its counter update.
FYB_DEV void df_output(const DecodeParams &p, const DfSync &ds, const Phase &ph, const DfBuf &bf, unsigned tile,
    float yA, float yB, unsigned lane, unsigned long long &key, const TileIn &in, unsigned ta, float &scale)
{
    const unsigned gid = lane >> 2, l = ph.layer;
    const bool mine = (lane & 3) == 0;
    const int k = tile == ta ? 0 : tile == ta + 1 ? 1 : -1;  // the fetched inputs, if any
    if (ph.kind == PH_QKV || ph.kind == PH_GATEUP || ph.kind == PH_LOGITS) {
        if (scale < 0.f) scale = df_scale(p, bf, ph.nblk, lane);
        yA *= scale;
        yB *= scale;
    }
    if (ph.kind == PH_QKV) {
        const unsigned tq = p.H * p.hd / 16, tk = p.Hkv * p.hd / 16, hd = p.hd;
        const unsigned seg = tile < tq ? 0 : tile < tq + tk ? 1 : 2;
        const unsigned lt = tile - (seg == 0 ? 0 : seg == 1 ? tq : tq + tk);
        const unsigned rowA = lt * 16 + 2 * gid;
        if (mine) {
            const unsigned pos = __ldcg(p.request + 1), pair = (rowA % hd) >> 1;
            float a = yA, b = yB;
            if (seg <= 1) {  // llm_cpu.c:298-327
                const float c = k == 0 ? in.a0 : k == 1 ? in.a1 : p.rope_cos[(size_t)pos * (hd >> 1) + pair];
                const float s = k == 0 ? in.b0 : k == 1 ? in.b1 : p.rope_sin[(size_t)pos * (hd >> 1) + pair];
                a = __fsub_rn(__fmul_rn(yA, c), __fmul_rn(yB, s));
                b = __fadd_rn(__fmul_rn(yA, s), __fmul_rn(yB, c));
            }
            if (seg == 0) {
                *reinterpret_cast<float2 *>(p.q + rowA) = make_float2(a, b);
            } else {
                const unsigned kvh = rowA / hd, dd = rowA % hd;
                __half *cache = seg == 1 ? kv_layer(p, l, false) : kv_layer(p, l, true);
                *reinterpret_cast<__half2 *>(cache + ((size_t)kvh * p.capacity + pos) * hd + dd) =
                    __halves2half2(__float2half_rn(a), __float2half_rn(b));
            }
        }
        if (mine) __threadfence();  // the lanes that wrote, before the counter
        __syncwarp();
        if (lane == 0) atomicAdd(p.sync.qkv_done + l * p.Hkv + qkv_kvh(p, tile), 1u);
        return;
    }
    if (ph.kind == PH_O || ph.kind == PH_DOWN) {
        const unsigned rA = tile * 16 + gid, rB = rA + 8;
        if (mine) {
            float rsA, rsB;
            if (k >= 0 && !(ph.kind == PH_O && l == 0)) {
                rsA = k == 0 ? in.a0 : in.a1;
                rsB = k == 0 ? in.b0 : in.b1;
            } else if (ph.kind == PH_O) {
                rsA = residual_in(p, l, rA); rsB = residual_in(p, l, rB);
            } else {
                rsA = __ldcg(p.xm + rA); rsB = __ldcg(p.xm + rB);
            }
            float *dst = ph.kind == PH_O ? p.xm : p.xa;
            dst[rA] = __fadd_rn(rsA, yA);
            dst[rB] = __fadd_rn(rsB, yB);
        }
        if (mine) __threadfence();  // the lanes that wrote, before the counter
        __syncwarp();
        if (lane == 0) atomicAdd((ph.kind == PH_O ? ds.bo : ds.bdn) + l * (p.d / 256) + tile / 16, 1u);
        return;
    }
    if (ph.kind == PH_GATEUP) {
        if (mine) {  // llm_cpu.c:336-342: gate / (1 + expf(-gate)) * up
            const float g = __fdiv_rn(yA, __fadd_rn(1.0f, expf(-yA)));
            p.h[tile * 8 + gid] = __fmul_rn(g, yB);
        }
        if (mine) __threadfence();  // the lanes that wrote, before the counter
        __syncwarp();
        if (lane == 0) atomicAdd(ds.bgu + l * (p.ffn / 256) + tile / 32, 1u);
        return;
    }
    // PH_LOGITS: store and fold into the warp's key (ties to the lowest index)
    const unsigned rA = tile * 16 + gid, rB = rA + 8;
    unsigned long long kk = 0ull;
    if (mine) {
        const bool okA = rA < p.V, okB = rB < p.V;
        if (okA) p.logits[rA] = yA;
        if (okB) p.logits[rB] = yB;
        if (((okA && !isfinite(yA)) || (okB && !isfinite(yB))) && p.error) atomicCAS(p.error, 0u, ERR_NONFINITE);
        const unsigned long long kA = okA ? ((unsigned long long)float_order_key(yA) << 32) | (0xffffffffu - rA) : 0ull;
        const unsigned long long kB = okB ? ((unsigned long long)float_order_key(yB) << 32) | (0xffffffffu - rB) : 0ull;
        kk = kA > kB ? kA : kB;
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, kk, o);
        kk = other > kk ? other : kk;
    }
    key = kk > key ? kk : key;
}

// One GEMV phase of this warp (phase number seq; buffer seq & 1).
template <unsigned TYPE>
FYB_DEV bool df_gemv(const DecodeParams &p, const DfSync &ds, const DfShared &sh, const Phase &ph, Ring &r,
    unsigned seq, unsigned step, unsigned lane)
{
    wstamp(p, ph, 0, lane);
    const unsigned warp = threadIdx.x >> 5, par = seq & 1, use = seq >> 1, n = r.n;
    if (warp_aborted(p)) {  // leave at once (the ring may not hold this phase's units)
        if (lane == 0) atomicAdd(sh.exits + par, 1u);
        return false;
    }
    const DfBuf bf = par ? sh.b : sh.a;
    while (r.issued < n && r.issued < r.S) ring_issue(r, lane);  // the ring may have started shallow
    const unsigned nblk = ph.nblk, gid = lane >> 2, tig = lane & 3;
    // the previous use of this buffer (two phases back) is over for every warp of the CTA
    bool ok = true;
    if (lane == 0) ok = spin_smem_geq(p, sh.exits + par, QG_WARPS * use);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    if (ok) ok = df_eager_blocks(p, ds, ph, bf, seq, step, lane);
    wstamp(p, ph, 4, lane);
    unsigned tb, te;
    cta_tiles(ph, tb, te);
    // tiles this warp touches (it may produce any of them: a shared tile's
    // output comes from whichever warp completes it)
    const unsigned ta = (unsigned)(r.u0 / nblk), tz = (unsigned)((r.u0 + n + nblk - 1) / nblk);
    TileIn in;
    fetch_rope(p, ph, ta, tz, lane, in);
    const bool want_resid = ph.kind == PH_DOWN || (ph.kind == PH_O && ph.layer > 0);
    PartSlot *mine = sh.slots + (par * QG_WARPS + warp) * 2;
    float accA = 0.f, accB = 0.f, scale = -1.f;
    unsigned tile = ta, tile_units = 0;
    unsigned blk = (unsigned)(r.u0 - (unsigned long long)tile * nblk);
    unsigned long long key = 0ull;
    long long wait_cycles = 0, block_cycles = 0, out_cycles = 0;
    for (unsigned i = 0; i < n && ok; ++i) {
        const long long b0 = p.wtrace ? clock64() : 0;
        ok = df_ensure_block(p, ds, ph, bf, blk, seq, step, lane);
        if (p.wtrace) block_cycles += clock64() - b0;
        if (!ok) break;
        if (i == 0 && want_resid) fetch_resid(p, ph, ta, tz, lane, in);
        const long long c0 = p.wtrace ? clock64() : 0;
        const unsigned char *unit = ring_wait(r);
        if (!unit) { raise_abort(p, ERR_TIMEOUT); ok = false; break; }
        if (p.wtrace) wait_cycles += clock64() - c0;
        compute_unit<TYPE, 1>(unit, blk, bf.xl, bf.xstride, bf.exps, nblk, bf.gsums, ph.K / 32, lane, accA, accB);
        __syncwarp();
        if (r.issued < n) ring_issue(r, lane);
        ++tile_units;
        const bool tile_end = blk + 1 == nblk;
        blk = tile_end ? 0 : blk + 1;
        if (tile_end || i + 1 == n) {
            const long long o0 = p.wtrace ? clock64() : 0;
            const float yA = lane_total<1>(accA), yB = lane_total<1>(accB);
            if (tile_units == nblk) {
                df_output(p, ds, ph, bf, tile, yA, yB, lane, key, in, ta, scale);
            } else {
                // a tile shared with other warps of the CTA (only a warp's
                // first and last tiles can be): leave this part; the warp
                // whose units complete the tile adds the parts in warp order
                PartSlot &ps = mine[tile == ta ? 0 : 1];
                if (tig == 0) { ps.v[gid] = yA; ps.v[gid + 8] = yB; }
                __threadfence_block();
                __syncwarp();
                unsigned old = 0;
                unsigned *tc = sh.tcount + par * DF_TILES_PER_CTA + (tile - tb);
                if (lane == 0) old = atomicAdd(tc, tile_units);
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old + tile_units == nblk) {
                    __threadfence_block();
                    // the warps whose unit ranges meet this tile, and which of their slots holds it
                    const unsigned Uc = (te - tb) * nblk, lo = (tile - tb) * nblk, hi = lo + nblk;
                    float sA = 0.f, sB = 0.f;
                    for (unsigned w = 0; w < QG_WARPS; ++w) {
                        const unsigned a = Uc * w / QG_WARPS, e = Uc * (w + 1) / QG_WARPS;
                        if (a >= e || a >= hi || e <= lo) continue;
                        const PartSlot &q = sh.slots[(par * QG_WARPS + w) * 2 + (a >= lo ? 0 : 1)];
                        sA += q.v[gid];
                        sB += q.v[gid + 8];
                    }
                    if (lane == 0) *tc = 0;
                    df_output(p, ds, ph, bf, tile, sA, sB, lane, key, in, ta, scale);
                }
            }
            accA = 0.f; accB = 0.f;
            tile_units = 0;
            if (tile_end) ++tile;
            if (p.wtrace) out_cycles += clock64() - o0;
        }
    }
    wrecord(p, ph, 1, lane, (unsigned long long)wait_cycles);
    wrecord(p, ph, 5, lane, (unsigned long long)block_cycles);
    wrecord(p, ph, 6, lane, (unsigned long long)out_cycles);
    wstamp(p, ph, 2, lane);
    // the ring is empty: the next phase's weights start now
    if (ok && !warp_aborted(p)) ring_next(p, ph, r, lane);
    if (ph.kind == PH_LOGITS) {
        // the CTA's best key, then one global update per CTA; the CTA that
        // completes the last tile publishes the token
        if (lane == 0) atomicMax(sh.cta_key, key);
        __threadfence_block();
        __syncwarp();
        unsigned last = 0;
        if (lane == 0) last = atomicAdd(sh.cta_logit_warps, 1u) == QG_WARPS - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last && lane == 0) {
            __threadfence_block();
            const unsigned long long best = atomicExch(sh.cta_key, 0ull);
            *sh.cta_logit_warps = 0;
            if (te > tb) {
                __threadfence();
                atomicMax(p.argmax_key, best);
                __threadfence();
                if (atomicAdd(p.sync.logit_tiles, te - tb) + (te - tb) == ph.w.tiles) {
                    __threadfence();
                    const unsigned long long kk = atomicExch(p.argmax_key, 0ull);
                    *p.argmax_token = 0xffffffffu - (unsigned)(kk & 0xffffffffu);
                    atomicExch(p.sync.logit_tiles, 0u);
                }
            }
        }
    }
    __syncwarp();
    if (lane == 0) atomicAdd(sh.exits + par, 1u);
    wstamp(p, ph, 3, lane);
    return ok;
}

FYB_DEV bool df_run(const DecodeParams &p, const DfSync &ds, const DfShared &sh, const Phase &ph, Ring &r,
    unsigned seq, unsigned step, unsigned lane)
{
    return ph.w.type == T_Q4_K ? df_gemv<T_Q4_K>(p, ds, sh, ph, r, seq, step, lane)
                               : df_gemv<T_Q6_K>(p, ds, sh, ph, r, seq, step, lane);
}

// ------------------------------------------------------------ layout and kernel
struct DfLayout {
    size_t bars, a_xl, a_exps, a_gsums, a_state, a_bss, b_xl, b_exps, b_gsums, b_state, b_bss;
    size_t slots, tcount, misc, total;
    unsigned ka, kb;  // columns of the phases using buffer a / b
};

FYB_HOST_DEV size_t df_align16(size_t x) { return (x + 15) / 16 * 16; }

// Rings first (ring_bytes per warp), then the barriers, the two limb buffers
// (buffer b also holds the attention scratch, idle then) and the small state.
FYB_HOST_DEV DfLayout df_layout(unsigned d, unsigned ffn, unsigned H, unsigned Hkv, unsigned hd,
    unsigned ring_bytes)
{
    DfLayout s;
    s.ka = d;
    s.kb = H * hd > ffn ? H * hd : ffn;
    const size_t abytes = attn_smem_floats(H / Hkv, hd) * 4, xb = (size_t)4 * (s.kb + QG_XPAD);
    s.bars = (size_t)QG_WARPS * ring_bytes;
    s.a_xl = s.bars + (size_t)QG_WARPS * RING_BARS * 8;
    s.a_exps = s.a_xl + df_align16((size_t)4 * (s.ka + QG_XPAD));
    s.a_gsums = s.a_exps + df_align16((size_t)(s.ka / 256) * 4);
    s.a_state = s.a_gsums + df_align16((size_t)(s.ka / 32) * 4);
    s.a_bss = s.a_state + df_align16((size_t)(s.ka / 256) * 4);
    s.b_xl = s.a_bss + df_align16((size_t)(s.ka / 256) * 8);
    s.b_exps = s.b_xl + df_align16(xb > abytes ? xb : abytes);
    s.b_gsums = s.b_exps + df_align16((size_t)(s.kb / 256) * 4);
    s.b_state = s.b_gsums + df_align16((size_t)(s.kb / 32) * 4);
    s.b_bss = s.b_state + df_align16((size_t)(s.kb / 256) * 4);
    s.slots = s.b_bss + df_align16((size_t)(s.kb / 256) * 8);
    s.tcount = s.slots + df_align16((size_t)2 * QG_WARPS * 2 * sizeof(PartSlot));
    s.misc = s.tcount + (size_t)2 * DF_TILES_PER_CTA * 4;
    s.total = s.misc + 48;  // exits[2], cta_logit_warps, flag words; cta_key at +32
    return s;
}

// The dataflow form of decode_kernel (single GPU): the same phases, with
// GEMV phases that start per input block instead of behind CTA barriers.
template <int HD, int G>
__global__ void __launch_bounds__(QG_THREADS, 1) decode_df_kernel(const DecodeParams p)
{
    extern __shared__ __align__(128) unsigned char smem[];
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const DfLayout lay = df_layout(p.d, p.ffn, p.H, p.Hkv, p.hd, p.ring_bytes);
    Ring ring;
    ring.base = smem + (size_t)warp * p.ring_bytes;
    ring.bars = reinterpret_cast<uint64_t *>(smem + lay.bars) + warp * RING_BARS;
    ring.bytes = p.ring_bytes;
    ring.pre = p.ring_pre;
    ring.par = 0;
    ring.issued = ring.consumed = ring.n = 0;
    DfShared sh;
    sh.a.xl = reinterpret_cast<signed char *>(smem + lay.a_xl);
    sh.a.xstride = lay.ka + QG_XPAD;
    sh.a.exps = reinterpret_cast<int *>(smem + lay.a_exps);
    sh.a.gsums = reinterpret_cast<float *>(smem + lay.a_gsums);
    sh.a.state = reinterpret_cast<unsigned *>(smem + lay.a_state);
    sh.a.bss = reinterpret_cast<double *>(smem + lay.a_bss);
    sh.b.xl = reinterpret_cast<signed char *>(smem + lay.b_xl);
    sh.b.xstride = lay.kb + QG_XPAD;
    sh.b.exps = reinterpret_cast<int *>(smem + lay.b_exps);
    sh.b.gsums = reinterpret_cast<float *>(smem + lay.b_gsums);
    sh.b.state = reinterpret_cast<unsigned *>(smem + lay.b_state);
    sh.b.bss = reinterpret_cast<double *>(smem + lay.b_bss);
    sh.slots = reinterpret_cast<PartSlot *>(smem + lay.slots);
    sh.tcount = reinterpret_cast<unsigned *>(smem + lay.tcount);
    unsigned *misc = reinterpret_cast<unsigned *>(smem + lay.misc);
    sh.exits = misc;
    sh.cta_logit_warps = misc + 2;
    unsigned *flag = misc + 3;
    sh.cta_key = reinterpret_cast<unsigned long long *>(misc + 8);
    AttnSmem as;  // overlays buffer b, idle between the QKV and O phases
    as.wm = reinterpret_cast<float *>(sh.b.xl);
    as.wl = as.wm + QG_WARPS * G;
    as.wo = as.wl + QG_WARPS * G;
    as.flag = misc + 4;

    for (unsigned i = threadIdx.x; i < lay.ka / 256; i += QG_THREADS) sh.a.state[i] = 0;
    for (unsigned i = threadIdx.x; i < lay.kb / 256; i += QG_THREADS) sh.b.state[i] = 0;
    for (unsigned i = threadIdx.x; i < 2 * DF_TILES_PER_CTA; i += QG_THREADS) sh.tcount[i] = 0;
    if (threadIdx.x < 8) misc[threadIdx.x] = 0;
    if (threadIdx.x == 0) *sh.cta_key = 0ull;
    if (lane == 0) {
        for (unsigned s = 0; s < RING_BARS; ++s) mbar_init(ring.bars + s, 1);
        fence_barrier_init();
    }
    __syncthreads();

    const unsigned step = __ldcg(p.request + 3) + 1;
    const DfSync ds = p.df;
    unsigned ts = 0, seq = 0;
    bool ok = true;
    stamp(p, ts);
    Phase cur = make_phase(p, PH_QKV, 0), nx0;
    ring_begin(cur, ring, lane, phase_after(p, PH_QKV, 0, nx0) ? &nx0 : nullptr, p.l2_prefetch);
    // A failed phase raises the abort word, so the CTA-wide wait before the
    // next attention phase fails for every warp: the CTA barriers stay in step.
    for (unsigned l = 0; l < p.nl; ++l) {
        df_run(p, ds, sh, cur, ring, seq++, step, lane); advance(p, cur);  // QKV; now O
        ok = cta_wait(p, nullptr, 0, flag, ts) && attention_phase<HD, G>(p, l, step, as);
        stamp(p, ts);
        if (!ok) break;
        df_run(p, ds, sh, cur, ring, seq++, step, lane); advance(p, cur);  // O; now gate/up
        df_run(p, ds, sh, cur, ring, seq++, step, lane); advance(p, cur);  // gate/up; now down
        df_run(p, ds, sh, cur, ring, seq++, step, lane); advance(p, cur);  // down; now QKV or logits
    }
    if (ok && p.logits_mode) df_run(p, ds, sh, cur, ring, seq++, step, lane);
    ring_drain(ring);
    end_step(p, flag, ts);
}

}  // namespace fyb
