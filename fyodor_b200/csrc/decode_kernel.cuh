// decode_kernel.cuh - one decode step of a dense LLaMA model as one persistent
// kernel (the engine's per-token graph, CUDA/resident.inc:470-552, and its
// CPU reference, backend/core/llm_cpu.c:424-578).
//
// One 512-thread CTA per SM, launched cooperatively so that every CTA is
// resident and waits between CTAs cannot deadlock. Per layer the CTAs walk
// the phases QKV(+RoPE, fp16 KV append) -> attention -> O -> gate/up(+SwiGLU)
// -> down, then logits(+argmax). Each GEMV phase splits its (16-row tile,
// 256-column block) units over all warps of the grid like the stand-alone
// GEMV (qgemv.cu); phases meet through counters in global memory instead of
// kernel boundaries:
//   qkv_done[l][kv head]  Q/K/V tiles of that KV head's group finished
//   attn_done[l]          KV heads whose attention output is final
//   o_done / gu_done / down_done[l]   finished tiles of those phases
// Counters only grow (modulo 2^32): step e waits for e * (tiles per step),
// compared wrap-safe, so nothing is reset between steps. The step number is
// request[3] + 1; the last CTA to leave increments request[3].
// Producers write their outputs, fence, then add to a counter; the waiting
// thread reads it with ld.acquire.gpu and the CTA reads produced data through
// L2 (ld.cg), never through the non-coherent read-only path. Every wait is
// bounded: on timeout the kernel records ERR_TIMEOUT and raises an abort word
// at which all CTAs leave (after their in-flight bulk copies land).
//
// Weights stream through a per-warp ring of shared memory sized in bytes
// (4 Q4_K or 3 Q6_K units for the 8B shapes). A warp that finishes its units
// of a phase fills its ring with its first units of the next phase at once,
// so while the CTA waits for the next phase's input those weights are already
// on their way; small phases (QKV, O) arrive almost entirely during the wait.
// Inside a phase a warp only computes: outputs of tiles it owns completely
// are written as they finish, while fences, counter updates and the stream-K
// fix-up of tiles shared with neighbouring warps wait until its last unit.
//
// The residual adds and the RMSNorm sums of squares live in the epilogues of
// the O and down tiles (x_mid = x + o_out, x_next = x_mid + down_out, one
// double per 16-row tile, summed in a fixed order by the consumers), so the
// input preparation of a phase is one round of loads, x * scale * weight and
// the limb split.
#pragma once
#include "qgemv_core.cuh"
#include "dequant.cuh"

namespace fyb {

constexpr unsigned WAIT_LIMIT = 1u << 22;  // polls (with a short sleep) before ERR_TIMEOUT
constexpr unsigned RING_BARS = 8;          // mbarriers (max units in flight) per warp

struct DecodeParams {
    const DecodeLayer *layers;
    unsigned nl, d, H, Hkv, hd, ffn, V, capacity;
    QWeights out_head;
    const float *out_norm;
    const unsigned char *embd;
    unsigned long long embd_row_bytes;
    unsigned embd_type;
    float eps, attn_scale;
    const float *rope_cos, *rope_sin;
    unsigned *request;
    float *xa, *xm, *q, *attn, *h, *logits;
    double *ss_o, *ss_d;
    DecodeSync sync;
    float *partials;
    float *attn_partials;
    unsigned attn_splits;
    unsigned long long *argmax_key;
    unsigned *argmax_token, *tokens_log;
    unsigned *error;
    int logits_mode;
    unsigned ring_bytes;        // per warp, a multiple of 16
    unsigned ring_pre;          // units a warp requests when it starts a phase's ring early (0: all S)
    int l2_prefetch;            // L2 prefetch of weights: 0 none, 1 the phase after next, 2 the rest of the next phase
    unsigned long long *trace;  // optional [stamp][CTA] globaltimer values
    unsigned trace_slots;
    unsigned long long *wtrace;  // optional [layer][phase kind][warp][WTRACE_POINTS] records
    // tensor parallelism (tp > 1): H, Hkv, ffn and V above are this rank's
    unsigned tp, tp_rank, vocab0;
    unsigned char *const *peers;  // [tp] exchange regions, this rank's at tp_rank
    XchgLayout xl;
    __half *kcache, *vcache;      // all layers' caches in one allocation each (null: use the layer table)
    DecodeDfSync df;  // dataflow form only (df.bo null otherwise)
};

enum PhaseKind { PH_QKV = 0, PH_O = 1, PH_GATEUP = 2, PH_DOWN = 3, PH_LOGITS = 4 };

struct Phase {
    QWeights w;
    unsigned K, nblk, kind, layer;
};

// A warp's weight ring. Per phase it holds S = min(RING_BARS, bytes / unit)
// units; unit k of the phase goes to slot k % S. Bit s of `par` is the
// parity the next wait on mbarrier s expects. The ring is empty between
// phases, so each phase may use its own unit size.
struct Ring {
    unsigned char *base;
    uint64_t *bars;
    unsigned bytes, par, pre;
    unsigned S, ub, issued, consumed, n;
    unsigned long long u0;
    const unsigned char *src;
};

struct XBuf {
    signed char *xl;
    unsigned xstride;
    int *exps;
    float *gsums;
};

FYB_DEV unsigned ld_acquire(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

FYB_DEV unsigned ld_acquire_sys(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

FYB_DEV bool reached(unsigned value, unsigned target) { return (int)(value - target) >= 0; }

// Exchange counters of rank j (tensor parallelism): o_x[l] at l, d_x[l] at
// nl + l, argmax keys at 2 nl, the shared abort word at 2 nl + 1.
FYB_DEV unsigned *xctr(const DecodeParams &p, unsigned j)
{
    return reinterpret_cast<unsigned *>(p.peers[j] + p.xl.ctr);
}

FYB_DEV void raise_abort(const DecodeParams &p, unsigned code)
{
    if (p.error) atomicCAS(p.error, 0u, code);
    atomicExch(p.sync.abort_flag, 1u);
    for (unsigned j = 0; p.tp > 1 && j < p.tp; ++j)  // the other ranks leave too
        if (j != p.tp_rank) atomicExch_system(xctr(p, j) + 2 * p.nl + 1, 1u);
}

FYB_DEV bool aborted(const DecodeParams &p) { return *(volatile unsigned *)p.sync.abort_flag != 0; }
// The same answer for every lane of the warp (ring counters must not diverge).
FYB_DEV bool warp_aborted(const DecodeParams &p) { return __shfl_sync(0xffffffffu, aborted(p) ? 1 : 0, 0) != 0; }

FYB_DEV unsigned long long globaltimer()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Profiling: thread 0 records the time of trace point `ts` (every CTA passes
// the same trace points in the same order).
FYB_DEV void stamp(const DecodeParams &p, unsigned &ts)
{
    if (p.trace && threadIdx.x == 0 && ts < p.trace_slots)
        p.trace[(size_t)ts * gridDim.x + blockIdx.x] = globaltimer();
    ++ts;
}

// Whole-CTA wait until *ctr reached target (ctr null: only the abort check).
// Thread 0 polls; false (for every thread) on abort or timeout. Trace points:
// the CTA is idle (all its warps arrived), the wait is over.
FYB_DEV bool cta_wait(const DecodeParams &p, const unsigned *ctr, unsigned target, unsigned *flag, unsigned &ts,
    bool sys = false)
{
    __syncthreads();
    stamp(p, ts);
    if (threadIdx.x == 0) {
        unsigned ok = 0;
        for (unsigned i = 0;; ++i) {
            if (aborted(p)) break;
            if (!ctr || reached(sys ? ld_acquire_sys(ctr) : ld_acquire(ctr), target)) { ok = 1; break; }
            if (i >= WAIT_LIMIT) { raise_abort(p, ERR_TIMEOUT); break; }
#ifndef FYB_POLL_NS
#define FYB_POLL_NS 32
#endif
            if (FYB_POLL_NS) __nanosleep(FYB_POLL_NS);
        }
        *flag = ok;
    }
    stamp(p, ts);
    __syncthreads();
    return *flag != 0;
}

// ------------------------------------------------------------ weight ring
// CTA c owns tiles [T*c/C, T*(c+1)/C) of the phase (whole tiles, balanced to
// one tile); its warps split that range of units evenly.
FYB_DEV void cta_tiles(const Phase &ph, unsigned &tb, unsigned &te)
{
    const unsigned long long T = ph.w.tiles, C = gridDim.x;
    tb = (unsigned)(T * blockIdx.x / C);
    te = (unsigned)(T * (blockIdx.x + 1) / C);
}

FYB_DEV void warp_range(const Phase &ph, unsigned long long &u0, unsigned &n)
{
    unsigned tb, te;
    cta_tiles(ph, tb, te);
    const unsigned Uc = (te - tb) * ph.nblk, w = threadIdx.x >> 5;
    const unsigned a = Uc * w / QG_WARPS, b = Uc * (w + 1) / QG_WARPS;
    u0 = (unsigned long long)tb * ph.nblk + a;
    n = b - a;
}

FYB_DEV void ring_issue(Ring &r, unsigned lane)
{
    const unsigned slot = r.issued % r.S;
    if (lane == 0) {
        fence_proxy_async();
        mbar_expect_tx(r.bars + slot, r.ub);
        bulk_copy_g2s(r.base + slot * r.ub, r.src + (r.u0 + r.issued) * r.ub, r.ub, r.bars + slot);
    }
    ++r.issued;
}

// Start a phase on an empty ring: this warp's range, and its first units.
// L2 prefetch (one bulk prefetch per warp) mode 2: the warp's units of this
// phase beyond the ring's first S, so HBM streams the whole phase into L2
// while the CTAs still wait for its input; mode 1 (with `next`): the warp's
// units of the phase after this one.
FYB_DEV void ring_begin(const Phase &ph, Ring &r, unsigned lane, const Phase *next, int l2_prefetch)
{
    warp_range(ph, r.u0, r.n);
    r.ub = unit_bytes(ph.w.type);
    r.S = min(RING_BARS, r.bytes / r.ub);
    r.src = ph.w.units;
    r.issued = r.consumed = 0;
    const unsigned pre = r.pre ? min(r.pre, r.S) : r.S;
    while (r.issued < r.n && r.issued < pre) ring_issue(r, lane);
    if (l2_prefetch == 2 && r.n > r.S && lane == 0)
        bulk_prefetch_l2(r.src + (r.u0 + r.S) * r.ub, (r.n - r.S) * r.ub);
    if (next && l2_prefetch == 1 && lane == 0) {
        unsigned long long v0;
        unsigned nn;
        warp_range(*next, v0, nn);
        const unsigned ubn = unit_bytes(next->w.type);
        if (nn) bulk_prefetch_l2(next->w.units + v0 * ubn, nn * ubn);
    }
}

// Wait for the next unit; its shared-memory address, or null on timeout.
FYB_DEV const unsigned char *ring_wait(Ring &r)
{
    const unsigned slot = r.consumed % r.S;
    const bool landed = mbar_wait_bounded(r.bars + slot, (r.par >> slot) & 1u);
    if (!__all_sync(0xffffffffu, landed)) return nullptr;
    r.par ^= 1u << slot;
    ++r.consumed;
    return r.base + slot * r.ub;
}

// Before leaving early: let the copies still in flight land (bounded).
FYB_DEV void ring_drain(Ring &r)
{
    while (r.consumed != r.issued)
        if (!ring_wait(r)) break;
}

// ------------------------------------------------------------ input preparation
// x = the embedding row of the request's token (layer 0) or a buffer written
// earlier in this step, RMS-normalized when norm_w is set (scale from the
// per-tile sums `ss`, or a block reduction for the embedding row), split into
// limbs in shared memory. All loads of a pass are issued before any result
// is used, so a pass costs one round trip to L2.
FYB_DEV void prep_input(const DecodeParams &p, bool embed, const float *buf, const double *ss, unsigned ss_n,
    const float *norm_w, unsigned K, const XBuf &xb, double *red, float *scale_smem)
{
    const unsigned tid = threadIdx.x, nslot = K / 16, nblk = K / 256;
    const unsigned char *erow = nullptr;
    if (embed) erow = p.embd + (unsigned long long)__ldcg(p.request) * p.embd_row_bytes;
    auto load = [&](unsigned sl, float (&x)[16]) {
        if (embed) {
#pragma unroll
            for (int j = 0; j < 16; ++j) x[j] = dequant_any(erow, 16ull * sl + j, p.embd_type);
        } else {
            load16(buf + 16 * sl, x);
        }
    };
    if (norm_w && nslot <= QG_THREADS) {
        // one pass: x and the norm weight stay in registers while the scale forms
        const bool ok = tid < nslot;
        const unsigned sl = ok ? tid : 0;
        float x[16], w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) { x[j] = 0.f; w[j] = 0.f; }
        if (ok) { load(sl, x); load16(norm_w + 16 * sl, w); }
        double total = 0.0;
        if (embed) {
            if (ok) {
#pragma unroll
                for (int j = 0; j < 16; ++j) total += (double)x[j] * (double)x[j];
            }
            total = block_sum_double(total, red);
            if (tid == 0) *scale_smem = (float)(1.0 / sqrt(total / (double)K + (double)p.eps));
        } else if (tid < 32) {
#pragma unroll 8
            for (unsigned i = tid; i < ss_n; i += 32) total += __ldcg(ss + i);
#pragma unroll
            for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
            if (tid == 0) *scale_smem = (float)(1.0 / sqrt(total / (double)K + (double)p.eps));
        }
        __syncthreads();
        const float scale = *scale_smem;
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] = __fmul_rn(__fmul_rn(x[j], scale), w[j]);
        prep_slot(x, ok, 0, sl, K, nblk, xb.xl, xb.xstride, xb.exps, xb.gsums, p.error);
        __syncthreads();
        return;
    }
    float scale = 1.f;
    if (norm_w) {  // larger vectors: the scale first, then the passes
        double total = 0.0;
        if (embed) {
            for (unsigned s = tid; s < nslot; s += QG_THREADS) {
                float x[16];
                load(s, x);
#pragma unroll
                for (int j = 0; j < 16; ++j) total += (double)x[j] * (double)x[j];
            }
            total = block_sum_double(total, red);
            if (tid == 0) *scale_smem = (float)(1.0 / sqrt(total / (double)K + (double)p.eps));
        } else if (tid < 32) {
#pragma unroll 8
            for (unsigned i = tid; i < ss_n; i += 32) total += __ldcg(ss + i);
#pragma unroll
            for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
            if (tid == 0) *scale_smem = (float)(1.0 / sqrt(total / (double)K + (double)p.eps));
        }
        __syncthreads();
        scale = *scale_smem;
    }
    // two passes per round of loads
    for (unsigned s0 = 0; s0 < nslot; s0 += 2 * QG_THREADS) {
        const unsigned sa = s0 + tid, sb = s0 + QG_THREADS + tid;
        const bool oka = sa < nslot, okb = sb < nslot;
        float xa[16], xb2[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) { xa[j] = 0.f; xb2[j] = 0.f; }
        if (oka) load(sa, xa);
        if (okb) load(sb, xb2);
        if (norm_w) {
            float w[16];
            if (oka) {
                load16(norm_w + 16 * sa, w);
#pragma unroll
                for (int j = 0; j < 16; ++j) xa[j] = __fmul_rn(__fmul_rn(xa[j], scale), w[j]);
            }
            if (okb) {
                load16(norm_w + 16 * sb, w);
#pragma unroll
                for (int j = 0; j < 16; ++j) xb2[j] = __fmul_rn(__fmul_rn(xb2[j], scale), w[j]);
            }
        }
        prep_slot(xa, oka, 0, oka ? sa : 0, K, nblk, xb.xl, xb.xstride, xb.exps, xb.gsums, p.error);
        if (s0 + QG_THREADS < nslot)  // uniform: whether a second pass exists
            prep_slot(xb2, okb, 0, okb ? sb : 0, K, nblk, xb.xl, xb.xstride, xb.exps, xb.gsums, p.error);
    }
    __syncthreads();
}

// Tensor-parallel input of QKV, gate/up and the logits: x = base + the ranks'
// partial rows in rank order (so every rank computes the same x), or the
// embedding row; x is written back in shares (slot s by CTA s % grid) when
// `share` is set, its sum of squares reduced over the CTA, and x * scale * w
// split into limbs. One slot per thread (d <= 16 * threads).
FYB_DEV void prep_tp(const DecodeParams &p, bool embed, const float *base, const float *parts, float *share,
    const float *norm_w, const XBuf &xb, double *red)
{
    const unsigned tid = threadIdx.x, K = p.d, nslot = K / 16, nblk = K / 256;
    const bool ok = tid < nslot;
    const unsigned sl = ok ? tid : 0;
    float x[16], w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) { x[j] = 0.f; w[j] = 0.f; }
    if (ok) {
        load16(norm_w + 16 * sl, w);
        if (embed) {
            const unsigned char *erow = p.embd + (unsigned long long)__ldcg(p.request) * p.embd_row_bytes;
#pragma unroll
            for (int j = 0; j < 16; ++j) x[j] = dequant_any(erow, 16ull * sl + j, p.embd_type);
        } else {
            load16(base + 16 * sl, x);
#pragma unroll 8
            for (unsigned r = 0; r < 8; ++r) {
                if (r < p.tp) {
                    float y[16];
                    load16(parts + (size_t)r * K + 16 * sl, y);
#pragma unroll
                    for (int j = 0; j < 16; ++j) x[j] = __fadd_rn(x[j], y[j]);
                }
            }
        }
        if (share && sl % gridDim.x == blockIdx.x) {
            float4 *o4 = reinterpret_cast<float4 *>(share + 16 * sl);
#pragma unroll
            for (int i = 0; i < 4; ++i) o4[i] = make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
        }
    }
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < 16; ++j) ss += (double)x[j] * (double)x[j];
    ss = block_sum_double(ss, red);
    const float scale = (float)(1.0 / sqrt(ss / (double)K + (double)p.eps));
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = __fmul_rn(__fmul_rn(x[j], scale), w[j]);
    prep_slot(x, ok, 0, sl, K, nblk, xb.xl, xb.xstride, xb.exps, xb.gsums, p.error);
    __syncthreads();
}

// ------------------------------------------------------------ tile outputs
FYB_DEV float residual_in(const DecodeParams &p, unsigned layer, unsigned r)
{
    if (layer == 0)
        return dequant_any(p.embd + (unsigned long long)__ldcg(p.request) * p.embd_row_bytes, r, p.embd_type);
    return __ldcg(p.xa + r);
}

FYB_DEV unsigned qkv_kvh(const DecodeParams &p, unsigned tile)
{
    const unsigned tq = p.H * p.hd / 16, tk = p.Hkv * p.hd / 16;
    if (tile < tq) return (tile * 16 / p.hd) / (p.H / p.Hkv);
    return ((tile < tq + tk ? tile - tq : tile - tq - tk) * 16) / p.hd;
}

// Layer l's K (or V) cache: one allocation for all layers when the plan gives
// its base (no pointer chase through the layer table), else the table.
FYB_DEV __half *kv_layer(const DecodeParams &p, unsigned l, bool v)
{
    if (p.kcache) return (v ? p.vcache : p.kcache) + (size_t)l * p.Hkv * p.capacity * p.hd;
    return v ? p.layers[l].vcache : p.layers[l].kcache;
}

// Inputs the output tiles of a warp need besides the GEMV result (for the
// first two tiles it touches): RoPE factors (QKV) or residual rows (O, down).
struct TileIn {
    float a0, a1, b0, b1;
};

// RoPE factors of the QKV tiles (constant tables: loaded at phase start).
FYB_DEV void fetch_rope(const DecodeParams &p, const Phase &ph, unsigned ta, unsigned tz, unsigned lane,
    TileIn &in)
{
    const unsigned gid = lane >> 2;
    const unsigned tq = p.H * p.hd / 16, tk = p.Hkv * p.hd / 16, hd = p.hd;
    in.a0 = in.a1 = in.b0 = in.b1 = 0.f;
    if (ph.kind != PH_QKV || (lane & 3)) return;
    const unsigned pos = __ldcg(p.request + 1);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const unsigned t = ta + k;
        if (t >= tz || t >= tq + tk) continue;
        const unsigned lt = t < tq ? t : t - tq, pair = ((lt * 16 + 2 * gid) % hd) >> 1;
        const float c = p.rope_cos[(size_t)pos * (hd >> 1) + pair], s = p.rope_sin[(size_t)pos * (hd >> 1) + pair];
        if (k == 0) { in.a0 = c; in.b0 = s; } else { in.a1 = c; in.b1 = s; }
    }
}

// Residual rows of the O (layers after the first) and down tiles. The
// barrier form loads them at phase start (their writers finished phases
// ago); the dataflow form once the warp's first input block is ready, which
// orders them after their writers.
FYB_DEV void fetch_resid(const DecodeParams &p, const Phase &ph, unsigned ta, unsigned tz, unsigned lane,
    TileIn &in)
{
    const unsigned gid = lane >> 2;
    if (lane & 3) return;
    const float *src = ph.kind == PH_O ? p.xa : p.xm;
    if (ta < tz) { in.a0 = __ldcg(src + ta * 16 + gid); in.b0 = __ldcg(src + ta * 16 + gid + 8); }
    if (ta + 1 < tz) { in.a1 = __ldcg(src + (ta + 1) * 16 + gid); in.b1 = __ldcg(src + (ta + 1) * 16 + gid + 8); }
}

// Output of one complete tile (no fences, no counters). Lanes with tig == 0
// hold yA (MMA row gid) and yB (row gid + 8). LOGITS folds the tile's rows
// into the warp's running argmax key. `in` holds the RoPE factors or
// residual rows of tiles ta and ta + 1 (other tiles load them here).
FYB_DEV void tile_output(const DecodeParams &p, const Phase &ph, unsigned tile, float yA, float yB, unsigned lane,
    unsigned long long &key, const TileIn &in, unsigned ta)
{
    const int k = tile == ta ? 0 : tile == ta + 1 ? 1 : -1;
    const unsigned gid = lane >> 2;
    const bool mine = (lane & 3) == 0;
    const unsigned l = ph.layer;
    if (ph.kind == PH_QKV) {
        // rows 2*gid and 2*gid+1 of the tile form one RoPE pair (llm_cpu.c:298-327)
        const unsigned tq = p.H * p.hd / 16, tk = p.Hkv * p.hd / 16, hd = p.hd;
        const unsigned seg = tile < tq ? 0 : tile < tq + tk ? 1 : 2;
        const unsigned lt = tile - (seg == 0 ? 0 : seg == 1 ? tq : tq + tk);
        const unsigned rowA = lt * 16 + 2 * gid;
        if (mine) {
            const unsigned pos = __ldcg(p.request + 1), pair = (rowA % hd) >> 1;
            float a = yA, b = yB;
            if (seg <= 1) {
                const float c = k == 0 ? in.a0 : k == 1 ? in.a1 : p.rope_cos[(size_t)pos * (hd >> 1) + pair];
                const float s = k == 0 ? in.b0 : k == 1 ? in.b1 : p.rope_sin[(size_t)pos * (hd >> 1) + pair];
                a = __fsub_rn(__fmul_rn(yA, c), __fmul_rn(yB, s));
                b = __fadd_rn(__fmul_rn(yA, s), __fmul_rn(yB, c));
            }
            if (seg == 0) {
                *reinterpret_cast<float2 *>(p.q + rowA) = make_float2(a, b);
            } else {
                const unsigned kvh = rowA / hd, dd = rowA % hd;
                __half *cache = kv_layer(p, l, seg == 2);
                *reinterpret_cast<__half2 *>(cache + ((size_t)kvh * p.capacity + pos) * hd + dd) =
                    __halves2half2(__float2half_rn(a), __float2half_rn(b));
            }
        }
        return;
    }
    if ((ph.kind == PH_O || ph.kind == PH_DOWN) && p.tp > 1) {
        // this rank's partial rows go to every rank's exchange region; the
        // residual add and the sum of squares follow the exchange
        if (mine) {
            const size_t off = (ph.kind == PH_O ? p.xl.xo : p.xl.xd) + ((size_t)p.tp_rank * p.d + tile * 16 + gid) * 4;
            for (unsigned j = 0; j < p.tp; ++j) {
                float *dst = reinterpret_cast<float *>(p.peers[j] + off);
                dst[0] = yA;
                dst[8] = yB;
            }
        }
        return;
    }
    if (ph.kind == PH_O || ph.kind == PH_DOWN) {
        const unsigned rA = tile * 16 + gid, rB = rA + 8;
        double sq = 0.0;
        if (mine) {
            float xA, xB;
            const bool pre = k >= 0 && !(ph.kind == PH_O && l == 0);  // prefetched residual rows
            if (ph.kind == PH_O) {
                xA = __fadd_rn(pre ? (k ? in.a1 : in.a0) : residual_in(p, l, rA), yA);
                xB = __fadd_rn(pre ? (k ? in.b1 : in.b0) : residual_in(p, l, rB), yB);
                p.xm[rA] = xA; p.xm[rB] = xB;
            } else {
                xA = __fadd_rn(pre ? (k ? in.a1 : in.a0) : __ldcg(p.xm + rA), yA);
                xB = __fadd_rn(pre ? (k ? in.b1 : in.b0) : __ldcg(p.xm + rB), yB);
                p.xa[rA] = xA; p.xa[rB] = xB;
            }
            sq = (double)xA * (double)xA + (double)xB * (double)xB;
        }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) (ph.kind == PH_O ? p.ss_o : p.ss_d)[tile] = sq;
        return;
    }
    if (ph.kind == PH_GATEUP) {
        if (mine) {  // llm_cpu.c:336-342: gate / (1 + expf(-gate)) * up
            const float g = __fdiv_rn(yA, __fadd_rn(1.0f, expf(-yA)));
            p.h[tile * 8 + gid] = __fmul_rn(g, yB);
        }
        return;
    }
    // PH_LOGITS: store; argmax key = (order key, ~index) so ties go to the
    // lowest index (llm_cpu.c:896-905)
    const unsigned rA = tile * 16 + gid, rB = rA + 8;  // this rank's rows; p.vocab0 + row is the token
    unsigned long long kk = 0ull;
    if (mine) {
        const bool okA = rA < p.V, okB = rB < p.V;
        if (p.tp == 1) {
            if (okA) p.logits[rA] = yA;
            if (okB) p.logits[rB] = yB;
        } else if (p.logits_mode == 1) {  // every rank gathers the whole vocabulary
            for (unsigned j = 0; j < p.tp; ++j) {
                float *lg = reinterpret_cast<float *>(p.peers[j] + p.xl.logits) + p.vocab0;
                if (okA) lg[rA] = yA;
                if (okB) lg[rB] = yB;
            }
        }
        if (((okA && !isfinite(yA)) || (okB && !isfinite(yB))) && p.error) atomicCAS(p.error, 0u, ERR_NONFINITE);
        const unsigned gA = p.vocab0 + rA, gB = p.vocab0 + rB;
        const unsigned long long kA = okA ? ((unsigned long long)float_order_key(yA) << 32) | (0xffffffffu - gA) : 0ull;
        const unsigned long long kB = okB ? ((unsigned long long)float_order_key(yB) << 32) | (0xffffffffu - gB) : 0ull;
        kk = kA > kB ? kA : kB;
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, kk, o);
        kk = other > kk ? other : kk;
    }
    key = kk > key ? kk : key;
}

// Counter updates for `count` complete tiles starting at `first` (lane 0,
// after the fence that orders their outputs).
FYB_DEV void signal_tiles(const DecodeParams &p, const Phase &ph, unsigned first, unsigned count)
{
    if (!count) return;
    const unsigned l = ph.layer;
    if (ph.kind == PH_QKV) {
        for (unsigned t = first; t < first + count; ++t) atomicAdd(p.sync.qkv_done + l * p.Hkv + qkv_kvh(p, t), 1u);
    } else if (ph.kind == PH_O) {
        atomicAdd(p.sync.o_done + l, count);
    } else if (ph.kind == PH_GATEUP) {
        atomicAdd(p.sync.gu_done + l, count);
    } else if (ph.kind == PH_DOWN) {
        atomicAdd(p.sync.down_done + l, count);
    }
}

// ------------------------------------------------------------ phases
FYB_DEV Phase make_phase(const DecodeParams &p, unsigned kind, unsigned l)
{
    Phase ph;
    ph.kind = kind; ph.layer = l;
    if (kind == PH_LOGITS) { ph.w = p.out_head; ph.K = p.d; }
    else {
        const DecodeLayer &Ly = p.layers[l];
        if (kind == PH_QKV) { ph.w = Ly.qkv; ph.K = p.d; }
        else if (kind == PH_O) { ph.w = Ly.o; ph.K = p.H * p.hd; }
        else if (kind == PH_GATEUP) { ph.w = Ly.gateup; ph.K = p.d; }
        else { ph.w = Ly.down; ph.K = p.ffn; }
    }
    ph.nblk = ph.K / 256;
    return ph;
}

// The GEMV phase after (kind, l) in the step; false at the end.
FYB_DEV bool phase_after(const DecodeParams &p, unsigned kind, unsigned l, Phase &nx)
{
    if (kind == PH_QKV) { nx = make_phase(p, PH_O, l); return true; }
    if (kind == PH_O) { nx = make_phase(p, PH_GATEUP, l); return true; }
    if (kind == PH_GATEUP) { nx = make_phase(p, PH_DOWN, l); return true; }
    if (kind == PH_DOWN) {
        if (l + 1 < p.nl) { nx = make_phase(p, PH_QKV, l + 1); return true; }
        if (p.logits_mode) { nx = make_phase(p, PH_LOGITS, 0); return true; }
    }
    return false;
}

// cur <- the GEMV phase after cur (unchanged at the end of the step)
FYB_DEV void advance(const DecodeParams &p, Phase &cur)
{
    Phase nx;
    if (phase_after(p, cur.kind, cur.layer, nx)) cur = nx;
}

// Start the ring on the phase after `ph` (and prefetch the one after that into L2).
FYB_DEV void ring_next(const DecodeParams &p, const Phase &ph, Ring &r, unsigned lane)
{
    Phase nx, nx2;
    if (!phase_after(p, ph.kind, ph.layer, nx)) return;
    const bool has2 = phase_after(p, nx.kind, nx.layer, nx2);
    ring_begin(nx, r, lane, has2 ? &nx2 : nullptr, p.l2_prefetch);
}

// ------------------------------------------------------------ GEMV phase
// Profiling: per-warp records of a GEMV phase, WTRACE_POINTS words each:
// 0 entry (ns), 1 SM clock cycles spent waiting for weights, 2 all units
// computed (ns), 3 outputs done (ns); then in the barrier form the times
// (ns) after 4 the CTA barrier following the units, 5 the shared tiles'
// outputs, 6 the fence, 7 the second CTA barrier; in the dataflow form
// 4 its input preparation at phase entry done (ns), 5 cycles waiting for
// input blocks between units, 6 cycles spent in tile outputs.
FYB_DEV void wrecord(const DecodeParams &p, const Phase &ph, unsigned point, unsigned lane, unsigned long long value)
{
    if (!p.wtrace || lane) return;
    const unsigned long long NW = (unsigned long long)gridDim.x * QG_WARPS;
    const unsigned long long gw = (unsigned long long)blockIdx.x * QG_WARPS + (threadIdx.x >> 5);
    const unsigned slot = ph.kind == PH_LOGITS ? p.nl * 5 : ph.layer * 5 + ph.kind;
    p.wtrace[((size_t)slot * NW + gw) * WTRACE_POINTS + point] = value;
}
FYB_DEV void wstamp(const DecodeParams &p, const Phase &ph, unsigned point, unsigned lane)
{
    if (p.wtrace) wrecord(p, ph, point, lane, globaltimer());
}

// A warp's partial result for a tile it shares with other warps of its CTA.
struct PartSlot {
    unsigned tile;   // ~0u: empty
    unsigned last;   // 1: this segment holds the tile's last unit
    float v[16];     // rows 0..15 of the tile
};
constexpr unsigned PART_SLOTS_BYTES = QG_WARPS * 2 * sizeof(PartSlot) + QG_WARPS * 8;

// One GEMV phase of this CTA: its warps compute their units (ring_begin
// issued the first ones); a tile a warp covers completely produces its
// output at once, while the at most two tiles it shares with neighbouring
// warps (its first and last) leave partial sums in shared memory. After one
// CTA barrier the warp holding a shared tile's last unit adds the partials
// in warp order (so results do not depend on timing) and produces the
// output. Then one fence and one counter update per CTA publish its tiles.
template <unsigned TYPE>
FYB_DEV bool gemv_phase(const DecodeParams &p, const Phase &ph, Ring &r, const XBuf &xb, unsigned lane,
    PartSlot *parts, unsigned long long *keys)
{
    wstamp(p, ph, 0, lane);
    const unsigned warp = threadIdx.x >> 5, n = r.n;
    const unsigned nblk = ph.nblk, gid = lane >> 2, tig = lane & 3;
    while (r.issued < n && r.issued < r.S) ring_issue(r, lane);  // the ring may have started shallow
    // side inputs of the first two tiles this warp touches, loaded while the units run
    const unsigned ta = (unsigned)(r.u0 / nblk), tz = (unsigned)((r.u0 + n + nblk - 1) / nblk);
    TileIn in;
    fetch_rope(p, ph, ta, tz, lane, in);
    if (p.tp == 1 && (ph.kind == PH_DOWN || (ph.kind == PH_O && ph.layer > 0))) fetch_resid(p, ph, ta, tz, lane, in);
    PartSlot *mine = parts + warp * 2;
    if (lane < 2) mine[lane].tile = ~0u;
    float accA = 0.f, accB = 0.f;
    unsigned tile = (unsigned)(r.u0 / nblk), tile_units = 0, np = 0;
    unsigned blk = (unsigned)(r.u0 - (unsigned long long)tile * nblk);  // advanced per unit, no division
    unsigned long long key = 0ull;
    long long wait_cycles = 0;
    bool ok = true;
    for (unsigned i = 0; i < n; ++i) {
        const long long c0 = p.wtrace ? clock64() : 0;
        const unsigned char *unit = ring_wait(r);
        if (!unit) { raise_abort(p, ERR_TIMEOUT); ok = false; break; }
        if (p.wtrace) wait_cycles += clock64() - c0;
        compute_unit<TYPE, 1>(unit, blk, xb.xl, xb.xstride, xb.exps, nblk, xb.gsums, ph.K / 32, lane, accA, accB);
        __syncwarp();
        if (r.issued < n) ring_issue(r, lane);
        ++tile_units;
        const bool tile_end = blk + 1 == nblk;
        blk = tile_end ? 0 : blk + 1;
        if (!tile_end && i + 1 != n) continue;
        const float yA = lane_total<1>(accA), yB = lane_total<1>(accB);
        if (tile_units == nblk) {
            tile_output(p, ph, tile, yA, yB, lane, key, in, ta);
        } else if (np < 2) {  // only the first and the last tile can be shared
            if (tig == 0) { mine[np].v[gid] = yA; mine[np].v[gid + 8] = yB; }
            if (lane == 0) { mine[np].tile = tile; mine[np].last = tile_end ? 1u : 0u; }
            ++np;
        }
        accA = 0.f; accB = 0.f;
        tile_units = 0;
        if (tile_end) ++tile;
    }
    wrecord(p, ph, 1, lane, (unsigned long long)wait_cycles);
    wstamp(p, ph, 2, lane);
    // the ring is empty: the next phase's weights start now
    if (ok && !warp_aborted(p)) ring_next(p, ph, r, lane);
    __syncthreads();
    wstamp(p, ph, 4, lane);
    // shared tiles: the warp with the tile's last unit sums every warp's part
    for (unsigned k = 0; k < 2; ++k) {
        const unsigned t = mine[k].tile;
        if (t == ~0u || !mine[k].last) continue;
        float yA = 0.f, yB = 0.f;
        for (unsigned w = 0; w <= warp; ++w)
#pragma unroll
            for (unsigned j = 0; j < 2; ++j)
                if (parts[w * 2 + j].tile == t) { yA += parts[w * 2 + j].v[gid]; yB += parts[w * 2 + j].v[gid + 8]; }
        tile_output(p, ph, t, yA, yB, lane, key, in, ta);
    }
    if (ph.kind == PH_LOGITS && lane == 0) keys[warp] = key;
    wstamp(p, ph, 5, lane);
    // the lanes that wrote outputs (tig 0) order them before the CTA's counter update
    if ((lane & 3) == 0 || p.tp > 1) {  // (prep_tp's shares are written by any thread)
        // phases whose outputs other GPUs read (the exchanged O and down rows,
        // the gathered logits) order them at system scope before the counters
        if (p.tp > 1 && (ph.kind == PH_O || ph.kind == PH_DOWN || ph.kind == PH_LOGITS)) __threadfence_system();
        else fence_acq_rel_gpu();
    }
    wstamp(p, ph, 6, lane);
    __syncthreads();
    wstamp(p, ph, 7, lane);
    unsigned tb, te;
    cta_tiles(ph, tb, te);
    if (ph.kind == PH_QKV) {
        if (warp == 0)
            for (unsigned t = tb + lane; t < te; t += 32) atomicAdd(p.sync.qkv_done + ph.layer * p.Hkv + qkv_kvh(p, t), 1u);
    } else if (threadIdx.x == 0 && te > tb) {
        if (ph.kind == PH_LOGITS) {
            unsigned long long best = 0ull;
            for (unsigned w = 0; w < QG_WARPS; ++w) best = keys[w] > best ? keys[w] : best;
            atomicMax(p.argmax_key, best);
            __threadfence();
            // the CTA that completes the last tile publishes the token (with
            // tensor parallelism: this rank's best key, to every rank)
            if (atomicAdd(p.sync.logit_tiles, te - tb) + (te - tb) == ph.w.tiles) {
                __threadfence();
                const unsigned long long k = atomicExch(p.argmax_key, 0ull);
                atomicExch(p.sync.logit_tiles, 0u);
                if (p.tp == 1) {
                    *p.argmax_token = 0xffffffffu - (unsigned)(k & 0xffffffffu);
                } else {
                    for (unsigned j = 0; j < p.tp; ++j)
                        reinterpret_cast<unsigned long long *>(p.peers[j] + p.xl.keys)[p.tp_rank] = k;
                    __threadfence_system();
                    for (unsigned j = 0; j < p.tp; ++j) atomicAdd_system(xctr(p, j) + 2 * p.nl, 1u);
                }
            }
        } else if (p.tp > 1 && (ph.kind == PH_O || ph.kind == PH_DOWN)) {
            const unsigned idx = (ph.kind == PH_O ? 0 : p.nl) + ph.layer;
            for (unsigned j = 0; j < p.tp; ++j) atomicAdd_system(xctr(p, j) + idx, te - tb);
        } else {
            signal_tiles(p, ph, tb, te - tb);
        }
    }
    wstamp(p, ph, 3, lane);
    return ok;
}

FYB_DEV bool run_gemv(const DecodeParams &p, const Phase &ph, Ring &r, const XBuf &xb, unsigned lane,
    PartSlot *parts, unsigned long long *keys)
{
    return ph.w.type == T_Q4_K ? gemv_phase<T_Q4_K>(p, ph, r, xb, lane, parts, keys)
                               : gemv_phase<T_Q6_K>(p, ph, r, xb, lane, parts, keys);
}

// ------------------------------------------------------------ attention
struct AttnSmem {
    float *wm, *wl;  // [warps][G] running max and sum of each warp
    float *wo;       // [warps][G][HD] unnormalized outputs
    unsigned *flag;
};

FYB_HOST_DEV size_t attn_smem_floats(unsigned G, unsigned hd)
{
    return 2 * (size_t)QG_WARPS * G + (size_t)QG_WARPS * G * hd;
}

// Partitions of the context per KV head for attended length L: one per
// ATT_CHUNK positions, at most the plan's maximum.
#ifndef FYB_ATT_CHUNK
#define FYB_ATT_CHUNK 32
#endif
constexpr unsigned ATT_CHUNK = FYB_ATT_CHUNK;
constexpr unsigned ATT_MAX_PARTS = 16;  // partitions per KV head (the plan caps its maximum here)
FYB_DEV unsigned attn_parts(const DecodeParams &p, unsigned L)
{
    return max(1u, min(min(p.attn_splits, ATT_MAX_PARTS), (L + ATT_CHUNK - 1) / ATT_CHUNK));
}

// Widen DPL fp16 values (DPL 4: uint2, DPL 2: one word) to float.
template <int DPL>
FYB_DEV void load_half_row(const __half *src, float (&out)[DPL])
{
    if constexpr (DPL == 4) {
        uint2 v = __ldcg(reinterpret_cast<const uint2 *>(src));
        const float2 a = __half22float2(*reinterpret_cast<__half2 *>(&v.x));
        const float2 b = __half22float2(*reinterpret_cast<__half2 *>(&v.y));
        out[0] = a.x; out[1] = a.y; out[2] = b.x; out[3] = b.y;
    } else {
        unsigned v = __ldcg(reinterpret_cast<const unsigned *>(src));
        const float2 a = __half22float2(*reinterpret_cast<__half2 *>(&v));
        out[0] = a.x; out[1] = a.y;
    }
}

// One (KV head, partition) item with all warps of the CTA. Lane i owns head
// dimensions [DPL*i, DPL*i + DPL); warp w takes positions c0 + w, c0 + w + 16,
// ... in batches of PB, loading the q slices, and the K and V rows of a whole
// batch, before using any of them, so a batch costs one round trip to
// memory. Scores are lane partial dots reduced over the warp; an online
// softmax per query head keeps (max, sum, unnormalized output) per warp, and
// the warps merge in shared memory. The CTA's result goes to the item's slot;
// the last partition of a KV head merges the slots in partition order and
// publishes the head group (attention.cu does the same across launches).
template <int HD, int G>
FYB_DEV void attention_item(const DecodeParams &p, unsigned l, unsigned kvh, unsigned sp, const AttnSmem &sm)
{
    constexpr int DPL = HD / 32, PB = G <= 2 ? 4 : G <= 4 ? 2 : 1;
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned L = __ldcg(p.request + 1) + 1;
    const unsigned S = attn_parts(p, L);
    const unsigned chunk = (L + S - 1) / S;
    const unsigned c0 = min(L, sp * chunk), c1 = min(L, c0 + chunk);
    const __half *K = kv_layer(p, l, false) + (size_t)kvh * p.capacity * HD + DPL * lane;
    const __half *V = kv_layer(p, l, true) + (size_t)kvh * p.capacity * HD + DPL * lane;
    float qr[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float *qg = p.q + ((size_t)kvh * G + g) * HD + DPL * lane;
        if constexpr (DPL == 4) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(qg));
            qr[g][0] = v.x; qr[g][1] = v.y; qr[g][2] = v.z; qr[g][3] = v.w;
        } else {
            const float2 v = __ldcg(reinterpret_cast<const float2 *>(qg));
            qr[g][0] = v.x; qr[g][1] = v.y;
        }
    }
    float m[G], lsum[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY; lsum[g] = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[g][e] = 0.f;
    }
    for (unsigned t0 = c0 + warp; t0 < c1; t0 += QG_WARPS * PB) {
        float kf[PB][DPL], vf[PB][DPL];
        bool valid[PB];
#pragma unroll
        for (int j = 0; j < PB; ++j) {
            const unsigned t = t0 + QG_WARPS * j;
            valid[j] = t < c1;
            const size_t row = (size_t)(valid[j] ? t : t0) * HD;
            load_half_row<DPL>(K + row, kf[j]);
            load_half_row<DPL>(V + row, vf[j]);
        }
        float sc[PB][G];
#pragma unroll
        for (int j = 0; j < PB; ++j)
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float d = qr[g][0] * kf[j][0];
#pragma unroll
                for (int e = 1; e < DPL; ++e) d = fmaf(qr[g][e], kf[j][e], d);
                sc[j][g] = d;
            }
#pragma unroll
        for (int off = 16; off; off >>= 1)
#pragma unroll
            for (int j = 0; j < PB; ++j)
#pragma unroll
                for (int g = 0; g < G; ++g) sc[j][g] += __shfl_xor_sync(0xffffffffu, sc[j][g], off);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float mb = m[g];
#pragma unroll
            for (int j = 0; j < PB; ++j)
                if (valid[j]) mb = fmaxf(mb, sc[j][g] * p.attn_scale);
            const float alpha = m[g] == -INFINITY ? 0.f : expf(m[g] - mb);
            lsum[g] *= alpha;
#pragma unroll
            for (int e = 0; e < DPL; ++e) o[g][e] *= alpha;
#pragma unroll
            for (int j = 0; j < PB; ++j) {
                const float pj = valid[j] ? expf(sc[j][g] * p.attn_scale - mb) : 0.f;
                lsum[g] += pj;
#pragma unroll
                for (int e = 0; e < DPL; ++e) o[g][e] = fmaf(pj, vf[j][e], o[g][e]);
            }
            m[g] = mb;
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (lane == 0) { sm.wm[warp * G + g] = m[g]; sm.wl[warp * G + g] = lsum[g]; }
#pragma unroll
        for (int e = 0; e < DPL; ++e) sm.wo[(warp * G + g) * HD + lane * DPL + e] = o[g][e];
    }
    __syncthreads();
    constexpr unsigned SLOT = G * (HD + 2);
    float *slot = p.attn_partials + ((size_t)kvh * S + sp) * SLOT;
    for (unsigned i = threadIdx.x; i < G * HD; i += QG_THREADS) {
        const unsigned g = i / HD, dd = i % HD;
        float M = -INFINITY;
        for (int w = 0; w < QG_WARPS; ++w) M = fmaxf(M, sm.wm[w * G + g]);
        float acc = 0.f, den = 0.f;
        for (int w = 0; w < QG_WARPS; ++w) {
            const float wmv = sm.wm[w * G + g];
            const float f = wmv == -INFINITY ? 0.f : expf(wmv - M);
            acc = fmaf(sm.wo[(w * G + g) * HD + dd], f, acc);
            den = fmaf(sm.wl[w * G + g], f, den);
        }
        slot[g * (HD + 2) + dd] = acc;
        if (dd == 0) { slot[g * (HD + 2) + HD] = M; slot[g * (HD + 2) + HD + 1] = den; }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *sm.flag = atomicAdd(p.sync.attn_counters + kvh, 1u) == S - 1;
    __syncthreads();
    if (!*sm.flag) return;
    __threadfence();
    // merge the S slots: their maxima and sums staged in shared memory (one
    // round of loads), then every output element loads its S values at once
    const float *all = p.attn_partials + (size_t)kvh * S * SLOT;
    float *sM = sm.wo, *sD = sm.wo + ATT_MAX_PARTS * G;
    for (unsigned i = threadIdx.x; i < S * G; i += QG_THREADS) {
        const unsigned s2 = i / G, g = i % G;
        sM[i] = __ldcg(all + s2 * SLOT + g * (HD + 2) + HD);
        sD[i] = __ldcg(all + s2 * SLOT + g * (HD + 2) + HD + 1);
    }
    __syncthreads();
    for (unsigned i = threadIdx.x; i < G * HD; i += QG_THREADS) {
        const unsigned g = i / HD, dd = i % HD;
        float v[ATT_MAX_PARTS];
#pragma unroll
        for (unsigned s2 = 0; s2 < ATT_MAX_PARTS; ++s2)
            v[s2] = s2 < S ? __ldcg(all + s2 * SLOT + g * (HD + 2) + dd) : 0.f;
        float M = -INFINITY;
        for (unsigned s2 = 0; s2 < S; ++s2) M = fmaxf(M, sM[s2 * G + g]);
        float acc = 0.f, den = 0.f;
#pragma unroll
        for (unsigned s2 = 0; s2 < ATT_MAX_PARTS; ++s2) {
            if (s2 < S) {
                const float ms = sM[s2 * G + g];
                const float f = ms == -INFINITY ? 0.f : expf(ms - M);
                acc = fmaf(v[s2], f, acc);
                den = fmaf(sD[s2 * G + g], f, den);
            }
        }
        p.attn[((size_t)kvh * G + g) * HD + dd] = acc / den;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        p.sync.attn_counters[kvh] = 0;
        __threadfence();
        if (p.df.attn_kv) atomicAdd(p.df.attn_kv + l * p.Hkv + kvh, 1u);
        else atomicAdd(p.sync.attn_done + l, 1u);
    }
}

template <int HD, int G>
FYB_DEV bool attention_phase(const DecodeParams &p, unsigned l, unsigned step, const AttnSmem &sm)
{
    const unsigned S = attn_parts(p, __ldcg(p.request + 1) + 1);
    const unsigned items = p.Hkv * S;
    const unsigned per_step = G * HD / 16 + 2 * HD / 16;
    for (unsigned it = blockIdx.x; it < items; it += gridDim.x) {
        const unsigned kvh = it / S, sp = it % S;
        unsigned untraced = ~0u - 4;  // item counts differ between CTAs: not traced
        if (!cta_wait(p, p.sync.qkv_done + l * p.Hkv + kvh, step * per_step, sm.flag, untraced)) return false;
        attention_item<HD, G>(p, l, kvh, sp, sm);
    }
    return true;
}

// ------------------------------------------------------------ the kernel
struct SmemLayout {
    size_t rings, bars, xbuf, exps, gsums, red, parts, misc, total;
};

// Everything but the rings; the rings take what is left of the 227 KB.
FYB_HOST_DEV SmemLayout smem_layout(unsigned d, unsigned ffn, unsigned H, unsigned Hkv, unsigned hd,
    unsigned ring_bytes)
{
    SmemLayout s;
    const unsigned kmax = ffn > d ? ffn : d, kin = H * hd > kmax ? H * hd : kmax;
    const size_t xbytes = (size_t)4 * (kin + QG_XPAD);
    const size_t abytes = attn_smem_floats(H / Hkv, hd) * 4;
    s.rings = 0;
    s.bars = (size_t)QG_WARPS * ring_bytes;
    s.xbuf = s.bars + (size_t)QG_WARPS * RING_BARS * 8;
    s.exps = s.xbuf + ((xbytes > abytes ? xbytes : abytes) + 15) / 16 * 16;
    s.gsums = s.exps + ((size_t)(kin / 256) * 4 + 15) / 16 * 16;
    s.red = s.gsums + ((size_t)(kin / 32) * 4 + 15) / 16 * 16;
    s.parts = s.red + QG_WARPS * sizeof(double);
    s.misc = s.parts + PART_SLOTS_BYTES;
    s.total = s.misc + 16;
    return s;
}

// End of a step (every CTA): the last CTA out advances the step counter and,
// for greedy steps, the request. Nothing happens after an abort: the plan is
// failed and its sync words are not trusted again.
FYB_DEV void end_step(const DecodeParams &p, unsigned *flag, unsigned &ts)
{
    const bool tp = p.tp > 1;
    if (!cta_wait(p, nullptr, 0, flag, ts)) return;
    // the last CTA out advances the step (and, for greedy steps, the request)
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.sync.exit_count, 1u) == gridDim.x - 1) {
            __threadfence();
            p.sync.exit_count[0] = 0;
            if (tp && p.logits_mode) {  // the token: the best of the ranks' keys
                // keys move once per step with logits: request[4] counts those steps
                const unsigned *kc = xctr(p, p.tp_rank) + 2 * p.nl;
                const unsigned lstep = p.request[4] + 1;
                bool got = false;
                for (unsigned i = 0; i < WAIT_LIMIT && !aborted(p); ++i) {
                    if (reached(ld_acquire_sys(kc), lstep * p.tp)) { got = true; break; }
                    __nanosleep(32);
                }
                if (!got) { raise_abort(p, ERR_TIMEOUT); return; }
                const unsigned long long *kk = reinterpret_cast<const unsigned long long *>(p.peers[p.tp_rank] + p.xl.keys);
                unsigned long long best = 0ull;
                for (unsigned j = 0; j < p.tp; ++j) {
                    const unsigned long long v = __ldcg(kk + j);
                    best = v > best ? v : best;
                }
                *p.argmax_token = 0xffffffffu - (unsigned)(best & 0xffffffffu);
            }
            if (p.logits_mode == 2) {
                const unsigned t = __ldcg(p.argmax_token);
                p.tokens_log[p.request[2]] = t;
                p.request[0] = t;
                p.request[1] += 1;
                p.request[2] += 1;
            }
            p.request[3] += 1;
            if (p.logits_mode) p.request[4] += 1;
        }
    }
}

// One instantiation per (head dimension, query heads per KV head): a plan
// runs exactly one, so its registers are sized for that attention variant.
template <int HD, int G>
__global__ void __launch_bounds__(QG_THREADS, 1) decode_kernel(const DecodeParams p)
{
    extern __shared__ __align__(128) unsigned char smem[];
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const SmemLayout lay = smem_layout(p.d, p.ffn, p.H, p.Hkv, p.hd, p.ring_bytes);
    Ring ring;
    ring.base = smem + lay.rings + (size_t)warp * p.ring_bytes;
    ring.bars = reinterpret_cast<uint64_t *>(smem + lay.bars) + warp * RING_BARS;
    ring.bytes = p.ring_bytes;
    ring.pre = p.ring_pre;
    ring.par = 0;
    ring.issued = ring.consumed = ring.n = 0;
    XBuf xb;
    const unsigned kmax = p.ffn > p.d ? p.ffn : p.d;
    xb.xstride = (p.H * p.hd > kmax ? p.H * p.hd : kmax) + QG_XPAD;
    xb.xl = reinterpret_cast<signed char *>(smem + lay.xbuf);
    xb.exps = reinterpret_cast<int *>(smem + lay.exps);
    xb.gsums = reinterpret_cast<float *>(smem + lay.gsums);
    double *red = reinterpret_cast<double *>(smem + lay.red);
    PartSlot *parts = reinterpret_cast<PartSlot *>(smem + lay.parts);
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(smem + lay.parts + QG_WARPS * 2 * sizeof(PartSlot));
    unsigned *flag = reinterpret_cast<unsigned *>(smem + lay.misc);
    float *scale_smem = reinterpret_cast<float *>(flag + 1);
    AttnSmem as;  // overlays the limb buffer, which is idle during attention
    as.wm = reinterpret_cast<float *>(smem + lay.xbuf);
    as.wl = as.wm + QG_WARPS * G;
    as.wo = as.wl + QG_WARPS * G;
    as.flag = flag + 2;

    if (lane == 0) {
        for (unsigned s = 0; s < RING_BARS; ++s) mbar_init(ring.bars + s, 1);
        fence_barrier_init();
    }
    __syncwarp();

    const unsigned step = __ldcg(p.request + 3) + 1;
    const unsigned dt = p.d / 16;
    bool ok = true;
    unsigned ts = 0;
    const bool tp = p.tp > 1;
    // this rank's exchange region as floats (the partial rows all ranks wrote)
    const float *xparts = tp ? reinterpret_cast<const float *>(p.peers[p.tp_rank]) : nullptr;
    stamp(p, ts);
    Phase cur = make_phase(p, PH_QKV, 0), nx0;
    ring_begin(cur, ring, lane, phase_after(p, PH_QKV, 0, nx0) ? &nx0 : nullptr, p.l2_prefetch);
    for (unsigned l = 0; l < p.nl && ok; ++l) {
        // Q/K/V + RoPE + KV append
        if (tp) {  // x = x_mid + the ranks' down rows (or the embedding row); written to xa
            ok = cta_wait(p, l ? xctr(p, p.tp_rank) + p.nl + l - 1 : nullptr, step * p.tp * dt, flag, ts, true);
            if (!ok) break;
            prep_tp(p, l == 0, p.xm, xparts + p.xl.xd / 4, p.xa, p.layers[l].attn_norm, xb, red);
        } else {
            ok = cta_wait(p, l ? p.sync.down_done + (l - 1) : nullptr, step * dt, flag, ts);
            if (!ok) break;
            if (l == 0) prep_input(p, true, nullptr, nullptr, 0, p.layers[0].attn_norm, p.d, xb, red, scale_smem);
            else prep_input(p, false, p.xa, p.ss_d, dt, p.layers[l].attn_norm, p.d, xb, red, scale_smem);
        }
        stamp(p, ts);
        run_gemv(p, cur, ring, xb, lane, parts, keys); advance(p, cur);  // now the O projection
        // attention (its scratch overlays the limb buffer, idle now)
        ok = cta_wait(p, nullptr, 0, flag, ts) && attention_phase<HD, G>(p, l, step, as);
        stamp(p, ts);
        if (!ok) break;
        // output projection; residual add in the tile outputs
        ok = cta_wait(p, p.sync.attn_done + l, step * p.Hkv, flag, ts);
        if (!ok) break;
        prep_input(p, false, p.attn, nullptr, 0, nullptr, p.H * p.hd, xb, red, scale_smem);
        stamp(p, ts);
        run_gemv(p, cur, ring, xb, lane, parts, keys); advance(p, cur);  // gate/up
        // gate/up + SwiGLU
        if (tp) {  // x_mid = x + the ranks' O rows; written to xm
            ok = cta_wait(p, xctr(p, p.tp_rank) + l, step * p.tp * dt, flag, ts, true);
            if (!ok) break;
            prep_tp(p, false, p.xa, xparts + p.xl.xo / 4, p.xm, p.layers[l].ffn_norm, xb, red);
        } else {
            ok = cta_wait(p, p.sync.o_done + l, step * dt, flag, ts);
            if (!ok) break;
            prep_input(p, false, p.xm, p.ss_o, dt, p.layers[l].ffn_norm, p.d, xb, red, scale_smem);
        }
        stamp(p, ts);
        run_gemv(p, cur, ring, xb, lane, parts, keys); advance(p, cur);  // down
        // down; residual add in the tile outputs
        ok = cta_wait(p, p.sync.gu_done + l, step * (p.ffn / 8), flag, ts);
        if (!ok) break;
        prep_input(p, false, p.h, nullptr, 0, nullptr, p.ffn, xb, red, scale_smem);
        stamp(p, ts);
        run_gemv(p, cur, ring, xb, lane, parts, keys); advance(p, cur);  // the next layer's QKV, or the logits
    }
    if (ok && p.logits_mode) {
        if (tp) ok = cta_wait(p, xctr(p, p.tp_rank) + 2 * p.nl - 1, step * p.tp * dt, flag, ts, true);
        else ok = cta_wait(p, p.sync.down_done + (p.nl - 1), step * dt, flag, ts);
        if (ok) {
            if (tp) prep_tp(p, false, p.xm, xparts + p.xl.xd / 4, nullptr, p.out_norm, xb, red);
            else prep_input(p, false, p.xa, p.ss_d, dt, p.out_norm, p.d, xb, red, scale_smem);
            stamp(p, ts);
            run_gemv(p, cur, ring, xb, lane, parts, keys);
        }
    }
    ring_drain(ring);
    end_step(p, flag, ts);
}

using DecodeKernel = void (*)(const DecodeParams);

}  // namespace fyb
