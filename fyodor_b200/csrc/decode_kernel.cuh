// decode_kernel.cuh - one decode step of a dense LLaMA model as one persistent
// kernel (the engine's per-token graph, CUDA/resident.inc:470-552, and its
// CPU reference, backend/core/llm_cpu.c:424-578).
//
// One 512-thread CTA per SM, launched cooperatively so that every CTA is
// resident and waits between CTAs cannot deadlock. Per layer the CTAs walk
// the phases QKV(+RoPE, fp16 KV append) -> attention -> O(+residual) ->
// gate/up(+SwiGLU) -> down(+residual), then logits(+argmax).
//
// Hand-off between phases: every vector a phase produces for another CTA
// (q, the new K/V rows, the attention output, x after O, h, x after down, and
// with tensor parallelism the ranks' partial rows) is stored as 8-byte words
// {value, tag} with tag = (step, layer). A consumer polls the words it needs
// until every tag matches; an aligned 8-byte store and load are single-copy
// atomic, so a matching tag means a complete value, and no fence, counter or
// grid barrier sits between a producer's store and its consumer's load. The
// dependency chain of the step (every phase needs every tile of the phase
// before it, through attention or the full-vector products) guarantees that
// a word is not overwritten by its next layer before all its readers read it.
//
// GEMV phases. CTA c owns whole 16-row tiles [T*c/C, T*(c+1)/C) of the phase;
// they are processed in chunks of up to CHUNK tiles. Inside a chunk the
// (tile, 256-column block) units are ordered block-major and split evenly
// over the 16 warps, so a warp multiplies one or a few input blocks against
// several tiles: it polls and prepares only those blocks (256 values: the
// RMSNorm weight product, per-block exponent and four signed 8-bit limbs,
// the integer-MMA unit math of qgemv_core.cuh) into its private limb slot,
// with no CTA barrier before its first unit. Each unit's result is added to
// the warp's partial row slots in shared memory; after one CTA barrier per
// chunk the rows are summed over the warps in warp order (results do not
// depend on timing), scaled by the RMSNorm factor 1/sqrt(mean(x^2) + eps)
// (W (x * s * w) = s * W (x * w); the block sums of squares come from the
// warps that prepared the blocks), and the tile outputs are stored.
//
// Weights stream through a per-warp ring of shared memory (bulk copies with
// an mbarrier per slot, bounded waits); a warp that finishes its units of a
// phase fills its ring with its first units of the next phase at once.
//
// Every wait is bounded: on timeout the kernel records ERR_TIMEOUT and raises
// an abort word at which all CTAs leave (after their in-flight bulk copies
// land); CTA barriers inside a phase are __syncthreads_or over the CTA's
// abort state, so an abort never leaves part of a CTA at a barrier.
#pragma once
#include "qgemv_core.cuh"
#include "dequant.cuh"

namespace fyb {

constexpr unsigned WAIT_LIMIT = 1u << 22;  // polls (with a short sleep) before ERR_TIMEOUT
constexpr unsigned POLL_NS_MAX = 256;      // poll back-off: sleeps double from 16 ns up to this
constexpr unsigned RING_BARS = 8;          // mbarriers (max units in flight) per warp
constexpr unsigned CHUNK = 16;             // tiles per reduction chunk
constexpr unsigned LIMB_STRIDE = 256 + QG_XPAD;  // limb-row stride of a one-block slot (64 mod 128)
constexpr unsigned LIMB_SLOT = 4 * LIMB_STRIDE + 16 + 32 + 16;  // 4 limb rows | exponent | 8 group sums | pad
constexpr unsigned LIMB_SLOTS = 1;                 // per warp: the input block of its current units
constexpr unsigned NORM_BLOCKS_MAX = 64;   // 256-value blocks of a normalized input (d <= 16384)
constexpr unsigned DTRACE_POINTS = 32;     // per-warp detail records (profiling)

typedef unsigned long long u64;

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
    DecodeLL ll;                // tagged vectors
    float *logits;
    DecodeSync sync;
    float *attn_partials;
    unsigned attn_splits;
    unsigned long long *argmax_key;
    unsigned *argmax_token, *tokens_log;
    unsigned *error;
    int logits_mode;
    unsigned ring_bytes;        // per warp, a multiple of 16
    unsigned long long *trace;  // optional [point][CTA] globaltimer values
    unsigned trace_slots;
    unsigned long long *dtrace; // optional [CTA][warp][DTRACE_POINTS] records of layer nl / 2

    // tensor parallelism (tp > 1): H, Hkv, ffn and V above are this rank's
    unsigned tp, tp_rank, vocab0;
    unsigned char *const *peers;  // [tp] exchange regions, this rank's at tp_rank
    XchgLayout xl;
    __half *kcache, *vcache;      // all layers' caches, layer l at l * Hkv * capacity * hd
};

enum PhaseKind { PH_QKV = 0, PH_O = 1, PH_GATEUP = 2, PH_DOWN = 3, PH_LOGITS = 4 };

struct Phase {
    QWeights w;
    unsigned K, nblk, kind, layer;
};

// ------------------------------------------------------------ tagged words
// Tag of the words written by layer l (l = -1: before the first layer) of
// step `step`; 0 is never a tag, and a zeroed buffer never matches.
FYB_DEV unsigned ll_tag(unsigned step, int l) { return (step << 8) | (unsigned)((l + 1) & 0xff); }
FYB_DEV u64 ll_pack(float v, unsigned tag) { return ((u64)tag << 32) | (u64)__float_as_uint(v); }
FYB_DEV void ll_put(u64 *dst, float v, unsigned tag)
{
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" :: "l"(dst), "l"(ll_pack(v, tag)) : "memory");
}
// a word for another GPU (peer memory over NVLink)
FYB_DEV void ll_put_sys(u64 *dst, float v, unsigned tag)
{
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" :: "l"(dst), "l"(ll_pack(v, tag)) : "memory");
}
FYB_DEV u64 ll_get(const u64 *src)
{
    u64 v;
    asm volatile("ld.volatile.global.b64 %0, [%1];" : "=l"(v) : "l"(src) : "memory");
    return v;
}
FYB_DEV void ll_get2(const u64 *src, u64 &a, u64 &b)
{
    asm volatile("ld.volatile.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(src) : "memory");
}
FYB_DEV bool ll_ok(u64 w, unsigned tag) { return (unsigned)(w >> 32) == tag; }
FYB_DEV float ll_val(u64 w) { return __uint_as_float((unsigned)w); }

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

FYB_DEV unsigned ld_acquire_sys(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
FYB_DEV bool reached(unsigned value, unsigned target) { return (int)(value - target) >= 0; }

// One word, by one thread, until its tag matches (bounded). False on abort.
FYB_DEV bool ll_wait1(const DecodeParams &p, const u64 *src, unsigned tag, float &v)
{
    u64 w = ll_get(src);
    unsigned ns = 16;
    for (unsigned i = 0; !ll_ok(w, tag); ++i) {
        if (i >= WAIT_LIMIT) { raise_abort(p, ERR_TIMEOUT); return false; }
        if (aborted(p)) return false;
        __nanosleep(ns);
        ns = min(ns * 2, POLL_NS_MAX);
        w = ll_get(src);
    }
    v = ll_val(w);
    return true;
}

// Eight consecutive words per lane (src is this lane's first word, 16-byte
// aligned), warp-uniform: returns when every lane's words carry `tag`; false
// for the whole warp on abort or timeout.
FYB_DEV void ll_load8(const u64 *src, u64 (&r)[8])
{
#pragma unroll
    for (int i = 0; i < 4; ++i) ll_get2(src + 2 * i, r[2 * i], r[2 * i + 1]);
}

// `pre`: the words already requested from src (so that two blocks' loads
// are in flight together), or null.
FYB_DEV bool ll_wait8(const DecodeParams &p, const u64 *src, unsigned tag, float (&v)[8], const u64 *pre = nullptr)
{
    u64 r[8];
    if (pre) {
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = pre[i];
    } else {
        ll_load8(src, r);
    }
    unsigned ns = 16;
    for (unsigned it = 0;; ++it) {
        bool ok = true;
#pragma unroll
        for (int i = 0; i < 8; ++i) ok = ok && ll_ok(r[i], tag);
        if (__all_sync(0xffffffffu, ok)) break;
        if (it >= WAIT_LIMIT) {
            if ((threadIdx.x & 31) == 0) raise_abort(p, ERR_TIMEOUT);
            return false;
        }
        if (warp_aborted(p)) return false;
        __nanosleep(ns);
        ns = min(ns * 2, POLL_NS_MAX);
        if (!ok) {
#pragma unroll
            for (int i = 0; i < 4; ++i) ll_get2(src + 2 * i, r[2 * i], r[2 * i + 1]);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = ll_val(r[i]);
    return true;
}

FYB_DEV unsigned long long globaltimer()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Profiling: thread 0 records the time of trace point `ts` (every CTA passes
// the same trace points in the same order).
FYB_DEV void stamp(const DecodeParams &p, unsigned ts)
{
    if (p.trace && threadIdx.x == 0 && ts < p.trace_slots) p.trace[(size_t)ts * gridDim.x + blockIdx.x] = globaltimer();
}

// Profiling detail of one layer (nl / 2), lane 0 of every warp: per GEMV
// phase kind k (QKV, O, gate/up, down) at 6k: entry (ns), first input block
// prepared (ns), SM cycles waiting for weights, SM cycles preparing inputs,
// units done (ns), outputs done (ns); attention (warp 0) at 24: entry, first
// item's inputs polled, first item published, merge done (ns, 0 if none),
// phase end.
#ifndef FYB_DETAIL_TRACE
#define FYB_DETAIL_TRACE 0  // build flag: per-warp detail records (registers and branches in the unit loop)
#endif
FYB_DEV bool dtraced(const DecodeParams &p, unsigned l) { return FYB_DETAIL_TRACE && p.dtrace && l == p.nl / 2; }
FYB_DEV void drecord(const DecodeParams &p, unsigned point, unsigned long long v)
{
    if ((threadIdx.x & 31) == 0)
        p.dtrace[((size_t)blockIdx.x * QG_WARPS + (threadIdx.x >> 5)) * DTRACE_POINTS + point] = v;
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

FYB_DEV void cta_tiles(const Phase &ph, unsigned &tb, unsigned &te)
{
    const unsigned long long T = ph.w.tiles, C = gridDim.x;
    tb = (unsigned)(T * blockIdx.x / C);
    te = (unsigned)(T * (blockIdx.x + 1) / C);
}

// A warp's units of one phase: chunk by chunk, and inside chunk c (Tc tiles)
// the units u = b * Tc + t in [Uc * w / W, Uc * (w + 1) / W), Uc = nblk * Tc.
struct Walk {
    unsigned T, nblk, c, k, e, Tc, b, t;  // (b, t): block and chunk-local tile of unit k
};

FYB_DEV void walk_chunk(Walk &wk, unsigned warp)
{
    wk.Tc = min(CHUNK, wk.T - wk.c * CHUNK);
    const unsigned Uc = wk.Tc * wk.nblk;
    wk.k = Uc * warp / QG_WARPS;
    wk.e = Uc * (warp + 1) / QG_WARPS;
    wk.b = wk.k / wk.Tc;
    wk.t = wk.k - wk.b * wk.Tc;
}

FYB_DEV void walk_begin(Walk &wk, unsigned T, unsigned nblk, unsigned warp)
{
    wk.T = T; wk.nblk = nblk; wk.c = 0;
    wk.k = wk.e = wk.Tc = wk.b = wk.t = 0;
    if (T) walk_chunk(wk, warp);
}

// Next unit (t: tile index within the CTA's range, b: block); false at the end.
FYB_DEV bool walk_next(Walk &wk, unsigned warp, unsigned &t, unsigned &b)
{
    while (wk.k == wk.e) {
        if ((wk.c + 1) * CHUNK >= wk.T) return false;
        ++wk.c;
        walk_chunk(wk, warp);
    }
    b = wk.b;
    t = wk.c * CHUNK + wk.t;
    ++wk.k;
    if (++wk.t == wk.Tc) { wk.t = 0; ++wk.b; }
    return true;
}

FYB_DEV unsigned walk_count(unsigned T, unsigned nblk, unsigned warp)
{
    unsigned n = 0;
    for (unsigned c = 0; c * CHUNK < T; ++c) {
        const unsigned Uc = min(CHUNK, T - c * CHUNK) * nblk;
        n += Uc * (warp + 1) / QG_WARPS - Uc * warp / QG_WARPS;
    }
    return n;
}

// ------------------------------------------------------------ weight ring
// A warp's weight ring. Per phase it holds S = min(RING_BARS, bytes / unit)
// units; unit k of the phase goes to slot k % S. Bit s of `par` is the
// parity the next wait on mbarrier s expects. The ring is empty between
// phases, so each phase may use its own unit size.
// The issue side of a warp's ring, kept in shared memory: only lane 0 forms
// copy addresses, so these words take no registers in the unit loop.
struct RingIssue {
    const unsigned char *src;
    unsigned tb, nblk, ub;
    Walk iw;  // issue cursor
};

struct Ring {
    unsigned char *base;
    uint64_t *bars;
    RingIssue *is;    // this warp's issue state (shared memory)
    unsigned bytes, par;
    unsigned S, ub, issued, consumed, n;
    unsigned si, sc;  // slots of the next issue and the next consumption (issued % S, consumed % S)
};

FYB_DEV void ring_issue(Ring &r, unsigned lane)
{
    const unsigned slot = r.si;
    if (lane == 0) {
        RingIssue &q = *r.is;
        unsigned t = 0, b = 0;
        walk_next(q.iw, threadIdx.x >> 5, t, b);
        mbar_expect_tx(r.bars + slot, q.ub);
        bulk_copy_g2s(r.base + slot * q.ub, q.src + ((unsigned long long)(q.tb + t) * q.nblk + b) * q.ub, q.ub,
                      r.bars + slot);
    }
    ++r.issued;
    if (++r.si == r.S) r.si = 0;
}

// Start a phase on an empty ring: this warp's units and its first S copies.
FYB_DEV void ring_begin(const Phase &ph, Ring &r, unsigned lane)
{
    unsigned tb, te;
    cta_tiles(ph, tb, te);
    const unsigned warp = threadIdx.x >> 5;
    r.n = walk_count(te - tb, ph.nblk, warp);
    r.ub = unit_bytes(ph.w.type);
    r.S = min(RING_BARS, r.bytes / r.ub);
    if (lane == 0) {
        RingIssue &q = *r.is;
        q.src = ph.w.units; q.tb = tb; q.nblk = ph.nblk; q.ub = r.ub;
        walk_begin(q.iw, te - tb, ph.nblk, warp);
    }
    r.issued = r.consumed = 0;
    r.si = r.sc = 0;
    while (r.issued < r.n && r.issued < r.S) ring_issue(r, lane);
}

// Wait for the next unit; its shared-memory address, or null on timeout.
FYB_DEV const unsigned char *ring_wait(Ring &r)
{
    const unsigned slot = r.sc;
    const bool landed = mbar_wait_bounded(r.bars + slot, (r.par >> slot) & 1u);
    if (!__all_sync(0xffffffffu, landed)) return nullptr;
    r.par ^= 1u << slot;
    ++r.consumed;
    if (++r.sc == r.S) r.sc = 0;
    return r.base + slot * r.ub;
}

// Before leaving early: let the copies still in flight land (bounded).
FYB_DEV void ring_drain(Ring &r)
{
    while (r.consumed != r.issued)
        if (!ring_wait(r)) break;
}

FYB_DEV void ring_next(const DecodeParams &p, const Phase &ph, Ring &r, unsigned lane)
{
    Phase nx;
    if (phase_after(p, ph.kind, ph.layer, nx)) ring_begin(nx, r, lane);
}

// ------------------------------------------------------------ shared memory of a CTA
struct LimbSlot {           // one prepared 256-value block (a warp's private slot)
    signed char *xl;        // 4 limb rows, stride LIMB_STRIDE
    int *exps;              // the block exponent
    float *gsums;           // 8 group sums of 32 values
};

struct Cta {
    float *parts;           // [2][CHUNK][warps][16] partial rows of a chunk's tiles
    double *bss;            // [2][NORM_BLOCKS_MAX] block sums of squares of a phase's input
    unsigned long long *keys;  // [warps] logits argmax keys
    unsigned *flag;
};

// Slot `which` of the limb slots starting at `base` (a warp's first slot).
FYB_DEV LimbSlot limb_slot(unsigned char *base, unsigned which)
{
    LimbSlot s;
    unsigned char *b = base + (size_t)which * LIMB_SLOT;
    s.xl = reinterpret_cast<signed char *>(b);
    s.exps = reinterpret_cast<int *>(b + 4 * LIMB_STRIDE);
    s.gsums = reinterpret_cast<float *>(b + 4 * LIMB_STRIDE + 16);
    return s;
}

// ------------------------------------------------------------ input preparation
// Lane i holds values 8i..8i+7 of a 256-value block (x * w already): the
// block exponent, four signed limbs per value (the same split as prep_slot in
// qgemv_core.cuh, stored in its lane-major layout) and the eight 32-value
// group sums.
FYB_DEV void split_block(float (&x)[8], unsigned lane, const LimbSlot &s, unsigned *error)
{
    float gs = 0.f, mx = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) { gs = __fadd_rn(gs, x[j]); mx = fmaxf(mx, fabsf(x[j])); }
    gs = __fadd_rn(gs, __shfl_xor_sync(0xffffffffu, gs, 1));
    gs = __fadd_rn(gs, __shfl_xor_sync(0xffffffffu, gs, 2));
    if ((lane & 3) == 0) s.gsums[lane >> 2] = gs;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int E = 0;
    const bool bad = !(mx <= 3.0e38f);  // inf or NaN in the block
    if (!bad && mx > 0.f) {
        frexpf(mx, &E);
        if (E < -120) E = -120;  // below 2^-121 the limbs round to zero anyway
    }
    if (lane == 0) *s.exps = E;
    if (lane == 0 && bad && error) *(volatile unsigned *)error = ERR_NONFINITE;
    const float sc = pow2f(6 - E);
    unsigned words[4][2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
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
    // natural words 2i and 2i+1 of the limb row: chunk (i / 8), word w = 2 (i % 8) (+1)
    const unsigned chunk = (lane >> 3) * 64u, w0 = (lane & 7u) * 2u, w1 = w0 + 1u;
    const unsigned p0 = chunk + ((w0 & 3u) * 4u + (w0 >> 2)) * 4u, p1 = chunk + ((w1 & 3u) * 4u + (w1 >> 2)) * 4u;
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        *reinterpret_cast<unsigned *>(s.xl + l * LIMB_STRIDE + p0) = words[l][0];
        *reinterpret_cast<unsigned *>(s.xl + l * LIMB_STRIDE + p1) = words[l][1];
    }
}

// Block b of a phase's input into the warp's limb slot; the block's sum of
// squares (before the norm weight) into bss[b] for normalized inputs. Sources:
// QKV: the embedding row (layer 0) or x after the previous layer; O: the
// attention output; gate/up: x after O; down: h; logits: x after the last
// layer. With tensor parallelism the d-row inputs are a base vector plus the
// ranks' partial rows, added in rank order (every rank computes the same x),
// and the last CTA stores the summed x for the next exchange's base.
// The lane's first word of block b for phases with one tagged source (O,
// down, and without tensor parallelism QKV after layer 0, gate/up and the
// logits); null for the others.
FYB_DEV const u64 *single_source(const DecodeParams &p, const Phase &ph, unsigned b, unsigned lane)
{
    const unsigned i0 = b * 256 + lane * 8;
    if (ph.kind == PH_O) return p.ll.attn + i0;
    if (ph.kind == PH_DOWN) return p.ll.h + i0;
    if (p.tp > 1 || (ph.kind == PH_QKV && ph.layer == 0)) return nullptr;
    return (ph.kind == PH_GATEUP ? p.ll.xm : p.ll.xa) + i0;
}

FYB_DEV bool prep_block(const DecodeParams &p, const Phase &ph, unsigned b, unsigned step, const LimbSlot &s,
    double *bss, unsigned lane, const u64 *pre = nullptr)
{
    const unsigned i0 = b * 256 + lane * 8;
    const int l = (int)ph.layer;
    float x[8];
    const bool norm = ph.kind == PH_QKV || ph.kind == PH_GATEUP || ph.kind == PH_LOGITS;
    const int prev = ph.kind == PH_LOGITS ? (int)p.nl - 1 : l - 1;  // the layer whose output QKV / logits read
    if (ph.kind == PH_QKV && l == 0) {
        const unsigned char *erow = p.embd + (unsigned long long)__ldcg(p.request) * p.embd_row_bytes;
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = dequant_any(erow, (unsigned long long)i0 + j, p.embd_type);
        if (p.tp > 1 && blockIdx.x == gridDim.x - 1) {  // the base of layer 0's O exchange
#pragma unroll
            for (int j = 0; j < 8; ++j) ll_put(p.ll.xa + i0 + j, x[j], ll_tag(step, -1));
        }
    } else if (ph.kind == PH_O || ph.kind == PH_DOWN) {
        if (!ll_wait8(p, single_source(p, ph, b, lane), ll_tag(step, l), x, pre)) return false;
    } else if (p.tp == 1) {
        const unsigned tag = ll_tag(step, ph.kind == PH_GATEUP ? l : prev);
        if (!ll_wait8(p, single_source(p, ph, b, lane), tag, x, pre)) return false;
    } else {
        // x = base + the ranks' partial rows: QKV / logits: x after O plus the
        // down rows; gate/up: x after the previous exchange plus the O rows
        // tags: the base is tagged with the layer whose output it completes
        // (gate/up: the previous layer), the partial rows with their layer
        const bool gu = ph.kind == PH_GATEUP;
        const unsigned tag = ll_tag(step, gu ? l : prev);
        const u64 *base = gu ? p.ll.xa : p.ll.xm;
        const u64 *parts = reinterpret_cast<const u64 *>(p.peers[p.tp_rank] + (gu ? p.xl.xo : p.xl.xd));
        if (!ll_wait8(p, base + i0, ll_tag(step, gu ? l - 1 : prev), x)) return false;
        for (unsigned r = 0; r < p.tp; ++r) {
            float y[8];
            if (!ll_wait8(p, parts + (size_t)r * p.d + i0, tag, y)) return false;
#pragma unroll
            for (int j = 0; j < 8; ++j) x[j] = __fadd_rn(x[j], y[j]);
        }
        if (ph.kind != PH_LOGITS && blockIdx.x == gridDim.x - 1) {  // the next exchange's base
            u64 *dst = gu ? p.ll.xm : p.ll.xa;
            const unsigned wt = ll_tag(step, gu ? l : prev);
#pragma unroll
            for (int j = 0; j < 8; ++j) ll_put(dst + i0 + j, x[j], wt);
        }
    }
    if (norm) {
        double ss = 0.0;
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += (double)x[j] * (double)x[j];
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) bss[b] = ss;
        const float *nw = ph.kind == PH_QKV ? p.layers[l].attn_norm
                        : ph.kind == PH_GATEUP ? p.layers[l].ffn_norm : p.out_norm;
        const float4 w0 = __ldg(reinterpret_cast<const float4 *>(nw + i0));
        const float4 w1 = __ldg(reinterpret_cast<const float4 *>(nw + i0 + 4));
        const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = __fmul_rn(x[j], w[j]);
    }
    split_block(x, lane, s, p.error);
    __syncwarp();
    return true;
}

// ------------------------------------------------------------ tile outputs
FYB_DEV __half *kv_layer(const DecodeParams &p, unsigned l, bool v)
{
    return (v ? p.vcache : p.kcache) + (size_t)l * p.Hkv * p.capacity * p.hd;
}

// Output of rows j and j + 8 of `tile` (the MMA rows gid and gid + 8 of the
// repacked layouts): QKV: the RoPE pair (2i, 2i+1) of a head, q or K/V;
// O / down: x rows (residual added) or, with tensor parallelism, this
// rank's partial rows for every rank; gate/up: gate and up row j of the
// tile's 8 FFN rows; logits: two vocabulary rows and their argmax key.
FYB_DEV bool pair_output(const DecodeParams &p, const Phase &ph, unsigned step, unsigned tile, unsigned j, float yA,
    float yB, unsigned long long &key)
{
    const unsigned l = ph.layer;
    const unsigned tag = ll_tag(step, (int)l);
    if (ph.kind == PH_QKV) {
        // rows 2*j and 2*j+1 of the tile form one RoPE pair (llm_cpu.c:298-327)
        const unsigned tq = p.H * p.hd / 16, tk = p.Hkv * p.hd / 16, hd = p.hd;
        const unsigned seg = tile < tq ? 0 : tile < tq + tk ? 1 : 2;
        const unsigned lt = tile - (seg == 0 ? 0 : seg == 1 ? tq : tq + tk);
        const unsigned rowA = lt * 16 + 2 * j;
        const unsigned pos = __ldcg(p.request + 1), pair = (rowA % hd) >> 1;
        float a = yA, b = yB;
        if (seg <= 1) {
            const float c = __ldg(p.rope_cos + (size_t)pos * (hd >> 1) + pair);
            const float s = __ldg(p.rope_sin + (size_t)pos * (hd >> 1) + pair);
            a = __fsub_rn(__fmul_rn(yA, c), __fmul_rn(yB, s));
            b = __fadd_rn(__fmul_rn(yA, s), __fmul_rn(yB, c));
        }
        if (seg == 0) {
            ll_put(p.ll.q + rowA, a, tag);
            ll_put(p.ll.q + rowA + 1, b, tag);
        } else {
            const unsigned kvh = rowA / hd, dd = rowA % hd;
            const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
            *reinterpret_cast<__half2 *>(kv_layer(p, l, seg == 2) + ((size_t)kvh * p.capacity + pos) * hd + dd) =
                __halves2half2(ha, hb);
            u64 *nw = p.ll.kvnew + (seg == 2 ? p.Hkv * hd : 0u) + rowA;  // the attention reads row pos here
            ll_put(nw, __half2float(ha), tag);
            ll_put(nw + 1, __half2float(hb), tag);
        }
        return true;
    }
    if (ph.kind == PH_O || ph.kind == PH_DOWN) {
        const unsigned rA = tile * 16 + j;
        if (p.tp > 1) {  // this rank's partial rows, to every rank's exchange region
            const size_t off = (ph.kind == PH_O ? p.xl.xo : p.xl.xd) + ((size_t)p.tp_rank * p.d + rA) * 8;
            for (unsigned r = 0; r < p.tp; ++r) {
                u64 *dst = reinterpret_cast<u64 *>(p.peers[r] + off);
                if (r == p.tp_rank) { ll_put(dst, yA, tag); ll_put(dst + 8, yB, tag); }
                else { ll_put_sys(dst, yA, tag); ll_put_sys(dst + 8, yB, tag); }
            }
            return true;
        }
        if (ph.kind == PH_O && l == 0) {  // layer 0: the residual is the embedding row
            const unsigned char *erow = p.embd + (unsigned long long)__ldcg(p.request) * p.embd_row_bytes;
            yA = __fadd_rn(dequant_any(erow, rA, p.embd_type), yA);
            yB = __fadd_rn(dequant_any(erow, rA + 8, p.embd_type), yB);
        }  // other layers: the caller added the residual rows
        u64 *dst = ph.kind == PH_O ? p.ll.xm : p.ll.xa;
        ll_put(dst + rA, yA, tag);
        ll_put(dst + rA + 8, yB, tag);
        return true;
    }
    if (ph.kind == PH_GATEUP) {  // llm_cpu.c:336-342: gate / (1 + expf(-gate)) * up
        const float g = __fdiv_rn(yA, __fadd_rn(1.0f, expf(-yA)));
        ll_put(p.ll.h + tile * 8 + j, __fmul_rn(g, yB), tag);
        return true;
    }
    // PH_LOGITS: store; argmax key = (order key, ~index) so ties go to the
    // lowest index (llm_cpu.c:896-905)
    const unsigned rA = tile * 16 + j, rB = rA + 8;  // this rank's rows; p.vocab0 + row is the token
    const bool okA = rA < p.V, okB = rB < p.V;
    if (p.tp == 1) {
        if (okA) p.logits[rA] = yA;
        if (okB) p.logits[rB] = yB;
    } else if (p.logits_mode == 1) {  // every rank gathers the whole vocabulary
        for (unsigned r = 0; r < p.tp; ++r) {
            float *lg = reinterpret_cast<float *>(p.peers[r] + p.xl.logits) + p.vocab0;
            if (okA) lg[rA] = yA;
            if (okB) lg[rB] = yB;
        }
    }
    if (((okA && !isfinite(yA)) || (okB && !isfinite(yB))) && p.error) atomicCAS(p.error, 0u, ERR_NONFINITE);
    const unsigned gA = p.vocab0 + rA, gB = p.vocab0 + rB;
    const unsigned long long kA = okA ? ((unsigned long long)float_order_key(yA) << 32) | (0xffffffffu - gA) : 0ull;
    const unsigned long long kB = okB ? ((unsigned long long)float_order_key(yB) << 32) | (0xffffffffu - gB) : 0ull;
    const unsigned long long kk = kA > kB ? kA : kB;
    key = kk > key ? kk : key;
    return true;
}

// ------------------------------------------------------------ GEMV phase
// One GEMV phase of this CTA (see the file comment). `seq` counts the chunks
// this CTA has reduced (it picks the partial-row buffer) and `pseq` the
// phases (it picks the block sums of squares). False for every thread on
// abort.
template <unsigned TYPE>
FYB_DEV bool gemv_phase(const DecodeParams &p, const Phase &ph, unsigned step, Ring &r, unsigned char *slots,
    const Cta &cta, unsigned lane, unsigned &seq, unsigned pseq, unsigned long long &key)
{
    const unsigned warp = threadIdx.x >> 5, gid = lane >> 2, tig = lane & 3;
    unsigned tb, te;
    cta_tiles(ph, tb, te);
    const unsigned T = te - tb, nblk = ph.nblk;
    const bool norm = ph.kind == PH_QKV || ph.kind == PH_GATEUP || ph.kind == PH_LOGITS;
    double *bss = cta.bss + (pseq & 1) * NORM_BLOCKS_MAX;
    bool ok = true;
    unsigned plo = ~0u, cur_b = ~0u;  // plo: the block in the limb slot; cur_b: the block of bc
    BlockConst bc;
    const bool dt = dtraced(p, ph.layer) && ph.kind != PH_LOGITS;
    const unsigned dbase = ph.kind * 6;
    long long wait_cycles = 0, prep_cycles = 0;
    if (dt) drecord(p, dbase, globaltimer());
    if (r.n == 0 && !warp_aborted(p)) ring_next(p, ph, r, lane);  // no units here: only the next ring
    if (T == 0) return __syncthreads_or(aborted(p)) == 0;  // keeps the CTA's phases in step (bss, parts)
    for (unsigned c = 0; c * CHUNK < T; ++c) {
        Walk wk;
        wk.T = T; wk.nblk = nblk; wk.c = c;
        walk_chunk(wk, warp);
        const unsigned Tc = wk.Tc;
        float *parts = cta.parts + (size_t)(seq & 1) * CHUNK * QG_WARPS * 16;
        // the abort word is read here and used at the chunk barrier, so its
        // load is not in front of the barrier (a failure of this thread since
        // the last barrier raised it, and this thread sees its own store)
        const bool abort_seen = lane == 0 && aborted(p);
        // a warp whose units are exactly one block column of the chunk writes
        // each of its partial rows once; any other warp starts them at zero
        // and adds to them
        const bool column = wk.e - wk.k == Tc && wk.t == 0;
        if (!column) {
            for (unsigned i = lane; i < Tc * 16; i += 32) parts[((i >> 4) * QG_WARPS + warp) * 16 + (i & 15)] = 0.f;
            __syncwarp();
        }
        {
        unsigned b = wk.b, t = wk.t;
        for (unsigned k = wk.k; k < wk.e && ok;) {
            if (b != plo) {  // prepare block b into the limb slot
                const long long c0 = dt ? clock64() : 0;
                ok = prep_block(p, ph, b, step, limb_slot(slots, 0), bss, lane);
                if (dt) {
                    prep_cycles += clock64() - c0;
                    if (plo == ~0u) drecord(p, dbase + 1, globaltimer());
                }
                plo = b;
                if (!ok) break;
            }
            const LimbSlot slot = limb_slot(slots, 0);
            if (b != cur_b) { bc = block_const(slot.exps, slot.gsums, lane); cur_b = b; }
            // two units of the same block run as two independent MMA chains
            const bool two = k + 1 < wk.e && t + 1 < Tc;
            const long long w0 = dt ? clock64() : 0;
            const unsigned char *u0 = ring_wait(r);
            const unsigned char *u1 = two && u0 ? ring_wait(r) : u0;
            if (dt) wait_cycles += clock64() - w0;
            if (!u0 || !u1) { if (lane == 0) raise_abort(p, ERR_TIMEOUT); ok = false; break; }
            float acc[2][2];
            if (two) {
                const unsigned char *const uu[2] = {u0, u1};
                compute_units<TYPE, 2>(uu, slot.xl, LIMB_STRIDE, bc, lane, acc);
            } else {
                const unsigned char *const uu[1] = {u0};
                float a1[1][2];
                compute_units<TYPE, 1>(uu, slot.xl, LIMB_STRIDE, bc, lane, a1);
                acc[0][0] = a1[0][0]; acc[0][1] = a1[0][1];
            }
            __syncwarp();
            if (r.issued < r.n) ring_issue(r, lane);
            if (two && r.issued < r.n) ring_issue(r, lane);
#pragma unroll
            for (int n = 0; n < 2; ++n) {
                if (n == 1 && !two) break;
                const float yA = lane_total<1>(acc[n][0]), yB = lane_total<1>(acc[n][1]);
                if (tig == 0) {
                    float *row = parts + ((t + n) * QG_WARPS + warp) * 16;
                    if (column) { row[gid] = yA; row[gid + 8] = yB; }
                    else { row[gid] += yA; row[gid + 8] += yB; }
                }
            }
            const unsigned adv = two ? 2u : 1u;
            k += adv;
            t += adv;
            if (t == Tc) { t = 0; ++b; }
            // the ring is empty after this warp's last unit: the next phase's weights start now
            if (r.consumed == r.n && !warp_aborted(p)) ring_next(p, ph, r, lane);
        }
        }
        if (dt && (c + 1) * CHUNK >= T) {
            drecord(p, dbase + 2, (unsigned long long)wait_cycles);
            drecord(p, dbase + 3, (unsigned long long)prep_cycles);
            drecord(p, dbase + 4, globaltimer());
        }
        // reducer threads (t * 8 + j) read their residual rows before the barrier
        const unsigned i = threadIdx.x, t = i >> 3, j = i & 7;
        const bool reducer = i < Tc * 8;
        const bool resid = p.tp == 1 && (ph.kind == PH_DOWN || (ph.kind == PH_O && ph.layer > 0));
        u64 ra = 0, rb = 0;
        const u64 *rsrc = ph.kind == PH_O ? p.ll.xa : p.ll.xm;
        const unsigned rA = (tb + c * CHUNK + t) * 16 + j;
        if (reducer && resid) { ra = ll_get(rsrc + rA); rb = ll_get(rsrc + rA + 8); }
        // every failure raised the abort word before this barrier
        if (__syncthreads_or(!ok || abort_seen)) return false;
        if (reducer) {
            float yA = 0.f, yB = 0.f;
#pragma unroll 4
            for (unsigned w = 0; w < QG_WARPS; ++w) {
                yA += parts[(t * QG_WARPS + w) * 16 + j];
                yB += parts[(t * QG_WARPS + w) * 16 + j + 8];
            }
            if (norm) {
                double ss = 0.0;
                for (unsigned bb = 0; bb < nblk; ++bb) ss += bss[bb];
                const float scale = (float)(1.0 / sqrt(ss / (double)ph.K + (double)p.eps));
                yA = __fmul_rn(yA, scale);
                yB = __fmul_rn(yB, scale);
            }
            if (resid) {
                const unsigned rtag = ll_tag(step, ph.kind == PH_O ? (int)ph.layer - 1 : (int)ph.layer);
                float xa_, xb_;
                if (ll_ok(ra, rtag)) xa_ = ll_val(ra); else ll_wait1(p, rsrc + rA, rtag, xa_);
                if (ll_ok(rb, rtag)) xb_ = ll_val(rb); else ll_wait1(p, rsrc + rA + 8, rtag, xb_);
                yA = __fadd_rn(xa_, yA);
                yB = __fadd_rn(xb_, yB);
            }
            // a failed wait raised the abort word; the next CTA barrier sees it
            pair_output(p, ph, step, tb + c * CHUNK + t, j, yA, yB, key);
        }
        ++seq;
    }
    if (dt) drecord(p, dbase + 5, globaltimer());
    return true;
}

FYB_DEV bool run_gemv(const DecodeParams &p, const Phase &ph, unsigned step, Ring &r, unsigned char *slots,
    const Cta &cta, unsigned lane, unsigned &seq, unsigned pseq, unsigned long long &key)
{
    return ph.w.type == T_Q4_K ? gemv_phase<T_Q4_K>(p, ph, step, r, slots, cta, lane, seq, pseq, key)
                               : gemv_phase<T_Q6_K>(p, ph, step, r, slots, cta, lane, seq, pseq, key);
}

// ------------------------------------------------------------ attention
struct AttnSmem {
    float *wm, *wl;  // [warps][G] running max and sum of each warp
    float *wo;       // [warps][G][HD] unnormalized outputs
    float *qkv;      // [G * HD + 2 * HD] the group's query rows, the new K and V rows
    unsigned *flag;
};

FYB_HOST_DEV size_t attn_smem_floats(unsigned G, unsigned hd)
{
    return 2 * (size_t)QG_WARPS * G + (size_t)QG_WARPS * G * hd + (size_t)(G + 2) * hd;
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
// ... in batches of PB, loading the K and V rows of a whole batch before
// using any of them, so a batch costs one round trip to memory. The query
// rows and the new position's K/V rows (tagged words of this layer) are
// polled first; older positions come from the fp16 cache. Scores are lane
// partial dots reduced over the warp; an online softmax per query head keeps
// (max, sum, unnormalized output) per warp, and the warps merge in shared
// memory. The CTA's result goes to the item's slot; the last partition of a
// KV head merges the slots in partition order and stores the head group's
// attention output as tagged words.
template <int HD, int G>
FYB_DEV bool attention_item(const DecodeParams &p, unsigned step, unsigned l, unsigned kvh, unsigned sp,
    const AttnSmem &sm)
{
    constexpr int DPL = HD / 32, PB = G <= 2 ? 4 : G <= 4 ? 2 : 1;
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned pos = __ldcg(p.request + 1), L = pos + 1;
    const unsigned S = attn_parts(p, L);
    const unsigned chunk = (L + S - 1) / S;
    const unsigned c0 = min(L, sp * chunk), c1 = min(L, c0 + chunk);
    const unsigned tag = ll_tag(step, (int)l);
    const __half *K = kv_layer(p, l, false) + (size_t)kvh * p.capacity * HD + DPL * lane;
    const __half *V = kv_layer(p, l, true) + (size_t)kvh * p.capacity * HD + DPL * lane;
    // the query rows of the group and, in the partition holding it, the new
    // position's K and V rows: one tagged word per thread, polled by the whole
    // CTA into shared memory, then every warp reads them from there
    const bool has_new = pos >= c0 && pos < c1;
    bool ok = true;
    for (unsigned i = threadIdx.x; i < G * HD + (has_new ? 2 * HD : 0); i += QG_THREADS) {
        const u64 *src = i < G * HD ? p.ll.q + (size_t)kvh * G * HD + i
                       : p.ll.kvnew + (size_t)(i < G * HD + HD ? kvh : p.Hkv + kvh) * HD + (i - G * HD) % HD;
        float v = 0.f;
        ok = ok && ll_wait1(p, src, tag, v);
        sm.qkv[i] = v;
    }
    if (__syncthreads_or(!ok)) return false;
    const bool dt = dtraced(p, l) && warp == 0 && sp + kvh * S == blockIdx.x;  // the CTA's first item
    if (dt) drecord(p, 25, globaltimer());
    float qr[G][DPL], knew[DPL], vnew[DPL];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < DPL; ++e) qr[g][e] = sm.qkv[g * HD + DPL * lane + e];
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
        knew[e] = has_new ? sm.qkv[G * HD + DPL * lane + e] : 0.f;
        vnew[e] = has_new ? sm.qkv[G * HD + HD + DPL * lane + e] : 0.f;
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
            if (valid[j] && t == pos) {
#pragma unroll
                for (int e = 0; e < DPL; ++e) { kf[j][e] = knew[e]; vf[j][e] = vnew[e]; }
            } else {
                const size_t row = (size_t)(valid[j] ? t : t0) * HD;
                load_half_row<DPL>(K + row, kf[j]);
                load_half_row<DPL>(V + row, vf[j]);
            }
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
    // the CTA's partial result: per query head its maximum, sum and
    // unnormalized output, merged over the warps in warp order; thread i
    // owns output elements i + r * QG_THREADS
    constexpr unsigned SLOT = G * (HD + 2);
    constexpr unsigned EPT = (G * HD + QG_THREADS - 1) / QG_THREADS;  // elements per thread (1 or 2)
    u64 *const parts_all = reinterpret_cast<u64 *>(p.attn_partials) + (size_t)kvh * ATT_MAX_PARTS * SLOT;
    float acc0[EPT], M0[EPT], den0[EPT];
#pragma unroll
    for (unsigned r = 0; r < EPT; ++r) {
        const unsigned e = threadIdx.x + r * QG_THREADS, g = e / HD, dd = e % HD;
        acc0[r] = 0.f; M0[r] = -INFINITY; den0[r] = 0.f;
        if (e < G * HD) {
            for (int w = 0; w < QG_WARPS; ++w) M0[r] = fmaxf(M0[r], sm.wm[w * G + g]);
            for (int w = 0; w < QG_WARPS; ++w) {
                const float wmv = sm.wm[w * G + g];
                const float f = wmv == -INFINITY ? 0.f : expf(wmv - M0[r]);
                acc0[r] = fmaf(sm.wo[(w * G + g) * HD + dd], f, acc0[r]);
                den0[r] = fmaf(sm.wl[w * G + g], f, den0[r]);
            }
        }
    }
    if (sp != 0) {
        // partitions after the first publish their result as tagged words;
        // the first partition's CTA merges them
        u64 *slot = parts_all + (size_t)sp * SLOT;
#pragma unroll
        for (unsigned r = 0; r < EPT; ++r) {
            const unsigned e = threadIdx.x + r * QG_THREADS, g = e / HD, dd = e % HD;
            if (e < G * HD) {
                ll_put(slot + g * (HD + 2) + dd, acc0[r], tag);
                if (dd == 0) {
                    ll_put(slot + g * (HD + 2) + HD, M0[r], tag);
                    ll_put(slot + g * (HD + 2) + HD + 1, den0[r], tag);
                }
            }
        }
        if (dt) drecord(p, 26, globaltimer());
        __syncthreads();  // the shared scratch is free again
        return true;
    }
    if (dt) drecord(p, 26, globaltimer());
    // merge: the other partitions' slots polled into shared memory, eight
    // words in flight per thread (slot s2 at index (s2 - 1) * SLOT), this
    // partition's own result stays in registers; then the sums run in
    // partition order
    __syncthreads();  // every thread has read the warps' outputs
    float *const sp_all = sm.wo;
    bool mok = true;
    const unsigned n = (S - 1) * SLOT;
    for (unsigned q0 = threadIdx.x; q0 < n; q0 += 8 * QG_THREADS) {
        u64 w[8];
#pragma unroll
        for (unsigned j = 0; j < 8; ++j) {
            const unsigned q = q0 + j * QG_THREADS;
            w[j] = q < n ? ll_get(parts_all + SLOT + q) : 0ull;
        }
#pragma unroll
        for (unsigned j = 0; j < 8; ++j) {
            const unsigned q = q0 + j * QG_THREADS;
            if (q >= n) break;
            float v;
            if (ll_ok(w[j], tag)) v = ll_val(w[j]);
            else if (!ll_wait1(p, parts_all + SLOT + q, tag, v)) mok = false;
            sp_all[q] = v;
        }
    }
    if (__syncthreads_or(!mok)) return false;
#pragma unroll
    for (unsigned r = 0; r < EPT; ++r) {
        const unsigned e = threadIdx.x + r * QG_THREADS, g = e / HD, dd = e % HD;
        if (e >= G * HD) continue;
        const float *gs = sp_all + g * (HD + 2);  // gs[(s2 - 1) * SLOT + k]: partition s2 >= 1
        float M = M0[r];
        for (unsigned s2 = 1; s2 < S; ++s2) M = fmaxf(M, gs[(s2 - 1) * SLOT + HD]);
        float acc = 0.f, den = 0.f;
        for (unsigned s2 = 0; s2 < S; ++s2) {
            const float ms = s2 ? gs[(s2 - 1) * SLOT + HD] : M0[r];
            const float f = ms == -INFINITY ? 0.f : expf(ms - M);
            acc = fmaf(s2 ? gs[(s2 - 1) * SLOT + dd] : acc0[r], f, acc);
            den = fmaf(s2 ? gs[(s2 - 1) * SLOT + HD + 1] : den0[r], f, den);
        }
        ll_put(p.ll.attn + ((size_t)kvh * G + g) * HD + dd, acc / den, tag);
    }
    if (dt) drecord(p, 27, globaltimer());
    __syncthreads();  // the shared scratch is free again
    return true;
}

template <int HD, int G>
FYB_DEV bool attention_phase(const DecodeParams &p, unsigned step, unsigned l, const AttnSmem &sm)
{
    const unsigned S = attn_parts(p, __ldcg(p.request + 1) + 1);
    const unsigned items = p.Hkv * S;
    for (unsigned it = blockIdx.x; it < items; it += gridDim.x)
        if (!attention_item<HD, G>(p, step, l, it / S, it % S, sm)) return false;
    return true;
}

// ------------------------------------------------------------ the kernel
struct SmemLayout {
    size_t rings, bars, uni, parts, bss, keys, issue, misc, total;
};

// Everything but the rings; the rings take what is left of the 227 KB. The
// limb slots and the attention scratch share one region (attention runs
// between GEMV phases, behind CTA barriers).
FYB_HOST_DEV SmemLayout smem_layout(unsigned H, unsigned Hkv, unsigned hd, unsigned ring_bytes)
{
    SmemLayout s;
    const size_t limbs = (size_t)QG_WARPS * LIMB_SLOTS * LIMB_SLOT;
    const size_t abytes = attn_smem_floats(H / Hkv, hd) * 4;
    s.rings = 0;
    s.bars = (size_t)QG_WARPS * ring_bytes;
    s.uni = s.bars + (size_t)QG_WARPS * RING_BARS * 8;
    s.parts = s.uni + ((limbs > abytes ? limbs : abytes) + 15) / 16 * 16;
    s.bss = s.parts + (size_t)2 * CHUNK * QG_WARPS * 16 * 4;
    s.keys = s.bss + (size_t)2 * NORM_BLOCKS_MAX * 8;
    s.issue = s.keys + (size_t)QG_WARPS * 8;
    s.misc = s.issue + ((size_t)QG_WARPS * sizeof(RingIssue) + 15) / 16 * 16;
    s.total = s.misc + 16;
    return s;
}

// End of a step (every CTA): the logits argmax key of the CTA, then the last
// CTA out advances the step counter and, for greedy steps, the request.
// Nothing happens after an abort: the plan is failed and its sync words are
// not trusted again.
FYB_DEV void end_step(const DecodeParams &p, const Cta &cta, unsigned long long key, bool logits_done)
{
    const bool tp = p.tp > 1;
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (logits_done) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
            key = other > key ? other : key;
        }
        if (lane == 0) cta.keys[warp] = key;
    }
    if (__syncthreads_or(threadIdx.x == 0 && aborted(p))) return;
    if (threadIdx.x != 0) return;
    if (logits_done) {
        unsigned tb, te;
        const Phase lg = make_phase(p, PH_LOGITS, 0);
        cta_tiles(lg, tb, te);
        if (te > tb) {
            unsigned long long best = 0ull;
            for (unsigned w = 0; w < QG_WARPS; ++w) best = cta.keys[w] > best ? cta.keys[w] : best;
            atomicMax(p.argmax_key, best);
            __threadfence();
            // the CTA that completes the last tile publishes the token (with
            // tensor parallelism: this rank's best key, to every rank)
            if (atomicAdd(p.sync.logit_tiles, te - tb) + (te - tb) == lg.w.tiles) {
                __threadfence();
                const unsigned long long k = atomicExch(p.argmax_key, 0ull);
                atomicExch(p.sync.logit_tiles, 0u);
                if (!tp) {
                    *p.argmax_token = 0xffffffffu - (unsigned)(k & 0xffffffffu);
                } else {
                    for (unsigned j = 0; j < p.tp; ++j)
                        reinterpret_cast<unsigned long long *>(p.peers[j] + p.xl.keys)[p.tp_rank] = k;
                    __threadfence_system();
                    for (unsigned j = 0; j < p.tp; ++j) atomicAdd_system(xctr(p, j) + 2 * p.nl, 1u);
                }
            }
        }
    }
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

// One instantiation per (head dimension, query heads per KV head): a plan
// runs exactly one, so its registers are sized for that attention variant.
template <int HD, int G>
__global__ void __launch_bounds__(QG_THREADS, 1) decode_kernel(const DecodeParams p)
{
    extern __shared__ __align__(128) unsigned char smem[];
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const SmemLayout lay = smem_layout(p.H, p.Hkv, p.hd, p.ring_bytes);
    Ring ring;
    ring.base = smem + lay.rings + (size_t)warp * p.ring_bytes;
    ring.bars = reinterpret_cast<uint64_t *>(smem + lay.bars) + warp * RING_BARS;
    ring.bytes = p.ring_bytes;
    ring.is = reinterpret_cast<RingIssue *>(smem + lay.issue) + warp;
    ring.par = 0;
    ring.issued = ring.consumed = ring.n = 0;
    unsigned char *const slots = smem + lay.uni + (size_t)warp * LIMB_SLOTS * LIMB_SLOT;  // this warp's limb slots
    Cta cta;
    cta.parts = reinterpret_cast<float *>(smem + lay.parts);
    cta.bss = reinterpret_cast<double *>(smem + lay.bss);
    cta.keys = reinterpret_cast<unsigned long long *>(smem + lay.keys);
    cta.flag = reinterpret_cast<unsigned *>(smem + lay.misc);
    AttnSmem as;  // overlays the limb slots, idle during attention
    as.wm = reinterpret_cast<float *>(smem + lay.uni);
    as.wl = as.wm + QG_WARPS * G;
    as.wo = as.wl + QG_WARPS * G;
    as.qkv = as.wo + QG_WARPS * G * HD;
    as.flag = cta.flag;

    if (lane == 0) {
        for (unsigned s = 0; s < RING_BARS; ++s) mbar_init(ring.bars + s, 1);
        fence_barrier_init();
    }
    __syncwarp();

    const unsigned step = __ldcg(p.request + 3) + 1;
    bool ok = true;
    unsigned seq = 0, pseq = 0, ts = 0;
    unsigned long long key = 0ull;
    stamp(p, ts++);
    Phase cur = make_phase(p, PH_QKV, 0);
    ring_begin(cur, ring, lane);
    for (unsigned l = 0; l < p.nl && ok; ++l) {
        for (unsigned k = 0; k < 5 && ok; ++k) {
            if (k == 1) {  // attention; its scratch overlays the limb slots, so all warps leave it together
                if (dtraced(p, l) && warp == 0) drecord(p, 24, globaltimer());
                ok = attention_phase<HD, G>(p, step, l, as);
                ok = __syncthreads_or(!ok || aborted(p)) == 0;
                if (dtraced(p, l) && warp == 0) drecord(p, 28, globaltimer());
            } else {
                ok = run_gemv(p, cur, step, ring, slots, cta, lane, seq, pseq++, key);
                Phase nx;
                if (phase_after(p, cur.kind, cur.layer, nx)) cur = nx;
            }
            stamp(p, ts++);
        }
    }
    bool logits_done = false;
    if (ok && p.logits_mode) {
        ok = run_gemv(p, cur, step, ring, slots, cta, lane, seq, pseq++, key);
        logits_done = ok;
    }
    stamp(p, 1 + 5 * p.nl);
    ring_drain(ring);
    if (ok) {
        end_step(p, cta, key, logits_done);
        stamp(p, 2 + 5 * p.nl);
    }
}

using DecodeKernel = void (*)(const DecodeParams);

}  // namespace fyb
