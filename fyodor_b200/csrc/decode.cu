// decode.cu - host side of the persistent decode kernel: shared-memory
// sizing, support checks, grid choice and the cooperative launch. The kernel
// itself (decode_kernel.cuh) is instantiated once per (head dimension, group
// size) in decode_inst.cu, which the build compiles once per variant so the
// instantiations compile in parallel.
#include "decode_kernel.cuh"

namespace fyb {

#define FYB_DK_DECL(HD, G) DecodeKernel decode_entry_##HD##_##G();
FYB_DK_DECL(128, 1) FYB_DK_DECL(128, 2) FYB_DK_DECL(128, 4) FYB_DK_DECL(128, 8)
FYB_DK_DECL(64, 1) FYB_DK_DECL(64, 2) FYB_DK_DECL(64, 4) FYB_DK_DECL(64, 8)
#undef FYB_DK_DECL

constexpr size_t SMEM_LIMIT = 227 * 1024;

// Ring bytes per warp for the rest of the layout taking `other` bytes: what
// is left (or `want`, when smaller but at least two Q6_K units), at most
// RING_BARS Q6_K units; 0 when fewer than two Q6_K units fit.
static unsigned ring_bytes_left(size_t other, unsigned want)
{
    if (other >= SMEM_LIMIT) return 0;
    size_t rb = (SMEM_LIMIT - other) / QG_WARPS / 16 * 16;
    rb = std::min<size_t>(rb, (size_t)RING_BARS * Q6_UNIT);
    if (want) rb = std::min<size_t>(rb, std::max<size_t>(want / 16 * 16, 2 * Q6_UNIT));
    return rb >= 2 * Q6_UNIT ? (unsigned)rb : 0;
}

static unsigned ring_bytes_for(const DecodeGeometry &g, unsigned want = 0)
{
    return ring_bytes_left(smem_layout(g.H, g.Hkv, g.hd, 0).total, want);
}

static size_t decode_smem_bytes(const DecodeGeometry &g, unsigned want = 0)
{
    return smem_layout(g.H, g.Hkv, g.hd, ring_bytes_for(g, want)).total;
}

int decode_supported(const DecodeGeometry &g, unsigned type_out)
{
    if (!g.nl || g.nl > 254 || !g.Hkv || g.H % g.Hkv) return 0;
    const unsigned G = g.H / g.Hkv;
    if ((g.hd != 64 && g.hd != 128) || !(G == 1 || G == 2 || G == 4 || G == 8)) return 0;
    if (g.d % 256 || g.ffn % 256 || (g.H * g.hd) % 256 || g.d / 256 > NORM_BLOCKS_MAX || g.ffn > 65536) return 0;
    if (type_out != T_Q4_K && type_out != T_Q6_K) return 0;
    return ring_bytes_for(g) != 0 && decode_smem_bytes(g) <= SMEM_LIMIT;
}

static DecodeKernel decode_kernel_for(const DecodeGeometry &g)
{
    const unsigned G = g.Hkv ? g.H / g.Hkv : 0;
#define FYB_DK(HDV, GV) \
    if (g.hd == HDV && G == GV) return decode_entry_##HDV##_##GV();
    FYB_DK(128, 1) FYB_DK(128, 2) FYB_DK(128, 4) FYB_DK(128, 8)
    FYB_DK(64, 1) FYB_DK(64, 2) FYB_DK(64, 4) FYB_DK(64, 8)
#undef FYB_DK
    return nullptr;
}

// One CTA per SM when one fits with the geometry's shared memory, else 0.
int decode_grid(int sms, const DecodeGeometry &g)
{
    const DecodeKernel decode_kernel = decode_kernel_for(g);
    if (!decode_kernel) return 0;
    const size_t smem = decode_smem_bytes(g);
    int per_sm = 0;
    if (cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel, QG_THREADS, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return per_sm >= 1 ? sms : 0;
}

int launch_decode(const DecodeLaunch &L, cudaStream_t s)
{
    if (!decode_supported(L.g, L.out_head.type) || L.grid <= 0 || !L.layers) return -1;
    if (!L.ll.xa || !L.ll.xm || !L.ll.q || !L.ll.kvnew || !L.ll.attn || !L.ll.h || !L.attn_partials) return -1;
    if (L.tp > 1 && !L.peers) return -1;
    DecodeParams p = {};
    p.layers = L.layers;
    p.nl = L.g.nl; p.d = L.g.d; p.H = L.g.H; p.Hkv = L.g.Hkv; p.hd = L.g.hd; p.ffn = L.g.ffn; p.V = L.g.V;
    p.capacity = L.g.capacity;
    p.out_head = L.out_head; p.out_norm = L.out_norm;
    p.embd = L.embd; p.embd_row_bytes = L.embd_row_bytes; p.embd_type = L.embd_type;
    p.eps = L.eps; p.attn_scale = L.attn_scale;
    p.rope_cos = L.rope_cos; p.rope_sin = L.rope_sin;
    p.request = L.request;
    p.ll = L.ll;
    p.logits = L.logits;
    p.sync = L.sync;
    p.attn_partials = L.attn_partials; p.attn_splits = L.attn_splits;
    p.argmax_key = L.argmax_key; p.argmax_token = L.argmax_token; p.tokens_log = L.tokens_log;
    p.error = L.error;
    p.logits_mode = L.logits_mode;
    p.ring_bytes = ring_bytes_for(L.g, L.ring_bytes);
    p.kcache = L.kcache; p.vcache = L.vcache;
    p.trace = L.trace; p.trace_slots = L.trace_slots; p.dtrace = L.dtrace;
    p.tp = L.tp; p.tp_rank = L.tp_rank; p.vocab0 = L.vocab0; p.peers = L.peers; p.xl = L.xl;
    if (p.ring_bytes < 2 * Q6_UNIT || !p.kcache || !p.vcache) return -1;  // every unit size needs two ring slots
    const size_t smem = decode_smem_bytes(L.g, L.ring_bytes);
    const DecodeKernel decode_kernel = decode_kernel_for(L.g);
    if (!decode_kernel) return -1;
    if (cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return -2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)L.grid);
    cfg.blockDim = dim3(QG_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_kernel, p) == cudaSuccess ? 0 : -2;
}

}  // namespace fyb
