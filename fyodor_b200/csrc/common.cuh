// common.cuh - device helpers shared by the sm_100a kernels of the provider.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#define FYB_DEV __device__ __forceinline__
#define FYB_HOST_DEV __host__ __device__ __forceinline__

namespace fyb {

// GGML storage ids (the engine's nya_llm_tensor_type).
enum : unsigned { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14, T_BF16 = 30 };

// Error words a kernel may raise instead of trapping. The host reads them
// from mapped memory after the stream is synchronized.
enum : unsigned { ERR_NONE = 0, ERR_TIMEOUT = 1, ERR_NONFINITE = 2, ERR_BOUNDS = 4 };

FYB_DEV unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }

// Binary16 bytes to float, bit-exact for every encoding (hardware cvt keeps
// subnormals; NaN payloads are not produced by any GGUF scale we read).
FYB_DEV float half_bits_to_float(unsigned short h)
{
    float v;
    asm("cvt.f32.f16 %0, %1;" : "=f"(v) : "h"(h));
    return v;
}
FYB_DEV float half_at(const unsigned char *p)
{
    return half_bits_to_float((unsigned short)((unsigned)p[0] | ((unsigned)p[1] << 8)));
}

// ---- programmatic dependent launch ---------------------------------------
FYB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FYB_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- global loads for streamed (read-once) weights -------------------------
FYB_DEV uint2 ldg_stream_u2(const void *p)
{
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
FYB_DEV uint4 ldg_stream_u4(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
FYB_DEV unsigned ldg_stream_u1(const void *p)
{
    unsigned r;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}
FYB_DEV void prefetch_l2(const void *p) { asm volatile("prefetch.global.L2::evict_last [%0];" :: "l"(p)); }
// Bulk prefetch of [p, p + bytes) into L2 (16-byte aligned, bytes a multiple of 16).
// Release/acquire fence at GPU scope: orders this thread's earlier writes
// before its later ones (the counter update after a tile's outputs).
FYB_DEV void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

FYB_DEV void bulk_prefetch_l2(const void *p, unsigned bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(p), "r"(bytes) : "memory");
}

// ---- mbarrier + bulk (TMA, non-tensor) copies into shared memory ----------
FYB_DEV void mbar_init(uint64_t *bar, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
FYB_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
FYB_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
FYB_DEV void mbar_expect_tx(uint64_t *bar, unsigned bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
FYB_DEV bool mbar_try_wait(uint64_t *bar, unsigned phase)
{
    unsigned ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(phase) : "memory");
    return ok != 0;
}
// Waits for the phase with an iteration bound; false means the copy never
// landed (the caller raises ERR_TIMEOUT instead of spinning forever).
FYB_DEV bool mbar_wait_bounded(uint64_t *bar, unsigned phase)
{
    for (unsigned i = 0; i < (1u << 22); ++i)
        if (mbar_try_wait(bar, phase)) return true;
    return false;
}
// global -> shared bulk copy completing on `bar`; both addresses 16-byte
// aligned and `bytes` a multiple of 16. Weights are streamed once: evict first.
FYB_DEV void bulk_copy_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar)
{
    asm volatile(
        "{\n .reg .b64 pol;\n createpolicy.fractional.L2::evict_first.b64 pol, 1.0;\n"
        " cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], pol;\n}\n"
        :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
FYB_DEV void ldmatrix_x4(unsigned (&r)[4], const void *p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}

// L2-coherent loads for data produced by other CTAs of the same launch.
FYB_DEV float ldcg_f32(const float *p) { return __ldcg(p); }

// ---- integer tensor-core fragments -----------------------------------------
// D(16x8, s32) = A(16x32, u8, row) * B(32x8, s8, col) + C
FYB_DEV void mma_u8s8_k32(int (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// D(16x8, s32) = A(16x16, u8, row) * B(16x8, s8, col) + C
FYB_DEV void mma_u8s8_k16(int (&d)[4], unsigned a0, unsigned a1, unsigned b0)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

// Order-preserving key for a float: larger float -> larger unsigned.
FYB_DEV unsigned float_order_key(float f)
{
    unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
FYB_DEV float float_from_order_key(unsigned k)
{
    unsigned u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

FYB_DEV float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
FYB_DEV float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace fyb
