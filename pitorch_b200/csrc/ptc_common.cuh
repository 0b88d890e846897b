// ptc_common.cuh -- shared device helpers for the sm_100a kernels.
//
// * Error handling: a failed CUDA call in the product path prints the call
//   site and aborts, the host analogue of the reference's panic()
//   (pitorch/runtime/gpu.c:107-108, pitorch/pt.c:50-54).
// * pitorch's libm-free math (pitorch/ops/core/pt_math.c) restated for the
//   device with explicitly rounded multiplies/adds (__fmul_rn/__fadd_rn),
//   so nvcc cannot contract them into FMAs and every result carries the
//   same bits as the host C build. RoPE angles at positions up to 1023 are
//   sensitive to this.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#define PTC_CHECK(call)                                                        \
    do {                                                                       \
        cudaError_t e_ = (call);                                               \
        if (e_ != cudaSuccess) {                                               \
            fprintf(stderr, "pitorch_b200: CUDA error %s (%s) at %s:%d: %s\n", \
                    cudaGetErrorName(e_), cudaGetErrorString(e_), __FILE__,    \
                    __LINE__, #call);                                          \
            abort();                                                           \
        }                                                                      \
    } while (0)

#define PTC_FATAL(...)                                        \
    do {                                                      \
        fprintf(stderr, "pitorch_b200: fatal: " __VA_ARGS__); \
        fputc('\n', stderr);                                  \
        abort();                                              \
    } while (0)

namespace ptc {

// ---------------------------------------------------------------------------
// pitorch math on the device (pt_math.c), bit-compatible with the host build.
// ---------------------------------------------------------------------------

// pt_math.c:8-25
__device__ __forceinline__ float pt_expf(float x) {
    if (x > 88.7f) return 3.4028235e+38f;
    if (x < -87.3f) return 0.0f;
    float t = __fmul_rn(x, 1.4426950408889634f);
    int n = __float2int_rz(__fadd_rn(t, t >= 0.0f ? 0.5f : -0.5f));
    float r = __fsub_rn(x, __fmul_rn((float)n, 0.6931471805599453f));
    float p = 0.0083333333f;
    p = __fadd_rn(0.0416666667f, __fmul_rn(r, p));
    p = __fadd_rn(0.1666666667f, __fmul_rn(r, p));
    p = __fadd_rn(0.5f, __fmul_rn(r, p));
    p = __fadd_rn(1.0f, __fmul_rn(r, p));
    p = __fadd_rn(1.0f, __fmul_rn(r, p));
    return __fmul_rn(p, __int_as_float((n + 127) << 23));
}

// pt_math.c:31-44
__device__ __forceinline__ float pt_logf(float x) {
    if (x <= 0.0f) return -3.4028235e+38f;
    uint32_t u = __float_as_uint(x);
    int e = (int)((u >> 23) & 0xFF) - 127;
    float m = __uint_as_float((u & 0x007FFFFFu) | 0x3F800000u);
    if (m > 1.41421356f) { m = __fmul_rn(m, 0.5f); e++; }
    float f = __fsub_rn(m, 1.0f);
    float s = 0.11111111f;
    s = __fadd_rn(-0.125f, __fmul_rn(f, s));
    s = __fadd_rn(0.14285714f, __fmul_rn(f, s));
    s = __fadd_rn(-0.16666667f, __fmul_rn(f, s));
    s = __fadd_rn(0.2f, __fmul_rn(f, s));
    s = __fadd_rn(-0.25f, __fmul_rn(f, s));
    s = __fadd_rn(0.33333333f, __fmul_rn(f, s));
    s = __fadd_rn(-0.5f, __fmul_rn(f, s));
    s = __fadd_rn(1.0f, __fmul_rn(f, s));
    return __fadd_rn(__fmul_rn(f, s), __fmul_rn((float)e, 0.69314718f));
}

// pt_math.c:58-62
__device__ __forceinline__ float pt_reduce_2pi(float x) {
    float k = __fmul_rn(x, 0.15915494309190f);
    k = (float)__float2int_rz(__fadd_rn(k, k >= 0.0f ? 0.5f : -0.5f));
    return __fsub_rn(x, __fmul_rn(k, 6.28318530717959f));
}

// pt_math.c:64-74
__device__ __forceinline__ float pt_sinf(float x) {
    x = pt_reduce_2pi(x);
    if (x > 1.57079632679490f) x = __fsub_rn(3.14159265358979f, x);
    else if (x < -1.57079632679490f) x = __fsub_rn(-3.14159265358979f, x);
    float z = __fmul_rn(x, x);
    float s = 0.00000275573f;
    s = __fadd_rn(-0.00019841270f, __fmul_rn(z, s));
    s = __fadd_rn(0.00833333333f, __fmul_rn(z, s));
    s = __fadd_rn(-0.16666666667f, __fmul_rn(z, s));
    s = __fadd_rn(1.0f, __fmul_rn(z, s));
    return __fmul_rn(x, s);
}

// pt_math.c:76-87
__device__ __forceinline__ float pt_cosf(float x) {
    x = pt_reduce_2pi(x);
    float sign = 1.0f;
    if (x > 1.57079632679490f) { x = __fsub_rn(3.14159265358979f, x); sign = -1.0f; }
    else if (x < -1.57079632679490f) { x = __fsub_rn(-3.14159265358979f, x); sign = -1.0f; }
    float z = __fmul_rn(x, x);
    float c = 0.00002480159f;
    c = __fadd_rn(-0.00138888889f, __fmul_rn(z, c));
    c = __fadd_rn(0.04166666667f, __fmul_rn(z, c));
    c = __fadd_rn(-0.50000000000f, __fmul_rn(z, c));
    c = __fadd_rn(1.0f, __fmul_rn(z, c));
    return __fmul_rn(sign, c);
}

// pt_math.c:92-102 (IEEE division: the library is built without fast math)
__device__ __forceinline__ float pt_sqrtf(float x) {
    if (x <= 0.0f) return 0.0f;
    float y = __uint_as_float(0x1fbd1df5u + (__float_as_uint(x) >> 1));
    for (int i = 0; i < 3; i++) y = __fmul_rn(0.5f, __fadd_rn(y, __fdiv_rn(x, y)));
    return y;
}

// 1 / pt_sqrtf(sum_sq / dim + 1e-5), the rmsnorm scale of pt_ops.c:9.
__device__ __forceinline__ float rms_scale(float sum_sq, int dim) {
    return __fdiv_rn(1.0f, pt_sqrtf(__fadd_rn(__fdiv_rn(sum_sq, (float)dim), 1e-5f)));
}

// The RoPE rotation angle of pt_ops.c:36-37 for even index i.
__device__ __forceinline__ float rope_theta(int i, int head_dim, int pos) {
    float e = __fdiv_rn(__fmul_rn(-9.210340372f, (float)(i % head_dim)), (float)head_dim);
    return __fmul_rn((float)pos, pt_expf(e));
}

// silu(a) * b as pitorch computes it: a / (1 + exp(-a)), then times b
// (pt_ops.c:28-31 followed by vec_mul, pt_ops.c:56-59).
__device__ __forceinline__ float silu_mul(float a, float b) {
    return __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, pt_expf(-a))), b);
}

// ---------------------------------------------------------------------------
// Warp helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Streaming 128-bit load of weights: read-only path, no L1 allocation
// (weights are touched once per token).
__device__ __forceinline__ float4 ldg_stream(const float4 *p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    acc = fmaf(a.w, b.w, acc);
    return acc;
}

// Vector reduction into global memory (performed at L2): dst 16-byte aligned.
__device__ __forceinline__ void red_add_v4(float *dst, float4 v) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}

// Fire-and-forget 64-bit max at L2, and an add with acquire-release
// semantics at GPU scope that returns the old value.
__device__ __forceinline__ void red_max_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("red.relaxed.gpu.global.max.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Programmatic dependent launch (sm_90+): wait for the producer grid's
// memory, and let the next grid in the stream start its prologue early.
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// A pipeline link's mailbox in the receiving rank's memory: the message of
// one position ([pos | x], pitorch/dist/pt_dist_pipeline.c:287-302) and the
// number of messages delivered so far, published last with release
// semantics at system scope.
struct MailboxHeader {
    int pos;
    unsigned seq;   // messages delivered into this mailbox
    int pad[2];     // x starts 16-byte aligned
};

// One rank's classifier result in a vocab-parallel decode: the packed argmax
// key of its rows for position `pos`, published by `seq` (release, system
// scope) like a mailbox message. A combining rank's mailbox carries one slot
// per rank after its x.
struct KeySlot {
    unsigned long long key;
    unsigned seq;
    int pos;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Order-preserving map of a float to uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Argmax key: value in the high word, inverted index in the low word, so the
// 64-bit max picks the largest value and, among equals, the lowest index --
// the strict '>' scan of pt_ops.c:65-70.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    return ((unsigned long long)float_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ int argmax_key_index(unsigned long long k) {
    return (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
}

// ---------------------------------------------------------------------------
// Bulk (TMA) global->shared copies completed on an mbarrier. Only the
// form that writes the issuing CTA's own shared memory is used, and only on
// this GPU's own memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned smem_u32(const void *p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// L2 eviction priority of this kernel's own loads (createpolicy; no device
// setting changes): POL_NONE issues the plain forms.
enum L2Pol { POL_NONE = 0, POL_FIRST = 1, POL_LAST = 2, POL_NORMAL = 3 };
__device__ __forceinline__ uint64_t make_l2_policy(int kind) {
    uint64_t p = 0;
    if (kind == POL_FIRST) asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    else if (kind == POL_LAST) asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    else if (kind == POL_NORMAL) asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// bulk_g2s with an L2 cache policy (kind != POL_NONE) or without.
__device__ __forceinline__ void bulk_g2s_pol(void *dst, const void *src, unsigned bytes, uint64_t *bar, int kind,
                                             uint64_t pol) {
    if (kind == POL_NONE) {
        bulk_g2s(dst, src, bytes, bar);
        return;
    }
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// Per-thread asynchronous 16-byte global->shared copies (dst, src 16-byte
// aligned), completed by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16_pol(void *dst, const void *src, int kind, uint64_t pol) {
    if (kind == POL_NONE) {
        cp_async16(dst, src);
        return;
    }
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "l"(pol)
                 : "memory");
}
// 128-bit L2-only load with an L2 cache policy (or the plain __ldcg).
__device__ __forceinline__ float4 ldcg_pol(const float4 *p, int kind, uint64_t pol) {
    if (kind == POL_NONE) return __ldcg(p);
    float4 v;
    asm volatile("ld.global.cg.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Warm L2 with a global range (bulk prefetch; no data is returned).
// src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2(const void *src, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_l2_pol(const void *src, unsigned bytes, int kind, uint64_t pol) {
    if (kind == POL_NONE) {
        prefetch_l2(src, bytes);
        return;
    }
    asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(src), "r"(bytes), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for an mbarrier phase: gives up after `limit` polls (each
// try_wait itself blocks for a bounded hardware interval) and reports it.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, unsigned parity, int *err, int code) {
    for (long it = 0; it < (1L << 22); it++)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicExch(err, code);
    return false;
}

}  // namespace ptc
