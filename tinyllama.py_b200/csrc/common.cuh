// Shared device helpers for the sm_100a decode kernels: element traits,
// the per-device status word, and thin inline-PTX wrappers for mbarriers,
// bulk / tensor TMA copies, ldmatrix and the bf16/f16 mma.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tinyllama_b200.h"

namespace tlb {

// Per-device status word (TLB_STATUS_* bits). Defined in abi.cu.
extern __device__ unsigned int g_status;

__device__ __forceinline__ void flag_status(unsigned int bits) {
    atomicOr(&g_status, bits);
}

// ---------------------------------------------------------------- elements
template <typename T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float to_f(float x) { return x; }
    static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
    static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
    static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// Two floats -> packed pair of 16-bit values (low half = first argument).
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Probabilities as mma operands (in [0, 1] in the decode kernel, at most 2^8
// with the prefill kernel's lazy exponent base): fp16 keeps 11 significant bits,
// which is enough; bf16 keeps 8, so it is carried as a hi + lo pair whose sum
// holds 16 bits (lo is the bf16 rounding of the remainder).
template <typename T> constexpr bool kSplitP = false;
template <> constexpr bool kSplitP<__nv_bfloat16> = true;

template <typename T>
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    if constexpr (kSplitP<T>) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        const float2 hf = __bfloat1622float2(h);
        const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
        hi = *reinterpret_cast<const uint32_t*>(&h);
        lo = *reinterpret_cast<const uint32_t*>(&l);
    } else {
        hi = pack2<T>(a, b);
        lo = 0u;
    }
}

// Four consecutive outputs (scaled fp32 -> storage type) with one store:
// 8 bytes for half types, 16 for fp32.
template <typename T> struct Vec4Out;
template <> struct Vec4Out<__nv_bfloat16> {
    static __device__ __forceinline__ void store(__nv_bfloat16* p, float4 v, float s) {
        uint2 u;
        u.x = pack2<__nv_bfloat16>(v.x * s, v.y * s);
        u.y = pack2<__nv_bfloat16>(v.z * s, v.w * s);
        *reinterpret_cast<uint2*>(p) = u;
    }
};
template <> struct Vec4Out<__half> {
    static __device__ __forceinline__ void store(__half* p, float4 v, float s) {
        uint2 u;
        u.x = pack2<__half>(v.x * s, v.y * s);
        u.y = pack2<__half>(v.z * s, v.w * s);
        *reinterpret_cast<uint2*>(p) = u;
    }
};

// ------------------------------------------------------------- shared mem
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Orders this thread's generic-proxy global stores before later async-proxy
// (TMA) reads of the same addresses.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// NeoX rotation of the pair (x, y) = (v[i], v[i + rot/2]) by (c, s) =
// (cos_sin[pos, i], cos_sin[pos, rot/2 + i]) in fp32
// (pos_encoding_kernel.cu:24-65). Each product and the sum are rounded on
// their own (no fused multiply-add contraction): every kernel that rotates,
// in whatever code it is inlined into, rounds to the same bits, and those are
// the bits of the same fp32 expression evaluated step by step on the host.
__device__ __forceinline__ void rope_pair(float x, float y, float c, float s, float& xo,
                                          float& yo) {
    xo = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, s));
    yo = __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, s));
}

// Packed pair of 16-bit values (low half first) -> two floats.
template <typename T> __device__ __forceinline__ void unpack2(uint32_t w, float& lo, float& hi) {
    T v[2];
    memcpy(v, &w, 4);
    lo = Elem<T>::to_f(v[0]);
    hi = Elem<T>::to_f(v[1]);
}

// rope_pair on the two packed columns of x (first half) and of y (the same
// columns + rot/2), with their packed cos and sin.
template <typename T>
__device__ __forceinline__ void rope_packed2(uint32_t& x, uint32_t& y, uint32_t c, uint32_t s) {
    float x0, x1, y0, y1, c0, c1, s0, s1, xo0, xo1, yo0, yo1;
    unpack2<T>(x, x0, x1);
    unpack2<T>(y, y0, y1);
    unpack2<T>(c, c0, c1);
    unpack2<T>(s, s0, s1);
    rope_pair(x0, y0, c0, s0, xo0, yo0);
    rope_pair(x1, y1, c1, s1, xo1, yo1);
    x = pack2<T>(xo0, xo1);
    y = pack2<T>(yo0, yo1);
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
#ifdef TLB_MBAR_SPIN
    // Non-suspending probe: the waiting warp polls instead of sleeping.
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
#else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
#endif
    return ok != 0;
}
// Bounded wait: every try_wait may suspend the thread for a short,
// hardware-defined interval, so this limit is far above any legitimate wait
// (a few microseconds) while still ending a wait that would never complete.
constexpr uint32_t kWaitLimit = 1u << 22;
static_assert(kWaitLimit == TLB_WAIT_LIMIT_DEFAULT, "one default bound");
// `limit` probes at most (0: give up at once without probing).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  uint32_t limit = kWaitLimit) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    return false;
}

// ---------------------------------------------------------------- TMA copies
// L2 policy for data that is read exactly once per step (the KV stream).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 2-D tiled tensor load (no multicast) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, int32_t z, uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
        : "memory");
}
// Untiled bulk load: src and dst 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
        : "memory");
}
// One lane of the (converged, full) warp: the single-thread region that
// issues TMA copies, so their operands are known to be warp-uniform.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(pred));
    return pred != 0;
}
// Bulk prefetch of `bytes` (a multiple of 16, 16-byte aligned) into L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ----------------------------------------------------------- warp matrix ops
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D = A(16x16, row) * B(16x8, col) + D, fp32 accumulate.
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4],
                                                 uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// atomicInc with release-acquire semantics at GPU scope:
// *p = (*p >= limit) ? 0 : *p + 1, returns the old value.
// Acquire load / relaxed store at GPU scope.
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_gpu(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atomic_inc_acq_rel(unsigned* p, unsigned limit) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;"
                 : "=r"(old)
                 : "l"(p), "r"(limit)
                 : "memory");
    return old;
}

// Programmatic dependent launch: wait until the kernel this one was allowed
// to overlap has finished and its writes are visible (no-op otherwise), and
// let the next kernel's prologue start early.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 4-byte asynchronous global -> shared copy (Ampere-style cp.async), for
// small metadata that must arrive ahead of its use.
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(src))
                 : "memory");
}
// 16 bytes global -> shared, through L2 only (both addresses 16-byte aligned)
__device__ __forceinline__ void cp_async_cg16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(src))
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Named barrier among `count` threads (count a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// 128-bit vector of elements for the streaming kernels.
struct alignas(16) Vec16 {
    uint4 v;
};

}  // namespace tlb
