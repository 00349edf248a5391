// pkv_device.cuh -- sm_100a device primitives of the paged decode engine:
// mbarrier pipeline, TMA tensor loads, ldmatrix / mma.sync / movmatrix
// fragments and the bounded waits every kernel here uses.
#pragma once

#include <cuda.h>  // CUtensorMap (type only; the driver is reached at run time)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pkv {

constexpr int kHeadDim = 128;        // reference: kernels/persistentkv_attention.cuh:26
constexpr int kTileTokens = 32;      // work-item tile unit, reference cuh:28
constexpr int kStageTokens = 16;     // tokens staged per ring slot
#ifndef PKV_CONSUMER_WARPS
#define PKV_CONSUMER_WARPS 4
#endif
#ifndef PKV_MIN_CTAS_PER_SM
#define PKV_MIN_CTAS_PER_SM 2
#endif
constexpr int kConsumerWarps = PKV_CONSUMER_WARPS;  // math warps per CTA
constexpr int kThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kStateStride = kHeadDim + 2;  // {m, l, acc[128]} per state row
constexpr int kRowBytes = kHeadDim * 2;     // one token of one KV head
constexpr int kHalfRowBytes = 128;          // 64 elements: one SW128 line
constexpr int kSlotBytes = 4 * kStageTokens * kHalfRowBytes;  // K lo/hi, V lo/hi
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kNegFltMax = -3.402823466e38f;

// Bounded waits: a pipeline wait that exceeds this many nanoseconds gives up,
// raises PKV_DEVERR_TIMEOUT and lets the kernel drain and return.
constexpr unsigned long long kWaitLimitNs = 4000000000ull;

constexpr unsigned kErrPageId = 0x1u;
constexpr unsigned kErrLogicalPage = 0x2u;
constexpr unsigned kErrWorkItem = 0x4u;
constexpr unsigned kErrSlot = 0x8u;
constexpr unsigned kErrIndex = 0x10u;
constexpr unsigned kErrTimeout = 0x20u;
constexpr unsigned kErrPeer = 0x40u;  // a peer's state did not arrive in time
constexpr unsigned kErrNoPage = 0x80u;  // KV append: the free-page list ran out

// Sharded decode: each rank's states reach the other ranks' memory through
// plain peer stores over NVLink as 8-byte words carrying the step number;
// the owner polls them, bounded like every other wait.
constexpr unsigned long long kPeerWaitLimitNs = 2000000000ull;
constexpr int kMaxWorld = 8;

__device__ __forceinline__ unsigned ld_relaxed_gpu_u32(const unsigned* addr) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void raise_error(unsigned* error_word, unsigned bit) {
    if (error_word != nullptr) atomicOr(error_word, bit);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase of `bar` with the given parity to complete. Returns
// false if it did not within kWaitLimitNs, or as soon as another thread of
// the CTA has raised `*abort_flag`.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  const volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long start = global_timer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i) {
            if (mbar_try_wait(bar, parity)) return true;
        }
        if (abort_flag != nullptr && *abort_flag != 0) return false;
        if (global_timer_ns() - start > kWaitLimitNs) return false;
    }
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Named barrier among the consumer warps only (the producer never joins).
__device__ __forceinline__ void consumer_bar_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled TMA load (no multicast) of one box into shared memory; completion
// is signalled on `bar` as transaction bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 16-byte cp.async global -> shared (L2 only); bytes beyond src_bytes (0 or
// 16) are zero-filled, so a masked chunk reads nothing.
__device__ __forceinline__ void cp_async_16(uint32_t smem_dst, const void* src, uint32_t src_bytes,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(smem_dst),
        "l"(src), "r"(src_bytes), "l"(policy)
        : "memory");
}

// Arrives on `bar` once all prior cp.async of this thread have completed
// (the barrier's expected count includes this arrival).
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// One bulk copy (TMA, untiled, no multicast) of `bytes` contiguous bytes of
// global memory into shared memory, completing as transaction bytes on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t smem_dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_dst), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Orders this thread's generic-proxy global accesses (and those it has
// acquired) before its later async-proxy (bulk copy) accesses of global memory.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Atomic add at GPU scope with acquire-release semantics: the release half
// publishes every write that happens-before it (those of the CTA's other
// threads included, through a preceding barrier); the acquire half makes the
// writes released by earlier adds visible.  The issuing thread only waits for
// the result when it reads it.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int32_t* addr, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;"
                 : "=r"(old)
                 : "l"(addr), "r"(v)
                 : "memory");
    return old;
}

// ---------------------------------------------------------------- PDL
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- fragments
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <typename T>
struct ElemOps;

template <>
struct ElemOps<__half> {
    static constexpr bool kSplitP = false;
    static __device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
        asm(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
            "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ __half from_float(float x) { return __float2half_rn(x); }
};

template <>
struct ElemOps<__nv_bfloat16> {
    static constexpr bool kSplitP = true;
    static __device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
        asm(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
            "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    // The rounding residual x - bf16(x) of each value, itself as bf16.
    static __device__ __forceinline__ uint32_t pack_residual(float lo, float hi) {
        const float rlo = lo - __bfloat162float(__float2bfloat16_rn(lo));
        const float rhi = hi - __bfloat162float(__float2bfloat16_rn(hi));
        return pack(rlo, rhi);
    }
    static __device__ __forceinline__ __nv_bfloat16 from_float(float x) {
        return __float2bfloat16_rn(x);
    }
};

}  // namespace pkv
