// Shared device helpers for the Moonshine B200 kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace msb {

constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}

// Block-wide sum; `red` must hold >= 32 floats.  All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = (lane < nw) ? red[lane] : 0.f;
    t = warp_sum(t);
    return t;
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + expf(-x)); }

__device__ __forceinline__ float gelu_erf(float x) {
    return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
}

// L2-coherent loads for data written by other CTAs of the same launch.
__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float4 ldcg4(const float4* p) { return __ldcg(p); }

// Streaming read-only loads (weights): no L1 allocation.
__device__ __forceinline__ float4 ld_stream4(const float4* p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch
// A grid launched with programmatic stream serialization (launch_kernel under pdl_launches())
// may be scheduled while its predecessor in the stream still runs: it must call pdl_wait()
// before it reads anything the predecessor writes (the wait returns once that grid has
// completed and its writes are visible; without the launch attribute it returns at once).
// pdl_trigger() lets the next such grid start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// bf16 of v at p[0] and, when lo_off != 0, the bf16 of its remainder v - bf16(v) at
// p[lo_off] (the low plane of a split operand: v = hi + lo to ~2^-17 relative)
__device__ __forceinline__ void st_bf16_split(__nv_bfloat16* p, float v, size_t lo_off) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    p[0] = h;
    if (lo_off) p[lo_off] = __float2bfloat16_rn(v - __bfloat162float(h));
}

// ---------------------------------------------------------------- mbarriers and bulk copies
constexpr uint32_t WAIT_LIMIT = 1u << 22;  // polls of a bounded mbarrier wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// One plain arrival (no transaction bytes).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded parity wait; returns false after WAIT_LIMIT polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(a), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// Contiguous global -> shared bulk copy completing on `bar` (both addresses 16-byte
// aligned, bytes a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// bulk_load with an L2 eviction-priority policy (from make_l2_policy) attached.
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                               uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// L2 policy: a fraction `keep` of the accessed lines evict_last, the others evict_first.
__device__ __forceinline__ uint64_t make_l2_policy(float keep) {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.L2::evict_first.b64 %0, %1;" : "=l"(pol) : "f"(keep));
    return pol;
}

// Gumbel(0, 1) noise for temperature sampling by the Gumbel-max trick (the argmax of
// logit / T + g over the vocabulary is a draw from softmax(logit / T); Gumbel 1954, used
// for sampling by Maddison, Tarlow and Minka 2014).  The uniform comes from a counter-based
// hash of (seed, stream, index) with the SplitMix64 finalizer (Steele, Lea and Flood 2014),
// so a draw depends only on those three numbers.
__device__ __forceinline__ float gumbel_noise(uint32_t seed, uint32_t stream, uint32_t idx) {
    uint64_t z = (((uint64_t)seed << 32) | stream) + (uint64_t)(idx + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    const float u = ((float)(z >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1), 24 bits
    return -logf(-logf(u));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Grid-wide barrier for a cooperative (co-resident) launch.  `count` is zeroed by the
// host before the launch and only grows; barrier number `epoch` completes when it
// reaches epoch * gridDim.x.  The wait is bounded by `timeout_ns`; on expiry the
// status word is set and every CTA returns false so the kernel can exit cleanly.
__device__ __forceinline__ bool grid_barrier(unsigned* count, unsigned* status, unsigned& epoch,
                                             uint64_t timeout_ns = 2000000000ull) {
    __shared__ int s_ok;
    __syncthreads();
    epoch += 1;
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned target = epoch * gridDim.x;
        red_release_gpu_add(count, 1u);
        const uint64_t t0 = globaltimer_ns();
        while (true) {
            unsigned v = ld_acquire_gpu(count);
            if ((int)(v - target) >= 0) break;
            if (*(volatile unsigned*)status != DEV_OK) { ok = 0; break; }
            if (globaltimer_ns() - t0 > timeout_ns) {
                atomicCAS(status, DEV_OK, DEV_BARRIER_TIMEOUT);
                ok = 0;
                break;
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

}  // namespace msb
