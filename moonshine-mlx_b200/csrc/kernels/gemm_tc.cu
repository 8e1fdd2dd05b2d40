// bf16 tensor-core GEMM for sm_100a: TMA -> shared memory -> tcgen05.mma -> TMEM -> fused
// epilogue.  C[m, n] = epi( sum_k A[m, k] * B[n, k] ), A and B K-major bf16, fp32 accumulate.
//
// One CTA computes a 128 x BN output tile with four warps:
//   warp 0 (one lane)  TMA producer: STAGES-deep ring of 128x64 A / BNx64 B tiles, 128-byte
//                      swizzled, completion tracked by mbarrier transaction counts
//   warp 1 (one lane)  MMA issuer: 4 x tcgen05.mma (K = 16 each) per 64-wide k-block into a
//                      128 x BN fp32 accumulator in tensor memory; tcgen05.commit frees the
//                      stage and, after the last k-block, signals the epilogue
//   all four warps     epilogue: tcgen05.ld of their 32 accumulator lanes (= rows) into the
//                      idle stage buffers, then row by row (lanes along columns, so global
//                      accesses coalesce) bias / activation / residual / bf16 or fp32 store /
//                      K-V scatter / RoPE / SwiGLU / argmax / split-K atomics
//
// A is addressed through a 3-D tensor map (k, y, z) so a causal stride-2 convolution runs as
// `taps` accumulated GEMMs: tap t reads A at (k, y_t, m + z_t) and B at column t*K_tap + k.
// For a plain GEMM taps = 1, y = z = 0.
//
// Every mbarrier wait is bounded; a timeout records an error code and the CTA drains its
// in-flight copies (again bounded), frees its tensor memory and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"

namespace msb {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;         // bf16: 128 bytes = one 128B-swizzle row
constexpr int STAGES = 4;
constexpr int TC_THREADS = 128;
constexpr uint32_t WAIT_LIMIT = 1u << 22;   // polls of a bounded mbarrier wait

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

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// Shared-memory matrix descriptor: K-major tile of 128-byte rows with the 128B swizzle, 8-row
// groups 1024 bytes apart (stride byte offset), leading byte offset unused (1), version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor for kind::f16: bf16 A and B (K-major), fp32 accumulate, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN>
struct alignas(1024) TcSmem {
    __nv_bfloat16 a[STAGES][BM * BK];
    __nv_bfloat16 b[STAGES][BN * BK];
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t done;
    uint32_t tmem_base;
};

__device__ __forceinline__ void store_out(const TcGemmArgs& g, int m, int n, float v) {
    const GemmEpilogue& ep = g.ep;
    if (ep.bias) v += ep.bias[n];
    if (ep.act == ACT_SILU) v = silu(v);
    else if (ep.act == ACT_GELU) v = gelu_erf(v);
    if (ep.residual) v += ep.residual[(size_t)m * ep.ldr + n];
    if (ep.kv_scatter) {
        const int kvdim = ep.kv_heads * ep.head_dim;
        const int layer = n / (2 * kvdim);
        const int rem = n - layer * 2 * kvdim;
        const int kv = rem / kvdim;
        const int c = rem - kv * kvdim;
        const int head = c / ep.head_dim;
        const int dim = c - head * ep.head_dim;
        const size_t idx = ((((size_t)layer * 2 + kv) * ep.kv_heads + head) * ep.frame_cap +
                            (size_t)(m + ep.frame_offset)) * ep.head_dim + dim;
        if (ep.kv_out32) ep.kv_out32[idx] = v;
        if (ep.kv_out16) reinterpret_cast<__half*>(ep.kv_out16)[idx] = __float2half_rn(v);
        return;
    }
    if (ep.out) ep.out[(size_t)m * ep.ldc + n] = v;
    if (g.out_bf16) g.out_bf16[(size_t)m * g.ldc_bf16 + n] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // order-preserving as unsigned
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n);
}

// Epilogue of the accumulator column pair (n, n+1) of row m; n is even and has1 says
// whether column n+1 exists.  ROPE_KV and SWIGLU need even N, so their pairs are whole.
__device__ __forceinline__ void epilogue2(const TcGemmArgs& g, int m, int n, float a0, float a1, bool has1,
                                          float& best, int& bestn) {
    switch (g.mode) {
        case TC_EPI_ROPE_KV: {
            const TcRopeKv& r = g.rope;
            const int HD = r.H * r.hd, KVD = r.KVH * r.hd;
            const int t = *r.pos;
            const bool isq = n < HD, isk = !isq && n < HD + KVD;
            const int c = (isq ? n : (isk ? n - HD : n - HD - KVD)) % r.hd;
            if ((isq || isk) && c < r.nd) {
                const float cs = r.cos_t[(size_t)t * (r.nd >> 1) + (c >> 1)];
                const float sn = r.sin_t[(size_t)t * (r.nd >> 1) + (c >> 1)];
                const float b0 = a0 * cs - a1 * sn, b1 = a0 * sn + a1 * cs;
                a0 = b0;
                a1 = b1;
            }
            if (isq) {
                r.q[(size_t)m * HD + n] = a0;
                r.q[(size_t)m * HD + n + 1] = a1;
            } else {
                const int j = n - HD;
                r.kv_new[(size_t)m * 2 * KVD + j] = a0;
                r.kv_new[(size_t)m * 2 * KVD + j + 1] = a1;
                const int kv = j / KVD, c2 = j - kv * KVD;
                const int head = c2 / r.hd, dim = c2 - head * r.hd;
                const size_t idx = (((size_t)m * r.KVH + head) * r.t_cap + t) * r.hd + dim;
                void* base = kv ? r.v_cache : r.k_cache;
                if (r.kv_f16) {
                    reinterpret_cast<__half*>(base)[idx] = __float2half_rn(a0);
                    reinterpret_cast<__half*>(base)[idx + 1] = __float2half_rn(a1);
                } else {
                    reinterpret_cast<float*>(base)[idx] = a0;
                    reinterpret_cast<float*>(base)[idx + 1] = a1;
                }
            }
            break;
        }
        case TC_EPI_SWIGLU: {
            const float val = a0 + (g.ep.bias ? g.ep.bias[n] : 0.f);
            const float gate = a1 + (g.ep.bias ? g.ep.bias[n + 1] : 0.f);
            g.out_bf16[(size_t)m * g.ldc_bf16 + (n >> 1)] = __float2bfloat16_rn(val * silu(gate));
            break;
        }
        case TC_EPI_ARGMAX: {
            if (a0 > best) {  // columns arrive in increasing order per lane: strict > keeps the lowest
                best = a0;
                bestn = n;
            }
            if (has1 && a1 > best) {
                best = a1;
                bestn = n + 1;
            }
            if (g.ep.out) {
                g.ep.out[(size_t)m * g.ep.ldc + n] = a0;
                if (has1) g.ep.out[(size_t)m * g.ep.ldc + n + 1] = a1;
            }
            break;
        }
        case TC_EPI_ACCUM: {
            const bool add_bias = blockIdx.z == 0 && g.ep.bias;
            float* o = g.ep.out + (size_t)m * g.ep.ldc + n;
            atomicAdd(o, a0 + (add_bias ? g.ep.bias[n] : 0.f));
            if (has1) atomicAdd(o + 1, a1 + (add_bias ? g.ep.bias[n + 1] : 0.f));
            break;
        }
        default:
            store_out(g, m, n, a0);
            if (has1) store_out(g, m, n + 1, a1);
    }
}

template <int BN>
__global__ void __launch_bounds__(TC_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
               TcGemmArgs g) {
    extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
    TcSmem<BN>& s = *reinterpret_cast<TcSmem<BN>*>(
        (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    // this CTA's k-blocks: split blockIdx.z of g.splits
    const int nkb_all = g.taps * g.kb_per_tap;
    const int per_split = (nkb_all + g.splits - 1) / g.splits;
    const int kb_lo = blockIdx.z * per_split;
    const int nkb = max(0, min(nkb_all, kb_lo + per_split) - kb_lo);
    constexpr uint32_t A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
    __shared__ int s_fail;

    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        mbar_init(&s.done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {  // tensor memory: BN fp32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem_base)),
                     "r"((uint32_t)BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s.tmem_base;

    int issued = 0;  // producer: k-blocks whose copies were issued
    if (warp == 0 && lane == 0) {
        for (int kb = 0; kb < nkb; ++kb) {
            const int st = kb % STAGES;
            if (kb >= STAGES && !mbar_wait(&s.empty[st], ((kb / STAGES) - 1) & 1)) {
                atomicCAS(g.status, 0u, 5u);
                s_fail = 1;
                break;
            }
            const int gkb = kb_lo + kb;
            const int tap = gkb / g.kb_per_tap;
            const int k0 = (gkb - tap * g.kb_per_tap) * BK;
            mbar_expect_tx(&s.full[st], A_BYTES + B_BYTES);
            tma_load_3d(s.a[st], &tmap_a, &s.full[st], k0, g.tap_y[tap], m0 + g.tap_z[tap]);
            tma_load_2d(s.b[st], &tmap_b, &s.full[st], tap * g.k_per_tap + k0, n0);
            issued = kb + 1;
        }
    } else if (warp == 1 && lane == 0) {
        const uint32_t idesc = idesc_bf16(BM, BN);
        for (int kb = 0; kb < nkb; ++kb) {
            const int st = kb % STAGES;
            if (!mbar_wait(&s.full[st], (kb / STAGES) & 1)) {
                atomicCAS(g.status, 0u, 5u);
                s_fail = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a_addr = smem_u32(s.a[st]), b_addr = smem_u32(s.b[st]);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {  // 16 bf16 = 32 bytes per MMA along K
                mma_bf16(tmem, smem_desc_sw128(a_addr + k * 32), smem_desc_sw128(b_addr + k * 32), idesc,
                         (kb > 0 || k > 0) ? 1u : 0u);
            }
            mma_commit(&s.empty[st]);
        }
        if (nkb > 0) mma_commit(&s.done);
    }
    __syncwarp();
    __syncthreads();  // role loops finished; s_fail is final

    // epilogue: warp w owns accumulator lanes (rows) 32w .. 32w+31
    bool ok = nkb > 0 && mbar_wait(&s.done, 0);  // an empty k-split contributes nothing
    if (nkb > 0 && !ok) atomicCAS(g.status, 0u, 5u);
    ok = __all_sync(FULL, ok) && !s_fail;  // tcgen05.ld below is warp-collective
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // The accumulator tile goes through shared memory (the idle stage buffers) so that the
    // epilogue walks rows with lanes along columns: every global store / atomic of a warp
    // then touches one contiguous row segment instead of 32 rows.
    constexpr int LDS = BN + 1;  // +1: rows written by the 32 lanes of a warp hit distinct banks
    float* tile = reinterpret_cast<float*>(&s.a[0][0]);
    static_assert(sizeof(float) * BM * LDS <= sizeof(s.a) + sizeof(s.b), "epilogue tile must fit the stages");
    if (ok) {
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
        float* my = tile + (size_t)(warp * 32 + lane) * LDS;
        for (int c0 = 0; c0 < BN; c0 += 8) {
            float v[8];
            tmem_ld8(lane_addr + c0, v);
#pragma unroll
            for (int i = 0; i < 8; ++i) my[c0 + i] = v[i];
        }
    }
    __syncthreads();
    if (ok) {
        const int rows = min(BM, g.M - m0);
        for (int r = warp; r < rows; r += TC_THREADS / 32) {
            const int m = m0 + r;
            const float* row = tile + (size_t)r * LDS;
            float best = -INFINITY;
            int bestn = 0x7fffffff;
            for (int c = 2 * lane; c < BN; c += 64) {
                const int n = n0 + c;
                if (n >= g.N) break;
                epilogue2(g, m, n, row[c], row[c + 1], n + 1 < g.N, best, bestn);
            }
            if (g.mode == TC_EPI_ARGMAX) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float bo = __shfl_xor_sync(FULL, best, o);
                    const int no = __shfl_xor_sync(FULL, bestn, o);
                    if (bo > best || (bo == best && no < bestn)) {
                        best = bo;
                        bestn = no;
                    }
                }
                if (lane == 0 && best > -INFINITY) atomicMax(g.argmax + m, argmax_key(best, bestn));
            }
        }
    }
    // drain copies still in flight after a failure (bounded), then free tensor memory
    if (warp == 0 && lane == 0 && s_fail) {
        for (int kb = (issued > STAGES ? issued - STAGES : 0); kb < issued; ++kb)
            mbar_wait(&s.full[kb % STAGES], (kb / STAGES) & 1);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN)
                     : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

}  // namespace

bool tc_make_map_3d(CUtensorMap* map, const void* base, uint64_t dim_k, uint64_t dim_y, uint64_t dim_z,
                    uint64_t stride_y_bytes, uint64_t stride_z_bytes, uint32_t box_z) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {dim_k, dim_y, dim_z};
    const cuuint64_t strides[2] = {stride_y_bytes, stride_z_bytes};
    const cuuint32_t box[3] = {(cuuint32_t)BK, 1, box_z};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_make_map_2d(CUtensorMap* map, const void* base, uint64_t dim_k, uint64_t rows, uint64_t row_stride_bytes,
                    uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {dim_k, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_gemm_tc(const CUtensorMap& map_a, const CUtensorMap& map_b, const TcGemmArgs& g, int bn,
                           cudaStream_t stream) {
    if (g.M <= 0 || g.N <= 0) return cudaSuccess;
    if (g.taps < 1 || g.taps > 8 || g.kb_per_tap < 1 || !g.status) return cudaErrorInvalidValue;
    if (g.splits < 1 || (g.splits > 1 && g.mode != TC_EPI_ACCUM)) return cudaErrorInvalidValue;
    if ((g.mode == TC_EPI_ROPE_KV || g.mode == TC_EPI_SWIGLU) && (g.N & 1)) return cudaErrorInvalidValue;
    const dim3 grid((g.N + bn - 1) / bn, (g.M + BM - 1) / BM, g.splits);
    ++launch_counter();
    if (bn == 128) {
        const size_t smem = sizeof(TcSmem<128>) + 1024;
        static bool set128 = false;
        if (!set128) {
            cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem);
            if (e != cudaSuccess) return e;
            set128 = true;
        }
        gemm_tc_kernel<128><<<grid, TC_THREADS, smem, stream>>>(map_a, map_b, g);
    } else if (bn == 64) {
        const size_t smem = sizeof(TcSmem<64>) + 1024;
        static bool set64 = false;
        if (!set64) {
            cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem);
            if (e != cudaSuccess) return e;
            set64 = true;
        }
        gemm_tc_kernel<64><<<grid, TC_THREADS, smem, stream>>>(map_a, map_b, g);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace msb
