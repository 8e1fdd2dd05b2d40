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
//                      K-V scatter / RoPE / SwiGLU / argmax / residual update
//
// Split-K: the `splits` CTAs of one output tile (blockIdx.z) form a thread-block cluster.
// Each stages its partial tile in its own shared memory; after a cluster barrier, split z
// sums rows [z * R / S, (z + 1) * R / S) of all S partials in split order through
// distributed shared memory and runs the epilogue on them.  The sum order is fixed, so
// results do not depend on which split finishes first.
//
// Large GEMMs with the plain epilogue (more output tiles than SMs, no k-splits) run a
// persistent form instead: one CTA per SM walks its tiles with the producer and MMA warps
// running ahead into a second TMEM accumulator while four epilogue warps drain the first.
//
// A is addressed through a 3-D tensor map (k, y, z) so a causal stride-2 convolution runs as
// `taps` accumulated GEMMs: tap t reads A at (k, y_t, m + z_t) and B at column t*K_tap + k.
// For a plain GEMM taps = 1, y = z = 0.
//
// Every mbarrier wait is bounded; a timeout records an error code and the CTA drains its
// in-flight copies (again bounded), frees its tensor memory and exits.
#include <algorithm>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "cluster_common.cuh"
#include "common.cuh"
#include "kernels.h"

namespace msb {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;         // bf16: 128 bytes = one 128B-swizzle row
constexpr int TC_THREADS = 128;
static_assert(BM == TC_THREADS, "one thread per tile row (folded LayerNorm statistics)");

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

// 32 consecutive accumulator columns of this thread's lane, one wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// SP (split): A and B each come as a bf16 high plane and a bf16 low plane (x = hi + lo to
// ~2^-17 relative) and every MMA step accumulates hi.hi + hi.lo + lo.hi, which gives fp32
// checkpoints fp32-level products on the bf16 tensor pipe; 3 stages of both planes.
template <int BN, bool SP>
struct alignas(1024) TcSmem {
    static constexpr int ST = SP ? 3 : 4;  // ring stages
    static constexpr int P = SP ? 2 : 1;   // planes per operand
    __nv_bfloat16 a[ST][P][BM * BK];
    __nv_bfloat16 b[ST][P][BN * BK];
    uint64_t full[ST];
    uint64_t empty[ST];
    uint64_t done;
    uint32_t tmem_base;
};

__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // order-preserving as unsigned
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n);
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

__device__ __forceinline__ void st_bf16x4(__nv_bfloat16* p, float4 v) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p) = u;
}

// bf16 high part of four values, and (lo_off != 0) the bf16 of their remainders lo_off
// elements further on
__device__ __forceinline__ void st_bf16x4_split(__nv_bfloat16* p, float4 v, size_t lo_off) {
    st_bf16x4(p, v);
    if (lo_off) {
        const float4 r = make_float4(v.x - __bfloat162float(__float2bfloat16_rn(v.x)),
                                     v.y - __bfloat162float(__float2bfloat16_rn(v.y)),
                                     v.z - __bfloat162float(__float2bfloat16_rn(v.z)),
                                     v.w - __bfloat162float(__float2bfloat16_rn(v.w)));
        st_bf16x4(p + lo_off, r);
    }
}

__device__ __forceinline__ void st_f16x4(__half* p, float4 v) {
    __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p) = u;
}

// Row stride (floats) of the accumulator tile staged in shared memory: a multiple of 4 for
// 128-bit accesses, and 4 mod 32 so the 8 lanes of one 128-bit store phase hit distinct banks.
template <int BN>
__host__ __device__ constexpr int tile_ld() { return BN + 4; }

// Epilogue of a staged 128 x BN accumulator tile.  Thread t owns the four columns
// n = n0 + 4 (t mod BN/4) .. n + 3 for every row it visits, so column-only terms (bias,
// RoPE angles, K/V scatter base) are loaded once, and the BN/4 threads of a row write one
// contiguous row segment with 128-bit accesses.  N is a multiple of 4 (checked at launch).
// Rows [r_lo, r_hi) of the tile; lnr (folded LayerNorm) holds each tile row's (mean, rstd);
// res (ACCUM, optional) the residual rows [r_lo, r_hi) read ahead, BN / 4 float4 per row.
template <int BN, int MODE>
__device__ __forceinline__ void epilogue_tile(const TcGemmArgs& g, const float* tile, int m0, int n0, int r_lo,
                                              int r_hi, const float2* lnr, const float4* res, int t) {
    constexpr int TPR = BN / 4;            // threads per row
    constexpr int RPP = TC_THREADS / TPR;  // rows per pass
    constexpr int LDS = tile_ld<BN>();
    const int c = (t % TPR) * 4;
    const int n = n0 + c;
    const bool col_ok = n < g.N;
    const int r0 = r_lo + t / TPR;
    const int rows = r_hi;
    const int passes = (r_hi - r_lo + RPP - 1) / RPP;
    const GemmEpilogue& ep = g.ep;

    float4 bias = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (MODE == TC_EPI_STD || MODE == TC_EPI_SWIGLU || MODE == TC_EPI_ACCUM) {
        if (ep.bias && col_ok) bias = *reinterpret_cast<const float4*>(ep.bias + n);
    }
    float4 csum = make_float4(0.f, 0.f, 0.f, 0.f);
    if (lnr && col_ok) csum = *reinterpret_cast<const float4*>(g.lnf.csum + n);
    // K/V scatter: column part of the cache index (the four columns share one head)
    size_t kv_col = 0;
    if constexpr (MODE == TC_EPI_STD) {
        if (ep.kv_scatter && col_ok) {
            const int kvdim = ep.kv_heads * ep.head_dim;
            const int layer = n / (2 * kvdim);
            const int rem = n - layer * 2 * kvdim;
            const int kv = rem / kvdim;
            const int cc = rem - kv * kvdim;
            const int head = cc / ep.head_dim;
            const int dim = cc - head * ep.head_dim;
            kv_col = (((size_t)layer * 2 + kv) * ep.kv_heads + head) * ep.frame_cap * ep.head_dim + dim;
        }
    }
    // RoPE: region of the four columns and the angles of their two pairs
    int region = 0, rdim = 0;  // region 0 = q, 1 = k, 2 = v; rdim = column inside the region
    float cs0 = 1.f, sn0 = 0.f, cs1 = 1.f, sn1 = 0.f;
    int t_pos = 0;
    if constexpr (MODE == TC_EPI_ROPE_KV) {
        const TcRopeKv& r = g.rope;
        const int HD = r.H * r.hd, KVD = r.KVH * r.hd;
        region = n < HD ? 0 : (n < HD + KVD ? 1 : 2);
        rdim = region == 0 ? n : (region == 1 ? n - HD : n - HD - KVD);
        t_pos = *r.pos;
        const int ch = rdim % r.hd;
        if (col_ok && region < 2) {
            const float* cr = r.cos_t + (size_t)t_pos * (r.nd >> 1);
            const float* sr = r.sin_t + (size_t)t_pos * (r.nd >> 1);
            if (ch < r.nd) {
                cs0 = cr[ch >> 1];
                sn0 = sr[ch >> 1];
            }
            if (ch + 2 < r.nd) {
                cs1 = cr[(ch >> 1) + 1];
                sn1 = sr[(ch >> 1) + 1];
            }
        }
    }

#pragma unroll 2
    for (int p = 0; p < passes; ++p) {
        const int r = r0 + p * RPP;
        const bool ok = col_ok && r < rows;
        const int m = m0 + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ok) v = *reinterpret_cast<const float4*>(tile + (size_t)r * LDS + c);
        if (lnr && ok) {
            const float2 st = lnr[r];
            v = make_float4((v.x - st.x * csum.x) * st.y, (v.y - st.x * csum.y) * st.y,
                            (v.z - st.x * csum.z) * st.y, (v.w - st.x * csum.w) * st.y);
        }
        if constexpr (MODE == TC_EPI_STD) {
            if (ok) {
                v = add4(v, bias);
                if (ep.act == ACT_SILU) v = make_float4(silu(v.x), silu(v.y), silu(v.z), silu(v.w));
                else if (ep.act == ACT_GELU)
                    v = make_float4(gelu_erf(v.x), gelu_erf(v.y), gelu_erf(v.z), gelu_erf(v.w));
                if (ep.residual) v = add4(v, *reinterpret_cast<const float4*>(ep.residual + (size_t)m * ep.ldr + n));
                if (ep.kv_scatter) {
                    const size_t idx = kv_col + (size_t)(m + ep.frame_offset) * ep.head_dim;
                    if (ep.kv_out32) *reinterpret_cast<float4*>(ep.kv_out32 + idx) = v;
                    if (ep.kv_out16) st_f16x4(reinterpret_cast<__half*>(ep.kv_out16) + idx, v);
                } else {
                    if (ep.out) *reinterpret_cast<float4*>(ep.out + (size_t)m * ep.ldc + n) = v;
                    if (g.out_bf16) st_bf16x4_split(g.out_bf16 + (size_t)m * g.ldc_bf16 + n, v, g.bf16_lo_off);
                }
            }
        } else if constexpr (MODE == TC_EPI_ACCUM) {
            float4 nv = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ok) {
                float4* o = reinterpret_cast<float4*>(ep.out + (size_t)m * ep.ldc + n);
                nv = add4(res ? res[(r - r_lo) * TPR + (t % TPR)] : *o, add4(v, bias));
                *o = nv;
                if (g.out_bf16) st_bf16x4_split(g.out_bf16 + (size_t)m * g.ldc_bf16 + n, nv, g.bf16_lo_off);
            }
            if (g.stats_out) {  // (mean, M2) of the row's updated values over this tile's columns
                float sx = (nv.x + nv.y) + (nv.z + nv.w);
#pragma unroll
                for (int o = TPR / 2; o > 0; o >>= 1) sx += __shfl_xor_sync(FULL, sx, o);
                const float mean = sx / (float)min(BN, g.N - n0);
                float q = 0.f;
                if (ok) {
                    const float a = nv.x - mean, b = nv.y - mean, e = nv.z - mean, f = nv.w - mean;
                    q = (a * a + b * b) + (e * e + f * f);
                }
#pragma unroll
                for (int o = TPR / 2; o > 0; o >>= 1) q += __shfl_xor_sync(FULL, q, o);
                if ((t % TPR) == 0 && r < rows)
                    g.stats_out[(size_t)blockIdx.x * g.stats_ld + m] = make_float2(mean, q);
            }
        } else if constexpr (MODE == TC_EPI_SWIGLU) {
            if (ok) {  // columns (value, gate, value, gate) -> two outputs
                v = add4(v, bias);
                const float o0 = v.x * silu(v.y), o1 = v.z * silu(v.w);
                const __nv_bfloat162 o = __floats2bfloat162_rn(o0, o1);
                __nv_bfloat16* dst = g.out_bf16 + (size_t)m * g.ldc_bf16 + (n >> 1);
                *reinterpret_cast<__nv_bfloat162*>(dst) = o;
                if (g.bf16_lo_off)
                    *reinterpret_cast<__nv_bfloat162*>(dst + g.bf16_lo_off) =
                        __floats2bfloat162_rn(o0 - __low2float(o), o1 - __high2float(o));
            }
        } else if constexpr (MODE == TC_EPI_ROPE_KV) {
            if (ok) {
                const TcRopeKv& rp = g.rope;
                if (region < 2) {
                    const float x0 = v.x * cs0 - v.y * sn0, y0 = v.x * sn0 + v.y * cs0;
                    const float x1 = v.z * cs1 - v.w * sn1, y1 = v.z * sn1 + v.w * cs1;
                    v = make_float4(x0, y0, x1, y1);
                }
                if (region == 0) {
                    *reinterpret_cast<float4*>(rp.q + (size_t)m * rp.H * rp.hd + rdim) = v;
                } else {
                    const int KVD = rp.KVH * rp.hd;
                    const int j = (region - 1) * KVD + rdim;
                    *reinterpret_cast<float4*>(rp.kv_new + (size_t)m * 2 * KVD + j) = v;
                    const int head = rdim / rp.hd, dim = rdim - head * rp.hd;
                    const PagedKv& pk = rp.kv;
                    const int lp = t_pos / pk.page;
                    const int phys = lp < pk.table_stride ? pk.table[(size_t)m * pk.table_stride + lp] : -1;
                    if (phys >= 0) {  // rows past their own limit have no page here
                        const size_t idx = (size_t)phys * pk.page_elems + pk.layer_off +
                                           ((size_t)(region - 1) * rp.KVH + head) * pk.page * rp.hd +
                                           (size_t)(t_pos % pk.page) * rp.hd + dim;
                        if (pk.kv_f16) st_f16x4(reinterpret_cast<__half*>(pk.pool) + idx, v);
                        else *reinterpret_cast<float4*>(reinterpret_cast<float*>(pk.pool) + idx) = v;
                    }
                }
            }
        } else {  // TC_EPI_ARGMAX: the TPR threads of a row lie in one warp
            float best = -INFINITY;
            int bestn = 0x7fffffff;
            if (ok) {
                if (ep.out) *reinterpret_cast<float4*>(ep.out + (size_t)m * ep.ldc + n) = v;
                float4 k = v;
                if (g.inv_temp > 0.f) {  // temperature sampling: Gumbel-max keys
                    const unsigned st = (unsigned)(*g.step) + ((unsigned)m << 20);
                    k = make_float4(v.x * g.inv_temp + gumbel_noise(g.seed, st, (unsigned)n),
                                    v.y * g.inv_temp + gumbel_noise(g.seed, st, (unsigned)n + 1),
                                    v.z * g.inv_temp + gumbel_noise(g.seed, st, (unsigned)n + 2),
                                    v.w * g.inv_temp + gumbel_noise(g.seed, st, (unsigned)n + 3));
                }
                // increasing column order with strict > keeps the lowest index on ties
                if (k.x > best) { best = k.x; bestn = n; }
                if (k.y > best) { best = k.y; bestn = n + 1; }
                if (k.z > best) { best = k.z; bestn = n + 2; }
                if (k.w > best) { best = k.w; bestn = n + 3; }
            }
#pragma unroll
            for (int o = TPR / 2; o > 0; o >>= 1) {
                const float bo = __shfl_xor_sync(FULL, best, o);
                const int no = __shfl_xor_sync(FULL, bestn, o);
                if (bo > best || (bo == best && no < bestn)) {
                    best = bo;
                    bestn = no;
                }
            }
            if ((t % TPR) == 0 && r < rows && best > -INFINITY) atomicMax(g.argmax + m, argmax_key(best, bestn));
        }
    }
}

template <int BN, int MODE, bool SP>
__global__ void __launch_bounds__(TC_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
               const __grid_constant__ CUtensorMap tmap_a_lo, const __grid_constant__ CUtensorMap tmap_b_lo,
               TcGemmArgs g) {
    using Sm = TcSmem<BN, SP>;
    constexpr int STAGES = Sm::ST;
    extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
    Sm& s = *reinterpret_cast<Sm*>(
        (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    // this CTA's k-blocks: split blockIdx.z of g.splits
    const int nkb_all = g.taps * g.kb_per_tap;
    const int per_split = (nkb_all + g.splits - 1) / g.splits;
    const int kb_lo = blockIdx.z * per_split;
    const int nkb = max(0, min(nkb_all, kb_lo + per_split) - kb_lo);
    constexpr uint32_t A_BYTES = BM * BK * 2 * Sm::P, B_BYTES = BN * BK * 2 * Sm::P;
    __shared__ int s_fail;
    __shared__ float2 s_lnr[BM];  // folded LayerNorm: (mean, rstd) per tile row
    // ACCUM: this CTA's residual rows, read by the idle warps while the main loop runs
    constexpr int RES_F4 = 1024;
    __shared__ float4 s_res[MODE == TC_EPI_ACCUM ? RES_F4 : 1];
    const int S = (int)gridDim.z;
    const int rows = min(BM, g.M - m0);
    const int per_rows = (rows + S - 1) / S;  // epilogue rows of split z: [z per, (z + 1) per)
    const int r_lo = S == 1 ? 0 : min(rows, (int)blockIdx.z * per_rows);
    const int r_hi = S == 1 ? rows : min(rows, r_lo + per_rows);
    const bool res_ahead = MODE == TC_EPI_ACCUM && (r_hi - r_lo) * (BN / 4) <= RES_F4;

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

    // B (the weights) does not come from the previous kernel: the first stages' B tiles are
    // requested before waiting for it (programmatic dependent launch), A after
    const int pre = min(nkb, STAGES);
    if (warp == 0 && lane == 0)
        for (int kb = 0; kb < pre; ++kb) {
            const int gkb = kb_lo + kb;
            const int tap = gkb / g.kb_per_tap;
            const int k0 = (gkb - tap * g.kb_per_tap) * BK;
            mbar_expect_tx(&s.full[kb], A_BYTES + B_BYTES);
            tma_load_2d(s.b[kb][0], &tmap_b, &s.full[kb], tap * g.k_per_tap + k0, n0);
            if constexpr (SP) tma_load_2d(s.b[kb][1], &tmap_b_lo, &s.full[kb], tap * g.k_per_tap + k0, n0);
        }
    pdl_wait();
    pdl_trigger();

    int issued = 0;  // producer: k-blocks whose copies were issued
    if (warp == 0 && lane == 0) {
        for (int kb = 0; kb < nkb; ++kb) {
            const int st = kb % STAGES;
            if (kb >= STAGES && !mbar_wait(&s.empty[st], ((kb / STAGES) - 1) & 1)) {
                atomicCAS(g.status, 0u, (unsigned)DEV_WAIT_TIMEOUT);
                s_fail = 1;
                break;
            }
            const int gkb = kb_lo + kb;
            const int tap = gkb / g.kb_per_tap;
            const int k0 = (gkb - tap * g.kb_per_tap) * BK;
            if (kb >= pre) {
                mbar_expect_tx(&s.full[st], A_BYTES + B_BYTES);
                tma_load_2d(s.b[st][0], &tmap_b, &s.full[st], tap * g.k_per_tap + k0, n0);
                if constexpr (SP) tma_load_2d(s.b[st][1], &tmap_b_lo, &s.full[st], tap * g.k_per_tap + k0, n0);
            }
            tma_load_3d(s.a[st][0], &tmap_a, &s.full[st], k0, g.tap_y[tap], m0 + g.tap_z[tap]);
            if constexpr (SP) tma_load_3d(s.a[st][1], &tmap_a_lo, &s.full[st], k0, g.tap_y[tap], m0 + g.tap_z[tap]);
            issued = kb + 1;
        }
    } else if (warp == 1 && lane == 0) {
        const uint32_t idesc = idesc_bf16(BM, BN);
        for (int kb = 0; kb < nkb; ++kb) {
            const int st = kb % STAGES;
            if (!mbar_wait(&s.full[st], (kb / STAGES) & 1)) {
                atomicCAS(g.status, 0u, (unsigned)DEV_WAIT_TIMEOUT);
                s_fail = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a_addr = smem_u32(s.a[st][0]), b_addr = smem_u32(s.b[st][0]);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {  // 16 bf16 = 32 bytes per MMA along K
                mma_bf16(tmem, smem_desc_sw128(a_addr + k * 32), smem_desc_sw128(b_addr + k * 32), idesc,
                         (kb > 0 || k > 0) ? 1u : 0u);
                if constexpr (SP) {  // + hi.lo + lo.hi (lo.lo is below fp32 rounding of the sum)
                    const uint32_t al = smem_u32(s.a[st][Sm::P - 1]), bl = smem_u32(s.b[st][Sm::P - 1]);
                    mma_bf16(tmem, smem_desc_sw128(a_addr + k * 32), smem_desc_sw128(bl + k * 32), idesc, 1u);
                    mma_bf16(tmem, smem_desc_sw128(al + k * 32), smem_desc_sw128(b_addr + k * 32), idesc, 1u);
                }
            }
            mma_commit(&s.empty[st]);
        }
        if (nkb > 0) mma_commit(&s.done);
    } else if (warp >= 2 && res_ahead) {
        const GemmEpilogue& ep = g.ep;
        for (int e = threadIdx.x - 64; e < (r_hi - r_lo) * (BN / 4); e += 64) {
            const int r = r_lo + e / (BN / 4), n = n0 + (e % (BN / 4)) * 4;
            if (n < g.N) s_res[e] = *reinterpret_cast<const float4*>(ep.out + (size_t)(m0 + r) * ep.ldc + n);
        }
    } else if (warp >= 2 && MODE != TC_EPI_ACCUM && g.lnf.stats) {
        // folded LayerNorm: (mean, rstd) of every tile row from the producer's column-tile
        // statistics (final since pdl_wait), on the two warps the main loop leaves idle
        const TcLnFold& f = g.lnf;
        const int rows_here = min(BM, g.M - m0);
        for (int r = threadIdx.x - 64; r < rows_here; r += 64) {
            float na = 0.f, mean = 0.f, m2 = 0.f;
            for (int q = 0; q < f.ntiles; ++q) {
                const float2 st = f.stats[(size_t)q * f.ld + m0 + r];
                const float nb = (float)min(f.tile_n, f.K - q * f.tile_n);
                const float nn = na + nb, delta = st.x - mean;
                mean += delta * (nb / nn);
                m2 += st.y + delta * delta * (na * nb / nn);
                na = nn;
            }
            s_lnr[r] = make_float2(mean, rsqrtf(m2 / (float)f.K + 1e-5f));
        }
    }
    __syncwarp();
    __syncthreads();  // role loops finished; s_fail and s_lnr are final

    // epilogue: warp w owns accumulator lanes (rows) 32w .. 32w+31.  The tile goes through
    // shared memory (the idle stage buffers) so the global side is row-contiguous.
    bool ok = nkb > 0 && mbar_wait(&s.done, 0);  // an empty k-split stages zeros
    if (nkb > 0 && !ok) atomicCAS(g.status, 0u, (unsigned)DEV_WAIT_TIMEOUT);
    ok = __syncthreads_and(ok && !s_fail);      // uniform: the epilogue crosses warps
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    constexpr int LDS = tile_ld<BN>();
    float* tile = reinterpret_cast<float*>(&s.a[0][0][0]);
    static_assert(sizeof(float) * BM * LDS <= sizeof(s.a) + sizeof(s.b), "epilogue tile must fit the stages");
    if (warp * 32 < rows) {  // warp-uniform: lanes of rows past M hold nothing
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
        float* my = tile + (size_t)(warp * 32 + lane) * LDS;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
            float v[32];
            if (ok) tmem_ld32(lane_addr + c0, v);
            else
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = 0.f;
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(my + c0 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
    }
    __syncthreads();  // the whole tile is staged
    const float2* lnr = (MODE != TC_EPI_ACCUM && g.lnf.stats) ? s_lnr : nullptr;
    const float4* res = res_ahead ? s_res : nullptr;
    if (S == 1) {
        if (ok) epilogue_tile<BN, MODE>(g, tile, m0, n0, 0, rows, lnr, res, threadIdx.x);
    } else {
        // every split of the tile has staged its partial (barriers taken by all CTAs, also
        // after a failure, so none is left waiting)
        cluster_barrier();
        const int lo = r_lo, hi = r_hi;
        const bool any_fail = *reinterpret_cast<volatile unsigned*>(g.status) != 0u;
        if (!any_fail) {
            // rows [lo, hi): sum of the S partials in split order, into this CTA's own tile
            // (no other CTA reads these rows of it)
            constexpr int C4 = BN / 4;
            const uint32_t tile_a = smem_u32(tile);
            for (int e = threadIdx.x; e < (hi - lo) * C4; e += TC_THREADS) {
                const int r = lo + e / C4, c = (e % C4) * 4;
                const uint32_t off = (uint32_t)((r * LDS + c) * 4);
                // every split's value is requested before the first is added (the remote loads
                // overlap), then summed in split order
                float4 part[TC_MAX_SPLITS];
#pragma unroll
                for (int q = 0; q < TC_MAX_SPLITS; ++q)
                    if (q < S) part[q] = ld_dsmem4(mapa_rank(tile_a + off, (uint32_t)q));
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int q = 0; q < TC_MAX_SPLITS; ++q)
                    if (q < S) acc = add4(acc, part[q]);
                *reinterpret_cast<float4*>(tile + (size_t)r * LDS + c) = acc;
            }
        }
        cluster_barrier();  // every CTA has read the partials it needs from its peers
        if (!any_fail) epilogue_tile<BN, MODE>(g, tile, m0, n0, lo, hi, lnr, res, threadIdx.x);
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

// Persistent form for large GEMMs with the STD epilogue and no k-splits (the batched and
// streaming encoders): one CTA per SM walks the output tiles blockIdx.x, blockIdx.x +
// gridDim.x, ... (N fastest).  Six warps: warp 0 (one lane) the TMA producer and warp 1 (one
// lane) the MMA issuer run ahead across tiles, warps 2-5 the epilogue.  Two TMEM accumulators
// (2 BN columns) let the MMAs of tile i + 1 run while the epilogue drains tile i: tfull[a]
// (MMA commit) hands accumulator a to the epilogue, tempty[a] (one arrival per epilogue warp)
// hands it back.  The epilogue stages the accumulator in its own shared tile and runs
// epilogue_tile with its 128 threads.  Split operands take 2 ring stages, bf16 ones 4.
constexpr int TCP_THREADS = 192;
// Named barrier 1 of the four epilogue warps (128 threads); the _and form also returns
// whether every one of them passed `v`.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ bool epi_sync_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}
template <int BN, bool SP>
struct alignas(1024) TcPSmem {
    static constexpr int ST = SP ? 2 : 4;
    static constexpr int P = SP ? 2 : 1;
    __nv_bfloat16 a[ST][P][BM * BK];
    __nv_bfloat16 b[ST][P][BN * BK];
    float tile[BM * tile_ld<BN>()];
    uint64_t full[ST], empty[ST], tfull[2], tempty[2], done;
    uint32_t tmem_base;
};

template <int BN, bool SP>
__global__ void __launch_bounds__(TCP_THREADS, 1)
gemm_tc_persist_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                       const __grid_constant__ CUtensorMap tmap_a_lo, const __grid_constant__ CUtensorMap tmap_b_lo,
                       TcGemmArgs g) {
    using Sm = TcPSmem<BN, SP>;
    constexpr int STAGES = Sm::ST;
    extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
    Sm& s = *reinterpret_cast<Sm*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntn = (g.N + BN - 1) / BN, ntiles = ntn * ((g.M + BM - 1) / BM);
    const int nkb = g.taps * g.kb_per_tap;
    constexpr uint32_t A_BYTES = BM * BK * 2 * Sm::P, B_BYTES = BN * BK * 2 * Sm::P;
    __shared__ int s_fail;
    volatile int* failed = &s_fail;
    auto fail = [&]() {
        atomicCAS(g.status, 0u, (unsigned)DEV_WAIT_TIMEOUT);
        *failed = 1;
    };

    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s.tfull[i], 1);
            mbar_init(&s.tempty[i], 4);  // one arrival per epilogue warp
        }
        mbar_init(&s.done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {  // tensor memory: two accumulators of BN fp32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem_base)),
                     "r"((uint32_t)(2 * BN))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s.tmem_base;
    pdl_wait();
    pdl_trigger();

    int issued = 0;  // producer: k-blocks issued over all of this CTA's tiles
    if (warp == 0 && lane == 0) {
        for (int tile = blockIdx.x; tile < ntiles && !*failed; tile += gridDim.x) {
            const int m0 = (tile / ntn) * BM, n0 = (tile % ntn) * BN;
            for (int kb = 0; kb < nkb; ++kb, ++issued) {
                const int st = issued % STAGES;
                if (issued >= STAGES && !mbar_wait(&s.empty[st], ((issued / STAGES) - 1) & 1)) {
                    fail();
                    break;
                }
                const int tap = kb / g.kb_per_tap;
                const int k0 = (kb - tap * g.kb_per_tap) * BK;
                mbar_expect_tx(&s.full[st], A_BYTES + B_BYTES);
                tma_load_2d(s.b[st][0], &tmap_b, &s.full[st], tap * g.k_per_tap + k0, n0);
                tma_load_3d(s.a[st][0], &tmap_a, &s.full[st], k0, g.tap_y[tap], m0 + g.tap_z[tap]);
                if constexpr (SP) {
                    tma_load_2d(s.b[st][1], &tmap_b_lo, &s.full[st], tap * g.k_per_tap + k0, n0);
                    tma_load_3d(s.a[st][1], &tmap_a_lo, &s.full[st], k0, g.tap_y[tap], m0 + g.tap_z[tap]);
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        const uint32_t idesc = idesc_bf16(BM, BN);
        int used = 0, i = 0;  // k-blocks consumed, tiles started
        for (int tile = blockIdx.x; tile < ntiles && !*failed; tile += gridDim.x, ++i) {
            const int acc = i & 1;
            // the epilogue has drained this accumulator's previous tile
            if (i >= 2 && !mbar_wait(&s.tempty[acc], ((i >> 1) - 1) & 1)) {
                fail();
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t d = tmem + (uint32_t)(acc * BN);
            bool ok = true;
            for (int kb = 0; kb < nkb; ++kb, ++used) {
                const int st = used % STAGES;
                if (!mbar_wait(&s.full[st], (used / STAGES) & 1)) {
                    fail();
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t a_addr = smem_u32(s.a[st][0]), b_addr = smem_u32(s.b[st][0]);
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                    mma_bf16(d, smem_desc_sw128(a_addr + k * 32), smem_desc_sw128(b_addr + k * 32), idesc,
                             (kb > 0 || k > 0) ? 1u : 0u);
                    if constexpr (SP) {  // + hi.lo + lo.hi
                        const uint32_t al = smem_u32(s.a[st][Sm::P - 1]), bl = smem_u32(s.b[st][Sm::P - 1]);
                        mma_bf16(d, smem_desc_sw128(a_addr + k * 32), smem_desc_sw128(bl + k * 32), idesc, 1u);
                        mma_bf16(d, smem_desc_sw128(al + k * 32), smem_desc_sw128(b_addr + k * 32), idesc, 1u);
                    }
                }
                mma_commit(&s.empty[st]);
            }
            if (!ok) break;
            mma_commit(&s.tfull[acc]);
        }
        // every MMA issued here has finished before the tensor memory is freed
        mma_commit(&s.done);
        if (!mbar_wait(&s.done, 0)) fail();
    } else if (warp >= 2) {
        const int et = threadIdx.x - 64, q = warp & 3;  // warp q may read accumulator lanes 32q..32q+31
        constexpr int LDS = tile_ld<BN>();
        int i = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
            const int acc = i & 1;
            const bool ready = !*failed && mbar_wait(&s.tfull[acc], (i >> 1) & 1);
            if (!epi_sync_and(ready)) {  // uniform over the four epilogue warps
                fail();
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int m0 = (tile / ntn) * BM, n0 = (tile % ntn) * BN;
            const int rows = min(BM, g.M - m0);
            if (q * 32 < rows) {  // warp-uniform: lanes of rows past M hold nothing
                const uint32_t lane_addr = tmem + (uint32_t)(acc * BN) + ((uint32_t)(q * 32) << 16);
                float* my = s.tile + (size_t)(q * 32 + lane) * LDS;
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    float v[32];
                    tmem_ld32(lane_addr + c0, v);
#pragma unroll
                    for (int k = 0; k < 32; k += 4)
                        *reinterpret_cast<float4*>(my + c0 + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.tempty[acc]);  // the accumulator takes tile i + 2
            epi_sync();                                   // the tile is staged
            epilogue_tile<BN, TC_EPI_STD>(g, s.tile, m0, n0, 0, rows, nullptr, nullptr, et);
            epi_sync();  // consumed before the next tile is staged
        }
    }
    __syncwarp();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    // drain copies still in flight after a failure (bounded), then free tensor memory (the MMA
    // issuer waited for its last MMA)
    if (warp == 0 && lane == 0 && *failed)
        for (int it = (issued > STAGES ? issued - STAGES : 0); it < issued; ++it)
            mbar_wait(&s.full[it % STAGES], (it / STAGES) & 1);
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(2 * BN))
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

namespace {
bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

template <int BN, int MODE, bool SP>
cudaError_t launch_tc(const CUtensorMap& map_a, const CUtensorMap& map_b, const CUtensorMap& map_a_lo,
                      const CUtensorMap& map_b_lo, const TcGemmArgs& g, cudaStream_t stream) {
    const size_t smem = sizeof(TcSmem<BN, SP>) + 1024;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, MODE, SP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const dim3 grid((g.N + BN - 1) / BN, (g.M + BM - 1) / BM, g.splits);
    if (g.splits > 1)
        return launch_kernel_cluster_z(gemm_tc_kernel<BN, MODE, SP>, grid, dim3(TC_THREADS), smem, stream, g.splits,
                                       map_a, map_b, map_a_lo, map_b_lo, g);
    return launch_kernel(gemm_tc_kernel<BN, MODE, SP>, grid, dim3(TC_THREADS), smem, stream, map_a, map_b, map_a_lo,
                         map_b_lo, g);
}

int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            n = 1;
    }
    return n;
}

// The persistent form: one CTA per SM (its shared memory allows no second one).
template <int BN, bool SP>
cudaError_t launch_tc_persist(const CUtensorMap& map_a, const CUtensorMap& map_b, const CUtensorMap& map_a_lo,
                              const CUtensorMap& map_b_lo, const TcGemmArgs& g, cudaStream_t stream, int ntiles) {
    const size_t smem = sizeof(TcPSmem<BN, SP>) + 1024;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemm_tc_persist_kernel<BN, SP>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    return launch_kernel(gemm_tc_persist_kernel<BN, SP>, dim3(std::min(ntiles, num_sms())), dim3(TCP_THREADS), smem,
                         stream, map_a, map_b, map_a_lo, map_b_lo, g);
}

template <int BN, bool SP>
cudaError_t launch_tc_mode(const CUtensorMap& map_a, const CUtensorMap& map_b, const CUtensorMap& map_a_lo,
                           const CUtensorMap& map_b_lo, const TcGemmArgs& g, cudaStream_t stream) {
    const int ntiles = ((g.N + BN - 1) / BN) * ((g.M + BM - 1) / BM);
    switch (g.mode) {
        case TC_EPI_STD:
            // more tiles than SMs: the persistent form overlaps each tile's epilogue with the
            // next tile's loads and MMAs (its epilogue has no folded LayerNorm)
            if (g.splits == 1 && ntiles > num_sms() && !g.lnf.stats)
                return launch_tc_persist<BN, SP>(map_a, map_b, map_a_lo, map_b_lo, g, stream, ntiles);
            return launch_tc<BN, TC_EPI_STD, SP>(map_a, map_b, map_a_lo, map_b_lo, g, stream);
        case TC_EPI_ROPE_KV: return launch_tc<BN, TC_EPI_ROPE_KV, SP>(map_a, map_b, map_a_lo, map_b_lo, g, stream);
        case TC_EPI_SWIGLU: return launch_tc<BN, TC_EPI_SWIGLU, SP>(map_a, map_b, map_a_lo, map_b_lo, g, stream);
        case TC_EPI_ARGMAX: return launch_tc<BN, TC_EPI_ARGMAX, SP>(map_a, map_b, map_a_lo, map_b_lo, g, stream);
        case TC_EPI_ACCUM: return launch_tc<BN, TC_EPI_ACCUM, SP>(map_a, map_b, map_a_lo, map_b_lo, g, stream);
        default: return cudaErrorInvalidValue;
    }
}

// The epilogue moves four columns per thread with 128-bit (fp32) / 64-bit (bf16, fp16)
// accesses: every output it touches must allow that.  A folded LayerNorm needs statistics
// tiles that cover exactly its K inputs and a row sum per column.
bool epilogue_layout_ok(const TcGemmArgs& g) {
    const GemmEpilogue& ep = g.ep;
    if (g.N % 4) return false;
    if (g.stats_out && g.mode != TC_EPI_ACCUM) return false;
    if (g.lnf.stats) {
        const TcLnFold& f = g.lnf;
        if (!f.csum || !aligned(f.csum, 16) || f.tile_n <= 0 || f.ntiles <= 0 || f.ld < g.M || f.K <= 0 ||
            (f.ntiles - 1) * f.tile_n >= f.K || f.ntiles * f.tile_n < f.K)
            return false;
    }
    switch (g.mode) {
        case TC_EPI_STD:
            if (ep.bias && !aligned(ep.bias, 16)) return false;
            if (ep.residual && (ep.ldr % 4 || !aligned(ep.residual, 16))) return false;
            if (ep.kv_scatter)
                return ep.head_dim % 4 == 0 && (!ep.kv_out32 || aligned(ep.kv_out32, 16)) &&
                       (!ep.kv_out16 || aligned(ep.kv_out16, 8));
            if (ep.out && (ep.ldc % 4 || !aligned(ep.out, 16))) return false;
            if (g.out_bf16 && (g.ldc_bf16 % 4 || !aligned(g.out_bf16, 8))) return false;
            return true;
        case TC_EPI_ACCUM:
            if (g.lnf.stats) return false;
            if (g.stats_out && g.stats_ld < g.M) return false;
            if (g.out_bf16 && (g.ldc_bf16 % 4 || !aligned(g.out_bf16, 8))) return false;
            return ep.out && ep.ldc % 4 == 0 && aligned(ep.out, 16) && (!ep.bias || aligned(ep.bias, 16));
        case TC_EPI_SWIGLU:
            return g.out_bf16 && g.ldc_bf16 % 2 == 0 && aligned(g.out_bf16, 4) && (!ep.bias || aligned(ep.bias, 16));
        case TC_EPI_ROPE_KV: {
            const TcRopeKv& r = g.rope;
            return r.hd % 4 == 0 && aligned(r.q, 16) && aligned(r.kv_new, 16) && r.kv.table && r.kv.page > 0 &&
                   aligned(r.kv.pool, 16) && r.kv.page_elems % 4 == 0 && r.kv.layer_off % 4 == 0 &&
                   g.N == (r.H + 2 * r.KVH) * r.hd;
        }
        case TC_EPI_ARGMAX:
            return g.argmax && (!ep.out || (ep.ldc % 4 == 0 && aligned(ep.out, 16))) && (g.inv_temp <= 0.f || g.step);
        default:
            return false;
    }
}
}  // namespace

cudaError_t launch_gemm_tc_split(const CUtensorMap& map_a, const CUtensorMap* map_a_lo, const CUtensorMap& map_b,
                                 const CUtensorMap* map_b_lo, const TcGemmArgs& g, int bn, cudaStream_t stream) {
    if (g.M <= 0 || g.N <= 0) return cudaSuccess;
    if (g.taps < 1 || g.taps > 8 || g.kb_per_tap < 1 || !g.status) return cudaErrorInvalidValue;
    if (g.splits < 1 || g.splits > TC_MAX_SPLITS || g.splits > g.taps * g.kb_per_tap) return cudaErrorInvalidValue;
    if ((map_a_lo == nullptr) != (map_b_lo == nullptr)) return cudaErrorInvalidValue;
    if (!epilogue_layout_ok(g) || (g.bf16_lo_off % 4)) return cudaErrorInvalidValue;
    ++launch_counter();
    if (map_a_lo) {
        if (bn == 128) return launch_tc_mode<128, true>(map_a, map_b, *map_a_lo, *map_b_lo, g, stream);
        if (bn == 64) return launch_tc_mode<64, true>(map_a, map_b, *map_a_lo, *map_b_lo, g, stream);
        return cudaErrorInvalidValue;
    }
    if (bn == 128) return launch_tc_mode<128, false>(map_a, map_b, map_a, map_b, g, stream);
    if (bn == 64) return launch_tc_mode<64, false>(map_a, map_b, map_a, map_b, g, stream);
    return cudaErrorInvalidValue;
}

cudaError_t launch_gemm_tc(const CUtensorMap& map_a, const CUtensorMap& map_b, const TcGemmArgs& g, int bn,
                           cudaStream_t stream) {
    return launch_gemm_tc_split(map_a, nullptr, map_b, nullptr, g, bn, stream);
}

}  // namespace msb
