// Device helpers of the clustered batch-1 decode kernel (decode_cluster.cu): distributed
// shared memory, the hardware cluster barrier, tagged exchange words, the block GEMV, the
// cross-attention key pass over shared-memory K/V blocks and the row layout of the packed
// per-CTA weight streams.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace msb {
namespace {

constexpr int NW = 8;         // warps per CTA
constexpr int NT = NW * 32;   // threads per CTA

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_index() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t mapa_rank(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_dsmem(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_dsmem_i(uint32_t addr, int v) {
    asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
// 16-byte aligned address
__device__ __forceinline__ float4 ld_dsmem4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
// 64-bit exchange words: (tag << 32) | payload.  One aligned 8-byte access is single-copy
// atomic, so a reader that sees the expected tag also sees its payload; no fence is needed.
__device__ __forceinline__ void st_tagged(unsigned long long* p, unsigned tag, uint32_t payload) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(((unsigned long long)tag << 32) | payload)
                 : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cp16(void* s, const void* g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(s)), "l"(g) : "memory");
}

// GEMV rows of the packed streams are stored rf + 4 floats apart (rf % 8 == 0): an odd
// number of 16-byte units, so lanes that own consecutive rows read distinct bank groups.
__host__ __device__ inline int row_stride(int rf) { return rf + 4; }

// res[i] = rows[i][0 : rf) . vec for i < nr (nr <= 64, row i at rows + i * rs).  Long rows
// split their columns over warps 1-7 with lanes owning rows (rs / 4 odd, so the eight lanes
// of one 128-bit phase read eight different bank groups) and a per-row sum of the warp
// partials in fixed order; warp 0, whose lane 0 issues the ring's bulk copies right before,
// takes no columns.  Short rows take one thread each.  Ends with a barrier.
__device__ __noinline__ void block_gemv(const float* rows, int nr, int rf, int rs, const float* vec, float* part,
                                        float* res) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int c4 = rf >> 2;
    const float4* v4 = reinterpret_cast<const float4*>(vec);
    if (c4 >= 4 * NW) {
        constexpr int W0 = 1;  // first column warp
        constexpr int NWK = NW - W0;
        const int per = (c4 + NWK - 1) / NWK;
        const int k0 = (w - W0) * per, k1 = w < W0 ? k0 : min(c4, k0 + per);
        for (int i = lane; i < nr && w >= W0; i += 32) {
            const float4* row = reinterpret_cast<const float4*>(rows + (size_t)i * rs);
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
            int k = k0;
#pragma unroll 2
            for (; k + 1 < k1; k += 2) {
                const float4 x = row[k], y = row[k + 1], u = v4[k], v = v4[k + 1];
                a0 = fmaf(x.x, u.x, a0);
                a1 = fmaf(x.y, u.y, a1);
                a2 = fmaf(x.z, u.z, a2);
                a3 = fmaf(x.w, u.w, a3);
                a0 = fmaf(y.x, v.x, a0);
                a1 = fmaf(y.y, v.y, a1);
                a2 = fmaf(y.z, v.z, a2);
                a3 = fmaf(y.w, v.w, a3);
            }
            if (k < k1) {
                const float4 x = row[k], u = v4[k];
                a0 = fmaf(x.x, u.x, a0);
                a1 = fmaf(x.y, u.y, a1);
                a2 = fmaf(x.z, u.z, a2);
                a3 = fmaf(x.w, u.w, a3);
            }
            part[(w - W0) * 64 + i] = (a0 + a1) + (a2 + a3);
        }
        __syncthreads();
        for (int i = tid - 32 * W0; i < nr && i >= 0; i += NT - 32 * W0) {
            float sum = 0.f;
#pragma unroll
            for (int q = 0; q < NWK; ++q) sum += part[q * 64 + i];
            res[i] = sum;
        }
    } else {
        for (int i = tid; i < nr; i += NT) {
            const float4* row = reinterpret_cast<const float4*>(rows + (size_t)i * rs);
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
            for (int k = 0; k < c4; ++k) {
                const float4 x = row[k], u = v4[k];
                a0 = fmaf(x.x, u.x, a0);
                a1 = fmaf(x.y, u.y, a1);
                a2 = fmaf(x.z, u.z, a2);
                a3 = fmaf(x.w, u.w, a3);
            }
            res[i] = (a0 + a1) + (a2 + a3);
        }
    }
    __syncthreads();
}

// Dot product of one word of BITS-bit codes (lowest bits first) with its 32 / BITS inputs.
// A code field is turned into a float without a conversion instruction: OR-ing it into the
// mantissa of 2^23 and subtracting 2^23 gives field * 2^s exactly, s being the field's bit
// offset inside its 16-bit half of the word; x holds the inputs pre-scaled by 2^-s, so each
// product equals code * input exactly before the fused add.
template <int BITS>
__device__ __forceinline__ float dot_code_word(uint32_t wd, const float4* x4) {
    constexpr int PER = 32 / BITS;
    const uint32_t hi = wd >> 16;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int q = 0; q < PER / 4; ++q) {
        const float4 t = x4[q];
        const float xv[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int o = (4 * q + e) * BITS;
            const uint32_t src = o < 16 ? wd : hi;
            const uint32_t m = ((1u << BITS) - 1u) << (o & 15);
            const float f = __uint_as_float((src & m) | 0x4B000000u) - 8388608.f;
            if (e & 1) a1 = fmaf(f, xv[e], a1);
            else a0 = fmaf(f, xv[e], a0);
        }
    }
    return a0 + a1;
}

// Scale of input j of a row of BITS-bit codes in the pre-scaled vector block_gemv_q reads
// (2^-s, s = the bit offset of j's code field inside its 16-bit half word; exact).
__device__ __forceinline__ float quant_input_scale(int j, int bits) {
    const int sh = ((j % (32 / bits)) * bits) & 15;
    return __uint_as_float((uint32_t)(127 - sh) << 23);
}

// Input k (value v) of the vector block_gemv_q reads, for rows of rf inputs (rf % 64 == 0):
// xq[k] = v * quant_input_scale(k), and lane 16m of the warp stores xq[rf + k / 16] = the
// sum of the 16 inputs its half warp holds.  Called by whole warps holding 32 consecutive
// inputs (k = 32 w + lane).
template <int BITS>
__device__ __forceinline__ void quant_input(float v, int k, float* xq, int rf) {
    xq[k] = v * quant_input_scale(k, BITS);
    float t = v + __shfl_xor_sync(0xffffffffu, v, 8);
    t += __shfl_xor_sync(0xffffffffu, t, 4);
    t += __shfl_xor_sync(0xffffffffu, t, 2);
    t += __shfl_xor_sync(0xffffffffu, t, 1);
    if ((threadIdx.x & 15) == 0) xq[rf + (k >> 4)] = t;
}

// res[i] = W[i] . vec for a block of nr <= NT affine-quantized rows of rf inputs (the MLX
// layout w = scale * q + bias per group of gs inputs).  Row i is a record at rows + i * rs
// words: rf * BITS / 32 code words, then (scale, bias) float pairs per group.  The sum is
// taken as sum over 16-byte code chunks k of scale_g * (q . vec)_k + bias_g * (sum of vec)_k.
// The vector comes prepared (by the LayerNorm that produced it): xq[j] = vec[j] *
// quant_input_scale(j), then at xq + rf the sums of vec over each 16 inputs.  Lanes own
// rows; the eight warps split into 8 / T' row groups of 32 (T' = the number of 32-row groups
// rounded up to a power of two) and each group's warps take the chunks round robin, their
// partials summed per row in fixed order.  Ends with a barrier.
template <int BITS>
__device__ __noinline__ void block_gemv_q(const uint32_t* rows, int nr, int rf, int rs, int gs, const float* xq,
                                          float* part, float* res) {
    constexpr int PER = 32 / BITS;  // codes per word
    constexpr int CC = 4 * PER;     // inputs per 16-byte chunk of codes
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int nch = rf / CC;
    const float* x16 = xq + rf;
    const int T = (nr + 31) >> 5;
    const int Tp = T <= 1 ? 1 : T <= 2 ? 2 : T <= 4 ? 4 : 8;
    const int S = NW / Tp;  // warps per 32-row group
    const int rg = w / S, sp = w - rg * S;
    const int i = rg * 32 + lane;
    float acc = 0.f;
    if (i < nr) {
        const uint32_t* row = rows + (size_t)i * rs;
        const float2* sb = reinterpret_cast<const float2*>(row + rf / PER);
        for (int k = sp; k < nch; k += S) {
            const uint4 cw = *reinterpret_cast<const uint4*>(row + 4 * k);
            const float4* x4 = reinterpret_cast<const float4*>(xq + k * CC);
            float a0 = dot_code_word<BITS>(cw.x, x4);
            float a1 = dot_code_word<BITS>(cw.y, x4 + PER / 4);
            a0 += dot_code_word<BITS>(cw.z, x4 + 2 * (PER / 4));
            a1 += dot_code_word<BITS>(cw.w, x4 + 3 * (PER / 4));
            float xs = x16[k * (CC / 16)];
#pragma unroll
            for (int t = 1; t < CC / 16; ++t) xs += x16[k * (CC / 16) + t];
            const float2 g = sb[(k * CC) / gs];
            acc = fmaf(g.x, a0 + a1, fmaf(g.y, xs, acc));
        }
    }
    if (S == 1) {
        if (i < nr) res[i] = acc;
    } else {
        part[sp * (32 * Tp) + i] = acc;
        __syncthreads();
        for (int q = tid; q < nr; q += NT) {
            float v = 0.f;
            for (int t = 0; t < S; ++t) v += part[t * (32 * Tp) + q];
            res[q] = v;
        }
    }
    __syncthreads();
}

// Cross-attention key scoring layout (as the batched streaming kernel): G lanes per key,
// 16 bytes of the key row per lane.
template <int HDT, bool F16>
struct KeyShape {
    static constexpr int ESZ = F16 ? 2 : 4;
    static constexpr int NE = HDT * ESZ / 16;
    static constexpr int EP = 16 / ESZ;
    static constexpr int G = NE <= 4 ? 4 : (NE <= 8 ? 8 : 16);
    static constexpr int KPP = 32 / G;
};

// One warp's pass over keys [k0, k1) of a shared-memory K/V block (rows of HDT elements):
// scores with the grouped-lane layout, online softmax into (m, l), V accumulation into
// (a0, a1) = dims (2 lane, 2 lane + 1).  `qr` is this lane's q slice, `sc` 32 floats.
struct QSlice {
    float v[8];
};

template <int HDT, bool F16>
__device__ __noinline__ float4 attend_keys(const void* kblk, const void* vblk, int k0, int k1, QSlice q,
                                           float scale, float* sc, float4 st, int lane) {
    const float* qr = q.v;
    float m = st.x, l = st.y, a0 = st.z, a1 = st.w;
    using S = KeyShape<HDT, F16>;
    using E = typename std::conditional<F16, __half, float>::type;
    const E* kb = reinterpret_cast<const E*>(kblk);
    const E* vb = reinterpret_cast<const E*>(vblk);
    const int g = lane / S::G, sub = lane - (lane / S::G) * S::G;
    for (int c0 = k0; c0 < k1; c0 += 32) {
        const int nk = min(32, k1 - c0);
        for (int p = 0; p < 32 / S::KPP; ++p) {
            const int j = p * S::KPP + g;
            if (p * S::KPP >= nk) break;  // warp-uniform
            float dot = 0.f;
            if (j < nk && sub < S::NE) {
                const uint4 u = *reinterpret_cast<const uint4*>(kb + (size_t)(c0 + j) * HDT + sub * S::EP);
                if constexpr (F16) {
                    const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const float2 f = __half22float2(h2[t]);
                        dot = fmaf(qr[2 * t], f.x, fmaf(qr[2 * t + 1], f.y, dot));
                    }
                } else {
                    const float* f = reinterpret_cast<const float*>(&u);
#pragma unroll
                    for (int t = 0; t < 4; ++t) dot = fmaf(qr[t], f[t], dot);
                }
            }
#pragma unroll
            for (int o = S::G / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(FULL, dot, o);
            if (sub == 0) sc[j] = (j < nk) ? dot * scale : -INFINITY;
        }
        __syncwarp();
        const float sv = lane < nk ? sc[lane] : -INFINITY;
        const float mn = fmaxf(m, warp_max(sv));
        const float pv = (sv == -INFINITY) ? 0.f : expf(sv - mn);
        const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
        l = l * corr + warp_sum(pv);
        a0 *= corr;
        a1 *= corr;
        __syncwarp();
        sc[lane] = pv;
        __syncwarp();
        if (2 * lane < HDT) {
#pragma unroll 4
            for (int j = 0; j < nk; ++j) {
                const float pj = sc[j];
                float2 v;
                if constexpr (F16) v = __half22float2(*reinterpret_cast<const __half2*>(vb + (size_t)(c0 + j) * HDT + 2 * lane));
                else v = *reinterpret_cast<const float2*>(vb + (size_t)(c0 + j) * HDT + 2 * lane);
                a0 = fmaf(pj, v.x, a0);
                a1 = fmaf(pj, v.y, a1);
            }
        }
        __syncwarp();
        m = mn;
    }
    return make_float4(m, l, a0, a1);
}


// Rows of the next block of a segment (header + rows of rf floats, at most maxr rows, split
// at whole multiples of `gran` rows, the header only in the first block), or -1 when the
// segment is exhausted.
__host__ __device__ inline int next_block_rows(int hdr, int nrows, int rf, int gran, int slot_floats, int row0,
                                               bool first, int maxr) {
    if (!(first && hdr > 0) && row0 >= nrows) return -1;
    const int cap = slot_floats - (first ? hdr : 0);
    const int per = max(gran, min(maxr, cap / rf) / gran * gran);
    return min(nrows - row0, per);
}

struct BlockEnt {
    const void* s0;
    const void* s1;
    uint32_t b0, b1;
};

}  // namespace
}  // namespace msb
