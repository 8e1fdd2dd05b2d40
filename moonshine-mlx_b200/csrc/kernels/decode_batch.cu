// Batched greedy decode (B independent utterances in lockstep): the non-GEMM kernels of one
// decoder step.  The projections run on the tcgen05 GEMM (gemm_tc.cu) with bf16 weights
// and bf16 activations at the GEMM inputs; the residual stream, attention and softmax stay
// in fp32.  Row b of every [B, ...] buffer is utterance b.
//
//   embed_rows          x[b] = embed[next_id[b]], its bf16 planes and row statistics (the
//                       LayerNorms are folded into the GEMMs that consume them)
//   ln_bf16             LayerNorm (no bias, eps 1e-5) of fp32 rows -> bf16 GEMM input (encoder)
//   self_attn_batch     one 4-warp CTA per (b, head): keys 0..t in rounds staged in shared
//                       memory from b's pages (fp16|fp32), this step's fp32 K/V at t
//                       (MoonshineLayers.swift:106-125)
//   cross_attn_stream   one CTA per (b, head): bulk-copy ring of K/V chunks of utterance b's
//                       own frames through shared memory, online softmax -> bf16 rows
//   cross_attn_batch    generic head_dim: (b, head, 32-key chunk) partials over b's frames
//   cross_combine       merge the chunk partials -> bf16 attention rows
//   step_finalize       per-row argmax -> ids, EOS / limit bookkeeping, next ids, t + 1
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace msb {

namespace {

constexpr int CHB = 32;
constexpr int SA_WARPS = 4;  // batched self attention: warps per (row, head), key chunks interleaved
constexpr int MAXHD_B = 64;

// Sum over the block (128 threads) in a fixed order; every thread gets the total.
__device__ __forceinline__ float block_sum128(float v, float* red) {
    v = warp_sum(v);
    __syncthreads();  // red is free (earlier readers are done)
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    return (red[0] + red[1]) + (red[2] + red[3]);
}

__global__ void __launch_bounds__(128) embed_rows_kernel(const int* __restrict__ ids, const float* __restrict__ embed,
                                                         int d, int B, int V, float* __restrict__ x, unsigned* status,
                                                         __nv_bfloat16* __restrict__ xb, size_t lo_off,
                                                         float2* __restrict__ stats, int stats_ld, int tile_n) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[4];
    const int b = blockIdx.x;
    if (b >= B) return;
    int id = ids[b];
    if (id < 0 || id >= V) {
        if (threadIdx.x == 0) atomicCAS(status, 0u, (unsigned)DEV_BAD_TOKEN);
        id = 0;
    }
    const float* e = embed + (size_t)id * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float v = e[i];
        x[(size_t)b * d + i] = v;
        if (xb) st_bf16_split(xb + (size_t)b * d + i, v, lo_off);
    }
    if (stats) {  // (mean, M2) per column tile, two passes (block-uniform loop)
        for (int t0 = 0; t0 < d; t0 += tile_n) {
            const int nc = min(tile_n, d - t0);
            float s = 0.f;
            for (int i = threadIdx.x; i < nc; i += blockDim.x) s += e[t0 + i];
            const float mean = block_sum128(s, red) / (float)nc;
            float q = 0.f;
            for (int i = threadIdx.x; i < nc; i += blockDim.x) {
                const float a = e[t0 + i] - mean;
                q += a * a;
            }
            q = block_sum128(q, red);
            if (threadIdx.x == 0) stats[(size_t)(t0 / tile_n) * stats_ld + b] = make_float2(mean, q);
        }
    }
}

__global__ void ln_bf16_kernel(const float* __restrict__ x, int rows, int d, const float* __restrict__ w,
                               float w_offset, __nv_bfloat16* __restrict__ out, size_t lo_off) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[32];
    const int r = blockIdx.x;
    if (r >= rows) return;
    const float* xr = x + (size_t)r * d;
    float s = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) s += xr[i];
    const float mean = block_sum(s, red) / (float)d;
    float q = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float c = xr[i] - mean;
        q += c * c;
    }
    const float rstd = rsqrtf(block_sum(q, red) / (float)d + 1e-5f);
    for (int i = threadIdx.x; i < d; i += blockDim.x)
        st_bf16_split(out + (size_t)r * d + i, (xr[i] - mean) * rstd * (w[i] + w_offset), lo_off);
}

// The same LayerNorm with one warp per row for d % 4 == 0, d <= 32 * 4 * LNW_V4: the row
// stays in registers (LNW_V4 float4 per lane) across the mean, variance and output passes,
// reductions are warp shuffles only, LNW_ROWS rows per CTA.  x and w 16-byte aligned, out
// 8-byte aligned.
constexpr int LNW_ROWS = 8;
constexpr int LNW_V4 = 8;
__global__ void __launch_bounds__(LNW_ROWS * 32) ln_bf16_warp_kernel(const float* __restrict__ x, int rows, int d,
                                                                     const float* __restrict__ w, float w_offset,
                                                                     __nv_bfloat16* __restrict__ out, size_t lo_off) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * LNW_ROWS + (threadIdx.x >> 5);
    if (r >= rows) return;  // whole warps
    const int n4 = d >> 2;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)r * d);
    float4 v[LNW_V4];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < LNW_V4; ++j) {
        const int i = lane + 32 * j;
        v[j] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
    const float mean = warp_sum(s) / (float)d;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < LNW_V4; ++j)
        if (lane + 32 * j < n4) {
            const float a = v[j].x - mean, b = v[j].y - mean, c = v[j].z - mean, e = v[j].w - mean;
            q += (a * a + b * b) + (c * c + e * e);
        }
    const float rstd = rsqrtf(warp_sum(q) / (float)d + 1e-5f);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(out + (size_t)r * d);
#pragma unroll
    for (int j = 0; j < LNW_V4; ++j) {
        const int i = lane + 32 * j;
        if (i < n4) {
            const float4 g = w4[i];
            const float y0 = (v[j].x - mean) * rstd * (g.x + w_offset), y1 = (v[j].y - mean) * rstd * (g.y + w_offset);
            const float y2 = (v[j].z - mean) * rstd * (g.z + w_offset), y3 = (v[j].w - mean) * rstd * (g.w + w_offset);
            const __nv_bfloat162 lo = __floats2bfloat162_rn(y0, y1);
            const __nv_bfloat162 hi = __floats2bfloat162_rn(y2, y3);
            uint2 pk;
            pk.x = *reinterpret_cast<const uint32_t*>(&lo);
            pk.y = *reinterpret_cast<const uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(o2 + 2 * i) = pk;
            if (lo_off) {  // remainders: the low plane of a split operand
                const __nv_bfloat162 rl = __floats2bfloat162_rn(y0 - __low2float(lo), y1 - __high2float(lo));
                const __nv_bfloat162 rh = __floats2bfloat162_rn(y2 - __low2float(hi), y3 - __high2float(hi));
                pk.x = *reinterpret_cast<const uint32_t*>(&rl);
                pk.y = *reinterpret_cast<const uint32_t*>(&rh);
                *reinterpret_cast<uint2*>(o2 + 2 * i + lo_off / 2) = pk;
            }
        }
    }
}

__device__ __forceinline__ float load_kv(const void* base, size_t idx, int f16) {
    return f16 ? __half2float(reinterpret_cast<const __half*>(base)[idx]) : reinterpret_cast<const float*>(base)[idx];
}

// One CTA of W warps per (b, h) (SA_WARPS; one warp when a round of 32 keys covers the
// whole call).  Keys come in rounds of `keys` (at most SaShape::KEYS,
// fewer when the call's positions are fewer, which shrinks the shared memory and so raises
// the CTAs resident per SM): every thread
// first copies its share of the round's cached K and V rows (from row b's pages; a key
// without a page -- a row past its own limit -- is skipped) into shared memory with 16-byte
// cp.async, so a round costs one memory round trip; then warp w scores keys
// [w kw, (w + 1) kw) of the round, kw = keys / W (lanes own keys, rows read in
// 16-byte pieces against q staged in shared memory), keeps an online softmax and accumulates
// V with lane c owning dims (2c, 2c+1).  Key t is this step's fp32 K/V.  The warp states are merged in warp order.
template <bool F16>
struct SaShape {
    static constexpr int ESZ = F16 ? 2 : 4;
    static constexpr int KEYS = F16 ? 128 : 64;  // most keys per round (<= 32 per warp)
};
// shared-memory row of hd elements: an odd number of 16-byte pieces, so the eight lanes of
// one 128-bit phase reading eight different rows hit different bank groups
__host__ __device__ constexpr int sa_row_pieces(int hd, int esz) { return ((hd * esz) / 16) | 1; }
// shared memory of a round of `keys` K and V rows of hd elements
template <bool F16>
constexpr size_t sa_smem_bytes(int keys, int hd) {
    return (size_t)2 * keys * sa_row_pieces(hd, SaShape<F16>::ESZ) * 16;
}

template <bool F16, int KEYS, int W>
__global__ void __launch_bounds__(W * 32) self_attn_batch_kernel(
    const float* __restrict__ q, const float* __restrict__ kv_new, const PagedKv kv, const int* __restrict__ pos,
    int B, int H, int KVH, int hd, float scale, __nv_bfloat16* __restrict__ out, size_t lo_off) {
    using S = SaShape<F16>;
    static_assert(KEYS % W == 0 && KEYS / W <= 32 && KEYS <= S::KEYS, "round of whole warp slices");
    constexpr int keys = KEYS, kw = KEYS / W;  // keys per round, per warp per round
    using E = typename std::conditional<F16, __half, float>::type;
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) unsigned char sa_raw[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int item = blockIdx.x;
    if (item >= B * H) return;  // whole CTA
    const int b = item / H, h = item - b * H;
    const int kvh = h / (H / KVH);
    const int t = *pos;
    const int HD = H * hd, KVD = KVH * hd;
    const float* qr = q + (size_t)b * HD + h * hd;
    const float* fk = kv_new + (size_t)b * 2 * KVD + kvh * hd;
    const float* fv = fk + KVD;
    // element offsets of this (layer, head)'s K and V inside a page
    const size_t koff = (size_t)kv.layer_off + (size_t)kvh * kv.page * hd;
    const size_t voff = koff + (size_t)KVH * kv.page * hd;
    const int* tab = kv.table + (size_t)b * kv.table_stride;
    const E* pool = reinterpret_cast<const E*>(kv.pool);
    const int npc = hd * S::ESZ / 16;                 // 16-byte pieces per row
    const int rse = sa_row_pieces(hd, S::ESZ) * 16 / S::ESZ;  // shared row stride (elements)
    E* ks = reinterpret_cast<E*>(sa_raw);
    E* vs = ks + (size_t)keys * rse;
    // this head's q, staged once and read back as broadcast float4s
    __shared__ __align__(16) float qw[MAXHD_B];
    __shared__ float wm[W], wl[W];
    __shared__ float wacc[W][MAXHD_B];
    for (int c = threadIdx.x; c < hd; c += blockDim.x) qw[c] = qr[c];
    const float4* q4 = reinterpret_cast<const float4*>(qw);
    // pool element offset of cached key j's row, or -1 (no page)
    auto row_of = [&](int j) -> long long {
        const int lp = j / kv.page;
        const int phys = lp < kv.table_stride ? tab[lp] : -1;
        return phys >= 0 ? (long long)phys * kv.page_elems + (long long)(j % kv.page) * hd : -1ll;
    };
    float m = -INFINITY, l = 0.f, a0 = 0.f, a1 = 0.f;
    for (int base = 0; base <= t; base += keys) {
        const int ncached = max(0, min(keys, t - base));  // keys base .. base + ncached - 1 < t
        __syncthreads();  // the previous round's rows are consumed (and q is staged)
        for (int i = threadIdx.x; i < 2 * ncached * npc; i += blockDim.x) {
            const int kvsel = i >= ncached * npc, ii = kvsel ? i - ncached * npc : i;
            const int jj = ii / npc, pc = ii - jj * npc;
            const long long re = row_of(base + jj);
            if (re < 0) continue;
            const E* src = pool + (kvsel ? voff : koff) + re + (size_t)pc * (16 / S::ESZ);
            E* dst = (kvsel ? vs : ks) + (size_t)jj * rse + (size_t)pc * (16 / S::ESZ);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src) : "memory");
        }
        asm volatile("cp.async.commit_group;\ncp.async.wait_all;\n" ::: "memory");
        __syncthreads();
        const int k0 = base + w * kw;  // this warp's keys k0 .. k0 + kw - 1 (<= t)
        const int nk = max(0, min(kw, t + 1 - k0));
        if (nk == 0) continue;  // warp-uniform; the barrier of the next round is still taken
        const int j = k0 + lane;
        float s = -INFINITY;
        bool valid = false;
        if (lane < nk) {
            if (j == t) {
                float dot = 0.f;
                const float4* k4 = reinterpret_cast<const float4*>(fk);
                for (int p = 0; p < hd / 4; ++p) {
                    const float4 kk = k4[p], qq = q4[p];
                    dot = fmaf(qq.x, kk.x, fmaf(qq.y, kk.y, fmaf(qq.z, kk.z, fmaf(qq.w, kk.w, dot))));
                }
                s = dot * scale;
                valid = true;
            } else if (row_of(j) >= 0) {
                float dot = 0.f;
                const E* kr = ks + (size_t)(j - base) * rse;
                if constexpr (F16) {
                    for (int p = 0; p < hd / 8; ++p) {
                        const uint4 u = *reinterpret_cast<const uint4*>(kr + 8 * p);
                        const __half2* h2 = reinterpret_cast<const __half2*>(&u);
                        const float4 qa = q4[2 * p], qb = q4[2 * p + 1];
                        const float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]);
                        const float2 f2 = __half22float2(h2[2]), f3 = __half22float2(h2[3]);
                        dot = fmaf(qa.x, f0.x, fmaf(qa.y, f0.y, fmaf(qa.z, f1.x, fmaf(qa.w, f1.y, dot))));
                        dot = fmaf(qb.x, f2.x, fmaf(qb.y, f2.y, fmaf(qb.z, f3.x, fmaf(qb.w, f3.y, dot))));
                    }
                } else {
                    for (int p = 0; p < hd / 4; ++p) {
                        const float4 kk = *reinterpret_cast<const float4*>(kr + 4 * p), qq = q4[p];
                        dot = fmaf(qq.x, kk.x, fmaf(qq.y, kk.y, fmaf(qq.z, kk.z, fmaf(qq.w, kk.w, dot))));
                    }
                }
                s = dot * scale;
                valid = true;
            }
        }
        const float mn = fmaxf(m, warp_max(s));
        const float p = valid ? expf(s - mn) : 0.f;
        const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
        l = l * corr + warp_sum(p);
        a0 *= corr;
        a1 *= corr;
        const int c = 2 * lane;
        for (int u = 0; u < nk; ++u) {
            const float pu = __shfl_sync(FULL, p, u);
            if (pu == 0.f || c >= hd) continue;
            float2 v;
            if (k0 + u == t) v = make_float2(fv[c], fv[c + 1]);
            else if constexpr (F16)
                v = __half22float2(*reinterpret_cast<const __half2*>(vs + (size_t)(k0 + u - base) * rse + c));
            else v = *reinterpret_cast<const float2*>(vs + (size_t)(k0 + u - base) * rse + c);
            a0 = fmaf(pu, v.x, a0);
            a1 = fmaf(pu, v.y, a1);
        }
        m = mn;
    }
    // merge the warps' softmax states in warp order
    if (lane == 0) {
        wm[w] = m;
        wl[w] = l;
    }
    if (2 * lane < hd) {
        wacc[w][2 * lane] = a0;
        wacc[w][2 * lane + 1] = a1;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < hd; e += blockDim.x) {
        float mx = -INFINITY;
#pragma unroll
        for (int qq = 0; qq < W; ++qq) mx = fmaxf(mx, wm[qq]);
        float lsum = 0.f, o = 0.f;
#pragma unroll
        for (int qq = 0; qq < W; ++qq) {
            if (wm[qq] == -INFINITY) continue;
            const float f = expf(wm[qq] - mx);
            lsum = fmaf(wl[qq], f, lsum);
            o = fmaf(wacc[qq][e], f, o);
        }
        st_bf16_split(out + (size_t)b * HD + h * hd + e, o / lsum, lo_off);
    }
}

// One warp per (b, h, chunk); partial (m, l, o[hd]) at part[((b*H + h)*max_chunks + c)].
__global__ void cross_attn_batch_kernel(const float* __restrict__ qc, const float* __restrict__ cross32,
                                        const void* __restrict__ cross_st, int st_f16, const int* __restrict__ pos,
                                        const int* __restrict__ frame_off, const int* __restrict__ frames, int B,
                                        int H, int KVH, int hd, int m_cap, int layer, int max_chunks, float scale,
                                        float* __restrict__ part) {
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= B * H * max_chunks) return;
    const int c = item % max_chunks;
    const int bh = item / max_chunks;
    const int b = bh / H, h = bh - b * H;
    const int kvh = h / (H / KVH);
    const int M = frames[b];
    float* out = part + (size_t)item * (hd + 2);
    const int j0 = c * CHB;
    if (j0 >= M) {
        if (lane == 0) {
            out[0] = -INFINITY;
            out[1] = 0.f;
        }
        return;
    }
    const int nk = min(CHB, M - j0);
    const bool first = (*pos == 0);
    const int f16 = first ? 0 : st_f16;
    const void* src = first ? (const void*)cross32 : cross_st;
    const int HD = H * hd;
    const float* qr = qc + (size_t)b * HD + h * hd;
    const size_t kb = ((((size_t)layer * 2 + 0) * KVH + kvh) * m_cap + frame_off[b]) * hd;
    const size_t vb = ((((size_t)layer * 2 + 1) * KVH + kvh) * m_cap + frame_off[b]) * hd;
    float s = -INFINITY;
    if (lane < nk) {
        float dot = 0.f;
        const size_t kr = kb + (size_t)(j0 + lane) * hd;
        for (int e = 0; e < hd; ++e) dot = fmaf(qr[e], load_kv(src, kr + e, f16), dot);
        s = dot * scale;
    }
    const float mc = warp_max(s);
    const float p = (lane < nk) ? expf(s - mc) : 0.f;
    const float l = warp_sum(p);
    float a0 = 0.f, a1 = 0.f;
    for (int jj = 0; jj < nk; ++jj) {
        const float pp = __shfl_sync(FULL, p, jj);
        const int e = 2 * lane;
        if (e < hd) {
            const size_t vr = vb + (size_t)(j0 + jj) * hd + e;
            a0 = fmaf(pp, load_kv(src, vr, f16), a0);
            a1 = fmaf(pp, load_kv(src, vr + 1, f16), a1);
        }
    }
    if (lane == 0) {
        out[0] = mc;
        out[1] = l;
    }
    const int e = 2 * lane;
    if (e < hd) {
        out[2 + e] = a0;
        out[2 + e + 1] = a1;
    }
}

__global__ void cross_combine_kernel(const float* __restrict__ part, int B, int H, int hd, int max_chunks,
                                     __nv_bfloat16* __restrict__ out, size_t lo_off) {
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= B * H) return;
    const float* base = part + (size_t)item * max_chunks * (hd + 2);
    float M = -INFINITY;
    for (int k = lane; k < max_chunks; k += 32) M = fmaxf(M, base[(size_t)k * (hd + 2)]);
    M = warp_max(M);
    float L = 0.f;
    for (int k = lane; k < max_chunks; k += 32) {
        const float mk = base[(size_t)k * (hd + 2)];
        if (mk != -INFINITY) L += base[(size_t)k * (hd + 2) + 1] * expf(mk - M);
    }
    L = warp_sum(L);
    const int b = item / H, h = item - b * H;
    for (int e = lane; e < hd; e += 32) {
        float O = 0.f;
        for (int k = 0; k < max_chunks; ++k) {
            const float mk = base[(size_t)k * (hd + 2)];
            if (mk != -INFINITY) O += base[(size_t)k * (hd + 2) + 2 + e] * expf(mk - M);
        }
        st_bf16_split(out + (size_t)b * H * hd + h * hd + e, O / L, lo_off);
    }
}

// Cross attention of one (utterance b, head h) per CTA, streamed through shared memory.
// K rows and V rows of one head are contiguous over frames, so thread 0 keeps a ring of
// ST chunks of CH keys in flight as two bulk copies per chunk completing on one
// mbarrier.  Warp w scores keys [w*KW, (w+1)*KW) of each chunk with G lanes per key (16
// bytes of the row per lane, the matching q slice in registers, shuffle sum inside the
// group), keeps an online softmax, and accumulates V with lane c owning dims 2c, 2c+1.  The
// four warp states are merged in shared memory and written as bf16.  Semantics as the
// cross branch of MoonshineLayers.swift:150-160 (scale hd^-1/2, no mask over the frames).
template <int HDT, bool F16>
struct XsShape {
    static constexpr int ESZ = F16 ? 2 : 4;
    static constexpr int ROWB = HDT * ESZ;                        // bytes of one key row
    static constexpr int NE = ROWB / 16;                          // 16-byte pieces per row
    static constexpr int EP = 16 / ESZ;                           // elements per piece
    static constexpr int G = NE <= 4 ? 4 : (NE <= 8 ? 8 : 16);    // lanes per key
    static constexpr int KPP = 32 / G;                            // keys per warp pass
    static constexpr int CH = F16 ? 64 : 32;                      // keys per stage
    static constexpr int ST = 3;                                  // ring stages
    static constexpr int KW = CH / 4;                             // keys per warp per stage
    static constexpr int STAGE_ELEMS = CH * HDT;                  // per tensor
    static_assert(NE * 16 == ROWB && NE <= 16, "key rows must be whole 16-byte pieces");
    static_assert(KW % KPP == 0 && KW <= 32, "warp slice must be whole passes");
};
constexpr int XS_THREADS = 128;

template <int HDT, bool F16>
constexpr size_t xs_smem_bytes() {
    return 2 * (size_t)XsShape<HDT, F16>::ST * XsShape<HDT, F16>::STAGE_ELEMS * XsShape<HDT, F16>::ESZ;
}

template <int HDT, bool F16>
__global__ void __launch_bounds__(XS_THREADS) cross_attn_stream_kernel(
    const float* __restrict__ qc, const void* __restrict__ src, const int* __restrict__ frame_off,
    const int* __restrict__ frames, int H, int KVH, int m_cap, int layer, float scale,
    __nv_bfloat16* __restrict__ out, unsigned* status, size_t lo_off, const void* const* __restrict__ rows_src,
    const int* __restrict__ rows_cap) {
    pdl_wait();
    pdl_trigger();
    using S = XsShape<HDT, F16>;
    using E = typename std::conditional<F16, __half, float>::type;
    extern __shared__ __align__(128) unsigned char xs_raw[];
    E* ks = reinterpret_cast<E*>(xs_raw);
    E* vs = ks + S::ST * S::STAGE_ELEMS;
    __shared__ __align__(8) uint64_t full[S::ST];
    __shared__ float sc[4][S::KW];  // scores, then probabilities, of each warp's slice
    __shared__ float wm[4], wl[4];
    __shared__ float wacc[4][HDT];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int b = blockIdx.x / H, h = blockIdx.x - (blockIdx.x / H) * H;
    const int kvh = h / (H / KVH);
    const int M = frames[b];
    const int nchunks = (M + S::CH - 1) / S::CH;
    // concatenated layout (frames from frame_off[b], pitch m_cap) or row b's own buffer
    const E* base = reinterpret_cast<const E*>(rows_src ? rows_src[b] : src);
    const size_t mc = rows_src ? (size_t)rows_cap[b] : (size_t)m_cap;
    const size_t fo = rows_src ? 0 : (size_t)frame_off[b];
    const E* kg = base + ((((size_t)layer * 2 + 0) * KVH + kvh) * mc + fo) * HDT;
    const E* vg = base + ((((size_t)layer * 2 + 1) * KVH + kvh) * mc + fo) * HDT;
    auto issue = [&](int c) {
        const int st = c % S::ST;
        const uint32_t bytes = (uint32_t)min(S::CH, M - c * S::CH) * S::ROWB;
        mbar_expect_tx(&full[st], 2 * bytes);
        bulk_load(ks + (size_t)st * S::STAGE_ELEMS, kg + (size_t)c * S::STAGE_ELEMS, bytes, &full[st]);
        bulk_load(vs + (size_t)st * S::STAGE_ELEMS, vg + (size_t)c * S::STAGE_ELEMS, bytes, &full[st]);
    };
    if (threadIdx.x == 0) {
        for (int i = 0; i < S::ST; ++i) mbar_init(&full[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int c = 0; c < min(nchunks, S::ST); ++c) issue(c);
    }
    __syncthreads();  // the barriers are initialised before any thread waits on them
    // q slice of this lane's piece (lanes with sub >= NE only pad their group)
    const int g = lane / S::G, sub = lane - (lane / S::G) * S::G;
    float qr[S::EP];
    const float* qrow = qc + (size_t)b * H * HDT + h * HDT;
#pragma unroll
    for (int e = 0; e < S::EP; ++e) qr[e] = (sub < S::NE) ? qrow[sub * S::EP + e] : 0.f;

    float m_run = -INFINITY, l_run = 0.f, a0 = 0.f, a1 = 0.f;
    int failed_at = -1;
    for (int c = 0; c < nchunks; ++c) {
        const int st = c % S::ST;
        const bool ok = mbar_wait(&full[st], (c / S::ST) & 1);
        // every warp is past chunk c-1 here, so its stage can be refilled
        if (!__syncthreads_and(ok)) {
            failed_at = c;
            break;
        }
        if (threadIdx.x == 0 && c >= 1 && c - 1 + S::ST < nchunks) issue(c - 1 + S::ST);
        const int nk = min(S::CH, M - c * S::CH);
        const int k0 = wid * S::KW;
        const int kw = max(0, min(S::KW, nk - k0));
        const E* kst = ks + (size_t)st * S::STAGE_ELEMS + (size_t)k0 * HDT;
        const E* vst = vs + (size_t)st * S::STAGE_ELEMS + (size_t)k0 * HDT;
#pragma unroll
        for (int p = 0; p < S::KW / S::KPP; ++p) {
            const int j = p * S::KPP + g;
            float dot = 0.f;
            if (j < kw && sub < S::NE) {
                const uint4 u = *reinterpret_cast<const uint4*>(kst + (size_t)j * HDT + sub * S::EP);
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
            if (sub == 0) sc[wid][j] = (j < kw) ? dot * scale : -INFINITY;
        }
        __syncwarp();
        const float sv = lane < S::KW ? sc[wid][lane] : -INFINITY;
        const float mn = fmaxf(m_run, warp_max(sv));
        const float pv = (sv == -INFINITY) ? 0.f : expf(sv - mn);
        const float corr = (m_run == -INFINITY) ? 0.f : expf(m_run - mn);
        l_run = l_run * corr + warp_sum(pv);
        a0 *= corr;
        a1 *= corr;
        __syncwarp();
        if (lane < S::KW) sc[wid][lane] = pv;
        __syncwarp();
        if (2 * lane < HDT) {
#pragma unroll 4
            for (int j = 0; j < kw; ++j) {
                const float pj = sc[wid][j];
                float2 v;
                if constexpr (F16) v = __half22float2(*reinterpret_cast<const __half2*>(vst + (size_t)j * HDT + 2 * lane));
                else v = *reinterpret_cast<const float2*>(vst + (size_t)j * HDT + 2 * lane);
                a0 = fmaf(pj, v.x, a0);
                a1 = fmaf(pj, v.y, a1);
            }
        }
        m_run = mn;
    }
    if (failed_at >= 0) {  // uniform across the CTA (decided by __syncthreads_and)
        if (threadIdx.x == 0) {
            atomicCAS(status, 0u, (unsigned)DEV_WAIT_TIMEOUT);
            const int issued = min(nchunks, failed_at == 0 ? S::ST : failed_at - 1 + S::ST);
            for (int c = failed_at; c < issued; ++c) mbar_wait(&full[c % S::ST], (c / S::ST) & 1);
        }
        return;
    }
    if (lane == 0) {
        wm[wid] = m_run;
        wl[wid] = l_run;
    }
    if (2 * lane < HDT) {
        wacc[wid][2 * lane] = a0;
        wacc[wid][2 * lane + 1] = a1;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < HDT; e += blockDim.x) {
        float Mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) Mx = fmaxf(Mx, wm[w]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            if (wm[w] == -INFINITY) continue;
            const float f = expf(wm[w] - Mx);
            L = fmaf(wl[w], f, L);
            O = fmaf(wacc[w][e], f, O);
        }
        st_bf16_split(out + (size_t)b * H * HDT + h * HDT + e, O / L, lo_off);
    }
}

template <int HDT>
cudaError_t launch_cross_stream(bool f16, const float* qc, const void* src, const int* frame_off, const int* frames,
                                int B, int H, int KVH, int m_cap, int layer, float scale, __nv_bfloat16* out,
                                unsigned* status, cudaStream_t s, size_t lo_off, const void* const* rows_src,
                                const int* rows_cap) {
    static bool attr_set = false;
    if (!attr_set) {  // both variants at once: the fp16 one is first launched inside a graph capture
        cudaError_t e = cudaFuncSetAttribute(cross_attn_stream_kernel<HDT, true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)xs_smem_bytes<HDT, true>());
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(cross_attn_stream_kernel<HDT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)xs_smem_bytes<HDT, false>());
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    if (f16)
        return launch_kernel(cross_attn_stream_kernel<HDT, true>, dim3(B * H), dim3(XS_THREADS),
                             xs_smem_bytes<HDT, true>(), s, qc, src, frame_off, frames, H, KVH, m_cap, layer, scale,
                             out, status, lo_off, rows_src, rows_cap);
    return launch_kernel(cross_attn_stream_kernel<HDT, false>, dim3(B * H), dim3(XS_THREADS),
                         xs_smem_bytes<HDT, false>(), s, qc, src, frame_off, frames, H, KVH, m_cap, layer, scale,
                         out, status, lo_off, rows_src, rows_cap);
}

// One thread per row b.  Decodes the packed argmax, applies the greedy-loop rules of
// MoonshineModel.swift:204-232 per utterance, and advances the step counter.
__global__ void step_finalize_kernel(unsigned long long* amax, int B, int* pos, int* next_ids, int* ids_out,
                                     int t_cap, int* counts, const int* limits, int* done, int* hit_eos, int eos,
                                     int forced) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) {
        const int id = (int)(0xFFFFFFFFu - (uint32_t)(amax[b] & 0xFFFFFFFFull));
        amax[b] = 0ull;
        next_ids[b] = id;
        if (!done[b]) {
            if (!forced && id == eos) {
                done[b] = 1;
                hit_eos[b] = 1;
            } else {
                ids_out[(size_t)b * t_cap + counts[b]] = id;
                counts[b] += 1;
                if (counts[b] >= limits[b]) done[b] = 1;
            }
        }
    }
    __syncthreads();
    if (blockIdx.x == 0 && threadIdx.x == 0) *pos += 1;
}

}  // namespace

cudaError_t launch_embed_rows(const int* ids, const float* embed, int d, int B, int V, float* x, unsigned* status,
                              cudaStream_t s, __nv_bfloat16* xb, size_t lo_off, float2* stats, int stats_ld,
                              int tile_n) {
    if (stats && (tile_n <= 0 || stats_ld < B)) return cudaErrorInvalidValue;
    ++launch_counter();
    return launch_kernel(embed_rows_kernel, dim3(B), dim3(128), 0, s, ids, embed, d, B, V, x, status, xb, lo_off,
                         stats, stats_ld, tile_n);
}

cudaError_t launch_ln_bf16(const float* x, int rows, int d, const float* w, __nv_bfloat16* out, cudaStream_t s,
                          float w_offset, size_t lo_off) {
    if (rows <= 0) return cudaSuccess;
    ++launch_counter();
    const bool warp_rows = d % 4 == 0 && d <= 32 * 4 * LNW_V4 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                           reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 8 == 0 &&
                           lo_off % 4 == 0;
    if (warp_rows)
        return launch_kernel(ln_bf16_warp_kernel, dim3((rows + LNW_ROWS - 1) / LNW_ROWS), dim3(LNW_ROWS * 32), 0, s,
                             x, rows, d, w, w_offset, out, lo_off);
    return launch_kernel(ln_bf16_kernel, dim3(rows), dim3(128), 0, s, x, rows, d, w, w_offset, out, lo_off);
}

cudaError_t launch_self_attn_batch(const float* q, const float* kv_new, const PagedKv& kv, const int* pos, int B,
                                   int H, int KVH, int hd, float scale, __nv_bfloat16* out, cudaStream_t s,
                                   size_t lo_off) {
    if (hd > MAXHD_B || (hd & 7) || !kv.table || kv.page <= 0 || !kv.pool || kv.table_stride <= 0)
        return cudaErrorInvalidValue;
    ++launch_counter();
    // every position of the call is below table_stride * page: rounds of that many keys (32,
    // 64 or 128), at most KEYS
    const int reach = kv.reach > 0 ? std::min(kv.reach, kv.table_stride * kv.page) : kv.table_stride * kv.page;
    auto go = [&](auto f16, auto keys) {
        constexpr bool F = decltype(f16)::value;
        constexpr int KS = decltype(keys)::value;
        constexpr int W = KS == 32 ? 1 : SA_WARPS;  // one round of 32 keys: one warp per (b, h)
        return launch_kernel(self_attn_batch_kernel<F, KS, W>, dim3(B * H), dim3(W * 32), sa_smem_bytes<F>(KS, hd),
                             s, q, kv_new, kv, pos, B, H, KVH, hd, scale, out, lo_off);
    };
    using T_ = std::true_type;
    using F_ = std::false_type;
    using K32 = std::integral_constant<int, 32>;
    using K64 = std::integral_constant<int, 64>;
    using K128 = std::integral_constant<int, 128>;
    if (kv.kv_f16) return reach <= 32 ? go(T_(), K32()) : reach <= 64 ? go(T_(), K64()) : go(T_(), K128());
    return reach <= 32 ? go(F_(), K32()) : go(F_(), K64());
}

cudaError_t launch_cross_attn_batch(const float* qc, const float* cross32, const void* cross_st, int st_f16,
                                    const int* pos, const int* frame_off, const int* frames, int B, int H, int KVH,
                                    int hd, int m_cap, int layer, int max_frames, float scale, float* part,
                                    __nv_bfloat16* out, int first_step, unsigned* status, cudaStream_t s,
                                    size_t lo_off, const CrossRows* rows) {
    if (hd > MAXHD_B || (hd & 1)) return cudaErrorInvalidValue;
    if (rows && (first_step < 0 || !cross_rows_supported(hd) || !rows->src32 || !rows->src16 || !rows->cap))
        return cudaErrorInvalidValue;
    if (first_step >= 0 && cross_rows_supported(hd)) {
        // one CTA per (utterance, head); the first decoder call reads the fp32 copy
        const void* src = first_step ? (const void*)cross32 : cross_st;
        const bool f16 = !first_step && st_f16;
        const void* const* rsrc = rows ? (first_step ? rows->src32 : rows->src16) : nullptr;
        const int* rcap = rows ? rows->cap : nullptr;
        if ((!rows && (reinterpret_cast<uintptr_t>(src) & 15) != 0) || !status) return cudaErrorInvalidValue;
        ++launch_counter();
        switch (hd) {
            case 32: return launch_cross_stream<32>(f16, qc, src, frame_off, frames, B, H, KVH, m_cap, layer, scale, out, status, s, lo_off, rsrc, rcap);
            case 40: return launch_cross_stream<40>(f16, qc, src, frame_off, frames, B, H, KVH, m_cap, layer, scale, out, status, s, lo_off, rsrc, rcap);
            case 48: return launch_cross_stream<48>(f16, qc, src, frame_off, frames, B, H, KVH, m_cap, layer, scale, out, status, s, lo_off, rsrc, rcap);
            default: return launch_cross_stream<64>(f16, qc, src, frame_off, frames, B, H, KVH, m_cap, layer, scale, out, status, s, lo_off, rsrc, rcap);
        }
    }
    // generic head_dim: chunk partials + combine, fp32/stored copy chosen on the device
    const int max_chunks = (max_frames + CHB - 1) / CHB;
    const int items = B * H * max_chunks;
    launch_counter() += 2;
    cross_attn_batch_kernel<<<(items + 7) / 8, 256, 0, s>>>(qc, cross32, cross_st, st_f16, pos, frame_off, frames, B,
                                                            H, KVH, hd, m_cap, layer, max_chunks, scale, part);
    cross_combine_kernel<<<(B * H + 7) / 8, 256, 0, s>>>(part, B, H, hd, max_chunks, out, lo_off);
    return cudaGetLastError();
}

bool cross_rows_supported(int hd) { return hd == 32 || hd == 40 || hd == 48 || hd == 64; }

cudaError_t launch_step_finalize(unsigned long long* amax, int B, int* pos, int* next_ids, int* ids_out, int t_cap,
                                 int* counts, const int* limits, int* done, int* hit_eos, int eos, int forced,
                                 cudaStream_t s) {
    if (B > 1024) return cudaErrorInvalidValue;
    ++launch_counter();
    return launch_kernel(step_finalize_kernel, dim3(1), dim3(((B + 31) / 32) * 32), 0, s, amax, B, pos, next_ids,
                         ids_out, t_cap, counts, limits, done, hit_eos, eos, forced);
}

namespace {
// Block (segment s, row b): copy row b's M[b] frames of segment s of its own cross K/V
// ([segs][mcap[b]][hd], fp32 and optional fp16 copy) to frames off[b].. of segment s of
// the concatenated layout [segs][m_cap][hd].  Rows of hd elements are whole 16-byte units.
__global__ void gather_cross_kernel(const float* const* __restrict__ src32, const __half* const* __restrict__ src16,
                                    const int* __restrict__ mcap, const int* __restrict__ frames,
                                    const int* __restrict__ off, int hd, int m_cap, float* __restrict__ dst32,
                                    __half* __restrict__ dst16) {
    const int seg = blockIdx.x, b = blockIdx.y;
    const size_t n = (size_t)frames[b] * hd;
    const size_t so = (size_t)seg * mcap[b] * hd, dof = ((size_t)seg * m_cap + off[b]) * hd;
    const uint4* s32 = reinterpret_cast<const uint4*>(src32[b] + so);
    uint4* d32 = reinterpret_cast<uint4*>(dst32 + dof);
    for (size_t i = threadIdx.x; i < n / 4; i += blockDim.x) d32[i] = s32[i];
    if (dst16 && src16[b]) {
        const uint4* s16 = reinterpret_cast<const uint4*>(src16[b] + so);
        uint4* d16 = reinterpret_cast<uint4*>(dst16 + dof);
        for (size_t i = threadIdx.x; i < n / 8; i += blockDim.x) d16[i] = s16[i];
    }
}
}  // namespace

cudaError_t launch_gather_cross(const float* const* src32, const void* const* src16, const int* mcap,
                                const int* frames, const int* off, int B, int segs, int hd, int m_cap, float* dst32,
                                void* dst16, cudaStream_t s) {
    if (B <= 0 || segs <= 0) return cudaSuccess;
    if (hd & 7) return cudaErrorInvalidValue;
    ++launch_counter();
    gather_cross_kernel<<<dim3(segs, B), 256, 0, s>>>(src32, reinterpret_cast<const __half* const*>(src16), mcap,
                                                       frames, off, hd, m_cap, dst32,
                                                       reinterpret_cast<__half*>(dst16));
    return cudaGetLastError();
}

namespace {
// dst row r = src row r (interleave == 0) or, for the SwiGLU fc1, dst row 2j = src row j
// (value) and dst row 2j+1 = src row j + interleave (gate).
__global__ void f32_to_bf16_rows_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int rows,
                                        int K, int interleave, size_t lo_off, const float* __restrict__ colscale) {
    const int r = blockIdx.x;
    if (r >= rows) return;
    const int sr = interleave ? ((r & 1) ? interleave + (r >> 1) : (r >> 1)) : r;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float v = src[(size_t)sr * K + k];
        st_bf16_split(dst + (size_t)r * K + k, colscale ? v * colscale[k] : v, lo_off);
    }
}
// One block of 256 threads per row: strided double partial sums, then a fixed tree.
__global__ void bf16_row_sums_kernel(const __nv_bfloat16* __restrict__ w, int K, size_t lo_off,
                                     float* __restrict__ out) {
    __shared__ double red[256];
    const int r = blockIdx.x;
    const __nv_bfloat16* row = w + (size_t)r * K;
    double s = 0.0;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        s += (double)__bfloat162float(row[k]);
        if (lo_off) s += (double)__bfloat162float(row[lo_off + k]);
    }
    red[threadIdx.x] = s;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x == 0) out[r] = (float)red[0];
}
__global__ void interleave_f32_kernel(const float* __restrict__ src, float* __restrict__ dst, int n2, int half) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < n2) dst[r] = (r & 1) ? src[half + (r >> 1)] : src[r >> 1];
}
}  // namespace

cudaError_t launch_f32_to_bf16_rows(const float* src, __nv_bfloat16* dst, int rows, int K, int interleave,
                                    cudaStream_t s, size_t lo_off, const float* colscale) {
    ++launch_counter();
    f32_to_bf16_rows_kernel<<<rows, 256, 0, s>>>(src, dst, rows, K, interleave, lo_off, colscale);
    return cudaGetLastError();
}

cudaError_t launch_bf16_row_sums(const __nv_bfloat16* w, int rows, int K, size_t lo_off, float* out,
                                 cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    ++launch_counter();
    bf16_row_sums_kernel<<<rows, 256, 0, s>>>(w, K, lo_off, out);
    return cudaGetLastError();
}

cudaError_t launch_interleave_f32(const float* src, float* dst, int n2, int half, cudaStream_t s) {
    ++launch_counter();
    interleave_f32_kernel<<<(n2 + 255) / 256, 256, 0, s>>>(src, dst, n2, half);
    return cudaGetLastError();
}

size_t cross_batch_part_floats(int B, int H, int hd, int max_frames) {
    return (size_t)B * H * ((max_frames + CHB - 1) / CHB) * (hd + 2);
}

}  // namespace msb
