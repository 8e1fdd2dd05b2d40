// Batch-1 greedy decode as ONE persistent cooperative kernel (fp32 weights).
//
// A whole forced-length (or EOS-terminated) token loop runs inside a single launch: the
// argmax of step t is fed back as the embedding row of step t+1 on the device, so there
// is no host round trip per token (the reference syncs with `.item()` every token,
// Sources/MoonshineMLX/MoonshineModel.swift:216-229).
//
// Batch-1 decode is a chain of small dependent GEMVs, so the cost is the chain's latency
// rather than HBM bandwidth.  Each decoder layer (MoonshineLayers.swift:350-379) runs as
// eight grid-wide phases separated by a bounded grid barrier:
//
//   P1  LN1 (every CTA) + QKV rows + interleaved partial RoPE + KV append
//   P2  self-attention partials over 32-key chunks, [cache(fp16|fp32) ; this step's fp32 K/V]
//   P3  combine (every CTA) + O projection split by head -> ps[h][d]
//   P4  x1 = x + sum_h ps, LN2 + cross-attention Q rows
//   P5  cross-attention partials over 32-key chunks, pre-combined per CTA
//   P6  combine (every CTA) + cross O projection split by head -> pc[h][d]
//   P7  x2 = x1 + sum_h pc, LN3 + fc1 rows + bias + SwiGLU (first half value, second gate)
//   P8  fc2 rows + bias + residual -> next residual buffer
//   F   final LN + LM-head rows with per-CTA argmax; grid argmax (ties -> lowest id)
//
// Latency hiding: every warp owns a fixed slice of every phase's weight rows (and of the
// K/V chunks, which do not depend on the step's activations), and copies the NEXT phase's
// slice into its own shared-memory region with cp.async before it waits at the barrier.
// After the barrier only the activations (a few KB, L2-resident) are read from global
// memory; the weight rows are already on chip.  The LM head streams through a
// double-buffered cp.async pipeline.
//
// KV rounding follows the reference's fp16 cache rules (MoonshineLayers.swift:106-125):
// the current position's K/V enter attention in fp32 and are stored rounded; cross K/V
// are fp32 at step 0 and the stored (rounded) copy afterwards.
#include "common.cuh"
#include "kernels.h"

namespace msb {

namespace {

constexpr int NT = 256;
constexpr int NWB = NT / 32;   // warps per CTA
constexpr int CH = 32;         // keys per attention chunk
constexpr int MAXHD = 64;

// ------------------------------------------------------------------ async copies
__device__ __forceinline__ void cp16(void* s, const void* g) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(s);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
__device__ __forceinline__ void cp_wait_two_pending() { asm volatile("cp.async.wait_group 2;\n" ::: "memory"); }

// Warp-cooperative async copy; `bytes` is a multiple of 16, both ends 16-byte aligned.
__device__ __forceinline__ void warp_cp(void* s, const void* g, int bytes, int lane) {
    char* sd = reinterpret_cast<char*>(s);
    const char* gs = reinterpret_cast<const char*>(g);
    for (int o = lane * 16; o < bytes; o += 32 * 16) cp16(sd + o, gs + o);
}

// Dot product of two shared-memory vectors (n % 4 == 0), summed over the warp.
__device__ __forceinline__ float sdot(const float* w, const float* v, int n, int lane) {
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const float4* v4 = reinterpret_cast<const float4*>(v);
    float acc = 0.f;
    for (int i = lane; i < (n >> 2); i += 32) {
        const float4 a = w4[i], b = v4[i];
        acc = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, acc))));
    }
    return warp_sum(acc);
}

// ------------------------------------------------------------------ attention chunk
// One warp attends q (shared memory) over keys [j0, j0+nk).  Row `fresh_j` comes from the
// fp32 `fresh_k/fresh_v` (global); every other row j from base + (j - jb) * hd in `kb/vb`,
// which are shared memory (SMEM) or global memory (read through L2).  Lanes own keys for
// the scores and dims for the weighted sum; (m, l, acc) is an online-softmax state.
// Kept out of line: one copy of this code serves both attention phases, which keeps the
// persistent kernel's instruction footprint small.
__device__ __noinline__ void attend(bool SMEM, const float* q, const void* kb, const void* vb, int jb, int j0,
                                       int nk, int hd, float scale, int f16, const float* fresh_k,
                                       const float* fresh_v, int fresh_j, int lane, float& m, float& l,
                                       float acc[MAXHD / 32]) {
    const int j = j0 + lane;
    float s = -INFINITY;
    if (lane < nk) {
        float dot = 0.f;
        if (j == fresh_j) {
            for (int c = 0; c < hd; c += 4) {
                const float4 a = *reinterpret_cast<const float4*>(q + c);
                const float4 b = ldcg4(reinterpret_cast<const float4*>(fresh_k + c));
                dot = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, dot))));
            }
        } else if (f16) {
            const uint4* kr = reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(kb) + (size_t)(j - jb) * hd);
            uint4 rk[MAXHD / 8];
#pragma unroll
            for (int e = 0; e < MAXHD / 8; ++e)
                if (e * 8 < hd) rk[e] = SMEM ? kr[e] : __ldcg(kr + e);
#pragma unroll
            for (int e = 0; e < MAXHD / 8; ++e) {
                if (e * 8 < hd) {
                    const __half2* h2 = reinterpret_cast<const __half2*>(&rk[e]);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float2 b = __half22float2(h2[u]);
                        dot = fmaf(q[e * 8 + 2 * u], b.x, dot);
                        dot = fmaf(q[e * 8 + 2 * u + 1], b.y, dot);
                    }
                }
            }
        } else {
            const float4* kr = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(kb) + (size_t)(j - jb) * hd);
            for (int e = 0; e < (hd >> 2); ++e) {
                const float4 b = SMEM ? kr[e] : __ldcg(kr + e);
                const float4 a = *reinterpret_cast<const float4*>(q + 4 * e);
                dot = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, dot))));
            }
        }
        s = dot * scale;
    }
    const float mc = warp_max(s);
    const float mn = fmaxf(m, mc);
    const float pj = (lane < nk) ? expf(s - mn) : 0.f;
    const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
    l = l * corr + warp_sum(pj);
#pragma unroll
    for (int i = 0; i < MAXHD / 32; ++i) acc[i] *= corr;
#pragma unroll 4
    for (int jj = 0; jj < nk; ++jj) {
        const float pp = __shfl_sync(FULL, pj, jj);
        const int row = j0 + jj;
#pragma unroll
        for (int i = 0; i < MAXHD / 32; ++i) {
            const int c = 2 * lane + i;  // lane owns dims (2*lane, 2*lane+1)
            if (c < hd) {
                float vv;
                if (row == fresh_j) {
                    vv = ldcg(fresh_v + c);
                } else if (f16) {
                    const __half* vp = reinterpret_cast<const __half*>(vb) + (size_t)(row - jb) * hd + c;
                    vv = __half2float(SMEM ? *vp : __ldcg(vp));
                } else {
                    const float* vp = reinterpret_cast<const float*>(vb) + (size_t)(row - jb) * hd + c;
                    vv = SMEM ? *vp : ldcg(vp);
                }
                acc[i] = fmaf(pp, vv, acc[i]);
            }
        }
    }
    m = mn;
}

// Fast path of one attention chunk with everything on chip: q, the chunk's K/V rows (the
// warp's prefetch region, row j at j * HDT elements) and, for self-attention, the fresh
// fp32 K/V row that replaces local row `fresh`.  Lane j scores key j; lane c then owns
// dims (2c, 2c+1) of the weighted V sum, reading the probabilities from `pw` (per warp).
template <int HDT, bool F16>
__device__ __forceinline__ void attend_fast(const float* __restrict__ q, const unsigned char* __restrict__ kreg,
                                            const unsigned char* __restrict__ vreg, int nk, int fresh,
                                            const float* __restrict__ fk, const float* __restrict__ fv, float scale,
                                            float* pw, int lane, float& m, float& l, float& a0, float& a1) {
    float s = -INFINITY;
    if (lane < nk) {
        float dot = 0.f;
        if (lane == fresh) {
#pragma unroll
            for (int c = 0; c < HDT; c += 4) {
                const float4 a = *reinterpret_cast<const float4*>(q + c);
                const float4 b = *reinterpret_cast<const float4*>(fk + c);
                dot = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, dot))));
            }
        } else if (F16) {
            const uint4* kr = reinterpret_cast<const uint4*>(kreg + (size_t)lane * HDT * 2);
#pragma unroll
            for (int e = 0; e < HDT / 8; ++e) {
                const uint4 u = kr[e];
                const __half2* h2 = reinterpret_cast<const __half2*>(&u);
                const float4 qa = *reinterpret_cast<const float4*>(q + 8 * e);
                const float4 qb = *reinterpret_cast<const float4*>(q + 8 * e + 4);
                const float2 k0 = __half22float2(h2[0]), k1 = __half22float2(h2[1]);
                const float2 k2 = __half22float2(h2[2]), k3 = __half22float2(h2[3]);
                dot = fmaf(qa.x, k0.x, fmaf(qa.y, k0.y, fmaf(qa.z, k1.x, fmaf(qa.w, k1.y, dot))));
                dot = fmaf(qb.x, k2.x, fmaf(qb.y, k2.y, fmaf(qb.z, k3.x, fmaf(qb.w, k3.y, dot))));
            }
        } else {
            const float4* kr = reinterpret_cast<const float4*>(kreg + (size_t)lane * HDT * 4);
#pragma unroll
            for (int e = 0; e < HDT / 4; ++e) {
                const float4 b = kr[e];
                const float4 a = *reinterpret_cast<const float4*>(q + 4 * e);
                dot = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, dot))));
            }
        }
        s = dot * scale;
    }
    const float mc = warp_max(s);
    const float mn = fmaxf(m, mc);
    const float pj = (lane < nk) ? expf(s - mn) : 0.f;
    const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
    l = l * corr + warp_sum(pj);
    a0 *= corr;
    a1 *= corr;
    pw[lane] = pj;
    __syncwarp();
    if (2 * lane < HDT) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
        for (int j = 0; j < nk; ++j) {
            const float pp = pw[j];
            float2 v;
            if (j == fresh) v = *reinterpret_cast<const float2*>(fv + 2 * lane);
            else if (F16) v = __half22float2(reinterpret_cast<const __half2*>(vreg + (size_t)j * HDT * 2)[lane]);
            else v = reinterpret_cast<const float2*>(vreg + (size_t)j * HDT * 4)[lane];
            s0 = fmaf(pp, v.x, s0);
            s1 = fmaf(pp, v.y, s1);
        }
        a0 += s0;
        a1 += s1;
    }
    __syncwarp();
    m = mn;
}

// Online merge of one softmax partial (m, l, o) into a running (M, L, O).
__device__ __forceinline__ void merge_partial(float m, float l, float o, float& M, float& L, float& O) {
    const float Mn = fmaxf(M, m);
    const float a = (M == -INFINITY) ? 0.f : expf(M - Mn);
    const float b = expf(m - Mn);
    L = fmaf(L, a, l * b);
    O = fmaf(O, a, o * b);
    M = Mn;
}

// LayerNorm (biased variance, eps 1e-5) of x = base + sum_k parts[k] into `out` (shared
// memory), computed by every CTA.  `coh` selects L2-coherent loads for `base`.
__device__ __forceinline__ void cta_ln(const float* base, bool coh, const float* p0, const float* p1, int nparts,
                                       int d, const float* w, float* out, float* red) {
    float s = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        float v = coh ? ldcg(base + i) : base[i];
        for (int k = 0; k < nparts; ++k) v += ldcg(p0 + (size_t)k * d + i);
        if (p1)
            for (int k = 0; k < nparts; ++k) v += ldcg(p1 + (size_t)k * d + i);
        out[i] = v;
        s += v;
    }
    const float mean = block_sum(s, red) / (float)d;
    float q = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float c = out[i] - mean;
        q += c * c;
    }
    const float rstd = rsqrtf(block_sum(q, red) / (float)d + 1e-5f);
    for (int i = threadIdx.x; i < d; i += blockDim.x) out[i] = (out[i] - mean) * rstd * w[i];
    __syncthreads();
}

__device__ __forceinline__ void stage(const float* src, float* dst, int n) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = ldcg(src + i);
    __syncthreads();
}

// Chunk bookkeeping for the cross-attention rounds.
struct CrossMap {
    int nck, items, rounds;
};

template <int HDT>
__global__ void __launch_bounds__(NT, 1) decode_b1_kernel(DecodeParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ float red[32];
    __shared__ float s_bv[NWB];
    __shared__ int s_bi[NWB];
    __shared__ int s_whead[NWB];

    const int d = p.d, H = p.H, KVH = p.KVH, I = p.I, V = p.V, L = p.L;
    constexpr int hd = HDT;
    const int HD = H * hd, KVD = KVH * hd;
    const int rep = H / KVH;
    const int half_nd = p.nd >> 1;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int gw = blockIdx.x * NWB + wid;
    const int NW = gridDim.x * NWB;
    const int G = gridDim.x;
    const int kvesz = p.kv_f16 ? 2 : 4;

    // shared memory carve-up
    float* hs = reinterpret_cast<float*>(smem_raw);             // [d]
    float* vec = hs + ((d + 3) & ~3);                           // [max(I, HD, d)]
    const int vec_n = max(max(I, HD), d);
    float* comb = vec + ((vec_n + 3) & ~3);                      // [HD]
    float* wpart = comb + ((HD + 3) & ~3);                       // [NWB][hd + 2]
    float* fks = wpart + ((NWB * (hd + 2) + 3) & ~3);            // [2][KVD] this step's fp32 K/V
    float* pws = fks + ((2 * KVD + 3) & ~3);                      // [NWB][32] chunk probabilities
    unsigned char* regions = reinterpret_cast<unsigned char*>(pws + NWB * 32);
    float* reg = reinterpret_cast<float*>(regions + (size_t)wid * p.region_bytes);

    const CrossMap cm{(p.M + CH - 1) / CH, H * ((p.M + CH - 1) / CH), (H * ((p.M + CH - 1) / CH) + NW - 1) / NW};
    const int npairs = (HD + 2 * KVD) >> 1;
    const int per7 = (I + NW - 1) / NW;       // blocked SwiGLU items per warp, P7

    unsigned epoch = 0;
    // optional trace: CTA 0 stamps %globaltimer at the start, then per phase after the
    // activation loads, after its prefetched slice landed, after its math, and after the
    // grid barrier
    int tr = 0;
    const bool tracer = p.trace && blockIdx.x == 0 && threadIdx.x == 0;
    auto stamp = [&]() {
        if (tracer && tr < p.trace_cap) p.trace[tr] = globaltimer_ns();
        ++tr;
    };
    stamp();
    auto sync = [&]() -> bool {
        if (!grid_barrier(p.bar_count, p.status, epoch)) return false;
        stamp();
        return true;
    };

    // ---- prefetchers: each copies this warp's slice of the named phase into `reg`
    auto pf_p1 = [&](int l) {
        const float* w = p.layers[l].wqkv;
        int k = 0;
        for (int it = gw; it < npairs; it += NW, ++k)
            warp_cp(reg + (size_t)k * 2 * d, w + (size_t)(2 * it) * d, 2 * d * 4, lane);
    };
    auto pf_p2 = [&](int l, int t) {
        const int nck = (t + 1 + CH - 1) / CH;
        const int it = gw;
        if (it >= H * nck) return;
        const int h = it / nck, c = it - h * nck;
        const int kvh = h / rep;
        const int j0 = c * CH;
        const int ncached = min(j0 + CH, t) - j0;  // rows below t
        if (ncached <= 0) return;
        const size_t cb = (((size_t)l * KVH + kvh) * p.t_cap + j0) * hd * kvesz;
        const int bytes = ncached * hd * kvesz;
        warp_cp(reg, reinterpret_cast<const char*>(p.self_k) + cb, bytes, lane);
        warp_cp(reinterpret_cast<char*>(reg) + CH * hd * kvesz, reinterpret_cast<const char*>(p.self_v) + cb,
                bytes, lane);
    };
    auto pf_orows = [&](const float* w) {  // P3 / P6: output-projection rows r = gw + k*NW
        int k = 0;
        for (int r = gw; r < d; r += NW, ++k) warp_cp(reg + (size_t)k * HD, w + (size_t)r * HD, HD * 4, lane);
    };
    auto pf_p4 = [&](int l) {
        const float* w = p.layers[l].wcq;
        int k = 0;
        for (int r = gw; r < HD; r += NW, ++k) warp_cp(reg + (size_t)k * d, w + (size_t)r * d, d * 4, lane);
    };
    auto pf_p5 = [&](int l, int step) {
        const int it = gw;
        if (it >= cm.items) return;
        const int h = it / cm.nck, c = it - h * cm.nck;
        const int kvh = h / rep;
        const int j0 = c * CH, nk = min(CH, p.M - j0);
        const int esz = (step == 0) ? 4 : kvesz;
        const char* src = (step == 0) ? reinterpret_cast<const char*>(p.cross32)
                                      : reinterpret_cast<const char*>(p.cross_stored);
        const size_t kb = ((((size_t)l * 2 + 0) * KVH + kvh) * p.m_cap + j0) * hd * esz;
        const size_t vb = ((((size_t)l * 2 + 1) * KVH + kvh) * p.m_cap + j0) * hd * esz;
        warp_cp(reg, src + kb, nk * hd * esz, lane);
        warp_cp(reinterpret_cast<char*>(reg) + CH * hd * esz, src + vb, nk * hd * esz, lane);
    };
    auto pf_p7 = [&](int l) {
        const float* w = p.layers[l].w1;
        const int j0 = gw * per7, j1 = min(I, j0 + per7);
        for (int j = j0; j < j1; ++j) {
            warp_cp(reg + (size_t)(2 * (j - j0)) * d, w + (size_t)j * d, d * 4, lane);
            warp_cp(reg + (size_t)(2 * (j - j0) + 1) * d, w + (size_t)(j + I) * d, d * 4, lane);
        }
    };
    auto pf_p8 = [&](int l) {
        const float* w = p.layers[l].w2;
        int k = 0;
        for (int r = gw; r < d; r += NW, ++k) warp_cp(reg + (size_t)k * I, w + (size_t)r * I, I * 4, lane);
    };
    auto pf_lm = [&](int g, int buf) {  // LM head rows [4g, 4g+4) into buffer `buf`
        const int r0 = 4 * g;
        const int nr = min(4, V - r0);
        warp_cp(reg + (size_t)buf * 4 * d, p.lm_head + (size_t)r0 * d, nr * d * 4, lane);
    };
    auto land = [&]() {  // prefetched data of this phase is in shared memory
        stamp();
        cp_wait_all();
        __syncwarp();
        stamp();
    };

    int tok = p.start_token;
    int step = 0;
    bool stop = false;
    pf_p1(0);
    cp_commit();
    for (; step < p.n_steps && !stop; ++step) {
        const int t = step;
        if (tok < 0 || tok >= V) {
            if (threadIdx.x == 0) atomicCAS(p.status, DEV_OK, DEV_BAD_TOKEN);
            cp_wait_all();
            return;
        }
        const float* emb = p.embed + (size_t)tok * d;
        for (int l = 0; l < L; ++l) {
            const DecodeLayerW W = p.layers[l];
            const float* xin = (l == 0) ? emb : p.xb + (size_t)((l - 1) & 1) * d;
            float* xout = p.xb + (size_t)(l & 1) * d;
            const bool coh = l > 0;

            // ---- P1: LN1 + QKV + RoPE + KV append
            cta_ln(xin, coh, nullptr, nullptr, 0, d, W.ln1, hs, red);
            land();
            {
                int k = 0;
                for (int it = gw; it < npairs; it += NW, ++k) {
                    const int r = it << 1;
                    float a0 = sdot(reg + (size_t)k * 2 * d, hs, d, lane);
                    float a1 = sdot(reg + (size_t)k * 2 * d + d, hs, d, lane);
                    if (lane == 0) {
                        const bool isq = r < HD;
                        const bool isk = !isq && r < HD + KVD;
                        const int c = (isq ? r : (isk ? r - HD : r - HD - KVD)) % hd;
                        if ((isq || isk) && c < p.nd) {
                            const int i = c >> 1;
                            const float cs = p.rope_cos[(size_t)t * half_nd + i];
                            const float sn = p.rope_sin[(size_t)t * half_nd + i];
                            const float b0 = a0 * cs - a1 * sn;
                            const float b1 = a0 * sn + a1 * cs;
                            a0 = b0;
                            a1 = b1;
                        }
                        if (isq) {
                            p.qbuf[r] = a0;
                            p.qbuf[r + 1] = a1;
                        } else {
                            const int j = r - HD;
                            p.kvnew[j] = a0;
                            p.kvnew[j + 1] = a1;
                            const int kv = j / KVD;
                            const int c2 = j - kv * KVD;
                            const int head = c2 / hd, dim = c2 - head * hd;
                            const size_t idx = (((size_t)l * KVH + head) * p.t_cap + t) * hd + dim;
                            void* base = kv ? p.self_v : p.self_k;
                            if (p.kv_f16) {
                                __half* hb = reinterpret_cast<__half*>(base);
                                hb[idx] = __float2half_rn(a0);
                                hb[idx + 1] = __float2half_rn(a1);
                            } else {
                                float* fb = reinterpret_cast<float*>(base);
                                fb[idx] = a0;
                                fb[idx + 1] = a1;
                            }
                        }
                    }
                }
            }
            __syncwarp();
            stamp();
            pf_p2(l, t);
            cp_commit();
            if (!sync()) { cp_wait_all(); return; }

            // ---- P2: self-attention chunk partials
            for (int i = threadIdx.x; i < 2 * KVD; i += blockDim.x) fks[i] = ldcg(p.kvnew + i);
            stage(p.qbuf, vec, HD);
            land();
            {
                const int nck = (t + 1 + CH - 1) / CH;
                int k = 0;
                for (int it = gw; it < H * nck; it += NW, ++k) {
                    const int h = it / nck, c = it - h * nck;
                    const int kvh = h / rep;
                    const int j0 = c * CH, nk = min(CH, t + 1 - j0);
                    float m = -INFINITY, lsum = 0.f, acc[MAXHD / 32];
#pragma unroll
                    for (int i = 0; i < MAXHD / 32; ++i) acc[i] = 0.f;
                    const float* fk = p.kvnew + kvh * hd;
                    const float* fv = p.kvnew + KVD + kvh * hd;
                    if (k == 0) {
                        const int fr = (t - j0 < nk) ? t - j0 : -1;
                        const unsigned char* kr = reinterpret_cast<const unsigned char*>(reg);
                        if (p.kv_f16)
                            attend_fast<HDT, true>(vec + h * HDT, kr, kr + CH * HDT * 2, nk, fr, fks + kvh * HDT,
                                                   fks + KVD + kvh * HDT, p.scale, pws + wid * 32, lane, m, lsum,
                                                   acc[0], acc[1]);
                        else
                            attend_fast<HDT, false>(vec + h * HDT, kr, kr + CH * HDT * 4, nk, fr, fks + kvh * HDT,
                                                    fks + KVD + kvh * HDT, p.scale, pws + wid * 32, lane, m, lsum,
                                                    acc[0], acc[1]);
                    } else {
                        const size_t cb = ((size_t)l * KVH + kvh) * p.t_cap * hd * kvesz;
                        attend(false,vec + h * hd, reinterpret_cast<const char*>(p.self_k) + cb,
                                      reinterpret_cast<const char*>(p.self_v) + cb, 0, j0, nk, hd, p.scale, p.kv_f16,
                                      fk, fv, t, lane, m, lsum, acc);
                    }
                    float* out = p.spart + (size_t)it * (hd + 2);
                    if (lane == 0) {
                        out[0] = m;
                        out[1] = lsum;
                    }
#pragma unroll
                    for (int i = 0; i < MAXHD / 32; ++i) {
                        const int cc = 2 * lane + i;
                        if (cc < hd) out[2 + cc] = acc[i];
                    }
                }
            }
            __syncwarp();
            stamp();
            pf_orows(W.wo);
            cp_commit();
            if (!sync()) { cp_wait_all(); return; }

            // ---- P3: combine self-attention (every CTA) + head-split O projection
            {
                const int nck = (t + 1 + CH - 1) / CH;
                for (int it = threadIdx.x; it < HD; it += blockDim.x) {
                    const int h = it / hd, c = it - h * hd;
                    const float* base = p.spart + (size_t)h * nck * (hd + 2);
                    float M = -INFINITY, Ls = 0.f, O = 0.f;
#pragma unroll 8
                    for (int k = 0; k < nck; ++k) {
                        const float* pk = base + (size_t)k * (hd + 2);
                        merge_partial(ldcg(pk), ldcg(pk + 1), ldcg(pk + 2 + c), M, Ls, O);
                    }
                    comb[it] = O / Ls;
                }
                __syncthreads();
                land();
                int k = 0;
                for (int r = gw; r < d; r += NW, ++k) {
                    const float v = sdot(reg + (size_t)k * HD, comb, HD, lane);
                    if (lane == 0) p.x1[r] = (coh ? ldcg(xin + r) : xin[r]) + v;
                }
            }
            __syncwarp();
            stamp();
            pf_p4(l);
            cp_commit();
            if (!sync()) { cp_wait_all(); return; }

            // ---- P4: x1 = x + sum_h ps, LN2 + cross Q
            cta_ln(p.x1, true, nullptr, nullptr, 0, d, W.ln2, hs, red);
            land();
            {
                int k = 0;
                for (int r = gw; r < HD; r += NW, ++k) {
                    const float v = sdot(reg + (size_t)k * d, hs, d, lane);
                    if (lane == 0) {
                        p.qc[r] = v;
                        if (p.qc_trace) p.qc_trace[((size_t)step * L + l) * HD + r] = v;
                    }
                }
            }
            __syncwarp();
            stamp();
            pf_p5(l, step);
            cp_commit();
            if (!sync()) { cp_wait_all(); return; }

            // ---- P5: cross-attention chunk partials, pre-combined per CTA
            stage(p.qc, vec, HD);
            land();
            {
                const int f16 = (step == 0) ? 0 : p.kv_f16;
                const int esz = f16 ? 2 : 4;
                const void* src = (step == 0) ? (const void*)p.cross32 : p.cross_stored;
                for (int rd = 0; rd < cm.rounds; ++rd) {
                    const int it = rd * NW + gw;
                    float m = -INFINITY, lsum = 0.f, acc[MAXHD / 32];
#pragma unroll
                    for (int i = 0; i < MAXHD / 32; ++i) acc[i] = 0.f;
                    int head = -1;
                    if (it < cm.items) {
                        const int h = it / cm.nck, c = it - h * cm.nck;
                        const int kvh = h / rep;
                        const int j0 = c * CH, nk = min(CH, p.M - j0);
                        head = h;
                        if (rd == 0) {
                            const unsigned char* kr = reinterpret_cast<const unsigned char*>(reg);
                            if (f16)
                                attend_fast<HDT, true>(vec + h * HDT, kr, kr + CH * HDT * 2, nk, -1, nullptr, nullptr,
                                                       p.scale, pws + wid * 32, lane, m, lsum, acc[0], acc[1]);
                            else
                                attend_fast<HDT, false>(vec + h * HDT, kr, kr + CH * HDT * 4, nk, -1, nullptr, nullptr,
                                                        p.scale, pws + wid * 32, lane, m, lsum, acc[0], acc[1]);
                        } else {
                            const size_t kb = (((size_t)l * 2 + 0) * KVH + kvh) * p.m_cap * hd * esz;
                            const size_t vb = (((size_t)l * 2 + 1) * KVH + kvh) * p.m_cap * hd * esz;
                            attend(false,vec + h * hd, reinterpret_cast<const char*>(src) + kb,
                                          reinterpret_cast<const char*>(src) + vb, 0, j0, nk, hd, p.scale, f16,
                                          nullptr, nullptr, -1, lane, m, lsum, acc);
                        }
                    }
                    float* wp = wpart + (size_t)wid * (hd + 2);
                    if (lane == 0) {
                        wp[0] = m;
                        wp[1] = lsum;
                        s_whead[wid] = head;
                    }
#pragma unroll
                    for (int i = 0; i < MAXHD / 32; ++i) {
                        const int cc = 2 * lane + i;
                        if (cc < hd) wp[2 + cc] = acc[i];
                    }
                    __syncthreads();
                    const int first = s_whead[0];
                    if (first >= 0) {
                        int last = first;
                        for (int w = 1; w < NWB; ++w) last = max(last, s_whead[w]);
                        const int nslot = last - first + 1;
                        for (int e = threadIdx.x; e < nslot * (hd + 2); e += blockDim.x) {
                            const int s = e / (hd + 2), c = e - s * (hd + 2);
                            const int hh = first + s;
                            float mx = -INFINITY;
                            for (int w = 0; w < NWB; ++w)
                                if (s_whead[w] == hh) mx = fmaxf(mx, wpart[w * (hd + 2)]);
                            float v;
                            if (c == 0) {
                                v = mx;
                            } else {
                                v = 0.f;
                                for (int w = 0; w < NWB; ++w) {
                                    if (s_whead[w] != hh) continue;
                                    const float f = expf(wpart[w * (hd + 2)] - mx);
                                    v = fmaf(wpart[w * (hd + 2) + c], f, v);
                                }
                            }
                            p.cpart[(((size_t)rd * G + blockIdx.x) * NWB + s) * (hd + 2) + c] = v;
                        }
                    }
                    __syncthreads();
                }
            }
            stamp();
            pf_orows(W.wco);
            cp_commit();
            if (!sync()) { cp_wait_all(); return; }

            // ---- P6: combine cross-attention (every CTA) + head-split cross O projection
            {
                for (int it = threadIdx.x; it < HD; it += blockDim.x) {
                    const int h = it / hd, c = it - h * hd;
                    float M = -INFINITY, Ls = 0.f, O = 0.f;
                    // head h's chunks are items [h*nck, h*nck + nck); round rd holds items
                    // [rd*NW, rd*NW + NW) and CTA b of the round the 8 items from rd*NW + 8b
                    for (int rd = 0; rd < cm.rounds; ++rd) {
                        const int lo = max(h * cm.nck, rd * NW), hi = min(h * cm.nck + cm.nck, rd * NW + NW);
                        if (lo >= hi) continue;
                        const int b0 = (lo - rd * NW) / NWB, b1 = (hi - 1 - rd * NW) / NWB;
#pragma unroll 4
                        for (int b = b0; b <= b1; ++b) {
                            const int first_head = (rd * NW + b * NWB) / cm.nck;
                            const float* pe = p.cpart + ((((size_t)rd * G + b) * NWB) + (h - first_head)) * (hd + 2);
                            merge_partial(ldcg(pe), ldcg(pe + 1), ldcg(pe + 2 + c), M, Ls, O);
                        }
                    }
                    comb[it] = O / Ls;
                }
                __syncthreads();
                land();
                int k = 0;
                for (int r = gw; r < d; r += NW, ++k) {
                    const float v = sdot(reg + (size_t)k * HD, comb, HD, lane);
                    if (lane == 0) p.x2[r] = ldcg(p.x1 + r) + v;
                }
            }
            __syncwarp();
            stamp();
            pf_p7(l);
            cp_commit();
            if (!sync()) { cp_wait_all(); return; }

            // ---- P7: x2 = x1 + sum_h pc, LN3 + fc1 + SwiGLU
            cta_ln(p.x2, true, nullptr, nullptr, 0, d, W.ln3, hs, red);
            land();
            {
                const int j0 = gw * per7, j1 = min(I, j0 + per7);
                for (int j = j0; j < j1; ++j) {
                    const float a = sdot(reg + (size_t)(2 * (j - j0)) * d, hs, d, lane);
                    const float b = sdot(reg + (size_t)(2 * (j - j0) + 1) * d, hs, d, lane);
                    if (lane == 0) p.gbuf[j] = (a + W.b1[j]) * silu(b + W.b1[j + I]);
                }
            }
            __syncwarp();
            stamp();
            pf_p8(l);
            cp_commit();
            if (!sync()) { cp_wait_all(); return; }

            // ---- P8: fc2 + bias + residual -> xout
            stage(p.gbuf, vec, I);
            land();
            {
                int k = 0;
                for (int r = gw; r < d; r += NW, ++k) {
                    const float v = sdot(reg + (size_t)k * I, vec, I, lane);
                    if (lane == 0) xout[r] = ldcg(p.x2 + r) + (v + W.b2[r]);
                }
            }
            __syncwarp();
            stamp();
            if (l + 1 < L) pf_p1(l + 1);
            else if (gw * 4 < V) pf_lm(gw, 0);
            cp_commit();
            if (!sync()) { cp_wait_all(); return; }
        }

        // ---- F: final LN + LM head + argmax
        cta_ln(p.xb + (size_t)((L - 1) & 1) * d, true, nullptr, nullptr, 0, d, p.final_ln, hs, red);
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        {
            // 3-stage cp.async pipeline over this warp's 4-row groups: group gw sits in
            // buffer 0 (prefetched during P8), the next two are always in flight
            if (4 * (gw + NW) < V) pf_lm(gw + NW, 1);
            cp_commit();
            int k = 0;
            for (int g = gw; 4 * g < V; g += NW, ++k) {
                if (4 * (g + 2 * NW) < V) pf_lm(g + 2 * NW, (k + 2) % 3);
                cp_commit();
                cp_wait_two_pending();
                __syncwarp();
                const int r0 = 4 * g, nr = min(4, V - r0);
                const float* rows = reg + (size_t)(k % 3) * 4 * d;
                for (int r = 0; r < nr; ++r) {
                    const float v = sdot(rows + (size_t)r * d, hs, d, lane);
                    const float key = p.inv_temp > 0.f
                                          ? v * p.inv_temp + gumbel_noise(p.seed, (unsigned)step, (unsigned)(r0 + r))
                                          : v;
                    if (key > bv) {
                        bv = key;
                        bi = r0 + r;
                    }
                    if (p.logits_out && lane == 0) p.logits_out[(size_t)step * V + r0 + r] = v;
                }
                __syncwarp();
            }
            cp_wait_all();
            __syncwarp();
        }
        if (lane == 0) {
            s_bv[wid] = bv;
            s_bi[wid] = bi;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float v = s_bv[0];
            int i = s_bi[0];
            for (int w = 1; w < NWB; ++w) {
                if (s_bv[w] > v || (s_bv[w] == v && s_bi[w] < i)) {
                    v = s_bv[w];
                    i = s_bi[w];
                }
            }
            p.amax_val[blockIdx.x] = v;
            p.amax_idx[blockIdx.x] = i;
        }
        if (step + 1 < p.n_steps) pf_p1(0);
        cp_commit();
        if (!sync()) { cp_wait_all(); return; }
        if (wid == 0) {
            float v = -INFINITY;
            int i = 0x7fffffff;
            for (int b = lane; b < G; b += 32) {
                const float vb = ldcg(p.amax_val + b);
                const int ib = __ldcg(p.amax_idx + b);
                if (vb > v || (vb == v && ib < i)) {
                    v = vb;
                    i = ib;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float vo = __shfl_xor_sync(FULL, v, o);
                const int io = __shfl_xor_sync(FULL, i, o);
                if (vo > v || (vo == v && io < i)) {
                    v = vo;
                    i = io;
                }
            }
            if (lane == 0) s_bi[0] = i;
        }
        __syncthreads();
        const int best = s_bi[0];
        if (blockIdx.x == 0 && threadIdx.x == 0) p.ids_out[step] = best;
        if (!p.forced && best == p.eos) {
            if (blockIdx.x == 0 && threadIdx.x == 0) *p.hit_eos = 1;
            stop = true;
        }
        tok = p.teacher ? p.teacher[step] : best;
        __syncthreads();
    }
    cp_wait_all();
    if (blockIdx.x == 0 && threadIdx.x == 0) *p.n_done = step;
}

size_t region_bytes_for(const DecodeParams& p, int grid) {
    const int NW = grid * NWB;
    const int HD = p.H * p.hd, KVD = p.KVH * p.hd;
    const int npairs = (HD + 2 * KVD) / 2;
    auto cdiv = [](int a, int b) { return (a + b - 1) / b; };
    size_t r = 0;
    r = std::max<size_t>(r, (size_t)cdiv(npairs, NW) * 2 * p.d * 4);
    r = std::max<size_t>(r, (size_t)2 * CH * p.hd * 4);  // self / cross chunk, fp32 worst case
    r = std::max<size_t>(r, (size_t)cdiv(p.d, NW) * HD * 4);
    r = std::max<size_t>(r, (size_t)cdiv(HD, NW) * p.d * 4);
    r = std::max<size_t>(r, (size_t)cdiv(p.I, NW) * 2 * p.d * 4);
    r = std::max<size_t>(r, (size_t)cdiv(p.d, NW) * p.I * 4);
    r = std::max<size_t>(r, (size_t)3 * 4 * p.d * 4);
    return (r + 15) & ~(size_t)15;
}

}  // namespace

int decode_b1_block_threads() { return NT; }
int decode_chunk_keys() { return CH; }

size_t decode_b1_spart_floats(int H, int hd, int t_cap) {
    return (size_t)H * ((t_cap + CH) / CH + 1) * (hd + 2);
}

size_t decode_b1_cpart_floats(int H, int hd, int m_cap, int grid) {
    const int NW = grid * NWB;
    const int items = H * ((m_cap + CH - 1) / CH);
    const int rounds = std::max(1, (items + NW - 1) / NW);
    return (size_t)rounds * grid * NWB * (hd + 2);
}

cudaError_t launch_decode_b1(const DecodeParams& p, int grid, cudaStream_t stream) {
    // fp16 K/V rows must be whole 16-byte cp.async units: head_dim % 8 == 0
    if ((p.d & 3) || (p.hd & 7) || (p.I & 3) || p.H % p.KVH || p.hd > MAXHD || 2 * p.H > 32)
        return cudaErrorInvalidValue;
    DecodeParams pc = p;
    pc.region_bytes = (int)region_bytes_for(p, grid);
    const int HD = p.H * p.hd;
    const int vec_n = std::max(std::max(p.I, HD), p.d);
    const int KVD = p.KVH * p.hd;
    const size_t floats = (size_t)((p.d + 3) & ~3) + ((vec_n + 3) & ~3) + ((HD + 3) & ~3) +
                          (((size_t)NWB * (p.hd + 2) + 3) & ~(size_t)3) + ((2 * KVD + 3) & ~3) + NWB * 32;
    const size_t smem = floats * 4 + (size_t)NWB * pc.region_bytes;
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    const void* fn = nullptr;
    switch (p.hd) {  // head_dim is a compile-time constant inside the kernel
        case 32: fn = (const void*)decode_b1_kernel<32>; break;
        case 40: fn = (const void*)decode_b1_kernel<40>; break;
        case 48: fn = (const void*)decode_b1_kernel<48>; break;
        case 64: fn = (const void*)decode_b1_kernel<64>; break;
        default: return cudaErrorInvalidValue;
    }
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    void* args[] = {&pc};
    ++launch_counter();
    return cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(NT), args, smem, stream);
}

bool decode_b1_supports_head_dim(int hd) { return hd == 32 || hd == 40 || hd == 48 || hd == 64; }

cudaError_t preload_decode_b1(int hd) {
    cudaFuncAttributes a;
    switch (hd) {
        case 32: return cudaFuncGetAttributes(&a, decode_b1_kernel<32>);
        case 40: return cudaFuncGetAttributes(&a, decode_b1_kernel<40>);
        case 48: return cudaFuncGetAttributes(&a, decode_b1_kernel<48>);
        case 64: return cudaFuncGetAttributes(&a, decode_b1_kernel<64>);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace msb
