// Batch-1 greedy decode as ONE persistent cooperative kernel (fp32 weights).
//
// A whole forced-length (or EOS-terminated) token loop runs inside a single launch: the
// argmax of step t is fed back as the embedding row of step t+1 on the device, so there
// is no host round trip per token (the reference syncs with `.item()` every token,
// Sources/MoonshineMLX/MoonshineModel.swift:216-229).  Each decoder layer
// (MoonshineLayers.swift:350-379) is a sequence of grid-wide phases separated by a
// bounded grid barrier; every phase spreads its weight rows over all warps of the GPU
// with 128-bit streaming loads (batch-1 decode is a weight-bandwidth problem):
//
//   P1  LN1 (each CTA, redundantly) + QKV GEMV + interleaved partial RoPE + KV append
//   P2  self-attention, one CTA per head, over [cache(fp16|fp32) ; this step's fp32 K/V]
//   P3  O projection + residual
//   P4  LN2 + cross-attention Q GEMV
//   P5  cross-attention partials over 32-key chunks (flash-decode split)
//   P6  combine partials -> cross O projection + residual
//   P7  LN3 + fc1 GEMV + bias + SwiGLU (value = first half, gate = second half)
//   P8  fc2 GEMV + bias + residual
//   F   final LN + LM-head GEMV with per-CTA argmax, then a grid argmax (ties -> lowest id)
//
// KV rounding follows the reference's fp16 cache rules (MoonshineLayers.swift:106-125):
// the current position's K/V enter attention in fp32 and are stored rounded; cross K/V
// are fp32 at step 0 and the stored (rounded) copy afterwards.
#include "common.cuh"
#include "kernels.h"

namespace msb {

namespace {

constexpr int DEC_THREADS = 512;
constexpr int DEC_WARPS = DEC_THREADS / 32;
constexpr int CHUNK = 32;

// Dot product of a weight row (global, read once) with a vector staged in shared memory.
__device__ __forceinline__ float dot_row(const float* __restrict__ w, const float* v, int n,
                                         int lane) {
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const float4* v4 = reinterpret_cast<const float4*>(v);
    float acc = 0.f;
    for (int i = lane; i < (n >> 2); i += 32) {
        const float4 a = ld_stream4(w4 + i);
        const float4 b = v4[i];
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
        acc = fmaf(a.z, b.z, acc);
        acc = fmaf(a.w, b.w, acc);
    }
    return warp_sum(acc);
}

// Four independent rows at once (more loads in flight per warp).
__device__ __forceinline__ void dot_rows4(const float* __restrict__ w, int ld, int nrows,
                                          const float* v, int n, int lane, float out[4]) {
    const float4* v4 = reinterpret_cast<const float4*>(v);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int i = lane; i < (n >> 2); i += 32) {
        const float4 b = v4[i];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            if (r < nrows) {
                const float4 a = ld_stream4(reinterpret_cast<const float4*>(w + (size_t)r * ld) + i);
                acc[r] = fmaf(a.x, b.x, acc[r]);
                acc[r] = fmaf(a.y, b.y, acc[r]);
                acc[r] = fmaf(a.z, b.z, acc[r]);
                acc[r] = fmaf(a.w, b.w, acc[r]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) out[r] = warp_sum(acc[r]);
}

constexpr int MAXHD = 64;

// One warp attends a query (in shared memory) over keys [j0, j0+nk) of one head.
// Lanes own keys for the scores and dims for the weighted sum; (m, l, acc) is an online
// softmax state merged across calls.  `fresh_*` (fp32) replace the cached row `fresh_j`.
__device__ __forceinline__ void attend_rows(const float* q, const void* kb, const void* vb, int j0,
                                            int nk, int hd, float scale, int f16,
                                            const float* fresh_k, const float* fresh_v,
                                            int fresh_j, int lane, float& m, float& l,
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
            const uint4* kr = reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(kb) + (size_t)j * hd);
            uint4 rk[MAXHD / 8];
#pragma unroll
            for (int e = 0; e < MAXHD / 8; ++e)
                if (e * 8 < hd) rk[e] = __ldcg(kr + e);
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
            const float4* kr = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(kb) + (size_t)j * hd);
            float4 rk[MAXHD / 4];
#pragma unroll
            for (int e = 0; e < MAXHD / 4; ++e)
                if (e * 4 < hd) rk[e] = __ldcg(kr + e);
#pragma unroll
            for (int e = 0; e < MAXHD / 4; ++e) {
                if (e * 4 < hd) {
                    const float4 a = *reinterpret_cast<const float4*>(q + 4 * e);
                    dot = fmaf(a.x, rk[e].x, fmaf(a.y, rk[e].y, fmaf(a.z, rk[e].z, fmaf(a.w, rk[e].w, dot))));
                }
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
#pragma unroll 8
    for (int jj = 0; jj < nk; ++jj) {
        const float pp = __shfl_sync(FULL, pj, jj);
        const int row = j0 + jj;
#pragma unroll
        for (int i = 0; i < MAXHD / 32; ++i) {
            const int c = lane + 32 * i;
            if (c < hd) {
                float vv;
                if (row == fresh_j) vv = ldcg(fresh_v + c);
                else if (f16) vv = __half2float(__ldcg(reinterpret_cast<const __half*>(vb) + (size_t)row * hd + c));
                else vv = ldcg(reinterpret_cast<const float*>(vb) + (size_t)row * hd + c);
                acc[i] = fmaf(pp, vv, acc[i]);
            }
        }
    }
    m = mn;
}

// Self-attention chunk: cache rows below `pos`, the fresh fp32 row at `pos`.
__device__ __forceinline__ void warp_chunk(const float* q, const void* kcache, const void* vcache,
                                           size_t cbase, int j0, int nk, int hd, float scale,
                                           int f16, bool /*self*/, const float* fresh_k,
                                           const float* fresh_v, int pos, int lane, float& m,
                                           float& l, float acc[MAXHD / 32]) {
    const void* kb = f16 ? (const void*)(reinterpret_cast<const __half*>(kcache) + cbase)
                         : (const void*)(reinterpret_cast<const float*>(kcache) + cbase);
    const void* vb = f16 ? (const void*)(reinterpret_cast<const __half*>(vcache) + cbase)
                         : (const void*)(reinterpret_cast<const float*>(vcache) + cbase);
    attend_rows(q, kb, vb, j0, nk, hd, scale, f16, fresh_k, fresh_v, pos, lane, m, l, acc);
}

// Cross-attention chunk over the per-utterance K/V (no fresh row).
__device__ __forceinline__ void warp_chunk_kv(const float* q, const void* kv, size_t kb_off,
                                              size_t vb_off, int j0, int nk, int hd, float scale,
                                              int f16, int lane, float& m, float& l,
                                              float acc[MAXHD / 32]) {
    const void* kb = f16 ? (const void*)(reinterpret_cast<const __half*>(kv) + kb_off)
                         : (const void*)(reinterpret_cast<const float*>(kv) + kb_off);
    const void* vb = f16 ? (const void*)(reinterpret_cast<const __half*>(kv) + vb_off)
                         : (const void*)(reinterpret_cast<const float*>(kv) + vb_off);
    attend_rows(q, kb, vb, j0, nk, hd, scale, f16, nullptr, nullptr, -1, lane, m, l, acc);
}

// LayerNorm of a d-vector into shared memory, computed by every CTA.
__device__ __forceinline__ void cta_layernorm(const float* x, bool coherent, const float* w,
                                              float* out, int d, float* red) {
    float s = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float v = coherent ? ldcg(x + i) : x[i];
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

__global__ void __launch_bounds__(DEC_THREADS, 1) decode_b1_kernel(DecodeParams p) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float red[32];
    __shared__ float s_bv[DEC_WARPS];
    __shared__ int s_bi[DEC_WARPS];

    const int d = p.d, H = p.H, KVH = p.KVH, hd = p.hd, I = p.I, V = p.V;
    const int HD = H * hd, KVD = KVH * hd;
    const int rep = H / KVH;
    const int half_nd = p.nd >> 1;
    const int vec_n = max(max(I, HD), d);
    float* hs = sm;                                // [d]
    float* vec = hs + ((d + 3) & ~3);              // [vec_n]
    float* sc = vec + ((vec_n + 3) & ~3);          // [t_cap] scores / partial outputs
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int gw = blockIdx.x * DEC_WARPS + wid;
    const int NW = gridDim.x * DEC_WARPS;
    const int nchunks = (p.M + CHUNK - 1) / CHUNK;
    unsigned epoch = 0;

    int tok = p.start_token;
    int step = 0;
    bool stop = false;
    for (; step < p.n_steps && !stop; ++step) {
        const int pos = step;
        if (tok < 0 || tok >= V) {
            if (threadIdx.x == 0) atomicCAS(p.status, DEV_OK, DEV_BAD_TOKEN);
            return;
        }
        const float* emb = p.embed + (size_t)tok * d;
        for (int l = 0; l < p.L; ++l) {
            const DecodeLayerW W = p.layers[l];
            const float* xin = (l == 0) ? emb : p.x;
            const bool xin_coh = l > 0;

            // ---- P1: LN1 + QKV + RoPE + KV append
            cta_layernorm(xin, xin_coh, W.ln1, hs, d, red);
            const int npairs = (HD + 2 * KVD) >> 1;
            for (int it = gw; it < npairs; it += NW) {
                const int r = it << 1;
                float a0 = dot_row(W.wqkv + (size_t)r * d, hs, d, lane);
                float a1 = dot_row(W.wqkv + (size_t)(r + 1) * d, hs, d, lane);
                if (lane == 0) {
                    const bool isq = r < HD;
                    const bool isk = !isq && r < HD + KVD;
                    const int c = (isq ? r : (isk ? r - HD : r - HD - KVD)) % hd;
                    if ((isq || isk) && c < p.nd) {
                        const int i = c >> 1;
                        const float cs = p.rope_cos[(size_t)pos * half_nd + i];
                        const float sn = p.rope_sin[(size_t)pos * half_nd + i];
                        const float b0 = a0 * cs - a1 * sn;
                        const float b1 = a0 * sn + a1 * cs;
                        a0 = b0;
                        a1 = b1;
                    }
                    if (isq) {
                        p.qbuf[r] = a0;
                        p.qbuf[r + 1] = a1;
                    } else {
                        const int j = r - HD;             // [0, 2*KVD)
                        p.kvnew[j] = a0;
                        p.kvnew[j + 1] = a1;
                        const int kv = j / KVD;
                        const int c2 = j - kv * KVD;
                        const int head = c2 / hd, dim = c2 - head * hd;
                        const size_t idx = (((size_t)l * KVH + head) * p.t_cap + pos) * hd + dim;
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
            if (!grid_barrier(p.bar_count, p.status, epoch)) return;

            // ---- P2: self-attention, one CTA per head; warp w takes key chunks w, w+16, ...
            for (int h = blockIdx.x; h < H; h += gridDim.x) {
                const int kvh = h / rep;
                const int n = pos + 1;
                stage(p.qbuf + h * hd, vec, hd);
                const size_t cbase = ((size_t)l * KVH + kvh) * p.t_cap * hd;
                float m = -INFINITY, lsum = 0.f, acc[MAXHD / 32];
#pragma unroll
                for (int i = 0; i < MAXHD / 32; ++i) acc[i] = 0.f;
                for (int j0 = wid * CHUNK; j0 < n; j0 += DEC_WARPS * CHUNK)
                    warp_chunk(vec, p.self_k, p.self_v, cbase, j0, min(CHUNK, n - j0), hd, p.scale,
                               p.kv_f16, true, p.kvnew + kvh * hd, p.kvnew + KVD + kvh * hd, pos,
                               lane, m, lsum, acc);
                float* po = sc;  // [DEC_WARPS][hd + 2]
                if (lane == 0) {
                    po[wid * (hd + 2)] = m;
                    po[wid * (hd + 2) + 1] = lsum;
                }
#pragma unroll
                for (int i = 0; i < MAXHD / 32; ++i) {
                    const int c = lane + 32 * i;
                    if (c < hd) po[wid * (hd + 2) + 2 + c] = acc[i];
                }
                __syncthreads();
                for (int c = threadIdx.x; c < hd; c += blockDim.x) {
                    float mx = -INFINITY;
                    for (int w = 0; w < DEC_WARPS; ++w) mx = fmaxf(mx, po[w * (hd + 2)]);
                    float L = 0.f, O = 0.f;
                    for (int w = 0; w < DEC_WARPS; ++w) {
                        const float mw = po[w * (hd + 2)];
                        if (mw == -INFINITY) continue;
                        const float f = expf(mw - mx);
                        L = fmaf(po[w * (hd + 2) + 1], f, L);
                        O = fmaf(po[w * (hd + 2) + 2 + c], f, O);
                    }
                    p.attn[h * hd + c] = O / L;
                }
                __syncthreads();
            }
            if (!grid_barrier(p.bar_count, p.status, epoch)) return;

            // ---- P3: O projection + residual
            stage(p.attn, vec, HD);
            for (int r = gw; r < d; r += NW) {
                const float v = dot_row(W.wo + (size_t)r * HD, vec, HD, lane);
                if (lane == 0) p.x[r] = (xin_coh ? ldcg(xin + r) : xin[r]) + v;
            }
            if (!grid_barrier(p.bar_count, p.status, epoch)) return;

            // ---- P4: LN2 + cross Q
            cta_layernorm(p.x, true, W.ln2, hs, d, red);
            for (int r = gw; r < HD; r += NW) {
                const float v = dot_row(W.wcq + (size_t)r * d, hs, d, lane);
                if (lane == 0) p.qbuf[r] = v;
            }
            if (!grid_barrier(p.bar_count, p.status, epoch)) return;

            // ---- P5: cross-attention partials over 32-key chunks
            {
                const int f16 = (step == 0) ? 0 : p.kv_f16;
                const void* kvsrc = (step == 0) ? (const void*)p.cross32 : p.cross_stored;
                stage(p.qbuf, vec, HD);
                for (int it = gw; it < H * nchunks; it += NW) {
                    const int h = it / nchunks, c = it - h * nchunks;
                    const int kvh = h / rep;
                    const size_t kb = (((size_t)l * 2 + 0) * KVH + kvh) * p.m_cap * hd;
                    const size_t vb = (((size_t)l * 2 + 1) * KVH + kvh) * p.m_cap * hd;
                    float m = -INFINITY, lsum = 0.f, acc[MAXHD / 32];
#pragma unroll
                    for (int i = 0; i < MAXHD / 32; ++i) acc[i] = 0.f;
                    warp_chunk_kv(vec + h * hd, kvsrc, kb, vb, c * CHUNK, min(CHUNK, p.M - c * CHUNK),
                                  hd, p.scale, f16, lane, m, lsum, acc);
                    float* out = p.part + (size_t)it * (hd + 2);
                    if (lane == 0) {
                        out[0] = m;
                        out[1] = lsum;
                    }
#pragma unroll
                    for (int i = 0; i < MAXHD / 32; ++i) {
                        const int cc = lane + 32 * i;
                        if (cc < hd) out[2 + cc] = acc[i];
                    }
                }
            }
            if (!grid_barrier(p.bar_count, p.status, epoch)) return;

            // ---- P6a: combine partials, one warp per head
            for (int h = gw; h < H; h += NW) {
                const float* base = p.part + (size_t)h * nchunks * (hd + 2);
                float mx = -INFINITY;
                for (int k = lane; k < nchunks; k += 32) mx = fmaxf(mx, ldcg(base + (size_t)k * (hd + 2)));
                mx = warp_max(mx);
                float L = 0.f;
                for (int k = lane; k < nchunks; k += 32) {
                    const float* pk = base + (size_t)k * (hd + 2);
                    L = fmaf(ldcg(pk + 1), expf(ldcg(pk) - mx), L);
                }
                L = warp_sum(L);
                for (int cb = 0; cb < hd; cb += 32) {
                    const int c = cb + lane;
                    float O = 0.f;
                    if (c < hd) {
#pragma unroll 4
                        for (int k = 0; k < nchunks; ++k) {
                            const float* pk = base + (size_t)k * (hd + 2);
                            O = fmaf(ldcg(pk + 2 + c), expf(ldcg(pk) - mx), O);
                        }
                        p.attn[h * hd + c] = O / L;
                    }
                }
            }
            if (!grid_barrier(p.bar_count, p.status, epoch)) return;

            // ---- P6b: cross O projection + residual
            stage(p.attn, vec, HD);
            for (int r = gw; r < d; r += NW) {
                const float v = dot_row(W.wco + (size_t)r * HD, vec, HD, lane);
                if (lane == 0) p.x[r] = ldcg(p.x + r) + v;
            }
            if (!grid_barrier(p.bar_count, p.status, epoch)) return;

            // ---- P7: LN3 + fc1 + SwiGLU
            cta_layernorm(p.x, true, W.ln3, hs, d, red);
            for (int j = gw; j < I; j += NW) {
                const float a = dot_row(W.w1 + (size_t)j * d, hs, d, lane);
                const float b = dot_row(W.w1 + (size_t)(j + I) * d, hs, d, lane);
                if (lane == 0) p.gbuf[j] = (a + W.b1[j]) * silu(b + W.b1[j + I]);
            }
            if (!grid_barrier(p.bar_count, p.status, epoch)) return;

            // ---- P8: fc2 + bias + residual
            stage(p.gbuf, vec, I);
            for (int r = gw; r < d; r += NW) {
                const float v = dot_row(W.w2 + (size_t)r * I, vec, I, lane);
                if (lane == 0) p.x[r] = ldcg(p.x + r) + W.b2[r] + v;
            }
            if (!grid_barrier(p.bar_count, p.status, epoch)) return;
        }

        // ---- F: final LN + LM head + argmax
        cta_layernorm(p.x, true, p.final_ln, hs, d, red);
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int r0 = gw * 4; r0 < V; r0 += NW * 4) {
            const int nr = min(4, V - r0);
            float o[4];
            dot_rows4(p.lm_head + (size_t)r0 * d, d, nr, hs, d, lane, o);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                if (r < nr) {
                    if (o[r] > bv) {
                        bv = o[r];
                        bi = r0 + r;
                    }
                    if (p.logits_out && lane == 0) p.logits_out[(size_t)step * V + r0 + r] = o[r];
                }
            }
        }
        if (lane == 0) {
            s_bv[wid] = bv;
            s_bi[wid] = bi;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float v = s_bv[0];
            int i = s_bi[0];
            for (int w = 1; w < DEC_WARPS; ++w) {
                if (s_bv[w] > v || (s_bv[w] == v && s_bi[w] < i)) {
                    v = s_bv[w];
                    i = s_bi[w];
                }
            }
            p.amax_val[blockIdx.x] = v;
            p.amax_idx[blockIdx.x] = i;
        }
        if (!grid_barrier(p.bar_count, p.status, epoch)) return;
        if (wid == 0) {
            float v = -INFINITY;
            int i = 0x7fffffff;
            for (int b = lane; b < (int)gridDim.x; b += 32) {
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
    if (blockIdx.x == 0 && threadIdx.x == 0) *p.n_done = step;
}

}  // namespace

int decode_b1_block_threads() { return DEC_THREADS; }
int decode_chunk_keys() { return CHUNK; }

cudaError_t launch_decode_b1(const DecodeParams& p, int grid, int block, cudaStream_t stream) {
    if (block != DEC_THREADS) return cudaErrorInvalidValue;
    if ((p.d & 3) || (p.hd & 3) || (p.I & 3) || p.H % p.KVH) return cudaErrorInvalidValue;
    const int vec_n = (p.I > p.H * p.hd ? (p.I > p.d ? p.I : p.d) : (p.H * p.hd > p.d ? p.H * p.hd : p.d));
    const size_t smem = sizeof(float) * ((size_t)((p.d + 3) & ~3) + ((vec_n + 3) & ~3) +
                                         ((p.t_cap + 3) & ~3) + (size_t)DEC_WARPS * p.hd + 64);
    static thread_local size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(decode_b1_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured = smem;
    }
    DecodeParams pc = p;
    void* args[] = {&pc};
    ++launch_counter();
    return cudaLaunchCooperativeKernel((void*)decode_b1_kernel, dim3(grid), dim3(block), args,
                                       smem, stream);
}

}  // namespace msb
