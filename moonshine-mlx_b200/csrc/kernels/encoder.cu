// Audio frontend and encoder-side kernels (fp32).
//
//   frame_features   : CMVN + asinh + Linear(frame_len -> d) + SiLU, one warp per frame
//                      (Sources/MoonshineMLX/MoonshineEncoder.swift:15-34, 84-86)
//   layernorm_rows   : LayerNorm with optional unit offset and a fused row add, used for
//                      the encoder norms and final_norm + pos_emb (prepareMemory,
//                      MoonshineDecoder.swift:39-47)
//   window_attention : sliding-window MHA, keys restricted to the band instead of a
//                      dense [T,T] additive mask (MoonshineLayers.swift:266-290); for
//                      windows the band of 32 query rows is staged in shared memory per CTA
#include "common.cuh"
#include "kernels.h"

namespace msb {

namespace {

constexpr int FF_WARPS = 8;
constexpr int MAX_FRAME = 128;

__device__ __forceinline__ void store_feature(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// One frame (warp): CMVN, asinh, Linear + SiLU into the output row o; fr is the warp's
// MAX_FRAME floats of shared memory.
template <class OutT>
__device__ __forceinline__ void frame_feature(const float* a, int frame_len, const float* __restrict__ log_k,
                                              const float* __restrict__ w, int dim, OutT* o, float* fr, int lane) {
    float s = 0.f;
    for (int i = lane; i < frame_len; i += 32) s += a[i];
    const float mean = warp_sum(s) / (float)frame_len;
    float v = 0.f;
    for (int i = lane; i < frame_len; i += 32) {
        const float c = a[i] - mean;
        v += c * c;
    }
    const float rms = sqrtf(warp_sum(v) / (float)frame_len + 1e-6f);
    const float k = expf(*log_k);
    for (int i = lane; i < frame_len; i += 32) fr[i] = asinhf(k * ((a[i] - mean) / rms));
    __syncwarp();
    for (int j = lane; j < dim; j += 32) {
        const float* wr = w + (size_t)j * frame_len;
        float acc = 0.f;
        for (int i = 0; i < frame_len; ++i) acc = fmaf(fr[i], __ldg(wr + i), acc);
        store_feature(o + j, silu(acc));
    }
}

template <class OutT>
__global__ void __launch_bounds__(FF_WARPS * 32)
frame_features_kernel(const float* __restrict__ audio, int n_frames, int frame_len,
                      const float* __restrict__ log_k, const float* __restrict__ w, int dim,
                      OutT* __restrict__ out, int ld_out) {
    __shared__ float fr[FF_WARPS][MAX_FRAME];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int f = blockIdx.x * FF_WARPS + wid;
    if (f >= n_frames) return;
    frame_feature(audio + (size_t)f * frame_len, frame_len, log_k, w, dim, out + (size_t)f * ld_out, fr[wid], lane);
}

// Frame features of FFB_FRAMES frames per CTA (fp32 out): each warp normalises frames into
// shared memory as frame_feature does, then thread j computes output j of every frame of the
// CTA, so a weight row is read once per CTA instead of once per frame.  Each output is summed
// in the same order as frame_feature's (bitwise the same values).
constexpr int FFB_FRAMES = 16, FFB_THREADS = 256;

__device__ __forceinline__ void frame_features_block(const float* __restrict__ a, int nf, int frame_len,
                                                     const float* __restrict__ log_k, const float* __restrict__ w,
                                                     int dim, float* __restrict__ out, int ld_out, bool w4) {
    __shared__ __align__(16) float fr[FFB_FRAMES][MAX_FRAME];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int f0 = blockIdx.x * FFB_FRAMES;
    const int nfb = min(FFB_FRAMES, nf - f0);
    if (nfb <= 0) return;  // whole CTA
    for (int f = wid; f < nfb; f += FFB_THREADS / 32) {
        const float* af = a + (size_t)(f0 + f) * frame_len;
        float s = 0.f;
        for (int i = lane; i < frame_len; i += 32) s += af[i];
        const float mean = warp_sum(s) / (float)frame_len;
        float v = 0.f;
        for (int i = lane; i < frame_len; i += 32) {
            const float c = af[i] - mean;
            v += c * c;
        }
        const float rms = sqrtf(warp_sum(v) / (float)frame_len + 1e-6f);
        const float k = expf(*log_k);
        for (int i = lane; i < frame_len; i += 32) fr[f][i] = asinhf(k * ((af[i] - mean) / rms));
    }
    __syncthreads();
    for (int j = threadIdx.x; j < dim; j += FFB_THREADS) {
        const float* wr = w + (size_t)j * frame_len;
        float acc[FFB_FRAMES];
#pragma unroll
        for (int f = 0; f < FFB_FRAMES; ++f) acc[f] = 0.f;
        if (w4) {  // frame_len % 4 == 0 and 16-byte aligned rows
            for (int i = 0; i < frame_len; i += 4) {
                const float4 wv = __ldg(reinterpret_cast<const float4*>(wr + i));
#pragma unroll
                for (int f = 0; f < FFB_FRAMES; ++f) {
                    const float4 x = *reinterpret_cast<const float4*>(&fr[f][i]);
                    acc[f] = fmaf(x.w, wv.w, fmaf(x.z, wv.z, fmaf(x.y, wv.y, fmaf(x.x, wv.x, acc[f]))));
                }
            }
        } else {
            for (int i = 0; i < frame_len; ++i) {
                const float wv = __ldg(wr + i);
#pragma unroll
                for (int f = 0; f < FFB_FRAMES; ++f) acc[f] = fmaf(fr[f][i], wv, acc[f]);
            }
        }
#pragma unroll
        for (int f = 0; f < FFB_FRAMES; ++f)
            if (f < nfb) out[(size_t)(f0 + f) * ld_out + j] = silu(acc[f]);
    }
}

__global__ void __launch_bounds__(FFB_THREADS)
frame_features_block_kernel(const float* __restrict__ audio, int n_frames, int frame_len, const float* __restrict__ log_k,
                            const float* __restrict__ w, int dim, float* __restrict__ out, int ld_out, int w4) {
    frame_features_block(audio, n_frames, frame_len, log_k, w, dim, out, ld_out, w4 != 0);
}

__global__ void __launch_bounds__(FFB_THREADS)
frame_features_block_batch_kernel(const float* __restrict__ audio, const long long* __restrict__ aoff,
                                  const int* __restrict__ nf, float* const* __restrict__ out, int frame_len,
                                  const float* __restrict__ log_k, const float* __restrict__ w, int dim, int ld_out,
                                  int w4) {
    const int z = blockIdx.y;
    frame_features_block(audio + aoff[z], nf[z], frame_len, log_k, w, dim, out[z], ld_out, w4 != 0);
}

// dst[z][0 .. n[z]) = src[z][0 .. n[z]) (zeros where src[z] is null); n[z] % 4 == 0, 16-byte
// aligned rows.
__global__ void copy_rows_batch_kernel(const float* const* __restrict__ src, float* const* __restrict__ dst,
                                       const int* __restrict__ n) {
    const int z = blockIdx.x;
    const float4* s4 = reinterpret_cast<const float4*>(src[z]);
    float4* d4 = reinterpret_cast<float4*>(dst[z]);
    for (int i = threadIdx.x; i < n[z] / 4; i += blockDim.x) d4[i] = s4 ? s4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
}

constexpr int LN_MAXV = 32;  // up to 1024 features per row (32 per lane)

__global__ void layernorm_rows_kernel(const float* __restrict__ x, int rows, int dim,
                                      const float* __restrict__ w, float w_offset, float eps,
                                      const float* __restrict__ add, int add_row0,
                                      float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const float* xr = x + (size_t)r * dim;
    float v[LN_MAXV];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < LN_MAXV; ++j) {
        const int i = lane + 32 * j;
        v[j] = (i < dim) ? xr[i] : 0.f;
        s += v[j];
    }
    const float mean = warp_sum(s) / (float)dim;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < LN_MAXV; ++j) {
        const int i = lane + 32 * j;
        const float c = (i < dim) ? v[j] - mean : 0.f;
        q += c * c;
    }
    const float rstd = rsqrtf(warp_sum(q) / (float)dim + eps);
    float* o = out + (size_t)r * dim;
    const float* ar = add ? add + (size_t)(add_row0 + r) * dim : nullptr;
#pragma unroll
    for (int j = 0; j < LN_MAXV; ++j) {
        const int i = lane + 32 * j;
        if (i < dim) {
            float y = (v[j] - mean) * rstd * (w[i] + w_offset);
            if (ar) y += ar[i];
            o[i] = y;
        }
    }
}

constexpr int WA_MAXHD = 128;

// One warp per (query, head).  Keys are visited 32 at a time with an online softmax.
__global__ void window_attention_kernel(const float* __restrict__ qkv, int T, int H, int KVH,
                                        int hd, int left, int right, float scale,
                                        float* __restrict__ out, int seg_rows, const int* __restrict__ seg_len,
                                        __nv_bfloat16* __restrict__ out_bf16, size_t lo_off) {
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= T * H) return;
    const int t = item / H, h = item - t * H;
    const int kvh = h / (H / KVH);
    const int ld = (H + 2 * KVH) * hd;
    const float* q = qkv + (size_t)t * ld + h * hd;
    const float* kbase = qkv + H * hd + kvh * hd;
    const float* vbase = qkv + (H + KVH) * hd + kvh * hd;
    // segments: rows [s * seg_rows, s * seg_rows + seg_len[s]) are one utterance; a query sees
    // keys of its own utterance only, and rows past its length are written as zeros
    int base = 0, len = T, tl = t;
    if (seg_rows > 0) {
        const int sgi = t / seg_rows;
        base = sgi * seg_rows;
        len = seg_len[sgi];
        tl = t - base;
        if (tl >= len) {
            for (int d = lane; d < hd; d += 32) {
                if (out) out[(size_t)t * (H * hd) + h * hd + d] = 0.f;
                if (out_bf16) st_bf16_split(out_bf16 + (size_t)t * (H * hd) + h * hd + d, 0.f, lo_off);
            }
            return;
        }
    }
    int lo = base, hi = base + len;
    if (left > 0) {
        lo = base + max(0, tl - left + 1);
        hi = base + min(len, tl + (right > 0 ? right : 1));
    }
    float m = -INFINITY, l = 0.f;
    float acc[WA_MAXHD / 32];
#pragma unroll
    for (int j = 0; j < WA_MAXHD / 32; ++j) acc[j] = 0.f;
    for (int k0 = lo; k0 < hi; k0 += 32) {
        const int kk = k0 + lane;
        float s = -INFINITY;
        if (kk < hi) {
            const float* kr = kbase + (size_t)kk * ld;
            float dot = 0.f;
            for (int d = 0; d < hd; d += 4) {
                const float4 a = *reinterpret_cast<const float4*>(q + d);
                const float4 b = *reinterpret_cast<const float4*>(kr + d);
                dot = fmaf(a.x, b.x, dot);
                dot = fmaf(a.y, b.y, dot);
                dot = fmaf(a.z, b.z, dot);
                dot = fmaf(a.w, b.w, dot);
            }
            s = dot * scale;
        }
        const float mc = warp_max(s);
        const float mn = fmaxf(m, mc);
        const float p = (kk < hi) ? expf(s - mn) : 0.f;
        const float corr = expf(m - mn);  // 0 on the first chunk (m = -inf)
        l = l * corr + warp_sum(p);
#pragma unroll
        for (int j = 0; j < WA_MAXHD / 32; ++j) acc[j] *= corr;
        const int nk = min(32, hi - k0);
        for (int j = 0; j < nk; ++j) {
            const float pj = __shfl_sync(FULL, p, j);
            const float* vr = vbase + (size_t)(k0 + j) * ld;
#pragma unroll
            for (int c = 0; c < WA_MAXHD / 32; ++c) {
                const int d = lane + 32 * c;
                if (d < hd) acc[c] = fmaf(pj, vr[d], acc[c]);
            }
        }
        m = mn;
    }
    const size_t o = (size_t)t * (H * hd) + h * hd;
    const float inv = 1.f / l;
#pragma unroll
    for (int c = 0; c < WA_MAXHD / 32; ++c) {
        const int d = lane + 32 * c;
        if (d < hd) {
            if (out) out[o + d] = acc[c] * inv;
            if (out_bf16) st_bf16_split(out_bf16 + o + d, acc[c] * inv, lo_off);
        }
    }
}

// The same attention for windows (left > 0), one CTA per (tile of WT_Q consecutive query rows
// of one segment, head): the K and V rows of the band those queries see are staged in shared
// memory once with coalesced loads (rows padded to hd + 4 floats, so lanes reading different
// rows hit different banks), then each warp takes every WT_WARPS-th query with the arithmetic
// of window_attention_kernel in the same order, so the results are the same bit for bit;
// the per-query kernel read every key row from global memory once per query.
constexpr int WT_Q = 32;
constexpr int WT_WARPS = 4;
__global__ void __launch_bounds__(WT_WARPS * 32) window_attention_tile_kernel(
    const float* __restrict__ qkv, int T, int H, int KVH, int hd, int left, int right, float scale,
    float* __restrict__ out, int seg_rows, const int* __restrict__ seg_len, __nv_bfloat16* __restrict__ out_bf16,
    size_t lo_off, int tiles_per_seg, int kmax) {
    extern __shared__ __align__(16) float wt_smem[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int h = blockIdx.y, kvh = h / (H / KVH);
    const int seg = blockIdx.x / tiles_per_seg, tile = blockIdx.x - seg * tiles_per_seg;
    const int srows = seg_rows > 0 ? seg_rows : T;
    const int base = seg * srows, len = seg_rows > 0 ? seg_len[seg] : T;
    const int q0 = tile * WT_Q, q1 = min(srows, q0 + WT_Q);  // local rows of this tile's queries
    const int ld = (H + 2 * KVH) * hd, rs = hd + 4, n4 = hd >> 2;
    float* ks = wt_smem;
    float* vs = ks + (size_t)kmax * rs;
    float* qw = vs + (size_t)kmax * rs + wid * hd;  // this warp's query row
    // the band of the valid queries: local keys [klo, khi) (at most kmax rows, host-checked)
    const int qv1 = min(q1, len);
    const int klo = q0 < qv1 ? max(0, q0 - left + 1) : 0;
    const int khi = q0 < qv1 ? min(len, (qv1 - 1) + (right > 0 ? right : 1)) : 0;
    const int nrows = khi - klo;
    const float* kg = qkv + (size_t)(base + klo) * ld + H * hd + kvh * hd;
    const float* vg = kg + KVH * hd;
    for (int i = threadIdx.x; i < 2 * nrows * n4; i += blockDim.x) {
        const int kv = i >= nrows * n4, ii = kv ? i - nrows * n4 : i;
        const int r = ii / n4, c4 = ii - r * n4;
        const float4 v = *reinterpret_cast<const float4*>((kv ? vg : kg) + (size_t)r * ld + 4 * c4);
        *reinterpret_cast<float4*>((kv ? vs : ks) + (size_t)r * rs + 4 * c4) = v;
    }
    __syncthreads();
    for (int qi = q0 + wid; qi < q1; qi += WT_WARPS) {
        const int t = base + qi;
        const size_t o = (size_t)t * (H * hd) + h * hd;
        if (qi >= len) {  // rows past the segment's length are written as zeros
            for (int d = lane; d < hd; d += 32) {
                if (out) out[o + d] = 0.f;
                if (out_bf16) st_bf16_split(out_bf16 + o + d, 0.f, lo_off);
            }
            continue;
        }
        __syncwarp();  // the previous query's row is no longer read
        for (int d = lane; d < hd; d += 32) qw[d] = qkv[(size_t)t * ld + h * hd + d];
        __syncwarp();
        const int lo = max(0, qi - left + 1), hi = min(len, qi + (right > 0 ? right : 1));
        float m = -INFINITY, l = 0.f;
        float acc[WA_MAXHD / 32];
#pragma unroll
        for (int j = 0; j < WA_MAXHD / 32; ++j) acc[j] = 0.f;
        for (int k0 = lo; k0 < hi; k0 += 32) {
            const int kk = k0 + lane;
            float s = -INFINITY;
            if (kk < hi) {
                const float* kr = ks + (size_t)(kk - klo) * rs;
                float dot = 0.f;
                for (int d = 0; d < hd; d += 4) {
                    const float4 a = *reinterpret_cast<const float4*>(qw + d);
                    const float4 b = *reinterpret_cast<const float4*>(kr + d);
                    dot = fmaf(a.x, b.x, dot);
                    dot = fmaf(a.y, b.y, dot);
                    dot = fmaf(a.z, b.z, dot);
                    dot = fmaf(a.w, b.w, dot);
                }
                s = dot * scale;
            }
            const float mc = warp_max(s);
            const float mn = fmaxf(m, mc);
            const float p = (kk < hi) ? expf(s - mn) : 0.f;
            const float corr = expf(m - mn);  // 0 on the first chunk (m = -inf)
            l = l * corr + warp_sum(p);
#pragma unroll
            for (int j = 0; j < WA_MAXHD / 32; ++j) acc[j] *= corr;
            const int nk = min(32, hi - k0);
            for (int j = 0; j < nk; ++j) {
                const float pj = __shfl_sync(FULL, p, j);
                const float* vr = vs + (size_t)(k0 + j - klo) * rs;
#pragma unroll
                for (int c = 0; c < WA_MAXHD / 32; ++c) {
                    const int d = lane + 32 * c;
                    if (d < hd) acc[c] = fmaf(pj, vr[d], acc[c]);
                }
            }
            m = mn;
        }
        const float inv = 1.f / l;
#pragma unroll
        for (int c = 0; c < WA_MAXHD / 32; ++c) {
            const int d = lane + 32 * c;
            if (d < hd) {
                if (out) out[o + d] = acc[c] * inv;
                if (out_bf16) st_bf16_split(out_bf16 + o + d, acc[c] * inv, lo_off);
            }
        }
    }
}

// CMVN + asinh of the 80-sample frames of a batch in segment-row layout: row r holds frame
// r % seg_rows - 4 of utterance r / seg_rows (bf16, frame_len values), or zeros where there is
// none (the causal padding in front and the tail), so the following Linear + SiLU GEMM
// writes exact zeros there.
__global__ void frame_norm_rows_kernel(const float* const* __restrict__ audio, const int* __restrict__ n_frames,
                                       int rows, int seg_rows, int frame_len, const float* __restrict__ log_k,
                                       __nv_bfloat16* __restrict__ out, size_t lo_off) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int sgi = r / seg_rows, f = r - sgi * seg_rows - 4;
    __nv_bfloat16* o = out + (size_t)r * frame_len;
    if (f < 0 || f >= n_frames[sgi]) {
        for (int i = lane; i < frame_len; i += 32) st_bf16_split(o + i, 0.f, lo_off);
        return;
    }
    const float* a = audio[sgi] + (size_t)f * frame_len;
    float s = 0.f;
    for (int i = lane; i < frame_len; i += 32) s += a[i];
    const float mean = warp_sum(s) / (float)frame_len;
    float v = 0.f;
    for (int i = lane; i < frame_len; i += 32) {
        const float c = a[i] - mean;
        v += c * c;
    }
    const float rms = sqrtf(warp_sum(v) / (float)frame_len + 1e-6f);
    const float k = expf(*log_k);
    for (int i = lane; i < frame_len; i += 32) st_bf16_split(o + i, asinhf(k * ((a[i] - mean) / rms)), lo_off);
}

// Final encoder LayerNorm of segment rows (rows [s * seg_rows, s * seg_rows + len[s]) hold
// utterance s) plus pos_emb[t], gathered to memory rows off[s] + t (fp32 and bf16).
__global__ void ln_gather_rows_kernel(const float* __restrict__ x, int rows, int seg_rows, int dim,
                                      const float* __restrict__ w, float w_offset, float eps,
                                      const float* __restrict__ pos_emb, const int* __restrict__ len,
                                      const int* __restrict__ off, float* __restrict__ out,
                                      __nv_bfloat16* __restrict__ out_bf16, size_t lo_off) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int sgi = r / seg_rows, t = r - sgi * seg_rows;
    if (t >= len[sgi]) return;
    const float* xr = x + (size_t)r * dim;
    float v[LN_MAXV];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < LN_MAXV; ++j) {
        const int i = lane + 32 * j;
        v[j] = (i < dim) ? xr[i] : 0.f;
        s += v[j];
    }
    const float mean = warp_sum(s) / (float)dim;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < LN_MAXV; ++j) {
        const int i = lane + 32 * j;
        const float c = (i < dim) ? v[j] - mean : 0.f;
        q += c * c;
    }
    const float rstd = rsqrtf(warp_sum(q) / (float)dim + eps);
    const size_t orow = (size_t)(off[sgi] + t) * dim;
    const float* pe = pos_emb + (size_t)t * dim;
#pragma unroll
    for (int j = 0; j < LN_MAXV; ++j) {
        const int i = lane + 32 * j;
        if (i < dim) {
            const float y = (v[j] - mean) * rstd * (w[i] + w_offset) + pe[i];
            out[orow + i] = y;
            st_bf16_split(out_bf16 + orow + i, y, lo_off);
        }
    }
}

// Segment rows from per-segment sources: row t of segment b = src[b] + t * dim for t < T[b],
// zeros for t in [T[b], seg_rows) (block (t, b), dim % 4 == 0, 16-byte aligned sources).
__global__ void gather_seg_rows_kernel(const float* const* __restrict__ src, const int* __restrict__ T,
                                       int seg_rows, int dim, float* __restrict__ out) {
    const int t = blockIdx.x, b = blockIdx.y;
    float4* o = reinterpret_cast<float4*>(out + ((size_t)b * seg_rows + t) * dim);
    const bool has = t < T[b];
    const float4* sr = has ? reinterpret_cast<const float4*>(src[b] + (size_t)t * dim) : nullptr;
    for (int i = threadIdx.x; i < (dim >> 2); i += blockDim.x) o[i] = has ? sr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
}

// Final encoder LayerNorm + positions of a window per segment, scattered to each segment's
// own output: for i < cnt[b], row b * seg_rows + off[b] + i -> dst[b] + i * dim, adding
// pos_emb[pos[b] + i] (one warp per (b, i); the arithmetic of ln_gather_rows_kernel).
__global__ void ln_scatter_rows_kernel(const float* __restrict__ x, int nseg, int max_cnt, int seg_rows, int dim,
                                       const float* __restrict__ w, float w_offset, float eps,
                                       const float* __restrict__ pos_emb, const int* __restrict__ off,
                                       const int* __restrict__ cnt, const int* __restrict__ pos,
                                       float* const* __restrict__ dst) {
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= nseg * max_cnt) return;
    const int b = item / max_cnt, i = item - b * max_cnt;
    if (i >= cnt[b]) return;
    const float* xr = x + ((size_t)b * seg_rows + off[b] + i) * dim;
    float v[LN_MAXV];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < LN_MAXV; ++j) {
        const int k = lane + 32 * j;
        v[j] = (k < dim) ? xr[k] : 0.f;
        s += v[j];
    }
    const float mean = warp_sum(s) / (float)dim;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < LN_MAXV; ++j) {
        const int k = lane + 32 * j;
        const float c = (k < dim) ? v[j] - mean : 0.f;
        q += c * c;
    }
    const float rstd = rsqrtf(warp_sum(q) / (float)dim + eps);
    float* o = dst[b] + (size_t)i * dim;
    const float* pe = pos_emb + (size_t)(pos[b] + i) * dim;
#pragma unroll
    for (int j = 0; j < LN_MAXV; ++j) {
        const int k = lane + 32 * j;
        if (k < dim) o[k] = (v[j] - mean) * rstd * (w[k] + w_offset) + pe[k];
    }
}

}  // namespace

cudaError_t launch_gather_seg_rows(const float* const* src, const int* T, int nseg, int seg_rows, int dim, float* out,
                                   cudaStream_t stream) {
    if (nseg <= 0 || seg_rows <= 0) return cudaSuccess;
    if (dim % 4) return cudaErrorInvalidValue;
    ++launch_counter();
    gather_seg_rows_kernel<<<dim3(seg_rows, nseg), 128, 0, stream>>>(src, T, seg_rows, dim, out);
    return cudaGetLastError();
}

cudaError_t launch_ln_scatter_rows(const float* x, int nseg, int max_cnt, int seg_rows, int dim, const float* w,
                                   float w_offset, float eps, const float* pos_emb, const int* off, const int* cnt,
                                   const int* pos, float* const* dst, cudaStream_t stream) {
    if (nseg <= 0 || max_cnt <= 0) return cudaSuccess;
    if (dim > 32 * LN_MAXV) return cudaErrorInvalidValue;
    ++launch_counter();
    const int wpb = 8, items = nseg * max_cnt;
    ln_scatter_rows_kernel<<<(items + wpb - 1) / wpb, wpb * 32, 0, stream>>>(x, nseg, max_cnt, seg_rows, dim, w,
                                                                           w_offset, eps, pos_emb, off, cnt, pos,
                                                                           dst);
    return cudaGetLastError();
}

cudaError_t launch_frame_features(const float* audio, int n_frames, int frame_len,
                                  const float* log_k, const float* w, int dim, float* out,
                                  int ld_out, cudaStream_t stream) {
    if (n_frames <= 0) return cudaSuccess;
    if (frame_len > MAX_FRAME) return cudaErrorInvalidValue;
    ++launch_counter();
    const int w4 = (frame_len % 4 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) ? 1 : 0;
    frame_features_block_kernel<<<(n_frames + FFB_FRAMES - 1) / FFB_FRAMES, FFB_THREADS, 0, stream>>>(
        audio, n_frames, frame_len, log_k, w, dim, out, ld_out, w4);
    return cudaGetLastError();
}

cudaError_t launch_frame_features_batch(const float* audio, const long long* aoff, const int* nf, float* const* out,
                                        int nb, int nf_max, int frame_len, const float* log_k, const float* w,
                                        int dim, int ld_out, cudaStream_t stream) {
    if (nb <= 0 || nf_max <= 0) return cudaSuccess;
    if (frame_len > MAX_FRAME || nb > 65535) return cudaErrorInvalidValue;
    ++launch_counter();
    const int w4 = (frame_len % 4 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) ? 1 : 0;
    frame_features_block_batch_kernel<<<dim3((nf_max + FFB_FRAMES - 1) / FFB_FRAMES, nb), FFB_THREADS, 0, stream>>>(
        audio, aoff, nf, out, frame_len, log_k, w, dim, ld_out, w4);
    return cudaGetLastError();
}

cudaError_t launch_copy_rows_batch(const float* const* src, float* const* dst, const int* n, int nb,
                                   cudaStream_t stream) {
    if (nb <= 0) return cudaSuccess;
    ++launch_counter();
    copy_rows_batch_kernel<<<nb, 128, 0, stream>>>(src, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_frame_features_bf16(const float* audio, int n_frames, int frame_len, const float* log_k,
                                       const float* w, int dim, __nv_bfloat16* out, int ld_out,
                                       cudaStream_t stream) {
    if (n_frames <= 0) return cudaSuccess;
    if (frame_len > MAX_FRAME) return cudaErrorInvalidValue;
    ++launch_counter();
    frame_features_kernel<__nv_bfloat16><<<(n_frames + FF_WARPS - 1) / FF_WARPS, FF_WARPS * 32, 0, stream>>>(
        audio, n_frames, frame_len, log_k, w, dim, out, ld_out);
    return cudaGetLastError();
}

cudaError_t launch_layernorm_rows(const float* x, int rows, int dim, const float* w,
                                  float w_offset, float eps, const float* add, int add_row0,
                                  float* out, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    if (dim > 32 * LN_MAXV) return cudaErrorInvalidValue;
    ++launch_counter();
    const int wpb = 8;
    layernorm_rows_kernel<<<(rows + wpb - 1) / wpb, wpb * 32, 0, stream>>>(
        x, rows, dim, w, w_offset, eps, add, add_row0, out);
    return cudaGetLastError();
}

cudaError_t launch_window_attention(const float* qkv, int T, int H, int kv_heads, int hd,
                                    int left, int right, float scale, float* out,
                                    cudaStream_t stream, int seg_rows, const int* seg_len,
                                    __nv_bfloat16* out_bf16, size_t lo_off) {
    if (T <= 0) return cudaSuccess;
    if (hd > WA_MAXHD || (hd & 3) || H % kv_heads) return cudaErrorInvalidValue;
    if ((seg_rows > 0) != (seg_len != nullptr) || (!out && !out_bf16)) return cudaErrorInvalidValue;
    ++launch_counter();
    if (left > 0 && (seg_rows == 0 || T % seg_rows == 0)) {  // windows: the band staged per tile
        const int kmax = WT_Q + left + (right > 0 ? right : 1);
        const size_t smem = ((size_t)2 * kmax * (hd + 4) + (size_t)WT_WARPS * hd) * 4;
        if (smem <= 48 * 1024) {
            const int srows = seg_rows > 0 ? seg_rows : T, nseg = T / srows;
            const int tiles = (srows + WT_Q - 1) / WT_Q;
            window_attention_tile_kernel<<<dim3(nseg * tiles, H), WT_WARPS * 32, smem, stream>>>(
                qkv, T, H, kv_heads, hd, left, right, scale, out, seg_rows, seg_len, out_bf16, lo_off, tiles, kmax);
            return cudaGetLastError();
        }
    }
    const int wpb = 8;
    const int items = T * H;
    window_attention_kernel<<<(items + wpb - 1) / wpb, wpb * 32, 0, stream>>>(
        qkv, T, H, kv_heads, hd, left, right, scale, out, seg_rows, seg_len, out_bf16, lo_off);
    return cudaGetLastError();
}

cudaError_t launch_frame_norm_rows(const float* const* audio, const int* n_frames, int rows, int seg_rows,
                                   int frame_len, const float* log_k, __nv_bfloat16* out, cudaStream_t stream,
                                   size_t lo_off) {
    if (rows <= 0) return cudaSuccess;
    if (seg_rows <= 4) return cudaErrorInvalidValue;
    ++launch_counter();
    const int wpb = 8;
    frame_norm_rows_kernel<<<(rows + wpb - 1) / wpb, wpb * 32, 0, stream>>>(audio, n_frames, rows, seg_rows,
                                                                          frame_len, log_k, out, lo_off);
    return cudaGetLastError();
}

cudaError_t launch_ln_gather_rows(const float* x, int rows, int seg_rows, int dim, const float* w, float w_offset,
                                  float eps, const float* pos_emb, const int* len, const int* off, float* out,
                                  __nv_bfloat16* out_bf16, cudaStream_t stream, size_t lo_off) {
    if (rows <= 0) return cudaSuccess;
    if (dim > 32 * LN_MAXV || seg_rows <= 0) return cudaErrorInvalidValue;
    ++launch_counter();
    const int wpb = 8;
    ln_gather_rows_kernel<<<(rows + wpb - 1) / wpb, wpb * 32, 0, stream>>>(x, rows, seg_rows, dim, w, w_offset, eps,
                                                                         pos_emb, len, off, out, out_bf16, lo_off);
    return cudaGetLastError();
}

}  // namespace msb
