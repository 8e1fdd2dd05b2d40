// Audio frontend and encoder-side kernels (fp32).
//
//   frame_features   : CMVN + asinh + Linear(frame_len -> d) + SiLU, one warp per frame
//                      (Sources/MoonshineMLX/MoonshineEncoder.swift:15-34, 84-86)
//   layernorm_rows   : LayerNorm with optional unit offset and a fused row add, used for
//                      the encoder norms and final_norm + pos_emb (prepareMemory,
//                      MoonshineDecoder.swift:39-47)
//   window_attention : sliding-window MHA, keys restricted to the band instead of a
//                      dense [T,T] additive mask (MoonshineLayers.swift:266-290)
#include "common.cuh"
#include "kernels.h"

namespace msb {

namespace {

constexpr int FF_WARPS = 8;
constexpr int MAX_FRAME = 128;

__global__ void __launch_bounds__(FF_WARPS * 32)
frame_features_kernel(const float* __restrict__ audio, int n_frames, int frame_len,
                      const float* __restrict__ log_k, const float* __restrict__ w, int dim,
                      float* __restrict__ out, int ld_out) {
    __shared__ float fr[FF_WARPS][MAX_FRAME];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int f = blockIdx.x * FF_WARPS + wid;
    if (f >= n_frames) return;
    const float* a = audio + (size_t)f * frame_len;
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
    for (int i = lane; i < frame_len; i += 32) fr[wid][i] = asinhf(k * ((a[i] - mean) / rms));
    __syncwarp();
    for (int o = lane; o < dim; o += 32) {
        const float* wr = w + (size_t)o * frame_len;
        float acc = 0.f;
        for (int i = 0; i < frame_len; ++i) acc = fmaf(fr[wid][i], __ldg(wr + i), acc);
        out[(size_t)f * ld_out + o] = silu(acc);
    }
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
                                        float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= T * H) return;
    const int t = item / H, h = item - t * H;
    const int kvh = h / (H / KVH);
    const int ld = (H + 2 * KVH) * hd;
    const float* q = qkv + (size_t)t * ld + h * hd;
    const float* kbase = qkv + H * hd + kvh * hd;
    const float* vbase = qkv + (H + KVH) * hd + kvh * hd;
    int lo = 0, hi = T;
    if (left > 0) {
        lo = max(0, t - left + 1);
        hi = min(T, t + (right > 0 ? right : 1));
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
    float* o = out + (size_t)t * (H * hd) + h * hd;
    const float inv = 1.f / l;
#pragma unroll
    for (int c = 0; c < WA_MAXHD / 32; ++c) {
        const int d = lane + 32 * c;
        if (d < hd) o[d] = acc[c] * inv;
    }
}

}  // namespace

cudaError_t launch_frame_features(const float* audio, int n_frames, int frame_len,
                                  const float* log_k, const float* w, int dim, float* out,
                                  int ld_out, cudaStream_t stream) {
    if (n_frames <= 0) return cudaSuccess;
    if (frame_len > MAX_FRAME) return cudaErrorInvalidValue;
    ++launch_counter();
    frame_features_kernel<<<(n_frames + FF_WARPS - 1) / FF_WARPS, FF_WARPS * 32, 0, stream>>>(
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
                                    cudaStream_t stream) {
    if (T <= 0) return cudaSuccess;
    if (hd > WA_MAXHD || (hd & 3) || H % kv_heads) return cudaErrorInvalidValue;
    ++launch_counter();
    const int wpb = 8;
    const int items = T * H;
    window_attention_kernel<<<(items + wpb - 1) / wpb, wpb * 32, 0, stream>>>(
        qkv, T, H, kv_heads, hd, left, right, scale, out);
    return cudaGetLastError();
}

}  // namespace msb
