// Cross-attention alignment rows for word timestamps.
//
// The reference (generateWithWordTimestamps, MoonshineModel.swift:241-316) asks every
// decoder layer for its cross-attention scores q.K^T * scale (MoonshineLayers.swift:150-154)
// and findAlignment (MoonshineTimestamps.swift:106-146) turns them, per decoder call, into
// one row over the memory frames:
//   row[f]  = mean over layers of mean over heads of softmax_f(q_lh . K_lh[f] * scale)
//   z       = (row - mean(row)) / (std(row) + 1e-6)            (population std)
//   out[f]  = median of z over [max(0, f - w/2), min(M - 1, f + w/2)]  (element count/2 of
//             the sorted window, so the upper median where the clipped window is even)
// Here the decode kernels store each call's cross queries (qc_trace [steps][L][H*hd]) and
// two kernels rebuild the rows from the cross K the decode used: the fp32 copy for the
// first call and the stored copy (fp16 when the cache is fp16) for the others, exactly as
// the attention itself did.
//
//   cross_weights_kernel  grid (step groups, L): the head-mean softmax rows of one layer
//                         for up to SG calls that read the same K copy, so each K row is
//                         loaded once per group; scores and the head sums live in shared
//                         memory ([SG][M] each).  Output part [steps][L][M].
//   alignment_rows_kernel grid (steps): layer mean, z-score, median filter, and the
//                         softmax probability of the call's chosen id from its logits.
#include "kernels.h"

#include <cuda_fp16.h>

namespace msb {

namespace {

constexpr int AL_THREADS = 256;
constexpr int AL_MAX_SG = 8;
constexpr int AL_MAX_HD = 128;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide reduction of SG values per thread (max when is_max, else sum); every thread
// gets the results in out[]. red: [SG][32] shared floats.
template <int SG>
__device__ void block_reduce(float (&v)[SG], bool is_max, float* red, float (&out)[SG]) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int s = 0; s < SG; ++s) {
        const float x = is_max ? warp_max(v[s]) : warp_sum(v[s]);
        if (lane == 0) red[s * 32 + w] = x;
    }
    __syncthreads();
#pragma unroll
    for (int s = 0; s < SG; ++s) {
        float x = is_max ? -INFINITY : 0.f;
        for (int k = 0; k < nw; ++k) x = is_max ? fmaxf(x, red[s * 32 + k]) : x + red[s * 32 + k];
        out[s] = x;
    }
    __syncthreads();
}

template <int SG>
__global__ void __launch_bounds__(AL_THREADS) cross_weights_kernel(const float* __restrict__ qtr,
                                                                   const float* __restrict__ c32,
                                                                   const void* __restrict__ cst, int st_f16,
                                                                   int n_steps, int L, int H, int KVH, int hd,
                                                                   int m_cap, int M, float scale, float* part) {
    extern __shared__ float sm[];
    __shared__ float red[SG * 32];
    const int l = blockIdx.y;
    const int g = blockIdx.x;
    // group 0 is the first call alone (fp32 K); group g >= 1 holds calls 1 + (g-1)*SG ...
    const int s0 = g == 0 ? 0 : 1 + (g - 1) * SG;
    const int ns = g == 0 ? 1 : min(SG, n_steps - s0);
    if (ns <= 0) return;
    const bool f16 = g > 0 && st_f16;
    const int HD = H * hd, rep = H / KVH;
    float* qs = sm;                       // [SG][HD]
    float* sc = qs + (size_t)SG * HD;     // [SG][M]
    float* acc = sc + (size_t)SG * M;     // [SG][M]
    for (int i = threadIdx.x; i < SG * HD; i += blockDim.x) {
        const int s = i / HD;
        qs[i] = s < ns ? qtr[((size_t)(s0 + s) * L + l) * HD + (i - s * HD)] * scale : 0.f;
    }
    for (int i = threadIdx.x; i < SG * M; i += blockDim.x) acc[i] = 0.f;
    __syncthreads();
    for (int h = 0; h < H; ++h) {
        const size_t kbase = ((size_t)(l * 2) * KVH + h / rep) * m_cap * hd;
        // scores of every frame for the group's calls
        for (int f = threadIdx.x; f < M; f += blockDim.x) {
            float dot[SG];
#pragma unroll
            for (int s = 0; s < SG; ++s) dot[s] = 0.f;
            if (f16) {
                const __half* kr = reinterpret_cast<const __half*>(cst) + kbase + (size_t)f * hd;
                for (int e = 0; e < hd; ++e) {
                    const float kv = __half2float(kr[e]);
#pragma unroll
                    for (int s = 0; s < SG; ++s) dot[s] = fmaf(qs[s * HD + h * hd + e], kv, dot[s]);
                }
            } else {
                const float* kr = (g == 0 ? c32 : reinterpret_cast<const float*>(cst)) + kbase + (size_t)f * hd;
                for (int e = 0; e < hd; ++e) {
                    const float kv = kr[e];
#pragma unroll
                    for (int s = 0; s < SG; ++s) dot[s] = fmaf(qs[s * HD + h * hd + e], kv, dot[s]);
                }
            }
#pragma unroll
            for (int s = 0; s < SG; ++s) sc[(size_t)s * M + f] = dot[s];
        }
        // softmax over frames, accumulated into the head sum
        float mx[SG], sum[SG], r[SG];
#pragma unroll
        for (int s = 0; s < SG; ++s) mx[s] = -INFINITY;
        for (int f = threadIdx.x; f < M; f += blockDim.x)
#pragma unroll
            for (int s = 0; s < SG; ++s) mx[s] = fmaxf(mx[s], sc[(size_t)s * M + f]);
        block_reduce<SG>(mx, true, red, r);
#pragma unroll
        for (int s = 0; s < SG; ++s) {
            mx[s] = r[s];
            sum[s] = 0.f;
        }
        for (int f = threadIdx.x; f < M; f += blockDim.x)
#pragma unroll
            for (int s = 0; s < SG; ++s) {
                const float e = expf(sc[(size_t)s * M + f] - mx[s]);
                sc[(size_t)s * M + f] = e;
                sum[s] += e;
            }
        block_reduce<SG>(sum, false, red, r);
        for (int f = threadIdx.x; f < M; f += blockDim.x)
#pragma unroll
            for (int s = 0; s < SG; ++s) acc[(size_t)s * M + f] += sc[(size_t)s * M + f] / r[s];
        __syncthreads();
    }
    const float inv_h = 1.f / (float)H;
    for (int s = 0; s < ns; ++s)
        for (int f = threadIdx.x; f < M; f += blockDim.x)
            part[((size_t)(s0 + s) * L + l) * M + f] = acc[(size_t)s * M + f] * inv_h;
}

// k-th smallest of n values (k < n) by rank counting: v[i] is the answer when
// #(v < v[i]) <= k < #(v < v[i]) + #(v == v[i]).
__device__ float select_kth(const float* v, int n, int k) {
    for (int i = 0; i < n; ++i) {
        int lt = 0, eq = 0;
        for (int j = 0; j < n; ++j) {
            lt += v[j] < v[i];
            eq += v[j] == v[i];
        }
        if (lt <= k && k < lt + eq) return v[i];
    }
    return v[0];
}

__global__ void __launch_bounds__(AL_THREADS) alignment_rows_kernel(const float* __restrict__ part, int L, int M,
                                                                    int width, const float* __restrict__ logits,
                                                                    const int* __restrict__ ids, int V,
                                                                    float* raw_out, float* filt_out, float* probs) {
    extern __shared__ float sm[];
    __shared__ float red[32];
    const int s = blockIdx.x;
    float* row = sm;     // [M]
    float* z = sm + M;   // [M]
    const float inv_l = 1.f / (float)L;
    float loc = 0.f;
    for (int f = threadIdx.x; f < M; f += blockDim.x) {
        float a = 0.f;
        for (int l = 0; l < L; ++l) a += part[((size_t)s * L + l) * M + f];
        a *= inv_l;
        row[f] = a;
        loc += a;
        if (raw_out) raw_out[(size_t)s * M + f] = a;
    }
    float v1[1] = {loc}, o1[1];
    block_reduce<1>(v1, false, red, o1);
    const float mean = o1[0] / (float)max(M, 1);
    loc = 0.f;
    for (int f = threadIdx.x; f < M; f += blockDim.x) {
        const float dlt = row[f] - mean;
        loc += dlt * dlt;
    }
    v1[0] = loc;
    block_reduce<1>(v1, false, red, o1);
    const float sd = sqrtf(o1[0] / (float)max(M, 1)) + 1e-6f;
    for (int f = threadIdx.x; f < M; f += blockDim.x) z[f] = (row[f] - mean) / sd;
    __syncthreads();
    const int half = width > 1 ? width / 2 : 0;
    for (int f = threadIdx.x; f < M; f += blockDim.x) {
        float out = z[f];
        if (half > 0) {
            const int lo = max(0, f - half), hi = min(M - 1, f + half);
            float w[64];
            const int n = hi - lo + 1;
            for (int i = 0; i < n; ++i) w[i] = z[lo + i];
            out = select_kth(w, n, n / 2);
        }
        filt_out[(size_t)s * M + f] = out;
    }
    // probability of the chosen id: softmax(logits)[id]
    const float* lg = logits + (size_t)s * V;
    float mx = -INFINITY;
    for (int v = threadIdx.x; v < V; v += blockDim.x) mx = fmaxf(mx, lg[v]);
    v1[0] = mx;
    block_reduce<1>(v1, true, red, o1);
    mx = o1[0];
    float sum = 0.f;
    for (int v = threadIdx.x; v < V; v += blockDim.x) sum += expf(lg[v] - mx);
    v1[0] = sum;
    block_reduce<1>(v1, false, red, o1);
    if (threadIdx.x == 0) {
        const int id = ids[s];
        probs[s] = (id >= 0 && id < V) ? expf(lg[id] - mx) / o1[0] : 0.f;
    }
}

size_t cross_weights_smem(int SG, int HD, int M) { return ((size_t)SG * HD + (size_t)2 * SG * M) * 4; }

}  // namespace

int alignment_max_median_width() { return 63; }

size_t alignment_part_floats(int n_steps, int L, int M) { return (size_t)n_steps * L * M; }

cudaError_t launch_alignment_rows(const float* qc_trace, const float* cross32, const void* cross_stored, int st_f16,
                                  int n_steps, int L, int H, int KVH, int hd, int m_cap, int M, float scale,
                                  const float* logits, const int* ids, int V, int width, float* part, float* raw_out,
                                  float* filt_out, float* probs, cudaStream_t s) {
    if (n_steps <= 0 || M <= 0) return cudaSuccess;
    if (H % KVH || hd > AL_MAX_HD || width > alignment_max_median_width()) return cudaErrorInvalidValue;
    const int HD = H * hd;
    // widest step group whose shared rows fit (the first call is always a group of one)
    int max_smem = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    const size_t budget = (size_t)max_smem - 2048;
    int SG = AL_MAX_SG;
    while (SG > 1 && cross_weights_smem(SG, HD, M) > budget) SG >>= 1;
    if (cross_weights_smem(SG, HD, M) > budget || (size_t)2 * M * 4 > budget) return cudaErrorInvalidValue;
    const int groups = 1 + (n_steps - 1 + SG - 1) / SG;
    const size_t sm1 = cross_weights_smem(SG, HD, M);
    cudaError_t e = cudaSuccess;
#define AL_LAUNCH(N)                                                                                             \
    case N:                                                                                                      \
        e = cudaFuncSetAttribute(cross_weights_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1); \
        if (e != cudaSuccess) return e;                                                                          \
        ++launch_counter();                                                                                      \
        cross_weights_kernel<N><<<dim3(groups, L), AL_THREADS, sm1, s>>>(qc_trace, cross32, cross_stored, st_f16, \
                                                                         n_steps, L, H, KVH, hd, m_cap, M,        \
                                                                         scale, part);                           \
        break;
    switch (SG) {
        AL_LAUNCH(8)
        AL_LAUNCH(4)
        AL_LAUNCH(2)
        AL_LAUNCH(1)
        default: return cudaErrorInvalidValue;
    }
#undef AL_LAUNCH
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const size_t sm2 = (size_t)2 * M * 4;
    e = cudaFuncSetAttribute(alignment_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2);
    if (e != cudaSuccess) return e;
    ++launch_counter();
    alignment_rows_kernel<<<n_steps, AL_THREADS, sm2, s>>>(part, L, M, width, logits, ids, V, raw_out, filt_out,
                                                           probs);
    return cudaGetLastError();
}

}  // namespace msb
