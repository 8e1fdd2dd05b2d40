// fp32 SIMT GEMM with fused epilogues, C = A * B^T (both operands K-contiguous).
// Used by the fp32 encoder path: causal convs as implicit GEMMs (strided A rows over a
// zero-padded activation buffer), QKV / O / MLP projections with bias, activation and
// residual fused, and the once-per-utterance cross-attention K/V projection scattered
// straight into the decoder's KV layout (fp32 and fp16 copies).  Two batched forms for many
// streaming states at once: one GEMM over rows gathered from anywhere (a row pointer each),
// writing each row to its own place (the frontend convs of every stream) or through a K/V
// scatter per row (the cross K/V of every stream's new memory rows).
#include "common.cuh"
#include "kernels.h"

namespace msb {

namespace {

constexpr int BN = 64;
constexpr int BK = 16;
constexpr int NT = 256;

// Column n of a cross K/V projection -> (layer, k|v, head, dim) of the decoder's layout
// [L][2][kv_heads][frame_cap][head_dim], at frame `frame`.
__device__ __forceinline__ void kv_store(float* out32, void* out16, int kv_heads, int head_dim, int frame_cap,
                                         int frame, int n, float v) {
    const int kvdim = kv_heads * head_dim;
    const int layer = n / (2 * kvdim);
    const int rem = n - layer * 2 * kvdim;
    const int kv = rem / kvdim;
    const int c = rem - kv * kvdim;
    const int head = c / head_dim;
    const int dim = c - head * head_dim;
    const size_t idx = ((((size_t)layer * 2 + kv) * kv_heads + head) * frame_cap + (size_t)frame) * head_dim + dim;
    if (out32) out32[idx] = v;
    if (out16) reinterpret_cast<__half*>(out16)[idx] = __float2half_rn(v);
}

__device__ __forceinline__ void epilogue_store(const GemmEpilogue& ep, int m, int n, float v) {
    if (ep.bias) v += ep.bias[n];
    if (ep.act == ACT_SILU) v = silu(v);
    else if (ep.act == ACT_GELU) v = gelu_erf(v);
    if (ep.residual) v += ep.residual[(size_t)m * ep.ldr + n];
    if (!ep.kv_scatter) {
        ep.out[(size_t)m * ep.ldc + n] = v;
        return;
    }
    kv_store(ep.kv_out32, ep.kv_out16, ep.kv_heads, ep.head_dim, ep.frame_cap, m + ep.frame_offset, n, v);
}

// One BM x BN output tile at (blockIdx.y * BM, blockIdx.x * BN).  With a_rows, row m of A is
// at a_rows[m] (lda unused) and the result goes either through the per-row K/V scatter
// kv_rows[m] (ep gives kv_heads and head_dim) or, with bias and activation, to out_rows[m];
// the arithmetic is the same in every form.
template <int BM>
__device__ __forceinline__ void gemm_f32_tile(const float* __restrict__ A, int lda, const float* __restrict__ B,
                                              int ldb, int M, int N, int K, const GemmEpilogue& ep,
                                              const float* const* __restrict__ a_rows = nullptr,
                                              const KvRowDst* __restrict__ kv_rows = nullptr,
                                              float* const* __restrict__ out_rows = nullptr) {
    constexpr int TM = BM / 16;          // rows per thread
    constexpr int A_F4 = BM * BK / 4;    // float4 per A tile
    constexpr int A_PER_T = A_F4 / NT;   // 2 (BM=128) or 1 (BM=64)
    __shared__ float As[2][BK][BM + 4];
    __shared__ float Bs[2][BK][BN + 4];

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;

    float4 ra[A_PER_T];
    float4 rb;
    const float* arow[A_PER_T];  // this thread's A rows (null past M)
#pragma unroll
    for (int i = 0; i < A_PER_T; ++i) {
        const int m = m0 + ((tid + i * NT) >> 2);
        arow[i] = m < M ? (a_rows ? a_rows[m] : A + (size_t)m * lda) : nullptr;
    }

    auto load_tiles = [&](int k0) {
#pragma unroll
        for (int i = 0; i < A_PER_T; ++i) {
            const int f = tid + i * NT;
            const int kq = (f & 3) << 2;
            const int k = k0 + kq;
            ra[i] = (arow[i] && k < K) ? __ldg(reinterpret_cast<const float4*>(arow[i] + k))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        {
            const int row = tid >> 2, kq = (tid & 3) << 2;
            const int n = n0 + row, k = k0 + kq;
            rb = (n < N && k < K) ? __ldg(reinterpret_cast<const float4*>(B + (size_t)n * ldb + k))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store_tiles = [&](int s) {
#pragma unroll
        for (int i = 0; i < A_PER_T; ++i) {
            const int f = tid + i * NT;
            const int row = f >> 2, kq = (f & 3) << 2;
            As[s][kq + 0][row] = ra[i].x;
            As[s][kq + 1][row] = ra[i].y;
            As[s][kq + 2][row] = ra[i].z;
            As[s][kq + 3][row] = ra[i].w;
        }
        const int row = tid >> 2, kq = (tid & 3) << 2;
        Bs[s][kq + 0][row] = rb.x;
        Bs[s][kq + 1][row] = rb.y;
        Bs[s][kq + 2][row] = rb.z;
        Bs[s][kq + 3][row] = rb.w;
    };

    float acc[TM][4];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

    const int ktiles = (K + BK - 1) / BK;
    load_tiles(0);
    store_tiles(0);
    __syncthreads();
    for (int kt = 0; kt < ktiles; ++kt) {
        const int s = kt & 1;
        if (kt + 1 < ktiles) load_tiles((kt + 1) * BK);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[TM];
#pragma unroll
            for (int i = 0; i < TM; i += 4) {
                const float4 t = *reinterpret_cast<const float4*>(&As[s][kk][ty * TM + i]);
                a[i] = t.x; a[i + 1] = t.y; a[i + 2] = t.z; a[i + 3] = t.w;
            }
            const float4 b = *reinterpret_cast<const float4*>(&Bs[s][kk][tx * 4]);
#pragma unroll
            for (int i = 0; i < TM; ++i) {
                acc[i][0] = fmaf(a[i], b.x, acc[i][0]);
                acc[i][1] = fmaf(a[i], b.y, acc[i][1]);
                acc[i][2] = fmaf(a[i], b.z, acc[i][2]);
                acc[i][3] = fmaf(a[i], b.w, acc[i][3]);
            }
        }
        if (kt + 1 < ktiles) store_tiles(s ^ 1);
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int m = m0 + ty * TM + i;
        if (m >= M) continue;
        if (kv_rows) {
            const KvRowDst d = kv_rows[m];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = n0 + tx * 4 + j;
                if (n < N) kv_store(d.out32, d.out16, ep.kv_heads, ep.head_dim, d.frame_cap, d.frame_row, n, acc[i][j]);
            }
            continue;
        }
        if (out_rows) {
            float* o = out_rows[m];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = n0 + tx * 4 + j;
                if (n >= N) continue;
                float v = acc[i][j];
                if (ep.bias) v += ep.bias[n];
                if (ep.act == ACT_SILU) v = silu(v);
                else if (ep.act == ACT_GELU) v = gelu_erf(v);
                o[n] = v;
            }
            continue;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n < N) epilogue_store(ep, m, n, acc[i][j]);
        }
    }
}

template <int BM>
__global__ void __launch_bounds__(NT) gemm_f32_kernel(const float* __restrict__ A, int lda,
                                                       const float* __restrict__ B, int ldb,
                                                       int M, int N, int K, GemmEpilogue ep) {
    gemm_f32_tile<BM>(A, lda, B, ldb, M, N, K, ep);
}

template <int BM>
__global__ void __launch_bounds__(NT) gemm_f32_rows_kernel(const float* const* __restrict__ a_rows,
                                                            const KvRowDst* __restrict__ kv_rows,
                                                            float* const* __restrict__ out_rows, int M,
                                                            const float* __restrict__ B, int ldb, int N, int K,
                                                            GemmEpilogue ep) {
    gemm_f32_tile<BM>(nullptr, 0, B, ldb, M, N, K, ep, a_rows, kv_rows, out_rows);
}

cudaError_t launch_rows(const float* const* a_rows, const KvRowDst* kv_rows, float* const* out_rows, int M,
                        const float* B, int ldb, int N, int K, const GemmEpilogue& ep, cudaStream_t stream) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if ((K & 3) || (ldb & 3) || (reinterpret_cast<uintptr_t>(B) & 15) || (M + 63) / 64 > 65535)
        return cudaErrorInvalidValue;
    const int gx = (N + BN - 1) / BN;
    ++launch_counter();
    if ((long long)gx * ((M + 127) / 128) >= 2 * 148) {
        dim3 grid(gx, (M + 127) / 128);
        gemm_f32_rows_kernel<128><<<grid, NT, 0, stream>>>(a_rows, kv_rows, out_rows, M, B, ldb, N, K, ep);
    } else {
        dim3 grid(gx, (M + 63) / 64);
        gemm_f32_rows_kernel<64><<<grid, NT, 0, stream>>>(a_rows, kv_rows, out_rows, M, B, ldb, N, K, ep);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_f32(const float* A, int lda, const float* B, int ldb, int M, int N,
                            int K, const GemmEpilogue& ep, cudaStream_t stream) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if ((K & 3) || (lda & 3) || (ldb & 3) || (reinterpret_cast<uintptr_t>(A) & 15) ||
        (reinterpret_cast<uintptr_t>(B) & 15))
        return cudaErrorInvalidValue;
    const int gx = (N + BN - 1) / BN;
    const int tiles128 = gx * ((M + 127) / 128);
    ++launch_counter();
    if (tiles128 >= 2 * 148) {
        dim3 grid(gx, (M + 127) / 128);
        gemm_f32_kernel<128><<<grid, NT, 0, stream>>>(A, lda, B, ldb, M, N, K, ep);
    } else {
        dim3 grid(gx, (M + 63) / 64);
        gemm_f32_kernel<64><<<grid, NT, 0, stream>>>(A, lda, B, ldb, M, N, K, ep);
    }
    return cudaGetLastError();
}

cudaError_t launch_gemm_f32_rows(const float* const* a_rows, float* const* out_rows, int M, const float* B, int ldb,
                                 int N, int K, const float* bias, int act, cudaStream_t stream) {
    GemmEpilogue ep;
    ep.bias = bias;
    ep.act = act;
    return launch_rows(a_rows, nullptr, out_rows, M, B, ldb, N, K, ep, stream);
}

cudaError_t launch_gemm_f32_kv_rows(const float* const* a_rows, const KvRowDst* dst, int M, const float* B, int ldb,
                                    int N, int K, int kv_heads, int head_dim, cudaStream_t stream) {
    if (kv_heads <= 0 || head_dim <= 0) return cudaErrorInvalidValue;
    GemmEpilogue ep;
    ep.kv_scatter = 1;
    ep.kv_heads = kv_heads;
    ep.head_dim = head_dim;
    return launch_rows(a_rows, dst, nullptr, M, B, ldb, N, K, ep, stream);
}

cudaError_t preload_gemm_f32() {
    cudaFuncAttributes a;
    cudaError_t e = cudaFuncGetAttributes(&a, gemm_f32_kernel<64>);
    return e != cudaSuccess ? e : cudaFuncGetAttributes(&a, gemm_f32_kernel<128>);
}

}  // namespace msb
