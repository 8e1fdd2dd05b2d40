// Batch-1 greedy decode on head clusters (fp32 weights), one persistent launch per token
// loop.  Same arithmetic and greedy-loop rules as decode_b1.cu; a different schedule.
//
// The grid is H clusters of CL = 8 CTAs: cluster c owns attention head c in every layer.
// Values that only one head needs are exchanged inside the cluster through distributed
// shared memory (remote st.shared::cluster, then the hardware cluster barrier), so a decoder
// layer (MoonshineLayers.swift:350-379) needs only three grid-wide exchanges:
//
//   QKV     LN1 (every CTA) + this CTA's rows of head c's q|k|v -> all 8 CTAs    [cluster]
//           RoPE on q, k (every CTA); rank 0 appends K/V to the self cache
//   SELF    this CTA's key range -> (max, sum, acc) -> all 8 CTAs, merge         [cluster]
//   O       rows of W_o[:, head c] . attn_c -> partial[c][d]                      [grid]
//           x1 = x + sum_c partial[c]            (every CTA keeps the residual in smem)
//   CQ      LN2 + this CTA's rows of head c's cross q -> all 8 CTAs              [cluster]
//   CROSS   this CTA's memory frames -> partial -> all 8 CTAs, merge             [cluster]
//   CO      as O with the cross output projection                                [grid]
//   FC1     LN3 + this CTA's gr (value, gate) row pairs + bias + SwiGLU (local)
//   FC2     W2[:, its gr columns] . g -> d partial; reduce-scatter in cluster    [cluster]
//           + b2 (cluster 0) -> partial[c][d]                                    [grid]
//   LM      final LN + this CTA's vocabulary rows, per-CTA argmax                [grid]
//
// A grid exchange needs no barrier: partial sums travel as 64-bit words (exchange number,
// value) and a reader polls the H words it needs until every one carries the current number.
//
// Weights: every CTA reads only its own slices, packed once at load time into one
// contiguous per-CTA stream in consumption order with the small per-phase vectors (LayerNorm
// weights, bias slices) in front of the rows they precede.  Thread 0 keeps NSLOT blocks of
// that stream (and of the CTA's cross K/V frames) in flight with bulk copies on mbarriers,
// refilling a slot as soon as the CTA releases it, so weight traffic overlaps the exchanges.
//
// Every wait is bounded (ring blocks by poll count, the grid counter by %globaltimer).  A CTA
// whose wait gives up records an error and from then on skips waits and copies but keeps
// executing the same sequence of cluster barriers; the end-of-step decision (next token,
// stop) is taken identically by every CTA of a cluster, so no barrier is left waiting and a
// failure never hangs the GPU.
#include <algorithm>
#include <type_traits>

#include "cluster_common.cuh"
#include "common.cuh"
#include "kernels.h"

namespace msb {

namespace {

constexpr int CL = 8;         // CTAs per cluster (one cluster per head)
constexpr int NSLOT = 3;      // weight-stream ring slots
constexpr uint64_t GSYNC_TIMEOUT_NS = 2000000000ull;

// ---------------------------------------------------------------- packed stream layout
// Per CTA and layer, segments in consumption order; each is [header][rows] (GEMV rows padded
// to row_stride):
//   QKV  [ln1 (d)]                   [rq  rows x d ]   rows of head c's q|k|v
//   O    []                          [ro  rows x hd]   W_o rows, head c's columns
//   CQ   [ln2 (d)]                   [rcq rows x d ]   rows of head c's cross q
//   CO   []                          [ro  rows x hd]
//   FC1  [ln3 (d), b1 pairs (2 gr)]  [2gr rows x d ]   (value, gate) row pairs
//   FC2  [b2 slice (ro, padded)]     [d rows x gr  ]   W2[:, this CTA's gr columns]
// then after the last layer LM [final_ln (d)][rlm rows x d].
// GEMV rows are stored rf + 4 floats apart (rf % 8 == 0): an odd number of 16-byte units,
// so lanes that own consecutive rows read distinct shared-memory bank groups.  With
// g.qbits the QKV, CQ and FC1 rows (with g.lm_qbits the LM rows) are quantized records
// (quant_row_stride words: codes, then (scale, bias) pairs), at most NT rows per block.

// stored row stride (words) of the QKV / CQ / FC1 rows and of the LM rows (cluster_geom);
// QR = false: the geometry has fp32 rows only and the strides are row_stride(d)
template <bool QR = true>
__host__ __device__ inline int rows_stride_d(const ClusterGeom& g, int d) { return QR ? g.rs_rows : row_stride(d); }
template <bool QR = true>
__host__ __device__ inline int lm_stride(const ClusterGeom& g, int d) { return QR ? g.rs_lm : row_stride(d); }

struct Segs {
    size_t qkv, o, cq, co, fc1, fc2, layer;
    int ro4;
};
template <bool QR = true>
__host__ __device__ inline Segs make_segs(const ClusterGeom& g, int d, int hd) {
    Segs s;
    const int sd = rows_stride_d<QR>(g, d), sh = row_stride(hd);
    s.ro4 = (g.ro + 3) & ~3;
    s.qkv = 0;
    s.o = s.qkv + (size_t)d + (size_t)g.rq * sd;
    s.cq = s.o + (size_t)g.ro * sh;
    s.co = s.cq + (size_t)d + (size_t)g.rcq * sd;
    s.fc1 = s.co + (size_t)g.ro * sh;
    s.fc2 = s.fc1 + (size_t)d + 2 * g.gr + (size_t)2 * g.gr * sd;
    s.layer = s.fc2 + (size_t)s.ro4 + (size_t)d * g.gr;
    return s;
}

enum SegId { SEG_QKV = 0, SEG_O, SEG_CQ, SEG_XKV, SEG_CO, SEG_FC1, SEG_FC2, SEG_LM };

constexpr int MAXB = 320;  // blocks per step a CTA's schedule may have (checked at launch)
constexpr int FC2_MAXR = 1024;  // fc2 rows per block: a CTA's whole fc2 slice is one block for tiny
constexpr int LM_ROWS = 32;     // fp32 LM rows per block (one full lane round of block_gemv)

// Per-warp sums of the values in s and of their squares -> red[0][w], red[1][w] (the
// LayerNorm statistics of the residual, gathered while it is written; a barrier must follow
// before they are read).
__device__ __forceinline__ void warp_stats(float s, float q, float* red) {
    s = warp_sum(s);
    q = warp_sum(q);
    if ((threadIdx.x & 31) == 0) {
        red[threadIdx.x >> 5] = s;
        red[NW + (threadIdx.x >> 5)] = q;
    }
}

struct SegPlan {
    size_t off;  // floats from the CTA's stream base
    int hdr, nrows, rf, gran;  // rf: stored row stride (floats)
    int maxr;                  // rows per block at most
};
// Segment `seg` of `layer` for cluster rank r (CTA index cta); SEG_LM ignores `layer`.
template <bool QR = true>
__host__ __device__ inline SegPlan seg_plan(int seg, int layer, const ClusterGeom& g, const Segs& sg, int d, int hd,
                                           int L, int V, int r, int cta) {
    const size_t lw = (size_t)layer * sg.layer;
    const int nq = max(0, min(g.rq, 3 * hd - r * g.rq));
    const int no = max(0, min(g.ro, d - r * g.ro));
    const int ncq = max(0, min(g.rcq, hd - r * g.rcq));
    const int nlm = max(0, min(g.rlm, V - cta * g.rlm));
    const int sd = rows_stride_d<QR>(g, d), mq = QR && g.qbits ? NT : 64;
    switch (seg) {
        case SEG_QKV: return {lw + sg.qkv, d, nq, sd, 1, mq};
        case SEG_O: return {lw + sg.o, 0, no, row_stride(hd), 1, 64};
        case SEG_CQ: return {lw + sg.cq, d, ncq, sd, 1, mq};
        case SEG_CO: return {lw + sg.co, 0, no, row_stride(hd), 1, 64};
        case SEG_FC1: return {lw + sg.fc1, d + 2 * g.gr, 2 * g.gr, sd, 2, mq};
        case SEG_FC2: return {lw + sg.fc2, sg.ro4, d, g.gr, 1, FC2_MAXR};
        default: return {(size_t)L * sg.layer, d, nlm, lm_stride<QR>(g, d), 1, QR && g.lm_qbits ? NT : LM_ROWS};
    }
}

// Blocks of one step of a CTA's schedule (cross K/V element size esz).
__host__ __device__ inline int blocks_per_step(const ClusterGeom& g, const Segs& sg, int d, int hd, int L, int V,
                                               int r, int cta, int M, int esz) {
    const int slot_floats = g.slot_bytes / 4;
    const int fr = (M + 7) / 8, f0 = min(M, r * fr), f1 = min(M, f0 + fr);
    const int fpb = g.slot_bytes / (2 * hd * esz);
    int n = 0;
    for (int l = 0; l <= L; ++l)
        for (int seg = (l == L ? SEG_LM : SEG_QKV); seg <= (l == L ? SEG_LM : SEG_FC2); ++seg) {
            if (seg == SEG_XKV) {
                n += (f1 - f0 + fpb - 1) / fpb;
                continue;
            }
            const SegPlan sp = seg_plan(seg, l, g, sg, d, hd, L, V, r, cta);
            int row0 = 0;
            bool first = true;
            for (;;) {
                const int nr = next_block_rows(sp.hdr, sp.nrows, sp.rf, sp.gran, slot_floats, row0, first, sp.maxr);
                if (nr < 0) break;
                ++n;
                row0 += nr;
                first = false;
            }
        }
    return n;
}


// xs[k] += the H clusters' partial words pb[q * d + k] of exchange `tag`, summed in cluster
// order, for every k < d; each thread polls exactly the words it adds until their tags match
// (or the CTA has failed; a wait past GSYNC_TIMEOUT_NS records DEV_BARRIER_TIMEOUT).  With
// eight clusters and NT < d <= NT + NT / 4 it is one round of polls: element tid (8 words) and
// a quarter of element NT + tid / 4 (words 2 (tid % 4), +1), all loads in flight together,
// whose four pair sums meet by shuffles in fixed order.  Ends with a barrier; returns the
// cycles spent polling.
__device__ __forceinline__ long long add_cluster_partials(const unsigned long long* pb, float* xs, int d, int H,
                                                          unsigned tag, volatile int* failed, unsigned* status,
                                                          float* red) {
    const int tid = threadIdx.x;
    long long cyc = 0;
    float st1 = 0.f, st2 = 0.f;  // this thread's share of sum(x), sum(x^2)
    auto timed_out = [&](uint64_t& t0) {
        if (t0 == 0) {
            t0 = globaltimer_ns();
        } else if (globaltimer_ns() - t0 > GSYNC_TIMEOUT_NS) {
            atomicCAS(status, DEV_OK, DEV_BARRIER_TIMEOUT);
            *failed = 1;
            return true;
        }
        return false;
    };
    if (H == 8 && d > NT && d - NT <= NT / 4) {
        const int e = d - NT, xi = tid >> 2, qq = (tid & 3) * 2;
        const bool hasx = xi < e;
        const int nb = hasx ? 2 : 0;
        const unsigned long long* srcA = pb + tid;
        const unsigned long long* srcB = pb + NT + min(xi, e - 1) + (size_t)qq * d;
        unsigned long long va[8], vb[2] = {0ull, 0ull};
#pragma unroll
        for (int q = 0; q < 8; ++q) va[q] = ld_tagged(srcA + (size_t)q * d);
#pragma unroll
        for (int q = 0; q < 2; ++q)
            if (q < nb) vb[q] = ld_tagged(srcB + (size_t)q * d);
        const long long c0 = clock64();
        uint64_t t0 = 0;
        for (;;) {
            bool done = true;
#pragma unroll
            for (int q = 0; q < 8; ++q)
                if ((unsigned)(va[q] >> 32) != tag) {
                    done = false;
                    va[q] = ld_tagged(srcA + (size_t)q * d);
                }
#pragma unroll
            for (int q = 0; q < 2; ++q)
                if (q < nb && (unsigned)(vb[q] >> 32) != tag) {
                    done = false;
                    vb[q] = ld_tagged(srcB + (size_t)q * d);
                }
            if (done || *failed || timed_out(t0)) break;
        }
        cyc = clock64() - c0;
        float v = xs[tid];
#pragma unroll
        for (int q = 0; q < 8; ++q) v += __uint_as_float((uint32_t)va[q]);
        xs[tid] = v;
        const float s2 = __uint_as_float((uint32_t)vb[0]) + __uint_as_float((uint32_t)vb[1]);
        const float o1 = __shfl_xor_sync(FULL, s2, 1);
        const float pr = (tid & 1) ? o1 + s2 : s2 + o1;  // words 0-3 / 4-7 of the element
        const float o2 = __shfl_xor_sync(FULL, pr, 2);
        const float tot = (tid & 2) ? o2 + pr : pr + o2;
        if (hasx && (tid & 3) == 0) {
            const float xv = xs[NT + xi] + tot;
            xs[NT + xi] = xv;
            st1 += xv;
            st2 += xv * xv;
        }
        st1 += v;
        st2 += v * v;
    } else {
        for (int k = tid; k < d; k += NT) {
            unsigned long long v[16];
#pragma unroll
            for (int q = 0; q < 16; ++q)
                if (q < H) v[q] = ld_tagged(pb + (size_t)q * d + k);
            const long long c0 = clock64();
            uint64_t t0 = 0;
            for (;;) {
                bool done = true;
#pragma unroll
                for (int q = 0; q < 16; ++q)
                    if (q < H && (unsigned)(v[q] >> 32) != tag) {
                        done = false;
                        v[q] = ld_tagged(pb + (size_t)q * d + k);
                    }
                if (done || *failed || timed_out(t0)) break;
            }
            cyc += clock64() - c0;
            float a = xs[k];
            for (int q = 0; q < H; ++q) a += __uint_as_float((uint32_t)v[q]);
            xs[k] = a;
            st1 += a;
            st2 += a * a;
        }
    }
    warp_stats(st1, st2, red);
    __syncthreads();
    return cyc;
}
// The same as one out-of-line copy: the quantized-row kernels (measured faster so; the fp32
// kernel is faster with the body inlined at its three exchanges per layer).
__device__ __noinline__ long long add_cluster_partials_call(const unsigned long long* pb, float* xs, int d, int H,
                                                            unsigned tag, volatile int* failed, unsigned* status,
                                                            float* red) {
    return add_cluster_partials(pb, xs, d, H, tag, failed, status, red);
}

// xl = LN(xs) * wln over d inputs from statistics gathered with the residual (red: per-warp
// sums of x and x^2, see warp_stats): mean = sum / d, variance = sum(x^2) / d - mean^2; for
// rows quantized to qb (= QB) bits also the vector block_gemv_q reads (d % 64 == 0 there, so
// every iteration covers whole warps).  One out-of-line copy serves every call site of the
// kernel, so its instructions stay cached between the segments of a layer.  Ends with a
// barrier.
template <int QB>
__device__ __noinline__ void ln_apply(const float* xs, const float* wln, float* xl, int d, float* xq, int qb,
                                      const float* red) {
    float s = 0.f, q = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        s += red[w];
        q += red[NW + w];
    }
    const float mean = s / (float)d;
    const float rstd = rsqrtf(fmaxf(q / (float)d - mean * mean, 0.f) + 1e-5f);
    for (int k = threadIdx.x; k < d; k += NT) {
        const float v = (xs[k] - mean) * rstd * wln[k];
        xl[k] = v;
        if constexpr (QB != 0)
            if (qb) quant_input<QB>(v, k, xq, d);
    }
    __syncthreads();
}

// QB: code width of the quantized rows the geometry streams (gm.qbits / gm.lm_qbits, each QB
// or 0); the fp32 instantiation (QB = 0) carries none of their code.
template <int HDT, int QB>
__global__ void __launch_bounds__(NT, 1) decode_cluster_kernel(DecodeParams p, ClusterGeom gm) {
    constexpr bool QR = QB != 0;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[NSLOT];
    __shared__ int s_failed;
    __shared__ int x_best[CL], x_fail[CL];  // end-of-step decision inputs (remote-written)
    __shared__ float s_bv[NW];
    __shared__ int s_bi[NW];
    __shared__ BlockEnt s_tab[2][MAXB];
    __shared__ int s_nb[2];

    const int d = p.d, H = p.H, V = p.V, L = p.L, M = p.M;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int c = (int)cluster_index(), r = (int)cluster_rank();
    const int cta = c * CL + r, ncta = H * CL;
    const int slot_bytes = gm.slot_bytes, slot_floats = slot_bytes / 4;
    const Segs sg = make_segs<QR>(gm, d, HDT);
    const int nq = max(0, min(gm.rq, 3 * HDT - r * gm.rq));
    const int no = max(0, min(gm.ro, d - r * gm.ro));
    const int ncq = max(0, min(gm.rcq, HDT - r * gm.rcq));
    const int nlm = max(0, min(gm.rlm, V - cta * gm.rlm));
    const int fr = (M + CL - 1) / CL;
    const int f0 = min(M, r * fr), f1 = min(M, f0 + fr);
    const float scale = p.scale;
    const int half_nd = p.nd >> 1;

    // shared memory carve-up (same offsets in every CTA: remote addresses come from mapa)
    unsigned char* ring = smem_raw;
    float* skv = reinterpret_cast<float*>(smem_raw + (size_t)NSLOT * slot_bytes);  // [2][skv_keys][HDT] (fp32 worst)
    float* xs = skv + (size_t)2 * gm.skv_keys * HDT;  // [d] residual
    float* xl = xs + d;                                // [d] LayerNorm output
    float* qkv_s = xl + d;                             // [3 HDT] head c's q|k|v (remote-written)
    float* qc_s = qkv_s + 3 * HDT;                     // [HDT] cross q (remote-written)
    float* sp_s = qc_s + HDT;                          // [CL][HDT + 4] self partials (remote-written)
    float* cp_s = sp_s + CL * (HDT + 4);               // [CL][HDT + 4] cross partials (remote-written)
    float* fp2_s = cp_s + CL * (HDT + 4);              // [d] this CTA's fc2 partial (remote-read)
    float* attn_s = fp2_s + d;                         // [HDT]
    float* wpart = attn_s + HDT;                       // [NW][HDT + 4]
    float* g_s = wpart + NW * (HDT + 4);               // [gr] SwiGLU outputs
    float* gb_s = g_s + ((gm.gr + 3) & ~3);            // [2 gr] b1 (value, gate) pairs
    float* b2_s = gb_s + 2 * gm.gr;                    // [ro4] b2 slice
    float* sc = b2_s + sg.ro4;                         // [NW][32]
    float* gpart = sc + NW * 32;                       // [NW][64] block_gemv warp partials
    float* gres = gpart + NW * 64;                     // [64] block_gemv results ([NT], then
                                                       // [d + d / 16] quantized GEMV input, when QR)
    float* xq_s = gres + NT;

    if (tid == 0) {
        for (int i = 0; i < NSLOT; ++i) mbar_init(&full[i], 1);
        s_failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    cluster_barrier();  // every CTA of the cluster is running before any remote store

    // ------------------------------------------------------------ producer (thread 0)
    // The block schedule of a step is the same for every step after the first (which reads
    // the fp32 cross K/V), so thread 0 records two tables once and then only indexes them.
    uint32_t n_iss = 0, n_con = 0, n_ok = 0;  // issued, consumed, confirmed landed
    const float* pbase = gm.packed + (size_t)cta * gm.cta_floats;
    if (tid == 0) {
        for (int tb = 0; tb < 2; ++tb) {
            const int esz = (tb == 0 || !p.kv_f16) ? 4 : 2;
            const char* xsrc = tb == 0 ? reinterpret_cast<const char*>(p.cross32)
                                       : reinterpret_cast<const char*>(p.cross_stored);
            const int fpb = slot_bytes / (2 * HDT * esz);
            int n = 0;
            for (int l = 0; l <= L; ++l)
                for (int seg = (l == L ? SEG_LM : SEG_QKV); seg <= (l == L ? SEG_LM : SEG_FC2); ++seg) {
                    if (seg == SEG_XKV) {
                        for (int a = f0; a < f1 && n < MAXB; a += fpb) {
                            const int nf = min(fpb, f1 - a);
                            const size_t kr = ((((size_t)l * 2 + 0) * H + c) * p.m_cap + a) * HDT * esz;
                            const size_t vr = ((((size_t)l * 2 + 1) * H + c) * p.m_cap + a) * HDT * esz;
                            const uint32_t b = (uint32_t)nf * HDT * esz;
                            s_tab[tb][n++] = {xsrc + kr, xsrc + vr, b, b};
                        }
                        continue;
                    }
                    const SegPlan sp = seg_plan<QR>(seg, l, gm, sg, d, HDT, L, V, r, cta);
                    int row0 = 0;
                    bool first = true;
                    while (n < MAXB) {
                        const int nr = next_block_rows(sp.hdr, sp.nrows, sp.rf, sp.gran, slot_floats, row0, first, sp.maxr);
                        if (nr < 0) break;
                        const float* src = pbase + sp.off + (first ? 0 : sp.hdr + (size_t)row0 * sp.rf);
                        const uint32_t floats = (first ? sp.hdr : 0) + (uint32_t)nr * sp.rf;
                        s_tab[tb][n++] = {src, nullptr, floats * 4, 0u};
                        row0 += nr;
                        first = false;
                    }
                }
            s_nb[tb] = n;
        }
    }
    __syncthreads();
    const uint32_t nb0 = (uint32_t)s_nb[0], nb1 = (uint32_t)s_nb[1];
    const uint32_t n_total = p.n_steps > 0 ? nb0 + (uint32_t)(p.n_steps - 1) * nb1 : 0u;
    // issue block n_iss of the whole launch (thread 0; nothing once failed or exhausted)
    const bool hint = gm.l2_keep > 0.f;
    const uint64_t l2pol = hint ? make_l2_policy(fminf(gm.l2_keep, 1.f)) : 0ull;
    auto issue_next = [&]() {
        if (n_iss >= n_total || s_failed) return;
        const BlockEnt e = n_iss < nb0 ? s_tab[0][n_iss] : s_tab[1][(n_iss - nb0) % nb1];
        const int slot = n_iss % NSLOT;
        mbar_expect_tx(&full[slot], e.b0 + e.b1);
        unsigned char* dst = ring + (size_t)slot * slot_bytes;
        if (hint) {
            bulk_load_hint(dst, e.s0, e.b0, &full[slot], l2pol);
            if (e.b1) bulk_load_hint(dst + e.b0, e.s1, e.b1, &full[slot], l2pol);
        } else {
            bulk_load(dst, e.s0, e.b0, &full[slot]);
            if (e.b1) bulk_load(dst + e.b0, e.s1, e.b1, &full[slot]);
        }
        ++n_iss;
    };
    if (tid == 0)
        for (int i = 0; i < NSLOT; ++i) issue_next();

    // ------------------------------------------------------------ helpers
    long long cyc_take = 0, cyc_cbar = 0, cyc_poll = 0;  // trace-only accumulators (CTA 0)
    const bool tr0 = p.trace != nullptr && cta == 0 && tid == 0;
    auto fail = [&](unsigned code) {
        atomicCAS(p.status, DEV_OK, code);
        s_failed = 1;
    };
    // the next block (every thread); once failed, no wait and the slot holds stale data
    auto take = [&]() -> const float* {
        const int slot = n_con % NSLOT;
        const long long c0 = tr0 ? clock64() : 0;
        if (!s_failed) {
            if (mbar_wait(&full[slot], (n_con / NSLOT) & 1)) n_ok = n_con + 1;
            else fail(DEV_WAIT_TIMEOUT);
        }
        if (tr0) cyc_take += clock64() - c0;
        __syncthreads();
        // every thread is done with the previous block: its slot takes the next copy
        if (tid == 0 && n_con >= 1) issue_next();
        return reinterpret_cast<const float*>(ring + (size_t)slot * slot_bytes);
    };
    auto release = [&]() { ++n_con; };
    // walk the blocks of one segment: body(block, rows, row0, nr, first)
    auto for_blocks = [&](int seg, int layer, auto&& body) {
        const SegPlan sp = seg_plan<QR>(seg, layer, gm, sg, d, HDT, L, V, r, cta);
        int row0 = 0;
        bool first = true;
        for (;;) {
            const int nr = next_block_rows(sp.hdr, sp.nrows, sp.rf, sp.gran, slot_floats, row0, first, sp.maxr);
            if (nr < 0) break;
            const float* blk = take();
            body(blk, blk + (first ? sp.hdr : 0), row0, nr, first);
            release();
            row0 += nr;
            first = false;
        }
    };
    // block GEMV of rows of d inputs against xl: quantized records (rs words apart) or fp32 rows
    auto rows_gemv = [&](const float* rows, int nr, bool quant, int rs) {
        if constexpr (QR) {
            if (quant) {
                block_gemv_q<QB>(reinterpret_cast<const uint32_t*>(rows), nr, d, rs, gm.qgroup, xq_s, gpart, gres);
                return;
            }
        }
        block_gemv(rows, nr, d, row_stride(d), xl, gpart, gres);
    };
    auto cbar = [&]() {
        const long long c0 = tr0 ? clock64() : 0;
        cluster_barrier();
        if (tr0) cyc_cbar += clock64() - c0;
    };
    // Grid exchanges carry their data in tagged words: exchange number `epoch` (the same
    // sequence in every CTA) is the tag, and a reader polls the words it needs until every
    // tag matches.  The buffers are zeroed before each launch, so no stale word matches.
    unsigned epoch = 0;
    // wait until the n words at src[q * stride] (q < n <= 16) carry `tag`; payloads -> out
    auto wait_tagged = [&](const unsigned long long* src, size_t stride, int n, unsigned tag, uint32_t* out) {
        unsigned long long v[16];
#pragma unroll
        for (int q = 0; q < 16; ++q)
            if (q < n) v[q] = ld_tagged(src + q * stride);
        const long long c0 = tr0 ? clock64() : 0;
        uint64_t t0 = 0;
        for (;;) {
            bool done = true;
#pragma unroll
            for (int q = 0; q < 16; ++q)
                if (q < n && (unsigned)(v[q] >> 32) != tag) {
                    done = false;
                    v[q] = ld_tagged(src + q * stride);
                }
            if (done || s_failed) break;
            if (t0 == 0) t0 = globaltimer_ns();
            else if (globaltimer_ns() - t0 > GSYNC_TIMEOUT_NS) {
                fail(DEV_BARRIER_TIMEOUT);
                break;
            }
        }
        if (tr0) cyc_poll += clock64() - c0;
#pragma unroll
        for (int q = 0; q < 16; ++q)
            if (q < n) out[q] = (uint32_t)v[q];
    };
    // xl = LN(xs) * wln (wln in shared memory); for rows quantized to qb bits also the
    // vector block_gemv_q reads: xl pre-scaled per input, then sums over each 16 inputs
    // (d % 64 == 0 there, so every iteration below covers whole warps)
    // LayerNorm statistics of xs, gathered where xs is written (the embedding row and every
    // partial-sum exchange) so that the LayerNorm itself is one elementwise pass
    __shared__ float s_red[2 * NW];
    auto layer_norm = [&](const float* wln, int qb) { ln_apply<QB>(xs, wln, xl, d, xq_s, qb, s_red); };
    int par = 0;
    // xs += sum over clusters (fixed order) of partial[par][.] of exchange `epoch`
    auto add_partials = [&]() {
        const unsigned long long* pb = gm.part + (size_t)par * H * d;
        long long cy;
        if constexpr (QR) cy = add_cluster_partials_call(pb, xs, d, H, epoch, &s_failed, p.status, s_red);
        else cy = add_cluster_partials(pb, xs, d, H, epoch, &s_failed, p.status, s_red);
        if (tr0) cyc_poll += cy;
        par ^= 1;
    };
    // output-projection partial of head c: rows r*ro + i of W[:, head c] . attn_s
    auto out_proj = [&](int seg, int layer) {
        ++epoch;
        unsigned long long* pb = gm.part + (size_t)par * H * d + (size_t)c * d;
        for_blocks(seg, layer, [&](const float*, const float* rows, int row0, int nr, bool) {
            block_gemv(rows, nr, HDT, row_stride(HDT), attn_s, gpart, gres);
            for (int i = tid; i < nr; i += NT) st_tagged(pb + r * gm.ro + row0 + i, epoch, __float_as_uint(gres[i]));
        });
    };
    // merge of the per-warp softmax states in wpart -> slot r of `dst` in every cluster CTA
    auto publish_partial = [&](float* dst) {
        __syncthreads();
        // every thread merges the warp states for its elements e of (m, l, acc[0..HDT))
        float m = -INFINITY;
        for (int q = 0; q < NW; ++q) m = fmaxf(m, wpart[q * (HDT + 4)]);
        const uint32_t base_a = smem_u32(dst + r * (HDT + 4));
        for (int e = tid; e < HDT + 2; e += NT) {
            float v = 0.f;
            if (e == 0) {
                v = m;
            } else {
                for (int q = 0; q < NW; ++q) {
                    const float* wp = wpart + q * (HDT + 4);
                    if (wp[0] != -INFINITY) v = fmaf(e == 1 ? wp[1] : wp[4 + e - 2], expf(wp[0] - m), v);
                }
            }
            const uint32_t off = (e < 2) ? e * 4 : (4 + (e - 2)) * 4;
            for (int q = 0; q < CL; ++q) st_dsmem(mapa_rank(base_a + off, q), v);
        }
        cbar();
    };
    auto merge_cluster = [&](const float* src) {  // attn_s = merge of the CL partials
        for (int e = tid; e < HDT; e += NT) {
            float mx = -INFINITY;
            for (int q = 0; q < CL; ++q) mx = fmaxf(mx, src[q * (HDT + 4)]);
            float lsum = 0.f, o = 0.f;
            for (int q = 0; q < CL; ++q) {
                const float* sq = src + q * (HDT + 4);
                if (sq[0] == -INFINITY) continue;
                const float f = expf(sq[0] - mx);
                lsum = fmaf(sq[1], f, lsum);
                o = fmaf(sq[4 + e], f, o);
            }
            attn_s[e] = (lsum > 0.f) ? o / lsum : 0.f;
        }
        __syncthreads();
    };
    auto store_warp_state = [&](float m, float lsum, float a0, float a1) {
        float* wp = wpart + w * (HDT + 4);
        if (lane == 0) {
            wp[0] = m;
            wp[1] = lsum;
        }
        if (2 * lane < HDT) {
            wp[4 + 2 * lane] = a0;
            wp[4 + 2 * lane + 1] = a1;
        }
    };

    // optional %globaltimer trace of CTA 0: per step [start, 9 per layer, LM rows, LM argmax, clock64,
    // cycles waiting for ring blocks, in cluster barriers, polling the grid counter]
    const bool tracing = p.trace != nullptr && cta == 0 && tid == 0;
    int tpos = 0;
    auto stamp = [&]() {
        if (tracing && tpos < p.trace_cap) p.trace[tpos++] = globaltimer_ns();
    };

    const uint32_t qkv_a = smem_u32(qkv_s), qc_a = smem_u32(qc_s), fp2_a = smem_u32(fp2_s);
    const uint32_t xb_a = smem_u32(x_best), xf_a = smem_u32(x_fail);
    unsigned long long* xam = gm.part + (size_t)2 * H * d;  // [ncta][value, index] per step
    unsigned epoch_lm = 0;
    int tok = p.start_token;
    int step = 0;
    bool stop = false;
    for (; step < p.n_steps && !stop; ++step) {
        const int t = step;
        stamp();
        {
            float e1 = 0.f, e2 = 0.f;
            for (int k = tid; k < d; k += NT) {
                const float v = __ldg(p.embed + (size_t)tok * d + k);
                xs[k] = v;
                e1 += v;
                e2 += v * v;
            }
            warp_stats(e1, e2, s_red);
        }
        __syncthreads();
        for (int l = 0; l < L; ++l) {
            // ---- self-K/V prefetch of this CTA's cached keys [j0, min(j1, t))
            const int nk = t + 1, kr = (nk + CL - 1) / CL;
            const int j0 = min(nk, r * kr), j1 = min(nk, j0 + kr), jc = min(j1, t);
            const int kesz = p.kv_f16 ? 2 : 4;
            {
                const int rowb = HDT * kesz, pieces = rowb / 16;
                const char* kc = reinterpret_cast<const char*>(p.self_k);
                const char* vc = reinterpret_cast<const char*>(p.self_v);
                char* sk = reinterpret_cast<char*>(skv);
                char* sv = sk + (size_t)gm.skv_keys * HDT * 4;
                const int total = (jc > j0 ? jc - j0 : 0) * pieces;
                for (int i = tid; i < 2 * total; i += NT) {
                    const int kv = i >= total, ii = kv ? i - total : i;
                    const int j = j0 + ii / pieces, pc = ii % pieces;
                    const size_t src = ((((size_t)l * H + c) * p.t_cap + j) * HDT) * kesz + (size_t)pc * 16;
                    cp16((kv ? sv : sk) + (size_t)(j - j0) * rowb + pc * 16, (kv ? vc : kc) + src);
                }
                asm volatile("cp.async.commit_group;\n" ::: "memory");
            }
            // ---- LN1 + this CTA's q|k|v rows -> every CTA of the cluster
            for_blocks(SEG_QKV, l, [&](const float* blk, const float* rows, int row0, int nr, bool first) {
                if (first) layer_norm(blk, gm.qbits);
                rows_gemv(rows, nr, gm.qbits != 0, gm.rs_rows);
                for (int e = tid; e < nr * CL; e += NT) {  // row i -> rank q
                    const int i = e / CL, q = e - (e / CL) * CL;
                    st_dsmem(mapa_rank(qkv_a + 4 * (r * gm.rq + row0 + i), q), gres[i]);
                }
            });
            cbar();
            stamp();
            // RoPE on q and k (interleaved pairs of the first nd dims), every CTA
            for (int i = tid; i < 2 * half_nd; i += NT) {
                const int which = i / half_nd, pi = i - which * half_nd;  // 0: q, 1: k
                float* v = qkv_s + which * HDT + 2 * pi;
                const float cs = p.rope_cos[(size_t)t * half_nd + pi], sn = p.rope_sin[(size_t)t * half_nd + pi];
                const float a0 = v[0], a1 = v[1];
                v[0] = a0 * cs - a1 * sn;
                v[1] = a0 * sn + a1 * cs;
            }
            __syncthreads();
            if (r == 0 && !s_failed) {  // K/V append, stored rounded when the cache is fp16
                for (int e = tid; e < 2 * HDT; e += NT) {
                    const int kv = e / HDT, dim = e - kv * HDT;
                    const float v = qkv_s[HDT + e];
                    const size_t idx = (((size_t)l * H + c) * p.t_cap + t) * HDT + dim;
                    void* base = kv ? p.self_v : p.self_k;
                    if (p.kv_f16) reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v);
                    else reinterpret_cast<float*>(base)[idx] = v;
                }
            }
            // ---- self-attention over keys [j0, j1): cached rows from skv, key t fresh fp32
            asm volatile("cp.async.wait_all;\n" ::: "memory");
            __syncthreads();
            {
                float m = -INFINITY, lsum = 0.f, a0 = 0.f, a1 = 0.f;
                const float q0 = (2 * lane < HDT) ? qkv_s[2 * lane] : 0.f;
                const float q1 = (2 * lane < HDT) ? qkv_s[2 * lane + 1] : 0.f;
                for (int j = j0 + w; j < j1; j += NW) {
                    float k0v = 0.f, k1v = 0.f, v0 = 0.f, v1 = 0.f;
                    if (2 * lane < HDT) {
                        if (j == t) {
                            k0v = qkv_s[HDT + 2 * lane];
                            k1v = qkv_s[HDT + 2 * lane + 1];
                            v0 = qkv_s[2 * HDT + 2 * lane];
                            v1 = qkv_s[2 * HDT + 2 * lane + 1];
                        } else if (p.kv_f16) {
                            const __half* sk = reinterpret_cast<const __half*>(skv);
                            const __half* sv = sk + (size_t)gm.skv_keys * HDT * 2;
                            const float2 kf = __half22float2(*reinterpret_cast<const __half2*>(sk + (size_t)(j - j0) * HDT + 2 * lane));
                            const float2 vf = __half22float2(*reinterpret_cast<const __half2*>(sv + (size_t)(j - j0) * HDT + 2 * lane));
                            k0v = kf.x; k1v = kf.y; v0 = vf.x; v1 = vf.y;
                        } else {
                            const float* sk = skv;
                            const float* sv = skv + (size_t)gm.skv_keys * HDT;
                            const float2 kf = *reinterpret_cast<const float2*>(sk + (size_t)(j - j0) * HDT + 2 * lane);
                            const float2 vf = *reinterpret_cast<const float2*>(sv + (size_t)(j - j0) * HDT + 2 * lane);
                            k0v = kf.x; k1v = kf.y; v0 = vf.x; v1 = vf.y;
                        }
                    }
                    const float s = warp_sum(fmaf(q0, k0v, q1 * k1v)) * scale;
                    const float mn = fmaxf(m, s);
                    const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
                    const float pj = expf(s - mn);
                    lsum = lsum * corr + pj;
                    a0 = fmaf(a0, corr, pj * v0);
                    a1 = fmaf(a1, corr, pj * v1);
                    m = mn;
                }
                store_warp_state(m, lsum, a0, a1);
            }
            publish_partial(sp_s);
            stamp();
            merge_cluster(sp_s);
            // ---- output projection -> x1
            out_proj(SEG_O, l);
            stamp();
            add_partials();
            // ---- LN2 + cross q rows -> every CTA of the cluster
            for_blocks(SEG_CQ, l, [&](const float* blk, const float* rows, int row0, int nr, bool first) {
                if (first) layer_norm(blk, gm.qbits);
                rows_gemv(rows, nr, gm.qbits != 0, gm.rs_rows);
                for (int e = tid; e < nr * CL; e += NT) {
                    const int i = e / CL, q = e - (e / CL) * CL;
                    st_dsmem(mapa_rank(qc_a + 4 * (r * gm.rcq + row0 + i), q), gres[i]);
                }
                if (p.qc_trace)
                    for (int i = tid; i < nr; i += NT)
                        p.qc_trace[((size_t)step * L + l) * H * HDT + c * HDT + r * gm.rcq + row0 + i] = gres[i];
            });
            cbar();
            stamp();
            // ---- cross attention over frames [f0, f1): fp32 at step 0, stored copy after
            {
                const bool f16 = step > 0 && p.kv_f16;
                const int esz = f16 ? 2 : 4;
                const int fpb = slot_bytes / (2 * HDT * esz);
                float m = -INFINITY, lsum = 0.f, a0 = 0.f, a1 = 0.f;
                QSlice qs;
                float* qr = qs.v;
                {
                    const int G = f16 ? KeyShape<HDT, true>::G : KeyShape<HDT, false>::G;
                    const int NE = f16 ? KeyShape<HDT, true>::NE : KeyShape<HDT, false>::NE;
                    const int EP = f16 ? 8 : 4;
                    const int sub = lane % G;
#pragma unroll
                    for (int e = 0; e < 8; ++e) qr[e] = (e < EP && sub < NE) ? qc_s[sub * EP + e] : 0.f;
                }
                for (int a = f0; a < f1; a += fpb) {
                    const int nf = min(fpb, f1 - a);
                    const float* blk = take();
                    const int kpw = (nf + NW - 1) / NW;
                    const int k0 = min(nf, w * kpw), k1 = min(nf, k0 + kpw);
                    const void* vblk = reinterpret_cast<const unsigned char*>(blk) + (size_t)nf * HDT * esz;
                    const float4 st0 = make_float4(m, lsum, a0, a1);
                    const float4 st1 = f16 ? attend_keys<HDT, true>(blk, vblk, k0, k1, qs, scale, sc + w * 32, st0, lane)
                                           : attend_keys<HDT, false>(blk, vblk, k0, k1, qs, scale, sc + w * 32, st0, lane);
                    m = st1.x;
                    lsum = st1.y;
                    a0 = st1.z;
                    a1 = st1.w;
                    release();
                }
                store_warp_state(m, lsum, a0, a1);
            }
            publish_partial(cp_s);
            stamp();
            merge_cluster(cp_s);
            // ---- cross output projection -> x2
            out_proj(SEG_CO, l);
            stamp();
            add_partials();
            // ---- LN3 + fc1 + SwiGLU on this CTA's gr indices (rows alternate value, gate)
            for_blocks(SEG_FC1, l, [&](const float* blk, const float* rows, int row0, int nr, bool first) {
                if (first) {
                    for (int i = tid; i < 2 * gm.gr; i += NT) gb_s[i] = blk[d + i];
                    layer_norm(blk, gm.qbits);  // ends with a barrier: gb_s is visible too
                }
                rows_gemv(rows, nr, gm.qbits != 0, gm.rs_rows);
                for (int i = tid; i < (nr >> 1); i += NT) {  // row0 and nr even: whole pairs
                    const int pr = (row0 >> 1) + i;
                    const float val = gres[2 * i] + gb_s[2 * pr], gate = gres[2 * i + 1] + gb_s[2 * pr + 1];
                    g_s[pr] = val * silu(gate);
                }
            });
            stamp();
            // ---- fc2 partial over this CTA's gr columns, reduce-scatter in the cluster
            for_blocks(SEG_FC2, l, [&](const float* blk, const float* rows, int row0, int nr, bool first) {
                if (first)
                    for (int i = tid; i < sg.ro4; i += NT) b2_s[i] = blk[i];
                for (int i = tid; i < nr; i += NT) {
                    const float4* row = reinterpret_cast<const float4*>(rows + (size_t)i * gm.gr);
                    const float4* g4 = reinterpret_cast<const float4*>(g_s);
                    float a = 0.f;
                    for (int q = 0; q < (gm.gr >> 2); ++q) {
                        const float4 wv = row[q], gv = g4[q];
                        a = fmaf(wv.x, gv.x, fmaf(wv.y, gv.y, fmaf(wv.z, gv.z, fmaf(wv.w, gv.w, a))));
                    }
                    fp2_s[row0 + i] = a;
                }
            });
            cbar();
            stamp();
            {
                ++epoch;
                unsigned long long* pb = gm.part + (size_t)par * H * d + (size_t)c * d;
                for (int i = tid; i < no; i += NT) {
                    const int k = r * gm.ro + i;
                    float v = 0.f;
                    for (int q = 0; q < CL; ++q) v += ld_dsmem(mapa_rank(fp2_a + 4 * k, q));
                    if (c == 0) v += b2_s[i];
                    st_tagged(pb + k, epoch, __float_as_uint(v));
                }
            }
            stamp();
            add_partials();
        }

        // ---- final LN + LM head rows + argmax
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        const int lm_row0 = cta * gm.rlm;
        for_blocks(SEG_LM, 0, [&](const float* blk, const float* rows, int row0, int nr, bool first) {
            if (first) layer_norm(blk, gm.lm_qbits);
            rows_gemv(rows, nr, gm.lm_qbits != 0, gm.rs_lm);
            for (int i = tid; i < nr; i += NT) {
                const float v = gres[i];
                const int row = lm_row0 + row0 + i;
                const float key =
                    p.inv_temp > 0.f ? v * p.inv_temp + gumbel_noise(p.seed, (unsigned)step, (unsigned)row) : v;
                if (key > bv) {  // a thread sees its rows in increasing order: ties keep the lowest
                    bv = key;
                    bi = row;
                }
                if (p.logits_out) p.logits_out[(size_t)step * V + row] = v;
            }
        });
        stamp();
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float vo = __shfl_xor_sync(FULL, bv, o);
            const int io = __shfl_xor_sync(FULL, bi, o);
            if (vo > bv || (vo == bv && io < bi)) {
                bv = vo;
                bi = io;
            }
        }
        if (lane == 0) {
            s_bv[w] = bv;
            s_bi[w] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            float v = s_bv[0];
            int i = s_bi[0];
            for (int q = 1; q < NW; ++q)
                if (s_bv[q] > v || (s_bv[q] == v && s_bi[q] < i)) {
                    v = s_bv[q];
                    i = s_bi[q];
                }
            ++epoch_lm;
            st_tagged(xam + 2 * cta, epoch_lm, __float_as_uint(v));
            st_tagged(xam + 2 * cta + 1, epoch_lm, (uint32_t)i);
        }
        if (tid != 0) ++epoch_lm;
        stamp();
        if (w == 0) {
            float v = -INFINITY;
            int i = 0x7fffffff;
            for (int b = lane; b < ncta; b += 32) {
                uint32_t u[2];
                wait_tagged(xam + 2 * b, 1, 2, epoch_lm, u);
                const float vb = __uint_as_float(u[0]);
                const int ib = (int)u[1];
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
            // every CTA of the cluster decides from the same inputs: rank r's view -> slot r
            if (lane < CL) {
                st_dsmem_i(mapa_rank(xb_a + 4 * r, lane), i);
                st_dsmem_i(mapa_rank(xf_a + 4 * r, lane), s_failed);
            }
        }
        cbar();
        const int best = x_best[0];
        int anyfail = 0;
        for (int q = 0; q < CL; ++q) anyfail |= x_fail[q] | (x_best[q] != best);
        if (anyfail) {
            if (tid == 0) atomicCAS(p.status, DEV_OK, (unsigned)DEV_WAIT_TIMEOUT);
            stop = true;
        } else {
            if (cta == 0 && tid == 0) p.ids_out[step] = best;
            if (!p.forced && best == p.eos) {
                if (cta == 0 && tid == 0) *p.hit_eos = 1;
                stop = true;
            }
            tok = p.teacher ? p.teacher[step] : best;
            if (!stop && step + 1 < p.n_steps && (tok < 0 || tok >= V)) {
                if (tid == 0) atomicCAS(p.status, DEV_OK, (unsigned)DEV_BAD_TOKEN);
                stop = true;
            }
        }
        if (tracing && tpos + 4 <= p.trace_cap) {
            p.trace[tpos++] = (unsigned long long)clock64();
            p.trace[tpos++] = (unsigned long long)cyc_take;
            p.trace[tpos++] = (unsigned long long)cyc_cbar;
            p.trace[tpos++] = (unsigned long long)cyc_poll;
            cyc_take = cyc_cbar = cyc_poll = 0;
        }
        __syncthreads();  // x_best / x_fail are rewritten next step only after two more barriers
    }
    if (cta == 0 && tid == 0) *p.n_done = step;
    // drain every copy not confirmed landed (bounded), then leave together with the cluster
    if (tid == 0)
        for (uint32_t k = n_ok; k < n_iss; ++k) mbar_wait(&full[k % NSLOT], (k / NSLOT) & 1);
    __syncthreads();
    cluster_barrier();
}

size_t cluster_smem_bytes(const ClusterGeom& g, int d, int hd) {
    const int ro4 = (g.ro + 3) & ~3;
    const size_t floats = (size_t)2 * g.skv_keys * hd + 2 * d + 3 * hd + hd + 2 * CL * (hd + 4) + d + hd +
                          NW * (hd + 4) + ((g.gr + 3) & ~3) + 2 * g.gr + ro4 + NW * 32 + NW * 64 +
                          (g.qbits || g.lm_qbits ? NT + d + d / 16 + 4 : 64);
    return (size_t)NSLOT * g.slot_bytes + floats * 4;
}

}  // namespace

bool cluster_quant_ok(int d, int bits, int gs) {
    if (!(bits == 2 || bits == 4 || bits == 8) || gs <= 0 || d % gs) return false;
    return gs % (128 / bits) == 0;  // a 16-byte chunk of codes lies inside one group
}

bool cluster_geom(int d, int H, int KVH, int hd, int I, int V, int L, int t_cap, ClusterGeom* g, int qbits,
                  int lm_qbits, int qgroup) {
    if (KVH != H || (d & 7) || (hd & 7) || hd > 64 || I % (H * CL) || ((I / (H * CL)) & 3)) return false;
    if ((qbits && !cluster_quant_ok(d, qbits, qgroup)) || (lm_qbits && !cluster_quant_ok(d, lm_qbits, qgroup)))
        return false;
    ClusterGeom r{};
    r.qbits = qbits;
    r.lm_qbits = lm_qbits;
    r.qgroup = qbits || lm_qbits ? qgroup : 0;
    r.rs_rows = qbits ? quant_row_stride(d, qbits, qgroup) : row_stride(d);
    r.rs_lm = lm_qbits ? quant_row_stride(d, lm_qbits, qgroup) : row_stride(d);
    r.rq = (3 * hd + CL - 1) / CL;
    r.ro = (d + CL - 1) / CL;
    r.rcq = (hd + CL - 1) / CL;
    r.gr = I / (H * CL);
    r.rlm = (V + H * CL - 1) / (H * CL);
    const int sd = rows_stride_d(r, d), sl = lm_stride(r, d);
    // ring slot: at least 52 KB, and large enough that a CTA's whole fc1 segment (header and
    // every (value, gate) row pair, at most 64 fp32 / NT quantized rows) is one block when
    // that stays within 56 KB (wider models take their fc1 rows in several blocks); with a
    // quantized LM head, large enough for NT of its rows behind the final-norm header when
    // that stays within 56 KB
    {
        const size_t fc1 = ((size_t)d + 2 * r.gr + (size_t)std::min(2 * r.gr, qbits ? NT : 64) * sd) * 4;
        size_t want = 52 * 1024;
        if (fc1 <= 56 * 1024) want = std::max(want, fc1);
        const size_t lm = ((size_t)d + (size_t)std::min(r.rlm, NT) * sl) * 4;
        if (lm_qbits && lm <= 56 * 1024) want = std::max(want, lm);
        r.slot_bytes = (int)((want + 127) / 128 * 128);
    }
    r.skv_keys = (t_cap + CL - 1) / CL;
    const Segs s = make_segs(r, d, hd);
    r.cta_floats = (size_t)L * s.layer + (size_t)d + (size_t)r.rlm * sl;
    // every segment's first block (header + one row group) and a fp32 K/V frame fit a slot
    const size_t slot_f = (size_t)r.slot_bytes / 4;
    if ((size_t)d + std::max(sd, sl) > slot_f || (size_t)d + 2 * r.gr + 2 * sd > slot_f ||
        (size_t)s.ro4 + r.gr > slot_f ||
        (size_t)2 * hd * 4 > slot_f)
        return false;
    if (cluster_smem_bytes(r, d, hd) > 208 * 1024) return false;  // + ~16 KB of static shared memory
    *g = r;
    return true;
}

int cluster_ctas(int H) { return H * CL; }

// Packed per-CTA stream of the decoder weights in consumption order (see make_segs):
// device-to-device copies, once per model.
cudaError_t pack_cluster_weights(const ClusterGeom& g, const DecodeLayerW* layers_host, int L, const float* lm_head,
                                 const uint32_t* lm_q, const float* final_ln, int d, int H, int hd, int I, int V,
                                 float* packed, cudaStream_t s) {
    const Segs sg = make_segs(g, d, hd);
    const int HD = H * hd;
    const int sd = rows_stride_d(g, d), sh = row_stride(hd), sl = lm_stride(g, d);
    // source rows of d inputs: fp32 rows (pitch d, d floats copied) or quantized records
    // (pitch and copied width sd words)
    const int rw = g.qbits ? sd : d;
    if ((g.qbits && (!layers_host[0].qkv_q || !layers_host[0].cq_q || !layers_host[0].w1_q)) ||
        (g.lm_qbits && !lm_q))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaSuccess;
    auto copy_rows = [&](float* dst, const float* src, size_t row_floats, size_t src_pitch_floats, size_t nrows,
                         size_t dst_pitch_floats) {
        if (e != cudaSuccess || nrows == 0) return;
        e = cudaMemcpy2DAsync(dst, dst_pitch_floats * 4, src, src_pitch_floats * 4, row_floats * 4, nrows,
                              cudaMemcpyDeviceToDevice, s);
    };
    auto copy_vec = [&](float* dst, const float* src, size_t n) {
        if (n) copy_rows(dst, src, n, n, 1, n);
    };
    for (int c = 0; c < H; ++c)
        for (int r = 0; r < CL; ++r) {
            const int cta = c * CL + r;
            float* base = packed + (size_t)cta * g.cta_floats;
            for (int l = 0; l < L; ++l) {
                const DecodeLayerW& W = layers_host[l];
                float* lw = base + (size_t)l * sg.layer;
                // QKV: ln1, then head c's q|k|v rows: local row i -> global (i / hd) * HD + c * hd + i % hd
                copy_vec(lw + sg.qkv, W.ln1, d);
                const float* qkv = g.qbits ? reinterpret_cast<const float*>(W.qkv_q) : W.wqkv;
                const float* cq = g.qbits ? reinterpret_cast<const float*>(W.cq_q) : W.wcq;
                const float* w1 = g.qbits ? reinterpret_cast<const float*>(W.w1_q) : W.w1;
                for (int i = r * g.rq; i < std::min(3 * hd, (r + 1) * g.rq);) {
                    const int grp = i / hd, end = std::min(std::min(3 * hd, (r + 1) * g.rq), (grp + 1) * hd);
                    copy_rows(lw + sg.qkv + d + (size_t)(i - r * g.rq) * sd,
                              qkv + ((size_t)grp * HD + c * hd + i % hd) * rw, rw, rw, end - i, sd);
                    i = end;
                }
                const int r0o = r * g.ro, no = std::max(0, std::min(g.ro, d - r0o));
                copy_rows(lw + sg.o, W.wo + (size_t)r0o * HD + c * hd, hd, HD, no, sh);
                copy_rows(lw + sg.co, W.wco + (size_t)r0o * HD + c * hd, hd, HD, no, sh);
                const int r0q = r * g.rcq, ncq = std::max(0, std::min(g.rcq, hd - r0q));
                copy_vec(lw + sg.cq, W.ln2, d);
                copy_rows(lw + sg.cq + d, cq + ((size_t)c * hd + r0q) * rw, rw, rw, ncq, sd);
                // FC1: ln3, (value, gate) bias pairs, (value, gate) row pairs
                const int jb = c * g.gr * CL + r * g.gr;
                float* f1 = lw + sg.fc1;
                copy_vec(f1, W.ln3, d);
                copy_rows(f1 + d, W.b1 + jb, 1, 1, g.gr, 2);
                copy_rows(f1 + d + 1, W.b1 + I + jb, 1, 1, g.gr, 2);
                copy_rows(f1 + d + 2 * g.gr, w1 + (size_t)jb * rw, rw, rw, g.gr, 2 * sd);
                copy_rows(f1 + d + 2 * g.gr + sd, w1 + ((size_t)I + jb) * rw, rw, rw, g.gr, 2 * sd);
                // FC2: b2 slice of this rank's reduce-scatter range, then W2[:, jb .. jb + gr)
                copy_vec(lw + sg.fc2, W.b2 + r0o, no);
                copy_rows(lw + sg.fc2 + sg.ro4, W.w2 + jb, g.gr, I, d, g.gr);
            }
            float* lm = base + (size_t)L * sg.layer;
            copy_vec(lm, final_ln, d);
            const int r0 = cta * g.rlm, nr = std::max(0, std::min(g.rlm, V - r0));
            if (g.lm_qbits)
                copy_rows(lm + d, reinterpret_cast<const float*>(lm_q) + (size_t)r0 * sl, sl, sl, nr, sl);
            else
                copy_rows(lm + d, lm_head + (size_t)r0 * d, d, d, nr, sl);
        }
    return e;
}

template <int HDT>
const void* cluster_kernel_for(int qb) {
    switch (qb) {
        case 2: return (const void*)decode_cluster_kernel<HDT, 2>;
        case 4: return (const void*)decode_cluster_kernel<HDT, 4>;
        case 8: return (const void*)decode_cluster_kernel<HDT, 8>;
        default: return (const void*)decode_cluster_kernel<HDT, 0>;
    }
}

cudaError_t launch_decode_cluster(const DecodeParams& p, const ClusterGeom& g, cudaStream_t stream) {
    const void* fn = nullptr;
    const int qb = g.qbits ? g.qbits : g.lm_qbits;
    if (g.qbits && g.lm_qbits && g.qbits != g.lm_qbits) return cudaErrorInvalidValue;
    switch (p.hd) {
        case 32: fn = cluster_kernel_for<32>(qb); break;
        case 40: fn = cluster_kernel_for<40>(qb); break;
        case 48: fn = cluster_kernel_for<48>(qb); break;
        case 64: fn = cluster_kernel_for<64>(qb); break;
        default: return cudaErrorInvalidValue;
    }
    if (p.KVH != p.H || p.t_cap > g.skv_keys * CL || !g.packed || !g.part) return cudaErrorInvalidValue;
    {
        const Segs sg = make_segs(g, p.d, p.hd);
        for (int cta = 0; cta < p.H * CL; ++cta)
            for (int esz : {2, 4})
                if (blocks_per_step(g, sg, p.d, p.hd, p.L, p.V, cta % CL, cta, p.M, esz) > MAXB)
                    return cudaErrorCooperativeLaunchTooLarge;  // schedule too long: caller keeps the grid kernel
    }
    const size_t smem = cluster_smem_bytes(g, p.d, p.hd);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.H * CL, 1, 1);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = CL;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int active = 0;
    e = cudaOccupancyMaxActiveClusters(&active, fn, &cfg);
    if (e != cudaSuccess) return e;
    if (active < p.H) return cudaErrorCooperativeLaunchTooLarge;  // every cluster must be resident
    void* args[] = {const_cast<DecodeParams*>(&p), const_cast<ClusterGeom*>(&g)};
    ++launch_counter();
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace msb
