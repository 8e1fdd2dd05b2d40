// Host-side launchers of the Moonshine B200 kernels.  Plain device pointers and sizes;
// every launcher enqueues on `stream` and returns cudaGetLastError().
#pragma once

#include <utility>

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace msb {

// Count of kernel launches issued through these launchers on this thread.
int64_t& launch_counter();

// Launches of the kernels that call pdl_wait() (the batched decode step's) carry the
// programmatic-stream-serialization attribute while this thread-local flag is set, so each
// can launch while its predecessor finishes (CUDA graphs keep the programmatic edges).
bool& pdl_launches();
template <class... Params, class... Args>
cudaError_t launch_kernel(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_launches() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
// The same with thread-block clusters of (1, 1, cluster_z) CTAs (cluster_z > 1).
template <class... Params, class... Args>
cudaError_t launch_kernel_cluster_z(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t stream, int cluster_z, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = (unsigned)cluster_z;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_launches() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Device-side error codes reported through a kernel's status word.
enum : unsigned { DEV_OK = 0, DEV_BARRIER_TIMEOUT = 1, DEV_BAD_TOKEN = 2, DEV_WAIT_TIMEOUT = 5 };

// ---------------------------------------------------------------- frontend
// Frame features: per 80-sample frame CMVN, asinh(exp(log_k) x), SiLU(x W^T).
// audio [n_frames * frame_len]; w [dim, frame_len]; out rows at out + f * ld_out.
cudaError_t launch_frame_features(const float* audio, int n_frames, int frame_len,
                                  const float* log_k, const float* w, int dim,
                                  float* out, int ld_out, cudaStream_t stream);
// The same for nb streams in one launch (device tables): stream z's nf[z] frames start at
// audio + aoff[z] and its rows at out[z]; nf_max >= every nf[z].
cudaError_t launch_frame_features_batch(const float* audio, const long long* aoff, const int* nf, float* const* out,
                                        int nb, int nf_max, int frame_len, const float* log_k, const float* w,
                                        int dim, int ld_out, cudaStream_t stream);
// dst[z][0, n[z]) = src[z][0, n[z]) for z < nb (zeros where src[z] is null); device tables,
// every n[z] a multiple of 4 floats and every row 16-byte aligned.
cudaError_t launch_copy_rows_batch(const float* const* src, float* const* dst, const int* n, int nb,
                                   cudaStream_t stream);

// ---------------------------------------------------------------- fp32 GEMM
// C[m, n] = epilogue( sum_k A[m*lda + k] * B[n*ldb + k] ).
enum GemmAct { ACT_NONE = 0, ACT_SILU = 1, ACT_GELU = 2 };
struct GemmEpilogue {
    const float* bias = nullptr;       // [N]
    int act = ACT_NONE;
    const float* residual = nullptr;   // added after the activation, [M, ldr]
    int ldr = 0;
    float* out = nullptr;              // [M, ldc]
    int ldc = 0;
    // Cross-attention K/V scatter: column n -> (layer, k|v, head, dim); rows are frames.
    // Writes out32 (fp32, nullable) and out16 (fp16, nullable) at
    // (((layer*2 + kv)*kv_heads + head)*frame_cap + m)*head_dim + dim.
    int kv_scatter = 0;
    float* kv_out32 = nullptr;
    void* kv_out16 = nullptr;
    int kv_heads = 0, head_dim = 0, frame_cap = 0, frame_offset = 0;
};
cudaError_t launch_gemm_f32(const float* A, int lda, const float* B, int ldb, int M, int N,
                            int K, const GemmEpilogue& ep, cudaStream_t stream);
// C = act(A B^T + bias) over M rows gathered from anywhere: row r of A at a_rows[r] (16-byte
// aligned, K floats), its result at out_rows[r] (device tables).  Each value is the same as
// launch_gemm_f32 gives.
cudaError_t launch_gemm_f32_rows(const float* const* a_rows, float* const* out_rows, int M, const float* B, int ldb,
                                 int N, int K, const float* bias, int act, cudaStream_t stream);
// Where row r of a gathered-rows cross K/V GEMM lands: the K/V scatter of GemmEpilogue
// into out32 / out16 (either nullable) with frame_cap rows per segment, at frame frame_row.
struct KvRowDst {
    float* out32;
    void* out16;
    int frame_cap, frame_row;
};
// Cross K/V projection of M memory rows from anywhere (row r at a_rows[r], 16-byte aligned,
// K floats) scattered per row as dst[r] says (device tables): many streams' new memory rows
// in one launch.  Each value is the same as launch_gemm_f32 with kv_scatter gives.
cudaError_t launch_gemm_f32_kv_rows(const float* const* a_rows, const KvRowDst* dst, int M, const float* B, int ldb,
                                    int N, int K, int kv_heads, int head_dim, cudaStream_t stream);

// ---------------------------------------------------------------- bf16 tensor-core GEMM
// C = epi(A * B^T) with A [M, K] and B [N, K] bf16 (K-major), fp32 accumulation in TMEM.
// A goes through a 3-D tensor map (k, y, z); k-block kb belongs to tap kb / kb_per_tap and
// reads A at (k, tap_y[tap], m + tap_z[tap]) and B at column tap * k_per_tap + k.
enum TcEpiMode {
    TC_EPI_STD = 0,      // bias / activation / residual / fp32 + bf16 stores / K-V scatter
    TC_EPI_ROPE_KV = 1,  // decoder q|k|v: partial interleaved RoPE, K/V appended to the cache
    TC_EPI_SWIGLU = 2,   // interleaved (value, gate) columns -> bf16 value * silu(gate)
    TC_EPI_ARGMAX = 3,   // per-row argmax (ties -> lowest column) + optional fp32 logits
    TC_EPI_ACCUM = 4,    // out += acc (+ bias): the residual update (one CTA finalises each element)
};

// Paged self-attention K/V of the batched engine.  A page holds `page` consecutive positions
// of one row for every layer, K and V: the element of (layer, k|v, kv head, position j, dim)
// lives at pool + phys * page_elems + layer_off + kv * KVH * page * hd
//                  + (head * page + j % page) * hd + dim   (elements of the KV dtype),
// with phys = table[row * table_stride + j / page] the row's physical page (-1: no page; a
// write there is dropped and a read sees no key).  layer_off selects the layer.
struct PagedKv {
    void* pool = nullptr;
    const int* table = nullptr;
    int table_stride = 0;         // logical pages per row in the table
    int page = 16;                // positions per page
    long long page_elems = 0;     // elements per page (all layers, K and V)
    long long layer_off = 0;      // elements from a page's start to this layer's K
    int kv_f16 = 0;
    int reach = 0;                // > 0: no position the launch sees reaches this (sizes the
                                  // self-attention rounds); 0: table_stride * page
};

// Decoder q|k|v epilogue parameters (row m = batch slot b).
struct TcRopeKv {
    const int* pos = nullptr;       // device: position of this step
    const float* cos_t = nullptr;   // [pos][nd/2]
    const float* sin_t = nullptr;
    int nd = 0, hd = 0, H = 0, KVH = 0;
    float* q = nullptr;             // [M, H*hd] fp32
    float* kv_new = nullptr;        // [M, 2*KVH*hd] fp32 (k then v)
    PagedKv kv;                     // this step's K/V go to position *pos of row m
};

constexpr int TC_MAX_SPLITS = 8;  // portable cluster size
// LayerNorm folded into the GEMM that consumes it (batched decoder): B holds W[n][k] * w[k]
// (w the LayerNorm weight) and csum[n] is the sum of that stored row, so row m of
// LN(x) W^T = rstd_m (x_m . W'_n - mean_m csum[n]) with A the raw residual x.  The row
// statistics come from the kernel that last wrote the residual, as (mean, M2) pairs of
// column tiles of tile_n columns (stats[t * ld + m]), merged here in tile order
// (Chan, Golub and LeVeque 1979); eps 1e-5.
struct TcLnFold {
    const float2* stats = nullptr;
    const float* csum = nullptr;  // [N]
    int ntiles = 0, tile_n = 0, ld = 0, K = 0;
};

struct TcGemmArgs {
    int M = 0, N = 0;
    int taps = 1, kb_per_tap = 0, k_per_tap = 0;
    int tap_y[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int tap_z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int splits = 1;                       // k-splits over blockIdx.z (<= TC_MAX_SPLITS): the splits
                                          // of a tile form one thread-block cluster and sum their
                                          // partial tiles in split order through distributed
                                          // shared memory (deterministic), every mode
    int mode = TC_EPI_STD;
    GemmEpilogue ep;                      // fp32 outputs / scatter (as the fp32 GEMM)
    __nv_bfloat16* out_bf16 = nullptr;    // optional bf16 copy of the output [M, ldc_bf16]
    int ldc_bf16 = 0;
    size_t bf16_lo_off = 0;               // != 0: out_bf16 (STD, SWIGLU) also gets the bf16 of the
                                          // remainder v - bf16(v) this many elements further on
    TcRopeKv rope;
    TcLnFold lnf;                         // stats != null: LayerNorm folded in (STD, ROPE_KV,
                                          // SWIGLU, ARGMAX), applied before the mode's epilogue
    float2* stats_out = nullptr;          // ACCUM: (mean, M2) of each updated residual row over
    int stats_ld = 0;                     //   this tile's columns at [blockIdx.x * stats_ld + m];
                                          //   out_bf16 (+ bf16_lo_off) gets its bf16 planes
    unsigned long long* argmax = nullptr; // [M] packed (ordered value, ~column) maxima
    float inv_temp = 0.f;                 // ARGMAX: 0 greedy, else maxima of logit * inv_temp + Gumbel
    unsigned seed = 0;                    //   noise of (seed, step + (row << 20), column);
    const int* step = nullptr;            //   step from this device word
    unsigned* status = nullptr;           // device word; 5 = a bounded wait gave up
};
}  // namespace msb
struct CUtensorMap_st;
namespace msb {
// Tensor maps (128B swizzle, 64-element k boxes).  A: dims (k, y, z) with byte strides of
// y and z, box z rows; B: dims (k, rows) with a row stride, box `box_rows` rows.
bool tc_make_map_3d(CUtensorMap_st* map, const void* base, uint64_t dim_k, uint64_t dim_y, uint64_t dim_z,
                    uint64_t stride_y_bytes, uint64_t stride_z_bytes, uint32_t box_z);
bool tc_make_map_2d(CUtensorMap_st* map, const void* base, uint64_t dim_k, uint64_t rows, uint64_t row_stride_bytes,
                    uint32_t box_rows);
cudaError_t launch_gemm_tc(const CUtensorMap_st& map_a, const CUtensorMap_st& map_b, const TcGemmArgs& g, int bn,
                           cudaStream_t stream);
// The same with split operands (both lo maps set): A = A_hi + A_lo and B = B_hi + B_lo as bf16
// planes, accumulated as A_hi B_hi + A_hi B_lo + A_lo B_hi (about fp32 accuracy: each operand
// is kept to ~2^-17 relative).  With both lo maps null it is launch_gemm_tc.
cudaError_t launch_gemm_tc_split(const CUtensorMap_st& map_a, const CUtensorMap_st* map_a_lo,
                                 const CUtensorMap_st& map_b, const CUtensorMap_st* map_b_lo, const TcGemmArgs& g,
                                 int bn, cudaStream_t stream);

// ---------------------------------------------------------------- encoder
// Row LayerNorm (biased variance): out = (x-mean)/sqrt(var+eps) * (w + w_offset)
// (+ add[(add_row0 + r) * dim] when add != nullptr).
cudaError_t launch_layernorm_rows(const float* x, int rows, int dim, const float* w,
                                  float w_offset, float eps, const float* add, int add_row0,
                                  float* out, cudaStream_t stream);

// Multi-head attention over a [T, 3*H*hd] q|k|v buffer with a per-query key window
// [t-left+1, t+right-1] (left <= 0 means no window: all keys).  out [T, H*hd].
// Segments (seg_rows > 0): rows [s * seg_rows, s * seg_rows + seg_len[s]) are one utterance;
// queries see keys of their own utterance, rows past its length get zeros.  out and
// out_bf16 are each nullable (not both).
cudaError_t launch_window_attention(const float* qkv, int T, int H, int kv_heads, int hd,
                                    int left, int right, float scale, float* out,
                                    cudaStream_t stream, int seg_rows = 0, const int* seg_len = nullptr,
                                    __nv_bfloat16* out_bf16 = nullptr, size_t lo_off = 0);
// CMVN + asinh of every frame of a batch into segment rows (row r: frame r % seg_rows - 4 of
// utterance r / seg_rows, zeros where there is none), bf16 [rows][frame_len]: the input of
// the frame Linear as one GEMM.  audio / n_frames: device arrays of the utterances.
// (lo_off here and in the two launchers around it: the low plane of a split operand, as for
// launch_ln_bf16.)
cudaError_t launch_frame_norm_rows(const float* const* audio, const int* n_frames, int rows, int seg_rows,
                                   int frame_len, const float* log_k, __nv_bfloat16* out, cudaStream_t stream,
                                   size_t lo_off = 0);
// Frame features written as bf16 (same math as launch_frame_features).
cudaError_t launch_frame_features_bf16(const float* audio, int n_frames, int frame_len, const float* log_k,
                                       const float* w, int dim, __nv_bfloat16* out, int ld_out,
                                       cudaStream_t stream);
// Final encoder LayerNorm of segment rows + pos_emb[t], gathered to rows off[s] + t of out
// (fp32) and out_bf16 for t < len[s].
cudaError_t launch_ln_gather_rows(const float* x, int rows, int seg_rows, int dim, const float* w, float w_offset,
                                  float eps, const float* pos_emb, const int* len, const int* off, float* out,
                                  __nv_bfloat16* out_bf16, cudaStream_t stream, size_t lo_off = 0);

// Segment rows gathered from per-segment device pointers (device arrays src[nseg], T[nseg]):
// row t of segment b = src[b] + t * dim for t < T[b], zero rows up to seg_rows.
cudaError_t launch_gather_seg_rows(const float* const* src, const int* T, int nseg, int seg_rows, int dim, float* out,
                                   cudaStream_t stream);
// Final encoder LayerNorm + pos_emb of cnt[b] rows of segment b starting at row off[b],
// written to dst[b] (positions pos[b]..); device arrays of nseg entries.
cudaError_t launch_ln_scatter_rows(const float* x, int nseg, int max_cnt, int seg_rows, int dim, const float* w,
                                   float w_offset, float eps, const float* pos_emb, const int* off, const int* cnt,
                                   const int* pos, float* const* dst, cudaStream_t stream);

// ---------------------------------------------------------------- decoder
struct DecodeLayerW {
    const float* wqkv;   // [3*d, d]  (q rows, k rows, v rows)
    const float* wo;     // [d, d]
    const float* wcq;    // [d, d]
    const float* wco;    // [d, d]
    const float* w1;     // [2I, d]
    const float* b1;     // [2I]
    const float* w2;     // [d, I]
    const float* b2;     // [d]
    const float* ln1;    // [d]
    const float* ln2;    // [d]
    const float* ln3;    // [d]
    // Affine-quantized row records of q|k|v, cross q and fc1 (quant_row_stride words per row:
    // the checkpoint's packed codes, then one (scale, bias) float pair per group), or null.
    // Only the clustered batch-1 kernel reads them; every other kernel uses the fp32 rows.
    const uint32_t* qkv_q;
    const uint32_t* cq_q;
    const uint32_t* w1_q;
};

// Words per quantized row record of rf inputs: rf * bits / 32 code words, then rf / gs
// (scale, bias) float pairs, padded to an odd number of 16-byte units so that lanes owning
// consecutive rows read distinct shared-memory bank groups.
__host__ __device__ inline int quant_row_stride(int rf, int bits, int gs) {
    const int words = rf * bits / 32 + 2 * (rf / gs);
    int units = (words + 3) / 4;
    if (!(units & 1)) ++units;
    return units * 4;
}

struct DecodeParams {
    int d, H, KVH, hd, I, V, L, nd;   // dims; nd = rotary dims
    float scale;
    const DecodeLayerW* layers;       // device array [L]
    const float* final_ln;            // [d]
    const float* lm_head;             // [V, d]
    const float* embed;               // [V, d]
    const float* rope_cos;            // [max_pos, nd/2]
    const float* rope_sin;
    int max_pos;
    // self KV [L][KVH][t_cap][hd]; fp16 when kv_f16
    void* self_k;
    void* self_v;
    int t_cap;
    int kv_f16;
    // cross KV [L][2][KVH][m_cap][hd]: fp32 copy (step 0) and stored copy (fp16 when kv_f16)
    const float* cross32;
    const void* cross_stored;
    int m_cap, M;
    // scratch (device)
    float* xb;         // [2][d] residual stream, ping-pong across layers
    float* qbuf;       // [H*hd] self-attention query (after RoPE)
    float* qc;         // [H*hd] cross-attention query
    float* kvnew;      // [2*KVH*hd] this step's K/V (fp32)
    float* x1;         // [d] residual after self-attention
    float* x2;         // [d] residual after cross-attention
    float* spart;      // [H * self_chunks][hd + 2] self-attention chunk partials
    float* cpart;      // [rounds][grid][8][hd + 2] cross-attention per-CTA partials
    float* gbuf;       // [I] SwiGLU output
    float* amax_val;   // [gridDim]
    int* amax_idx;     // [gridDim]
    // token loop
    int start_token;
    int n_steps;          // decoder calls to run
    int forced;           // 1: never stop on EOS
    float inv_temp;       // 0: greedy argmax; else sample softmax(logit * inv_temp) (Gumbel-max)
    unsigned seed;        // sampling: noise of (seed, step, vocabulary index)
    const int* teacher;   // nullable [n_steps]: next input ids
    int eos;
    int* ids_out;         // [n_steps]
    float* logits_out;    // nullable [n_steps, V]
    float* qc_trace;      // nullable [n_steps][L][H*hd]: every decoder call's cross-attention queries
    int* n_done;          // decoder calls completed
    int* hit_eos;
    unsigned* bar_count;
    unsigned* status;
    unsigned long long* trace;  // nullable: %globaltimer stamps (start + after each barrier)
    int trace_cap;
    int region_bytes;           // per-warp prefetch region (set by the launcher)
};

// ---------------------------------------------------------------- batched decode step
// x[b] = embed[ids[b]]; with xb also its bf16 planes (xb [B][d], low plane lo_off further),
// and with stats the (mean, M2) of each row over column tiles of tile_n at
// stats[t * stats_ld + b] (the layout TcGemmArgs::lnf reads).
cudaError_t launch_embed_rows(const int* ids, const float* embed, int d, int B, int V, float* x, unsigned* status,
                              cudaStream_t s, __nv_bfloat16* xb = nullptr, size_t lo_off = 0,
                              float2* stats = nullptr, int stats_ld = 0, int tile_n = 0);
// The bf16 outputs below take an optional lo_off: != 0 also writes the low plane of a split
// operand (bf16 of v - bf16(v)) lo_off elements after each value.
cudaError_t launch_ln_bf16(const float* x, int rows, int d, const float* w, __nv_bfloat16* out, cudaStream_t s,
                          float w_offset = 0.f, size_t lo_off = 0);
cudaError_t launch_self_attn_batch(const float* q, const float* kv_new, const PagedKv& kv, const int* pos, int B,
                                   int H, int KVH, int hd, float scale, __nv_bfloat16* out, cudaStream_t s,
                                   size_t lo_off = 0);
// Per-row cross K/V read in place: row b's [layers][2][KVH][cap[b]][hd] at src32[b] (fp32) and
// at src16[b] (the stored copy: fp16, or the fp32 rows again when the cache is fp32); device
// tables, every pointer 16-byte aligned.  Needs a head_dim of 32, 40, 48 or 64.
struct CrossRows {
    const void* const* src32 = nullptr;
    const void* const* src16 = nullptr;
    const int* cap = nullptr;
};
// rows == nullptr: the concatenated layout [layers][2][KVH][m_cap][hd] at cross32 / cross_st,
// row b's frames from frame_off[b]; otherwise rows (cross32, cross_st, frame_off, m_cap unused).
cudaError_t launch_cross_attn_batch(const float* qc, const float* cross32, const void* cross_st, int st_f16,
                                    const int* pos, const int* frame_off, const int* frames, int B, int H, int KVH,
                                    int hd, int m_cap, int layer, int max_frames, float scale, float* part,
                                    __nv_bfloat16* out, int first_step, unsigned* status, cudaStream_t s,
                                    size_t lo_off = 0, const CrossRows* rows = nullptr);
bool cross_rows_supported(int hd);
cudaError_t launch_step_finalize(unsigned long long* amax, int B, int* pos, int* next_ids, int* ids_out, int t_cap,
                                 int* counts, const int* limits, int* done, int* hit_eos, int eos, int forced,
                                 cudaStream_t s);
// colscale (optional, [K]): each row times colscale[k] before rounding (a LayerNorm weight
// folded into the GEMM that consumes it).
cudaError_t launch_f32_to_bf16_rows(const float* src, __nv_bfloat16* dst, int rows, int K, int interleave,
                                    cudaStream_t s, size_t lo_off = 0, const float* colscale = nullptr);
// out[r] = sum over k of row r of a bf16 matrix [rows][K] (plus its low plane lo_off further,
// when lo_off != 0), accumulated in double in a fixed order.
cudaError_t launch_bf16_row_sums(const __nv_bfloat16* w, int rows, int K, size_t lo_off, float* out,
                                 cudaStream_t s);
cudaError_t launch_interleave_f32(const float* src, float* dst, int n2, int half, cudaStream_t s);
size_t cross_batch_part_floats(int B, int H, int hd, int max_frames);
// Per-row cross K/V ([segs][mcap[b]][hd] at src32[b] / src16[b], device pointer arrays) into
// the concatenated layout [segs][m_cap][hd] at frame offset off[b]; src16 entries may be null.
cudaError_t launch_gather_cross(const float* const* src32, const void* const* src16, const int* mcap,
                                const int* frames, const int* off, int B, int segs, int hd, int m_cap, float* dst32,
                                void* dst16, cudaStream_t s);

// Head-clustered batch-1 decode (one 8-CTA cluster per head, packed per-CTA weight streams).
struct ClusterGeom {
    int rq = 0, ro = 0, rcq = 0, gr = 0, rlm = 0;  // rows per CTA: q|k|v, out-proj, cross q, SwiGLU, vocab
    int slot_bytes = 0;                           // weight-stream ring slot
    int skv_keys = 0;                             // cached self keys per CTA (ceil(t_cap / 8))
    size_t cta_floats = 0;                        // packed stream length per CTA
    const float* packed = nullptr;                // [H * 8][cta_floats]
    unsigned long long* part = nullptr;           // tagged exchange words: [2][H][d] partial sums, then
                                                  // [H * 8][2] per-CTA argmax; zeroed before each launch
    size_t part_words = 0;
    float l2_keep = 0.f;                          // > 0: this fraction of the streamed weight and
                                                  // cross K/V lines is loaded L2 evict_last, the rest
                                                  // evict_first (the stream is re-read every token)
    int qbits = 0, lm_qbits = 0, qgroup = 0;      // > 0: the q|k|v, cross q and fc1 rows (qbits) and
                                                  // the LM-head rows (lm_qbits) are streamed as
                                                  // quantized records (2, 4 or 8 bits, groups of qgroup)
    int rs_rows = 0, rs_lm = 0;                   // stored row strides (words) of those rows
};
// Whether the clustered kernel can stream rows of d inputs quantized to `bits` in groups of
// gs: every 16-byte chunk of codes must lie inside one group.
bool cluster_quant_ok(int d, int bits, int gs);
// false when the dims do not fit the clustered kernel (the caller keeps decode_b1)
bool cluster_geom(int d, int H, int KVH, int hd, int I, int V, int L, int t_cap, ClusterGeom* g, int qbits = 0,
                  int lm_qbits = 0, int qgroup = 0);
int cluster_ctas(int H);
// lm_q: quantized LM-head records (when g.lm_qbits), else lm_head's fp32 rows are packed.
cudaError_t pack_cluster_weights(const ClusterGeom& g, const DecodeLayerW* layers_host, int L, const float* lm_head,
                                 const uint32_t* lm_q, const float* final_ln, int d, int H, int hd, int I, int V,
                                 float* packed, cudaStream_t s);
cudaError_t launch_decode_cluster(const DecodeParams& p, const ClusterGeom& g, cudaStream_t stream);

// Word-timestamp alignment rows from the cross queries a decode stored (qc_trace) and the
// cross K it read: raw_out (nullable) and filt_out [n_steps][M] are the head/layer-mean
// softmax rows and their z-scored, median-filtered (width) form; probs [n_steps] the softmax
// probability of ids[s] under logits [n_steps][V].  part: alignment_part_floats scratch.
int alignment_max_median_width();
size_t alignment_part_floats(int n_steps, int L, int M);
cudaError_t launch_alignment_rows(const float* qc_trace, const float* cross32, const void* cross_stored, int st_f16,
                                  int n_steps, int L, int H, int KVH, int hd, int m_cap, int M, float scale,
                                  const float* logits, const int* ids, int V, int width, float* part, float* raw_out,
                                  float* filt_out, float* probs, cudaStream_t s);

// Persistent cooperative decode kernel: runs up to n_steps greedy decoder calls.
cudaError_t launch_decode_b1(const DecodeParams& p, int grid, cudaStream_t stream);
int decode_b1_block_threads();
bool decode_b1_supports_head_dim(int hd);
// Load the code of decode_b1_kernel<hd> / both gemm_f32_kernel instantiations now (under lazy
// module loading the first launch would otherwise do it, reserving device memory then).
cudaError_t preload_decode_b1(int hd);
cudaError_t preload_gemm_f32();
int decode_chunk_keys();
// Scratch sizes (floats) the decode kernel needs for `grid` CTAs.
size_t decode_b1_spart_floats(int H, int hd, int t_cap);
size_t decode_b1_cpart_floats(int H, int hd, int m_cap, int grid);

}  // namespace msb
