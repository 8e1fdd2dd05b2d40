// Batched greedy decode engine: B utterances decoded in lockstep with bf16 tcgen05 GEMMs.
#pragma once

#include <cuda.h>

#include <memory>
#include <vector>

#include "model.hpp"

namespace msb {

struct BatchEngine {
    // fp32 checkpoints (not forced to bf16) take split operands in every GEMM
    explicit BatchEngine(Model& model) : m(model), split(!model.enc_bf16), esplit(!model.enc_bf16) {}
    // growth of the engine's scratch, stream-ordered on the model stream from the model's pool
    // (a cudaFree / cudaMalloc pair in the middle of serving stalled for up to ~0.8 s)
    void grow(DevBuf& b, size_t n) { b.ensure_on(n, m.stream, m.streams_pool()); }
    ~BatchEngine();

    static constexpr int kKvPage = 16;  // positions per self-attention K/V page
    int64_t pages_used = 0;             // pages the last call assigned
    int64_t pages_capacity = 0;         // pages the pool holds

    struct Result {
        std::vector<int32_t> ids;      // [B][t_cap]
        std::vector<int32_t> counts;   // [B]
        std::vector<int32_t> hit_eos;  // [B]
        std::vector<float> logits;     // [steps][B][V] when requested
        int t_cap = 0, steps = 0;
        double encode_ms = 0, decode_ms = 0;
    };
    // Encode each utterance (one chunk each), project all cross K/V at once, then run the
    // step loop.  limits[b] decoder calls at most per utterance (forced: exactly).
    // temperature > 0 samples each row's tokens (Gumbel-max keys of (seed, step, row, column)).
    Result run(const std::vector<const float*>& audio_dev, const std::vector<int64_t>& n_samples,
               const std::vector<int>& limits, bool forced, bool want_logits, float temperature = 0.f,
               unsigned seed = 0);

    // Decode rows whose cross K/V already exist (streaming segments): row b's layout is
    // [L][2][KVH][m_cap][hd] with `frames` valid rows, fp32 plus the fp16 copy.
    struct CrossSrc {
        const float* c32;
        const void* c16;
        int m_cap, frames;
    };
    Result run_cross(const std::vector<CrossSrc>& src, const std::vector<int>& limits, bool forced,
                     float temperature = 0.f, unsigned seed = 0);

    // One utterance through the tensor-core encoder (split operands for fp32 checkpoints):
    // memory rows and cross K/V ([L][2][KVH][*m_cap][hd], fp32 and, with an fp16 KV cache,
    // the fp16 copy) in this engine's buffers, for the batch-1 decode.  Returns the memory
    // frames, or -1 when the dims do not fit the tensor-core encoder (the caller encodes on
    // CUDA cores).
    int encode_one(const float* audio_dev, int64_t n_samples, const float** cross32_out, const void** cross16_out,
                   int* m_cap);

    // Incremental encoders of many streams in one pass (transcribe_batch): every stream's
    // window of features goes through the encoder layers as one segment of the longest
    // window's rows; the final norm + positions of its new rows land at its `dst`.  false
    // when the dims do not fit the tensor-core encoder (the caller encodes stream by stream).
    struct StreamWindow {
        const float* feat;  // window rows [T, e_hidden]
        int T, off, nnew, pos;
        float* dst;         // the stream's memory at its current length
    };
    bool encode_windows(const std::vector<StreamWindow>& w);
    // The same result for the new rows with each layer run only over the rows whose value can
    // have changed since the stream's previous incremental encode, plus their left attention
    // context: a stream keeps every layer's output rows (`layer_out`, one buffer per layer but
    // the last).  A layer-l output row r depends on features up to r + (right contexts of
    // layers 0..l), so rows below prev - that sum were final at the previous encode (prev =
    // the feature count then) and are kept; from there on they are recomputed with the band
    // clipped at the current feature count, exactly as the reference's window does.  The
    // window's left edge never reaches a committed row's receptive field (16 frames per
    // layer of left context), so the committed rows are the window's.
    struct StreamIncWindow {
        const float* feat;                // the segment's features [total, e_hidden]
        std::vector<float*> layer_out;    // [e_layers - 1] buffers of >= total rows
        int total, prev;                  // feature count now / at the previous incremental encode
        int emitted, nnew, pos;           // new memory rows: frames emitted .. emitted + nnew
        float* dst;                       // the stream's memory at its current length
    };
    bool encode_windows_inc(const std::vector<StreamIncWindow>& w);
    bool tc_encoder_fits() const;  // the dims the tensor-core encoder supports

   private:
    struct LayerB {
        __nv_bfloat16 *wqkv, *wo, *wcq, *wco, *w1i, *w2;
        float* b1i;
        float *cs_qkv, *cs_cq, *cs_w1;  // row sums of the LayerNorm-folded weights
        CUtensorMap m_qkv, m_o, m_cq, m_co, m_w1, m_w2;
        CUtensorMap m_qkv_lo, m_o_lo, m_cq_lo, m_co_lo, m_w1_lo, m_w2_lo;  // low planes (split)
    };
    Model& m;
    bool split;  // fp32 checkpoint: split bf16 operands (fp32-level products)
    bool weights_ready = false;
    std::vector<DevBuf*> own;
    std::vector<LayerB> layers;
    __nv_bfloat16* lm = nullptr;
    float* cs_lm = nullptr;
    CUtensorMap m_lm, m_lm_lo;
    int Bc = 0, Tc = 0, Mc = 0, Fc = 0;  // capacities: rows, steps, total frames, frames per row
    DevBuf x, hb, attn, g, q, qc, kvnew, part, amax, ids, next_ids, counts, limits_d, done, hit,
        pos, frame_off, frames, cross32, cross16, memory, status;
    // LayerNorms folded into the GEMMs that consume them: hb holds the bf16 planes of the
    // residual x, and lnst the (mean, M2) of each row over column tiles of kStatTile,
    // written by whichever kernel last updated x ([tile][Bc])
    DevBuf lnst;
    // paged self-attention K/V: page pool and per-row page table of the current call
    DevBuf kvpool, ptable;
    int table_stride = 0;
    void assign_pages(int B, int T, const std::vector<int>& limits);
    CUtensorMap a_hb, a_attn, a_g, a_hb_lo, a_attn_lo, a_g_lo;

    // Utterances are encoded concurrently on the model's encoder lanes.
    void encode_all(const std::vector<const float*>& audio_dev, const std::vector<int64_t>& n_samples,
                    const std::vector<int>& off);
    // All utterances in one pass of bf16 tcgen05 GEMMs (model.enc_bf16): each utterance owns a
    // fixed number of rows (its padded length), so the causal convs are 5-tap GEMMs over the
    // whole batch and every encoder projection is one GEMM; also the cross K/V of all memory
    // rows.  false when the dims do not fit (the caller keeps the per-utterance path).
    bool encode_tc(const std::vector<const float*>& audio_dev, const std::vector<int64_t>& n_samples,
                   const std::vector<int>& off, const std::vector<int>& fr);
    void encoder_layers_tc(size_t rows3, int R3, const int* seg_len, int l0 = 0, int l1 = -1);
    TableUpload inc_tables;  // launch tables of encode_windows_inc
    size_t erows_cap = 0;
    size_t enc_rows_capacity(size_t rows3);
    DevBuf wtab;  // device tables of encode_windows
    struct EncLayerB {
        __nv_bfloat16 *wqkv, *wo, *w1, *w2;
        CUtensorMap m_qkv, m_o, m_w1, m_w2;
        CUtensorMap m_qkv_lo, m_o_lo, m_w1_lo, m_w2_lo;
    };
    bool enc_weights_ready = false;
    bool esplit;  // fp32 checkpoint: the encoder GEMMs take split operands
    std::vector<EncLayerB> elayers;
    __nv_bfloat16 *elin = nullptr, *econv1 = nullptr, *econv2 = nullptr, *ecross = nullptr;
    CUtensorMap m_lin, m_conv1, m_conv2, m_ecross, m_lin_lo, m_conv1_lo, m_conv2_lo, m_ecross_lo;
    DevBuf enorm, epad1, epad2, ex, eh, eqkv, eattn, ef, emem16, eseg, eaud;
    void ensure_enc_weights();

    template <class T> T* alloc(size_t n);
    void ensure_weights();
    Result decode_prepared(int B, int T, int maxM, const std::vector<int>& off, const std::vector<int>& fr,
                           const std::vector<int>& limits, bool forced, bool want_logits);
    DevBuf xsrc;  // device pointer tables of run_cross
    // run_cross: the cross attention reads every stream's own cross K/V through these tables
    // (no copy into cross32 / cross16) when the head size has the streamed kernel
    CrossRows xrows;
    bool xrows_on = false;
    void ensure_ws(int B, int T, int Mtot, int maxM);
    void enqueue_step(int B, int max_frames, bool forced, bool first, float* logits);
    // positions the steps being enqueued can reach (0: the call's limit); the steps of a call
    // are captured in up to three graphs, for positions below 32, below 64 and the rest, so
    // that early steps run self attention in shorter rounds (less shared memory per CTA)
    int sa_reach = 0;
    float inv_temp = 0.f;  // sampling state of the current run
    unsigned seed = 0;
    void gemm(const CUtensorMap& a, const CUtensorMap& b, TcGemmArgs& g, int K, int bn,
              const CUtensorMap* a_lo = nullptr, const CUtensorMap* b_lo = nullptr);
};

}  // namespace msb
