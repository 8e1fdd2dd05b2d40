// Batched greedy decode engine: B utterances decoded in lockstep with bf16 tcgen05 GEMMs.
#pragma once

#include <cuda.h>

#include <memory>
#include <vector>

#include "model.hpp"

namespace msb {

struct BatchEngine {
    explicit BatchEngine(Model& model) : m(model) {}
    ~BatchEngine();

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
    Result run(const std::vector<const float*>& audio_dev, const std::vector<int64_t>& n_samples,
               const std::vector<int>& limits, bool forced, bool want_logits);

   private:
    struct LayerB {
        __nv_bfloat16 *wqkv, *wo, *wcq, *wco, *w1i, *w2;
        float* b1i;
        CUtensorMap m_qkv, m_o, m_cq, m_co, m_w1, m_w2;
    };
    Model& m;
    bool weights_ready = false;
    std::vector<DevBuf*> own;
    std::vector<LayerB> layers;
    __nv_bfloat16* lm = nullptr;
    CUtensorMap m_lm;
    int Bc = 0, Tc = 0, Mc = 0, Fc = 0;  // capacities: rows, steps, total frames, frames per row
    DevBuf x, hb, attn, g, q, qc, kvnew, kcache, vcache, part, amax, ids, next_ids, counts, limits_d, done, hit,
        pos, frame_off, frames, cross32, cross16, memory, status;
    CUtensorMap a_hb, a_attn, a_g;

    // Concurrent encoder lanes: each has its own scratch buffers and stream, so independent
    // utterances' (latency-bound) encoders overlap on the GPU.
    struct EncLane {
        DevBuf feat1p, feat2p, x, h, qkv, attn, f, memory, memproj;
        cudaStream_t stream = nullptr;
        cudaEvent_t done = nullptr;
        EncBufs bufs() { return {&feat1p, &feat2p, &x, &h, &qkv, &attn, &f, &memory, &memproj}; }
    };
    std::vector<std::unique_ptr<EncLane>> lanes;
    cudaEvent_t ev_start = nullptr;
    void encode_all(const std::vector<const float*>& audio_dev, const std::vector<int64_t>& n_samples,
                    const std::vector<int>& off);

    template <class T> T* alloc(size_t n);
    void ensure_weights();
    void ensure_ws(int B, int T, int Mtot, int maxM);
    void enqueue_step(int B, int max_frames, bool forced, bool first, float* logits);
    void gemm(const CUtensorMap& a, const CUtensorMap& b, TcGemmArgs& g, int K, int bn);
};

}  // namespace msb
