// Streaming transcription state (StreamingState, Sources/MoonshineMLX/MoonshineStreaming.swift:8-43)
// with its frontend conv buffers, features, memory and cross K/V resident on the device.
#pragma once

#include <memory>
#include <vector>

#include "model.hpp"

namespace msb {

// Seed of a sampled decode: the caller's seed mixed with a call counter.
inline unsigned mix_seed(unsigned seed, uint32_t call) { return seed ^ (call * 0x9E3779B9u); }

struct StreamState {
    Model* model = nullptr;
    // frontend (persists across segments)
    std::vector<float> sample_buffer;   // leftover samples (< frame_len), host side
    bool have_conv1 = false, have_conv2 = false;
    DevBuf conv1_buf, conv2_buf;         // last 4 rows of the conv inputs
    DevBuf xin1, xin2, chunk_audio;      // per-chunk scratch
    // page-locked staging of a chunk's frames, so its upload does not wait for the stream;
    // stage_done marks when the last upload from it has finished
    float* stage = nullptr;
    size_t stage_cap = 0;
    cudaEvent_t stage_done = nullptr;
    // accumulated encoder-input features [count, e_hidden]
    DevBuf features;
    int feat_count = 0, feat_cap = 0;
    int encoder_frames_emitted = 0;
    int pos_offset = 0;
    // memory [memory_len, hidden] and its cross K/V [L][2][KVH][mem_cap][hd]
    DevBuf memory, cross32, cross16;
    int memory_len = 0, mem_cap = 0;
    bool cross_f16 = false;
    // incremental encoder (batched transcribe): every encoder layer's output rows of the
    // segment so far ([e_layers - 1] buffers of enc_rows rows), valid up to the feature count
    // of the last incremental encode (enc_valid; rows past its final ones are recomputed);
    // enc_inc false once another encode path has advanced the segment (until its reset)
    std::unique_ptr<DevBuf[]> enc_x;
    int enc_rows = 0, enc_valid = 0;
    bool enc_inc = true;
    std::vector<std::vector<int32_t>> emitted;
    bool last_hit_eos = false;
    bool active = false;
    uint32_t calls = 0;  // transcribe calls so far (separates the draws of successive calls)

    explicit StreamState(Model* m);
    ~StreamState();
    StreamState(const StreamState&) = delete;
    StreamState& operator=(const StreamState&) = delete;
    void start();
    void stop() { active = false; }
    // addAudio; `s` (nullable: the model's stream) is the CUDA stream the frontend runs on
    void add_audio(const float* chunk, int64_t n, cudaStream_t s = nullptr);
    struct Result {
        std::vector<int32_t> ids;
        bool hit_eos = false;
        bool emitted = false;
    };
    Result transcribe(bool is_final, const ms_streaming_config& sc, int32_t max_tokens);
    // transcribe in two halves around an external decode of the segment's memory:
    // begin() encodes the new frames and returns the decode limit (0: nothing to decode,
    // the call is already complete); finish() applies the segment rules to the ids.
    // `lane` (nullable) runs the encoder on that lane's scratch and stream.
    int64_t begin(bool is_final, int32_t max_tokens, Result* done_early, EncLane* lane = nullptr);

    // begin() split for encoding many streams' new frames in one batched pass:
    // note_call(); plan_new_frames() (false: nothing new to encode); the caller encodes the
    // window and writes the new memory rows at memory_row(); commit_new_frames(); then
    // decode_limit() as begin() would return it.
    struct EncPlan {
        int win_start = 0, T = 0, off = 0, nnew = 0, stable = 0;
    };
    void note_call() { ++calls; }
    bool plan_new_frames(bool is_final, EncPlan* p, cudaStream_t s);
    const float* window(const EncPlan& p) const;
    float* memory_row() const;
    void commit_new_frames(const EncPlan& p, cudaStream_t s);
    // commit_new_frames without the cross K/V (computed by the caller, e.g. for many streams
    // at once by commit_new_frames_batch)
    void advance_new_frames(const EncPlan& p);
    // The incremental encoder's layer-output buffers, grown (stream-ordered on s, keeping the
    // valid rows) to hold feat_count rows; one pointer per layer but the last.
    std::vector<float*> inc_buffers(cudaStream_t s);
    int64_t decode_limit(bool is_final, int32_t max_tokens, Result* done_early);
    Result finish(std::vector<int32_t> ids, bool hit_eos, bool is_final, const ms_streaming_config& sc);

   private:
    void reset_segment();
    void encode_new_frames(bool is_final, EncLane* lane = nullptr);
    void ensure_memory(int rows, cudaStream_t s);
    std::pair<std::vector<int32_t>, bool> decode_memory(int32_t max_tokens, float temperature, unsigned seed);
};

// addAudio of n streams of model m in one pass on stream s: chunks[i] (ns[i] samples) goes to
// ss[i], with the same results as n calls of add_audio in order (a stream that appears more
// than once takes its chunks one after the other).  One upload of all the streams' whole
// frames and launch tables, then five launches for the lot: the conv histories, the frame
// features, conv1, the new histories, conv2.
void add_audio_batch(Model& m, StreamState* const* ss, int n, const float* const* chunks, const int64_t* ns,
                     cudaStream_t s);

// commit_new_frames of n streams (plans[i] for ss[i], new memory rows already written at
// their memory_row()) with one gathered-rows cross K/V launch for all their new rows, on s.
void commit_new_frames_batch(Model& m, StreamState* const* ss, const StreamState::EncPlan* plans, int n,
                             cudaStream_t s);

}  // namespace msb
