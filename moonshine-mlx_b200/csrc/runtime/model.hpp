// Host runtime of the Moonshine B200 path: config, weights on the device, device
// workspaces, and the encode / decode orchestration behind the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../../include/moonshine_b200.h"
#include "../kernels/kernels.h"

namespace msb {

struct MsError : std::runtime_error {
    ms_status status;
    MsError(ms_status s, const std::string& m) : std::runtime_error(m), status(s) {}
};

void cuda_check(cudaError_t e, const char* what);
#define MSB_CUDA(x) ::msb::cuda_check((x), #x)

// Parsed config.json, mirroring MoonshineConfig.swift:5-178.
struct Config {
    int hidden = 320, inter = 1280, layers = 6, heads = 8, kv_heads = 8, head_dim = 40;
    int vocab = 32768, max_pos = 4096;
    bool tie = false;
    int enc_hidden_size = 320;  // encoder_hidden_size (memory width before proj)
    // encoder
    int e_hidden = 320, e_inter = 1280, e_layers = 6, e_heads = 8, e_kv_heads = 8, e_head_dim = 40;
    double frame_ms = 5.0;
    int sample_rate = 16000, e_max_pos = 4096;
    bool has_windows = false;
    std::vector<std::pair<int, int>> windows;
    int bos = 1, eos = 2, dec_start = 1, pad = 0;
    double partial_rotary = 0.8, rope_theta = 10000.0, max_tok_per_s = 6.5;
    bool quantized = false;  // config.json "quantization" (MoonshineConfig.swift:147-153)
    int q_group = 64, q_bits = 8;

    int frame_len() const { return (int)(frame_ms * (double)sample_rate / 1000.0); }
    int rotary_ndims() const {
        int nd = (int)((double)head_dim * partial_rotary);
        return nd - nd % 2;
    }
    // window of encoder layer i: left <= 0 means full attention
    std::pair<int, int> window(int i) const {
        if (has_windows && i < (int)windows.size()) return windows[i];
        return {0, 0};
    }
    static Config from_json_file(const std::string& path);
};

// Device buffer that grows on demand.
struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf();
    void ensure(size_t n);
    // ensure, stream-ordered: the old block is freed on s and the new one taken from `pool`
    // on s (neither synchronises the device nor, once the pool holds freed blocks, maps new
    // memory); for buffers used only on s.  The contents are not kept.
    void ensure_on(size_t n, cudaStream_t s, cudaMemPool_t pool);
    template <class T> T* as() const { return reinterpret_cast<T*>(p); }
};

// Launch tables of one call, filled on the host and uploaded on one stream: page-locked
// staging (reused once its last upload has finished) and its device copy.  Kernels that read
// the device copy must run on the stream of the upload, so the next upload waits for them.
struct TableUpload {
    char* stage = nullptr;
    size_t cap = 0;
    cudaEvent_t done = nullptr;
    DevBuf dev;
    TableUpload() = default;
    TableUpload(const TableUpload&) = delete;
    TableUpload& operator=(const TableUpload&) = delete;
    ~TableUpload();
    // Host area of at least `bytes` (waits for the previous upload from it).
    char* host(size_t bytes);
    // Uploads the first `bytes` on s (the device copy grows stream-ordered from `pool`);
    // returns the device address of the area.
    char* upload(size_t bytes, cudaStream_t s, cudaMemPool_t pool);
};

struct EncLayer {
    float *wqkv, *wo, *w1, *b1, *w2, *b2, *ln_in, *ln_post;
};

// Encoder scratch of one utterance (the model's own set lives in Workspace; the batched
// engine keeps extra sets to encode several utterances concurrently).
struct EncBufs {
    DevBuf *feat1p, *feat2p, *x, *h, *qkv, *attn, *f, *memory, *memproj;
};

// A concurrent encoder lane: its own scratch set and CUDA stream.
struct EncLane {
    DevBuf feat1p, feat2p, x, h, qkv, attn, f, memory, memproj;
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    EncBufs bufs() { return {&feat1p, &feat2p, &x, &h, &qkv, &attn, &f, &memory, &memproj}; }
    ~EncLane();
};

// Per-call device workspace for one utterance chunk (batch 1).
struct Workspace {
    DevBuf audio, feat1p, feat2p, x, h, qkv, attn, f, memory, memproj;
    DevBuf cross32, cross16, self_k, self_v;
    DevBuf dx, dq, dqc, dkvnew, dps, dpc, dspart, dpart, dg, amax_v, amax_i, ids, logits, flags;
    DevBuf qtrace, apart, arows, afilt, aprobs;  // word-timestamp alignment
    int m_cap = 0, t_cap = 0;
};

struct StreamState;
struct BatchEngine;

struct Model {
    Config cfg;
    ms_options opts{};
    int device = 0, num_sms = 0;
    bool kv_f16 = true;
    bool enc_bf16 = false;  // batched encodes run on bf16 tensor cores (bf16 / f16 checkpoint or MS_W_BF16)
    cudaStream_t stream = nullptr;
    cudaEvent_t ev[4] = {};
    std::mutex mu;

    // weights (device, fp32)
    std::vector<DevBuf*> owned;
    float *lin_w = nullptr, *log_k = nullptr, *conv1_w = nullptr, *conv1_b = nullptr,
          *conv2_w = nullptr, *conv2_b = nullptr, *enc_final = nullptr;
    std::vector<EncLayer> enc;
    float *embed = nullptr, *pos_emb = nullptr, *proj = nullptr, *lm_head = nullptr,
          *dec_norm = nullptr, *cross_w = nullptr;
    std::vector<DecodeLayerW> dec;
    DecodeLayerW* dec_dev = nullptr;
    DevBuf dec_layers_buf, rope_cos, rope_sin;
    int rope_cap = 0;

    Workspace ws;
    // head-clustered batch-1 decode: packed per-CTA weight streams, built on first use
    bool cl_tried = false, cl_ok = false;
    ClusterGeom cl_geom;
    DevBuf cl_packed, cl_part;
    // quantized checkpoints: bits of the quantized row records the clustered kernel streams
    // for q|k|v, cross q and fc1 (DecodeLayerW::*_q) and for the LM head (lm_q); 0 = fp32 rows
    int cl_qbits = 0, cl_lm_qbits = 0;
    const uint32_t* lm_q = nullptr;
    bool prepare_cluster_decode();
    std::unique_ptr<BatchEngine> batch;  // batched bf16 tensor-core decode, built on first use
    bool trace_enabled = false;
    DevBuf trace_buf;
    std::vector<unsigned long long> last_trace;

    ~Model();
    float* upload(const std::vector<float>& v);
    const uint32_t* upload_words(const std::vector<uint32_t>& v);
    void ensure_rope(int positions);

    // --- orchestration (all on `stream`)
    // Frontend + encoder + prepareMemory for one chunk already on the device.
    // Returns the number of memory frames; memory rows land in ws.memory (or memproj).
    int encode_device(const float* audio_dev, int64_t n_samples, int pos_offset);
    const float* memory_ptr() const;
    // Encoder over already computed features [T, e_hidden] (streaming windows).
    void encoder_layers(float* x, int T);
    // The same on explicit scratch buffers and stream (concurrent encodes).
    EncBufs own_enc_bufs();
    int encode_into(const EncBufs& b, const float* audio_dev, int64_t n_samples, int pos_offset, cudaStream_t s);
    const float* memory_of(const EncBufs& b) const;
    void encoder_layers_on(const EncBufs& b, float* x, int T, cudaStream_t s);
    // Grow `b` once for utterances of up to max_samples (no reallocation while encoding).
    void reserve_encoder(const EncBufs& b, int64_t max_samples);
    // Cross K/V of `frames` memory rows into the decode cache at row offset `row0`.
    void cross_kv(const float* memory, int frames, int row0);
    // Decode scratch for `m_frames` memory rows and `t_cap` decoder calls.
    void ensure_decode(int m_frames, int t_cap, bool want_logits, int V);
    void ensure_cross_ws(int m_cap);
    struct DecodeResult {
        int n_calls = 0;
        bool hit_eos = false;
        int kernel = MS_DECODE_GRID;  // which batch-1 kernel ran
    };
    // Greedy (temperature 0) or sampled decode against cross K/V laid out
    // [L][2][KVH][m_cap][hd] (fp32 copy for the first decoder call, stored copy afterwards).
    DecodeResult decode(const float* cross32, const void* cross_stored, int m_cap, int M, int n_steps,
                        bool forced, const int* teacher_dev, bool logits, float temperature = 0.f,
                        unsigned seed = 0, float* qc_trace = nullptr);
    // Cross K/V of `frames` memory rows into explicit buffers at row offset `row0`.
    void cross_kv_into(const float* memory, int frames, int row0, float* out32, void* out16, int m_cap,
                       cudaStream_t s = nullptr);
    // Encoder lanes 0..k-1 (created on first use); `fork` makes them wait for the work
    // queued so far on the model stream, `join` makes the model stream wait for them.
    std::vector<std::unique_ptr<EncLane>> enc_lanes;
    cudaEvent_t lanes_fork = nullptr;
    EncLane& enc_lane(int k);
    void fork_lanes(int k);
    void join_lanes(int k);
    // Memory pool of the streams' growing buffers (stream-ordered allocations).  Freed blocks
    // stay in the pool (no release threshold), so growth reuses memory instead of mapping
    // new memory from the driver every time many streams grow at once.
    cudaMemPool_t stream_pool = nullptr;
    cudaMemPool_t streams_pool();
    // Batched streaming frontend (addAudio of many streams in one pass): the upload of the
    // chunks' frames and launch tables, and the conv inputs of all the streams; and the
    // tables of the streams' batched cross K/V of new memory rows.
    TableUpload fe_tables, kv_tables;
    DevBuf fe_x;
};

// Throws the MsError that a decode kernel's device status word stands for (no-op for DEV_OK).
void throw_device_status(unsigned code, const char* what);

// Allocation-free decode (ms_decode_memory_static): looks up the device address of the
// static scratch array on `device` (which must be current) and loads the kernels that path
// launches, so that the calls themselves load and reserve nothing.  Called by model load.
void noalloc_prepare(int device, int head_dim);

ms_status to_status(const std::exception& e);
// Sets the thread-local message returned by ms_last_error().
void set_last_error(const std::string& m);

}  // namespace msb
