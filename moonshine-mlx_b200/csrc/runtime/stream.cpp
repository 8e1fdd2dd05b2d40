// Streaming state machine of MoonshineStreaming.swift over device-resident buffers.
//
// Frontend (Embedder.processChunk, MoonshineEncoder.swift:100-151): leftover samples stay
// on the host (< one frame); whole frames go through the fused frame-feature kernel and
// the two causal convs as implicit GEMMs whose 4-row history buffers live on the device.
// encodeNewFrames (MoonshineStreaming.swift:178-214) re-runs the encoder over the
// 16*L-frame left context plus new frames and appends memory rows AND their cross K/V:
// memory rows never change once appended, so their cross K/V is computed once instead of
// on every transcribe call as the reference does (identical values).  decodeMemory
// (:229-276) re-decodes from BOS on every call with the same greedy kernel as generate.
#include "stream.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <unordered_set>

namespace msb {

namespace {

// Grow `b` to `new_bytes`, keeping its first `keep_bytes` (device-to-device copy).
// Growth of a stream's buffers is stream-ordered (allocated from the model's stream pool and
// freed with cudaFreeAsync on the stream that uses them): many streams growing at the same
// chunk neither synchronise the device nor each map new memory from the driver.
void grow_keep(DevBuf& b, size_t keep_bytes, size_t new_bytes, cudaStream_t s, cudaMemPool_t pool) {
    if (new_bytes <= b.bytes) return;
    void* p = nullptr;
    MSB_CUDA(cudaMallocFromPoolAsync(&p, new_bytes, pool, s));
    if (b.p && keep_bytes) MSB_CUDA(cudaMemcpyAsync(p, b.p, keep_bytes, cudaMemcpyDeviceToDevice, s));
    if (b.p) MSB_CUDA(cudaFreeAsync(b.p, s));
    b.p = p;
    b.bytes = new_bytes;
}

}  // namespace

StreamState::StreamState(Model* m) : model(m) {
    // createStream pre-fills frameLen-1 zero samples (MoonshineStreaming.swift:69-71)
    sample_buffer.assign((size_t)std::max(0, m->cfg.frame_len() - 1), 0.f);
}

StreamState::~StreamState() {
    if (stage_done) {
        cudaEventSynchronize(stage_done);
        cudaEventDestroy(stage_done);
    }
    if (stage) cudaFreeHost(stage);
}

void StreamState::start() {  // MoonshineStreaming.swift:74-78
    active = true;
    reset_segment();
    emitted.clear();
}

void StreamState::reset_segment() {  // MoonshineStreaming.swift:217-226
    feat_count = 0;
    enc_valid = 0;
    enc_inc = true;
    encoder_frames_emitted = 0;
    pos_offset = 0;
    memory_len = 0;
    last_hit_eos = false;
}

void StreamState::add_audio(const float* chunk, int64_t n, cudaStream_t s_in) {  // MoonshineStreaming.swift:87-105
    Model& m = *model;
    const Config& c = m.cfg;
    const int fl = c.frame_len(), ed = c.e_hidden;
    cudaStream_t s = s_in ? s_in : m.stream;
    const size_t have = sample_buffer.size() + (size_t)n;
    const int64_t nf64 = (int64_t)have / fl;
    if (nf64 > (1 << 24)) throw MsError(MS_ERR_INVALID_ARG, "audio chunk too long");
    if (nf64 == 0) {  // everything stays in the remainder buffer
        sample_buffer.insert(sample_buffer.end(), chunk, chunk + n);
        return;
    }
    // leftover samples + the chunk, in page-locked memory the upload reads asynchronously
    if (!stage_done) MSB_CUDA(cudaEventCreateWithFlags(&stage_done, cudaEventDisableTiming));
    MSB_CUDA(cudaEventSynchronize(stage_done));  // the previous upload from it is done
    if (have > stage_cap) {
        if (stage) MSB_CUDA(cudaFreeHost(stage));
        stage = nullptr;
        const size_t cap = std::max(have, 2 * stage_cap);
        MSB_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&stage), cap * 4, cudaHostAllocDefault));
        stage_cap = cap;
    }
    std::copy(sample_buffer.begin(), sample_buffer.end(), stage);
    std::copy(chunk, chunk + n, stage + sample_buffer.size());
    const int64_t rem = (int64_t)have - nf64 * fl;
    sample_buffer.assign(stage + nf64 * fl, stage + have);
    (void)rem;
    const int nf = (int)nf64;
    chunk_audio.ensure((size_t)nf * fl * 4);
    MSB_CUDA(cudaMemcpyAsync(chunk_audio.p, stage, (size_t)nf * fl * 4, cudaMemcpyHostToDevice, s));
    MSB_CUDA(cudaEventRecord(stage_done, s));
    const int T2 = (nf - 1) / 2 + 1, T3 = (T2 - 1) / 2 + 1;
    xin1.ensure((size_t)(4 + nf) * ed * 4);
    xin2.ensure((size_t)(4 + T2) * 2 * ed * 4);
    conv1_buf.ensure((size_t)4 * ed * 4);
    conv2_buf.ensure((size_t)4 * 2 * ed * 4);
    float* x1 = xin1.as<float>();
    float* x2 = xin2.as<float>();
    if (have_conv1) MSB_CUDA(cudaMemcpyAsync(x1, conv1_buf.p, (size_t)4 * ed * 4, cudaMemcpyDeviceToDevice, s));
    else MSB_CUDA(cudaMemsetAsync(x1, 0, (size_t)4 * ed * 4, s));
    if (have_conv2) MSB_CUDA(cudaMemcpyAsync(x2, conv2_buf.p, (size_t)4 * 2 * ed * 4, cudaMemcpyDeviceToDevice, s));
    else MSB_CUDA(cudaMemsetAsync(x2, 0, (size_t)4 * 2 * ed * 4, s));
    MSB_CUDA(launch_frame_features(chunk_audio.as<float>(), nf, fl, m.log_k, m.lin_w, ed, x1 + 4 * ed, ed, s));
    GemmEpilogue c1;
    c1.bias = m.conv1_b;
    c1.act = ACT_SILU;
    c1.out = x2 + 4 * 2 * ed;
    c1.ldc = 2 * ed;
    MSB_CUDA(launch_gemm_f32(x1, 2 * ed, m.conv1_w, 5 * ed, T2, 2 * ed, 5 * ed, c1, s));
    // conv1Buffer = last 4 rows of [buffer; x] (MoonshineEncoder.swift:137)
    MSB_CUDA(cudaMemcpyAsync(conv1_buf.p, x1 + (size_t)nf * ed, (size_t)4 * ed * 4, cudaMemcpyDeviceToDevice, s));
    have_conv1 = true;
    if (feat_count + T3 > feat_cap) {
        const int cap = std::max(feat_count + T3, std::max(2 * feat_cap, 256));
        grow_keep(features, (size_t)feat_count * ed * 4, (size_t)cap * ed * 4, s, m.streams_pool());
        feat_cap = cap;
    }
    GemmEpilogue c2;
    c2.bias = m.conv2_b;
    c2.out = features.as<float>() + (size_t)feat_count * ed;
    c2.ldc = ed;
    MSB_CUDA(launch_gemm_f32(x2, 4 * ed, m.conv2_w, 10 * ed, T3, ed, 10 * ed, c2, s));
    MSB_CUDA(cudaMemcpyAsync(conv2_buf.p, x2 + (size_t)T2 * 2 * ed, (size_t)4 * 2 * ed * 4,
                             cudaMemcpyDeviceToDevice, s));
    have_conv2 = true;
    feat_count += T3;
}

namespace {

// One pass of add_audio_batch over streams that each appear once and each have whole frames.
struct FrontJob {
    StreamState* st;
    const float* chunk;
    int64_t n;
    int nf, T2, T3;
    size_t aoff, x1, x2;  // offsets (floats) of the frames in the upload and of the conv inputs in fe_x
};

void frontend_pass(Model& m, const std::vector<FrontJob>& jobs, size_t audio_f, size_t x_f, int nf_max, int rows1,
                   int rows2, cudaStream_t s) {
    const Config& c = m.cfg;
    const int fl = c.frame_len(), ed = c.e_hidden, nb = (int)jobs.size();
    const size_t tb = (audio_f * 4 + 15) & ~(size_t)15;
    size_t off = tb;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 15) & ~(size_t)15;
        return o;
    };
    const size_t o_aoff = take(8 * (size_t)nb), o_ffout = take(8 * (size_t)nb);
    const size_t o_pre_src = take(16 * (size_t)nb), o_pre_dst = take(16 * (size_t)nb);
    const size_t o_post_src = take(16 * (size_t)nb), o_post_dst = take(16 * (size_t)nb);
    // conv1 / conv2 as implicit GEMMs over every stream's rows: A row and output row pointers
    const size_t o_g1a = take(8 * (size_t)rows1), o_g1o = take(8 * (size_t)rows1);
    const size_t o_g2a = take(8 * (size_t)rows2), o_g2o = take(8 * (size_t)rows2);
    const size_t o_nf = take(4 * (size_t)nb), o_cnt = take(8 * (size_t)nb);
    const size_t total = off;

    // conv inputs (grow by half again at least, so a slowly growing batch rarely reallocates)
    if (x_f * 4 > m.fe_x.bytes)
        m.fe_x.ensure_on(std::max(x_f * 4, m.fe_x.bytes + m.fe_x.bytes / 2), s, m.streams_pool());
    // per-stream buffers, allocated and grown stream-ordered before the tables point at them
    for (const FrontJob& j : jobs) {
        StreamState& st = *j.st;
        grow_keep(st.conv1_buf, 0, (size_t)4 * ed * 4, s, m.streams_pool());
        grow_keep(st.conv2_buf, 0, (size_t)4 * 2 * ed * 4, s, m.streams_pool());
        if (st.feat_count + j.T3 > st.feat_cap) {
            const int cap = std::max(st.feat_count + j.T3, std::max(2 * st.feat_cap, 256));
            grow_keep(st.features, (size_t)st.feat_count * ed * 4, (size_t)cap * ed * 4, s, m.streams_pool());
            st.feat_cap = cap;
        }
    }

    char* h = m.fe_tables.host(total);
    float* x = m.fe_x.as<float>();
    auto hp = [&](size_t o) { return reinterpret_cast<void*>(h + o); };
    long long* aoff = static_cast<long long*>(hp(o_aoff));
    float** ffout = static_cast<float**>(hp(o_ffout));
    const float** pre_src = static_cast<const float**>(hp(o_pre_src));
    float** pre_dst = static_cast<float**>(hp(o_pre_dst));
    const float** post_src = static_cast<const float**>(hp(o_post_src));
    float** post_dst = static_cast<float**>(hp(o_post_dst));
    const float** g1a = static_cast<const float**>(hp(o_g1a));
    float** g1o = static_cast<float**>(hp(o_g1o));
    const float** g2a = static_cast<const float**>(hp(o_g2a));
    float** g2o = static_cast<float**>(hp(o_g2o));
    int* nfv = static_cast<int*>(hp(o_nf));
    int* cnt = static_cast<int*>(hp(o_cnt));
    int r1 = 0, r2 = 0;
    for (int z = 0; z < nb; ++z) {
        const FrontJob& j = jobs[z];
        StreamState& st = *j.st;
        // the stream's whole frames: leftover samples, then the head of the chunk
        float* a = reinterpret_cast<float*>(h) + j.aoff;
        const size_t used = (size_t)j.nf * fl, sb = st.sample_buffer.size();
        const size_t from_sb = std::min(sb, used);
        std::copy(st.sample_buffer.begin(), st.sample_buffer.begin() + from_sb, a);
        std::copy(j.chunk, j.chunk + (used - from_sb), a + from_sb);
        float* x1 = x + j.x1;
        float* x2 = x + j.x2;
        aoff[z] = (long long)j.aoff;
        nfv[z] = j.nf;
        ffout[z] = x1 + 4 * ed;
        pre_src[z] = st.have_conv1 ? st.conv1_buf.as<float>() : nullptr;
        pre_dst[z] = x1;
        pre_src[nb + z] = st.have_conv2 ? st.conv2_buf.as<float>() : nullptr;
        pre_dst[nb + z] = x2;
        // conv1Buffer / conv2Buffer = last 4 rows of [buffer; x] (MoonshineEncoder.swift:137)
        post_src[z] = x1 + (size_t)j.nf * ed;
        post_dst[z] = st.conv1_buf.as<float>();
        post_src[nb + z] = x2 + (size_t)j.T2 * 2 * ed;
        post_dst[nb + z] = st.conv2_buf.as<float>();
        cnt[z] = 4 * ed;
        cnt[nb + z] = 4 * 2 * ed;
        // conv1 row t reads x1 rows 2t..2t+4 (stride 2, kernel 5) and lands in x2 row 4 + t;
        // conv2 row t reads x2 rows 2t..2t+4 and lands in feature row feat_count + t
        for (int t = 0; t < j.T2; ++t, ++r1) {
            g1a[r1] = x1 + (size_t)t * 2 * ed;
            g1o[r1] = x2 + (size_t)(4 + t) * 2 * ed;
        }
        float* feat = st.features.as<float>() + (size_t)st.feat_count * ed;
        for (int t = 0; t < j.T3; ++t, ++r2) {
            g2a[r2] = x2 + (size_t)t * 4 * ed;
            g2o[r2] = feat + (size_t)t * ed;
        }
    }
    char* d = m.fe_tables.upload(total, s, m.streams_pool());
    auto dp = [&](size_t o) { return reinterpret_cast<void*>(d + o); };
    MSB_CUDA(launch_copy_rows_batch(static_cast<const float* const*>(dp(o_pre_src)),
                                    static_cast<float* const*>(dp(o_pre_dst)), static_cast<const int*>(dp(o_cnt)),
                                    2 * nb, s));
    MSB_CUDA(launch_frame_features_batch(reinterpret_cast<const float*>(d), static_cast<const long long*>(dp(o_aoff)),
                                         static_cast<const int*>(dp(o_nf)), static_cast<float* const*>(dp(o_ffout)),
                                         nb, nf_max, fl, m.log_k, m.lin_w, ed, ed, s));
    MSB_CUDA(launch_gemm_f32_rows(static_cast<const float* const*>(dp(o_g1a)), static_cast<float* const*>(dp(o_g1o)),
                                  rows1, m.conv1_w, 5 * ed, 2 * ed, 5 * ed, m.conv1_b, ACT_SILU, s));
    MSB_CUDA(launch_gemm_f32_rows(static_cast<const float* const*>(dp(o_g2a)), static_cast<float* const*>(dp(o_g2o)),
                                  rows2, m.conv2_w, 10 * ed, ed, 10 * ed, m.conv2_b, ACT_NONE, s));
    MSB_CUDA(launch_copy_rows_batch(static_cast<const float* const*>(dp(o_post_src)),
                                    static_cast<float* const*>(dp(o_post_dst)), static_cast<const int*>(dp(o_cnt)),
                                    2 * nb, s));
    for (const FrontJob& j : jobs) {
        StreamState& st = *j.st;
        const size_t used = (size_t)j.nf * fl, sb = st.sample_buffer.size();
        std::vector<float> rest;
        rest.reserve(sb + (size_t)j.n - used);
        for (size_t k = used; k < sb; ++k) rest.push_back(st.sample_buffer[k]);
        const size_t c0 = used > sb ? used - sb : 0;
        rest.insert(rest.end(), j.chunk + c0, j.chunk + j.n);
        st.sample_buffer.swap(rest);
        st.have_conv1 = st.have_conv2 = true;
        st.feat_count += j.T3;
    }
}

}  // namespace

void add_audio_batch(Model& m, StreamState* const* ss, int n, const float* const* chunks, const int64_t* ns,
                     cudaStream_t s) {
    const Config& c = m.cfg;
    const int fl = c.frame_len(), ed = c.e_hidden;
    bool dup = false;
    {
        std::unordered_set<const StreamState*> seen;
        for (int i = 0; i < n && !dup; ++i) dup = !seen.insert(ss[i]).second;
    }
    if (dup) {  // a stream's chunks must be taken in order: one call at a time
        for (int i = 0; i < n; ++i) ss[i]->add_audio(chunks[i], ns[i], s);
        return;
    }
    for (int i = 0; i < n; ++i)
        if ((int64_t)(ss[i]->sample_buffer.size() + (size_t)ns[i]) / fl > (1 << 24))
            throw MsError(MS_ERR_INVALID_ARG, "audio chunk too long");
    // streams per pass (the frame-feature grid takes up to 65535 streams in y) and conv rows
    // per pass (the conv GEMM grids take up to 65535 row tiles)
    constexpr int kGroup = 16384, kRows = 1 << 20;
    std::vector<FrontJob> jobs;
    size_t audio_f = 0, x_f = 0;
    int nf_max = 0, rows1 = 0, rows2 = 0;
    auto flush = [&]() {
        if (!jobs.empty()) frontend_pass(m, jobs, audio_f, x_f, nf_max, rows1, rows2, s);
        jobs.clear();
        audio_f = x_f = 0;
        nf_max = rows1 = rows2 = 0;
    };
    for (int i = 0; i < n; ++i) {
        StreamState& st = *ss[i];
        const size_t have = st.sample_buffer.size() + (size_t)ns[i];
        const int nf = (int)((int64_t)have / fl);
        if (nf == 0) {  // everything stays in the remainder buffer
            st.sample_buffer.insert(st.sample_buffer.end(), chunks[i], chunks[i] + ns[i]);
            continue;
        }
        FrontJob j;
        j.st = &st;
        j.chunk = chunks[i];
        j.n = ns[i];
        j.nf = nf;
        j.T2 = (nf - 1) / 2 + 1;
        j.T3 = (j.T2 - 1) / 2 + 1;
        j.aoff = audio_f;
        audio_f += ((size_t)nf * fl + 3) & ~(size_t)3;
        j.x1 = x_f;
        x_f += (size_t)(4 + nf) * ed;
        j.x2 = x_f;
        x_f += (size_t)(4 + j.T2) * 2 * ed;
        nf_max = std::max(nf_max, nf);
        rows1 += j.T2;
        rows2 += j.T3;
        jobs.push_back(j);
        if ((int)jobs.size() == kGroup || rows1 > kRows) flush();
    }
    flush();
}

void StreamState::ensure_memory(int rows, cudaStream_t s) {
    Model& m = *model;
    const Config& c = m.cfg;
    if (rows <= mem_cap) return;
    const int cap = std::max(rows, std::max(2 * mem_cap, 256));
    grow_keep(memory, (size_t)memory_len * c.hidden * 4, (size_t)cap * c.hidden * 4, s, m.streams_pool());
    // the K/V layout [L][2][KVH][cap][hd] depends on the capacity: the rows kept move to the
    // new pitch with one strided copy per buffer (no recomputation)
    const size_t segs = (size_t)c.layers * 2 * c.kv_heads, hd = c.head_dim;
    const size_t n = segs * cap * hd;
    auto regrid = [&](DevBuf& b, size_t esz) {
        void* p = nullptr;
        MSB_CUDA(cudaMallocFromPoolAsync(&p, n * esz, m.streams_pool(), s));
        if (b.p && memory_len > 0)
            MSB_CUDA(cudaMemcpy2DAsync(p, (size_t)cap * hd * esz, b.p, (size_t)mem_cap * hd * esz,
                                       (size_t)memory_len * hd * esz, segs, cudaMemcpyDeviceToDevice, s));
        if (b.p) MSB_CUDA(cudaFreeAsync(b.p, s));
        b.p = p;
        b.bytes = n * esz;
    };
    regrid(cross32, 4);
    regrid(cross16, 2);
    mem_cap = cap;
}

bool StreamState::plan_new_frames(bool is_final, EncPlan* p, cudaStream_t s) {  // MoonshineStreaming.swift:178-214
    const Config& c = model->cfg;
    if (feat_count <= 0) return false;
    const int total = feat_count;
    int look = 0;
    if (c.has_windows)
        for (auto& w : c.windows) look = std::max(look, w.second);
    const int stable = is_final ? total : std::max(0, total - look);
    const int nnew = stable - encoder_frames_emitted;
    if (nnew <= 0) return false;
    if (pos_offset + nnew > c.max_pos)
        throw MsError(MS_ERR_INVALID_ARG, "segment longer than the positional table");
    const int left_ctx = 16 * c.e_layers;
    p->win_start = std::max(0, encoder_frames_emitted - left_ctx);
    p->T = total - p->win_start;
    p->off = encoder_frames_emitted - p->win_start;
    p->nnew = nnew;
    p->stable = stable;
    ensure_memory(memory_len + nnew, s);
    return true;
}

const float* StreamState::window(const EncPlan& p) const {
    return features.as<float>() + (size_t)p.win_start * model->cfg.e_hidden;
}

float* StreamState::memory_row() const { return memory.as<float>() + (size_t)memory_len * model->cfg.hidden; }

void StreamState::commit_new_frames(const EncPlan& p, cudaStream_t s) {
    Model& m = *model;
    m.cross_kv_into(memory_row(), p.nnew, memory_len, cross32.as<float>(), cross16.p, mem_cap, s);
    advance_new_frames(p);
}

std::vector<float*> StreamState::inc_buffers(cudaStream_t s) {
    Model& m = *model;
    const int L = m.cfg.e_layers, ed = m.cfg.e_hidden;
    if (!enc_x) enc_x.reset(new DevBuf[std::max(1, L - 1)]);
    if (feat_count > enc_rows) {
        const int cap = std::max(feat_count, std::max(2 * enc_rows, 256));
        for (int l = 0; l < L - 1; ++l)
            grow_keep(enc_x[l], (size_t)enc_valid * ed * 4, (size_t)cap * ed * 4, s, m.streams_pool());
        enc_rows = cap;
    }
    std::vector<float*> out((size_t)std::max(0, L - 1));
    for (int l = 0; l < L - 1; ++l) out[l] = enc_x[l].as<float>();
    return out;
}

void StreamState::advance_new_frames(const EncPlan& p) {
    pos_offset += p.nnew;
    encoder_frames_emitted = p.stable;
    memory_len += p.nnew;
}

void commit_new_frames_batch(Model& m, StreamState* const* ss, const StreamState::EncPlan* plans, int n,
                             cudaStream_t s) {
    const Config& c = m.cfg;
    int rows = 0;
    for (int i = 0; i < n; ++i) rows += plans[i].nnew;
    if (rows > 0) {
        const size_t o_dst = ((size_t)rows * 8 + 15) & ~(size_t)15;
        const size_t total = o_dst + (size_t)rows * sizeof(KvRowDst);
        char* h = m.kv_tables.host(total);
        const float** a = reinterpret_cast<const float**>(h);
        KvRowDst* dst = reinterpret_cast<KvRowDst*>(h + o_dst);
        int r = 0;
        for (int i = 0; i < n; ++i) {
            StreamState& st = *ss[i];
            const float* mem = st.memory_row();
            for (int j = 0; j < plans[i].nnew; ++j, ++r) {
                a[r] = mem + (size_t)j * c.hidden;
                dst[r] = KvRowDst{st.cross32.as<float>(), st.cross16.p, st.mem_cap, st.memory_len + j};
            }
        }
        char* d = m.kv_tables.upload(total, s, m.streams_pool());
        const int N = c.layers * 2 * c.kv_heads * c.head_dim;
        MSB_CUDA(launch_gemm_f32_kv_rows(reinterpret_cast<const float* const*>(d),
                                         reinterpret_cast<const KvRowDst*>(d + o_dst), rows, m.cross_w, c.hidden, N,
                                         c.hidden, c.kv_heads, c.head_dim, s));
    }
    for (int i = 0; i < n; ++i) ss[i]->advance_new_frames(plans[i]);
}

void StreamState::encode_new_frames(bool is_final, EncLane* lane) {  // MoonshineStreaming.swift:178-214
    Model& m = *model;
    const Config& c = m.cfg;
    const EncBufs eb = lane ? lane->bufs() : m.own_enc_bufs();
    const cudaStream_t s = lane ? lane->stream : m.stream;
    EncPlan p;
    if (!plan_new_frames(is_final, &p, s)) return;
    enc_inc = false;  // the incremental encoder's layer rows do not follow this encode
    const int ed = c.e_hidden;
    eb.x->ensure((size_t)p.T * ed * 4);
    float* x = eb.x->as<float>();
    MSB_CUDA(cudaMemcpyAsync(x, window(p), (size_t)p.T * ed * 4, cudaMemcpyDeviceToDevice, s));
    m.encoder_layers_on(eb, x, p.T, s);
    float* dst = memory_row();
    if (m.proj) {
        eb.memory->ensure((size_t)p.nnew * ed * 4);
        MSB_CUDA(launch_layernorm_rows(x + (size_t)p.off * ed, p.nnew, ed, m.enc_final, 1.0f, 1e-5f, m.pos_emb,
                                       pos_offset, eb.memory->as<float>(), s));
        GemmEpilogue e;
        e.out = dst;
        e.ldc = c.hidden;
        MSB_CUDA(launch_gemm_f32(eb.memory->as<float>(), ed, m.proj, ed, p.nnew, c.hidden, ed, e, s));
    } else {
        MSB_CUDA(launch_layernorm_rows(x + (size_t)p.off * ed, p.nnew, ed, m.enc_final, 1.0f, 1e-5f, m.pos_emb,
                                       pos_offset, dst, s));
    }
    commit_new_frames(p, s);
}

std::pair<std::vector<int32_t>, bool> StreamState::decode_memory(int32_t max_tokens, float temperature,
                                                                   unsigned seed) {
    Model& m = *model;
    const Config& c = m.cfg;
    if (memory_len <= 0) return {{}, false};
    // MoonshineStreaming.swift:234-236
    const double dur = (double)memory_len * 0.020;
    const int64_t limit = (int64_t)std::ceil(dur * c.max_tok_per_s);
    const int64_t max_tok = std::min<int64_t>(max_tokens, limit);
    if (max_tok <= 0) throw MsError(MS_ERR_INVALID_ARG, "token limit must be positive");
    m.ensure_decode(memory_len, (int)max_tok, false, c.vocab);
    Model::DecodeResult r = m.decode(cross32.as<float>(), m.kv_f16 ? cross16.p : cross32.p, mem_cap, memory_len,
                                     (int)max_tok, false, nullptr, false, temperature, seed);
    const int n_ids = r.n_calls - (r.hit_eos ? 1 : 0);
    std::vector<int32_t> ids((size_t)std::max(n_ids, 0));
    if (n_ids > 0) {
        MSB_CUDA(cudaMemcpyAsync(ids.data(), m.ws.ids.p, (size_t)n_ids * 4, cudaMemcpyDeviceToHost, m.stream));
        MSB_CUDA(cudaStreamSynchronize(m.stream));
    }
    return {ids, r.hit_eos};
}

int64_t StreamState::begin(bool is_final, int32_t max_tokens, Result* done_early, EncLane* lane) {
    // MoonshineStreaming.swift:122-131
    ++calls;
    encode_new_frames(is_final, lane);
    if (memory_len <= 0) MSB_CUDA(cudaStreamSynchronize(lane ? lane->stream : model->stream));
    return decode_limit(is_final, max_tokens, done_early);
}

int64_t StreamState::decode_limit(bool is_final, int32_t max_tokens, Result* done_early) {
    if (memory_len <= 0) {
        if (is_final) reset_segment();
        *done_early = Result();
        return 0;
    }
    // MoonshineStreaming.swift:234-236
    const double dur = (double)memory_len * 0.020;
    const int64_t limit = (int64_t)std::ceil(dur * model->cfg.max_tok_per_s);
    const int64_t max_tok = std::min<int64_t>(max_tokens, limit);
    if (max_tok <= 0) throw MsError(MS_ERR_INVALID_ARG, "token limit must be positive");
    return max_tok;
}

StreamState::Result StreamState::finish(std::vector<int32_t> ids, bool hit_eos, bool is_final,
                                        const ms_streaming_config& sc) {
    // MoonshineStreaming.swift:133-168
    Result res;
    res.ids = std::move(ids);
    res.hit_eos = hit_eos;
    last_hit_eos = res.hit_eos;
    if (res.hit_eos && memory_len >= sc.min_segment_frames) {
        emitted.push_back(res.ids);
        reset_segment();
        encode_new_frames(is_final);
        res.emitted = true;
        return res;
    }
    if (is_final || memory_len > sc.max_memory_frames) {
        emitted.push_back(res.ids);
        reset_segment();
        res.emitted = true;
    }
    return res;
}

StreamState::Result StreamState::transcribe(bool is_final, const ms_streaming_config& sc, int32_t max_tokens) {
    Result early;
    const int64_t max_tok = begin(is_final, max_tokens, &early);
    if (max_tok <= 0) return early;
    auto dm = decode_memory(max_tokens, sc.temperature, mix_seed((unsigned)sc.seed, calls - 1));
    return finish(std::move(dm.first), dm.second, is_final, sc);
}

}  // namespace msb
