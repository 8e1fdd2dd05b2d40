// extern "C" boundary: argument checks, status codes and the thread-local error message
// around the C++ runtime.
#include <cmath>
#include <cstring>
#include <limits>
#include <string>

#include "../../include/moonshine_b200.h"
#include "runtime/alignment.hpp"
#include "runtime/model.hpp"
#include "runtime/batch.hpp"
#include "runtime/stream.hpp"

namespace msb {
Model* load_model(const std::string& dir, const ms_options& o);

int64_t& launch_counter() {
    static thread_local int64_t n = 0;
    return n;
}

bool& pdl_launches() {
    static thread_local bool on = false;
    return on;
}

namespace {
thread_local std::string g_err;

ms_status fail(ms_status s, const std::string& m) {
    g_err = m;
    return s;
}
}  // namespace

void set_last_error(const std::string& m) { g_err = m; }

namespace {

template <class F>
ms_status guarded(F&& f) {
    try {
        g_err.clear();
        return f();
    } catch (const MsError& e) {
        return fail(e.status, e.what());
    } catch (const std::bad_alloc&) {
        return fail(MS_ERR_OOM, "host allocation failed");
    } catch (const std::exception& e) {
        return fail(MS_ERR_INVALID_ARG, e.what());
    }
}

struct GenOut {
    int32_t n_ids = 0;
    int32_t logit_rows = 0;
};

}  // namespace

// One offline chunk: upload, encode, cross K/V, decode; appends ids (and logits rows).
static void generate_chunk(Model& m, const float* audio, int64_t len, const ms_gen_params& gp,
                           int32_t max_tokens, int32_t* ids_out, int32_t cap, float* logits_out,
                           GenOut& out, ms_gen_stats& st, const int32_t* teacher, int32_t n_teacher,
                           bool device_io, unsigned chunk_index) {
    const Config& c = m.cfg;
    MSB_CUDA(cudaEventRecord(m.ev[0], m.stream));
    const float* audio_dev = audio;
    if (!device_io) {
        m.ws.audio.ensure((size_t)std::max<int64_t>(len, 1) * 4);
        MSB_CUDA(cudaMemcpyAsync(m.ws.audio.p, audio, (size_t)len * 4, cudaMemcpyHostToDevice, m.stream));
        audio_dev = m.ws.audio.as<float>();
    }
    // fp32 checkpoints under MS_W_AUTO encode on split-operand tensor-core GEMMs (the
    // batched engine's encoder, one utterance), anything else on the CUDA-core encoder
    const float* cross32 = nullptr;
    const void* cross_st = nullptr;
    int m_cap = 0;
    int M = -1;
    if (!m.enc_bf16 && m.opts.weight_dtype == MS_W_AUTO && len >= c.frame_len()) {
        if (!m.batch) m.batch.reset(new BatchEngine(m));
        M = m.batch->encode_one(audio_dev, len, &cross32, &cross_st, &m_cap);
    }
    const bool tc_encoded = M > 0;
    if (!tc_encoded) M = m.encode_device(audio_dev, len, 0);
    st.memory_frames = M;
    if (M == 0) return;  // fewer samples than one frame: nothing to decode
    const double dur = (double)len / (double)c.sample_rate;
    const int64_t limit64 = std::min<int64_t>(max_tokens, (int64_t)std::ceil(dur * c.max_tok_per_s));
    const bool forced = gp.forced_len != 0;  // < 0: this chunk's own limit, EOS ignored
    const int n_steps = gp.forced_len > 0 ? gp.forced_len : (int)limit64;
    if (n_steps <= 0) throw MsError(MS_ERR_INVALID_ARG, "token limit must be positive");
    const int* teacher_dev = nullptr;
    if (teacher) {
        if (gp.forced_len <= 0 || n_teacher < n_steps)
            throw MsError(MS_ERR_INVALID_ARG, "teacher_ids need forced_len <= n_teacher");
        m.ws.f.ensure((size_t)n_steps * 4);  // reuse: teacher ids after encode is done
    }
    const bool want_logits = logits_out != nullptr;
    m.ensure_decode(M, n_steps, want_logits, c.vocab);
    if (!tc_encoded) {
        m.cross_kv(m.memory_ptr(), M, 0);
        cross32 = m.ws.cross32.as<float>();
        cross_st = m.kv_f16 ? m.ws.cross16.p : m.ws.cross32.p;
        m_cap = m.ws.m_cap;
    }
    if (teacher) {
        MSB_CUDA(cudaMemcpyAsync(m.ws.f.p, teacher, (size_t)n_steps * 4, cudaMemcpyHostToDevice, m.stream));
        teacher_dev = m.ws.f.as<int>();
    }
    MSB_CUDA(cudaEventRecord(m.ev[1], m.stream));
    const unsigned seed = (unsigned)gp.seed ^ (chunk_index * 0x9E3779B9u);  // chunks draw independently
    Model::DecodeResult r = m.decode(cross32, cross_st, m_cap, M, n_steps, forced, teacher_dev, want_logits,
                                     gp.temperature, seed);
    MSB_CUDA(cudaEventRecord(m.ev[2], m.stream));
    const int n_ids = r.n_calls - (r.hit_eos ? 1 : 0);
    const int fit = std::max(0, std::min(n_ids, cap - out.n_ids));
    if (fit > 0)
        MSB_CUDA(cudaMemcpyAsync(ids_out + out.n_ids, m.ws.ids.p, (size_t)fit * 4,
                                 device_io ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, m.stream));
    if (want_logits) {
        const int rows = std::max(0, std::min(r.n_calls, cap - out.logit_rows));
        if (rows > 0)
            MSB_CUDA(cudaMemcpyAsync(logits_out + (size_t)out.logit_rows * c.vocab, m.ws.logits.p,
                                     (size_t)rows * c.vocab * 4, cudaMemcpyDeviceToHost, m.stream));
        out.logit_rows += rows;
    }
    MSB_CUDA(cudaEventRecord(m.ev[3], m.stream));
    MSB_CUDA(cudaStreamSynchronize(m.stream));
    float t_enc = 0, t_dec = 0;
    MSB_CUDA(cudaEventElapsedTime(&t_enc, m.ev[0], m.ev[1]));
    MSB_CUDA(cudaEventElapsedTime(&t_dec, m.ev[1], m.ev[2]));
    st.encode_ms += t_enc;
    st.decode_ms += t_dec;
    st.hit_eos = r.hit_eos ? 1 : 0;
    st.decode_kernel = r.kernel;
    out.n_ids += n_ids;
}

}  // namespace msb

using namespace msb;

extern "C" {

void ms_options_default(ms_options* o) {
    if (!o) return;
    std::memset(o, 0, sizeof(*o));
    o->device = 0;
    o->kv_dtype = MS_KV_F16;
    o->weight_dtype = MS_W_AUTO;
    o->max_batch = 64;
}

void ms_gen_params_default(ms_gen_params* p) {
    if (!p) return;
    std::memset(p, 0, sizeof(*p));
    p->chunk_duration = 30.0;
}

void ms_streaming_config_default(ms_streaming_config* c) {
    if (!c) return;
    c->max_memory_frames = 100000;
    c->min_segment_frames = 250;
    c->batch_decode = 0;
    c->temperature = 0.f;
    c->seed = 0;
}

const char* ms_last_error(void) { return g_err.c_str(); }
int32_t ms_model_decode_weight_bits(const ms_model* model, int32_t* lm_bits) {
    const Model* m = reinterpret_cast<const Model*>(model);
    if (lm_bits) *lm_bits = m ? m->cl_lm_qbits : 0;
    return m ? m->cl_qbits : 0;
}

int64_t ms_kernel_launches(void) { return launch_counter(); }
void ms_reset_kernel_launches(void) { launch_counter() = 0; }
const char* ms_version(void) { return "moonshine-b200 0.1 (sm_100a)"; }

size_t ms_struct_size(const char* name) {
    if (!name) return 0;
    const std::string n(name);
    if (n == "ms_options") return sizeof(ms_options);
    if (n == "ms_model_config") return sizeof(ms_model_config);
    if (n == "ms_gen_params") return sizeof(ms_gen_params);
    if (n == "ms_gen_stats") return sizeof(ms_gen_stats);
    if (n == "ms_alignment") return sizeof(ms_alignment);
    if (n == "ms_streaming_config") return sizeof(ms_streaming_config);
    return 0;
}

ms_status ms_enable_decode_trace(ms_model* model, int32_t enabled) {
    if (!model) return fail(MS_ERR_INVALID_ARG, "null model");
    Model* m = reinterpret_cast<Model*>(model);
    std::lock_guard<std::mutex> g(m->mu);
    m->trace_enabled = enabled != 0;
    return MS_OK;
}

ms_status ms_decode_trace(ms_model* model, uint64_t* stamps_out, int32_t cap, int32_t* n_out) {
    if (!model || !n_out || cap < 0 || (cap > 0 && !stamps_out)) return fail(MS_ERR_INVALID_ARG, "bad argument");
    Model* m = reinterpret_cast<Model*>(model);
    std::lock_guard<std::mutex> g(m->mu);
    const int32_t n = (int32_t)m->last_trace.size();
    *n_out = n;
    for (int32_t i = 0; i < n && i < cap; ++i) stamps_out[i] = m->last_trace[i];
    if (n > cap) return fail(MS_ERR_CAPACITY, "stamps buffer too small");
    return MS_OK;
}

ms_status ms_model_load(const char* dir, const ms_options* opts, ms_model** out) {
    return guarded([&]() -> ms_status {
        if (!dir || !out) return fail(MS_ERR_INVALID_ARG, "dir and out must be non-null");
        *out = nullptr;
        ms_options o;
        ms_options_default(&o);
        if (opts) o = *opts;
        if (o.max_batch <= 0) o.max_batch = 64;
        Model* m = load_model(dir, o);
        *out = reinterpret_cast<ms_model*>(m);
        return MS_OK;
    });
}

void ms_model_free(ms_model* model) {
    try {
        delete reinterpret_cast<Model*>(model);
    } catch (...) {
    }
}

ms_status ms_model_enable_fp16_kv_cache(ms_model* model, int32_t enabled) {
    if (!model) return fail(MS_ERR_INVALID_ARG, "null model");
    Model* m = reinterpret_cast<Model*>(model);
    std::lock_guard<std::mutex> g(m->mu);
    m->kv_f16 = enabled != 0;
    return MS_OK;
}

int32_t ms_model_sample_rate(const ms_model* model) {
    if (!model) return 0;
    return reinterpret_cast<const Model*>(model)->cfg.sample_rate;
}

ms_status ms_model_get_config(const ms_model* model, ms_model_config* out) {
    if (!model || !out) return fail(MS_ERR_INVALID_ARG, "null argument");
    const Config& c = reinterpret_cast<const Model*>(model)->cfg;
    std::memset(out, 0, sizeof(*out));
    out->hidden_size = c.hidden;
    out->intermediate_size = c.inter;
    out->num_hidden_layers = c.layers;
    out->num_attention_heads = c.heads;
    out->num_key_value_heads = c.kv_heads;
    out->head_dim = c.head_dim;
    out->vocab_size = c.vocab;
    out->max_position_embeddings = c.max_pos;
    out->tie_word_embeddings = c.tie;
    out->encoder_hidden_size = c.enc_hidden_size;
    out->enc_hidden_size = c.e_hidden;
    out->enc_intermediate_size = c.e_inter;
    out->enc_num_hidden_layers = c.e_layers;
    out->enc_num_attention_heads = c.e_heads;
    out->enc_num_key_value_heads = c.e_kv_heads;
    out->enc_head_dim = c.e_head_dim;
    out->enc_frame_len = c.frame_len();
    out->enc_sample_rate = c.sample_rate;
    out->enc_max_position_embeddings = c.e_max_pos;
    out->bos_token_id = c.bos;
    out->eos_token_id = c.eos;
    out->decoder_start_token_id = c.dec_start;
    out->pad_token_id = c.pad;
    out->rotary_ndims = c.rotary_ndims();
    out->rope_theta = (float)c.rope_theta;
    out->max_tokens_per_second = c.max_tok_per_s;
    out->num_sliding_windows = c.has_windows ? (int32_t)std::min<size_t>(c.windows.size(), 64) : 0;
    for (int i = 0; i < out->num_sliding_windows; ++i) {
        out->sliding_windows[i][0] = c.windows[i].first;
        out->sliding_windows[i][1] = c.windows[i].second;
    }
    return MS_OK;
}

static ms_status generate_impl(ms_model* model, const float* audio, int64_t n_samples,
                               const ms_gen_params* params, int32_t* ids_out, int32_t cap, int32_t* n_out,
                               float* logits_out, ms_gen_stats* stats, bool device_io);

ms_status ms_generate(ms_model* model, const float* audio, int64_t n_samples,
                      const ms_gen_params* params, int32_t* ids_out, int32_t cap, int32_t* n_out,
                      float* logits_out, ms_gen_stats* stats) {
    return generate_impl(model, audio, n_samples, params, ids_out, cap, n_out, logits_out, stats, false);
}

ms_status ms_generate_device(ms_model* model, const float* audio_dev, int64_t n_samples,
                             const ms_gen_params* params, int32_t* ids_dev, int32_t cap, int32_t* n_out,
                             ms_gen_stats* stats) {
    return generate_impl(model, audio_dev, n_samples, params, ids_dev, cap, n_out, nullptr, stats, true);
}

ms_status ms_generate_long(ms_model* model, const float* audio, int64_t n_samples,
                           const ms_streaming_config* config, int32_t* ids_out, int32_t cap, int32_t* n_out,
                           ms_gen_stats* stats) {
    return guarded([&]() -> ms_status {
        if (!model || !n_out) return fail(MS_ERR_INVALID_ARG, "model and n_out must be non-null");
        if (n_samples < 0 || (n_samples > 0 && !audio)) return fail(MS_ERR_INVALID_ARG, "bad audio buffer");
        if (cap < 0 || (cap > 0 && !ids_out)) return fail(MS_ERR_INVALID_ARG, "bad ids buffer");
        ms_streaming_config sc;
        ms_streaming_config_default(&sc);
        if (config) sc = *config;
        if (sc.max_memory_frames <= 0) return fail(MS_ERR_INVALID_ARG, "max_memory_frames must be positive");
        Model& m = *reinterpret_cast<Model*>(model);
        std::lock_guard<std::mutex> g(m.mu);
        MSB_CUDA(cudaSetDevice(m.device));
        const Config& c = m.cfg;
        ms_gen_stats st;
        std::memset(&st, 0, sizeof(st));
        cudaEvent_t t0, t1, t2;
        MSB_CUDA(cudaEventCreate(&t0));
        MSB_CUDA(cudaEventCreate(&t1));
        MSB_CUDA(cudaEventCreate(&t2));
        MSB_CUDA(cudaEventRecord(t0, m.stream));
        // one full encode (MoonshineStreaming.swift:297-301) and the cross K/V of every row
        m.ws.audio.ensure((size_t)std::max<int64_t>(n_samples, 1) * 4);
        if (n_samples > 0)
            MSB_CUDA(cudaMemcpyAsync(m.ws.audio.p, audio, (size_t)n_samples * 4, cudaMemcpyHostToDevice, m.stream));
        const int total = m.encode_device(m.ws.audio.as<float>(), n_samples, 0);
        st.memory_frames = total;
        if (total > 0) m.cross_kv(m.memory_ptr(), total, 0);
        MSB_CUDA(cudaEventRecord(t1, m.stream));
        int32_t n = 0;
        auto put = [&](int32_t id) {
            if (n < cap) ids_out[n] = id;
            ++n;
        };
        int mem_start = 0;
        while (mem_start < total) {  // :312-360
            const int mem_end = std::min(mem_start + sc.max_memory_frames, total);
            const int frames = mem_end - mem_start;
            const int tok_limit = (int)std::ceil((double)frames * 0.02 * c.max_tok_per_s);
            if (tok_limit <= 0) break;
            m.ensure_decode(m.ws.m_cap, tok_limit, false, c.vocab);
            // a segment is a row slice of the cross K/V: same layout, base moved by mem_start rows
            const float* c32 = m.ws.cross32.as<float>() + (size_t)mem_start * c.head_dim;
            const char* cst = reinterpret_cast<const char*>(m.kv_f16 ? m.ws.cross16.p : m.ws.cross32.p) +
                              (size_t)mem_start * c.head_dim * (m.kv_f16 ? 2 : 4);
            Model::DecodeResult r = m.decode(c32, cst, m.ws.m_cap, frames, tok_limit, false, nullptr, false);
            const int n_ids = r.n_calls - (r.hit_eos ? 1 : 0);
            std::vector<int32_t> seg((size_t)std::max(n_ids, 0));
            if (n_ids > 0) {
                MSB_CUDA(cudaMemcpyAsync(seg.data(), m.ws.ids.p, (size_t)n_ids * 4, cudaMemcpyDeviceToHost, m.stream));
                MSB_CUDA(cudaStreamSynchronize(m.stream));
            }
            // the reference's hitEOS is set only by an EOS before the last decoder call
            const bool hit = r.hit_eos && r.n_calls < tok_limit;
            if (!seg.empty()) {
                for (int32_t id : seg) put(id);
                put(-1);
                st.n_chunks += 1;
            }
            st.n_tokens += (int32_t)seg.size();
            st.hit_eos = hit ? 1 : 0;
            st.decode_kernel = r.kernel;
            if (hit && frames > sc.min_segment_frames) {  // :354-359 (tokens include the start token)
                const int used = std::max(sc.min_segment_frames,
                                          (int)((double)(seg.size() + 1) / c.max_tok_per_s * 50.0));
                mem_start += std::min(used, frames);
            } else {
                mem_start = mem_end;
            }
        }
        MSB_CUDA(cudaEventRecord(t2, m.stream));
        MSB_CUDA(cudaEventSynchronize(t2));
        float te = 0, tt = 0;
        cudaEventElapsedTime(&te, t0, t1);
        cudaEventElapsedTime(&tt, t0, t2);
        cudaEventDestroy(t0);
        cudaEventDestroy(t1);
        cudaEventDestroy(t2);
        st.encode_ms = te;
        st.decode_ms = tt - te;
        st.total_ms = tt;
        const double dur = (double)n_samples / (double)c.sample_rate;
        st.tokens_per_second = tt > 0 ? dur / (tt / 1000.0) : 0.0;
        if (stats) *stats = st;
        *n_out = n;
        if (n > cap) return fail(MS_ERR_CAPACITY, "ids buffer too small");
        return MS_OK;
    });
}

ms_status ms_generate_alignment(ms_model* model, const float* audio, int64_t n_samples, int32_t max_tokens,
                                int32_t medfilt_width, ms_alignment* out, ms_gen_stats* stats) {
    return guarded([&]() -> ms_status {
        if (!model || !out) return fail(MS_ERR_INVALID_ARG, "model and out must be non-null");
        if (n_samples < 0 || (n_samples > 0 && !audio)) return fail(MS_ERR_INVALID_ARG, "bad audio buffer");
        if (out->cap < 0 || (out->cap > 0 && (!out->ids || !out->token_probs || !out->jump_frames)))
            return fail(MS_ERR_INVALID_ARG, "ids, token_probs and jump_frames must hold cap entries");
        if (out->attn_cap < 0) return fail(MS_ERR_INVALID_ARG, "attn_cap must be >= 0");
        if (medfilt_width > alignment_max_median_width())
            return fail(MS_ERR_INVALID_ARG, "medfilt_width must be at most " +
                                                std::to_string(alignment_max_median_width()));
        Model& m = *reinterpret_cast<Model*>(model);
        std::lock_guard<std::mutex> g(m.mu);
        MSB_CUDA(cudaSetDevice(m.device));
        const Config& c = m.cfg;
        out->n_tokens = out->n_steps = out->n_frames = out->hit_eos = 0;
        ms_gen_stats st;
        std::memset(&st, 0, sizeof(st));
        cudaEvent_t t0, t1, t2;
        MSB_CUDA(cudaEventCreate(&t0));
        MSB_CUDA(cudaEventCreate(&t1));
        MSB_CUDA(cudaEventCreate(&t2));
        MSB_CUDA(cudaEventRecord(t0, m.stream));
        // one encode of the whole audio (MoonshineModel.swift:253-256)
        m.ws.audio.ensure((size_t)std::max<int64_t>(n_samples, 1) * 4);
        if (n_samples > 0)
            MSB_CUDA(cudaMemcpyAsync(m.ws.audio.p, audio, (size_t)n_samples * 4, cudaMemcpyHostToDevice, m.stream));
        const int M = m.encode_device(m.ws.audio.as<float>(), n_samples, 0);
        st.memory_frames = M;
        out->n_frames = M;
        const double dur = (double)n_samples / (double)c.sample_rate;
        int limit = (int)std::ceil(dur * c.max_tok_per_s);  // :258-259
        if (max_tokens > 0) limit = std::min(limit, (int)max_tokens);
        std::vector<int32_t> ids;
        std::vector<float> probs, filt;
        int n_steps = 0;
        if (M > 0 && limit > 0) {
            m.cross_kv(m.memory_ptr(), M, 0);
            MSB_CUDA(cudaEventRecord(t1, m.stream));
            m.ensure_decode(m.ws.m_cap, limit, true, c.vocab);
            const int HD = c.heads * c.head_dim;
            m.ws.qtrace.ensure((size_t)limit * c.layers * HD * 4);
            const void* cst = m.kv_f16 ? m.ws.cross16.p : m.ws.cross32.p;
            Model::DecodeResult r = m.decode(m.ws.cross32.as<float>(), cst, m.ws.m_cap, M, limit, false, nullptr,
                                             true, 0.f, 0, m.ws.qtrace.as<float>());
            n_steps = r.n_calls;
            st.decode_kernel = r.kernel;
            st.hit_eos = r.hit_eos ? 1 : 0;
            if (n_steps > 0) {
                m.ws.apart.ensure(alignment_part_floats(n_steps, c.layers, M) * 4);
                m.ws.arows.ensure((size_t)n_steps * M * 4);
                m.ws.afilt.ensure((size_t)n_steps * M * 4);
                m.ws.aprobs.ensure((size_t)n_steps * 4);
                MSB_CUDA(launch_alignment_rows(m.ws.qtrace.as<float>(), m.ws.cross32.as<float>(), cst,
                                               m.kv_f16 ? 1 : 0, n_steps, c.layers, c.heads, c.kv_heads,
                                               c.head_dim, m.ws.m_cap, M, std::pow((float)c.head_dim, -0.5f),
                                               m.ws.logits.as<float>(), m.ws.ids.as<int>(), c.vocab,
                                               std::max(1, (int)medfilt_width), m.ws.apart.as<float>(),
                                               m.ws.arows.as<float>(), m.ws.afilt.as<float>(),
                                               m.ws.aprobs.as<float>(), m.stream));
                ids.resize(n_steps);
                probs.resize(n_steps);
                filt.resize((size_t)n_steps * M);
                MSB_CUDA(cudaMemcpyAsync(ids.data(), m.ws.ids.p, (size_t)n_steps * 4, cudaMemcpyDeviceToHost,
                                         m.stream));
                MSB_CUDA(cudaMemcpyAsync(probs.data(), m.ws.aprobs.p, (size_t)n_steps * 4,
                                         cudaMemcpyDeviceToHost, m.stream));
                MSB_CUDA(cudaMemcpyAsync(filt.data(), m.ws.afilt.p, filt.size() * 4, cudaMemcpyDeviceToHost,
                                         m.stream));
                const size_t rows_floats = (size_t)n_steps * M;
                if (out->attn_rows && (int64_t)rows_floats <= out->attn_cap)
                    MSB_CUDA(cudaMemcpyAsync(out->attn_rows, m.ws.arows.p, rows_floats * 4, cudaMemcpyDeviceToHost,
                                             m.stream));
            }
        } else {
            MSB_CUDA(cudaEventRecord(t1, m.stream));
        }
        MSB_CUDA(cudaStreamSynchronize(m.stream));
        const int n_tok = n_steps - (st.hit_eos ? 1 : 0);
        // the reference's DTW and jump extraction (MoonshineTimestamps.swift:148-184)
        const std::vector<int32_t> jumps = n_tok > 0 ? dtw_jump_frames(filt.data(), n_steps, M)
                                                     : std::vector<int32_t>();
        MSB_CUDA(cudaEventRecord(t2, m.stream));
        MSB_CUDA(cudaEventSynchronize(t2));
        float te = 0, tt = 0;
        cudaEventElapsedTime(&te, t0, t1);
        cudaEventElapsedTime(&tt, t0, t2);
        cudaEventDestroy(t0);
        cudaEventDestroy(t1);
        cudaEventDestroy(t2);
        out->n_tokens = std::max(n_tok, 0);
        out->n_steps = n_steps;
        out->hit_eos = st.hit_eos;
        const size_t rows_floats = (size_t)n_steps * M;
        if (out->attn_filtered && (int64_t)rows_floats <= out->attn_cap)
            std::memcpy(out->attn_filtered, filt.data(), rows_floats * 4);
        if (n_steps > out->cap) return fail(MS_ERR_CAPACITY, "ids / token_probs / jump_frames hold fewer than " +
                                                              std::to_string(n_steps) + " entries");
        for (int k = 0; k < out->n_tokens; ++k) out->ids[k] = ids[k];
        for (int k = 0; k < n_steps; ++k) out->token_probs[k] = probs[k];
        for (size_t k = 0; k < jumps.size(); ++k) out->jump_frames[k] = jumps[k];
        st.n_tokens = out->n_tokens;
        st.n_chunks = 1;
        st.encode_ms = te;
        st.decode_ms = tt - te;
        st.total_ms = tt;
        st.tokens_per_second = tt > 0 ? out->n_tokens / (tt / 1000.0) : 0.0;
        if (stats) *stats = st;
        if ((out->attn_rows || out->attn_filtered) && (int64_t)rows_floats > out->attn_cap)
            return fail(MS_ERR_CAPACITY, "attention buffers hold fewer than " + std::to_string(rows_floats) +
                                             " floats");
        return MS_OK;
    });
}

ms_status ms_alignment_jump_frames(const float* filtered, int32_t n_rows, int32_t n_frames,
                                   int32_t* jump_frames_out) {
    return guarded([&]() -> ms_status {
        if (n_rows < 0 || n_frames < 0) return fail(MS_ERR_INVALID_ARG, "negative size");
        if (n_rows > 0 && n_frames > 0 && (!filtered || !jump_frames_out))
            return fail(MS_ERR_INVALID_ARG, "null buffer");
        const std::vector<int32_t> j = dtw_jump_frames(filtered, n_rows, n_frames);
        for (size_t k = 0; k < j.size(); ++k) jump_frames_out[k] = j[k];
        return MS_OK;
    });
}

ms_status ms_word_timings(const int32_t* jump_frames, int32_t n_jumps, const float* token_probs, int32_t n_probs,
                          const int32_t* word_first, int32_t n_words, int32_t n_tokens, int32_t n_frames,
                          double time_offset, double* start_out, double* end_out, double* prob_out,
                          int32_t* n_out) {
    return guarded([&]() -> ms_status {
        if (n_jumps < 0 || n_probs < 0 || n_words < 0 || n_tokens < 0 || !n_out)
            return fail(MS_ERR_INVALID_ARG, "negative count or null n_out");
        if ((n_jumps && !jump_frames) || (n_probs && !token_probs) || (n_words && !word_first) ||
            (n_words && (!start_out || !end_out || !prob_out)))
            return fail(MS_ERR_INVALID_ARG, "null buffer");
        for (int w = 0; w < n_words; ++w)
            if (word_first[w] < 0 || word_first[w] >= n_tokens || (w && word_first[w] <= word_first[w - 1]))
                return fail(MS_ERR_INVALID_ARG, "word_first must ascend strictly within [0, n_tokens)");
        *n_out = 0;
        if (n_tokens == 0) return MS_OK;  // the reference returns no words without tokens (:104)
        const std::vector<WordTime> wt = word_times(jump_frames, n_jumps, token_probs, n_probs, word_first, n_words,
                                                    n_tokens, n_frames, time_offset);
        for (size_t k = 0; k < wt.size(); ++k) {
            start_out[k] = wt[k].start;
            end_out[k] = wt[k].end;
            prob_out[k] = wt[k].probability;
        }
        *n_out = (int32_t)wt.size();
        return MS_OK;
    });
}

void* ms_model_stream(ms_model* model) {
    return model ? (void*)reinterpret_cast<Model*>(model)->stream : nullptr;
}

ms_status ms_model_batch_kv_pages(ms_model* model, int64_t* used, int64_t* capacity, int32_t* page_positions) {
    if (!model) return fail(MS_ERR_INVALID_ARG, "null model");
    Model& m = *reinterpret_cast<Model*>(model);
    std::lock_guard<std::mutex> g(m.mu);
    if (used) *used = m.batch ? m.batch->pages_used : 0;
    if (capacity) *capacity = m.batch ? m.batch->pages_capacity : 0;
    if (page_positions) *page_positions = BatchEngine::kKvPage;
    return MS_OK;
}

static ms_status generate_impl(ms_model* model, const float* audio, int64_t n_samples,
                               const ms_gen_params* params, int32_t* ids_out, int32_t cap, int32_t* n_out,
                               float* logits_out, ms_gen_stats* stats, bool device_io) {
    return guarded([&]() -> ms_status {
        if (!model || !n_out) return fail(MS_ERR_INVALID_ARG, "model and n_out must be non-null");
        if (n_samples < 0 || (n_samples > 0 && !audio)) return fail(MS_ERR_INVALID_ARG, "bad audio buffer");
        if (cap < 0 || (cap > 0 && !ids_out)) return fail(MS_ERR_INVALID_ARG, "bad ids buffer");
        ms_gen_params gp;
        ms_gen_params_default(&gp);
        if (params) gp = *params;
        if (!(gp.temperature >= 0.f)) return fail(MS_ERR_INVALID_ARG, "temperature must be >= 0");
        if (gp.teacher_ids && gp.n_teacher <= 0) return fail(MS_ERR_INVALID_ARG, "n_teacher must be positive");
        Model& m = *reinterpret_cast<Model*>(model);
        std::lock_guard<std::mutex> g(m.mu);
        MSB_CUDA(cudaSetDevice(m.device));
        const int32_t max_tokens = gp.max_tokens > 0 ? gp.max_tokens : std::numeric_limits<int32_t>::max();
        const double cd = gp.chunk_duration > 0 ? gp.chunk_duration : 30.0;
        const int64_t chunk = (int64_t)(cd * (double)m.cfg.sample_rate);
        if (chunk <= 0) return fail(MS_ERR_INVALID_ARG, "chunk_duration too small");
        ms_gen_stats st;
        std::memset(&st, 0, sizeof(st));
        GenOut out;
        cudaEvent_t t0, t1;
        MSB_CUDA(cudaEventCreate(&t0));
        MSB_CUDA(cudaEventCreate(&t1));
        MSB_CUDA(cudaEventRecord(t0, m.stream));
        for (int64_t off = 0; off < n_samples; off += chunk) {
            const int64_t len = std::min(chunk, n_samples - off);
            generate_chunk(m, audio + off, len, gp, max_tokens, ids_out, cap, logits_out, out, st,
                           gp.teacher_ids, gp.n_teacher, device_io, (unsigned)st.n_chunks);
            st.n_chunks += 1;
        }
        MSB_CUDA(cudaEventRecord(t1, m.stream));
        MSB_CUDA(cudaEventSynchronize(t1));
        float tot = 0;
        cudaEventElapsedTime(&tot, t0, t1);
        cudaEventDestroy(t0);
        cudaEventDestroy(t1);
        st.n_tokens = out.n_ids;
        st.total_ms = tot;
        st.tokens_per_second = tot > 0 ? out.n_ids / (tot / 1000.0) : 0.0;
        if (stats) *stats = st;
        *n_out = out.n_ids;
        if (out.n_ids > cap) return fail(MS_ERR_CAPACITY, "ids buffer too small");
        return MS_OK;
    });
}

ms_status ms_encode(ms_model* model, const float* audio, int64_t n_samples, float* memory_out,
                    int64_t cap_floats, int32_t* n_frames) {
    return guarded([&]() -> ms_status {
        if (!model || !n_frames) return fail(MS_ERR_INVALID_ARG, "null argument");
        if (n_samples < 0 || (n_samples > 0 && !audio)) return fail(MS_ERR_INVALID_ARG, "bad audio buffer");
        Model& m = *reinterpret_cast<Model*>(model);
        std::lock_guard<std::mutex> g(m.mu);
        MSB_CUDA(cudaSetDevice(m.device));
        m.ws.audio.ensure((size_t)std::max<int64_t>(n_samples, 1) * 4);
        if (n_samples > 0)
            MSB_CUDA(cudaMemcpyAsync(m.ws.audio.p, audio, (size_t)n_samples * 4, cudaMemcpyHostToDevice,
                                     m.stream));
        const int M = m.encode_device(m.ws.audio.as<float>(), n_samples, 0);
        *n_frames = M;
        const int64_t need = (int64_t)M * m.cfg.hidden;
        if (need > cap_floats) {
            MSB_CUDA(cudaStreamSynchronize(m.stream));
            return fail(MS_ERR_CAPACITY, "memory buffer too small");
        }
        if (need > 0) {
            if (!memory_out) return fail(MS_ERR_INVALID_ARG, "null memory_out");
            MSB_CUDA(cudaMemcpyAsync(memory_out, m.memory_ptr(), (size_t)need * 4, cudaMemcpyDeviceToHost,
                                     m.stream));
        }
        MSB_CUDA(cudaStreamSynchronize(m.stream));
        return MS_OK;
    });
}

ms_status ms_generate_batch(ms_model* model, const float* const* audios, const int64_t* n_samples,
                            int32_t batch, const ms_gen_params* params, int32_t* ids_out, int32_t cap,
                            int32_t* n_out, ms_gen_stats* stats) {
    return guarded([&]() -> ms_status {
        if (!model || !audios || !n_samples || !n_out || batch < 0)
            return fail(MS_ERR_INVALID_ARG, "null argument");
        if (cap < 0 || (cap > 0 && !ids_out)) return fail(MS_ERR_INVALID_ARG, "bad ids buffer");
        ms_gen_stats total;
        std::memset(&total, 0, sizeof(total));
        ms_status worst = MS_OK;
        ms_gen_params gp;
        ms_gen_params_default(&gp);
        if (params) gp = *params;
        if (!(gp.temperature >= 0.f)) return fail(MS_ERR_INVALID_ARG, "temperature must be >= 0");
        Model& m = *reinterpret_cast<Model*>(model);
        const double cd = gp.chunk_duration > 0 ? gp.chunk_duration : 30.0;
        const int64_t chunk = (int64_t)(cd * (double)m.cfg.sample_rate);
        bool one_chunk = batch > 0 && !gp.teacher_ids;
        for (int32_t b = 0; b < batch && one_chunk; ++b)
            one_chunk = audios[b] && n_samples[b] >= m.cfg.frame_len() && n_samples[b] <= chunk;
        if (one_chunk) {
            // lockstep decode of the whole batch on the tensor-core engine
            std::lock_guard<std::mutex> g(m.mu);
            MSB_CUDA(cudaSetDevice(m.device));
            const int32_t max_tokens = gp.max_tokens > 0 ? gp.max_tokens : std::numeric_limits<int32_t>::max();
            std::vector<int> limits(batch);
            for (int32_t b = 0; b < batch; ++b) {
                const double dur = (double)n_samples[b] / (double)m.cfg.sample_rate;
                limits[b] = gp.forced_len > 0 ? gp.forced_len
                                              : (int)std::min<int64_t>(max_tokens,
                                                                       (int64_t)std::ceil(dur * m.cfg.max_tok_per_s));
                if (limits[b] <= 0) return fail(MS_ERR_INVALID_ARG, "token limit must be positive");
            }
            int64_t total_samples = 0;
            std::vector<int64_t> offs(batch);
            for (int32_t b = 0; b < batch; ++b) {
                offs[b] = total_samples;
                total_samples += (n_samples[b] + 63) / 64 * 64;  // keep every utterance 256-byte aligned
            }
            m.ws.audio.ensure((size_t)total_samples * 4);
            std::vector<const float*> dev(batch);
            std::vector<int64_t> lens(n_samples, n_samples + batch);
            for (int32_t b = 0; b < batch; ++b) {
                dev[b] = m.ws.audio.as<float>() + offs[b];
                MSB_CUDA(cudaMemcpyAsync(const_cast<float*>(dev[b]), audios[b], (size_t)n_samples[b] * 4,
                                         cudaMemcpyHostToDevice, m.stream));
            }
            if (!m.batch) m.batch.reset(new BatchEngine(m));
            cudaEvent_t t0, t1;
            MSB_CUDA(cudaEventCreate(&t0));
            MSB_CUDA(cudaEventCreate(&t1));
            MSB_CUDA(cudaEventRecord(t0, m.stream));
            BatchEngine::Result r = m.batch->run(dev, lens, limits, gp.forced_len != 0, gp.batch_logits != nullptr,
                                                 gp.temperature, (unsigned)gp.seed);
            MSB_CUDA(cudaEventRecord(t1, m.stream));
            MSB_CUDA(cudaEventSynchronize(t1));
            float tot = 0;
            cudaEventElapsedTime(&tot, t0, t1);
            cudaEventDestroy(t0);
            cudaEventDestroy(t1);
            const int V = m.cfg.vocab;
            for (int32_t b = 0; b < batch; ++b) {
                const int n = r.counts[b];
                n_out[b] = n;
                if (n > cap) worst = MS_ERR_CAPACITY;
                for (int i = 0; i < std::min(n, cap); ++i) ids_out[(size_t)b * cap + i] = r.ids[(size_t)b * r.t_cap + i];
                if (gp.batch_logits)
                    for (int st = 0; st < std::min(r.steps, cap); ++st)
                        std::memcpy(gp.batch_logits + ((size_t)b * cap + st) * V,
                                    r.logits.data() + ((size_t)st * batch + b) * V, (size_t)V * 4);
                total.n_tokens += n;
            }
            total.n_chunks = batch;
            total.encode_ms = r.encode_ms;
            total.decode_ms = r.decode_ms;
            total.total_ms = tot;
            total.tokens_per_second = tot > 0 ? total.n_tokens / (tot / 1000.0) : 0.0;
            if (stats) *stats = total;
            if (worst != MS_OK) return fail(worst, "ids buffer too small");
            return MS_OK;
        }
        for (int32_t b = 0; b < batch; ++b) {
            ms_gen_stats st;
            ms_status s = ms_generate(model, audios[b], n_samples[b], params, ids_out + (size_t)b * cap, cap,
                                      n_out + b, nullptr, &st);
            if (s != MS_OK && s != MS_ERR_CAPACITY) return s;
            if (s == MS_ERR_CAPACITY) worst = s;
            total.n_tokens += st.n_tokens;
            total.n_chunks += st.n_chunks;
            total.encode_ms += st.encode_ms;
            total.decode_ms += st.decode_ms;
            total.total_ms += st.total_ms;
        }
        total.tokens_per_second = total.total_ms > 0 ? total.n_tokens / (total.total_ms / 1000.0) : 0.0;
        if (stats) *stats = total;
        if (worst != MS_OK) return fail(worst, "ids buffer too small");
        return MS_OK;
    });
}

// ------------------------------------------------------------------- streaming

ms_status ms_stream_create(ms_model* model, ms_stream** out) {
    return guarded([&]() -> ms_status {
        if (!model || !out) return fail(MS_ERR_INVALID_ARG, "null argument");
        Model* m = reinterpret_cast<Model*>(model);
        std::lock_guard<std::mutex> g(m->mu);
        MSB_CUDA(cudaSetDevice(m->device));
        *out = reinterpret_cast<ms_stream*>(new StreamState(m));
        return MS_OK;
    });
}

void ms_stream_free(ms_stream* stream) {
    if (!stream) return;
    StreamState* s = reinterpret_cast<StreamState*>(stream);
    {
        std::lock_guard<std::mutex> g(s->model->mu);
        cudaSetDevice(s->model->device);
        cudaStreamSynchronize(s->model->stream);
    }
    delete s;
}

ms_status ms_stream_start(ms_stream* stream) {
    if (!stream) return fail(MS_ERR_INVALID_ARG, "null stream");
    StreamState* s = reinterpret_cast<StreamState*>(stream);
    std::lock_guard<std::mutex> g(s->model->mu);
    s->start();
    return MS_OK;
}

ms_status ms_stream_stop(ms_stream* stream) {
    if (!stream) return fail(MS_ERR_INVALID_ARG, "null stream");
    StreamState* s = reinterpret_cast<StreamState*>(stream);
    std::lock_guard<std::mutex> g(s->model->mu);
    s->stop();
    return MS_OK;
}

ms_status ms_stream_add_audio(ms_stream* stream, const float* chunk, int64_t n_samples) {
    return guarded([&]() -> ms_status {
        if (!stream || n_samples < 0 || (n_samples > 0 && !chunk)) return fail(MS_ERR_INVALID_ARG, "bad argument");
        StreamState* s = reinterpret_cast<StreamState*>(stream);
        std::lock_guard<std::mutex> g(s->model->mu);
        MSB_CUDA(cudaSetDevice(s->model->device));
        s->add_audio(chunk, n_samples);
        return MS_OK;
    });
}

ms_status ms_stream_add_audio_batch(ms_stream* const* streams, int32_t n, const float* const* chunks,
                                    const int64_t* n_samples) {
    return guarded([&]() -> ms_status {
        if (!streams || n < 0 || (n > 0 && (!chunks || !n_samples))) return fail(MS_ERR_INVALID_ARG, "bad argument");
        for (int32_t i = 0; i < n; ++i)
            if (!streams[i] || n_samples[i] < 0 || (n_samples[i] > 0 && !chunks[i]))
                return fail(MS_ERR_INVALID_ARG, "bad stream or chunk in batch");
        Model* shared = n > 0 ? reinterpret_cast<StreamState*>(streams[0])->model : nullptr;
        for (int32_t i = 1; i < n && shared; ++i)
            if (reinterpret_cast<StreamState*>(streams[i])->model != shared) shared = nullptr;
        if (!shared) {  // streams of several models: one at a time
            for (int32_t i = 0; i < n; ++i) {
                const ms_status st = ms_stream_add_audio(streams[i], chunks[i], n_samples[i]);
                if (st != MS_OK) return st;
            }
            return MS_OK;
        }
        std::lock_guard<std::mutex> g(shared->mu);
        MSB_CUDA(cudaSetDevice(shared->device));
        // all the streams' frontends in one pass on the model stream: one upload, five launches
        add_audio_batch(*shared, reinterpret_cast<StreamState* const*>(streams), n, chunks, n_samples,
                        shared->stream);
        return MS_OK;
    });
}

static ms_status transcribe_one(StreamState* s, int32_t is_final, const ms_streaming_config& sc,
                                int32_t max_tokens, int32_t* ids_out, int32_t cap, int32_t* n_out,
                                int32_t* hit_eos, int32_t* emitted) {
    StreamState::Result r = s->transcribe(is_final != 0, sc, max_tokens);
    const int32_t n = (int32_t)r.ids.size();
    *n_out = n;
    const int32_t fit = std::min(n, cap);
    if (fit > 0) std::memcpy(ids_out, r.ids.data(), (size_t)fit * 4);
    if (hit_eos) *hit_eos = r.hit_eos ? 1 : 0;
    if (emitted) *emitted = r.emitted ? 1 : 0;
    if (n > cap) return fail(MS_ERR_CAPACITY, "ids buffer too small");
    return MS_OK;
}

ms_status ms_stream_transcribe(ms_stream* stream, int32_t is_final, const ms_streaming_config* config,
                               int32_t max_tokens, int32_t* ids_out, int32_t cap, int32_t* n_out,
                               int32_t* hit_eos, int32_t* emitted) {
    return guarded([&]() -> ms_status {
        if (!stream || !n_out || cap < 0 || (cap > 0 && !ids_out)) return fail(MS_ERR_INVALID_ARG, "bad argument");
        ms_streaming_config sc;
        ms_streaming_config_default(&sc);
        if (config) sc = *config;
        if (!(sc.temperature >= 0.f)) return fail(MS_ERR_INVALID_ARG, "temperature must be >= 0");
        const int32_t mt = max_tokens > 0 ? max_tokens : std::numeric_limits<int32_t>::max();
        StreamState* s = reinterpret_cast<StreamState*>(stream);
        std::lock_guard<std::mutex> g(s->model->mu);
        MSB_CUDA(cudaSetDevice(s->model->device));
        return transcribe_one(s, is_final, sc, mt, ids_out, cap, n_out, hit_eos, emitted);
    });
}

ms_status ms_stream_transcribe_batch(ms_stream* const* streams, int32_t n, int32_t is_final,
                                     const ms_streaming_config* config, int32_t max_tokens, int32_t* ids_out,
                                     int32_t cap, int32_t* n_out, int32_t* hit_eos, int32_t* emitted) {
    return guarded([&]() -> ms_status {
        if (!streams || !n_out || n < 0 || cap < 0 || (cap > 0 && !ids_out))
            return fail(MS_ERR_INVALID_ARG, "bad argument");
        ms_streaming_config sc;
        ms_streaming_config_default(&sc);
        if (config) sc = *config;
        if (!(sc.temperature >= 0.f)) return fail(MS_ERR_INVALID_ARG, "temperature must be >= 0");
        const int32_t mt = max_tokens > 0 ? max_tokens : std::numeric_limits<int32_t>::max();
        ms_status worst = MS_OK;
        for (int32_t i = 0; i < n; ++i)
            if (!streams[i]) return fail(MS_ERR_INVALID_ARG, "null stream in batch");
        Model* shared = n > 0 ? reinterpret_cast<StreamState*>(streams[0])->model : nullptr;
        for (int32_t i = 1; i < n && shared; ++i)
            if (reinterpret_cast<StreamState*>(streams[i])->model != shared) shared = nullptr;
        if (sc.batch_decode && shared) {
            // encode each stream's new frames, decode every segment with memory in lockstep
            std::lock_guard<std::mutex> g(shared->mu);
            MSB_CUDA(cudaSetDevice(shared->device));
            std::vector<StreamState::Result> res(n);
            std::vector<int64_t> lim(n);
            std::vector<BatchEngine::CrossSrc> src;
            std::vector<int> limits, rows;
            if (!shared->batch) shared->batch.reset(new BatchEngine(*shared));
            BatchEngine& be = *shared->batch;
            if (be.tc_encoder_fits() && shared->opts.weight_dtype != MS_W_F32) {
                // every stream's new frames through one tensor-core encoder pass (split operands
                // for fp32 checkpoints, bf16 for bf16 ones)
                std::vector<StreamState::EncPlan> plan(n);
                std::vector<char> has(n, 0);
                std::vector<BatchEngine::StreamWindow> wins;
                std::vector<BatchEngine::StreamIncWindow> incs;
                // batch_decode 1: each layer over the rows that can have changed (incremental);
                // 2: the whole window again every call, as the reference does
                const bool incremental = sc.batch_decode != 2;
                for (int32_t i = 0; i < n; ++i) {
                    StreamState* s = reinterpret_cast<StreamState*>(streams[i]);
                    s->note_call();
                    has[i] = s->plan_new_frames(is_final != 0, &plan[i], shared->stream) ? 1 : 0;
                    if (!has[i]) continue;
                    if (incremental && s->enc_inc) {
                        incs.push_back({s->features.as<float>(), s->inc_buffers(shared->stream), s->feat_count,
                                        s->enc_valid, s->encoder_frames_emitted, plan[i].nnew, s->pos_offset,
                                        s->memory_row()});
                        s->enc_valid = s->feat_count;
                    } else {
                        wins.push_back({s->window(plan[i]), plan[i].T, plan[i].off, plan[i].nnew, s->pos_offset,
                                        s->memory_row()});
                        s->enc_inc = false;
                    }
                }
                be.encode_windows(wins);
                be.encode_windows_inc(incs);
                // the cross K/V of every stream's new memory rows in one launch
                std::vector<StreamState*> enc_ss;
                std::vector<StreamState::EncPlan> enc_plans;
                for (int32_t i = 0; i < n; ++i)
                    if (has[i]) {
                        enc_ss.push_back(reinterpret_cast<StreamState*>(streams[i]));
                        enc_plans.push_back(plan[i]);
                    }
                commit_new_frames_batch(*shared, enc_ss.data(), enc_plans.data(), (int)enc_ss.size(),
                                        shared->stream);
                for (int32_t i = 0; i < n; ++i)
                    lim[i] = reinterpret_cast<StreamState*>(streams[i])->decode_limit(is_final != 0, mt, &res[i]);
            } else {
                const int lanes = std::min<int32_t>(n, 8);  // concurrent incremental encoders
                shared->fork_lanes(lanes);
                for (int32_t i = 0; i < n; ++i)
                    lim[i] = reinterpret_cast<StreamState*>(streams[i])
                                 ->begin(is_final != 0, mt, &res[i], &shared->enc_lane(i % lanes));
                shared->join_lanes(lanes);
            }
            for (int32_t i = 0; i < n; ++i) {
                StreamState* s = reinterpret_cast<StreamState*>(streams[i]);
                if (lim[i] > 0) {
                    src.push_back({s->cross32.as<float>(), s->cross16.p, s->mem_cap, s->memory_len});
                    limits.push_back((int)lim[i]);
                    rows.push_back(i);
                }
            }
            if (!src.empty()) {
                // one seed for the lockstep batch: the rows (stream positions) separate the draws
                unsigned seed = (unsigned)sc.seed;
                if (sc.temperature > 0.f)
                    seed = mix_seed(seed, reinterpret_cast<StreamState*>(streams[rows[0]])->calls - 1);
                BatchEngine::Result r = shared->batch->run_cross(src, limits, false, sc.temperature, seed);
                for (size_t k = 0; k < rows.size(); ++k) {
                    const int32_t i = rows[k];
                    std::vector<int32_t> ids(r.ids.begin() + (size_t)k * r.t_cap,
                                             r.ids.begin() + (size_t)k * r.t_cap + r.counts[k]);
                    res[i] = reinterpret_cast<StreamState*>(streams[i])->finish(std::move(ids), r.hit_eos[k] != 0,
                                                                                  is_final != 0, sc);
                }
            }
            for (int32_t i = 0; i < n; ++i) {
                const int32_t cnt = (int32_t)res[i].ids.size();
                n_out[i] = cnt;
                for (int32_t j = 0; j < std::min(cnt, cap); ++j) ids_out[(size_t)i * cap + j] = res[i].ids[j];
                if (hit_eos) hit_eos[i] = res[i].hit_eos ? 1 : 0;
                if (emitted) emitted[i] = res[i].emitted ? 1 : 0;
                if (cnt > cap) worst = MS_ERR_CAPACITY;
            }
            if (worst != MS_OK) return fail(worst, "ids buffer too small");
            return MS_OK;
        }
        for (int32_t i = 0; i < n; ++i) {
            StreamState* s = reinterpret_cast<StreamState*>(streams[i]);
            std::lock_guard<std::mutex> g(s->model->mu);
            MSB_CUDA(cudaSetDevice(s->model->device));
            ms_status st = transcribe_one(s, is_final, sc, mt, ids_out + (size_t)i * cap, cap, n_out + i,
                                          hit_eos ? hit_eos + i : nullptr, emitted ? emitted + i : nullptr);
            if (st != MS_OK) worst = st;
        }
        if (worst != MS_OK) return fail(worst, "ids buffer too small");
        return MS_OK;
    });
}

ms_status ms_stream_emitted(ms_stream* stream, int32_t* ids_out, int32_t cap, int32_t* n_out) {
    if (!stream || !n_out || cap < 0 || (cap > 0 && !ids_out)) return fail(MS_ERR_INVALID_ARG, "bad argument");
    StreamState* s = reinterpret_cast<StreamState*>(stream);
    std::lock_guard<std::mutex> g(s->model->mu);
    int32_t n = 0;
    for (auto& seg : s->emitted) {
        for (int32_t id : seg) {
            if (n < cap) ids_out[n] = id;
            ++n;
        }
        if (n < cap) ids_out[n] = -1;
        ++n;
    }
    *n_out = n;
    if (n > cap) return fail(MS_ERR_CAPACITY, "ids buffer too small");
    return MS_OK;
}

int32_t ms_stream_memory_len(const ms_stream* stream) {
    if (!stream) return 0;
    return reinterpret_cast<const StreamState*>(stream)->memory_len;
}

ms_status ms_stream_memory(ms_stream* stream, float* memory_out, int64_t cap_floats, int32_t* rows_out) {
    return guarded([&]() -> ms_status {
        if (!stream || !rows_out || cap_floats < 0 || (cap_floats > 0 && !memory_out))
            return fail(MS_ERR_INVALID_ARG, "bad argument");
        StreamState* s = reinterpret_cast<StreamState*>(stream);
        std::lock_guard<std::mutex> g(s->model->mu);
        MSB_CUDA(cudaSetDevice(s->model->device));
        *rows_out = s->memory_len;
        const int64_t need = (int64_t)s->memory_len * s->model->cfg.hidden;
        if (need > cap_floats) return fail(MS_ERR_CAPACITY, "memory buffer too small");
        if (need > 0)
            MSB_CUDA(cudaMemcpyAsync(memory_out, s->memory.p, (size_t)need * 4, cudaMemcpyDeviceToHost,
                                     s->model->stream));
        MSB_CUDA(cudaStreamSynchronize(s->model->stream));
        return MS_OK;
    });
}

}  // extern "C"
