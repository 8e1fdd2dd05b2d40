// Model loading (config.json + safetensors) and the batch-1 encode / decode orchestration.
#include "model.hpp"

#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>

#include "batch.hpp"
#include "json.hpp"

namespace msb {

void cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        throw MsError(MS_ERR_OOM, std::string("CUDA out of memory in ") + what);
    }
    throw MsError(MS_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

ms_status to_status(const std::exception& e) {
    if (auto* m = dynamic_cast<const MsError*>(&e)) return m->status;
    if (dynamic_cast<const std::bad_alloc*>(&e)) return MS_ERR_OOM;
    return MS_ERR_INVALID_ARG;
}

DevBuf::~DevBuf() {
    if (p) cudaFree(p);
}

TableUpload::~TableUpload() {
    if (done) {
        cudaEventSynchronize(done);
        cudaEventDestroy(done);
    }
    if (stage) cudaFreeHost(stage);
}

char* TableUpload::host(size_t bytes) {
    if (!done) MSB_CUDA(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
    MSB_CUDA(cudaEventSynchronize(done));
    if (bytes > cap) {
        if (stage) MSB_CUDA(cudaFreeHost(stage));
        stage = nullptr;
        const size_t c = std::max(bytes, 2 * cap);
        MSB_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&stage), c, cudaHostAllocDefault));
        cap = c;
    }
    return stage;
}

char* TableUpload::upload(size_t bytes, cudaStream_t s, cudaMemPool_t pool) {
    // grows by half again at least, so a slowly growing call rarely reallocates
    if (bytes > dev.bytes) dev.ensure_on(std::max(bytes, dev.bytes + dev.bytes / 2), s, pool);
    MSB_CUDA(cudaMemcpyAsync(dev.p, stage, bytes, cudaMemcpyHostToDevice, s));
    MSB_CUDA(cudaEventRecord(done, s));
    return dev.as<char>();
}

void DevBuf::ensure_on(size_t n, cudaStream_t s, cudaMemPool_t pool) {
    if (n <= bytes) return;
    if (p) MSB_CUDA(cudaFreeAsync(p, s));
    p = nullptr;
    bytes = 0;
    MSB_CUDA(cudaMallocFromPoolAsync(&p, n, pool, s));
    bytes = n;
}

void DevBuf::ensure(size_t n) {
    if (n <= bytes) return;
    if (p) {
        cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    MSB_CUDA(cudaMalloc(&p, n));
    bytes = n;
}

// ------------------------------------------------------------------ config

static std::string read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw MsError(MS_ERR_NOT_FOUND, "cannot open " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

Config Config::from_json_file(const std::string& path) {
    std::string txt = read_file(path);
    Json d;
    try {
        d = Json::parse(txt.data(), txt.size());
    } catch (const std::exception& e) {
        throw MsError(MS_ERR_BAD_CONFIG, std::string("Failed to parse config.json: ") + e.what());
    }
    if (d.kind != Json::Object) throw MsError(MS_ERR_BAD_CONFIG, "Failed to parse config.json");
    Config c;
    // MoonshineConfig.swift:134-177
    c.hidden = (int)d.int_or("hidden_size", 320);
    c.inter = (int)d.int_or("intermediate_size", 1280);
    c.layers = (int)d.int_or("num_hidden_layers", 6);
    c.heads = (int)d.int_or("num_attention_heads", 8);
    c.kv_heads = (int)d.int_or("num_key_value_heads", 8);
    c.head_dim = (int)d.int_or("head_dim", 40);
    c.vocab = (int)d.int_or("vocab_size", 32768);
    c.max_pos = (int)d.int_or("max_position_embeddings", 4096);
    c.tie = d.bool_or("tie_word_embeddings", false);
    const Json* ehs = d.get("encoder_hidden_size");
    const bool has_ehs = ehs && ehs->kind == Json::Number;
    c.bos = (int)d.int_or("bos_token_id", 1);
    c.eos = (int)d.int_or("eos_token_id", 2);
    c.dec_start = (int)d.int_or("decoder_start_token_id", 1);
    c.pad = (int)d.int_or("pad_token_id", 0);
    c.partial_rotary = d.num_or("partial_rotary_factor", 0.8);
    c.rope_theta = d.num_or("rope_theta", 10000.0);
    if (const Json* rp = d.get("rope_parameters"); rp && rp->kind == Json::Object) {
        c.partial_rotary = rp->num_or("partial_rotary_factor", c.partial_rotary);
        c.rope_theta = rp->num_or("rope_theta", c.rope_theta);
    }
    c.max_tok_per_s = d.num_or("max_tokens_per_second", 6.5);
    if (const Json* q = d.get("quantization"); q && q->kind == Json::Object) {
        c.quantized = true;
        c.q_group = (int)q->int_or("group_size", 64);
        c.q_bits = (int)q->int_or("bits", 8);
    }
    if (const Json* e = d.get("encoder_config"); e && e->kind == Json::Object) {
        // MoonshineConfig.swift:43-56
        c.e_hidden = (int)e->int_or("hidden_size", 320);
        c.e_inter = (int)e->int_or("intermediate_size", 1280);
        c.e_layers = (int)e->int_or("num_hidden_layers", 6);
        c.e_heads = (int)e->int_or("num_attention_heads", 8);
        c.e_kv_heads = (int)e->int_or("num_key_value_heads", 8);
        c.e_head_dim = (int)e->int_or("head_dim", 40);
        c.frame_ms = e->num_or("frame_ms", 5.0);
        c.sample_rate = (int)e->int_or("sample_rate", 16000);
        c.e_max_pos = (int)e->int_or("max_position_embeddings", 4096);
        if (const Json* sw = e->get("sliding_windows"); sw && sw->kind == Json::Array) {
            c.has_windows = true;
            for (const Json& w : sw->arr) {
                if (w.kind != Json::Array || w.arr.size() < 2 || w.arr[0].kind != Json::Number ||
                    w.arr[1].kind != Json::Number)
                    throw MsError(MS_ERR_BAD_CONFIG, "sliding_windows entries must be [left, right]");
                c.windows.emplace_back((int)w.arr[0].num, (int)w.arr[1].num);
            }
        }
    } else {
        // MoonshineConfig.swift:115-122
        const int eh = has_ehs ? (int)ehs->num : c.hidden;
        c.e_hidden = eh;
        c.e_inter = eh * 4;
        c.e_layers = c.layers;
        c.e_heads = c.heads;
        c.e_kv_heads = c.kv_heads;
        c.e_head_dim = c.head_dim;
    }
    c.enc_hidden_size = has_ehs ? (int)ehs->num : c.e_hidden;
    return c;
}

// ------------------------------------------------------------------ safetensors

namespace {

struct Tensor {
    std::string dtype;
    std::vector<int64_t> shape;
    const uint8_t* data = nullptr;
    size_t bytes = 0;
    int64_t numel() const {
        int64_t n = 1;
        for (auto s : shape) n *= s;
        return n;
    }
};

struct SafeTensors {
    int fd = -1;
    void* map = nullptr;
    size_t size = 0;
    std::map<std::string, Tensor> tensors;
    ~SafeTensors() {
        if (map && map != MAP_FAILED) munmap(map, size);
        if (fd >= 0) close(fd);
    }
    void open_file(const std::string& path) {
        fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) throw MsError(MS_ERR_NOT_FOUND, "cannot open " + path);
        struct stat st;
        if (fstat(fd, &st) != 0) throw MsError(MS_ERR_BAD_WEIGHTS, "stat failed: " + path);
        size = (size_t)st.st_size;
        if (size < 8) throw MsError(MS_ERR_BAD_WEIGHTS, "truncated safetensors: " + path);
        map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (map == MAP_FAILED) throw MsError(MS_ERR_BAD_WEIGHTS, "mmap failed: " + path);
        const uint8_t* b = reinterpret_cast<const uint8_t*>(map);
        uint64_t hn = 0;
        std::memcpy(&hn, b, 8);
        if (hn > size - 8) throw MsError(MS_ERR_BAD_WEIGHTS, "bad safetensors header size");
        Json h;
        try {
            h = Json::parse(reinterpret_cast<const char*>(b + 8), (size_t)hn);
        } catch (const std::exception& e) {
            throw MsError(MS_ERR_BAD_WEIGHTS, std::string("bad safetensors header: ") + e.what());
        }
        const uint8_t* data = b + 8 + hn;
        const size_t data_size = size - 8 - hn;
        for (auto& kv : h.obj) {
            if (kv.first == "__metadata__") continue;
            const Json& m = kv.second;
            Tensor t;
            t.dtype = m.str_or("dtype", "");
            if (const Json* sh = m.get("shape"))
                for (auto& s : sh->arr) t.shape.push_back((int64_t)s.num);
            const Json* off = m.get("data_offsets");
            if (!off || off->arr.size() != 2) throw MsError(MS_ERR_BAD_WEIGHTS, "bad offsets: " + kv.first);
            const size_t a = (size_t)off->arr[0].num, e = (size_t)off->arr[1].num;
            if (a > e || e > data_size) throw MsError(MS_ERR_BAD_WEIGHTS, "offsets out of range: " + kv.first);
            t.data = data + a;
            t.bytes = e - a;
            size_t esz = (t.dtype == "F32" || t.dtype == "U32") ? 4 : (t.dtype == "F16" || t.dtype == "BF16") ? 2 : 0;
            if (esz && (size_t)t.numel() * esz != t.bytes)
                throw MsError(MS_ERR_BAD_WEIGHTS, "size mismatch: " + kv.first);
            tensors[kv.first] = t;
        }
    }
};

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f, mant = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) bits = sign;
        else {
            exp = 127 - 15 + 1;
            while (!(mant & 0x400)) {
                mant <<= 1;
                --exp;
            }
            mant &= 0x3ff;
            bits = sign | (exp << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

std::vector<float> to_f32(const Tensor& t) {
    std::vector<float> out((size_t)t.numel());
    if (t.dtype == "F32") {
        std::memcpy(out.data(), t.data, t.bytes);
    } else if (t.dtype == "F16") {
        const uint16_t* s = reinterpret_cast<const uint16_t*>(t.data);
        for (size_t i = 0; i < out.size(); ++i) out[i] = half_to_float(s[i]);
    } else if (t.dtype == "BF16") {
        const uint16_t* s = reinterpret_cast<const uint16_t*>(t.data);
        for (size_t i = 0; i < out.size(); ++i) {
            uint32_t b = (uint32_t)s[i] << 16;
            std::memcpy(&out[i], &b, 4);
        }
    } else {
        throw MsError(MS_ERR_BAD_WEIGHTS, "unsupported tensor dtype " + t.dtype);
    }
    return out;
}

std::string find_weights(const std::string& dir) {
    // ModelLoader.swift:115-130: prefer model.safetensors, else any *.safetensors
    std::string first;
    DIR* dp = opendir(dir.c_str());
    if (!dp) throw MsError(MS_ERR_NOT_FOUND, "No safetensors weights found in: " + dir);
    while (dirent* e = readdir(dp)) {
        std::string n = e->d_name;
        if (n.size() > 12 && n.substr(n.size() - 12) == ".safetensors") {
            if (n == "model.safetensors") {
                closedir(dp);
                return dir + "/" + n;
            }
            if (first.empty() || n < first) first = n;
        }
    }
    closedir(dp);
    if (first.empty()) throw MsError(MS_ERR_NOT_FOUND, "No safetensors weights found in: " + dir);
    return dir + "/" + first;
}

// Sanitised view of the checkpoint (ModelLoader.swift:75-101).
struct WeightSource {
    SafeTensors st;
    bool hf = false;
    std::map<std::string, const Tensor*> byname;

    void load(const std::string& path) {
        st.open_file(path);
        for (auto& kv : st.tensors)
            if (kv.first.rfind("model.", 0) == 0) hf = true;
        for (auto& kv : st.tensors) {
            std::string k = kv.first;
            if (hf) {
                if (k.rfind("model.", 0) == 0) k = k.substr(6);
                size_t p;
                while ((p = k.find(".gamma")) != std::string::npos) k.replace(p, 6, ".weight");
            }
            byname[k] = &kv.second;
        }
    }
    const Tensor& need(const std::string& k, std::vector<int64_t> shape) const {
        auto it = byname.find(k);
        if (it == byname.end()) throw MsError(MS_ERR_BAD_WEIGHTS, "missing weight " + k);
        const Tensor& t = *it->second;
        if (t.shape != shape) {
            std::string s = "shape mismatch for " + k + ": got [";
            for (auto v : t.shape) s += std::to_string(v) + ",";
            s += "] want [";
            for (auto v : shape) s += std::to_string(v) + ",";
            throw MsError(MS_ERR_BAD_WEIGHTS, s + "]");
        }
        return t;
    }
    bool has(const std::string& k) const { return byname.count(k) != 0; }
    const Tensor& need_any(const std::string& k) const {
        auto it = byname.find(k);
        if (it == byname.end()) throw MsError(MS_ERR_BAD_WEIGHTS, "missing weight " + k);
        return *it->second;
    }
    // Affine quantization of Linear weights (MLX format): a uint32 `.weight` of packed
    // `q_bits`-bit codes, lowest bits first, with per-group `.scales` / `.biases`.
    int q_group = 0, q_bits = 0;
    std::vector<float> f32(const std::string& k, std::vector<int64_t> shape) const {
        auto it = byname.find(k);
        if (it != byname.end() && it->second->dtype == "U32" && q_bits > 0 && shape.size() == 2)
            return dequantize(k, shape[0], shape[1]);
        return to_f32(need(k, shape));
    }
    // w = scale * q + bias per group of q_group inputs: the matrix quantized_matmul multiplies by
    // (ModelLoader.swift:47-49,103-111).
    std::vector<float> dequantize(const std::string& k, int64_t out, int64_t in) const {
        const std::string base = k.substr(0, k.size() - std::string(".weight").size());
        if (k.size() < 7 || k.compare(k.size() - 7, 7, ".weight") != 0 || in % q_group)
            throw MsError(MS_ERR_BAD_WEIGHTS, "unexpected quantized tensor " + k);
        const int per = 32 / q_bits;
        const Tensor& packed = need(k, {out, in / per});
        const std::vector<float> sc = to_f32(need(base + ".scales", {out, in / q_group}));
        const std::vector<float> bi = to_f32(need(base + ".biases", {out, in / q_group}));
        const uint32_t* q = reinterpret_cast<const uint32_t*>(packed.data);
        const uint32_t mask = (1u << q_bits) - 1u;
        std::vector<float> w((size_t)out * in);
        for (int64_t o = 0; o < out; ++o)
            for (int64_t i = 0; i < in; ++i) {
                const uint32_t word = q[(size_t)o * (in / per) + i / per];
                const float code = (float)((word >> ((i % per) * q_bits)) & mask);
                const size_t gi = (size_t)o * (in / q_group) + i / q_group;
                w[(size_t)o * in + i] = sc[gi] * code + bi[gi];
            }
        return w;
    }
    bool is_quantized(const std::string& k) const {
        auto it = byname.find(k);
        return q_bits > 0 && it != byname.end() && it->second->dtype == "U32";
    }
    // Rows of a quantized Linear as the clustered decode kernel streams them: per row its
    // packed codes (in * q_bits / 32 words, as stored), then one (scale, bias) fp32 pair per
    // group, zero padded to quant_row_stride words.
    std::vector<uint32_t> quant_records(const std::string& k, int64_t out, int64_t in) const {
        if (!is_quantized(k) || in % q_group)
            throw MsError(MS_ERR_BAD_WEIGHTS, "unexpected quantized tensor " + k);
        const std::string base = k.substr(0, k.size() - std::string(".weight").size());
        const int per = 32 / q_bits;
        const int64_t ng = in / q_group, cw = in / per;
        const Tensor& packed = need(k, {out, cw});
        const std::vector<float> sc = to_f32(need(base + ".scales", {out, ng}));
        const std::vector<float> bi = to_f32(need(base + ".biases", {out, ng}));
        const int rs = quant_row_stride((int)in, q_bits, q_group);
        std::vector<uint32_t> r((size_t)out * rs, 0u);
        for (int64_t o = 0; o < out; ++o) {
            uint32_t* dst = r.data() + (size_t)o * rs;
            std::memcpy(dst, packed.data + (size_t)o * cw * 4, (size_t)cw * 4);
            for (int64_t g = 0; g < ng; ++g) {
                std::memcpy(dst + cw + 2 * g, &sc[(size_t)o * ng + g], 4);
                std::memcpy(dst + cw + 2 * g + 1, &bi[(size_t)o * ng + g], 4);
            }
        }
        return r;
    }
    // Conv weight as [out][k][in] from HF [out,in,k] or MLX [out,k,in].
    std::vector<float> conv(const std::string& k, int out, int in, int ks) const {
        if (hf) {
            std::vector<float> w = f32(k, {out, in, ks});
            std::vector<float> r((size_t)out * in * ks);
            for (int o = 0; o < out; ++o)
                for (int i = 0; i < in; ++i)
                    for (int t = 0; t < ks; ++t)
                        r[((size_t)o * ks + t) * in + i] = w[((size_t)o * in + i) * ks + t];
            return r;
        }
        return f32(k, {out, ks, in});
    }
};

void append(std::vector<float>& dst, const std::vector<float>& src) {
    dst.insert(dst.end(), src.begin(), src.end());
}

}  // namespace

// ------------------------------------------------------------------ model

Model::~Model() {
    enc_lanes.clear();
    if (lanes_fork) cudaEventDestroy(lanes_fork);
    if (stream) {
        cudaSetDevice(device);
        cudaStreamSynchronize(stream);
    }
    // released by the driver once the last block allocated from it is freed
    if (stream_pool) cudaMemPoolDestroy(stream_pool);
    for (auto* b : owned) delete b;
    for (auto& e : ev)
        if (e) cudaEventDestroy(e);
    if (stream) cudaStreamDestroy(stream);
}

cudaMemPool_t Model::streams_pool() {
    if (!stream_pool) {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        MSB_CUDA(cudaMemPoolCreate(&stream_pool, &props));
        uint64_t keep = UINT64_MAX;
        MSB_CUDA(cudaMemPoolSetAttribute(stream_pool, cudaMemPoolAttrReleaseThreshold, &keep));
    }
    return stream_pool;
}

const uint32_t* Model::upload_words(const std::vector<uint32_t>& v) {
    DevBuf* b = new DevBuf();
    owned.push_back(b);
    b->ensure(std::max<size_t>(16, v.size() * sizeof(uint32_t)));
    MSB_CUDA(cudaMemcpy(b->p, v.data(), v.size() * sizeof(uint32_t), cudaMemcpyHostToDevice));
    return reinterpret_cast<const uint32_t*>(b->p);
}

float* Model::upload(const std::vector<float>& v) {
    DevBuf* b = new DevBuf();
    owned.push_back(b);
    b->ensure(std::max<size_t>(16, v.size() * sizeof(float)));
    MSB_CUDA(cudaMemcpy(b->p, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
    return b->as<float>();
}

void throw_device_status(unsigned code, const char* what) {
    const std::string w(what);
    switch (code) {
        case DEV_OK: return;
        case DEV_BARRIER_TIMEOUT: throw MsError(MS_ERR_TIMEOUT, w + ": grid exchange timed out");
        case DEV_WAIT_TIMEOUT: throw MsError(MS_ERR_TIMEOUT, w + ": a pipeline wait timed out");
        case DEV_BAD_TOKEN: throw MsError(MS_ERR_INVALID_ARG, w + ": token id out of range");
        default: throw MsError(MS_ERR_CUDA, w + ": device status " + std::to_string(code));
    }
}

void Model::ensure_rope(int positions) {
    if (positions <= rope_cap) return;
    const int nd = cfg.rotary_ndims(), half = nd / 2;
    const int cap = std::max(positions, 4096);
    std::vector<float> c((size_t)cap * std::max(half, 1)), s(c.size());
    for (int p = 0; p < cap; ++p)
        for (int i = 0; i < half; ++i) {
            const double inv = std::pow(cfg.rope_theta, -2.0 * i / (double)nd);
            const double a = (double)p * inv;
            c[(size_t)p * half + i] = (float)std::cos(a);
            s[(size_t)p * half + i] = (float)std::sin(a);
        }
    MSB_CUDA(cudaStreamSynchronize(stream));
    rope_cos.ensure(c.size() * 4);
    rope_sin.ensure(s.size() * 4);
    MSB_CUDA(cudaMemcpy(rope_cos.p, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
    MSB_CUDA(cudaMemcpy(rope_sin.p, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
    rope_cap = cap;
}

static void validate(const Config& c) {
    auto bad = [](const std::string& m) { throw MsError(MS_ERR_UNSUPPORTED, m); };
    if (c.quantized && !(c.q_bits == 2 || c.q_bits == 4 || c.q_bits == 8))
        bad("quantized checkpoints need bits 2, 4 or 8");
    if (c.quantized && (c.q_group < 8 || c.q_group % 8)) bad("quantization group_size must be a multiple of 8");
    if (c.hidden % 4 || c.e_hidden % 4 || c.inter % 4 || c.e_inter % 4)
        bad("hidden/intermediate sizes must be multiples of 4");
    if (c.head_dim % 4 || c.e_head_dim % 4 || c.head_dim > 64 || c.e_head_dim > 128)
        bad("head_dim must be a multiple of 4 (decoder <= 64, encoder <= 128)");
    if (c.heads % c.kv_heads || c.e_heads % c.e_kv_heads) bad("heads must be a multiple of kv heads");
    if (!decode_b1_supports_head_dim(c.head_dim)) bad("decoder head_dim must be 32, 40, 48 or 64");
    if (c.heads > 16) bad("at most 16 decoder heads");
    if (c.hidden > 1024 || c.e_hidden > 1024) bad("hidden size above 1024");
    if (c.frame_len() <= 0 || c.frame_len() > 128) bad("frame length must be in [1, 128]");
    if (c.layers <= 0 || c.e_layers <= 0 || c.vocab <= 0) bad("empty model");
    for (auto& w : c.windows)
        if (w.first < 1 || w.second < 0) bad("sliding windows need left >= 1 and right >= 0");
    if (c.enc_hidden_size != c.e_hidden) bad("encoder_hidden_size must equal the encoder width");
}

Model* load_model(const std::string& dir, const ms_options& o) {
    std::unique_ptr<Model> m(new Model());
    m->opts = o;
    m->device = o.device;
    m->kv_f16 = o.kv_dtype == MS_KV_F16;
    int ndev = 0;
    MSB_CUDA(cudaGetDeviceCount(&ndev));
    if (o.device < 0 || o.device >= ndev) throw MsError(MS_ERR_INVALID_ARG, "bad device ordinal");
    MSB_CUDA(cudaSetDevice(o.device));
    cudaDeviceProp prop;
    MSB_CUDA(cudaGetDeviceProperties(&prop, o.device));
    if (prop.major != 10) throw MsError(MS_ERR_UNSUPPORTED, "this library targets sm_100a (B200)");
    m->num_sms = prop.multiProcessorCount;
    m->cfg = Config::from_json_file(dir + "/config.json");
    validate(m->cfg);
    MSB_CUDA(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    for (auto& e : m->ev) MSB_CUDA(cudaEventCreate(&e));

    WeightSource ws;
    if (m->cfg.quantized) {
        ws.q_group = m->cfg.q_group;
        ws.q_bits = m->cfg.q_bits;
    }
    ws.load(find_weights(dir));
    {
        // bf16 tensor-core encoder for batches: bf16 / f16 checkpoints (MS_W_AUTO) or on request
        const std::string k = "encoder.layers.0.mlp.fc1.weight";
        const std::string dt = ws.has(k) ? ws.need_any(k).dtype : "";
        m->enc_bf16 = o.weight_dtype == MS_W_BF16 ||
                      (o.weight_dtype == MS_W_AUTO && (dt == "BF16" || dt == "F16"));
    }
    const Config& c = m->cfg;
    const int ed = c.e_hidden, d = c.hidden, fl = c.frame_len();
    const int eHD = c.e_heads * c.e_head_dim, eKVD = c.e_kv_heads * c.e_head_dim;
    const int HD = c.heads * c.head_dim, KVD = c.kv_heads * c.head_dim;

    // log_k is a scalar; writers store it as shape [] or [1]
    m->log_k = m->upload(ws.has("encoder.embedder.comp.log_k") &&
                                 ws.need_any("encoder.embedder.comp.log_k").numel() == 1
                             ? to_f32(ws.need_any("encoder.embedder.comp.log_k"))
                             : ws.f32("encoder.embedder.comp.log_k", {}));
    m->lin_w = m->upload(ws.f32("encoder.embedder.linear.weight", {ed, fl}));
    m->conv1_w = m->upload(ws.conv("encoder.embedder.conv1.weight", 2 * ed, ed, 5));
    m->conv1_b = m->upload(ws.f32("encoder.embedder.conv1.bias", {2 * ed}));
    m->conv2_w = m->upload(ws.conv("encoder.embedder.conv2.weight", ed, 2 * ed, 5));
    m->conv2_b = m->upload(ws.f32("encoder.embedder.conv2.bias", {ed}));
    for (int i = 0; i < c.e_layers; ++i) {
        const std::string p = "encoder.layers." + std::to_string(i) + ".";
        EncLayer L{};
        std::vector<float> qkv = ws.f32(p + "self_attn.q_proj.weight", {eHD, ed});
        append(qkv, ws.f32(p + "self_attn.k_proj.weight", {eKVD, ed}));
        append(qkv, ws.f32(p + "self_attn.v_proj.weight", {eKVD, ed}));
        L.wqkv = m->upload(qkv);
        L.wo = m->upload(ws.f32(p + "self_attn.o_proj.weight", {ed, eHD}));
        L.w1 = m->upload(ws.f32(p + "mlp.fc1.weight", {c.e_inter, ed}));
        L.b1 = m->upload(ws.f32(p + "mlp.fc1.bias", {c.e_inter}));
        L.w2 = m->upload(ws.f32(p + "mlp.fc2.weight", {ed, c.e_inter}));
        L.b2 = m->upload(ws.f32(p + "mlp.fc2.bias", {ed}));
        L.ln_in = m->upload(ws.f32(p + "input_layernorm.weight", {ed}));
        L.ln_post = m->upload(ws.f32(p + "post_attention_layernorm.weight", {ed}));
        m->enc.push_back(L);
    }
    m->enc_final = m->upload(ws.f32("encoder.final_norm.weight", {ed}));
    m->embed = m->upload(ws.f32("decoder.embed_tokens.weight", {c.vocab, d}));
    m->pos_emb = m->upload(ws.f32("decoder.pos_emb.weight", {c.max_pos, ed}));
    if (ed != d) m->proj = m->upload(ws.f32("decoder.proj.weight", {d, ed}));
    // Quantized checkpoints: unless fp32 weights or the single-grid kernel are asked for, the
    // clustered batch-1 kernel can stream the rows of d inputs it splits by rows (q|k|v, cross
    // q, fc1, and an untied LM head) as the checkpoint's codes with their scales and biases
    // instead of fp32 rows (ms_options.quant_stream).
    static const char* const kRowKeys[] = {"self_attn.q_proj.weight", "self_attn.k_proj.weight",
                                           "self_attn.v_proj.weight", "encoder_attn.q_proj.weight",
                                           "mlp.fc1.weight"};
    if (o.quant_stream < MS_QSTREAM_AUTO || o.quant_stream > MS_QSTREAM_NONE)
        throw MsError(MS_ERR_INVALID_ARG, "bad quant_stream");
    if (c.quantized && o.weight_dtype != MS_W_F32 && o.decode_kernel != MS_DECODE_GRID &&
        o.quant_stream != MS_QSTREAM_NONE && cluster_quant_ok(d, c.q_bits, c.q_group)) {
        // AUTO streams the LM head only: on the tiny model at batch 1 that measured fastest for
        // 2, 4 and 8 bits (the small per-layer row blocks gain less from fewer bytes than their
        // in-kernel dequantization costs)
        bool all = o.quant_stream == MS_QSTREAM_ALL;
        for (int i = 0; i < c.layers; ++i)
            for (const char* k : kRowKeys) all = all && ws.is_quantized("decoder.layers." + std::to_string(i) + "." + k);
        m->cl_qbits = all ? c.q_bits : 0;
        m->cl_lm_qbits = !c.tie && ws.is_quantized("proj_out.weight") ? c.q_bits : 0;
    }
    auto records = [&](const std::string& p, std::initializer_list<std::pair<const char*, int>> parts) {
        std::vector<uint32_t> r;
        for (const auto& kp : parts) {
            const std::vector<uint32_t> x = ws.quant_records(p + kp.first, kp.second, d);
            r.insert(r.end(), x.begin(), x.end());
        }
        return m->upload_words(r);
    };
    std::vector<float> crossw;
    for (int i = 0; i < c.layers; ++i) {
        const std::string p = "decoder.layers." + std::to_string(i) + ".";
        DecodeLayerW L{};
        if (m->cl_qbits) {
            L.qkv_q = records(p, {{kRowKeys[0], HD}, {kRowKeys[1], KVD}, {kRowKeys[2], KVD}});
            L.cq_q = records(p, {{kRowKeys[3], HD}});
            L.w1_q = records(p, {{kRowKeys[4], 2 * c.inter}});
        }
        std::vector<float> qkv = ws.f32(p + "self_attn.q_proj.weight", {HD, d});
        append(qkv, ws.f32(p + "self_attn.k_proj.weight", {KVD, d}));
        append(qkv, ws.f32(p + "self_attn.v_proj.weight", {KVD, d}));
        L.wqkv = m->upload(qkv);
        L.wo = m->upload(ws.f32(p + "self_attn.o_proj.weight", {d, HD}));
        L.wcq = m->upload(ws.f32(p + "encoder_attn.q_proj.weight", {HD, d}));
        L.wco = m->upload(ws.f32(p + "encoder_attn.o_proj.weight", {d, HD}));
        append(crossw, ws.f32(p + "encoder_attn.k_proj.weight", {KVD, d}));
        append(crossw, ws.f32(p + "encoder_attn.v_proj.weight", {KVD, d}));
        L.w1 = m->upload(ws.f32(p + "mlp.fc1.weight", {2 * c.inter, d}));
        L.b1 = m->upload(ws.f32(p + "mlp.fc1.bias", {2 * c.inter}));
        L.w2 = m->upload(ws.f32(p + "mlp.fc2.weight", {d, c.inter}));
        L.b2 = m->upload(ws.f32(p + "mlp.fc2.bias", {d}));
        L.ln1 = m->upload(ws.f32(p + "input_layernorm.weight", {d}));
        L.ln2 = m->upload(ws.f32(p + "post_attention_layernorm.weight", {d}));
        L.ln3 = m->upload(ws.f32(p + "final_layernorm.weight", {d}));
        m->dec.push_back(L);
    }
    m->cross_w = m->upload(crossw);
    m->dec_norm = m->upload(ws.f32("decoder.norm.weight", {d}));
    m->lm_head = c.tie ? m->embed : m->upload(ws.f32("proj_out.weight", {c.vocab, d}));
    if (m->cl_lm_qbits) m->lm_q = records("", {{"proj_out.weight", c.vocab}});
    m->dec_layers_buf.ensure(sizeof(DecodeLayerW) * m->dec.size());
    MSB_CUDA(cudaMemcpy(m->dec_layers_buf.p, m->dec.data(), sizeof(DecodeLayerW) * m->dec.size(),
                        cudaMemcpyHostToDevice));
    m->dec_dev = m->dec_layers_buf.as<DecodeLayerW>();
    m->ensure_rope(4096);
    noalloc_prepare(o.device, c.head_dim);
    MSB_CUDA(cudaDeviceSynchronize());
    return m.release();
}

// ------------------------------------------------------------------ encode

EncBufs Model::own_enc_bufs() {
    return {&ws.feat1p, &ws.feat2p, &ws.x, &ws.h, &ws.qkv, &ws.attn, &ws.f, &ws.memory, &ws.memproj};
}

const float* Model::memory_ptr() const { return proj ? ws.memproj.as<float>() : ws.memory.as<float>(); }

const float* Model::memory_of(const EncBufs& b) const {
    return proj ? b.memproj->as<float>() : b.memory->as<float>();
}

void Model::encoder_layers(float* x, int T) { encoder_layers_on(own_enc_bufs(), x, T, stream); }

int Model::encode_device(const float* audio_dev, int64_t n_samples, int pos_offset) {
    return encode_into(own_enc_bufs(), audio_dev, n_samples, pos_offset, stream);
}

void Model::encoder_layers_on(const EncBufs& b, float* x, int T, cudaStream_t s) {
    const Config& c = cfg;
    const int ed = c.e_hidden, hd = c.e_head_dim;
    const int eHD = c.e_heads * hd, QKV = (c.e_heads + 2 * c.e_kv_heads) * hd;
    b.h->ensure((size_t)T * ed * 4);
    b.qkv->ensure((size_t)T * QKV * 4);
    b.attn->ensure((size_t)T * eHD * 4);
    b.f->ensure((size_t)T * c.e_inter * 4);
    float *h = b.h->as<float>(), *qkv = b.qkv->as<float>(), *attn = b.attn->as<float>(), *f = b.f->as<float>();
    const float scale = std::pow((float)hd, -0.5f);
    for (int i = 0; i < c.e_layers; ++i) {
        const EncLayer& L = enc[i];
        MSB_CUDA(launch_layernorm_rows(x, T, ed, L.ln_in, 1.0f, 1e-5f, nullptr, 0, h, s));
        GemmEpilogue e1;
        e1.out = qkv;
        e1.ldc = QKV;
        MSB_CUDA(launch_gemm_f32(h, ed, L.wqkv, ed, T, QKV, ed, e1, s));
        auto w = c.window(i);
        MSB_CUDA(launch_window_attention(qkv, T, c.e_heads, c.e_kv_heads, hd, w.first, w.second, scale, attn, s));
        GemmEpilogue e2;
        e2.out = x;
        e2.ldc = ed;
        e2.residual = x;
        e2.ldr = ed;
        MSB_CUDA(launch_gemm_f32(attn, eHD, L.wo, eHD, T, ed, eHD, e2, s));
        MSB_CUDA(launch_layernorm_rows(x, T, ed, L.ln_post, 1.0f, 1e-5f, nullptr, 0, h, s));
        GemmEpilogue e3;
        e3.out = f;
        e3.ldc = c.e_inter;
        e3.bias = L.b1;
        e3.act = ACT_GELU;
        MSB_CUDA(launch_gemm_f32(h, ed, L.w1, ed, T, c.e_inter, ed, e3, s));
        GemmEpilogue e4;
        e4.out = x;
        e4.ldc = ed;
        e4.bias = L.b2;
        e4.residual = x;
        e4.ldr = ed;
        MSB_CUDA(launch_gemm_f32(f, c.e_inter, L.w2, c.e_inter, T, ed, c.e_inter, e4, s));
    }
}

void Model::reserve_encoder(const EncBufs& b, int64_t max_samples) {
    const Config& c = cfg;
    const int ed = c.e_hidden;
    const int T1 = (int)(max_samples / c.frame_len());
    if (T1 <= 0) return;
    const int T2 = (T1 - 1) / 2 + 1, T3 = (T2 - 1) / 2 + 1;
    const int QKV = (c.e_heads + 2 * c.e_kv_heads) * c.e_head_dim;
    b.feat1p->ensure((size_t)(4 + T1) * ed * 4);
    b.feat2p->ensure((size_t)(4 + T2) * 2 * ed * 4);
    b.x->ensure((size_t)T3 * ed * 4);
    b.memory->ensure((size_t)T3 * ed * 4);
    b.h->ensure((size_t)T3 * ed * 4);
    b.qkv->ensure((size_t)T3 * QKV * 4);
    b.attn->ensure((size_t)T3 * c.e_heads * c.e_head_dim * 4);
    b.f->ensure((size_t)T3 * c.e_inter * 4);
    if (proj) b.memproj->ensure((size_t)T3 * c.hidden * 4);
}

int Model::encode_into(const EncBufs& b, const float* audio_dev, int64_t n_samples, int pos_offset,
                       cudaStream_t s) {
    const Config& c = cfg;
    const int fl = c.frame_len(), ed = c.e_hidden;
    const int T1 = (int)(n_samples / fl);
    if (T1 <= 0) return 0;
    const int T2 = (T1 - 1) / 2 + 1, T3 = (T2 - 1) / 2 + 1;
    if (pos_offset + T3 > c.max_pos)
        throw MsError(MS_ERR_INVALID_ARG, "audio longer than the positional table (" +
                                              std::to_string(c.max_pos) + " frames)");
    b.feat1p->ensure((size_t)(4 + T1) * ed * 4);
    b.feat2p->ensure((size_t)(4 + T2) * 2 * ed * 4);
    b.x->ensure((size_t)T3 * ed * 4);
    b.memory->ensure((size_t)T3 * ed * 4);
    float* f1 = b.feat1p->as<float>();
    float* f2 = b.feat2p->as<float>();
    float* x = b.x->as<float>();
    MSB_CUDA(cudaMemsetAsync(f1, 0, (size_t)4 * ed * 4, s));
    MSB_CUDA(cudaMemsetAsync(f2, 0, (size_t)4 * 2 * ed * 4, s));
    MSB_CUDA(launch_frame_features(audio_dev, T1, fl, log_k, lin_w, ed, f1 + 4 * ed, ed, s));
    // causal conv1 (k5 s2, left pad 4) as a GEMM over strided rows of the padded buffer
    GemmEpilogue c1;
    c1.bias = conv1_b;
    c1.act = ACT_SILU;
    c1.out = f2 + 4 * 2 * ed;
    c1.ldc = 2 * ed;
    MSB_CUDA(launch_gemm_f32(f1, 2 * ed, conv1_w, 5 * ed, T2, 2 * ed, 5 * ed, c1, s));
    GemmEpilogue c2;
    c2.bias = conv2_b;
    c2.out = x;
    c2.ldc = ed;
    MSB_CUDA(launch_gemm_f32(f2, 4 * ed, conv2_w, 10 * ed, T3, ed, 10 * ed, c2, s));
    encoder_layers_on(b, x, T3, s);
    MSB_CUDA(launch_layernorm_rows(x, T3, ed, enc_final, 1.0f, 1e-5f, pos_emb, pos_offset, b.memory->as<float>(), s));
    if (proj) {
        b.memproj->ensure((size_t)T3 * c.hidden * 4);
        GemmEpilogue e;
        e.out = b.memproj->as<float>();
        e.ldc = c.hidden;
        MSB_CUDA(launch_gemm_f32(b.memory->as<float>(), ed, proj, ed, T3, c.hidden, ed, e, s));
    }
    return T3;
}

// ------------------------------------------------------------------ decode

void Model::ensure_decode(int m_cap, int t_cap, bool want_logits, int V) {  // m_cap: memory rows
    const Config& c = cfg;
    const int hd = c.head_dim, KVH = c.kv_heads, L = c.layers, d = c.hidden, H = c.heads;
    const int HD = H * hd;
    if (t_cap > ws.t_cap) {
        const size_t n = (size_t)L * KVH * t_cap * hd;
        ws.self_k.ensure(n * 4);
        ws.self_v.ensure(n * 4);
        ws.ids.ensure((size_t)t_cap * 4);
        ws.t_cap = t_cap;
    }
    if (want_logits) ws.logits.ensure((size_t)t_cap * V * 4);
    ws.dx.ensure((size_t)2 * d * 4);
    ws.dq.ensure((size_t)HD * 4);
    ws.dqc.ensure((size_t)HD * 4);
    ws.dkvnew.ensure((size_t)2 * KVH * hd * 4);
    ws.dps.ensure((size_t)H * d * 4);
    ws.dpc.ensure((size_t)H * d * 4);
    ws.dspart.ensure(decode_b1_spart_floats(H, hd, ws.t_cap) * 4);
    ws.dpart.ensure(decode_b1_cpart_floats(H, hd, m_cap, num_sms) * 4);
    ws.dg.ensure((size_t)c.inter * 4);
    ws.amax_v.ensure(num_sms * 4);
    ws.amax_i.ensure(num_sms * 4);
    ws.flags.ensure(64);
}

void Model::ensure_cross_ws(int m_cap) {
    if (m_cap <= ws.m_cap) return;
    const Config& c = cfg;
    const size_t n = (size_t)c.layers * 2 * c.kv_heads * m_cap * c.head_dim;
    ws.cross32.ensure(n * 4);
    ws.cross16.ensure(n * 2);
    ws.m_cap = m_cap;
}

void Model::cross_kv(const float* memory, int frames, int row0) {
    ensure_cross_ws(row0 + frames);
    cross_kv_into(memory, frames, row0, ws.cross32.as<float>(), kv_f16 ? ws.cross16.p : nullptr, ws.m_cap);
}

EncLane::~EncLane() {
    if (stream) cudaStreamDestroy(stream);
    if (done) cudaEventDestroy(done);
}

EncLane& Model::enc_lane(int k) {
    while ((int)enc_lanes.size() <= k) {
        auto l = std::make_unique<EncLane>();
        MSB_CUDA(cudaStreamCreateWithFlags(&l->stream, cudaStreamNonBlocking));
        MSB_CUDA(cudaEventCreateWithFlags(&l->done, cudaEventDisableTiming));
        enc_lanes.push_back(std::move(l));
    }
    return *enc_lanes[k];
}

void Model::fork_lanes(int k) {
    if (!lanes_fork) MSB_CUDA(cudaEventCreateWithFlags(&lanes_fork, cudaEventDisableTiming));
    MSB_CUDA(cudaEventRecord(lanes_fork, stream));
    for (int i = 0; i < k; ++i) MSB_CUDA(cudaStreamWaitEvent(enc_lane(i).stream, lanes_fork, 0));
}

void Model::join_lanes(int k) {
    for (int i = 0; i < k; ++i) {
        EncLane& l = enc_lane(i);
        MSB_CUDA(cudaEventRecord(l.done, l.stream));
        MSB_CUDA(cudaStreamWaitEvent(stream, l.done, 0));
    }
}

void Model::cross_kv_into(const float* memory, int frames, int row0, float* out32, void* out16, int m_cap,
                          cudaStream_t s) {
    if (frames <= 0) return;
    const Config& c = cfg;
    GemmEpilogue e;
    e.kv_scatter = 1;
    e.kv_out32 = out32;
    e.kv_out16 = out16;
    e.kv_heads = c.kv_heads;
    e.head_dim = c.head_dim;
    e.frame_cap = m_cap;
    e.frame_offset = row0;
    const int N = c.layers * 2 * c.kv_heads * c.head_dim;
    MSB_CUDA(launch_gemm_f32(memory, c.hidden, cross_w, c.hidden, frames, N, c.hidden, e, s ? s : stream));
}

// Fraction of the clustered batch-1 kernel's streamed weight and cross K/V lines loaded L2
// evict_last: the per-token stream (~98 MB for the tiny model) is re-read every decoder call
// but does not stay resident as a whole, so a subset is kept and the rest streams through
// (measured +7% decode tokens/s at 0.5 over no hint; 1.0 loses it again).
constexpr float kL2Keep = 0.5f;

bool Model::prepare_cluster_decode() {
    if (cl_tried) return cl_ok;
    cl_tried = true;
    const Config& c = cfg;
    ClusterGeom g;
    if (!cluster_geom(c.hidden, c.heads, c.kv_heads, c.head_dim, c.inter, c.vocab, c.layers, 0, &g, cl_qbits,
                      cl_lm_qbits, c.q_group))
        return false;
    cl_packed.ensure((size_t)cluster_ctas(c.heads) * g.cta_floats * 4);
    g.part_words = (size_t)2 * c.heads * c.hidden + (size_t)2 * cluster_ctas(c.heads);
    cl_part.ensure(g.part_words * 8);
    MSB_CUDA(pack_cluster_weights(g, dec.data(), c.layers, lm_head, lm_q, dec_norm, c.hidden, c.heads, c.head_dim,
                                  c.inter, c.vocab, cl_packed.as<float>(), stream));
    g.packed = cl_packed.as<float>();
    g.part = cl_part.as<unsigned long long>();
    cl_geom = g;
    cl_ok = true;
    return true;
}

Model::DecodeResult Model::decode(const float* cross32, const void* cross_stored, int m_cap, int M,
                                  int n_steps, bool forced, const int* teacher_dev, bool logits, float temperature,
                                  unsigned seed, float* qc_trace) {
    const Config& c = cfg;
    ensure_rope(n_steps + 1);
    DecodeParams p{};
    p.d = c.hidden;
    p.H = c.heads;
    p.KVH = c.kv_heads;
    p.hd = c.head_dim;
    p.I = c.inter;
    p.V = c.vocab;
    p.L = c.layers;
    p.nd = c.rotary_ndims();
    p.scale = std::pow((float)c.head_dim, -0.5f);
    p.layers = dec_dev;
    p.final_ln = dec_norm;
    p.lm_head = lm_head;
    p.embed = embed;
    p.rope_cos = rope_cos.as<float>();
    p.rope_sin = rope_sin.as<float>();
    p.max_pos = rope_cap;
    p.self_k = ws.self_k.p;
    p.self_v = ws.self_v.p;
    p.t_cap = ws.t_cap;
    p.kv_f16 = kv_f16 ? 1 : 0;
    p.cross32 = cross32;
    p.cross_stored = cross_stored;
    p.m_cap = m_cap;
    p.M = M;
    p.xb = ws.dx.as<float>();
    p.qbuf = ws.dq.as<float>();
    p.qc = ws.dqc.as<float>();
    p.kvnew = ws.dkvnew.as<float>();
    p.x1 = ws.dps.as<float>();
    p.x2 = ws.dpc.as<float>();
    p.spart = ws.dspart.as<float>();
    p.cpart = ws.dpart.as<float>();
    p.gbuf = ws.dg.as<float>();
    p.amax_val = ws.amax_v.as<float>();
    p.amax_idx = ws.amax_i.as<int>();
    p.start_token = c.dec_start;
    p.n_steps = n_steps;
    p.forced = forced ? 1 : 0;
    p.inv_temp = temperature > 0.f ? 1.f / temperature : 0.f;
    p.seed = seed;
    p.teacher = teacher_dev;
    p.eos = c.eos;
    p.ids_out = ws.ids.as<int>();
    p.logits_out = logits ? ws.logits.as<float>() : nullptr;
    p.qc_trace = qc_trace;
    unsigned* flags = ws.flags.as<unsigned>();
    p.bar_count = flags;
    p.status = flags + 1;
    p.n_done = reinterpret_cast<int*>(flags + 2);
    p.hit_eos = reinterpret_cast<int*>(flags + 3);
    int trace_n = 0;
    if (trace_enabled) {
        trace_n = 2 + n_steps * (c.layers * 8 * 4 + 4);
        trace_buf.ensure((size_t)trace_n * 8);
        MSB_CUDA(cudaMemsetAsync(trace_buf.p, 0, (size_t)trace_n * 8, stream));
        p.trace = trace_buf.as<unsigned long long>();
        p.trace_cap = trace_n;
    }
    MSB_CUDA(cudaMemsetAsync(flags, 0, 16, stream));
    bool launched = false;
    int ran = MS_DECODE_GRID;
    const int want = opts.decode_kernel;
    if ((want == MS_DECODE_AUTO || want == MS_DECODE_CLUSTER) && prepare_cluster_decode()) {
        ClusterGeom g = cl_geom;
        ClusterGeom sized;
        if (cluster_geom(c.hidden, c.heads, c.kv_heads, c.head_dim, c.inter, c.vocab, c.layers, ws.t_cap, &sized,
                         cl_qbits, cl_lm_qbits, c.q_group)) {
            g.skv_keys = sized.skv_keys;
            g.l2_keep = kL2Keep;
            MSB_CUDA(cudaMemsetAsync(g.part, 0, g.part_words * 8, stream));  // no stale exchange word
            const cudaError_t e = launch_decode_cluster(p, g, stream);
            if (e == cudaSuccess) {
                launched = true;
                ran = MS_DECODE_CLUSTER;
            } else if (e == cudaErrorCooperativeLaunchTooLarge) {
                (void)cudaGetLastError();  // not all clusters fit
            } else {
                MSB_CUDA(e);
            }
        }
    }
    if (!launched) MSB_CUDA(launch_decode_b1(p, num_sms, stream));
    unsigned hf[4];
    MSB_CUDA(cudaMemcpyAsync(hf, flags, 16, cudaMemcpyDeviceToHost, stream));
    if (trace_n) {
        last_trace.resize(trace_n);
        MSB_CUDA(cudaMemcpyAsync(last_trace.data(), trace_buf.p, (size_t)trace_n * 8, cudaMemcpyDeviceToHost,
                                 stream));
    }
    MSB_CUDA(cudaStreamSynchronize(stream));
    throw_device_status(hf[1], "decode kernel");
    DecodeResult r;
    r.n_calls = (int)hf[2];
    r.hit_eos = hf[3] != 0;
    r.kernel = ran;
    return r;
}

}  // namespace msb
