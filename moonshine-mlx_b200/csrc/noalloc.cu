// Allocation-free greedy decode: ms_decode_memory_static.
//
// Some callers must not allocate device memory once they are running: a real-time audio
// callback cannot risk cudaMalloc/cudaFree (they can block and synchronise the whole
// device, which blows the callback's deadline), and hosts that run under a fixed,
// pre-reserved GPU memory budget are not allowed to grow it.  This entry point serves
// them.  It decodes from encoder memory rows the caller already holds in device memory
// and writes token ids into a device buffer the caller owns; everything else it needs
// (the cross-attention K/V of the memory rows, the self-attention K/V cache and the
// decode kernel's working buffers) lives in one file-scope device array of a fixed size.
//
// That array exists once per device for the lifetime of the process (each process has its
// own copy).  Model load does the one-time set-up on its device (noalloc_prepare): it looks
// up the array's device address, which loads this file's module and so reserves the array,
// and loads the kernels the call launches, so the call itself loads and reserves nothing.
// Every call reuses the array; two calls whose GPU work overlapped would race on it.  Calls
// through this library cannot overlap: a process-wide lock serialises them and each call
// waits for its own GPU work before it returns.
//
// The decode always runs the single-grid kernel (decode_b1_kernel), whose scratch the
// array holds.  ms_generate_device may pick the head-clustered kernel, which sums in a
// different order, so the two agree to rounding (identical ids except at near-ties).
#include <cmath>
#include <cstring>
#include <mutex>

#include "../../include/moonshine_b200.h"
#include <cuda_fp16.h>

#include "kernels/kernels.h"
#include "runtime/model.hpp"

namespace msb {
namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB per device
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
unsigned char* g_static_ptr[kMaxDevices] = {};

// Device address of the array on `device` (the current device), looked up once.
unsigned char* static_scratch(int device) {
    if (device < 0 || device >= kMaxDevices) throw MsError(MS_ERR_INVALID_ARG, "device ordinal out of range");
    if (!g_static_ptr[device]) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (e != cudaSuccess)
            throw MsError(MS_ERR_CUDA, std::string("cudaGetSymbolAddress(static scratch): ") + cudaGetErrorString(e));
        g_static_ptr[device] = reinterpret_cast<unsigned char*>(ptr);
    }
    return g_static_ptr[device];
}

// Bump allocator over the static array (256-byte aligned segments).
struct Carve {
    unsigned char* base;
    size_t used = 0;
    template <class T>
    T* take(size_t count) {
        const size_t off = (used + 255) & ~size_t(255);
        used = off + count * sizeof(T);
        return reinterpret_cast<T*>(base + off);
    }
};

}  // namespace

void noalloc_prepare(int device, int head_dim) {
    std::lock_guard<std::mutex> g(g_static_mu);
    static_scratch(device);
    MSB_CUDA(preload_decode_b1(head_dim));
    MSB_CUDA(preload_gemm_f32());
}

}  // namespace msb

using namespace msb;

extern "C" ms_status ms_decode_memory_static(ms_model* model, const float* memory_dev, int32_t frames,
                                             int32_t n_tokens, int32_t forced, int32_t* ids_dev,
                                             int32_t* n_out, int32_t* hit_eos) {
    try {
        set_last_error("");
        if (!model || !memory_dev || !ids_dev || !n_out || frames <= 0 || n_tokens <= 0)
            throw MsError(MS_ERR_INVALID_ARG, "model, memory, ids and n_out must be set; frames and tokens > 0");
        if (reinterpret_cast<uintptr_t>(memory_dev) & 15)
            throw MsError(MS_ERR_INVALID_ARG, "memory rows must be 16-byte aligned");
        Model& m = *reinterpret_cast<Model*>(model);
        const Config& c = m.cfg;
        std::lock_guard<std::mutex> g_model(m.mu);
        std::lock_guard<std::mutex> g_static(g_static_mu);
        MSB_CUDA(cudaSetDevice(m.device));
        if (n_tokens > m.rope_cap)
            throw MsError(MS_ERR_CAPACITY, "n_tokens above the model's position table");

        // Size every segment first (null base) and reject requests the array cannot hold.
        const int L = c.layers, KVH = c.kv_heads, hd = c.head_dim, H = c.heads, d = c.hidden;
        const int KVD = KVH * hd, HD = H * hd, G = m.num_sms;
        const bool f16 = m.kv_f16;
        const size_t kvsz = f16 ? 2 : 4;
        const size_t cross_n = (size_t)L * 2 * KVH * frames * hd;
        const size_t self_n = (size_t)L * KVH * n_tokens * hd;
        auto layout = [&](unsigned char* base, DecodeParams* p) -> size_t {
            Carve cv{base};
            float* cross32 = cv.take<float>(cross_n);
            void* cross16 = f16 ? (void*)cv.take<__half>(cross_n) : nullptr;
            void* sk = cv.take<unsigned char>(self_n * kvsz);
            void* sv = cv.take<unsigned char>(self_n * kvsz);
            float* xb = cv.take<float>(2 * (size_t)d);
            float* qb = cv.take<float>(HD);
            float* qc = cv.take<float>(HD);
            float* kvnew = cv.take<float>(2 * (size_t)KVD);
            float* x1 = cv.take<float>(d);
            float* x2 = cv.take<float>(d);
            float* spart = cv.take<float>(decode_b1_spart_floats(H, hd, n_tokens));
            float* cpart = cv.take<float>(decode_b1_cpart_floats(H, hd, frames, G));
            float* gbuf = cv.take<float>(c.inter);
            float* av = cv.take<float>(G);
            int* ai = cv.take<int>(G);
            unsigned* flags = cv.take<unsigned>(4);
            if (p) {
                p->cross32 = cross32;
                p->cross_stored = f16 ? cross16 : (const void*)cross32;
                p->self_k = sk;
                p->self_v = sv;
                p->xb = xb;
                p->qbuf = qb;
                p->qc = qc;
                p->kvnew = kvnew;
                p->x1 = x1;
                p->x2 = x2;
                p->spart = spart;
                p->cpart = cpart;
                p->gbuf = gbuf;
                p->amax_val = av;
                p->amax_idx = ai;
                p->bar_count = flags;
                p->status = flags + 1;
                p->n_done = reinterpret_cast<int*>(flags + 2);
                p->hit_eos = reinterpret_cast<int*>(flags + 3);
            }
            return cv.used;
        };
        const size_t need = layout(nullptr, nullptr);
        if (need > kStaticScratchBytes)
            throw MsError(MS_ERR_CAPACITY, "static decode scratch needs " + std::to_string(need) +
                                               " bytes for this model, frames and tokens; the limit is " +
                                               std::to_string(kStaticScratchBytes));

        unsigned char* base = m.device >= 0 && m.device < kMaxDevices ? g_static_ptr[m.device] : nullptr;
        if (!base) throw MsError(MS_ERR_CUDA, "static scratch was not set up by model load on this device");
        DecodeParams p{};
        layout(base, &p);
        p.d = d;
        p.H = H;
        p.KVH = KVH;
        p.hd = hd;
        p.I = c.inter;
        p.V = c.vocab;
        p.L = L;
        p.nd = c.rotary_ndims();
        p.scale = std::pow((float)hd, -0.5f);
        p.layers = m.dec_dev;
        p.final_ln = m.dec_norm;
        p.lm_head = m.lm_head;
        p.embed = m.embed;
        p.rope_cos = m.rope_cos.as<float>();
        p.rope_sin = m.rope_sin.as<float>();
        p.max_pos = m.rope_cap;
        p.t_cap = n_tokens;
        p.kv_f16 = f16 ? 1 : 0;
        p.m_cap = frames;
        p.M = frames;
        p.start_token = c.dec_start;
        p.n_steps = n_tokens;
        p.forced = forced ? 1 : 0;
        p.teacher = nullptr;
        p.eos = c.eos;
        p.ids_out = ids_dev;
        p.logits_out = nullptr;
        p.trace = nullptr;
        p.trace_cap = 0;

        // The array keeps the previous call's contents: the barrier counter and the status
        // words must start at zero.
        MSB_CUDA(cudaMemsetAsync(p.bar_count, 0, 4 * sizeof(unsigned), m.stream));
        m.cross_kv_into(memory_dev, frames, 0, const_cast<float*>(p.cross32),
                        f16 ? const_cast<void*>(p.cross_stored) : nullptr, frames);
        MSB_CUDA(launch_decode_b1(p, m.num_sms, m.stream));
        unsigned hf[4];
        MSB_CUDA(cudaMemcpyAsync(hf, p.bar_count, sizeof(hf), cudaMemcpyDeviceToHost, m.stream));
        MSB_CUDA(cudaStreamSynchronize(m.stream));
        throw_device_status(hf[1], "decode kernel");
        const int calls = (int)hf[2];
        *n_out = calls - (hf[3] ? 1 : 0);
        if (hit_eos) *hit_eos = hf[3] ? 1 : 0;
        return MS_OK;
    } catch (const MsError& e) {
        set_last_error(e.what());
        return e.status;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return MS_ERR_CUDA;
    }
}
