// Batched greedy decode: B utterances step in lockstep; every projection is one tcgen05 GEMM
// over all B rows (bf16 weights and GEMM inputs, fp32 accumulation and residual stream).
// Step 0 runs eagerly, the remaining steps replay one captured CUDA graph of the step.
#include "batch.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace msb {

namespace {
constexpr int kBnNarrow = 64;   // q|k|v and cross-q projections (more CTAs for small N)
constexpr int kBnWide = 128;
constexpr int kStatTile = kBnWide;  // residual statistics tiles: the N tiles of the ACCUM GEMMs

void make_b_map(CUtensorMap* map, const __nv_bfloat16* w, int N, int K, int bn) {
    if (!tc_make_map_2d(map, w, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, (uint32_t)bn))
        throw MsError(MS_ERR_CUDA, "cuTensorMapEncodeTiled failed for a weight matrix");
}

void make_a_map(CUtensorMap* map, const __nv_bfloat16* a, int rows, int K) {
    if (!tc_make_map_3d(map, a, (uint64_t)K, 1, (uint64_t)rows, (uint64_t)K * 2, (uint64_t)K * 2, 128))
        throw MsError(MS_ERR_CUDA, "cuTensorMapEncodeTiled failed for an activation matrix");
}
}  // namespace

BatchEngine::~BatchEngine() {
    for (auto* b : own) delete b;
}

// Encode every utterance into memory rows [off[b], off[b] + frames) of the batch memory.
// Utterance b runs on lane b % K; the model stream waits for all lanes at the end.
void BatchEngine::encode_all(const std::vector<const float*>& audio_dev, const std::vector<int64_t>& n_samples,
                             const std::vector<int>& off) {
    constexpr int kLanes = 8;
    const int B = (int)audio_dev.size();
    const int K = std::min(B, kLanes);
    const int64_t longest = *std::max_element(n_samples.begin(), n_samples.end());
    for (int k = 0; k < K; ++k) m.reserve_encoder(m.enc_lane(k).bufs(), longest);  // before any lane runs
    m.fork_lanes(K);
    const int hidden = m.cfg.hidden;
    for (int b = 0; b < B; ++b) {
        EncLane& l = m.enc_lane(b % K);
        const EncBufs eb = l.bufs();
        const int M = m.encode_into(eb, audio_dev[b], n_samples[b], 0, l.stream);
        if (M <= 0) throw MsError(MS_ERR_CUDA, "frame count mismatch");
        MSB_CUDA(cudaMemcpyAsync(memory.as<float>() + (size_t)off[b] * hidden, m.memory_of(eb),
                                 (size_t)M * hidden * 4, cudaMemcpyDeviceToDevice, l.stream));
    }
    m.join_lanes(K);
}

template <class T>
T* BatchEngine::alloc(size_t n) {
    DevBuf* b = new DevBuf();
    own.push_back(b);
    b->ensure(std::max<size_t>(n * sizeof(T), 256));
    return b->as<T>();
}

void BatchEngine::ensure_weights() {
    if (weights_ready) return;
    const Config& c = m.cfg;
    const int d = c.hidden, HD = c.heads * c.head_dim, KVD = c.kv_heads * c.head_dim, I = c.inter;
    cudaStream_t s = m.stream;
    // fp32 checkpoints keep fp32-level GEMM products (split): every weight and GEMM input as
    // a bf16 high plane plus a bf16 low plane; bf16 / f16 checkpoints, or bf16 on request,
    // use one bf16 plane
    // bf16 copy of src [rows, K] (rows interleaved value/gate when `il`), its weight map and,
    // when split, the low plane right behind it with its own map
    // With a LayerNorm weight `lnw` the rows are stored times lnw[k] (the LayerNorm folds into
    // the GEMM) and *csum gets each stored row's sum.
    auto weight = [&](const float* src, int rows, int K, int il, int bn, CUtensorMap* hi, CUtensorMap* lo,
                      const float* lnw = nullptr, float** csum = nullptr) {
        const size_t n = (size_t)rows * K;
        __nv_bfloat16* w = alloc<__nv_bfloat16>(split ? 2 * n : n);
        MSB_CUDA(launch_f32_to_bf16_rows(src, w, rows, K, il, s, split ? n : 0, lnw));
        make_b_map(hi, w, rows, K, bn);
        if (split) make_b_map(lo, w + n, rows, K, bn);
        if (csum) {
            *csum = alloc<float>((size_t)rows);
            MSB_CUDA(launch_bf16_row_sums(w, rows, K, split ? n : 0, *csum, s));
        }
        return w;
    };
    layers.resize(c.layers);
    for (int l = 0; l < c.layers; ++l) {
        const DecodeLayerW& W = m.dec[l];
        LayerB& B = layers[l];
        B.wqkv = weight(W.wqkv, HD + 2 * KVD, d, 0, kBnNarrow, &B.m_qkv, &B.m_qkv_lo, W.ln1, &B.cs_qkv);
        B.wo = weight(W.wo, d, HD, 0, kBnWide, &B.m_o, &B.m_o_lo);
        B.wcq = weight(W.wcq, HD, d, 0, kBnNarrow, &B.m_cq, &B.m_cq_lo, W.ln2, &B.cs_cq);
        B.wco = weight(W.wco, d, HD, 0, kBnWide, &B.m_co, &B.m_co_lo);
        B.w1i = weight(W.w1, 2 * I, d, I, kBnWide, &B.m_w1, &B.m_w1_lo, W.ln3, &B.cs_w1);
        B.w2 = weight(W.w2, d, I, 0, kBnWide, &B.m_w2, &B.m_w2_lo);
        B.b1i = alloc<float>((size_t)2 * I);
        MSB_CUDA(launch_interleave_f32(W.b1, B.b1i, 2 * I, I, s));
    }
    lm = weight(m.lm_head, c.vocab, d, 0, kBnWide, &m_lm, &m_lm_lo, m.dec_norm, &cs_lm);
    MSB_CUDA(cudaStreamSynchronize(s));
    weights_ready = true;
}

void BatchEngine::ensure_ws(int B, int T, int Mtot, int maxM) {
    const Config& c = m.cfg;
    const int d = c.hidden, HD = c.heads * c.head_dim, KVD = c.kv_heads * c.head_dim, I = c.inter;
    const size_t kvsz = m.kv_f16 ? 2 : 4;
    bool remap = false;
    const size_t P = split ? 2 : 1;  // bf16 planes of the GEMM inputs
    if (B > Bc) {
        Bc = B;
        remap = true;
        grow(x, (size_t)Bc * d * 4);
        grow(hb, (size_t)Bc * d * 2 * P);
        grow(attn, (size_t)Bc * HD * 2 * P);
        grow(g, (size_t)Bc * I * 2 * P);
        grow(q, (size_t)Bc * HD * 4);
        grow(qc, (size_t)Bc * HD * 4);
        grow(kvnew, (size_t)Bc * 2 * KVD * 4);
        grow(amax, (size_t)Bc * 8);
        grow(next_ids, (size_t)Bc * 4);
        grow(counts, (size_t)Bc * 4);
        grow(limits_d, (size_t)Bc * 4);
        grow(done, (size_t)Bc * 4);
        grow(hit, (size_t)Bc * 4);
        grow(frame_off, (size_t)Bc * 4);
        grow(frames, (size_t)Bc * 4);
        grow(lnst, (size_t)((d + kStatTile - 1) / kStatTile) * Bc * sizeof(float2));
    }
    // capacities grow by half again at least, so a workload that grows a little per call
    // (streams whose memories lengthen every chunk) reallocates rarely
    auto cap_for = [](int cur, int need) { return need <= cur ? cur : std::max(need, cur + cur / 2); };
    if (T > Tc || remap) {
        Tc = cap_for(Tc, T);
        grow(ids, (size_t)Bc * Tc * 4);
    }
    (void)kvsz;
    if (Mtot > Mc) {
        Mc = cap_for(Mc, Mtot);
        const size_t n = (size_t)c.layers * 2 * KVD * Mc;
        grow(cross32, n * 4);
        grow(cross16, n * 2);
        grow(memory, (size_t)Mc * d * 4);
    }
    if (maxM > Fc || remap) {
        Fc = cap_for(Fc, maxM);
        grow(part, cross_batch_part_floats(Bc, c.heads, c.head_dim, Fc) * 4);
    }
    grow(status, 16);
    grow(pos, 16);
    if (remap) {
        make_a_map(&a_hb, hb.as<__nv_bfloat16>(), Bc, d);
        make_a_map(&a_attn, attn.as<__nv_bfloat16>(), Bc, HD);
        make_a_map(&a_g, g.as<__nv_bfloat16>(), Bc, I);
        if (split) {
            make_a_map(&a_hb_lo, hb.as<__nv_bfloat16>() + (size_t)Bc * d, Bc, d);
            make_a_map(&a_attn_lo, attn.as<__nv_bfloat16>() + (size_t)Bc * HD, Bc, HD);
            make_a_map(&a_g_lo, g.as<__nv_bfloat16>() + (size_t)Bc * I, Bc, I);
        }
    }
}

// Self-attention K/V pages for this call: row b gets ceil(limits[b] / kKvPage) pages (the
// positions it can reach), numbered consecutively from 0; the pool grows to the largest call
// seen and every page returns to it when the call ends.  Table entries past a row's pages
// are -1 (rows that have reached their limit keep stepping in lockstep; their writes there
// are dropped).
void BatchEngine::assign_pages(int B, int T, const std::vector<int>& limits) {
    const Config& c = m.cfg;
    const int KVD = c.kv_heads * c.head_dim;
    table_stride = (T + kKvPage - 1) / kKvPage;
    std::vector<int> tab((size_t)B * table_stride, -1);
    int64_t next = 0;
    for (int b = 0; b < B; ++b) {
        const int need = (std::max(limits[b], 1) + kKvPage - 1) / kKvPage;
        for (int q = 0; q < need && q < table_stride; ++q) tab[(size_t)b * table_stride + q] = (int)next++;
    }
    const size_t page_bytes = (size_t)c.layers * 2 * KVD * kKvPage * 4;  // fp32-sized: the KV dtype may change
    grow(kvpool, (size_t)std::max<int64_t>(next, 1) * page_bytes);
    pages_used = next;
    pages_capacity = (int64_t)(kvpool.bytes / page_bytes);
    grow(ptable, tab.size() * 4);
    MSB_CUDA(cudaMemcpyAsync(ptable.p, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, m.stream));
    // the host vector goes away at return: the copy must have read it
    MSB_CUDA(cudaStreamSynchronize(m.stream));
}

void BatchEngine::gemm(const CUtensorMap& a, const CUtensorMap& b, TcGemmArgs& ga, int K, int bn,
                       const CUtensorMap* a_lo, const CUtensorMap* b_lo) {
    ga.taps = 1;
    ga.kb_per_tap = (K + 63) / 64;
    ga.k_per_tap = K;
    ga.status = status.as<unsigned>();
    // k-splits (one cluster per output tile, summed in split order) until the grid covers
    // the SMs; every split keeps at least one k-block
    const int tiles = ((ga.N + bn - 1) / bn) * ((ga.M + 127) / 128);
    int sp = std::max(1, std::min({TC_MAX_SPLITS, ga.kb_per_tap, m.num_sms / std::max(tiles, 1)}));
    const int per = (ga.kb_per_tap + sp - 1) / sp;
    ga.splits = (ga.kb_per_tap + per - 1) / per;
    MSB_CUDA(launch_gemm_tc_split(a, a_lo, b, b_lo, ga, bn, m.stream));
}

namespace {
// Programmatic dependent launches for the kernels of one decode step (each waits for its
// predecessor before reading its results; a weight GEMM prefetches its first weight tiles
// while the previous kernel finishes).
struct PdlScope {
    bool prev;
    PdlScope() : prev(pdl_launches()) { pdl_launches() = true; }
    ~PdlScope() { pdl_launches() = prev; }
};
}  // namespace

void BatchEngine::enqueue_step(int B, int max_frames, bool forced, bool first, float* logits) {
    PdlScope pdl;
    const Config& c = m.cfg;
    const int d = c.hidden, H = c.heads, KVH = c.kv_heads, hd = c.head_dim, I = c.inter;
    const int HD = H * hd, KVD = KVH * hd;
    const float scale = std::pow((float)hd, -0.5f);
    cudaStream_t s = m.stream;
    const int* posp = pos.as<int>();
    float* X = x.as<float>();
    // split operands: low planes of the GEMM inputs (lo_* element offsets) and their maps
    const size_t lo_hb = split ? (size_t)Bc * d : 0, lo_attn = split ? (size_t)Bc * HD : 0;
    const size_t lo_g = split ? (size_t)Bc * I : 0;
    const CUtensorMap* hb_lo = split ? &a_hb_lo : nullptr;
    const CUtensorMap* attn_lo = split ? &a_attn_lo : nullptr;
    const CUtensorMap* g_lo = split ? &a_g_lo : nullptr;
    auto wlo = [&](const CUtensorMap& mlo) { return split ? &mlo : nullptr; };
    // LayerNorms folded into their consumers: the GEMMs after LN1, LN2, LN3 and the final
    // norm read the residual's bf16 planes (hb) and the statistics of its rows (lnst), which
    // the embedding and every residual update (ACCUM GEMM) write
    const int ntiles = (d + kStatTile - 1) / kStatTile;
    float2* st = lnst.as<float2>();
    auto fold = [&](TcGemmArgs& ga, const float* csum) {
        ga.lnf.stats = st;
        ga.lnf.csum = csum;
        ga.lnf.ntiles = ntiles;
        ga.lnf.tile_n = kStatTile;
        ga.lnf.ld = Bc;
        ga.lnf.K = d;
    };
    auto update = [&](TcGemmArgs& ga) {
        ga.out_bf16 = hb.as<__nv_bfloat16>();
        ga.ldc_bf16 = d;
        ga.bf16_lo_off = lo_hb;
        ga.stats_out = st;
        ga.stats_ld = Bc;
    };
    MSB_CUDA(launch_embed_rows(next_ids.as<int>(), m.embed, d, B, c.vocab, X, status.as<unsigned>(), s,
                               hb.as<__nv_bfloat16>(), lo_hb, st, Bc, kStatTile));
    for (int l = 0; l < c.layers; ++l) {
        const DecodeLayerW& W = m.dec[l];
        LayerB& L = layers[l];
        PagedKv pk;
        pk.pool = kvpool.p;
        pk.table = ptable.as<int>();
        pk.table_stride = table_stride;
        pk.page = kKvPage;
        pk.page_elems = (long long)c.layers * 2 * KVD * kKvPage;
        pk.layer_off = (long long)l * 2 * KVD * kKvPage;
        pk.kv_f16 = m.kv_f16 ? 1 : 0;
        pk.reach = sa_reach;
        // self-attention block
        {
            TcGemmArgs ga;
            ga.M = B;
            ga.N = HD + 2 * KVD;
            ga.mode = TC_EPI_ROPE_KV;
            ga.rope.pos = posp;
            ga.rope.cos_t = m.rope_cos.as<float>();
            ga.rope.sin_t = m.rope_sin.as<float>();
            ga.rope.nd = c.rotary_ndims();
            ga.rope.hd = hd;
            ga.rope.H = H;
            ga.rope.KVH = KVH;
            ga.rope.q = q.as<float>();
            ga.rope.kv_new = kvnew.as<float>();
            ga.rope.kv = pk;
            fold(ga, L.cs_qkv);
            gemm(a_hb, L.m_qkv, ga, d, kBnNarrow, hb_lo, wlo(L.m_qkv_lo));
        }
        MSB_CUDA(launch_self_attn_batch(q.as<float>(), kvnew.as<float>(), pk, posp, B, H, KVH, hd, scale,
                                        attn.as<__nv_bfloat16>(), s, lo_attn));
        {
            TcGemmArgs ga;
            ga.M = B;
            ga.N = d;
            ga.mode = TC_EPI_ACCUM;
            ga.ep.out = X;
            ga.ep.ldc = d;
            update(ga);
            gemm(a_attn, L.m_o, ga, HD, kBnWide, attn_lo, wlo(L.m_o_lo));
        }
        // cross-attention block
        {
            TcGemmArgs ga;
            ga.M = B;
            ga.N = HD;
            ga.ep.out = qc.as<float>();
            ga.ep.ldc = HD;
            fold(ga, L.cs_cq);
            gemm(a_hb, L.m_cq, ga, d, kBnNarrow, hb_lo, wlo(L.m_cq_lo));
        }
        MSB_CUDA(launch_cross_attn_batch(qc.as<float>(), cross32.as<float>(), m.kv_f16 ? cross16.p : cross32.p,
                                         m.kv_f16 ? 1 : 0, posp, frame_off.as<int>(), frames.as<int>(), B, H, KVH,
                                         hd, Mc, l, max_frames, scale, part.as<float>(), attn.as<__nv_bfloat16>(),
                                         first ? 1 : 0, status.as<unsigned>(), s, lo_attn,
                                         xrows_on ? &xrows : nullptr));
        {
            TcGemmArgs ga;
            ga.M = B;
            ga.N = d;
            ga.mode = TC_EPI_ACCUM;
            ga.ep.out = X;
            ga.ep.ldc = d;
            update(ga);
            gemm(a_attn, L.m_co, ga, HD, kBnWide, attn_lo, wlo(L.m_co_lo));
        }
        // SwiGLU MLP
        {
            TcGemmArgs ga;
            ga.M = B;
            ga.N = 2 * I;
            ga.mode = TC_EPI_SWIGLU;
            ga.ep.bias = L.b1i;
            ga.out_bf16 = g.as<__nv_bfloat16>();
            ga.ldc_bf16 = I;
            ga.bf16_lo_off = lo_g;
            fold(ga, L.cs_w1);
            gemm(a_hb, L.m_w1, ga, d, kBnWide, hb_lo, wlo(L.m_w1_lo));
        }
        {
            TcGemmArgs ga;
            ga.M = B;
            ga.N = d;
            ga.mode = TC_EPI_ACCUM;
            ga.ep.out = X;
            ga.ep.ldc = d;
            ga.ep.bias = W.b2;
            update(ga);
            gemm(a_g, L.m_w2, ga, I, kBnWide, g_lo, wlo(L.m_w2_lo));
        }
    }
    {
        TcGemmArgs ga;
        ga.M = B;
        ga.N = c.vocab;
        ga.mode = TC_EPI_ARGMAX;
        ga.argmax = amax.as<unsigned long long>();
        ga.ep.out = logits;
        ga.ep.ldc = c.vocab;
        ga.inv_temp = inv_temp;
        ga.seed = seed;
        ga.step = pos.as<int>();
        fold(ga, cs_lm);
        gemm(a_hb, m_lm, ga, d, kBnWide, hb_lo, wlo(m_lm_lo));
    }
    MSB_CUDA(launch_step_finalize(amax.as<unsigned long long>(), B, pos.as<int>(), next_ids.as<int>(), ids.as<int>(),
                                  Tc, counts.as<int>(), limits_d.as<int>(), done.as<int>(), hit.as<int>(), c.eos,
                                  forced ? 1 : 0, s));
}

void BatchEngine::ensure_enc_weights() {
    if (enc_weights_ready) return;
    const Config& c = m.cfg;
    const int ed = c.e_hidden, hd = c.e_head_dim, EI = c.e_inter;
    const int eHD = c.e_heads * hd, QKV = (c.e_heads + 2 * c.e_kv_heads) * hd;
    const int NKV = c.layers * 2 * c.kv_heads * c.head_dim;
    cudaStream_t s = m.stream;
    auto weight = [&](const float* src, int rows, int K, CUtensorMap* hi, CUtensorMap* lo) {
        const size_t n = (size_t)rows * K;
        __nv_bfloat16* w = alloc<__nv_bfloat16>(esplit ? 2 * n : n);
        MSB_CUDA(launch_f32_to_bf16_rows(src, w, rows, K, 0, s, esplit ? n : 0));
        make_b_map(hi, w, rows, K, kBnWide);
        if (esplit) make_b_map(lo, w + n, rows, K, kBnWide);
        return w;
    };
    elin = weight(m.lin_w, ed, c.frame_len(), &m_lin, &m_lin_lo);
    econv1 = weight(m.conv1_w, 2 * ed, 5 * ed, &m_conv1, &m_conv1_lo);
    econv2 = weight(m.conv2_w, ed, 10 * ed, &m_conv2, &m_conv2_lo);
    elayers.resize(c.e_layers);
    for (int i = 0; i < c.e_layers; ++i) {
        const EncLayer& L = m.enc[i];
        EncLayerB& E = elayers[i];
        E.wqkv = weight(L.wqkv, QKV, ed, &E.m_qkv, &E.m_qkv_lo);
        E.wo = weight(L.wo, ed, eHD, &E.m_o, &E.m_o_lo);
        E.w1 = weight(L.w1, EI, ed, &E.m_w1, &E.m_w1_lo);
        E.w2 = weight(L.w2, ed, EI, &E.m_w2, &E.m_w2_lo);
    }
    ecross = weight(m.cross_w, NKV, c.hidden, &m_ecross, &m_ecross_lo);
    MSB_CUDA(cudaStreamSynchronize(s));
    enc_weights_ready = true;
}

// Encoder-layer scratch rows: the capacity grows by half again at least, so stream windows
// that lengthen a little every chunk reallocate (free + malloc, a device synchronisation)
// only now and then.
size_t BatchEngine::enc_rows_capacity(size_t rows3) {
    if (rows3 > erows_cap) erows_cap = std::max(rows3, erows_cap + erows_cap / 2);
    return erows_cap;
}

// Encoder layers l0 .. l1 - 1 (all by default; MoonshineLayers.swift:297-310) over
// X = ex [rows3, e_hidden] in segments of R3 rows; attention of segment s sees its first
// seg_len[s] rows only.  Uses eh, eqkv, eattn
// and ef (grown here) and the encoder weights (split operands for fp32 checkpoints).
void BatchEngine::encoder_layers_tc(size_t rows3, int R3, const int* seg_len, int l0, int l1) {
    const Config& c = m.cfg;
    const int ed = c.e_hidden, hd = c.e_head_dim, EI = c.e_inter;
    const int eHD = c.e_heads * hd, QKV = (c.e_heads + 2 * c.e_kv_heads) * hd;
    cudaStream_t s = m.stream;
    const size_t P = esplit ? 2 : 1;
    const size_t cap = enc_rows_capacity(rows3);  // low planes sit cap rows behind the high ones
    const size_t lo_h = esplit ? cap * ed : 0, lo_attn = esplit ? cap * eHD : 0, lo_f = esplit ? cap * EI : 0;
    grow(eh, cap * ed * 2 * P);
    grow(eqkv, cap * QKV * 4);
    grow(eattn, cap * eHD * 2 * P);
    grow(ef, cap * EI * 2 * P);
    float* X = ex.as<float>();
    auto amap = [&](CUtensorMap* hi, CUtensorMap* lo, const __nv_bfloat16* p, size_t rows, int K, size_t lo_off) {
        make_a_map(hi, p, (int)rows, K);
        if (esplit) make_a_map(lo, p + lo_off, (int)rows, K);
    };
    auto lo_of = [&](const CUtensorMap& mlo) { return esplit ? &mlo : nullptr; };
    CUtensorMap a_h, a_attn, a_f, a_h_lo, a_attn_lo, a_f_lo;
    amap(&a_h, &a_h_lo, eh.as<__nv_bfloat16>(), rows3, ed, lo_h);
    amap(&a_attn, &a_attn_lo, eattn.as<__nv_bfloat16>(), rows3, eHD, lo_attn);
    amap(&a_f, &a_f_lo, ef.as<__nv_bfloat16>(), rows3, EI, lo_f);
    const CUtensorMap* h_lo = esplit ? &a_h_lo : nullptr;
    const CUtensorMap* attn_lo = esplit ? &a_attn_lo : nullptr;
    const CUtensorMap* f_lo = esplit ? &a_f_lo : nullptr;
    const float scale = std::pow((float)hd, -0.5f);
    for (int i = l0; i < (l1 < 0 ? c.e_layers : l1); ++i) {
        const EncLayer& L = m.enc[i];
        const EncLayerB& E = elayers[i];
        MSB_CUDA(launch_ln_bf16(X, (int)rows3, ed, L.ln_in, eh.as<__nv_bfloat16>(), s, 1.0f, lo_h));
        {
            TcGemmArgs ga;
            ga.M = (int)rows3;
            ga.N = QKV;
            ga.ep.out = eqkv.as<float>();
            ga.ep.ldc = QKV;
            gemm(a_h, E.m_qkv, ga, ed, kBnWide, h_lo, lo_of(E.m_qkv_lo));
        }
        const auto w = c.window(i);
        MSB_CUDA(launch_window_attention(eqkv.as<float>(), (int)rows3, c.e_heads, c.e_kv_heads, hd, w.first, w.second,
                                         scale, nullptr, s, R3, seg_len, eattn.as<__nv_bfloat16>(), lo_attn));
        {
            TcGemmArgs ga;
            ga.M = (int)rows3;
            ga.N = ed;
            ga.ep.out = X;
            ga.ep.ldc = ed;
            ga.ep.residual = X;
            ga.ep.ldr = ed;
            gemm(a_attn, E.m_o, ga, eHD, kBnWide, attn_lo, lo_of(E.m_o_lo));
        }
        MSB_CUDA(launch_ln_bf16(X, (int)rows3, ed, L.ln_post, eh.as<__nv_bfloat16>(), s, 1.0f, lo_h));
        {
            TcGemmArgs ga;
            ga.M = (int)rows3;
            ga.N = EI;
            ga.ep.bias = L.b1;
            ga.ep.act = ACT_GELU;
            ga.out_bf16 = ef.as<__nv_bfloat16>();
            ga.ldc_bf16 = EI;
            ga.bf16_lo_off = lo_f;
            gemm(a_h, E.m_w1, ga, ed, kBnWide, h_lo, lo_of(E.m_w1_lo));
        }
        {
            TcGemmArgs ga;
            ga.M = (int)rows3;
            ga.N = ed;
            ga.ep.bias = L.b2;
            ga.ep.out = X;
            ga.ep.ldc = ed;
            ga.ep.residual = X;
            ga.ep.ldr = ed;
            gemm(a_f, E.m_w2, ga, EI, kBnWide, f_lo, lo_of(E.m_w2_lo));
        }
    }
}

bool BatchEngine::tc_encoder_fits() const {
    const Config& c = m.cfg;
    const int ed = c.e_hidden, fl = c.frame_len(), hd = c.e_head_dim;
    const int eHD = c.e_heads * hd;
    return !m.proj && ed == c.hidden && ed % 64 == 0 && eHD % 64 == 0 && c.e_inter % 64 == 0 && ed <= 1024 &&
           hd <= 128 && hd % 4 == 0 && fl % 8 == 0 && fl <= 128;
}

bool BatchEngine::encode_tc(const std::vector<const float*>& audio_dev, const std::vector<int64_t>& n_samples,
                            const std::vector<int>& off, const std::vector<int>& fr) {
    const Config& c = m.cfg;
    const int ed = c.e_hidden, fl = c.frame_len(), d = c.hidden;
    if (!tc_encoder_fits()) return false;
    const int B = (int)audio_dev.size();
    int T1max = 0;
    std::vector<int> T1(B);
    for (int b = 0; b < B; ++b) {
        T1[b] = (int)(n_samples[b] / fl);
        T1max = std::max(T1max, T1[b]);
    }
    // rows per utterance: R in the conv1 input (4 zero rows + frames), R/2 in the conv2 input
    // (4 zero rows + conv1 outputs), R/4 in the encoder layers
    const int T3max = *std::max_element(fr.begin(), fr.end());
    if (T3max > c.max_pos)
        throw MsError(MS_ERR_INVALID_ARG, "audio longer than the positional table (" + std::to_string(c.max_pos) +
                                              " frames)");
    const int R = (T1max + 9 + 3) / 4 * 4, R2 = R / 2, R3 = R / 4;
    const size_t rows1 = (size_t)B * R, rows2 = (size_t)B * R2 + 4, rows3 = (size_t)B * R3;
    ensure_enc_weights();
    cudaStream_t s = m.stream;
    // bf16 GEMM inputs hold a low plane right after the high one when split (lo_* elements on)
    const size_t P = esplit ? 2 : 1;
    const size_t lo_norm = esplit ? rows1 * fl : 0, lo_pad1 = esplit ? rows1 * ed : 0;
    const size_t lo_pad2 = esplit ? rows2 * 2 * ed : 0;
    const size_t lo_mem = esplit ? (size_t)Mc * d : 0;
    grow(enorm, rows1 * fl * 2 * P);
    grow(eaud, (size_t)B * sizeof(float*));
    grow(epad1, rows1 * ed * 2 * P);
    grow(epad2, rows2 * 2 * ed * 2 * P);
    grow(ex, enc_rows_capacity(rows3) * ed * 4);
    grow(emem16, (size_t)Mc * d * 2 * P);
    grow(eseg, (size_t)3 * B * 4);
    __nv_bfloat16* pad1 = epad1.as<__nv_bfloat16>();
    __nv_bfloat16* pad2 = epad2.as<__nv_bfloat16>();
    float* X = ex.as<float>();
    int* seg_len = eseg.as<int>();
    int* seg_off = seg_len + B;
    // A maps of a bf16 input [rows, K] at p: the high plane, and when split the low one
    auto amap = [&](CUtensorMap* hi, CUtensorMap* lo, const __nv_bfloat16* p, size_t rows, int K, size_t lo_off) {
        make_a_map(hi, p, (int)rows, K);
        if (esplit) make_a_map(lo, p + lo_off, (int)rows, K);
    };
    auto lo_of = [&](const CUtensorMap& mlo) { return esplit ? &mlo : nullptr; };
    {
        std::vector<int> host(2 * (size_t)B);
        for (int b = 0; b < B; ++b) {
            host[b] = fr[b];
            host[B + b] = off[b];
        }
        MSB_CUDA(cudaMemcpyAsync(seg_len, host.data(), host.size() * 4, cudaMemcpyHostToDevice, s));
    }
    // frontend: frames of utterance b at rows b*R + 4 + f, every other row zero (normalised
    // frames of zeros give SiLU(0) = 0 out of the Linear)
    {
        std::vector<int> t1(T1);
        int* t1_dev = seg_len + 2 * B;
        MSB_CUDA(cudaMemcpyAsync(t1_dev, t1.data(), (size_t)B * 4, cudaMemcpyHostToDevice, s));
        MSB_CUDA(cudaMemcpyAsync(eaud.p, audio_dev.data(), (size_t)B * sizeof(float*), cudaMemcpyHostToDevice, s));
        // the pointer array is read by the next kernel: keep the host copy alive until then
        MSB_CUDA(launch_frame_norm_rows(reinterpret_cast<const float* const*>(eaud.p), t1_dev, (int)rows1, R, fl,
                                        m.log_k, enorm.as<__nv_bfloat16>(), s, lo_norm));
        CUtensorMap a_norm, a_norm_lo;
        for (int pl = 0; pl < (int)P; ++pl) {
            if (!tc_make_map_3d(pl ? &a_norm_lo : &a_norm, enorm.as<__nv_bfloat16>() + (pl ? lo_norm : 0),
                                (uint64_t)fl, 1, (uint64_t)rows1, (uint64_t)fl * 2, (uint64_t)fl * 2, 128))
                throw MsError(MS_ERR_CUDA, "cuTensorMapEncodeTiled failed for the frames");
        }
        TcGemmArgs ga;
        ga.M = (int)rows1;
        ga.N = ed;
        ga.ep.act = ACT_SILU;
        ga.out_bf16 = pad1;
        ga.ldc_bf16 = ed;
        ga.bf16_lo_off = lo_pad1;
        gemm(a_norm, m_lin, ga, fl, kBnWide, esplit ? &a_norm_lo : nullptr, lo_of(m_lin_lo));
        MSB_CUDA(cudaStreamSynchronize(s));  // t1 and the pointer array were copied from host vectors
    }
    // causal stride-2 convs as 5-tap GEMMs: output row m reads input rows 2m + tap, i.e.
    // (y, z) = (tap & 1, m + tap / 2) of the input viewed as row pairs
    auto conv = [&](const __nv_bfloat16* in, size_t in_rows, int cin, size_t in_lo, const CUtensorMap& wmap,
                    const CUtensorMap& wmap_lo, int M, int N, TcGemmArgs& ga) {
        CUtensorMap amap, amap_lo;
        for (int pl = 0; pl < (int)P; ++pl)
            if (!tc_make_map_3d(pl ? &amap_lo : &amap, in + (pl ? in_lo : 0), (uint64_t)cin, 2,
                                (uint64_t)(in_rows / 2), (uint64_t)cin * 2, (uint64_t)cin * 4, 128))
                throw MsError(MS_ERR_CUDA, "cuTensorMapEncodeTiled failed for a conv input");
        ga.M = M;
        ga.N = N;
        ga.taps = 5;
        ga.kb_per_tap = cin / 64;
        ga.k_per_tap = cin;
        for (int t = 0; t < 5; ++t) {
            ga.tap_y[t] = t & 1;
            ga.tap_z[t] = t >> 1;
        }
        ga.mode = TC_EPI_STD;
        ga.status = status.as<unsigned>();
        MSB_CUDA(launch_gemm_tc_split(amap, esplit ? &amap_lo : nullptr, wmap, lo_of(wmap_lo), ga, kBnWide, s));
    };
    {
        TcGemmArgs ga;
        ga.ep.bias = m.conv1_b;
        ga.ep.act = ACT_SILU;
        ga.out_bf16 = pad2 + (size_t)4 * 2 * ed;  // utterance b's conv1 outputs at rows b*R2 + 4 + t
        ga.ldc_bf16 = 2 * ed;
        ga.bf16_lo_off = lo_pad2;
        conv(pad1, rows1, ed, lo_pad1, m_conv1, m_conv1_lo, B * R2, 2 * ed, ga);
    }
    // the 4 rows in front of every utterance took the previous one's tail outputs: back to zero
    for (int pl = 0; pl < (int)P; ++pl)
        MSB_CUDA(cudaMemset2DAsync(pad2 + (pl ? lo_pad2 : 0), (size_t)R2 * 2 * ed * 2, 0, (size_t)4 * 2 * ed * 2, B,
                                   s));
    {
        TcGemmArgs ga;
        ga.ep.bias = m.conv2_b;
        ga.ep.out = X;
        ga.ep.ldc = ed;
        conv(pad2, rows2, 2 * ed, lo_pad2, m_conv2, m_conv2_lo, B * R3, ed, ga);
    }
    // encoder layers over all B * R3 rows; attention stays inside each utterance's rows
    encoder_layers_tc(rows3, R3, seg_len);
    // prepareMemory: final norm + positions, gathered to the batch memory rows
    MSB_CUDA(launch_ln_gather_rows(X, (int)rows3, R3, ed, m.enc_final, 1.0f, 1e-5f, m.pos_emb, seg_len, seg_off,
                                   memory.as<float>(), emem16.as<__nv_bfloat16>(), s, lo_mem));
    // cross K/V of every memory row in one GEMM (scatter epilogue: fp32 copy + fp16 store)
    int Mtot = 0;
    for (int b = 0; b < B; ++b) Mtot = std::max(Mtot, off[b] + fr[b]);
    CUtensorMap a_mem, a_mem_lo;
    amap(&a_mem, &a_mem_lo, emem16.as<__nv_bfloat16>(), Mtot, d, lo_mem);
    TcGemmArgs ga;
    ga.M = Mtot;
    ga.N = c.layers * 2 * c.kv_heads * c.head_dim;
    ga.ep.kv_scatter = 1;
    ga.ep.kv_out32 = cross32.as<float>();
    ga.ep.kv_out16 = m.kv_f16 ? cross16.p : nullptr;
    ga.ep.kv_heads = c.kv_heads;
    ga.ep.head_dim = c.head_dim;
    ga.ep.frame_cap = Mc;
    ga.ep.frame_offset = 0;
    gemm(a_mem, m_ecross, ga, d, kBnWide, esplit ? &a_mem_lo : nullptr, lo_of(m_ecross_lo));
    return true;
}

int BatchEngine::encode_one(const float* audio_dev, int64_t n_samples, const float** cross32_out,
                            const void** cross16_out, int* m_cap) {
    const Config& c = m.cfg;
    const int fl = c.frame_len();
    const int T1 = (int)(n_samples / fl);
    const int T2 = T1 > 0 ? (T1 - 1) / 2 + 1 : 0;
    const int M = T2 > 0 ? (T2 - 1) / 2 + 1 : 0;
    if (M <= 0) return -1;
    ensure_ws(1, 1, M, M);
    MSB_CUDA(cudaMemsetAsync(status.p, 0, 16, m.stream));  // the split-K epilogues read it
    if (!encode_tc({audio_dev}, {n_samples}, {0}, {M})) return -1;
    unsigned st_word = 0;
    MSB_CUDA(cudaMemcpyAsync(&st_word, status.p, 4, cudaMemcpyDeviceToHost, m.stream));
    MSB_CUDA(cudaStreamSynchronize(m.stream));
    throw_device_status(st_word, "tensor-core encoder");
    *cross32_out = cross32.as<float>();
    *cross16_out = m.kv_f16 ? cross16.p : cross32.p;
    *m_cap = Mc;
    return M;
}

bool BatchEngine::encode_windows(const std::vector<StreamWindow>& w) {
    if (w.empty()) return true;
    if (!tc_encoder_fits()) return false;
    const Config& c = m.cfg;
    const int ed = c.e_hidden, B = (int)w.size();
    int R3 = 1, max_new = 1;
    for (const auto& x : w) {
        R3 = std::max(R3, x.T);
        max_new = std::max(max_new, x.nnew);
    }
    const size_t rows3 = (size_t)B * R3;
    ensure_enc_weights();
    cudaStream_t s = m.stream;
    grow(ex, enc_rows_capacity(rows3) * ed * 4);
    grow(status, 16);
    // tables: src[B], dst[B] pointers, then T, off, cnt, pos
    std::vector<unsigned char> tab((size_t)B * (2 * sizeof(void*) + 4 * sizeof(int)));
    const void** srcp = reinterpret_cast<const void**>(tab.data());
    void** dstp = reinterpret_cast<void**>(tab.data() + (size_t)B * sizeof(void*));
    int* ints = reinterpret_cast<int*>(tab.data() + (size_t)2 * B * sizeof(void*));
    for (int b = 0; b < B; ++b) {
        srcp[b] = w[b].feat;
        dstp[b] = w[b].dst;
        ints[b] = w[b].T;
        ints[B + b] = w[b].off;
        ints[2 * B + b] = w[b].nnew;
        ints[3 * B + b] = w[b].pos;
    }
    grow(wtab, tab.size());
    MSB_CUDA(cudaMemcpyAsync(wtab.p, tab.data(), tab.size(), cudaMemcpyHostToDevice, s));
    MSB_CUDA(cudaMemsetAsync(status.p, 0, 16, s));
    const char* t = reinterpret_cast<const char*>(wtab.p);
    const float* const* src_d = reinterpret_cast<const float* const*>(t);
    float* const* dst_d = reinterpret_cast<float* const*>(t + (size_t)B * sizeof(void*));
    const int* T_d = reinterpret_cast<const int*>(t + (size_t)2 * B * sizeof(void*));
    MSB_CUDA(launch_gather_seg_rows(src_d, T_d, B, R3, ed, ex.as<float>(), s));
    encoder_layers_tc(rows3, R3, T_d);
    MSB_CUDA(launch_ln_scatter_rows(ex.as<float>(), B, max_new, R3, ed, m.enc_final, 1.0f, 1e-5f, m.pos_emb, T_d + B,
                                    T_d + 2 * B, T_d + 3 * B, dst_d, s));
    unsigned st_word = 0;
    MSB_CUDA(cudaMemcpyAsync(&st_word, status.p, 4, cudaMemcpyDeviceToHost, s));
    MSB_CUDA(cudaStreamSynchronize(s));  // also: the host table is read
    throw_device_status(st_word, "tensor-core stream encoder");
    return true;
}

bool BatchEngine::encode_windows_inc(const std::vector<StreamIncWindow>& w) {
    if (w.empty()) return true;
    if (!tc_encoder_fits()) return false;
    const Config& c = m.cfg;
    const int ed = c.e_hidden, B = (int)w.size(), L = c.e_layers;
    ensure_enc_weights();
    cudaStream_t s = m.stream;
    grow(status, 16);
    // right context summed over layers 0..l
    std::vector<int> Ssum(L);
    for (int l = 0, acc = 0; l < L; ++l) Ssum[l] = (acc += std::max(0, c.window(l).second));
    // per layer and stream: rows recomputed from c (earlier ones final), segment from s0 (left
    // attention context of row c), n = total - s0 rows
    std::vector<int> R(L, 1);
    std::vector<int> c0((size_t)L * B), s0((size_t)L * B);
    int max_new = 1;
    size_t rows_max = 0;
    for (int l = 0; l < L; ++l) {
        const int left = std::max(0, c.window(l).first);
        for (int b = 0; b < B; ++b) {
            const StreamIncWindow& x = w[b];
            const int cl = std::max(0, std::min(x.prev, x.total) - Ssum[l]);
            const int sl = std::max(0, cl - left);
            c0[(size_t)l * B + b] = cl;
            s0[(size_t)l * B + b] = sl;
            R[l] = std::max(R[l], x.total - sl);
        }
        rows_max = std::max(rows_max, (size_t)B * R[l]);
    }
    for (const auto& x : w) {
        max_new = std::max(max_new, x.nnew);
        if ((int)x.layer_out.size() != L - 1 || x.emitted < 0 || x.emitted + x.nnew > x.total)
            throw MsError(MS_ERR_INVALID_ARG, "incremental encoder: bad stream window");
    }
    grow(ex, enc_rows_capacity(rows_max) * ed * 4);
    float* X = ex.as<float>();
    // tables (each array 16-byte aligned), per layer: gather src[B], gather rows[B]; copy
    // src[B], dst[B], floats[B] (layers but the last); then memory dst[B], off[B], cnt[B], pos[B]
    const size_t P8 = ((size_t)B * 8 + 15) & ~(size_t)15, P4 = ((size_t)B * 4 + 15) & ~(size_t)15;
    const size_t o_gT = P8, o_csrc = P8 + P4, o_cdst = 2 * P8 + P4, o_ccnt = 3 * P8 + P4;
    const size_t per_layer = 3 * P8 + 2 * P4, fin = P8 + 3 * P4;
    const size_t bytes = (size_t)L * per_layer + fin;
    char* h = inc_tables.host(bytes);
    for (int l = 0; l < L; ++l) {
        char* t = h + (size_t)l * per_layer;
        const float** gsrc = reinterpret_cast<const float**>(t);
        int* gT = reinterpret_cast<int*>(t + o_gT);
        const float** csrc = reinterpret_cast<const float**>(t + o_csrc);
        float** cdst = reinterpret_cast<float**>(t + o_cdst);
        int* ccnt = reinterpret_cast<int*>(t + o_ccnt);
        for (int b = 0; b < B; ++b) {
            const StreamIncWindow& x = w[b];
            const int cl = c0[(size_t)l * B + b], sl = s0[(size_t)l * B + b];
            gsrc[b] = (l == 0 ? x.feat : x.layer_out[l - 1]) + (size_t)sl * ed;
            gT[b] = x.total - sl;
            // layer l's recomputed rows c .. total of segment b into the stream's layer-l rows
            csrc[b] = X + ((size_t)b * R[l] + (cl - sl)) * ed;
            cdst[b] = l < L - 1 ? x.layer_out[l] + (size_t)cl * ed : nullptr;
            ccnt[b] = (x.total - cl) * ed;
        }
    }
    {
        char* t = h + (size_t)L * per_layer;
        float** dst = reinterpret_cast<float**>(t);
        int* off = reinterpret_cast<int*>(t + P8);
        int* cnt = reinterpret_cast<int*>(t + P8 + P4);
        int* pos = reinterpret_cast<int*>(t + P8 + 2 * P4);
        for (int b = 0; b < B; ++b) {
            dst[b] = w[b].dst;
            off[b] = w[b].emitted - s0[(size_t)(L - 1) * B + b];
            cnt[b] = w[b].nnew;
            pos[b] = w[b].pos;
        }
    }
    MSB_CUDA(cudaMemsetAsync(status.p, 0, 16, s));
    char* d = inc_tables.upload(bytes, s, m.streams_pool());
    for (int l = 0; l < L; ++l) {
        const char* t = d + (size_t)l * per_layer;
        const int* gT = reinterpret_cast<const int*>(t + o_gT);
        const size_t rows = (size_t)B * R[l];
        MSB_CUDA(launch_gather_seg_rows(reinterpret_cast<const float* const*>(t), gT, B, R[l], ed, X, s));
        encoder_layers_tc(rows, R[l], gT, l, l + 1);
        if (l < L - 1)
            MSB_CUDA(launch_copy_rows_batch(reinterpret_cast<const float* const*>(t + o_csrc),
                                            reinterpret_cast<float* const*>(t + o_cdst),
                                            reinterpret_cast<const int*>(t + o_ccnt), B, s));
    }
    const char* t = d + (size_t)L * per_layer;
    MSB_CUDA(launch_ln_scatter_rows(X, B, max_new, R[L - 1], ed, m.enc_final, 1.0f, 1e-5f, m.pos_emb,
                                    reinterpret_cast<const int*>(t + P8), reinterpret_cast<const int*>(t + P8 + P4),
                                    reinterpret_cast<const int*>(t + P8 + 2 * P4),
                                    reinterpret_cast<float* const*>(t), s));
    unsigned st_word = 0;
    MSB_CUDA(cudaMemcpyAsync(&st_word, status.p, 4, cudaMemcpyDeviceToHost, s));
    MSB_CUDA(cudaStreamSynchronize(s));
    throw_device_status(st_word, "tensor-core incremental stream encoder");
    return true;
}

BatchEngine::Result BatchEngine::run(const std::vector<const float*>& audio_dev, const std::vector<int64_t>& n_samples,
                                     const std::vector<int>& limits, bool forced, bool want_logits, float temperature,
                                     unsigned seed_) {
    inv_temp = temperature > 0.f ? 1.f / temperature : 0.f;
    seed = seed_;
    const Config& c = m.cfg;
    const int B = (int)audio_dev.size();
    cudaStream_t s = m.stream;
    Result res;
    ensure_weights();
    MSB_CUDA(cudaEventRecord(m.ev[0], s));
    // encode every utterance, gather the memory rows [Mtot, d]
    std::vector<int> off(B), fr(B);
    std::vector<float*> staged;
    int Mtot = 0, maxM = 0;
    // first pass: frame counts
    for (int b = 0; b < B; ++b) {
        const int fl = c.frame_len();
        const int T1 = (int)(n_samples[b] / fl);
        const int T2 = T1 > 0 ? (T1 - 1) / 2 + 1 : 0;
        fr[b] = T2 > 0 ? (T2 - 1) / 2 + 1 : 0;
        if (fr[b] <= 0) throw MsError(MS_ERR_INVALID_ARG, "an utterance has fewer samples than one frame");
        off[b] = Mtot;
        Mtot += fr[b];
        maxM = std::max(maxM, fr[b]);
    }
    const int T = *std::max_element(limits.begin(), limits.end());
    ensure_ws(B, T, Mtot, maxM);
    // the status word starts at zero before any of this call's kernels (the split-K
    // epilogues read it; the decode reports what encoder or decode recorded in it)
    MSB_CUDA(cudaMemsetAsync(status.p, 0, 16, s));
    if (!((m.enc_bf16 || m.opts.weight_dtype == MS_W_AUTO) && encode_tc(audio_dev, n_samples, off, fr))) {
        encode_all(audio_dev, n_samples, off);
        m.cross_kv_into(memory.as<float>(), Mtot, 0, cross32.as<float>(), m.kv_f16 ? cross16.p : nullptr, Mc);
    }
    MSB_CUDA(cudaEventRecord(m.ev[1], s));
    return decode_prepared(B, T, maxM, off, fr, limits, forced, want_logits);
}

BatchEngine::Result BatchEngine::run_cross(const std::vector<CrossSrc>& src, const std::vector<int>& limits,
                                           bool forced, float temperature, unsigned seed_) {
    inv_temp = temperature > 0.f ? 1.f / temperature : 0.f;
    seed = seed_;
    const Config& c = m.cfg;
    const int B = (int)src.size();
    cudaStream_t s = m.stream;
    ensure_weights();
    MSB_CUDA(cudaEventRecord(m.ev[0], s));
    std::vector<int> off(B), fr(B), mcap(B);
    int Mtot = 0, maxM = 0;
    for (int b = 0; b < B; ++b) {
        fr[b] = src[b].frames;
        mcap[b] = src[b].m_cap;
        if (fr[b] <= 0 || fr[b] > mcap[b]) throw MsError(MS_ERR_INVALID_ARG, "a stream has no memory to decode");
        off[b] = Mtot;
        Mtot += fr[b];
        maxM = std::max(maxM, fr[b]);
    }
    const int T = *std::max_element(limits.begin(), limits.end());
    // in place: the streams' buffers are read where they lie, so the engine holds no copy (the
    // copy and its capacity would grow with the sum of every stream's memory)
    const bool in_place = cross_rows_supported(c.head_dim);
    for (int b = 0; b < B && in_place; ++b)
        if ((reinterpret_cast<uintptr_t>(src[b].c32) & 15) || (m.kv_f16 && (reinterpret_cast<uintptr_t>(src[b].c16) & 15)))
            throw MsError(MS_ERR_CUDA, "stream cross K/V not 16-byte aligned");
    ensure_ws(B, T, in_place ? 0 : Mtot, maxM);
    MSB_CUDA(cudaMemsetAsync(status.p, 0, 16, s));
    // pointer tables: src32[B], src16[B] (the stored copy; the fp32 rows when the cache is
    // fp32), then mcap[B]
    std::vector<const void*> ptrs(2 * (size_t)B);
    for (int b = 0; b < B; ++b) {
        ptrs[b] = src[b].c32;
        ptrs[B + b] = m.kv_f16 ? src[b].c16 : (in_place ? src[b].c32 : nullptr);
    }
    grow(xsrc, (size_t)2 * B * sizeof(void*) + (size_t)B * 4);
    char* tab = reinterpret_cast<char*>(xsrc.p);
    MSB_CUDA(cudaMemcpyAsync(tab, ptrs.data(), ptrs.size() * sizeof(void*), cudaMemcpyHostToDevice, s));
    MSB_CUDA(cudaMemcpyAsync(tab + 2 * B * sizeof(void*), mcap.data(), (size_t)B * 4, cudaMemcpyHostToDevice, s));
    MSB_CUDA(cudaMemcpyAsync(frame_off.p, off.data(), (size_t)B * 4, cudaMemcpyHostToDevice, s));
    MSB_CUDA(cudaMemcpyAsync(frames.p, fr.data(), (size_t)B * 4, cudaMemcpyHostToDevice, s));
    if (in_place) {
        xrows.src32 = reinterpret_cast<const void* const*>(tab);
        xrows.src16 = reinterpret_cast<const void* const*>(tab + B * sizeof(void*));
        xrows.cap = reinterpret_cast<const int*>(tab + 2 * B * sizeof(void*));
    } else {
        MSB_CUDA(launch_gather_cross(reinterpret_cast<const float* const*>(tab),
                                     reinterpret_cast<const void* const*>(tab + B * sizeof(void*)),
                                     reinterpret_cast<const int*>(tab + 2 * B * sizeof(void*)), frames.as<int>(),
                                     frame_off.as<int>(), B, c.layers * 2 * c.kv_heads, c.head_dim, Mc,
                                     cross32.as<float>(), m.kv_f16 ? cross16.p : nullptr, s));
    }
    MSB_CUDA(cudaEventRecord(m.ev[1], s));
    xrows_on = in_place;
    try {
        Result r = decode_prepared(B, T, maxM, off, fr, limits, forced, false);
        xrows_on = false;
        return r;
    } catch (...) {
        xrows_on = false;
        throw;
    }
}

BatchEngine::Result BatchEngine::decode_prepared(int B, int T, int maxM, const std::vector<int>& off,
                                                 const std::vector<int>& fr, const std::vector<int>& limits,
                                                 bool forced, bool want_logits) {
    const Config& c = m.cfg;
    cudaStream_t s = m.stream;
    Result res;
    assign_pages(B, T, limits);
    // step state
    std::vector<int> bos(B, c.dec_start);
    MSB_CUDA(cudaMemcpyAsync(next_ids.p, bos.data(), (size_t)B * 4, cudaMemcpyHostToDevice, s));
    MSB_CUDA(cudaMemcpyAsync(limits_d.p, limits.data(), (size_t)B * 4, cudaMemcpyHostToDevice, s));
    MSB_CUDA(cudaMemcpyAsync(frame_off.p, off.data(), (size_t)B * 4, cudaMemcpyHostToDevice, s));
    MSB_CUDA(cudaMemcpyAsync(frames.p, fr.data(), (size_t)B * 4, cudaMemcpyHostToDevice, s));
    MSB_CUDA(cudaMemsetAsync(counts.p, 0, (size_t)B * 4, s));
    MSB_CUDA(cudaMemsetAsync(done.p, 0, (size_t)B * 4, s));
    MSB_CUDA(cudaMemsetAsync(hit.p, 0, (size_t)B * 4, s));
    MSB_CUDA(cudaMemsetAsync(amax.p, 0, (size_t)B * 8, s));
    MSB_CUDA(cudaMemsetAsync(pos.p, 0, 16, s));
    DevBuf logit_buf;
    if (want_logits) logit_buf.ensure((size_t)T * B * c.vocab * 4);
    auto logits_at = [&](int step) -> float* {
        return want_logits ? logit_buf.as<float>() + (size_t)step * B * c.vocab : nullptr;
    };
    // step st sees positions 0..st: its self attention needs rounds of at most st + 1 keys
    auto reach_for = [](int st) { return st < 32 ? 32 : (st < 64 ? 64 : 0); };
    sa_reach = reach_for(0);
    enqueue_step(B, maxM, forced, true, logits_at(0));
    if (want_logits) {
        for (int st = 1; st < T; ++st) {
            sa_reach = reach_for(st);
            enqueue_step(B, maxM, forced, false, logits_at(st));
        }
    } else if (T > 1) {
        // one graph per reach bucket, each replayed for its steps; every graph lives until
        // the stream has finished with it
        std::vector<cudaGraph_t> graphs;
        std::vector<cudaGraphExec_t> execs;
        auto release = [&]() {
            for (auto e : execs) cudaGraphExecDestroy(e);
            for (auto g : graphs) cudaGraphDestroy(g);
        };
        try {
            for (int st = 1; st < T;) {
                const int r = reach_for(st);
                int end = st;
                while (end < T && reach_for(end) == r) ++end;
                sa_reach = r;
                cudaGraph_t graph = nullptr;
                MSB_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
                try {
                    enqueue_step(B, maxM, forced, false, nullptr);
                } catch (...) {
                    cudaStreamEndCapture(s, &graph);
                    if (graph) cudaGraphDestroy(graph);
                    throw;
                }
                MSB_CUDA(cudaStreamEndCapture(s, &graph));
                graphs.push_back(graph);
                cudaGraphExec_t exec = nullptr;
                MSB_CUDA(cudaGraphInstantiate(&exec, graph, 0));
                execs.push_back(exec);
                for (; st < end; ++st) MSB_CUDA(cudaGraphLaunch(exec, s));
            }
            MSB_CUDA(cudaStreamSynchronize(s));
        } catch (...) {
            cudaStreamSynchronize(s);
            release();
            sa_reach = 0;
            throw;
        }
        release();
    }
    sa_reach = 0;
    MSB_CUDA(cudaEventRecord(m.ev[2], s));
    res.t_cap = Tc;
    res.steps = T;
    res.ids.resize((size_t)B * Tc);
    res.counts.resize(B);
    res.hit_eos.resize(B);
    unsigned st_word = 0;
    MSB_CUDA(cudaMemcpyAsync(res.ids.data(), ids.p, (size_t)B * Tc * 4, cudaMemcpyDeviceToHost, s));
    MSB_CUDA(cudaMemcpyAsync(res.counts.data(), counts.p, (size_t)B * 4, cudaMemcpyDeviceToHost, s));
    MSB_CUDA(cudaMemcpyAsync(res.hit_eos.data(), hit.p, (size_t)B * 4, cudaMemcpyDeviceToHost, s));
    MSB_CUDA(cudaMemcpyAsync(&st_word, status.p, 4, cudaMemcpyDeviceToHost, s));
    if (want_logits) {
        res.logits.resize((size_t)T * B * c.vocab);
        MSB_CUDA(cudaMemcpyAsync(res.logits.data(), logit_buf.p, res.logits.size() * 4, cudaMemcpyDeviceToHost, s));
    }
    MSB_CUDA(cudaStreamSynchronize(s));
    throw_device_status(st_word, "batched decode");
    float te = 0, td = 0;
    cudaEventElapsedTime(&te, m.ev[0], m.ev[1]);
    cudaEventElapsedTime(&td, m.ev[1], m.ev[2]);
    res.encode_ms = te;
    res.decode_ms = td;
    return res;
}

}  // namespace msb
