/*
 * moonshine_b200.h -- C ABI of the B200-native Moonshine V2 streaming speech-to-text path.
 *
 * Every entry point replaces one piece of the reference Swift API of
 * kylehowells/moonshine-mlx (paths below are inside that project).  Token ids cross
 * this boundary; turning them into text stays with the caller's tokenizer
 * (Sources/MoonshineMLX/MoonshineTokenizer.swift:21-23), exactly as the reference's
 * generate/transcribe call `decodeTokens` on the ids they produce.
 *
 * Conventions
 *   - Every call returns ms_status.  On failure a thread-local message is available
 *     from ms_last_error().  Inference never throws in the reference; here it returns
 *     a status and leaves the outputs untouched on error.
 *   - Caller owns every host buffer (audio in, ids/logits out).  Audio is float32 mono
 *     at the model's sample rate (16 kHz), copied to device memory during the call.
 *   - A model handle may be used from several threads for ms_generate* calls (each
 *     call gets its own CUDA stream and workspace when needed); calls on one stream
 *     handle must be serialised by the caller, as with the reference's StreamingState.
 *   - No function here allocates with malloc on the hot path after the first call of
 *     a given size; device buffers are pooled per model.
 */
#ifndef MOONSHINE_B200_H
#define MOONSHINE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference's MoonshineError (ModelLoader.swift:187-203) maps to
 * MS_ERR_BAD_CONFIG (invalidConfig), MS_ERR_NOT_FOUND (missingWeights) and
 * MS_ERR_BAD_WEIGHTS; downloadFailed/noTokenizer/audioLoadFailed have no
 * counterpart (no hub download, tokenizer and audio I/O stay with the caller). */
typedef enum {
    MS_OK = 0,
    MS_ERR_INVALID_ARG = 1,
    MS_ERR_OOM = 2,
    MS_ERR_CUDA = 3,
    MS_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up */
    MS_ERR_BAD_WEIGHTS = 5,
    MS_ERR_BAD_CONFIG = 6,
    MS_ERR_NOT_FOUND = 7,
    MS_ERR_UNSUPPORTED = 8,
    MS_ERR_CAPACITY = 9     /* output buffer too small; *n_out holds the needed size */
} ms_status;

typedef struct ms_model ms_model;
typedef struct ms_stream ms_stream;

/* KV-cache storage type.  The reference stores decoder K/V in fp32, or in fp16 after
 * enableFloat16KVCache(true) -- which its loader turns on by default
 * (MoonshineModel.swift:47-65). */
typedef enum { MS_KV_F32 = 0, MS_KV_F16 = 1 } ms_kv_dtype;

/* Matmul input type of batched generation, and the weight rows of quantized checkpoints in
 * the batch-1 decode.  The batch-1 kernels compute in fp32 from the checkpoint's values.
 * Batched generation runs tensor-core GEMMs: for BF16/F16 checkpoints under MS_W_AUTO, or
 * any checkpoint under MS_W_BF16, on bf16 inputs (the encoder too); otherwise (MS_W_F32, or
 * an F32 checkpoint under MS_W_AUTO) the decode GEMMs take every weight and input as a bf16
 * high plane plus a bf16 low plane and sum three products (hi.hi + hi.lo + lo.hi), which
 * keeps fp32-level accuracy, and the encoder runs fp32 CUDA-core GEMMs.  For a quantized checkpoint the clustered batch-1 kernel
 * streams the quantized codes of its row-split weights (ms_model_decode_weight_bits) except
 * under MS_W_F32, which streams them dequantized to fp32. */
typedef enum { MS_W_AUTO = 0, MS_W_F32 = 1, MS_W_BF16 = 2 } ms_weight_dtype;

typedef struct {
    int32_t device;          /* CUDA device ordinal */
    int32_t kv_dtype;        /* ms_kv_dtype; default MS_KV_F16 like prepareForInference */
    int32_t weight_dtype;    /* ms_weight_dtype */
    int32_t max_batch;       /* largest ms_generate_batch / stream batch (default 64) */
    int32_t decode_kernel;   /* batch-1 decode kernel: MS_DECODE_AUTO or MS_DECODE_CLUSTER
                                (head-clustered when the dims and the GPU allow it, else
                                single-grid) or MS_DECODE_GRID (single-grid persistent kernel).
                                Both compute the same greedy loop. */
    int32_t quant_stream;    /* quantized checkpoints, clustered kernel: which weights stream as
                                codes (MS_QSTREAM_*); ignored otherwise */
    int32_t reserved[6];
} ms_options;

enum { MS_DECODE_AUTO = 0, MS_DECODE_GRID = 1, MS_DECODE_CLUSTER = 2 };

/* MS_QSTREAM_ALL: q|k|v, cross q, fc1 and the LM head; MS_QSTREAM_LM: the LM head only;
 * MS_QSTREAM_NONE: none (every row dequantized to fp32 at load); MS_QSTREAM_AUTO: the LM
 * head only, which measured fastest for 2, 4 and 8 bits on the tiny model (ALL streams the
 * fewest bytes but its small per-layer blocks cost more to dequantize than they save). */
enum { MS_QSTREAM_AUTO = 0, MS_QSTREAM_ALL = 1, MS_QSTREAM_LM = 2, MS_QSTREAM_NONE = 3 };

/* Fills *opts with the defaults (device 0, fp16 KV, auto weights, max_batch 64). */
void ms_options_default(ms_options* opts);

/* Parsed config.json (MoonshineConfig.swift:61-178), read-only view. */
typedef struct {
    int32_t hidden_size, intermediate_size, num_hidden_layers, num_attention_heads,
            num_key_value_heads, head_dim, vocab_size, max_position_embeddings;
    int32_t tie_word_embeddings, encoder_hidden_size;
    int32_t enc_hidden_size, enc_intermediate_size, enc_num_hidden_layers,
            enc_num_attention_heads, enc_num_key_value_heads, enc_head_dim,
            enc_frame_len, enc_sample_rate, enc_max_position_embeddings;
    int32_t bos_token_id, eos_token_id, decoder_start_token_id, pad_token_id;
    int32_t rotary_ndims;
    float rope_theta;
    double max_tokens_per_second;
    int32_t num_sliding_windows;  /* 0 when config.json has no sliding_windows */
    int32_t sliding_windows[64][2];
} ms_model_config;

/* MoonshineModel.load(from:hfToken:) (MoonshineModel.swift:409-414) for a LOCAL
 * directory holding config.json + *.safetensors (ModelLoader.swift:35-70,115-130).
 * Accepts HuggingFace key layout (``model.`` prefix, ``.gamma``, conv [out,in,k]) and
 * MLX layout, as sanitizeWeights does (ModelLoader.swift:75-101), and MLX affine-quantized
 * checkpoints (config.json "quantization", 2/4/8 bits, ModelLoader.swift:47-49,103-111).
 * Hub download is not supported. */
ms_status ms_model_load(const char* dir, const ms_options* opts, ms_model** out);
void ms_model_free(ms_model* model);

/* Code width of the weight rows the clustered batch-1 decode kernel streams for q|k|v,
 * cross q and fc1 of a quantized checkpoint (2, 4 or 8: the checkpoint's codes with their
 * per-group scale and bias, multiplied in the kernel), or 0 when it streams fp32 rows
 * (unquantized checkpoints, MS_W_F32, MS_DECODE_GRID, quant_stream other than
 * MS_QSTREAM_ALL, or dims the quantized rows do not fit).  *lm_bits (nullable) receives the
 * same for the LM head (0 when it is tied to the embedding or for MS_QSTREAM_NONE). */
int32_t ms_model_decode_weight_bits(const ms_model* model, int32_t* lm_bits);

/* MoonshineModel.enableFloat16KVCache(_:) (MoonshineModel.swift:60-65). */
ms_status ms_model_enable_fp16_kv_cache(ms_model* model, int32_t enabled);

/* MoonshineModel.sampleRate (MoonshineModel.swift:44). */
int32_t ms_model_sample_rate(const ms_model* model);

ms_status ms_model_get_config(const ms_model* model, ms_model_config* out);

/* Offline generation parameters (MoonshineModel.generate, MoonshineModel.swift:130-136). */
typedef struct {
    int32_t max_tokens;        /* maxTokens; <= 0 means Int.max (no cap) */
    int32_t forced_len;        /* > 0: decode exactly this many tokens per chunk, EOS fed
                                  back like any id (benchmark / parity harness mode);
                                  < 0: each chunk (ms_generate_batch: each utterance) decodes
                                  exactly its own limit min(max_tokens, ceil(seconds * 6.5)),
                                  EOS fed back like any id */
    float temperature;         /* 0: greedy argMax; > 0: each token is a draw from
                                  softmax(logits / temperature) (MLXRandom.categorical,
                                  MoonshineModel.swift:211-213), by the Gumbel-max trick */
    float reserved_f;
    double chunk_duration;     /* seconds per independently decoded chunk; <= 0 -> 30 */
    const int32_t* teacher_ids;/* nullable: feed these ids instead of the argmax (one per
                                  decoder call after BOS; needs forced_len = count) */
    int32_t n_teacher;
    int32_t seed;              /* temperature > 0: a draw depends only on (seed, chunk, step,
                                  vocabulary index; plus the row in ms_generate_batch) */
    float* batch_logits;       /* nullable, ms_generate_batch only: [batch][cap][vocab]
                                  logits of every decoder call */
    int32_t reserved[4];
} ms_gen_params;

void ms_gen_params_default(ms_gen_params* p);

/* Timings of the last call (the reference's `profile:` output,
 * MoonshineModel.swift:167-183). */
typedef struct {
    int32_t n_tokens;
    int32_t n_chunks;
    int32_t hit_eos;           /* last chunk ended on EOS */
    int32_t memory_frames;     /* encoder frames of the last chunk */
    int32_t decode_kernel;     /* batch-1 kernel of the last chunk: MS_DECODE_GRID or MS_DECODE_CLUSTER */
    double encode_ms, decode_ms, total_ms;
    double tokens_per_second;  /* n_tokens / total (MoonshineModel.swift:182) */
} ms_gen_stats;

/* MoonshineModel.generate(audio:maxTokens:temperature:chunkDuration:profile:)
 * (MoonshineModel.swift:130-237): per 30 s chunk, frontend + encoder + greedy decode.
 *   ids_out    [cap]      generated ids of all chunks, BOS/EOS excluded
 *   logits_out nullable;  [cap * vocab] float32 logits of every decoder call
 *   stats      nullable */
ms_status ms_generate(ms_model* model, const float* audio, int64_t n_samples,
                      const ms_gen_params* params, int32_t* ids_out, int32_t cap,
                      int32_t* n_out, float* logits_out, ms_gen_stats* stats);

/* ms_generate for audio that is already in device memory of the model's GPU (no
 * counterpart in the reference, whose MLXArray audio is device-resident by design):
 * audio_dev [n_samples] and ids_dev [cap] are device pointers; nothing crosses PCIe
 * except a few status words. */
ms_status ms_generate_device(ms_model* model, const float* audio_dev, int64_t n_samples,
                             const ms_gen_params* params, int32_t* ids_dev, int32_t cap,
                             int32_t* n_out, ms_gen_stats* stats);

/* The CUDA stream (cudaStream_t) the model's work runs on, for callers that bracket
 * calls with their own events. */
void* ms_model_stream(ms_model* model);

/* Self-attention K/V pages of the batched engine (ms_generate_batch and the lockstep
 * ms_stream_transcribe_batch; no counterpart in the reference, whose cache grows by
 * concatenation, MoonshineLayers.swift:106-115).  Each call gives every row
 * ceil(limit / page_positions) pages of page_positions positions (all layers, K and V), so a
 * ragged batch holds the sum of its rows' needs rather than rows x the longest, and every
 * page returns to the pool when the call ends.  *used: pages the last call assigned;
 * *capacity: pages the pool holds (the largest call so far).  Any output may be null. */
ms_status ms_model_batch_kv_pages(ms_model* model, int64_t* used, int64_t* capacity, int32_t* page_positions);

/* Batched offline generation: B independent utterances decoded together (no counterpart
 * in the reference, which is batch 1).  Utterances of at most one chunk (chunk_duration)
 * are decoded in lockstep: every projection is one tensor-core GEMM over all B rows (fp32
 * accumulation, residual stream and softmax; inputs as ms_weight_dtype describes), so logits
 * agree with a per-utterance ms_generate to bf16 precision for bf16 checkpoints and to fp32
 * precision for fp32 ones.  Longer utterances fall back to per-utterance decoding.
 * ids_out is [B * cap], n_out [B]; teacher ids are not supported. */
ms_status ms_generate_batch(ms_model* model, const float* const* audios,
                            const int64_t* n_samples, int32_t batch,
                            const ms_gen_params* params, int32_t* ids_out, int32_t cap,
                            int32_t* n_out, ms_gen_stats* stats);

/* Intermediate results for parity checks: memory (= prepareMemory(encoder(embed(x))),
 * MoonshineModel.swift:194-196) of one chunk, [frames * hidden] float32. */
ms_status ms_encode(ms_model* model, const float* audio, int64_t n_samples,
                    float* memory_out, int64_t cap_floats, int32_t* n_frames);

/* Greedy decode that allocates no device memory.  No counterpart in the reference: it
 * exists for callers that cannot call cudaMalloc once they are running -- a real-time
 * audio callback, where an allocation can block and synchronise the device past the
 * callback's deadline, or a host that runs inside a fixed, pre-reserved GPU memory budget.
 *
 * The caller passes encoder memory rows already in device memory of the model's GPU
 * (memory_dev, [frames * hidden] float32, 16-byte aligned; e.g. ms_encode's output copied
 * to the device) and a device buffer ids_dev of n_tokens int32.  The rows must be fully
 * written before the call: the call's work runs on the model's own stream (ms_model_stream),
 * which does not wait for other streams, so synchronise the stream that wrote them (or make
 * the model's stream wait on an event recorded after the write).  The call runs up to
 * n_tokens decoder calls from BOS (forced != 0: exactly n_tokens, EOS fed back like any
 * id), writes the ids to ids_dev and their count to *n_out (host), like ms_generate_device
 * for one chunk.  It always uses the single-grid decode kernel; ms_generate_device may pick
 * the head-clustered one, which sums in another order, so the two agree to rounding.
 *
 * The cross-attention K/V, the self-attention K/V cache and the decode working buffers
 * live in one static 16 MiB device array that every GPU loading this library holds until
 * the process exits: with the tiny model that covers 500 memory frames (10 s of audio) and
 * 128 decoder calls; larger requests fail with MS_ERR_CAPACITY and a message giving the
 * bytes needed.  ms_model_load reserves the array on its device and loads the kernels this
 * call launches, so the call itself neither allocates nor loads code.  Every call reuses
 * the array: two calls whose GPU work overlapped would race on it, which this library
 * prevents by serialising the calls and waiting for each call's work before returning. */
ms_status ms_decode_memory_static(ms_model* model, const float* memory_dev, int32_t frames,
                                  int32_t n_tokens, int32_t forced, int32_t* ids_dev,
                                  int32_t* n_out, int32_t* hit_eos);

/* ------------------------------------------------------------------- word timestamps */

/* Outputs of ms_generate_alignment.  The caller sets the buffers and capacities; the call
 * sets the counts. */
typedef struct {
    int32_t* ids;              /* [cap] generated ids, BOS/EOS excluded (the reference's gen) */
    float* token_probs;        /* [cap] softmax probability of each decoder call's chosen id
                                  (tokenProbs, MoonshineModel.swift:278-283; the EOS call included) */
    int32_t* jump_frames;      /* [cap] jumpTimes (MoonshineTimestamps.swift:176-184): the memory
                                  frame at which the DTW path enters each call's row */
    int32_t cap;               /* capacity of ids, token_probs and jump_frames */
    int32_t reserved0;
    float* attn_rows;          /* nullable [attn_cap]: per decoder call, the mean over layers and
                                  heads of the cross-attention softmax over memory frames,
                                  row-major [n_steps][n_frames] (:106-130) */
    float* attn_filtered;      /* nullable [attn_cap]: the same rows z-scored and median-filtered
                                  (:132-146); the DTW cost is their negation */
    int64_t attn_cap;          /* floats in each of attn_rows / attn_filtered */
    int32_t n_tokens;          /* out: ids */
    int32_t n_steps;           /* out: decoder calls = attention rows = jump frames
                                  (n_tokens, plus one when the last call produced EOS) */
    int32_t n_frames;          /* out: memory frames (numFrames) */
    int32_t hit_eos;           /* out */
} ms_alignment;

/* generateWithWordTimestamps(audio:maxTokens:timeOffset:) (MoonshineModel.swift:241-316) up
 * to the tokenizer: the whole audio is encoded in one pass, then greedy decoding of up to
 * min(max_tokens, ceil(seconds * 6.5)) decoder calls stops at EOS (max_tokens <= 0: no
 * cap).  Every call's cross-attention queries are kept on the device; afterwards the GPU
 * rebuilds the attention rows, z-scores and median-filters them (medfilt_width, the
 * reference's 7; <= 1 disables the filter, at most 63), and the DTW path over them gives
 * jump_frames.  Grouping ids into words needs the tokenizer and stays with the caller, who
 * passes the word boundaries to ms_word_timings.  The audio's memory must fit the
 * positional table (max_position_embeddings frames). */
ms_status ms_generate_alignment(ms_model* model, const float* audio, int64_t n_samples,
                                int32_t max_tokens, int32_t medfilt_width, ms_alignment* out,
                                ms_gen_stats* stats);

/* The DTW step of findAlignment on rows the caller holds (host only, no GPU work): dtw
 * (MoonshineTimestamps.swift:20-65) over cost = -filtered ([n_rows][n_frames], row-major),
 * then the jump extraction (:176-184).  jump_frames_out receives n_rows frames. */
ms_status ms_alignment_jump_frames(const float* filtered, int32_t n_rows, int32_t n_frames,
                                   int32_t* jump_frames_out);

/* Word timings of findAlignment (MoonshineTimestamps.swift:186-239) for words given by the
 * index of their first token (word_first, ascending; word w covers tokens
 * [word_first[w], word_first[w+1]) and the last word ends at n_tokens; the reference starts
 * a word at every token whose piece begins with U+2581).  start_out/end_out are seconds
 * (time_offset + frame * 0.02, rounded to 1 ms; overlapping neighbours meet at the rounded
 * midpoint), prob_out the mean token probability rounded to 1e-4.  Each output is
 * [n_words]; *n_out receives the number of words written. */
ms_status ms_word_timings(const int32_t* jump_frames, int32_t n_jumps, const float* token_probs,
                          int32_t n_probs, const int32_t* word_first, int32_t n_words,
                          int32_t n_tokens, int32_t n_frames, double time_offset,
                          double* start_out, double* end_out, double* prob_out, int32_t* n_out);

/* ------------------------------------------------------------------- streaming */

/* StreamingConfig (MoonshineStreaming.swift:47-62), plus fields of this library: transcribe's
 * temperature argument and the seed of its draws. */
typedef struct {
    int32_t max_memory_frames;   /* default 100000 */
    int32_t min_segment_frames;  /* default 250 */
    int32_t batch_decode;        /* ms_stream_transcribe_batch only (default 0): 1 encodes the
                                    new frames of all streams of one model in one tensor-core
                                    pass and decodes them in lockstep on tensor cores (the
                                    batched engine; fp32 checkpoints keep fp32-level products,
                                    bf16 ones bf16), so ids match a per-stream call except
                                    where the top two logits are closer than that precision.
                                    The pass runs each encoder layer over the rows whose value
                                    can have changed since the stream's previous call plus
                                    their left attention context (the committed memory rows
                                    are those of the reference's window); 2 re-encodes each
                                    stream's whole window instead, as the reference does */
    float temperature;           /* transcribe(temperature:) (:122-128): 0 greedy (default);
                                    > 0 draws each token from softmax(logits / temperature)
                                    (decodeMemory, :238-268) by the Gumbel-max trick */
    int32_t seed;                /* temperature > 0: a draw depends only on (seed, the stream's
                                    number of transcribe calls so far, step, vocabulary index;
                                    plus the stream's row in a lockstep batch) */
} ms_streaming_config;

void ms_streaming_config_default(ms_streaming_config* c);

/* createStream() (MoonshineStreaming.swift:69-71). */
ms_status ms_stream_create(ms_model* model, ms_stream** out);
void ms_stream_free(ms_stream* stream);
/* startStream(_:) (:74-78) and stopStream(_:) (:81-83). */
ms_status ms_stream_start(ms_stream* stream);
ms_status ms_stream_stop(ms_stream* stream);
/* addAudio(_:chunk:) (:87-105). */
ms_status ms_stream_add_audio(ms_stream* stream, const float* chunk, int64_t n_samples);

/* addAudio of many streams at once (no counterpart in the reference, which feeds one stream
 * per call): chunks[i] (n_samples[i] samples) goes to streams[i], with the same effect as n
 * calls of ms_stream_add_audio (a stream listed twice takes its chunks in order).  When all
 * streams share one model their frontends run as one batched pass (one upload of every
 * stream's whole frames, five launches for all of them), which is what serving many streams
 * needs. */
ms_status ms_stream_add_audio_batch(ms_stream* const* streams, int32_t n, const float* const* chunks,
                                    const int64_t* n_samples);
/* transcribe(_:isFinal:streamingConfig:maxTokens:temperature:) (:122-168).
 *   ids_out  ids of the current segment decode (the returned "text")
 *   hit_eos  the decode ended on EOS          (nullable)
 *   emitted  the ids were appended to the emitted segments (nullable) */
ms_status ms_stream_transcribe(ms_stream* stream, int32_t is_final,
                               const ms_streaming_config* config, int32_t max_tokens,
                               int32_t* ids_out, int32_t cap, int32_t* n_out,
                               int32_t* hit_eos, int32_t* emitted);
/* getEmittedText(_:) (:171-173): ids of every emitted segment, each segment followed
 * by the separator id -1. */
ms_status ms_stream_emitted(ms_stream* stream, int32_t* ids_out, int32_t cap,
                            int32_t* n_out);
/* Frames currently in the segment's memory (StreamingState.memoryLen, :26-27). */
int32_t ms_stream_memory_len(const ms_stream* stream);
/* The segment's memory rows (StreamingState.memory, :25-26): memory_len x hidden floats into
 * memory_out (cap_floats of room; MS_ERR_CAPACITY, with *rows_out set, when it is too small). */
ms_status ms_stream_memory(ms_stream* stream, float* memory_out, int64_t cap_floats, int32_t* rows_out);

/* transcribe over many streams at once (no counterpart in the reference).  Each stream's
 * new frames are encoded on its own; with config->batch_decode == 0 each stream is then
 * decoded on its own (results equal ms_stream_transcribe on it alone), with 1 the
 * decodes of all streams that share one model run in lockstep (see batch_decode).
 * ids_out is [n * cap], n_out/hit_eos/emitted are [n] (hit_eos and emitted nullable). */
ms_status ms_stream_transcribe_batch(ms_stream* const* streams, int32_t n, int32_t is_final,
                                     const ms_streaming_config* config, int32_t max_tokens,
                                     int32_t* ids_out, int32_t cap, int32_t* n_out,
                                     int32_t* hit_eos, int32_t* emitted);

/* generateLong(audio:streamingConfig:) (MoonshineStreaming.swift:287-376): the whole
 * audio is encoded in one pass, then decoded in segments of at most max_memory_frames
 * memory rows with EOS-driven advance (an early EOS in a segment longer than
 * min_segment_frames moves the start by max(min_segment_frames, tokens / 6.5 * 50) frames).
 * ids_out receives the ids of every segment that produced tokens, each followed by the
 * separator -1 (the reference joins the non-empty segment texts).  stats->n_chunks is the
 * number of segments; stats->tokens_per_second holds audio seconds per wall second, as
 * the reference's generateLong reports it.  The audio's memory must fit the positional
 * table (max_position_embeddings frames). */
ms_status ms_generate_long(ms_model* model, const float* audio, int64_t n_samples,
                           const ms_streaming_config* config, int32_t* ids_out, int32_t cap,
                           int32_t* n_out, ms_gen_stats* stats);

/* ------------------------------------------------------------------- diagnostics */

/* Thread-local message of the last failing call on this thread ("" if none). */
const char* ms_last_error(void);

/* Number of kernel launches issued by this library on this thread since the last
 * reset (launch accounting for benchmarks). */
int64_t ms_kernel_launches(void);
void ms_reset_kernel_launches(void);

/* Phase trace of the batch-1 decode kernel (the device-side counterpart of the
 * reference's `profile:` timings, MoonshineModel.swift:167-175): when enabled, the next
 * decode records a %globaltimer stamp (ns) at its start and after every grid-wide phase
 * barrier; ms_decode_trace copies the stamps of the last decode. */
ms_status ms_enable_decode_trace(ms_model* model, int32_t enabled);
ms_status ms_decode_trace(ms_model* model, uint64_t* stamps_out, int32_t cap, int32_t* n_out);

/* Library version string. */
const char* ms_version(void);
/* sizeof of one of this header's structs by its name ("ms_options", "ms_model_config",
 * "ms_gen_params", "ms_gen_stats", "ms_alignment", "ms_streaming_config"), 0 for any other
 * name: a binding in another language checks its own layouts against it at load. */
size_t ms_struct_size(const char* name);

#ifdef __cplusplus
}
#endif

#endif /* MOONSHINE_B200_H */
