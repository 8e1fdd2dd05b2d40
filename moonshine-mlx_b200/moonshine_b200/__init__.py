"""Python mirror of the reference Swift API over the B200 C ABI (include/moonshine_b200.h).

Names follow kylehowells/moonshine-mlx's public surface
(Sources/MoonshineMLX/MoonshineModel.swift, MoonshineStreaming.swift):

    model = MoonshineModel.load(path)                  # MoonshineModel.load(from:)
    out = model.generate(audio)                        # generate(audio:maxTokens:...)
    model.enable_float16_kv_cache(False)               # enableFloat16KVCache(_:)
    st = model.create_stream(); model.start_stream(st) # createStream / startStream
    model.add_audio(st, chunk)                         # addAudio(_:chunk:)
    ids = model.transcribe(st, is_final=False)         # transcribe(_:isFinal:...)
    model.get_emitted(st)                              # getEmittedText(_:)

Token ids replace text (the tokenizer stays with the caller).  Every call goes through
the CUDA library; there is no CPU fallback -- importing this module fails loudly when
the library has not been built.
"""
from __future__ import annotations

import ctypes as C
import os
import weakref
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmoonshine_b200.so")

MS_OK = 0
MS_ERR_CAPACITY = 9
STATUS_NAMES = {0: "OK", 1: "INVALID_ARG", 2: "OOM", 3: "CUDA_ERROR", 4: "TIMEOUT",
                5: "BAD_WEIGHTS", 6: "BAD_CONFIG", 7: "NOT_FOUND", 8: "UNSUPPORTED",
                9: "CAPACITY"}
KV_F32, KV_F16 = 0, 1


class MoonshineError(RuntimeError):
    """Raised for every non-OK status (mirrors MoonshineError, ModelLoader.swift:187-203)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class _Options(C.Structure):
    _fields_ = [("device", C.c_int32), ("kv_dtype", C.c_int32), ("weight_dtype", C.c_int32),
                ("max_batch", C.c_int32), ("decode_kernel", C.c_int32), ("quant_stream", C.c_int32),
                ("reserved", C.c_int32 * 6)]


class _GenParams(C.Structure):
    _fields_ = [("max_tokens", C.c_int32), ("forced_len", C.c_int32),
                ("temperature", C.c_float), ("reserved_f", C.c_float),
                ("chunk_duration", C.c_double), ("teacher_ids", C.POINTER(C.c_int32)),
                ("n_teacher", C.c_int32), ("seed", C.c_int32),
                ("batch_logits", C.POINTER(C.c_float)), ("reserved", C.c_int32 * 4)]


DECODE_KERNEL_NAMES = {1: "grid", 2: "cluster"}


class _GenStats(C.Structure):
    _fields_ = [("n_tokens", C.c_int32), ("n_chunks", C.c_int32), ("hit_eos", C.c_int32),
                ("memory_frames", C.c_int32), ("decode_kernel", C.c_int32), ("encode_ms", C.c_double),
                ("decode_ms", C.c_double), ("total_ms", C.c_double),
                ("tokens_per_second", C.c_double)]


class _StreamingConfig(C.Structure):
    _fields_ = [("max_memory_frames", C.c_int32), ("min_segment_frames", C.c_int32),
                ("batch_decode", C.c_int32), ("temperature", C.c_float), ("seed", C.c_int32)]


class _Alignment(C.Structure):
    _fields_ = [("ids", C.POINTER(C.c_int32)), ("token_probs", C.POINTER(C.c_float)),
                ("jump_frames", C.POINTER(C.c_int32)), ("cap", C.c_int32), ("reserved0", C.c_int32),
                ("attn_rows", C.POINTER(C.c_float)), ("attn_filtered", C.POINTER(C.c_float)),
                ("attn_cap", C.c_int64), ("n_tokens", C.c_int32), ("n_steps", C.c_int32),
                ("n_frames", C.c_int32), ("hit_eos", C.c_int32)]


class _ModelConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
        "num_key_value_heads", "head_dim", "vocab_size", "max_position_embeddings",
        "tie_word_embeddings", "encoder_hidden_size", "enc_hidden_size",
        "enc_intermediate_size", "enc_num_hidden_layers", "enc_num_attention_heads",
        "enc_num_key_value_heads", "enc_head_dim", "enc_frame_len", "enc_sample_rate",
        "enc_max_position_embeddings", "bos_token_id", "eos_token_id",
        "decoder_start_token_id", "pad_token_id", "rotary_ndims")] + [
        ("rope_theta", C.c_float), ("max_tokens_per_second", C.c_double),
        ("num_sliding_windows", C.c_int32), ("sliding_windows", (C.c_int32 * 2) * 64)]


def _load_lib() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {os.path.dirname(_HERE)}`")
    lib = C.CDLL(LIB_PATH)
    P = C.c_void_p
    i32p = C.POINTER(C.c_int32)
    f32p = C.POINTER(C.c_float)
    sigs = {
        "ms_options_default": (None, [C.POINTER(_Options)]),
        "ms_gen_params_default": (None, [C.POINTER(_GenParams)]),
        "ms_streaming_config_default": (None, [C.POINTER(_StreamingConfig)]),
        "ms_model_load": (C.c_int, [C.c_char_p, C.POINTER(_Options), C.POINTER(P)]),
        "ms_model_free": (None, [P]),
        "ms_model_enable_fp16_kv_cache": (C.c_int, [P, C.c_int32]),
        "ms_model_sample_rate": (C.c_int32, [P]),
        "ms_model_decode_weight_bits": (C.c_int32, [P, C.POINTER(C.c_int32)]),
        "ms_model_get_config": (C.c_int, [P, C.POINTER(_ModelConfig)]),
        "ms_generate": (C.c_int, [P, f32p, C.c_int64, C.POINTER(_GenParams), i32p, C.c_int32,
                                  i32p, f32p, C.POINTER(_GenStats)]),
        "ms_generate_long": (C.c_int, [P, f32p, C.c_int64, C.POINTER(_StreamingConfig), i32p, C.c_int32,
                                       i32p, C.POINTER(_GenStats)]),
        "ms_generate_batch": (C.c_int, [P, C.POINTER(f32p), C.POINTER(C.c_int64), C.c_int32,
                                        C.POINTER(_GenParams), i32p, C.c_int32, i32p,
                                        C.POINTER(_GenStats)]),
        "ms_generate_device": (C.c_int, [P, C.c_void_p, C.c_int64, C.POINTER(_GenParams), C.c_void_p,
                                         C.c_int32, i32p, C.POINTER(_GenStats)]),
        "ms_generate_alignment": (C.c_int, [P, f32p, C.c_int64, C.c_int32, C.c_int32, C.POINTER(_Alignment),
                                            C.POINTER(_GenStats)]),
        "ms_word_timings": (C.c_int, [i32p, C.c_int32, f32p, C.c_int32, i32p, C.c_int32, C.c_int32, C.c_int32,
                                      C.c_double, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                      C.POINTER(C.c_double), i32p]),
        "ms_alignment_jump_frames": (C.c_int, [f32p, C.c_int32, C.c_int32, i32p]),
        "ms_model_stream": (C.c_void_p, [P]),
        "ms_stream_add_audio_batch": (C.c_int, [C.POINTER(C.c_void_p), C.c_int32, C.POINTER(C.POINTER(C.c_float)),
                                          C.POINTER(C.c_int64)]),
        "ms_model_batch_kv_pages": (C.c_int, [P, C.POINTER(C.c_int64), C.POINTER(C.c_int64), C.POINTER(C.c_int32)]),
        "ms_decode_memory_static": (C.c_int, [P, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                              i32p, i32p]),
        "ms_encode": (C.c_int, [P, f32p, C.c_int64, f32p, C.c_int64, i32p]),
        "ms_stream_create": (C.c_int, [P, C.POINTER(P)]),
        "ms_stream_free": (None, [P]),
        "ms_stream_start": (C.c_int, [P]),
        "ms_stream_stop": (C.c_int, [P]),
        "ms_stream_add_audio": (C.c_int, [P, f32p, C.c_int64]),
        "ms_stream_transcribe": (C.c_int, [P, C.c_int32, C.POINTER(_StreamingConfig), C.c_int32,
                                           i32p, C.c_int32, i32p, i32p, i32p]),
        "ms_stream_transcribe_batch": (C.c_int, [C.POINTER(P), C.c_int32, C.c_int32,
                                                 C.POINTER(_StreamingConfig), C.c_int32, i32p,
                                                 C.c_int32, i32p, i32p, i32p]),
        "ms_stream_emitted": (C.c_int, [P, i32p, C.c_int32, i32p]),
        "ms_stream_memory_len": (C.c_int32, [P]),
        "ms_stream_memory": (C.c_int, [P, C.POINTER(C.c_float), C.c_int64, i32p]),
        "ms_enable_decode_trace": (C.c_int, [P, C.c_int32]),
        "ms_decode_trace": (C.c_int, [P, C.POINTER(C.c_uint64), C.c_int32, i32p]),
        "ms_last_error": (C.c_char_p, []),
        "ms_kernel_launches": (C.c_int64, []),
        "ms_reset_kernel_launches": (None, []),
        "ms_version": (C.c_char_p, []),
        "ms_struct_size": (C.c_size_t, [C.c_char_p]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    # the structs passed by pointer must have the library's layout
    for cname, cls in (("ms_options", _Options), ("ms_model_config", _ModelConfig), ("ms_gen_params", _GenParams),
                       ("ms_gen_stats", _GenStats), ("ms_alignment", _Alignment),
                       ("ms_streaming_config", _StreamingConfig)):
        if lib.ms_struct_size(cname.encode()) != C.sizeof(cls):
            raise ImportError(f"{cname}: {C.sizeof(cls)} bytes here, {lib.ms_struct_size(cname.encode())} in "
                              f"{LIB_PATH} (a library built from another header)")
    return lib


_lib: Optional[C.CDLL] = None


def _L() -> C.CDLL:
    """The CUDA library, loaded on first use (importing `synth` needs no build)."""
    global _lib
    if _lib is None:
        _lib = _load_lib()
    return _lib


def _check(status: int) -> None:
    if status != MS_OK:
        raise MoonshineError(status, _L().ms_last_error().decode(errors="replace"))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32).reshape(-1))


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _iptr(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


@dataclass
class TranscriptionOutput:
    """TranscriptionOutput (MoonshineModel.swift:8-14) with token ids in place of text."""
    tokens: List[int]
    generation_tokens: int
    total_time: float
    tokens_per_second: float
    encode_ms: float = 0.0
    decode_ms: float = 0.0
    hit_eos: bool = False
    memory_frames: int = 0
    decode_kernel: str = ""   # batch-1 kernel of the last chunk: "grid" or "cluster"
    logits: Optional[np.ndarray] = None
    text: str = ""            # generate_with_word_timestamps: decoded text (caller's tokenizer)
    segments: list = field(default_factory=list)


@dataclass
class WordTiming:
    """WordTiming (MoonshineTimestamps.swift:9-15)."""
    word: str
    tokens: List[int]
    start: float
    end: float
    probability: float


@dataclass
class TranscriptionSegment:
    """TranscriptionSegment (MoonshineModel.swift:16-21)."""
    text: str
    start: float
    end: float
    words: List[WordTiming] = field(default_factory=list)


@dataclass
class Alignment:
    """Everything ms_generate_alignment returns: ids (EOS excluded), one probability and
    one jump frame per decoder call, and optionally the attention rows."""
    ids: List[int]
    token_probs: np.ndarray
    jump_frames: np.ndarray
    n_frames: int
    hit_eos: bool
    attn_rows: Optional[np.ndarray] = None
    attn_filtered: Optional[np.ndarray] = None
    stats: Optional[object] = None


def _default_piece(t: int) -> str:
    return ""


def _default_decode(ids: Sequence[int]) -> str:
    # the reference's decodeTokens without a tokenizer (MoonshineModel.swift:320-327)
    return "".join(chr(t) if t < 128 else f"<{t}>" for t in ids)


def alignment_jump_frames(filtered: np.ndarray) -> np.ndarray:
    """DTW jump frames of z-scored, median-filtered attention rows [n_rows, n_frames]
    (host-side step of findAlignment, MoonshineTimestamps.swift:148-184)."""
    f = np.ascontiguousarray(filtered, dtype=np.float32)
    n, m = (f.shape if f.ndim == 2 else (0, 0))
    out = np.zeros(max(n, 1), dtype=np.int32)
    _check(_L().ms_alignment_jump_frames(_fptr(f), n, m, _iptr(out)))
    return out[: (n if m > 0 else 0)]


def word_timings(alignment: "Alignment", token_to_string: Optional[Callable[[int], Optional[str]]] = None,
                 decode_tokens: Optional[Callable[[Sequence[int]], str]] = None,
                 time_offset: float = 0.0) -> List[WordTiming]:
    """Word grouping of findAlignment (MoonshineTimestamps.swift:154-173): a word starts at
    every token whose piece begins with U+2581; the timing arithmetic runs in the library
    (ms_word_timings)."""
    piece = token_to_string or _default_piece
    dec = decode_tokens or _default_decode
    toks = alignment.ids
    if not toks:
        return []
    first: List[int] = []
    for i, t in enumerate(toks):
        p = piece(t) or ""
        if not first or (p.startswith("\u2581") and i > first[-1]):
            first.append(i)
    nw = len(first)
    wf = np.asarray(first, dtype=np.int32)
    jf = np.ascontiguousarray(alignment.jump_frames, dtype=np.int32)
    pr = np.ascontiguousarray(alignment.token_probs, dtype=np.float32)
    st, en, pb = (np.zeros(nw, dtype=np.float64) for _ in range(3))
    n = C.c_int32()
    dp = C.POINTER(C.c_double)
    _check(_L().ms_word_timings(_iptr(jf), jf.shape[0], _fptr(pr), pr.shape[0], _iptr(wf), nw, len(toks),
                                int(alignment.n_frames), float(time_offset), st.ctypes.data_as(dp),
                                en.ctypes.data_as(dp), pb.ctypes.data_as(dp), C.byref(n)))
    out = []
    for w in range(n.value):
        lo = first[w]
        hi = first[w + 1] if w + 1 < nw else len(toks)
        ids = toks[lo:hi]
        out.append(WordTiming(word=dec(ids).strip(" "), tokens=list(ids), start=float(st[w]), end=float(en[w]),
                              probability=float(pb[w])))
    return out


@dataclass
class StreamingConfig:
    """StreamingConfig (MoonshineStreaming.swift:47-62)."""
    max_memory_frames: int = 100000
    min_segment_frames: int = 250
    # transcribe_batch: 1 (or True) encodes all streams' new frames in one tensor-core pass,
    # each encoder layer over the rows that can have changed since the stream's previous call,
    # and decodes in lockstep; 2 the same but re-encoding each stream's whole window, as the
    # reference does (same memory rows to rounding)
    batch_decode: int = 0

    def _c(self, temperature: float = 0.0, seed: int = 0) -> _StreamingConfig:
        return _StreamingConfig(self.max_memory_frames, self.min_segment_frames, int(self.batch_decode),
                                float(temperature), int(seed) & 0x7FFFFFFF)


class StreamingState:
    """Opaque handle over ms_stream (StreamingState, MoonshineStreaming.swift:8-43)."""

    def __init__(self, handle, model: "MoonshineModel"):
        self._h = handle
        self._model = model  # keeps the model alive while the stream exists
        self.last_hit_eos = False

    @property
    def memory_len(self) -> int:
        return int(_L().ms_stream_memory_len(self._h))

    def memory(self) -> np.ndarray:
        """The segment's memory rows (StreamingState.memory, MoonshineStreaming.swift:25-26),
        [memory_len, hidden] float32."""
        hidden = self._model.config.hidden_size
        out = np.zeros((max(self.memory_len, 0), hidden), dtype=np.float32)
        rows = C.c_int32()
        _check(_L().ms_stream_memory(self._h, _fptr(out), out.size, C.byref(rows)))
        return out[: rows.value]

    def close(self):
        # a stream is freed before its model (MoonshineModel.close frees the live ones first)
        if self._h and self._model._h:
            _L().ms_stream_free(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MoonshineModel:
    def __init__(self, handle):
        self._h = handle
        self._streams = weakref.WeakSet()  # live streams, freed before the model
        cfg = _ModelConfig()
        _check(_L().ms_model_get_config(self._h, C.byref(cfg)))
        self.config = cfg

    @staticmethod
    def load(path: str, device: int = 0, kv_fp16: bool = True, decode_kernel: str = "auto",
             weight_dtype: str = "auto", quant_stream: str = "auto") -> "MoonshineModel":
        """MoonshineModel.load(from:) for a local directory (MoonshineModel.swift:409-414).

        ``decode_kernel`` picks the batch-1 decode kernel: "auto" or "cluster" (one 8-CTA
        cluster per head when the dims and the GPU allow it, else single-grid) or "grid"
        (single-grid persistent kernel).  ``weight_dtype`` ("auto", "f32", "bf16") is
        ms_weight_dtype: "f32" also makes the clustered kernel stream a quantized
        checkpoint's rows dequantized instead of as codes.  ``quant_stream`` ("auto", "all",
        "lm", "none") is MS_QSTREAM_*: which weights of a quantized checkpoint the clustered
        kernel streams as codes."""
        kinds = {"auto": 0, "grid": 1, "cluster": 2}
        if decode_kernel not in kinds:
            raise ValueError("decode_kernel must be one of " + ", ".join(kinds))
        wkinds = {"auto": 0, "f32": 1, "bf16": 2}
        if weight_dtype not in wkinds:
            raise ValueError("weight_dtype must be one of " + ", ".join(wkinds))
        o = _Options()
        _L().ms_options_default(C.byref(o))
        o.device = device
        o.kv_dtype = KV_F16 if kv_fp16 else KV_F32
        o.decode_kernel = kinds[decode_kernel]
        o.weight_dtype = wkinds[weight_dtype]
        qkinds = {"auto": 0, "all": 1, "lm": 2, "none": 3}
        if quant_stream not in qkinds:
            raise ValueError("quant_stream must be one of " + ", ".join(qkinds))
        o.quant_stream = qkinds[quant_stream]
        h = C.c_void_p()
        _check(_L().ms_model_load(path.encode(), C.byref(o), C.byref(h)))
        return MoonshineModel(h)

    def close(self):
        if self._h:
            for st in list(self._streams):
                st.close()
            _L().ms_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def sample_rate(self) -> int:
        return int(_L().ms_model_sample_rate(self._h))

    @property
    def decode_weight_bits(self) -> Tuple[int, int]:
        """(bits of the q|k|v / cross q / fc1 rows, bits of the LM-head rows) that the
        clustered batch-1 kernel streams as quantized codes; 0 = fp32 rows."""
        lm = C.c_int32()
        rows = int(_L().ms_model_decode_weight_bits(self._h, C.byref(lm)))
        return rows, int(lm.value)

    def enable_float16_kv_cache(self, enabled: bool) -> None:
        _check(_L().ms_model_enable_fp16_kv_cache(self._h, 1 if enabled else 0))

    def _params(self, max_tokens, temperature, chunk_duration, forced_len, teacher, seed=0):
        p = _GenParams()
        _L().ms_gen_params_default(C.byref(p))
        p.max_tokens = 0 if max_tokens is None else int(max_tokens)
        p.forced_len = 0 if forced_len is None else int(forced_len)
        p.temperature = float(temperature)
        p.seed = int(seed) & 0x7FFFFFFF
        p.chunk_duration = float(chunk_duration)
        if teacher is not None:
            p.teacher_ids = _iptr(teacher)
            p.n_teacher = int(teacher.shape[0])
        return p

    def generate(self, audio, max_tokens: Optional[int] = None, temperature: float = 0.0,
                 chunk_duration: float = 30.0, forced_len: Optional[int] = None,
                 teacher_ids: Optional[Sequence[int]] = None,
                 return_logits: bool = False, seed: int = 0) -> TranscriptionOutput:
        """MoonshineModel.generate (MoonshineModel.swift:130-184); temperature > 0 samples
        (MLXRandom.categorical of logits / temperature) with draws keyed by ``seed``."""
        a = _f32(audio)
        sr = self.sample_rate
        chunk = int(chunk_duration * sr)
        n_chunks = max(1, -(-a.shape[0] // chunk)) if a.shape[0] else 0
        per_chunk = forced_len if forced_len and forced_len > 0 else int(np.ceil(min(chunk, a.shape[0]) / sr * 6.5)) + 1
        if max_tokens:
            per_chunk = min(per_chunk, max_tokens) if not forced_len else per_chunk
        cap = max(1, n_chunks * per_chunk + 1)
        teacher = None if teacher_ids is None else np.ascontiguousarray(teacher_ids, dtype=np.int32)
        p = self._params(max_tokens, temperature, chunk_duration, forced_len, teacher, seed)
        V = self.config.vocab_size
        while True:
            ids = np.zeros(cap, dtype=np.int32)
            logits = np.zeros((cap, V), dtype=np.float32) if return_logits else None
            n = C.c_int32()
            st = _GenStats()
            s = _L().ms_generate(self._h, _fptr(a), a.shape[0], C.byref(p), _iptr(ids), cap,
                                C.byref(n), _fptr(logits) if logits is not None else None,
                                C.byref(st))
            if s == MS_ERR_CAPACITY and n.value > cap:
                cap = n.value + 1
                continue
            _check(s)
            break
        out = TranscriptionOutput(tokens=ids[: n.value].tolist(), generation_tokens=n.value,
                                  total_time=st.total_ms / 1000.0,
                                  tokens_per_second=st.tokens_per_second,
                                  encode_ms=st.encode_ms, decode_ms=st.decode_ms,
                                  hit_eos=bool(st.hit_eos), memory_frames=st.memory_frames,
                                  decode_kernel=DECODE_KERNEL_NAMES.get(st.decode_kernel, ""))
        if return_logits:
            out.logits = logits
        return out

    def generate_long(self, audio, streaming_config: Optional["StreamingConfig"] = None):
        """generateLong (MoonshineStreaming.swift:287-376): returns (segments, output) where
        segments are the id lists of the segments that produced tokens and output carries
        the timings (its tokens_per_second is audio seconds per wall second, as in the
        reference)."""
        a = _f32(audio)
        sc = (streaming_config or StreamingConfig())._c()
        cap = max(16, int(np.ceil(a.shape[0] / self.sample_rate * 6.5)) * 4 + 64)
        while True:
            ids = np.zeros(cap, dtype=np.int32)
            n = C.c_int32()
            st = _GenStats()
            s = _L().ms_generate_long(self._h, _fptr(a), a.shape[0], C.byref(sc), _iptr(ids), cap,
                                      C.byref(n), C.byref(st))
            if s == MS_ERR_CAPACITY and n.value > cap:
                cap = n.value + 1
                continue
            _check(s)
            break
        segments, cur = [], []
        for t in ids[: n.value].tolist():
            if t == -1:
                segments.append(cur)
                cur = []
            else:
                cur.append(t)
        out = TranscriptionOutput(tokens=[t for seg in segments for t in seg], generation_tokens=len(segments),
                                  total_time=st.total_ms / 1000.0, tokens_per_second=st.tokens_per_second,
                                  encode_ms=st.encode_ms, decode_ms=st.decode_ms, hit_eos=bool(st.hit_eos),
                                  memory_frames=st.memory_frames,
                                  decode_kernel=DECODE_KERNEL_NAMES.get(st.decode_kernel, ""))
        return segments, out

    def generate_device(self, audio_dev_ptr: int, n_samples: int, ids_dev_ptr: int, cap: int,
                        forced_len: Optional[int] = None, max_tokens: Optional[int] = None,
                        chunk_duration: float = 30.0):
        """ms_generate_device: audio and ids stay in device memory.  Returns (n, stats)."""
        p = self._params(max_tokens, 0.0, chunk_duration, forced_len, None)
        n = C.c_int32()
        st = _GenStats()
        _check(_L().ms_generate_device(self._h, C.c_void_p(audio_dev_ptr), int(n_samples), C.byref(p),
                                       C.c_void_p(ids_dev_ptr), int(cap), C.byref(n), C.byref(st)))
        return n.value, st

    def enable_decode_trace(self, enabled: bool = True) -> None:
        _check(_L().ms_enable_decode_trace(self._h, 1 if enabled else 0))

    def decode_trace(self) -> np.ndarray:
        """%globaltimer stamps (ns) of the last traced decode: start, then one per barrier."""
        n = C.c_int32()
        _L().ms_decode_trace(self._h, None, 0, C.byref(n))
        buf = np.zeros(max(n.value, 1), dtype=np.uint64)
        _check(_L().ms_decode_trace(self._h, buf.ctypes.data_as(C.POINTER(C.c_uint64)), buf.shape[0],
                                    C.byref(n)))
        return buf[: n.value]

    def decode_memory_static(self, memory_dev_ptr: int, frames: int, ids_dev_ptr: int, n_tokens: int,
                             forced: bool = True):
        """ms_decode_memory_static: decode without any device allocation, from memory rows
        in device memory into a device ids buffer.  Returns (n_ids, hit_eos)."""
        n, hit = C.c_int32(), C.c_int32()
        _check(_L().ms_decode_memory_static(self._h, C.c_void_p(memory_dev_ptr), int(frames), int(n_tokens),
                                            1 if forced else 0, C.c_void_p(ids_dev_ptr), C.byref(n),
                                            C.byref(hit)))
        return n.value, bool(hit.value)

    def batch_kv_pages(self):
        """(pages the last batched call assigned, pages the pool holds, positions per page)."""
        u, c, p = C.c_int64(), C.c_int64(), C.c_int32()
        _check(_L().ms_model_batch_kv_pages(self._h, C.byref(u), C.byref(c), C.byref(p)))
        return u.value, c.value, p.value

    @property
    def cuda_stream(self) -> int:
        """cudaStream_t the model's work is enqueued on (as an integer handle)."""
        return int(_L().ms_model_stream(self._h) or 0)

    def generate_batch(self, audios: Sequence[np.ndarray], max_tokens: Optional[int] = None,
                       forced_len: Optional[int] = None, chunk_duration: float = 30.0,
                       return_logits: bool = False, temperature: float = 0.0, seed: int = 0):
        """Batched offline generation.  Returns (ids per utterance, stats[, logits
        [B, cap, vocab] of every decoder call])."""
        arrs = [_f32(a) for a in audios]
        B = len(arrs)
        sr = self.sample_rate
        longest = max((a.shape[0] for a in arrs), default=0)
        n_chunks = max(1, -(-longest // int(chunk_duration * sr)))
        per = forced_len if forced_len and forced_len > 0 else int(np.ceil(min(longest, chunk_duration * sr) / sr * 6.5)) + 1
        cap = n_chunks * per + 1
        ptrs = (C.POINTER(C.c_float) * B)(*[_fptr(a) for a in arrs])
        lens = (C.c_int64 * B)(*[a.shape[0] for a in arrs])
        ids = np.zeros((B, cap), dtype=np.int32)
        n = np.zeros(B, dtype=np.int32)
        p = self._params(max_tokens, temperature, chunk_duration, forced_len, None, seed)
        logits = None
        if return_logits:
            logits = np.zeros((B, cap, self.config.vocab_size), dtype=np.float32)
            p.batch_logits = _fptr(logits)
        st = _GenStats()
        _check(_L().ms_generate_batch(self._h, ptrs, lens, B, C.byref(p), _iptr(ids), cap,
                                     _iptr(n), C.byref(st)))
        out = [ids[b, : n[b]].tolist() for b in range(B)]
        return (out, st, logits) if return_logits else (out, st)

    def generate_alignment(self, audio, max_tokens: Optional[int] = None, medfilt_width: int = 7,
                           return_attention: bool = False) -> Alignment:
        """The GPU part of generateWithWordTimestamps (MoonshineModel.swift:241-316): one
        encode of the whole audio, greedy decode keeping every call's cross-attention
        queries, the attention rows (z-scored and median-filtered) and their DTW jump frames."""
        a = _f32(audio)
        sr = self.sample_rate
        cap = int(np.ceil(a.shape[0] / sr * self.config.max_tokens_per_second)) + 2
        if max_tokens:
            cap = min(cap, int(max_tokens) + 2)
        cap = max(cap, 1)
        frames = a.shape[0] // self.config.enc_frame_len // 4 + 2
        ids = np.zeros(cap, dtype=np.int32)
        probs = np.zeros(cap, dtype=np.float32)
        jumps = np.zeros(cap, dtype=np.int32)
        al = _Alignment()
        al.ids, al.token_probs, al.jump_frames, al.cap = _iptr(ids), _fptr(probs), _iptr(jumps), cap
        rows = filt = None
        if return_attention:
            rows = np.zeros(cap * frames, dtype=np.float32)
            filt = np.zeros(cap * frames, dtype=np.float32)
            al.attn_rows, al.attn_filtered, al.attn_cap = _fptr(rows), _fptr(filt), rows.shape[0]
        st = _GenStats()
        _check(_L().ms_generate_alignment(self._h, _fptr(a), a.shape[0], 0 if max_tokens is None else int(max_tokens),
                                          int(medfilt_width), C.byref(al), C.byref(st)))
        ns, M = al.n_steps, al.n_frames
        out = Alignment(ids=ids[: al.n_tokens].tolist(), token_probs=probs[:ns].copy(),
                        jump_frames=jumps[: (ns if al.n_tokens else 0)].copy(), n_frames=M,
                        hit_eos=bool(al.hit_eos), stats=st)
        if return_attention:
            out.attn_rows = rows[: ns * M].reshape(ns, M).copy()
            out.attn_filtered = filt[: ns * M].reshape(ns, M).copy()
        return out

    def generate_with_word_timestamps(self, audio, max_tokens: Optional[int] = None, time_offset: float = 0.0,
                                      token_to_string: Optional[Callable[[int], Optional[str]]] = None,
                                      decode_tokens: Optional[Callable[[Sequence[int]], str]] = None):
        """generateWithWordTimestamps(audio:maxTokens:timeOffset:) (MoonshineModel.swift:241-316).
        Returns (TranscriptionOutput, [WordTiming]); the output's ``segments`` holds one
        TranscriptionSegment over the whole audio."""
        a = _f32(audio)
        al = self.generate_alignment(a, max_tokens)
        words = word_timings(al, token_to_string, decode_tokens, time_offset)
        dec = decode_tokens or _default_decode
        text = dec(al.ids).strip(" ")
        st = al.stats
        dur = a.shape[0] / float(self.sample_rate)
        out = TranscriptionOutput(tokens=al.ids, generation_tokens=len(al.ids), total_time=st.total_ms / 1000.0,
                                  tokens_per_second=st.tokens_per_second, encode_ms=st.encode_ms,
                                  decode_ms=st.decode_ms, hit_eos=al.hit_eos, memory_frames=al.n_frames,
                                  decode_kernel=DECODE_KERNEL_NAMES.get(st.decode_kernel, ""))
        out.text = text
        out.segments = [TranscriptionSegment(text=text, start=0.0, end=dur, words=words)]
        return out, words

    def encode(self, audio) -> np.ndarray:
        """Memory = prepareMemory(encoder(embedder(audio))) for one chunk, [frames, hidden]."""
        a = _f32(audio)
        d = self.config.hidden_size
        cap = (a.shape[0] // self.config.enc_frame_len // 4 + 2) * d
        out = np.zeros(max(cap, d), dtype=np.float32)
        nf = C.c_int32()
        _check(_L().ms_encode(self._h, _fptr(a), a.shape[0], _fptr(out), out.shape[0], C.byref(nf)))
        return out[: nf.value * d].reshape(nf.value, d)

    # ---------------------------------------------------------------- streaming
    def create_stream(self) -> StreamingState:
        h = C.c_void_p()
        _check(_L().ms_stream_create(self._h, C.byref(h)))
        st = StreamingState(h, self)
        self._streams.add(st)
        return st

    def start_stream(self, state: StreamingState) -> None:
        _check(_L().ms_stream_start(state._h))

    def stop_stream(self, state: StreamingState) -> None:
        _check(_L().ms_stream_stop(state._h))

    def add_audio(self, state: StreamingState, chunk) -> None:
        a = _f32(chunk)
        _check(_L().ms_stream_add_audio(state._h, _fptr(a), a.shape[0]))

    def add_audio_batch(self, states: Sequence[StreamingState], chunks: Sequence) -> None:
        """add_audio of chunks[i] to states[i] for every i in one call (the frontends of all the
        streams of this model run as one batched pass: one upload, five launches)."""
        arrs = [_f32(c) for c in chunks]
        if len(arrs) != len(states):
            raise ValueError("one chunk per stream")
        B = len(arrs)
        hs = (C.c_void_p * B)(*[s._h for s in states])
        ptrs = (C.POINTER(C.c_float) * B)(*[_fptr(a) for a in arrs])
        lens = (C.c_int64 * B)(*[a.shape[0] for a in arrs])
        _check(_L().ms_stream_add_audio_batch(hs, B, ptrs, lens))

    def transcribe(self, state: StreamingState, is_final: bool = False,
                   streaming_config: Optional[StreamingConfig] = None,
                   max_tokens: Optional[int] = None, temperature: float = 0.0, seed: int = 0):
        """transcribe (MoonshineStreaming.swift:122-168).  Returns (ids, hit_eos, emitted);
        temperature > 0 samples (MLXRandom.categorical of logits / temperature) with draws
        keyed by ``seed`` and the stream's call count."""
        sc = (streaming_config or StreamingConfig())._c(temperature, seed)
        cap = max(16, int(np.ceil(state.memory_len * 0.02 * 6.5)) + 64)
        while True:
            ids = np.zeros(cap, dtype=np.int32)
            n, hit, em = C.c_int32(), C.c_int32(), C.c_int32()
            s = _L().ms_stream_transcribe(state._h, 1 if is_final else 0, C.byref(sc),
                                         0 if max_tokens is None else int(max_tokens),
                                         _iptr(ids), cap, C.byref(n), C.byref(hit), C.byref(em))
            if s == MS_ERR_CAPACITY:
                raise MoonshineError(s, "transcribe ids buffer too small")
            _check(s)
            break
        state.last_hit_eos = bool(hit.value)
        return ids[: n.value].tolist(), bool(hit.value), bool(em.value)

    def transcribe_batch(self, states: Sequence[StreamingState], is_final: bool = False,
                         streaming_config: Optional[StreamingConfig] = None,
                         max_tokens: Optional[int] = None, temperature: float = 0.0, seed: int = 0):
        B = len(states)
        sc = (streaming_config or StreamingConfig())._c(temperature, seed)
        cap = max(16, max((int(np.ceil(s.memory_len * 0.02 * 6.5)) for s in states), default=0) + 64)
        hs = (C.c_void_p * B)(*[s._h for s in states])
        ids = np.zeros((B, cap), dtype=np.int32)
        n = np.zeros(B, dtype=np.int32)
        hit = np.zeros(B, dtype=np.int32)
        em = np.zeros(B, dtype=np.int32)
        _check(_L().ms_stream_transcribe_batch(hs, B, 1 if is_final else 0, C.byref(sc),
                                              0 if max_tokens is None else int(max_tokens),
                                              _iptr(ids), cap, _iptr(n), _iptr(hit), _iptr(em)))
        return [(ids[b, : n[b]].tolist(), bool(hit[b]), bool(em[b])) for b in range(B)]

    def get_emitted(self, state: StreamingState) -> List[List[int]]:
        """getEmittedText (MoonshineStreaming.swift:171-173) as id segments."""
        cap = 1024
        while True:
            buf = np.zeros(cap, dtype=np.int32)
            n = C.c_int32()
            s = _L().ms_stream_emitted(state._h, _iptr(buf), cap, C.byref(n))
            if s == MS_ERR_CAPACITY:
                cap = n.value + 1
                continue
            _check(s)
            break
        segs, cur = [], []
        for t in buf[: n.value].tolist():
            if t == -1:
                segs.append(cur)
                cur = []
            else:
                cur.append(t)
        return segs


def kernel_launches() -> int:
    return int(_L().ms_kernel_launches())


def reset_kernel_launches() -> None:
    _L().ms_reset_kernel_launches()
