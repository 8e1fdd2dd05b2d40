"""CPU oracle for the Moonshine V2 streaming hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic of kylehowells/moonshine-mlx for the
path the CUDA library implements: the audio frontend, the sliding-window encoder, memory
preparation, the decoder step with its fp32 / fp16 KV-cache rounding rules, the greedy
token loop and the streaming state machine.  Each function cites the reference
file:line it follows (paths inside the reference project).

Only the test suite, the smoke check and the CPU-baseline leg of the benchmark may
import it, and only as the outputs to compare against or as the timed CPU restatement.
The product path never calls it.

Parity status: UNPINNED against the reference itself.  The reference is a Swift package
over mlx-swift 0.30.6 (Package.resolved:23-28); neither Swift nor MLX can run where this
library is built, and the reference ships no golden vectors or tests.  The restatement is
instead cross-checked against HuggingFace ``transformers``' MoonshineStreaming model (an
independent third-party implementation of the same architecture that reads the same
checkpoint layout) through fixtures under tests/golden/ made by
tests/golden/make_golden.py.  That cross-check covers fp32-KV decoding only; the fp16
KV rounding rules and the streaming state machine are reference-specific and rest on
this restatement alone.

dtype: ``np.float64`` (default) is the parity oracle; ``np.float32`` is the timed CPU
baseline (numpy over multi-threaded OpenBLAS).
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np


# ----------------------------------------------------------------------------- config

@dataclass
class EncoderConfig:
    """Sources/MoonshineMLX/MoonshineConfig.swift:5-57."""
    hidden_size: int = 320
    intermediate_size: int = 1280
    num_hidden_layers: int = 6
    num_attention_heads: int = 8
    num_key_value_heads: int = 8
    head_dim: int = 40
    frame_ms: float = 5.0
    sample_rate: int = 16000
    max_position_embeddings: int = 4096
    sliding_windows: Optional[List[List[int]]] = None

    @property
    def frame_len(self) -> int:  # MoonshineConfig.swift:17
        return int(self.frame_ms * self.sample_rate / 1000.0)

    @staticmethod
    def from_dict(d: dict) -> "EncoderConfig":  # MoonshineConfig.swift:43-56
        return EncoderConfig(
            hidden_size=d.get("hidden_size", 320),
            intermediate_size=d.get("intermediate_size", 1280),
            num_hidden_layers=d.get("num_hidden_layers", 6),
            num_attention_heads=d.get("num_attention_heads", 8),
            num_key_value_heads=d.get("num_key_value_heads", 8),
            head_dim=d.get("head_dim", 40),
            frame_ms=float(d.get("frame_ms", 5.0)),
            sample_rate=d.get("sample_rate", 16000),
            max_position_embeddings=d.get("max_position_embeddings", 4096),
            sliding_windows=d.get("sliding_windows"),
        )


@dataclass
class ModelConfig:
    """Sources/MoonshineMLX/MoonshineConfig.swift:61-178."""
    hidden_size: int = 320
    intermediate_size: int = 1280
    num_hidden_layers: int = 6
    num_attention_heads: int = 8
    num_key_value_heads: int = 8
    head_dim: int = 40
    vocab_size: int = 32768
    max_position_embeddings: int = 4096
    tie_word_embeddings: bool = False
    encoder_hidden_size: int = 320
    encoder: EncoderConfig = field(default_factory=EncoderConfig)
    bos_token_id: int = 1
    eos_token_id: int = 2
    decoder_start_token_id: int = 1
    pad_token_id: int = 0
    partial_rotary_factor: float = 0.8
    rope_theta: float = 10000.0
    max_tokens_per_second: float = 6.5

    @staticmethod
    def from_dict(d: dict) -> "ModelConfig":  # MoonshineConfig.swift:134-177
        hidden = d.get("hidden_size", 320)
        L = d.get("num_hidden_layers", 6)
        H = d.get("num_attention_heads", 8)
        KVH = d.get("num_key_value_heads", 8)
        hd = d.get("head_dim", 40)
        enc_hidden = d.get("encoder_hidden_size")
        if isinstance(d.get("encoder_config"), dict):
            enc = EncoderConfig.from_dict(d["encoder_config"])
        else:  # MoonshineConfig.swift:115-122
            eh = enc_hidden if enc_hidden is not None else hidden
            enc = EncoderConfig(hidden_size=eh, intermediate_size=eh * 4, num_hidden_layers=L,
                                num_attention_heads=H, num_key_value_heads=KVH, head_dim=hd)
        prf = d.get("partial_rotary_factor", 0.8)
        theta = d.get("rope_theta", 10000.0)
        rp = d.get("rope_parameters")
        if isinstance(rp, dict):  # MoonshineConfig.swift:142-145
            prf = rp.get("partial_rotary_factor", prf)
            theta = rp.get("rope_theta", theta)
        dst = d.get("decoder_start_token_id")
        return ModelConfig(
            hidden_size=hidden,
            intermediate_size=d.get("intermediate_size", 1280),
            num_hidden_layers=L, num_attention_heads=H, num_key_value_heads=KVH, head_dim=hd,
            vocab_size=d.get("vocab_size", 32768),
            max_position_embeddings=d.get("max_position_embeddings", 4096),
            tie_word_embeddings=bool(d.get("tie_word_embeddings", False)),
            encoder_hidden_size=enc_hidden if enc_hidden is not None else enc.hidden_size,
            encoder=enc,
            bos_token_id=d.get("bos_token_id", 1), eos_token_id=d.get("eos_token_id", 2),
            decoder_start_token_id=dst if isinstance(dst, int) else 1,
            pad_token_id=d.get("pad_token_id", 0),
            partial_rotary_factor=float(prf), rope_theta=float(theta),
            max_tokens_per_second=float(d.get("max_tokens_per_second", 6.5)),
        )

    @property
    def rotary_ndims(self) -> int:  # MoonshineLayers.swift:54-60
        nd = int(self.head_dim * self.partial_rotary_factor)
        return nd - nd % 2


# ----------------------------------------------------------------------------- weights

def sanitize_weights(w: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    """ModelLoader.swift:75-101: strip ``model.``, ``.gamma`` -> ``.weight``.  Conv
    weights stay in PyTorch [out, in, k] order here (the reference transposes them to
    MLX's [out, k, in]; the conv below indexes [out, in, k] directly)."""
    hf = any(k.startswith("model.") for k in w)
    out = {}
    for k, v in w.items():
        if hf:
            if k.startswith("model."):
                k = k[6:]
            k = k.replace(".gamma", ".weight")
        elif "conv" in k and k.endswith(".weight") and v.ndim == 3:
            v = np.transpose(v, (0, 2, 1))  # MLX [out,k,in] -> [out,in,k]
        out[k] = v
    return out


def dequantize_weights(w: Dict[str, np.ndarray], group_size: int, bits: int) -> Dict[str, np.ndarray]:
    """Quantized Linear layers (ModelLoader.swift:47-49,103-111, MLX affine format): a uint32
    ``.weight`` of packed ``bits``-bit codes (lowest bits first) with per-group ``.scales``
    and ``.biases`` becomes w = scale * q + bias, which is what quantized_matmul multiplies
    by.  Everything else passes through."""
    out = {}
    per = 32 // bits
    mask = (1 << bits) - 1
    for k, v in w.items():
        if k.endswith((".scales", ".biases")):
            continue
        base = k[: -len(".weight")] if k.endswith(".weight") else None
        if base is not None and v.dtype == np.uint32 and base + ".scales" in w:
            q = np.stack([(v >> np.uint32(j * bits)) & np.uint32(mask) for j in range(per)], axis=-1)
            q = q.reshape(v.shape[0], v.shape[1] * per).astype(np.float32)
            sc = np.repeat(w[base + ".scales"].astype(np.float32), group_size, axis=1)
            bi = np.repeat(w[base + ".biases"].astype(np.float32), group_size, axis=1)
            out[k] = sc * q + bi
        else:
            out[k] = v
    return out


def load_model_dir(path: str) -> Tuple[ModelConfig, Dict[str, np.ndarray]]:
    with open(os.path.join(path, "config.json")) as f:
        raw_cfg = json.load(f)
    cfg = ModelConfig.from_dict(raw_cfg)
    raw = _load_safetensors_any(os.path.join(path, "model.safetensors"))
    qc = raw_cfg.get("quantization")
    if isinstance(qc, dict):  # MoonshineConfig.swift:147-153 (defaults 64, 8)
        raw = dequantize_weights(raw, int(qc.get("group_size", 64)), int(qc.get("bits", 8)))
    return cfg, sanitize_weights(raw)


def _load_safetensors_any(fn: str) -> Dict[str, np.ndarray]:
    """safetensors reader that also widens BF16/F16 tensors to float32."""
    with open(fn, "rb") as f:
        n = int(np.frombuffer(f.read(8), dtype=np.uint64)[0])
        header = json.loads(f.read(n))
        base = 8 + n
        data = np.fromfile(f, dtype=np.uint8)
    out = {}
    for k, meta in header.items():
        if k == "__metadata__":
            continue
        a, b = meta["data_offsets"]
        buf = data[a:b]
        shape = tuple(meta["shape"])
        dt = meta["dtype"]
        if dt == "F32":
            v = buf.view(np.float32)
        elif dt == "F16":
            v = buf.view(np.float16).astype(np.float32)
        elif dt == "BF16":
            v = (buf.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        elif dt == "U32":
            v = buf.view(np.uint32)
        else:
            raise ValueError(f"unsupported dtype {dt} for {k}")
        out[k] = v.reshape(shape).copy()
    return out


# ----------------------------------------------------------------------------- math

def _layer_norm(x, w, eps=1e-5):
    """MLXFast.layerNorm / MLXNN.LayerNorm(bias: false): biased variance, eps 1e-5."""
    mu = x.mean(axis=-1, keepdims=True)
    c = x - mu
    var = (c * c).mean(axis=-1, keepdims=True)
    return c / np.sqrt(var + eps) * w


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _gelu_erf(x):
    """MLXNN.gelu: exact erf form."""
    from scipy.special import erf
    return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))


def _softmax(s, axis=-1):
    m = s.max(axis=axis, keepdims=True)
    e = np.exp(s - m)
    return e / e.sum(axis=axis, keepdims=True)


def _f16(x):
    """Round to IEEE half and back (the reference's ``asType(.float16)`` storage)."""
    return x.astype(np.float16).astype(x.dtype)


class Oracle:
    """Numpy restatement of MoonshineModel's encoder, decoder and greedy loops."""

    def __init__(self, cfg: ModelConfig, weights: Dict[str, np.ndarray], dtype=np.float64):
        self.cfg = cfg
        self.dt = dtype
        self.w = {k: np.asarray(v, dtype=dtype) for k, v in weights.items()}
        # Attention scale is a Float in the reference (MoonshineLayers.swift:40).
        self.scale = float(np.float32(cfg.head_dim) ** np.float32(-0.5))
        self.enc_scale = float(np.float32(cfg.encoder.head_dim) ** np.float32(-0.5))
        nd = cfg.rotary_ndims
        i = np.arange(nd // 2, dtype=np.float64)
        self.inv_freq = cfg.rope_theta ** (-2.0 * i / nd)

    @staticmethod
    def from_dir(path: str, dtype=np.float64) -> "Oracle":
        cfg, w = load_model_dir(path)
        return Oracle(cfg, w, dtype)

    # -------------------------------------------------------------- frontend (a1-a3)
    def _frames_to_features(self, frames):
        """FrameCMVN + AsinhCompression + SiLU(Linear) (MoonshineEncoder.swift:15-34,84-86)."""
        w = self.w
        mean = frames.mean(axis=-1, keepdims=True)
        c = frames - mean
        rms = np.sqrt((c * c).mean(axis=-1, keepdims=True) + 1e-6)
        x = c / rms
        x = np.arcsinh(np.exp(w["encoder.embedder.comp.log_k"]) * x)
        return _silu(x @ w["encoder.embedder.linear.weight"].T)

    def _conv(self, xp, name):
        """Conv1d(k=5, stride=2, no padding) over already-padded ``xp`` [T, C_in]."""
        W = self.w[f"encoder.embedder.{name}.weight"]  # [out, in, 5]
        b = self.w[f"encoder.embedder.{name}.bias"]
        T = xp.shape[0]
        n_out = (T - 5) // 2 + 1
        if n_out <= 0:
            return np.zeros((0, W.shape[0]), dtype=self.dt)
        out = np.broadcast_to(b, (n_out, W.shape[0])).copy()
        for k in range(5):
            out += xp[k:k + 2 * (n_out - 1) + 1:2] @ W[:, :, k].T
        return out

    def embed(self, audio):
        """Embedder batch forward (MoonshineEncoder.swift:73-97); audio 1-D."""
        a = np.asarray(audio, dtype=self.dt).reshape(-1)
        fl = self.cfg.encoder.frame_len
        n = a.shape[0] // fl
        x = self._frames_to_features(a[: n * fl].reshape(n, fl))
        pad = np.zeros((4, x.shape[1]), dtype=self.dt)
        x = _silu(self._conv(np.concatenate([pad, x]), "conv1"))
        pad = np.zeros((4, x.shape[1]), dtype=self.dt)
        return self._conv(np.concatenate([pad, x]), "conv2")

    # -------------------------------------------------------------- encoder (a5-a7)
    def _window_mask(self, layer: int, T: int):
        """EncoderLayer.slidingMask (MoonshineLayers.swift:266-290)."""
        sw = self.cfg.encoder.sliding_windows
        if sw is None or layer >= len(sw):
            return None
        left, right = sw[layer]
        pos = np.arange(T)
        diff = pos[:, None] - pos[None, :]
        valid = (diff >= 0) & (diff < left)
        if right > 0:
            valid |= (diff < 0) & (-diff < right)
        return np.where(valid, 0.0, -1e9).astype(self.dt)

    def _banded_attention(self, q, k, v, left: int, right: int):
        """The windowed softmax of slidingMask (MoonshineLayers.swift:266-290) evaluated over
        each query's band of keys [t - left + 1, t + right - 1] only.  The dense form adds
        -1e9 to every key outside the band, whose exp is exactly 0 in float64, so the two
        differ only in summation order; the float64 checker uses this form (the dense one
        spends its time in exp underflow at 30 s of audio), the float32 restatement keeps the
        reference's dense mask.  q, k, v [H, T, hd] -> [H, T, hd]."""
        T = q.shape[1]
        offs = np.arange(-(left - 1), max(right, 1))
        idx = np.arange(T)[:, None] + offs[None, :]                   # [T, W]
        valid = (idx >= 0) & (idx < T)
        idx = np.clip(idx, 0, T - 1)
        kb, vb = k[:, idx], v[:, idx]                                 # [H, T, W, hd]
        s = np.einsum("htd,htwd->htw", q, kb) * self.enc_scale
        s = np.where(valid[None], s, -np.inf)
        p = _softmax(s)
        return np.einsum("htw,htwd->htd", p, vb)

    def _encoder_layer(self, x, i):
        """EncoderLayer.callAsFunction (MoonshineLayers.swift:297-310)."""
        w = self.w
        ec = self.cfg.encoder
        p = f"encoder.layers.{i}."
        T = x.shape[0]
        H, hd = ec.num_attention_heads, ec.head_dim
        h = _layer_norm(x, w[p + "input_layernorm.weight"] + 1.0)
        q = (h @ w[p + "self_attn.q_proj.weight"].T).reshape(T, H, hd).transpose(1, 0, 2)
        k = (h @ w[p + "self_attn.k_proj.weight"].T).reshape(T, -1, hd).transpose(1, 0, 2)
        v = (h @ w[p + "self_attn.v_proj.weight"].T).reshape(T, -1, hd).transpose(1, 0, 2)
        rep = H // k.shape[0]
        if rep > 1:
            k = np.repeat(k, rep, axis=0)
            v = np.repeat(v, rep, axis=0)
        sw = ec.sliding_windows
        if self.dt == np.float64 and sw is not None and i < len(sw):
            o = self._banded_attention(q, k, v, *sw[i]).transpose(1, 0, 2).reshape(T, H * hd)
        else:
            s = q @ k.transpose(0, 2, 1) * self.enc_scale
            m = self._window_mask(i, T)
            if m is not None:
                s = s + m
            o = (_softmax(s) @ v).transpose(1, 0, 2).reshape(T, H * hd)
        x = x + o @ w[p + "self_attn.o_proj.weight"].T
        h = _layer_norm(x, w[p + "post_attention_layernorm.weight"] + 1.0)
        f = _gelu_erf(h @ w[p + "mlp.fc1.weight"].T + w[p + "mlp.fc1.bias"])
        return x + f @ w[p + "mlp.fc2.weight"].T + w[p + "mlp.fc2.bias"]

    def encode(self, features):
        """MoonshineEncoder.callAsFunction (MoonshineEncoder.swift:171-177)."""
        x = np.asarray(features, dtype=self.dt)
        if x.shape[0] == 0:
            return x
        for i in range(self.cfg.encoder.num_hidden_layers):
            x = self._encoder_layer(x, i)
        return _layer_norm(x, self.w["encoder.final_norm.weight"] + 1.0)

    def prepare_memory(self, enc, pos_offset: int = 0):
        """MoonshineDecoder.prepareMemory (MoonshineDecoder.swift:39-47)."""
        T = enc.shape[0]
        x = enc + self.w["decoder.pos_emb.weight"][pos_offset:pos_offset + T]
        if "decoder.proj.weight" in self.w:
            x = x @ self.w["decoder.proj.weight"].T
        return x

    def memory_for(self, audio):
        return self.prepare_memory(self.encode(self.embed(audio)))

    # -------------------------------------------------------------- decoder (a9-a14)
    def _rope(self, x, pos: int):
        """MLXFast.RoPE traditional=true on the first rotary_ndims dims
        (MoonshineLayers.swift:98-104); x [H, hd]."""
        nd = self.cfg.rotary_ndims
        ang = pos * self.inv_freq
        c = np.cos(ang).astype(self.dt)
        s = np.sin(ang).astype(self.dt)
        out = x.copy()
        a = x[:, 0:nd:2]
        b = x[:, 1:nd:2]
        out[:, 0:nd:2] = a * c - b * s
        out[:, 1:nd:2] = a * s + b * c
        return out

    def new_cache(self, memory, kv_fp16: bool):
        return DecoderCache(self, memory, kv_fp16)

    def decoder_step(self, token: int, cache: "DecoderCache", cross_qk: Optional[list] = None):
        """One decoder call for a single token (MoonshineDecoder.swift:55-85 with
        DecoderLayer MoonshineLayers.swift:350-379); returns final hidden state and
        logits (MoonshineModel.swift:71-85).  ``cross_qk`` (a list) receives each layer's
        cross-attention scores q.K^T * scale, [H, M] (returnCrossQK,
        MoonshineDecoder.swift:65-81, MoonshineLayers.swift:150-154)."""
        cfg, w = self.cfg, self.w
        H, hd = cfg.num_attention_heads, cfg.head_dim
        KVH = cfg.num_key_value_heads
        rep = H // KVH
        x = w["decoder.embed_tokens.weight"][token].astype(self.dt)
        pos = cache.length
        first = cache.length == 0
        for i in range(cfg.num_hidden_layers):
            p = f"decoder.layers.{i}."
            # self-attention with RoPE at offset = cache length (MoonshineLayers.swift:88-125)
            h = _layer_norm(x, w[p + "input_layernorm.weight"])
            q = self._rope((h @ w[p + "self_attn.q_proj.weight"].T).reshape(H, hd), pos)
            k = self._rope((h @ w[p + "self_attn.k_proj.weight"].T).reshape(KVH, hd), pos)
            v = (h @ w[p + "self_attn.v_proj.weight"].T).reshape(KVH, hd)
            # attention sees [cached (possibly fp16-rounded) rows ; this step's fp32 row]
            K = np.concatenate([cache.self_k[i], k[:, None, :]], axis=1)
            V = np.concatenate([cache.self_v[i], v[:, None, :]], axis=1)
            o = self._attend(q, K, V, rep)
            # stored cache rounds only the new row (concat of fp16 + fp32 promotes to
            # fp32, then ``asType(.float16)``; MoonshineLayers.swift:106-115)
            cache.self_k[i] = _f16(K) if cache.kv_fp16 else K
            cache.self_v[i] = _f16(V) if cache.kv_fp16 else V
            x = x + o @ w[p + "self_attn.o_proj.weight"].T
            # cross-attention: step 0 uses freshly projected fp32 K/V, later steps the
            # stored cache (fp16-rounded when enabled) (MoonshineLayers.swift:88-96,113-125)
            h = _layer_norm(x, w[p + "post_attention_layernorm.weight"])
            qc = (h @ w[p + "encoder_attn.q_proj.weight"].T).reshape(H, hd)
            if first:
                Kc, Vc = cache.cross_k32[i], cache.cross_v32[i]
            else:
                Kc, Vc = cache.cross_k[i], cache.cross_v[i]
            oc = self._attend(qc, Kc, Vc, rep)
            if cross_qk is not None:
                Kr = np.repeat(Kc, rep, axis=0) if rep > 1 else Kc
                cross_qk.append(np.einsum("hd,hsd->hs", qc, Kr) * self.scale)
            x = x + oc @ w[p + "encoder_attn.o_proj.weight"].T
            # SwiGLU MLP: first half value, second half gate (KernelFusion.swift:90-113)
            h = _layer_norm(x, w[p + "final_layernorm.weight"])
            f = h @ w[p + "mlp.fc1.weight"].T + w[p + "mlp.fc1.bias"]
            I = f.shape[-1] // 2
            g = f[:I] * _silu(f[I:])
            x = x + g @ w[p + "mlp.fc2.weight"].T + w[p + "mlp.fc2.bias"]
        cache.length += 1
        hfin = _layer_norm(x, w["decoder.norm.weight"])
        if cfg.tie_word_embeddings:
            logits = hfin @ w["decoder.embed_tokens.weight"].T
        else:
            logits = hfin @ w["proj_out.weight"].T
        return hfin, logits

    def _attend(self, q, K, V, rep):
        """SDPA for one query row per head; q [H, hd], K/V [KVH, S, hd]."""
        if rep > 1:
            K = np.repeat(K, rep, axis=0)
            V = np.repeat(V, rep, axis=0)
        s = np.einsum("hd,hsd->hs", q, K) * self.scale
        p = _softmax(s, axis=-1)
        return np.einsum("hs,hsd->hd", p, V).reshape(-1)

    # -------------------------------------------------------------- token loops (a15, a16)
    def greedy(self, memory, limit: int, kv_fp16: bool, forced_len: Optional[int] = None,
               teacher: Optional[List[int]] = None, keep_logits: bool = False):
        """Greedy decode against ``memory``.

        Default mode follows encodeAndDecodeChunk (MoonshineModel.swift:204-236) /
        decodeMemory (MoonshineStreaming.swift:238-275): BOS, then up to ``limit``
        decoder calls, stopping at EOS.  ``forced_len`` decodes exactly that many tokens
        with EOS fed back like any other id (the benchmark harness mode).  ``teacher``
        feeds the given ids instead of the argmax (for logits comparisons).
        Returns (ids, hit_eos, logits list or None, margins)."""
        cfg = self.cfg
        cache = self.new_cache(memory, kv_fp16)
        logits_all = [] if keep_logits else None
        margins = []
        ids: List[int] = []
        tok = cfg.decoder_start_token_id
        n_calls = forced_len if forced_len is not None else limit
        if teacher is not None:
            n_calls = len(teacher)
        hit_eos = False
        for step in range(n_calls):
            _, lg = self.decoder_step(tok, cache)
            nt = int(np.argmax(lg))
            srt = np.partition(lg, -2)[-2:]
            margins.append(float(srt[1] - srt[0]))
            if keep_logits:
                logits_all.append(np.array(lg, dtype=np.float64))
            if teacher is not None:
                ids.append(nt)
                tok = teacher[step]
                continue
            if forced_len is None and nt == cfg.eos_token_id:
                hit_eos = True
                break
            ids.append(nt)
            tok = nt
        return ids, hit_eos, logits_all, margins

    def token_limit(self, n_samples: int, max_tokens: Optional[int]) -> int:
        """MoonshineModel.swift:200-201."""
        dur = n_samples / float(self.cfg.encoder.sample_rate)
        lim = int(math.ceil(dur * self.cfg.max_tokens_per_second))
        return lim if max_tokens is None else min(max_tokens, lim)

    def generate(self, audio, max_tokens: Optional[int] = None, kv_fp16: bool = True,
                 chunk_duration: float = 30.0, forced_len: Optional[int] = None):
        """MoonshineModel.generate (MoonshineModel.swift:130-184) over 30 s chunks,
        returning the concatenated token ids (text decoding is out of scope)."""
        a = np.asarray(audio, dtype=np.float32).reshape(-1)
        sr = self.cfg.encoder.sample_rate
        chunk = int(chunk_duration * sr)
        ids: List[int] = []
        for off in range(0, a.shape[0], chunk):
            c = a[off:min(off + chunk, a.shape[0])]
            mem = self.memory_for(c)
            if mem.shape[0] == 0:
                continue
            limit = self.token_limit(c.shape[0], max_tokens)
            out, _, _, _ = self.greedy(mem, limit, kv_fp16, forced_len=forced_len)
            ids.extend(out)
        return ids

    def generate_long(self, audio, max_memory_frames: int = 100000, min_segment_frames: int = 250,
                      kv_fp16: bool = True) -> List[List[int]]:
        """generateLong (MoonshineStreaming.swift:287-376): one full encode, then segments of at
        most max_memory_frames memory rows with EOS-driven advance.  Returns the ids of every
        segment that produced tokens (the reference keeps the non-empty segment texts)."""
        mem = self.memory_for(np.asarray(audio, dtype=np.float32).reshape(-1))
        total = mem.shape[0]
        segments: List[List[int]] = []
        start = 0
        while start < total:  # :312
            end = min(start + max_memory_frames, total)
            frames = end - start
            limit = int(math.ceil(frames * 0.02 * self.cfg.max_tokens_per_second))  # :317
            ids, hit, _, _ = self.greedy(mem[start:end], limit, kv_fp16)
            # :324-345: the loop runs limit - 1 more calls and only an EOS inside it sets hitEOS;
            # an EOS from the last call is dropped without setting it
            calls = len(ids) + (1 if hit else 0)
            hit = hit and calls < limit
            if ids:
                segments.append(ids)
            if hit and frames > min_segment_frames:  # :354-359, tokens include the start token
                used = max(min_segment_frames, int((len(ids) + 1) / self.cfg.max_tokens_per_second * 50.0))
                start += min(used, frames)
            else:
                start = end
        return segments

    # ------------------------------------------------------------ word timestamps (f2)
    def generate_with_alignment(self, audio, max_tokens: Optional[int] = None, kv_fp16: bool = True,
                                medfilt_width: int = 7):
        """generateWithWordTimestamps (MoonshineModel.swift:241-316) up to the tokenizer: one
        encode of the whole audio, greedy decoding with every call's cross scores kept, EOS
        break after the call's probability is recorded.  Returns a dict with ids (EOS
        excluded), token_probs (one per call), attn_rows (layer/head-mean softmax rows),
        filtered (z-scored + median-filtered rows), jump_frames and n_frames."""
        a = np.asarray(audio, dtype=np.float32).reshape(-1)
        mem = self.memory_for(a)
        M = mem.shape[0]
        limit = self.token_limit(a.shape[0], max_tokens)  # :258-259
        cfg = self.cfg
        ids: List[int] = []
        probs: List[float] = []
        qk_steps: List[list] = []
        hit = False
        if M > 0:
            cache = self.new_cache(mem, kv_fp16)
            tok = cfg.decoder_start_token_id
            for _ in range(limit):  # :266-287
                qk: list = []
                _, lg = self.decoder_step(tok, cache, cross_qk=qk)
                qk_steps.append(qk)
                nt = int(np.argmax(lg))
                probs.append(float(_softmax(lg)[nt]))
                if nt == cfg.eos_token_id:
                    hit = True
                    break
                ids.append(nt)
                tok = nt
        rows = attention_rows(qk_steps, M)
        filt = median_filter_rows(zscore_rows(rows), medfilt_width)
        jumps = dtw_jump_frames(-filt) if ids and M > 0 else np.zeros(0, dtype=np.int64)
        return {"ids": ids, "token_probs": np.asarray(probs), "attn_rows": rows, "filtered": filt,
                "jump_frames": jumps, "n_frames": M, "hit_eos": hit}


def attention_rows(qk_steps: List[list], n_frames: int) -> np.ndarray:
    """findAlignment :106-130: per decoder call, the mean over layers of the head-mean
    softmax over frames of each layer's cross scores."""
    out = np.zeros((len(qk_steps), n_frames))
    for s, layers in enumerate(qk_steps):
        acc = np.zeros(n_frames)
        for qk in layers:
            acc += _softmax(np.asarray(qk, dtype=np.float64), axis=-1).mean(axis=0)[:n_frames]
        if layers:
            acc /= len(layers)
        out[s] = acc
    return out


def zscore_rows(rows: np.ndarray) -> np.ndarray:
    """findAlignment :132-139: (row - mean) / (population std + 1e-6) per row."""
    rows = np.asarray(rows, dtype=np.float64)
    if rows.size == 0:
        return rows.copy()
    mean = rows.mean(axis=1, keepdims=True)
    std = np.sqrt(((rows - mean) ** 2).mean(axis=1, keepdims=True)) + 1e-6
    return (rows - mean) / std


def median_filter_1d(x: np.ndarray, width: int) -> np.ndarray:
    """medianFilter1D (MoonshineTimestamps.swift:68-80): window clipped at the ends, element
    count/2 of the sorted window (the upper median of an even window)."""
    x = np.asarray(x)
    if width <= 1 or x.size == 0:
        return x.copy()
    half = width // 2
    out = np.empty_like(x)
    n = x.shape[0]
    for i in range(n):
        w = np.sort(x[max(0, i - half):min(n - 1, i + half) + 1])
        out[i] = w[w.shape[0] // 2]
    return out


def median_filter_rows(rows: np.ndarray, width: int) -> np.ndarray:
    return np.stack([median_filter_1d(r, width) for r in rows]) if len(rows) else np.asarray(rows).copy()


def dtw_path(cost: np.ndarray) -> Tuple[List[int], List[int]]:
    """dtw (MoonshineTimestamps.swift:20-65) in float32: diagonal wins ties, then vertical
    (skip text), then horizontal (skip time); backtrace from (N, M)."""
    cost = np.asarray(cost, dtype=np.float32)
    N, M = cost.shape
    if N == 0 or M == 0:
        return [], []
    inf = np.float32(np.inf)
    D = np.full((N + 1, M + 1), inf, dtype=np.float32)
    T = np.full((N + 1, M + 1), -1, dtype=np.int8)
    D[0, 0] = 0.0
    for i in range(1, N + 1):  # row order gives the same costs as the reference's column order
        for j in range(1, M + 1):
            c0, c1, c2 = D[i - 1, j - 1], D[i - 1, j], D[i, j - 1]
            if c0 <= c1 and c0 <= c2:
                c, t = c0, 0
            elif c1 <= c2:
                c, t = c1, 1
            else:
                c, t = c2, 2
            D[i, j] = np.float32(cost[i - 1, j - 1] + c)
            T[i, j] = t
    T[0, :] = 2
    T[:, 0] = 1
    i, j = N, M
    path = []
    while i > 0 or j > 0:
        path.append((i - 1, j - 1))
        t = T[i, j]
        if t == 0:
            i, j = i - 1, j - 1
        elif t == 1:
            i -= 1
        else:
            j -= 1
    path.reverse()
    return [p[0] for p in path], [p[1] for p in path]


def dtw_jump_frames(cost: np.ndarray) -> np.ndarray:
    """findAlignment :148-184: DTW path, then the time index at each change of text index."""
    text, time = dtw_path(cost)
    jumps = [time[k] for k in range(len(text)) if k == 0 or text[k] != text[k - 1]]
    return np.asarray(jumps, dtype=np.int64)


def word_timings(jump_frames, token_probs, word_first: List[int], n_tokens: int, n_frames: int,
                 time_offset: float = 0.0) -> List[Tuple[float, float, float]]:
    """findAlignment :186-239 for words given by their first token index: (start, end,
    probability) with the reference's rounding (Swift .rounded(): half away from zero) and
    the midpoint fix of overlapping neighbours."""
    def rnd(x, unit):
        v = abs(x) * unit
        f = math.floor(v)
        r = f + 1 if v - f >= 0.5 else f
        return (r if x >= 0 else -r) / unit

    jumps = [int(j) for j in jump_frames]
    probs = [float(p) for p in token_probs]
    out = []
    if n_tokens == 0:
        return out
    for w, first in enumerate(word_first):
        last = (word_first[w + 1] if w + 1 < len(word_first) else n_tokens) - 1
        sf = jumps[first] if first < len(jumps) else (jumps[-1] if jumps else 0)
        ef = jumps[last + 1] if last + 1 < len(jumps) else (jumps[-1] if jumps else n_frames)
        ps = np.float32(0.0)
        cnt = 0
        for k in range(first, last + 1):
            if k < len(probs):
                ps = np.float32(ps + np.float32(probs[k]))
                cnt += 1
        avg = float(ps) / cnt if cnt else 1.0
        out.append([rnd(time_offset + sf * 0.02, 1000.0), rnd(time_offset + ef * 0.02, 1000.0),
                    rnd(avg, 10000.0)])
    for k in range(1, len(out)):
        if out[k - 1][1] > out[k][0]:
            mid = rnd((out[k - 1][1] + out[k][0]) / 2.0, 1000.0)
            out[k - 1][1] = mid
            out[k][0] = mid
    return [tuple(o) for o in out]


class DecoderCache:
    """Per-layer self and cross K/V (MoonshineDecoder.swift:90-98) for one utterance."""

    def __init__(self, oracle: Oracle, memory, kv_fp16: bool):
        cfg, w = oracle.cfg, oracle.w
        KVH, hd = cfg.num_key_value_heads, cfg.head_dim
        M = memory.shape[0]
        self.kv_fp16 = kv_fp16
        self.length = 0
        self.self_k = [np.zeros((KVH, 0, hd), dtype=oracle.dt) for _ in range(cfg.num_hidden_layers)]
        self.self_v = [np.zeros((KVH, 0, hd), dtype=oracle.dt) for _ in range(cfg.num_hidden_layers)]
        self.cross_k32, self.cross_v32, self.cross_k, self.cross_v = [], [], [], []
        for i in range(cfg.num_hidden_layers):
            p = f"decoder.layers.{i}.encoder_attn."
            k = (memory @ w[p + "k_proj.weight"].T).reshape(M, KVH, hd).transpose(1, 0, 2)
            v = (memory @ w[p + "v_proj.weight"].T).reshape(M, KVH, hd).transpose(1, 0, 2)
            self.cross_k32.append(k)
            self.cross_v32.append(v)
            self.cross_k.append(_f16(k) if kv_fp16 else k)
            self.cross_v.append(_f16(v) if kv_fp16 else v)


# ----------------------------------------------------------------------------- streaming

@dataclass
class StreamingConfig:
    """MoonshineStreaming.swift:47-62."""
    max_memory_frames: int = 100000
    min_segment_frames: int = 250


class OracleStream:
    """StreamingState + createStream/startStream/addAudio/transcribe
    (MoonshineStreaming.swift:8-276, Embedder.processChunk MoonshineEncoder.swift:100-151).
    Token ids stand in for text."""

    def __init__(self, oracle: Oracle, kv_fp16: bool = True):
        self.o = oracle
        self.kv_fp16 = kv_fp16
        fl = oracle.cfg.encoder.frame_len
        # createStream pre-fills frameLen-1 zero samples (MoonshineStreaming.swift:69-71)
        self.sample_buffer = np.zeros(fl - 1, dtype=oracle.dt)
        self.conv1_buffer = None
        self.conv2_buffer = None
        self.features = None
        self.encoder_frames_emitted = 0
        self.pos_offset = 0
        self.memory = None
        self.emitted_segments: List[List[int]] = []
        self.last_decode_hit_eos = False
        self.active = False

    @property
    def memory_len(self) -> int:
        return 0 if self.memory is None else self.memory.shape[0]

    def start(self):  # MoonshineStreaming.swift:74-78
        self.active = True
        self._reset_segment()
        self.emitted_segments = []

    def stop(self):  # :81-83
        self.active = False

    def _process_chunk(self, chunk):
        """Embedder.processChunk (MoonshineEncoder.swift:100-151)."""
        o = self.o
        fl = o.cfg.encoder.frame_len
        c = np.asarray(chunk, dtype=o.dt).reshape(-1)
        if self.sample_buffer is not None and self.sample_buffer.shape[0] > 0:
            c = np.concatenate([self.sample_buffer, c])
        n = c.shape[0] // fl
        rem = c.shape[0] - n * fl
        self.sample_buffer = c[c.shape[0] - rem:] if rem > 0 else np.zeros(0, dtype=o.dt)
        if n == 0:
            return np.zeros((0, o.cfg.encoder.hidden_size), dtype=o.dt)
        x = o._frames_to_features(c[: n * fl].reshape(n, fl))
        if self.conv1_buffer is not None:
            xin1 = np.concatenate([self.conv1_buffer, x])
        else:
            xin1 = np.concatenate([np.zeros((4, x.shape[1]), dtype=o.dt), x])
        self.conv1_buffer = xin1[-4:]
        x = _silu(o._conv(xin1, "conv1"))
        if self.conv2_buffer is not None:
            xin2 = np.concatenate([self.conv2_buffer, x])
        else:
            xin2 = np.concatenate([np.zeros((4, x.shape[1]), dtype=o.dt), x])
        self.conv2_buffer = xin2[-4:]
        return o._conv(xin2, "conv2")

    def add_audio(self, chunk):  # MoonshineStreaming.swift:87-105
        f = self._process_chunk(chunk)
        if f.shape[0] > 0:
            self.features = f if self.features is None else np.concatenate([self.features, f])

    def _encode_new_frames(self, is_final: bool):  # MoonshineStreaming.swift:178-214
        o = self.o
        ec = o.cfg.encoder
        if self.features is None or self.features.shape[0] == 0:
            return
        total = self.features.shape[0]
        look = 0
        if ec.sliding_windows is not None:
            look = max([w[1] for w in ec.sliding_windows], default=0)
        stable = total if is_final else max(0, total - look)
        new = stable - self.encoder_frames_emitted
        if new <= 0:
            return
        left_ctx = 16 * ec.num_hidden_layers
        win_start = max(0, self.encoder_frames_emitted - left_ctx)
        enc = o.encode(self.features[win_start:total])
        off = self.encoder_frames_emitted - win_start
        mem = o.prepare_memory(enc[off:off + new], self.pos_offset)
        self.pos_offset += new
        self.encoder_frames_emitted = stable
        self.memory = mem if self.memory is None else np.concatenate([self.memory, mem])

    def _reset_segment(self):  # MoonshineStreaming.swift:217-226
        self.features = None
        self.encoder_frames_emitted = 0
        self.pos_offset = 0
        self.memory = None
        self.last_decode_hit_eos = False

    def _decode_memory(self, max_tokens: Optional[int]):  # MoonshineStreaming.swift:229-276
        o = self.o
        dur = float(self.memory_len) * 0.020
        limit = int(math.ceil(dur * o.cfg.max_tokens_per_second))
        max_tok = limit if max_tokens is None else min(max_tokens, limit)
        ids, hit, _, _ = o.greedy(self.memory, max_tok, self.kv_fp16)
        return ids, hit

    def transcribe(self, is_final: bool = False, config: StreamingConfig = StreamingConfig(),
                   max_tokens: Optional[int] = None):
        """MoonshineStreaming.swift:122-168.  Returns (ids, hit_eos, emitted) where
        ``emitted`` says whether the ids were appended to the emitted segments."""
        self._encode_new_frames(is_final)
        if self.memory_len == 0:
            if is_final:
                self._reset_segment()
            return [], False, False
        ids, hit = self._decode_memory(max_tokens)
        self.last_decode_hit_eos = hit
        if hit and self.memory_len >= config.min_segment_frames:
            self.emitted_segments.append(ids)
            self._reset_segment()
            self._encode_new_frames(is_final)
            return ids, hit, True
        if is_final:
            self.emitted_segments.append(ids)
            self._reset_segment()
            return ids, hit, True
        if self.memory_len > config.max_memory_frames:
            self.emitted_segments.append(ids)
            self._reset_segment()
            return ids, hit, True
        return ids, hit, False
