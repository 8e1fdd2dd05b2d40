"""Seeded synthetic model directories and audio for the Moonshine V2 streaming path.

No checkpoint or dataset can be downloaded on the machines this library is built and
measured on, so every model used by the tests and the benchmark is a random-init model
written to disk in the same layout a HuggingFace `UsefulSensors/moonshine-streaming-*`
checkpoint has (``config.json`` + ``model.safetensors`` with ``model.`` prefixed keys,
``.gamma`` encoder norms and PyTorch ``[out, in, k]`` conv weights).  That is the layout
the reference loader consumes (Sources/MoonshineMLX/ModelLoader.swift:35-101), so the
same directory feeds the CUDA runtime (``ms_model_load``) and the CPU oracle.

Weights: every Linear / Conv / Embedding weight and bias ~ N(0, 0.02) drawn from
``numpy.random.Generator(PCG64(seed))`` in sorted key order; ``log_k`` = 0; encoder
unit-offset norms stored as 0 (effective gamma 1); decoder LayerNorm weights 1.

Audio: N(0, 0.05) noise plus three sinusoids of amplitude 0.1 with frequency
~U(100, 3000) Hz and phase ~U(0, 2*pi), all from ``PCG64(seed)`` (frequencies, then
phases, then the noise), float32 at 16 kHz.
"""
from __future__ import annotations

import json
import math
import os
from typing import Dict, List, Optional

import numpy as np

SAMPLE_RATE = 16000

# Architectures.  "tiny" is the reference's own default config
# (Sources/MoonshineMLX/MoonshineConfig.swift:20-28, 84-103).  "small" and "medium" are
# not in the reference; their dims follow the published model cards' shapes.
_ARCH = {
    "tiny": dict(hidden_size=320, intermediate_size=1280, num_hidden_layers=6,
                 num_attention_heads=8, head_dim=40, seed=0),
    "small": dict(hidden_size=512, intermediate_size=2048, num_hidden_layers=10,
                  num_attention_heads=8, head_dim=64, seed=2),
    "medium": dict(hidden_size=640, intermediate_size=2560, num_hidden_layers=14,
                   num_attention_heads=10, head_dim=64, seed=3),
}


def sliding_windows_for(num_layers: int) -> List[List[int]]:
    """Encoder [left, right] windows: first two and last two layers see 4 frames of
    right context, the rest are causal.  For 6 layers this is the tiny model's
    published pattern [[16,4],[16,4],[16,0],[16,0],[16,4],[16,4]]."""
    out = []
    for i in range(num_layers):
        right = 4 if (i < 2 or i >= num_layers - 2) else 0
        out.append([16, right])
    return out


def make_config(arch: str = "tiny", **overrides) -> dict:
    """config.json contents for one architecture, in the key set the reference parses
    (Sources/MoonshineMLX/MoonshineConfig.swift:43-56, 134-177)."""
    a = dict(_ARCH[arch])
    a.pop("seed")
    a.update({k: v for k, v in overrides.items() if k in a})
    d = a["hidden_size"]
    L = a["num_hidden_layers"]
    cfg = {
        "model_type": "moonshine_streaming",
        "hidden_size": d,
        "intermediate_size": a["intermediate_size"],
        "num_hidden_layers": L,
        "num_attention_heads": a["num_attention_heads"],
        "num_key_value_heads": a["num_attention_heads"],
        "head_dim": a["head_dim"],
        "vocab_size": overrides.get("vocab_size", 32768),
        "max_position_embeddings": overrides.get("max_position_embeddings", 4096),
        "tie_word_embeddings": bool(overrides.get("tie_word_embeddings", False)),
        "bos_token_id": 1,
        "eos_token_id": 2,
        "decoder_start_token_id": 1,
        "pad_token_id": 0,
        "rope_parameters": {"rope_type": "default", "rope_theta": 10000.0,
                            "partial_rotary_factor": 0.8},
        "max_tokens_per_second": 6.5,
        "encoder_config": {
            "hidden_size": d,
            "intermediate_size": 4 * d,
            "num_hidden_layers": L,
            "num_attention_heads": a["num_attention_heads"],
            "num_key_value_heads": a["num_attention_heads"],
            "head_dim": a["head_dim"],
            "frame_ms": 5.0,
            "sample_rate": SAMPLE_RATE,
            "max_position_embeddings": overrides.get("max_position_embeddings", 4096),
            "sliding_windows": overrides.get("sliding_windows", sliding_windows_for(L)),
        },
    }
    return cfg


def default_seed(arch: str) -> int:
    return _ARCH[arch]["seed"]


def hf_weight_shapes(cfg: dict) -> Dict[str, tuple]:
    """Every tensor of a checkpoint in HuggingFace key layout, with its shape."""
    d = cfg["hidden_size"]
    I = cfg["intermediate_size"]
    L = cfg["num_hidden_layers"]
    H = cfg["num_attention_heads"]
    hd = cfg["head_dim"]
    V = cfg["vocab_size"]
    P = cfg["max_position_embeddings"]
    ec = cfg["encoder_config"]
    ed = ec["hidden_size"]
    eI = ec["intermediate_size"]
    eL = ec["num_hidden_layers"]
    eH = ec["num_attention_heads"]
    ehd = ec["head_dim"]
    frame_len = int(ec["frame_ms"] * ec["sample_rate"] / 1000.0)
    s = {}
    e = "model.encoder."
    s[e + "embedder.comp.log_k"] = ()
    s[e + "embedder.linear.weight"] = (ed, frame_len)
    s[e + "embedder.conv1.weight"] = (2 * ed, ed, 5)
    s[e + "embedder.conv1.bias"] = (2 * ed,)
    s[e + "embedder.conv2.weight"] = (ed, 2 * ed, 5)
    s[e + "embedder.conv2.bias"] = (ed,)
    for i in range(eL):
        p = f"{e}layers.{i}."
        for n in ("q", "k", "v"):
            s[p + f"self_attn.{n}_proj.weight"] = (eH * ehd, ed)
        s[p + "self_attn.o_proj.weight"] = (ed, eH * ehd)
        s[p + "mlp.fc1.weight"] = (eI, ed)
        s[p + "mlp.fc1.bias"] = (eI,)
        s[p + "mlp.fc2.weight"] = (ed, eI)
        s[p + "mlp.fc2.bias"] = (ed,)
        s[p + "input_layernorm.gamma"] = (ed,)
        s[p + "post_attention_layernorm.gamma"] = (ed,)
    s[e + "final_norm.gamma"] = (ed,)
    dd = "model.decoder."
    s[dd + "embed_tokens.weight"] = (V, d)
    s[dd + "pos_emb.weight"] = (P, ed)
    if ed != d:
        s[dd + "proj.weight"] = (d, ed)
    for i in range(L):
        p = f"{dd}layers.{i}."
        for att in ("self_attn", "encoder_attn"):
            for n in ("q", "k", "v"):
                s[p + f"{att}.{n}_proj.weight"] = (H * hd, d)
            s[p + f"{att}.o_proj.weight"] = (d, H * hd)
        s[p + "mlp.fc1.weight"] = (2 * I, d)
        s[p + "mlp.fc1.bias"] = (2 * I,)
        s[p + "mlp.fc2.weight"] = (d, I)
        s[p + "mlp.fc2.bias"] = (d,)
        for n in ("input_layernorm", "post_attention_layernorm", "final_layernorm"):
            s[p + f"{n}.weight"] = (d,)
    s[dd + "norm.weight"] = (d,)
    if not cfg.get("tie_word_embeddings", False):
        s["proj_out.weight"] = (V, d)
    return s


def make_weights(cfg: dict, seed: int, std: float = 0.02) -> Dict[str, np.ndarray]:
    """Seeded random-init weights in HuggingFace key layout (float32)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for key, shape in sorted(hf_weight_shapes(cfg).items()):
        if key.endswith("comp.log_k"):
            out[key] = np.zeros(shape, dtype=np.float32)
        elif key.endswith(".gamma"):
            out[key] = np.zeros(shape, dtype=np.float32)
        elif "layernorm" in key or key.endswith("decoder.norm.weight"):
            out[key] = np.ones(shape, dtype=np.float32)
        else:
            out[key] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std))
    return out


def write_model_dir(path: str, cfg: dict, weights: Dict[str, np.ndarray],
                    dtype: str = "float32") -> str:
    """Write config.json + model.safetensors.  ``dtype`` "bfloat16"/"float16" stores the
    checkpoint at reduced precision (the small/medium bf16 workloads)."""
    from safetensors.numpy import save_file

    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    if dtype == "float32":
        tensors = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in weights.items()}
        save_file(tensors, os.path.join(path, "model.safetensors"))
    else:
        _save_reduced(path, weights, dtype)
    return path


# Linear layers of the MLX module tree: the ones the reference quantizes when their input
# width is a multiple of the group size (ModelLoader.swift:103-111).  Embeddings, convs and
# norms stay floating point.
_LINEAR_SUFFIXES = ("_proj.weight", "mlp.fc1.weight", "mlp.fc2.weight", "embedder.linear.weight",
                    "decoder.proj.weight", "proj_out.weight")


def is_quantizable_linear(key: str, shape: tuple, group_size: int) -> bool:
    return key.endswith(_LINEAR_SUFFIXES) and len(shape) == 2 and shape[1] % group_size == 0


def quantize_affine(w: np.ndarray, group_size: int, bits: int):
    """MLX affine quantization of a [out, in] matrix (mlx.core.quantize, published format):
    per group of ``group_size`` consecutive inputs, w ~ scale * q + bias with q an unsigned
    ``bits``-bit integer; q values packed into uint32 words lowest bits first.  Returns
    (packed [out, in * bits / 32] uint32, scales [out, in / group], biases [out, in / group])."""
    out_dim, in_dim = w.shape
    levels = (1 << bits) - 1
    g = w.reshape(out_dim, in_dim // group_size, group_size).astype(np.float64)
    lo, hi = g.min(axis=-1), g.max(axis=-1)
    scale = np.where(hi > lo, (hi - lo) / levels, 1.0)
    q = np.clip(np.rint((g - lo[..., None]) / scale[..., None]), 0, levels).astype(np.uint32)
    q = q.reshape(out_dim, in_dim)
    per = 32 // bits
    q = q.reshape(out_dim, in_dim // per, per)
    packed = np.zeros((out_dim, in_dim // per), dtype=np.uint32)
    for j in range(per):
        packed |= q[:, :, j] << np.uint32(j * bits)
    return packed, scale.astype(np.float32), lo.astype(np.float32)


def dequantize_affine(packed: np.ndarray, scales: np.ndarray, biases: np.ndarray, group_size: int,
                      bits: int) -> np.ndarray:
    """Inverse of quantize_affine: w = scale * q + bias per group (float32)."""
    per = 32 // bits
    out_dim = packed.shape[0]
    in_dim = packed.shape[1] * per
    mask = np.uint32((1 << bits) - 1)
    q = np.stack([(packed >> np.uint32(j * bits)) & mask for j in range(per)], axis=-1).reshape(out_dim, in_dim)
    s = np.repeat(np.asarray(scales, np.float32), group_size, axis=1)
    b = np.repeat(np.asarray(biases, np.float32), group_size, axis=1)
    return (s * q.astype(np.float32) + b).astype(np.float32)


def to_mlx_layout(weights: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    """HuggingFace keys -> the MLX module layout (ModelLoader.swift:75-101 in reverse):
    no ``model.`` prefix, ``.gamma`` -> ``.weight``, conv weights [out, k, in]."""
    out = {}
    for k, v in weights.items():
        if k.startswith("model."):
            k = k[6:]
        k = k.replace(".gamma", ".weight")
        if "conv" in k and k.endswith(".weight") and v.ndim == 3:
            v = np.transpose(v, (0, 2, 1))
        out[k] = np.ascontiguousarray(v)
    return out


def write_quantized_model_dir(path: str, cfg: dict, weights: Dict[str, np.ndarray], group_size: int = 64,
                              bits: int = 8, scale_dtype: str = "float16") -> str:
    """A quantized checkpoint as MLX saves one: MLX key layout, config.json
    "quantization": {group_size, bits}, and for every quantizable Linear a uint32
    ``.weight`` with ``.scales`` / ``.biases`` (stored in ``scale_dtype``)."""
    os.makedirs(path, exist_ok=True)
    cfg = dict(cfg)
    cfg["quantization"] = {"group_size": group_size, "bits": bits}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    tensors = {}
    for k, v in to_mlx_layout(weights).items():
        if is_quantizable_linear(k, v.shape, group_size):
            packed, sc, bi = quantize_affine(v, group_size, bits)
            base = k[: -len(".weight")]
            tensors[k] = packed
            tensors[base + ".scales"] = sc
            tensors[base + ".biases"] = bi
        else:
            tensors[k] = np.ascontiguousarray(v, dtype=np.float32)
    _save_tensors(os.path.join(path, "model.safetensors"), tensors,
                  {k for k in tensors if k.endswith((".scales", ".biases"))}, scale_dtype)
    return path


def _save_tensors(fn: str, tensors: Dict[str, np.ndarray], reduced: set, reduced_dtype: str) -> None:
    """safetensors writer for float32 / uint32 tensors, ``reduced`` keys stored as f16/bf16."""
    header = {}
    blobs = []
    off = 0
    for k in sorted(tensors):
        v = tensors[k]
        if v.dtype == np.uint32:
            raw, tag = np.ascontiguousarray(v).tobytes(), "U32"
        elif k in reduced and reduced_dtype == "float16":
            raw, tag = np.ascontiguousarray(v, np.float32).astype(np.float16).tobytes(), "F16"
        elif k in reduced and reduced_dtype == "bfloat16":
            raw, tag = f32_to_bf16_bits(v).tobytes(), "BF16"
        else:
            raw, tag = np.ascontiguousarray(v, np.float32).tobytes(), "F32"
        header[k] = {"dtype": tag, "shape": list(v.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(fn, "wb") as f:
        f.write(np.uint64(len(hb)).tobytes())
        f.write(hb)
        for b in blobs:
            f.write(b)


def _save_reduced(path: str, weights: Dict[str, np.ndarray], dtype: str) -> None:
    """safetensors writer for bf16/f16 (numpy has no bfloat16): round-to-nearest-even."""
    header = {}
    blobs = []
    off = 0
    for k in sorted(weights):
        v = np.ascontiguousarray(weights[k], dtype=np.float32)
        if dtype == "float16":
            raw = v.astype(np.float16).tobytes()
            tag = "F16"
        elif dtype == "bfloat16":
            raw = f32_to_bf16_bits(v).tobytes()
            tag = "BF16"
        else:
            raise ValueError(dtype)
        header[k] = {"dtype": tag, "shape": list(v.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(os.path.join(path, "model.safetensors"), "wb") as f:
        f.write(np.uint64(len(hb)).tobytes())
        f.write(hb)
        for b in blobs:
            f.write(b)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def synth_audio(n_samples: int, seed: int, sample_rate: int = SAMPLE_RATE) -> np.ndarray:
    """Gaussian noise (std 0.05) + 3 sinusoids (amplitude 0.1), float32."""
    rng = np.random.Generator(np.random.PCG64(seed))
    freqs = rng.uniform(100.0, 3000.0, size=3)
    phases = rng.uniform(0.0, 2.0 * math.pi, size=3)
    noise = rng.normal(0.0, 0.05, size=n_samples)
    t = np.arange(n_samples, dtype=np.float64) / sample_rate
    x = noise
    for f, p in zip(freqs, phases):
        x = x + 0.1 * np.sin(2.0 * math.pi * f * t + p)
    return x.astype(np.float32)


def utterance_lengths(n: int, lo_s: float, hi_s: float, seed: int) -> np.ndarray:
    """Sample counts of a batch of utterances with durations ~U(lo_s, hi_s)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    secs = rng.uniform(lo_s, hi_s, size=n)
    return np.floor(secs * SAMPLE_RATE).astype(np.int64)


def ensure_model_dir(root: str, arch: str = "tiny", seed: Optional[int] = None,
                     dtype: str = "float32", quant: Optional[tuple] = None, **overrides) -> str:
    """Create (once) and return a seeded model directory under ``root``.  ``quant`` =
    (group_size, bits) writes an MLX affine-quantized checkpoint of the same weights."""
    if seed is None:
        seed = default_seed(arch)
    tag = f"{arch}_s{seed}_{dtype}"
    if quant:
        tag += f"_q{quant[0]}b{quant[1]}"
    if overrides:
        tag += "_" + "_".join(f"{k}{v}" for k, v in sorted(overrides.items())
                              if not isinstance(v, list))
    path = os.path.join(root, tag)
    if os.path.exists(os.path.join(path, "model.safetensors")):
        return path
    cfg = make_config(arch, **overrides)
    w = make_weights(cfg, seed)
    tmp = path + ".tmp%d" % os.getpid()
    if quant:
        write_quantized_model_dir(tmp, cfg, w, group_size=quant[0], bits=quant[1])
    else:
        write_model_dir(tmp, cfg, w, dtype=dtype)
    try:
        os.replace(tmp, path)
    except OSError:
        pass
    return path
