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
                     dtype: str = "float32", **overrides) -> str:
    """Create (once) and return a seeded model directory under ``root``."""
    if seed is None:
        seed = default_seed(arch)
    tag = f"{arch}_s{seed}_{dtype}"
    if overrides:
        tag += "_" + "_".join(f"{k}{v}" for k, v in sorted(overrides.items())
                              if not isinstance(v, list))
    path = os.path.join(root, tag)
    if os.path.exists(os.path.join(path, "model.safetensors")):
        return path
    cfg = make_config(arch, **overrides)
    w = make_weights(cfg, seed)
    tmp = path + ".tmp%d" % os.getpid()
    write_model_dir(tmp, cfg, w, dtype=dtype)
    try:
        os.replace(tmp, path)
    except OSError:
        pass
    return path
