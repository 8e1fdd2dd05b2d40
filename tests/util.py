"""Shared helpers for the parity tests (seeded models, oracle cache, tolerances)."""
import functools
import json
import os
import shutil

import numpy as np

from moonshine_b200 import synth

# fp32 logits tolerance: max |gpu - oracle| / max |oracle| per decoder call
FP32_LOGIT_TOL = 1e-3
# bf16 logits tolerance (same norm-relative measure)
BF16_LOGIT_TOL = 2e-2


def model_dir(root, arch="tiny", seed=None, dtype="float32", **overrides):
    return synth.ensure_model_dir(root, arch, seed=seed, dtype=dtype, **overrides)


def with_config(src_dir, dst_dir, **changes):
    """Copy of a model directory sharing its weights file, with config.json edits."""
    os.makedirs(dst_dir, exist_ok=True)
    with open(os.path.join(src_dir, "config.json")) as f:
        cfg = json.load(f)
    for k, v in changes.items():
        if k.startswith("encoder_config."):
            cfg["encoder_config"][k.split(".", 1)[1]] = v
        else:
            cfg[k] = v
    with open(os.path.join(dst_dir, "config.json"), "w") as f:
        json.dump(cfg, f)
    dst_w = os.path.join(dst_dir, "model.safetensors")
    if not os.path.exists(dst_w):
        os.symlink(os.path.join(src_dir, "model.safetensors"), dst_w)
    return dst_dir


@functools.lru_cache(maxsize=8)
def oracle_for(path, dtype=np.float64):
    from oracle.moonshine_oracle import Oracle
    return Oracle.from_dir(path, dtype)


def rel_err(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def assert_logits_close(gpu_rows, ref_rows, tol):
    assert len(gpu_rows) == len(ref_rows)
    errs = [rel_err(g, r) for g, r in zip(gpu_rows, ref_rows)]
    worst = max(errs) if errs else 0.0
    assert worst <= tol, f"worst per-step relative logits error {worst:.3e} > {tol} (steps: {np.round(errs, 6)})"
    return worst
