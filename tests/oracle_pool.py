"""Per-utterance oracle checks of a batched GPU run, spread over a process pool.

Large batches (64 utterances x 128 decoder calls) are too slow for one oracle process, so
the comparison of each utterance runs in a worker of a `spawn` pool (safe to start after
the GPU is in use; each worker keeps numpy's BLAS single-threaded).  The GPU side saves
its logits to a .npy file that the workers memory-map, so no large array is pickled."""
import functools
import multiprocessing as mp
import os

import numpy as np

from util import BF16_LOGIT_TOL


@functools.lru_cache(maxsize=2)
def _oracle(path, dtype_name):
    from oracle.moonshine_oracle import Oracle
    return Oracle.from_dir(path, getattr(np, dtype_name))


def check_row(job):
    """Greedy ids may part from the oracle's only at a near-tie (a step whose top-2 margin is
    within the bf16 tolerance of the logits scale); logits up to and including that step
    must agree within the tolerance.  Returns (row, error message or None, worst logits
    error, step the ids part at or -1, smallest relative top-2 margin seen)."""
    (row, path, dtype_name, n_samples, audio_seed, forced, kv_fp16, gpu_ids, logits_file, tol) = job
    from moonshine_b200 import synth
    o = _oracle(path, dtype_name)
    audio = synth.synth_audio(n_samples, audio_seed)
    mem = o.memory_for(audio)
    ref, _, ref_logits, margins = o.greedy(mem, forced, kv_fp16, forced_len=forced, keep_logits=True)
    gl = np.load(logits_file, mmap_mode="r")[row]
    k = next((i for i, (x, y) in enumerate(zip(gpu_ids, ref)) if x != y), None)
    rel_margins = [m / max(float(np.max(np.abs(l))), 1e-30) for m, l in zip(margins, ref_logits)]
    if k is None:
        if len(gpu_ids) != len(ref):
            return row, f"row {row}: {len(gpu_ids)} ids vs {len(ref)}", 0.0, -1, min(rel_margins)
        k_cmp = len(ref_logits) - 1
    else:
        if rel_margins[k] > tol:
            return (row, f"row {row}: ids part at step {k} with relative margin {rel_margins[k]:.4f}", 0.0, k,
                    min(rel_margins))
        k_cmp = k
    worst = 0.0
    for i in range(k_cmp + 1):
        r = np.asarray(ref_logits[i], np.float64)
        g = np.asarray(gl[i], np.float64)
        worst = max(worst, float(np.max(np.abs(g - r)) / max(np.max(np.abs(r)), 1e-30)))
    err = None if worst <= tol else f"row {row}: logits error {worst:.3e} > {tol}"
    return row, err, worst, (-1 if k is None else k), min(rel_margins)


def check_batch(path, lens, audio_seeds, forced, kv_fp16, gpu_ids, gpu_logits, tmpdir,
                dtype_name="float32", tol=BF16_LOGIT_TOL):
    """Checks every row of a batched run against the oracle in parallel; returns the list of
    per-row results of check_row."""
    f = os.path.join(str(tmpdir), "gpu_logits.npy")
    np.save(f, gpu_logits)
    jobs = [(b, path, dtype_name, int(lens[b]), int(audio_seeds[b]), forced, kv_fp16, list(gpu_ids[b]), f, tol)
            for b in range(len(lens))]
    n = max(1, min(len(jobs), os.cpu_count() or 1, 16))
    old = {k: os.environ.get(k) for k in ("OPENBLAS_NUM_THREADS", "OMP_NUM_THREADS", "MKL_NUM_THREADS")}
    for k in old:
        os.environ[k] = "1"
    try:
        with mp.get_context("spawn").Pool(n) as pool:
            out = pool.map(check_row, jobs, chunksize=1)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return out
