"""Benchmark: batch-1 Moonshine tiny transcription on B200 (decode tokens/s), plus the
batched, sharded and streaming workloads as extra keys of the same JSON line.

Headline workload (one "step"): 30 s of seeded synthetic 16 kHz audio through the frontend,
the sliding-window encoder, the once-per-utterance cross K/V projection and a 200-token
forced greedy decode (EOS ignored) of the tiny architecture (d 320, 6+6 layers, vocab
32768) with random-init fp32 weights and an fp16 KV cache.  Tokens/s counts encode time,
like the reference's tokensPerSecond (Sources/MoonshineMLX/MoonshineModel.swift:182).

Legs (keys of the same line; each can be skipped):
  word_timestamps  generateWithWordTimestamps on the headline audio
  quantized_4bit   the same weights as an MLX affine 4-bit checkpoint
  batched          small bf16, 64 utterances of U(5, 15) s, 128 forced tokens (per GPU)
  sharded          medium bf16, a fixed job of 256 utterances of U(2, 30) s, each decoding
                   its own limit ceil(6.5 s) with EOS ignored, partitioned over the N GPUs
                   (whole-box tokens/s, RTFx, per-rank imbalance)
  streaming        512 tiny fp32 streams split over the N GPUs, 80 ms chunks,
                   transcribe(isFinal: false, maxTokens: 16) after every chunk (aggregate
                   tokens/s, p50 / p99 per-chunk latency)

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 runs under torchrun, one process per GPU, each a full model replica (the path has no
cross-utterance state, so there is no collective on the data path; NCCL carries only the
timing barrier, the max-over-ranks reduction and the result gather).  `--impl reference`
times the CPU restatement of the reference on the host cores.
"""
import argparse
import gc
import hashlib
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "moonshine-mlx_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

ARCH = "tiny"
WEIGHT_SEED = 0
N_SAMPLES = 480000       # 30 s
AUDIO_SEED = 1
FORCED = 200
WORKLOAD = "tiny fp32 weights, fp16 KV, batch 1, 30 s audio, 200 forced tokens (encode + decode)"
FALLBACK_HBM_GBS = 6650.0


def decode_bytes_per_launch(cfg, M, n_tokens, kv_bytes=2):
    """Algorithmic HBM bytes of one decode launch (n_tokens decoder calls).

    Per call: every decoder weight once (layers, final norm, LM head), the embedding row,
    the cross K/V of all M frames (fp32 on the first call, stored dtype afterwards), the
    self K/V rows of earlier positions, and the new self K/V rows written."""
    d, I, L, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"], cfg["vocab_size"]
    HD = cfg["num_attention_heads"] * cfg["head_dim"]
    KVD = cfg["num_key_value_heads"] * cfg["head_dim"]
    per_layer = (HD + 2 * KVD) * d + d * HD + HD * d + d * HD + 2 * I * d + 2 * I + d * I + d + 3 * d
    w = (L * per_layer + d + V * d) * 4
    emb = d * 4
    cross0 = L * 2 * M * KVD * 4
    cross = L * 2 * M * KVD * kv_bytes
    self_reads = L * 2 * KVD * kv_bytes * (n_tokens * (n_tokens - 1) // 2)
    self_writes = L * 2 * KVD * kv_bytes * n_tokens
    return n_tokens * (w + emb) + cross0 + (n_tokens - 1) * cross + self_reads + self_writes


# DRAM traffic of one decode launch measured by ncu (dram__bytes_read.sum +
# dram__bytes_write.sum, 16 decoder calls at 1500 memory frames, fp16 KV), together with
# the sha256 of the kernel's source files at capture time.  Reported only while the sources
# are unchanged; otherwise the line carries traffic null.
KERNEL_SOURCES = {
    "cluster": ["csrc/kernels/decode_cluster.cu", "csrc/kernels/cluster_common.cuh", "csrc/kernels/common.cuh"],
    "grid": ["csrc/kernels/decode_b1.cu", "csrc/kernels/common.cuh"],
}
NCU_DECODE_TRAFFIC_16CALLS_1500F = {
    "cluster": {"bytes": 856079360 + 3237376, "sources_sha256": "4cf38cbb5ed3c704fa91609fc10d2fe26a5d52df23468cf10bf4b6eeab9b3a1b"},
}
DECODE_KERNEL_SYMBOL = {"cluster": "decode_cluster_kernel<40, 0>", "grid": "decode_b1_kernel<40>"}


def kernel_sources_sha256(kernel):
    h = hashlib.sha256()
    for rel in KERNEL_SOURCES.get(kernel, []):
        with open(os.path.join(PKG, rel), "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def decode_traffic_per_launch(M, n_tokens, kernel):
    rec = NCU_DECODE_TRAFFIC_16CALLS_1500F.get(kernel)
    if M != 1500 or rec is None or rec["sources_sha256"] != kernel_sources_sha256(kernel):
        return None
    return int(rec["bytes"] * n_tokens / 16)


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def bench_config(world):
    """The `config` object of both arms' lines."""
    return {"workload": WORKLOAD, "global_batch": world, "seq_len": FORCED,
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            "l2": "512 MB buffer written between timed steps"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.3)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[2:6]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU restatement

def oracle_setup():
    import numpy as np
    from moonshine_b200 import synth
    from oracle.moonshine_oracle import Oracle
    root = os.path.join(tempfile.gettempdir(), "moonshine_b200_bench")
    path = synth.ensure_model_dir(root, ARCH, seed=WEIGHT_SEED)
    return Oracle.from_dir(path, np.float32), synth.synth_audio(N_SAMPLES, AUDIO_SEED)


def oracle_step(o, audio):
    """One step of the headline workload on the numpy float32 restatement: the 30 s
    encode, the cross K/V and all FORCED decoder calls with greedy feedback."""
    import numpy as np
    t0 = time.perf_counter()
    cache = o.new_cache(o.memory_for(audio), True)
    tok = o.cfg.decoder_start_token_id
    for _ in range(FORCED):
        _, lg = o.decoder_step(tok, cache)
        tok = int(np.argmax(lg))
    return time.perf_counter() - t0


def cpu_baseline_oracle(n_steps=3):
    """The numpy float32 restatement on all host threads, timed over `n_steps` whole steps of
    the headline workload (median)."""
    o, audio = oracle_setup()
    times = [oracle_step(o, audio) for _ in range(n_steps)]
    t = statistics.median(times)
    return {"value": round(FORCED / t, 3), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"numpy float32 restatement of the reference (Swift/MLX cannot run here): "
                      f"{n_steps} whole steps (30 s encode + cross K/V + {FORCED} decoder calls), median",
            "s_per_step": round(t, 4)}


def run_reference(args, rank, world):
    if rank != 0:
        return
    o, audio = oracle_setup()
    for _ in range(args.warmup):
        oracle_step(o, audio)
    times = [oracle_step(o, audio) for _ in range(args.steps)]
    ms = 1e3 * sum(times) / len(times)
    val = FORCED / (ms / 1e3)
    line = {
        "impl": "reference", "metric": "decode tokens/s", "value": round(val, 3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(world),
        "cpu_baseline": {"value": round(val, 3), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"numpy float32 restatement of the reference (Swift/MLX cannot run here): "
                                   f"whole steps (30 s encode + cross K/V + {FORCED} decoder calls)"},
        "e2e": {"value": round(val, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU legs

def _events(torch, stream):
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    return a, b


def leg_batched(mb, synth, root, torch, barrier, rank, local, reps=3):
    """ms_generate_batch on small bf16: 64 utterances of U(5, 15) s, 128 forced tokens each,
    host buffers in and out; CUDA events on the model's stream around the public call."""
    import numpy as np
    if rank == 0:
        synth.ensure_model_dir(root, "small", seed=2, dtype="bfloat16")
    barrier()
    bpath = synth.ensure_model_dir(root, "small", seed=2, dtype="bfloat16")
    brng = np.random.Generator(np.random.PCG64(7))
    blens = (brng.uniform(5, 15, size=64) * 16000).astype(int) // 80 * 80
    baudio = [synth.synth_audio(int(n), 100 + i) for i, n in enumerate(blens)]
    bm = mb.MoonshineModel.load(bpath, device=local)
    s = torch.cuda.ExternalStream(bm.cuda_stream)
    bm.generate_batch(baudio, forced_len=128)
    b_enc, b_dec, b_ms = [], [], []
    torch.cuda.nvtx.range_push("batched")  # profilers can select this leg's kernels (ncu --nvtx)
    for _ in range(reps):
        e0, e1 = _events(torch, s)
        e0.record(s)
        bids, bst = bm.generate_batch(baudio, forced_len=128)
        e1.record(s)
        torch.cuda.synchronize()
        assert all(len(r) == 128 for r in bids)
        b_ms.append(e0.elapsed_time(e1))
        b_enc.append(bst.encode_ms)
        b_dec.append(bst.decode_ms)
    torch.cuda.nvtx.range_pop()
    bm.close()
    med = statistics.median(b_ms)
    return {"workload": "small bf16 weights, 64 utterances of U(5, 15) s, 128 forced tokens each",
            "encode_ms": round(statistics.median(b_enc), 2), "decode_ms": round(statistics.median(b_dec), 2),
            "ms": round(med, 2), "ms_per_step_decode": round(statistics.median(b_dec) / 128, 4),
            "tokens_per_s_per_gpu": round(64 * 128 / (med / 1e3), 1),
            "audio_s": round(float(blens.sum()) / 16000.0, 2),
            "timing": f"CUDA events on the model stream around the public call incl. host copies "
                      f"(median of {reps})"}


def leg_sharded(mb, synth, root, torch, dist, barrier, rank, world, local, reps=2, sub_batch=256):
    """A fixed job of 256 medium bf16 utterances of U(2, 30) s, each decoding its own limit
    ceil(6.5 s) with EOS ignored, partitioned by length over the ranks (shard.py).  Each rank
    runs its share through ms_generate_batch in length-sorted groups of at most `sub_batch`
    utterances (by default one call for the whole share: a lockstep step costs about the same
    for 256 rows as for 64); time per rank by CUDA events on its model stream, job time = max over ranks;
    ids gathered on rank 0."""
    import numpy as np
    from moonshine_b200 import shard
    if rank == 0:
        synth.ensure_model_dir(root, "medium", seed=3, dtype="bfloat16")
    barrier()
    path = synth.ensure_model_dir(root, "medium", seed=3, dtype="bfloat16")
    rng = np.random.Generator(np.random.PCG64(11))
    lens = (rng.uniform(2, 30, size=256) * 16000).astype(int) // 80 * 80
    share = shard.partition_by_length(lens.tolist(), world)[rank]
    order = sorted(share, key=lambda i: -int(lens[i]))
    groups = [order[k:k + sub_batch] for k in range(0, len(order), sub_batch)]
    audio = {i: synth.synth_audio(int(lens[i]), 1000 + i) for i in share}
    m = mb.MoonshineModel.load(path, device=local)
    s = torch.cuda.ExternalStream(m.cuda_stream)
    m.generate_batch([audio[i] for i in groups[0]], forced_len=-1)   # warm-up: weights, graphs
    times, results = [], {}
    for rep in range(reps):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = _events(torch, s)
        torch.cuda.nvtx.range_push(f"sharded_{rep}")  # one timed job's kernels, for ncu --nvtx
        e0.record(s)
        for g in groups:
            ids, _ = m.generate_batch([audio[i] for i in g], forced_len=-1)
            for i, r in zip(g, ids):
                results[i] = r
        e1.record(s)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / 1e3)
    m.close()
    t_rank = statistics.median(times)
    toks = sum(len(results[i]) for i in share)
    expect = sum(int(math.ceil(lens[i] / 16000.0 * 6.5)) for i in share)
    assert toks == expect, (toks, expect)
    t_max, t_mean, tok_all = t_rank, t_rank, toks
    if dist is not None:
        t = torch.tensor([t_rank, t_rank, float(toks)], dtype=torch.float64, device=f"cuda:{local}")
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        t_max, t_mean, tok_all = float(mx[0]), float(t[1]) / world, int(t[2])
    gathered = shard.gather_results([results[i] for i in share], share, len(lens))
    if rank != 0:
        return None
    assert all(r is not None for r in gathered)
    audio_s = float(lens.sum()) / 16000.0
    return {"workload": "medium bf16 weights, 256 utterances of U(2, 30) s (a fixed job, partitioned by length "
                        "over the GPUs), each decoding ceil(6.5 tokens per second) with EOS ignored",
            "n_gpus": world, "tokens": tok_all, "audio_s": round(audio_s, 1),
            "job_s": round(t_max, 4), "tokens_per_s": round(tok_all / t_max, 1),
            "rtfx": round(audio_s / t_max, 1), "rank_imbalance": round(t_max / t_mean, 4),
            "utterances_per_gpu_call": min(sub_batch, len(share)),
            "timing": "CUDA events on each rank's model stream around its generate_batch calls (host buffers, "
                      f"median of {reps}), job time = max over ranks"}


def leg_streaming(mb, synth, torch, dist, barrier, rank, world, local, root, n_streams=512, n_chunks=125,
                  chunk=1280, max_tokens=16):
    """512 tiny fp32 streams (split over the ranks), 80 ms chunks, after every chunk
    transcribe(isFinal: false, maxTokens: 16) of every stream of the rank: one
    ms_stream_add_audio_batch and one ms_stream_transcribe_batch per chunk, whose encoders run
    as one tensor-core pass and whose decodes run in lockstep on the tensor cores
    with split bf16 operands (fp32-level products for this fp32 checkpoint).  Per-chunk
    latency = the time of that call for the rank's streams (CUDA events); p50 / p99 over
    chunks and ranks."""
    import numpy as np
    if rank == 0:
        synth.ensure_model_dir(root, ARCH, seed=WEIGHT_SEED)
    barrier()
    path = synth.ensure_model_dir(root, ARCH, seed=WEIGHT_SEED)
    mine = list(range(rank, n_streams, world))
    m = mb.MoonshineModel.load(path, device=local, kv_fp16=True)
    s = torch.cuda.ExternalStream(m.cuda_stream)
    audio = {i: synth.synth_audio(n_chunks * chunk, 5000 + i) for i in mine}
    sc = mb.StreamingConfig(batch_decode=True)
    # warm-up on separate streams over the whole job, untimed: weight planes, and the device
    # memory of every buffer size the job reaches (stream-ordered pool growth maps new device
    # memory, which took up to ~1 s per growth on the B200 boxes; the blocks freed when the
    # warm-up streams close are reused by the timed ones), so the timed chunks are steady-state
    # serving
    warm = [m.create_stream() for _ in mine]
    for st in warm:
        m.start_stream(st)
    for k in range(n_chunks):
        m.add_audio_batch(warm, [audio[i][k * chunk:(k + 1) * chunk] for i in mine])
        m.transcribe_batch(warm, is_final=False, streaming_config=sc, max_tokens=max_tokens)
    for st in warm:
        st.close()
    # the harness's own objects out of the cyclic collector's scans (a full collection of them
    # took ~35 ms inside a timed chunk)
    gc.collect()
    gc.freeze()
    states = [m.create_stream() for _ in mine]
    for st in states:
        m.start_stream(st)
    lat, toks = [], 0
    barrier()
    torch.cuda.synchronize()
    t_all0, t_all1 = _events(torch, s)
    t_all0.record(s)
    for k in range(n_chunks):
        e0, e1 = _events(torch, s)
        torch.cuda.nvtx.range_push(f"streaming_chunk_{k}")  # one chunk's kernels, for ncu --nvtx
        e0.record(s)
        m.add_audio_batch(states, [audio[i][k * chunk:(k + 1) * chunk] for i in mine])
        out = m.transcribe_batch(states, is_final=False, streaming_config=sc, max_tokens=max_tokens)
        e1.record(s)
        torch.cuda.nvtx.range_pop()
        toks += sum(len(o[0]) for o in out)
        lat.append((e0, e1))
    t_all1.record(s)
    torch.cuda.synchronize()
    gc.unfreeze()
    lat_ms = [a.elapsed_time(b) for a, b in lat]
    total_s = t_all0.elapsed_time(t_all1) / 1e3
    for st in states:
        st.close()
    m.close()
    all_lat = lat_ms
    t_max, tok_all = total_s, toks
    if dist is not None:
        t = torch.tensor(lat_ms + [total_s, float(toks)], dtype=torch.float64, device=f"cuda:{local}")
        got = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(got, t)
        all_lat = [float(x) for g in got for x in g[:-2].tolist()]
        t_max = max(float(g[-2]) for g in got)
        tok_all = int(sum(float(g[-1]) for g in got))
    if rank != 0:
        return None
    a = np.asarray(all_lat)
    return {"workload": f"{n_streams} tiny fp32 streams (fp16 KV), {n_chunks} chunks of 80 ms each, "
                        f"transcribe(isFinal: false, maxTokens: {max_tokens}) of every stream after every chunk "
                        "(lockstep decode of the GPU's streams, split bf16 operands: fp32-level products)",
            "n_gpus": world, "streams_per_gpu": len(mine), "decoded_tokens": tok_all,
            "tokens_per_s": round(tok_all / t_max, 1), "chunk_ms_p50": round(float(np.percentile(a, 50)), 3),
            "chunk_ms_p99": round(float(np.percentile(a, 99)), 3), "job_s": round(t_max, 3),
            "timing": "CUDA events on each rank's model stream around add_audio + transcribe_batch of its streams "
                      "per chunk (host buffers); job time = max over ranks"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-timestamps", action="store_true", help="skip the word-timestamp leg")
    ap.add_argument("--no-quantized", action="store_true", help="skip the 4-bit checkpoint leg")
    ap.add_argument("--no-batched", action="store_true", help="skip the small-model batched leg")
    ap.add_argument("--no-sharded", action="store_true", help="skip the medium-model sharded job")
    ap.add_argument("--no-streaming", action="store_true", help="skip the 512-stream leg")
    ap.add_argument("--stream-chunks", type=int, default=125, help="80 ms chunks per stream")
    ap.add_argument("--seconds", type=float, default=30.0, help="audio length (profiling cases)")
    ap.add_argument("--tokens", type=int, default=200, help="forced decode length (profiling cases)")
    ap.add_argument("--flush-mb", type=int, default=512, help="L2-flush buffer written between steps")
    args = ap.parse_args()
    global N_SAMPLES, FORCED, WORKLOAD
    if args.seconds != 30.0 or args.tokens != 200:
        N_SAMPLES = int(args.seconds * 16000) // 80 * 80
        FORCED = args.tokens
        WORKLOAD = (f"tiny fp32 weights, fp16 KV, batch 1, {args.seconds:g} s audio, "
                    f"{FORCED} forced tokens (encode + decode)")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        args.warmup = 3

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    import moonshine_b200 as mb
    from moonshine_b200 import synth

    root = os.path.join(tempfile.gettempdir(), "moonshine_b200_bench")
    if rank == 0:
        path = synth.ensure_model_dir(root, ARCH, seed=WEIGHT_SEED)
    barrier()
    path = synth.ensure_model_dir(root, ARCH, seed=WEIGHT_SEED)
    model = mb.MoonshineModel.load(path, device=local, kv_fp16=True)
    cfg = json.load(open(os.path.join(path, "config.json")))
    stream = torch.cuda.ExternalStream(model.cuda_stream)

    audio_np = synth.synth_audio(N_SAMPLES, AUDIO_SEED)
    audio_pinned = torch.from_numpy(audio_np).pin_memory()
    audio_dev = audio_pinned.to(f"cuda:{local}")
    ids_dev = torch.zeros(FORCED + 8, dtype=torch.int32, device=f"cuda:{local}")
    # > 126 MB L2; profiling captures may shrink it (less device memory to save/restore)
    flush = torch.empty(max(1, args.flush_mb) << 20, dtype=torch.uint8, device=f"cuda:{local}")
    torch.cuda.synchronize()

    def run_device():
        return model.generate_device(audio_dev.data_ptr(), N_SAMPLES, ids_dev.data_ptr(), ids_dev.numel(),
                                     forced_len=FORCED)

    for _ in range(args.warmup):
        run_device()
    torch.cuda.synchronize()

    # ---- device-resident timing (value)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    dec_ms, enc_ms, ntok, kernels = [], [], 0, set()
    barrier()
    torch.cuda.synchronize()
    mb.reset_kernel_launches()
    with ClockSampler(local) as clocks:
        for k in range(args.steps):
            with torch.cuda.stream(stream):
                flush.fill_(k & 0xFF)            # evict L2 between steps (outside the events)
            evs[k][0].record(stream)
            n, st = run_device()
            evs[k][1].record(stream)
            ntok += n
            kernels.add(mb.DECODE_KERNEL_NAMES.get(st.decode_kernel, "?"))
            dec_ms.append(st.decode_ms)
            enc_ms.append(st.encode_ms)
        torch.cuda.synchronize()
    launches = mb.kernel_launches()
    barrier()
    t_rank = sum(a.elapsed_time(b) for a, b in evs)
    assert ntok == FORCED * args.steps, ntok

    # ---- end-to-end through the public API with host buffers (e2e)
    e2e_evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    host_audio = audio_pinned.numpy()
    for _ in range(args.warmup):  # the host-buffer path's own first-use work (its upload buffer), untimed
        model.generate(host_audio, forced_len=FORCED)
    barrier()
    torch.cuda.synchronize()
    for k in range(args.steps):
        with torch.cuda.stream(stream):
            flush.fill_(k & 0xFF)
        e2e_evs[k][0].record(stream)
        out = model.generate(host_audio, forced_len=FORCED)
        e2e_evs[k][1].record(stream)
        assert len(out.tokens) == FORCED
    torch.cuda.synchronize()
    barrier()
    t_e2e = sum(a.elapsed_time(b) for a, b in e2e_evs)

    # ---- word timestamps (generateWithWordTimestamps) on the same audio, host buffers: the
    # greedy decode with the cross queries kept, the attention-row kernels and the host DTW,
    # against a plain greedy generate of the same number of decoder calls
    ts = None
    if not args.no_timestamps:
        al = model.generate_alignment(host_audio)
        n_calls = len(al.token_probs)
        t_al, t_gen = [], []
        for k in range(3):
            for fn, acc in ((lambda: model.generate_alignment(host_audio), t_al),
                            (lambda: model.generate(host_audio, forced_len=n_calls), t_gen)):
                with torch.cuda.stream(stream):
                    flush.fill_(k & 0xFF)
                e0, e1 = _events(torch, stream)
                e0.record(stream)
                fn()
                e1.record(stream)
                torch.cuda.synchronize()
                acc.append(e0.elapsed_time(e1))
        ts = {"decoder_calls": n_calls, "memory_frames": al.n_frames,
              "ms_per_call": round(statistics.median(t_al), 3),
              "generate_same_calls_ms": round(statistics.median(t_gen), 3),
              "overhead_ms": round(statistics.median(t_al) - statistics.median(t_gen), 3),
              "timing": "CUDA events on the model stream around the public call (median of 3), L2 flushed "
                        "before each"}

    # ---- the same weights as an MLX affine 4-bit checkpoint (group 64), device-resident audio:
    # the clustered kernel streams the LM head as codes (the default quant_stream)
    qleg = None
    if not args.no_quantized:
        if rank == 0:
            synth.ensure_model_dir(root, ARCH, seed=WEIGHT_SEED, quant=(64, 4))
        barrier()
        qpath = synth.ensure_model_dir(root, ARCH, seed=WEIGHT_SEED, quant=(64, 4))
        qm = mb.MoonshineModel.load(qpath, device=local, kv_fp16=True)
        qstream = torch.cuda.ExternalStream(qm.cuda_stream)
        for _ in range(args.warmup):
            qm.generate_device(audio_dev.data_ptr(), N_SAMPLES, ids_dev.data_ptr(), ids_dev.numel(), forced_len=FORCED)
        q_evs, q_dec = [], []
        torch.cuda.synchronize()
        for k in range(min(args.steps, 8)):
            with torch.cuda.stream(qstream):
                flush.fill_(k & 0xFF)
            e0, e1 = _events(torch, qstream)
            e0.record(qstream)
            n, st = qm.generate_device(audio_dev.data_ptr(), N_SAMPLES, ids_dev.data_ptr(), ids_dev.numel(),
                                       forced_len=FORCED)
            e1.record(qstream)
            assert n == FORCED
            q_evs.append((e0, e1))
            q_dec.append(st.decode_ms)
        torch.cuda.synchronize()
        q_ms = statistics.mean(a.elapsed_time(b) for a, b in q_evs)
        qleg = {"checkpoint": "MLX affine 4-bit, group 64 (same weights)", "streamed_bits": list(qm.decode_weight_bits),
                "tokens_per_s_per_gpu": round(FORCED / (q_ms / 1e3), 2),
                "ms_per_token_decode": round(statistics.mean(q_dec) / FORCED, 5),
                "timing": "CUDA events per step (encode + decode), L2 flushed before each"}
        qm.close()
        barrier()

    bleg = None if args.no_batched else leg_batched(mb, synth, root, torch, barrier, rank, local)
    barrier()
    sleg = None if args.no_sharded else leg_sharded(mb, synth, root, torch, dist, barrier, rank, world, local)
    barrier()
    stleg = None
    if not args.no_streaming:
        stleg = leg_streaming(mb, synth, torch, dist, barrier, rank, world, local, root, n_chunks=args.stream_chunks)
    barrier()

    if dist is not None:
        t = torch.tensor([t_rank, t_e2e], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_rank, t_e2e = float(t[0]), float(t[1])

    if rank == 0:
        M = (((N_SAMPLES // 80) - 1) // 2 + 1 - 1) // 2 + 1
        bytes_launch = decode_bytes_per_launch(cfg, M, FORCED)
        dec_avg = statistics.mean(dec_ms)
        achieved = bytes_launch / (dec_avg / 1e3) / 1e9
        peak, peak_kind = measured_peak()
        total_tokens = world * FORCED * args.steps
        value = total_tokens / (t_rank / 1e3)
        kern = kernels.pop() if len(kernels) == 1 else "mixed"
        traffic = decode_traffic_per_launch(M, FORCED, kern)
        line = {
            "metric": "decode tokens/s", "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_rank / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, seeded noise+sinusoid audio)",
            "config": bench_config(world),
            "ms_per_token_decode": round(dec_avg / FORCED, 5),
            "encode_ms": round(statistics.mean(enc_ms), 4),
            "rtfx": round((N_SAMPLES / 16000.0) / (t_rank / args.steps / 1e3), 1),
            "gpu_launches": int(launches),
            "roofline": {"bound": "hbm", "kernel": DECODE_KERNEL_SYMBOL.get(kern, kern),
                         "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": peak_kind, "algorithmic_bytes_per_launch": int(bytes_launch),
                         "launch_ms": round(dec_avg, 4), "traffic": traffic,
                         "traffic_source": ("ncu dram__bytes of a 16-call launch at 1500 frames on the same kernel "
                                            "sources, scaled by decoder calls") if traffic else None},
            "e2e": {"value": round(total_tokens / (t_e2e / 1e3), 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": N_SAMPLES * 4, "d2h_bytes_per_step": FORCED * 4 + 16},
            "clocks": clocks.summary(),
        }
        if ts is not None:
            line["word_timestamps"] = ts
        if qleg is not None:
            line["quantized_4bit"] = qleg
        if bleg is not None:
            line["batched"] = bleg
        if sleg is not None:
            line["sharded"] = sleg
        if stleg is not None:
            line["streaming"] = stleg
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_oracle()
        print(json.dumps(line), flush=True)
    model.close()
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
