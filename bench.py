"""Benchmark: batch-1 Moonshine tiny transcription on B200 (decode tokens/s).

Workload (one "step"): 30 s of seeded synthetic 16 kHz audio through the frontend,
the sliding-window encoder, the once-per-utterance cross K/V projection and a 200-token
forced greedy decode (EOS ignored) of the tiny architecture (d 320, 6+6 layers,
vocab 32768) with random-init fp32 weights and an fp16 KV cache.  Tokens/s counts encode
time, like the reference's tokensPerSecond (Sources/MoonshineMLX/MoonshineModel.swift:182).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 runs under torchrun, one process per GPU, each an independent full replica
(the path has no cross-utterance state, so there is no collective on the data path).
`--impl reference` times the CPU restatement of the reference on the host cores.
"""
import argparse
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


# dram__bytes_read.sum + dram__bytes_write.sum of one decode launch (16 decoder calls, 1500
# memory frames, fp16 KV) from an ncu capture of each batch-1 kernel; per-call traffic is
# flat after the first call.
NCU_DECODE_BYTES_16CALLS_1500F = {
    "cluster": (857855232 + 3086336, "profiles/decode_cluster_tiny_30s_16tok.md"),
    "grid": (830.744e6 + 5.621e6, "profiles/decode_b1_tiny_30s_16tok.md"),
}
DECODE_KERNEL_SYMBOL = {"cluster": "decode_cluster_kernel<40, 0>", "grid": "decode_b1_kernel<40>"}


def decode_traffic_per_launch(M, n_tokens, kernel):
    if M != 1500 or kernel not in NCU_DECODE_BYTES_16CALLS_1500F:
        return None, None
    b, src = NCU_DECODE_BYTES_16CALLS_1500F[kernel]
    return int(b * n_tokens / 16), src


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


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


def cpu_baseline_oracle(budget_tokens=40):
    """Times the numpy restatement (float32, all host threads) on a bounded sample of the
    workload: the full 30 s encode + cross K/V and `budget_tokens` decoder calls; the
    200-token figure is extrapolated from the measured per-token time."""
    import numpy as np
    from moonshine_b200 import synth
    from oracle.moonshine_oracle import Oracle
    root = os.path.join(tempfile.gettempdir(), "moonshine_b200_bench")
    path = synth.ensure_model_dir(root, ARCH, seed=WEIGHT_SEED)
    o = Oracle.from_dir(path, np.float32)
    audio = synth.synth_audio(N_SAMPLES, AUDIO_SEED)
    t0 = time.perf_counter()
    mem = o.memory_for(audio)
    t1 = time.perf_counter()
    cache = o.new_cache(mem, True)
    t2 = time.perf_counter()
    tok = o.cfg.decoder_start_token_id
    for _ in range(budget_tokens):
        _, lg = o.decoder_step(tok, cache)
        tok = int(np.argmax(lg))
    t3 = time.perf_counter()
    per_tok = (t3 - t2) / budget_tokens
    total = (t1 - t0) + (t2 - t1) + per_tok * FORCED
    return {"value": FORCED / total, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"numpy float32 oracle: 30 s encode + cross K/V + {budget_tokens} decoder calls, "
                      f"{FORCED}-token time extrapolated ({per_tok * 1e3:.2f} ms/token)",
            "encode_s": round(t1 - t0, 4), "ms_per_token": round(per_tok * 1e3, 4)}


def run_reference(args, rank, world):
    if rank != 0:
        return
    import numpy as np
    from moonshine_b200 import synth
    from oracle.moonshine_oracle import Oracle
    root = os.path.join(tempfile.gettempdir(), "moonshine_b200_bench")
    path = synth.ensure_model_dir(root, ARCH, seed=WEIGHT_SEED)
    o = Oracle.from_dir(path, np.float32)
    audio = synth.synth_audio(N_SAMPLES, AUDIO_SEED)
    # each step: 30 s encode + cross K/V + `n_tok` decoder calls, n_tok sized so the whole
    # run stays within ~3 minutes; tokens/s extrapolates the decode to 200 tokens
    per_step_budget_s = 150.0 / max(1, args.steps + args.warmup)
    n_tok = max(4, min(FORCED, int((per_step_budget_s - 3.5) / 0.012)))

    def step():
        t0 = time.perf_counter()
        mem = o.memory_for(audio)
        cache = o.new_cache(mem, True)
        t1 = time.perf_counter()
        tok = o.cfg.decoder_start_token_id
        for _ in range(n_tok):
            _, lg = o.decoder_step(tok, cache)
            tok = int(np.argmax(lg))
        t2 = time.perf_counter()
        return (t1 - t0) + (t2 - t1) * FORCED / n_tok

    for _ in range(args.warmup):
        step()
    times = [step() for _ in range(args.steps)]
    ms = 1e3 * sum(times) / len(times)
    val = FORCED / (ms / 1e3)
    line = {
        "impl": "reference", "metric": "decode tokens/s", "value": round(val, 3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": 1, "parallelism": "replicas"},
        "cpu_baseline": {"value": round(val, 3), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"numpy float32 restatement of the reference (Swift/MLX cannot run here): "
                                   f"30 s encode + {n_tok} decoder calls per step, decode extrapolated to "
                                   f"{FORCED} tokens"},
        "e2e": {"value": round(val, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-timestamps", action="store_true", help="skip the word-timestamp leg")
    ap.add_argument("--no-quantized", action="store_true", help="skip the 4-bit checkpoint leg")
    ap.add_argument("--batched", action="store_true",
                    help="add the batched leg: small architecture, bf16 weights, 64 utterances of 5-15 s, "
                         "128 forced tokens each")
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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    import numpy as np
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
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                fn()
                torch.cuda.synchronize()
                acc.append((time.perf_counter() - t0) * 1e3)
        ts = {"decoder_calls": n_calls, "memory_frames": al.n_frames,
              "ms_per_call": round(statistics.median(t_al), 3),
              "generate_same_calls_ms": round(statistics.median(t_gen), 3),
              "overhead_ms": round(statistics.median(t_al) - statistics.median(t_gen), 3),
              "timing": "host wall clock around the public call (median of 3), L2 flushed before each"}

    # ---- the same weights as an MLX affine 4-bit checkpoint (group 64), device-resident audio:
    # the clustered kernel streams the LM head as codes (the default quant_stream)
    qleg = None
    if not args.no_quantized:
        if rank == 0:
            qpath = synth.ensure_model_dir(root, ARCH, seed=WEIGHT_SEED, quant=(64, 4))
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
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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
        del qm
        barrier()

    # ---- batched generation (ms_generate_batch): small architecture, bf16 checkpoint, 64
    # independent utterances of U(5, 15) s, 128 forced tokens each, host buffers in and out
    bleg = None
    if args.batched:
        if rank == 0:
            bpath = synth.ensure_model_dir(root, "small", seed=2, dtype="bfloat16")
        barrier()
        bpath = synth.ensure_model_dir(root, "small", seed=2, dtype="bfloat16")
        brng = np.random.Generator(np.random.PCG64(7))
        blens = (brng.uniform(5, 15, size=64) * 16000).astype(int) // 80 * 80
        baudio = [synth.synth_audio(int(n), 100 + i) for i, n in enumerate(blens)]
        bm = mb.MoonshineModel.load(bpath, device=local)
        bm.generate_batch(baudio, forced_len=128)
        b_enc, b_dec, b_wall = [], [], []
        for _ in range(3):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            bids, bst = bm.generate_batch(baudio, forced_len=128)
            b_wall.append((time.perf_counter() - t0) * 1e3)
            assert all(len(r) == 128 for r in bids)
            b_enc.append(bst.encode_ms)
            b_dec.append(bst.decode_ms)
        bleg = {"workload": "small bf16 weights, 64 utterances of U(5, 15) s, 128 forced tokens each",
                "encode_ms": round(statistics.median(b_enc), 2), "decode_ms": round(statistics.median(b_dec), 2),
                "wall_ms": round(statistics.median(b_wall), 2),
                "tokens_per_s_per_gpu": round(64 * 128 / (statistics.median(b_wall) / 1e3), 1),
                "audio_s": round(float(blens.sum()) / 16000.0, 2),
                "timing": "host wall clock around the public call incl. host copies (median of 3)"}
        del bm
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
        traffic, traffic_src = decode_traffic_per_launch(M, FORCED, kern)
        line = {
            "metric": "decode tokens/s", "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_rank / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, seeded noise+sinusoid audio)",
            "config": {"workload": WORKLOAD, "global_batch": world, "seq_len": FORCED,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": f"{args.flush_mb} MB buffer written between timed steps"},
            "ms_per_token_decode": round(dec_avg / FORCED, 5),
            "encode_ms": round(statistics.mean(enc_ms), 4),
            "rtfx": round((N_SAMPLES / 16000.0) / (t_rank / args.steps / 1e3), 1),
            "gpu_launches": int(launches),
            "roofline": {"bound": "hbm", "kernel": DECODE_KERNEL_SYMBOL.get(kern, kern),
                         "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": peak_kind, "algorithmic_bytes_per_launch": int(bytes_launch),
                         "launch_ms": round(dec_avg, 4), "traffic": traffic,
                         "traffic_source": (f"ncu dram__bytes of a 16-call launch at 1500 frames, scaled by "
                                            f"decoder calls ({traffic_src})") if traffic_src else None},
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
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_oracle()
        print(json.dumps(line), flush=True)
    del model
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
