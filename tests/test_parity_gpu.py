"""CUDA path vs the CPU oracle on seeded random-init models and synthetic audio.

Token ids must be identical; logits must agree within 1e-3 (fp32 weights) measured as
max |gpu - oracle| / max |oracle| per decoder call."""
import functools

import numpy as np
import pytest

from moonshine_b200 import synth
from util import (FP32_LOGIT_TOL, assert_logits_close, model_dir, oracle_for, rel_err,
                  with_config)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_dir(model_root):
    return model_dir(model_root, "tiny")


@pytest.fixture(scope="module")
def tiny(tiny_dir):
    import moonshine_b200 as mb
    return mb.MoonshineModel.load(tiny_dir)


@pytest.mark.parametrize("n_samples,seed", [(32000, 7), (105600, 0), (12345, 3)])
def test_encode_matches_oracle(tiny, tiny_dir, n_samples, seed):
    audio = synth.synth_audio(n_samples, seed)
    mem = tiny.encode(audio)
    ref = oracle_for(tiny_dir).memory_for(audio)
    assert mem.shape == ref.shape
    assert rel_err(mem, ref) < 1e-4


@pytest.mark.parametrize("kv_fp16", [False, True])
def test_forced_decode_6p6s(tiny, tiny_dir, kv_fp16):
    """6.6 s of audio, 64 forced tokens, EOS ignored (the batch-1 tiny workload)."""
    audio = synth.synth_audio(105600, 0)
    tiny.enable_float16_kv_cache(kv_fp16)
    out = tiny.generate(audio, forced_len=64, return_logits=True)
    o = oracle_for(tiny_dir)
    ids, _, logits, margins = o.greedy(o.memory_for(audio), 64, kv_fp16, forced_len=64, keep_logits=True)
    assert out.tokens == ids
    assert_logits_close(out.logits[:64], logits, FP32_LOGIT_TOL)


@pytest.mark.parametrize("kv_fp16", [False, True])
def test_teacher_forced_logits(tiny, tiny_dir, kv_fp16):
    """Random fed-back ids exercise many embedding rows and positions."""
    audio = synth.synth_audio(48000, 11)
    teacher = np.random.Generator(np.random.PCG64(5)).integers(0, 32768, size=40).astype(np.int32)
    tiny.enable_float16_kv_cache(kv_fp16)
    out = tiny.generate(audio, forced_len=40, teacher_ids=teacher, return_logits=True)
    o = oracle_for(tiny_dir)
    ids, _, logits, _ = o.greedy(o.memory_for(audio), 40, kv_fp16, teacher=teacher.tolist(), keep_logits=True)
    assert out.tokens == ids
    assert_logits_close(out.logits[:40], logits, FP32_LOGIT_TOL)


def test_default_token_limit_and_max_tokens(tiny, tiny_dir):
    """limit = min(maxTokens, ceil(dur * 6.5)) (MoonshineModel.swift:200-201)."""
    audio = synth.synth_audio(105600, 0)
    tiny.enable_float16_kv_cache(True)
    out = tiny.generate(audio)
    assert len(out.tokens) == int(np.ceil(6.6 * 6.5))
    assert out.tokens == oracle_for(tiny_dir).generate(audio, kv_fp16=True)
    out5 = tiny.generate(audio, max_tokens=5)
    assert out5.tokens == out.tokens[:5]


def test_eos_stops_like_the_reference(tiny_dir, model_root, tmp_path):
    """A model whose eos id is a token the greedy loop produces stops there and drops it."""
    import moonshine_b200 as mb
    audio = synth.synth_audio(64000, 21)
    o = oracle_for(tiny_dir)
    ids, _, _, _ = o.greedy(o.memory_for(audio), 30, True, forced_len=30)
    # stop on the first id that differs from the first one, else on the very first id
    k = next((i for i, t in enumerate(ids) if t != ids[0]), 0)
    eos_dir = with_config(tiny_dir, str(tmp_path / "eos"), eos_token_id=int(ids[k]))
    m = mb.MoonshineModel.load(eos_dir)
    out = m.generate(audio, max_tokens=30)
    ref = oracle_for(eos_dir).generate(audio, max_tokens=30, kv_fp16=True)
    assert out.tokens == ref == ids[:k]
    assert out.hit_eos


def test_multi_chunk_generate(tiny, tiny_dir):
    """Audio longer than chunkDuration is decoded chunk by chunk (MoonshineModel.swift:151-162)."""
    audio = synth.synth_audio(16000 * 12 + 4321, 13)
    tiny.enable_float16_kv_cache(True)
    out = tiny.generate(audio, chunk_duration=5.0, forced_len=12)
    ref = oracle_for(tiny_dir).generate(audio, kv_fp16=True, chunk_duration=5.0, forced_len=12)
    assert out.tokens == ref
    assert len(ref) == 3 * 12


@pytest.mark.parametrize("n", [0, 1, 79, 80, 81, 159, 161, 400])
def test_tiny_inputs(tiny, tiny_dir, n):
    """Empty audio, sub-frame audio and a handful of frames (tail samples dropped)."""
    audio = synth.synth_audio(n, 17) if n else np.zeros(0, np.float32)
    tiny.enable_float16_kv_cache(True)
    out = tiny.generate(audio)
    assert out.tokens == oracle_for(tiny_dir).generate(audio, kv_fp16=True)


def test_invalid_arguments(tiny):
    import moonshine_b200 as mb
    with pytest.raises(mb.MoonshineError) as ei:
        tiny.generate(np.zeros(1600, np.float32), temperature=-0.5)
    assert ei.value.status == 1
    with pytest.raises(mb.MoonshineError):
        mb.MoonshineModel.load("/nonexistent/model/dir")


def test_small_arch_head_dim_64(model_root):
    """hd 64 -> rotary width 50 (int(64*0.8)=51 rounded down), 10+10 layers."""
    import moonshine_b200 as mb
    d = model_dir(model_root, "small", vocab_size=2048, max_position_embeddings=512)
    m = mb.MoonshineModel.load(d)
    audio = synth.synth_audio(32000, 4)
    teacher = np.random.Generator(np.random.PCG64(6)).integers(0, 2048, size=16).astype(np.int32)
    o = oracle_for(d)
    mem = o.memory_for(audio)
    assert rel_err(m.encode(audio), mem) < 1e-4
    for kv in (False, True):
        m.enable_float16_kv_cache(kv)
        out = m.generate(audio, forced_len=16, teacher_ids=teacher, return_logits=True)
        ids, _, logits, _ = o.greedy(mem, 16, kv, teacher=teacher.tolist(), keep_logits=True)
        assert out.tokens == ids
        assert_logits_close(out.logits[:16], logits, FP32_LOGIT_TOL)


@pytest.mark.parametrize("kernel", ["grid", "cluster", "auto"])
def test_every_decode_kernel_30s(tiny_dir, kernel):
    """30 s of audio (1500 memory frames), fp16 KV, 48 forced tokens through each batch-1
    decode kernel: single-grid and one 8-CTA cluster per head ("auto" picks the latter on a
    B200)."""
    import moonshine_b200 as mb
    m = mb.MoonshineModel.load(tiny_dir, decode_kernel=kernel)
    audio = synth.synth_audio(480000, 1)
    out = m.generate(audio, forced_len=48, return_logits=True)
    assert out.decode_kernel == ("cluster" if kernel == "auto" else kernel)
    o = oracle_for(tiny_dir)
    ids, _, logits, _ = o.greedy(o.memory_for(audio), 48, True, forced_len=48, keep_logits=True)
    assert out.tokens == ids
    assert_logits_close(out.logits[:48], logits, FP32_LOGIT_TOL)


def test_generate_long_memory_cap(tiny, tiny_dir):
    """generateLong (MoonshineStreaming.swift:287-376) with a 100-frame memory cap: 6.6 s of
    audio (330 frames) decodes as 4 segments over slices of one full encode."""
    import moonshine_b200 as mb
    audio = synth.synth_audio(105600, 0)
    tiny.enable_float16_kv_cache(True)
    segs, out = tiny.generate_long(audio, mb.StreamingConfig(max_memory_frames=100, min_segment_frames=20))
    ref = oracle_for(tiny_dir).generate_long(audio, max_memory_frames=100, min_segment_frames=20)
    assert segs == ref
    assert len(ref) == 4 and out.generation_tokens == 4


def test_generate_long_eos_advance(model_root, tmp_path):
    """An EOS inside a segment longer than min_segment_frames moves the next segment's start
    by max(min_segment_frames, tokens / 6.5 * 50) frames instead of the full segment.  The
    weight seed 5 model's greedy ids vary within a segment; its eos id is set to one of
    them (16128, the sixth id of the first segment) so segments end early."""
    import moonshine_b200 as mb
    d = model_dir(model_root, "tiny", seed=5)
    audio = synth.synth_audio(105600, 0)
    eos_dir = with_config(d, str(tmp_path / "eos_long"), eos_token_id=16128)
    m = mb.MoonshineModel.load(eos_dir)
    sc = mb.StreamingConfig(max_memory_frames=120, min_segment_frames=10)
    segs, _ = m.generate_long(audio, sc)
    ref = oracle_for(eos_dir).generate_long(audio, max_memory_frames=120, min_segment_frames=10)
    assert segs == ref
    assert len(ref) >= 6  # 330 frames in 120-frame caps would give 3 segments


def _first_token_probs(d, audio, T):
    o = oracle_for(d)
    _, _, logits, _ = o.greedy(o.memory_for(audio), 1, True, forced_len=1, keep_logits=True)
    z = np.asarray(logits[0], np.float64) / T
    p = np.exp(z - z.max())
    return p / p.sum()


def _chi2(counts, p):
    n = counts.sum()
    keep = p * n >= 5
    return float(np.sum((counts[keep] - n * p[keep]) ** 2 / (n * p[keep])))


@pytest.mark.parametrize("kernel", ["grid", "cluster"])
def test_temperature_sampling_distribution(model_root, kernel):
    """temperature > 0 draws each token from softmax(logits / T) (MLXRandom.categorical,
    MoonshineModel.swift:211-213).  The random streams cannot match MLX's, so the test is
    distributional: 4000 seeds on a 16-token vocabulary against the oracle's softmax of the
    first decoder call (chi-square well above its 0.1 % point would fail), plus a fixed
    seed giving the same draws twice."""
    import moonshine_b200 as mb
    d = model_dir(model_root, "tiny", vocab_size=16)
    m = mb.MoonshineModel.load(d, decode_kernel=kernel)
    audio = synth.synth_audio(32000, 9)
    T = 0.7
    p = _first_token_probs(d, audio, T)
    counts = np.zeros(16)
    for seed in range(4000):
        out = m.generate(audio, forced_len=1, temperature=T, seed=seed)
        counts[out.tokens[0]] += 1
    chi2 = _chi2(counts, p)
    assert chi2 < 45.0, (chi2, counts, 4000 * p)
    a = m.generate(audio, max_tokens=20, temperature=T, seed=123)
    b = m.generate(audio, max_tokens=20, temperature=T, seed=123)
    assert a.tokens == b.tokens


def test_temperature_sampling_batch(model_root):
    """The batched engine samples per row: the first tokens of 16 x 256 rows of one utterance
    follow the same softmax (bf16 logits, well inside the chi-square margin)."""
    import moonshine_b200 as mb
    d = model_dir(model_root, "tiny", vocab_size=16)
    m = mb.MoonshineModel.load(d)
    audio = synth.synth_audio(32000, 9)
    T = 0.7
    p = _first_token_probs(d, audio, T)
    counts = np.zeros(16)
    for seed in range(16):
        ids, _ = m.generate_batch([audio] * 256, forced_len=1, temperature=T, seed=seed)
        for r in ids:
            counts[r[0]] += 1
    chi2 = _chi2(counts, p)
    assert chi2 < 45.0, (chi2, counts, counts.sum() * p)


@pytest.mark.parametrize("group,bits,streamed", [(64, 8, 8), (64, 4, 4), (64, 2, 2), (32, 4, 4), (32, 2, 0),
                                                 (128, 4, 0)])
def test_quantized_checkpoint(model_root, group, bits, streamed):
    """MLX affine-quantized checkpoints (ModelLoader.swift:47-49,103-111; config.json
    "quantization"): every Linear whose input width divides by the group size is stored as
    packed codes + scales + biases.  The clustered batch-1 kernel streams the q|k|v, cross q,
    fc1 and LM-head rows (quant_stream "all"; by default only the LM head) as those codes and
    multiplies them in the kernel (`streamed` bits;
    0 where the rows are not quantized at d = 320 with groups of 128, or where a 16-byte
    chunk of 2-bit codes would straddle two groups of 32); the single-grid kernel and
    weight_dtype "f32" use the rows dequantized at load.  Ids and logits of all four match
    the oracle on the same checkpoint at the fp32 tolerance, and the quantized stream's
    logits match the dequantized stream's within 1e-4 relative (both fp32; the kernel factors
    each group's scale out of its sum, a different rounding order that 32 dependent calls
    compound to ~1e-5)."""
    import moonshine_b200 as mb
    d = model_dir(model_root, "tiny", quant=(group, bits))
    audio = synth.synth_audio(105600, 0)
    o = oracle_for(d)
    ids, _, logits, _ = o.greedy(o.memory_for(audio), 32, True, forced_len=32, keep_logits=True)
    outs = {}
    expect = {"all": (streamed, streamed), "auto": (0, streamed), "grid": (0, 0), "f32": (0, 0)}
    for name, kw in (("all", {"quant_stream": "all"}), ("auto", {}), ("grid", {"decode_kernel": "grid"}),
                     ("f32", {"weight_dtype": "f32"})):
        m = mb.MoonshineModel.load(d, **kw)
        assert m.decode_weight_bits == expect[name], name
        out = m.generate(audio, forced_len=32, return_logits=True)
        assert out.tokens == ids, name
        assert_logits_close(out.logits[:32], logits, FP32_LOGIT_TOL)
        outs[name] = out.logits[:32]
        m.close()
    assert rel_err(outs["all"], outs["f32"]) < 1e-4
    assert rel_err(outs["auto"], outs["f32"]) < 1e-4


@functools.lru_cache(maxsize=1)
def _headline_reference(tiny_dir):
    o = oracle_for(tiny_dir)
    ids, _, logits, margins = o.greedy(o.memory_for(synth.synth_audio(480000, 1)), 200, True, forced_len=200,
                                       keep_logits=True)
    return ids, logits, margins


@pytest.mark.parametrize("kernel", ["auto", "grid"])
def test_headline_workload_200_tokens(tiny_dir, kernel):
    """The benchmarked workload itself: tiny weights (seed 0), 30 s of audio (seed 1), fp16
    KV cache, 200 forced decoder calls, through the default kernel ("auto": the head-clustered
    one on a B200) and the single-grid one.  Ids identical to the float64 oracle's, logits
    within 1e-3 per call; the smallest top-2 margin is printed."""
    import moonshine_b200 as mb
    m = mb.MoonshineModel.load(tiny_dir, decode_kernel=kernel, kv_fp16=True)
    out = m.generate(synth.synth_audio(480000, 1), forced_len=200, return_logits=True)
    assert out.decode_kernel == ("cluster" if kernel == "auto" else kernel)
    ids, logits, margins = _headline_reference(tiny_dir)
    assert out.tokens == ids
    worst = assert_logits_close(out.logits[:200], logits, FP32_LOGIT_TOL)
    rel = [mg / float(np.max(np.abs(lg))) for mg, lg in zip(margins, logits)]
    print(f"headline workload ({out.decode_kernel}): worst logits error {worst:.2e}, smallest relative "
          f"top-2 margin {min(rel):.3e} at call {int(np.argmin(rel))}")


def test_medium_arch_batch1(model_root):
    """Medium architecture (d 640, 10 heads of 64 -> 10 head clusters, 14 + 14 layers), fp32,
    fp16 KV, on the head-clustered kernel (the single-grid kernel's per-warp staging does not
    fit shared memory at d 640): teacher-forced logits and free-running ids."""
    import moonshine_b200 as mb
    d = model_dir(model_root, "medium", max_position_embeddings=1024)
    m = mb.MoonshineModel.load(d, kv_fp16=True)
    audio = synth.synth_audio(48000, 8)
    o = oracle_for(d)
    mem = o.memory_for(audio)
    assert rel_err(m.encode(audio), mem) < 1e-4
    teacher = np.random.Generator(np.random.PCG64(9)).integers(0, 32768, size=12).astype(np.int32)
    out = m.generate(audio, forced_len=12, teacher_ids=teacher, return_logits=True)
    assert out.decode_kernel == "cluster"
    ids, _, logits, _ = o.greedy(mem, 12, True, teacher=teacher.tolist(), keep_logits=True)
    assert out.tokens == ids
    assert_logits_close(out.logits[:12], logits, FP32_LOGIT_TOL)
    free = m.generate(audio, forced_len=12)
    assert free.tokens == o.greedy(mem, 12, True, forced_len=12)[0]
