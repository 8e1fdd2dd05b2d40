"""Batched lockstep decode (bf16 tcgen05 GEMMs) vs the CPU oracle, per utterance.

GEMM inputs are bf16, so logits are compared with the bf16 tolerance (2e-2, max-abs
relative per decoder call); token ids must match the oracle's greedy ids."""
import numpy as np
import pytest

from moonshine_b200 import synth
from util import BF16_LOGIT_TOL, FP32_LOGIT_TOL, assert_logits_close, model_dir, oracle_for, with_config

pytestmark = pytest.mark.gpu


def _check_batch(path, audios, forced, kv_fp16=True, max_tokens=None, model=None, tol=BF16_LOGIT_TOL):
    import moonshine_b200 as mb
    m = model or mb.MoonshineModel.load(path, kv_fp16=kv_fp16)
    ids, st, logits = m.generate_batch(audios, forced_len=forced, max_tokens=max_tokens, return_logits=True)
    o = oracle_for(path)
    for b, a in enumerate(audios):
        mem = o.memory_for(a)
        if forced:
            ref, _, ref_logits, margins = o.greedy(mem, forced, kv_fp16, forced_len=forced, keep_logits=True)
        else:
            limit = o.token_limit(len(a), max_tokens)
            ref, _, ref_logits, margins = o.greedy(mem, limit, kv_fp16, keep_logits=True)
        # Greedy ids may only part at a near-tie: a step whose top-2 logit margin is within
        # the bf16 tolerance.  Logits are compared up to and including that step (its
        # inputs are still identical on both sides).
        k = next((i for i, (x, y) in enumerate(zip(ids[b], ref)) if x != y), None)
        if k is None:
            assert len(ids[b]) == len(ref), f"utterance {b}"
            k = len(ref_logits) - 1
        else:
            scale = float(np.max(np.abs(ref_logits[k])))
            assert margins[k] <= tol * scale, (
                f"utterance {b}: ids part at step {k} with margin {margins[k]:.4f} (scale {scale:.3f})")
        assert_logits_close(logits[b, : k + 1], ref_logits[: k + 1], tol)
    return st


@pytest.mark.parametrize("kv_fp16", [True, False])
def test_batch_tiny_forced(model_root, kv_fp16):
    d = model_dir(model_root, "tiny")
    audios = [synth.synth_audio(n, 60 + i) for i, n in enumerate([16000, 40000, 23456, 32000])]
    _check_batch(d, audios, 12, kv_fp16=kv_fp16)


def test_batch_small_bf16_checkpoint(model_root):
    d = model_dir(model_root, "small", dtype="bfloat16", vocab_size=2048, max_position_embeddings=512)
    audios = [synth.synth_audio(n, 70 + i) for i, n in enumerate([24000, 17777, 32000])]
    _check_batch(d, audios, 8)


def test_batch_limits_and_eos(model_root, tmp_path):
    base = model_dir(model_root, "tiny")
    o = oracle_for(base)
    audios = [synth.synth_audio(n, 80 + i) for i, n in enumerate([8000, 12000, 20000])]
    first = o.greedy(o.memory_for(audios[1]), 3, True, forced_len=3)[0]
    eos_dir = with_config(base, str(tmp_path / "eos"), eos_token_id=int(first[1]))
    _check_batch(eos_dir, audios, None)            # per-utterance limits, EOS stops
    _check_batch(base, audios, None, max_tokens=4)


def test_batch_of_one_equals_generate(model_root):
    import moonshine_b200 as mb
    d = model_dir(model_root, "tiny")
    m = mb.MoonshineModel.load(d)
    a = synth.synth_audio(48000, 90)
    ids, _ = m.generate_batch([a], forced_len=20)
    assert ids[0] == m.generate(a, forced_len=20).tokens


def _config3_audio():
    """The small-model batched workload: 64 utterances of U(5, 15) s (lengths from PCG64(7),
    whole frames), audio seeds 100 + i."""
    rng = np.random.Generator(np.random.PCG64(7))
    lens = (rng.uniform(5, 15, size=64) * 16000).astype(int) // 80 * 80
    seeds = [100 + i for i in range(64)]
    return lens, seeds, [synth.synth_audio(int(n), s) for n, s in zip(lens, seeds)]


def test_batch_config3_shape_against_oracle(model_root, tmp_path):
    """Small architecture, bf16 checkpoint, vocabulary 32768, 64 utterances of U(5, 15) s,
    128 forced tokens each -- the batched workload at its full shape.  Every utterance is
    checked against the oracle (a pool of oracle processes): ids identical except where they
    part at a near-tie, logits within the bf16 tolerance up to there.  A second run of the
    same batch gives bit-identical ids (the split-K sums run in a fixed order)."""
    import moonshine_b200 as mb
    from oracle_pool import check_batch
    d = model_dir(model_root, "small", dtype="bfloat16")
    lens, seeds, audios = _config3_audio()
    m = mb.MoonshineModel.load(d)
    ids, st, logits = m.generate_batch(audios, forced_len=128, return_logits=True)
    assert all(len(r) == 128 for r in ids)
    ids2, _ = m.generate_batch(audios, forced_len=128)
    assert ids2 == ids
    res = check_batch(d, lens, seeds, 128, True, ids, logits[:, :128], tmp_path)
    errs = [e for _, e, _, _, _ in res if e]
    parted = [(r, k) for r, _, _, k, _ in res if k >= 0]
    worst = max(w for _, _, w, _, _ in res)
    print(f"config-3 shape: worst logits error {worst:.3e}, rows parting at a near-tie {parted}, "
          f"smallest relative top-2 margin {min(mm for *_, mm in res):.2e}")
    assert not errs, errs


def test_batch_runs_are_bit_identical(model_root):
    """The same batch twice: identical ids and bit-identical logits."""
    import moonshine_b200 as mb
    d = model_dir(model_root, "small", dtype="bfloat16", vocab_size=2048, max_position_embeddings=512)
    audios = [synth.synth_audio(16000 + 4000 * (i % 5), 300 + i) for i in range(24)]
    m = mb.MoonshineModel.load(d)
    a_ids, _, a_lg = m.generate_batch(audios, forced_len=24, return_logits=True)
    b_ids, _, b_lg = m.generate_batch(audios, forced_len=24, return_logits=True)
    assert a_ids == b_ids
    assert np.array_equal(a_lg, b_lg)


def test_batch_medium_arch(model_root):
    """Medium architecture (d 640, 10 heads of 64, 14 + 14 layers), bf16 checkpoint, three
    utterances, 8 forced tokens, against the oracle."""
    d = model_dir(model_root, "medium", dtype="bfloat16", max_position_embeddings=1024)
    audios = [synth.synth_audio(n, 400 + i) for i, n in enumerate([32000, 45678, 20000])]
    _check_batch(d, audios, 8)


def test_batch_kv_pages_ragged(model_root):
    """Paged self-attention K/V: rows with limits 4, 26, 9 and 17 (ceil(6.5 s)) get 1, 2, 1
    and 2 pages of 16 positions -- 6 pages in one pool instead of 4 rows x 2 -- and still
    match the oracle; a smaller call afterwards takes fewer pages from the same pool, and
    the lockstep streaming decode draws its pages from it too."""
    import moonshine_b200 as mb
    d = model_dir(model_root, "tiny")
    m = mb.MoonshineModel.load(d)
    lens = [8000, 64000, 20000, 40000]
    audios = [synth.synth_audio(n, 500 + i) for i, n in enumerate(lens)]
    _check_batch(d, audios, None, model=m)
    used, cap, page = m.batch_kv_pages()
    assert page == 16
    assert used == sum(-(-int(np.ceil(n / 16000 * 6.5)) // page) for n in lens) == 6
    assert cap >= used
    _check_batch(d, audios[:1], None, model=m)
    used2, cap2, _ = m.batch_kv_pages()
    assert used2 == 1 and cap2 == cap
    # lockstep streaming decode of three streams: pages per call, returned after it
    states = [m.create_stream() for _ in range(3)]
    for st in states:
        m.start_stream(st)
    sc = mb.StreamingConfig(batch_decode=True)
    for k in range(6):
        for i, st in enumerate(states):
            m.add_audio(st, synth.synth_audio(1280 * (i + 1), 600 + 10 * k + i))
        m.transcribe_batch(states, streaming_config=sc, max_tokens=16)
        u, c, _ = m.batch_kv_pages()
        assert 1 <= u <= 3 and c == cap
    for st in states:
        st.close()


@pytest.mark.parametrize("kv_fp16", [True, False])
def test_batch_fp32_checkpoint_split_operands(model_root, kv_fp16):
    """An fp32 checkpoint decodes in lockstep with split bf16 operands (high + low planes,
    three tensor-core products per step): logits within the fp32 tolerance (1e-3) of the
    float64 oracle and ids identical to it, like the batch-1 kernels."""
    d = model_dir(model_root, "tiny")
    audios = [synth.synth_audio(n, 700 + i) for i, n in enumerate([16000, 48000, 30000, 80000])]
    _check_batch(d, audios, 24, kv_fp16=kv_fp16, tol=FP32_LOGIT_TOL)
