"""Word timestamps on the GPU (generateWithWordTimestamps, MoonshineModel.swift:241-316)
against the oracle's restatement of the same loop and findAlignment.

Ids must be identical.  The attention rows (mean over layers and heads of the cross-attention
softmax) must agree within 1e-5 max-norm relative, and within 1e-3 after z-scoring (the
random-init models attend almost uniformly: a row's spread is ~0.5% of its mean, which the
z-score blows up to the unit scale the DTW sees); token probabilities within 1e-3
relative.  The DTW is checked exactly: the library's jump frames equal the oracle's DTW
over the library's own filtered rows; against the oracle's own rows they may move where two
DTW costs are within float noise, so that comparison is by mean frame distance."""
import numpy as np
import pytest

from moonshine_b200 import synth
from util import model_dir, oracle_for, rel_err, with_config

pytestmark = pytest.mark.gpu

ROW_TOL = 1e-5
Z_TOL = 1e-3
PROB_RTOL = 1e-3


@pytest.fixture(scope="module")
def varied_dir(model_root):
    """Weight seed 5: its greedy ids vary from call to call."""
    return model_dir(model_root, "tiny", seed=5)


def _check_against_oracle(al, ref, width=7):
    from oracle.moonshine_oracle import dtw_jump_frames, median_filter_rows, zscore_rows
    assert al.ids == ref["ids"]
    assert al.n_frames == ref["n_frames"]
    assert al.attn_rows.shape == ref["attn_rows"].shape
    assert rel_err(al.attn_rows, ref["attn_rows"]) < ROW_TOL
    assert rel_err(zscore_rows(al.attn_rows), zscore_rows(ref["attn_rows"])) < Z_TOL
    assert al.token_probs.shape == ref["token_probs"].shape
    np.testing.assert_allclose(al.token_probs, ref["token_probs"], rtol=PROB_RTOL, atol=0)
    # z-score + median filter of the library's own rows, restated on the CPU
    filt = median_filter_rows(zscore_rows(al.attn_rows.astype(np.float64)), width)
    assert rel_err(al.attn_filtered, filt) < Z_TOL
    # DTW over the same rows: bit-exact path
    assert al.jump_frames.tolist() == dtw_jump_frames(-al.attn_filtered).tolist()
    assert al.jump_frames.shape[0] == al.attn_rows.shape[0]
    # against the oracle's own rows
    dist = np.abs(al.jump_frames.astype(np.int64) - ref["jump_frames"])
    assert dist.mean() <= 2.0, dist


@pytest.mark.parametrize("kernel,kv_fp16", [("grid", True), ("cluster", True), ("cluster", False), ("grid", False)])
def test_alignment_matches_oracle(varied_dir, kernel, kv_fp16):
    """6.6 s of audio: 330 memory frames, ceil(6.6 * 6.5) = 43 decoder calls, through every
    batch-1 decode kernel (each stores the cross queries) and both K/V cache dtypes."""
    import moonshine_b200 as mb
    m = mb.MoonshineModel.load(varied_dir, decode_kernel=kernel)
    m.enable_float16_kv_cache(kv_fp16)
    audio = synth.synth_audio(105600, 0)
    al = m.generate_alignment(audio, return_attention=True)
    ref = oracle_for(varied_dir).generate_with_alignment(audio, kv_fp16=kv_fp16)
    assert len(al.ids) == 43 and not al.hit_eos
    _check_against_oracle(al, ref)


def test_alignment_eos_row_and_word_timings(varied_dir, tmp_path):
    """An EOS call adds an attention row and a probability but no id (the reference appends
    the EOS call's scores before breaking, MoonshineModel.swift:273-287); words then follow
    the ids with a stand-in tokenizer whose even ids start words."""
    import moonshine_b200 as mb
    from oracle.moonshine_oracle import word_timings
    eos_dir = with_config(varied_dir, str(tmp_path / "eos"), eos_token_id=16128)
    m = mb.MoonshineModel.load(eos_dir)
    audio = synth.synth_audio(105600, 0)
    al = m.generate_alignment(audio, return_attention=True)
    ref = oracle_for(eos_dir).generate_with_alignment(audio, kv_fp16=True)
    assert al.hit_eos and ref["hit_eos"]
    assert len(al.token_probs) == len(al.ids) + 1 == len(al.jump_frames)
    _check_against_oracle(al, ref)

    piece = lambda t: ("▁w" if t % 2 == 0 else "x")
    out, words = m.generate_with_word_timestamps(audio, time_offset=2.5, token_to_string=piece)
    assert out.tokens == al.ids and out.segments[0].words == words
    first = [i for i, t in enumerate(al.ids) if i == 0 or piece(t).startswith("▁")]
    exp = word_timings(al.jump_frames.tolist(), al.token_probs.tolist(), first, len(al.ids), al.n_frames, 2.5)
    assert [(w.start, w.end, w.probability) for w in words] == exp
    assert sum(len(w.tokens) for w in words) == len(al.ids)
    assert out.segments[0].end == pytest.approx(6.6)


def test_alignment_max_tokens_and_empty(varied_dir):
    import moonshine_b200 as mb
    m = mb.MoonshineModel.load(varied_dir)
    audio = synth.synth_audio(105600, 0)
    full = m.generate_alignment(audio)
    cut = m.generate_alignment(audio, max_tokens=5, return_attention=True)
    assert cut.ids == full.ids[:5] and len(cut.token_probs) == 5 and not cut.hit_eos
    np.testing.assert_allclose(cut.token_probs, full.token_probs[:5], atol=1e-6)
    empty = m.generate_alignment(np.zeros(0, np.float32))
    assert empty.ids == [] and empty.jump_frames.shape[0] == 0 and empty.n_frames == 0
    out, words = m.generate_with_word_timestamps(np.zeros(0, np.float32))
    assert words == [] and out.tokens == []
    with pytest.raises(mb.MoonshineError):
        m.generate_alignment(audio, medfilt_width=65)


def test_alignment_30s(varied_dir):
    """30 s (1500 frames, 195 decoder calls): the largest single-chunk case; the row kernel
    then groups calls in shared memory against 1500-frame rows."""
    import moonshine_b200 as mb
    m = mb.MoonshineModel.load(varied_dir)
    audio = synth.synth_audio(480000, 3)
    al = m.generate_alignment(audio, return_attention=True)
    ref = oracle_for(varied_dir).generate_with_alignment(audio, kv_fp16=True)
    assert al.attn_rows.shape == (195, 1500)
    _check_against_oracle(al, ref)
