"""Streaming state machine (MoonshineStreaming.swift) on the CUDA path vs the oracle."""
import numpy as np
import pytest

from moonshine_b200 import synth
from util import model_dir, oracle_for, with_config

pytestmark = pytest.mark.gpu


def _run_both(path, audio, chunk, max_tokens, sc_kwargs, kv_fp16=True, final=True):
    import moonshine_b200 as mb
    from oracle.moonshine_oracle import OracleStream, StreamingConfig
    m = mb.MoonshineModel.load(path, kv_fp16=kv_fp16)
    st = m.create_stream()
    m.start_stream(st)
    os_ = OracleStream(oracle_for(path), kv_fp16=kv_fp16)
    os_.start()
    sc = mb.StreamingConfig(**sc_kwargs)
    osc = StreamingConfig(**sc_kwargs)
    calls = []
    for off in range(0, len(audio), chunk):
        c = audio[off:off + chunk]
        m.add_audio(st, c)
        os_.add_audio(c)
        last = off + chunk >= len(audio)
        fin = final and last
        g = m.transcribe(st, is_final=fin, streaming_config=sc, max_tokens=max_tokens)
        r = os_.transcribe(is_final=fin, config=osc, max_tokens=max_tokens)
        calls.append((g, r))
        assert st.memory_len == os_.memory_len
    return calls, m.get_emitted(st), os_.emitted_segments


def test_stream_80ms_chunks_matches_oracle(model_root):
    d = model_dir(model_root, "tiny")
    audio = synth.synth_audio(16000 * 2, 31)
    calls, em, ref_em = _run_both(d, audio, 1280, 16, {})
    for i, (g, r) in enumerate(calls):
        assert list(g) == [r[0], r[1], r[2]], f"call {i}"
    assert em == ref_em


def test_stream_odd_chunks_and_fp32_kv(model_root):
    d = model_dir(model_root, "tiny")
    audio = synth.synth_audio(16000 + 777, 32)
    calls, em, ref_em = _run_both(d, audio, 1000, 8, {}, kv_fp16=False)
    for g, r in calls:
        assert list(g) == [r[0], r[1], r[2]]
    assert em == ref_em


def test_stream_eos_segmentation(model_root, tmp_path):
    """EOS with enough memory emits the segment and resets (MoonshineStreaming.swift:144-150)."""
    base = model_dir(model_root, "tiny")
    o = oracle_for(base)
    audio = synth.synth_audio(16000 * 2, 33)
    first = o.greedy(o.memory_for(audio[:8000]), 4, True)[0]
    d = with_config(base, str(tmp_path / "eos"), eos_token_id=int(first[0]))
    calls, em, ref_em = _run_both(d, audio, 1280, 16, {"min_segment_frames": 8})
    for g, r in calls:
        assert list(g) == [r[0], r[1], r[2]]
    assert em == ref_em
    assert len(ref_em) >= 2


def test_stream_memory_cap(model_root):
    d = model_dir(model_root, "tiny")
    audio = synth.synth_audio(16000 * 2, 34)
    calls, em, ref_em = _run_both(d, audio, 2560, 4, {"max_memory_frames": 20}, final=False)
    for g, r in calls:
        assert list(g) == [r[0], r[1], r[2]]
    assert em == ref_em
    assert len(ref_em) >= 1


def test_stream_batch_equals_single(model_root):
    import moonshine_b200 as mb
    d = model_dir(model_root, "tiny")
    m = mb.MoonshineModel.load(d)
    streams = [m.create_stream() for _ in range(3)]
    singles = [m.create_stream() for _ in range(3)]
    for s in streams + singles:
        m.start_stream(s)
    audios = [synth.synth_audio(6400, 40 + i) for i in range(3)]
    for off in range(0, 6400, 1280):
        for i in range(3):
            m.add_audio(streams[i], audios[i][off:off + 1280])
            m.add_audio(singles[i], audios[i][off:off + 1280])
        got = m.transcribe_batch(streams, max_tokens=16)
        want = [m.transcribe(s, max_tokens=16) for s in singles]
        assert got == want


def test_stream_batch_decode_lockstep(model_root):
    """transcribe_batch with batch_decode: 4 streams fed 80 ms chunks, every call's segment
    decoded in lockstep on bf16 tensor cores.  Per call and stream the ids follow the
    oracle's decodeMemory (MoonshineStreaming.swift:229-276) up to the first step whose
    top-2 logit margin is within the bf16 tolerance; the memories stay equal throughout."""
    import moonshine_b200 as mb
    from oracle.moonshine_oracle import OracleStream, StreamingConfig
    from util import BF16_LOGIT_TOL
    d = model_dir(model_root, "tiny")
    m = mb.MoonshineModel.load(d)
    o = oracle_for(d)
    n_streams, chunk, n_chunks, max_tokens = 4, 1280, 10, 16
    audios = [synth.synth_audio(chunk * n_chunks, 70 + i) for i in range(n_streams)]
    streams = [m.create_stream() for _ in range(n_streams)]
    refs = [OracleStream(o, kv_fp16=True) for _ in range(n_streams)]
    for s, r in zip(streams, refs):
        m.start_stream(s)
        r.start()
    sc = mb.StreamingConfig(batch_decode=True)
    checked = 0
    for k in range(n_chunks):
        for i in range(n_streams):
            piece = audios[i][k * chunk:(k + 1) * chunk]
            m.add_audio(streams[i], piece)
            refs[i].add_audio(piece)
        got = m.transcribe_batch(streams, streaming_config=sc, max_tokens=max_tokens)
        for i in range(n_streams):
            r = refs[i]
            r._encode_new_frames(False)
            assert streams[i].memory_len == r.memory_len
            if r.memory_len == 0:
                assert got[i] == ([], False, False)
                continue
            limit = min(max_tokens, int(np.ceil(r.memory_len * 0.020 * o.cfg.max_tokens_per_second)))
            ref, hit, ref_logits, margins = o.greedy(r.memory, limit, True, keep_logits=True)
            ids = got[i][0]
            j = next((t for t, (x, y) in enumerate(zip(ids, ref)) if x != y), None)
            if j is None:
                assert ids == ref and got[i][1] == hit, f"stream {i} chunk {k}"
            else:
                scale = float(np.max(np.abs(ref_logits[j])))
                assert margins[j] <= BF16_LOGIT_TOL * scale, f"stream {i} chunk {k}: ids part at step {j}"
            checked += 1
    assert checked >= n_streams * (n_chunks - 2)
