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


@pytest.mark.parametrize("kv_fp16", [True, False])
def test_stream_memory_growth_keeps_cross_kv(model_root, kv_fp16):
    """7 s fed in 0.5 s chunks: the stream's memory passes its first capacity (256 frames)
    and its cross K/V rows move to the larger layout; every call still matches the oracle."""
    d = model_dir(model_root, "tiny")
    audio = synth.synth_audio(16000 * 7, 35)
    calls, em, ref_em = _run_both(d, audio, 8000, 16, {}, kv_fp16=kv_fp16, final=False)
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
        # the batched streams take their chunks in one add_audio_batch call (uneven sizes:
        # the remainder buffers differ per stream), the single ones one call each
        sizes = [1280 - 80 * i + (off // 1280) % 2 * 37 for i in range(3)]
        m.add_audio_batch(streams, [audios[i][off:off + sizes[i]] for i in range(3)])
        for i in range(3):
            m.add_audio(singles[i], audios[i][off:off + sizes[i]])
        got = m.transcribe_batch(streams, max_tokens=16)
        want = [m.transcribe(s, max_tokens=16) for s in singles]
        assert got == want


def test_stream_batch_ragged_and_repeated(model_root):
    """add_audio_batch with chunks shorter than a frame (they only fill the remainder buffer),
    an empty chunk, and a stream listed twice (its chunks are taken in order) matches the same
    chunks fed one add_audio call at a time."""
    import moonshine_b200 as mb
    d = model_dir(model_root, "tiny")
    m = mb.MoonshineModel.load(d)
    streams = [m.create_stream() for _ in range(3)]
    singles = [m.create_stream() for _ in range(3)]
    for s in streams + singles:
        m.start_stream(s)
    audios = [synth.synth_audio(8000, 50 + i) for i in range(3)]
    pos = [0, 0, 0]

    def take(i, n):
        piece = audios[i][pos[i]:pos[i] + n]
        pos[i] += n
        return piece

    plans = [[(0, 50), (1, 1111), (2, 0)], [(0, 2000), (1, 30), (2, 1500)],
             [(2, 700), (0, 900), (2, 333), (1, 2100)], [(0, 1200), (1, 1200), (2, 1200)]]
    for plan in plans:
        pieces = [(i, take(i, n)) for i, n in plan]
        m.add_audio_batch([streams[i] for i, _ in pieces], [p for _, p in pieces])
        for i, p in pieces:
            m.add_audio(singles[i], p)
        got = m.transcribe_batch(streams, max_tokens=16)
        want = [m.transcribe(s, max_tokens=16) for s in singles]
        assert got == want
        assert [s.memory_len for s in streams] == [s.memory_len for s in singles]


@pytest.mark.parametrize("windows", [None, [[8, 2], [12, 3], [16, 0], [5, 4], [16, 1], [16, 4]]])
def test_stream_incremental_encoder_matches_window(model_root, tmp_path, windows):
    """transcribe_batch's incremental encoder (batch_decode 1: each layer recomputes only the
    rows that can have changed since the stream's previous call, plus their left attention
    context) against re-encoding each stream's whole window as the reference's
    encodeNewFrames does (batch_decode 2, MoonshineStreaming.swift:178-214): the same memory
    rows after every call, to fp32 rounding (the two passes differ only in how their GEMMs
    split K), through the left-context limit of 16 frames per layer, ragged chunks, a call
    with no new stable frames and the final call."""
    import moonshine_b200 as mb
    d = model_dir(model_root, "tiny")
    if windows is not None:  # right context in most layers, left windows of several sizes
        d = with_config(d, str(tmp_path / "w"), **{"encoder_config.sliding_windows": windows})
    m = mb.MoonshineModel.load(d)
    n_streams = 3
    inc = [m.create_stream() for _ in range(n_streams)]
    win = [m.create_stream() for _ in range(n_streams)]
    for s in inc + win:
        m.start_stream(s)
    sizes = [1280] * 30 + [320, 2000, 1280, 90, 4000] + [1280] * 12
    audios = [synth.synth_audio(sum(sizes), 60 + i) for i in range(n_streams)]
    sc_inc, sc_win = mb.StreamingConfig(batch_decode=1), mb.StreamingConfig(batch_decode=2)
    off, longest = 0, 0
    for k, n in enumerate(sizes):
        final = k == len(sizes) - 1
        pieces = [a[off:off + n] for a in audios]
        off += n
        m.add_audio_batch(inc, pieces)
        m.add_audio_batch(win, pieces)
        m.transcribe_batch(inc, is_final=final, streaming_config=sc_inc, max_tokens=8)
        m.transcribe_batch(win, is_final=final, streaming_config=sc_win, max_tokens=8)
        for a, b in zip(inc, win):
            ma, mb_ = a.memory(), b.memory()
            assert ma.shape == mb_.shape, (k, ma.shape, mb_.shape)
            if ma.size:
                assert float(np.abs(ma - mb_).max()) <= 1e-4 * max(1.0, float(np.abs(mb_).max())), k
            longest = max(longest, ma.shape[0])
    assert longest > 16 * 6  # past the window's left context (the final call resets the segment)


def test_stream_batch_decode_lockstep(model_root):
    """transcribe_batch with batch_decode: 4 streams fed 80 ms chunks, every call's segment
    decoded in lockstep on the tensor cores (split bf16 operands for this fp32 checkpoint).
    Per call and stream the ids follow the oracle's decodeMemory
    (MoonshineStreaming.swift:229-276); they may part only at a step whose top-2 logit
    margin is within the fp32 tolerance; the memories stay equal throughout."""
    import moonshine_b200 as mb
    from oracle.moonshine_oracle import OracleStream, StreamingConfig
    from util import FP32_LOGIT_TOL
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
                assert margins[j] <= FP32_LOGIT_TOL * scale, f"stream {i} chunk {k}: ids part at step {j}"
            checked += 1
    assert checked >= n_streams * (n_chunks - 2)


def _stream_first_token_probs(o, audio, T, chunk=1280):
    """Softmax(logits / T) of the first decoder call on the oracle stream's memory after
    feeding `audio` in chunks (the memory a non-final transcribe decodes against)."""
    from oracle.moonshine_oracle import OracleStream
    os_ = OracleStream(o, kv_fp16=True)
    os_.start()
    for off in range(0, len(audio), chunk):
        os_.add_audio(audio[off:off + chunk])
    os_._encode_new_frames(False)
    cache = o.new_cache(os_.memory, True)
    _, lg = o.decoder_step(o.cfg.decoder_start_token_id, cache)
    z = np.asarray(lg, np.float64) / T
    p = np.exp(z - z.max())
    return p / p.sum(), os_.memory_len


def _chi2(counts, p):
    n = counts.sum()
    keep = p * n >= 5
    return float(np.sum((counts[keep] - n * p[keep]) ** 2 / (n * p[keep])))


def test_stream_temperature_sampling(model_root):
    """transcribe(temperature:) (MoonshineStreaming.swift:122-128, decodeMemory :238-268):
    each non-final call decodes from BOS against the same memory, so 3000 one-token calls
    draw from softmax(logits / T) of its first decoder call; a repeated (seed, call) sequence
    repeats its draws.  The lockstep batch samples per stream row."""
    import moonshine_b200 as mb
    d = model_dir(model_root, "tiny", vocab_size=16)
    o = oracle_for(d)
    audio = synth.synth_audio(16000, 41)
    T = 0.7
    p, mem_len = _stream_first_token_probs(o, audio, T)
    eos = o.cfg.eos_token_id
    m = mb.MoonshineModel.load(d)

    def fed_stream():
        st = m.create_stream()
        m.start_stream(st)
        for off in range(0, len(audio), 1280):
            m.add_audio(st, audio[off:off + 1280])
        return st

    st = fed_stream()
    counts = np.zeros(16)
    for _ in range(3000):
        ids, hit, emitted = m.transcribe(st, max_tokens=1, temperature=T, seed=7)
        assert not emitted
        if ids:
            counts[ids[0]] += 1
        elif hit and eos < 16:
            counts[eos] += 1
    assert st.memory_len == mem_len
    assert counts.sum() > 2900
    chi2 = _chi2(counts, p)
    assert chi2 < 45.0, (chi2, counts, counts.sum() * p)

    a, b = fed_stream(), fed_stream()
    seq_a = [m.transcribe(a, max_tokens=8, temperature=T, seed=11)[0] for _ in range(5)]
    seq_b = [m.transcribe(b, max_tokens=8, temperature=T, seed=11)[0] for _ in range(5)]
    assert seq_a == seq_b and len({tuple(x) for x in seq_a}) > 1

    streams = [fed_stream() for _ in range(64)]
    counts = np.zeros(16)
    sc = mb.StreamingConfig(batch_decode=True)
    for _ in range(32):
        for ids, hit, _ in m.transcribe_batch(streams, streaming_config=sc, max_tokens=1, temperature=T, seed=3):
            if ids:
                counts[ids[0]] += 1
            elif hit and eos < 16:
                counts[eos] += 1
    chi2 = _chi2(counts, p)
    assert chi2 < 45.0, (chi2, counts, counts.sum() * p)

    with pytest.raises(mb.MoonshineError):
        m.transcribe(st, temperature=-1.0)
