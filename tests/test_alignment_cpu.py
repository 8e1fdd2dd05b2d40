"""Word-timestamp host logic without a GPU: the oracle's restatement of findAlignment's
pieces (MoonshineTimestamps.swift:20-242) on hand-checked cases, and the library's DTW and
word-timing arithmetic (ms_alignment_jump_frames, ms_word_timings) against the oracle on
seeded random cases.  The reference ships no tests or fixtures for this path, so the hand
cases below are worked out from its source."""
import numpy as np
import pytest

from oracle.moonshine_oracle import (dtw_jump_frames, dtw_path, median_filter_1d, word_timings,
                                     zscore_rows)


def test_dtw_hand_cases():
    # a cheap diagonal: the path follows it
    c = np.full((3, 3), 5.0, np.float32)
    np.fill_diagonal(c, -1.0)
    assert dtw_path(c) == ([0, 1, 2], [0, 1, 2])
    # one text row over four frames: horizontal steps only
    assert dtw_path(np.zeros((1, 4), np.float32)) == ([0, 0, 0, 0], [0, 1, 2, 3])
    # four text rows over one frame: vertical steps only
    assert dtw_path(np.zeros((4, 1), np.float32)) == ([0, 1, 2, 3], [0, 0, 0, 0])
    # all-equal costs: ties go to the diagonal first, so a 2x4 grid ends on the diagonal
    # into (1, 3) after horizontal moves in row 0
    assert dtw_path(np.zeros((2, 4), np.float32)) == ([0, 0, 0, 1], [0, 1, 2, 3])
    # jump frames: first frame of each text row along the path
    c = np.array([[0, 0, 9, 9], [9, 9, 0, 9], [9, 9, 9, 0]], np.float32)
    assert dtw_jump_frames(c).tolist() == [0, 2, 3]
    assert dtw_path(np.zeros((0, 3), np.float32)) == ([], [])


def test_median_filter_hand_cases():
    x = np.array([5, 1, 4, 2, 3, 9, 0, 7], np.float32)
    # width 7, clipped windows; index count/2 of the sorted window
    assert median_filter_1d(x, 7).tolist() == [4, 3, 4, 3, 3, 4, 3, 7]
    assert median_filter_1d(x, 3).tolist() == [5, 4, 2, 3, 3, 3, 7, 7]
    assert median_filter_1d(x, 1).tolist() == x.tolist()


def test_zscore_population_std():
    r = np.array([[1.0, 2.0, 3.0, 4.0]])
    z = zscore_rows(r)
    sd = np.sqrt(1.25) + 1e-6
    np.testing.assert_allclose(z[0], (r[0] - 2.5) / sd)


def test_word_timings_hand_case():
    # jumps 0,3,5,8,12 frames; words start at tokens 0, 2, 3 of 4
    w = word_timings([0, 3, 5, 8, 12], [0.9, 0.8, 0.7, 0.6, 0.5], [0, 2, 3], 4, 20, 0.0)
    assert w == [(0.0, 0.1, 0.85), (0.1, 0.16, 0.7), (0.16, 0.24, 0.6)]
    # the last word ends at the last jump when no later row exists; an offset shifts all
    w = word_timings([0, 10], [0.5, 0.5], [0, 1], 2, 50, 1.5)
    assert w == [(1.5, 1.7, 0.5), (1.7, 1.7, 0.5)]
    # a word ends where the next one starts (both read the next word's jump frame), so the
    # reference's overlap fix (:224-239) never moves a boundary, even on a non-monotone path
    w = word_timings([10, 4, 20], [1.0, 1.0, 1.0], [0, 1], 2, 30, 0.0)
    assert w == [(0.2, 0.08, 1.0), (0.08, 0.4, 1.0)]
    assert word_timings([], [], [], 0, 10) == []


def _lib():
    import moonshine_b200 as mb
    return mb


@pytest.mark.parametrize("shape,seed", [((1, 1), 0), ((1, 7), 1), ((7, 1), 2), ((5, 9), 3),
                                        ((17, 40), 4), ((40, 17), 5), ((23, 300), 6)])
def test_library_dtw_matches_oracle(shape, seed):
    mb = _lib()
    rng = np.random.Generator(np.random.PCG64(seed))
    rows = rng.standard_normal(shape).astype(np.float32)
    assert mb.alignment_jump_frames(rows).tolist() == dtw_jump_frames(-rows).tolist()
    # small integers make ties everywhere: the tie order decides the path
    ints = rng.integers(-2, 3, size=shape).astype(np.float32)
    assert mb.alignment_jump_frames(ints).tolist() == dtw_jump_frames(-ints).tolist()


def test_library_dtw_empty():
    mb = _lib()
    assert mb.alignment_jump_frames(np.zeros((0, 5), np.float32)).tolist() == []
    assert mb.alignment_jump_frames(np.zeros((3, 0), np.float32)).tolist() == []


@pytest.mark.parametrize("seed", range(6))
def test_library_word_timings_match_oracle(seed):
    import ctypes as C
    mb = _lib()
    rng = np.random.Generator(np.random.PCG64(100 + seed))
    n_tok = int(rng.integers(1, 30))
    n_steps = n_tok + int(rng.integers(0, 2))         # EOS call adds a row
    n_frames = int(rng.integers(5, 400))
    jumps = np.sort(rng.integers(0, n_frames, size=n_steps)).astype(np.int32)
    if seed % 2:
        rng.shuffle(jumps)                             # a non-monotone path
    probs = rng.random(n_steps).astype(np.float32)
    starts = sorted(set([0] + rng.integers(0, n_tok, size=max(1, n_tok // 3)).tolist()))
    offset = float(rng.choice([0.0, 0.25, 12.34]))
    ref = word_timings(jumps.tolist(), probs.tolist(), starts, n_tok, n_frames, offset)
    nw = len(starts)
    wf = np.asarray(starts, np.int32)
    st, en, pb = (np.zeros(nw) for _ in range(3))
    n = C.c_int32()
    dp = C.POINTER(C.c_double)
    mb._check(mb._L().ms_word_timings(mb._iptr(jumps), n_steps, mb._fptr(probs), n_steps, mb._iptr(wf), nw,
                                      n_tok, n_frames, offset, st.ctypes.data_as(dp), en.ctypes.data_as(dp),
                                      pb.ctypes.data_as(dp), C.byref(n)))
    assert n.value == len(ref)
    assert [(float(a), float(b), float(c)) for a, b, c in zip(st, en, pb)] == ref


def test_word_grouping_by_piece_marker():
    """findAlignment :154-173: a word starts at every piece that begins with U+2581."""
    mb = _lib()
    al = mb.Alignment(ids=[5, 6, 7, 8, 9], token_probs=np.full(6, 0.5, np.float32),
                      jump_frames=np.array([0, 2, 4, 6, 8, 10], np.int32), n_frames=50, hit_eos=True)
    pieces = {5: "▁a", 6: "b", 7: "▁c", 8: "▁d", 9: "e"}
    words = mb.word_timings(al, pieces.get, lambda ids: " " + "".join(pieces[i].lstrip("▁") for i in ids))
    assert [w.word for w in words] == ["ab", "c", "de"]
    assert [w.tokens for w in words] == [[5, 6], [7], [8, 9]]
    assert [(w.start, w.end) for w in words] == [(0.0, 0.08), (0.08, 0.12), (0.12, 0.2)]
    # without a tokenizer every piece is "" -> one word (the reference's nil tokenizer)
    words = mb.word_timings(al)
    assert len(words) == 1 and words[0].tokens == [5, 6, 7, 8, 9]


def test_word_timings_rejects_bad_boundaries():
    import ctypes as C
    mb = _lib()
    wf = np.array([0, 0], np.int32)
    out = np.zeros(2)
    n = C.c_int32()
    dp = C.POINTER(C.c_double)
    s = mb._L().ms_word_timings(None, 0, None, 0, mb._iptr(wf), 2, 3, 10, 0.0, out.ctypes.data_as(dp),
                                out.ctypes.data_as(dp), out.ctypes.data_as(dp), C.byref(n))
    assert s == 1
