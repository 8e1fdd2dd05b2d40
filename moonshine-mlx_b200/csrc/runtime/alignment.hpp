// Host side of word-timestamp alignment (findAlignment, MoonshineTimestamps.swift:94-242):
// the DTW path over the filtered attention rows and the word timing arithmetic.
#pragma once

#include <cstdint>
#include <vector>

namespace msb {

// dtw (MoonshineTimestamps.swift:20-65) on cost = -rows ([N][M], row-major), followed by
// the jump extraction of findAlignment (:175-184): the frame at which the path enters each
// text row.  Returns N frames (empty when N or M is 0).
std::vector<int32_t> dtw_jump_frames(const float* rows, int N, int M);

struct WordTime {
    double start, end, probability;
};

// Word timings (:186-239) for words given by their first token index (word_first, ascending,
// word w spans [word_first[w], word_first[w+1]) and the last word ends at n_tokens).
std::vector<WordTime> word_times(const int32_t* jump_frames, int n_jumps, const float* probs, int n_probs,
                                 const int32_t* word_first, int n_words, int n_tokens, int n_frames,
                                 double time_offset);

}  // namespace msb
