// DTW path and word timing arithmetic of findAlignment (MoonshineTimestamps.swift:20-242).
// The DTW runs in float with the reference's step order (diagonal, then vertical, then
// horizontal on ties) so the path is the one the reference takes on the same rows; the cost
// matrix is kept as two rolling rows and the trace as one byte per cell.
#include "alignment.hpp"

#include <cmath>
#include <limits>

namespace msb {

std::vector<int32_t> dtw_jump_frames(const float* rows, int N, int M) {
    std::vector<int32_t> jumps;
    if (N <= 0 || M <= 0) return jumps;
    const float inf = std::numeric_limits<float>::infinity();
    std::vector<float> prev((size_t)M + 1, inf), cur((size_t)M + 1, inf);
    std::vector<uint8_t> trace((size_t)N * M);  // trace[(i-1)*M + (j-1)] for cell (i, j)
    prev[0] = 0.f;                               // cost[0][0]
    for (int i = 1; i <= N; ++i) {
        cur[0] = inf;
        const float* row = rows + (size_t)(i - 1) * M;
        uint8_t* tr = trace.data() + (size_t)(i - 1) * M;
        for (int j = 1; j <= M; ++j) {
            const float c0 = prev[j - 1], c1 = prev[j], c2 = cur[j - 1];
            float c;
            uint8_t t;
            if (c0 <= c1 && c0 <= c2) {
                c = c0;
                t = 0;
            } else if (c1 <= c2) {
                c = c1;
                t = 1;
            } else {
                c = c2;
                t = 2;
            }
            cur[j] = -row[j - 1] + c;
            tr[j - 1] = t;
        }
        std::swap(prev, cur);
    }
    // backtrace from (N, M); row 0 moves left, column 0 moves up (:51-61)
    std::vector<int32_t> text, time;
    int i = N, j = M;
    while (i > 0 || j > 0) {
        text.push_back(i - 1);
        time.push_back(j - 1);
        const int t = i == 0 ? 2 : j == 0 ? 1 : trace[(size_t)(i - 1) * M + (j - 1)];
        if (t == 0) {
            --i;
            --j;
        } else if (t == 1) {
            --i;
        } else {
            --j;
        }
    }
    // path in forward order; a jump is where the text index changes (:176-184)
    const int P = (int)text.size();
    for (int k = P - 1; k >= 0; --k)
        if (k == P - 1 || text[k] != text[k + 1]) jumps.push_back(time[k]);
    return jumps;
}

static double round_to(double x, double unit) { return std::round(x * unit) / unit; }

std::vector<WordTime> word_times(const int32_t* jump_frames, int n_jumps, const float* probs, int n_probs,
                                 const int32_t* word_first, int n_words, int n_tokens, int n_frames,
                                 double time_offset) {
    constexpr double frame_s = 0.02;  // 50 Hz memory frames (MoonshineTimestamps.swift:5)
    std::vector<WordTime> out;
    for (int w = 0; w < n_words; ++w) {
        const int first = word_first[w];
        const int last = (w + 1 < n_words ? word_first[w + 1] : n_tokens) - 1;
        if (last < first) continue;
        const int start_f = first < n_jumps ? jump_frames[first] : (n_jumps ? jump_frames[n_jumps - 1] : 0);
        const int end_f = last + 1 < n_jumps ? jump_frames[last + 1] : (n_jumps ? jump_frames[n_jumps - 1] : n_frames);
        float psum = 0.f;  // Float sum, then Double mean (:210-213)
        int pc = 0;
        for (int k = first; k <= last; ++k)
            if (k < n_probs) {
                psum += probs[k];
                ++pc;
            }
        const double avg = pc ? (double)psum / (double)pc : 1.0;
        WordTime wt;
        wt.start = round_to(time_offset + start_f * frame_s, 1000.0);
        wt.end = round_to(time_offset + end_f * frame_s, 1000.0);
        wt.probability = round_to(avg, 10000.0);
        out.push_back(wt);
    }
    // overlapping neighbours meet at the rounded midpoint (:224-239)
    for (size_t k = 1; k < out.size(); ++k)
        if (out[k - 1].end > out[k].start) {
            const double mid = round_to((out[k - 1].end + out[k].start) / 2.0, 1000.0);
            out[k - 1].end = mid;
            out[k].start = mid;
        }
    return out;
}

}  // namespace msb
