"""The incremental streaming encoder's row bookkeeping (BatchEngine::encode_windows_inc in
moonshine-mlx_b200/csrc/runtime/batch.cpp) restated over the float64 oracle's encoder layers,
against encodeNewFrames' window re-encode (MoonshineStreaming.swift:178-214, the oracle's
OracleStream._encode_new_frames).

Per call and layer l the restatement recomputes rows from c = max(0, prev - S_l), where prev
is the feature count at the stream's previous call and S_l the right contexts of layers
0..l summed, over a segment that starts `left` rows earlier (the attention context of row
c), keeps every layer's output rows, and commits the new stable rows through the final norm
and positions.  The committed memory rows must equal the window's to float64 rounding, for
the tiny model's windows and for windows with right context in every layer, with chunks of
several sizes, calls that commit nothing and a final call."""
import numpy as np
import pytest

from util import model_dir, oracle_for, with_config


def _window_memory(o, feats, emitted, stable, pos):
    """encodeNewFrames: the encoder over [emitted - 16 L, total), new rows [emitted, stable)."""
    L = o.cfg.encoder.num_hidden_layers
    ws = max(0, emitted - 16 * L)
    enc = o.encode(feats[ws:])
    return o.prepare_memory(enc[emitted - ws:stable - ws], pos)


class _Incremental:
    def __init__(self, o):
        from oracle.moonshine_oracle import _layer_norm
        self.o, self.ln = o, _layer_norm
        ec = o.cfg.encoder
        self.L = ec.num_hidden_layers
        self.left = [max(0, w[0]) for w in ec.sliding_windows]
        self.S = np.cumsum([max(0, w[1]) for w in ec.sliding_windows])
        self.out = [np.zeros((0, ec.hidden_size)) for _ in range(self.L - 1)]
        self.prev = 0

    def memory(self, feats, emitted, stable, pos):
        o, total = self.o, feats.shape[0]
        for l in range(self.L):
            c = max(0, min(self.prev, total) - int(self.S[l]))
            s = max(0, c - self.left[l])
            src = feats if l == 0 else self.out[l - 1]
            y = o._encoder_layer(src[s:total], l)
            if l < self.L - 1:
                keep = self.out[l][:c]
                self.out[l] = np.concatenate([keep, y[c - s:]])
            else:
                last, last_s = y, s
        self.prev = total
        enc = self.ln(last[emitted - last_s:stable - last_s], o.w["encoder.final_norm.weight"] + 1.0)
        return o.prepare_memory(enc, pos)


@pytest.mark.parametrize("windows", [None, [[16, 4]] * 6, [[8, 2], [12, 3], [16, 0], [5, 4], [16, 1], [16, 4]]])
def test_incremental_encoder_rows_match_window(model_root, tmp_path, windows):
    base = model_dir(model_root, "tiny")
    d = base if windows is None else with_config(base, str(tmp_path / "w"), **{"encoder_config.sliding_windows": windows})
    o = oracle_for(d)
    ec = o.cfg.encoder
    look = max([w[1] for w in ec.sliding_windows], default=0)
    rng = np.random.default_rng(7)
    feats_all = rng.standard_normal((260, ec.hidden_size))
    inc = _Incremental(o)
    total = emitted = pos = 0
    steps = [4] * 30 + [1, 9, 2, 0, 17] + [4] * 20 + [6]
    checked = 0
    for k, n in enumerate(steps):
        final = k == len(steps) - 1
        total += n
        feats = feats_all[:total]
        stable = total if final else max(0, total - look)
        new = stable - emitted
        if new <= 0:
            continue
        want = _window_memory(o, feats, emitted, stable, pos)
        got = inc.memory(feats, emitted, stable, pos)
        assert got.shape == want.shape
        assert np.allclose(got, want, rtol=1e-10, atol=1e-10), (k, float(np.abs(got - want).max()))
        emitted, pos = stable, pos + new
        checked += 1
    assert checked > 40 and emitted > 16 * ec.num_hidden_layers  # past the window's left edge
