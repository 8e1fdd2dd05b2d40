"""The pooled per-utterance checker used by the large batched GPU tests, run on CPU against
outputs the oracle itself produced: exact copies pass, a planted logits error and a planted
id change at a wide margin fail."""
import numpy as np

from moonshine_b200 import synth
from oracle_pool import check_batch
from util import model_dir, oracle_for


def test_pool_checker_accepts_oracle_outputs_and_flags_planted_errors(model_root, tmp_path):
    path = model_dir(model_root, "tiny", vocab_size=512, max_position_embeddings=256)
    o = oracle_for(path, np.float32)
    lens, seeds, forced = [8000, 12000], [3, 4], 4
    ids, logits = [], []
    for n, s in zip(lens, seeds):
        r, _, lg, _ = o.greedy(o.memory_for(synth.synth_audio(n, s)), forced, True, forced_len=forced,
                               keep_logits=True)
        ids.append(r)
        logits.append(np.stack(lg).astype(np.float32))
    logits = np.stack(logits)
    res = check_batch(path, lens, seeds, forced, True, ids, logits, tmp_path)
    assert all(err is None for _, err, _, _, _ in res), res
    bad = logits.copy()
    bad[1, 2, 7] += 0.5 * float(np.max(np.abs(bad[1, 2])))
    res = check_batch(path, lens, seeds, forced, True, ids, bad, tmp_path)
    assert res[0][1] is None and res[1][1] is not None and "logits" in res[1][1]
    wrong = [list(ids[0]), list(ids[1])]
    wrong[0][1] = (wrong[0][1] + 1) % 512
    res = check_batch(path, lens, seeds, forced, True, wrong, logits, tmp_path)
    assert res[0][1] is not None and res[0][3] == 1
