"""ms_decode_memory_static: the decode entry point for callers that cannot allocate device
memory while running -- a real-time audio callback, where cudaMalloc can block and
synchronise the device past the callback's deadline, or a host held to a fixed GPU memory
budget.

The calls are checked against the float64 oracle fed the same float32 memory rows
(identical ids), twice in a row on a freshly loaded model: the static scratch array keeps
the previous call's contents, so the second call checks that what must start at zero is
reset.  Free device memory is read before and after the calls and must be unchanged (model
load sets the array up and loads the kernels; the calls reserve nothing).  A non-forced call
stops at a configured EOS id like the reference's greedy loop."""
import numpy as np
import pytest

from moonshine_b200 import synth
from util import model_dir, oracle_for, with_config

pytestmark = pytest.mark.gpu

N_TOKENS = 48


def _memories(path, cases):
    """Oracle memory rows (rounded to float32, as uploaded) and the oracle's ids on them."""
    o = oracle_for(path)
    out = []
    for seed, seconds, forced in cases:
        mem = o.memory_for(synth.synth_audio(int(seconds * 16000), seed)).astype(np.float32)
        ids, hit, _, _ = o.greedy(mem.astype(np.float64), N_TOKENS, True,
                                  forced_len=N_TOKENS if forced else None)
        out.append((mem, ids, hit, forced))
    return out


def _run(path, cases):
    import torch
    import moonshine_b200 as mb
    model = mb.MoonshineModel.load(path, kv_fp16=True)
    bufs = [(torch.from_numpy(mem).to("cuda:0"), torch.full((N_TOKENS,), -7, dtype=torch.int32, device="cuda:0"))
            for mem, _, _, _ in cases]
    # inputs fully written before the calls (the call's stream does not wait for torch's)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(0)
    got = []
    for (mem_dev, ids_dev), (mem, _, _, forced) in zip(bufs, cases):
        n, hit = model.decode_memory_static(mem_dev.data_ptr(), mem.shape[0], ids_dev.data_ptr(), N_TOKENS,
                                            forced=forced)
        got.append((n, hit))
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(0)
    assert free1 == free0, f"free device memory changed across the calls: {free0} -> {free1}"
    for (n, hit), (_, ids_dev), (_, ref, ref_hit, forced) in zip(got, bufs, cases):
        assert n == len(ref) and hit == ref_hit
        assert ids_dev.cpu().tolist()[:n] == ref
    model.close()


def test_static_decode_matches_oracle_twice_without_allocating(model_root):
    path = model_dir(model_root, "tiny")
    _run(path, _memories(path, [(51, 6.6, True), (52, 4.0, True)]))


def test_static_decode_stops_at_eos(model_root, tmp_path):
    """eos_token_id set to the fifth greedy id of the forced run: the non-forced call
    stops there, returns the four ids before it and reports the EOS; a forced call on the
    same model follows."""
    base = model_dir(model_root, "tiny")
    first = _memories(base, [(53, 5.0, True)])[0]
    eos_dir = with_config(base, str(tmp_path / "eos_static"), eos_token_id=int(first[1][4]))
    cases = _memories(eos_dir, [(53, 5.0, False), (54, 3.0, True)])
    assert cases[0][2] and len(cases[0][1]) == first[1].index(first[1][4])
    _run(eos_dir, cases)


def test_static_decode_rejects_oversize(model_root):
    import torch
    import moonshine_b200 as mb
    path = model_dir(model_root, "tiny")
    model = mb.MoonshineModel.load(path)
    mem_dev = torch.zeros((1500, 320), dtype=torch.float32, device="cuda:0")
    ids_dev = torch.zeros((256,), dtype=torch.int32, device="cuda:0")
    with pytest.raises(mb.MoonshineError) as ei:
        model.decode_memory_static(mem_dev.data_ptr(), 1500, ids_dev.data_ptr(), 256)
    assert ei.value.status == mb.MS_ERR_CAPACITY
    assert "limit" in str(ei.value)
