"""ms_decode_memory_static: the decode entry point for callers that cannot allocate device
memory while running (real-time audio callbacks, fixed GPU memory budgets).  It must give
the same token ids as the regular entry point, on two calls in a row (the static scratch
array keeps the previous call's contents, so the second call checks that it is reset)."""
import numpy as np
import pytest

from moonshine_b200 import synth
from util import model_dir

pytestmark = pytest.mark.gpu


def test_static_decode_matches_generate_twice(model_root):
    import torch
    import moonshine_b200 as mb
    path = model_dir(model_root, "tiny")
    model = mb.MoonshineModel.load(path, kv_fp16=True)
    n_tokens = 48
    for seed, seconds in ((51, 6.6), (52, 4.0)):
        audio = synth.synth_audio(int(seconds * 16000), seed)
        ref = model.generate(audio, forced_len=n_tokens).tokens
        memory = model.encode(audio)
        mem_dev = torch.from_numpy(np.ascontiguousarray(memory)).to("cuda:0")
        ids_dev = torch.full((n_tokens,), -7, dtype=torch.int32, device="cuda:0")
        torch.cuda.synchronize()
        n, hit = model.decode_memory_static(mem_dev.data_ptr(), memory.shape[0], ids_dev.data_ptr(), n_tokens)
        assert n == n_tokens and not hit
        assert ids_dev.cpu().tolist() == ref


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
