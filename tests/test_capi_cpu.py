"""Host-side checks of the C ABI that need no GPU: the library loads, exports every
symbol include/moonshine_b200.h declares, and reports argument errors with a status."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "moonshine_b200.h")


def declared_functions():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(ms_[a-z0-9_]+)\s*\(", txt)))


def test_header_declares_the_api():
    names = declared_functions()
    for n in ("ms_model_load", "ms_generate", "ms_stream_create", "ms_stream_transcribe",
              "ms_stream_add_audio", "ms_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    import moonshine_b200 as mb
    lib = ctypes.CDLL(mb.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_defaults_and_argument_errors():
    import moonshine_b200 as mb
    L = mb._L()
    o = mb._Options()
    L.ms_options_default(ctypes.byref(o))
    assert (o.device, o.kv_dtype, o.max_batch) == (0, mb.KV_F16, 64)
    p = mb._GenParams()
    L.ms_gen_params_default(ctypes.byref(p))
    assert p.chunk_duration == 30.0 and p.temperature == 0.0
    sc = mb._StreamingConfig()
    L.ms_streaming_config_default(ctypes.byref(sc))
    assert (sc.max_memory_frames, sc.min_segment_frames) == (100000, 250)
    h = ctypes.c_void_p()
    assert L.ms_model_load(None, None, ctypes.byref(h)) == 1
    assert b"non-null" in L.ms_last_error()
    n = ctypes.c_int32()
    assert L.ms_generate(None, None, 0, None, None, 0, ctypes.byref(n), None, None) == 1
    assert L.ms_stream_start(None) == 1
    assert L.ms_model_sample_rate(None) == 0
    assert b"sm_100a" in L.ms_version()
    assert (o.weight_dtype, o.decode_kernel, o.quant_stream) == (0, 0, 0)  # AUTO everywhere
    lm = ctypes.c_int32(-1)
    assert L.ms_model_decode_weight_bits(None, ctypes.byref(lm)) == 0 and lm.value == 0
    assert L.ms_model_decode_weight_bits(None, None) == 0


def test_python_load_rejects_unknown_options(tmp_path):
    import moonshine_b200 as mb
    for kw in ({"decode_kernel": "solo"}, {"weight_dtype": "f16"}, {"quant_stream": "some"}):
        with pytest.raises(ValueError):
            mb.MoonshineModel.load(str(tmp_path), **kw)


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="a GPU is present")
def test_load_without_gpu_reports_cuda_error(tmp_path):
    import moonshine_b200 as mb
    with pytest.raises(mb.MoonshineError) as ei:
        mb.MoonshineModel.load(str(tmp_path))
    assert ei.value.status in (3, 7)


def declared_param_counts():
    """Number of parameters of every prototype in the header (void -> 0)."""
    txt = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for name, params in re.findall(r"\b(ms_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", txt):
        p = " ".join(params.split())
        out[name] = 0 if p in ("", "void") else p.count(",") + 1
    return out


def test_python_bindings_match_the_header_prototypes():
    """Every function the Python mirror binds takes as many arguments as its C prototype."""
    import moonshine_b200 as mb
    L = mb._L()
    counts = declared_param_counts()
    bound = 0
    for name, n in counts.items():
        fn = getattr(L, name, None)
        if fn is None or fn.argtypes is None:
            continue
        assert len(fn.argtypes) == n, (name, len(fn.argtypes), n)
        bound += 1
    assert bound >= 30


def test_stream_batch_and_memory_argument_errors():
    import moonshine_b200 as mb
    L = mb._L()
    rows = ctypes.c_int32(-1)
    assert L.ms_stream_memory(None, None, 0, ctypes.byref(rows)) == 1
    assert L.ms_stream_add_audio_batch(None, 1, None, None) == 1
    assert L.ms_stream_add_audio_batch(None, 0, None, None) == 1  # null stream array
    n = ctypes.c_int32()
    assert L.ms_stream_transcribe_batch(None, 1, 0, None, 0, None, 0, ctypes.byref(n), None, None) == 1


def test_struct_layouts_match_the_library():
    """The ctypes mirrors of the header's structs have the library's sizes (checked at load)."""
    import moonshine_b200 as mb
    L = mb._L()
    for cname, cls in (("ms_options", mb._Options), ("ms_model_config", mb._ModelConfig),
                       ("ms_gen_params", mb._GenParams), ("ms_gen_stats", mb._GenStats),
                       ("ms_alignment", mb._Alignment), ("ms_streaming_config", mb._StreamingConfig)):
        assert L.ms_struct_size(cname.encode()) == ctypes.sizeof(cls) > 0, cname
    assert L.ms_struct_size(b"ms_nothing") == 0
