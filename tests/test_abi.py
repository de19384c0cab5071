"""C-ABI surface of librpgc.so, checked without a GPU (no compute calls)."""
import os
import re
import tempfile

import numpy as np
import pytest

import rpgbarengine_b200 as rb
from rpgbarengine_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions(path):
    src = open(path).read()
    return sorted(set(re.findall(r"RPGC_API\s+[\w\s\*]+?\b(rpgc_\w+)\s*\(", src)))


def test_library_exports_every_header_symbol():
    names = header_functions(os.path.join(ROOT, "include", "rpgc.h"))
    assert len(names) >= 20
    lib = rb.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_only_abi_symbols_are_exported():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", rb.LIB_PATH], capture_output=True,
                         text=True).stdout
    funcs = [l.split()[-1] for l in out.splitlines() if " T " in l]
    extra = [f for f in funcs if not f.startswith("rpgc_")]
    assert not extra, extra[:10]


def test_version_and_errors_without_gpu():
    assert rb.version()
    if rb.device_count() > 0:
        pytest.skip("a GPU is present; the no-device paths are not reachable")
    with pytest.raises(rb.RpgcError) as e:
        rb.Model.load_gguf("/nonexistent/model.gguf")
    assert e.value.code == rb.E_IO
    # invalid handles are state errors, destroy/free of unknown handles are no-ops
    assert rb.lib().rpgc_session_len(12345) == rb.E_STATE
    assert rb.lib().rpgc_session_destroy(12345) == rb.OK
    assert rb.lib().rpgc_model_free(12345) == rb.OK


def test_gguf_parse_reaches_device_check():
    if rb.device_count() > 0:
        pytest.skip("a GPU is present")
    d = tempfile.mkdtemp()
    p = os.path.join(d, "tiny.gguf")
    synth.write_model(p, synth.TINY_MIX, 1)
    with pytest.raises(rb.RpgcError) as e:
        rb.Model.load_gguf(p)
    # the file parsed and the tensor table validated; only the device is missing
    assert "device" in str(e.value).lower()


def test_gguf_reader_matches_the_reference_on_odd_files():
    # src/gguf.cc:84-93, 105-106, 124, 139-141: version 1 changes only the two
    # counts; a duplicate tensor name and a missing architecture are rejected
    if rb.device_count() > 0:
        pytest.skip("a GPU is present")
    d = tempfile.mkdtemp()
    shape = synth.TINY_MIX
    tens = synth.build_tensors(shape, 1)
    meta = synth.metadata(shape)
    p1 = os.path.join(d, "v1.gguf")
    rb.gguf.write(p1, meta, tens, version=1)
    assert len(rb.gguf.read(p1).tensors) == len(tens)
    with pytest.raises(rb.RpgcError) as e:
        rb.Model.load_gguf(p1)
    assert "device" in str(e.value).lower()  # parsed; only the device is missing
    p2 = os.path.join(d, "dup.gguf")
    rb.gguf.write(p2, meta, tens + [tens[-1]])
    with pytest.raises(rb.RpgcError) as e:
        rb.Model.load_gguf(p2)
    assert e.value.code == rb.E_IO and "duplicate" in str(e.value)
    p3 = os.path.join(d, "noarch.gguf")
    rb.gguf.write(p3, {k: v for k, v in meta.items() if k != "general.architecture"}, tens)
    with pytest.raises(rb.RpgcError) as e:
        rb.Model.load_gguf(p3)
    assert e.value.code == rb.E_IO and "architecture" in str(e.value)


def test_gguf_python_roundtrip():
    d = tempfile.mkdtemp()
    p = os.path.join(d, "t.gguf")
    tens = synth.write_model(p, synth.TINY_Q8, 3)
    f = rb.gguf.read(p)
    assert f.meta["general.architecture"] == "qwen3"
    assert f.meta["qwen3.block_count"] == synth.TINY_Q8.n_layers
    assert len(f.meta["tokenizer.ggml.tokens"]) == synth.TINY_Q8.vocab
    for a in tens:
        b = f.tensor(a.name)
        assert b.ggml_type == a.ggml_type and tuple(b.dims) == tuple(a.dims)
        assert np.array_equal(np.asarray(b.data), a.data)


def test_batching_entry_points_check_arguments_without_gpu():
    # argument and handle checks run before any device work
    import ctypes as C
    L = rb.lib()
    assert L.rpgc_model_set_batching(12345, 257, 0) == rb.E_ARG  # above 256 sessions
    assert b"max_batch" in L.rpgc_last_error()
    assert L.rpgc_model_set_batching(12345, 4, -1) == rb.E_ARG
    assert L.rpgc_model_set_batching(12345, 4, 1000001) == rb.E_ARG
    assert L.rpgc_model_set_batching(12345, 4, 100) == rb.E_STATE  # no such model
    assert b"model handle" in L.rpgc_last_error()
    b, r = C.c_int64(-1), C.c_int64(-1)
    assert L.rpgc_model_batching_stats(12345, C.byref(b), C.byref(r)) == rb.E_STATE
    assert L.rpgc_model_batching_stats(12345, None, None) == rb.E_ARG
    o = rb.GenOpts(4, None, 0, 0.0, 0, 1.0, 0)
    out = np.zeros(8, np.int32)
    n_out = np.zeros(2, np.int32)
    sessions = np.array([12345, 12346], np.int32)
    assert L.rpgc_generate_batch(None, 2, C.byref(o), out.ctypes.data, n_out.ctypes.data) == rb.E_ARG
    assert L.rpgc_generate_batch(sessions.ctypes.data, 0, C.byref(o), out.ctypes.data,
                                 n_out.ctypes.data) == rb.E_ARG  # empty batch
    assert L.rpgc_generate_batch(sessions.ctypes.data, 257, C.byref(o), out.ctypes.data,
                                 n_out.ctypes.data) == rb.E_ARG
    assert L.rpgc_generate_batch(sessions.ctypes.data, 2, C.byref(o), out.ctypes.data,
                                 n_out.ctypes.data) == rb.E_STATE  # unknown sessions
