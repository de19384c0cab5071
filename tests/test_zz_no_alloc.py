"""rpgc_matmul_noalloc: the prefill matmul for callers that cannot let this
library allocate device memory (a host whose GPU heap belongs to another
runtime, or a path where an allocation may block or fail).  It runs the same
tensor-core kernels as rpgc_matmul with their scratch in a fixed device array
of the library, so its results must agree with rpgc_matmul's, call after call
(the array keeps the previous call's contents), and sizes beyond the array
must be refused.  This file is collected last on purpose: a run that stops at
its first failure has run every other test before it.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import rpgbarengine_b200 as rb  # noqa: E402
from rpgbarengine_b200 import gguf, synth  # noqa: E402
from tests.gpu_util import ROW_GATE  # noqa: E402


def _noalloc():
    fn = rb.lib().rpgc_matmul_noalloc
    vp, i64 = C.c_void_p, C.c_int64
    fn.argtypes = [C.c_uint32, vp, i64, i64, vp, i64, vp, vp]
    fn.restype = C.c_int
    return fn


def _row_gate_vs(got, want, W, X):
    """max over (t, r) of |got - want| / sum_k |x_k w_k|: the per-row matmul
    gate, taken against the allocating entry point's result."""
    den = np.abs(X.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
    return float((np.abs(got.astype(np.float64) - want.astype(np.float64)) / np.maximum(den, 1e-30)).max())


def test_noalloc_matmul_matches_rpgc_matmul_on_consecutive_calls():
    if rb.device_count() == 0:
        pytest.fail("GPU test collected without a CUDA device")
    fn = _noalloc()
    rng = np.random.default_rng(7)
    stream = torch.cuda.current_stream().cuda_stream
    # second call: a different type and shape, split-K (its partial sums in
    # the array), over what the first call left there
    for ty, rows, cols, n in [(gguf.Q4_K, 9728, 2560, 64), (gguf.Q6_K, 2560, 9728, 200),
                              (gguf.Q8_0, 1024, 4096, 1)]:
        w = torch.from_numpy(synth.random_blocks(rng, ty, rows, cols)).cuda()
        X = torch.from_numpy(rng.standard_normal((n, cols)).astype(np.float32)).cuda()
        want = rb.matmul_batch(ty, w, rows, cols, X)
        got = torch.full((n, rows), float("nan"), device="cuda")
        rc = fn(ty, w.data_ptr(), rows, cols, X.data_ptr(), n, got.data_ptr(), stream)
        assert rc == rb.OK, rb.lib().rpgc_last_error()
        torch.cuda.synchronize()
        W = rb.dequantize_rows(ty, w, rows, cols).cpu().numpy()
        g, wt = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all()
        assert _row_gate_vs(g, wt, W, X.cpu().numpy()) <= ROW_GATE, (ty, rows, cols, n)


def test_noalloc_matmul_refuses_sizes_beyond_its_array():
    if rb.device_count() == 0:
        pytest.fail("GPU test collected without a CUDA device")
    fn = _noalloc()
    rows, cols, n = 256, 9728, 2048  # ~152 MB of scratch, above the 32 MiB array
    w = torch.from_numpy(synth.random_blocks(np.random.default_rng(1), gguf.Q8_0, rows, cols)).cuda()
    X = torch.zeros((n, cols), device="cuda")
    out = torch.zeros((n, rows), device="cuda")
    rc = fn(gguf.Q8_0, w.data_ptr(), rows, cols, X.data_ptr(), n, out.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    assert rc == rb.E_ARG
    assert b"scratch" in rb.lib().rpgc_last_error()
