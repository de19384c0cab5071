"""The allocation-free decode attention entry point.

Callers that cannot allocate device memory (a host whose GPU heap belongs to
another runtime, or a latency-critical path that must stay out of the
allocator) use rpgc_attention_decode_noalloc, which guarantees that a call
allocates nothing and keeps no state between calls (its position splits merge
inside a thread-block cluster).  It must give the same result as
rpgc_attention_decode on consecutive calls of different shapes.  This file is
collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import rpgbarengine_b200 as rb  # noqa: E402

TOL = 1e-5  # relative L2, as for the other attention parity tests


def _noalloc():
    fn = rb.lib().rpgc_attention_decode_noalloc
    vp, i32, i64 = C.c_void_p, C.c_int32, C.c_int64
    fn.argtypes = [vp, vp, vp, i64, i32, i32, i32, i64, vp, vp]
    fn.restype = C.c_int
    return fn


def _case(seed, n_heads, n_kv, max_seq):
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.standard_normal(n_heads * 128).astype(np.float32)).cuda()
    kc = torch.from_numpy(rng.standard_normal((n_kv, max_seq, 128)).astype(np.float32)).cuda()
    vc = torch.from_numpy(rng.standard_normal((n_kv, max_seq, 128)).astype(np.float32)).cuda()
    return q, kc, vc


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


def test_noalloc_matches_allocating_entry_point_twice():
    if rb.device_count() == 0:
        pytest.fail("GPU test collected without a CUDA device")
    fn = _noalloc()
    stream = torch.cuda.current_stream().cuda_stream
    for seed, (n_heads, n_kv, max_seq, pos) in enumerate([(32, 8, 1152, 767), (16, 8, 300, 41)]):
        q, kc, vc = _case(seed, n_heads, n_kv, max_seq)
        want = rb.attention_decode(q, kc, vc, pos, n_heads, n_kv)
        got = torch.empty_like(q)
        rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), max_seq, n_heads, n_kv, 128, pos,
                got.data_ptr(), stream)
        assert rc == rb.OK, rb.lib().rpgc_last_error()
        torch.cuda.synchronize()
        assert _rel(got, want) <= TOL


def test_noalloc_rejects_unsupported_groups():
    if rb.device_count() == 0:
        pytest.fail("GPU test collected without a CUDA device")
    fn = _noalloc()
    q, kc, vc = _case(3, 24, 8, 16)  # 3 query heads per kv head
    out = torch.empty_like(q)
    rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), 16, 24, 8, 128, 3, out.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    assert rc == rb.E_ARG
    assert b"group" in rb.lib().rpgc_last_error()
