"""Synthetic model builders on CPU: the torch-drawn Q8_0 tensors that the
tp8b benchmark uploads (same table, layout and value ranges as
build_tensors, which the oracle tests use)."""
import numpy as np
import pytest

from rpgbarengine_b200 import gguf, synth


def _q8_fields(raw: np.ndarray):
    b = raw.reshape(-1, 34)
    d = b[:, 0:2].copy().view("<f2").astype(np.float32).reshape(-1)
    q = b[:, 2:].view(np.int8)
    return d, q


def test_torch_tensors_match_the_numpy_table():
    pytest.importorskip("torch")
    shape = synth.TINY_TP
    a = synth.build_tensors(shape, 5)
    b = synth.build_tensors_torch(shape, 5, "cpu")
    assert [t.name for t in a] == [t.name for t in b]
    for ta, tb in zip(a, b):
        assert ta.ggml_type == tb.ggml_type and tuple(ta.dims) == tuple(tb.dims)
        assert ta.data.nbytes == tb.data.nbytes
    for name, ty, rows, cols in shape.matrices():
        assert ty == gguf.Q8_0
    d, q = _q8_fields(b[0].data)
    assert d.min() >= np.float32(np.float16(1e-4)) and d.max() <= np.float32(np.float16(2e-4))
    assert q.min() >= -127 and q.max() <= 127  # -128 never drawn
    # roughly uniform over the 255 values
    assert abs(float(q.astype(np.float64).mean())) < 2.0
    assert len(np.unique(q)) == 255


def test_torch_tensors_are_seeded():
    pytest.importorskip("torch")
    shape = synth.TINY_TP
    x = synth.build_tensors_torch(shape, 9, "cpu")[0].data
    y = synth.build_tensors_torch(shape, 9, "cpu")[0].data
    z = synth.build_tensors_torch(shape, 10, "cpu")[0].data
    assert np.array_equal(x, y)
    assert not np.array_equal(x, z)


def test_torch_builder_rejects_k_quants():
    pytest.importorskip("torch")
    with pytest.raises(ValueError):
        synth.build_tensors_torch(synth.TINY_MIX, 1, "cpu")


@pytest.mark.parametrize("ty", [gguf.Q4_K, gguf.Q6_K, gguf.Q8_0])
def test_torch_blocks_have_the_benchmark_fields(ty):
    torch = pytest.importorskip("torch")
    gen = torch.Generator(device="cpu")
    gen.manual_seed(3)
    rows, cols = 64, 512
    b = synth.random_blocks_torch(ty, rows, cols, gen, "cpu").numpy()
    assert b.nbytes == rows * gguf.row_bytes(ty, cols)
    if ty == gguf.Q8_0:
        d, q = _q8_fields(b)
        assert d.min() >= np.float32(np.float16(1e-4)) and d.max() <= np.float32(np.float16(2e-4))
        assert q.min() >= -127
        return
    blk = b.reshape(-1, 144 if ty == gguf.Q4_K else 210)
    if ty == gguf.Q4_K:
        d = blk[:, 0:2].copy().view("<f2").astype(np.float32)
        dmin = blk[:, 2:4].copy().view("<f2").astype(np.float32)
        assert d.min() >= np.float32(np.float16(1e-3)) and d.max() <= np.float32(np.float16(4e-3))
        assert dmin.min() >= 0 and dmin.max() <= np.float32(np.float16(1e-3))
    else:
        sc = blk[:, 192:208].view(np.int8)
        d = blk[:, 208:210].copy().view("<f2").astype(np.float32)
        assert sc.min() >= -32 and sc.max() <= 31
        assert d.min() >= np.float32(np.float16(1e-3)) and d.max() <= np.float32(np.float16(4e-3))
