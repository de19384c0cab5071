"""Kernel parity on the GPU through the C ABI, against the oracle."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import rpgbarengine_b200 as rb  # noqa: E402
from rpgbarengine_b200 import gguf, synth  # noqa: E402
from tests.gpu_util import ROW_GATE, row_gate  # noqa: E402

TYPES = [gguf.Q8_0, gguf.Q4_K, gguf.Q6_K]
# the microbench shapes (rows x cols) plus ragged ones: odd row counts, partial tiles,
# odd block counts per row (unaligned Q6_K rows)
SHAPES = [(6144, 2048), (2048, 6144), (9728, 2560), (37, 512), (5, 768), (33, 256)]


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available() or rb.device_count() == 0:
        pytest.fail("GPU test collected without a CUDA device")


def dev_u8(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def legal_random(ty, rows, cols, seed):
    """Selftest-style structurally legal blocks: finite scales, random quant bytes."""
    rng = np.random.default_rng(seed)
    return synth.random_blocks(rng, ty, rows, cols)


@pytest.mark.parametrize("ty", TYPES + [gguf.F32])
@pytest.mark.parametrize("rows,cols", [(7, 512), (64, 2560), (3, 768)])
def test_dequant_bit_exact(orc, ty, rows, cols):
    if ty == gguf.F32:
        w = synth.f32_values(np.random.default_rng(1).standard_normal(rows * cols).astype(np.float32))
    else:
        w = legal_random(ty, rows, cols, 11 + rows)
    got = rb.dequantize_rows(ty, dev_u8(w), rows, cols).cpu().numpy()
    want = orc.dequantize_rows(ty, w, rows, cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_dequant_f16_bit_exact(orc):
    h = np.arange(0, 65536, dtype=np.uint32).astype(np.uint16)  # every half, NaNs included
    got = rb.dequantize_rows(gguf.F16, dev_u8(h.view(np.uint8)), 1, h.size).cpu().numpy()[0]
    want = orc.dequantize_rows(gguf.F16, h.view(np.uint8), 1, h.size)[0]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("ty", TYPES)
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_matvec_row_gate(orc, ty, rows, cols):
    w = legal_random(ty, rows, cols, rows * 7 + cols)
    x = np.random.default_rng(rows).standard_normal(cols).astype(np.float32)
    y = rb.matvec(ty, dev_u8(w), rows, cols, torch.from_numpy(x).cuda()).cpu().numpy()
    assert row_gate(orc, ty, w, rows, cols, x, y) <= ROW_GATE


@pytest.mark.parametrize("ty", TYPES)
def test_matvec_lm_head_shape(orc, ty):
    rows, cols = 151936, 2560
    w = legal_random(ty, rows, cols, 5)
    x = np.random.default_rng(2).standard_normal(cols).astype(np.float32) * 3
    y = rb.matvec(ty, dev_u8(w), rows, cols, torch.from_numpy(x).cuda()).cpu().numpy()
    idx = np.unique(np.concatenate([np.arange(64), np.arange(rows - 64, rows),
                                    np.random.default_rng(3).integers(0, rows, 2048)]))
    assert row_gate(orc, ty, w, rows, cols, x, y, idx) <= ROW_GATE
    assert np.isfinite(y).all()


def test_matvec_activation_edge_values(orc):
    # zeros, a single huge outlier, tiny values: the fixed-point activation copy
    ty, rows, cols = gguf.Q4_K, 64, 1024
    w = legal_random(ty, rows, cols, 9)
    x = np.zeros(cols, np.float32)
    x[5] = 3.0e4
    x[300:340] = 1e-30
    x[600] = -7.0
    y = rb.matvec(ty, dev_u8(w), rows, cols, torch.from_numpy(x).cuda()).cpu().numpy()
    assert row_gate(orc, ty, w, rows, cols, x, y) <= ROW_GATE


@pytest.mark.parametrize("ty", TYPES)
@pytest.mark.parametrize("rows,cols,n", [(6144, 2048, 64), (2048, 6144, 64), (9728, 2560, 64),
                                         (37, 512, 11), (5, 768, 9),
                                         (300, 12288, 8),  # the 8B down projection's input width
                                         # prefill sizes: two or three 256-token tiles, a partly
                                         # live last tile, ragged rows, split K
                                         (9728, 2560, 512), (333, 2560, 300), (1000, 4096, 700),
                                         (2560, 9728, 512)])
def test_matmul_row_gate(orc, ty, rows, cols, n):
    w = legal_random(ty, rows, cols, rows + cols + n)
    X = np.random.default_rng(n).standard_normal((n, cols)).astype(np.float32)
    out = rb.matmul_batch(ty, dev_u8(w), rows, cols, torch.from_numpy(X).cuda()).cpu().numpy()
    assert row_gate(orc, ty, w, rows, cols, X, out) <= ROW_GATE


OPTS = [(0.0, 0, 1.0), (0.7, 20, 0.8), (1.0, 0, 0.95), (0.5, 0, 1.0), (1.3, 50, 0.5),
        (2.0, 1, 0.9), (1.0, 0, 1e-9)]


@pytest.mark.parametrize("n", [3000, 151936])
@pytest.mark.parametrize("T,k,p", OPTS)
def test_sampler_matches_oracle(orc, n, T, k, p):
    rng = np.random.default_rng(n + int(T * 10) + k)
    for trial in range(4):
        logits = (rng.standard_normal(n) * (1 + 3 * trial)).astype(np.float32)
        u = orc.counter_uniform(1234, trial)
        want = orc.sample_token(logits, T, k, p, u)
        got = rb.sample_token(torch.from_numpy(logits).cuda(), T, k, p, u)
        assert got == want, (trial, got, want)


def test_sampler_golden(golden):
    g = golden["sampler"]
    for i, (t, k, p) in enumerate(g["opts"]):
        for j, l in enumerate(g["logits"]):
            got = rb.sample_token(torch.from_numpy(l).cuda(), float(t), int(k), float(p),
                                  float(g["u"][j]))
            assert got == g["tokens"][i, j]


def test_sampler_known_answers():
    # tools/selftest.cc:551-644
    def s(lg, t, k, p, u):
        return rb.sample_token(torch.tensor(lg, dtype=torch.float32).cuda(), t, k, p, u)
    assert [s([0, 0, 0, 0], 1.0, 0, 1.0, u) for u in (0.0, 0.24, 0.26, 0.99)] == [0, 0, 1, 3]
    assert [s([4, 2, 0], t, 0, 1.0, 0.95) for t in (0.5, 1.0, 2.0)] == [0, 1, 2]
    assert s([1, 9, 3], 0.0, 0, 1.0, 0.123) == 1
    assert s([3, 9, 9, 1], 0.0, 0, 1.0, 0.5) == 1  # ties -> lowest index


@pytest.mark.parametrize("n_heads,n_kv,max_seq,pos", [(32, 8, 1152, 0), (32, 8, 1152, 767),
                                                      (16, 8, 96, 95), (4, 2, 40, 17),
                                                      (8, 8, 4200, 4100), (64, 8, 200, 150),
                                                      (32, 8, 8192, 8191)])
def test_attention_decode_matches_oracle(orc, n_heads, n_kv, max_seq, pos):
    rng = np.random.default_rng(pos + n_heads)
    q = rng.standard_normal(n_heads * 128).astype(np.float32)
    kc = rng.standard_normal((n_kv, max_seq, 128)).astype(np.float32)
    vc = rng.standard_normal((n_kv, max_seq, 128)).astype(np.float32)
    want = orc.attention_one(q, kc, vc, pos, n_heads, n_kv)
    got = rb.attention_decode(torch.from_numpy(q).cuda(), torch.from_numpy(kc).cuda(),
                              torch.from_numpy(vc).cuda(), pos, n_heads, n_kv).cpu().numpy()
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= 1e-5, err
