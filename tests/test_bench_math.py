"""Roofline arithmetic of bench.py, checked on the CPU: the algorithmic bytes of
one decode step that the bench divides by a measured duration, recomputed here
from the ggml block sizes (Q4_K 144 B / 256 weights, Q6_K 210 B / 256, Q8_0
34 B / 32, src/quant.h:22-38) and the shapes' dimensions."""
import importlib.util
import os

from rpgbarengine_b200 import gguf, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BLOCK = {gguf.Q4_K: (256, 144), gguf.Q6_K: (256, 210), gguf.Q8_0: (32, 34), gguf.F32: (1, 4)}


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)  # defines functions only; main() runs under __main__
    return mod


def matrix_bytes(ty, rows, cols):
    per, nbytes = BLOCK[ty]
    assert cols % per == 0
    return rows * (cols // per) * nbytes


def step_weight_bytes(shape):
    # every layer matrix and the lm_head once; of the embedding table one row
    tot = 0
    for name, ty, rows, cols in shape.matrices():
        if name == "token_embd.weight":
            tot += matrix_bytes(ty, 1, cols)
            if shape.tied:  # the table is also the lm_head
                tot += matrix_bytes(ty, rows, cols)
        else:
            tot += matrix_bytes(ty, rows, cols)
    return tot


def test_config2_step_bytes():
    b = load_bench()
    s = synth.QWEN3_4B_Q4KM
    w = step_weight_bytes(s)
    assert w == s.weight_bytes(per_token=True)
    assert abs(w - 2.618e9) < 1e6  # the 2.62 GB per token the decode roofline quotes
    kv_per_pos = 2 * s.n_layers * s.n_kv_heads * s.head_dim * 4  # fp32 K and V
    assert kv_per_pos == 294912
    for ctx in (1, 514, 767, 1088):
        assert b.decode_bytes_per_token(s, ctx) == w + kv_per_pos * ctx


def test_config4_step_bytes_all_q8_0():
    b = load_bench()
    s = synth.QWEN3_8B_Q8_0
    assert not s.tied
    w = step_weight_bytes(s)
    assert w == s.weight_bytes(per_token=True)
    assert abs(w - 8.04e9) < 0.01e9  # the 8.04 GB re-streamed every step at TP 1
    assert b.decode_bytes_per_token(s, 0) == w


def test_every_bench_shape_is_whole_blocks():
    for s in (synth.QWEN3_1_7B_Q8_0, synth.QWEN3_4B_Q4KM, synth.QWEN3_8B_Q8_0):
        for name, ty, rows, cols in s.matrices():
            assert cols % BLOCK[ty][0] == 0, (s.name, name)
            assert gguf.row_bytes(ty, cols) == matrix_bytes(ty, 1, cols)
