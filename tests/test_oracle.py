"""The oracle (oracle/rpg_oracle.c) pinned before it is trusted.

1. The reference's own known-answer tests (tools/selftest.cc:429-645).
2. Golden fixtures produced by the reference itself in scalar mode
   (tests/golden/make_golden.py): bit-exact equality.
3. Live comparison with the reference build when oracle/_ref exists.
"""
import math
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

from rpgbarengine_b200 import gguf, synth


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# ---------------------------------------------------------------- selftest KATs
def test_q8_0_known_answer(orc):
    # tools/selftest.cc:432-447: d=1.0, qs = -16..15 -> exactly -16..15
    blk = np.zeros(34, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    blk[2:] = (np.arange(32) - 16).astype(np.int8).view(np.uint8)
    out = orc.dequantize_rows(gguf.Q8_0, blk, 1, 32)
    assert np.array_equal(out[0], np.arange(32, dtype=np.float32) - 16)


@pytest.mark.parametrize("f,h", [(1.0, 0x3C00), (0.5, 0x3800), (-2.5, 0xC100), (65504.0, 0x7BFF),
                                 (65505.0, 0x7BFF), (70000.0, 0x7C00), (1e30, 0x7C00), (0.0, 0),
                                 (1.0 / 16777216.0, 1), (1e-30, 0)])
def test_f16_anchors(orc, f, h):
    # tools/selftest.cc:528-543 (round to nearest even, overflow, subnormal)
    assert orc.f32_to_f16(f) == h


def test_f16_roundtrip_all(orc):
    for h in range(0, 0x10000, 7):
        v = orc.f16_to_f32(h)
        want = np.frombuffer(np.uint16(h).tobytes(), np.float16)[0].astype(np.float32)
        if math.isnan(want):
            assert math.isnan(v)
        else:
            assert v == want and (math.copysign(1, v) == math.copysign(1, want))


def test_sampler_known_answers(orc):
    # tools/selftest.cc:551-644
    assert orc.counter_uniform(42, 0) == orc.counter_uniform(42, 0)
    assert orc.counter_uniform(42, 0) != orc.counter_uniform(43, 0)
    assert all(0.0 <= orc.counter_uniform(7, i) < 1.0 for i in range(256))
    l3 = np.array([4, 2, 0], np.float32)
    hot, cold = orc.filter_to_probs(l3, 2.0, 0, 1.0), orc.filter_to_probs(l3, 0.5, 0, 1.0)
    assert cold[0] > hot[0] and abs(hot.sum() - 1) < 1e-5
    oh = orc.filter_to_probs(np.array([1, 9, 3], np.float32), 0.0, 0, 1.0)
    assert list(oh) == [0.0, 1.0, 0.0]
    assert orc.sample_token(np.array([1, 9, 3], np.float32), 0.0, 0, 1.0, 0.123) == 1
    pk = orc.filter_to_probs(np.array([5, 4, 3, 2, 1, 0], np.float32), 1.0, 2, 1.0)
    assert (pk > 0).sum() == 2 and pk[0] > 0 and pk[1] > 0 and pk[5] == 0
    lp = np.log(np.array([0.5, 0.3, 0.15, 0.05], np.float32))
    p9 = orc.filter_to_probs(lp, 1.0, 0, 0.9)
    assert (p9 > 0).sum() == 3 and p9[3] == 0
    p3 = orc.filter_to_probs(lp, 1.0, 0, 0.3)
    assert p3[0] == 1.0 and p3[1] == 0.0
    u4 = np.zeros(4, np.float32)
    assert [orc.sample_token(u4, 1.0, 0, 1.0, u) for u in (0.0, 0.24, 0.26, 0.99)] == [0, 0, 1, 3]
    assert [orc.sample_token(l3, t, 0, 1.0, 0.95) for t in (0.5, 1.0, 2.0)] == [0, 1, 2]


def test_splitmix64_vector(orc):
    # SplitMix64 of 0 (published test vector of the generator)
    assert orc.splitmix64(0) == 0xE220A8397B1DCDAF


# ---------------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("ty,cols", [(gguf.Q8_0, 512), (gguf.Q4_K, 1024), (gguf.Q6_K, 768)])
def test_golden_kernels(orc, golden, ty, cols):
    g = golden["kernels"]
    w, X = g[f"w_{ty}"], g[f"x_{ty}"]
    assert np.array_equal(bits(orc.dequantize_rows(ty, w, 5, cols)), bits(g[f"deq_{ty}"]))
    assert np.array_equal(bits(orc.matmul(ty, w, 5, cols, X)), bits(g[f"mm_{ty}"]))


def test_golden_sampler(orc, golden):
    g = golden["sampler"]
    for i, (t, k, p) in enumerate(g["opts"]):
        for j, l in enumerate(g["logits"]):
            pr = orc.filter_to_probs(l, float(t), int(k), float(p))
            assert np.array_equal(bits(pr), bits(g["probs"][i, j])), (t, k, p, j)
            assert orc.sample_token(l, float(t), int(k), float(p), float(g["u"][j])) == g["tokens"][i, j]
    for si, s in enumerate((0, 42, 2**63 + 5)):
        assert [orc.counter_uniform(s, c) for c in range(16)] == list(g["rng_u"][si])


def _tiny(orc, golden):
    g = golden["tiny_model"]
    shape = synth.TINY_MIX
    tensors = synth.build_tensors(shape, int(g["seed"]))
    return g, orc.model(shape, tensors, max_pos=256)


def test_golden_tiny_model(orc, golden):
    g, m = _tiny(orc, golden)
    assert np.array_equal(bits(m.rope_table()), bits(g["rope"]))
    ids = g["ids"]
    assert np.array_equal(bits(m.forward(ids, all_rows=True)), bits(g["logits_nokv"]))
    kv = m.kv(64)
    lg = m.forward(ids, kv, all_rows=True)
    assert np.array_equal(bits(lg), bits(g["logits_kv"]))
    assert list(m.generate(kv, lg[-1], 8)) == list(g["greedy"])
    kv2 = m.kv(64)
    lg2 = m.forward(ids, kv2)
    toks = m.generate(kv2, lg2[-1], 8, temperature=0.7, top_k=20, top_p=0.8, seed=99)
    assert list(toks) == list(g["sampled"])
    assert kv2.len == len(ids) + 8


def test_kv_path_equals_full_sequence(orc, golden):
    # tools/gen_check.cc:144-162: prefill through the cache == no-cache forward
    g, m = _tiny(orc, golden)
    ids = g["ids"]
    kv = m.kv(64)
    assert np.array_equal(bits(m.forward(ids, kv, all_rows=True)), bits(m.forward(ids, all_rows=True)))


def test_prefix_reuse_warm_equals_cold(orc, golden):
    # src/engine.cc:383-431: reuse = set_len(lcp) then prefill the rest
    g, m = _tiny(orc, golden)
    ids = g["ids"]
    cold = m.kv(64)
    lc = m.forward(ids, cold)
    warm = m.kv(64)
    m.forward(ids[:7], warm)
    m.forward(np.array([5, 6, 7], np.int32), warm)  # diverging turn
    warm.set_len(7)
    lw = m.forward(ids[7:], warm)
    assert np.array_equal(bits(lc), bits(lw))


def test_generate_stops_and_forwards_stop_token(orc, golden):
    g, m = _tiny(orc, golden)
    kv = m.kv(64)
    lg = m.forward(g["ids"], kv)
    first = m.generate(kv, lg[-1], 8)
    kv2 = m.kv(64)
    lg2 = m.forward(g["ids"], kv2)
    stop = int(first[2])
    n = list(first).index(stop) + 1  # first occurrence ends generation
    toks = m.generate(kv2, lg2[-1], 8, stop_ids=[stop])
    assert list(toks) == list(first[:n])
    assert kv2.len == len(g["ids"]) + n  # the stop token is forwarded too


def test_context_full_is_an_error(orc, golden):
    g, m = _tiny(orc, golden)
    kv = m.kv(len(g["ids"]) + 2)
    lg = m.forward(g["ids"], kv)
    with pytest.raises(OverflowError):
        m.generate(kv, lg[-1], 8)


# ---------------------------------------------------------------- live reference
def _ref_script(body: str) -> str:
    return ("import sys, numpy as np; sys.path.insert(0, %r)\n" % os.path.dirname(os.path.dirname(__file__))
            + "from oracle import Oracle, Reference\nfrom rpgbarengine_b200 import synth, gguf\n" + body)


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(__file__)),
                                                    "oracle", "_ref", "librpgref.so")),
                    reason="reference build (oracle/_ref) not present")
def test_live_reference_scalar_bit_exact():
    body = r'''
import tempfile, os
orc, ref = Oracle(), Reference()
assert ref.kernel == "scalar"
shape = synth.TINY_UNTIED
p = os.path.join(tempfile.mkdtemp(), "m.gguf")
tens = synth.write_model(p, shape, 17)
om, rm = orc.model(shape, tens, 512), ref.load(p, 2, 512)
ids = synth.prompt_ids(4, 20, shape.vocab)
ok, kv = om.kv(96), rm.kv(96)
a, b = om.forward(ids, ok, all_rows=True), rm.forward(ids, kv)
assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
ga = om.generate(ok, a[-1], 12, temperature=1.1, top_k=0, top_p=0.95, seed=3)
gb = rm.generate(kv, b[-1], 12, temperature=1.1, top_k=0, top_p=0.95, seed=3)
assert list(ga) == list(gb), (ga, gb)
print("OK")
'''
    env = dict(os.environ, RPGBAR_NO_SIMD="1", RPGBAR_ENGINE_LOG="off")
    r = subprocess.run([sys.executable, "-c", _ref_script(body)], env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr
