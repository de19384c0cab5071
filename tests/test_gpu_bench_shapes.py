"""Parity at the benchmarked model shapes, not only the tiny ones.

The decode step kernel is instantiated per (block-type mix, query heads per
kv head) and plans its phases from the matrix widths, so the shapes that the
benchmarks time are checked here against the oracle directly:

  * the 4B Q4_K_M mix (36 layers, hidden 2560, FFN 9728, 32 query / 8 kv
    heads: four query heads per kv head, vocabulary 151936, tied output)
    through rpgc_forward + rpgc_generate: prompt logits, teacher-forced
    single-token steps (each one launch of the persistent step kernel),
    greedy and sampled generation (temperature 0.7, top-k 20, top-p 0.8);
  * the same model decoding eight sessions at once (rpgc_generate_batch)
    after a shared prompt prefix copied between sessions on the device;
  * the 8B Q8_0 layout (hidden 4096, FFN 12288, untied output head,
    four query heads per kv head) at full width and full vocabulary with
    two layers, so the step kernel's K-dependent plans are the 8B model's.

The oracle is the C restatement of the reference's scalar path
(src/qwen3.cc:208-355, src/sampler.cc:36-112).
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import rpgbarengine_b200 as rb  # noqa: E402
from rpgbarengine_b200 import synth  # noqa: E402
from tests.gpu_util import LOGIT_REL_L2, compare_tokens, rel_l2  # noqa: E402

PROMPT = 48
DECODE = 24
SAMPLED = dict(temperature=0.7, top_k=20, top_p=0.8, seed=20251)


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if rb.device_count() == 0:
        pytest.fail("GPU test collected without a CUDA device")


@pytest.fixture(scope="module")
def m4b(orc):
    orc.set_threads(os.cpu_count() or 8)
    shape = synth.QWEN3_4B_Q4KM
    tens = synth.build_tensors(shape, 2)
    gm = rb.Model.upload(shape, tens, 0, 1024)
    om = orc.model(shape, tens, 1024)
    ids = synth.prompt_ids(12, PROMPT)
    okv = om.kv(256)
    first = om.forward(ids, okv)[0]
    yield gm, om, ids, okv, first
    gm.free()


def test_4b_prompt_and_greedy_steps(m4b):
    gm, om, ids, okv, first = m4b
    s = gm.session(256)
    got_first = s.forward_full(ids)
    assert rel_l2(got_first, first) <= LOGIT_REL_L2
    okv.set_len(PROMPT)
    want, want_logits = om.generate(okv, first, DECODE, want_logits=True)
    # greedy decode on the device (the captured step graph: sampler + step kernel)
    got = s.generate(DECODE)
    n_cmp = compare_tokens(got, want, want_logits)
    assert n_cmp >= 4, "the reference's top-2 margins were too small to compare anything"
    assert s.len == PROMPT + len(got)
    # teacher-forced single-token forwards: every step's logits against the
    # oracle's at the same position (each forward is one step-kernel launch)
    t = gm.session(256)
    t.forward_full(ids)
    for i in range(DECODE - 1):
        lg = t.forward_full(np.array([want[i]], np.int32))
        err = rel_l2(lg, want_logits[i + 1])
        assert err <= LOGIT_REL_L2, (i, err)
        assert err <= 1e-4, (i, err)  # far inside the gate: a kernel slip shows here first


def test_4b_sampled(m4b):
    gm, om, ids, okv, first = m4b
    s = gm.session(256)
    s.forward_full(ids)
    got = s.generate(DECODE, **SAMPLED)
    okv.set_len(PROMPT)
    want = om.generate(okv, first, DECODE, **SAMPLED)
    assert list(got) == list(want)
    assert s.len == PROMPT + len(got)


def test_4b_batch_of_eight_after_shared_prefix(m4b):
    # eight sessions open with the 48-token prompt (computed once, copied on
    # the device), add 1-4 tokens of their own and decode 5 tokens together;
    # each must match the oracle run for that session alone
    gm, om, ids, okv, _ = m4b
    base = gm.session(128)
    base.forward_full(ids)
    sess, suffixes = [], []
    for i in range(8):
        suf = synth.prompt_ids(900 + i, 1 + i % 4)
        s = gm.session(96)
        s.copy_prefix_from(base, PROMPT)
        s.forward_full(suf)
        sess.append(s)
        suffixes.append(suf)
    opts = [dict(), SAMPLED]
    for k, o in enumerate(opts):
        if k:  # second round: back to the end of each session's own prompt
            for s, suf in zip(sess, suffixes):
                s.set_len(PROMPT)
                s.forward_full(suf)
        got = rb.generate_batch(sess, 5, **o)
        for s, suf, g in zip(sess, suffixes, got):
            okv.set_len(PROMPT)
            lg = om.forward(suf, okv)[0]
            ref, ref_logits = om.generate(okv, lg, 5, want_logits=True, **o)
            if o:
                assert list(g) == list(ref)
            else:
                compare_tokens(list(g), ref, ref_logits)
            assert s.len == PROMPT + len(suf) + len(g)


def test_8b_layout_two_layers_full_width(orc):
    orc.set_threads(os.cpu_count() or 8)
    shape = synth.replace(synth.QWEN3_8B_Q8_0, name="qwen3-8b-q8_0-2layer", n_layers=2)
    tens = synth.build_tensors(shape, 8)
    gm = rb.Model.upload(shape, tens, 0, 1024)
    try:
        om = orc.model(shape, tens, 1024)
        ids = synth.prompt_ids(13, 20)
        s = gm.session(128)
        got_first = s.forward_full(ids)
        okv = om.kv(128)
        first = om.forward(ids, okv)[0]
        assert rel_l2(got_first, first) <= LOGIT_REL_L2
        want, want_logits = om.generate(okv, first, 16, want_logits=True)
        got = s.generate(16)
        compare_tokens(got, want, want_logits)
        t = gm.session(128)
        t.forward_full(ids)
        for i in range(15):
            lg = t.forward_full(np.array([want[i]], np.int32))
            err = rel_l2(lg, want_logits[i + 1])
            assert err <= 1e-4, (i, err)
    finally:
        gm.free()
