"""The tcgen05 prefill attention (selected with RPGC_ATTN_TC=1) against the
oracle: logits and KV cache of a ragged multi-tile prompt (several 128-query
and 64-key tiles, a partial last tile), a prefill split into chunks that start
mid-tile (pos0 > 0), and agreement with the default mma.sync kernel.  Same
gates as the default path: logits rel-L2 <= 1e-3 (asserted far tighter), K/V
rows <= 3e-5."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import rpgbarengine_b200 as rb  # noqa: E402
from rpgbarengine_b200 import synth  # noqa: E402
from tests.gpu_util import LOGIT_REL_L2, rel_l2  # noqa: E402

SHAPE = synth.TINY_MIX
MODELS = {}


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if rb.device_count() == 0:
        pytest.fail("GPU test collected without a CUDA device")


def pair(orc):
    if "m" not in MODELS:
        tens = synth.build_tensors(SHAPE, 5)
        MODELS["m"] = (rb.Model.upload(SHAPE, tens, 0, 1024), orc.model(SHAPE, tens, 1024))
    return MODELS["m"]


def test_tc_attention_ragged_prompt_matches_oracle(orc, monkeypatch):
    gm, om = pair(orc)
    ids = synth.prompt_ids(33, 300, SHAPE.vocab)  # 2 full 128-query tiles + 44
    monkeypatch.setenv("RPGC_ATTN_TC", "1")
    s = gm.session(512)
    got = s.forward_full(ids, all_rows=True)
    okv = om.kv(512)
    want = om.forward(ids, okv, all_rows=True)
    for t in range(len(ids)):
        assert rel_l2(got[t], want[t]) <= LOGIT_REL_L2, t
    assert rel_l2(got, want) <= 1e-4
    k, v = s.read_kv()
    ok, ov = okv.arrays()
    n = len(ids)
    assert rel_l2(k[:, :, :n], ok[:, :, :n]) <= 3e-5
    assert rel_l2(v[:, :, :n], ov[:, :, :n]) <= 3e-5
    # the default kernel on the same prompt: both inside the gate, close to each other
    monkeypatch.setenv("RPGC_ATTN_TC", "0")
    s2 = gm.session(512)
    base = s2.forward_full(ids, all_rows=True)
    assert rel_l2(got, base) <= 1e-4


def test_tc_attention_chunks_match_oracle(orc, monkeypatch):
    # chunks of 77, 130 and 93 tokens: the later chunks' query tiles start at
    # pos0 = 77 and 207, mid key tile, and read the earlier chunks' cache rows
    gm, om = pair(orc)
    ids = synth.prompt_ids(34, 300, SHAPE.vocab)
    monkeypatch.setenv("RPGC_ATTN_TC", "1")
    s = gm.session(512)
    got = np.concatenate([s.forward_full(ids[:77], all_rows=True), s.forward_full(ids[77:207], all_rows=True),
                          s.forward_full(ids[207:], all_rows=True)])
    want = om.forward(ids, om.kv(512), all_rows=True)
    for t in range(len(ids)):
        assert rel_l2(got[t], want[t]) <= LOGIT_REL_L2, t
    assert rel_l2(got, want) <= 1e-4
