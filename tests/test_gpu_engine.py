"""The token-level engine (rpgc_engine_*) against the oracle's replay of the
reference's per-turn session logic (src/engine.cc:383-487): a conversation of
several turns through the C ABI, each turn's whole prompt as token ids --
a first turn, a prompt grown by the reply and a new message (prefix reuse),
an identical resend (the cache holds the whole prompt: one position is
recomputed), a diverging turn (the cache is cut back to the common prefix),
a prompt that makes the forward fail (the cache is reset), and a prompt too
long for the session (refused before the cache is touched)."""
import pytest

pytestmark = pytest.mark.gpu

import rpgbarengine_b200 as rb  # noqa: E402
from oracle import OracleEngineSession  # noqa: E402
from rpgbarengine_b200 import synth  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if rb.device_count() == 0:
        pytest.fail("GPU test collected without a CUDA device")


@pytest.fixture(scope="module")
def models(orc):
    shape = synth.TINY_MIX
    tens = synth.build_tensors(shape, 77)
    gm = rb.Model.upload(shape, tens, 0, 1024)
    om = orc.model(shape, tens, 1024)
    yield shape, gm, om
    gm.free()


def turn(es, oe, ids, **req):
    got = es.generate(ids, **req)
    want = oe.generate(ids, **req)
    assert list(got[0]) == list(want[0]), (list(got[0]), list(want[0]))
    assert got[1:] == want[1:], (got[1:], want[1:])
    assert list(es.cached()) == oe.cached
    return got


def test_conversation_matches_the_reference_session_logic(models):
    shape, gm, om = models
    V = shape.vocab
    eos, im_end = 7, 11
    gm.set_special_ids(eos, im_end)
    assert gm.special_ids == (eos, im_end)
    opts = dict(max_seq=160, max_tokens=10, temperature=0.8, seed=5, stop_ids=[13])
    es = gm.engine_session(**opts)
    oe = OracleEngineSession(om, eos_id=eos, im_end_id=im_end, **opts)
    a = list(synth.prompt_ids(1, 24, V))
    # 1. first turn: nothing cached
    g1, _, n1, reused1 = turn(es, oe, a)
    assert n1 == 24 and reused1 == 0
    # 2. the prompt grows by the reply and a new message: only those are new
    p2 = a + list(g1) + list(synth.prompt_ids(2, 9, V))
    _, _, _, reused2 = turn(es, oe, p2, seed=9)
    assert reused2 == len(a) + len(g1)
    # 3. identical resend: the cache holds it all, one position is recomputed
    _, _, n3, reused3 = turn(es, oe, p2, seed=9)
    assert reused3 == n3 - 1
    # 4. a greedy turn that diverges after ten ids: the cache is cut back
    p4 = a[:10] + list(synth.prompt_ids(3, 15, V))
    _, _, _, reused4 = turn(es, oe, p4, temperature=0.0, max_tokens=6)
    assert reused4 == 10
    # 5. an id outside the vocabulary: the forward fails and the cache resets
    with pytest.raises(rb.RpgcError):
        es.generate(p4 + [V + 3])
    with pytest.raises(ValueError):
        oe.generate(p4 + [V + 3])
    assert list(es.cached()) == [] == oe.cached
    _, _, _, reused5 = turn(es, oe, p4)
    assert reused5 == 0
    # 6. too long for the session: refused, the cache untouched
    before = list(es.cached())
    with pytest.raises(rb.ContextFull):
        es.generate(list(synth.prompt_ids(4, 150, V)))
    assert list(es.cached()) == before
    # 7. reset: the next turn starts from nothing
    es.reset()
    oe.reset()
    _, _, _, reused7 = turn(es, oe, a)
    assert reused7 == 0
    es.close()


def test_stop_ids_and_finish_reasons(models):
    shape, gm, om = models
    V = shape.vocab
    p = list(synth.prompt_ids(30, 16, V))
    gm.set_special_ids(-1, -1)
    # learn the greedy continuation, then make its third token a stop id
    probe = gm.engine_session(max_seq=96, max_tokens=8)
    free, fin, _, _ = probe.generate(p)
    assert len(free) == 8 and fin == "length"
    probe.close()
    gm.set_special_ids(-1, int(free[2]))  # <|im_end|> stands in as the stop
    es = gm.engine_session(max_seq=96, max_tokens=8)
    oe = OracleEngineSession(om, 96, 8, eos_id=-1, im_end_id=int(free[2]))

    def first_stop(stops):  # the continuation ends at its first stop id, kept
        return next(i for i, t in enumerate(free) if int(t) in stops) + 1

    g, fin, _, _ = turn(es, oe, p)
    assert list(g) == list(free[:first_stop({int(free[2])})]) and fin == "stop"
    # a request stop id adds to the model's
    es.reset()
    oe.reset()
    g, fin, _, _ = turn(es, oe, p, stop_ids=[int(free[1])])
    assert list(g) == list(free[:first_stop({int(free[1]), int(free[2])})]) and fin == "stop"
    es.close()
    gm.set_special_ids(-1, -1)


def test_engine_arguments_are_checked(models):
    shape, gm, _ = models
    with pytest.raises(rb.RpgcError):
        gm.engine_session(max_seq=-1)
    with pytest.raises(rb.RpgcError):
        gm.engine_session(max_tokens=-3)
    with pytest.raises(rb.RpgcError):
        gm.engine_session(stop_ids=[shape.vocab])
    es = gm.engine_session(max_seq=64, max_tokens=500)  # narrowed to max_seq - 1
    with pytest.raises(rb.RpgcError):
        es.generate([])
    with pytest.raises(rb.RpgcError):
        es.generate([1, 2, 3], max_tokens=8, out_cap=4)  # out_ids too small, cache untouched
    assert list(es.cached()) == []
    es.close()
    assert rb.lib().rpgc_engine_session_destroy(99999) == rb.OK
