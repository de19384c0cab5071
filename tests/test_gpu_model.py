"""Whole token loop on the GPU vs the oracle: logits, KV cache, greedy and
sampled generation, prefix reuse, errors."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import rpgbarengine_b200 as rb  # noqa: E402
from rpgbarengine_b200 import synth  # noqa: E402
from tests.gpu_util import LOGIT_REL_L2, compare_tokens, rel_l2  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if rb.device_count() == 0:
        pytest.fail("GPU test collected without a CUDA device")


MODELS = {}


def pair(orc, shape, seed=5, max_pos=1024):
    key = (shape.name, seed, max_pos)
    if key not in MODELS:
        tens = synth.build_tensors(shape, seed)
        MODELS[key] = (rb.Model.upload(shape, tens, 0, max_pos), orc.model(shape, tens, max_pos), tens)
    return MODELS[key][:2]


@pytest.mark.parametrize("shape", [synth.TINY_MIX, synth.TINY_Q8, synth.TINY_UNTIED])
def test_forward_logits_and_kv(orc, shape):
    gm, om = pair(orc, shape)
    ids = synth.prompt_ids(21, 40, shape.vocab)
    s = gm.session(128)
    got = s.forward_full(ids, all_rows=True)
    okv = om.kv(128)
    want = om.forward(ids, okv, all_rows=True)
    for t in range(len(ids)):
        assert rel_l2(got[t], want[t]) <= LOGIT_REL_L2, t
    assert rel_l2(got, want) <= 1e-4  # far inside the gate
    assert s.len == len(ids)
    k, v = s.read_kv()
    ok, ov = okv.arrays()
    n = len(ids)
    # layer 0's rows come from the matmuls alone; later layers' rows inherit
    # the attention's error (fp16 hi/lo three-product split on the tensor
    # cores: ~2^-21 of sum |p v| per output, a few 1e-6 after the o projection)
    assert rel_l2(k[0, :, :n], ok[0, :, :n]) <= 1e-5
    assert rel_l2(v[0, :, :n], ov[0, :, :n]) <= 1e-5
    assert rel_l2(k[:, :, :n], ok[:, :, :n]) <= 3e-5
    assert rel_l2(v[:, :, :n], ov[:, :, :n]) <= 3e-5
    assert np.all(k[:, :, n:] == 0)


def test_single_token_steps_match_prefill(orc):
    # decode-path kernels (one token at a time) vs the oracle's cached forward
    shape = synth.TINY_MIX
    gm, om = pair(orc, shape)
    ids = synth.prompt_ids(3, 12, shape.vocab)
    s = gm.session(64)
    okv = om.kv(64)
    for t in range(len(ids)):
        got = s.forward_full(ids[t:t + 1])
        want = om.forward(ids[t:t + 1], okv)[0]
        assert rel_l2(got, want) <= LOGIT_REL_L2
        assert rel_l2(got, want) <= 1e-4


@pytest.mark.parametrize("T,k,p,seed", [(0.0, 0, 1.0, 0), (0.7, 20, 0.8, 99), (1.0, 0, 0.95, 7),
                                        (1.2, 5, 1.0, 3)])
@pytest.mark.parametrize("shape", [synth.TINY_MIX, synth.TINY_Q8])
def test_generate_matches_oracle(orc, shape, T, k, p, seed):
    gm, om = pair(orc, shape)
    ids = synth.prompt_ids(8, 17, shape.vocab)
    s = gm.session(96)
    s.forward_full(ids)
    got = s.generate(24, temperature=T, top_k=k, top_p=p, seed=seed)
    okv = om.kv(96)
    lg = om.forward(ids, okv)
    want, wl = om.generate(okv, lg[-1], 24, temperature=T, top_k=k, top_p=p, seed=seed,
                           want_logits=True)
    if T > 0:  # sampling consumes u = CounterUniform(seed, pos): sequences must agree
        assert list(got) == list(want)
    else:
        compare_tokens(got, want, wl)
    assert s.len == len(ids) + len(got)


def test_stop_token_is_forwarded(orc):
    shape = synth.TINY_MIX
    gm, om = pair(orc, shape)
    ids = synth.prompt_ids(9, 10, shape.vocab)
    s = gm.session(96)
    s.forward_full(ids)
    free = s.generate(12)
    stop = int(free[3])
    n = list(free).index(stop) + 1
    s2 = gm.session(96)
    s2.forward_full(ids)
    toks = s2.generate(12, stop_ids=[stop])
    assert list(toks) == list(free[:n])
    assert s2.len == len(ids) + n


def test_prefix_reuse_warm_equals_cold(orc):
    shape = synth.TINY_MIX
    gm, _ = pair(orc, shape)
    ids = synth.prompt_ids(4, 30, shape.vocab)
    cold = gm.session(64)
    lc = cold.forward_full(ids)
    warm = gm.session(64)
    warm.forward_full(ids[:19])
    warm.forward_full(np.array([1, 2, 3, 4], np.int32))
    warm.set_len(19)  # src/engine.cc:425-431
    lw = warm.forward_full(ids[19:])
    assert np.array_equal(lc.view(np.uint32), lw.view(np.uint32))
    assert np.array_equal(cold.generate(8), warm.generate(8))


def test_errors(orc):
    shape = synth.TINY_MIX
    gm, _ = pair(orc, shape)
    s = gm.session(20)
    with pytest.raises(rb.RpgcError):
        s.generate(4)  # no forward yet
    with pytest.raises(rb.RpgcError):
        s.forward_full(np.array([shape.vocab], np.int32))
    s.forward_full(synth.prompt_ids(1, 18, shape.vocab))
    with pytest.raises(rb.ContextFull):
        s.generate(8)  # 18 + 8 > 20: the reference throws once the cache is full
    with pytest.raises(rb.ContextFull):
        gm.session(20).forward_full(synth.prompt_ids(1, 21, shape.vocab))


def test_gguf_load_matches_upload(orc, tmp_path):
    shape = synth.TINY_UNTIED
    p = str(tmp_path / "m.gguf")
    tens = synth.write_model(p, shape, 31)
    a = rb.Model.load_gguf(p, 0, 512)
    b = rb.Model.upload(shape, tens, 0, 512)
    ids = synth.prompt_ids(2, 9, shape.vocab)
    la = a.session(32).forward_full(ids)
    lb = b.session(32).forward_full(ids)
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    assert a.weight_bytes == b.weight_bytes


@pytest.mark.slow
def test_config0_full_size(orc):
    """Qwen3-1.7B shape, all Q8_0, full size: 32-token prompt + 32 greedy tokens."""
    shape = synth.QWEN3_1_7B_Q8_0
    orc.set_threads(os.cpu_count() or 8)
    gm, om = pair(orc, shape, seed=0, max_pos=4096)
    ids = synth.prompt_ids(0, 32)
    s = gm.session(128)
    got_l = s.forward_full(ids)
    okv = om.kv(128)
    want_l = om.forward(ids, okv)[0]
    assert rel_l2(got_l, want_l) <= LOGIT_REL_L2
    got = s.generate(32)
    want, wl = om.generate(okv, want_l, 32, want_logits=True)
    compare_tokens(got, want, wl)


def test_copy_prefix_then_forward_matches_one_session(orc):
    # a shared prefix across sessions: session b takes positions [0, 20) from a on
    # the device, forwards the rest, and must agree with a's own forward
    shape = synth.TINY_MIX
    gm, om = pair(orc, shape)
    ids = synth.prompt_ids(5, 48, shape.vocab)
    a = gm.session(128)
    full = a.forward_full(ids, all_rows=True)
    b = gm.session(96)
    b.copy_prefix_from(a, 20)
    assert b.len == 20
    rest = b.forward_full(ids[20:], all_rows=True)
    assert b.len == len(ids)
    for t in range(len(ids) - 20):
        assert rel_l2(rest[t], full[20 + t]) <= 1e-4, t
    okv = om.kv(96)
    want = om.forward(ids, okv, all_rows=True)
    assert rel_l2(rest[-1], want[-1]) <= LOGIT_REL_L2
    ref, ref_logits = om.generate(okv, want[-1], 8, want_logits=True)
    compare_tokens(list(b.generate(8)), ref, ref_logits)
    # the source is untouched and keeps going
    assert a.len == len(ids)
    k_a, _ = a.read_kv()
    k_b, _ = b.read_kv()
    assert np.array_equal(k_a[:, :, :20], k_b[:, :, :20])


def test_copy_prefix_rejects_bad_requests(orc):
    gm, _ = pair(orc, synth.TINY_MIX)
    a = gm.session(64)
    a.forward_full(synth.prompt_ids(6, 10, synth.TINY_MIX.vocab))
    b = gm.session(64)
    with pytest.raises(rb.RpgcError):
        b.copy_prefix_from(a, 11)  # more than the source holds
    with pytest.raises(rb.RpgcError):
        b.copy_prefix_from(b, 1)  # itself
    small = gm.session(4)
    with pytest.raises(rb.ContextFull):
        small.copy_prefix_from(a, 10)
    other, _ = pair(orc, synth.TINY_Q8)
    c = other.session(64)
    with pytest.raises(rb.RpgcError):
        c.copy_prefix_from(a, 5)  # another model
    b.copy_prefix_from(a, 0)
    assert b.len == 0


def test_out_of_range_device_ids_are_reported_not_faulted(orc):
    # ids given on the device skip the host's range check: the embedding
    # kernel must not read outside the table, and the session reports it
    torch = pytest.importorskip("torch")
    gm, _ = pair(orc, synth.TINY_MIX)
    s = gm.session(64)
    ids = torch.tensor([3, synth.TINY_MIX.vocab + 12345, 7, -4], dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    s.forward_device(ids.data_ptr(), 4)
    with pytest.raises(rb.RpgcError) as e:
        s.sync()
    assert e.value.code == rb.E_ARG and "vocabulary" in str(e.value)
    s.sync()  # reported once; the session stays usable
    s.set_len(0)
    good = synth.prompt_ids(8, 6, synth.TINY_MIX.vocab)
    assert np.isfinite(s.forward_full(good)).all()


def test_generate_batch_matches_each_session_alone(orc):
    # three sessions with different prompt lengths decode together; each must
    # produce what the oracle gives it alone (greedy, then seeded sampling)
    shape = synth.TINY_MIX
    gm, om = pair(orc, shape)
    prompts = [synth.prompt_ids(40 + i, n, shape.vocab) for i, n in enumerate((9, 23, 5))]
    for opts in (dict(), dict(temperature=0.8, top_k=40, top_p=0.9, seed=77)):
        sess = [gm.session(64) for _ in prompts]
        for s, p in zip(sess, prompts):
            s.forward_full(p)
        got = rb.generate_batch(sess, 10, **opts)
        for s, p, g in zip(sess, prompts, got):
            okv = om.kv(64)
            first = om.forward(p, okv)[-1]
            ref, ref_logits = om.generate(okv, first, 10, want_logits=True, **opts)
            compare_tokens(list(g), ref, ref_logits)
            assert s.len == len(p) + len(g)
        # the sessions carry on singly after the batch
        nxt = sess[1].generate(3)
        assert len(nxt) == 3


@pytest.mark.parametrize("n_sessions", [24, 150])
def test_generate_batch_many_sessions(orc, n_sessions):
    # large batches split each session's positions less (2 kv heads: 24 sessions
    # take 8 splits, 150 take none); every session still matches the oracle
    shape = synth.TINY_MIX
    gm, om = pair(orc, shape)
    prompts = [synth.prompt_ids(300 + i, 3 + i % 7, shape.vocab) for i in range(n_sessions)]
    sess = [gm.session(16) for _ in prompts]
    for s, p in zip(sess, prompts):
        s.forward_full(p)
    got = rb.generate_batch(sess, 4)
    for p, g in zip(prompts, got):
        okv = om.kv(16)
        first = om.forward(p, okv)[-1]
        ref, ref_logits = om.generate(okv, first, 4, want_logits=True)
        compare_tokens(list(g), ref, ref_logits)


def test_generate_batch_stops_sessions_independently(orc):
    # a stop id taken from session a's own greedy continuation: a stops on it
    # (the stop token is kept), b runs on unless it meets it too
    shape = synth.TINY_MIX
    gm, om = pair(orc, shape)
    p0, p1 = synth.prompt_ids(50, 12, shape.vocab), synth.prompt_ids(51, 7, shape.vocab)
    okv = om.kv(64)
    ref0, _ = om.generate(okv, om.forward(p0, okv)[-1], 6, want_logits=True)
    stop = [int(ref0[2])]
    a, b = gm.session(64), gm.session(64)
    a.forward_full(p0)
    b.forward_full(p1)
    got = rb.generate_batch([a, b], 6, stop_ids=stop)
    for s, p, g in ((a, p0, got[0]), (b, p1, got[1])):
        kv = om.kv(64)
        ref, ref_logits = om.generate(kv, om.forward(p, kv)[-1], 6, stop_ids=stop, want_logits=True)
        compare_tokens(list(g), ref, ref_logits)
        assert s.len == len(p) + len(g)
    assert len(got[0]) <= 3


def test_generate_batch_rejects_bad_batches(orc):
    gm, _ = pair(orc, synth.TINY_MIX)
    a = gm.session(16)
    a.forward_full(synth.prompt_ids(52, 10, synth.TINY_MIX.vocab))
    with pytest.raises(rb.RpgcError):
        rb.generate_batch([a, a], 2)  # twice
    with pytest.raises(rb.ContextFull):
        rb.generate_batch([a], 7)  # room for 6
    fresh = gm.session(16)
    with pytest.raises(rb.RpgcError):
        rb.generate_batch([a, fresh], 2)  # fresh has no pending logits


def test_generate_calls_from_threads_are_batched(orc):
    # rpgc_generate from six threads on one model's sessions, each call with
    # its own length, sampling options and stop ids, with batching on: the
    # calls meet in batches (the model's counters say so) and each result
    # matches the oracle for its session alone
    import threading

    shape = synth.TINY_MIX
    gm, om = pair(orc, shape)
    prompts = [synth.prompt_ids(500 + i, 4 + 3 * i, shape.vocab) for i in range(6)]
    opts = [dict(), dict(temperature=0.8, top_k=40, top_p=0.9, seed=11), dict(),
            dict(temperature=0.7, top_k=0, top_p=0.8, seed=12), dict(), dict(temperature=1.0, seed=13)]
    lengths = [3 + i for i in range(6)]
    okv = om.kv(64)
    ref2, _ = om.generate(okv, om.forward(prompts[2], okv)[-1], lengths[2], want_logits=True)
    opts[2]["stop_ids"] = [int(ref2[1])]  # call 2 stops on its second token
    sess = [gm.session(64) for _ in prompts]
    for s, p in zip(sess, prompts):
        s.forward_full(p)
    got, errs = [None] * 6, []
    start = threading.Barrier(6)

    def run(i):
        try:
            start.wait()
            got[i] = sess[i].generate(lengths[i], **opts[i])
        except Exception as e:  # reported below
            errs.append(e)

    gm.set_batching(8, 200000)  # all six calls arrive well inside the window
    try:
        threads = [threading.Thread(target=run, args=(i,)) for i in range(6)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(120)
    finally:
        gm.set_batching(0)
    assert not errs, errs
    batches, requests = gm.batching_stats()
    assert batches >= 1 and requests >= 4, (batches, requests)
    for s, p, n, o, g in zip(sess, prompts, lengths, opts, got):
        kv = om.kv(64)
        ref, ref_logits = om.generate(kv, om.forward(p, kv)[-1], n, want_logits=True, **o)
        compare_tokens(list(g), ref, ref_logits)
        assert s.len == len(p) + len(g)
    assert len(got[2]) <= 2
    # off again: a call decodes alone and the counters stay
    assert len(sess[0].generate(2)) == 2
    assert gm.batching_stats() == (batches, requests)


def test_batching_setting_is_checked(orc):
    gm, _ = pair(orc, synth.TINY_MIX)
    with pytest.raises(rb.RpgcError):
        gm.set_batching(257, 0)
    with pytest.raises(rb.RpgcError):
        gm.set_batching(4, -1)
    gm.set_batching(4, 100)
    try:
        # a call that is not eligible (no pending logits) runs unbatched and reports its error
        s = gm.session(16)
        with pytest.raises(rb.RpgcError):
            s.generate(2)
        # one eligible call alone: the window passes, it decodes unbatched
        s.forward_full(synth.prompt_ids(53, 5, synth.TINY_MIX.vocab))
        assert len(s.generate(3)) == 3
    finally:
        gm.set_batching(0)


# Hidden 1024 and FFN 2048 give the matmuls 16-32 stages of K: the grouped
# launches (q/k/v, gate+up) and the single ones split K at small token counts
# (partial sums per matrix), which the 512-wide tiny shapes never do.
MID = synth.Qwen3Shape("mid-mix", 1, 1024, 2048, 8, 2, vocab=1024, context_length=1024)


def test_split_k_shapes_prefill_and_batch(orc):
    gm, om = pair(orc, MID)
    prompts = [synth.prompt_ids(700 + i, n, MID.vocab) for i, n in enumerate((40, 9, 130, 17, 66, 3))]
    sess = []
    for p in prompts:
        s = gm.session(200)
        got = s.forward_full(p, all_rows=True)
        okv = om.kv(200)
        want = om.forward(p, okv, all_rows=True)
        for t in range(len(p)):
            assert rel_l2(got[t], want[t]) <= LOGIT_REL_L2, (len(p), t)
        sess.append(s)
    got = rb.generate_batch(sess, 6)
    for s, p, g in zip(sess, prompts, got):
        okv = om.kv(200)
        ref, ref_logits = om.generate(okv, om.forward(p, okv)[-1], 6, want_logits=True)
        compare_tokens(list(g), ref, ref_logits)
        assert s.len == len(p) + len(g)


def test_batched_wait_that_gives_up_fails_only_its_session(orc):
    # a bounded device wait that runs out in one session's slice of the
    # batched attention (the test hook makes session 1's layer-0 blocks wait
    # on a barrier nothing completes) flags that session alone: the call
    # reports RPGC_E_TIMEOUT, the other sessions finish with their tokens
    import ctypes as C

    shape = synth.TINY_MIX
    gm, om = pair(orc, shape)
    prompts = [synth.prompt_ids(60 + i, n, shape.vocab) for i, n in enumerate((6, 9, 4))]
    sess = [gm.session(64) for _ in prompts]
    for s, p in zip(sess, prompts):
        s.forward_full(p)
    L = rb.lib()
    assert L.rpgc_test_stall_next_batch(1) == rb.OK
    handles = (C.c_int32 * 3)(*[s.handle for s in sess])
    o = rb.GenOpts(3, None, 0, 0.0, 0, 1.0, 0)
    out = np.zeros((3, 3), np.int32)
    n_out = np.zeros(3, np.int32)
    rc = L.rpgc_generate_batch(C.cast(handles, C.c_void_p), 3, C.byref(o), out.ctypes.data, n_out.ctypes.data)
    assert rc == rb.E_TIMEOUT, L.rpgc_last_error()
    assert f"session {sess[1].handle}".encode() in L.rpgc_last_error()
    assert n_out[1] == 0 and sess[1].len == len(prompts[1])
    for i in (0, 2):
        assert n_out[i] == 3 and sess[i].len == len(prompts[i]) + 3
        okv = om.kv(64)
        ref, ref_logits = om.generate(okv, om.forward(prompts[i], okv)[-1], 3, want_logits=True)
        compare_tokens(list(out[i]), ref, ref_logits)
    # the failed session needs a forward before it generates again; then it works
    with pytest.raises(rb.RpgcError):
        sess[1].generate(2)
    sess[1].set_len(len(prompts[1]) - 1)
    sess[1].forward_full(prompts[1][-1:])
    assert len(sess[1].generate(2)) == 2
