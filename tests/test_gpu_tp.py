"""Tensor parallelism on 2 GPUs (the 8B shape's layout, small): every rank's
logits and generated tokens against the oracle, the decode steps through the
persistent step kernel whose row-split projections exchange partial rows
with plain peer stores (no collective call per token), and a rank that never
signals: the other rank's bounded wait gives up and reports RPGC_E_TIMEOUT.
Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import rpgbarengine_b200 as rb  # noqa: E402
from rpgbarengine_b200 import synth  # noqa: E402
from tests.gpu_util import LOGIT_REL_L2, compare_tokens, rel_l2  # noqa: E402

WORLD = 2
SHAPE = synth.TINY_TP


def _rank(rank, world, nccl_id, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"  # plain peer paths (no multicast objects) in tests
    try:
        import rpgbarengine_b200 as rbl
        from rpgbarengine_b200 import synth as sy
        tens = sy.build_tensors(SHAPE, 11)
        model = rbl.Model.upload_tp(SHAPE, tens, rank, rank, world, nccl_id, 1024)
        s = model.session(128)
        ids = sy.prompt_ids(4, 33, SHAPE.vocab)
        logits = s.forward_full(ids, all_rows=True)
        k0 = rbl.kernel_launches()
        toks = s.generate(16)
        launches = rbl.kernel_launches() - k0
        s2 = model.session(64)  # decode steps one token at a time (the per-token path)
        steps = [s2.forward_full(ids[t:t + 1]) for t in range(8)]
        q.put((rank, None, logits, list(toks), np.stack(steps), launches))
    except Exception as e:  # report, do not hang the parent
        q.put((rank, repr(e), None, None, None, None))


def test_tensor_parallel_matches_oracle(orc):
    if rb.device_count() < WORLD:
        pytest.skip(f"tensor parallelism needs {WORLD} GPUs")
    import torch.multiprocessing as mp
    nccl_id = rb.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, WORLD, nccl_id, q), daemon=True) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(WORLD):
        r, err, logits, toks, steps, launches = q.get(timeout=300)
        assert err is None, f"rank {r}: {err}"
        out[r] = (logits, toks, steps)
        # one sampler + one step kernel per token (the per-launch path with
        # its collectives takes ~10 launches per layer)
        assert launches <= 3 * 16, (r, launches)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    tens = synth.build_tensors(SHAPE, 11)
    om = orc.model(SHAPE, tens, 1024)
    ids = synth.prompt_ids(4, 33, SHAPE.vocab)
    okv = om.kv(128)
    want = om.forward(ids, okv, all_rows=True)
    ref, ref_logits = om.generate(okv, want[-1], 16, want_logits=True)
    okv2 = om.kv(64)
    want_steps = np.stack([om.forward(ids[t:t + 1], okv2)[0] for t in range(8)])
    for r in range(WORLD):
        logits, toks, steps = out[r]
        for t in range(len(ids)):
            assert rel_l2(logits[t], want[t]) <= LOGIT_REL_L2, (r, t)
        for t in range(8):
            assert rel_l2(steps[t], want_steps[t]) <= LOGIT_REL_L2, (r, t)
        compare_tokens(toks, ref, ref_logits)
    # every rank holds the same logits and picks the same tokens
    assert np.array_equal(out[0][0], out[1][0])
    assert out[0][1] == out[1][1]


def _stall_rank(rank, world, nccl_id, q, go):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import rpgbarengine_b200 as rbl
        from rpgbarengine_b200 import synth as sy
        tens = sy.build_tensors(SHAPE, 11)
        model = rbl.Model.upload_tp(SHAPE, tens, rank, rank, world, nccl_id, 1024)
        s = model.session(128)
        s.forward_full(sy.prompt_ids(4, 20, SHAPE.vocab))
        s.generate(2)  # both ranks: the step plan and the peer mappings
        if rank == 0:
            # rank 1 never launches this step: every exchange wait gives up
            try:
                s.generate(4)
                q.put((rank, "no error"))
            except rbl.RpgcError as e:
                q.put((rank, e.code))
        else:
            q.put((rank, "idle"))
            go.get(timeout=300)  # stay alive (nothing in flight) until rank 0 is done
    except Exception as e:
        q.put((rank, repr(e)))


def test_tensor_parallel_wait_that_gives_up():
    if rb.device_count() < WORLD:
        pytest.skip(f"tensor parallelism needs {WORLD} GPUs")
    import torch.multiprocessing as mp
    nccl_id = rb.tp_unique_id()
    ctx = mp.get_context("spawn")
    q, go = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_stall_rank, args=(r, WORLD, nccl_id, q, go), daemon=True) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(WORLD):
            r, v = q.get(timeout=300)
            got[r] = v
    finally:
        go.put("done")
        for p in procs:
            p.join(timeout=60)
    assert got[1] == "idle", got
    assert got[0] == rb.E_TIMEOUT, got
