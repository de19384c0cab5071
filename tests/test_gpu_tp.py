"""Tensor parallelism on 2 GPUs (the 8B shape's layout, small): every rank's
logits and generated tokens against the oracle.  Skipped with fewer than 2
GPUs."""
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
        toks = s.generate(16)
        s2 = model.session(64)  # decode steps one token at a time (the per-token path)
        steps = [s2.forward_full(ids[t:t + 1]) for t in range(8)]
        q.put((rank, None, logits, list(toks), np.stack(steps), None))
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
        r, err, logits, toks, steps, _ = q.get(timeout=300)
        assert err is None, f"rank {r}: {err}"
        out[r] = (logits, toks, steps)
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
