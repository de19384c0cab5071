"""Tensor-parallel shard arithmetic on CPU, as world-size-2 `gloo` ranks (no
GPU): each rank takes its ranges from the library (rpgc_tp_shard_of, the
ranges rpgc_model_upload_tp copies), slices the raw blocks of a small model's
matrices the way the upload does (whole rows of q/k/v/gate/up/output; for o
and down the same block range of every row), dequantises its slices with the
oracle and computes its part of every projection.  The gathered row slices
must equal the unsharded products, and the all-reduced partial sums of the
column-split projections must match them to fp32 rounding.  The matrices
split are those of the reference's layer (src/qwen3.cc:119-206)."""
import os
import socket

import numpy as np
import pytest

import rpgbarengine_b200 as rb
from rpgbarengine_b200 import gguf, synth

SHAPE = synth.TINY_TP
SEED = 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _mat(tens, name):
    t = next(t for t in tens if t.name == name)
    cols, rows = t.dims
    return t, rows, cols


def _rows_slice(t, cols, r0, r1):
    rb_ = gguf.row_bytes(t.ggml_type, cols)
    return t.data.reshape(-1)[r0 * rb_:r1 * rb_]


def _cols_slice(t, rows, cols, c0, c1):
    # the same block range of every row: bytes [c0 / be * bb, c1 / be * bb)
    be, bb = gguf.TYPE_BLOCK[t.ggml_type]
    assert c0 % be == 0 and c1 % be == 0
    raw = t.data.reshape(rows, gguf.row_bytes(t.ggml_type, cols))
    return np.ascontiguousarray(raw[:, c0 // be * bb:c1 // be * bb])


def _vectors():
    rng = np.random.default_rng(7)
    return {"x": rng.standard_normal(SHAPE.hidden).astype(np.float32),
            "a": rng.standard_normal(SHAPE.q_dim).astype(np.float32),
            "h": rng.standard_normal(SHAPE.intermediate).astype(np.float32)}


def _rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from oracle import Oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        orc = Oracle()
        tens = synth.build_tensors(SHAPE, SEED)
        v = _vectors()
        sh = rb.tp_shard(SHAPE, rank, world)
        out = {}
        # row-split: this rank's rows of the product, gathered in rank order
        for name, key, vec in (("blk.0.attn_q.weight", "q_rows", "x"), ("blk.0.attn_k.weight", "kv_rows", "x"),
                               ("blk.1.attn_v.weight", "kv_rows", "x"), ("blk.0.ffn_gate.weight", "ffn_rows", "x"),
                               ("blk.1.ffn_up.weight", "ffn_rows", "x"), ("output.weight", "vocab_rows", "x")):
            t, rows, cols = _mat(tens, name)
            r0, r1 = sh[key]
            w = orc.dequantize_rows(t.ggml_type, _rows_slice(t, cols, r0, r1), r1 - r0, cols)
            part = torch.from_numpy((w.astype(np.float64) @ v[vec].astype(np.float64)))
            parts = [torch.zeros(r1 - r0, dtype=torch.float64) for _ in range(world)]
            dist.all_gather(parts, part)
            out[name] = torch.cat(parts).numpy()
        # column-split: this rank's partial sums, all-reduced
        for name, key, vec in (("blk.0.attn_output.weight", "o_cols", "a"), ("blk.1.ffn_down.weight", "down_cols", "h")):
            t, rows, cols = _mat(tens, name)
            c0, c1 = sh[key]
            w = orc.dequantize_rows(t.ggml_type, _cols_slice(t, rows, cols, c0, c1), rows, c1 - c0)
            part = torch.from_numpy(w.astype(np.float64) @ v[vec][c0:c1].astype(np.float64))
            dist.all_reduce(part)
            out[name] = part.numpy()
        q.put((rank, None, sh, out))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None, None))
    finally:
        dist.destroy_process_group()


def test_two_rank_shards_reproduce_the_whole_products(orc):
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, err, sh, out = q.get(timeout=300)
        assert err is None, f"rank {r}: {err}"
        res[r] = (sh, out)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # the ranges tile every matrix in rank order
    for key, total in (("q_rows", SHAPE.q_dim), ("kv_rows", SHAPE.kv_dim), ("ffn_rows", SHAPE.intermediate),
                       ("vocab_rows", SHAPE.vocab), ("o_cols", SHAPE.q_dim), ("down_cols", SHAPE.intermediate)):
        got = [res[r][0][key] for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == total and all(got[i][1] == got[i + 1][0] for i in range(world - 1))
    assert res[0][0]["n_heads"] * world == SHAPE.n_heads
    tens = synth.build_tensors(SHAPE, SEED)
    v = _vectors()
    vec_of = {"blk.0.attn_output.weight": "a", "blk.1.ffn_down.weight": "h"}
    for name, whole in res[0][1].items():
        t, rows, cols = _mat(tens, name)
        w = orc.dequantize_rows(t.ggml_type, t.data, rows, cols).astype(np.float64)
        want = w @ v[vec_of.get(name, "x")].astype(np.float64)
        for r in range(world):
            got = res[r][1][name]
            if name in vec_of:  # partial sums over column blocks: rounding of the split sum
                assert np.allclose(got, want, rtol=1e-12, atol=1e-12 * np.abs(want).max()), name
            else:
                assert np.array_equal(got, want), name


def test_shard_shapes_checked():
    with pytest.raises(rb.RpgcError) as e:
        rb.tp_shard(SHAPE, 0, 3)  # 4 heads, 2 kv heads do not divide by 3
    assert e.value.code == rb.E_ARG
    with pytest.raises(rb.RpgcError):
        rb.tp_shard(SHAPE, 2, 2)
    one = rb.tp_shard(synth.QWEN3_8B_Q8_0, 3, 8)
    assert one["n_kv_heads"] == 1 and one["kv_rows"] == (384, 512)
    assert one["vocab_rows"] == (3 * 151936 // 8, 4 * 151936 // 8)
