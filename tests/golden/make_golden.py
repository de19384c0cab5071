"""Generate tests/golden/*.npz from the reference itself.

Runs the reference's own code (oracle/_ref/librpgref.so, compiled from the
reference sources by oracle/Makefile) in its SCALAR mode (RPGBAR_NO_SIMD=1,
read by the reference at load time, src/matmul.cc:41-44) and stores inputs
and outputs as small fixtures.  The tests check the oracle against these
fixtures on machines where the reference is not present.

Usage (where the reference sources exist):
    make -C oracle && RPGBAR_NO_SIMD=1 python tests/golden/make_golden.py
"""
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import Reference  # noqa: E402
from rpgbarengine_b200 import gguf, synth  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def main():
    if os.environ.get("RPGBAR_NO_SIMD") != "1":
        sys.exit("run with RPGBAR_NO_SIMD=1 so the reference uses its scalar path")
    ref = Reference()
    assert ref.kernel == "scalar", ref.kernel
    rng = np.random.default_rng(20261201)

    # 1. dequant + per-row dots on structurally legal random blocks
    kern = {}
    for ty, cols in ((gguf.Q8_0, 512), (gguf.Q4_K, 1024), (gguf.Q6_K, 768)):
        rows = 5
        w = synth.random_blocks(rng, ty, rows, cols)
        X = rng.standard_normal((3, cols)).astype(np.float32) * 3
        kern[f"w_{ty}"] = w
        kern[f"x_{ty}"] = X
        kern[f"deq_{ty}"] = ref.dequantize_rows(ty, w, rows, cols)
        kern[f"mm_{ty}"] = ref.matmul(ty, w, rows, cols, X)
    np.savez_compressed(os.path.join(OUT, "kernels.npz"), **kern)

    # 2. sampler: filter_to_probs + sample_token over several option sets
    smp = {}
    logits = (rng.standard_normal((4, 3000)) * 4).astype(np.float32)
    opts = [(0.7, 20, 0.8), (1.0, 0, 0.95), (0.5, 0, 1.0), (1.3, 50, 0.5), (0.0, 0, 1.0),
            (2.0, 1, 0.9)]
    smp["logits"] = logits
    smp["opts"] = np.array(opts, np.float64)
    probs, toks = [], []
    us = np.array([ref.counter_uniform(7, c) for c in range(4)], np.float32)
    smp["u"] = us
    for (t, k, p) in opts:
        probs.append(np.stack([ref.filter_to_probs(l, t, int(k), p) for l in logits]))
        toks.append([ref.sample_token(l, t, int(k), p, float(u)) for l, u in zip(logits, us)])
    smp["probs"] = np.stack(probs)
    smp["tokens"] = np.array(toks, np.int32)
    smp["rng_u"] = np.array([[ref.counter_uniform(s, c) for c in range(16)] for s in (0, 42, 2**63 + 5)],
                            np.float32)
    np.savez_compressed(os.path.join(OUT, "sampler.npz"), **smp)

    # 3. whole-model: tiny synthetic model, forward logits and generation
    shape, seed = synth.TINY_MIX, 5
    d = tempfile.mkdtemp()
    path = os.path.join(d, "tiny.gguf")
    synth.write_model(path, shape, seed)
    m = ref.load(path, threads=1, max_pos=256)
    ids = synth.prompt_ids(11, 12, shape.vocab)
    mod = {"seed": np.int64(seed), "ids": ids, "rope": m.rope_table()}
    mod["logits_nokv"] = m.forward(ids)
    kv = m.kv(64)
    lg = m.forward(ids, kv)
    mod["logits_kv"] = lg
    mod["greedy"] = m.generate(kv, lg[-1], 8)
    kv2 = m.kv(64)
    lg2 = m.forward(ids, kv2)
    mod["sampled"] = m.generate(kv2, lg2[-1], 8, temperature=0.7, top_k=20, top_p=0.8, seed=99)
    np.savez_compressed(os.path.join(OUT, "tiny_model.npz"), **mod)
    for f in ("kernels.npz", "sampler.npz", "tiny_model.npz"):
        print(f, os.path.getsize(os.path.join(OUT, f)), "bytes")


if __name__ == "__main__":
    main()
