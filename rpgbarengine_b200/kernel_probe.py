"""Run one kernel of the token loop a few times on config-2 (Qwen3-4B Q4_K_M
mix) shapes, for timing and profiler captures of a single kernel.

  python -m rpgbarengine_b200.kernel_probe gemv-gate     # Q4_K 9728 x 2560, batch 1
  python -m rpgbarengine_b200.kernel_probe gemv-down     # Q6_K 2560 x 9728, batch 1
  python -m rpgbarengine_b200.kernel_probe gemv-lm       # Q6_K 151936 x 2560, batch 1
  python -m rpgbarengine_b200.kernel_probe gemm-gate 512 # Q4_K 9728 x 2560, 512 tokens
  python -m rpgbarengine_b200.kernel_probe gemm-q 512    # Q4_K 4096 x 2560
  python -m rpgbarengine_b200.kernel_probe gemm-down 512 # Q6_K 2560 x 9728
  python -m rpgbarengine_b200.kernel_probe attn 767      # decode attention, 32 / 8 heads, pos 767
  python -m rpgbarengine_b200.kernel_probe step 4        # config-2 model: 512-token prefill, 4 decode steps
  python -m rpgbarengine_b200.kernel_probe batch 64      # 64 sessions at position 1024, batched steps

Weights are seeded random blocks of the benchmark's distributions; each
launch reads its own weight copy, the copies together larger than L2.
Prints the mean launch time from CUDA events around a loop of launches.
"""
from __future__ import annotations

import sys

import numpy as np


def main(argv):
    import torch

    import rpgbarengine_b200 as rb
    from rpgbarengine_b200 import gguf, synth

    name = argv[0] if argv else "gemv-gate"
    arg = int(argv[1]) if len(argv) > 1 else 0
    reps = int(argv[2]) if len(argv) > 2 else 6
    rng = np.random.default_rng(0)
    mats = {"gate": (gguf.Q4_K, 9728, 2560), "down": (gguf.Q6_K, 2560, 9728),
            "lm": (gguf.Q6_K, 151936, 2560), "q": (gguf.Q4_K, 4096, 2560),
            "o": (gguf.Q4_K, 2560, 4096)}
    kind, _, which = name.partition("-")
    if kind in ("gemv", "gemm"):
        ty, rows, cols = mats[which]
        one = torch.from_numpy(synth.random_blocks(rng, ty, rows, cols)).cuda()
        ws = [one] + [one.clone() for _ in range(int(np.ceil(160e6 / one.numel())) - 1)]
        n = 1 if kind == "gemv" else (arg or 512)
        X = torch.randn(n, cols, device="cuda")
        out = torch.empty(n, rows, device="cuda")

        def launch(i):
            w = ws[i % len(ws)]
            if kind == "gemv":
                rb.matvec(ty, w, rows, cols, X[0], out=out[0])
            else:
                rb.matmul_batch(ty, w, rows, cols, X, out=out)
        work = f"{name} {rows}x{cols} n={n}"
    elif kind == "step":  # the whole token loop: prefill launches, then persistent decode steps
        shape = synth.QWEN3_4B_Q4KM
        model = rb.Model.upload(shape, synth.build_tensors(shape, 1234), 0, 4096)
        sess = model.session(800)
        sess.forward_full(synth.prompt_ids(42, 512))
        print("tokens", sess.generate(arg or 4))
        return
    elif kind == "batch":  # batched decode: one 1024-token prefill copied into every session
        shape = synth.QWEN3_4B_Q4KM
        model = rb.Model.upload(shape, synth.build_tensors(shape, 1234), 0, 4096)
        n = arg or 64
        first = model.session(1100)
        first.forward_full(synth.prompt_ids(42, 1024))
        sess = [first]
        for i in range(1, n):
            s = model.session(1100)
            s.copy_prefix_from(first, 1024)
            s.forward_full([7 + i])
            sess.append(s)
        torch.cuda.synchronize()
        # a profiler started with --profile-from-start off sees the batched steps only
        torch.cuda.profiler.start()
        rb.generate_batch(sess, reps)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print("batch", n, "steps", reps)
        return
    elif kind == "attn":
        pos = arg or 767
        max_seq = pos + 1
        q = torch.randn(32 * 128, device="cuda")
        kc = torch.randn(8, max_seq, 128, device="cuda")
        vc = torch.randn(8, max_seq, 128, device="cuda")
        o = torch.empty_like(q)

        def launch(i):
            rb.attention_decode(q, kc, vc, pos, 32, 8, out=o)
        work = f"attention decode 32/8 heads pos {pos}"
    else:
        raise SystemExit(f"unknown kernel {name}")
    for i in range(2):
        launch(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(reps):
        launch(i)
    e1.record()
    torch.cuda.synchronize()
    print(f"{work}: {e0.elapsed_time(e1) * 1e3 / reps:.1f} us per call (host-side calls included)")


if __name__ == "__main__":
    main(sys.argv[1:])
