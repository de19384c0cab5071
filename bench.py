"""Benchmark: Qwen3-4B Q4_K_M-mix token loop on B200 (the default workload, config2).

One step = one session pass over the config-2 workload: a 512-token prefill of
seeded uniform ids, then 256 greedy decode steps, then (prefix reuse back to
the 512-token prompt) 256 sampled decode steps at T=0.7, top-k 20, top-p 0.8.
Weights are random, in the benchmark's block distributions (synthetic data,
no checkpoint).  The weights (2.62 GB) exceed L2 (126 MB) and are streamed
again by every decode step, so no L2 flush is needed between steps.

  value  decode tok/s (greedy + sampled tokens / decode time), whole job,
         inputs resident on the device (rpgc_forward_device /
         rpgc_generate_device), CUDA events on the session stream.
  e2e    the same through the public host API (rpgc_forward with host ids ->
         host logits, rpgc_generate -> host token ids).
  roofline  the decode step against HBM: (weight bytes streamed per token +
         KV bytes read) / time per token, over the measured copy bandwidth.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
  python bench.py --workload tp8b --steps 1 --warmup 1   # 8B Q8_0 tensor parallel, under torchrun
  python bench.py --workload microbench --steps 5          # matmul kernels per quant type
  python bench.py --workload sessions64                    # 64 sessions, under torchrun for N > 1

N > 1: one process per GPU (torchrun), each rank runs its own independent
session (sessions shard with no communication), value = all ranks' tokens /
the slowest rank's time.  --impl reference times the reference's own CPU code
(oracle/_ref, AVX2, all host threads) on a bounded sample of the same
workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT, DECODE = 512, 256
SAMPLED = dict(temperature=0.7, top_k=20, top_p=0.8, seed=20261201)
METRIC = "Qwen3-4B Q4_K_M decode tok/s (% HBM roofline); 512-tok prefill tok/s"
SEED_WEIGHTS, SEED_PROMPT = 1234, 42


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(float(r[2]) for r in rows),
                "reasons": reasons, "samples": len(rows)}


# DRAM bytes of one step_kernel launch (ncu dram__bytes_read.sum +
# dram__bytes_write.sum; the 4B Q4_K_M-mix model after the 512-token prompt,
# attention over 516 keys)
STEP_TRAFFIC = 2_784_180_480
STEP_TRAFFIC_CTX = 516


def decode_bytes_per_token(shape, ctx: int) -> float:
    """Algorithmic HBM bytes of one decode step: every layer weight + lm_head
    (the embedding table contributes one row) + the fp32 KV read at ctx."""
    w = shape.weight_bytes(per_token=True)
    kv = 2 * shape.n_layers * shape.n_kv_heads * shape.head_dim * 4 * ctx
    return w + kv


def run_gpu(args):
    import torch

    import rpgbarengine_b200 as rb
    from rpgbarengine_b200 import dist as rdist
    from rpgbarengine_b200 import synth

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    torch.cuda.set_device(local)
    dev = local

    shape = synth.QWEN3_4B_Q4KM
    prompt_n, decode_n = args.prompt, args.decode  # the benchmark's 512 and 256 unless profiling a small case
    t0 = time.time()
    tensors = synth.build_tensors(shape, SEED_WEIGHTS)
    # the per-tensor pageable copy (one synchronous host-to-device copy per
    # tensor: the loader's former path) beside rpgc_model_upload's pipelined
    # pinned copy, both from the same resident host arrays
    torch.cuda.synchronize(dev)
    t_pg = time.time()
    for t in tensors:
        torch.from_numpy(np.ascontiguousarray(t.data).reshape(-1).view(np.uint8)).to(f"cuda:{dev}")
    torch.cuda.synchronize(dev)
    pageable_s = time.time() - t_pg
    t_up = time.time()
    model = rb.Model.upload(shape, tensors, dev, 4096)
    upload_s = time.time() - t_up
    del tensors
    build_s = time.time() - t0
    max_seq = prompt_n + decode_n + 8
    sess = model.session(max_seq)
    stream = torch.cuda.ExternalStream(sess.stream_ptr, device=dev)
    # one session per rank: global session index = rank
    (session,) = rdist.shard_sessions(world, rank, world)
    ids_host = synth.prompt_ids(rdist.session_seed(SEED_PROMPT, session), prompt_n)
    ids_dev = torch.from_numpy(ids_host).to(f"cuda:{dev}")
    out_dev = torch.zeros(decode_n + 8, dtype=torch.int32, device=f"cuda:{dev}")
    n_dev = torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
    torch.cuda.synchronize(dev)  # the ids are on the device before the session's own stream reads them

    def ev():
        return torch.cuda.Event(enable_timing=True)

    def device_step(marks):
        sess.set_len(0)
        marks[0].record(stream)
        sess.forward_device(ids_dev.data_ptr(), prompt_n)
        marks[1].record(stream)
        sess.generate_device(decode_n, out_dev.data_ptr(), n_dev.data_ptr())
        sess.set_len(prompt_n)  # prefix reuse: back to the prompt
        # logits for the sampled run: forward the last prompt token again
        sess.set_len(prompt_n - 1)
        sess.forward_device(ids_dev.data_ptr() + 4 * (prompt_n - 1), 1)
        marks[2].record(stream)
        sess.generate_device(decode_n, out_dev.data_ptr(), n_dev.data_ptr(), **SAMPLED)
        marks[3].record(stream)

    def barrier():
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()

    for _ in range(args.warmup):
        device_step([ev() for _ in range(4)])
    barrier()
    clocks = Clocks(dev) if rank == 0 else None
    marks = [[ev() for _ in range(4)] for _ in range(args.steps)]
    start, stop = ev(), ev()
    kl0 = rb.kernel_launches()
    start.record(stream)
    for k in range(args.steps):
        device_step(marks[k])
    stop.record(stream)
    barrier()
    launches = rb.kernel_launches() - kl0
    clk = clocks.stop() if clocks else None
    total_ms = start.elapsed_time(stop)
    pre_ms = sum(m[0].elapsed_time(m[1]) for m in marks)
    dec_ms = sum(m[1].elapsed_time(m[2]) + m[2].elapsed_time(m[3]) for m in marks)
    greedy_ms = sum(m[1].elapsed_time(m[2]) for m in marks)
    sampled_ms = sum(m[2].elapsed_time(m[3]) for m in marks)

    # ---- end to end through the public host API (host ids in, host results out)
    e2e_steps = max(1, min(args.steps, 3))
    ids_pinned = torch.from_numpy(ids_host).pin_memory()
    barrier()
    e0 = time.perf_counter()
    for _ in range(e2e_steps):
        sess.set_len(0)
        sess.forward_full(ids_pinned.numpy())
        sess.generate(decode_n)
        sess.set_len(prompt_n - 1)
        sess.forward_full(ids_pinned.numpy()[prompt_n - 1:])
        sess.generate(decode_n, **SAMPLED)
    barrier()
    e2e_s = time.perf_counter() - e0
    hbm, _, src = peaks()

    total_ms, pre_ms, dec_ms, e2e_s, greedy_ms, sampled_ms = rdist.max_over_ranks(
        [total_ms, pre_ms, dec_ms, e2e_s, greedy_ms, sampled_ms], dist, f"cuda:{dev}")
    if dist:
        dist.destroy_process_group()
    if rank != 0:
        return

    n_dec = 2 * decode_n * args.steps * world
    value = n_dec / (dec_ms / 1e3)
    prefill_tok_s = prompt_n * args.steps * world / (pre_ms / 1e3)
    ctx_avg = prompt_n + decode_n / 2.0
    bytes_tok = decode_bytes_per_token(shape, ctx_avg)
    per_tok_s = (dec_ms / 1e3) / (2 * decode_n * args.steps)
    achieved = bytes_tok / per_tok_s / 1e9
    layer_macs = shape.n_layers * (shape.hidden * (shape.q_dim + 2 * shape.kv_dim) +
                                   shape.q_dim * shape.hidden + 3 * shape.hidden * shape.intermediate)
    attn_flops = shape.n_layers * shape.n_heads * shape.head_dim * 4 * (prompt_n * (prompt_n + 1) / 2)
    prefill_flops = 2 * layer_macs * prompt_n + 2 * shape.vocab * shape.hidden + attn_flops
    if world == 1 and not args.skip_cpu:  # the host cores' reference sample, timed at N=1 only
        cpu = cpu_baseline(shape, args)
    else:
        cpu = {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference",
               "sample": "timed at N=1 only" if world > 1 else "skipped (--skip-cpu)"}
    e2e_tok = e2e_steps * 2 * decode_n * world / e2e_s
    _, bf16, _ = peaks()
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8 dp4a + fp32 (decode), fp16 hi/lo tcgen05 + fp32 (prefill)",
        "data": "synthetic",
        "config": {"workload": "config2: qwen3-4b q4_k_m-mix, 512-tok prefill + 256 greedy + 256 "
                               "sampled (T0.7 k20 p0.8) decode per session",
                   "model": shape.name, "global_batch": world, "seq_len": prompt_n + decode_n,
                   "parallelism": f"sessions x{world} (no communication)",
                   "weights": "raw Q4_K/Q6_K blocks in HBM", "kv": "fp32",
                   "decode_math": "dp4a on 24-bit fixed-point activation limbs, fp32 scales",
                   "l2": "inputs > L2: 2.62 GB of weights re-streamed every decode step",
                   "seed_weights": SEED_WEIGHTS, "seed_prompt": SEED_PROMPT},
        "prefill_tok_s": round(prefill_tok_s, 1),
        "prefill_ms": round(pre_ms / args.steps, 3),
        "prefill_tflops": round(prefill_flops / (pre_ms / args.steps / 1e3) / 1e12, 2),
        "prefill_roofline": {"bound": "tensor",
                             "achieved": round(prefill_flops / (pre_ms / args.steps / 1e3) / 1e12, 2),
                             "peak": bf16, "unit": "TFLOP/s",
                             "frac": round(prefill_flops / (pre_ms / args.steps / 1e3) / 1e12 / bf16, 4),
                             "peak_source": src,
                             "flops": "useful: 2 x the weight MACs of the prompt's tokens, causal "
                                      "attention, one lm_head row; the fp16 hi/lo matmuls issue three "
                                      "MMAs per useful MAC"},
        "greedy_tok_s": round(decode_n * args.steps * world / (greedy_ms / 1e3), 2),
        "sampled_tok_s": round(decode_n * args.steps * world / (sampled_ms / 1e3), 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4),
                     "traffic": (int(STEP_TRAFFIC + (bytes_tok - decode_bytes_per_token(shape, STEP_TRAFFIC_CTX)))
                                 if STEP_TRAFFIC else None),
                     "peak_source": src,
                     "kernel": "step_kernel: one launch per decode token runs all 36 layers and the "
                               "lm_head, whose phase also leaves per-CTA argmax / top-32 candidates; "
                               "the time per launch is the whole decode step (step_kernel + the "
                               "single-block sampler that reads the candidates), greedy and sampled",
                     "algorithmic_bytes_per_launch": int(bytes_tok),
                     "launch_us": round(per_tok_s * 1e6, 2),
                     "timing": "CUDA events on the session stream around the decode loops",
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at "
                                       f"context {STEP_TRAFFIC_CTX}, KV bytes scaled to the mean context"},
        "e2e": {"value": round(e2e_tok, 2), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * (prompt_n + 1),
                "d2h_bytes_per_step": 4 * (2 * shape.vocab + 2 * decode_n)},
        "gpu_launches": launches,
        "clocks": clk,
        "cpu_baseline": cpu,
        "build_s": round(build_s, 1),
        "upload": {"seconds": round(upload_s, 3), "gb": round(model.weight_bytes / 1e9, 3),
                   "gbs": round(model.weight_bytes / 1e9 / upload_s, 2),
                   "pageable_per_tensor_gbs": round(model.weight_bytes / 1e9 / pageable_s, 2),
                   "what": "rpgc_model_upload of the 4B Q4_K_M-mix weights from resident host arrays "
                           "(pinned staging, host threads) vs one pageable copy per tensor"},
    }
    print(json.dumps(line))


TP_PROMPT, TP_DECODE = 4096, 128
TP_METRIC = "Qwen3-8B Q8_0 tensor-parallel decode tok/s (% HBM roofline); 4096-tok prefill tok/s"


def run_tp8b(args):
    """The tp8b workload: the 8B shape (Q8_0, untied output), a 4096-token
    prefill of seeded uniform ids then 128 greedy decode steps, one session
    tensor-parallel over the torchrun ranks (rpgc_model_upload_tp; NCCL
    all-reduce after the row-split o and down projections, vocabulary slices
    of the logits all-gathered).  Strong scaling: the job is fixed, N GPUs
    share it.  value = decode tok/s of the session; the roofline counts the
    bytes all ranks stream per token against N x the measured copy bandwidth."""
    import torch

    import rpgbarengine_b200 as rb
    from rpgbarengine_b200 import dist as rdist
    from rpgbarengine_b200 import synth

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    dev = local
    shape = synth.QWEN3_8B_Q8_0
    t0 = time.time()
    tensors = synth.build_tensors_torch(shape, SEED_WEIGHTS, f"cuda:{dev}")
    if world > 1:
        nid = [rb.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(nid, src=0)
        model = rb.Model.upload_tp(shape, tensors, dev, rank, world, nid[0], TP_PROMPT + TP_DECODE + 64)
    else:
        model = rb.Model.upload(shape, tensors, dev, TP_PROMPT + TP_DECODE + 64)
    del tensors
    build_s = time.time() - t0
    sess = model.session(TP_PROMPT + TP_DECODE + 8)
    stream = torch.cuda.ExternalStream(sess.stream_ptr, device=dev)
    ids = torch.from_numpy(synth.prompt_ids(SEED_PROMPT, TP_PROMPT)).to(f"cuda:{dev}")
    out_dev = torch.zeros(TP_DECODE + 8, dtype=torch.int32, device=f"cuda:{dev}")
    n_dev = torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
    torch.cuda.synchronize(dev)  # the ids are on the device before the session's own stream reads them

    def ev():
        return torch.cuda.Event(enable_timing=True)

    def step(m):
        sess.set_len(0)
        m[0].record(stream)
        sess.forward_device(ids.data_ptr(), TP_PROMPT)
        m[1].record(stream)
        sess.generate_device(TP_DECODE, out_dev.data_ptr(), n_dev.data_ptr())
        m[2].record(stream)

    def barrier():
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()

    for _ in range(args.warmup):
        step([ev() for _ in range(3)])
    barrier()
    clocks = Clocks(dev) if rank == 0 else None
    marks = [[ev() for _ in range(3)] for _ in range(args.steps)]
    kl0 = rb.kernel_launches()
    for k in range(args.steps):
        step(marks[k])
    barrier()
    launches = rb.kernel_launches() - kl0
    clk = clocks.stop() if clocks else None
    pre_ms = sum(m[0].elapsed_time(m[1]) for m in marks)
    dec_ms = sum(m[1].elapsed_time(m[2]) for m in marks)
    total_ms = sum(m[0].elapsed_time(m[2]) for m in marks)
    # the tokens must agree across ranks (every rank samples the same logits)
    toks = out_dev[:TP_DECODE].cpu().numpy()
    digest = int(np.bitwise_xor.reduce(toks.astype(np.int64) * (np.arange(TP_DECODE) + 1)))
    pre_ms, dec_ms, total_ms = rdist.max_over_ranks([pre_ms, dec_ms, total_ms], dist, f"cuda:{dev}")
    digests = [digest]
    if dist:
        digests = [None] * world
        dist.all_gather_object(digests, digest)
        dist.destroy_process_group()
    if rank != 0:
        return
    hbm, _, src = peaks()
    value = TP_DECODE * args.steps / (dec_ms / 1e3)
    prefill_tok_s = TP_PROMPT * args.steps / (pre_ms / 1e3)
    bytes_tok = decode_bytes_per_token(shape, TP_PROMPT + TP_DECODE / 2.0)
    per_tok_s = (dec_ms / 1e3) / (TP_DECODE * args.steps)
    achieved = bytes_tok / per_tok_s / 1e9
    layer_macs = shape.n_layers * (shape.hidden * (shape.q_dim + 2 * shape.kv_dim) +
                                   shape.q_dim * shape.hidden + 3 * shape.hidden * shape.intermediate)
    attn_flops = shape.n_layers * shape.n_heads * shape.head_dim * 4 * (TP_PROMPT * (TP_PROMPT + 1) / 2)
    prefill_flops = 2 * layer_macs * TP_PROMPT + 2 * shape.vocab * shape.hidden + attn_flops
    print(json.dumps({
        "metric": TP_METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "int8 dp4a + fp32 (decode), fp16 hi/lo tcgen05 + fp32 (prefill)",
        "data": "synthetic",
        "config": {"workload": "config4: qwen3-8b q8_0, 4096-tok prefill + 128 greedy decode, "
                               f"tensor parallel x{world}",
                   "model": shape.name, "global_batch": 1, "seq_len": TP_PROMPT + TP_DECODE,
                   "parallelism": (f"tp{world} (column-split q/k/v/gate/up, row-split o/down; decode: "
                                   "partial rows stored into every rank's inbox by the step kernel "
                                   "over peer memory, summed in rank order, vocabulary-split lm_head "
                                   "rows written to every rank; prefill: NCCL all-reduce / all-gather)"
                                   if world > 1 else "tp1 (one GPU, no communication)"),
                   "weights": "raw Q8_0 blocks in HBM", "kv": "fp32",
                   "l2": "inputs > L2: 8.04 GB of weights re-streamed every decode step",
                   "seed_weights": SEED_WEIGHTS, "seed_prompt": SEED_PROMPT},
        "prefill_tok_s": round(prefill_tok_s, 1),
        "prefill_ms": round(pre_ms / args.steps, 3),
        "prefill_tflops": round(prefill_flops / (pre_ms / args.steps / 1e3) / 1e12, 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": round(hbm * world, 1),
                     "unit": "GB/s", "frac": round(achieved / (hbm * world), 4), "traffic": None,
                     "peak_source": src + f" copy bandwidth x {world} GPUs",
                     "kernel": ("whole decode step: the persistent step kernel on every rank, "
                                "two peer-memory exchanges per layer and one for the logits, no "
                                "collective call" if world > 1 else
                                "whole decode step: the persistent step kernel"),
                     "algorithmic_bytes_per_launch": int(bytes_tok),
                     "launch_us": round(per_tok_s * 1e6, 2),
                     "timing": "CUDA events on the session stream, max over ranks"},
        "ranks_agree": len(set(digests)) == 1,
        "gpu_launches": launches,
        "clocks": clk,
        "cpu_baseline": {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference",
                         "sample": "not run for the tp8b workload (the reference's 4096-token CPU "
                                   "prefill alone takes minutes); see the config2 line"},
        "build_s": round(build_s, 1),
    }))


S3_SESSIONS, S3_PREFIX, S3_UNIQUE, S3_DECODE = 64, 256, 768, 128


def run_sessions64(args):
    """The sessions64 workload: 64 independent sessions of the 4B shape, each
    prefilled to 1024 tokens of which the first 256 are a shared prefix, then
    128 greedy decode tokens per session; the sessions are sharded over the
    torchrun ranks with no communication.  Each rank computes the shared
    prefix once and copies its KV into every session on the device
    (rpgc_session_copy_prefix), prefills the 768 unique tokens, then decodes
    all its sessions together with rpgc_generate_batch (one weight stream per
    step for every session).  Device time from CUDA events: the prefills one
    session at a time (each synchronised before the next, so the intervals do
    not overlap, summed), the batched decode around its call; max over ranks."""
    import torch

    import rpgbarengine_b200 as rb
    from rpgbarengine_b200 import dist as rdist
    from rpgbarengine_b200 import synth

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    dev = local
    shape = synth.QWEN3_4B_Q4KM
    model = rb.Model.upload(shape, synth.build_tensors(shape, SEED_WEIGHTS), dev, 4096)
    max_seq = S3_PREFIX + S3_UNIQUE + S3_DECODE + 8
    mine = rdist.shard_sessions(S3_SESSIONS, rank, world)
    shared = torch.from_numpy(synth.prompt_ids(SEED_PROMPT, S3_PREFIX)).to(f"cuda:{dev}")
    unique = {i: torch.from_numpy(synth.prompt_ids(rdist.session_seed(SEED_PROMPT, 1000 + i), S3_UNIQUE))
              .to(f"cuda:{dev}") for i in mine}
    out_dev = torch.zeros(S3_DECODE + 8, dtype=torch.int32, device=f"cuda:{dev}")
    n_dev = torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
    # torch's copies run on its own stream; the sessions' streams do not wait for it
    torch.cuda.synchronize(dev)

    def ev():
        return torch.cuda.Event(enable_timing=True)

    def run(indices):
        pre = ev(), ev()
        psess = model.session(S3_PREFIX + 8)
        pstream = torch.cuda.ExternalStream(psess.stream_ptr, device=dev)
        pre[0].record(pstream)
        psess.forward_device(shared.data_ptr(), S3_PREFIX)
        pre[1].record(pstream)
        pstream.synchronize()
        sessions, pre_ms = [], []
        for i in indices:
            s = model.session(max_seq)
            st = torch.cuda.ExternalStream(s.stream_ptr, device=dev)
            ids = unique[i]
            e = ev(), ev()
            e[0].record(st)
            s.copy_prefix_from(psess, S3_PREFIX)
            s.forward_device(ids.data_ptr(), S3_UNIQUE)
            e[1].record(st)
            st.synchronize()  # one session at a time: the intervals must not overlap
            sessions.append((s, st, ids))
            pre_ms.append(e)
        # every session of the rank in one batched decode (rpgc_generate_batch
        # runs on the first session's stream and returns when all are done)
        torch.cuda.synchronize(dev)
        bst = sessions[0][1]
        e = ev(), ev()
        e[0].record(bst)
        toks = rb.generate_batch([s for s, _, _ in sessions], S3_DECODE)
        e[1].record(bst)
        torch.cuda.synchronize(dev)
        assert all(len(t) == S3_DECODE for t in toks)
        p_ms = pre[0].elapsed_time(pre[1]) + sum(a.elapsed_time(b) for a, b in pre_ms)
        d_ms = e[0].elapsed_time(e[1])
        for s, _, _ in sessions:
            s.close()
        psess.close()
        return p_ms, d_ms

    run(mine[:1])  # warm-up: graphs, plans, module loads
    if dist:
        dist.barrier()
    clocks = Clocks(dev) if rank == 0 else None
    kl0 = rb.kernel_launches()
    pre_ms, dec_ms = run(mine)
    launches = rb.kernel_launches() - kl0
    clk = clocks.stop() if clocks else None
    pre_ms, dec_ms = rdist.max_over_ranks([pre_ms, dec_ms], dist, f"cuda:{dev}")
    if dist:
        dist.destroy_process_group()
    if rank != 0:
        return
    hbm, _, src = peaks()
    # the reference serves sessions one after another: its aggregate rate over
    # the 64 sessions is its one-session decode rate on the same 4B weights
    if world == 1:
        cpu = cpu_baseline(shape, args)
        cpu["sample"] += " (one session; the reference decodes sessions one at a time)"
    else:
        cpu = {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference",
               "sample": "timed at N=1 only"}
    n_tok = S3_SESSIONS * S3_DECODE
    value = n_tok / (dec_ms / 1e3)
    ctx = S3_PREFIX + S3_UNIQUE + S3_DECODE / 2.0
    w_tok = shape.weight_bytes(per_token=True)
    kv_tok = decode_bytes_per_token(shape, ctx) - w_tok
    step_bytes = w_tok + (S3_SESSIONS / world) * kv_tok  # one batched step on one GPU
    achieved = step_bytes * S3_DECODE / (dec_ms / 1e3) / 1e9  # per GPU
    batched_ideal = hbm * 1e9 / (shape.weight_bytes(per_token=True) / S3_SESSIONS +
                                 decode_bytes_per_token(shape, ctx) - shape.weight_bytes(per_token=True))
    print(json.dumps({
        "metric": "sessions64 aggregate decode tok/s, 64 sessions with a shared 256-token prefix",
        "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": 1, "warmup": 1,
        "ms_per_step": round(pre_ms + dec_ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8 dp4a + fp32 (decode), fp16 hi/lo tcgen05 + fp32 (prefill)",
        "data": "synthetic",
        "config": {"workload": "config3: qwen3-4b q4_k_m-mix, 64 sessions x (256 shared + 768 unique "
                               "prefill, 128 greedy decode), sessions sharded over the GPUs",
                   "model": shape.name, "global_batch": S3_SESSIONS, "seq_len": max_seq - 8,
                   "parallelism": f"sessions x{world} (no communication)",
                   "prefix": "computed once per GPU, KV copied device-to-device into each session",
                   "decode": "all of a rank's sessions in one rpgc_generate_batch (tensor-core "
                             "matmuls over the session rows, per-session attention)"},
        "prefill_tok_s": round(S3_SESSIONS * S3_UNIQUE / (pre_ms / 1e3), 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": None, "peak_source": src,
                     "kernel": "batched decode step: weights once per step + every session's KV at ~1088",
                     "batched_ideal_tok_s_per_gpu": round(batched_ideal, 1)},
        "gpu_launches": launches, "clocks": clk,
        "cpu_baseline": cpu,
    }))


MB_SHAPES = [(6144, 2048), (2048, 6144), (9728, 2560), (151936, 2560)]  # rows x cols


def run_microbench(args):
    """The microbench workload: the fused-dequant matmuls per quant type (Q4_K, Q6_K,
    Q8_0) at rows x cols 6144x2048, 2048x6144, 9728x2560 and 151936x2560, on
    f32 N(0,1) activations at batch 1 (rpgc_matvec, the decode GEMV: HBM
    roofline) and batch 64 (rpgc_matmul, the tensor-core GEMM: useful
    TFLOP/s).  Every call reads its own copy of the weights (the copies
    together exceed L2); the calls are captured in a CUDA graph so that the
    time is device time only (CUDA events around graph replays)."""
    import torch

    import rpgbarengine_b200 as rb
    from rpgbarengine_b200 import gguf, synth

    dev = int(os.environ.get("LOCAL_RANK", "0"))
    if int(os.environ.get("RANK", "0")) != 0:
        return
    torch.cuda.set_device(dev)
    hbm, bf16, src = peaks()
    gen = torch.Generator(device=f"cuda:{dev}")
    gen.manual_seed(SEED_WEIGHTS)
    rows_out = []
    stream = torch.cuda.Stream(device=dev)
    cases = [(ty, tname, rows, cols) for ty, tname in ((gguf.Q4_K, "Q4_K"), (gguf.Q6_K, "Q6_K"), (gguf.Q8_0, "Q8_0"))
             for rows, cols in MB_SHAPES]
    if args.mb_only:  # one case, for a profiler capture
        tname, _, rc = args.mb_only.partition(":")
        rows, cols = (int(v) for v in rc.split("x"))
        cases = [(getattr(gguf, tname), tname, rows, cols)]
    for ty, tname, rows, cols in cases:
        if True:
            w0 = synth.random_blocks_torch(ty, rows, cols, gen, f"cuda:{dev}")
            copies = max(1, int(np.ceil(256e6 / w0.numel())))
            ws = [w0] + [w0.clone() for _ in range(copies - 1)]
            wbytes = rows * gguf.row_bytes(ty, cols)
            line = {"type": tname, "rows": rows, "cols": cols, "weight_mb": round(wbytes / 1e6, 2)}
            for n in (1, args.mb_batch):
                X = torch.randn(n, cols, device=f"cuda:{dev}", generator=gen)
                out = torch.empty(n, rows, device=f"cuda:{dev}")
                reps = max(len(ws), 8)

                def calls():
                    for i in range(reps):
                        rb.matmul_batch(ty, ws[i % len(ws)], rows, cols, X, out=out)
                with torch.cuda.stream(stream):
                    calls()  # warm-up (module load, attributes, allocator)
                stream.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    calls()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(stream):  # replays and events on one stream
                    g.replay()
                    stream.synchronize()
                    e0.record(stream)
                    for _ in range(args.steps):
                        g.replay()
                    e1.record(stream)
                torch.cuda.synchronize(dev)
                us = e0.elapsed_time(e1) * 1e3 / (args.steps * reps)
                if n == 1:
                    gbs = (wbytes + 4 * (cols + rows)) / (us * 1e-6) / 1e9
                    line.update(gemv_us=round(us, 2), gemv_gbs=round(gbs, 1), gemv_frac=round(gbs / hbm, 4))
                else:
                    tf = 2.0 * rows * cols * n / (us * 1e-6) / 1e12
                    line.update(gemm_rows=n, gemm64_us=round(us, 2), gemm64_tflops=round(tf, 2),
                                gemm64_frac=round(tf / bf16, 4))
                del g
            rows_out.append(line)
            del ws, w0
            torch.cuda.empty_cache()
    fr = [r["gemv_frac"] for r in rows_out]
    print(json.dumps({
        "metric": "microbench: fused-dequant GEMV (batch 1, HBM roofline) / GEMM (batch 64) per quant type",
        "value": round(float(np.mean(fr)), 4), "unit": "mean GEMV fraction of measured HBM copy bandwidth",
        "n_gpus": 1, "steps": args.steps, "warmup": 1, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8 dp4a + fp32 (GEMV), fp16 hi/lo tcgen05 + fp32 (GEMM)",
        "data": "synthetic", "config": {"workload": "config1: Q4_K/Q6_K/Q8_0 x 4 shapes, batch 1 and 64",
                                        "l2": "each call reads its own weight copy; copies > 256 MB"},
        "peak_hbm_gbs": hbm, "peak_bf16_tflops": bf16, "peak_source": src,
        "table": rows_out,
    }))


REF_DECODE = 8  # greedy and sampled tokens per reference step, each run from position PROMPT


def reference_decode(shape, threads, reps, warmup, path=None):
    """Time the reference's own code (oracle/_ref) at the benchmark's context:
    one PROMPT-token prefill (ForwardFull over the seeded prompt, timed once),
    then per step, from position PROMPT (the cache set back to the prompt as
    the GPU step does), REF_DECODE greedy tokens and REF_DECODE sampled tokens
    at the benchmark's sampling options.  Returns decode tok/s over the timed
    steps (greedy + sampled tokens / their time) and the prefill tok/s."""
    from oracle import Reference
    from rpgbarengine_b200 import synth

    tmp = None
    if path is None:
        tmp = tempfile.mkdtemp(prefix="rpgref_")
        path = os.path.join(tmp, "model.gguf")
        synth.write_model(path, shape, SEED_WEIGHTS)
    ref = Reference()
    m = ref.load(path, threads, 4096)
    ids = synth.prompt_ids(SEED_PROMPT, PROMPT)
    kv = m.kv(PROMPT + 2 * REF_DECODE + 8)
    t = time.perf_counter()
    first = m.forward(ids, kv)[-1].copy()
    pre_s = time.perf_counter() - t
    dec_s = 0.0
    for k in range(warmup + reps):
        t = time.perf_counter()
        kv.set_len(PROMPT)
        m.generate(kv, first, REF_DECODE)
        kv.set_len(PROMPT)
        m.generate(kv, first, REF_DECODE, **SAMPLED)
        if k >= warmup:
            dec_s += time.perf_counter() - t
    kern = ref.kernel
    del kv, m
    if tmp:
        os.remove(path)
        os.rmdir(tmp)
    return reps * 2 * REF_DECODE / dec_s, PROMPT / pre_s, kern


def cpu_baseline(shape, args):
    from oracle import reference_available
    if not reference_available():
        return {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference",
                "sample": "oracle/_ref not built"}
    threads = os.cpu_count() or 1
    os.environ.setdefault("RPGBAR_ENGINE_LOG", "off")
    dec, pre, kern = reference_decode(shape, threads, 1, 0)
    return {"value": round(dec, 3), "unit": "tok/s", "cores": threads, "kind": "reference",
            "sample": f"reference ({kern}) on the same weights: the {PROMPT}-token prefill "
                      f"({pre:.2f} tok/s), then {REF_DECODE} greedy + {REF_DECODE} sampled decode "
                      f"tokens from position {PROMPT}",
            "prefill_tok_s": round(pre, 3)}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from rpgbarengine_b200 import synth
    from oracle import reference_available
    if not reference_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/librpgref.so not built"}))
        return
    os.environ.setdefault("RPGBAR_ENGINE_LOG", "off")
    shape = synth.QWEN3_4B_Q4KM
    threads = os.cpu_count() or 1
    dec, pre, kern = reference_decode(shape, threads, args.steps, args.warmup)
    sample = (f"reference ({kern}) on the same weights, {threads} threads: one {PROMPT}-token "
              f"prefill ({pre:.2f} tok/s), then per step {REF_DECODE} greedy + {REF_DECODE} sampled "
              f"(T0.7 k20 p0.8) decode tokens from position {PROMPT}")
    print(json.dumps({
        "metric": METRIC, "value": round(dec, 3), "unit": "tok/s", "impl": "reference",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2: qwen3-4b q4_k_m-mix, 512-tok prefill, then greedy and sampled "
                               "(T0.7 k20 p0.8) decode from position 512 (CPU reference: "
                               f"{REF_DECODE} + {REF_DECODE} tokens per step)",
                   "model": shape.name, "seq_len": PROMPT + REF_DECODE,
                   "seed_weights": SEED_WEIGHTS, "seed_prompt": SEED_PROMPT},
        "prefill_tok_s": round(pre, 3),
        "cpu_baseline": {"value": round(dec, 3), "unit": "tok/s", "cores": threads,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": round(dec, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--prompt", type=int, default=PROMPT,
                    help="config2 prompt tokens (the benchmark's 512; smaller only for profiler captures)")
    ap.add_argument("--decode", type=int, default=DECODE,
                    help="config2 greedy and sampled tokens per step (the benchmark's 256)")
    ap.add_argument("--skip-cpu", action="store_true",
                    help="leave out the CPU reference sample (profiler captures)")
    ap.add_argument("--mb-batch", type=int, default=64, help="microbench: token rows of the matmul leg")
    ap.add_argument("--mb-only", default="",
                    help="microbench: one case TYPE:ROWSxCOLS (e.g. Q4_K:9728x2560), for profiler captures")
    ap.add_argument("--workload", default="config2", choices=["config2", "tp8b", "microbench", "sessions64"],
                    help="config2 (default): the 4B decode/prefill benchmark; tp8b: the 8B Q8_0 "
                         "shape tensor-parallel over the torchrun ranks; microbench: the matmul "
                         "kernels per quant type; sessions64: 64 sessions with a shared prefix")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "tp8b":
        run_tp8b(args)
    elif args.workload == "microbench":
        run_microbench(args)
    elif args.workload == "sessions64":
        run_sessions64(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
