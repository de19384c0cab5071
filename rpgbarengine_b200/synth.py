"""Seeded synthetic Qwen3 weights in raw ggml blocks (no network, no checkpoints).

Value distributions follow the benchmark configurations:
  Q8_0  d = fp16(U[1e-4, 2e-4]), qs = U{-127..127}
  Q4_K  d = fp16(U[1e-3, 4e-3]), dmin = fp16(U[0, 1e-3]), 12 random scale
        bytes (uniform 6-bit sc/m), 128 random quant bytes
  Q6_K  ql/qh random bytes, sc = U{-32..31} (int8), d = fp16(U[1e-3, 4e-3])
  norms F32 = 1.0
Block byte layouts are ggml's (reference src/quant.cc:207-217, 327-354,
396-429).  Shapes follow Qwen3 naming (reference src/model.cc:229-269).
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np

from . import gguf
from .gguf import F32, Q4_K, Q6_K, Q8_0, Tensor


@dataclass(frozen=True)
class Qwen3Shape:
    name: str
    n_layers: int
    hidden: int
    intermediate: int
    n_heads: int
    n_kv_heads: int
    head_dim: int = 128
    vocab: int = 151936
    tied: bool = True
    context_length: int = 8192
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    # ggml type per tensor role
    t_q: int = Q4_K
    t_k: int = Q4_K
    t_v: int = Q6_K
    t_o: int = Q4_K
    t_gate: int = Q4_K
    t_up: int = Q4_K
    t_down: int = Q6_K
    t_embd: int = Q6_K
    t_out: int = Q8_0

    @property
    def q_dim(self):
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self):
        return self.n_kv_heads * self.head_dim

    def matrices(self):
        """(name, ggml type, rows, cols) of every 2-D weight."""
        out = [("token_embd.weight", self.t_embd, self.vocab, self.hidden)]
        if not self.tied:
            out.append(("output.weight", self.t_out, self.vocab, self.hidden))
        for l in range(self.n_layers):
            p = f"blk.{l}."
            out += [
                (p + "attn_q.weight", self.t_q, self.q_dim, self.hidden),
                (p + "attn_k.weight", self.t_k, self.kv_dim, self.hidden),
                (p + "attn_v.weight", self.t_v, self.kv_dim, self.hidden),
                (p + "attn_output.weight", self.t_o, self.hidden, self.q_dim),
                (p + "ffn_gate.weight", self.t_gate, self.intermediate, self.hidden),
                (p + "ffn_up.weight", self.t_up, self.intermediate, self.hidden),
                (p + "ffn_down.weight", self.t_down, self.hidden, self.intermediate),
            ]
        return out

    def weight_bytes(self, per_token: bool = False) -> int:
        """Raw block bytes of all 2-D weights; per_token=True counts what one
        decode step streams (every layer matrix + lm_head, not the embedding
        table, of which one row is read)."""
        tot = 0
        for name, ty, rows, cols in self.matrices():
            nb = rows * gguf.row_bytes(ty, cols)
            if per_token and name == "token_embd.weight":
                nb = gguf.row_bytes(ty, cols) + (nb if self.tied else 0)
            tot += nb
        return tot


# The benchmarked shapes: 1.7B all-Q8_0 (tied), 4B Q4_K_M mix (tied), 8B all-Q8_0 (untied).
QWEN3_1_7B_Q8_0 = Qwen3Shape("qwen3-1.7b-q8_0", 28, 2048, 6144, 16, 8,
                             t_q=Q8_0, t_k=Q8_0, t_v=Q8_0, t_o=Q8_0, t_gate=Q8_0, t_up=Q8_0,
                             t_down=Q8_0, t_embd=Q8_0)
QWEN3_4B_Q4KM = Qwen3Shape("qwen3-4b-q4_k_m", 36, 2560, 9728, 32, 8)
QWEN3_8B_Q8_0 = Qwen3Shape("qwen3-8b-q8_0", 36, 4096, 12288, 32, 8, tied=False,
                           t_q=Q8_0, t_k=Q8_0, t_v=Q8_0, t_o=Q8_0, t_gate=Q8_0, t_up=Q8_0,
                           t_down=Q8_0, t_embd=Q8_0, t_out=Q8_0)
# Small shapes for parity tests (same block types and code paths).
TINY_MIX = Qwen3Shape("tiny-mix", 2, 512, 768, 4, 2, vocab=1024, context_length=1024)
TINY_Q8 = replace(QWEN3_1_7B_Q8_0, name="tiny-q8_0", n_layers=2, hidden=256, intermediate=512,
                  n_heads=2, n_kv_heads=1, vocab=768, context_length=1024)
TINY_UNTIED = replace(TINY_MIX, name="tiny-untied", tied=False, t_out=Q6_K)
# The 8B shape's block types and untied output, small enough for a 2-GPU
# tensor-parallel parity test (every split block-aligned at 2 ranks).
TINY_TP = replace(QWEN3_8B_Q8_0, name="tiny-tp-q8_0", n_layers=2, hidden=512, intermediate=1024,
                  n_heads=4, n_kv_heads=2, vocab=1024, context_length=1024)

SHAPES = {s.name: s for s in (QWEN3_1_7B_Q8_0, QWEN3_4B_Q4KM, QWEN3_8B_Q8_0, TINY_MIX, TINY_Q8,
                              TINY_UNTIED, TINY_TP)}


def _f16_bytes(x: np.ndarray) -> np.ndarray:
    return x.astype("<f2").view(np.uint8).reshape(-1, 2)


def q8_0_blocks(rng: np.random.Generator, n_blocks: int, d=(1e-4, 2e-4)) -> np.ndarray:
    b = np.empty((n_blocks, 34), np.uint8)
    b[:, 0:2] = _f16_bytes(rng.uniform(d[0], d[1], n_blocks))
    b[:, 2:] = rng.integers(-127, 128, (n_blocks, 32), dtype=np.int8).view(np.uint8)
    return b.reshape(-1)


def q4_k_blocks(rng: np.random.Generator, n_blocks: int, d=(1e-3, 4e-3), dmin=(0.0, 1e-3)):
    b = np.frombuffer(rng.bytes(n_blocks * 144), np.uint8).reshape(n_blocks, 144).copy()
    b[:, 0:2] = _f16_bytes(rng.uniform(d[0], d[1], n_blocks))
    b[:, 2:4] = _f16_bytes(rng.uniform(dmin[0], dmin[1], n_blocks))
    return b.reshape(-1)


def q6_k_blocks(rng: np.random.Generator, n_blocks: int, d=(1e-3, 4e-3)):
    b = np.frombuffer(rng.bytes(n_blocks * 210), np.uint8).reshape(n_blocks, 210).copy()
    b[:, 192:208] = rng.integers(-32, 32, (n_blocks, 16), dtype=np.int8).view(np.uint8)
    b[:, 208:210] = _f16_bytes(rng.uniform(d[0], d[1], n_blocks))
    return b.reshape(-1)


def f32_values(values: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(values, dtype="<f4").view(np.uint8).reshape(-1)


def random_blocks(rng: np.random.Generator, ggml_type: int, rows: int, cols: int) -> np.ndarray:
    """rows x cols weights of one type as raw bytes (row-major blocks)."""
    n = rows * cols
    if ggml_type == Q8_0:
        return q8_0_blocks(rng, n // 32)
    if ggml_type == Q4_K:
        return q4_k_blocks(rng, n // 256)
    if ggml_type == Q6_K:
        return q6_k_blocks(rng, n // 256)
    if ggml_type == F32:
        return f32_values(rng.standard_normal(n).astype(np.float32))
    raise ValueError(f"no generator for ggml type {ggml_type}")


def norm_tensors(shape: Qwen3Shape) -> list:
    """The F32 norm gains (all 1.0): output norm, then per layer attention,
    FFN, q and k norms."""
    ones_h = f32_values(np.ones(shape.hidden, np.float32))
    ones_d = f32_values(np.ones(shape.head_dim, np.float32))
    out = [Tensor("output_norm.weight", F32, (shape.hidden,), ones_h)]
    for l in range(shape.n_layers):
        p = f"blk.{l}."
        out.append(Tensor(p + "attn_norm.weight", F32, (shape.hidden,), ones_h))
        out.append(Tensor(p + "ffn_norm.weight", F32, (shape.hidden,), ones_h))
        out.append(Tensor(p + "attn_q_norm.weight", F32, (shape.head_dim,), ones_d))
        out.append(Tensor(p + "attn_k_norm.weight", F32, (shape.head_dim,), ones_d))
    return out


def build_tensors(shape: Qwen3Shape, seed: int) -> list:
    """All tensors of a synthetic model, in Qwen3/GGUF naming order."""
    rng = np.random.default_rng(seed)
    out = []
    for name, ty, rows, cols in shape.matrices():
        out.append(Tensor(name, ty, (cols, rows), random_blocks(rng, ty, rows, cols)))
    return out + norm_tensors(shape)


def random_blocks_torch(ggml_type: int, rows: int, cols: int, gen, device):
    """random_blocks drawn by torch on `device` (a uint8 tensor there): the
    same block layout and distributions (Q8_0: fp16 d in [1e-4, 2e-4], quants
    in [-127, 127]; Q4_K: d in [1e-3, 4e-3], dmin in [0, 1e-3], random scale
    and quant bytes; Q6_K: random ql/qh, int8 scales in [-32, 31], d in
    [1e-3, 4e-3]), a different stream of numbers."""
    import torch

    def f16(n, lo, hi):
        return torch.empty(n, dtype=torch.float32, device=device).uniform_(lo, hi, generator=gen) \
            .to(torch.float16).view(torch.uint8).view(n, 2)

    if ggml_type == Q8_0:
        nb = rows * cols // 32
        blk = torch.empty((nb, 34), dtype=torch.uint8, device=device)
        blk[:, 0:2] = f16(nb, 1e-4, 2e-4)
        blk[:, 2:] = torch.randint(-127, 128, (nb, 32), dtype=torch.int8, device=device,
                                   generator=gen).view(torch.uint8)
    elif ggml_type == Q4_K:
        nb = rows * cols // 256
        blk = torch.randint(0, 256, (nb, 144), dtype=torch.uint8, device=device, generator=gen)
        blk[:, 0:2] = f16(nb, 1e-3, 4e-3)
        blk[:, 2:4] = f16(nb, 0.0, 1e-3)
    elif ggml_type == Q6_K:
        nb = rows * cols // 256
        blk = torch.randint(0, 256, (nb, 210), dtype=torch.uint8, device=device, generator=gen)
        blk[:, 192:208] = torch.randint(-32, 32, (nb, 16), dtype=torch.int8, device=device,
                                        generator=gen).view(torch.uint8)
        blk[:, 208:210] = f16(nb, 1e-3, 4e-3)
    else:
        raise ValueError(f"no torch generator for ggml type {ggml_type}")
    return blk.view(-1)


def build_tensors_torch(shape: Qwen3Shape, seed: int, device) -> list:
    """build_tensors for all-Q8_0 shapes (the 8B benchmark shape), the random
    blocks drawn by torch on `device` (8.7 GB in seconds instead of minutes)
    and returned as host bytes: the same distributions (fp16 d uniform in
    [1e-4, 2e-4], int8 quants uniform in [-127, 127]), a different stream of
    numbers from build_tensors(shape, seed)."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out = []
    for name, ty, rows, cols in shape.matrices():
        if ty != Q8_0:
            raise ValueError("build_tensors_torch covers Q8_0 matrices only")
        blk = random_blocks_torch(ty, rows, cols, gen, device)
        out.append(Tensor(name, ty, (cols, rows), blk.cpu().numpy()))
        del blk
    return out + norm_tensors(shape)


def metadata(shape: Qwen3Shape, with_tokenizer: bool = True) -> dict:
    """GGUF metadata the reference's Model::Load needs (src/model.cc:159-211,
    src/tokenizer.cc:135-162): qwen3.* hyper-parameters plus a dummy BBPE
    vocabulary of `vocab` tokens and one merge."""
    a = "qwen3."
    m = {
        "general.architecture": "qwen3",
        "general.name": shape.name,
        "general.alignment": gguf.ALIGN,
        a + "block_count": shape.n_layers,
        a + "context_length": shape.context_length,
        a + "embedding_length": shape.hidden,
        a + "feed_forward_length": shape.intermediate,
        a + "attention.head_count": shape.n_heads,
        a + "attention.head_count_kv": shape.n_kv_heads,
        a + "attention.key_length": shape.head_dim,
        a + "attention.value_length": shape.head_dim,
        a + "rope.freq_base": float(shape.rope_theta),
        a + "attention.layer_norm_rms_epsilon": float(shape.rms_eps),
    }
    if with_tokenizer:
        m["tokenizer.ggml.model"] = "gpt2"
        m["tokenizer.ggml.pre"] = "qwen2"
        m["tokenizer.ggml.tokens"] = [f"<t{i}>" for i in range(shape.vocab)]
        m["tokenizer.ggml.token_type"] = [1] * shape.vocab
        m["tokenizer.ggml.merges"] = ["< t"]
    return m


def write_model(path: str, shape: Qwen3Shape, seed: int) -> list:
    tensors = build_tensors(shape, seed)
    gguf.write(path, metadata(shape), tensors)
    return tensors


def prompt_ids(seed: int, n: int, vocab: int = 151936, hi: int = 151643) -> np.ndarray:
    """Seeded uniform token ids in [0, min(hi, vocab))."""
    return np.random.default_rng(seed).integers(0, min(hi, vocab), n).astype(np.int32)
