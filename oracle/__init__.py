"""ctypes loaders for the parity checkers (test infrastructure only).

  Oracle     liboracle.so, the C restatement of the reference token loop
             (rpg_oracle.c).  Pinned bit-exactly against the reference's own
             scalar path and the reference's known-answer tests.
  Reference  _ref/librpgref.so, the reference's own sources compiled in place
             (see Makefile) behind ref_driver.cc.  Present wherever it was
             built; absent is reported, never faked.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "librpgref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


class OrcConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("hidden", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("intermediate", C.c_int32), ("vocab", C.c_int32),
                ("context_length", C.c_int32), ("max_pos", C.c_int32),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float)]


class OrcTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("type", C.c_uint32), ("n_dims", C.c_int32),
                ("dims", C.c_int64 * 4), ("data", C.c_void_p), ("n_bytes", C.c_int64)]


class OrcGenOpts(C.Structure):
    _fields_ = [("max_tokens", C.c_int32), ("stop_ids", C.POINTER(C.c_int32)),
                ("n_stop", C.c_int32), ("temperature", C.c_float), ("top_k", C.c_int32),
                ("top_p", C.c_float), ("seed", C.c_uint64)]


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a).view(np.uint8).reshape(-1))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class Oracle:
    """The C restatement; thread count only splits independent outputs."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        L = self.lib = C.CDLL(path)
        L.orc_f16_to_f32.argtypes, L.orc_f16_to_f32.restype = [C.c_uint16], C.c_float
        L.orc_f32_to_f16.argtypes, L.orc_f32_to_f16.restype = [C.c_float], C.c_uint16
        L.orc_row_bytes.argtypes, L.orc_row_bytes.restype = [C.c_uint32, C.c_int64], C.c_int64
        L.orc_dequantize_row.argtypes = [C.c_uint32, _u8p, C.c_int64, _f32p]
        L.orc_dot_row.argtypes, L.orc_dot_row.restype = [C.c_uint32, _f32p, _u8p, C.c_int64], C.c_float
        L.orc_dot_row_f64.argtypes = [C.c_uint32, _f32p, _u8p, C.c_int64, C.POINTER(C.c_double)]
        L.orc_dot_row_f64.restype = C.c_double
        L.orc_matmul.argtypes = [C.c_uint32, _u8p, C.c_int64, C.c_int64, _f32p, C.c_int64, _f32p]
        L.orc_argmax.argtypes, L.orc_argmax.restype = [_f32p, C.c_int64], C.c_int32
        L.orc_rmsnorm.argtypes = [_f32p, _f32p, C.c_int64, C.c_float, _f32p]
        L.orc_splitmix64.argtypes, L.orc_splitmix64.restype = [C.c_uint64], C.c_uint64
        L.orc_counter_uniform.argtypes = [C.c_uint64, C.c_uint64]
        L.orc_counter_uniform.restype = C.c_float
        L.orc_filter_to_probs.argtypes = [_f32p, C.c_int64, C.c_float, C.c_int32, C.c_float, _f32p]
        L.orc_sample_token.argtypes = [_f32p, C.c_int64, C.c_float, C.c_int32, C.c_float, C.c_float]
        L.orc_sample_token.restype = C.c_int32
        L.orc_model_create.argtypes = [C.POINTER(OrcConfig), C.POINTER(OrcTensor), C.c_int]
        L.orc_model_create.restype = C.c_void_p
        L.orc_model_free.argtypes = [C.c_void_p]
        L.orc_model_rope_positions.argtypes, L.orc_model_rope_positions.restype = [C.c_void_p], C.c_int64
        L.orc_model_rope_table.argtypes = [C.c_void_p]
        L.orc_model_rope_table.restype = C.POINTER(C.c_float)
        L.orc_kv_create.argtypes, L.orc_kv_create.restype = [C.c_void_p, C.c_int64], C.c_void_p
        L.orc_kv_free.argtypes = [C.c_void_p]
        L.orc_kv_len.argtypes, L.orc_kv_len.restype = [C.c_void_p], C.c_int64
        L.orc_kv_set_len.argtypes = [C.c_void_p, C.c_int64]
        L.orc_kv_k.argtypes, L.orc_kv_k.restype = [C.c_void_p], C.POINTER(C.c_float)
        L.orc_kv_v.argtypes, L.orc_kv_v.restype = [C.c_void_p], C.POINTER(C.c_float)
        L.orc_forward.argtypes = [C.c_void_p, C.c_void_p, _i32p, C.c_int64, _f32p, C.c_int]
        L.orc_generate.argtypes = [C.c_void_p, C.c_void_p, _f32p, C.POINTER(OrcGenOpts), _i32p,
                                   C.POINTER(C.c_int32), C.c_void_p]
        L.orc_attention_one.argtypes = [_f32p, _f32p, _f32p, C.c_int64, C.c_int32, C.c_int32,
                                        C.c_int32, C.c_int64, _f32p]
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_max_threads.restype = C.c_int

    # -- kernels ---------------------------------------------------------
    def f16_to_f32(self, h: int) -> float:
        return self.lib.orc_f16_to_f32(h)

    def f32_to_f16(self, f: float) -> int:
        return self.lib.orc_f32_to_f16(f)

    def row_bytes(self, ty: int, n: int) -> int:
        return self.lib.orc_row_bytes(ty, n)

    def dequantize_rows(self, ty: int, w, rows: int, cols: int) -> np.ndarray:
        w = _u8(w)
        out = np.empty((rows, cols), np.float32)
        if self.lib.orc_dequantize_row(ty, w, rows * cols, out.reshape(-1)) != 0:
            raise ValueError("unsupported type or size")
        return out

    def dot_row(self, ty: int, a, w) -> float:
        a = _f32(a)
        return float(self.lib.orc_dot_row(ty, a, _u8(w), a.size))

    def dot_row_f64(self, ty: int, a, w):
        a = _f32(a)
        s = C.c_double()
        v = self.lib.orc_dot_row_f64(ty, a, _u8(w), a.size, C.byref(s))
        return v, s.value

    def matmul(self, ty: int, w, rows: int, cols: int, X) -> np.ndarray:
        X = _f32(X).reshape(-1, cols)
        out = np.empty((X.shape[0], rows), np.float32)
        if self.lib.orc_matmul(ty, _u8(w), rows, cols, X, X.shape[0], out) != 0:
            raise ValueError("bad matmul arguments")
        return out

    def argmax(self, x) -> int:
        x = _f32(x)
        return int(self.lib.orc_argmax(x, x.size))

    def rmsnorm(self, x, w, eps: float) -> np.ndarray:
        x, w = _f32(x), _f32(w)
        out = np.empty_like(x)
        self.lib.orc_rmsnorm(x, w, x.size, eps, out)
        return out

    def splitmix64(self, x: int) -> int:
        return int(self.lib.orc_splitmix64(x))

    def counter_uniform(self, seed: int, counter: int) -> float:
        return float(self.lib.orc_counter_uniform(seed, counter))

    def filter_to_probs(self, logits, temperature, top_k, top_p) -> np.ndarray:
        x = _f32(logits)
        out = np.empty_like(x)
        self.lib.orc_filter_to_probs(x, x.size, temperature, top_k, top_p, out)
        return out

    def sample_token(self, logits, temperature, top_k, top_p, u) -> int:
        x = _f32(logits)
        return int(self.lib.orc_sample_token(x, x.size, temperature, top_k, top_p, u))

    def attention_one(self, q, kc, vc, pos: int, n_heads: int, n_kv: int) -> np.ndarray:
        """One query token over one layer's cache [n_kv, max_seq, hd]."""
        q, kc, vc = _f32(q).reshape(-1), _f32(kc), _f32(vc)
        hd = q.size // n_heads
        out = np.empty(q.size, np.float32)
        if self.lib.orc_attention_one(q, kc.reshape(-1), vc.reshape(-1), kc.shape[-2], n_heads,
                                      n_kv, hd, pos, out) != 0:
            raise ValueError("bad attention arguments")
        return out

    def set_threads(self, n: int):
        self.lib.orc_set_threads(n)

    def max_threads(self) -> int:
        return int(self.lib.orc_max_threads())

    # -- model -------------------------------------------------------------
    def model(self, shape, tensors, max_pos: int = 4096) -> "OracleModel":
        return OracleModel(self, shape, tensors, max_pos)


def tensor_table(tensors, struct_type=OrcTensor):
    """ctypes array over a list of gguf.Tensor (keeps the byte buffers alive)."""
    arr = (struct_type * len(tensors))()
    keep = []
    for i, t in enumerate(tensors):
        data = np.ascontiguousarray(t.data)
        keep.append(data)
        nm = t.name.encode()
        keep.append(nm)
        arr[i].name = nm
        arr[i].type = t.ggml_type
        arr[i].n_dims = len(t.dims)
        for j, d in enumerate(t.dims):
            arr[i].dims[j] = d
        arr[i].data = data.ctypes.data
        arr[i].n_bytes = data.nbytes
    return arr, keep


class OracleModel:
    def __init__(self, orc: Oracle, shape, tensors, max_pos: int):
        self.orc, self.shape = orc, shape
        cfg = OrcConfig(shape.n_layers, shape.hidden, shape.n_heads, shape.n_kv_heads,
                        shape.head_dim, shape.intermediate, shape.vocab, shape.context_length,
                        max_pos, shape.rope_theta, shape.rms_eps)
        self._tab, self._keep = tensor_table(tensors)
        self.h = orc.lib.orc_model_create(C.byref(cfg), self._tab, len(tensors))
        if not self.h:
            raise ValueError("oracle rejected the tensor table")
        self.rope_positions = orc.lib.orc_model_rope_positions(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            self.orc.lib.orc_model_free(self.h)
            self.h = None

    def rope_table(self) -> np.ndarray:
        n = self.rope_positions * self.shape.head_dim
        p = self.orc.lib.orc_model_rope_table(self.h)
        return np.ctypeslib.as_array(p, shape=(n,)).copy().reshape(self.rope_positions, -1)

    def kv(self, max_seq: int) -> "OracleKv":
        return OracleKv(self, max_seq)

    def forward(self, ids, kv=None, all_rows: bool = False) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        rows = ids.size if all_rows else 1
        out = np.empty((rows, self.shape.vocab), np.float32)
        rc = self.orc.lib.orc_forward(self.h, kv.h if kv else None, ids, ids.size, out,
                                      1 if all_rows else 0)
        if rc != 0:
            raise ValueError("oracle forward rejected its arguments")
        return out

    def generate(self, kv, first_logits, max_tokens, stop_ids=(), temperature=0.0, top_k=0,
                 top_p=1.0, seed=0, want_logits=False):
        stop = (C.c_int32 * max(1, len(stop_ids)))(*stop_ids)
        o = OrcGenOpts(max_tokens, stop, len(stop_ids), temperature, top_k, top_p, seed)
        out = np.zeros(max_tokens, np.int32)
        n = C.c_int32()
        lg = np.zeros((max_tokens, self.shape.vocab), np.float32) if want_logits else None
        rc = self.orc.lib.orc_generate(self.h, kv.h, _f32(first_logits), C.byref(o), out,
                                       C.byref(n), lg.ctypes.data if want_logits else None)
        if rc == -1:
            raise ValueError("oracle generate rejected its arguments")
        toks = out[: n.value].copy()
        if rc == -2:
            raise OverflowError(f"context full after {n.value} tokens")
        return (toks, lg[: n.value]) if want_logits else toks


class OracleKv:
    def __init__(self, m: OracleModel, max_seq: int):
        self.m, self.max_seq = m, max_seq
        self.h = m.orc.lib.orc_kv_create(m.h, max_seq)
        if not self.h:
            raise MemoryError("oracle kv allocation failed")

    def __del__(self):
        if getattr(self, "h", None):
            self.m.orc.lib.orc_kv_free(self.h)
            self.h = None

    @property
    def len(self) -> int:
        return int(self.m.orc.lib.orc_kv_len(self.h))

    def set_len(self, n: int):
        if self.m.orc.lib.orc_kv_set_len(self.h, n) != 0:
            raise ValueError("kv length out of range")

    def arrays(self):
        s = self.m.shape
        shp = (s.n_layers, s.n_kv_heads, self.max_seq, s.head_dim)
        n = int(np.prod(shp))
        k = np.ctypeslib.as_array(self.m.orc.lib.orc_kv_k(self.h), shape=(n,)).reshape(shp)
        v = np.ctypeslib.as_array(self.m.orc.lib.orc_kv_v(self.h), shape=(n,)).reshape(shp)
        return k.copy(), v.copy()


class OracleEngineSession:
    """The reference's per-turn session logic (src/engine.cc:383-487) replayed
    over the oracle's forward and generate, on token ids: the checker for the
    library's token-level engine (rpgc_engine_generate).

    Cached ids and the LCP (src/engine.cc:383-397), options from the request
    else the session (:399-411), the capacity check before the cache is
    touched (:412-419), the cache cut to the prefix and the rest forwarded,
    reset on a failed forward (:421-448), stop ids eos / <|im_end|> / request /
    session (:451-456), top_k 0 and top_p 0.95 (:463-467), the finish reason
    by tokens (:477-487)."""

    DEFAULT_MAX_TOKENS, SEQ_MARGIN, TOP_K, TOP_P, MAX_T = 256, 4, 0, 0.95, 2.0

    def __init__(self, m: OracleModel, max_seq: int, max_tokens: int = 0, temperature: float = 0.0,
                 seed: int = 0, stop_ids=(), eos_id: int = -1, im_end_id: int = -1):
        self.m, self.max_seq = m, max_seq
        self.kv = m.kv(max_seq)
        self.cached = []
        mt = max_tokens or self.DEFAULT_MAX_TOKENS
        self.max_tokens = min(mt, max_seq - 1)
        self.temperature = self._clamp(temperature)
        self.seed = seed
        self.stop = list(stop_ids)
        self.eos_id, self.im_end_id = eos_id, im_end_id

    @classmethod
    def _clamp(cls, t):
        return 0.0 if not t > 0 else min(t, cls.MAX_T)

    def reset(self):
        self.kv.set_len(0)
        self.cached = []

    def generate(self, ids, max_tokens=0, temperature=None, seed=None, stop_ids=()):
        ids = [int(i) for i in ids]
        n = len(ids)
        if n == 0:
            raise ValueError("the prompt is empty")
        assert len(self.cached) == self.kv.len
        lcp = 0
        while lcp < len(self.cached) and lcp < n and self.cached[lcp] == ids[lcp]:
            lcp += 1
        if lcp == n:
            lcp = n - 1
        mt = max_tokens if max_tokens > 0 else self.max_tokens
        t = self._clamp(self.temperature if temperature is None else temperature)
        sd = self.seed if seed is None else seed
        stop = []
        for i in [self.eos_id, self.im_end_id] + list(stop_ids) + self.stop:
            if i >= 0 and i not in stop:
                stop.append(int(i))
        if n + mt + self.SEQ_MARGIN > self.max_seq:
            raise OverflowError("sequence too long")
        if any(i < 0 or i >= self.m.shape.vocab for i in ids):
            self.reset()  # the forward fails: the cache is not reused
            raise ValueError("prompt id outside the vocabulary")
        self.kv.set_len(lcp)
        first = self.m.forward(np.asarray(ids[lcp:], np.int32), self.kv)[0]
        self.cached = list(ids)
        gen = [int(x) for x in self.m.generate(self.kv, first, mt, stop_ids=stop, temperature=t,
                                               top_k=self.TOP_K, top_p=self.TOP_P, seed=sd)]
        self.cached += gen
        stopped = bool(gen) and gen[-1] in stop
        finish = "length" if len(gen) >= mt and not stopped else "stop"
        return gen, finish, n, lcp


class Reference:
    """The reference's own code (oracle/_ref/librpgref.so), when built.

    The reference picks its matmul backend once at load time from
    RPGBAR_NO_SIMD, so the scalar and AVX2 paths need separate processes."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref` where the "
                                    "reference sources exist")
        L = self.lib = C.CDLL(path)
        L.refd_last_error.restype = C.c_char_p
        L.refd_active_kernel.restype = C.c_char_p
        L.refd_f16_to_f32.argtypes, L.refd_f16_to_f32.restype = [C.c_uint16], C.c_float
        L.refd_f32_to_f16.argtypes, L.refd_f32_to_f16.restype = [C.c_float], C.c_uint16
        L.refd_dequantize_row.argtypes = [C.c_uint32, _u8p, C.c_int64, _f32p]
        for fn in (L.refd_dot_row, L.refd_dot_row_ref):
            fn.argtypes = [C.c_uint32, _f32p, _u8p, C.c_int64, C.POINTER(C.c_float)]
        L.refd_matmul.argtypes = [C.c_uint32, _u8p, C.c_int64, C.c_int64, _f32p, C.c_int64,
                                  _f32p, C.c_int]
        L.refd_counter_uniform.argtypes = [C.c_uint64, C.c_uint64]
        L.refd_counter_uniform.restype = C.c_float
        L.refd_splitmix64.argtypes, L.refd_splitmix64.restype = [C.c_uint64], C.c_uint64
        L.refd_filter_to_probs.argtypes = [_f32p, C.c_int64, C.c_float, C.c_int32, C.c_float, _f32p]
        L.refd_sample_token.argtypes = [_f32p, C.c_int64, C.c_float, C.c_int32, C.c_float, C.c_float]
        L.refd_sample_token.restype = C.c_int32
        L.refd_model_load.argtypes = [C.c_char_p, C.c_int, C.c_int32]
        L.refd_model_load.restype = C.c_void_p
        L.refd_model_free.argtypes = [C.c_void_p]
        L.refd_model_config.argtypes = [C.c_void_p, C.POINTER(C.c_int64)]
        L.refd_model_rope.argtypes = [C.c_void_p, _f32p, C.c_int64]
        L.refd_kv_create.argtypes, L.refd_kv_create.restype = [C.c_void_p, C.c_int64], C.c_void_p
        L.refd_kv_free.argtypes = [C.c_void_p]
        L.refd_kv_len.argtypes, L.refd_kv_len.restype = [C.c_void_p], C.c_int64
        L.refd_kv_set_len.argtypes = [C.c_void_p, C.c_int64]
        L.refd_forward.argtypes = [C.c_void_p, C.c_void_p, _i32p, C.c_int64, _f32p]
        L.refd_generate.argtypes = [C.c_void_p, C.c_void_p, _f32p, C.c_int32, _i32p, C.c_int32,
                                    C.c_float, C.c_int32, C.c_float, C.c_uint64, _i32p,
                                    C.POINTER(C.c_int32)]

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(self.lib.refd_last_error().decode("utf-8", "replace"))

    @property
    def kernel(self) -> str:
        return self.lib.refd_active_kernel().decode()

    def dequantize_rows(self, ty, w, rows, cols):
        out = np.empty((rows, cols), np.float32)
        self._check(self.lib.refd_dequantize_row(ty, _u8(w), rows * cols, out.reshape(-1)))
        return out

    def dot_row(self, ty, a, w, scalar=False):
        a = _f32(a)
        out = C.c_float()
        fn = self.lib.refd_dot_row_ref if scalar else self.lib.refd_dot_row
        self._check(fn(ty, a, _u8(w), a.size, C.byref(out)))
        return float(out.value)

    def matmul(self, ty, w, rows, cols, X, threads=0):
        X = _f32(X).reshape(-1, cols)
        out = np.empty((X.shape[0], rows), np.float32)
        self._check(self.lib.refd_matmul(ty, _u8(w), rows, cols, X, X.shape[0], out, threads))
        return out

    def counter_uniform(self, seed, counter):
        return float(self.lib.refd_counter_uniform(seed, counter))

    def filter_to_probs(self, logits, temperature, top_k, top_p):
        x = _f32(logits)
        out = np.empty_like(x)
        self._check(self.lib.refd_filter_to_probs(x, x.size, temperature, top_k, top_p, out))
        return out

    def sample_token(self, logits, temperature, top_k, top_p, u):
        x = _f32(logits)
        return int(self.lib.refd_sample_token(x, x.size, temperature, top_k, top_p, u))

    def load(self, path: str, threads: int = 0, max_pos: int = 4096) -> "RefModel":
        h = self.lib.refd_model_load(path.encode(), threads, max_pos)
        if not h:
            raise RuntimeError(self.lib.refd_last_error().decode("utf-8", "replace"))
        return RefModel(self, h)


class RefModel:
    def __init__(self, ref: Reference, h):
        self.ref, self.h = ref, h
        cfg = (C.c_int64 * 10)()
        ref.lib.refd_model_config(h, cfg)
        (self.n_layers, self.hidden, self.n_heads, self.n_kv_heads, self.head_dim,
         self.intermediate, self.vocab, self.context_length, self.rope_positions,
         self.tied) = list(cfg)

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.refd_model_free(self.h)
            self.h = None

    def rope_table(self):
        out = np.empty(self.rope_positions * self.head_dim, np.float32)
        self.ref._check(self.ref.lib.refd_model_rope(self.h, out, out.size))
        return out.reshape(self.rope_positions, -1)

    def kv(self, max_seq):
        h = self.ref.lib.refd_kv_create(self.h, max_seq)
        if not h:
            raise RuntimeError(self.ref.lib.refd_last_error().decode("utf-8", "replace"))
        return RefKv(self.ref, h)

    def forward(self, ids, kv=None):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty((ids.size, self.vocab), np.float32)
        self.ref._check(self.ref.lib.refd_forward(self.h, kv.h if kv else None, ids, ids.size,
                                                  out))
        return out

    def generate(self, kv, first_logits, max_tokens, stop_ids=(), temperature=0.0, top_k=0,
                 top_p=1.0, seed=0):
        stop = np.asarray(list(stop_ids) or [-1], np.int32)
        out = np.zeros(max_tokens, np.int32)
        n = C.c_int32()
        self.ref._check(self.ref.lib.refd_generate(self.h, kv.h, _f32(first_logits), max_tokens,
                                                   stop, len(stop_ids), temperature, top_k,
                                                   top_p, seed, out, C.byref(n)))
        return out[: n.value].copy()


class RefKv:
    def __init__(self, ref, h):
        self.ref, self.h = ref, h

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.refd_kv_free(self.h)
            self.h = None

    @property
    def len(self):
        return int(self.ref.lib.refd_kv_len(self.h))

    def set_len(self, n):
        self.ref._check(self.ref.lib.refd_kv_set_len(self.h, n))


def reference_available() -> bool:
    return os.path.exists(REF_SO)
