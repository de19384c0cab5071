"""rpgbarengine_b200 -- B200 (sm_100a) token loop behind a C ABI.

Python host mirror of the reference's token-level interface:

  Model / Model.load_gguf      Model::Load               (src/model.cc:147-281)
  Session                      KvCache + ForwardScratch  (src/kv_cache.h, src/qwen3.h:38-59)
  Session.forward_full         ForwardFull/ForwardStep   (src/qwen3.cc:208-300)
  Session.generate             Generate                  (src/qwen3.cc:302-355)
  dequantize_rows              DequantizeRow             (src/quant.h:65)
  matvec / matmul_batch        MatVec / MatMulBatch      (src/model.cc:23-69)
  sample_token                 SampleToken / ArgMax      (src/sampler.cc:96-112)

Every call goes through librpgc.so (include/rpgc.h).  There is no CPU
fallback: without the built library, or without a CUDA device, calls fail.
Errors raise RpgcError carrying the C status code and rpgc_last_error().
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import gguf as _gguf

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librpgc.so")

OK, E_ARG, E_CUDA, E_OOM, E_STATE, E_CONTEXT_FULL, E_TIMEOUT, E_IO = 0, -1, -2, -3, -4, -5, -6, -7
F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
MAX_STOP = 16


class RpgcError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[rpgc {code}] {msg}")
        self.code = code


class ContextFull(RpgcError):
    pass


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("type", C.c_uint32), ("n_dims", C.c_int32),
                ("dims", C.c_int64 * 4), ("data", C.c_void_p), ("n_bytes", C.c_int64)]


class ModelConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("hidden", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("intermediate", C.c_int32), ("vocab", C.c_int32),
                ("context_length", C.c_int32), ("max_pos", C.c_int32),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float)]


class TpShard(C.Structure):
    """rpgc_tp_shard: one rank's head counts and row / column ranges."""
    _fields_ = [("n_heads", C.c_int32), ("n_kv_heads", C.c_int32), ("intermediate", C.c_int32),
                ("q_rows", C.c_int64 * 2), ("kv_rows", C.c_int64 * 2), ("ffn_rows", C.c_int64 * 2),
                ("vocab_rows", C.c_int64 * 2), ("o_cols", C.c_int64 * 2), ("down_cols", C.c_int64 * 2)]


class GenOpts(C.Structure):
    _fields_ = [("max_tokens", C.c_int32), ("stop_ids", C.POINTER(C.c_int32)),
                ("n_stop", C.c_int32), ("temperature", C.c_float), ("top_k", C.c_int32),
                ("top_p", C.c_float), ("seed", C.c_uint64)]


class EngineSessionOpts(C.Structure):
    _fields_ = [("max_seq", C.c_int32), ("max_tokens", C.c_int32), ("temperature", C.c_float),
                ("seed", C.c_uint64), ("stop_ids", C.POINTER(C.c_int32)), ("n_stop", C.c_int32)]


class EngineRequest(C.Structure):
    _fields_ = [("max_tokens", C.c_int32), ("set_temperature", C.c_int32), ("temperature", C.c_float),
                ("set_seed", C.c_int32), ("seed", C.c_uint64), ("stop_ids", C.POINTER(C.c_int32)),
                ("n_stop", C.c_int32)]


class EngineResult(C.Structure):
    _fields_ = [("n_out", C.c_int32), ("finish", C.c_int32), ("prompt_tokens", C.c_int64),
                ("reused", C.c_int64)]


FINISH = {0: "stop", 1: "length"}

_lib = None


def lib() -> C.CDLL:
    """Load librpgc.so once; raise if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RpgcError(E_STATE, f"{LIB_PATH} not built: run `python -m rpgbarengine_b200.build`")
    L = C.CDLL(LIB_PATH)
    vp, i32, i64, u32, f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint32, C.c_float
    sig = {
        "rpgc_version": ([], C.c_char_p),
        "rpgc_kernel_launches": ([], C.c_int64),
        "rpgc_last_error": ([], C.c_char_p),
        "rpgc_device_count": ([], C.c_int),
        "rpgc_model_upload": ([C.c_int, C.POINTER(ModelConfig), C.POINTER(Tensor), i32], i32),
        "rpgc_tp_id": ([C.c_void_p, C.c_int64], C.c_int),
        "rpgc_tp_shard_of": ([C.POINTER(ModelConfig), i32, i32, C.POINTER(TpShard)], C.c_int),
        "rpgc_model_upload_tp": ([C.c_int, C.POINTER(ModelConfig), C.POINTER(Tensor), i32, i32, i32,
                                  C.c_void_p], i32),
        "rpgc_model_load_gguf": ([C.c_int, C.c_char_p, i32], i32),
        "rpgc_model_get_config": ([i32, C.POINTER(ModelConfig)], C.c_int),
        "rpgc_model_weight_bytes": ([i32], i64),
        "rpgc_model_free": ([i32], C.c_int),
        "rpgc_session_create": ([i32, i32], i32),
        "rpgc_session_destroy": ([i32], C.c_int),
        "rpgc_session_len": ([i32], i64),
        "rpgc_session_set_len": ([i32, i64], C.c_int),
        "rpgc_session_stream": ([i32], vp),
        "rpgc_session_read_kv": ([i32, vp, vp], C.c_int),
        "rpgc_forward": ([i32, vp, i64, vp, vp], C.c_int),
        "rpgc_generate": ([i32, C.POINTER(GenOpts), vp, C.POINTER(i32)], C.c_int),
        "rpgc_forward_device": ([i32, vp, i64], C.c_int),
        "rpgc_session_copy_prefix": ([i32, i32, i64], C.c_int),
        "rpgc_generate_batch": ([vp, i32, C.POINTER(GenOpts), vp, vp], C.c_int),
        "rpgc_model_set_batching": ([i32, i32, i32], C.c_int),
        "rpgc_model_batching_stats": ([i32, C.POINTER(C.c_int64), C.POINTER(C.c_int64)], C.c_int),
        "rpgc_generate_device": ([i32, C.POINTER(GenOpts), vp, vp], C.c_int),
        "rpgc_session_sync": ([i32], C.c_int),
        "rpgc_test_stall_next_batch": ([i32], C.c_int),
        "rpgc_engine_session_create": ([i32, C.POINTER(EngineSessionOpts)], i32),
        "rpgc_engine_session_destroy": ([i32], C.c_int),
        "rpgc_engine_session_reset": ([i32], C.c_int),
        "rpgc_engine_session_cached": ([i32, vp, i64], i64),
        "rpgc_engine_generate": ([i32, vp, i64, C.POINTER(EngineRequest), vp, i32,
                                  C.POINTER(EngineResult)], C.c_int),
        "rpgc_model_set_special_ids": ([i32, i32, i32], C.c_int),
        "rpgc_model_special_ids": ([i32, C.POINTER(i32), C.POINTER(i32)], C.c_int),
        "rpgc_dequantize_rows": ([u32, vp, i64, i64, vp, vp], C.c_int),
        "rpgc_matvec": ([u32, vp, i64, i64, vp, vp, vp], C.c_int),
        "rpgc_matmul": ([u32, vp, i64, i64, vp, i64, vp, vp], C.c_int),
        "rpgc_sample": ([vp, i64, f32, i32, f32, f32, vp, vp], C.c_int),
        "rpgc_attention_decode": ([vp, vp, vp, i64, i32, i32, i32, i64, vp, vp], C.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes, fn.restype = args, res
    _lib = L
    return L


def exported_symbols() -> list:
    return [n for n in ("rpgc_version", "rpgc_last_error", "rpgc_device_count") if hasattr(lib(), n)]


def _check(rc: int):
    if rc < 0:
        msg = lib().rpgc_last_error().decode("utf-8", "replace")
        raise (ContextFull if rc == E_CONTEXT_FULL else RpgcError)(rc, msg)
    return rc


def version() -> str:
    return lib().rpgc_version().decode()


def device_count() -> int:
    return int(lib().rpgc_device_count())


def tensor_table(tensors):
    """ctypes rpgc_tensor[] over gguf.Tensor objects (buffers kept alive)."""
    arr = (Tensor * len(tensors))()
    keep = []
    for i, t in enumerate(tensors):
        data = np.ascontiguousarray(t.data)
        nm = t.name.encode()
        keep += [data, nm]
        arr[i].name, arr[i].type, arr[i].n_dims = nm, t.ggml_type, len(t.dims)
        for j, d in enumerate(t.dims):
            arr[i].dims[j] = d
        arr[i].data, arr[i].n_bytes = data.ctypes.data, data.nbytes
    return arr, keep


class Model:
    """Weights resident in HBM as raw ggml blocks (one device)."""

    def __init__(self, handle: int):
        self.handle = handle
        c = ModelConfig()
        _check(lib().rpgc_model_get_config(handle, C.byref(c)))
        self.config = c
        self.vocab = c.vocab

    @classmethod
    def upload(cls, shape, tensors, device: int = 0, max_pos: int = 4096) -> "Model":
        cfg = ModelConfig(shape.n_layers, shape.hidden, shape.n_heads, shape.n_kv_heads,
                          shape.head_dim, shape.intermediate, shape.vocab, shape.context_length,
                          max_pos, shape.rope_theta, shape.rms_eps)
        tab, keep = tensor_table(tensors)
        h = _check(lib().rpgc_model_upload(device, C.byref(cfg), tab, len(tensors)))
        del keep
        return cls(h)

    @classmethod
    def upload_tp(cls, shape, tensors, device: int, rank: int, world: int, nccl_id: bytes,
                  max_pos: int = 4096) -> "Model":
        """Rank `rank` of a `world`-way tensor-parallel model (rpgc_model_upload_tp):
        every rank passes the whole tensor table and the same NCCL id."""
        cfg = ModelConfig(shape.n_layers, shape.hidden, shape.n_heads, shape.n_kv_heads,
                          shape.head_dim, shape.intermediate, shape.vocab, shape.context_length,
                          max_pos, shape.rope_theta, shape.rms_eps)
        tab, keep = tensor_table(tensors)
        idbuf = C.create_string_buffer(bytes(nccl_id), len(nccl_id))
        h = _check(lib().rpgc_model_upload_tp(device, C.byref(cfg), tab, len(tensors), rank, world,
                                              C.cast(idbuf, C.c_void_p)))
        del keep
        return cls(h)

    @classmethod
    def load_gguf(cls, path: str, device: int = 0, max_pos: int = 4096) -> "Model":
        return cls(_check(lib().rpgc_model_load_gguf(device, path.encode(), max_pos)))

    @property
    def weight_bytes(self) -> int:
        return int(_check(lib().rpgc_model_weight_bytes(self.handle)))

    def set_batching(self, max_batch: int, window_us: int = 2000):
        """rpgc_model_set_batching: gather concurrent generate calls on this
        model's sessions (from different threads) into batched decodes of up
        to max_batch sessions; 0 or 1 turns it off."""
        _check(lib().rpgc_model_set_batching(self.handle, max_batch, window_us))

    def batching_stats(self):
        """(batches of two or more sessions run, generate calls they served)."""
        b, r = C.c_int64(0), C.c_int64(0)
        _check(lib().rpgc_model_batching_stats(self.handle, C.byref(b), C.byref(r)))
        return b.value, r.value

    def session(self, max_seq: int) -> "Session":
        return Session(self, max_seq)

    def set_special_ids(self, eos_id: int, im_end_id: int):
        """The model-level stop ids of the token-level engine (-1: none)."""
        _check(lib().rpgc_model_set_special_ids(self.handle, eos_id, im_end_id))

    @property
    def special_ids(self):
        e, i = C.c_int32(-1), C.c_int32(-1)
        _check(lib().rpgc_model_special_ids(self.handle, C.byref(e), C.byref(i)))
        return e.value, i.value

    def engine_session(self, **kw) -> "EngineSession":
        return EngineSession(self, **kw)

    def free(self):
        if self.handle:
            lib().rpgc_model_free(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Session:
    """One inference context: device KV cache + stream (src/kv_cache.h:35-82)."""

    def __init__(self, model: Model, max_seq: int):
        self.model = model
        self.max_seq = max_seq
        self.handle = _check(lib().rpgc_session_create(model.handle, max_seq))

    @property
    def len(self) -> int:
        return int(_check(lib().rpgc_session_len(self.handle)))

    def set_len(self, n: int):
        _check(lib().rpgc_session_set_len(self.handle, n))

    def reset(self):
        self.set_len(0)

    def copy_prefix_from(self, src: "Session", n: int):
        """KV positions [0, n) of `src` copied into this session on the device
        (rpgc_session_copy_prefix); a forward of the remaining tokens follows."""
        _check(lib().rpgc_session_copy_prefix(self.handle, src.handle, n))

    @property
    def stream_ptr(self) -> int:
        return int(lib().rpgc_session_stream(self.handle) or 0)

    def forward_full(self, ids, all_rows: bool = False):
        """Append ids; returns the last-row logits, or all rows if asked."""
        ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
        V = self.model.vocab
        last = np.empty(V, np.float32)
        allr = np.empty((ids.size, V), np.float32) if all_rows else None
        _check(lib().rpgc_forward(self.handle, ids.ctypes.data, ids.size, last.ctypes.data,
                                  allr.ctypes.data if all_rows else None))
        return allr if all_rows else last

    forward = forward_full

    def generate(self, max_tokens: int, stop_ids=(), temperature: float = 0.0, top_k: int = 0,
                 top_p: float = 1.0, seed: int = 0) -> np.ndarray:
        stop = (C.c_int32 * max(1, len(stop_ids)))(*stop_ids)
        o = GenOpts(max_tokens, stop, len(stop_ids), temperature, top_k, top_p, seed)
        out = np.zeros(max_tokens, np.int32)
        n = C.c_int32(0)
        rc = lib().rpgc_generate(self.handle, C.byref(o), out.ctypes.data, C.byref(n))
        if rc < 0:
            _check(rc)
        return out[: n.value].copy()

    def forward_device(self, ids_dev_ptr: int, n: int):
        _check(lib().rpgc_forward_device(self.handle, ids_dev_ptr, n))

    def generate_device(self, max_tokens: int, out_dev_ptr: int, n_out_dev_ptr: int,
                        temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                        seed: int = 0):
        o = GenOpts(max_tokens, None, 0, temperature, top_k, top_p, seed)
        _check(lib().rpgc_generate_device(self.handle, C.byref(o), out_dev_ptr, n_out_dev_ptr))

    def sync(self):
        _check(lib().rpgc_session_sync(self.handle))

    def read_kv(self):
        c = self.model.config
        shp = (c.n_layers, c.n_kv_heads, self.max_seq, c.head_dim)
        k = np.empty(shp, np.float32)
        v = np.empty(shp, np.float32)
        _check(lib().rpgc_session_read_kv(self.handle, k.ctypes.data, v.ctypes.data))
        return k, v

    def close(self):
        if self.handle:
            lib().rpgc_session_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# -------------------------------------------------------------- kernel calls
def _ptr(t) -> int:
    return int(t.data_ptr())


def _stream(stream) -> int:
    if stream is None:
        import torch
        return int(torch.cuda.current_stream().cuda_stream)
    return int(stream)


def generate_batch(sessions, max_tokens: int, stop_ids=(), temperature: float = 0.0, top_k: int = 0,
                   top_p: float = 1.0, seed: int = 0) -> list:
    """rpgc_generate_batch: max_tokens steps decoding one token for every
    session at once; returns one array of generated ids per session."""
    n = len(sessions)
    handles = (C.c_int32 * n)(*[s.handle for s in sessions])
    stop = (C.c_int32 * max(1, len(stop_ids)))(*stop_ids)
    o = GenOpts(max_tokens, stop, len(stop_ids), temperature, top_k, top_p, seed)
    out = np.zeros((n, max_tokens), np.int32)
    n_out = np.zeros(n, np.int32)
    _check(lib().rpgc_generate_batch(C.cast(handles, C.c_void_p), n, C.byref(o), out.ctypes.data,
                                     n_out.ctypes.data))
    return [out[i, : n_out[i]].copy() for i in range(n)]


def tp_shard(shape, rank: int, world: int) -> dict:
    """Rank `rank`'s shard of a `world`-way tensor-parallel model of `shape`
    (rpgc_tp_shard_of, the ranges rpgc_model_upload_tp uploads): head counts
    and [begin, end) row / column ranges per matrix kind.  Needs no device."""
    cfg = ModelConfig(shape.n_layers, shape.hidden, shape.n_heads, shape.n_kv_heads, shape.head_dim,
                      shape.intermediate, shape.vocab, shape.context_length, shape.context_length,
                      shape.rope_theta, shape.rms_eps)
    out = TpShard()
    _check(lib().rpgc_tp_shard_of(C.byref(cfg), rank, world, C.byref(out)))
    d = {k: getattr(out, k) for k in ("n_heads", "n_kv_heads", "intermediate")}
    for k in ("q_rows", "kv_rows", "ffn_rows", "vocab_rows", "o_cols", "down_cols"):
        d[k] = (int(getattr(out, k)[0]), int(getattr(out, k)[1]))
    return d


def tp_unique_id() -> bytes:
    """A new 128-byte NCCL unique id for rpgc_model_upload_tp (one rank makes
    it and shares it with the others)."""
    buf = C.create_string_buffer(128)
    _check(lib().rpgc_tp_id(C.cast(buf, C.c_void_p), 128))
    return buf.raw


def kernel_launches() -> int:
    """Kernels the library has enqueued so far (graph replays count their kernels)."""
    return int(lib().rpgc_kernel_launches())


def dequantize_rows(ggml_type: int, w, rows: int, cols: int, out=None, stream=None):
    """w: uint8 CUDA tensor of raw blocks -> float32 [rows, cols] (bit-exact)."""
    import torch
    out = out if out is not None else torch.empty((rows, cols), dtype=torch.float32, device=w.device)
    _check(lib().rpgc_dequantize_rows(ggml_type, _ptr(w), rows, cols, _ptr(out), _stream(stream)))
    return out


def matvec(ggml_type: int, w, rows: int, cols: int, x, out=None, stream=None):
    import torch
    out = out if out is not None else torch.empty(rows, dtype=torch.float32, device=x.device)
    _check(lib().rpgc_matvec(ggml_type, _ptr(w), rows, cols, _ptr(x), _ptr(out), _stream(stream)))
    return out


def matmul_batch(ggml_type: int, w, rows: int, cols: int, X, out=None, stream=None):
    """OUT[t, r] = dot(X[t], W[r]); X float32 [n, cols] on the device."""
    import torch
    n = X.shape[0]
    out = out if out is not None else torch.empty((n, rows), dtype=torch.float32, device=X.device)
    _check(lib().rpgc_matmul(ggml_type, _ptr(w), rows, cols, _ptr(X), n, _ptr(out), _stream(stream)))
    return out


def sample_token(logits, temperature: float, top_k: int, top_p: float, u: float, stream=None) -> int:
    import torch
    tok = torch.empty(1, dtype=torch.int32, device=logits.device)
    _check(lib().rpgc_sample(_ptr(logits), logits.numel(), temperature, top_k, top_p, u, _ptr(tok),
                             _stream(stream)))
    return int(tok.item())


def attention_decode(q, k_cache, v_cache, pos: int, n_heads: int, n_kv_heads: int,
                     out=None, stream=None):
    """Attention of one query token over cache positions [0, pos]
    (AttentionFromCache, src/qwen3.cc:79-117).  q: [n_heads*128] float32;
    caches: [n_kv_heads, max_seq, 128] float32, all on the device."""
    import torch
    out = out if out is not None else torch.empty_like(q)
    max_seq = k_cache.shape[-2]
    _check(lib().rpgc_attention_decode(_ptr(q), _ptr(k_cache), _ptr(v_cache), max_seq, n_heads,
                                       n_kv_heads, 128, pos, _ptr(out), _stream(stream)))
    return out


row_bytes = _gguf.row_bytes


def _ids_array(ids):
    a = (C.c_int32 * max(1, len(ids)))(*[int(i) for i in ids])
    return a, len(ids)


class EngineSession:
    """Token-level engine session (rpgc_engine_*): the reference's
    rpg_engine_session_* / rpg_engine_generate (src/engine.cc:259-515) with
    prompts and completions as token ids; the host keeps the text side."""

    def __init__(self, model: Model, max_seq: int = 0, max_tokens: int = 0, temperature: float = 0.0,
                 seed: int = 0, stop_ids=()):
        self.model = model
        self._stop = _ids_array(stop_ids)
        o = EngineSessionOpts(max_seq, max_tokens, temperature, seed, self._stop[0], self._stop[1])
        self.handle = _check(lib().rpgc_engine_session_create(model.handle, C.byref(o)))

    def generate(self, ids, max_tokens: int = 0, temperature=None, seed=None, stop_ids=(), out_cap=None):
        """One turn: ids = the whole prompt so far.  Returns (completion ids,
        finish "stop"/"length", prompt_tokens, reused prefix length)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
        stop = _ids_array(stop_ids)
        req = EngineRequest(max_tokens, temperature is not None, temperature or 0.0, seed is not None,
                            seed or 0, stop[0], stop[1])
        cap = out_cap if out_cap is not None else max(max_tokens, 1 << 16)
        out = np.zeros(max(1, cap), np.int32)
        res = EngineResult()
        _check(lib().rpgc_engine_generate(self.handle, ids.ctypes.data, ids.size, C.byref(req),
                                          out.ctypes.data, cap, C.byref(res)))
        return out[: res.n_out].copy(), FINISH[res.finish], int(res.prompt_tokens), int(res.reused)

    def reset(self):
        _check(lib().rpgc_engine_session_reset(self.handle))

    def cached(self) -> np.ndarray:
        n = _check(lib().rpgc_engine_session_cached(self.handle, None, 0))
        out = np.zeros(max(1, n), np.int32)
        _check(lib().rpgc_engine_session_cached(self.handle, out.ctypes.data, n))
        return out[:n]

    def close(self):
        if self.handle:
            lib().rpgc_engine_session_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
