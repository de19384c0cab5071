"""Shared helpers for the GPU parity tests (checked against the oracle)."""
import numpy as np

from rpgbarengine_b200 import gguf

# north_star gates
ROW_GATE = 1e-5      # per-row matmul error: max|d| / sum|a*w|
LOGIT_REL_L2 = 1e-3  # final logits, relative L2
MARGIN = 1e-2        # greedy tokens must agree where the top-2 margin exceeds this


def row_gate(orc, ty, w, rows, cols, X, out, row_idx=None):
    """max over (t, r) of |out - exact| / sum_k |a_k w_k|, exact in float64 from the
    oracle's bit-exact dequantised weights."""
    rb = gguf.row_bytes(ty, cols)
    if row_idx is None:
        row_idx = np.arange(rows)
    wr = np.ascontiguousarray(w.reshape(rows, rb)[row_idx])
    W = orc.dequantize_rows(ty, wr, len(row_idx), cols).astype(np.float64)
    Xd = np.asarray(X, np.float64).reshape(-1, cols)
    exact = Xd @ W.T
    den = np.abs(Xd) @ np.abs(W).T
    got = np.asarray(out, np.float64).reshape(Xd.shape[0], rows)[:, row_idx]
    return float((np.abs(got - exact) / np.maximum(den, 1e-30)).max())


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def top2_margin(logits):
    s = np.sort(np.asarray(logits, np.float64))
    return float(s[-1] - s[-2])


def compare_tokens(got, ref, ref_logits, margin=MARGIN):
    """Tokens must match up to the first position where the reference's top-2
    margin is below `margin` (after that the sequences may legitimately split)."""
    n = min(len(got), len(ref))
    for i in range(n):
        if top2_margin(ref_logits[i]) <= margin:
            return i  # compared up to here
        assert got[i] == ref[i], f"token {i}: got {got[i]} want {ref[i]}"
    assert len(got) == len(ref), (len(got), len(ref))
    return n
