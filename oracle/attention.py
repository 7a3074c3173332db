"""CPU oracle for the forward attention path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module,
and only as the checker / the timed CPU baseline; the product (fa.forward) never calls it.

A numpy restatement of the reference's ground truth ``attention_reference``
(fa/reference.py:8-18 of aligoldenhat/flash-attention-from-scratch):
  1. upcast q, k, v (fp16) to fp32                        fa/reference.py:12
  2. scores = q k^T * (1 / sqrt(d))                        fa/reference.py:13
  3. causal: entries strictly above the diagonal -> -inf  fa/reference.py:14-17
  4. softmax over keys, then @ v                          fa/reference.py:18
The output is fp32. Parity is pinned: tests/golden/ holds input/output vectors produced by the
reference's own attention_reference (tests/golden/make_golden.py), and tests/test_oracle.py
checks this module against them.

Extension over the reference oracle: an explicit ``softmax_scale`` (the reference tests a
custom scale through the identity ref(q * scale * sqrt(d)), tests/test_flash_fwd.py:97-103).
"""

from __future__ import annotations

import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np


def _attention_heads(q32: np.ndarray, k32: np.ndarray, v32: np.ndarray, causal: bool, scale: np.float32) -> np.ndarray:
    """q32, k32, v32: [h, N, d] float32 -> [h, N, d] float32."""
    s = np.matmul(q32, np.swapaxes(k32, -1, -2))
    s *= scale
    if causal:
        n = s.shape[-1]
        s[:, np.triu(np.ones((n, n), dtype=bool), k=1)] = -np.inf
    s -= s.max(axis=-1, keepdims=True)
    np.exp(s, out=s)
    s /= s.sum(axis=-1, keepdims=True)
    return np.matmul(s, v32)


def attention(
    q,
    k,
    v,
    causal: bool = False,
    softmax_scale: float | None = None,
    threads: int | None = None,
    max_chunk_bytes: int = 1 << 30,
) -> np.ndarray:
    """softmax(q k^T * scale) v in fp32 for [..., N, d] inputs (fp16 or castable).

    The N x N score matrix is materialised per chunk of heads (bounded by max_chunk_bytes);
    chunks run on a thread pool of `threads` workers (numpy releases the GIL in matmul/exp).
    """
    q = np.asarray(q)
    k = np.asarray(k)
    v = np.asarray(v)
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("oracle: q, k, v must have the same shape")
    lead, (n, d) = q.shape[:-2], q.shape[-2:]
    scale = np.float32(1.0 / math.sqrt(d) if softmax_scale is None else softmax_scale)
    qh = q.reshape(-1, n, d).astype(np.float32)
    kh = k.reshape(-1, n, d).astype(np.float32)
    vh = v.reshape(-1, n, d).astype(np.float32)
    heads = qh.shape[0]
    out = np.empty((heads, n, d), dtype=np.float32)
    if heads == 0 or n == 0:
        return out.reshape(q.shape)
    per_head = max(1, n * n * 4)
    chunk = max(1, min(heads, max_chunk_bytes // per_head))
    ranges = [(i, min(heads, i + chunk)) for i in range(0, heads, chunk)]

    def run(r):
        a, b = r
        out[a:b] = _attention_heads(qh[a:b], kh[a:b], vh[a:b], causal, scale)

    workers = threads if threads is not None else 1
    if workers <= 1 or len(ranges) == 1:
        for r in ranges:
            run(r)
    else:
        with ThreadPoolExecutor(max_workers=workers) as ex:
            list(ex.map(run, ranges))
    return out.reshape(q.shape)


def attention_sampled_heads(q, k, v, head_ids, causal=False, softmax_scale=None, threads=None) -> np.ndarray:
    """Oracle on a subset of flattened (b, h) heads: returns [len(head_ids), N, d] fp32."""
    q = np.asarray(q)
    n, d = q.shape[-2:]
    idx = np.asarray(list(head_ids), dtype=np.int64)
    qs = q.reshape(-1, n, d)[idx]
    ks = np.asarray(k).reshape(-1, n, d)[idx]
    vs = np.asarray(v).reshape(-1, n, d)[idx]
    return attention(qs, ks, vs, causal=causal, softmax_scale=softmax_scale, threads=threads)


def default_threads() -> int:
    return max(1, os.cpu_count() or 1)
