"""numpy restatement of the reference's ``fp_attention`` Triton kernel.

TEST INFRASTRUCTURE ONLY (the oracle).  Nothing in ``fusionpass_b200`` imports it.

Follows ``lib/Plan/TritonEmitter.cpp:73-104`` (twin
``python/fusionpass/kernels.py:58-89``) step by step, per (batch*head, 64-row
query tile):

* q, k, v are contiguous ``[BH, S, D]`` and upcast to float32 (``:66-67,74-75,82-83``);
* ``m_i = -inf``, ``l_i = 0``, ``acc = 0`` in float32 (``:68-70``);
* for each 64-key tile: ``s = (q @ k^T) * scale`` with IEEE f32 dots (``:76``),
  out-of-range keys set to ``-inf`` (``:77``), ``m_new = max(m_i, rowmax(s))``,
  ``alpha = exp(m_i - m_new)``, ``p = exp(s - m_new)``, ``l_i = l_i*alpha + rowsum(p)``,
  ``acc = acc*alpha + p @ v`` (``:78-85``);
* ``out = acc / l_i`` rounded once to the output dtype (``:86-88``).

The Triton interpreter evaluates ``tl.dot`` as ``np.matmul(a, b) + acc`` in
float32, which is what this restatement does as well.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
BLOCK_M = 64  # reference kernels.py:34
BLOCK_N = 64  # reference kernels.py:35


def _tile(qt, k, v, S, scale):
    m_i = np.full((qt.shape[0],), -np.inf, dtype=F32)
    l_i = np.zeros((qt.shape[0],), dtype=F32)
    acc = np.zeros((qt.shape[0], qt.shape[1]), dtype=F32)
    D = qt.shape[1]
    for start in range(0, S, BLOCK_N):
        # masked tile loads read 0.0 past the end (kernels.py:74-75,82-83)
        kt = np.zeros((BLOCK_N, D), dtype=F32)
        vt = np.zeros((BLOCK_N, D), dtype=F32)
        n = min(BLOCK_N, S - start)
        kt[:n] = k[start:start + n]
        vt[:n] = v[start:start + n]
        s = (np.matmul(qt, kt.T, dtype=F32) + F32(0.0)) * F32(scale)
        s[:, n:] = -np.inf  # kernels.py:77
        m_new = np.maximum(m_i, s.max(axis=1))
        alpha = np.exp((m_i - m_new).astype(F32)).astype(F32)
        p = np.exp((s - m_new[:, None]).astype(F32)).astype(F32)
        l_i = (l_i * alpha + p.sum(axis=1, dtype=F32)).astype(F32)
        acc = (acc * alpha[:, None] + (np.matmul(p, vt, dtype=F32) + F32(0.0))).astype(F32)
        m_i = m_new
    return acc / l_i[:, None]


def attention_fwd(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float,
                  out_dtype=None, bh_slices=None) -> np.ndarray:
    """``softmax(scale * q @ k^T) @ v`` over ``[..., S, D]`` with the reference tiling.

    ``bh_slices`` (optional iterable of flat batch*head indices) restricts the
    work to those slices; the other slices of the result are left as zeros.
    Every (tile, bh) program is independent in the reference grid
    (``kernels.py:320``), so a slice-wise run is exact for the slices it covers.
    """
    out_dtype = out_dtype or q.dtype
    shape = q.shape
    S, D = shape[-2], shape[-1]
    bh = int(np.prod(shape[:-2])) if len(shape) > 2 else 1
    q3 = np.asarray(q).reshape(bh, S, D).astype(F32)
    k3 = np.asarray(k).reshape(bh, S, D).astype(F32)
    v3 = np.asarray(v).reshape(bh, S, D).astype(F32)
    out = np.zeros((bh, S, D), dtype=F32)
    which = range(bh) if bh_slices is None else bh_slices
    for b in which:
        for m0 in range(0, S, BLOCK_M):
            # masked query loads read 0.0 past the end (kernels.py:66-67)
            qt = np.zeros((BLOCK_M, D), dtype=F32)
            n = min(BLOCK_M, S - m0)
            qt[:n] = q3[b, m0:m0 + n]
            out[b, m0:m0 + n] = _tile(qt, k3[b], v3[b], S, scale)[:n]
    return out.astype(out_dtype).reshape(shape)
