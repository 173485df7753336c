"""An independent numpy restatement of the reference's attention math (float64), used to
cross-check the C oracle.  Written from src/forward.nim:108-211 semantics, vectorised."""
from __future__ import annotations

import numpy as np


def rope_cols(x: np.ndarray, nHead: int, headDim: int, ropeDim: int, base: float,
              positions: np.ndarray) -> np.ndarray:
    """Rotate pairs (2i, 2i+1) of every head at the given per-column positions (float64)."""
    y = np.array(x, np.float64, copy=True)
    S = y.shape[1]
    i = np.arange(ropeDim // 2)
    theta = np.power(np.float32(1.0) / np.float32(base),
                     (2 * i).astype(np.float32) / np.float32(ropeDim)).astype(np.float64)
    ang = np.outer(theta, positions.astype(np.float64))  # [pairs, S]
    c, s = np.cos(ang), np.sin(ang)
    for h in range(nHead):
        r0 = h * headDim + 2 * i
        r1 = r0 + 1
        v0, v1 = y[r0, :S].copy(), y[r1, :S].copy()
        y[r0, :S] = v0 * c - v1 * s
        y[r1, :S] = v0 * s + v1 * c
    return y


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, nHead: int, nHeadKv: int,
              headDim: int, qpos: np.ndarray, nkeys: int) -> np.ndarray:
    """q: [nHead*headDim, Sq], k,v: [nHeadKv*headDim, >= nkeys]; query column i attends keys
    0..qpos[i].  Returns ctx [nHead*headDim, Sq] in float64."""
    group = nHead // nHeadKv
    Sq = q.shape[1]
    ctx = np.zeros((nHead * headDim, Sq))
    for h in range(nHead):
        kvh = h // group
        qh = q[h * headDim:(h + 1) * headDim].astype(np.float64)
        kh = k[kvh * headDim:(kvh + 1) * headDim, :nkeys].astype(np.float64)
        vh = v[kvh * headDim:(kvh + 1) * headDim, :nkeys].astype(np.float64)
        s = (qh.T @ kh) / np.sqrt(headDim)  # [Sq, nkeys]
        mask = np.arange(nkeys)[None, :] > qpos[:, None]
        s[mask] = -np.inf
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        ctx[h * headDim:(h + 1) * headDim] = vh @ p.T
    return ctx
