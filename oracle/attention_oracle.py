"""CPU oracle for the hybrid-attention decode step — TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may import this module; the product path never does.  It
restates, in numpy fp32, the one-token cached step of FonaTech/Project_Chronos's
two attention modules as the reference computes it, so the decode kernels
(which cache rotated rope keys and fold the key/value up-projections into the
query and the output) can be checked against the unfolded arithmetic:

* ``MLADecodeOracle`` — ``MLAAttention.forward`` (chronos/model/hybrid_attention.py:
  116-179) with S = 1: q_nope / q_rope per-head RMSNorms, RoPE on q_rope at the
  new position with the first rope_dim table columns (:129-132), the latent
  c = RMSNorm(kv_down(x)) appended to the cached latents (:136-142), keys and
  values recomputed from ALL cached latents (k_nope, k_rope rotated at every
  position, v; :147-155), scores / sqrt(head_dim), softmax, weighted values;
* ``SlidingWindowDecodeOracle`` — ``SlidingWindowAttention.forward`` (:213-258)
  with S = 1: q/k RMSNorms, RoPE at past_len = the CUT cache's length (:217-225),
  append, cut to the last ``window`` keys (:231-234), attention over them;
* ``rmsnorm`` — minimind RMSNorm (x * rsqrt(mean(x^2) + eps) * weight);
* ``rope`` — minimind apply_rotary_pos_emb: x * cos + rotate_half(x) * sin.

Every step takes the projection output row of the new token (the layout the
kernels take: MLA [q_nope | q_rope | kv_down], sliding window [q | k | v]).
"""
from __future__ import annotations

from typing import List

import numpy as np


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.asarray(x, np.float32)
    inv = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + np.float32(eps))
    return (np.asarray(w, np.float32) * (x * inv)).astype(np.float32)


def rope(x: np.ndarray, cos_row: np.ndarray, sin_row: np.ndarray) -> np.ndarray:
    """x [..., d]; cos_row/sin_row [d] (or broadcastable)."""
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return (x * cos_row + rot * sin_row).astype(np.float32)


def _attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, n_rep: int, scale: float) -> np.ndarray:
    """q [nH, d]; k, v [T, nKV, d]: softmax(q k^T * scale) v per head (repeat_kv)."""
    out = []
    for h in range(q.shape[0]):
        g = h // n_rep
        s = (k[:, g, :] @ q[h]) * np.float32(scale)
        p = np.exp(s - s.max())
        p = p / p.sum()
        out.append(p @ v[:, g, :])
    return np.concatenate(out).astype(np.float32)


class MLADecodeOracle:
    def __init__(self, heads, kv_heads, head_dim, rope_dim, latent, eps, norm_q_nope, norm_q_rope, norm_kv,
                 w_knope, w_krope, w_v, cos, sin):
        self.nh, self.nkv, self.d, self.r, self.l, self.eps = heads, kv_heads, head_dim, rope_dim, latent, eps
        self.nope = head_dim - rope_dim
        self.wq1, self.wq2, self.wkv = (np.asarray(a, np.float32) for a in (norm_q_nope, norm_q_rope, norm_kv))
        self.w_knope, self.w_krope, self.w_v = (np.asarray(a, np.float32) for a in (w_knope, w_krope, w_v))
        self.cos, self.sin = np.asarray(cos, np.float32), np.asarray(sin, np.float32)
        self.latents: List[np.ndarray] = []

    def step(self, proj_row: np.ndarray) -> np.ndarray:
        nh, nope, R, L = self.nh, self.nope, self.r, self.l
        pos = len(self.latents)
        p = np.asarray(proj_row, np.float32)
        q_nope = rmsnorm(p[:nh * nope].reshape(nh, nope), self.wq1, self.eps)
        q_rope = rmsnorm(p[nh * nope:nh * (nope + R)].reshape(nh, R), self.wq2, self.eps)
        q_rope = rope(q_rope, self.cos[pos, :R], self.sin[pos, :R])
        q = np.concatenate([q_nope, q_rope], axis=-1)
        self.latents.append(rmsnorm(p[nh * (nope + R):nh * (nope + R) + L], self.wkv, self.eps))
        c = np.stack(self.latents)                                   # [T, L]
        T = c.shape[0]
        k_nope = (c @ self.w_knope.T).reshape(T, self.nkv, nope)
        k_rope = (c @ self.w_krope.T).reshape(T, self.nkv, R)
        k_rope = rope(k_rope, self.cos[:T, None, :R], self.sin[:T, None, :R])
        k = np.concatenate([k_nope, k_rope], axis=-1)
        v = (c @ self.w_v.T).reshape(T, self.nkv, self.d)
        return _attend(q, k, v, nh // self.nkv, 1.0 / np.sqrt(self.d))


class SlidingWindowDecodeOracle:
    def __init__(self, heads, kv_heads, head_dim, window, eps, norm_q, norm_k, cos, sin):
        self.nh, self.nkv, self.d, self.w, self.eps = heads, kv_heads, head_dim, window, eps
        self.wq, self.wk = np.asarray(norm_q, np.float32), np.asarray(norm_k, np.float32)
        self.cos, self.sin = np.asarray(cos, np.float32), np.asarray(sin, np.float32)
        self.keys: List[np.ndarray] = []
        self.values: List[np.ndarray] = []

    def step(self, proj_row: np.ndarray) -> np.ndarray:
        nh, nkv, D = self.nh, self.nkv, self.d
        past_len = len(self.keys)            # the cut cache's length
        p = np.asarray(proj_row, np.float32)
        q = rmsnorm(p[:nh * D].reshape(nh, D), self.wq, self.eps)
        k = rmsnorm(p[nh * D:(nh + nkv) * D].reshape(nkv, D), self.wk, self.eps)
        v = p[(nh + nkv) * D:(nh + 2 * nkv) * D].reshape(nkv, D)
        q = rope(q, self.cos[past_len], self.sin[past_len])
        k = rope(k, self.cos[past_len], self.sin[past_len])
        self.keys.append(k)
        self.values.append(v)
        self.keys, self.values = self.keys[-self.w:], self.values[-self.w:]
        return _attend(q, np.stack(self.keys), np.stack(self.values), nh // nkv, 1.0 / np.sqrt(D))
