"""CPU oracle for the Chronos MoE feed-forward layer — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module.  It is the checker for the CUDA
extension, never part of the product path (``project_chronos_b200`` never
imports it and fails loudly when its CUDA library is missing).

What it restates (all citations are files of FonaTech/Project_Chronos):

* routing — ``chronos/model/moe_chronos.py:112`` (gate GEMM, softmax) and
  ``:124-128`` (top-k, ``norm_topk_prob`` renormalisation with ``+1e-20``),
  computed by ``router_oracle.c`` under the bit-exact routing contract of
  ``include/chronos_moe.h`` (fp32 fmaf chain over h, ties -> lower index);
* the expert FFN — minimind ``FeedForward``, restated in the reference at
  ``chronos/mlx/moe.py:13-23``: ``down(silu(gate(x)) * up(x))``, bias-free;
* shared experts — ``moe_chronos.py:90-93``: the MEAN of the shared FFNs;
* the lookahead router — ``chronos/model/lookahead_router.py:36-55``
  (``lookahead``);
* the training load-balance loss — ``moe_chronos.py:175-185`` and
  ``:270-276`` (``aux_loss``);
* the blend and combine — ``moe_chronos.py:190-268`` with the arithmetic form
  of ``chronos/mlx/moe.py:160-166``:
  ``y_t = sum_k w_tk (a_e E_e(x_t) + (1 - a_e) S(x_t)) + S(x_t)``.

Parity pin: the routing and the layer output are checked against golden
vectors produced by the reference's own ``ChronosMOEFeedForward`` (imported
in the build container through a minimind shim; see
``tests/golden/make_golden.py``).  The minimind ``FeedForward`` itself is a
third-party dependency absent from the reference tree (``chronos/deps.py:17-18``
pins only the ``master`` branch of github.com/jingyaogong/minimind); its
SwiGLU form is the one restated in ``chronos/mlx/moe.py:13-23``.

Arithmetic: fp32 numpy (BLAS) on the operand values.  ``emulate_device``
additionally rounds the SwiGLU hidden activation and the final output to the
input dtype, which is where the CUDA path rounds, so tight tolerances can be
used in tests.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "librouter_oracle.so")
_lib = None


def build() -> str:
    """Compile router_oracle.c into librouter_oracle.so (gcc, no fast-math)."""
    src = os.path.join(_HERE, "router_oracle.c")
    if (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(
            ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
             "-o", _LIB_PATH, src, "-lm"])
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(_LIB_PATH)
        f32p = ctypes.POINTER(ctypes.c_float)
        i32p = ctypes.POINTER(ctypes.c_int32)
        lib.oracle_route.argtypes = [f32p, f32p, f32p, ctypes.c_int64, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int, i32p,
                                     f32p, f32p, f32p]
        lib.oracle_route.restype = None
        lib.oracle_router_logits.argtypes = [f32p, f32p, f32p, ctypes.c_int64,
                                             ctypes.c_int, ctypes.c_int, f32p]
        lib.oracle_router_logits.restype = None
        _lib = lib
    return _lib


def _fp(a: Optional[np.ndarray]):
    if a is None:
        return ctypes.POINTER(ctypes.c_float)()
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


# ---------------------------------------------------------------------------
# dtype helpers (round-to-nearest-even, as torch / the device round)
# ---------------------------------------------------------------------------

def round_to_bf16(a: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 value (RNE), returned as fp32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def round_to_dtype(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_to_bf16(a)
    if dtype == "fp16":
        return a.astype(np.float16).astype(np.float32)
    return np.asarray(a, dtype=np.float32)


# ---------------------------------------------------------------------------
# routing
# ---------------------------------------------------------------------------

def route(x: np.ndarray, router_w: np.ndarray, k: int, norm_topk: bool,
          bias: Optional[np.ndarray] = None):
    """Routing contract of include/chronos_moe.h on fp32 operand values.

    Returns (idx [N,k] int32 in rank order, weight [N,k] fp32, probs [N,E] fp32,
    logits [N,E] fp32).
    """
    lib = _load()
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(router_w, dtype=np.float32)
    n, h = x.shape
    e = w.shape[0]
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    idx = np.zeros((n, k), dtype=np.int32)
    wt = np.zeros((n, k), dtype=np.float32)
    probs = np.zeros((n, e), dtype=np.float32)
    logits = np.zeros((n, e), dtype=np.float32)
    lib.oracle_route(_fp(x), _fp(w), _fp(b), n, h, e, k, int(bool(norm_topk)),
                     idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), _fp(wt),
                     _fp(probs), _fp(logits))
    return idx, wt, probs, logits


# ---------------------------------------------------------------------------
# the layer
# ---------------------------------------------------------------------------

def _silu(v: np.ndarray) -> np.ndarray:
    return v / (1.0 + np.exp(-v))


def swiglu(x: np.ndarray, wg: np.ndarray, wu: np.ndarray, wd: np.ndarray,
           round_hidden: Optional[str] = None) -> np.ndarray:
    """down(silu(gate(x)) * up(x)) with nn.Linear [out, in] weights, fp32."""
    g = x @ wg.T
    u = x @ wu.T
    hdn = (_silu(g) * u).astype(np.float32)
    if round_hidden is not None:
        hdn = round_to_dtype(hdn, round_hidden)
    return (hdn @ wd.T).astype(np.float32)


def moe_forward(x: np.ndarray, router_w: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray,
                w_down: np.ndarray, sh_gate: np.ndarray, sh_up: np.ndarray,
                sh_down: np.ndarray, k: int, norm_topk: bool,
                avail: Optional[np.ndarray] = None, bias: Optional[np.ndarray] = None,
                dtype: str = "fp32", emulate_device: bool = False, route_out=None):
    """The blended MoE output for every row of ``x`` (fp32 result).

    ``x`` [N,H]; ``router_w`` [E,H]; ``w_gate``/``w_up`` [E,F,H]; ``w_down``
    [E,H,F]; ``sh_*`` the same with S_h leading; ``avail`` [E] in [0,1] or
    None (all available).  Returns (y [N,H], idx, weight, probs).
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, h = x.shape
    e = router_w.shape[0]
    s_h = sh_gate.shape[0]
    if route_out is None:
        idx, wt, probs, _ = route(x, router_w, k, norm_topk, bias)
    else:
        idx, wt, probs = route_out
    a = np.ones(e, dtype=np.float32) if avail is None else np.asarray(avail, np.float32)
    rh = dtype if (emulate_device and dtype != "fp32") else None

    shared = np.zeros((n, h), dtype=np.float32)
    for j in range(s_h):
        shared += swiglu(x, sh_gate[j], sh_up[j], sh_down[j], rh)
    if s_h > 0:
        shared /= np.float32(s_h)

    y = np.zeros((n, h), dtype=np.float32)
    shared_coef = np.ones(n, dtype=np.float32)
    for ex in range(e):
        rows, cols = np.nonzero(idx == ex)
        if rows.size == 0:
            continue
        w_sel = wt[rows, cols]
        ae = a[ex]
        shared_coef[rows] += w_sel * (1.0 - ae)
        if ae > 0.0:
            out = swiglu(x[rows], w_gate[ex], w_up[ex], w_down[ex], rh)
            np.add.at(y, rows, out * (w_sel * ae)[:, None])
    if s_h > 0:
        y += shared * shared_coef[:, None]
    if emulate_device and dtype != "fp32":
        y = round_to_dtype(y, dtype)
    return y, idx, wt, probs


def lookahead(x: np.ndarray, w1: np.ndarray, w2: np.ndarray, num_experts: int, steps: int) -> np.ndarray:
    """Lookahead router probabilities [N, K, E] (chronos/model/lookahead_router.py:36-55):
    softmax over the experts of W2 . silu(W1 . x), per step, fp32."""
    x = np.asarray(x, np.float32)
    h1 = _silu((x @ np.asarray(w1, np.float32).T).astype(np.float32)).astype(np.float32)
    lg = (h1 @ np.asarray(w2, np.float32).T).astype(np.float32).reshape(x.shape[0], steps, num_experts)
    lg = lg - lg.max(axis=-1, keepdims=True)
    e = np.exp(lg)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def aux_loss(idx: np.ndarray, probs: np.ndarray, num_experts: int) -> float:
    """Raw load-balance loss of a training forward (``moe_chronos.py:177-178``):
    ``E * sum_{j,e} onehot(idx)[:, j, e].mean(0) * probs.mean(0)[e]``, i.e. E
    times the sum over experts of (selections of e / tokens) x (mean router
    probability of e); float64 accumulation."""
    idx = np.asarray(idx)
    n = idx.shape[0]
    if n == 0:
        return 0.0
    load = np.bincount(idx.reshape(-1), minlength=num_experts).astype(np.float64) / n
    return float(num_experts * np.sum(load * np.asarray(probs, np.float64).mean(axis=0)))


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b.ravel())
    num = np.linalg.norm((a - b).ravel())
    if den == 0.0:
        return float(num)
    return float(num / den)
