"""CPU restatement of the expert-parallel kernels — TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may use this module: it stands in for the sm_100a extension so
that the host orchestration of ``project_chronos_b200.ep.ExpertParallelMoE``
(splits, all-to-all order, combine) can run on gloo CPU ranks.  The product
path never imports it.

``CpuEpBackend`` exposes the four calls ``ExpertParallelMoE`` makes, with the
same arguments and results as ``project_chronos_b200.ops``:

* ``moe_route``   — the routing contract of include/chronos_moe.h
  (``router_oracle.c``; reference ``chronos/model/moe_chronos.py:112-128``);
* ``ep_dispatch`` — include/chronos_ep.h: rows grouped by (expert chunk, destination rank),
  metadata (local expert, w*a), ``pair_slot``, shared share w*(1-a); inside a
  rank this restatement orders rows by (token, choice), the kernel's order is
  unspecified and nothing downstream depends on it.  ``dedup``: one row per
  (token, destination rank), opened by the token's first available selection
  there, metadata [P, 2] = that rank's selections in choice order, padded with
  (-1, 0.0); ``seg_rows`` > 0: rank g's rows start at g * seg_rows, the rest of
  each segment is padding metadata (fixed all-to-all splits);
* ``moe_forward`` — the blended layer (``moe_oracle.moe_forward``) on pre-routed
  selections, with ``slot_of_expert < 0`` meaning a = 0;
* ``ep_combine``  — y_t = y_shared_t + sum_j rows[pair_slot(t, j)].

The arithmetic of the layer itself is ``chronos/mlx/moe.py:160-166``; see
``moe_oracle``.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import moe_oracle as O


def _np(t: Optional[torch.Tensor]) -> Optional[np.ndarray]:
    return None if t is None else t.detach().to(torch.float32).cpu().numpy()


class CpuEpBackend:
    """fp32 CPU stand-ins for the extension calls of the expert-parallel layer."""

    @staticmethod
    def moe_route(x, router_w, top_k, norm_topk, num_shared=0, ffn=64, router_bias=None,
                  want_probs=True, workspace=None):
        idx, wt, probs, _ = O.route(_np(x), _np(router_w), int(top_k), bool(norm_topk), _np(router_bias))
        return dict(topk_idx=torch.from_numpy(idx), topk_weight=torch.from_numpy(wt),
                    probs=torch.from_numpy(probs) if want_probs else None, counts=None, mass=None)

    @staticmethod
    def ep_dispatch(x, topk_idx, topk_weight, num_experts, world_size, avail=None, num_chunks=1, dedup=False,
                    seg_rows=0):
        xn = x.detach()
        idx = topk_idx.to(torch.int64).numpy()
        wt = topk_weight.to(torch.float32).numpy()
        n, k = idx.shape
        epr = num_experts // world_size
        a_all = np.ones(num_experts, np.float32) if avail is None else \
            np.clip(_np(avail), 0.0, 1.0).astype(np.float32)
        a = a_all[idx]
        shared_w = (wt * (np.float32(1.0) - a)).astype(np.float32)
        num_chunks = max(1, int(num_chunks))
        dest = idx // epr
        key = ((idx % epr) // (epr // num_chunks)) * world_size + dest
        pairs = min(k, epr) if dedup and num_chunks == 1 else 1
        sent = a > 0
        if pairs > 1:   # only a token's first available selection on each rank opens a row
            for t in range(n):
                seen = set()
                for j in range(k):
                    if sent[t, j]:
                        if dest[t, j] in seen:
                            sent[t, j] = False
                        seen.add(dest[t, j])
        counts = np.array([int(np.sum(sent & (key == q))) for q in range(num_chunks * world_size)], np.int32)
        seg_rows = int(seg_rows)
        if seg_rows > 0:
            assert num_chunks == 1 and counts.max(initial=0) <= seg_rows
            offs = np.arange(world_size, dtype=np.int64) * seg_rows
            rows = world_size * seg_rows
        else:
            offs = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int64)
            rows = n * k
        send_x = torch.zeros(rows, xn.shape[1], dtype=xn.dtype)
        meta = np.zeros((rows, pairs, 2), np.int32)
        meta[:, :, 0] = -1
        pair_slot = np.full(n * k, -1, np.int32)
        fill = offs.copy()
        for i in range(n * k):                       # (token, choice) order inside a rank
            t, j = divmod(i, k)
            if not sent[t, j]:
                continue
            g = dest[t, j]
            q = key[t, j]
            s = int(fill[q])
            fill[q] += 1
            pair_slot[i] = s
            send_x[s] = xn[t]
            picks = [jj for jj in range(j, k) if a[t, jj] > 0 and dest[t, jj] == g] if pairs > 1 else [j]
            for qq, jj in enumerate(picks):
                meta[s, qq, 0] = idx[t, jj] - g * epr
                meta[s, qq, 1] = np.float32(wt[t, jj] * a[t, jj]).view(np.int32)
        return dict(send_counts=torch.from_numpy(counts).view(num_chunks, world_size), send_x=send_x,
                    send_meta=torch.from_numpy(meta), pair_slot=torch.from_numpy(pair_slot),
                    shared_weight=torch.from_numpy(shared_w), pairs=pairs)

    @staticmethod
    def moe_forward(x, router_w, w_gate, w_up, w_down, sh_gate, sh_up, sh_down, top_k, norm_topk,
                    avail=None, router_bias=None, slot_of_expert=None, want_probs=True, topk=None,
                    **_):
        xn = _np(x)
        e = router_w.shape[0]
        a = np.ones(e, np.float32) if avail is None else _np(avail)
        if slot_of_expert is not None:
            a = np.where(slot_of_expert.cpu().numpy() < 0, np.float32(0.0), a).astype(np.float32)
        if topk is not None:
            # padding selections (expert -1) contribute nothing: weight 0 on expert 0
            ti = topk[0].to(torch.int32).numpy().copy()
            tw = topk[1].to(torch.float32).numpy().copy()
            tw[ti < 0] = 0.0
            ti[ti < 0] = 0
            route_out = (ti, tw, None)
        else:
            idx, wt, probs, _l = O.route(xn, _np(router_w), int(top_k), bool(norm_topk), _np(router_bias))
            route_out = (idx, wt, probs)
        h = xn.shape[1]
        f = w_gate.shape[1]
        s_h = 0 if sh_gate is None else sh_gate.shape[0]
        shg = _np(sh_gate) if s_h else np.zeros((0, f, h), np.float32)
        shu = _np(sh_up) if s_h else np.zeros((0, f, h), np.float32)
        shd = _np(sh_down) if s_h else np.zeros((0, h, f), np.float32)
        # slot p of the pools serves expert p (the layer's own pools)
        y, _, _, _ = O.moe_forward(xn, np.zeros((e, h), np.float32), _np(w_gate), _np(w_up), _np(w_down),
                                   shg, shu, shd, int(top_k), bool(norm_topk), avail=a,
                                   route_out=route_out)
        return dict(y=torch.from_numpy(y).to(x.dtype), probs=None, topk_idx=None, topk_weight=None)

    @staticmethod
    def ep_combine(recv_y, pair_slot, top_k, y_shared=None, num_tokens=None, out=None):
        n = int(num_tokens if num_tokens is not None else pair_slot.numel() // top_k)
        h = recv_y.shape[1]
        rows = recv_y.to(torch.float32)
        y = torch.zeros(n, h) if y_shared is None else y_shared.to(torch.float32).clone()
        ps = pair_slot.view(n, top_k)
        for j in range(top_k):
            s = ps[:, j].to(torch.int64)
            ok = s >= 0
            y[ok] += rows[s[ok]]
        return y.to(recv_y.dtype)
