"""Expert-parallel Chronos MoE layer: routed experts sharded over a process group.

The reference runs every expert of a layer on one device
(``chronos/model/moe_chronos.py:146-173, 190-268``).  Here rank g of a group of
G owns the routed experts ``[g*E/G, (g+1)*E/G)``; the router and the shared
experts are replicated; tokens stay on their rank.  One forward (with one rank
and ``dispatch_single_rank=False``, the default, it is the single-device layer
call instead):

1. route the rank's tokens (router kernels, bit-exact routing contract);
2. ``chronos_ep_dispatch``: rows of x grouped by destination rank, with
   (local expert, w*a) metadata; selections of unavailable experts (a = 0)
   are not sent, their weight moves to the shared term;
3. all-to-all of the counts (the one host synchronisation: NCCL's variable
   all-to-all needs the split sizes), then of the rows and metadata (NCCL over
   NVLink); the shared term (1 + sum w(1-a)) * mean_j Shared_j(x) is computed
   while the rows travel;
4. the received rows through the grouped expert kernels (pre-routed, k = 1):
   w*a*SwiGLU_e(x) per row;
5. all-to-all of the result rows back to their source ranks;
6. ``chronos_ep_combine``: y_t = shared term + sum_j returned row (t, j).

Same arithmetic as the single-device layer (the blend of
``chronos/mlx/moe.py:160-166``); each routed contribution is rounded once to the
layer dtype before the fp32 combine.  All compute runs in the sm_100a
extension; ``backend`` exists so the host orchestration can be exercised
with CPU stand-ins in tests.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from . import ops


class ExpertParallelMoE(nn.Module):
    def __init__(self, config, group: Optional["dist.ProcessGroup"] = None, backend=None,
                 dispatch_single_rank: bool = False):
        super().__init__()
        self.dispatch_single_rank = bool(dispatch_single_rank)
        self.config = config
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.rank = dist.get_rank(group)
            self.world = dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1
        E = int(config.num_experts)
        if E % self.world:
            raise ValueError(f"num_experts {E} is not a multiple of the group size {self.world}")
        self.num_experts = E
        self.experts_per_rank = E // self.world
        self.first_expert = self.rank * self.experts_per_rank
        self.top_k = int(config.num_experts_per_tok)
        self.norm_topk_prob = bool(config.norm_topk_prob)
        self.num_shared = int(getattr(config, "num_shared_experts", 1))
        self.router_logit_bias: Optional[torch.Tensor] = None
        self.backend = backend if backend is not None else ops
        self.router = None
        self.w_gate = self.w_up = self.w_down = None
        self.sh_gate = self.sh_up = self.sh_down = None
        self.last_send_counts = None
        self.last_recv_counts = None

    @classmethod
    def from_stacked(cls, config, router: torch.Tensor, gate: torch.Tensor, up: torch.Tensor,
                     down: torch.Tensor, sh_gate: Optional[torch.Tensor] = None,
                     sh_up: Optional[torch.Tensor] = None, sh_down: Optional[torch.Tensor] = None,
                     group=None, backend=None, local: bool = False,
                     dispatch_single_rank: bool = False) -> "ExpertParallelMoE":
        """Build from stacked weights.  ``local=False``: gate/up/down hold all E
        experts and this rank keeps its slice (a view); ``local=True``: they
        already hold only this rank's E/G experts."""
        m = cls(config, group=group, backend=backend, dispatch_single_rank=dispatch_single_rank)
        lo, n = m.first_expert, m.experts_per_rank
        if not local:
            gate, up, down = gate[lo:lo + n], up[lo:lo + n], down[lo:lo + n]
        if gate.shape[0] != n:
            raise ValueError(f"expected {n} local experts, got {gate.shape[0]}")
        m.router = router
        m.w_gate, m.w_up, m.w_down = gate.contiguous(), up.contiguous(), down.contiguous()
        if m.num_shared:
            m.sh_gate, m.sh_up, m.sh_down = sh_gate, sh_up, sh_down
        return m

    @classmethod
    def from_layer(cls, layer, group=None, backend=None) -> "ExpertParallelMoE":
        """Shard a single-device ``ChronosMOEFeedForward`` (its live experts)."""
        m = cls(layer.config, group=group, backend=backend)
        lo, n = m.first_expert, m.experts_per_rank
        ex = [layer.experts[e] for e in range(lo, lo + n)]
        stack = lambda mods, name: torch.stack([getattr(x, name).weight.detach() for x in mods])  # noqa: E731
        sh = list(layer.shared_experts)
        return cls.from_stacked(
            layer.config, layer.gate.weight.detach(), stack(ex, "gate_proj"), stack(ex, "up_proj"),
            stack(ex, "down_proj"), stack(sh, "gate_proj") if sh else None,
            stack(sh, "up_proj") if sh else None, stack(sh, "down_proj") if sh else None,
            group=group, backend=backend, local=True)

    # ------------------------------------------------------------------
    def _exchange(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, async_op=False):
        return dist.all_to_all_single(out, inp, output_split_sizes=out_splits,
                                      input_split_sizes=in_splits, group=self.group,
                                      async_op=async_op)

    def forward(self, x: torch.Tensor, available_expert_mask: Optional[torch.Tensor] = None
                ) -> torch.Tensor:
        be = self.backend
        shp = x.shape
        H = shp[-1]
        xf = x.reshape(-1, H)
        dev, dt = xf.device, xf.dtype
        k, E, G = self.top_k, self.num_experts, self.world
        F = self.w_gate.shape[1]
        avail = None
        if available_expert_mask is not None:
            avail = available_expert_mask.to(device=dev, dtype=torch.float32)

        if G == 1 and not self.dispatch_single_rank:
            # one rank owns every expert: the single-device layer, no dispatch
            y = be.moe_forward(xf, self.router, self.w_gate, self.w_up, self.w_down, self.sh_gate,
                               self.sh_up, self.sh_down, k, self.norm_topk_prob, avail=avail,
                               router_bias=self.router_logit_bias, want_probs=False)["y"]
            self.last_send_counts = self.last_recv_counts = None
            return y.view(shp)

        # 1-2: route, build the send buffers
        r = be.moe_route(xf, self.router, k, self.norm_topk_prob, num_shared=self.num_shared,
                         ffn=F, router_bias=self.router_logit_bias, want_probs=False)
        d = be.ep_dispatch(xf, r["topk_idx"], r["topk_weight"], E, G, avail=avail)

        # 3: counts, then rows + metadata (async) while the shared term runs
        send_counts = d["send_counts"]
        recv_counts = send_counts if G == 1 else torch.empty_like(send_counts)
        if G > 1:
            self._exchange(recv_counts, send_counts, None, None)
        both = torch.cat([send_counts, recv_counts]).cpu().tolist()
        sc, rc = both[:G], both[G:]
        self.last_send_counts, self.last_recv_counts = sc, rc
        n_send, n_recv = sum(sc), sum(rc)
        if G == 1:  # nothing to exchange: the send buffers are the receive buffers
            recv_x, recv_meta = d["send_x"][:n_send], d["send_meta"][:n_send]
            w1 = w2 = None
        else:
            recv_x = torch.empty(n_recv, H, dtype=dt, device=dev)
            recv_meta = torch.empty(n_recv, 2, dtype=torch.int32, device=dev)
            w1 = self._exchange(recv_x, d["send_x"][:n_send], rc, sc, async_op=True)
            w2 = self._exchange(recv_meta, d["send_meta"][:n_send], rc, sc, async_op=True)

        y_shared = None
        if self.num_shared:
            no_slot = torch.full((E,), -1, dtype=torch.int32, device=dev)
            y_shared = be.moe_forward(
                xf, self.router, self.w_gate, self.w_up, self.w_down, self.sh_gate, self.sh_up,
                self.sh_down, k, self.norm_topk_prob, avail=torch.zeros(E, dtype=torch.float32, device=dev),
                slot_of_expert=no_slot, want_probs=False,
                topk=[r["topk_idx"], d["shared_weight"]])["y"]
        for w in (w1, w2):
            if w is not None:
                w.wait()

        # 4: this rank's experts on the rows it received
        eid = recv_meta[:, 0:1].contiguous()
        wgt = recv_meta[:, 1:2].contiguous().view(torch.float32)
        local_router = torch.empty(self.experts_per_rank, H, dtype=dt, device=dev)
        y_loc = be.moe_forward(recv_x, local_router, self.w_gate, self.w_up, self.w_down, None, None,
                               None, 1, False, want_probs=False, topk=[eid, wgt])["y"]

        # 5-6: rows back to their source ranks, combine
        if G == 1:
            back = y_loc
        else:
            back = torch.empty(n_send, H, dtype=dt, device=dev)
            self._exchange(back, y_loc, sc, rc)
        y = be.ep_combine(back, d["pair_slot"], k, y_shared=y_shared, num_tokens=xf.shape[0])
        return y.view(shp)
