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
   NVLink), in C chunks of each rank's experts, all issued at once; the shared
   term (1 + sum w(1-a)) * mean_j Shared_j(x) is computed while the rows travel.
   With ``segment_rows`` > 0 (the same on every rank) the send buffers hold one
   fixed segment of that many rows per destination and both exchanges use equal
   splits: no counts, no host synchronisation, padding rows (expert -1) travel;
4. as each chunk lands, its rows through the grouped expert kernels
   (pre-routed, k = 1): w*a*SwiGLU_e(x) per row (with C > 1 on at most
   ``gemm_ctas`` SMs, leaving the rest to the exchange);
5. all-to-all of each chunk's result rows back to their source ranks, in
   flight while the next chunk's experts run;
6. ``chronos_ep_combine``: y_t = shared term + sum_j returned row (t, j).

Same arithmetic as the single-device layer (the blend of
``chronos/mlx/moe.py:160-166``); each routed contribution is rounded once to the
layer dtype before the fp32 combine.  ``available_expert_mask`` is applied as
that arithmetic availability, a_e = mask[e], in eval as in training: every
expert of a sharded layer is resident, so there is no live-but-marked-
unavailable expert to run anyway, as the torch module does in eval
(``moe_chronos.py:221-227``).  A mask with zeros therefore sends those
experts' selections to the shared term here, while
``ChronosMOEFeedForward`` in eval would still run its loaded experts.  All compute runs in the sm_100a
extension; ``backend`` exists so the host orchestration can be exercised
with CPU stand-ins in tests.
"""
from __future__ import annotations

import contextlib

from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from . import ops

_MAX_KEYS = 32  # chunks x ranks of one dispatch (CHRONOS_EP_MAX_RANKS)


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
        # expert chunks of the exchange pipeline (dividing E/G, chunks * ranks <= 32), and
        # the CTAs the expert GEMMs may use while chunks are exchanged beside them
        self.chunks = 1
        self.gemm_ctas = 132
        # unchunked exchange: one row per (token, destination rank), every selection of
        # the token on that rank in the row's metadata (False: one row per selection)
        self.dedup = True
        # > 0: fixed all-to-all segments of this many rows per destination rank (every
        # rank must use the same value, and a forward's rows per destination must fit:
        # its token count when deduplicated); 0: split sizes exchanged and read on the host
        self.segment_rows = 0
        self.last_send_counts_dev = None
        # optional phase timing: a list that each forward appends
        # {phase: torch.cuda.Event} to (events on the compute stream)
        self.phase_events = None

    def _side_stream(self, dev) -> torch.cuda.Stream:
        """One side stream per device for the shared experts' term."""
        streams = self.__dict__.setdefault("_side_streams", {})
        st = streams.get(dev.index)
        if st is None:
            st = torch.cuda.Stream(device=dev)
            streams[dev.index] = st
        return st

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

    def read_send_counts(self):
        """Rows sent to each rank by the last forward (a host read of the device
        counts when the exchange used fixed segments)."""
        if self.last_send_counts is not None or self.last_send_counts_dev is None:
            return self.last_send_counts
        return [int(v) for v in self.last_send_counts_dev.reshape(-1).cpu().tolist()]

    # ------------------------------------------------------------------
    def _exchange(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, async_op=False):
        if self.world == 1:  # a single rank sends everything to itself
            out.copy_(inp)
            return None
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

        marks = {} if self.phase_events is not None else None

        def mark(name):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks[name] = ev

        mark("start")
        # 1-2: route, build the send buffers (rows ordered by token chunk, then rank)
        r = be.moe_route(xf, self.router, k, self.norm_topk_prob, num_shared=self.num_shared,
                         ffn=F, router_bias=self.router_logit_bias, want_probs=False)
        C = max(c for c in range(1, max(1, min(self.chunks, _MAX_KEYS // G)) + 1)
                if self.experts_per_rank % c == 0)
        # with chunks, the exchange runs beside the expert GEMMs: leave it SMs
        max_ctas = 0 if C == 1 else self.gemm_ctas
        seg = int(self.segment_rows) if C == 1 else 0
        if seg:
            need = xf.shape[0] if self.dedup else xf.shape[0] * min(k, self.experts_per_rank)
            if need > seg:
                raise ValueError(f"{need} rows per destination do not fit segment_rows {seg}")
        # one row per (token, destination rank) when unchunked: each x row crosses
        # to a rank once, carrying all of the token's selections there
        d = be.ep_dispatch(xf, r["topk_idx"], r["topk_weight"], E, G, avail=avail, num_chunks=C,
                           dedup=self.dedup, seg_rows=seg)
        P = int(d.get("pairs", 1))

        mark("dispatched")
        # the shared experts' term needs only the routing: on a CUDA device it runs on a
        # side stream from here, so the GPU has work while the host waits for the split
        # sizes below (the row exchange still overlaps it, as before)
        y_shared = None
        side = None
        if self.num_shared:
            cur = torch.cuda.current_stream(dev) if xf.is_cuda else None
            if cur is not None:
                side = self._side_stream(dev)
                side.wait_stream(cur)
            with (torch.cuda.stream(side) if side is not None else contextlib.nullcontext()):
                no_slot = torch.full((E,), -1, dtype=torch.int32, device=dev)
                y_shared = be.moe_forward(
                    xf, self.router, self.w_gate, self.w_up, self.w_down, self.sh_gate, self.sh_up,
                    self.sh_down, k, self.norm_topk_prob, avail=torch.zeros(E, dtype=torch.float32, device=dev),
                    slot_of_expert=no_slot, want_probs=False,
                    topk=[r["topk_idx"], d["shared_weight"]])["y"]
                mark("shared_done")
        if seg:
            # 3 (fixed segments): equal splits, nothing for the host to wait for
            sc = rc = [[seg] * G]
            self.last_send_counts = self.last_recv_counts = None
            self.last_send_counts_dev = d["send_counts"]
        else:
            # 3: counts [C, G] -> per destination [G, C]; one host sync for every split size
            send_gc = d["send_counts"].reshape(C, G).t().contiguous()
            recv_gc = torch.empty_like(send_gc)
            self._exchange(recv_gc, send_gc, None, None)
            both = torch.cat([send_gc.reshape(-1), recv_gc.reshape(-1)]).cpu().tolist()
            sc = [[both[g * C + c] for g in range(G)] for c in range(C)]          # sent, [c][g]
            rc = [[both[G * C + g * C + c] for g in range(G)] for c in range(C)]  # received, [c][g]
            self.last_send_counts = [sum(sc[c][g] for c in range(C)) for g in range(G)]
            self.last_recv_counts = [sum(rc[c][g] for c in range(C)) for g in range(G)]
            self.last_send_counts_dev = None
        send_off = [0]
        for c in range(C):
            send_off.append(send_off[-1] + sum(sc[c]))
        n_send = send_off[-1]

        # rows and metadata of every chunk, in flight while the shared term runs
        recv_x, recv_meta, works = [], [], []
        for c in range(C):
            lo, hi = send_off[c], send_off[c + 1]
            rx = torch.empty(sum(rc[c]), H, dtype=dt, device=dev)
            rm = torch.empty(sum(rc[c]), P, 2, dtype=torch.int32, device=dev)
            works.append((self._exchange(rx, d["send_x"][lo:hi], rc[c], sc[c], async_op=True),
                          self._exchange(rm, d["send_meta"][lo:hi], rc[c], sc[c], async_op=True)))
            recv_x.append(rx)
            recv_meta.append(rm)

        mark("counts_exchanged")

        # 4-5: per expert chunk, as it lands: its experts on its rows, rows sent back
        # (the return of chunk c overlaps the experts of chunk c + 1)
        local_router = torch.empty(self.experts_per_rank, H, dtype=dt, device=dev)
        back = torch.empty(n_send, H, dtype=dt, device=dev)
        back_works = []
        for c in range(C):
            for w in works[c]:
                if w is not None:
                    w.wait()
            if c == 0:
                mark("rows_arrived")
            rm = recv_meta[c]
            eid = rm[:, :, 0].contiguous()                      # [rows, P], -1 = padding
            wgt = rm[:, :, 1].contiguous().view(torch.float32)  # [rows, P] w * a
            y_loc = be.moe_forward(recv_x[c], local_router, self.w_gate, self.w_up, self.w_down, None,
                                   None, None, P, False, want_probs=False, topk=[eid, wgt],
                                   max_ctas=max_ctas)["y"]
            back_works.append(self._exchange(back[send_off[c]:send_off[c + 1]], y_loc, sc[c], rc[c],
                                             async_op=True))
        mark("experts_done")
        for w in back_works:
            if w is not None:
                w.wait()
        mark("rows_returned")

        # 6: fold the returned rows and the shared term
        if side is not None:
            cur = torch.cuda.current_stream(dev)
            cur.wait_stream(side)
            y_shared.record_stream(cur)
        y = be.ep_combine(back, d["pair_slot"], k, y_shared=y_shared, num_tokens=xf.shape[0])
        mark("combined")
        if marks is not None:
            self.phase_events.append(marks)
        return y.view(shp)
