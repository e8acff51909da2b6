"""Drop-in ``ChronosMOEFeedForward`` whose arithmetic runs in the sm_100a kernels.

Mirrors ``chronos/model/moe_chronos.py`` of FonaTech/Project_Chronos:

* same constructor argument (a Chronos/MiniMind config), same submodules and
  parameter shapes (``gate``, ``experts[e].{gate,up,down}_proj``,
  ``shared_experts[j].*``), so ``state_dict`` keys load unchanged
  (``chronos/io/expert_store.py:233-243``);
* ``forward(x [B,S,H], available_expert_mask=None) -> [B,S,H]`` with the
  reference's semantics for both branches (``moe_chronos.py:146-188`` and
  ``:190-279``): placeholder (``LazyExpertPlaceholder``) experts and, in
  training, mask-off experts are served by the shared-expert fallback; in eval
  a live expert runs even when the mask calls it unavailable
  (``moe_chronos.py:222-227``);
* side effects kept: ``last_router_probs``, ``last_router_probs_grad``,
  ``aux_loss``, ``aux_loss_raw``, ``last_on_demand_experts``,
  ``last_fallback_experts``, ``last_on_demand_weight_mass``,
  ``last_fallback_weight_mass``; runtime hooks ``runtime_miss_policy``,
  ``runtime_on_demand_loader``, ``runtime_touch_expert`` (set by the
  reference's inference engine, ``inference_engine.py:118-173``) are called in
  ascending expert order for the selected experts, as the reference does.

Fast path (no hooks installed): one C-ABI call, no host synchronisation; the
bookkeeping lists are computed lazily from device tensors the first time they
are read.  Hook path: routing runs first, the selected experts are read back
once (one sync instead of the reference's two per expert), the hooks run, and
the expert GEMMs run with the resulting availability.

Expert weights live in stacked per-layer pools (``[E, F, H]``, ``[E, F, H]``,
``[E, H, F]``); each expert's ``nn.Linear.weight`` is re-bound as a view into
its pool slot, so ``load_state_dict`` writes straight into the layout the
kernels read with TMA.  Modules swapped in later (``ExpertStore`` promoting a
placeholder) are adopted into the pool on the next forward.

There is no CPU implementation: CPU inputs raise.  Backward is not
implemented (training-mode forward with autograd enabled raises).
"""
from __future__ import annotations

from typing import List, Optional

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops


def _act_fn(name: str):
    if name in ("silu", "swish"):
        return F.silu
    raise ValueError(f"hidden_act={name!r}: the fused kernels implement SwiGLU with silu only")


class FeedForward(nn.Module):
    """Bias-free SwiGLU expert with minimind's parameter names
    (``gate_proj``, ``up_proj``, ``down_proj``), restated at
    ``chronos/mlx/moe.py:13-23``.  Its own ``forward`` (used only when called
    directly, never by ``ChronosMOEFeedForward``) is the plain torch math."""

    def __init__(self, config, intermediate_size: Optional[int] = None):
        super().__init__()
        inter = intermediate_size if intermediate_size is not None else config.intermediate_size
        self.gate_proj = nn.Linear(config.hidden_size, inter, bias=False)
        self.down_proj = nn.Linear(inter, config.hidden_size, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, inter, bias=False)
        self.dropout = nn.Dropout(getattr(config, "dropout", 0.0))
        self.act_fn = _act_fn(getattr(config, "hidden_act", "silu"))

    def forward(self, x):
        return self.dropout(self.down_proj(self.act_fn(self.gate_proj(x)) * self.up_proj(x)))


class LazyExpertPlaceholder(nn.Module):
    """Parameter-free stand-in for an expert that is not resident
    (``moe_chronos.py:13-29``); raises if executed."""

    def __init__(self, hidden_size: int, intermediate_size: int, dtype: torch.dtype):
        super().__init__()
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.dtype = dtype
        self.loaded = False

    def forward(self, _x):
        raise RuntimeError("lazy expert placeholder executed before materialization")


def _is_placeholder(m: nn.Module) -> bool:
    # any parameter-free module is a placeholder, including the reference's own class
    if isinstance(m, LazyExpertPlaceholder):
        return True
    if type(m).__name__ == "LazyExpertPlaceholder":
        return True
    return next(m.parameters(recurse=True), None) is None


class _ExpertList(nn.ModuleList):
    """ModuleList that tells its owner when an expert module is swapped."""

    def __init__(self, modules, owner_ref):
        super().__init__(modules)
        object.__setattr__(self, "_owner_ref", owner_ref)

    def __setitem__(self, idx, module):
        super().__setitem__(idx, module)
        owner = self._owner_ref()
        if owner is not None:
            owner._pool_dirty = True


class ChronosMOEFeedForward(nn.Module):
    def __init__(self, config):
        super().__init__()
        import weakref

        self.config = config
        self.num_experts = config.num_experts
        self.num_experts_per_tok = config.num_experts_per_tok
        self.norm_topk_prob = config.norm_topk_prob
        self.router_aux_loss_coef = config.router_aux_loss_coef
        _act_fn(getattr(config, "hidden_act", "silu"))

        self.gate = nn.Linear(config.hidden_size, config.num_experts, bias=False)
        self.experts = _ExpertList([
            FeedForward(config, intermediate_size=config.moe_intermediate_size)
            for _ in range(config.num_experts)
        ], weakref.ref(self))
        self.shared_experts = nn.ModuleList([
            FeedForward(config, intermediate_size=config.moe_intermediate_size)
            for _ in range(getattr(config, "num_shared_experts", 1))
        ])
        self.aux_loss = torch.zeros(1)
        self.aux_loss_raw: Optional[torch.Tensor] = None
        self.last_router_probs: Optional[torch.Tensor] = None
        self.last_router_probs_grad: Optional[torch.Tensor] = None
        self.fallback_mask_prob = float(getattr(config, "fallback_mask_prob", 0.0))
        self.runtime_miss_policy = "fallback_diagnostic"
        self.runtime_on_demand_loader = None
        self.runtime_touch_expert = None
        self._stats_pending = None
        self._last_on_demand_experts: List[int] = []
        self._last_fallback_experts: List[int] = []
        self._last_on_demand_weight_mass = 0.0
        self._last_fallback_weight_mass = 0.0
        # Benchmark knob: fp32 [E] offset added to the router logits (None in models).
        self.router_logit_bias: Optional[torch.Tensor] = None
        # How an eval-time mask is read.  "reference": as moe_chronos.py:221-227
        # (a live expert runs even where the mask says unavailable; only
        # placeholders fall back).  "residency": the mask names the experts that
        # are resident, a_e = mask_e (the blend of chronos/mlx/moe.py:160-166), as a
        # pooled store whose non-resident experts are placeholders behaves; a CUDA
        # mask is then applied on the device without a host read, so the call can
        # be captured in a CUDA graph.
        self.mask_semantics = "reference"
        # Expert residency (set by a pooled ExpertStore): per-expert device ready
        # flags the GEMMs wait on for selected experts only.
        self.expert_ready_flags: Optional[torch.Tensor] = None
        self.expert_ready_epoch: int = 0
        self.expert_ready_timeout_ns: int = 0
        self._pool = None
        self._pool_dirty = True
        self._live_np = None
        self._avail_cache = {}
        # Slot pools owned by a pooled ExpertStore (attach_expert_pool), or None.
        self._ext_pool = None
        # bound fast-path call (ops.LayerCall) and the key of what it was bound to
        self._call = None
        self._call_key = None
        self._eval_zero: Optional[torch.Tensor] = None
        self._has_placeholder = None  # (live array, any placeholder in it)

    # ------------------------------------------------------------------
    # bookkeeping attributes (lazy: resolved from device tensors on read)
    # ------------------------------------------------------------------
    def _resolve_stats(self):
        pend = self._stats_pending
        if pend is None:
            return
        self._stats_pending = None
        counts = pend["counts"].cpu().numpy()
        mass = pend["mass"].cpu().numpy().astype(np.float64)
        if isinstance(pend["a"], torch.Tensor):  # availability built on the device
            pend = dict(pend, a=pend["a"].cpu().numpy())
        od, fb = [], []
        odm = fbm = 0.0
        for e in range(self.num_experts):
            if counts[e] <= 0:
                continue
            if pend["a"][e] > 0.0:
                if pend["on_demand"][e]:
                    od.append(e)
                    odm += float(mass[e])
            else:
                fb.append(e)
                fbm += float(mass[e])
        self._last_on_demand_experts = od
        self._last_fallback_experts = fb
        self._last_on_demand_weight_mass = odm
        self._last_fallback_weight_mass = fbm

    def _stat_prop(name):  # noqa: N805 - property factory
        def getter(self):
            self._resolve_stats()
            return getattr(self, "_" + name)

        def setter(self, v):
            self._stats_pending = None
            setattr(self, "_" + name, v)

        return property(getter, setter)

    last_on_demand_experts = _stat_prop("last_on_demand_experts")
    last_fallback_experts = _stat_prop("last_fallback_experts")
    last_on_demand_weight_mass = _stat_prop("last_on_demand_weight_mass")
    last_fallback_weight_mass = _stat_prop("last_fallback_weight_mass")
    del _stat_prop

    @classmethod
    def from_stacked(cls, config, router: torch.Tensor, gate: torch.Tensor, up: torch.Tensor,
                     down: torch.Tensor, sh_gate: Optional[torch.Tensor] = None,
                     sh_up: Optional[torch.Tensor] = None,
                     sh_down: Optional[torch.Tensor] = None) -> "ChronosMOEFeedForward":
        """Build a layer around already-stacked weights (no copy): gate/up
        ``[E, F, H]``, down ``[E, H, F]``, shared ``[S, ...]``; the per-expert
        parameters become views of these tensors."""
        with torch.device("meta"):
            m = cls(config)
        dev, dt = gate.device, gate.dtype
        S = len(m.shared_experts)
        pool = dict(gate=gate, up=up, down=down,
                    sh_gate=sh_gate if S else None, sh_up=sh_up if S else None,
                    sh_down=sh_down if S else None)
        m.gate.weight = nn.Parameter(router, requires_grad=False)
        for e, ex in enumerate(m.experts):
            ex.gate_proj.weight = nn.Parameter(gate[e], requires_grad=False)
            ex.up_proj.weight = nn.Parameter(up[e], requires_grad=False)
            ex.down_proj.weight = nn.Parameter(down[e], requires_grad=False)
        for j, ex in enumerate(m.shared_experts):
            ex.gate_proj.weight = nn.Parameter(sh_gate[j], requires_grad=False)
            ex.up_proj.weight = nn.Parameter(sh_up[j], requires_grad=False)
            ex.down_proj.weight = nn.Parameter(sh_down[j], requires_grad=False)
        m._pool = pool
        m._sync_pool(dev, dt)
        return m

    def attach_expert_pool(self, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
                           slot_of_expert: torch.Tensor, slot_host: np.ndarray,
                           ready_flags: Optional[torch.Tensor] = None,
                           ready_timeout_ns: int = 0) -> None:
        """Serve the routed experts from slot pools owned by an expert store.

        gate/up ``[P, F, H]``, down ``[P, H, F]``: P resident slots.
        ``slot_of_expert`` (device int32 ``[E]``) and ``slot_host`` (the store's
        host copy) map expert -> slot, -1 = not resident.  ``ready_flags``
        (device int32 ``[E]``, this layer's row) is 1 once the slot's copy of
        the expert has landed; the GEMMs wait on it for selected experts only.
        Expert modules stay ``experts[e]`` (live views of their slot, or
        placeholders), so the reference's residency checks keep working."""
        self._ext_pool = dict(gate=gate, up=up, down=down, slot=slot_of_expert, slot_host=slot_host)
        self.expert_ready_flags = ready_flags
        self.expert_ready_epoch = 1 if ready_flags is not None else 0
        self.expert_ready_timeout_ns = int(ready_timeout_ns)
        self._pool_dirty = True

    def detach_expert_pool(self) -> None:
        self._ext_pool = None
        self._pool = None
        self.expert_ready_flags = None
        self.expert_ready_epoch = 0
        self._pool_dirty = True

    # ------------------------------------------------------------------
    def _apply(self, fn, *args, **kwargs):
        self._pool_dirty = True
        return super()._apply(fn, *args, **kwargs)

    def _shared_expert_output(self, x_flat: torch.Tensor) -> torch.Tensor:
        """Average output of all shared experts (``moe_chronos.py:90-93``)."""
        out = sum(e(x_flat) for e in self.shared_experts)
        return out / len(self.shared_experts)

    def _sync_pool(self, device: torch.device, dtype: torch.dtype) -> None:
        """Adopt every live expert's weights into the stacked pools (views)."""
        E = self.num_experts
        H = self.config.hidden_size
        Fd = self.config.moe_intermediate_size
        S = len(self.shared_experts)
        ext = self._ext_pool
        if ext is not None:
            self._sync_ext_pool(ext, device, dtype)
            return
        pool = self._pool
        if pool is None or pool.get("slot") is not None or pool["gate"].device != device \
                or pool["gate"].dtype != dtype:
            pool = dict(
                gate=torch.empty(E, Fd, H, device=device, dtype=dtype),
                up=torch.empty(E, Fd, H, device=device, dtype=dtype),
                down=torch.empty(E, H, Fd, device=device, dtype=dtype),
                sh_gate=torch.empty(S, Fd, H, device=device, dtype=dtype) if S else None,
                sh_up=torch.empty(S, Fd, H, device=device, dtype=dtype) if S else None,
                sh_down=torch.empty(S, H, Fd, device=device, dtype=dtype) if S else None,
            )
            self._pool = pool
        live = np.zeros(E, dtype=np.float32)

        def adopt(mod, names_pools, idx):
            for name, pt in names_pools:
                lin = getattr(mod, name)
                wt = lin.weight
                dst = pt[idx]
                if wt.data_ptr() != dst.data_ptr() or wt.shape != dst.shape:
                    if tuple(wt.shape) != tuple(dst.shape):
                        raise RuntimeError(f"expert weight {name} has shape {tuple(wt.shape)}, "
                                           f"expected {tuple(dst.shape)}")
                    with torch.no_grad():
                        dst.copy_(wt.detach())
                    lin.weight = nn.Parameter(dst, requires_grad=wt.requires_grad)

        for e, ex in enumerate(self.experts):
            if _is_placeholder(ex):
                continue
            live[e] = 1.0
            adopt(ex, (("gate_proj", pool["gate"]), ("up_proj", pool["up"]),
                       ("down_proj", pool["down"])), e)
        for j, ex in enumerate(self.shared_experts):
            adopt(ex, (("gate_proj", pool["sh_gate"]), ("up_proj", pool["sh_up"]),
                       ("down_proj", pool["sh_down"])), j)
        self._live_np = live
        self._avail_cache = {}
        self._pool_dirty = False

    def _sync_ext_pool(self, ext, device: torch.device, dtype: torch.dtype) -> None:
        """Pooled-store mode: routed experts live in the store's slots; shared
        experts are adopted into this layer's own stacked pool."""
        if ext["gate"].device != device or ext["gate"].dtype != dtype:
            raise RuntimeError(f"expert slot pool is {ext['gate'].dtype} on {ext['gate'].device}, "
                               f"input is {dtype} on {device}")
        E = self.num_experts
        H = self.config.hidden_size
        Fd = self.config.moe_intermediate_size
        S = len(self.shared_experts)
        old = self._pool or {}
        sh = old.get("sh_gate")
        if S and (sh is None or sh.device != device or sh.dtype != dtype):
            sh_pools = dict(sh_gate=torch.empty(S, Fd, H, device=device, dtype=dtype),
                            sh_up=torch.empty(S, Fd, H, device=device, dtype=dtype),
                            sh_down=torch.empty(S, H, Fd, device=device, dtype=dtype))
        else:
            sh_pools = dict(sh_gate=old.get("sh_gate"), sh_up=old.get("sh_up"),
                            sh_down=old.get("sh_down"))
        for j, ex in enumerate(self.shared_experts):
            for name, key in (("gate_proj", "sh_gate"), ("up_proj", "sh_up"), ("down_proj", "sh_down")):
                lin = getattr(ex, name)
                dst = sh_pools[key][j]
                if lin.weight.data_ptr() != dst.data_ptr():
                    with torch.no_grad():
                        dst.copy_(lin.weight.detach())
                    lin.weight = nn.Parameter(dst, requires_grad=lin.weight.requires_grad)
        slot_host = ext["slot_host"]
        live = np.zeros(E, dtype=np.float32)
        for e, ex in enumerate(self.experts):
            if _is_placeholder(ex):
                continue
            s = int(slot_host[e])
            if s < 0:
                raise RuntimeError(f"expert {e} is live but has no slot in the store's pool")
            for name, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
                lin = getattr(ex, name)
                dst = ext[key][s]
                if lin.weight.data_ptr() != dst.data_ptr():
                    if tuple(lin.weight.shape) != tuple(dst.shape):
                        raise RuntimeError(f"expert weight {name} has shape {tuple(lin.weight.shape)}, "
                                           f"expected {tuple(dst.shape)}")
                    with torch.no_grad():
                        dst.copy_(lin.weight.detach())
                    lin.weight = nn.Parameter(dst, requires_grad=False)
            live[e] = 1.0
        self._pool = dict(gate=ext["gate"], up=ext["up"], down=ext["down"], slot=ext["slot"],
                          **sh_pools)
        self._live_np = live
        self._avail_cache = {}
        self._pool_dirty = False

    def _layer_call(self, pool, bias) -> "ops.LayerCall":
        """The bound fast-path call for the current weights (rebuilt when any of
        them, the router bias or the readiness settings change)."""
        w = self.gate.weight
        key = (w.data_ptr(), w.dtype, pool["gate"].data_ptr(), pool["up"].data_ptr(),
               pool["down"].data_ptr(), None if pool["sh_gate"] is None else pool["sh_gate"].data_ptr(),
               None if bias is None else (bias.data_ptr(), bias._version),
               None if pool.get("slot") is None else pool["slot"].data_ptr(),
               None if self.expert_ready_flags is None else self.expert_ready_flags.data_ptr(),
               self.expert_ready_epoch, self.expert_ready_timeout_ns, bool(self.norm_topk_prob))
        if self._call_key != key:
            self._call = ops.LayerCall(
                w, pool["gate"], pool["up"], pool["down"], pool["sh_gate"], pool["sh_up"], pool["sh_down"],
                self.num_experts_per_tok, bool(self.norm_topk_prob), router_bias=bias,
                slot_of_expert=pool.get("slot"), ready_flags=self.expert_ready_flags,
                ready_epoch=self.expert_ready_epoch, spin_limit_ns=self.expert_ready_timeout_ns)
            self._call_key = key
        return self._call

    def _avail_tensor(self, a: np.ndarray, device) -> torch.Tensor:
        key = (a.tobytes(), str(device))
        t = self._avail_cache.get(key)
        if t is None:
            t = torch.from_numpy(a.astype(np.float32)).to(device, non_blocking=False)
            if len(self._avail_cache) > 64:
                self._avail_cache = {}
            self._avail_cache[key] = t
        return t

    # ------------------------------------------------------------------
    def forward(self, x: torch.Tensor, available_expert_mask: Optional[torch.Tensor] = None
                ) -> torch.Tensor:
        return self._forward(x, available_expert_mask, acc_out=False)

    def forward_acc(self, x: torch.Tensor, available_expert_mask: Optional[torch.Tensor] = None
                    ) -> torch.Tensor:
        """``forward`` whose result is the layer's fp32 accumulator, not yet rounded
        to the layer dtype (CHRONOS_FLAG_ACC_OUT: no finalize pass), for a caller
        whose next kernel reads it and rounds it (``ops.add_rmsnorm`` with an fp32
        x).  Calls that take the host-hook path return ``forward``'s output in the
        layer dtype; the caller accepts either."""
        return self._forward(x, available_expert_mask, acc_out=True)

    def _forward(self, x: torch.Tensor, available_expert_mask: Optional[torch.Tensor], acc_out: bool
                 ) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("ChronosMOEFeedForward (sm_100a kernels) needs CUDA tensors; "
                               f"got x on {x.device}")
        if self.training and torch.is_grad_enabled():
            raise NotImplementedError(
                "ChronosMOEFeedForward runs forward-only kernels; backward is not implemented "
                "(call it under torch.no_grad() or in eval mode)")
        B, S, H = x.shape
        E = self.num_experts
        k = self.num_experts_per_tok
        x_flat = x.reshape(-1, H)
        dev, dt = x.device, x.dtype
        if self._pool_dirty or self._pool is None or self._pool["gate"].device != dev:
            self._sync_pool(dev, dt)
        pool = self._pool
        live = self._live_np
        # per-call bookkeeping: plain attributes (never parameters, buffers or
        # submodules), written past nn.Module.__setattr__'s type checks, which
        # cost more host time than the kernels of a one-token call
        _set = object.__setattr__
        _set(self, "_stats_pending", None)
        _set(self, "_last_on_demand_experts", [])
        _set(self, "_last_fallback_experts", [])
        _set(self, "_last_on_demand_weight_mass", 0.0)
        _set(self, "_last_fallback_weight_mass", 0.0)

        training_fallback_mask = None
        if (available_expert_mask is None and self.training and self.fallback_mask_prob > 0.0
                and len(self.shared_experts) > 0):
            keep = torch.rand(self.num_experts, device=dev) >= self.fallback_mask_prob
            if not torch.any(keep):
                keep[torch.randint(0, self.num_experts, (1,), device=dev)] = True
            training_fallback_mask = keep

        masked = available_expert_mask is not None or training_fallback_mask is not None
        mask_t = available_expert_mask if available_expert_mask is not None else training_fallback_mask
        eval_with_mask = available_expert_mask is not None and not self.training
        hp = self._has_placeholder
        if hp is None or hp[0] is not live:  # recomputed only when the pool was re-synced
            hp = (live, bool((live == 0).any()))
            _set(self, "_has_placeholder", hp)
        has_placeholder = hp[1]
        touch = getattr(self, "runtime_touch_expert", None)
        loader = getattr(self, "runtime_on_demand_loader", None)
        policy = getattr(self, "runtime_miss_policy", "fallback_diagnostic")
        loader_active = (eval_with_mask and loader is not None
                         and policy in {"on_demand", "sync_on_demand"} and has_placeholder)
        touch_active = eval_with_mask and touch is not None
        standard_with_placeholder = (not masked) and has_placeholder

        mask_np = None
        if masked and not eval_with_mask:
            # training with a mask: a_e = live and mask > 0 (moe_chronos.py:221, 227)
            if mask_t.is_cuda:
                avail_dev = (mask_t.to(torch.float32) > 0).to(torch.float32) * \
                    torch.from_numpy(live).to(dev)
            else:
                mask_np = np.array(mask_t.detach().to(torch.float32).numpy(), copy=True)
                avail_dev = None
        if masked and available_expert_mask is not None and not available_expert_mask.is_cuda:
            # a snapshot: the statistics read later must see the mask of this call
            mask_np = np.array(available_expert_mask.detach().to(torch.float32).numpy(), copy=True)

        bias = self.router_logit_bias
        probs = None
        if touch_active or loader_active or standard_with_placeholder:
            # ---- hook path: route, read back the selected experts once ----
            r = ops.moe_route(x_flat, self.gate.weight, k, bool(self.norm_topk_prob),
                              num_shared=len(self.shared_experts),
                              ffn=self.config.moe_intermediate_size, router_bias=bias)
            probs = r["probs"]
            counts = r["counts"].cpu().numpy()
            mass = r["mass"].cpu().numpy().astype(np.float64)
            if mask_np is None and mask_t is not None:
                mask_np = mask_t.detach().to(torch.float32).cpu().numpy()
            a = np.ones(E, dtype=np.float32)
            od, fb = [], []
            odm = fbm = 0.0
            topk = [r["topk_idx"], r["topk_weight"]]
            # A pooled store smaller than this call's set of experts: loading
            # into a full pool evicts, possibly an expert this call already
            # counts on.  Then the experts are computed in passes (routed only)
            # before each such load, as the reference computes each expert
            # before loading the next (moe_chronos.py:228-254), and the shared
            # term is added once at the end with the fallback weights.
            state = dict(chunk=[], y=None, pool=pool)

            def pool_full() -> bool:
                ext = self._ext_pool
                return ext is not None and \
                    int((ext["slot_host"] >= 0).sum()) >= int(ext["gate"].shape[0])

            def routed_pass(experts) -> torch.Tensor:
                if self._pool_dirty:
                    self._sync_pool(dev, dt)
                    state["pool"] = self._pool
                pl = state["pool"]
                a_c = np.zeros(E, dtype=np.float32)
                a_c[experts] = 1.0
                o = ops.moe_forward(
                    x_flat, self.gate.weight, pl["gate"], pl["up"], pl["down"], None, None, None, k,
                    bool(self.norm_topk_prob), avail=self._avail_tensor(a_c, dev), router_bias=bias,
                    slot_of_expert=pl.get("slot"), ready_flags=self.expert_ready_flags,
                    ready_epoch=self.expert_ready_epoch, spin_limit_ns=self.expert_ready_timeout_ns,
                    want_probs=False, topk=topk)
                return o["y"].float()

            def flush() -> None:
                if state["chunk"]:
                    yc = routed_pass(state["chunk"])
                    state["y"] = yc if state["y"] is None else state["y"] + yc
                    state["chunk"] = []

            for i in range(E):
                if counts[i] <= 0:
                    continue
                if not masked:
                    if live[i] == 0:
                        raise RuntimeError("lazy expert placeholder executed before materialization")
                    continue
                expert_live = not _is_placeholder(self.experts[i])
                expert_available = float(mask_np[i]) > 0.0
                stale = eval_with_mask and expert_live
                if expert_live and (expert_available or stale):
                    if touch is not None and not self.training:
                        touch(int(i))
                    if not expert_available and eval_with_mask:
                        od.append(i)
                        odm += float(mass[i])
                    a[i] = 1.0
                    state["chunk"].append(i)
                else:
                    loaded = False
                    if eval_with_mask and policy in {"on_demand", "sync_on_demand"} and loader is not None:
                        if state["chunk"] and pool_full():
                            flush()
                        res = loader(int(i))
                        loaded = bool(res.get("ok", False)) if isinstance(res, dict) else bool(res)
                    if loaded and not _is_placeholder(self.experts[i]):
                        od.append(i)
                        odm += float(mass[i])
                        a[i] = 1.0
                        state["chunk"].append(i)
                    else:
                        fb.append(i)
                        fbm += float(mass[i])
                        a[i] = 0.0
            if self._pool_dirty:
                # the loader promoted experts: adopt the new modules into the pool
                self._sync_pool(dev, dt)
            pool = self._pool
            if state["y"] is None:
                out = ops.moe_forward(
                    x_flat, self.gate.weight, pool["gate"], pool["up"], pool["down"],
                    pool["sh_gate"], pool["sh_up"], pool["sh_down"], k, bool(self.norm_topk_prob),
                    avail=self._avail_tensor(a, dev), router_bias=bias,
                    slot_of_expert=pool.get("slot"),
                    ready_flags=self.expert_ready_flags, ready_epoch=self.expert_ready_epoch,
                    spin_limit_ns=self.expert_ready_timeout_ns, want_probs=False, topk=topk)
            else:
                flush()
                y_acc = state["y"]
                if len(self.shared_experts) > 0:
                    # shared term once: (1 + sum of the fallback selections' weights) * S(x)
                    fb_t = torch.zeros(E, dtype=torch.float32, device=dev)
                    if fb:
                        fb_t[torch.tensor(fb, device=dev)] = 1.0
                    w_fb = (r["topk_weight"] * fb_t[r["topk_idx"].long()]).contiguous()
                    o = ops.moe_forward(
                        x_flat, self.gate.weight, pool["gate"], pool["up"], pool["down"],
                        pool["sh_gate"], pool["sh_up"], pool["sh_down"], k,
                        bool(self.norm_topk_prob), avail=self._avail_tensor(np.zeros(E, np.float32), dev),
                        router_bias=bias, slot_of_expert=pool.get("slot"), want_probs=False,
                        topk=[r["topk_idx"], w_fb])
                    y_acc = y_acc + o["y"].float()
                out = dict(y=y_acc.to(dt), topk_idx=r["topk_idx"])
            self._last_on_demand_experts = od
            self._last_fallback_experts = fb
            self._last_on_demand_weight_mass = odm
            self._last_fallback_weight_mass = fbm
        else:
            # ---- fast path: one call, no host synchronisation ----
            on_demand = _NO_ON_DEMAND
            avail_is_mask = False
            if not masked:
                a_np = None
                avail_t = None
            elif eval_with_mask and self.mask_semantics == "residency":
                # the mask names the resident experts: a_e = mask_e for live experts
                # (a CUDA mask is applied on the device, with no host read)
                if mask_np is not None:
                    a_np = ((mask_np > 0.0) & (live > 0)).astype(np.float32)
                    avail_t = self._avail_tensor(a_np, dev)
                elif not has_placeholder:
                    # every expert live: the kernels threshold the mask themselves
                    # (one snapshot copy instead of three elementwise passes)
                    a_np = None
                    m = available_expert_mask.detach()
                    avail_t = (m.clone() if m.dtype == torch.float32 else m.to(torch.float32)).contiguous()
                    avail_is_mask = True
                else:
                    a_np = None
                    avail_t = (available_expert_mask.to(torch.float32) > 0).to(torch.float32) * \
                        self._avail_tensor(live, dev)
            elif eval_with_mask:
                a_np = live.copy()  # live experts run even when marked unavailable
                if mask_np is not None:
                    on_demand = _LazyOnDemand(mask_np, live)  # built when the statistics are read
                avail_t = self._avail_tensor(a_np, dev)
            else:
                if mask_np is not None:
                    a_np = ((mask_np > 0.0) & (live > 0)).astype(np.float32)
                    avail_t = self._avail_tensor(a_np, dev)
                else:
                    a_np = None
                    avail_t = avail_dev
            out = self._layer_call(pool, bias)(x_flat, avail=avail_t, want_probs=True,
                                               want_stats=masked, want_topk=self.training,
                                               avail_is_mask=avail_is_mask, acc_out=acc_out)
            probs = out["probs"]
            if masked:
                if a_np is None:
                    a_np = avail_t  # read back only when the statistics are read
                if eval_with_mask and self.mask_semantics == "residency":
                    _set(self, "_stats_pending", dict(counts=out["counts"], mass=out["mass"], a=a_np,
                                                      on_demand=_NO_ON_DEMAND))
                elif eval_with_mask and mask_np is None:
                    # CUDA mask in eval: read lazily together with the counts
                    _set(self, "_stats_pending", dict(
                        counts=out["counts"], mass=out["mass"], a=a_np,
                        on_demand=_LazyOnDemand(available_expert_mask.detach().clone(), live)))
                else:
                    _set(self, "_stats_pending", dict(counts=out["counts"], mass=out["mass"], a=a_np,
                                                      on_demand=on_demand))

        y = out["y"]
        scores_bse = probs.view(B, S, E)
        _set(self, "last_router_probs_grad", scores_bse)
        _set(self, "last_router_probs", scores_bse.detach())
        if self.training:
            topk_idx = out["topk_idx"].long()
            load = torch.bincount(topk_idx.reshape(-1), minlength=E).float() / max(1, x_flat.shape[0])
            aux_raw = (load * probs.float().mean(0)).sum() * E
            _set(self, "aux_loss_raw", aux_raw)
            _set(self, "aux_loss", aux_raw * self.router_aux_loss_coef)
        else:
            # eval: a zero scalar on the layer's device, made once and reused (a
            # fresh one per call is a device fill per call)
            z = self._eval_zero
            if z is None or z.device != probs.device or z.dtype != probs.dtype:
                z = probs.new_zeros(())
                _set(self, "_eval_zero", z)
            _set(self, "aux_loss_raw", z)
            _set(self, "aux_loss", z)
        return y.view(B, S, H)


class _LazyOnDemand:
    """on_demand[e] = mask[e] <= 0 and live[e], computed on first use (from a host
    array, or read back from a CUDA mask)."""

    def __init__(self, mask, live: np.ndarray):
        self.mask = mask
        self.live = live
        self._v = None

    def __getitem__(self, e):
        if self._v is None:
            m = self.mask
            if isinstance(m, torch.Tensor):
                m = m.detach().to(torch.float32).cpu().numpy()
            self._v = (m <= 0.0) & (self.live > 0)
        return self._v[e]


class _NoOnDemand:
    """on_demand[e] = False for every e (calls without an eval-time mask)."""

    def __getitem__(self, e):
        return False


_NO_ON_DEMAND = _NoOnDemand()

