"""Torch-facing calls of the sm_100a MoE extension.

``moe_forward`` / ``moe_route`` take CUDA tensors, allocate the outputs and
the workspace through torch's caching allocator, and call the C ABI on the
current CUDA stream.  They never fall back to another implementation: a CPU
tensor, a missing library or a failing call raises.

``moe_forward`` is also registered as the custom op ``chronos::moe_forward``
(with a fake implementation) so ``torch.compile`` traces the whole layer as
one node.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional

import torch

from . import _native as N

_DTYPES = {torch.bfloat16: N.DTYPE_BF16, torch.float16: N.DTYPE_FP16, torch.float32: N.DTYPE_FP32}

_status_words: Dict[int, torch.Tensor] = {}


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def status_word(device: torch.device) -> torch.Tensor:
    """Persistent per-device int32 word the kernels report device-side failures in."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = w
    return w


def check_status(device: Optional[torch.device] = None, reset: bool = True) -> int:
    """Synchronise, read the device status word, raise on a recorded failure."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    w = status_word(device)
    code = int(w.item())
    if reset and code:
        w.zero_()
    if code:
        raise N.ChronosMoeError(code, "device-side failure recorded by a MoE kernel")
    return code


def _check_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("chronos MoE kernels need CUDA tensors (no CPU path exists); "
                               f"got a tensor on {t.device}")


def _contig(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    return None if t is None else t.contiguous()


def _shape(n: int, h: int, e: int, k: int, f: int, s: int, dtype: torch.dtype) -> N.ChronosMoeShape:
    if dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {dtype}")
    return N.ChronosMoeShape(n, h, e, k, f, s, _DTYPES[dtype])


def workspace_bytes(n: int, h: int, e: int, k: int, f: int, s: int, dtype: torch.dtype) -> int:
    lib = N.load_library()
    shp = _shape(n, h, e, k, f, s, dtype)
    size = lib.chronos_moe_workspace_size(ctypes.byref(shp))
    if size == 0 and n >= 0:
        N.check(N.CHRONOS_ERR_INVALID_ARG)
    return int(size)


def moe_forward(x: torch.Tensor, router_w: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
                w_down: torch.Tensor, sh_gate: Optional[torch.Tensor], sh_up: Optional[torch.Tensor],
                sh_down: Optional[torch.Tensor], top_k: int, norm_topk: bool,
                avail: Optional[torch.Tensor] = None, router_bias: Optional[torch.Tensor] = None,
                slot_of_expert: Optional[torch.Tensor] = None,
                ready_flags: Optional[torch.Tensor] = None, ready_epoch: int = 0,
                spin_limit_ns: int = 0, want_probs: bool = True, want_stats: bool = False,
                topk: Optional[List[torch.Tensor]] = None, status: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None,
                max_ctas: int = 0):
    """One MoE layer.  x [N, H]; router_w [E, H]; w_gate/w_up [P, F, H]; w_down [P, H, F];
    sh_* [S, F, H] / [S, H, F] (or None when S = 0); avail [E] fp32 in [0, 1].

    ``topk`` = [topk_idx int32 [N,k], topk_weight fp32 [N,k]] from an earlier
    ``moe_route`` call skips routing (the host-hook slow path).

    Returns dict(y, probs, topk_idx, topk_weight, counts, mass); probs/counts/mass
    are None unless requested.
    """
    _check_cuda(x, router_w, w_gate, w_up, w_down, sh_gate, sh_up, sh_down, avail, router_bias,
                slot_of_expert, ready_flags)
    x = x.contiguous()
    n, h = x.shape
    e = router_w.shape[0]
    p_slots, f, _ = w_gate.shape
    s = 0 if sh_gate is None else sh_gate.shape[0]
    dt = x.dtype
    for name, t in (("router_w", router_w), ("w_gate", w_gate), ("w_up", w_up), ("w_down", w_down),
                    ("sh_gate", sh_gate), ("sh_up", sh_up), ("sh_down", sh_down)):
        if t is not None and t.dtype != dt:
            raise TypeError(f"{name} dtype {t.dtype} != x dtype {dt}")
    dev = x.device
    lib = N.load_library()
    shp = _shape(n, h, e, top_k, f, s, dt)
    ws_bytes = int(lib.chronos_moe_workspace_size(ctypes.byref(shp)))
    if ws_bytes == 0 and n > 0:
        N.check(N.CHRONOS_ERR_INVALID_ARG)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    y = out if out is not None else torch.empty(n, h, dtype=dt, device=dev)
    probs = torch.empty(n, e, dtype=dt, device=dev) if want_probs else None
    if topk is not None:
        topk_idx, topk_w = topk
        flags = N.FLAG_PREROUTED
    else:
        topk_idx = torch.empty(n, top_k, dtype=torch.int32, device=dev)
        topk_w = torch.empty(n, top_k, dtype=torch.float32, device=dev)
        flags = 0
    counts = torch.empty(e, dtype=torch.int32, device=dev) if want_stats else None
    mass = torch.empty(e, dtype=torch.float32, device=dev) if want_stats else None
    if status is None:
        status = status_word(dev)
    w_gate, w_up, w_down = w_gate.contiguous(), w_up.contiguous(), w_down.contiguous()
    sh_gate, sh_up, sh_down = _contig(sh_gate), _contig(sh_up), _contig(sh_down)
    router_w = router_w.contiguous()
    avail = None if avail is None else avail.to(device=dev, dtype=torch.float32).contiguous()
    rb = None if router_bias is None else router_bias.to(device=dev, dtype=torch.float32).contiguous()
    args = N.ChronosMoeArgs(
        shape=shp, norm_topk=int(bool(norm_topk)), flags=flags,
        x=_ptr(x), router_w=_ptr(router_w), router_bias=_ptr(rb),
        w_gate=_ptr(w_gate), w_up=_ptr(w_up), w_down=_ptr(w_down), pool_slots=int(p_slots),
        slot_of_expert=_ptr(slot_of_expert), w_shared_gate=_ptr(sh_gate),
        w_shared_up=_ptr(sh_up), w_shared_down=_ptr(sh_down), avail=_ptr(avail),
        ready_flags=_ptr(ready_flags), ready_epoch=int(ready_epoch),
        spin_limit_ns=int(spin_limit_ns), y=_ptr(y), router_probs=_ptr(probs),
        topk_idx=_ptr(topk_idx), topk_weight=_ptr(topk_w), expert_counts=_ptr(counts),
        expert_mass=_ptr(mass), workspace=_ptr(workspace), workspace_bytes=int(workspace.numel()),
        status=_ptr(status), max_ctas=int(max_ctas))
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        N.check(lib.chronos_moe_forward(ctypes.byref(args), ctypes.c_void_p(stream)))
    return dict(y=y, probs=probs, topk_idx=topk_idx, topk_weight=topk_w, counts=counts, mass=mass)


def _raw_stream(index: int) -> int:
    """Handle of the current CUDA stream of device `index` (torch's raw accessor when
    present: a fraction of the host time of building a torch.cuda.Stream)."""
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return raw(index)
    return torch.cuda.current_stream(index).cuda_stream


class _SharedWorkspace:
    """One workspace per (device, stream), shared by every layer that runs there.

    Calls on one stream run one after another, so every layer can use the same
    buffer; it grows to the largest size requested and never shrinks (a
    smaller call uses a prefix: the extension only requires ``workspace_bytes
    >= need``).  A buffer is allocated while its stream is the current stream,
    so when a larger one replaces it the caching allocator hands the old block
    out again only after the work already queued on that stream.  The memory
    held is the workspace of the largest call per stream, e.g. ~0.45 GB for
    8192 tokens of the d_model 2048, 64-expert top-6 layer (~9.4 MB for 64).

    A buffer that a CUDA graph captured is never freed: the graph replays
    into its address, so when it is outgrown it is retired, not released."""

    def __init__(self):
        self._bufs: Dict[tuple, torch.Tensor] = {}
        self._captured: set = set()              # data_ptr of buffers a graph holds
        self._retired: List[torch.Tensor] = []    # outgrown buffers graphs still hold

    def get(self, dev: torch.device, stream: int, nbytes: int) -> torch.Tensor:
        key = (dev.index, stream)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            if buf is not None and buf.data_ptr() in self._captured:
                self._retired.append(buf)
            # round up so that slowly growing token counts do not reallocate every call
            buf = torch.empty(max(256, nbytes + nbytes // 8), dtype=torch.uint8, device=dev)
            self._bufs[key] = buf
        if torch.cuda.is_current_stream_capturing():
            self._captured.add(buf.data_ptr())
        return buf

    def release(self) -> None:
        """Drop the cached buffers no captured graph holds (call when no layer
        call is in flight)."""
        self._bufs = {k: b for k, b in self._bufs.items() if b.data_ptr() in self._captured}


shared_workspace = _SharedWorkspace()


class LayerCall:
    """One layer's static arguments bound once, for repeated calls with little host work.

    ``LayerCall(router_w, w_gate, ...)(x, avail=...)`` computes what
    ``moe_forward`` computes.  The weights, pools, slot map, ready flags and
    router bias are checked and converted once; each call allocates only its
    outputs, takes the workspace shared by all layers on the current stream
    (``shared_workspace``) and copies a prebuilt argument struct.  Rebuild it
    when any bound tensor is replaced."""

    def __init__(self, router_w, w_gate, w_up, w_down, sh_gate, sh_up, sh_down, top_k: int,
                 norm_topk: bool, router_bias=None, slot_of_expert=None, ready_flags=None,
                 ready_epoch: int = 0, spin_limit_ns: int = 0):
        _check_cuda(router_w, w_gate, w_up, w_down, sh_gate, sh_up, sh_down, router_bias, slot_of_expert,
                    ready_flags)
        dt = router_w.dtype
        for name, t in (("w_gate", w_gate), ("w_up", w_up), ("w_down", w_down), ("sh_gate", sh_gate),
                        ("sh_up", sh_up), ("sh_down", sh_down)):
            if t is not None and t.dtype != dt:
                raise TypeError(f"{name} dtype {t.dtype} != router dtype {dt}")
        self.dev = router_w.device
        self.dtype = dt
        self.e = router_w.shape[0]
        self.p_slots, self.f, self.h = w_gate.shape
        self.s = 0 if sh_gate is None else sh_gate.shape[0]
        self.k = int(top_k)
        # keep the (contiguous) tensors alive: the struct holds their addresses
        self._keep = [t.contiguous() if t is not None else None
                      for t in (router_w, w_gate, w_up, w_down, sh_gate, sh_up, sh_down)]
        rb = None if router_bias is None else router_bias.to(device=self.dev, dtype=torch.float32).contiguous()
        self._keep += [rb, slot_of_expert, ready_flags]
        r, g, u, d, sg, su, sd = self._keep[:7]
        self._lib = N.load_library()
        self._tmpl = N.ChronosMoeArgs(
            shape=_shape(0, self.h, self.e, self.k, self.f, self.s, dt), norm_topk=int(bool(norm_topk)),
            flags=0, router_w=_ptr(r), router_bias=_ptr(rb), w_gate=_ptr(g), w_up=_ptr(u), w_down=_ptr(d),
            pool_slots=int(self.p_slots), slot_of_expert=_ptr(slot_of_expert), w_shared_gate=_ptr(sg),
            w_shared_up=_ptr(su), w_shared_down=_ptr(sd), ready_flags=_ptr(ready_flags),
            ready_epoch=int(ready_epoch), spin_limit_ns=int(spin_limit_ns),
            status=_ptr(status_word(self.dev)))
        self._need = {}   # token count -> workspace bytes

    def _workspace_bytes(self, n: int) -> int:
        size = self._need.get(n)
        if size is None:
            shp = _shape(n, self.h, self.e, self.k, self.f, self.s, self.dtype)
            size = int(self._lib.chronos_moe_workspace_size(ctypes.byref(shp)))
            if size == 0 and n > 0:
                N.check(N.CHRONOS_ERR_INVALID_ARG)
            if len(self._need) > 64:
                self._need.clear()
            self._need[n] = size
        return size

    def __call__(self, x: torch.Tensor, avail: Optional[torch.Tensor] = None, want_probs: bool = True,
                 want_stats: bool = False, want_topk: bool = False, avail_is_mask: bool = False,
                 acc_out: bool = False) -> dict:
        """``avail_is_mask``: ``avail`` is a residency mask, a_e = (avail[e] > 0),
        thresholded by the kernels (CHRONOS_FLAG_AVAIL_MASK).  ``acc_out``: ``y`` is
        the layer's fp32 accumulator, not rounded to the layer dtype
        (CHRONOS_FLAG_ACC_OUT; for a caller whose next kernel rounds it)."""
        if not x.is_cuda or x.dtype != self.dtype:
            raise TypeError(f"x must be a CUDA {self.dtype} tensor")
        x = x.contiguous()
        n = x.shape[0]
        dev = self.dev
        stream = _raw_stream(dev.index)
        ws = shared_workspace.get(dev, stream, self._workspace_bytes(n))
        y = torch.empty(n, self.h, dtype=torch.float32 if acc_out else self.dtype, device=dev)
        probs = torch.empty(n, self.e, dtype=self.dtype, device=dev) if want_probs else None
        topk_idx = torch.empty(n, self.k, dtype=torch.int32, device=dev) if want_topk else None
        topk_w = torch.empty(n, self.k, dtype=torch.float32, device=dev) if want_topk else None
        counts = torch.empty(self.e, dtype=torch.int32, device=dev) if want_stats else None
        mass = torch.empty(self.e, dtype=torch.float32, device=dev) if want_stats else None
        if avail is not None and (avail.dtype != torch.float32 or not avail.is_cuda
                                  or not avail.is_contiguous()):
            avail = avail.to(device=dev, dtype=torch.float32).contiguous()
        a = N.ChronosMoeArgs.from_buffer_copy(self._tmpl)
        a.shape.num_tokens = n
        a.x = x.data_ptr()
        a.y = y.data_ptr()
        a.router_probs = _ptr(probs)
        a.avail = _ptr(avail)
        a.topk_idx = _ptr(topk_idx)
        a.topk_weight = _ptr(topk_w)
        a.expert_counts = _ptr(counts)
        a.expert_mass = _ptr(mass)
        a.workspace = ws.data_ptr()
        a.workspace_bytes = ws.numel()
        if avail_is_mask and avail is not None:
            a.flags |= N.FLAG_AVAIL_MASK
        if acc_out:
            a.flags |= N.FLAG_ACC_OUT
        if torch.cuda.current_device() == dev.index:
            rc = self._lib.chronos_moe_forward(ctypes.byref(a), ctypes.c_void_p(stream))
        else:
            with torch.cuda.device(dev):
                rc = self._lib.chronos_moe_forward(ctypes.byref(a), ctypes.c_void_p(stream))
        N.check(rc)
        return dict(y=y, probs=probs, topk_idx=topk_idx, topk_weight=topk_w, counts=counts, mass=mass)


def moe_route(x: torch.Tensor, router_w: torch.Tensor, top_k: int, norm_topk: bool,
              num_shared: int = 0, ffn: int = 64, router_bias: Optional[torch.Tensor] = None,
              want_probs: bool = True, workspace: Optional[torch.Tensor] = None):
    """Routing only: dict(probs, topk_idx, topk_weight, counts, mass) on the device."""
    _check_cuda(x, router_w, router_bias)
    x = x.contiguous()
    n, h = x.shape
    e = router_w.shape[0]
    dt = x.dtype
    if router_w.dtype != dt:
        raise TypeError(f"router_w dtype {router_w.dtype} != x dtype {dt}")
    dev = x.device
    lib = N.load_library()
    shp = _shape(n, h, e, top_k, ffn, num_shared, dt)
    ws_bytes = int(lib.chronos_moe_workspace_size(ctypes.byref(shp)))
    if ws_bytes == 0 and n > 0:
        N.check(N.CHRONOS_ERR_INVALID_ARG)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    probs = torch.empty(n, e, dtype=dt, device=dev) if want_probs else None
    topk_idx = torch.empty(n, top_k, dtype=torch.int32, device=dev)
    topk_w = torch.empty(n, top_k, dtype=torch.float32, device=dev)
    counts = torch.empty(e, dtype=torch.int32, device=dev)
    mass = torch.empty(e, dtype=torch.float32, device=dev)
    router_w = router_w.contiguous()
    rb = None if router_bias is None else router_bias.to(device=dev, dtype=torch.float32).contiguous()
    args = N.ChronosMoeArgs(
        shape=shp, norm_topk=int(bool(norm_topk)), flags=0, x=_ptr(x), router_w=_ptr(router_w),
        router_bias=_ptr(rb), router_probs=_ptr(probs), topk_idx=_ptr(topk_idx),
        topk_weight=_ptr(topk_w), expert_counts=_ptr(counts), expert_mass=_ptr(mass),
        workspace=_ptr(workspace), workspace_bytes=int(workspace.numel()),
        status=_ptr(status_word(dev)))
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        N.check(lib.chronos_moe_route(ctypes.byref(args), ctypes.c_void_p(stream)))
    return dict(probs=probs, topk_idx=topk_idx, topk_weight=topk_w, counts=counts, mass=mass)


def ep_dispatch(x: torch.Tensor, topk_idx: torch.Tensor, topk_weight: torch.Tensor, num_experts: int,
                world_size: int, avail: Optional[torch.Tensor] = None, num_chunks: int = 1,
                dedup: bool = False, seg_rows: int = 0) -> dict:
    """Send buffers of one rank for expert parallelism (include/chronos_ep.h).

    Rows are ordered by (expert chunk, destination rank): each rank's E/G local
    experts split into ``num_chunks`` chunks (which must divide E/G).
    Returns dict(send_counts [C, G] int32, send_x [N*k, H], send_meta [N*k, P, 2] int32
    (local expert id, fp32 bits of w*a), pair_slot [N*k] int32, shared_weight [N, k]
    fp32, pairs P); the first ``send_counts.sum()`` rows of the send buffers are used.
    ``dedup`` (one chunk): one row per (token, destination rank), P = min(k, E/G)
    selections per row (padding: expert -1); else one row per selection, P = 1.
    ``seg_rows`` > 0 (one chunk): fixed segments, rank g's rows at g * seg_rows (the
    buffers hold world_size * seg_rows rows, unused rows carry padding metadata), so
    an all-to-all with equal splits needs no counts on the host."""
    _check_cuda(x, topk_idx, topk_weight, avail)
    x = x.contiguous()
    n, h = x.shape
    k = topk_idx.shape[1]
    dev = x.device
    if x.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {x.dtype}")
    topk_idx = topk_idx.to(torch.int32).contiguous()
    topk_weight = topk_weight.to(torch.float32).contiguous()
    av = None if avail is None else avail.to(device=dev, dtype=torch.float32).contiguous()
    num_chunks = max(1, int(num_chunks))
    pairs = min(k, int(num_experts) // int(world_size)) if dedup and num_chunks == 1 else 1
    seg_rows = max(0, int(seg_rows))
    rows = int(world_size) * seg_rows if seg_rows else n * k
    out = dict(send_counts=torch.empty(num_chunks, world_size, dtype=torch.int32, device=dev),
               send_x=torch.empty(rows, h, dtype=x.dtype, device=dev),
               send_meta=torch.empty(rows, pairs, 2, dtype=torch.int32, device=dev),
               pair_slot=torch.empty(n * k, dtype=torch.int32, device=dev),
               shared_weight=torch.empty(n, k, dtype=torch.float32, device=dev))
    scratch = torch.empty(max(n * k, 1), dtype=torch.int32, device=dev)
    args = N.ChronosEpDispatchArgs(
        num_tokens=n, hidden=h, num_experts=int(num_experts), top_k=k, world_size=int(world_size),
        dtype=_DTYPES[x.dtype], num_chunks=num_chunks, meta_pairs=pairs if pairs > 1 else 0, x=_ptr(x), topk_idx=_ptr(topk_idx), topk_weight=_ptr(topk_weight),
        avail=_ptr(av), send_counts=_ptr(out["send_counts"]), send_x=_ptr(out["send_x"]),
        send_meta=_ptr(out["send_meta"]),
        pair_slot=_ptr(out["pair_slot"]), shared_weight=_ptr(out["shared_weight"]),
        scratch=_ptr(scratch), seg_rows=seg_rows)
    lib = N.load_library()
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        N.check(lib.chronos_ep_dispatch(ctypes.byref(args), ctypes.c_void_p(stream)))
    out["pairs"] = pairs
    return out


def ep_combine(recv_y: torch.Tensor, pair_slot: torch.Tensor, top_k: int,
               y_shared: Optional[torch.Tensor] = None, num_tokens: Optional[int] = None,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y_t = y_shared_t + sum_j recv_y[pair_slot[t, j]] (fp32, j ascending)."""
    _check_cuda(recv_y, pair_slot, y_shared)
    h = recv_y.shape[1]
    n = int(num_tokens if num_tokens is not None else pair_slot.numel() // top_k)
    dev = recv_y.device
    dt = recv_y.dtype
    if y_shared is not None and y_shared.dtype != dt:
        raise TypeError(f"y_shared dtype {y_shared.dtype} != recv_y dtype {dt}")
    recv_y = recv_y.contiguous()
    y_shared = _contig(y_shared)
    pair_slot = pair_slot.to(torch.int32).contiguous()
    y = out if out is not None else torch.empty(n, h, dtype=dt, device=dev)
    args = N.ChronosEpCombineArgs(num_tokens=n, hidden=h, top_k=int(top_k), dtype=_DTYPES[dt],
                                  y_shared=_ptr(y_shared), recv_y=_ptr(recv_y),
                                  pair_slot=_ptr(pair_slot), y=_ptr(y))
    lib = N.load_library()
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        N.check(lib.chronos_ep_combine(ctypes.byref(args), ctypes.c_void_p(stream)))
    return y


def lookahead_forward(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, num_experts: int,
                      steps: int) -> torch.Tensor:
    """Lookahead router (include/chronos_lookahead.h): x [N, H], w1 [H/4, H],
    w2 [E*K, H/4] -> probs [N, K, E] in x's dtype."""
    _check_cuda(x, w1, w2)
    x = x.contiguous()
    n, h = x.shape
    for name, t in (("w1", w1), ("w2", w2)):
        if t.dtype != x.dtype:
            raise TypeError(f"{name} dtype {t.dtype} != x dtype {x.dtype}")
    if x.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {x.dtype}")
    w1, w2 = w1.contiguous(), w2.contiguous()
    probs = torch.empty(n, steps, num_experts, dtype=x.dtype, device=x.device)
    args = N.ChronosLookaheadArgs(num_tokens=n, hidden=h, inner=w1.shape[0], num_experts=int(num_experts),
                                  steps=int(steps), dtype=_DTYPES[x.dtype], x=_ptr(x), w1=_ptr(w1),
                                  w2=_ptr(w2), probs=_ptr(probs))
    lib = N.load_library()
    stream = torch.cuda.current_stream(x.device).cuda_stream
    with torch.cuda.device(x.device):
        N.check(lib.chronos_lookahead_forward(ctypes.byref(args), ctypes.c_void_p(stream)))
    return probs


def add_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
                sum_out: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """RMSNorm(x + residual) * weight over the last dim (include/chronos_attention.h);
    ``sum_out`` (may be ``x`` or ``residual``) receives x + residual.  The layer
    dtype is ``weight``'s; an fp32 ``x`` with a bf16/fp16 ``weight`` (a MoE
    layer's fp32 accumulator) is rounded to that dtype as it is read."""
    _check_cuda(x, weight, residual, sum_out, out)
    dt = weight.dtype
    x_fp32 = x.dtype == torch.float32 and dt != torch.float32
    if dt not in _DTYPES or (x.dtype != dt and not x_fp32):
        raise TypeError(f"x {x.dtype} / weight {weight.dtype}: one supported dtype expected")
    for t in (residual, sum_out, out):
        if t is not None and t.dtype != dt:
            raise TypeError("residual, sum_out and out must have weight's dtype")
    w = x.shape[-1]
    for t in (x, residual, sum_out, out):
        if t is not None and not t.is_contiguous():
            raise ValueError("add_rmsnorm needs contiguous tensors")
    if x_fp32 and sum_out is not None and sum_out.data_ptr() == x.data_ptr():
        raise ValueError("sum_out cannot alias an fp32 x")
    out = torch.empty(x.shape, dtype=dt, device=x.device) if out is None else out
    args = N.ChronosNormArgs(rows=x.numel() // max(w, 1), width=w, dtype=_DTYPES[dt], eps=float(eps),
                             x_fp32=1 if x_fp32 else 0,
                             x=_ptr(x), residual=_ptr(residual), sum_out=_ptr(sum_out),
                             weight=_ptr(weight.contiguous()), out=_ptr(out))
    lib = N.load_library()
    N.check(lib.chronos_add_rmsnorm(ctypes.byref(args), ctypes.c_void_p(_raw_stream(x.device.index))))
    return out


def argmax_rows(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """torch.argmax(x, dim=-1) as one kernel (include/chronos_attention.h): the
    index of the first maximal value of every row (NaN counts as the maximum),
    int64 [*x.shape[:-1]]."""
    _check_cuda(x, out)
    if x.dtype not in _DTYPES:
        raise TypeError(f"x {x.dtype}: bf16, fp16 or fp32 expected")
    if not x.is_contiguous():
        raise ValueError("argmax_rows needs a contiguous tensor")
    cols = x.shape[-1]
    rows = x.numel() // max(cols, 1)
    if out is None:
        out = torch.empty(x.shape[:-1], dtype=torch.int64, device=x.device)
    elif out.dtype != torch.int64 or out.numel() != rows or not out.is_contiguous():
        raise ValueError("out must be a contiguous int64 tensor with one value per row")
    lib = N.load_library()
    N.check(lib.chronos_argmax_rows(ctypes.c_void_p(_ptr(x)), rows, cols, _DTYPES[x.dtype],
                                    ctypes.c_void_p(_ptr(out)), ctypes.c_void_p(_raw_stream(x.device.index))))
    return out


def attn_decode(kind: str, proj: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                cache_a: torch.Tensor, cache_b: torch.Tensor, heads: int, kv_heads: int, head_dim: int,
                rope_dim: int, latent: int, window: int, eps: float, norm_q: torch.Tensor,
                norm_q2: torch.Tensor, norm_kv: Optional[torch.Tensor] = None,
                w_krope: Optional[torch.Tensor] = None, w_knope: Optional[torch.Tensor] = None,
                w_v: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One cached decode step of an MLA (``kind="mla"``) or sliding-window
    (``"sw"``) layer: proj [B, width] -> out [B, heads*head_dim]; appends the new
    token to the caches.  ``pos`` is a device int32 scalar (the new token's
    position).  Every tensor must be contiguous, on one device, in one dtype."""
    _check_cuda(proj, pos, cos, sin, cache_a, cache_b, norm_q, norm_q2, norm_kv, w_krope, w_knope, w_v, out)
    dt = proj.dtype
    if dt not in _DTYPES:
        raise TypeError(f"unsupported dtype {dt}")
    for t in (cos, sin, cache_a, cache_b, norm_q, norm_q2, norm_kv, w_krope, w_knope, w_v):
        if t is not None and (t.dtype != dt or not t.is_contiguous()):
            raise TypeError("attention operands must be contiguous and share proj's dtype")
    if pos.dtype != torch.int32:
        raise TypeError("pos must be a device int32 scalar")
    b = proj.shape[0]
    out = torch.empty(b, heads * head_dim, dtype=dt, device=proj.device) if out is None else out
    args = N.ChronosAttnArgs(
        batch=b, heads=heads, kv_heads=kv_heads, head_dim=head_dim, rope_dim=rope_dim, latent=latent,
        window=window, max_len=cache_a.shape[1], table_len=cos.shape[0], dtype=_DTYPES[dt], eps=float(eps),
        pos=_ptr(pos), proj=_ptr(proj), norm_q=_ptr(norm_q), norm_q2=_ptr(norm_q2), norm_kv=_ptr(norm_kv),
        w_krope=_ptr(w_krope), w_knope=_ptr(w_knope), w_v=_ptr(w_v), cos=_ptr(cos), sin=_ptr(sin),
        cache_a=_ptr(cache_a), cache_b=_ptr(cache_b), out=_ptr(out))
    lib = N.load_library()
    fn = lib.chronos_mla_decode if kind == "mla" else lib.chronos_sw_decode
    N.check(fn(ctypes.byref(args), ctypes.c_void_p(_raw_stream(proj.device.index))))
    return out


def profile_begin(max_calls: int) -> None:
    """Record per-stage CUDA events for the next ``max_calls`` layer calls (this thread)."""
    lib = N.load_library()
    N.check(lib.chronos_moe_profile_begin(int(max_calls)))


def profile_end() -> dict:
    """Synchronise and return {"calls": c, stage: (total_ms, launches), ...}."""
    lib = N.load_library()
    ms = (ctypes.c_float * len(N.STAGES))()
    cnt = (ctypes.c_int32 * len(N.STAGES))()
    calls = lib.chronos_moe_profile_end(ms, cnt, len(N.STAGES))
    if calls < 0:
        N.check(-calls)
    out = {"calls": int(calls)}
    for i, name in enumerate(N.STAGES):
        out[name] = (float(ms[i]), int(cnt[i]))
    return out


def set_option(name: str, value: int) -> None:
    """Process-wide launch-sequence switch (``chronos_moe_set_option``), e.g.
    ``set_option("fused_route", 0)`` for the two-kernel decode routing."""
    N.check(N.load_library().chronos_moe_set_option(name.encode(), int(value)))


def kernel_launches() -> int:
    """Kernels launched by the extension since it was loaded."""
    return int(N.load_library().chronos_moe_kernel_launches())


# ---------------------------------------------------------------------------
# torch.library registration (one graph node for torch.compile)
# ---------------------------------------------------------------------------

@torch.library.custom_op("chronos::moe_forward", mutates_args=())
def moe_forward_op(x: torch.Tensor, router_w: torch.Tensor, w_gate: torch.Tensor,
                   w_up: torch.Tensor, w_down: torch.Tensor, sh_gate: Optional[torch.Tensor],
                   sh_up: Optional[torch.Tensor], sh_down: Optional[torch.Tensor],
                   avail: Optional[torch.Tensor], top_k: int,
                   norm_topk: bool) -> List[torch.Tensor]:
    r = moe_forward(x, router_w, w_gate, w_up, w_down, sh_gate, sh_up, sh_down, top_k, norm_topk,
                    avail=avail, want_probs=True)
    return [r["y"], r["probs"], r["topk_idx"], r["topk_weight"]]


@moe_forward_op.register_fake
def _moe_forward_fake(x, router_w, w_gate, w_up, w_down, sh_gate, sh_up, sh_down, avail, top_k,
                      norm_topk):
    n, h = x.shape
    e = router_w.shape[0]
    return [x.new_empty(n, h), x.new_empty(n, e),
            x.new_empty(n, top_k, dtype=torch.int32), x.new_empty(n, top_k, dtype=torch.float32)]
