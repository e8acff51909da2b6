"""Run one MoE-layer workload a few times (for profilers such as ncu).

    python -m project_chronos_b200.profile_case --workload prefill --calls 3
    python -m project_chronos_b200.profile_case --workload decode --tokens 1 --calls 3
    python -m project_chronos_b200.profile_case --workload ep --calls 3
    python -m project_chronos_b200.profile_case --workload decode --tokens 64 --fused-route --calls 3
    python -m project_chronos_b200.profile_case --workload model --tokens 32 --calls 3
    python -m project_chronos_b200.profile_case --workload attn --kind sw --tokens 32 --calls 20
    python -m project_chronos_b200.profile_case --workload lookahead --tokens 32 --calls 20
    python -m project_chronos_b200.profile_case --workload model-pieces --tokens 32

Builds the named synthetic workload on cuda:0 (``synthetic.WORKLOADS``),
calls ``ops.moe_forward`` ``--calls`` times with an L2 flush (256 MB write)
before each call, synchronises, checks the device status word and prints the
average device time per call.  Nothing else runs, so a kernel filter with a
launch skip count selects a steady-state call.
"""
from __future__ import annotations

import argparse
import sys

import torch

from . import ops, synthetic as syn


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="prefill",
                    choices=sorted(syn.WORKLOADS) + ["model", "model-pieces", "attn", "lookahead"])
    ap.add_argument("--kind", default="sw", choices=["sw", "mla"], help="attention kind (--workload attn)")
    ap.add_argument("--positions", type=int, default=516, help="cached positions (--workload attn)")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--fused-route", action="store_true",
                    help="decode routing as one cluster launch (chronos_moe_set_option)")
    ap.add_argument("--option", action="append", default=[], metavar="NAME=VALUE",
                    help="any chronos_moe_set_option switch, e.g. down_split_target=4")
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ops.set_option("fused_route", 1 if args.fused_route else 0)
    for opt in args.option:
        name, _, value = opt.partition("=")
        ops.set_option(name, int(value))
    if args.workload == "ep":
        return _ep(args, dev)
    if args.workload == "model":
        return _model(args, dev)
    if args.workload == "model-pieces":
        return _model_pieces(args, dev)
    if args.workload == "attn":
        return _attn(args, dev)
    if args.workload == "lookahead":
        return _lookahead(args, dev)
    wl = syn.named_workload(args.workload, tokens=args.tokens, seed=args.seed, device=dev)
    w = wl.weights
    s = wl.shape
    avail = None if wl.mask is None else wl.mask.to(torch.float32)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    total_ms = 0.0
    for _ in range(args.calls):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        ops.moe_forward(wl.x, w.router, w.gate, w.up, w.down,
                        w.sh_gate if s.num_shared else None, w.sh_up if s.num_shared else None,
                        w.sh_down if s.num_shared else None, s.top_k, s.norm_topk, avail=avail,
                        router_bias=wl.bias)
        b.record()
        torch.cuda.synchronize()
        total_ms += a.elapsed_time(b)
    ops.check_status(dev)
    print(f"{args.workload} tokens={wl.x.shape[0]} calls={args.calls} "
          f"avg_ms={total_ms / args.calls:.4f}")
    return 0


def _model(args, dev) -> int:
    """Eager decode steps of the 8-layer model (synthetic.DECODE_MODEL): a
    512-token prompt of --tokens rows, then --calls one-token steps."""
    import types
    from .model import ChronosForCausalLM
    cfg = types.SimpleNamespace(**syn.DECODE_MODEL)
    lm = ChronosForCausalLM.on_device(cfg, dev, torch.bfloat16)
    syn.init_model_(lm, args.seed, dev)
    lm.eval()
    b = args.tokens or 32
    g = torch.Generator(device=dev).manual_seed(args.seed + 1)
    ids = torch.randint(0, cfg.vocab_size, (b, 512), generator=g, device=dev)
    total_ms = 0.0
    with torch.no_grad():
        out, _ = lm(ids, use_cache=True, cache_capacity=512 + args.calls + 8)
        cache = out.past_key_values
        nxt = torch.argmax(out.logits[:, -1], dim=-1).view(-1, 1)
        for _ in range(args.calls):
            a = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            a.record()
            out, _ = lm(nxt, past_key_values=cache, use_cache=True)
            e.record()
            torch.cuda.synchronize()
            total_ms += a.elapsed_time(e)
            nxt = torch.argmax(out.logits[:, -1], dim=-1).view(-1, 1)
    ops.check_status(dev)
    print(f"model batch={b} steps={args.calls} avg_ms={total_ms / args.calls:.4f}")
    return 0


def _graph_chain_us(fn, reps: int = 20, iters: int = 20) -> float:
    """Device time of one ``fn()`` inside a CUDA graph of ``reps`` back-to-back calls
    (launch gaps included, as in a graph-replayed decode step), in us."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        graph.replay()
    e.record()
    torch.cuda.synchronize()
    return a.elapsed_time(e) * 1e3 / (iters * reps)


def _model_pieces(args, dev) -> int:
    """The 8-layer model's graph-replayed decode step (synthetic.DECODE_MODEL, a
    512-token prompt of --tokens rows), then each piece of a step alone as a chain
    of graph-captured calls: the residual add + RMSNorm (fp32 MoE accumulator or
    bf16 input), the input projection and o_proj (cuBLAS), the two attention
    decode kernels, one MoE layer (fp32 hand-off, and with its finalize), one whole
    sliding-window block, the lookahead router, the LM head and the greedy pick."""
    import json
    import types
    import torch.nn.functional as F
    from .model import ChronosForCausalLM, GraphedDecoder
    cfg = types.SimpleNamespace(**syn.DECODE_MODEL)
    lm = ChronosForCausalLM.on_device(cfg, dev, torch.bfloat16)
    syn.init_model_(lm, args.seed, dev)
    lm.eval()
    B, H = args.tokens or 32, cfg.hidden_size
    g = torch.Generator(device=dev).manual_seed(args.seed + 1)
    ids = torch.randint(0, cfg.vocab_size, (B, 512), generator=g, device=dev)
    res = {}
    with torch.no_grad():
        out, _ = lm(ids, use_cache=True, cache_capacity=512 + 200)
        cache = out.past_key_values
        dec = GraphedDecoder(lm, cache)
        for _ in range(3):
            dec.step()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(50):
            dec.step()
        e.record()
        torch.cuda.synchronize()
        res["step"] = a.elapsed_time(e) * 1e3 / 50
        m = lm.model
        L0, L1 = m.layers[0], m.layers[1]
        hid = torch.randn(B, 1, H, generator=g, device=dev, dtype=torch.bfloat16)
        acc = torch.randn(B, 1, H, generator=g, device=dev, dtype=torch.float32)
        bf = torch.randn(B, 1, H, generator=g, device=dev, dtype=torch.bfloat16)
        x2 = bf.view(B, H)
        cos, sin = m.freqs_cos, m.freqs_sin
        a0, a1 = L0.self_attn, L1.self_attn
        p0, p1 = F.linear(x2, a0._in_weight()), F.linear(x2, a1._in_weight())
        mask = dec.masks[1]
        res["norm_fp32_acc"] = _graph_chain_us(lambda: L1.input_layernorm(acc, residual=hid, sum_out=hid))
        res["norm_bf16"] = _graph_chain_us(lambda: L1.post_attention_layernorm(bf, residual=hid, sum_out=hid))
        res["in_proj_sw"] = _graph_chain_us(lambda: F.linear(x2, a1._in_weight()))
        res["in_proj_mla"] = _graph_chain_us(lambda: F.linear(x2, a0._in_weight()))
        res["o_proj"] = _graph_chain_us(lambda: F.linear(x2, a1.o_proj.weight))
        res["attn_sw"] = _graph_chain_us(lambda: ops.attn_decode(
            "sw", p1, cache.pos, cos, sin, cache.a[1], cache.b[1], a1.n_heads, a1.n_kv_heads, a1.head_dim,
            a1.head_dim, 0, a1.window_size, a1.eps, a1.q_norm.weight, a1.k_norm.weight))
        res["attn_mla"] = _graph_chain_us(lambda: ops.attn_decode(
            "mla", p0, cache.pos, cos, sin, cache.a[0], cache.b[0], a0.n_heads, a0.n_kv_heads, a0.head_dim,
            a0.rope_dim, a0.kv_latent_dim, 0, a0.eps, a0.q_nope_norm.weight, a0.q_rope_norm.weight,
            norm_kv=a0.kv_down_norm.weight, w_krope=a0.k_rope_proj.weight, w_knope=a0.k_nope_proj.weight,
            w_v=a0.v_proj.weight))
        res["moe_fp32_handoff"] = _graph_chain_us(lambda: L1.mlp.forward_acc(bf, mask), reps=8)
        res["moe_with_finalize"] = _graph_chain_us(lambda: L1.mlp(bf, mask), reps=8)

        def block():
            h_in = L1.input_layernorm(acc, residual=hid, sum_out=hid)
            at = a1.decode(h_in.view(B, H), cos, sin, cache).view(B, 1, H)
            mi = L1.post_attention_layernorm(at, residual=hid, sum_out=hid)
            return L1.mlp.forward_acc(mi, mask)
        res["block_sw"] = _graph_chain_us(block, reps=8)
        res["lookahead"] = _graph_chain_us(lambda: m.lookahead_router(hid), reps=8)
        res["lm_head"] = _graph_chain_us(lambda: F.linear(x2, lm.lm_head.weight))
        logits = F.linear(x2, lm.lm_head.weight)
        nxt = torch.empty(B, dtype=torch.long, device=dev)
        res["argmax"] = _graph_chain_us(lambda: ops.argmax_rows(logits, out=nxt))
    ops.check_status(dev)
    print(json.dumps({k + "_us": round(v, 2) for k, v in res.items()}))
    return 0


def _timed(fn, calls: int) -> float:
    """Average device time of ``fn()`` over ``calls`` back-to-back calls, in µs."""
    fn()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(calls):
        fn()
    e.record()
    torch.cuda.synchronize()
    return a.elapsed_time(e) * 1e3 / calls


def _attn(args, dev) -> int:
    """One attention decode kernel of the 8-layer model's shape (synthetic.DECODE_MODEL):
    --tokens batch rows, --positions cached tokens, random cache contents."""
    import types
    from .model import HybridCache, make_attention, precompute_freqs_cis
    cfg = types.SimpleNamespace(**syn.DECODE_MODEL)
    b = args.tokens or 32
    layer = 0 if args.kind == "mla" else 1
    dt = torch.bfloat16
    attn = make_attention(layer, cfg).to(dev, dt).eval()
    g = torch.Generator(device=dev).manual_seed(args.seed)
    with torch.no_grad():
        for name, p in sorted(attn.named_parameters()):
            if name.endswith("norm.weight"):
                p.normal_(1.0, 0.1, generator=g)
            else:
                p.normal_(0.0, 0.02, generator=g)
    cache = HybridCache(cfg, b, args.positions + 8, dev, dt)
    for t in (cache.a[layer], cache.b[layer]):
        t.normal_(0.0, 1.0, generator=g)
    cache.pos.fill_(args.positions)
    cache.length = args.positions
    cos, sin = precompute_freqs_cis(cfg.head_dim, cfg.max_position_embeddings, cfg.rope_theta)
    cos, sin = cos.to(dev, dt), sin.to(dev, dt)
    x = torch.randn(b, cfg.hidden_size, generator=g, device=dev, dtype=dt)
    proj = torch.nn.functional.linear(x, attn._in_weight())
    if args.kind == "mla":
        fn = lambda: ops.attn_decode(  # noqa: E731
            "mla", proj, cache.pos, cos, sin, cache.a[layer], cache.b[layer], attn.n_heads, attn.n_kv_heads,
            attn.head_dim, attn.rope_dim, attn.kv_latent_dim, 0, attn.eps, attn.q_nope_norm.weight,
            attn.q_rope_norm.weight, norm_kv=attn.kv_down_norm.weight, w_krope=attn.k_rope_proj.weight,
            w_knope=attn.k_nope_proj.weight, w_v=attn.v_proj.weight)
    else:
        fn = lambda: ops.attn_decode(  # noqa: E731
            "sw", proj, cache.pos, cos, sin, cache.a[layer], cache.b[layer], attn.n_heads, attn.n_kv_heads,
            attn.head_dim, attn.head_dim, 0, attn.window_size, attn.eps, attn.q_norm.weight, attn.k_norm.weight)
    us = _timed(fn, args.calls)
    ops.check_status(dev)
    print(f"attn kind={args.kind} batch={b} positions={args.positions} calls={args.calls} avg_us={us:.2f}")
    return 0


def _lookahead(args, dev) -> int:
    """The lookahead router of the 8-layer model on --tokens rows."""
    import types
    from .lookahead import LookaheadRouter
    cfg = types.SimpleNamespace(**syn.DECODE_MODEL)
    m = LookaheadRouter(cfg).to(dev, torch.bfloat16).eval()
    g = torch.Generator(device=dev).manual_seed(args.seed)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0.0, 0.02, generator=g)
    n = args.tokens or 32
    x = torch.randn(1, n, cfg.hidden_size, generator=g, device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        us = _timed(lambda: m(x), args.calls)
    ops.check_status(dev)
    print(f"lookahead tokens={n} calls={args.calls} avg_us={us:.2f}")
    return 0


def _ep(args, dev) -> int:
    """The expert-parallel layer on one GPU (all experts local, no exchange)."""
    import types
    from .ep import ExpertParallelMoE
    spec = syn.WORKLOADS["ep"]
    shape = spec["shape"]
    n = args.tokens or spec["tokens"]
    w = syn.make_ep_weights(shape, 0, 1, seed=args.seed, dtype=torch.bfloat16, device=dev)
    x = syn.make_hidden(n, shape.hidden, syn.make_generator(args.seed + 1, dev), dtype=torch.bfloat16,
                        device=dev)
    cfg = types.SimpleNamespace(hidden_size=shape.hidden, num_experts=shape.num_experts,
                                num_experts_per_tok=shape.top_k, moe_intermediate_size=shape.ffn,
                                num_shared_experts=shape.num_shared, norm_topk_prob=shape.norm_topk)
    m = ExpertParallelMoE.from_stacked(cfg, w.router, w.gate, w.up, w.down, w.sh_gate, w.sh_up,
                                       w.sh_down, local=True)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    total_ms = 0.0
    for _ in range(args.calls):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        m(x)
        b.record()
        torch.cuda.synchronize()
        total_ms += a.elapsed_time(b)
    ops.check_status(dev)
    print(f"ep tokens={n} calls={args.calls} avg_ms={total_ms / args.calls:.4f}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
