"""Rank bodies for the expert-parallel tests (run in spawned processes).

``cpu_rank``: gloo rank with the oracle's CPU stand-ins for the extension
(host orchestration only).  ``gpu_rank``: NCCL rank on its own GPU with the
sm_100a extension.  Both compare the expert-parallel layer on the rank's own
tokens against the single-device result on the same global weights.
"""
import os
import sys
import traceback
from datetime import timedelta

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def _weights(E, H, F, S, seed=0):
    import torch
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: (torch.randn(*s, generator=g) * 0.05)  # noqa: E731
    return dict(router=r(E, H), gate=r(E, F, H), up=r(E, F, H), down=r(E, H, F),
                sh_gate=r(S, F, H), sh_up=r(S, F, H), sh_down=r(S, H, F))


def _cfg(E, k, H, F, S):
    import types
    return types.SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                                 moe_intermediate_size=F, num_shared_experts=S, norm_topk_prob=True)


def _ref(x, w, k, mask):
    from oracle import moe_oracle as O
    ref, _, _, _ = O.moe_forward(x.numpy(), w["router"].numpy(), w["gate"].numpy(), w["up"].numpy(),
                                 w["down"].numpy(), w["sh_gate"].numpy(), w["sh_up"].numpy(),
                                 w["sh_down"].numpy(), k, True, avail=None if mask is None else mask.numpy())
    return ref


def cpu_rank(rank, world, port, q, scenario):
    import numpy as np
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        from oracle import moe_oracle as O
        from oracle.ep_oracle import CpuEpBackend
        from project_chronos_b200.ep import ExpertParallelMoE
        E, k, H, F, S = 8, 2, 32, 16, 1
        w = _weights(E, H, F, S)
        x = torch.randn(5 + 3 * rank, H, generator=torch.Generator().manual_seed(100 + rank))
        mask = None
        if scenario == "mask":
            mask = torch.tensor([1, 0, 1, 1, 0, 1, 1, 1], dtype=torch.float32)
        if scenario == "fail" and rank == 1:
            raise RuntimeError("injected rank failure before the exchange")
        m = ExpertParallelMoE.from_stacked(_cfg(E, k, H, F, S), w["router"], w["gate"], w["up"],
                                           w["down"], w["sh_gate"], w["sh_up"], w["sh_down"],
                                           backend=CpuEpBackend())
        m.chunks = 3 if scenario == "mask" else 1
        if scenario == "fixed":
            m.segment_rows = 16   # every rank's tokens (at most 14) fit one segment
        y = m(x, available_expert_mask=mask)
        if scenario == "fixed":
            q.put(("ok", rank, O.rel_l2(y.numpy(), _ref(x, w, k, mask)), m.read_send_counts(), None))
            return
        ref, _, _, _ = O.moe_forward(x.numpy(), w["router"].numpy(), w["gate"].numpy(),
                                     w["up"].numpy(), w["down"].numpy(), w["sh_gate"].numpy(),
                                     w["sh_up"].numpy(), w["sh_down"].numpy(), k, True,
                                     avail=None if mask is None else mask.numpy())
        q.put(("ok", rank, O.rel_l2(y.numpy(), ref), m.last_send_counts, m.last_recv_counts))
    except Exception as exc:  # reported to the test, which decides
        q.put(("error", rank, f"{type(exc).__name__}: {exc}", None, None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def gpu_rank(rank, world, port, q, cfg_d):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        from project_chronos_b200 import ops
        from project_chronos_b200.ep import ExpertParallelMoE
        E, k, H, F, S, n = (cfg_d[key] for key in ("E", "k", "H", "F", "S", "n"))
        dt = torch.bfloat16
        w = {key: v.to(dev, dt) for key, v in _weights(E, H, F, S).items()}
        x = torch.randn(n, H, generator=torch.Generator().manual_seed(100 + rank)).to(dev, dt)
        m = ExpertParallelMoE.from_stacked(_cfg(E, k, H, F, S), w["router"], w["gate"], w["up"],
                                           w["down"], w["sh_gate"], w["sh_up"], w["sh_down"])
        m.segment_rows = int(cfg_d.get("seg", 0))
        y = m(x)
        full = ops.moe_forward(x, w["router"], w["gate"], w["up"], w["down"], w["sh_gate"], w["sh_up"],
                               w["sh_down"], k, True, want_probs=False)["y"]
        torch.cuda.synchronize()
        ops.check_status(dev)
        rel = (torch.linalg.vector_norm(y.float() - full.float()) /
               torch.linalg.vector_norm(full.float())).item()
        if m.segment_rows:
            q.put(("ok", rank, rel, m.read_send_counts(), None))
        else:
            q.put(("ok", rank, rel, m.last_send_counts, m.last_recv_counts))
    except Exception:
        q.put(("error", rank, traceback.format_exc(), None, None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass
