"""Drop-in ``LookaheadRouter`` whose forward is one sm_100a kernel.

Mirrors ``chronos/model/lookahead_router.py`` of FonaTech/Project_Chronos:
same constructor (a Chronos config with ``hidden_size``, ``num_experts``,
``lookahead_steps``), same parameters (``proj.0.weight`` [H/4, H],
``proj.2.weight`` [E*K, H/4], bias-free, SiLU between), so ``state_dict`` keys
(``model.lookahead_router.proj.{0,2}.weight``) load unchanged;
``forward(hidden_states [B, S, H]) -> [B, S, K, E]`` softmax probabilities
(K = lookahead_steps + 1, index 0 the current step) and
``predict_next_experts(hidden_states, top_k)``.

The two projections, the SiLU and the K softmaxes run in one launch
(``chronos_lookahead_forward``), accumulating in fp32.  CUDA inputs only;
backward is not implemented (call it under ``torch.no_grad()``).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import ops


class LookaheadRouter(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.lookahead_steps = int(config.lookahead_steps)
        self.num_experts = int(config.num_experts)
        H = int(config.hidden_size)
        K = self.lookahead_steps + 1
        self.proj = nn.Sequential(
            nn.Linear(H, H // 4, bias=False),
            nn.SiLU(),
            nn.Linear(H // 4, self.num_experts * K, bias=False),
        )

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        if not hidden_states.is_cuda:
            raise RuntimeError("LookaheadRouter (sm_100a kernel) needs CUDA tensors; "
                               f"got {hidden_states.device}")
        if torch.is_grad_enabled() and self.training:
            raise NotImplementedError("LookaheadRouter runs a forward-only kernel; backward is not "
                                      "implemented (call it under torch.no_grad() or in eval mode)")
        B, S, H = hidden_states.shape
        K = self.lookahead_steps + 1
        probs = ops.lookahead_forward(hidden_states.reshape(-1, H), self.proj[0].weight,
                                      self.proj[2].weight, self.num_experts, K)
        return probs.view(B, S, K, self.num_experts)

    def predict_next_experts(self, hidden_states: torch.Tensor, top_k: int = 1) -> torch.Tensor:
        """Top-k expert indices of every future step: [B, S, lookahead_steps, top_k]."""
        probs = self.forward(hidden_states)
        return torch.topk(probs[:, :, 1:, :], k=top_k, dim=-1).indices
