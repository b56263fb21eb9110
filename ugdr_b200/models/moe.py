"""MoE router for the expert-parallel all-to-all workload: seeded uniform router logits, top-k
experts per token, softmax weights renormalised over the chosen k."""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class MoEConfig:
    tokens: int = 16384  # per rank
    hidden: int = 7168
    topk: int = 8
    experts: int = 256


def route(tokens: int, experts: int, topk: int, seed: int, device="cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """(expert ids [tokens, topk] int32, weights [tokens, topk] float32)."""
    g = torch.Generator(device=device).manual_seed(seed)
    logits = torch.rand(tokens, experts, generator=g, device=device)
    top, ids = torch.topk(logits, topk, dim=-1)
    w = torch.softmax(top, dim=-1)
    return ids.to(torch.int32), w.to(torch.float32)


def reference_positions(ids: torch.Tensor, experts: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Row counts per expert and each row's rank inside its expert group, in row order
    (the semantics of the fused route kernel), computed with plain torch ops."""
    flat = ids.reshape(-1).long()
    counts = torch.bincount(flat, minlength=experts)
    order = torch.sort(flat, stable=True).indices
    starts = torch.cumsum(counts, 0) - counts
    rank_sorted = torch.arange(flat.numel(), device=flat.device) - starts[flat[order]]
    pos = torch.empty_like(flat)
    pos[order] = rank_sorted
    return counts.to(torch.int32), pos.view(ids.shape).to(torch.int32)
