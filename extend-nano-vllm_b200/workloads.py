"""Seeded synthetic inputs with the shapes and distributions of the benchmark
configurations (no datasets or checkpoints are used anywhere).

Layer shapes:
  QWEN3_30B_A3B   hidden 2048, 128 experts, top-8, moe_intermediate 768
  QWEN3_235B_A22B hidden 4096, 128 experts, top-8, moe_intermediate 1536
  QWEN3_NEXT_80B_A3B hidden 2048, 512 experts, top-10, moe_intermediate 512,
                  shared expert 512
Distributions: hidden states N(0, 1) bf16; router gate N(0, 0.02) fp32;
expert weights N(0, 0.02) bf16; decode router logits U(0, 1) fp32; prefill
logits N(0, 1) + Zipf(alpha) popularity bias over a seeded expert permutation.

Generators draw on the CPU with torch.Generator so every machine with the
same torch version produces identical tensors; ``device`` only chooses where
the result is placed.  Large expert weights can instead be drawn directly on
the GPU (``on_device=True``) when bit-identical CPU copies are not needed.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class LayerShape:
    name: str
    hidden: int
    intermediate: int
    num_experts: int
    top_k: int
    norm_topk_prob: bool = True
    shared_intermediate: int | None = None

    @property
    def expert_bytes(self) -> int:
        """bf16 bytes of one expert's gate/up + down weights."""
        return 3 * self.hidden * self.intermediate * 2

    @property
    def flops_per_route(self) -> int:
        """Multiply-adds x 2 of one route through gate/up and down."""
        return 2 * 3 * self.hidden * self.intermediate


QWEN3_30B_A3B = LayerShape("qwen3-30b-a3b-moe", 2048, 768, 128, 8)
QWEN3_235B_A22B = LayerShape("qwen3-235b-a22b-moe", 4096, 1536, 128, 8)
# Qwen3-Next-style layer with a shared expert as wide as the routed ones.
QWEN3_NEXT_80B_A3B = LayerShape("qwen3-next-80b-a3b-moe", 2048, 512, 512, 10,
                                shared_intermediate=512)


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return g


def hidden_states(tokens: int, hidden: int, seed: int, device="cpu") -> torch.Tensor:
    x = torch.randn((tokens, hidden), generator=_gen(seed), dtype=torch.float32)
    return x.to(torch.bfloat16).to(device)


def gate_weight(shape: LayerShape, seed: int, device="cpu") -> torch.Tensor:
    g = torch.randn((shape.num_experts, shape.hidden), generator=_gen(seed), dtype=torch.float32)
    return (g * 0.02).to(device)


def expert_weights(shape: LayerShape, seed: int, num_local: int | None = None,
                   first_expert: int = 0, device="cpu", on_device: bool = False
                   ) -> tuple[torch.Tensor, torch.Tensor]:
    """(W13 [E_loc, 2I, H], W2 [E_loc, H, I]) bf16, N(0, 0.02).

    Expert e's weights depend only on (seed, e), so EP shards cut from the same
    seed equal slices of the full tensors."""
    num_local = shape.num_experts if num_local is None else num_local
    H, I = shape.hidden, shape.intermediate
    w13 = torch.empty((num_local, 2 * I, H), dtype=torch.bfloat16, device=device)
    w2 = torch.empty((num_local, H, I), dtype=torch.bfloat16, device=device)
    for i in range(num_local):
        e = first_expert + i
        if on_device:
            g = torch.Generator(device=device)
            g.manual_seed(seed * 100003 + e)
            w13[i] = (torch.randn((2 * I, H), generator=g, device=device) * 0.02).bfloat16()
            w2[i] = (torch.randn((H, I), generator=g, device=device) * 0.02).bfloat16()
        else:
            g = _gen(seed * 100003 + e)
            w13[i] = (torch.randn((2 * I, H), generator=g) * 0.02).bfloat16()
            w2[i] = (torch.randn((H, I), generator=g) * 0.02).bfloat16()
    return w13, w2


def shared_expert_weights(shape: LayerShape, seed: int, device="cpu"
                          ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Shared expert (gate/up [2I_s, H], down [H, I_s], gate [1, H]) bf16, N(0, 0.02)."""
    H, I = shape.hidden, shape.shared_intermediate
    g = _gen(seed * 100003 + 99991)
    w13 = (torch.randn((2 * I, H), generator=g) * 0.02).bfloat16()
    w2 = (torch.randn((H, I), generator=g) * 0.02).bfloat16()
    wg = (torch.randn((1, H), generator=g) * 0.02).bfloat16()
    return w13.to(device), w2.to(device), wg.to(device)


def uniform_logits(tokens: int, num_experts: int, seed: int, device="cpu") -> torch.Tensor:
    """Decode buckets: U(0, 1) fp32 router logits."""
    return torch.rand((tokens, num_experts), generator=_gen(seed), dtype=torch.float32).to(device)


def zipf_bias(num_experts: int, alpha: float, seed: int) -> torch.Tensor:
    """b_e = log(r_e^-alpha / sum_j j^-alpha), r = seeded permutation of 1..E."""
    rank = torch.randperm(num_experts, generator=_gen(seed)).to(torch.float64) + 1.0
    norm = sum(j ** -alpha for j in range(1, num_experts + 1))
    return torch.log(rank.pow(-alpha) / norm).to(torch.float32)


def zipf_logits(tokens: int, num_experts: int, seed: int, alpha: float = 1.2,
                device="cpu") -> torch.Tensor:
    """Prefill: N(0, 1) noise plus the Zipf(alpha) popularity bias."""
    noise = torch.randn((tokens, num_experts), generator=_gen(seed), dtype=torch.float32)
    return (noise + zipf_bias(num_experts, alpha, seed + 1)[None, :]).to(device)


def capacity_for(tokens: int, shape: LayerShape, factor: float) -> int:
    """Token-scaled capacity, the reference formula (moe.py:882-885)."""
    return max(1, math.ceil(factor * tokens * shape.top_k / shape.num_experts))
