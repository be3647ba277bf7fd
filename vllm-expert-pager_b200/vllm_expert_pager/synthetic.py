"""Seeded synthetic inputs for the expert-paging benchmarks and tests.

There are no model checkpoints or routing logs offline, so every configuration
is regenerated from seeds with CPU torch generators (deterministic for a given
torch build):

* ``fp8_expert``: one expert of a Qwen3-style FP8 MoE layer.  w13 ``[1024, 2048]``
  and w2 ``[2048, 512]`` drawn from N(0, 0.02) in bf16 and quantised to
  float8_e4m3fn with one fp32 scale (amax / 448) per 128x128 block.
* ``zipf_trace``: batch-1 top-8 decode routing over 256 experts.  Expert ranks
  follow Zipf(s=1.1) (``p[r] ~ (r+1)**-s``) over a per-layer seeded
  permutation; each step draws 8 distinct ranks.
* ``uniform_routing``: prefill routing, every token picks ``topk`` distinct
  experts uniformly at random.

This module imports nothing else from the package, so the golden-fixture
generator can load it by path next to the reference implementation.
"""

from __future__ import annotations

import torch

HIDDEN = 2048
MOE_INTER = 512
NUM_EXPERTS = 256
TOPK = 8
BLOCK = 128
FP8_MAX = 448.0

# (rows, cols) of the two per-expert weights, in name order.
SHAPES = {"w13_weight": (2 * MOE_INTER, HIDDEN), "w2_weight": (HIDDEN, MOE_INTER)}


def quantize_block_fp8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 ``[R, C]`` -> (float8_e4m3fn ``[R, C]``, fp32 scales ``[R/128, C/128]``)."""
    R, C = w.shape
    blocks = w.float().view(R // BLOCK, BLOCK, C // BLOCK, BLOCK)
    scale = blocks.abs().amax(dim=(1, 3)) / FP8_MAX
    q = (blocks / scale[:, None, :, None]).to(torch.float8_e4m3fn)
    return q.view(R, C), scale


def fp8_expert(gen: torch.Generator) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
    """One expert: ``{name: (fp8 weight, fp32 block scales)}``, w13 drawn before w2."""
    out = {}
    for name, shape in SHAPES.items():
        w = (torch.randn(shape, generator=gen) * 0.02).to(torch.bfloat16)
        out[name] = quantize_block_fp8(w)
    return out


def fp8_experts(count: int, seed: int = 0):
    """``count`` experts from one generator seeded ``seed`` (config 1 uses 8, seed 0)."""
    gen = torch.Generator().manual_seed(seed)
    return [fp8_expert(gen) for _ in range(count)]


def fp8_experts_device(count: int, device: torch.device, seed: int = 0, batch: int = 32):
    """``count`` experts drawn on the device (torch's CUDA generator seeded ``seed``).

    Same distribution and quantisation as ``fp8_expert`` but generated
    ``batch`` experts at a time on the GPU (the CPU generator is too slow for
    hundreds of experts).  Returns ``{name: (fp8 [count, r, c], fp32 scales
    [count, r/128, c/128])}``.
    """
    gen = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for name, (r, c) in SHAPES.items():
        q = torch.empty((count, r, c), dtype=torch.float8_e4m3fn, device=device)
        sc = torch.empty((count, r // BLOCK, c // BLOCK), dtype=torch.float32, device=device)
        for e0 in range(0, count, batch):
            n = min(batch, count - e0)
            w = (torch.randn((n, r, c), generator=gen, device=device) * 0.02).to(torch.bfloat16)
            blocks = w.float().view(n, r // BLOCK, BLOCK, c // BLOCK, BLOCK)
            amax = blocks.abs().amax(dim=(2, 4)) / FP8_MAX
            q[e0 : e0 + n] = (blocks / amax[:, :, None, :, None]).to(torch.float8_e4m3fn).view(n, r, c)
            sc[e0 : e0 + n] = amax
        out[name] = (q, sc)
    return out


def row_bytes(q: torch.Tensor) -> torch.Tensor:
    """The raw bytes of a weight as a flat uint8 tensor."""
    return q.contiguous().view(torch.uint8).reshape(-1)


def zipf_trace(steps: int = 4096, num_experts: int = NUM_EXPERTS, topk: int = TOPK,
               s: float = 1.1, layer: int = 0) -> torch.Tensor:
    """Decode routing ``int32 [steps, topk]`` for one layer (distinct ids per step)."""
    perm = torch.randperm(num_experts, generator=torch.Generator().manual_seed(layer))
    p = (torch.arange(num_experts, dtype=torch.float64) + 1.0) ** -s
    gen = torch.Generator().manual_seed(1000 + layer)
    out = torch.empty((steps, topk), dtype=torch.int32)
    for i in range(steps):
        ranks = torch.multinomial(p, topk, replacement=False, generator=gen)
        out[i] = perm[ranks].to(torch.int32)
    return out


def uniform_routing(tokens: int, num_experts: int = NUM_EXPERTS, topk: int = TOPK,
                    seed: int = 0) -> torch.Tensor:
    """Prefill routing ``int32 [tokens, topk]``: distinct uniform experts per token."""
    gen = torch.Generator().manual_seed(seed)
    return torch.rand((tokens, num_experts), generator=gen).topk(topk).indices.to(torch.int32)
