"""vLLM's Triton FP8 fused MoE, split at the top-k sum.

The MoE GEMMs are vLLM's (``fused_moe_kernel``), the callee of the paging path,
not part of it.  The reference plugin reaches them through
``RoutedExperts.forward_modular`` and intercepts ``TritonExperts.moe_sum`` to
take the top-k sum once across chunks (experts.py:541-556).  This module runs
the same sequence as vLLM's ``fused_experts_impl`` (quantise the input, align
tokens to experts honouring ``expert_map``, w13 GEMM, SiLU-and-mul, quantise,
w2 GEMM into ``intermediate_cache3``) and stops before ``moe_sum``, so callers
outside a vLLM model (the benchmark, the bit-exactness tests) can collect the
per-expert contributions themselves.  Experts whose ``expert_map`` entry is -1
contribute exact zeros (vLLM writes zeros for them).
"""

from __future__ import annotations

import functools

import torch


@functools.lru_cache(maxsize=1)
def _vllm():
    from vllm import _custom_ops as ops
    from vllm.model_executor.layers.fused_moe import fused_moe as fm
    from vllm.model_executor.layers.fused_moe.activation import MoEActivation, apply_moe_activation
    from vllm.model_executor.layers.fused_moe.utils import moe_kernel_quantize_input

    return ops, fm, MoEActivation, apply_moe_activation, moe_kernel_quantize_input


def moe_config(w13_shape, w2_shape, topk: int, tokens: int, block_shape=(128, 128)) -> dict:
    """vLLM's kernel config for these weight shapes and token count (fp8 w8a8)."""
    _, fm, *_ = _vllm()
    dtype = fm._get_config_dtype_str(use_fp8_w8a8=True, dtype=torch.bfloat16)
    return fm.try_get_optimal_moe_config(tuple(w13_shape), tuple(w2_shape), topk, dtype, tokens,
                                         block_shape=list(block_shape))


def contributions(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor,
                  w13_scale: torch.Tensor, w2_scale: torch.Tensor, topk_weights: torch.Tensor,
                  topk_ids: torch.Tensor, expert_map: torch.Tensor | None,
                  global_num_experts: int, config: dict | None = None,
                  block_shape=(128, 128)) -> torch.Tensor:
    """Per-(token, k) expert outputs ``[T, topk, hidden]`` (bf16), before the top-k sum.

    ``w13``/``w2`` are the expert rows the kernel indexes (a slab in slot order
    with ``expert_map`` mapping expert ids to slots, or all experts with
    ``expert_map=None``).
    """
    ops, fm, MoEActivation, apply_moe_activation, quantize = _vllm()
    T, H = x.shape
    topk = topk_ids.shape[1]
    N = w13.shape[1]
    if config is None:
        config = moe_config(w13.shape, w2.shape, topk, T, block_shape)
    bs = list(block_shape)
    qx, a1_scale = quantize(A=x, A_scale=None, quant_dtype=torch.float8_e4m3fn,
                            per_act_token_quant=False, block_shape=bs)
    sorted_ids, expert_ids, padded = fm._prepare_expert_assignment(
        topk_ids, config, T, topk, global_num_experts, expert_map, block_shape=bs,
        ignore_invalid_experts=True)
    cache1 = torch.empty((T, topk, N), dtype=x.dtype, device=x.device)
    common = dict(compute_type=fm.tl.bfloat16, use_fp8_w8a8=True, use_int8_w8a8=False,
                  use_int8_w8a16=False, use_int4_w4a16=False, per_channel_quant=False,
                  block_shape=bs)
    fm.dispatch_fused_moe_kernel(qx, w13, cache1, a1_scale, w13_scale, None, topk_weights,
                                 sorted_ids, expert_ids, padded, False, topk, config, **common)
    cache2 = torch.empty((T * topk, N // 2), dtype=x.dtype, device=x.device)
    apply_moe_activation(MoEActivation.SILU, cache2, cache1.view(-1, N))
    q2, a2_scale = quantize(A=cache2, A_scale=None, quant_dtype=torch.float8_e4m3fn,
                            per_act_token_quant=False, block_shape=bs)
    cache3 = torch.zeros((T, topk, H), dtype=x.dtype, device=x.device)
    fm.dispatch_fused_moe_kernel(q2, w2, cache3, a2_scale, w2_scale, None, topk_weights,
                                 sorted_ids, expert_ids, padded, True, 1, config, **common)
    return cache3


def moe_sum(cache3: torch.Tensor, out: torch.Tensor) -> None:
    """vLLM's top-k sum (``ops.moe_sum``: fp32 sum, one rounding to bf16)."""
    ops, *_ = _vllm()
    ops.moe_sum(cache3, out)
