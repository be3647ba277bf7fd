"""A stand-in for vLLM >= 0.28's ``RoutedExperts`` (test infrastructure).

The image ships vLLM 0.22, which has no ``vllm.model_executor.layers.fused_moe.
routed_experts``.  This module provides a minimal class with the attributes and
methods the plugin's hook uses (the reference's experts.py reads them): expert
and parallel configuration, ``w13_weight``/``w2_weight`` and their block scales
as parameters, ``quant_method`` with ``process_weights_after_loading``,
``weight_scale_name``, ``fp8_backend`` and ``moe_kernel.fused_experts`` (a real
vLLM ``TritonExperts``), ``weight_loader``, the ``expert_map`` property, and a
``forward_modular`` that runs vLLM's Triton FP8 fused MoE on the current
parameters and finishes with ``fused_experts.moe_sum`` as vLLM does.
"""

from __future__ import annotations

import sys
import types
from types import SimpleNamespace

import torch

MODULE = "vllm.model_executor.layers.fused_moe.routed_experts"


def install() -> type:
    if MODULE in sys.modules and hasattr(sys.modules[MODULE], "RoutedExperts"):
        return sys.modules[MODULE].RoutedExperts
    from vllm_expert_pager import moe

    class RoutedExperts(torch.nn.Module):
        registered = None

        @classmethod
        def register_oot(cls, sub):
            cls.registered = sub

        def __init__(self, num_experts, hidden, inter, layer_name, quant_method, device,
                     tp_size=1, use_ep=False):
            super().__init__()
            E = num_experts
            self.global_num_experts = self.local_num_experts = E
            self.use_ep = use_ep
            self.layer_name = layer_name
            self.moe_config = SimpleNamespace(moe_parallel_config=SimpleNamespace(tp_size=tp_size))
            self.hidden_size, self.intermediate_size_per_partition = hidden, inter
            self.quant_method = quant_method
            fp8 = torch.float8_e4m3fn
            P = torch.nn.Parameter
            self.w13_weight = P(torch.zeros((E, 2 * inter, hidden), dtype=fp8, device=device),
                                requires_grad=False)
            self.w2_weight = P(torch.zeros((E, hidden, inter), dtype=fp8, device=device),
                               requires_grad=False)
            self.w13_weight_scale_inv = P(torch.zeros((E, 2 * inter // 128, hidden // 128),
                                                      device=device), requires_grad=False)
            self.w2_weight_scale_inv = P(torch.zeros((E, hidden // 128, inter // 128),
                                                     device=device), requires_grad=False)

        @property
        def expert_map(self):
            return None

        def weight_loader(self, param, loaded_weight, weight_name, shard_id, expert_id,
                          return_success=False):
            n = self.intermediate_size_per_partition // 128
            if param is self.w13_weight_scale_inv:
                half = 0 if shard_id == "w1" else n
                param.data[expert_id][half : half + n].copy_(loaded_weight)
            else:
                param.data[expert_id].copy_(loaded_weight)
            return True if return_success else None

        def forward_modular(self, x, topk_weights, topk_ids, shared_experts=None,
                            shared_experts_input=None):
            cache3 = moe.contributions(x, self.w13_weight, self.w2_weight,
                                       self.w13_weight_scale_inv, self.w2_weight_scale_inv,
                                       topk_weights, topk_ids, self.expert_map,
                                       self.global_num_experts, config=self.quant_method.config)
            out = torch.empty_like(x)
            self.quant_method.moe_kernel.fused_experts.moe_sum(cache3, out)
            return out

    mod = types.ModuleType(MODULE)
    mod.RoutedExperts = RoutedExperts
    sys.modules[MODULE] = mod
    return RoutedExperts


def quant_method(config: dict, backend=None):
    """A quant_method with the fields the hook reads; fused_experts is a real TritonExperts."""
    from vllm.model_executor.layers.fused_moe.experts.triton_moe import TritonExperts
    from vllm.model_executor.layers.fused_moe.oracle.fp8 import Fp8MoeBackend

    return SimpleNamespace(
        process_weights_after_loading=lambda layer: None,
        weight_scale_name="weight_scale_inv",
        fp8_backend=backend if backend is not None else Fp8MoeBackend.TRITON,
        moe_kernel=SimpleNamespace(fused_experts=TritonExperts.__new__(TritonExperts)),
        config=config,
    )
