"""The vLLM hook (experts.py) end to end: load, setup, decode and prefill steps.

Drives ``ExpertPagerRoutedExperts`` on top of the stand-in ``RoutedExperts``
(tests/vllm_standin.py; vLLM 0.22 in this image has none) through the same
calls vLLM makes: construction, ``weight_loader`` per shard (w1/w3 halves, w2,
block scales), ``process_weights_after_loading``, then ``forward_modular``.
Every output must equal, bit for bit, vLLM's fused MoE over all experts
resident (same kernel config).
"""

import importlib
import os
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
E, H, I, TOPK, L = 32, 2048, 512, 8, 2


@pytest.fixture
def experts_mod(tmp_path, monkeypatch):
    import vllm_standin

    vllm_standin.install()
    env = {"VLLM_EXPERT_PAGER_CACHE_SLOTS": "8", "VLLM_EXPERT_PAGER_RAM_SLOTS": "16",
           "VLLM_EXPERT_PAGER_SSD_PATH": str(tmp_path / "pager.bin"),
           "VLLM_EXPERT_PAGER_WORKING_ROWS": "8", "VLLM_EXPERT_PAGER_LOG_INTERVAL": "3"}
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    import vllm_expert_pager.experts as ex

    ex = importlib.reload(ex)
    cfg = SimpleNamespace(model_config=SimpleNamespace(
        hf_text_config=SimpleNamespace(num_hidden_layers=L)))
    monkeypatch.setattr(ex, "get_current_vllm_config", lambda: cfg)
    yield ex
    if ex._store is not None:
        ex._store.release()
    ex._store = None
    ex._working = None


def make_layers(ex, weights, config):
    import vllm_standin

    layers = []
    for layer in range(L):
        m = ex.ExpertPagerRoutedExperts(E, H, I, f"model.layers.{layer}.mlp.experts",
                                        vllm_standin.quant_method(config), DEV)
        (w13, s13), (w2, s2) = weights[layer]["w13_weight"], weights[layer]["w2_weight"]
        for e in range(E):
            # vLLM loads gate (w1) and up (w3) halves separately, then w2, then scales.
            m.weight_loader(m.w13_weight, w13[e, :I].cpu(), "w13", "w1", e)
            m.weight_loader(m.w13_weight, w13[e, I:].cpu(), "w13", "w3", e)
            m.weight_loader(m.w2_weight, w2[e].cpu(), "w2", "w2", e)
            m.weight_loader(m.w13_weight_scale_inv, s13[e, : I // 128], "s13", "w1", e)
            m.weight_loader(m.w13_weight_scale_inv, s13[e, I // 128 :], "s13", "w3", e)
            m.weight_loader(m.w2_weight_scale_inv, s2[e], "s2", "w2", e)
        m.quant_method.process_weights_after_loading(m)
        layers.append(m)
    return layers


def test_hook_outputs_match_unpaged_moe(experts_mod):
    from vllm_expert_pager import moe, synthetic

    ex = experts_mod
    weights = [synthetic.fp8_experts_device(E, DEV, seed=10 + layer) for layer in range(L)]
    config = moe.moe_config((E, 2 * I, H), (E, H, I), TOPK, 64)
    layers = make_layers(ex, weights, config)
    assert ex._store.compress and ex._store.path is not None  # R < E: compressed + SSD
    g = torch.Generator(device=DEV).manual_seed(0)
    for step in range(12):
        T = 64 if step in (3, 9) else 1  # two prefill-sized steps (working path)
        x = (torch.randn((T, H), generator=g, device=DEV) * 0.5).to(torch.bfloat16)
        ids = torch.rand((T, E), generator=g, device=DEV).topk(TOPK).indices.to(torch.int32)
        tw = torch.softmax(torch.randn((T, TOPK), generator=g, device=DEV), -1)
        for layer, m in enumerate(layers):
            out = m.forward_modular(x, tw, ids)
            (w13, s13), (w2, s2) = weights[layer]["w13_weight"], weights[layer]["w2_weight"]
            ref3 = moe.contributions(x, w13, w2, s13, s2, tw, ids, None, E, config)
            ref = torch.empty_like(x)
            moe.moe_sum(ref3, ref)
            torch.cuda.synchronize()
            assert torch.equal(out, ref), f"step {step} layer {layer}"
    assert ex._store.failed is None and ex._store.reads > 0
    assert all(m._expert_pager.step_errors() == 0 for m in layers)
    # Parameters are back to their one-row placeholders after every forward.
    assert layers[0].w13_weight.shape[0] == 1 and layers[0].expert_map is None
    # A decode-step wait that gave up (planted in the pinned host copy the kernel
    # keeps) stops the next eager forward, as a failed SSD read does.
    layers[1]._expert_pager.step_errors_host[0] = 2
    with pytest.raises(RuntimeError, match="gave up"):
        layers[1].forward_modular(x, tw, ids)
    layers[1]._expert_pager.step_errors_host[0] = 0


def test_hook_replays_in_a_cuda_graph(experts_mod):
    """forward_modular of a batch-1 decode step, captured once in a CUDA graph with no
    host synchronisation inside the capture, then replayed with new x / topk_ids /
    topk_weights written into the captured buffers: every replay equals the eager
    unpaged MoE bit for bit (compressed RAM tier + SSD tier, both layers)."""
    from vllm_expert_pager import moe, synthetic

    ex = experts_mod
    weights = [synthetic.fp8_experts_device(E, DEV, seed=40 + layer) for layer in range(L)]
    config = moe.moe_config((E, 2 * I, H), (E, H, I), TOPK, 64)
    layers = make_layers(ex, weights, config)
    g = torch.Generator(device=DEV).manual_seed(3)

    def draw():
        x = (torch.randn((1, H), generator=g, device=DEV) * 0.5).to(torch.bfloat16)
        ids = torch.rand((1, E), generator=g, device=DEV).topk(TOPK).indices.to(torch.int32)
        tw = torch.softmax(torch.randn((1, TOPK), generator=g, device=DEV), -1)
        return x, ids, tw

    x, ids, tw = (t.clone() for t in draw())
    for _ in range(2):  # eager warm-up: Triton compilation, tables
        for m in layers:
            m.forward_modular(x, tw, ids)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(graph, stream=s):
        # Any torch operation that would synchronise with the host raises here.
        torch.cuda.set_sync_debug_mode("error")
        try:
            outs = [m.forward_modular(x, tw, ids) for m in layers]
        finally:
            torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()
    for step in range(10):
        nx, nids, ntw = draw()
        x.copy_(nx)
        ids.copy_(nids)
        tw.copy_(ntw)
        graph.replay()
        torch.cuda.synchronize()
        for layer, out in enumerate(outs):
            (w13, s13), (w2, s2) = weights[layer]["w13_weight"], weights[layer]["w2_weight"]
            ref = torch.empty_like(x)
            moe.moe_sum(moe.contributions(x, w13, w2, s13, s2, tw, ids, None, E, config), ref)
            assert torch.equal(out, ref), f"replay {step} layer {layer}"
    del graph
    assert ex._store.failed is None and ex._store.reads > 0
    assert all(m._expert_pager.step_errors() == 0 for m in layers)


def test_hook_rejects_unsupported_setups(experts_mod, monkeypatch):
    import vllm_standin
    from vllm.model_executor.layers.fused_moe.oracle.fp8 import Fp8MoeBackend

    ex = experts_mod
    with pytest.raises(RuntimeError, match="expert parallelism"):
        ex.ExpertPagerRoutedExperts(E, H, I, "l", vllm_standin.quant_method({}), DEV, use_ep=True)
    with pytest.raises(RuntimeError, match="tensor parallelism"):
        ex.ExpertPagerRoutedExperts(E, H, I, "l", vllm_standin.quant_method({}), DEV, tp_size=2)
    with pytest.raises(RuntimeError, match="MARLIN"):
        ex.ExpertPagerRoutedExperts(E, H, I, "l",
                                    vllm_standin.quant_method({}, Fp8MoeBackend.MARLIN), DEV)
    m = ex.ExpertPagerRoutedExperts(E, H, I, "l", vllm_standin.quant_method({}), DEV)
    with pytest.raises(RuntimeError, match="monolithic"):
        m.forward_monolithic()


def test_hook_validates_settings(experts_mod, monkeypatch):
    import vllm_standin

    ex = experts_mod
    monkeypatch.setattr(ex, "RAM_SLOTS", "4")
    with pytest.raises(ValueError, match="must be >= VLLM_EXPERT_PAGER_CACHE_SLOTS"):
        ex.ExpertPagerRoutedExperts(E, H, I, "l", vllm_standin.quant_method({}), DEV)
    monkeypatch.setattr(ex, "RAM_SLOTS", None)
    monkeypatch.setattr(ex, "COMPRESS", "maybe")
    with pytest.raises(ValueError, match="auto, on or off"):
        ex.ExpertPagerRoutedExperts(E, H, I, "l", vllm_standin.quant_method({}), DEV)


def test_plugin_registers_the_subclass(experts_mod):
    import vllm_standin
    from vllm_expert_pager import plugin

    base = vllm_standin.install()
    plugin.register()
    assert base.registered is experts_mod.ExpertPagerRoutedExperts or \
        base.registered.__name__ == "ExpertPagerRoutedExperts"
    assert os.environ["VLLM_EXPERT_PAGER_CACHE_SLOTS"] == "8"
