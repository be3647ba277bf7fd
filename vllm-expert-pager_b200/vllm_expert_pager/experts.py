"""Hook vLLM's ``RoutedExperts`` so expert weights are referenced through a slab.

Drop-in for src/vllm_expert_pager/experts.py of monochromegane/vllm-expert-pager:
the same class (``ExpertPagerRoutedExperts``), overrides (``__init__``,
``expert_map``, ``weight_loader``, ``forward_modular``, ``forward_monolithic``,
the wrapped ``process_weights_after_loading``), settings
(``VLLM_EXPERT_PAGER_*``, same defaults and validation messages) and errors.
It targets the vLLM API the reference targets (0.28 / 0.29: ``RoutedExperts``,
``TritonExperts.moe_sum``, ``Fp8MoeBackend``).

The paging itself lives in ``pager.LayerPager`` (one per MoE layer): decode
steps page the step's experts into the layer's cache slab, steps with more
experts than slots run them through the shared working slab in chunks, and
vLLM's own fused MoE runs on the slab with ``expert_map``.  New setting:
``VLLM_EXPERT_PAGER_OVERLAP`` (default 1) overlaps chunk k+1's copies with
chunk k's MoE using a working slab of 2 x WORKING_ROWS rows; 0 keeps the
reference's serial order and W rows.
"""

import os

import torch
from vllm.config import get_current_vllm_config
from vllm.logger import init_logger
from vllm.model_executor.layers.fused_moe.experts.triton_moe import TritonExperts
from vllm.model_executor.layers.fused_moe.oracle.fp8 import Fp8MoeBackend
from vllm.model_executor.layers.fused_moe.routed_experts import RoutedExperts

from vllm_expert_pager.pager import PARAMS, LayerPager, WorkingSlab
from vllm_expert_pager.store import Store

# A logger outside the "vllm." namespace inherits the root's WARNING level in
# vLLM's logging setup and drops info lines (experts.py:33-37).
logger = init_logger(f"vllm.{__name__}")

CACHE_SLOTS = int(os.environ.get("VLLM_EXPERT_PAGER_CACHE_SLOTS", "32"))
RAM_SLOTS = os.environ.get("VLLM_EXPERT_PAGER_RAM_SLOTS")
SSD_PATH = os.environ.get("VLLM_EXPERT_PAGER_SSD_PATH")
COMPRESS = os.environ.get("VLLM_EXPERT_PAGER_COMPRESS", "auto")
PITCH_RATIO = float(os.environ.get("VLLM_EXPERT_PAGER_PITCH", "0.89"))
WORKING_ROWS = int(os.environ.get("VLLM_EXPERT_PAGER_WORKING_ROWS", "64"))
LOG_INTERVAL = int(os.environ.get("VLLM_EXPERT_PAGER_LOG_INTERVAL", "1000"))
OVERLAP = os.environ.get("VLLM_EXPERT_PAGER_OVERLAP", "1") not in ("0", "false", "off")

_store: Store | None = None
# One WorkingSlab serves every layer.  vLLM calls the MoE layers in order on a
# single stream, so a layer's chunk loop never overlaps another layer's
# (experts.py:79-83).
_working: WorkingSlab | None = None


class ExpertPagerRoutedExperts(RoutedExperts):
    """``RoutedExperts`` whose expert weights are paged through a slab.

    The path is chosen from the shape of ``topk_ids`` alone (decode when it has
    no more elements than cache slots), so graph capture and replay agree.
    """

    _expert_pager_expert_map: torch.Tensor | None = None
    _expert_pager_calls = 0

    def __init__(self, *args, **kwargs) -> None:
        super().__init__(*args, **kwargs)
        if self.use_ep or self.local_num_experts != self.global_num_experts:
            raise RuntimeError(
                f"{self.layer_name}: vllm-expert-pager does not support expert "
                f"parallelism (local={self.local_num_experts}, "
                f"global={self.global_num_experts})"
            )
        if self.moe_config.moe_parallel_config.tp_size != 1:
            raise RuntimeError(
                f"{self.layer_name}: vllm-expert-pager does not support tensor parallelism"
            )
        E = self.global_num_experts
        params = {name: getattr(self, name) for name in PARAMS}

        global _store
        if _store is None:
            R = int(RAM_SLOTS) if RAM_SLOTS else E
            if R < CACHE_SLOTS:
                raise ValueError(
                    f"VLLM_EXPERT_PAGER_RAM_SLOTS={R} must be >= "
                    f"VLLM_EXPERT_PAGER_CACHE_SLOTS={CACHE_SLOTS}"
                )
            if WORKING_ROWS < 1:
                raise ValueError(
                    f"VLLM_EXPERT_PAGER_WORKING_ROWS must be >= 1, got {WORKING_ROWS}"
                )
            if COMPRESS not in ("auto", "on", "off"):
                raise ValueError(
                    f"VLLM_EXPERT_PAGER_COMPRESS must be auto, on or off, got {COMPRESS!r}"
                )
            compress = R < E if COMPRESS == "auto" else COMPRESS == "on"
            _store = Store(
                num_layers=get_current_vllm_config().model_config.hf_text_config.num_hidden_layers,
                num_experts=E,
                ram_slots=R,
                # RAM-tier rows for the SSD reads of the working path: 2 x W, so
                # that the reads of one chunk never land in rows whose previous
                # contents an earlier chunk is still copying to the GPU.
                working_rows=2 * WORKING_ROWS,
                row_bytes={n: p[0].numel() * p.element_size() for n, p in params.items()},
                compress=compress,
                pitch_ratio=PITCH_RATIO,
                path=SSD_PATH,
                device=params["w13_weight"].device,
            )
        self._expert_pager_store = _store
        self._expert_pager_layer = _store.add_layer()

        # The codec splits each fp8 byte into its exponent and sign/mantissa
        # bits; weights in Marlin's repacked layout break that assumption.
        if _store.compress and (
            getattr(self.quant_method, "fp8_backend", None) == Fp8MoeBackend.MARLIN
        ):
            raise RuntimeError(
                f"{self.layer_name}: vllm-expert-pager compresses raw fp8 rows and "
                "does not support the MARLIN backend; set VLLM_EXPERT_PAGER_COMPRESS=off"
            )
        # The weights are paged, so the layer keeps a single real row per param;
        # a stride-0 view makes it look [E, ...] to process_weights_after_loading
        # (experts.py:160-167), and _expert_pager_setup trims it back.
        for p in params.values():
            p.data = torch.empty((1, *p.shape[1:]), dtype=p.dtype, device=p.device).expand(p.shape)
        # The loader delivers w1 (gate) and w3 (up) separately; their halves of
        # an expert's w13 row are collected here until the row is complete.
        self._expert_pager_stage: dict[int, tuple[torch.Tensor, set[str]]] = {}

        original = self.quant_method.process_weights_after_loading

        def process_weights_after_loading(layer: RoutedExperts) -> None:
            original(layer)
            layer._expert_pager_setup()

        self.quant_method.process_weights_after_loading = process_weights_after_loading

    # ---- expert_map override ----

    @property
    def expert_map(self) -> torch.Tensor | None:
        if self._expert_pager_expert_map is not None:
            return self._expert_pager_expert_map
        return super().expert_map

    # ---- loading ----

    def weight_loader(self, param: torch.nn.Parameter, loaded_weight: torch.Tensor,
                      weight_name: str, shard_id: str, expert_id: int,
                      return_success: bool = False) -> bool | None:
        if param is self.w13_weight:
            N, H = self.intermediate_size_per_partition, self.hidden_size
            buf, seen = self._expert_pager_stage.setdefault(
                expert_id,
                (torch.empty((2 * N, H), dtype=loaded_weight.dtype, device="cpu"), set()),
            )
            half = 0 if shard_id == "w1" else N  # w13 row = [w1; w3]
            buf[half : half + N].copy_(loaded_weight)
            seen.add(shard_id)
            if seen != {"w1", "w3"}:
                return True if return_success else None
            del self._expert_pager_stage[expert_id]
            self._expert_pager_store.write(self._expert_pager_layer, expert_id, "w13_weight", buf)
        elif param is self.w2_weight:
            self._expert_pager_store.write(self._expert_pager_layer, expert_id, "w2_weight",
                                           loaded_weight)
        else:
            return super().weight_loader(param, loaded_weight, weight_name, shard_id, expert_id,
                                         return_success)
        return True if return_success else None

    # ---- after loading ----

    def _expert_pager_setup(self) -> None:
        store = self._expert_pager_store
        params = {name: getattr(self, name) for name in PARAMS}
        shapes = {}
        for name, p in params.items():
            p.data = p.data[:1].clone()  # undo the expand; keep one row
            if p.data.numel() * p.element_size() != store.row_bytes[name]:
                raise RuntimeError(
                    f"{self.layer_name}: {name} row has {p.data.numel() * p.element_size()} B "
                    f"after process_weights_after_loading, expected {store.row_bytes[name]}"
                )
            shapes[name] = (tuple(p.shape[1:]), p.dtype)
        scale_name = getattr(self.quant_method, "weight_scale_name", None)
        if scale_name is None:
            raise RuntimeError(
                f"{self.layer_name}: {type(self.quant_method).__name__} has no "
                "weight_scale_name; vllm-expert-pager only knows how to stage FP8 scales"
            )
        self._expert_pager_scale_names = [f"{w}_{scale_name}" for w in ("w13", "w2")]
        scales = {n: getattr(self, n).data for n in self._expert_pager_scale_names}

        global _working
        if _working is None:
            all_shapes = dict(shapes)
            all_shapes.update({n: (tuple(s.shape[1:]), s.dtype) for n, s in scales.items()})
            _working = WorkingSlab(WORKING_ROWS, all_shapes, store, store.device,
                                   halves=2 if OVERLAP else 1)
        self._expert_pager = LayerPager(store, self._expert_pager_layer, CACHE_SLOTS, scales,
                                        shapes, _working)
        self._expert_pager_table = self._expert_pager.vram
        self._expert_pager_ram = self._expert_pager.ram
        self._expert_pager_map = self._expert_pager.expert_map
        self._expert_pager_params = {n: getattr(self, n) for n in
                                     list(PARAMS) + self._expert_pager_scale_names}
        experts = self.quant_method.moe_kernel.fused_experts
        if getattr(type(experts), "moe_sum", None) is not TritonExperts.moe_sum:
            raise RuntimeError(
                f"{self.layer_name}: vllm-expert-pager chunks the prefill through "
                f"TritonExperts.moe_sum, but the kernel is {type(experts).__name__}"
            )
        self._expert_pager_experts = experts
        logger.info_once(
            "vllm-expert-pager: %d cache slots/layer, %d RAM slots/layer, %d working rows%s, "
            "rows %s", CACHE_SLOTS, store.ram_slots, WORKING_ROWS,
            " x2 (overlapped chunks)" if OVERLAP else "",
            f"compressed to {'+'.join(str(store.pitch[n]) for n in PARAMS)} B"
            if store.compress else "raw",
        )  # fmt: skip

    # ---- forward ----

    def forward_modular(self, x: torch.Tensor, topk_weights: torch.Tensor,
                        topk_ids: torch.Tensor, shared_experts=None,
                        shared_experts_input: torch.Tensor | None = None) -> torch.Tensor:
        store = self._expert_pager_store
        if store.failed is not None:
            raise RuntimeError(f"vllm-expert-pager: SSD read failed\n{store.failed}")
        gave_up = self._expert_pager.step_errors()
        if gave_up:
            raise RuntimeError(
                f"vllm-expert-pager: {self.layer_name}: {gave_up} wait(s) of the decode step "
                "gave up, so its slab holds stale rows"
            )
        if topk_ids.numel() > self._expert_pager.cache_slots:
            return self._expert_pager_forward_working(x, topk_weights, topk_ids, shared_experts,
                                                      shared_experts_input)
        res = self._expert_pager.decode(topk_ids)
        self._expert_pager_log()
        return self._expert_pager_run(res.slabs, x, topk_weights, topk_ids, shared_experts,
                                      shared_experts_input)

    def _expert_pager_forward_working(self, x, topk_weights, topk_ids, shared_experts,
                                      shared_experts_input):
        """Run the step's experts through the working slab in chunks (experts.py:455-577).

        Every chunk's MoE writes its experts' contributions (exact zeros for the
        others) to intermediate_cache3; ``moe_sum`` is intercepted to add them
        up, and the real top-k sum runs once, in the last chunk, so the result
        equals a single unchunked run bit for bit.
        """
        experts = self._expert_pager_experts
        moe_sum = type(experts).moe_sum
        acc: dict[str, torch.Tensor] = {}
        state = {"k": 0, "n": 1}

        def collect(cache3: torch.Tensor, output: torch.Tensor) -> None:
            acc["c"] = cache3.clone() if "c" not in acc else acc["c"].add_(cache3)
            if state["k"] == state["n"] - 1:
                moe_sum(experts, acc["c"], output)

        def run_chunk(k, n, slabs, expert_map):
            state["k"], state["n"] = k, n
            return self._expert_pager_run(
                slabs, x, topk_weights, topk_ids,
                shared_experts if k == 0 else None,
                shared_experts_input if k == 0 else None,
            )  # fmt: skip

        experts.moe_sum = collect  # the instance attribute shadows the method, for the chunks only
        try:
            out = self._expert_pager.working_chunks(topk_ids, run_chunk, overlap=OVERLAP)
        finally:
            del experts.moe_sum
        self._expert_pager_log()
        return out

    def _expert_pager_run(self, slabs, x, topk_weights, topk_ids, shared_experts,
                          shared_experts_input):
        """Point the weights and scales at the slab and run vLLM's MoE (experts.py:579-604)."""
        saved = {name: param.data for name, param in self._expert_pager_params.items()}
        try:
            for name, param in self._expert_pager_params.items():
                param.data = slabs[name]
            self._expert_pager_expert_map = self._expert_pager_map
            return super().forward_modular(x=x, topk_weights=topk_weights, topk_ids=topk_ids,
                                           shared_experts=shared_experts,
                                           shared_experts_input=shared_experts_input)
        finally:
            self._expert_pager_expert_map = None
            for name, data in saved.items():
                self._expert_pager_params[name].data = data

    def forward_monolithic(self, *args, **kwargs) -> torch.Tensor:
        raise RuntimeError(
            f"{self.layer_name}: vllm-expert-pager only supports modular MoE kernels, "
            f"but {type(self.quant_method).__name__} is monolithic. Expert weights "
            "would not be staged."
        )

    def _expert_pager_log(self) -> None:
        self._expert_pager_calls += 1
        if LOG_INTERVAL <= 0 or self._expert_pager_calls % LOG_INTERVAL:
            return
        if torch.cuda.is_current_stream_capturing():  # reading counters would sync
            return
        vram, ram = self._expert_pager.vram, self._expert_pager.ram
        vh, vm, rh, rm = torch.cat([vram.counters[1:], ram.counters[1:]]).tolist()
        logger.info(
            "vllm-expert-pager %s: vram hit %.1f%% (%d/%d), ram hit %.1f%% (%d/%d)",
            self.layer_name, 100.0 * vh / (vh + vm) if vh + vm else 0.0, vh, vh + vm,
            100.0 * rh / (rh + rm) if rh + rm else 0.0, rh, rh + rm,
        )  # fmt: skip
        store = self._expert_pager_store
        if self._expert_pager_layer == 0 and store.fetches:
            logger.info(
                "vllm-expert-pager ssd: %d fetches, %d reads, %.3f s, %.2f ms/fetch, "
                "%d re-publishes, %d give-ups, %d missed",
                store.fetches, store.reads, store.io_seconds,
                1e3 * store.io_seconds / store.fetches, int(store.req[store.retry_at]),
                int(store.req[store.giveup_at]), store.missed,
            )  # fmt: skip
        gave_up = self._expert_pager.step_errors()
        if gave_up:
            logger.warning("vllm-expert-pager %s: %d decode-step wait(s) gave up",
                           self.layer_name, gave_up)


def register() -> None:
    RoutedExperts.register_oot(ExpertPagerRoutedExperts)
