"""HuggingFace ``transformers`` fallback rollout engine and the
prepare / generate / finish generation interface (reference:
``lumenrl/engine/inference/hf_engine.py:19-183``,
``lumenrl/engine/inference/generation.py:17-91``).

The native engine (``engine.py``: paged KV, CUDA-graph decode, tcgen05
kernels) serves the Qwen3 family.  ``HFEngine`` covers what it does not: any
architecture ``transformers`` can build from a local directory or an
in-memory module, at eager PyTorch speed.  It is a correctness and coverage
path, not a fast one, and it is never used by the benchmark.

Weights reach it three ways: a local HF directory (``from_pretrained``, no
network), an existing module, or ``from_native`` (a native ``Qwen3Model``
exported through ``hf_state_dict``).  ``update_weights`` loads an HF-named
state dict and fails on incomplete coverage (a parameter not updated, or a
tensor of the state dict that matches no parameter).
"""

from __future__ import annotations

import gc
from typing import Any, Optional

import torch
import torch.nn.functional as F
from torch import Tensor

from lumenrl_b200.core.protocol import DataProto


class HFEngine:
    """Generation and per-token log-probs through a ``transformers`` causal LM."""

    def __init__(self, model: Optional[torch.nn.Module] = None, model_path: Optional[str] = None,
                 dtype: torch.dtype = torch.bfloat16, device: str | torch.device = "cuda",
                 pad_token_id: int = 0, eos_token_id: Optional[int] = None) -> None:
        if model is None and model_path is None:
            raise ValueError("HFEngine needs a module or a local model directory")
        self._model = model
        self._path = model_path
        self.dtype = dtype
        self.device = torch.device(device)
        self.pad_token_id = pad_token_id
        self.eos_token_id = eos_token_id
        self._asleep = False

    # -- construction --------------------------------------------------------------
    @classmethod
    def from_native(cls, native, device: str | torch.device = "cpu", dtype: torch.dtype = torch.float32,
                    **kw) -> "HFEngine":
        """An HF twin of a native ``Qwen3Model`` (same config, same weights)."""
        import transformers
        from lumenrl_b200.utils.checkpoint import hf_config
        cfg = dict(hf_config(native.args))
        arch = cfg.pop("architectures")[0]
        mtype = cfg.pop("model_type")
        cfg.pop("torch_dtype", None)
        config = transformers.AutoConfig.for_model(mtype, **cfg)
        model = getattr(transformers, arch)(config)
        eng = cls(model=model, dtype=dtype, device=device, **kw)
        eng.init()
        eng.update_weights({k: v.detach() for k, v in native.hf_state_dict().items()})   # experts routed in
        return eng

    def init(self) -> None:
        if self._model is None:
            from transformers import AutoModelForCausalLM
            self._model = AutoModelForCausalLM.from_pretrained(self._path, torch_dtype=self.dtype,
                                                               local_files_only=True)
        self._model.to(device=self.device, dtype=self.dtype)
        self._model.eval()

    @property
    def model(self) -> torch.nn.Module:
        if self._model is None:
            raise RuntimeError("HFEngine: call init() first")
        return self._model

    # -- generation ----------------------------------------------------------------
    @torch.no_grad()
    def generate(self, input_ids: Tensor, attention_mask: Optional[Tensor] = None, max_new_tokens: int = 512,
                 temperature: float = 1.0, top_p: float = 1.0, top_k: int = 0, do_sample: bool = True,
                 seed: Optional[int] = None) -> tuple[Tensor, Tensor]:
        """Left-padded prompts [B, L] -> (sequences [B, L + new], mask of the
        same shape: prompt mask, then 1 for generated tokens up to the end)."""
        m = self.model
        ids = input_ids.to(self.device)
        am = attention_mask.to(self.device) if attention_mask is not None else torch.ones_like(ids)
        kw: dict[str, Any] = {"max_new_tokens": max_new_tokens, "pad_token_id": self.pad_token_id,
                              "do_sample": bool(do_sample and temperature > 0)}
        if self.eos_token_id is not None:
            kw["eos_token_id"] = self.eos_token_id
        if kw["do_sample"]:
            kw["temperature"] = float(temperature)
            kw["top_p"] = float(top_p)
            kw["top_k"] = int(top_k) if top_k > 0 else 0
        if seed is not None:
            torch.manual_seed(seed)
        out = m.generate(input_ids=ids, attention_mask=am, **kw)
        L = ids.shape[1]
        mask = torch.ones_like(out)
        mask[:, :L] = am
        gen = out[:, L:]
        if self.eos_token_id is not None:
            # tokens after the first end-of-sequence are padding
            is_eos = (gen == self.eos_token_id).long()
            mask[:, L:] = ((is_eos.cumsum(-1) - is_eos) == 0).long()
        return out, mask

    @torch.no_grad()
    def compute_log_probs(self, input_ids: Tensor, attention_mask: Optional[Tensor] = None,
                          temperature: float = 1.0) -> Tensor:
        """[B, T] sequences -> [B, T-1] log p(token t+1 | prefix), fp32."""
        ids = input_ids.to(self.device)
        am = attention_mask.to(self.device) if attention_mask is not None else None
        logits = self.model(input_ids=ids, attention_mask=am).logits[:, :-1].float() / max(temperature, 1e-6)
        return F.log_softmax(logits, -1).gather(-1, ids[:, 1:].unsqueeze(-1)).squeeze(-1)

    # -- weights and lifecycle -------------------------------------------------------
    @torch.no_grad()
    def update_weights(self, state_dict: dict[str, Tensor]) -> int:
        """Load HF-named tensors; raises KeyError unless every parameter of
        the module is covered and every tensor is used."""
        from lumenrl_b200.sync.moe_weights import assert_weight_sync_coverage, route_expert_weights
        m = self.model
        params = dict(m.named_parameters())
        tied = getattr(getattr(m, "config", None), "tie_word_embeddings", False)
        # per-expert checkpoint tensors <-> the module's fused expert parameters
        state_dict = route_expert_weights(state_dict, params)
        try:
            assert_weight_sync_coverage(state_dict, {k: tuple(p.shape) for k, p in params.items()},
                                        optional=("lm_head.weight",) if tied else ())
        except KeyError as e:
            raise KeyError(f"HFEngine {e.args[0]}") from None
        for k, v in state_dict.items():
            if k in params:
                params[k].copy_(v.to(device=params[k].device, dtype=params[k].dtype))
        return len(state_dict)

    def sleep(self) -> None:
        if self._model is not None and not self._asleep:
            self._model.to("cpu")
            self._asleep = True
            gc.collect()
            if torch.cuda.is_available():
                torch.cuda.empty_cache()

    def wake(self) -> None:
        if self._model is not None and self._asleep:
            self._model.to(self.device)
            self._asleep = False

    def shutdown(self) -> None:
        self._model = None
        gc.collect()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()


class GenerationInterface:
    """prepare -> generate (DataProto in, DataProto out) -> finish around any
    engine with ``generate(input_ids, attention_mask, **sampling)``: the
    set-up cost is paid once per rollout phase and released after it."""

    def __init__(self, engine_factory) -> None:
        self._factory = engine_factory
        self._engine = None
        self.sampling_defaults: dict[str, Any] = {"max_new_tokens": 64, "temperature": 1.0}

    def prepare_for_generation(self) -> None:
        if self._engine is None:
            self._engine = self._factory()
            if hasattr(self._engine, "init"):
                self._engine.init()
        elif hasattr(self._engine, "wake"):
            self._engine.wake()

    def generate(self, batch: DataProto) -> DataProto:
        if self._engine is None:
            raise RuntimeError("GenerationInterface: call prepare_for_generation() first")
        if "input_ids" not in batch.tensors:
            raise KeyError("GenerationInterface: the batch needs an 'input_ids' column")
        sampling = {**self.sampling_defaults, **dict(batch.meta.get("sampling_params", {}))}
        seqs, mask = self._engine.generate(batch["input_ids"], batch.tensors.get("attention_mask"), **sampling)
        return DataProto(tensors={"sequences": seqs.cpu(), "attention_mask": mask.cpu()},
                         meta={**batch.meta, "sampling_params": sampling})

    def finish_generation(self, release: bool = False) -> None:
        if self._engine is None:
            return
        if release and hasattr(self._engine, "shutdown"):
            self._engine.shutdown()
            self._engine = None
        elif hasattr(self._engine, "sleep"):
            self._engine.sleep()
