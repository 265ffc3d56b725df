"""Typed configuration: dataclass schema + YAML + CLI dot-list overrides.

The key names and nesting are the public recipe format of LumenRL
(``lumenrl/core/config.py:23-931`` in the reference), so an existing recipe
loads unchanged.  The loader is written here from scratch (the reference uses
OmegaConf, which this framework does not depend on):

* ``LumenRLConfig.from_yaml(path, overrides)`` reads YAML, resolves
  ``${oc.env:VAR[,default]}`` and ``${dotted.key}`` interpolations, merges the
  result into the dataclass defaults, then applies ``a.b.c=value`` overrides.
* Unknown keys are rejected (strict schema), values are coerced to the field's
  annotated type (``int``/``float``/``bool``/``str``/``Optional``/``list``/
  ``dict``/nested dataclass).
* Fields typed ``dict``/``Any`` accept free-form mappings.
"""

from __future__ import annotations

import argparse
import dataclasses
import logging
import os
import re
import typing
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Optional

import yaml

logger = logging.getLogger(__name__)


# ---------------------------------------------------------------------------
# Schema (field names follow the reference recipe format)
# ---------------------------------------------------------------------------


@dataclass
class FSDPEngineConfig:
    strategy: str = "fsdp2"
    fsdp_size: int = -1
    param_offload: bool = False
    optimizer_offload: bool = False
    grad_offload: bool = False
    reshard_after_forward: bool = True
    forward_only: bool = False
    seed: int = 42
    model_dtype: str = "bf16"
    mixed_precision: Optional[dict] = None
    use_remove_padding: bool = True
    ulysses_sequence_parallel_size: int = 1
    forward_prefetch: bool = False
    use_orig_params: bool = True
    use_torch_compile: bool = False


@dataclass
class OptimizerConfig:
    optimizer_type: str = "adamw"
    lr: float = 1e-6
    weight_decay: float = 0.01
    clip_grad: float = 1.0
    lr_scheduler_type: str = "cosine"
    lr_warmup_steps: int = 10
    lr_warmup_steps_ratio: float = 0.0
    total_training_steps: int = 1000
    min_lr_ratio: float = 0.0
    num_cycles: float = 0.5
    adam_beta1: float = 0.9
    adam_beta2: float = 0.95
    adam_eps: float = 1e-8


@dataclass
class LoRAConfig:
    enabled: bool = False
    rank: int = 0
    alpha: int = 16
    target_modules: Optional[list] = None
    exclude_modules: Optional[list] = None
    merge: bool = False
    adapter_path: Optional[str] = None


@dataclass
class HFModelConfig:
    local_path: str = ""
    model_type: str = "language_model"
    trust_remote_code: bool = True
    use_remove_padding: bool = True
    enable_gradient_checkpointing: bool = True
    lora: LoRAConfig = field(default_factory=LoRAConfig)
    use_liger: bool = False
    use_fused_kernels: bool = False
    calculate_entropy: bool = False
    calculate_sum_pi_squared: bool = False


@dataclass
class ClusterConfig:
    num_nodes: int = 1
    gpus_per_node: int = 1
    ray_address: Optional[str] = None


@dataclass
class RayWorkerRoleConfig:
    num_workers: int = 0
    dispatch_mode: str = "dp_compute_proto"
    mesh_mapping: Optional[list] = None
    lazy_dispatch_key: Optional[str] = None
    detached: bool = False
    process_on_nodes: Optional[list] = None
    max_colocate_count: int = 1
    topology_tags: dict = field(default_factory=dict)


@dataclass
class RayControllerConfig:
    enabled: bool = False
    fuse_actor_ref: bool = False
    actor: RayWorkerRoleConfig = field(default_factory=RayWorkerRoleConfig)
    ref: RayWorkerRoleConfig = field(default_factory=RayWorkerRoleConfig)
    rollout: RayWorkerRoleConfig = field(default_factory=RayWorkerRoleConfig)
    topology_map: dict = field(default_factory=dict)


@dataclass
class ControllerConfig:
    ray: RayControllerConfig = field(default_factory=RayControllerConfig)


@dataclass
class MegatronConfig:
    tensor_model_parallel_size: int = 1
    pipeline_model_parallel_size: int = 1
    context_parallel_size: int = 1
    expert_model_parallel_size: int = 1
    sequence_parallel: bool = False
    num_experts: Optional[int] = None
    moe_grouped_gemm: bool = True
    expert_tensor_parallel_size: Optional[int] = None
    moe_router_topk: Optional[int] = None
    moe_router_load_balancing_type: str = "aux_loss"
    moe_router_pre_softmax: Optional[bool] = None
    moe_router_score_function: Optional[str] = None
    moe_router_dtype: Optional[str] = "fp32"
    moe_router_topk_scaling_factor: Optional[float] = None
    moe_shared_expert_intermediate_size: Optional[int] = None
    moe_aux_loss_coeff: float = 0.0
    moe_router_bias_update_rate: Optional[float] = None
    moe_token_dispatcher_type: str = "alltoall"
    moe_permute_fusion: bool = False
    use_distributed_optimizer: bool = True
    grad_reduce_in_fp32: bool = True
    attention_softmax_in_fp32: bool = True
    recompute_granularity: Optional[str] = None
    recompute_method: Optional[str] = None
    recompute_num_layers: Optional[int] = None
    attention_backend: str = "unfused"
    use_packed_sequences: bool = True
    log_probs_chunk_size: int = 0
    enable_dynamic_batch: bool = False
    max_tokens_per_gpu: int = 0
    dist_checkpoint_path: Optional[str] = None
    deterministic_mode: Optional[bool] = None
    build_optimizer: bool = True
    optimizer_cpu_offload: bool = False
    optimizer_offload_fraction: float = 1.0
    overlap_cpu_optimizer_d2h_h2d: bool = True


@dataclass
class AtomConfig:
    tensor_parallel_size: int = 1
    kv_cache_dtype: str = "auto"
    max_model_len: Optional[int] = None
    gpu_memory_utilization: float = 0.6
    gpu_id: Optional[int] = None
    transport: str = "fifo"
    data_parallel_size: int = 1
    expert_parallel_size: int = 1
    enable_prefix_caching: bool = False
    online_quant_config: Optional[dict] = None
    engine_kwargs: dict = field(default_factory=dict)


@dataclass
class VLLMConfig:
    tensor_parallel_size: int = 1
    kv_cache_dtype: str = "auto"
    max_model_len: Optional[int] = None
    gpu_memory_utilization: float = 0.6
    gpu_id: Optional[int] = None
    dtype: str = "bfloat16"
    enforce_eager: bool = True
    enable_chunked_prefill: bool = True
    max_num_batched_tokens: int = 8192
    max_num_seqs: int = 64
    swap_space: int = 4
    trust_remote_code: bool = True
    quantization: str = ""
    moe_backend: str = ""
    calculate_log_probs: bool = False
    seed: Optional[int] = None
    persistent: bool = True
    data_parallel_rollout: bool = True
    online: bool = True
    transport: str = "fifo"
    ray_http_base_port: int = 8700
    ray_http_start_server: bool = True
    enable_sleep_mode: bool = True
    sleep_level: int = 2
    update_weights_bucket_megabytes: int = 512
    use_shm: bool = False
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1


@dataclass
class TrainingConfig:
    megatron_cfg: MegatronConfig = field(default_factory=MegatronConfig)
    fsdp_cfg: Optional[dict] = None
    optimizer_dtype: str = "bf16"


@dataclass
class GenerationConfig:
    atom_cfg: AtomConfig = field(default_factory=AtomConfig)
    vllm_cfg: VLLMConfig = field(default_factory=VLLMConfig)


@dataclass
class PolicyConfig:
    model_name: str = ""
    training_backend: str = "fsdp2"
    generation_backend: str = "atom"
    training: TrainingConfig = field(default_factory=TrainingConfig)
    generation: GenerationConfig = field(default_factory=GenerationConfig)
    max_total_sequence_length: int = 4096
    max_response_length: int = 20480
    train_global_batch_size: int = 64
    gen_batch_size: int = 0
    train_micro_batch_size: int = 8
    max_token_len_per_gpu: int = 0
    ppo_mini_batch_size: int = 0
    learning_rate: float = 1e-6
    lr_warmup_steps: int = 10
    weight_decay: float = 0.01
    max_grad_norm: float = 1.0
    adam_beta1: float = 0.9
    adam_beta2: float = 0.95
    adam_eps: float = 1e-8
    warmup_ratio: float = 0.0
    min_lr: float = 0.0
    lr_decay_style: str = "cosine"
    wsd_decay_ratio: float = 0.2
    wsd_decay_style: str = "cosine"
    balance_batch: bool = False


@dataclass
class GRPOConfig:
    num_generations: int = 8
    kl_coeff: float = 0.0
    clip_ratio: float = 0.2
    num_ppo_epochs: int = 1
    num_mini_batches: int = 1
    discount: float = 1.0


@dataclass
class FilterGroupsConfig:
    enable: bool = False
    metric: str = "acc"
    max_num_gen_batches: int = 0


@dataclass
class OverlongBufferConfig:
    enable: bool = False
    len: int = 0
    penalty_factor: float = 0.0
    log: bool = False


@dataclass
class DAPOConfig:
    num_generations: int = 8
    kl_coeff: float = 0.0
    clip_ratio_low: float = 0.2
    clip_ratio_high: float = 0.28
    clip_ratio_c: float = 3.0
    dynamic_sampling: bool = True
    token_level_pg: bool = True
    overlong_reward_shaping: bool = True
    loss_mode: str = "token_level"
    discount: float = 1.0
    filter_groups: FilterGroupsConfig = field(default_factory=FilterGroupsConfig)
    overlong_buffer: OverlongBufferConfig = field(default_factory=OverlongBufferConfig)
    max_resp_len: int = 0


@dataclass
class PPOConfig:
    kl_coeff: float = 0.02
    clip_ratio: float = 0.2
    num_ppo_epochs: int = 4
    num_mini_batches: int = 4
    gae_lambda: float = 0.95
    discount: float = 1.0


@dataclass
class OPDConfig:
    kl_direction: str = "reverse"
    temperature: float = 1.0
    position_weighting: bool = False
    position_decay: float = 0.8
    opd_coeff: float = 1.0
    lazy_logits: bool = True
    teacher_micro_batch_size: int = 4


@dataclass
class SpecDistillConfig:
    draft_type: str = "eagle3"
    loss_type: str = "forward_kl"
    position_decay: float = 0.8
    loss_decay_gamma: float = 7.0
    num_target_layers: int = 1
    aux_hidden_state_layer_ids: Optional[list] = None
    anchor_num: int = 512
    spec_length: int = 5


@dataclass
class TeacherConfig:
    model_name: str = ""
    key: str = ""
    lm_head_key: str = "lm_head.weight"
    norm_key: str = "model.norm.weight"
    load_norm: bool = False
    inference_backend: str = "hf"
    quantization: str = ""
    tensor_parallel_size: int = 1
    gpu_ids: Optional[list] = None
    transport: str = "mooncake"
    atom: Any = None
    mori_io_host: str = "127.0.0.1"
    mori_io_port: int = 0
    mori_io_qp_per_transfer: int = 2
    atom_plugin: bool = False


@dataclass
class DraftModelConfig:
    model_name: str = ""
    from_scratch: bool = False
    head_dim: Optional[int] = None
    num_layers: Optional[int] = None
    num_heads: Optional[int] = None
    num_kv_heads: Optional[int] = None
    ffn_dim: Optional[int] = None
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    rope_scaling_type: Optional[str] = None
    rope_scaling_factor: float = 64.0
    rope_original_max_pos: int = 4096
    rope_beta_fast: float = 32.0
    rope_beta_slow: float = 1.0
    rope_mscale: float = 1.0
    rope_mscale_all_dim: float = 1.0
    rope_low_freq_factor: float = 1.0
    rope_high_freq_factor: float = 4.0
    use_aux_hidden_state: bool = True
    use_input_layernorm_in_first_layer: bool = True
    use_last_layernorm: bool = True
    use_mtp_layernorm: bool = False
    attention_bias: bool = False
    mlp_bias: bool = False
    max_window_layers: Optional[int] = None
    dtype: str = "float16"
    resume_from: Optional[str] = None


@dataclass
class DistillationConfig:
    enabled: bool = False
    teacher_key: str = "data_source"
    teachers: dict = field(default_factory=dict)
    loss_mode: str = "reverse_kl"
    topk: Optional[int] = None
    use_task_rewards: bool = False
    distillation_loss_coef: float = 1.0


@dataclass
class RolloutCorrectionConfig:
    enabled: bool = False
    method: str = "tis"
    clip: float = 1.5
    rollout_is: str = ""
    rollout_is_threshold: Any = "2.0"
    rollout_is_batch_normalize: bool = False
    rollout_is_seq_reduction: str = "sum"
    rollout_rs: str = ""
    rollout_rs_threshold: Any = ""
    bypass_mode: bool = False
    loss_type: str = "ppo_clip"

    def __post_init__(self) -> None:
        # Thresholds may be a number, an IcePop "lower_upper" pair or a comma
        # list; keep them as strings so one field carries all three forms.
        if not isinstance(self.rollout_is_threshold, str):
            self.rollout_is_threshold = str(self.rollout_is_threshold)
        if not isinstance(self.rollout_rs_threshold, str):
            self.rollout_rs_threshold = str(self.rollout_rs_threshold)
        if self.rollout_is_seq_reduction not in ("sum", "mean"):
            raise ValueError(
                f"rollout_is_seq_reduction must be 'sum' or 'mean', got {self.rollout_is_seq_reduction!r}")


@dataclass
class AlgorithmConfig:
    name: str = "grpo"
    adv_estimator: str = ""
    grpo: GRPOConfig = field(default_factory=GRPOConfig)
    dapo: DAPOConfig = field(default_factory=DAPOConfig)
    ppo: PPOConfig = field(default_factory=PPOConfig)
    opd: OPDConfig = field(default_factory=OPDConfig)
    spec_distill: SpecDistillConfig = field(default_factory=SpecDistillConfig)
    teacher: TeacherConfig = field(default_factory=TeacherConfig)
    draft: DraftModelConfig = field(default_factory=DraftModelConfig)
    distillation: DistillationConfig = field(default_factory=DistillationConfig)
    kl_ctrl_type: str = "fixed"
    kl_penalty: str = "kl"
    kl_target: float = 0.01
    kl_horizon: int = 10000
    use_kl_in_reward: bool = False
    loss_mode: str = ""
    loss_agg_mode: str = "token-mean"
    clip_ratio: float = 0.2
    clip_ratio_low: Optional[float] = None
    clip_ratio_high: Optional[float] = None
    clip_ratio_c: float = 3.0
    rollout_correction: Optional[RolloutCorrectionConfig] = None


@dataclass
class RolloutQuantConfig:
    precision: str = "bf16"
    use_deep_gemm: bool = True
    num_first_layers_in_bf16: int = 0
    num_last_layers_in_bf16: int = 0


@dataclass
class TrainingQuantConfig:
    fp8: Optional[str] = None
    fp8_recipe: str = "blockwise"
    fp8_weight_cache: bool = False
    lumen_norm: bool = False
    fused_mlp: bool = False
    fused_rope: bool = False
    lumen_linear: bool = False
    hf_attn_patch: bool = False


@dataclass
class QuantizationConfig:
    rollout: RolloutQuantConfig = field(default_factory=RolloutQuantConfig)
    training: TrainingQuantConfig = field(default_factory=TrainingQuantConfig)
    rollout_correction: RolloutCorrectionConfig = field(default_factory=RolloutCorrectionConfig)


@dataclass
class R3Config:
    enabled: bool = False
    record_router_logits: bool = True
    replay_mode: str = "distribution"
    rollout_replay: bool = False


@dataclass
class MoEConfig:
    r3: R3Config = field(default_factory=R3Config)


@dataclass
class RewardConfig:
    type: str = "function"
    function: str = "math_reward"
    dataset: str = ""
    dataset_split: str = "train"
    model_name: Optional[str] = None
    shuffle: bool = True
    shuffle_seed: Optional[int] = None


@dataclass
class DatasetConfig:
    chat_template: str = ""
    last_turn_loss_only: str = "false"
    min_loss_tokens: int = 0
    num_preprocess_workers: int = 16
    cache_dir: str = "/dev/shm/lumenrl_cache"


@dataclass
class EvalConfig:
    enabled: bool = False
    interval: int = 1000
    num_samples: int = 256
    micro_batch_size: int = 8


@dataclass
class CriticConfig:
    enabled: bool = False
    model_name: str = ""
    training_backend: str = "fsdp2"
    learning_rate: float = 1e-5
    weight_decay: float = 0.01
    max_grad_norm: float = 1.0
    value_clip_ratio: float = 0.2
    num_critic_epochs: int = 1


@dataclass
class CheckpointConfig:
    checkpoint_dir: str = "results/default"
    save_steps: int = 50
    save_total_limit: int = 3
    resume: bool = True


@dataclass
class WandbConfig:
    project: str = "lumenrl"
    name: str = ""
    entity: Optional[str] = None


@dataclass
class LoggerConfig:
    wandb_enabled: bool = False
    wandb: WandbConfig = field(default_factory=WandbConfig)
    log_interval: int = 1
    num_val_samples_to_print: int = 5


@dataclass
class MooncakeTransferConfig:
    master_server_address: Optional[str] = None
    metadata_server: Optional[str] = None
    local_hostname: str = ""
    protocol: str = "rdma"
    device_name: str = ""
    global_segment_size: str = "16GB"
    local_buffer_size: str = "4GB"
    host_buffer_size: int = 536870912
    gpu_buffer_size: int = 536870912
    async_put_pool_size: int = 4
    enable_gpu_direct: bool = False
    enable_hard_pin: bool = False
    kv_lease_ttl_s: float = 120.0
    get_retry_wait_seconds: float = 1.0
    get_retry_max_wait_seconds: float = 90.0


@dataclass
class RDMAWeightSyncConfig:
    backend: str = "rccl"
    require_rdma: bool = True
    hca: str = "mlx5_0"
    interface: str = "ens11np0"
    gid_index: int = 3
    gdr_mode: str = "auto"


@dataclass
class WeightSyncConfig:
    # "auto" picks the fastest path for the placement: in-place (colocated,
    # one GPU), NVLink all-gather/broadcast (several GPUs, same node),
    # shared_folder (safetensors) or rdma-style bucket stream (cross node).
    backend: str = "auto"
    shared_folder: str = "/volumes/oss1/lumenrl_weight_sync"
    bucket_size_mb: int = 1024
    timeout_s: int = 600
    verify_full_load: bool = True
    rdma: RDMAWeightSyncConfig = field(default_factory=RDMAWeightSyncConfig)


@dataclass
class AsyncTrainingConfig:
    enabled: bool = False
    require_batches: int = 4
    trigger_parameter_sync_step: int = 4
    staleness_threshold: float = 0.0
    partial_rollout: bool = False
    use_rollout_log_probs: bool = True
    rollout_n_gpus: int = 0
    trainer_n_gpus: int = 0
    queue_maxsize: int = 64
    weight_sync_dir: str = "/tmp/lumenrl_weight_sync"


@dataclass
class TorchProfilerScheduleConfig:
    skip_first: int = 0
    wait: int = 0
    warmup: int = 1
    active: int = 3
    repeat: int = 0


@dataclass
class TorchProfilerToolConfig:
    contents: list = field(default_factory=lambda: ["cpu", "cuda"])
    schedule: Optional[TorchProfilerScheduleConfig] = None


@dataclass
class ProfilerConfig:
    # "torch" (torch.profiler chrome traces), "nvtx" (NVTX ranges only, for an
    # external Nsight capture) or "ncu" (emits an ncu command line per step).
    tool: str = "torch"
    enable: bool = False
    all_ranks: bool = False
    ranks: list = field(default_factory=list)
    save_path: str = "outputs/profile"
    steps: Optional[list] = None
    profile_continuous_steps: bool = False
    tool_config: Any = field(default_factory=TorchProfilerToolConfig)


@dataclass
class RuntimeAssemblyConfig:
    training_backend: str = "fsdp2"
    inference_backend: str = "atom"
    topology: str = "decoupled"
    strict_policy: bool = True
    use_new_assembler: bool = True
    role_impl_keys: dict = field(default_factory=dict)


@dataclass
class KernelsConfig:
    """B200 kernel and collective selection (no counterpart in the reference,
    whose kernels come from its inference / training libraries).  Each field
    mirrors one ``LRL_*`` environment variable; ``None`` keeps the variable's
    value or the built-in default, a value overrides both
    (``lumenrl_b200.ops.kernel_flags.apply_kernels_config``)."""
    train_gemm: Optional[str] = None       # LRL_TRAIN_GEMM: own (CTA-pair tcgen05) | cublas
    train_attn: Optional[str] = None       # LRL_TRAIN_ATTN: tc (tcgen05 flash) | fa2
    train_attn_bwd: Optional[str] = None   # LRL_TRAIN_ATTN_BWD: tc | fa2
    decode_gemm: Optional[str] = None      # LRL_DECODE_GEMM: auto | sk | skinny | cublas
    fp8_decode_gemm: Optional[str] = None  # LRL_FP8_DECODE_GEMM: stream | gemm
    decode_attn: Optional[str] = None      # LRL_DECODE_ATTN: tma | cp
    nvls: Optional[bool] = None            # LRL_NVLS: NVLink-SHARP multicast collectives
    cp_ring: Optional[str] = None          # LRL_CP_RING: nvlink | pg
    draft_allreduce: Optional[str] = None  # LRL_DRAFT_ALLREDUCE: nvlink | nccl
    debug_bounds: Optional[bool] = None    # LRL_DEBUG_BOUNDS: bounds-checked NVLink kernels
    eagle_kernels: Optional[bool] = None   # LRL_EAGLE_KERNELS: fused Eagle3 draft kernels


@dataclass
class LumenRLConfig:
    cluster: ClusterConfig = field(default_factory=ClusterConfig)
    policy: PolicyConfig = field(default_factory=PolicyConfig)
    algorithm: AlgorithmConfig = field(default_factory=AlgorithmConfig)
    reward: RewardConfig = field(default_factory=RewardConfig)
    quantization: QuantizationConfig = field(default_factory=QuantizationConfig)
    moe: MoEConfig = field(default_factory=MoEConfig)
    critic: CriticConfig = field(default_factory=CriticConfig)
    checkpointing: CheckpointConfig = field(default_factory=CheckpointConfig)
    logger: LoggerConfig = field(default_factory=LoggerConfig)
    mooncake: MooncakeTransferConfig = field(default_factory=MooncakeTransferConfig)
    weight_sync: WeightSyncConfig = field(default_factory=WeightSyncConfig)
    async_training: AsyncTrainingConfig = field(default_factory=AsyncTrainingConfig)
    profiler: ProfilerConfig = field(default_factory=ProfilerConfig)
    controller: ControllerConfig = field(default_factory=ControllerConfig)
    assembly: RuntimeAssemblyConfig = field(default_factory=RuntimeAssemblyConfig)
    dataset: DatasetConfig = field(default_factory=DatasetConfig)
    eval: EvalConfig = field(default_factory=EvalConfig)
    kernels: KernelsConfig = field(default_factory=KernelsConfig)
    num_training_steps: int = 1000
    seed: int = 42
    val_dataset: str = ""
    val_steps: int = 0
    val_batch_size: int = 16

    # -- loading -----------------------------------------------------------
    @classmethod
    def from_dict(cls, data: dict | None, overrides: list[str] | None = None) -> "LumenRLConfig":
        tree = dict(data or {})
        for item in overrides or []:
            key, value = _parse_override(item)
            _set_dotted(tree, key, value)
        tree = _resolve_interpolations(tree)
        return _build(cls, tree, "")

    @classmethod
    def from_yaml(cls, path: str | Path, overrides: list[str] | None = None) -> "LumenRLConfig":
        with open(path, "r", encoding="utf-8") as f:
            data = yaml.safe_load(f) or {}
        return cls.from_dict(data, overrides)

    @classmethod
    def from_cli(cls, argv: list[str] | None = None) -> "LumenRLConfig":
        parser = argparse.ArgumentParser(description="lumenrl_b200")
        parser.add_argument("--config", type=str, required=True, help="Path to YAML config")
        args, unknown = parser.parse_known_args(argv)
        return cls.from_yaml(args.config, overrides=unknown)

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)


def load_config(config_path: str | Path, overrides: list[str] | None = None) -> LumenRLConfig:
    return LumenRLConfig.from_yaml(config_path, overrides=overrides)


# ---------------------------------------------------------------------------
# Loader internals
# ---------------------------------------------------------------------------

_INTERP = re.compile(r"\$\{([^}]+)\}")


def _parse_override(item: str) -> tuple[str, Any]:
    item = item.lstrip("-")
    if "=" not in item:
        raise ValueError(f"override must look like key=value, got {item!r}")
    key, raw = item.split("=", 1)
    value = yaml.safe_load(raw) if raw != "" else ""
    return key.strip(), value


def _set_dotted(tree: dict, key: str, value: Any) -> None:
    parts = key.split(".")
    node = tree
    for p in parts[:-1]:
        nxt = node.get(p)
        if not isinstance(nxt, dict):
            nxt = {}
            node[p] = nxt
        node = nxt
    node[parts[-1]] = value


def _get_dotted(tree: dict, key: str) -> Any:
    node: Any = tree
    for p in key.split("."):
        if not isinstance(node, dict) or p not in node:
            raise KeyError(f"interpolation target {key!r} not found")
        node = node[p]
    return node


def _resolve_interpolations(tree: dict) -> dict:
    def resolve(value: Any, depth: int = 0) -> Any:
        if depth > 16:
            raise ValueError("interpolation recursion too deep")
        if isinstance(value, dict):
            return {k: resolve(v, depth) for k, v in value.items()}
        if isinstance(value, list):
            return [resolve(v, depth) for v in value]
        if not isinstance(value, str) or "${" not in value:
            return value

        def one(expr: str) -> Any:
            expr = expr.strip()
            if expr.startswith("oc.env:"):
                body = expr[len("oc.env:"):]
                name, _, default = body.partition(",")
                env = os.environ.get(name.strip())
                if env is not None:
                    return env
                if _:
                    return yaml.safe_load(default.strip()) if default.strip() else ""
                raise KeyError(f"environment variable {name!r} not set and no default given")
            return resolve(_get_dotted(tree, expr), depth + 1)

        whole = _INTERP.fullmatch(value.strip())
        if whole:
            return one(whole.group(1))
        return _INTERP.sub(lambda m: str(one(m.group(1))), value)

    return resolve(tree)


def _strip_optional(tp: Any) -> tuple[Any, bool]:
    origin = typing.get_origin(tp)
    if origin is typing.Union or (hasattr(typing, "UnionType") and origin is getattr(__import__("types"), "UnionType", None)):
        args = [a for a in typing.get_args(tp) if a is not type(None)]
        if len(args) == 1:
            return args[0], True
        return Any, True
    return tp, False


def _coerce(tp: Any, value: Any, path: str) -> Any:
    tp, optional = _strip_optional(tp)
    if value is None:
        if optional or tp is Any:
            return None
        # YAML "~" for a non-optional scalar: keep the schema's semantics by
        # rejecting it, as a structured config would.
        raise TypeError(f"{path}: null is not allowed")
    if tp is Any:
        return value
    if dataclasses.is_dataclass(tp):
        if isinstance(value, tp):
            return value
        if not isinstance(value, dict):
            raise TypeError(f"{path}: expected a mapping for {tp.__name__}")
        return _build(tp, value, path)
    origin = typing.get_origin(tp) or tp
    if origin in (list, tuple):
        if not isinstance(value, (list, tuple)):
            value = [value]
        return list(value)
    if origin is dict:
        if not isinstance(value, dict):
            raise TypeError(f"{path}: expected a mapping")
        return dict(value)
    if tp is bool:
        if isinstance(value, bool):
            return value
        if isinstance(value, str) and value.lower() in ("true", "false", "1", "0", "yes", "no"):
            return value.lower() in ("true", "1", "yes")
        if isinstance(value, int):
            return bool(value)
        raise TypeError(f"{path}: expected bool, got {value!r}")
    if tp is int:
        if isinstance(value, bool):
            raise TypeError(f"{path}: expected int, got bool")
        if isinstance(value, float) and value.is_integer():
            return int(value)
        return int(value)
    if tp is float:
        return float(value)
    if tp is str:
        return value if isinstance(value, str) else str(value)
    return value


def _build(cls: type, data: dict, prefix: str) -> Any:
    hints = typing.get_type_hints(cls)
    names = {f.name for f in dataclasses.fields(cls)}
    unknown = set(data) - names
    if unknown:
        where = prefix or cls.__name__
        raise KeyError(f"unknown config key(s) under {where}: {sorted(unknown)}")
    kwargs = {}
    for f in dataclasses.fields(cls):
        if f.name not in data:
            continue
        kwargs[f.name] = _coerce(hints[f.name], data[f.name], f"{prefix}.{f.name}" if prefix else f.name)
    obj = cls(**kwargs)
    return obj
