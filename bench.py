"""Headline benchmark: GRPO step tokens/s (rollout + train), Qwen3-8B, B200.

    python bench.py --gpus N --steps K --warmup W          # N=1
    torchrun --nproc-per-node N bench.py --gpus N ...       # N>1, one rank per GPU
    python bench.py --impl reference ...                    # the reference's own arm

Workload (BASELINE config "Qwen3-8B architecture, bf16, random init, GRPO
colocated"), weak scaling: every GPU runs 8 prompts x group 8 = 64 sequences
(so N=8 is the named 64 x 8 batch); prompts are 512 uniform-random token ids
from [0, 151643) by seed; responses up to 1024 tokens at temperature 1.0;
parity reward; micro-batch 4; one AdamW step per GRPO step; the updated bf16
weights reach the rollout engine every step (full weight sync).

A step is everything: rollout (prefill + decode), rewards, old log-probs,
advantages, fwd+bwd of every micro-batch, the optimizer step and the weight
sync.  `value` is total tokens (prompt + response, all ranks) / device time of
K steps (CUDA events, barrier + synchronize on both sides, max over ranks).
`e2e` repeats K steps through the public trainer API on the wall clock, each
step including the pinned host->device copy of its prompts and a
device->host read of its metrics.  The model weights (16 GB) dwarf the 126 MB
L2, so every step streams its inputs from HBM.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

METRIC = "GRPO step tokens/s (rollout+train) Qwen3-8B at 1/2/4/8 B200; weight-sync ms"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--prompts-per-gpu", type=int, default=8)
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--max-new", type=int, default=1024)
    ap.add_argument("--micro", type=int, default=4)
    ap.add_argument("--recompute", choices=["auto", "on", "off"], default="auto")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--placement", choices=["colocated", "separated", "async"], default="colocated",
                    help="colocated: every GPU generates and trains; separated: half the GPUs generate, half "
                         "train, in lockstep; async: the same split with the rollout one step ahead")
    ap.add_argument("--recipe", choices=["grpo", "dapo-fp8"], default="grpo",
                    help="grpo: the headline bf16 GRPO config; dapo-fp8: DAPO with W8A8 FP8 rollout, FP8 KV "
                         "cache and hybrid FP8 training linears (E4M3 forward, E5M2 gradients)")
    return ap.parse_args()


def recipe_config(args, model_name: str) -> dict:
    """Trainer config of the chosen recipe (the YAML schema of ``configs/``)."""
    vllm = {"temperature": 1.0, "top_p": 1.0}
    cfg = {"policy": {"model_name": model_name, "learning_rate": 1e-6, "lr_warmup_steps": 0,
                      "lr_decay_style": "constant", "train_micro_batch_size": args.micro,
                      "max_grad_norm": 1.0, "weight_decay": 0.01, "generation": {"vllm_cfg": vllm}},
           "algorithm": {"name": "grpo", "grpo": {"num_generations": args.group, "kl_coeff": 0.0,
                                                  "clip_ratio": 0.2}},
           "num_training_steps": args.warmup + 2 * args.steps, "seed": 1234}
    if args.recipe == "dapo-fp8":
        vllm.update(kv_cache_dtype="fp8", quantization="fp8_per_block", calculate_log_probs=True)
        cfg["algorithm"] = {"name": "dapo", "dapo": {
            "num_generations": args.group, "clip_ratio_low": 0.2, "clip_ratio_high": 0.28,
            "token_level_pg": True, "filter_groups": {"enable": True}}}
        cfg["quantization"] = {"rollout": {"precision": "fp8"},
                               "training": {"fp8": "hybrid", "fp8_recipe": "blockwise"},
                               "rollout_correction": {"rollout_is": "token", "rollout_is_threshold": 2.0}}
    return cfg


def reference_arm(args) -> None:
    """The reference's own GRPO path, unmodified, from ``baseline/_ref``.

    It cannot run on this image: its trainer imports OmegaConf and drives
    rollouts through Ray with the ROCm-only ATOM / vLLM-ROCm engines and the
    AITER / MORI kernels (git submodules absent from its source tree), and
    neither Ray nor OmegaConf has a wheel in the offline wheelhouse.  The
    line printed names what is missing on the machine it runs on."""
    import importlib.util
    here = os.path.dirname(os.path.abspath(__file__))
    ref = os.path.join(here, "baseline", "_ref")
    needed = ("ray", "omegaconf", "atom", "aiter", "mori")
    missing = [m for m in needed if importlib.util.find_spec(m) is None]
    if not os.path.isdir(os.path.join(ref, "lumenrl")):
        where = "the reference package is not installed under baseline/_ref"
    else:
        sys.path.insert(0, ref)
        try:
            import lumenrl.trainer.rl_trainer  # noqa: F401
            where = "lumenrl.trainer.rl_trainer imports"
        except Exception as e:
            where = f"import lumenrl.trainer.rl_trainer fails ({type(e).__name__}: {str(e).splitlines()[0][:120]})"
    why = (f"{where}; missing modules {missing}: Ray and OmegaConf have no offline wheel, and the GRPO rollout "
           "needs the ROCm-only ATOM/AITER/MORI submodules (absent from the reference source) -- no NVIDIA path")
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "metric": METRIC, "unavailable": why}))


class ClockSampler:
    """nvidia-smi samples (200 ms) of the GPUs in use during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, n: int) -> None:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        self.ids = vis.split(",")[:n] if vis else [str(i) for i in range(n)]
        self.proc = None
        self.lines: list[str] = []

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", ",".join(self.ids)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def main() -> None:
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    import torch
    import torch.distributed as dist

    from lumenrl_b200.core.config import LumenRLConfig
    from lumenrl_b200.models.config import resolve_model
    from lumenrl_b200.ops.ext import LAUNCHES, ext
    from lumenrl_b200.parallel.dist import init_distributed
    from lumenrl_b200.trainer.rl_trainer import RLRunSpec, RLTrainer

    st = init_distributed(timeout_s=900)
    ext()  # the kernels must be there
    world, rank = st.world_size, st.rank
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    margs = resolve_model(args.model)
    recompute = {"on": True, "off": False, "auto": "auto"}[args.recompute]
    cfg = LumenRLConfig.from_dict(recipe_config(args, margs.name))
    colocated = args.placement == "colocated"
    n_roll = world if colocated else world // 2     # GPUs that generate
    if not colocated and world < 2:
        raise SystemExit("--placement separated / async needs at least 2 GPUs")
    spec = RLRunSpec(prompts_per_step=args.prompts_per_gpu * n_roll, prompt_len=args.prompt_len, prompt_low=0,
                     prompt_high=151643, max_new_tokens=args.max_new, eos_token_id=151645, reward="parity",
                     rows_per_micro=args.micro, use_cuda_graph=not args.no_graph,
                     gradient_checkpointing=recompute)
    if colocated:
        tr = RLTrainer(cfg, margs, spec, st).setup()
    else:
        from lumenrl_b200.trainer.separated_trainer import SeparatedRLTrainer
        tr = SeparatedRLTrainer(cfg, margs, spec, st, num_rollout=n_roll,
                                async_lag=1 if args.placement == "async" else 0).setup()

    def sync():
        if dist.is_initialized():
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        tr.step()
    # ---- device-timed region ----
    clocks = ClockSampler(world) if rank == 0 else None
    sync()
    if clocks:
        clocks.start()
    l0 = LAUNCHES[0]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    toks = 0.0
    hist = []
    for _ in range(args.steps):
        m = tr.step()
        hist.append(m)
        toks += m.get("perf/total_num_tokens", 0.0)   # rank 0 trains in every placement
    e1.record()
    sync()
    launches = LAUNCHES[0] - l0
    dev_s = e0.elapsed_time(e1) / 1e3
    t = torch.tensor([dev_s], device=st.device, dtype=torch.float64)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_s = float(t.item())
    clk = clocks.stop() if clocks else None
    # ---- end-to-end region: public API, pinned H2D in, D2H of metrics out ----
    sync()
    w0 = time.perf_counter()
    toks_e2e = 0.0
    for _ in range(args.steps):
        m = tr.step()           # copies the pinned prompt batch H2D inside
        toks_e2e += float(m.get("perf/total_num_tokens", 0.0))   # metrics are host values (D2H inside step)
    sync()
    wall = time.perf_counter() - w0
    tw = torch.tensor([wall], device=st.device, dtype=torch.float64)
    if dist.is_initialized():
        dist.all_reduce(tw, op=dist.ReduceOp.MAX)
    wall = float(tw.item())
    # ---- multi-GPU correctness, outside the timed regions: replicas agree
    # bit for bit, and one fused NVLink optimizer step equals the NCCL path ----
    # host<->device bytes per step, summed over the ranks that move them
    io = torch.tensor([float(tr.io_bytes.get("h2d", 0)), float(tr.io_bytes.get("d2h", 0))], device=st.device,
                      dtype=torch.float64)
    if dist.is_initialized():
        dist.all_reduce(io)
    checks = {}
    if not colocated:
        tr.finish()             # async: the rollout side takes the last pushed update
    if world > 1 and colocated:
        from lumenrl_b200.parallel.symm import fused_vs_nccl_max_err, replica_agreement
        opt = tr.actor.opt
        checks.update(replica_agreement(tr.actor.model.flat, opt.master, opt.lo))
        fv = fused_vs_nccl_max_err(64 << 20, rank, world)
        checks["fused_vs_nccl_max_err"] = fv["weights_max_err"]
        checks["fused_vs_nccl"] = fv
    if rank == 0:
        last = hist[-1]
        B = args.prompts_per_gpu * args.group
        out = {
            "metric": METRIC, "value": toks / dev_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dev_s / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if args.recipe == "grpo" else "fp8 (E4M3 fwd / E5M2 grads, bf16 weights)",
            "data": "synthetic: uniform-random prompt ids [0,151643) by seed, random-init weights N(0,0.02)",
            "config": {"model": "Qwen3-8B (36L, h4096, 32q/8kv, hd128, ffn12288, vocab151936, qk-norm)",
                       "global_batch": B * world, "prompts": args.prompts_per_gpu * world, "group": args.group,
                       "seq_len": args.prompt_len + args.max_new, "prompt_len": args.prompt_len,
                       "max_new_tokens": args.max_new, "micro_batch": args.micro,
                       "parallelism": (f"dp{world} (sharded AdamW, resident bf16 weights; rollout TP=1 per GPU)"
                                       if colocated else
                                       f"separated: {world - n_roll} trainer GPU(s) (sharded AdamW) + {n_roll} "
                                       f"rollout GPU(s), weights pushed by NVLink peer stores"
                                       + (", rollout one step ahead" if args.placement == "async" else "")),
                       "placement": args.placement,
                       "recompute": recompute, "recipe": args.recipe,
                       "cache": "inputs larger than L2 (16 GB of weights per step)"},
            "clocks": clk,
            "e2e": {"value": toks_e2e / wall, "unit": "tokens/s", "h2d_bytes_per_step": int(io[0]),
                    "d2h_bytes_per_step": int(io[1])},
            "gpu_launches": launches,
            "breakdown_s": {k.replace("timing/", ""): v for k, v in last.items() if k.startswith("timing/")},
            "recompute_layers": last.get("actor/recompute_layers"),
            "weight_sync_ms": last.get("weight_sync/ms"),
            "weight_sync_GBps": last.get("weight_sync/GBps"),
            "gen_tokens_per_s": last.get("perf/gen_tokens_per_s"),
            "mean_response_len": last.get("response_length/mean"),
            **({k: last[k] for k in ("dapo/gen_rounds", "dapo/kept_frac", "rollout_corr/kl") if k in last}
               if args.recipe != "grpo" else {}),
            **checks,
        }
        print(json.dumps(out))
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
