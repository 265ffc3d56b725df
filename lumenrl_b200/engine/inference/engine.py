"""Native rollout engine: batched sampling with a paged KV cache.

Replaces the reference's external engines (vLLM/ATOM subprocesses driven over
FIFOs, ``lumenrl/engine/inference/{vllm,atom}_engine.py``) with an in-process
engine on the trainer's own weights:

* GRPO prefix sharing: each prompt is prefilled ONCE; its ``n`` samples share
  the prompt's full KV blocks (reference counted) and copy only the partial
  tail block, so prefill work and prompt KV memory drop by ``n``.
* Static batches up to ``max_num_seqs``.  Requests with more rows than slots
  run with continuous batching (``continuous_batching=True``, the default for
  dense models): a row that emits EOS frees its slot and the next queued
  sample takes it over -- its prompt prefilled on admission, the prompt's
  full KV blocks shared, the slot's block table / position / RNG counters
  rewritten in place so the captured decode graph stays valid.  Each row
  draws from its own counter-based stream keyed by (sample index, token
  index), so the samples equal those of static waves.  MoE models (routing
  capture per row) fall back to static waves.  The decode step always has
  static shapes and is replayed from a CUDA graph.
* Returns token ids, per-token rollout log-probs (under softmax(logits/T),
  the quantity TIS/MIS rollout correction needs) and, for MoE models, the
  routed expert ids per generated token (R3).
* ``sleep()``/``wake()`` free and re-create the KV pool for colocated
  training; ``update_weights`` is a no-op in colocated mode (the engine reads
  the trainer's flat bf16 buffer directly) and a copy otherwise.
"""

from __future__ import annotations

import logging
import math
from dataclasses import dataclass, field
from typing import Optional

import torch
from torch import Tensor

from lumenrl_b200.engine.inference.kv_cache import KVSpec, PagedKVCache
from lumenrl_b200.engine.inference.runner import DecodeGraph, ModelRunner, RoutingRecorder
from lumenrl_b200.models.qwen3 import Qwen3Model

logger = logging.getLogger(__name__)


@dataclass
class SamplingParams:
    max_new_tokens: int = 1024
    temperature: float = 1.0
    top_p: float = 1.0
    n: int = 1
    seed: int = 0
    eos_token_id: Optional[int] = 2
    stop_at_eos: bool = True
    # global index of this call's first row: a replica that serves a slice of
    # a larger batch draws exactly the samples one engine would draw for it
    row_offset: int = 0


@dataclass
class GenerationOutput:
    prompts: list[list[int]]
    responses: Tensor          # [N, max_new] int64, pad_id after the end
    response_lengths: Tensor   # [N] int64
    logprobs: Tensor           # [N, max_new] fp32 (0 past the end)
    prompt_index: Tensor       # [N] which prompt each row came from
    routed_experts: list = field(default_factory=list)  # per row: [len, layers, k] int16 (MoE only)
    stats: dict = field(default_factory=dict)


class RolloutEngine:
    def __init__(self, model: Qwen3Model, max_num_seqs: int = 64, max_model_len: int = 2048,
                 kv_cache_bytes: Optional[int] = None, block_size: int = 64, kv_dtype: torch.dtype = torch.bfloat16,
                 use_cuda_graph: bool = True, pad_token_id: int = 0, shared_prefix_attention: bool = True,
                 fp8_rollout=None, continuous_batching: bool = True, vocab_limit: Optional[int] = None,
                 tp_group=None) -> None:
        """``tp_group``: a process group of size T > 1 serves the model with
        tensor parallelism (``runner.TPShards``): every member calls
        ``generate`` with the same prompts and sampling parameters and gets the
        same samples, each GPU holding 1/T of the decoder linears' reads and of
        the KV cache."""
        self.model = model
        self.args = model.args
        self.device = model.flat.device
        self.max_num_seqs = max_num_seqs
        self.max_model_len = max_model_len
        self.block_size = block_size
        self.pad_token_id = pad_token_id
        self.shared_prefix_attention = shared_prefix_attention
        self.continuous_batching = continuous_batching
        # MoE decode steps are captured too when their routing and expert GEMMs
        # run on the device (no host read of the routes inside the step)
        from lumenrl_b200.models.moe import moe_graph_ok
        self.use_cuda_graph = (use_cuda_graph and self.device.type == "cuda"
                               and (self.args.num_experts == 0 or moe_graph_ok(model)))
        tp = None
        if tp_group is not None:
            import torch.distributed as dist
            if dist.get_world_size(tp_group) > 1:
                from lumenrl_b200.engine.inference.runner import TPShards
                tp = TPShards(model, tp_group, dist.get_rank(tp_group), dist.get_world_size(tp_group))
                if fp8_rollout is not None and fp8_rollout.is_fp8_enabled():
                    raise ValueError("rollout TP with FP8 rollout weights is not supported: use TP=1 per GPU")
        self.tp = tp
        if tp is not None:
            # no collective inside a captured decode graph: under TP the decode
            # step runs eagerly (its all-reduces are ordinary NCCL calls)
            self.use_cuda_graph = False
        kv_heads = tp.num_kv_heads if tp is not None else self.args.num_kv_heads
        spec = KVSpec(self.args.num_layers, kv_heads, self.args.head_dim, block_size, kv_dtype)
        self.max_blocks_per_seq = math.ceil(max_model_len / block_size) + 1
        if kv_cache_bytes is None:
            nblocks = max_num_seqs * self.max_blocks_per_seq + 1
        else:
            nblocks = PagedKVCache.blocks_for_budget(spec, kv_cache_bytes)
        self.cache = PagedKVCache(spec, nblocks, self.device)
        self.runner = ModelRunner(model, self.cache, tp)
        self.runner.max_len = max_model_len
        if vocab_limit is not None:
            if not 0 < vocab_limit <= self.args.vocab_size:
                raise ValueError(f"vocab_limit {vocab_limit} outside (0, {self.args.vocab_size}]")
            self.runner.vocab_limit = int(vocab_limit)
        if fp8_rollout is not None and fp8_rollout.is_fp8_enabled():
            # W8A8 blockwise rollout (128x128 E4M3 weight blocks, 1x128 activation
            # blocks); requantised from the bf16 weights at every weight sync
            from lumenrl_b200.quant.fp8 import FP8RolloutQuantizer
            self.runner.fp8 = FP8RolloutQuantizer(fp8_rollout, self.args.num_layers)
            self.runner.fp8.quantize_model(model)
        self._graphs: dict[tuple, DecodeGraph] = {}
        self._graphs_pool_ptr = self.cache.pool_ptr
        self.weight_version = 0

    # -- lifecycle ---------------------------------------------------------------
    def sleep(self, release_memory: bool = False) -> None:
        """Free the KV pool.  The block stays in the caching allocator (so the
        trainer's activations reuse it and the next wake is a cache hit)
        unless ``release_memory`` returns it to the driver.  Captured decode
        graphs point at the pool; they are kept, and dropped at the next wake
        only if the pool comes back at another address."""
        self.cache.sleep()
        if release_memory and self.device.type == "cuda":
            self._graphs.clear()
            torch.cuda.empty_cache()

    def wake(self) -> None:
        self.cache.wake()
        if self.cache.pool_ptr != self._graphs_pool_ptr:
            self._graphs.clear()
            self._graphs_pool_ptr = self.cache.pool_ptr

    def update_weights(self, flat: Optional[Tensor] = None, version: Optional[int] = None) -> None:
        """Colocated: the engine aliases the trainer buffer, nothing to move.
        Separated: copy a full bf16 flat buffer in (one contiguous copy)."""
        if flat is not None and flat.data_ptr() != self.model.flat.data_ptr():
            self.model.flat.copy_(flat, non_blocking=True)
        if self.runner.fp8 is not None:
            # re-quantised in place: the captured graphs read the same buffers
            self.runner.fp8.quantize_model(self.model)
        if self.tp is not None:
            self.tp.refresh()      # this rank's slices, copied in place
        self.weight_version = self.weight_version + 1 if version is None else version

    # -- generation ------------------------------------------------------------------
    def _graph(self, batch: int, sp: SamplingParams, share: Optional[tuple] = None) -> DecodeGraph:
        key = (batch, sp.temperature, sp.top_p, share)
        g = self._graphs.get(key)
        if g is None:
            g = DecodeGraph(self.runner, batch, self.max_blocks_per_seq, sp.temperature, sp.top_p,
                            self.use_cuda_graph, share)
            self._graphs[key] = g
        return g

    @torch.no_grad()
    def generate(self, prompts, sp: SamplingParams) -> GenerationOutput:
        """``prompts``: list of token-id lists, or an int64 tensor [P, L] of
        equal-length prompts (already on the device for the fast path)."""
        if not self.cache.awake:
            self.wake()
        rows_per_prompt = sp.n
        if (self.continuous_batching and self.args.num_experts == 0
                and len(prompts) * rows_per_prompt > self.max_num_seqs):
            return self._generate_continuous(prompts, sp)
        per_wave = max(1, self.max_num_seqs // rows_per_prompt)
        outs = []
        for w0 in range(0, len(prompts), per_wave):
            outs.append(self._generate_wave(prompts[w0: w0 + per_wave], sp, w0))
        if len(outs) == 1:
            return outs[0]
        width = max(o.responses.shape[1] for o in outs)

        def padw(t: Tensor, fill) -> Tensor:
            return torch.nn.functional.pad(t, (0, width - t.shape[1]), value=fill)
        return GenerationOutput(
            prompts=(torch.cat(list(o.prompts for o in outs)) if isinstance(outs[0].prompts, Tensor)
                     else [p for o in outs for p in o.prompts]),
            responses=torch.cat([padw(o.responses, self.pad_token_id) for o in outs]),
            response_lengths=torch.cat([o.response_lengths for o in outs]),
            logprobs=torch.cat([padw(o.logprobs, 0.0) for o in outs]),
            prompt_index=torch.cat([o.prompt_index for o in outs]),
            routed_experts=[r for o in outs for r in o.routed_experts],
            stats={k: sum(o.stats.get(k, 0) for o in outs) for k in outs[0].stats})

    # -- continuous batching ---------------------------------------------------------
    def _generate_continuous(self, prompts, sp: SamplingParams) -> GenerationOutput:
        """Slots are refilled as rows finish.  Host bookkeeping (block tables,
        admissions) runs every ``check_every`` decode steps; between checks
        the graph replays with finished slots masked (their writes go to a
        trash row)."""
        from lumenrl_b200 import ops
        dev, bs, n, S = self.device, self.block_size, sp.n, self.max_num_seqs
        ev0 = self._ev()
        as_tensor = isinstance(prompts, Tensor)
        P = len(prompts)
        plist = [prompts[i] for i in range(P)] if as_tensor else [list(p) for p in prompts]
        plens = [int(p.shape[0]) if as_tensor else len(p) for p in plist]
        max_new = min(sp.max_new_tokens, self.max_model_len - max(plens))
        if max_new <= 0:
            raise ValueError("prompt longer than max_model_len")
        total = P * n
        eos = sp.eos_token_id if sp.stop_at_eos else None
        alloc = self.cache.allocator
        g = self._graph(S, sp, None)
        base_seed = sp.seed * 1_000_003 + sp.row_offset
        # outputs (one trash row at the end absorbs the writes of idle slots)
        out_tok = torch.full((total + 1, max_new), self.pad_token_id, dtype=torch.long, device=dev)
        out_lp = torch.zeros(total + 1, max_new, dtype=torch.float32, device=dev)
        lengths = torch.full((total + 1,), max_new, dtype=torch.long, device=dev)
        flat_tok, flat_lp = out_tok.view(-1), out_lp.view(-1)
        slot_row = torch.full((S,), total, dtype=torch.long, device=dev)     # trash row when idle
        active = torch.zeros(S, dtype=torch.bool, device=dev)
        g.block_table.zero_()
        g.positions.zero_()
        g.step.zero_()
        g.prefix_len.zero_()
        host_row = [-1] * S
        slot_blocks: list[list[int]] = [[] for _ in range(S)]
        prompt_blocks: dict[int, list[int]] = {}
        pending_rows_of: dict[int, int] = {}
        next_row = 0
        stats = {"decode_steps": 0, "prefill_tokens": 0, "admissions": 0}

        def admit(free: list[int]) -> None:
            nonlocal next_row
            rows = list(range(next_row, min(total, next_row + len(free))))
            next_row += len(rows)
            if not rows:
                return
            new_p = sorted({r // n for r in rows} - set(prompt_blocks))
            logits_of: dict[int, Tensor] = {}
            if new_p:
                e0 = self._ev()
                ids = torch.cat([plist[i].to(dev, torch.long).reshape(-1) if as_tensor else
                                 torch.tensor(plist[i], dtype=torch.long, device=dev) for i in new_p])
                pos = torch.cat([torch.arange(plens[i], device=dev) for i in new_p])
                lens_t = torch.tensor([plens[i] for i in new_p], device=dev)
                cu = torch.zeros(len(new_p) + 1, dtype=torch.int32, device=dev)
                cu[1:] = torch.cumsum(lens_t, 0)
                slots_l = []
                for i in new_p:
                    blk = alloc.alloc(math.ceil(plens[i] / bs))
                    prompt_blocks[i] = blk
                    pending_rows_of[i] = n
                    slots_l.extend(blk[j // bs] * bs + j % bs for j in range(plens[i]))
                lg = self.runner.prefill(ids, pos, cu, int(lens_t.max()), torch.tensor(slots_l, dtype=torch.long,
                                                                                     device=dev))
                for k, i in enumerate(new_p):
                    logits_of[i] = lg[k]
                stats["prefill_tokens"] += int(lens_t.sum())
                e1 = self._ev()
                if e0 is not None:
                    self._pending_ev.append((e0, e1))      # prefill time, read after the loop
            first_logits, seeds, slots_used = [], [], []
            for slot, r in zip(free, rows):
                i, L = r // n, plens[r // n]
                full = L // bs
                shared = alloc.share(prompt_blocks[i][:full])
                private = alloc.alloc(math.ceil((L + max_new) / bs) - full)
                if L % bs:
                    self.cache.copy_block(prompt_blocks[i][full], private[0])
                table = shared + private
                slot_blocks[slot] = table
                host_row[slot] = r
                g.block_table[slot].zero_()
                g.block_table[slot, : len(table)] = torch.tensor(table, dtype=torch.int32, device=dev)
                g.positions[slot] = L
                first_logits.append(logits_of[i] if i in logits_of else self._prompt_logits[i])
                seeds.append(base_seed + r)
                slots_used.append(slot)
            for i, lg in logits_of.items():
                self._prompt_logits[i] = lg
            sl = torch.tensor(slots_used, dtype=torch.long, device=dev)
            rr = torch.tensor(rows, dtype=torch.long, device=dev)
            g.row_seed[sl] = torch.tensor(seeds, dtype=torch.long, device=dev)
            g.step[sl] = 0
            tok, lp = ops.sample_tokens_device(torch.stack(first_logits), sp.temperature, sp.top_p,
                                               g.row_seed[sl], torch.zeros(len(rows), dtype=torch.long, device=dev))
            out_tok[rr, 0], out_lp[rr, 0] = tok, lp
            g.tokens[sl] = tok
            slot_row[sl] = rr
            done = (tok == eos) if eos is not None else torch.zeros_like(tok, dtype=torch.bool)
            if max_new == 1:
                done = torch.ones_like(done)
            lengths[rr] = torch.where(done, torch.ones_like(tok), torch.full_like(tok, max_new))
            active[sl] = ~done
            g.step[sl] = 1
            stats["admissions"] += len(rows)

        self._prompt_logits: dict[int, Tensor] = {}
        self._pending_ev = []
        ev1 = self._ev()
        admit(list(range(S)))
        check_every = 4
        while True:
            for _ in range(check_every):
                tok, lp = g.run()
                stats["decode_steps"] += 1
                t = g.step                                   # token index each slot just sampled
                idx = slot_row * max_new + t.clamp(max=max_new - 1)
                flat_tok.index_copy_(0, idx, torch.where(active, tok, torch.full_like(tok, self.pad_token_id)))
                flat_lp.index_copy_(0, idx, torch.where(active, lp, torch.zeros_like(lp)))
                fin = active & ((t + 1 >= max_new) | ((tok == eos) if eos is not None else torch.zeros_like(active)))
                lengths.index_copy_(0, slot_row, torch.where(fin, t + 1, lengths[slot_row]))
                active &= ~fin
                slot_row.masked_fill_(fin, total)           # later replays write to the trash row
                g.tokens.copy_(tok)
                g.positions.add_(active.long())
                g.step.add_(active.long())
            # host bookkeeping: release finished slots, admit queued rows
            act = active.tolist()
            free = []
            for slot in range(S):
                if not act[slot] and host_row[slot] >= 0:
                    r = host_row[slot]
                    alloc.release(slot_blocks[slot])
                    slot_blocks[slot] = []
                    host_row[slot] = -1
                    i = r // n
                    pending_rows_of[i] -= 1
                    if pending_rows_of[i] == 0:       # last sample of the prompt: drop its own references
                        alloc.release(prompt_blocks.pop(i))
                        self._prompt_logits.pop(i, None)
                if host_row[slot] < 0:
                    free.append(slot)
                    slot_row[slot] = total
                    g.block_table[slot].zero_()
                    g.positions[slot] = 0
            if next_row < total and free:
                admit(free)
            if next_row >= total and not any(active.tolist()):
                break
        ev2 = self._ev()
        lens_out = lengths[:total]
        steps = int(lens_out.max()) if total else 0
        ar = torch.arange(max_new, device=dev).unsqueeze(0)
        valid = ar < lens_out.unsqueeze(1)
        tok_o = torch.where(valid, out_tok[:total], torch.full_like(out_tok[:total], self.pad_token_id))[:, :steps]
        lp_o = torch.where(valid, out_lp[:total], torch.zeros_like(out_lp[:total]))[:, :steps]
        # decode steps static waves of the same rows would have run (each wave
        # runs until its longest row ends), for the saved-steps statistic
        per_wave = max(1, S // n) * n
        lh = lens_out.tolist()
        static_steps = sum(max(lh[w: w + per_wave]) - 1 for w in range(0, total, per_wave))
        pf = sum(a.elapsed_time(b) for a, b in self._pending_ev) if ev0 is not None else 0.0
        self._pending_ev, self._prompt_logits = [], {}
        stats.update({"gen_tokens": int(lens_out.sum()), "static_wave_decode_steps": static_steps,
                      "decode_steps_saved": static_steps - stats["decode_steps"]})
        if ev0 is not None:
            stats.update({"prefill_ms": pf, "setup_ms": ev0.elapsed_time(ev1),
                          "decode_ms": ev1.elapsed_time(ev2) - pf})
        prompt_index = torch.arange(total, device=dev) // n
        return GenerationOutput(
            prompts=(prompts.repeat_interleave(n, 0) if as_tensor else [p for p in prompts for _ in range(n)]),
            responses=tok_o, response_lengths=lens_out, logprobs=lp_o, prompt_index=prompt_index,
            routed_experts=[], stats=stats)

    def _ev(self):
        if self.device.type != "cuda":
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def _generate_wave(self, prompts, sp: SamplingParams, prompt_offset: int) -> GenerationOutput:
        dev, bs, n = self.device, self.block_size, sp.n
        ev0 = self._ev()
        P = len(prompts)
        B = P * n
        alloc = self.cache.allocator
        as_tensor = isinstance(prompts, Tensor)
        plens = [int(prompts.shape[1])] * P if as_tensor else [len(p) for p in prompts]
        max_new = min(sp.max_new_tokens, self.max_model_len - max(plens))
        if max_new <= 0:
            raise ValueError("prompt longer than max_model_len")
        # 1) blocks: prompt blocks per prompt, per-row private tail + generation blocks
        tables: list[list[int]] = []
        owned: list[list[int]] = []
        prompt_blocks: list[list[int]] = []
        for L in plens:
            prompt_blocks.append(alloc.alloc(math.ceil(L / bs)))
        # 2) prefill unique prompts
        if as_tensor:
            ids = prompts.to(dev, torch.long).reshape(-1)
        else:
            ids = torch.tensor([t for p in prompts for t in p], dtype=torch.long, device=dev)
        pos = torch.cat([torch.arange(L, device=dev) for L in plens])
        lens = torch.tensor(plens, device=dev)
        cu = torch.zeros(P + 1, dtype=torch.int32, device=dev)
        cu[1:] = torch.cumsum(lens, 0)
        slots = torch.tensor([prompt_blocks[i][j // bs] * bs + j % bs for i, L in enumerate(plens)
                              for j in range(L)], dtype=torch.long, device=dev)
        recorder = None
        moe_layers = [i for i in range(self.args.num_layers) if self.args.is_moe_layer(i)]
        if moe_layers:
            recorder = RoutingRecorder(moe_layers)
            self.runner.routing_recorder = recorder
        logits = self.runner.prefill(ids, pos, cu, int(lens.max()), slots)
        ev1 = self._ev()
        prompt_routes = recorder.take() if recorder else None   # [sumL, layers, k]
        for i, L in enumerate(plens):
            full = L // bs
            need = math.ceil((L + max_new) / bs)
            for _ in range(n):
                shared = alloc.share(prompt_blocks[i][:full])
                private = alloc.alloc(need - full)
                if L % bs:
                    self.cache.copy_block(prompt_blocks[i][full], private[0])
                tables.append(shared + private)
                owned.append(shared + private)
        alloc.release([b for pb in prompt_blocks for b in pb])   # rows hold their own references now
        # 3) first token from the prefill logits (row r samples prompt r // n)
        row_logits = logits.repeat_interleave(n, dim=0)
        share = None
        group = 1
        if self.shared_prefix_attention and n > 1:
            from lumenrl_b200 import ops
            group = ops.shared_prefix_group(n, self.args.num_heads // self.args.num_kv_heads)
        if group > 1 and max(plens) >= bs:
            # static bounds, bucketed so graphs are reused: the shared whole
            # prompt blocks, and the private part (partial block + generation)
            max_prefix = -(-max((L // bs) * bs for L in plens) // 256) * 256
            max_suffix = -(-(bs + max_new) // 256) * 256
            share = (group, max_prefix, max_suffix)
        g = self._graph(B, sp, share)
        ev2 = self._ev()
        g.row_seed.copy_(torch.arange(B, device=dev) + (sp.seed * 1_000_003 + sp.row_offset + prompt_offset * n))
        g.step.fill_(0)
        from lumenrl_b200 import ops
        tok, lp = ops.sample_tokens_device(row_logits, sp.temperature, sp.top_p, g.row_seed, g.step)
        out_tok = torch.full((B, max_new), self.pad_token_id, dtype=torch.long, device=dev)
        out_lp = torch.zeros(B, max_new, dtype=torch.float32, device=dev)
        out_tok[:, 0], out_lp[:, 0] = tok, lp
        bt = torch.zeros(B, self.max_blocks_per_seq, dtype=torch.int32, device=dev)
        for r, t in enumerate(tables):
            bt[r, : len(t)] = torch.tensor(t, dtype=torch.int32)
        g.block_table.copy_(bt)
        plen = lens.repeat_interleave(n)
        g.positions.copy_(plen)
        g.prefix_len.copy_(((plen // bs) * bs).to(torch.int32))
        g.tokens.copy_(tok)
        routes_rows: list[list[Tensor]] = [[] for _ in range(B)]
        if recorder:
            self.runner.routing_recorder = recorder
        finished = torch.zeros(B, dtype=torch.bool, device=dev)
        eos = sp.eos_token_id if sp.stop_at_eos else None
        if eos is not None:
            finished |= tok == eos
        lengths = torch.full((B,), max_new, dtype=torch.long, device=dev)
        steps = 1
        check_every = 16
        for t in range(1, max_new):
            g.step.fill_(t)
            tok, lp = g.run()
            if recorder:
                step_routes = g.recorder.take()     # the routes of the step just replayed
                for r in range(B):
                    routes_rows[r].append(step_routes[r])
            out_tok[:, t] = tok
            out_lp[:, t] = lp
            g.tokens.copy_(tok)
            g.positions.add_(1)
            steps += 1
            if eos is not None:
                newly = (~finished) & (tok == eos)
                lengths = torch.where(newly, torch.full_like(lengths, t + 1), lengths)
                finished |= newly
                if t % check_every == 0 and bool(finished.all()):
                    break
        ev3 = self._ev()
        if eos is not None:
            first = (out_tok[:, 0] == eos)
            lengths = torch.where(first, torch.ones_like(lengths), lengths)
        lengths = lengths.clamp(max=steps)
        ar = torch.arange(out_tok.shape[1], device=dev).unsqueeze(0)
        valid = ar < lengths.unsqueeze(1)
        out_tok = torch.where(valid, out_tok, torch.full_like(out_tok, self.pad_token_id))[:, :steps]
        out_lp = torch.where(valid, out_lp, torch.zeros_like(out_lp))[:, :steps]
        for t in owned:
            alloc.release(t)
        routed = []
        if recorder:
            self.runner.routing_recorder = None
            offs = [0] + torch.cumsum(lens, 0).tolist()
            lens_host = lengths.tolist()
            for r in range(B):
                i = r // n
                pr = prompt_routes[offs[i]: offs[i + 1]]
                gen = torch.stack(routes_rows[r]) if routes_rows[r] else pr[:0]
                # routes of prompt tokens + tokens that were fed back (all but the last sample)
                routed.append(torch.cat([pr, gen[: max(lens_host[r] - 1, 0)]]).cpu())
        return GenerationOutput(
            prompts=(prompts.repeat_interleave(n, 0) if as_tensor else [p for p in prompts for _ in range(n)]),
            responses=out_tok, response_lengths=lengths,
            logprobs=out_lp, prompt_index=torch.arange(P, device=dev).repeat_interleave(n) + prompt_offset,
            routed_experts=routed,
            stats={"decode_steps": steps, "prefill_tokens": int(lens.sum()), "gen_tokens": int(lengths.sum()),
                   **({"prefill_ms": ev0.elapsed_time(ev1), "setup_ms": ev1.elapsed_time(ev2),
                       "decode_ms": ev2.elapsed_time(ev3)} if ev0 is not None else {})})
