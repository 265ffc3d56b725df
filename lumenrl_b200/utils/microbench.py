"""Micro-benchmarks of the hot paths on one GPU (random weights).

    python -m lumenrl_b200.utils.microbench decode --batch 64 --ctx 1024 --steps 20
    python -m lumenrl_b200.utils.microbench train  --rows 4 --seq 1536 --steps 3
    python -m lumenrl_b200.utils.microbench logprob --rows 8 --seq 1536

Each prints one JSON line with CUDA-event timings (warm-up first).  They run
the production code paths (engine decode graph, packed fwd/bwd, fused
log-prob) and are the commands the ncu summaries under profiles/ were made
with.
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch


def _model(name: str, trainable: bool):
    from lumenrl_b200.models.config import resolve_model
    from lumenrl_b200.models.qwen3 import Qwen3Model
    args = resolve_model(name)
    m = Qwen3Model(args, device="cuda", dtype=torch.bfloat16, requires_grad=trainable)
    m.init_weights(0)
    return m


def _model_args(name: str):
    from lumenrl_b200.models.config import resolve_model
    return resolve_model(name)


def _time(fn, steps: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def _time_sustained(fn, steps: int, warmup: int, sustain_ms: float) -> float:
    """_time after ``sustain_ms`` of back-to-back calls, so that the clocks
    have settled where the power limit holds them for a long kernel stream."""
    if sustain_ms > 0:
        import time
        t0 = time.perf_counter()
        while (time.perf_counter() - t0) * 1e3 < sustain_ms:
            for _ in range(8):
                fn()
            torch.cuda.synchronize()
    return _time(fn, steps, warmup)


def bench_decode(ns) -> dict:
    from lumenrl_b200.engine.inference.engine import RolloutEngine
    from lumenrl_b200.engine.inference.runner import DecodeGraph
    from lumenrl_b200 import ops
    m = _model(ns.model, False)
    B, ctx = ns.batch, ns.ctx
    fp8 = None
    if ns.fp8:
        from lumenrl_b200.quant.fp8 import FP8Config
        fp8 = FP8Config(precision="fp8")
    eng = RolloutEngine(m, max_num_seqs=B, max_model_len=ctx + 64, use_cuda_graph=not ns.no_graph,
                        kv_dtype=torch.float8_e4m3fn if ns.fp8_kv else torch.bfloat16, fp8_rollout=fp8)
    bs = eng.block_size
    n, P = ns.group, (ns.prefix // bs) * bs    # rows of a group share a P-token prompt (in ctx)
    grp = ops.shared_prefix_group(n, m.args.num_heads // m.args.num_kv_heads) if n > 1 and P > 0 else 1
    share = (grp, -(-P // 256) * 256, -(-(ctx - P + bs) // 256) * 256) if grp > 1 else None
    g = DecodeGraph(eng.runner, B, eng.max_blocks_per_seq, 1.0, 1.0, not ns.no_graph, share)
    nb = math.ceil((ctx + 64) / bs)
    pb = P // bs if grp > 1 else 0
    bt = torch.zeros(B, nb, dtype=torch.int32)
    nxt = 1 + (B // max(grp, 1)) * pb
    for r in range(B):
        if pb:
            bt[r, :pb] = 1 + (r // grp) * pb + torch.arange(pb, dtype=torch.int32)
        bt[r, pb:] = nxt + torch.arange(nb - pb, dtype=torch.int32)
        nxt += nb - pb
    g.block_table[:, :nb].copy_(bt.cuda())
    g.prefix_len.fill_(pb * bs)
    g.positions.fill_(ctx)
    g.tokens.random_(0, m.args.vocab_size)
    ms = _time(g.run, ns.steps, ns.warmup)
    wbytes = m.flat.numel() * 2
    if fp8 is not None:   # E4M3 copies replace the bf16 decoder linears in the step
        wbytes -= sum(qw.numel() for qw, _ in eng.runner.fp8.weights.values())
    kvbytes = B * ctx * m.args.kv_bytes_per_token() // (2 if ns.fp8_kv else 1)
    return {"op": "decode_step", "batch": B, "ctx": ctx, "shared_prefix": pb * bs, "group": grp,
            "attn": ops.DECODE_ATTN, "gemm": ops.DECODE_GEMM, "ms": ms, "fp8_weights": bool(ns.fp8),
            "fp8_kv": bool(ns.fp8_kv), "fp8_decode_gemm": ops.FP8_DECODE_GEMM if ns.fp8 else None,
            "weights_GB": wbytes / 1e9, "kv_GB": kvbytes / 1e9, "achieved_TBps": (wbytes + kvbytes) / ms / 1e9}


def bench_attn(ns) -> dict:
    """Decode attention of one layer (the model's heads): the per-row paged
    kernel vs the shared-prefix kernel on GRPO-shaped rows (``--group``
    samples share a ``--prefix``-token prompt, each with ``--ctx`` private
    tokens).  Bytes are the K/V bytes each variant must read."""
    from lumenrl_b200 import ops
    args = _model_args(ns.model)
    B, Hq, Hk, D, bs = ns.batch, args.num_heads, args.num_kv_heads, args.head_dim, 64
    n, P, S = ns.group, ns.prefix, ns.ctx
    groups = B // n
    pb, sb = P // bs, (S + bs - 1) // bs
    nblocks = 1 + groups * pb + B * sb
    kc = torch.randn(nblocks, bs, Hk, D, device="cuda").to(torch.bfloat16)
    vc = torch.randn_like(kc)
    ar_p = torch.arange(pb, dtype=torch.int32, device="cuda")
    ar_s = torch.arange(sb, dtype=torch.int32, device="cuda")
    bt = torch.zeros(B, pb + sb, dtype=torch.int32, device="cuda")
    for r in range(B):
        bt[r, :pb] = 1 + (r // n) * pb + ar_p
        bt[r, pb:] = 1 + groups * pb + r * sb + ar_s
    lens = torch.full((B,), P + S, dtype=torch.int32, device="cuda")
    pre = torch.full((B,), P, dtype=torch.int32, device="cuda")
    q = torch.randn(B, Hq, D, device="cuda").to(torch.bfloat16)
    sc = D ** -0.5
    grp = ops.shared_prefix_group(n, Hq // Hk)
    t_plain = _time(lambda: ops.paged_decode_attention(q, kc, vc, bt, lens, sc, max_len=P + S), ns.steps, ns.warmup)
    t_shared = _time(lambda: ops.paged_decode_attention_shared(q, kc, vc, bt, lens, pre, grp, sc, max_prefix=P,
                                                               max_suffix=S), ns.steps, ns.warmup)
    tok = Hk * D * 2 * 2
    plain_bytes = B * (P + S) * tok
    shared_bytes = (groups * P + B * S) * tok
    return {"op": "decode_attention", "batch": B, "group": n, "prefix": P, "suffix": S,
            "plain_ms": t_plain, "shared_ms": t_shared, "speedup": t_plain / t_shared,
            "plain_TBps": plain_bytes / t_plain / 1e9, "shared_TBps": shared_bytes / t_shared / 1e9}


def bench_skinny(ns) -> dict:
    """Decode-size GEMMs (M tokens x the model's projection shapes): the
    weight-streaming tcgen05 kernel vs cuBLAS.  Each timed call reads a
    different copy of the weight (copies > 256 MB in total), so weights come
    from HBM as in a decode step, not from L2."""
    from lumenrl_b200 import ops
    M = ns.batch
    out = []
    for N, K in [(6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288), (151936, 4096)]:
        x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        nbytes = N * K * 2
        copies = max(2, -(-(256 << 20) // nbytes) + 1)
        ws = [(torch.randn(N, K, device="cuda") / K ** 0.5).to(torch.bfloat16) for _ in range(copies)]
        it = {"i": 0}

        def nxt():
            it["i"] = (it["i"] + 1) % copies
            return ws[it["i"]]
        t_sk = _time(lambda: ops.skinny_linear(x, nxt()), ns.steps, ns.warmup)
        t_cb = _time(lambda: x @ nxt().t(), ns.steps, ns.warmup)
        err = (ops.skinny_linear(x, ws[0]).float() - (x.float() @ ws[0].float().t())).abs().max().item()
        out.append({"M": M, "N": N, "K": K, "skinny_ms": t_sk, "cublas_ms": t_cb,
                    "skinny_TBps": nbytes / t_sk / 1e9, "cublas_TBps": nbytes / t_cb / 1e9, "max_err": err})
        del ws
    from lumenrl_b200.ops.ext import ext
    return {"op": "skinny_gemm", "status": int(ext().skinny_gemm_status()), "shapes": out}


def bench_attn_train(ns) -> dict:
    """Packed causal attention forward + backward (training shapes: --rows
    sequences of --seq tokens, the model's heads) for each backend."""
    from lumenrl_b200 import ops
    args = _model_args(ns.model)
    T = ns.rows * ns.seq
    cu = torch.arange(0, T + 1, ns.seq, dtype=torch.int32, device="cuda")
    q = torch.randn(T, args.num_heads, args.head_dim, device="cuda").to(torch.bfloat16).requires_grad_(True)
    k = torch.randn(T, args.num_kv_heads, args.head_dim, device="cuda").to(torch.bfloat16).requires_grad_(True)
    v = torch.randn_like(k).requires_grad_(True)
    do = torch.randn_like(q)
    res = {"op": "train_attention", "tokens": T, "seq": ns.seq}
    flops = 4 * ns.rows * (ns.seq * ns.seq / 2) * args.num_heads * args.head_dim * 3.5  # fwd + bwd (2.5x)

    def step():
        o = ops.attention_varlen(q, k, v, cu, ns.seq, causal=True, scale=args.head_dim ** -0.5)
        o.backward(do)
    t = _time(step, ns.steps, ns.warmup)
    res["ms"] = t
    res["tflops"] = flops / t / 1e9
    # forward alone: library kernel vs the tcgen05 kernel
    from lumenrl_b200.ops.ext import ext
    fflops = 4 * ns.rows * (ns.seq * ns.seq / 2) * args.num_heads * args.head_dim
    sc = args.head_dim ** -0.5
    with torch.no_grad():
        qd, kd, vd = q.detach(), k.detach(), v.detach()
        t2 = _time(lambda: torch.ops.aten._flash_attention_forward(qd, kd, vd, cu, cu, ns.seq, ns.seq, 0.0, True,
                                                                    False, scale=sc), ns.steps, ns.warmup)
        t3 = _time(lambda: ext().fa_fwd(qd, kd, vd, cu, ns.seq, sc), ns.steps, ns.warmup)
        for var in range(5):
            tv = _time(lambda: ext().fa_fwd(qd, kd, vd, cu, ns.seq, sc, var), ns.steps, ns.warmup)
            res[f"fwd_tc_v{var}_tflops"] = round(fflops / tv / 1e9, 1)
        out, lse = ext().fa_fwd(qd, kd, vd, cu, ns.seq, sc)
        zero = torch.zeros((), dtype=torch.int64, device="cuda")
        outf, lsef, _, _, _ = torch.ops.aten._flash_attention_forward(qd, kd, vd, cu, cu, ns.seq, ns.seq, 0.0, True,
                                                                     False, scale=sc)
        tb2 = _time(lambda: torch.ops.aten._flash_attention_backward(do, qd, kd, vd, outf, lsef, cu, cu, ns.seq, ns.seq,
                                                                     0.0, True, zero, zero, scale=sc),
                    ns.steps, ns.warmup)
        tb3 = _time(lambda: ext().fa_bwd(do, qd, kd, vd, out, lse, cu, ns.seq, sc), ns.steps, ns.warmup)
        for var in range(2):
            tv = _time(lambda: ext().fa_bwd(do, qd, kd, vd, out, lse, cu, ns.seq, sc, variant=var), ns.steps,
                       ns.warmup)
            res[f"bwd_tc_v{var}_tflops"] = round(2.5 * fflops / tv / 1e9, 1)
    bflops = 2.5 * fflops
    res.update(fwd_fa2_ms=t2, fwd_fa2_tflops=fflops / t2 / 1e9, fwd_tc_ms=t3, fwd_tc_tflops=fflops / t3 / 1e9,
               fwd_tc_status=int(ext().fa_fwd_status()), bwd_fa2_ms=tb2, bwd_fa2_tflops=bflops / tb2 / 1e9,
               bwd_tc_ms=tb3, bwd_tc_tflops=bflops / tb3 / 1e9, bwd_tc_status=int(ext().fa_bwd_status()))
    return res


def bench_dgemm(ns) -> dict:
    """Decode-size linears (M = --batch rows) of the model: F.linear (cuBLAS)
    and the weight-streaming tcgen05 kernel, each call on the next of several
    weight copies so the weights stream from HBM as in the decode step."""
    from lumenrl_b200 import ops
    a = _model_args(ns.model)
    shapes = {"qkv": (a.qkv_dim, a.hidden_size), "o": (a.hidden_size, a.q_dim),
              "w13": (2 * a.intermediate_size, a.hidden_size), "w2": (a.hidden_size, a.intermediate_size),
              "lm_head": (a.vocab_size, a.hidden_size)}
    out = {"op": "decode_linears", "M": ns.batch, "cache": "weights rotate through > 300 MB of copies (HBM, not L2)"}
    for name, (N, K) in shapes.items():
        x = torch.randn(ns.batch, K, device="cuda").to(torch.bfloat16)
        copies = max(2, -(-300_000_000 // (N * K * 2)))
        ws = [(torch.randn(N, K, device="cuda") / K ** 0.5).to(torch.bfloat16) for _ in range(copies)]
        it = [0]

        def nxt():
            it[0] = (it[0] + 1) % copies
            return ws[it[0]]
        res = {"weight_MB": round(N * K * 2 / 1e6, 1)}
        res["linear_us"] = round(_time(lambda: torch.nn.functional.linear(x, nxt()), ns.steps, ns.warmup) * 1e3, 1)
        res["skinny_us"] = round(_time(lambda: ops.skinny_linear(x, nxt()), ns.steps, ns.warmup) * 1e3, 1)
        from lumenrl_b200.ops.ext import ext
        res["stream_k_us"] = round(_time(lambda: ext().skinny_sk(x, nxt(), 0), ns.steps, ns.warmup) * 1e3, 1)
        res["stream_k_TBps"] = round(N * K * 2 / res["stream_k_us"] / 1e6, 2)
        out[name] = res
        del ws
    return out


def bench_fp8dgemm(ns) -> dict:
    """FP8 rollout decode linears (M = --batch rows, E4M3 weights with 128x128
    scales): the weight-streaming W8A8 path (quantiser + stream-K kernel)
    against the two-kernel path (1x128 activation quantiser + block-scaled
    GEMM) and the bf16 cuBLAS linear; weights rotate through > 300 MB of
    copies so every call streams them from HBM."""
    from lumenrl_b200 import ops
    from lumenrl_b200.ops.ext import ext
    from lumenrl_b200.quant.fp8 import quant_weight_128x128
    a = _model_args(ns.model)
    shapes = {"qkv": (a.qkv_dim, a.hidden_size), "o": (a.hidden_size, a.q_dim),
              "w13": (2 * a.intermediate_size, a.hidden_size), "w2": (a.hidden_size, a.intermediate_size)}
    out = {"op": "fp8_decode_linears", "M": ns.batch, "cache": "weights rotate through > 300 MB of copies"}
    total = {"stream_us": 0.0, "two_kernel_us": 0.0, "bf16_cublas_us": 0.0}
    for name, (N, K) in shapes.items():
        x = torch.randn(ns.batch, K, device="cuda").to(torch.bfloat16)
        copies = max(2, -(-300_000_000 // (N * K)))
        qs = [quant_weight_128x128((torch.randn(N, K, device="cuda") / K ** 0.5).to(torch.bfloat16))
              for _ in range(copies)]
        wb = [(torch.randn(N, K, device="cuda") / K ** 0.5).to(torch.bfloat16) for _ in range(max(2, copies // 2))]
        it = [0]

        def nxt(pool):
            it[0] = (it[0] + 1) % len(pool)
            return pool[it[0]]
        res = {"weight_MB": round(N * K / 1e6, 1)}
        res["stream_us"] = round(_time(lambda: ext().skinny_fp8(x, *nxt(qs), 0), ns.steps, ns.warmup) * 1e3, 1)
        res["two_kernel_us"] = round(_time(lambda: ops.fp8_gemm_blockwise(x, *nxt(qs)), ns.steps, ns.warmup) * 1e3, 1)
        res["bf16_cublas_us"] = round(_time(lambda: torch.nn.functional.linear(x, nxt(wb)), ns.steps,
                                            ns.warmup) * 1e3, 1)
        res["stream_TBps"] = round(N * K / res["stream_us"] / 1e6, 2)
        res["status"] = int(ext().skinny_fp8_status())
        for k in total:
            total[k] += res[k]
        out[name] = res
        del qs, wb
    out["per_layer_us"] = {k: round(v, 1) for k, v in total.items()}
    return out


def bench_train(ns) -> dict:
    from lumenrl_b200 import ops
    m = _model(ns.model, True)
    m.gradient_checkpointing = ns.recompute
    grad = torch.zeros(m.flat.numel(), dtype=torch.float32, device="cuda")
    m.attach_main_grad(grad)
    T = ns.rows * ns.seq
    ids = torch.randint(0, m.args.vocab_size, (T,), device="cuda")
    pos = torch.arange(ns.seq, device="cuda").repeat(ns.rows)
    cu = torch.arange(0, T + 1, ns.seq, dtype=torch.int32, device="cuda")

    def step():
        h = m.forward_packed(ids, pos, cu, ns.seq)
        lp, _ = ops.token_logprob(h, m.lm_head, ids, want_entropy=False)
        lp.sum().backward()
    ms = _time(step, ns.steps, ns.warmup)
    flops = (8 if ns.recompute else 6) * m.args.num_params() * T
    return {"op": "train_micro_step", "tokens": T, "ms": ms, "tflops": flops / ms / 1e9, "recompute": ns.recompute}


def bench_logprob(ns) -> dict:
    from lumenrl_b200 import ops
    m = _model(ns.model, False)
    T = ns.rows * ns.seq
    h = torch.randn(T, m.args.hidden_size, device="cuda", dtype=torch.bfloat16)
    tgt = torch.randint(0, m.args.vocab_size, (T,), device="cuda")
    ms = _time(lambda: ops.token_logprob(h, m.lm_head, tgt), ns.steps, ns.warmup)
    return {"op": "lmhead_logprob", "tokens": T, "ms": ms,
            "tflops": 2 * T * m.args.vocab_size * m.args.hidden_size / ms / 1e9}


def bench_gemm(ns) -> dict:
    """tcgen05 GEMM vs cuBLAS (torch.matmul) on the model's GEMM shapes."""
    from lumenrl_b200 import ops
    shapes = [(6144, 6144, 4096), (6144, 24576, 4096), (6144, 4096, 12288), (6144, 4096, 4096),
              (4096, 151936, 4096), (8192, 8192, 8192), (64, 24576, 4096), (64, 6144, 4096)]
    out = []
    for M, N, K in shapes:
        a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        b = (torch.randn(N, K, device="cuda") / K ** 0.5).to(torch.bfloat16)
        t_tc = _time(lambda: ops.tc_gemm(a, b), ns.steps, ns.warmup)
        t_cb = _time(lambda: a @ b.t(), ns.steps, ns.warmup)
        fl = 2 * M * N * K
        out.append({"M": M, "N": N, "K": K, "tc_ms": t_tc, "cublas_ms": t_cb, "tc_tflops": fl / t_tc / 1e9,
                    "cublas_tflops": fl / t_cb / 1e9})
    from lumenrl_b200.ops.ext import ext
    for M, N, K in [(64, 6144, 4096), (64, 4096, 4096), (64, 24576, 4096), (64, 4096, 12288), (64, 151936, 4096)]:
        a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        b = (torch.randn(N, K, device="cuda") / K ** 0.5).to(torch.bfloat16)
        t_sk = _time(lambda: ext().tc_gemm_splitk(a, b, 0).to(torch.bfloat16), ns.steps, ns.warmup)
        t_cb = _time(lambda: a @ b.t(), ns.steps, ns.warmup)
        out.append({"M": M, "N": N, "K": K, "splitk_ms": t_sk, "cublas_ms": t_cb,
                    "splitk_TBps": N * K * 2 / t_sk / 1e9, "cublas_TBps": N * K * 2 / t_cb / 1e9})
    st = ops.tc_gemm_status()
    return {"op": "gemm", "status": st, "shapes": out}


def bench_gemm2(ns) -> dict:
    """CTA-pair tcgen05 GEMM vs cuBLAS on the three GEMMs of every Qwen3-8B
    training linear (T = --rows x --seq tokens) and the LM-head chunk:
    forward (x . W^T), dgrad (dy . W) and wgrad (main_grad += dy^T . x)."""
    from lumenrl_b200.ops.ext import ext
    a = _model_args(ns.model)
    T = ns.rows * ns.seq
    shapes = {"qkv": (a.qkv_dim, a.hidden_size), "o": (a.hidden_size, a.q_dim),
              "w13": (2 * a.intermediate_size, a.hidden_size), "w2": (a.hidden_size, a.intermediate_size),
              "lm_head": (a.vocab_size, a.hidden_size)}
    out = {"op": "train_gemms", "tokens": T, "cache": "operands > L2 except where noted by size"}
    tot = {"own": 0.0, "cublas": 0.0}
    for name, (N, K) in shapes.items():
        M = 2048 if name == "lm_head" else T
        x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        w = (torch.randn(N, K, device="cuda") / K ** 0.5).to(torch.bfloat16)
        dy = (torch.randn(M, N, device="cuda") / 8).to(torch.bfloat16)
        mg = torch.zeros(N, K, device="cuda")
        fl = 2 * M * N * K
        r = {}
        for kind, own, lib in [
                ("fwd", lambda: ext().gemm2sm(x, False, w, False, None, 0, ns.bn), lambda: x @ w.t()),
                ("dgrad", lambda: ext().gemm2sm(dy, False, w, True, None, 0, ns.bn), lambda: dy @ w),
                ("wgrad", lambda: ext().gemm2sm(dy, True, x, True, mg, 2, ns.bn),
                 lambda: torch.addmm(mg, dy.t(), x, out_dtype=torch.float32, out=mg))]:
            t_own = _time_sustained(own, ns.steps, ns.warmup, ns.sustain_ms)
            t_lib = _time_sustained(lib, ns.steps, ns.warmup, ns.sustain_ms)
            tot["own"] += t_own
            tot["cublas"] += t_lib
            r[kind] = {"own_tflops": round(fl / t_own / 1e9, 1), "cublas_tflops": round(fl / t_lib / 1e9, 1),
                       "ratio": round(t_lib / t_own, 3)}
        ref = x[:256].float() @ w.float().t()
        r["fwd_max_err"] = (ext().gemm2sm(x[:256], False, w, False, None, 0, 0).float() - ref).abs().max().item()
        out[name] = r
        del x, w, dy, mg
    out["sum_ms"] = {k: round(v, 3) for k, v in tot.items()}
    out["status"] = int(ext().gemm2sm_status())
    return out


def _nvml_handle():
    """NVML handle of the GPU this process runs on (first visible device)."""
    import pynvml
    pynvml.nvmlInit()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")[0].strip()
    if vis.startswith("GPU-"):
        return pynvml.nvmlDeviceGetHandleByUUID(vis)
    return pynvml.nvmlDeviceGetHandleByIndex(int(vis) if vis else 0)


def bench_gemm2energy(ns) -> dict:
    """Energy per FLOP of the training GEMMs: each GEMM runs back to back for
    --sustain-ms (clocks settle under the power limit), then for ~2 s more
    while NVML's energy counter and CUDA events are read; reports TFLOP/s,
    joules per PFLOP and the mean SM clock for the pair GEMM at 256- and
    128-wide tiles and for cuBLAS."""
    import time

    import pynvml
    from lumenrl_b200.ops.ext import ext
    h = _nvml_handle()
    a = _model_args(ns.model)
    T = ns.rows * ns.seq
    shapes = {"qkv": (a.qkv_dim, a.hidden_size), "w13": (2 * a.intermediate_size, a.hidden_size),
              "w2": (a.hidden_size, a.intermediate_size)}
    out = {"op": "gemm_energy", "tokens": T}
    for name, (N, K) in shapes.items():
        x = torch.randn(T, K, device="cuda").to(torch.bfloat16)
        w = (torch.randn(N, K, device="cuda") / K ** 0.5).to(torch.bfloat16)
        dy = (torch.randn(T, N, device="cuda") / 8).to(torch.bfloat16)
        fl = 2 * T * N * K
        r = {}
        for tag, fn in [("own512_fwd", lambda: ext().gemm2sm(x, False, w, False, None, 0, 512)),
                        ("own512_dgrad", lambda: ext().gemm2sm(dy, False, w, True, None, 0, 512)),
                        ("own256_fwd", lambda: ext().gemm2sm(x, False, w, False, None, 0, 256)),
                        ("own128_fwd", lambda: ext().gemm2sm(x, False, w, False, None, 0, 128)),
                        ("cublas_fwd", lambda: x @ w.t()),
                        ("own256_dgrad", lambda: ext().gemm2sm(dy, False, w, True, None, 0, 256)),
                        ("cublas_dgrad", lambda: dy @ w)]:
            _time_sustained(fn, 1, 0, ns.sustain_ms)
            n, clk = 0, []
            e0 = pynvml.nvmlDeviceGetTotalEnergyConsumption(h)
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            t0 = time.perf_counter()
            while time.perf_counter() - t0 < 2.0:
                for _ in range(16):
                    fn()
                n += 16
                clk.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                torch.cuda.synchronize()
            ev1.record()
            torch.cuda.synchronize()
            e1 = pynvml.nvmlDeviceGetTotalEnergyConsumption(h)
            ms = ev0.elapsed_time(ev1)
            r[tag] = {"tflops": round(fl * n / ms / 1e9, 1), "J_per_PFLOP": round((e1 - e0) / 1e3 / (fl * n / 1e15), 1),
                      "W": round((e1 - e0) / ms, 1), "sm_mhz": round(sum(clk) / len(clk))}
        out[name] = r
        del x, w, dy
    out["status"] = int(ext().gemm2sm_status())
    return out


def bench_eagle(ns) -> dict:
    """One Eagle3 draft training step (forward over the 7 TTT steps + backward)
    at Qwen3-8B width on --rows sequences of --seq tokens: teacher hidden
    states random, draft vocabulary 32000.  Run once with the package's
    kernels and once with LRL_EAGLE_KERNELS=0 (PyTorch path) to compare."""
    from lumenrl_b200.models import eagle3
    a = _model_args(ns.model)
    T = ns.rows * ns.seq
    torch.manual_seed(0)
    m = eagle3.Eagle3Model(a.hidden_size, a.vocab_size, 32000, a.num_heads, a.num_kv_heads, a.head_dim,
                           a.intermediate_size, 1, 7, a.rms_norm_eps, a.rope_theta).cuda().to(torch.bfloat16)
    ids = torch.randint(0, a.vocab_size, (T,), device="cuda")
    aux = (torch.randn(T, 3 * a.hidden_size, device="cuda") * 0.5).to(torch.bfloat16)
    tgt = (torch.randn(T, a.hidden_size, device="cuda") * 0.5).to(torch.bfloat16)
    emb = (torch.randn(a.vocab_size, a.hidden_size, device="cuda") * 0.02).to(torch.bfloat16)
    head = (torch.randn(a.vocab_size, a.hidden_size, device="cuda") * 0.02).to(torch.bfloat16)
    cu = torch.arange(0, T + 1, ns.seq, dtype=torch.int32, device="cuda")
    mask = torch.ones(T, device="cuda")

    def step():
        out = m(ids, aux, tgt, emb, head, cu, mask)
        out["loss"].backward()
        m.zero_grad(set_to_none=True)
    ms = _time(step, ns.steps, ns.warmup)
    return {"op": "eagle3_draft_step", "tokens": T, "ttt_steps": 7, "kernels": eagle3._KERNELS, "ms": ms,
            "tokens_per_s": T / ms * 1e3, "peak_mem_GB": torch.cuda.max_memory_allocated() / 1e9}


def bench_fp8gemm(ns) -> dict:
    """Block-scaled FP8 tcgen05 GEMM (csrc/gemm/fp8_gemm.cu) on the forward
    GEMMs of the Qwen3-8B training linears (E4M3 x E4M3, 1x128 activation
    and 128x128 weight scales), against the bf16 CTA-pair GEMM and cuBLAS bf16
    on the same shapes; plus the E5M2-gradient dgrad shape.  Quantisation is
    outside the timed region (weights are quantised once per optimizer step)."""
    from lumenrl_b200.ops.ext import ext
    from lumenrl_b200.quant import fp8 as q8
    a = _model_args(ns.model)
    T = ns.rows * ns.seq
    shapes = {"qkv": (a.qkv_dim, a.hidden_size), "o": (a.hidden_size, a.q_dim),
              "w13": (2 * a.intermediate_size, a.hidden_size), "w2": (a.hidden_size, a.intermediate_size)}
    out = {"op": "fp8_gemm", "tokens": T}
    for name, (N, K) in shapes.items():
        x = torch.randn(T, K, device="cuda").to(torch.bfloat16)
        w = (torch.randn(N, K, device="cuda") / K ** 0.5).to(torch.bfloat16)
        qx, sx = q8.quant_act_1x128(x)
        qw, sw = q8.quant_weight_128x128(w)
        fl = 2 * T * N * K
        t8 = _time(lambda: q8.fp8_matmul(qx, sx, qw, sw), ns.steps, ns.warmup)
        t16 = _time(lambda: ext().gemm2sm(x, False, w, False, None, 0, 0), ns.steps, ns.warmup)
        tcb = _time(lambda: x @ w.t(), ns.steps, ns.warmup)
        ref = q8.dequant_1x128(qx[:256], sx[:256]) @ q8.dequant_128x128(qw, sw).t()
        err = (q8.fp8_matmul(qx[:256].contiguous(), sx[:256].contiguous(), qw, sw).float() - ref).abs().max().item()
        out[name] = {"fp8_tflops": round(fl / t8 / 1e9, 1), "bf16_pair_tflops": round(fl / t16 / 1e9, 1),
                     "cublas_bf16_tflops": round(fl / tcb / 1e9, 1), "fp8_ms": round(t8, 4),
                     "max_err_vs_dequant": err}
        del x, w, qx, sx, qw, sw
    out["status"] = int(q8.fp8_gemm_status())
    return out


def bench_gemm2probe(ns) -> dict:
    """Operand-layout / epilogue probe of the pair GEMM on one shape
    (--rows x --seq tokens by the qkv projection, or --mnk M,N,K): every
    majorness pair with the bf16 epilogue and with the result dropped
    (mainloop-only time).  --case restricts it to one layout (kk, kn, nn, nk)."""
    from lumenrl_b200.ops.ext import ext
    a = _model_args(ns.model)
    M, N, K = (ns.rows * ns.seq, a.qkv_dim, a.hidden_size) if not ns.mnk else tuple(
        int(v) for v in ns.mnk.split(","))
    A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    B = (torch.randn(N, K, device="cuda") / K ** 0.5).to(torch.bfloat16)
    At, Bt = A.t().contiguous(), B.t().contiguous()
    fl = 2 * M * N * K
    out = {"op": "gemm2_probe", "M": M, "N": N, "K": K}
    cases = {"kk": (A, False, B, False), "kn": (A, False, Bt, True), "nn": (At, True, Bt, True),
             "nk": (At, True, B, False)}
    for name, (x, xm, y, ym) in cases.items():
        if ns.case and name != ns.case:
            continue
        for epi, tag in ((0, "bf16"), (3, "none")):
            t = _time(lambda: ext().gemm2sm(x, xm, y, ym, None, epi, ns.bn or 256), ns.steps, ns.warmup)
            out[f"{name}_{tag}_tflops"] = round(fl / t / 1e9, 1)
    if not ns.case:
        t = _time(lambda: A @ B.t(), ns.steps, ns.warmup)
        out["cublas_tflops"] = round(fl / t / 1e9, 1)
    out["status"] = int(ext().gemm2sm_status())
    return out


def bench_comm(ns) -> dict:
    """Fused NVLink optimizer step vs the NCCL path on a Qwen3-8B-sized flat
    buffer (launch under torchrun, one rank per GPU)."""
    import torch.distributed as dist
    from lumenrl_b200.engine.training.optimizer import ShardedFlatAdamW
    from lumenrl_b200.parallel.dist import init_distributed
    from lumenrl_b200.parallel.symm import NVLinkOptimizerComm
    st = init_distributed()
    W, r = st.world_size, st.rank
    n = (ns.numel // (W * 128)) * W * 128
    comm = NVLinkOptimizerComm(n, r, W)
    fused = ShardedFlatAdamW(comm.weights.tensor, W, r, lr=1e-6, comm=comm)
    fused.grad.normal_()

    def fstep():
        fused.comm.fused_step(fused.lo, fused.shard, fused.master, fused.grad_shard, fused.m, fused.v, 1e-6,
                              fused.betas, fused.eps, fused.wd, 1, 1.0)
    t_f = _time(fstep, ns.steps, ns.warmup)
    fstep()
    split = dict(comm.last_timing)          # device time of the two kernels of one step
    sp = torch.tensor([split.get("opt_rs_s", 0.0), split.get("opt_bcast_s", 0.0)], device="cuda",
                      dtype=torch.float64)
    del fused
    plain_w = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    plain = ShardedFlatAdamW(plain_w, W, r, lr=1e-6)

    def pstep():
        plain.grad.normal_() if False else None
        plain._reduce_scatter()
        plain._global_norm()
        from lumenrl_b200.ops.ext import ext
        ext().adamw_step(plain.master, plain.grad_shard, plain.m, plain.v, plain.w16[plain.lo: plain.hi], 1e-6,
                         0.9, 0.999, 1e-8, 0.01, 1, 1.0)
        plain._all_gather()
    t_p = _time(pstep, ns.steps, ns.warmup)
    t = torch.tensor([t_f, t_p], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(sp, op=dist.ReduceOp.MAX)
    nvls = comm.nvls
    comm.close()
    grad_bytes, w_bytes = n * 4, n * 2
    rs_link = (W - 1) / W * grad_bytes       # fp32 gradients a rank pulls from its peers
    ag_link = (W - 1) / W * w_bytes          # bf16 weights a rank pushes to its peers
    return {"op": "optimizer_collective", "world": W, "numel": n, "nvls": nvls, "fused_ms": float(t[0]),
            "nccl_ms": float(t[1]), "rs_norm_ms": float(sp[0]) * 1e3, "adamw_ag_ms": float(sp[1]) * 1e3,
            "rs_link_GBps": rs_link / max(float(sp[0]), 1e-12) / 1e9,
            "ag_link_GBps": ag_link / max(float(sp[1]), 1e-12) / 1e9,
            "nvlink_bytes_per_gpu": rs_link + ag_link}


def bench_allreduce(ns) -> dict:
    """Replicated-DP gradient all-reduce (launch under torchrun): this
    package's NVLink kernel (peer two-shot; NVLS with LRL_NVLS=1) against
    NCCL ``all_reduce`` on an fp32 buffer of --numel elements already in the
    symmetric staging buffer (so only the collective is timed).  Bus bytes per
    GPU = 2 (W-1)/W x size, the all-reduce convention."""
    import torch.distributed as dist
    from lumenrl_b200.ops.ext import ext
    from lumenrl_b200.parallel.dist import init_distributed
    from lumenrl_b200.parallel.symm import NVLinkAllReduce
    st = init_distributed()
    W, r = st.world_size, st.rank
    n = ns.numel // 4 * 4
    comm = NVLinkAllReduce(n, r, W)
    buf = comm.buf.tensor[:n]
    buf.normal_()

    def own():
        comm.epoch += 1
        if comm.nvls:
            ext().nvlink_allreduce_mc(comm.buf.mc, comm.signals.ptrs, r, n, 1.0, comm.epoch, comm.status,
                                      comm.wait_cycles)
        else:
            ext().nvlink_allreduce(comm.buf.ptrs, comm.signals.ptrs, r, n, 1.0, comm.epoch, comm.status,
                                   comm.wait_cycles)
    x = torch.randn(n, device="cuda")
    t_own = _time(own, ns.steps, ns.warmup)
    comm.check()
    t_nccl = _time(lambda: dist.all_reduce(x), ns.steps, ns.warmup)
    t = torch.tensor([t_own, t_nccl], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    comm.close()
    bus = 2 * (W - 1) / W * n * 4
    return {"op": "allreduce_fp32", "world": W, "numel": n, "nvls": comm.nvls, "own_ms": float(t[0]),
            "nccl_ms": float(t[1]), "own_busbw_GBps": bus / float(t[0]) / 1e6,
            "nccl_busbw_GBps": bus / float(t[1]) / 1e6}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["decode", "attn", "attn_train", "skinny", "train", "logprob", "gemm", "comm",
                                     "dgemm", "gemm2", "gemm2probe", "fp8gemm", "gemm2energy", "eagle", "fp8dgemm", "allreduce"])
    ap.add_argument("--blas", choices=["default", "cublas", "cublaslt"], default="default",
                    help="torch's preferred BLAS library for the library GEMMs")
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--prefix", type=int, default=512)
    ap.add_argument("--numel", type=int, default=8_200_000_000)
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--rows", type=int, default=4)
    ap.add_argument("--seq", type=int, default=1536)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--recompute", action="store_true")
    ap.add_argument("--bn", type=int, default=0, help="pair GEMM tile width (0 = auto, 128, 256, 512)")
    ap.add_argument("--mnk", default="", help="gemm2probe shape M,N,K")
    ap.add_argument("--case", default="", help="gemm2probe operand layout: kk, kn, nn or nk")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--fp8", action="store_true", help="decode: W8A8 FP8 rollout linears (128x128 weight blocks)")
    ap.add_argument("--fp8-kv", action="store_true", help="decode: E4M3 KV cache")
    ap.add_argument("--sustain-ms", type=float, default=0.0,
                    help="gemm2: run each GEMM back to back this long before timing it (power-limited clocks)")
    ns = ap.parse_args(argv)
    if ns.blas != "default":
        torch.backends.cuda.preferred_blas_library(ns.blas)
    fn = {"decode": bench_decode, "attn": bench_attn, "skinny": bench_skinny, "attn_train": bench_attn_train, "train": bench_train, "dgemm": bench_dgemm, "logprob": bench_logprob, "gemm": bench_gemm, "fp8gemm": bench_fp8gemm, "fp8dgemm": bench_fp8dgemm, "allreduce": bench_allreduce, "eagle": bench_eagle, "gemm2energy": bench_gemm2energy,
          "comm": bench_comm, "gemm2": bench_gemm2,
          "gemm2probe": bench_gemm2probe}[ns.what]
    res = fn(ns)
    import os
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(res))


if __name__ == "__main__":
    main()
