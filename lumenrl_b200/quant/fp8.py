"""FP8 configuration, blockwise quantisers, W8A8 rollout linear, FP8 KV-cache
calibration and hybrid FP8 training (reference ``lumenrl/quantization/*``).

Formats: E4M3 (max 448) for weights/activations, E5M2 (max 57344) for
gradients in hybrid training.  Granularities: 1x128 along the contraction dim
(activations; the reference's ``WeightQuantizer.quantize_tensor``) and
128x128 blocks (rollout weights, ``fp8_per_block``).  On CUDA the quantisers
are the ``quant_act_1x128`` / ``quant_weight_128x128`` kernels; CPU uses the
PyTorch definitions below.  Scales are ``amax / fp8_max`` (optionally rounded
to a power of two); a zero block gets scale ``tiny``/1 so it stays zero.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Any, Literal, Optional

import torch
from torch import Tensor

logger = logging.getLogger(__name__)

E4M3, E5M2 = torch.float8_e4m3fn, torch.float8_e5m2
FP8_MAX = {E4M3: 448.0, E5M2: 57344.0}


def fp8_e4m3_max() -> float:
    return 448.0


@dataclass(frozen=True)
class FP8Config:
    precision: str = "bf16"
    recipe: Literal["blockwise", "tensorwise"] = "blockwise"
    use_deep_gemm: bool = True
    num_first_layers_in_bf16: int = 0
    num_last_layers_in_bf16: int = 0
    use_weight_pow2_scale: bool = False
    use_activation_pow2_scale: bool = False

    def is_fp8_enabled(self) -> bool:
        p = self.precision.lower().strip()
        return p in {"fp8", "float8", "e4m3", "e5m2", "hybrid_fp8", "hybrid"} or "fp8" in p

    @classmethod
    def from_config(cls, quant_config) -> "FP8Config":
        r, t = quant_config.rollout, quant_config.training
        precision = t.fp8 if t.fp8 else r.precision
        recipe = t.fp8_recipe if t.fp8_recipe in ("blockwise", "tensorwise") else "blockwise"
        return cls(precision=precision, recipe=recipe, use_deep_gemm=r.use_deep_gemm,
                   num_first_layers_in_bf16=r.num_first_layers_in_bf16,
                   num_last_layers_in_bf16=r.num_last_layers_in_bf16)


def _pow2(s: Tensor) -> Tensor:
    return torch.pow(2.0, torch.round(torch.log2(s.clamp(min=torch.finfo(s.dtype).tiny))))


def quant_1x128_ref(x: Tensor, dtype=E4M3, pow2: bool = False) -> tuple[Tensor, Tensor]:
    lead, K = x.shape[:-1], x.shape[-1]
    nkb = (K + 127) // 128
    xp = torch.nn.functional.pad(x.float().reshape(-1, K), (0, nkb * 128 - K))
    blocks = xp.view(-1, nkb, 128)
    amax = blocks.abs().amax(-1)
    s = torch.where(amax > 0, amax / FP8_MAX[dtype], torch.ones_like(amax))
    if pow2:
        s = _pow2(s)
    q = (blocks / s.unsqueeze(-1)).clamp(-FP8_MAX[dtype], FP8_MAX[dtype]).to(dtype)
    return q.view(-1, nkb * 128)[:, :K].reshape(*lead, K), s.reshape(*lead, nkb)


def quant_128x128_ref(w: Tensor, dtype=E4M3, pow2: bool = False) -> tuple[Tensor, Tensor]:
    N, K = w.shape
    nn_, nk = (N + 127) // 128, (K + 127) // 128
    wp = torch.nn.functional.pad(w.float(), (0, nk * 128 - K, 0, nn_ * 128 - N))
    blocks = wp.view(nn_, 128, nk, 128).permute(0, 2, 1, 3)
    amax = blocks.abs().amax((-1, -2))
    s = torch.where(amax > 0, amax / FP8_MAX[dtype], torch.ones_like(amax))
    if pow2:
        s = _pow2(s)
    q = (blocks / s[..., None, None]).clamp(-FP8_MAX[dtype], FP8_MAX[dtype]).to(dtype)
    q = q.permute(0, 2, 1, 3).reshape(nn_ * 128, nk * 128)[:N, :K]
    return q.contiguous(), s


def quant_act_1x128(x: Tensor, dtype=E4M3) -> tuple[Tensor, Tensor]:
    if x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2:
        from lumenrl_b200.ops.ext import ext
        return tuple(ext().quant_act_1x128(x.contiguous(), dtype == E5M2))
    return quant_1x128_ref(x, dtype)


def quant_weight_128x128(w: Tensor, dtype=E4M3) -> tuple[Tensor, Tensor]:
    if w.is_cuda and w.dtype == torch.bfloat16:
        from lumenrl_b200.ops.ext import ext
        return tuple(ext().quant_weight_128x128(w.contiguous(), dtype == E5M2))
    return quant_128x128_ref(w, dtype)


def dequant_1x128(q: Tensor, s: Tensor) -> Tensor:
    K = q.shape[-1]
    return (q.float() * s.repeat_interleave(128, -1)[..., :K]).to(torch.float32)


def dequant_128x128(q: Tensor, s: Tensor) -> Tensor:
    N, K = q.shape
    full = s.repeat_interleave(128, 0)[:N].repeat_interleave(128, 1)[:, :K]
    return q.float() * full


class WeightQuantizer:
    """BF16 <-> FP8 E4M3 blockwise (1x128 along the last dim) for state dicts."""

    def __init__(self, config: FP8Config = FP8Config()) -> None:
        self.config = config

    def quantize_tensor(self, tensor: Tensor, block_size: int = 128) -> tuple[Tensor, Tensor]:
        if tensor.dim() < 1:
            raise ValueError("quantize_tensor expects tensor.dim() >= 1")
        if tensor.shape[-1] % block_size:
            raise ValueError(f"Last dim {tensor.shape[-1]} must be divisible by block_size={block_size}")
        if block_size != 128:
            raise ValueError("only 128-wide blocks are supported")
        return quant_1x128_ref(tensor, E4M3, self.config.use_weight_pow2_scale)

    def dequantize_tensor(self, quantized: Tensor, scales: Tensor, block_size: int = 128) -> Tensor:
        return dequant_1x128(quantized, scales).reshape(quantized.shape)

    def quantize_state_dict(self, sd: dict[str, Any]) -> dict[str, Any]:
        out: dict[str, Any] = {}
        for k, v in sd.items():
            if (isinstance(v, Tensor) and v.is_floating_point() and v.dtype not in (E4M3, E5M2) and v.ndim == 2
                    and v.shape[1] % 128 == 0):
                q, s = self.quantize_tensor(v.float())
                out[k] = q
                out[f"{k}_fp8_scales"] = s.to(torch.bfloat16)
                out[f"{k}_fp8_meta"] = torch.tensor(list(v.shape), dtype=torch.int64)
            else:
                out[k] = v
        return out

    def dequantize_state_dict(self, sd: dict[str, Any], dtype=torch.bfloat16) -> dict[str, Any]:
        out: dict[str, Any] = {}
        for k, v in sd.items():
            if k.endswith("_fp8_scales") or k.endswith("_fp8_meta"):
                continue
            s = sd.get(f"{k}_fp8_scales")
            out[k] = self.dequantize_tensor(v, s.float()).to(dtype) if s is not None else v
        return out


class FP8RolloutQuantizer:
    """W8A8 blockwise rollout weights: 128x128 E4M3 weight blocks with fp32
    scales, 1x128 activation blocks quantised on the fly.  The first/last
    ``num_*_layers_in_bf16`` decoder layers stay bf16."""

    def __init__(self, config: FP8Config, num_layers: int) -> None:
        self.config = config
        self.num_layers = num_layers
        self.weights: dict[str, tuple[Tensor, Tensor]] = {}

    def layer_in_fp8(self, i: int) -> bool:
        c = self.config
        return c.num_first_layers_in_bf16 <= i < self.num_layers - c.num_last_layers_in_bf16

    def quantize_model(self, model) -> dict:
        """(Re)quantise every eligible linear weight of ``model`` (used after
        each weight sync).  A re-quantisation writes into the tensors of the
        first one, so decode graphs captured against them stay valid."""
        for name, p in model.named_flat_params():
            if not any(name.endswith(s) for s in ("wqkv", "wo", "w13", "w2")):
                continue
            layer = int(name.split(".")[1])
            if self.layer_in_fp8(layer):
                qw, sw = quant_weight_128x128(p.detach())
                old = self.weights.get(name)
                if old is not None and old[0].shape == qw.shape and old[1].shape == sw.shape:
                    old[0].copy_(qw)
                    old[1].copy_(sw)
                else:
                    self.weights[name] = (qw, sw)
        return {"fp8/quantized_tensors": len(self.weights)}

    def linear(self, name: str, x: Tensor, w_bf16: Tensor, decode: bool = False) -> Tensor:
        """``decode``: x holds one token per live sequence; the weight-streaming
        W8A8 kernel serves it (the weights are read once)."""
        if name not in self.weights:
            return x @ w_bf16.t()
        qw, sw = self.weights[name]
        if x.is_cuda:
            from lumenrl_b200.ops import fp8_decode_linear, fp8_gemm_blockwise
            return fp8_decode_linear(x, qw, sw) if decode else fp8_gemm_blockwise(x, qw, sw)
        qx, sx = quant_1x128_ref(x)
        return (dequant_1x128(qx, sx) @ dequant_128x128(qw, sw).t()).to(x.dtype)


class FP8KVCacheQuantizer:
    """Per-layer K/V scales from observed amax (``scale = amax / 448``),
    recalibrated from prefill activations (reference
    ``quantization/fp8_kv_cache.py:26-80``)."""

    def __init__(self, num_layers: int, margin: float = 1.0) -> None:
        self.k_amax = [0.0] * num_layers
        self.v_amax = [0.0] * num_layers
        self.margin = margin

    def observe(self, layer: int, k: Tensor, v: Tensor) -> None:
        self.k_amax[layer] = max(self.k_amax[layer], float(k.abs().amax()))
        self.v_amax[layer] = max(self.v_amax[layer], float(v.abs().amax()))

    def scales(self) -> tuple[list[float], list[float]]:
        ks = [max(a * self.margin / 448.0, 1e-8) if a > 0 else 1.0 for a in self.k_amax]
        vs = [max(a * self.margin / 448.0, 1e-8) if a > 0 else 1.0 for a in self.v_amax]
        return ks, vs

    def apply(self, cache) -> None:
        cache.k_scale, cache.v_scale = self.scales()


def quant_t_1x128(x: Tensor, dtype=E4M3, kb_major: bool = False) -> tuple[Tensor, Tensor]:
    """x [R, C] -> (x^T quantised 1x128 along R: [C, Rpad] with Rpad = R
    rounded up to 128 (zero rows), scales [C, Rpad/128] or, ``kb_major``,
    [Rpad/128, Cpad] with Cpad = C rounded up to 128)."""
    if x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2:
        from lumenrl_b200.ops.ext import ext
        return tuple(ext().quant_t_1x128(x.contiguous(), dtype == E5M2, kb_major))
    R, C = x.shape
    Rpad = (R + 127) // 128 * 128
    xt = torch.nn.functional.pad(x.float().t(), (0, Rpad - R))
    q, s = quant_1x128_ref(xt, dtype)
    if kb_major:
        Cpad = (C + 127) // 128 * 128
        s = torch.nn.functional.pad(s.t(), (0, Cpad - C)).contiguous()
    return q, s


_FP8_ERR: dict = {}


def _err_word(dev) -> Tensor:
    if dev not in _FP8_ERR:
        _FP8_ERR[dev] = torch.zeros(1, dtype=torch.int32, device=dev)
    return _FP8_ERR[dev]


def fp8_matmul(qa: Tensor, sa: Tensor, qb: Tensor, sb: Tensor, out: Optional[Tensor] = None,
               b_row: bool = False) -> Tensor:
    """sum_kb (qa[:, kb] . qb[:, kb]^T) * sa[:, kb] * sb(kb): block-scaled
    FP8 GEMM (E4M3 / E5M2 in any combination).  ``b_row``: ``sb`` holds one
    scale per row of ``qb`` and K block, K-block-major ([K/128, Npad]); else
    128x128 blocks ([N/128, K/128]).  Returns bf16, or accumulates into the
    fp32 ``out``."""
    if qa.is_cuda:
        from lumenrl_b200.ops.ext import ext
        return ext().fp8_gemm_ex(qa, sa.contiguous(), qb, sb.contiguous(), _err_word(qa.device), out, b_row)
    a = dequant_1x128(qa, sa)
    if b_row:
        N = qb.shape[0]
        b = dequant_1x128(qb, sb[:, :N].t())
    else:
        b = dequant_128x128(qb, sb)
    r = a @ b.t()
    if out is not None:
        out += r
        return out
    return r.to(torch.bfloat16)


def fp8_gemm_status() -> int:
    v = 0
    for t in _FP8_ERR.values():
        v = max(v, int(t.item()))
        t.zero_()
    return v


class _FP8Linear(torch.autograd.Function):
    """y = x W^T with E4M3 forward operands; E5M2 gradients in dgrad and
    wgrad; the weight gradient accumulates in fp32 into W.main_grad."""

    @staticmethod
    def forward(ctx, x: Tensor, w: Tensor, w_handle: Tensor, mgr: "FP8TrainingManager", name: str):
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        qx, sx = quant_act_1x128(x2, E4M3)
        qw, sw = mgr.forward_weight(name, w)
        y = fp8_matmul(qx, sx, qw, sw)
        ctx.save_for_backward(x2, w)
        ctx.meta = (w_handle, mgr, name, x.shape)
        return y.to(x.dtype).view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy: Tensor):
        x2, w = ctx.saved_tensors
        w_handle, mgr, name, xshape = ctx.meta
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        if dy2.dtype != torch.bfloat16 and dy2.is_cuda:
            dy2 = dy2.to(torch.bfloat16)
        # dgrad: dx = dy . W   (E5M2 gradient x E4M3 transposed weight)
        qdy, sdy = quant_act_1x128(dy2, E5M2)
        qwt, swt = mgr.backward_weight(name, w)
        dx = fp8_matmul(qdy, sdy, qwt, swt).to(x2.dtype).view(xshape)
        # wgrad: dW += dy^T . x, contraction over tokens: both operands
        # quantised 1x128 along the token dimension
        qdt, sdt = quant_t_1x128(dy2, E5M2)
        qxt, sxt = quant_t_1x128(x2.to(dy2.dtype) if not x2.is_cuda else x2, E4M3, kb_major=True)
        mg = getattr(w_handle, "main_grad", None)
        if mg is not None:
            fp8_matmul(qdt, sdt, qxt, sxt, out=mg, b_row=True)
        else:
            g = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
            fp8_matmul(qdt, sdt, qxt, sxt, out=g, b_row=True)
            w_handle.grad = g.to(w_handle.dtype) if w_handle.grad is None else w_handle.grad + g.to(w_handle.dtype)
        return dx, None, None, None, None


class FP8TrainingManager:
    """Hybrid FP8 training (reference ``lumenrl/quantization/fp8_training.py:41-134``
    and the Lumen recipe of ``engine/training/fsdp_backend.py:251-366``).

    Every decoder linear (qkv, o, gate/up, down) runs three block-scaled FP8
    GEMMs on the tcgen05 tensor cores (``csrc/gemm/fp8_gemm.cu``):

    * forward: E4M3 activations (1x128 scales) x E4M3 weights (128x128);
    * dgrad: E5M2 output gradient (1x128) x E4M3 transposed weight (128x128);
    * wgrad: E5M2 gradient^T x E4M3 activations^T, both quantised 1x128 along
      the token dimension, accumulated in fp32 into ``main_grad``.

    Master weights and the optimizer stay fp32 / bf16 as before; the LM head,
    embeddings and norms stay bf16.  Quantised weights (and their transposes)
    are computed once per optimizer step and reused by every micro-batch;
    ``weights_updated()`` drops them after the step."""

    TARGETS = ("wqkv", "wo", "w13", "w2")

    def __init__(self, config: FP8Config) -> None:
        self.config = config
        self.enabled = config.is_fp8_enabled()
        self._fwd: dict[str, tuple[Tensor, Tensor]] = {}
        self._bwd: dict[str, tuple[Tensor, Tensor]] = {}

    def applies_to(self, name: str) -> bool:
        return self.enabled and name.rsplit(".", 1)[-1] in self.TARGETS

    def attach(self, model) -> None:
        model.fp8_training = self if self.enabled else None

    def weights_updated(self) -> None:
        self._fwd.clear()
        self._bwd.clear()

    def forward_weight(self, name: str, w: Tensor) -> tuple[Tensor, Tensor]:
        if name not in self._fwd:
            self._fwd[name] = quant_weight_128x128(w, E4M3)
        return self._fwd[name]

    def backward_weight(self, name: str, w: Tensor) -> tuple[Tensor, Tensor]:
        if name not in self._bwd:
            qw, sw = self.forward_weight(name, w)
            # the 128x128 blocks of W^T are those of W transposed: same bytes, same scales
            self._bwd[name] = (qw.t().contiguous(), sw.t().contiguous())
        return self._bwd[name]

    def linear(self, name: str, x: Tensor, w: Tensor) -> Tensor:
        if torch.is_grad_enabled() and w.requires_grad:
            return _FP8Linear.apply(x, w.detach(), w, self, name)
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        qx, sx = quant_act_1x128(x2, E4M3)
        qw, sw = self.forward_weight(name, w.detach())
        return fp8_matmul(qx, sx, qw, sw).to(x.dtype).view(*x.shape[:-1], w.shape[0])

    def reset_fp8_state(self, model=None) -> None:
        """Per-step hook of the reference API: quantised weights are dropped;
        scales come from each tensor's current blocks (no amax history)."""
        self.weights_updated()
