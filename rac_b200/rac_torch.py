"""PyTorch API of the RAC hot path, bound to librac_b200.so.

Mirrors the public surface of the reference's rac_torch/rac_torch.py
(names, constructor arguments, forward signatures, knobs) so that code
written against it runs unchanged:

    rac_matmul, rac_linear, RACLinear, FusedRACLinear, RACFusedQKV,
    RACFusedFFN, RACRoPE, RACRMSNorm, RACLayerNorm, RACRoPEAttention,
    RACLlamaBlock, patch_model, unpatch_model, rac_set_precision,
    rac_get_precision, rac_set_mode, rac_get_mode, rac_info.

Differences, all deliberate:
  * no CPU fallback: the reference silently runs torch ops when its
    extension is unavailable (rac_torch.py:183, :232); here a CPU tensor in
    a forward pass raises ValueError and a missing library raises RacError;
  * every matmul of a module goes through the rotation-accumulate GEMM in
    the process-wide mode (FAST or CORDIC with n iterations); the reference's
    CUDA build ignores the mode (rac_torch.cu:1181-1214);
  * bias, activation and residual adds are fused into the GEMM epilogue,
    and FusedRACLinear does not recompute F.linear in no-grad mode
    (rac_torch.py:423-426 does);
  * RMSNorm, RoPE and softmax run on this library's kernels;
  * RACLlamaBlock takes `gated=True` for the SwiGLU FFN of
    bench/bench_rac_transformer.c:441-453 (the reference module is ungated,
    rac_torch.py:1374).
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.autograd import Function

from . import _lib, ext
from .ext import ACT_GELU, ACT_NONE, ACT_RELU, ACT_SILU, MODE_CORDIC, MODE_FAST, MODE_SHIFTADD

__all__ = [
    "rac_matmul", "rac_linear", "RACLinear", "FusedRACLinear", "RACFusedQKV", "RACFusedFFN",
    "RACRoPE", "RACRMSNorm", "RACLayerNorm", "RACRoPEAttention", "RACLlamaBlock",
    "patch_model", "unpatch_model", "rac_set_precision", "rac_get_precision",
    "rac_set_mode", "rac_get_mode", "rac_info", "MODE_FAST", "MODE_CORDIC", "MODE_SHIFTADD",
    "ACT_NONE", "ACT_RELU", "ACT_GELU", "ACT_SILU",
]

# ── knobs (rac_torch.py:1009-1118) ─────────────────────────────────────────

_MODE_NAMES = {"fast": MODE_FAST, "cordic": MODE_CORDIC, "shiftadd": MODE_SHIFTADD,
               0: MODE_FAST, 1: MODE_CORDIC, 2: MODE_SHIFTADD}


def _resolve_mode(m) -> int:
    if isinstance(m, int):
        return m if m in (0, 1, 2) else MODE_FAST
    if isinstance(m, str) and m.lower() in _MODE_NAMES:
        return _MODE_NAMES[m.lower()]
    raise ValueError(f"Unknown RAC mode: {m}. Use 'fast', 'cordic', or 'shiftadd'.")


_RAC_CORDIC_ITERS = max(4, min(24, int(os.environ.get("RAC_CORDIC_ITERS", "24"))))
_RAC_CORDIC_MODE = _resolve_mode(os.environ.get("RAC_CORDIC_MODE", "fast"))


def rac_set_mode(mode) -> None:
    """'fast' (sign-XOR FMA), 'cordic' (iterative micro-rotations) or
    'shiftadd' (integer shift-add product, rac_kernels.hip:84-122)."""
    global _RAC_CORDIC_MODE
    _RAC_CORDIC_MODE = _resolve_mode(mode)
    ext.set_cordic_mode(_RAC_CORDIC_MODE)


def rac_get_mode() -> int:
    return _RAC_CORDIC_MODE


def rac_set_precision(iters: int) -> None:
    """CORDIC iteration count, clamped to [4, 24] (rac_torch.py:1099)."""
    global _RAC_CORDIC_ITERS
    _RAC_CORDIC_ITERS = max(4, min(24, int(iters)))
    ext.set_cordic_iters(_RAC_CORDIC_ITERS)


def rac_get_precision() -> int:
    return _RAC_CORDIC_ITERS


def _kw():
    return {"iters": _RAC_CORDIC_ITERS, "mode": _RAC_CORDIC_MODE}


# ── autograd functions ─────────────────────────────────────────────────────

class RACMatmulFunction(Function):
    """C = A @ B; backward dA = dC @ B^T (NT), dB = A^T @ dC (TN)."""

    @staticmethod
    def forward(ctx, A, B):
        ctx.save_for_backward(A, B)
        return ext.matmul_forward(A, B, **_kw())

    @staticmethod
    def backward(ctx, grad_C):
        A, B = ctx.saved_tensors
        gA, gB = ext.matmul_backward(grad_C, A, B, ctx.needs_input_grad[0],
                                     ctx.needs_input_grad[1], **_kw())
        return gA, gB


class RACLinearFunction(Function):
    """out = input @ weight^T + bias (bias fused into the GEMM epilogue)."""

    @staticmethod
    def forward(ctx, input, weight, bias):
        ctx.save_for_backward(input, weight)
        ctx.has_bias = bias is not None
        return ext.linear_forward(input, weight, bias, **_kw())

    @staticmethod
    def backward(ctx, grad_output):
        input, weight = ctx.saved_tensors
        gi, gw, gb = ext.linear_backward(grad_output, input, weight, ctx.has_bias, **_kw())
        return (gi if ctx.needs_input_grad[0] else None,
                gw if ctx.needs_input_grad[1] else None,
                gb.to(grad_output.dtype) if ctx.has_bias else None)


class RACFusedLinearFunction(Function):
    """out = act(input @ weight^T + bias) in one kernel (rac_torch.py:405-455)."""

    @staticmethod
    def forward(ctx, input, weight, bias, act_id):
        ctx.act_id = act_id
        ctx.has_bias = bias is not None
        if act_id == ACT_NONE or not any(ctx.needs_input_grad[:3]):
            out = ext.linear_forward(input, weight, bias, act=act_id, **_kw())
            ctx.save_for_backward(input, weight, out)
            return out
        pre = ext.linear_forward(input, weight, bias, **_kw())
        ctx.save_for_backward(input, weight, pre)
        return _act_torch(pre, act_id)

    @staticmethod
    def backward(ctx, grad_output):
        input, weight, pre = ctx.saved_tensors
        gi, gw, gb = ext.fused_linear_backward(grad_output, input, weight, None, pre,
                                               ctx.act_id, ctx.has_bias, **_kw())
        return gi, gw, (gb if ctx.has_bias else None), None


def _act_torch(x, act_id):
    if act_id == ACT_RELU:
        return torch.relu(x)
    if act_id == ACT_GELU:
        return F.gelu(x)
    if act_id == ACT_SILU:
        return F.silu(x)
    return x


def rac_matmul(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """Drop-in for torch.mm on 2-D CUDA tensors (rac_torch.py:277-285)."""
    return RACMatmulFunction.apply(A, B)


def rac_linear(input, weight, bias=None):
    """Drop-in for F.linear (rac_torch.py:288-302)."""
    return RACLinearFunction.apply(input, weight, bias)


# ── modules ────────────────────────────────────────────────────────────────

class RACLinear(nn.Module):
    """nn.Linear with the RAC GEMM (rac_torch.py:305-376); same parameters and init."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True,
                 device=None, dtype=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        fk = {"device": device, "dtype": dtype}
        self.weight = nn.Parameter(torch.empty((out_features, in_features), **fk))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, **fk))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self):
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)
        if self.bias is not None:
            fan_in = self.weight.shape[1]
            bound = 1.0 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, input):
        return RACLinearFunction.apply(input, self.weight, self.bias)

    def forward_residual(self, input, residual, act: int = ACT_NONE):
        """residual + act(input @ W^T + b) with the add fused into the epilogue
        (inference path: no autograd graph)."""
        return ext.linear_forward(input, self.weight, self.bias, act=act, residual=residual, **_kw())

    @classmethod
    def from_linear(cls, linear: nn.Linear) -> "RACLinear":
        rac = cls(linear.in_features, linear.out_features, bias=linear.bias is not None,
                  device=linear.weight.device, dtype=linear.weight.dtype)
        with torch.no_grad():
            rac.weight.copy_(linear.weight)
            if linear.bias is not None:
                rac.bias.copy_(linear.bias)
        return rac

    def extra_repr(self):
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, backend=RAC-B200")


def _resolve_act(act) -> int:
    table = {"none": ACT_NONE, None: ACT_NONE, "relu": ACT_RELU, "gelu": ACT_GELU,
             "silu": ACT_SILU, "swish": ACT_SILU}
    if isinstance(act, int):
        return act
    key = act.lower() if isinstance(act, str) else act
    if key in table:
        return table[key]
    raise ValueError(f"Unknown activation: {act}. Use 'relu', 'gelu', 'silu', or None.")


class FusedRACLinear(RACLinear):
    """act(input @ W^T + b) in one kernel (rac_torch.py:506-563)."""

    def __init__(self, in_features, out_features, bias=True, activation="relu",
                 device=None, dtype=None):
        super().__init__(in_features, out_features, bias, device, dtype)
        self.activation = activation
        self.act_id = _resolve_act(activation)

    def forward(self, input):
        return RACFusedLinearFunction.apply(input, self.weight, self.bias, self.act_id)

    @classmethod
    def from_linear_and_act(cls, linear, activation="relu"):
        f = cls(linear.in_features, linear.out_features, bias=linear.bias is not None,
                activation=activation, device=linear.weight.device, dtype=linear.weight.dtype)
        with torch.no_grad():
            f.weight.copy_(linear.weight)
            if linear.bias is not None:
                f.bias.copy_(linear.bias)
        return f

    def extra_repr(self):
        return super().extra_repr() + f", activation={self.activation}"


class RACFusedQKV(nn.Module):
    """One [3d, d] projection split into Q, K, V (rac_torch.py:586-628)."""

    def __init__(self, d_model, bias=True, device=None, dtype=None):
        super().__init__()
        self.d_model = d_model
        self.qkv = RACLinear(d_model, 3 * d_model, bias=bias, device=device, dtype=dtype)

    def forward(self, x):
        return self.qkv(x).chunk(3, dim=-1)


class RACFusedFFN(nn.Module):
    """fc2(act(fc1(x))) (rac_torch.py:631-655)."""

    def __init__(self, d_model, ff_dim, activation="gelu", bias=True, device=None, dtype=None):
        super().__init__()
        self.fc1 = FusedRACLinear(d_model, ff_dim, bias=bias, activation=activation,
                                  device=device, dtype=dtype)
        self.fc2 = RACLinear(ff_dim, d_model, bias=bias, device=device, dtype=dtype)

    def forward(self, x):
        return self.fc2(self.fc1(x))

    def forward_residual(self, x, residual):
        h = ext.linear_forward(x, self.fc1.weight, self.fc1.bias, act=self.fc1.act_id, **_kw())
        return self.fc2.forward_residual(h, residual)


class RACGatedFFN(nn.Module):
    """SwiGLU FFN: down(silu(gate(x)) * up(x)), the gated layer of the reference's
    CPU decoder bench (bench/bench_rac_transformer.c:441-453)."""

    def __init__(self, d_model, ff_dim, bias=False, device=None, dtype=None):
        super().__init__()
        self.gate = FusedRACLinear(d_model, ff_dim, bias=bias, activation="silu",
                                   device=device, dtype=dtype)
        self.up = RACLinear(d_model, ff_dim, bias=bias, device=device, dtype=dtype)
        self.down = RACLinear(ff_dim, d_model, bias=bias, device=device, dtype=dtype)

    def forward(self, x):
        return self.down(self.gate(x) * self.up(x))

    def _gate_up(self) -> torch.Tensor:
        """gate and up weights row-interleaved ([2F, d]) for the one-GEMM SwiGLU;
        derived state, rebuilt whenever either weight's storage or version changes."""
        key = tuple((w.data_ptr(), w._version, tuple(w.shape), w.device)
                    for w in (self.gate.weight, self.up.weight))
        if getattr(self, "_gu_key", None) != key:
            with torch.no_grad():
                self._gu = torch.stack([self.gate.weight, self.up.weight], 1).reshape(
                    -1, self.gate.weight.shape[1]).float().contiguous()
            self._gu_key = key
        return self._gu

    def forward_residual(self, x, residual):
        if self.gate.bias is None and self.up.bias is None:
            h = ext.linear_forward(x, self._gate_up(), None, act=ext.ACT_SWIGLU, **_kw())
            return self.down.forward_residual(h, residual)
        g = ext.linear_forward(x, self.gate.weight, self.gate.bias, act=ACT_SILU, **_kw())
        u = ext.linear_forward(x, self.up.weight, self.up.bias, **_kw())
        return self.down.forward_residual(g.mul_(u), residual)


class RACRoPE(nn.Module):
    """Rotary embeddings (rac_torch.py:1132-1196).  The cos/sin cache is built
    with the reference's torch formula; the pair rotation runs on the RoPE
    kernel in the reference module's rounding form (form 1)."""

    def __init__(self, head_dim: int, max_seq_len: int = 2048, base: float = 10000.0,
                 device=None, dtype=torch.float32):
        super().__init__()
        assert head_dim % 2 == 0, f"head_dim must be even, got {head_dim}"
        self.head_dim, self.max_seq_len, self.base = head_dim, max_seq_len, base
        half = head_dim // 2
        inv_freq = 1.0 / (base ** (torch.arange(0, half, dtype=torch.float32) * 2 / head_dim))
        angles = torch.arange(max_seq_len, dtype=torch.float32).unsqueeze(1) * inv_freq.unsqueeze(0)
        self.register_buffer("cos_cache", angles.cos().to(dtype=dtype, device=device), persistent=False)
        self.register_buffer("sin_cache", angles.sin().to(dtype=dtype, device=device), persistent=False)

    def _rotate(self, x, positions):
        out = x.float().contiguous().clone() if x.is_contiguous() and x.dtype == torch.float32 \
            else x.float().contiguous()
        seq = x.shape[-2]
        if positions is None:
            c, s = self.cos_cache[:seq], self.sin_cache[:seq]
        else:
            if positions.dim() != 1:
                raise ValueError("RACRoPE: positions must be a 1-D index over the sequence")
            c, s = self.cos_cache[positions], self.sin_cache[positions]
        ext.rope_apply_(out, c.float().contiguous(), s.float().contiguous(), form=1)
        return out if x.dtype == torch.float32 else out.to(x.dtype)

    def forward(self, q, k, positions=None):
        return self._rotate(q, positions), self._rotate(k, positions)

    def extra_repr(self):
        return f"head_dim={self.head_dim}, max_seq_len={self.max_seq_len}, base={self.base}"


class RACRMSNorm(nn.Module):
    """y = x * rsqrt(mean(x^2) + eps) * weight (rac_torch.py:1205-1234)."""

    def __init__(self, d_model: int, eps: float = 1e-6, device=None, dtype=None):
        super().__init__()
        self.d_model, self.eps = d_model, eps
        self.weight = nn.Parameter(torch.ones(d_model, device=device, dtype=dtype))

    def forward(self, x):
        y = ext.rmsnorm(x.float().contiguous(), self.weight.float().contiguous(), self.eps)
        return y if x.dtype == torch.float32 else y.to(x.dtype)

    def extra_repr(self):
        return f"d_model={self.d_model}, eps={self.eps}"


class RACLayerNorm(nn.Module):
    """(x - mean) * rsqrt(var + eps) * weight + bias (rac_torch.py:1239-1276)."""

    def __init__(self, d_model: int, eps: float = 1e-5, bias: bool = True, device=None, dtype=None):
        super().__init__()
        self.d_model, self.eps = d_model, eps
        self.weight = nn.Parameter(torch.ones(d_model, device=device, dtype=dtype))
        if bias:
            self.bias = nn.Parameter(torch.zeros(d_model, device=device, dtype=dtype))
        else:
            self.register_parameter("bias", None)

    def forward(self, x):
        b = self.bias.float().contiguous() if self.bias is not None else None
        y = ext.layernorm(x.float().contiguous(), self.weight.float().contiguous(), b, self.eps)
        return y if x.dtype == torch.float32 else y.to(x.dtype)


class RACRoPEAttention(nn.Module):
    """Llama-style attention (rac_torch.py:1279-1343): fused qkv RACLinear, RoPE on
    Q and K, softmax(QK^T * scale + mask) V, out_proj RACLinear.  In inference
    the attention core is this library's fused kernel (rac_attention, no
    [B, H, T, T] tensor); under autograd it is torch.matmul + softmax in fp32,
    as in the reference module."""

    def __init__(self, d_model: int, n_heads: int, max_seq_len: int = 4096, bias: bool = False,
                 dropout: float = 0.0, rope_base: float = 10000.0, device=None, dtype=None):
        super().__init__()
        assert d_model % n_heads == 0
        self.d_model, self.n_heads = d_model, n_heads
        self.d_head = d_model // n_heads
        self.scale = self.d_head ** -0.5
        self.qkv = RACLinear(d_model, 3 * d_model, bias=bias, device=device, dtype=dtype)
        self.out_proj = RACLinear(d_model, d_model, bias=bias, device=device, dtype=dtype)
        self.rope = RACRoPE(self.d_head, max_seq_len=max_seq_len, base=rope_base,
                            device=device, dtype=dtype or torch.float32)
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()

    def _context(self, x, mask=None, is_causal=False, positions=None, n_heads=None):
        """Attention output before out_proj, [B, T, heads*d_head]."""
        B, T, _ = x.shape
        H = n_heads or self.n_heads
        qkv = self.qkv(x)
        q, k, v = qkv.chunk(3, dim=-1)
        q = q.view(B, T, H, self.d_head).transpose(1, 2)
        k = k.view(B, T, H, self.d_head).transpose(1, 2)
        v = v.view(B, T, H, self.d_head).transpose(1, 2)
        q, k = self.rope(q, k, positions=positions)
        fused_ok = (not torch.is_grad_enabled() and isinstance(self.dropout, nn.Identity)
                    and self.d_head in (32, 64, 128)
                    and (mask is None or tuple(mask.shape) == (T, T)))
        if fused_ok:
            # One streaming kernel: no [B, H, T, T] score tensor (rac_attention).
            m = mask.to(device=x.device, dtype=torch.float32).contiguous() if mask is not None else None
            out = ext.attention(q, k, v.contiguous(), m, is_causal)
            return out.transpose(1, 2).reshape(B, T, H * self.d_head)
        scores = torch.matmul(q, k.transpose(-2, -1)) * self.scale
        if is_causal:
            scores = scores + torch.triu(torch.full((T, T), float("-inf"), device=x.device,
                                                    dtype=scores.dtype), diagonal=1)
        if mask is not None:
            scores = scores + mask
        if torch.is_grad_enabled() and scores.requires_grad:
            attn = torch.softmax(scores, dim=-1)      # autograd needs the torch op
        else:
            attn = ext.softmax(scores.contiguous())
        attn = self.dropout(attn)
        out = torch.matmul(attn, v)
        return out.transpose(1, 2).reshape(B, T, H * self.d_head)

    def forward(self, x, mask=None, is_causal=False, positions=None):
        return self.out_proj(self._context(x, mask, is_causal, positions))

    def extra_repr(self):
        return f"d_model={self.d_model}, n_heads={self.n_heads}, d_head={self.d_head}"


class RACLlamaBlock(nn.Module):
    """x + attn(RMSNorm(x)); x + ffn(RMSNorm(x))  (rac_torch.py:1348-1383).

    Same submodule names and parameter shapes as the reference, so its
    state_dict loads unchanged.  gated=True swaps the FFN for the SwiGLU
    form (RACGatedFFN).  In inference (no grad) the two residual adds are
    fused into the out_proj / down-projection GEMM epilogues."""

    def __init__(self, d_model: int, n_heads: int, ff_dim: int = None, max_seq_len: int = 4096,
                 activation: str = "silu", dropout: float = 0.0, bias: bool = False,
                 rms_eps: float = 1e-6, rope_base: float = 10000.0, gated: bool = False,
                 device=None, dtype=None):
        super().__init__()
        ff_dim = ff_dim or 4 * d_model
        self.gated = gated
        self.norm1 = RACRMSNorm(d_model, eps=rms_eps, device=device, dtype=dtype)
        self.attn = RACRoPEAttention(d_model, n_heads, max_seq_len=max_seq_len, bias=bias,
                                     dropout=dropout, rope_base=rope_base, device=device, dtype=dtype)
        self.norm2 = RACRMSNorm(d_model, eps=rms_eps, device=device, dtype=dtype)
        if gated:
            self.ffn = RACGatedFFN(d_model, ff_dim, bias=bias, device=device, dtype=dtype)
        else:
            self.ffn = RACFusedFFN(d_model, ff_dim, activation=activation, bias=bias,
                                   device=device, dtype=dtype)

    def forward(self, x, mask=None, is_causal=False, positions=None):
        if torch.is_grad_enabled():
            x = x + self.attn(self.norm1(x), mask=mask, is_causal=is_causal, positions=positions)
            return x + self.ffn(self.norm2(x))
        ctx = self.attn._context(self.norm1(x), mask, is_causal, positions)
        h = self.attn.out_proj.forward_residual(ctx, x)
        return self.ffn.forward_residual(self.norm2(h), h)

    def extra_repr(self):
        return f"d_model={self.norm1.d_model}, n_heads={self.attn.n_heads}, gated={self.gated}"


# ── model patching (rac_torch.py:865-942) ──────────────────────────────────

def patch_model(model: nn.Module, verbose: bool = True, min_features: int = 64) -> nn.Module:
    """Replaces every nn.Linear whose in and out features are both >= min_features
    by RACLinear (same signature and default as rac_torch.py:865-869: layers
    smaller than 64 stay torch's)."""
    count = 0

    def _replace(mod, prefix=""):
        nonlocal count
        for name, child in list(mod.named_children()):
            if isinstance(child, nn.Linear) and not isinstance(child, RACLinear) and \
                    min(child.in_features, child.out_features) >= min_features:
                setattr(mod, name, RACLinear.from_linear(child))
                count += 1
            else:
                _replace(child, f"{prefix}{name}.")

    _replace(model)
    if verbose:
        print(f"[rac_b200] patched {count} Linear layer(s)")
    return model


def unpatch_model(model: nn.Module, verbose: bool = True) -> nn.Module:
    """Inverse of patch_model: RACLinear -> nn.Linear with the same weights."""
    count = 0

    def _restore(mod):
        nonlocal count
        for name, child in list(mod.named_children()):
            if type(child) is RACLinear:
                lin = nn.Linear(child.in_features, child.out_features, bias=child.bias is not None,
                                device=child.weight.device, dtype=child.weight.dtype)
                with torch.no_grad():
                    lin.weight.copy_(child.weight)
                    if child.bias is not None:
                        lin.bias.copy_(child.bias)
                setattr(mod, name, lin)
                count += 1
            else:
                _restore(child)

    _restore(model)
    if verbose:
        print(f"[rac_b200] restored {count} Linear layer(s)")
    return model


def rac_info() -> dict:
    """Library and knob status (rac_torch.py:1388-1409), returned and printed."""
    L = _lib.lib()
    info = {
        "library": _lib.LIB_PATH, "version": L.rac_b200_version().decode(),
        "devices": L.rac_b200_device_count(), "cordic_iters": _RAC_CORDIC_ITERS,
        "mode": {0: "fast", 1: "cordic", 2: "shiftadd"}[_RAC_CORDIC_MODE],
        "cpu_fallback": False,
    }
    for k, v in info.items():
        print(f"  {k:14s} {v}")
    return info
