"""Torch-tensor front end of librac_b200.so.

The first half mirrors the pybind surface of the reference extension
``rac_cuda_ext`` (rac_torch/rac_torch_bind.cpp:223-258 and
rac_torch/rac_torch.cu:1181-1214): same function names, argument names,
defaults and conventions --

* ``iters <= 0`` takes the process-wide iteration knob, ``mode < 0`` the
  process-wide mode (rac_torch_bind.cpp:81-82);
* fp16/bf16 inputs are computed in fp32 and cast back (rac_torch.cu:867-872);
* an empty bias tensor means "no bias";
* kernels run on the current torch CUDA stream.

The second half exposes the elementwise / row-wise kernels on tensors.
Every call needs CUDA tensors: there is no CPU path, and a CPU tensor is a
``ValueError``.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import LAYOUT_NN, LAYOUT_NT, LAYOUT_TN

MODE_FAST, MODE_CORDIC, MODE_SHIFTADD = 0, 1, 2
ACT_NONE, ACT_RELU, ACT_GELU, ACT_SILU = 0, 1, 2, 3
# silu(v[:, 2c]) * v[:, 2c+1] over row-interleaved gate/up weights (N/2 outputs)
ACT_SWIGLU = 4

# Process-wide knobs of the torch binding (rac_torch_bind.cpp:54-55):
# defaults iters = 24, mode = FAST.
_iters = 24
_mode = MODE_FAST


def set_cordic_iters(iters: int) -> None:
    """rac_torch_bind.cpp:205-212: <= 0 resets to 24, else clamp to [1, 24]."""
    global _iters
    _iters = 24 if iters <= 0 else max(1, min(24, int(iters)))


def get_cordic_iters() -> int:
    return _iters


def set_cordic_mode(mode: int) -> None:
    """rac_torch_bind.cpp:216-219: unknown modes fall back to FAST."""
    global _mode
    _mode = mode if mode in (MODE_FAST, MODE_CORDIC, MODE_SHIFTADD) else MODE_FAST


def get_cordic_mode() -> int:
    return _mode


def _resolve(iters: int, mode: int) -> tuple[int, int]:
    it = _iters if iters <= 0 else max(1, min(24, int(iters)))
    md = _mode if mode < 0 else int(mode)
    return it, md


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("librac_b200 runs on CUDA tensors only (no CPU path)")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.float32 else t.float()


def _ptr(t):
    return None if t is None else t.data_ptr()


def gemm(A: torch.Tensor, B: torch.Tensor, layout: int = LAYOUT_NN, iters: int = 0,
         mode: int = -1, bias: torch.Tensor | None = None, act: int = ACT_NONE,
         residual: torch.Tensor | None = None, alpha: float = 1.0, beta: float | None = None,
         out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """C = act(alpha * op(A) op(B) + beta * residual + bias) for 2-D fp32 CUDA tensors.

    layout NN: A[M,K] B[K,N]; NT: A[M,K] B[N,K]; TN: A[K,M] B[K,N].
    Inner (last) dims must be contiguous; leading dims may be strided."""
    _need_cuda(A, B, bias, residual)
    it, md = _resolve(iters, mode)
    A, B = _f32(A), _f32(B)
    if A.dim() != 2 or B.dim() != 2:
        raise ValueError("gemm: 2-D operands required")
    if A.stride(1) != 1:
        A = A.contiguous()
    if B.stride(1) != 1:
        B = B.contiguous()
    if layout == LAYOUT_TN:
        K, M = A.shape
    else:
        M, K = A.shape
    N = B.shape[0] if layout == LAYOUT_NT else B.shape[1]
    Kb = B.shape[1] if layout == LAYOUT_NT else B.shape[0]
    if Kb != K:
        raise ValueError(f"gemm: inner dimensions differ ({K} vs {Kb})")
    if act == ACT_SWIGLU:
        if N % 2 or residual is not None or (beta or 0.0) != 0.0:
            raise ValueError("gemm: SwiGLU needs an even N and no residual")
    if out is None:
        out = torch.empty((M, N // 2 if act == ACT_SWIGLU else N), device=A.device,
                          dtype=torch.float32)
    if residual is not None:
        residual = _f32(residual)
        if residual.stride(-1) != 1:
            residual = residual.contiguous()
        b = 1.0 if beta is None else float(beta)
    else:
        b = 0.0 if beta is None else float(beta)
        if b != 0.0:
            residual = out
    if bias is not None:
        bias = _f32(bias).contiguous()
        if bias.numel() == 0:
            bias = None
    if M == 0 or N == 0:
        return out
    if K == 0:
        return out.zero_() if residual is None else out.copy_(residual).mul_(b)
    with torch.cuda.device(A.device):
        _lib.call("rac_gemm_async", _ptr(A), A.stride(0), _ptr(B), B.stride(0), _ptr(out),
                  out.stride(0), _ptr(residual), residual.stride(0) if residual is not None else 0,
                  _ptr(bias), M, N, K, layout, md, it, float(alpha), b, act, variant, _stream(A))
    return out


# ── rac_cuda_ext surface ───────────────────────────────────────────────────

def matmul_forward(A: torch.Tensor, B: torch.Tensor, iters: int = 0, mode: int = -1) -> torch.Tensor:
    """rac_torch_bind.cpp:61-88: C = A @ B (NN)."""
    if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[0]:
        raise ValueError("RAC: 2D tensors with matching inner dimension required")
    dt = A.dtype
    C = gemm(A.contiguous(), B.contiguous(), LAYOUT_NN, iters, mode)
    return C if dt == torch.float32 else C.to(dt)


def matmul_backward(grad_C, A, B, need_grad_A=True, need_grad_B=True, iters=0, mode=-1):
    """rac_torch_bind.cpp:130-162: dA = dC @ B^T (NT), dB = A^T @ dC (TN)."""
    gC, A_, B_ = _f32(grad_C).contiguous(), _f32(A).contiguous(), _f32(B).contiguous()
    gA = gemm(gC, B_, LAYOUT_NT, iters, mode) if need_grad_A else None
    gB = gemm(A_, gC, LAYOUT_TN, iters, mode) if need_grad_B else None
    if gA is not None and A.dtype != torch.float32:
        gA = gA.to(A.dtype)
    if gB is not None and B.dtype != torch.float32:
        gB = gB.to(B.dtype)
    return [gA, gB]


def linear_forward(input, weight, bias, iters=0, mode=-1, act: int = ACT_NONE,
                   residual: torch.Tensor | None = None):
    """rac_torch_bind.cpp:90-128: out = input @ weight^T + bias (NT), bias and an
    optional activation / residual add fused into the GEMM epilogue."""
    dt = input.dtype
    shape = list(input.shape)
    x2 = input.reshape(-1, weight.shape[1])
    r2 = residual.reshape(-1, weight.shape[0]) if residual is not None else None
    out = gemm(x2, weight, LAYOUT_NT, iters, mode,
               bias=bias if (bias is not None and bias.numel() > 0) else None,
               act=act, residual=r2)
    shape[-1] = weight.shape[0] // 2 if act == ACT_SWIGLU else weight.shape[0]
    out = out.reshape(shape)
    return out if dt == torch.float32 else out.to(dt)


def linear_backward(grad_output, input, weight, need_bias_grad, iters=0, mode=-1):
    """rac_torch_bind.cpp:164-199: grad_input (NN), grad_weight (TN), grad_bias."""
    out_f, in_f = weight.shape
    go = _f32(grad_output).reshape(-1, out_f).contiguous()
    inp = _f32(input).reshape(-1, in_f).contiguous()
    gi = gemm(go, _f32(weight).contiguous(), LAYOUT_NN, iters, mode)
    gw = gemm(go, inp, LAYOUT_TN, iters, mode)
    gb = go.sum(0) if need_bias_grad else None
    return [gi.reshape(list(input.shape[:-1]) + [in_f]), gw, gb]


def fused_linear_forward(input, weight, bias, act, iters=0, mode=-1):
    """rac_torch.cu:1037-1086: act(input @ weight^T + bias) in one kernel."""
    return linear_forward(input, weight, bias, iters, mode, act=int(act))


def act_grad(pre_act: torch.Tensor, act: int) -> torch.Tensor:
    """Derivative of the activation at pre_act (rac_torch.cu:680-697)."""
    x = pre_act.float()
    if act == ACT_RELU:
        return (x > 0).float()
    if act == ACT_GELU:
        cdf = 0.5 * (1.0 + torch.erf(x * 0.7071067811865))
        pdf = 0.3989422804 * torch.exp(-0.5 * x * x)
        return cdf + x * pdf
    if act == ACT_SILU:
        sig = torch.sigmoid(x)
        return sig * (1.0 + x * (1.0 - sig))
    return torch.ones_like(x)


def fused_linear_backward(grad_output, input, weight, bias, pre_act, act, has_bias,
                          iters=0, mode=-1):
    """rac_torch.cu:1093-1177: gradient through act, then the linear backward."""
    d = _f32(grad_output) * act_grad(pre_act, int(act))
    gi, gw, gb = linear_backward(d, input, weight, bool(has_bias), iters, mode)
    return [gi, gw, gb]


# ── elementwise and row-wise kernels on tensors ───────────────────────────

def _prep(t: torch.Tensor) -> torch.Tensor:
    _need_cuda(t)
    if t.dtype != torch.float32:
        raise ValueError("float32 tensor required")
    return t.contiguous()


def rotate_batch(v: torch.Tensor, theta: torch.Tensor, iters: int | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """v[..., 2] rotated by theta[...]: rac_rotate_batch (iters None: literal
    RAC_K_INV, 16 iterations, lib/c/rac_cpu.c:136-139) or rac_rotate_n."""
    v, theta = _prep(v), _prep(theta)
    if v.shape[-1] != 2 or v.numel() != 2 * theta.numel():
        raise ValueError("v must be [..., 2] with one angle per vector")
    out = torch.empty_like(v) if out is None else out
    lit = 1 if iters is None else 0
    with torch.cuda.device(v.device):
        _lib.call("rac_rotate_batch_async", v.data_ptr(), theta.data_ptr(), out.data_ptr(),
                  theta.numel(), 16 if iters is None else int(iters), lit, _stream(v))
    return out


def project_batch(v: torch.Tensor, theta: torch.Tensor, iters: int = 16) -> torch.Tensor:
    """rac_project_n per element (lib/c/rac_cpu.c:282-288)."""
    v, theta = _prep(v), _prep(theta)
    if v.shape[-1] != 2 or v.numel() != 2 * theta.numel():
        raise ValueError("v must be [..., 2] with one angle per vector")
    out = torch.empty_like(theta)
    with torch.cuda.device(v.device):
        _lib.call("rac_project_batch_async", v.data_ptr(), theta.data_ptr(), out.data_ptr(),
                  theta.numel(), int(iters), _stream(v))
    return out


def sincos(theta: torch.Tensor):
    """rac_sincos per element: (sin, cos)."""
    theta = _prep(theta)
    s, c = torch.empty_like(theta), torch.empty_like(theta)
    with torch.cuda.device(theta.device):
        _lib.call("rac_sincos_batch_async", theta.data_ptr(), s.data_ptr(), c.data_ptr(),
                  theta.numel(), _stream(theta))
    return s, c


def _unary(x: torch.Tensor, op: int) -> torch.Tensor:
    x = _prep(x)
    y = torch.empty_like(x)
    with torch.cuda.device(x.device):
        _lib.call("rac_unary_async", x.data_ptr(), y.data_ptr(), x.numel(), op, _stream(x))
    return y


def exp(x):
    return _unary(x, _lib.UNARY_EXP)


def tanh(x):
    return _unary(x, _lib.UNARY_TANH)


def rsqrt(x):
    return _unary(x, _lib.UNARY_RSQRT)


def sigmoid(x):
    return _unary(x, _lib.UNARY_SIGMOID)


def softmax(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Row softmax over the last dim (lib/c/rac_cpu.c:258-271)."""
    x = _prep(x)
    y = torch.empty_like(x) if out is None else out
    d = x.shape[-1]
    with torch.cuda.device(x.device):
        _lib.call("rac_softmax_async", x.data_ptr(), y.data_ptr(), x.numel() // max(d, 1), d,
                  _stream(x))
    return y


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor | None = None, eps: float = 1e-6,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """lib/c/rac_cpu.c:548-574 over the last dim."""
    x = _prep(x)
    g = _prep(gamma) if gamma is not None else None
    y = torch.empty_like(x) if out is None else out
    d = x.shape[-1]
    with torch.cuda.device(x.device):
        _lib.call("rac_rmsnorm_async", x.data_ptr(), y.data_ptr(), _ptr(g), float(eps),
                  x.numel() // max(d, 1), d, _stream(x))
    return y


def layernorm(x, gamma=None, beta=None, eps: float = 1e-5,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """lib/c/rac_cpu.c:507-546 over the last dim."""
    x = _prep(x)
    g = _prep(gamma) if gamma is not None else None
    b = _prep(beta) if beta is not None else None
    y = torch.empty_like(x) if out is None else out
    d = x.shape[-1]
    with torch.cuda.device(x.device):
        _lib.call("rac_layernorm_async", x.data_ptr(), y.data_ptr(), _ptr(g), _ptr(b), float(eps),
                  x.numel() // max(d, 1), d, _stream(x))
    return y


def rope_cache(max_seq: int, head_dim: int, base: float = 10000.0, device="cuda"):
    """rac_rope_cache (lib/c/rac_cpu.c:576-598): (cos, sin) [max_seq, head_dim/2]."""
    c = torch.empty((max_seq, head_dim // 2), device=device, dtype=torch.float32)
    s = torch.empty_like(c)
    with torch.cuda.device(c.device):
        _lib.call("rac_rope_cache_async", c.data_ptr(), s.data_ptr(), max_seq, head_dim,
                  float(base), _stream(c))
    return c, s


def rope_apply_(x: torch.Tensor, cos_tab: torch.Tensor, sin_tab: torch.Tensor,
                positions: torch.Tensor | None = None, form: int = 0) -> torch.Tensor:
    """In place on contiguous x[..., seq, head_dim]. form 0 = lib/c fmaf form,
    1 = torch RACRoPE form.  positions: optional int index per seq row."""
    _need_cuda(x)
    if not x.is_contiguous() or x.dtype != torch.float32:
        raise ValueError("rope_apply_ needs a contiguous float32 tensor")
    seq, hd = x.shape[-2], x.shape[-1]
    ct, st = _prep(cos_tab), _prep(sin_tab)
    pos = positions.to(device=x.device, dtype=torch.int32).contiguous() if positions is not None else None
    with torch.cuda.device(x.device):
        _lib.call("rac_rope_apply_async", x.data_ptr(), ct.data_ptr(), st.data_ptr(), _ptr(pos),
                  x.numel() // (seq * hd), seq, hd, int(form), _stream(x))
    return x


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None = None,
              is_causal: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused softmax(q k^T / sqrt(hd) + mask) v on [B, H, S, hd] (rac_attention)."""
    q, k, v = _prep(q), _prep(k), _prep(v)
    m = _prep(mask) if mask is not None else None
    if m is not None and m.shape != (q.shape[-2], q.shape[-2]):
        raise ValueError("attention mask must be [seq, seq]")
    o = torch.empty_like(q) if out is None else out
    b, h, s_, hd = q.shape
    with torch.cuda.device(q.device):
        _lib.call("rac_attention_async", q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(m),
                  int(bool(is_causal)), o.data_ptr(), b, h, s_, hd, _stream(q))
    return o


def check_device_errors(device=None) -> None:
    """Synchronises the current stream and raises if a bounded device loop gave up."""
    dev = torch.device("cuda") if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().rac_check_device_errors(torch.cuda.current_stream().cuda_stream))
