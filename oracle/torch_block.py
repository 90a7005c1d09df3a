"""Plain torch (CPU, fp32) restatement of the reference RACLlamaBlock -- TEST
INFRASTRUCTURE ONLY (a checker and the timed CPU baseline, never the product).

Off the GPU the reference module computes every RAC op with torch's own FMA
arithmetic (rac_torch/rac_torch.py:183 and :232 fall back to torch.matmul /
F.linear), so its CPU path is:

* RMSNorm  y = x * rsqrt(mean(x^2) + eps) * weight   (rac_torch.py:1205-1231)
* qkv = x Wqkv^T, heads split, RoPE on interleaved pairs (x[2i], x[2i+1])
  with the torch cos/sin cache                         (rac_torch.py:1132-1181)
* softmax(Q K^T * hd^-0.5 + causal mask) V, out_proj   (rac_torch.py:1279-1343)
* x + attn(RMS(x)); h + ffn(RMS(h))                   (rac_torch.py:1348-1383)
* FFN: fc2(act(fc1 x)) (RACFusedFFN, rac_torch.py:631-655), or the gated
  form down(silu(gate x) * up x), the SwiGLU of
  bench/bench_rac_transformer.c:441-453.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rope_cache(head_dim: int, max_seq: int, base: float = 10000.0):
    half = head_dim // 2
    inv_freq = 1.0 / (base ** (torch.arange(0, half, dtype=torch.float32) * 2 / head_dim))
    ang = torch.arange(max_seq, dtype=torch.float32).unsqueeze(1) * inv_freq.unsqueeze(0)
    return ang.cos(), ang.sin()


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(t, c, s):
    t1, t2 = t[..., 0::2], t[..., 1::2]
    out = torch.empty_like(t)
    out[..., 0::2] = t1 * c - t2 * s
    out[..., 1::2] = t1 * s + t2 * c
    return out


def block_forward(p: dict, x: torch.Tensor, n_heads: int, eps: float = 1e-6,
                  cos=None, sin=None, causal: bool = True, operand=None) -> torch.Tensor:
    """p: {"norm1", "qkv", "out", "norm2"} plus {"gate", "up", "down"} (gated)
    or {"fc1", "fc2"} (SiLU FFN): fp32 tensors, weights [out, in].  x [B, T, d].

    operand: a function applied to the activation operand of each of the four
    projections before its product with the weight (None: identity).  With
    oracle.cordic_operand it turns every projection into the CORDIC-mode GEMM
    (CORDIC(A, W) == FAST(r(A), W) bit for bit), while the attention core stays
    plain fp32 as in the reference module (rac_torch.py:1325-1337 uses
    torch.matmul there)."""
    op = operand or (lambda t: t)
    B, T, d = x.shape
    hd = d // n_heads
    if cos is None:
        cos, sin = rope_cache(hd, T)
    c, s = cos[:T], sin[:T]
    q, k, v = (op(_rms(x, p["norm1"], eps)) @ p["qkv"].T).chunk(3, -1)
    q, k, v = (t.reshape(B, T, n_heads, hd).transpose(1, 2) for t in (q, k, v))
    q, k = _rope(q, c, s), _rope(k, c, s)
    scores = torch.matmul(q, k.transpose(-2, -1)) * hd ** -0.5
    if causal:
        scores = scores + torch.full((T, T), float("-inf")).triu(1)
    o = torch.matmul(torch.softmax(scores, -1), v).transpose(1, 2).reshape(B, T, d)
    h = x + op(o) @ p["out"].T
    n = op(_rms(h, p["norm2"], eps))
    if "fc1" in p:
        return h + op(F.silu(n @ p["fc1"].T)) @ p["fc2"].T
    return h + op(F.silu(n @ p["gate"].T) * (n @ p["up"].T)) @ p["down"].T


def params_of(blk) -> dict:
    """The restatement's parameter dict from a RACLlamaBlock (gated or not)."""
    g = lambda t: t.detach().float().cpu()                      # noqa: E731
    p = {"norm1": g(blk.norm1.weight), "qkv": g(blk.attn.qkv.weight),
         "out": g(blk.attn.out_proj.weight), "norm2": g(blk.norm2.weight)}
    if hasattr(blk.ffn, "gate"):
        p.update(gate=g(blk.ffn.gate.weight), up=g(blk.ffn.up.weight), down=g(blk.ffn.down.weight))
    else:
        p.update(fc1=g(blk.ffn.fc1.weight), fc2=g(blk.ffn.fc2.weight))
    return p
