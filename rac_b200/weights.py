"""Real weights for RACLlamaBlock: a safetensors reader and the Llama-layer mapping.

The reference reads TinyLlama-shaped checkpoints with its own C safetensors
reader (bench/safetensors_reader.c: F32 / F16 / BF16 tensors, header =
8-byte little-endian length + JSON {name: {dtype, shape, data_offsets}}) and
maps `model.layers.L.*` tensors into its CPU decoder
(bench/bench_rac_transformer.c:170-190, 660-677).  This module does the same for
RACLlamaBlock(gated=True):

* q/k/v/o_proj -> attn.qkv (concatenated) and attn.out_proj;
* grouped-query K/V heads (n_kv_heads < n_heads) are repeated per query
  head, as the reference decoder does (bench_rac_transformer.c:402-427);
* q/k rows are permuted from the rotate-half RoPE layout of HF checkpoints to
  the interleaved pairs (x[2i], x[2i+1]) that RACRoPE rotates
  (rac_torch/rac_torch.py:1165-1181), so the block computes the checkpoint's
  own attention (the reference's C decoder applies no RoPE at all);
* gate/up/down_proj -> ffn.gate / ffn.up / ffn.down; input_layernorm and
  post_attention_layernorm -> norm1 / norm2.
"""
from __future__ import annotations

import json
import struct

import numpy as np
import torch

from .rac_torch import RACLlamaBlock

_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16}


def read_safetensors(path: str, names=None) -> dict[str, np.ndarray]:
    """{name: float32 array} for the F32 / F16 / BF16 tensors of a file
    (all of them, or only `names`)."""
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hlen))
        base = 8 + hlen
        out = {}
        for name, meta in header.items():
            if name == "__metadata__" or (names is not None and name not in names):
                continue
            dt = meta["dtype"]
            if dt not in _DTYPES:
                raise ValueError(f"{name}: unsupported dtype {dt}")
            start, end = meta["data_offsets"]
            f.seek(base + start)
            raw = np.frombuffer(f.read(end - start), dtype=_DTYPES[dt])
            if dt == "BF16":
                arr = (raw.astype(np.uint32) << 16).view(np.float32)
            else:
                arr = raw.astype(np.float32)
            out[name] = arr.reshape(meta["shape"])
    return out


def write_safetensors(path: str, tensors: dict[str, np.ndarray], dtype: str = "F32") -> None:
    """Writes float tensors as F32, F16 or BF16 (BF16: round to nearest even)."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr, dtype=np.float32)
        if dtype == "F32":
            b = a.tobytes()
        elif dtype == "F16":
            with np.errstate(over="ignore"):    # beyond the F16 range: inf, as IEEE rounding gives
                b = a.astype(np.float16).tobytes()
        elif dtype == "BF16":
            u = a.view(np.uint32).astype(np.uint64)
            u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
            b = u.astype(np.uint16).tobytes()
        else:
            raise ValueError(dtype)
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def rotate_half_to_interleaved(w: torch.Tensor, n_heads: int) -> torch.Tensor:
    """Rows of a q/k projection from the rotate-half RoPE layout (dims i and
    i + hd/2 form a pair) to the interleaved layout (dims 2i and 2i+1)."""
    out_f, in_f = w.shape
    hd = out_f // n_heads
    return w.reshape(n_heads, 2, hd // 2, in_f).transpose(1, 2).reshape(out_f, in_f)


def load_llama_layer(tensors_or_path, layer: int, n_heads: int, n_kv_heads: int | None = None,
                     rms_eps: float = 1e-5, rope_base: float = 10000.0, max_seq_len: int = 2048,
                     hf_rope: bool = True, prefix: str = "model.layers", device="cuda") -> RACLlamaBlock:
    """RACLlamaBlock(gated=True) holding layer `layer` of a Llama checkpoint."""
    p = f"{prefix}.{layer}."
    keys = ["self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
            "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
            "mlp.down_proj.weight", "input_layernorm.weight", "post_attention_layernorm.weight"]
    if isinstance(tensors_or_path, str):
        t = read_safetensors(tensors_or_path, {p + k for k in keys})
    else:
        t = tensors_or_path
    missing = [p + k for k in keys if p + k not in t]
    if missing:
        raise KeyError(f"missing tensors: {missing}")
    g = {k: torch.from_numpy(np.ascontiguousarray(t[p + k], dtype=np.float32)) for k in keys}
    wq, wk, wv = g["self_attn.q_proj.weight"], g["self_attn.k_proj.weight"], g["self_attn.v_proj.weight"]
    d = wq.shape[1]
    if d % n_heads:
        raise ValueError(f"d_model {d} is not a multiple of n_heads {n_heads}")
    hd = d // n_heads
    n_kv = n_kv_heads or wk.shape[0] // hd      # default: read off k_proj's rows
    if n_kv < 1 or n_heads % n_kv:
        raise ValueError("n_heads must be a multiple of n_kv_heads")
    ff = g["mlp.gate_proj.weight"].shape[0]
    want = {"self_attn.q_proj.weight": (d, d), "self_attn.k_proj.weight": (n_kv * hd, d),
            "self_attn.v_proj.weight": (n_kv * hd, d), "self_attn.o_proj.weight": (d, d),
            "mlp.gate_proj.weight": (ff, d), "mlp.up_proj.weight": (ff, d),
            "mlp.down_proj.weight": (d, ff), "input_layernorm.weight": (d,),
            "post_attention_layernorm.weight": (d,)}
    for k, shp in want.items():
        if tuple(g[k].shape) != shp:
            raise ValueError(f"{p + k}: shape {tuple(g[k].shape)}, expected {shp}")
    if hf_rope:
        wq = rotate_half_to_interleaved(wq, n_heads)
        wk = rotate_half_to_interleaved(wk, n_kv)
    rep = n_heads // n_kv
    # K/V head j serves query heads j*rep .. j*rep+rep-1.
    wk = wk.reshape(n_kv, hd, d).repeat_interleave(rep, dim=0).reshape(n_heads * hd, d)
    wv = wv.reshape(n_kv, hd, d).repeat_interleave(rep, dim=0).reshape(n_heads * hd, d)
    blk = RACLlamaBlock(d, n_heads, ff_dim=ff, max_seq_len=max_seq_len, bias=False,
                        rms_eps=rms_eps, rope_base=rope_base, gated=True)
    with torch.no_grad():
        blk.attn.qkv.weight.copy_(torch.cat([wq, wk, wv], 0))
        blk.attn.out_proj.weight.copy_(g["self_attn.o_proj.weight"])
        blk.ffn.gate.weight.copy_(g["mlp.gate_proj.weight"])
        blk.ffn.up.weight.copy_(g["mlp.up_proj.weight"])
        blk.ffn.down.weight.copy_(g["mlp.down_proj.weight"])
        blk.norm1.weight.copy_(g["input_layernorm.weight"])
        blk.norm2.weight.copy_(g["post_attention_layernorm.weight"])
    return blk.to(device)
