"""Real-weight loading: safetensors reader/writer and the Llama-layer mapping.

The reference decoder reads F32 / F16 / BF16 safetensors
(bench/safetensors_reader.c) and loads `model.layers.L.*` by the HF Llama
names (bench/bench_rac_transformer.c:182-190).  The mapping is pinned
against transformers' own LlamaDecoderLayer (rotate-half RoPE, grouped-query
K/V): the CPU tests check the loaded block's parameters in plain torch fp32,
the GPU test runs the block on this library's kernels.
"""
import numpy as np
import pytest
import torch

from rac_b200 import weights as W


def _hf_layer(d=128, heads=4, kv=2, ff=192, seed=0):
    tr = pytest.importorskip("transformers")
    from transformers.models.llama.modeling_llama import LlamaDecoderLayer, LlamaRotaryEmbedding
    cfg = tr.LlamaConfig(hidden_size=d, intermediate_size=ff, num_attention_heads=heads,
                         num_key_value_heads=kv, rms_norm_eps=1e-5, max_position_embeddings=64,
                         attn_implementation="eager")
    torch.manual_seed(seed)
    layer = LlamaDecoderLayer(cfg, 0).eval()
    with torch.no_grad():
        for p in layer.parameters():
            p.copy_(torch.randn_like(p) * (0.08 if p.dim() == 2 else 0.3) + (1.0 if p.dim() == 1 else 0.0))
    return cfg, layer, LlamaRotaryEmbedding(cfg)


def _hf_forward(layer, rot, x):
    B, T, _ = x.shape
    pos = torch.arange(T)[None].expand(B, T)
    mask = torch.full((T, T), float("-inf")).triu(1)[None, None].expand(B, 1, T, T)
    with torch.no_grad():
        return layer(x, attention_mask=mask, position_embeddings=rot(x, pos), position_ids=pos)


def _plain_block(blk, x):
    """The loaded block's math in plain torch fp32 (the oracle restatement)."""
    from oracle import torch_block as TB
    return TB.block_forward(TB.params_of(blk), x, blk.attn.n_heads, eps=blk.norm1.eps,
                            cos=blk.attn.rope.cos_cache, sin=blk.attn.rope.sin_cache)


def test_safetensors_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    t = {"a": rng.standard_normal((3, 5)).astype(np.float32),
         "b.c": rng.standard_normal(7).astype(np.float32) * 1e3,
         "empty": np.zeros((0, 4), np.float32)}
    for dt in ("F32", "F16", "BF16"):
        path = str(tmp_path / f"t_{dt}.safetensors")
        W.write_safetensors(path, t, dtype=dt)
        got = W.read_safetensors(path)
        assert set(got) == set(t)
        for k, v in t.items():
            if dt == "F32":
                want = v
            elif dt == "F16":
                want = v.astype(np.float16).astype(np.float32)
            else:
                want = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
            assert got[k].dtype == np.float32 and got[k].shape == v.shape
            assert np.array_equal(got[k], want), (dt, k)
    sub = W.read_safetensors(str(tmp_path / "t_F32.safetensors"), names={"a"})
    assert list(sub) == ["a"]


def test_safetensors_rejects_other_dtypes(tmp_path):
    import json
    import struct
    path = tmp_path / "i.safetensors"
    h = json.dumps({"__metadata__": {"format": "pt"},
                    "x": {"dtype": "I32", "shape": [2], "data_offsets": [0, 8]}}).encode()
    path.write_bytes(struct.pack("<Q", len(h)) + h + bytes(8))
    with pytest.raises(ValueError, match="unsupported dtype I32"):
        W.read_safetensors(str(path))


def test_rotate_half_permutation():
    w = torch.arange(2 * 8, dtype=torch.float32).reshape(8, 2)     # 1 head, hd 8
    p = W.rotate_half_to_interleaved(w, 1)
    # interleaved pair i = (rotate-half dims i, i + hd/2)
    assert p[:, 0].tolist() == [0, 8, 2, 10, 4, 12, 6, 14]


@pytest.mark.parametrize("dtype", ["F32", "BF16"])
def test_llama_layer_mapping_matches_transformers(tmp_path, dtype):
    cfg, layer, rot = _hf_layer()
    sd = {f"model.layers.3.{k}": v.numpy() for k, v in layer.state_dict().items()}
    path = str(tmp_path / "layer.safetensors")
    W.write_safetensors(path, sd, dtype=dtype)
    if dtype == "BF16":       # compare against the checkpoint as stored
        with torch.no_grad():
            for p in layer.parameters():
                p.copy_(p.to(torch.bfloat16).float())
    blk = W.load_llama_layer(path, 3, n_heads=4, rms_eps=1e-5, max_seq_len=64, device="cpu")
    assert blk.gated and blk.attn.qkv.weight.shape == (3 * 128, 128)
    x = torch.randn(2, 9, 128)
    with torch.no_grad():
        y = _plain_block(blk, x)
    assert (y - _hf_forward(layer, rot, x)).abs().max() < 2e-5


def test_llama_layer_errors(tmp_path):
    cfg, layer, _ = _hf_layer()
    sd = {f"model.layers.0.{k}": v.numpy() for k, v in layer.state_dict().items()}
    with pytest.raises(KeyError, match="missing tensors"):
        W.load_llama_layer(sd, 1, n_heads=4, device="cpu")
    with pytest.raises(ValueError, match="multiple of n_kv_heads"):
        W.load_llama_layer(sd, 0, n_heads=4, n_kv_heads=3, device="cpu")
    bad = dict(sd)
    bad["model.layers.0.mlp.down_proj.weight"] = np.zeros((128, 100), np.float32)
    with pytest.raises(ValueError, match="down_proj.weight: shape"):
        W.load_llama_layer(bad, 0, n_heads=4, device="cpu")


@pytest.mark.gpu
@pytest.mark.parametrize("mode,tol", [("fast", 1e-4), ("cordic", 2e-3)])
def test_llama_layer_on_gpu_matches_transformers(tmp_path, cuda, mode, tol):
    from rac_b200 import rac_torch as R
    cfg, layer, rot = _hf_layer()
    sd = {f"model.layers.0.{k}": v.numpy() for k, v in layer.state_dict().items()}
    path = str(tmp_path / "layer.safetensors")
    W.write_safetensors(path, sd)
    blk = W.load_llama_layer(path, 0, n_heads=4, n_kv_heads=2, rms_eps=1e-5, max_seq_len=64,
                             device=cuda)
    x = torch.randn(2, 33, 128)
    want = _hf_forward(layer, rot, x)
    R.rac_set_mode(mode)
    R.rac_set_precision(24 if mode == "fast" else 16)
    try:
        with torch.no_grad():
            y = blk(x.to(cuda), is_causal=True).cpu()        # fused attention + residual epilogues
        y_g = blk(x.to(cuda), is_causal=True).detach().cpu()  # autograd path
    finally:
        R.rac_set_mode("fast")
        R.rac_set_precision(24)
    scale = want.abs().max().item()
    assert (y - want).abs().max().item() < tol * scale
    assert (y_g - want).abs().max().item() < tol * scale


@pytest.mark.skipif(not __import__("oracle").st_available(),
                    reason="oracle/_ref/libst_ref.so not built (no reference checkout)")
@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
def test_reader_equals_reference_reader(tmp_path, dtype):
    """rac_b200.weights.read_safetensors against the reference decoder bench's own
    reader (bench/safetensors_reader.c, compiled from the reference checkout by
    oracle/Makefile): same names, shapes and float32 bits for every tensor, F32 /
    F16 / BF16, on random values plus zeros, signed zeros, subnormal and
    out-of-range magnitudes, infinities and NaN; and a Llama layer loaded from
    the reference reader's tensors equals the one loaded from ours."""
    import oracle as O
    rng = np.random.default_rng(len(dtype))
    edge = np.array([0.0, -0.0, 1.0, -1.0, 1e-6, -3e-8, 6e-5, 65504.0, 1e5, -1e-40,
                     3e38, np.inf, -np.inf, np.nan, 0.333333], np.float32)
    tensors = {"edge": edge, "vec": rng.standard_normal(37).astype(np.float32),
               "mat": (rng.standard_normal((16, 24)) * 0.05).astype(np.float32)}
    cfg, layer, _ = _hf_layer()
    prefix = "model.layers.0."
    for name, p in layer.state_dict().items():
        tensors[prefix + name] = p.numpy()
    path = str(tmp_path / f"w_{dtype}.safetensors")
    W.write_safetensors(path, tensors, dtype)
    ours = W.read_safetensors(path)
    theirs = O.ref_read_safetensors(path)
    assert sorted(ours) == sorted(theirs)
    for k in ours:
        a, b = ours[k], theirs[k]
        assert a.shape == b.shape, k
        same = (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))
        assert same.all(), (k, a[~same][:4], b[~same][:4])
    blk_a = W.load_llama_layer(ours, 0, cfg.num_attention_heads, cfg.num_key_value_heads, device="cpu")
    blk_b = W.load_llama_layer(theirs, 0, cfg.num_attention_heads, cfg.num_key_value_heads, device="cpu")
    for (na, pa), (nb, pb) in zip(blk_a.state_dict().items(), blk_b.state_dict().items()):
        assert na == nb and torch.equal(pa, pb), na
