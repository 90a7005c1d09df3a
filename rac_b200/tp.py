"""Multi-GPU layouts of the RAC hot path (one process per GPU, torch.distributed).

* ``column_shard`` / ``sharded_matmul``: rac_matmul split by N-column blocks.
  A is replicated, rank r owns B[:, n0:n1] and C[:, n0:n1]; there is no
  exchange on the data path (the reference's MPI path splits M rows instead,
  lib/c/rac_mpi.c:52-112; N-columns also balances the M=16 skinny case).
  ``gather_columns`` is the optional NCCL all-gather of C.
* ``TPLlamaBlock``: RACLlamaBlock with Megatron-style tensor parallelism --
  qkv and the FFN up-projections split by output rows (whole heads / ff
  slices per rank), out_proj and the down-projection split by input columns,
  one NCCL all-reduce (sum, fp32) after each of the two row-split GEMMs.
  The batch can run in pieces, so each piece's all-reduce overlaps the next
  piece's GEMMs (off by default: at TP2 it did not pay).  The gated FFN's gate and up shards run as one GEMM over
  row-interleaved weights whose epilogue writes silu(gate) * up.
  Rank 0 adds the residual in its GEMM epilogue so the all-reduce yields
  x + sum of partials directly.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import ext
from .rac_torch import RACLlamaBlock, RACRoPEAttention, RACRMSNorm, _kw


def column_shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """[n0, n1) columns owned by `rank` (sizes differ by at most one)."""
    return n * rank // world, n * (rank + 1) // world


def sharded_matmul(A: torch.Tensor, B_local: torch.Tensor, iters: int = 16, mode: int = 1,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """This rank's C[:, n0:n1] = A @ B[:, n0:n1]; no communication."""
    return ext.gemm(A, B_local, ext.LAYOUT_NN, iters, mode, out=out)


def gather_columns(C_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather of the column blocks into the full C (equal block sizes)."""
    import torch.distributed as dist
    parts = [torch.empty_like(C_local) for _ in range(world)]
    dist.all_gather(parts, C_local.contiguous(), group=group)
    return torch.cat(parts, dim=1)


class TPLlamaBlock(nn.Module):
    """One rank's shard of an RACLlamaBlock (inference forward)."""

    def __init__(self, full: RACLlamaBlock, world: int, rank: int, group=None):
        super().__init__()
        a = full.attn
        H, hd, d = a.n_heads, a.d_head, a.d_model
        if H % world:
            raise ValueError(f"n_heads={H} not divisible by world={world}")
        self.world, self.rank, self.group = world, rank, group
        self.h_local = H // world
        h0, h1 = rank * self.h_local * hd, (rank + 1) * self.h_local * hd
        dev = a.qkv.weight.device
        self.norm1 = full.norm1
        self.norm2 = full.norm2
        self.attn = RACRoPEAttention(d, H, max_seq_len=a.rope.max_seq_len, bias=False,
                                     rope_base=a.rope.base, device=dev)
        self.attn.n_heads = self.h_local
        wq = a.qkv.weight.data
        with torch.no_grad():
            self.attn.qkv = _linear_from(torch.cat([wq[h0:h1], wq[d + h0:d + h1],
                                                    wq[2 * d + h0:2 * d + h1]], 0))
            self.attn.out_proj = _linear_from(a.out_proj.weight.data[:, h0:h1])
        self.gated = full.gated
        f = full.ffn
        if self.gated:
            ff = f.up.out_features
            f0, f1 = ff * rank // world, ff * (rank + 1) // world
            self.w_down = _linear_from(f.down.weight.data[:, f0:f1])
            # gate and up rows interleaved: one GEMM with the SwiGLU epilogue
            self.w_gu = _linear_from(interleave_rows(f.gate.weight.data[f0:f1],
                                                     f.up.weight.data[f0:f1]))
        else:
            ff = f.fc1.out_features
            f0, f1 = ff * rank // world, ff * (rank + 1) // world
            self.act_id = f.fc1.act_id
            self.w_fc1 = _linear_from(f.fc1.weight.data[f0:f1])
            self.w_fc2 = _linear_from(f.fc2.weight.data[:, f0:f1])

    def full_params(self) -> dict:
        """The block's weights as CPU fp32 tensors keyed norm1/qkv/out/norm2 and
        gate/up/down (or fc1/fc2) -- the whole block only when world == 1."""
        g = lambda t: t.detach().float().cpu()                  # noqa: E731
        p = {"norm1": g(self.norm1.weight), "qkv": g(self.attn.qkv.weight),
             "out": g(self.attn.out_proj.weight), "norm2": g(self.norm2.weight)}
        if self.gated:
            gu = g(self.w_gu.weight)
            p.update(gate=gu[0::2].contiguous(), up=gu[1::2].contiguous(), down=g(self.w_down.weight))
        else:
            p.update(fc1=g(self.w_fc1.weight), fc2=g(self.w_fc2.weight))
        return p

    def _allreduce(self, t, async_op: bool = False):
        if self.world > 1:
            import torch.distributed as dist
            return dist.all_reduce(t, group=self.group, async_op=async_op)
        return None

    def _attn_half(self, x, mask, is_causal, positions):
        res = x if self.rank == 0 else None
        ctx = self.attn._context(self.norm1(x), mask, is_causal, positions, n_heads=self.h_local)
        return _apply(ctx, self.attn.out_proj, residual=res)

    def _ffn_half(self, h):
        n2 = self.norm2(h)
        res = h if self.rank == 0 else None
        if self.gated:
            return _apply(_apply(n2, self.w_gu, act=ext.ACT_SWIGLU), self.w_down, residual=res)
        return _apply(_apply(n2, self.w_fc1, act=self.act_id), self.w_fc2, residual=res)

    @torch.no_grad()
    def forward(self, x, mask=None, is_causal=True, positions=None, chunks: int | None = None):
        """chunks: split the batch into this many pieces so that each piece's
        all-reduce runs on NCCL's stream while the next piece's GEMMs run (the
        sequences of a batch are independent; at world 2 the result is the same
        bits as one piece).  Default 1: at TP2 in FAST mode the two all-reduces
        cost ~1 % of the step and halving the GEMMs' M cost more (32.3 ms with
        2 pieces, 33.7 with 4, 31.9 with 1)."""
        B = x.shape[0]
        c = chunks if chunks is not None else 1
        c = max(1, min(c, B))
        if c == 1:
            h = self._attn_half(x, mask, is_causal, positions)
            self._allreduce(h)
            y = self._ffn_half(h)
            self._allreduce(y)
            return y
        hs, works = [], []
        for xc in x.chunk(c, dim=0):
            h = self._attn_half(xc, mask, is_causal, positions)
            works.append(self._allreduce(h, async_op=True))
            hs.append(h)
        ys, works2 = [], []
        for h, w in zip(hs, works):
            if w is not None:
                w.wait()                   # this stream waits for the reduced h
            y = self._ffn_half(h)
            works2.append(self._allreduce(y, async_op=True))
            ys.append(y)
        for w in works2:
            if w is not None:
                w.wait()
        return torch.cat(ys, 0)


class _ShardLinear(nn.Module):
    """A bias-free weight shard applied with the RAC GEMM (inference only).

    In FAST mode x W^T runs as an NN GEMM on a k-major copy W^T, which
    measured faster than the NT form on this GPU (4096^3: 3.05 against
    3.66 ms) and gives the same bits (each output still accumulates
    fma(x_k, w_k) over k in order).  The copy is derived state: it is rebuilt
    whenever the weight's storage or version counter changes (load_state_dict,
    an in-place edit, a reassigned .data), so it can never go stale, and it
    costs one more weight-sized buffer per shard while FAST mode is used."""

    def __init__(self, w: torch.Tensor):
        super().__init__()
        self.weight = nn.Parameter(w.contiguous().clone(), requires_grad=False)
        self.bias = None
        self._wt = None
        self._wt_key = None

    def weight_t(self) -> torch.Tensor:
        w = self.weight
        key = (w.data_ptr(), w._version, tuple(w.shape), w.device)
        if self._wt is None or self._wt_key != key:
            self._wt = w.detach().t().contiguous()
            self._wt_key = key
        return self._wt

    def forward(self, x):
        return _apply(x, self)


def _apply(x: torch.Tensor, lin: _ShardLinear, act: int = ext.ACT_NONE,
           residual: torch.Tensor | None = None) -> torch.Tensor:
    """act(x W^T + residual) for a shard: NN on W^T in FAST mode, else NT on W."""
    kw = _kw()
    if kw["mode"] != ext.MODE_FAST:
        return ext.linear_forward(x, lin.weight, None, act=act, residual=residual, **kw)
    out_f, in_f = lin.weight.shape
    shape = list(x.shape)
    r2 = residual.reshape(-1, out_f) if residual is not None else None
    out = ext.gemm(x.reshape(-1, in_f), lin.weight_t(), ext.LAYOUT_NN, kw["iters"], kw["mode"],
                   act=act, residual=r2)
    shape[-1] = out.shape[-1]
    return out.reshape(shape)


def interleave_rows(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[2F, d] with gate row c at 2c and up row c at 2c+1 (the SwiGLU GEMM's B)."""
    return torch.stack([gate, up], dim=1).reshape(2 * gate.shape[0], gate.shape[1]).contiguous()


def _linear_from(w: torch.Tensor) -> nn.Module:
    return _ShardLinear(w)


def make_block(d: int, H: int, ff: int, max_seq: int, gated: bool, device, seed: int = 0):
    """RACLlamaBlock with the benchmark's random init: weights ~N(0, 0.02),
    norm gains 1 (identical on every rank for a given seed)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    blk = RACLlamaBlock(d, H, ff_dim=ff, max_seq_len=max_seq, activation="silu", bias=False,
                        gated=gated, device="meta")
    blk = blk.to_empty(device=device)
    with torch.no_grad():
        for name, p in blk.named_parameters():
            if p.dim() > 1:
                p.copy_((torch.randn(p.shape, generator=g) * 0.02).to(device))
            else:
                p.fill_(1.0)
    # rebuild the RoPE caches (to_empty left them uninitialised)
    from .rac_torch import RACRoPE
    blk.attn.rope = RACRoPE(d // H, max_seq_len=max_seq, base=10000.0, device=device)
    return blk


def bench_llama(args, world, rank, local, barrier, max_over_ranks, ClockSampler) -> dict | None:
    """RACLlamaBlock tokens/s: d 4096, 32 heads, ff 11008 SwiGLU, x [4, 2048, 4096],
    CORDIC 16 iterations (or --mode fast), tensor-parallel over `world` ranks."""
    import statistics
    import time

    from . import rac_torch as R
    dev = torch.device("cuda", local)
    R.rac_set_mode("cordic" if args.mode == "cordic" else "fast")
    R.rac_set_precision(args.iters)
    d, H, ff, Bt, T = 4096, 32, 11008, 4, 2048
    if args.size != 4096:            # reduced shape for quick checks
        d, H, ff, Bt, T = args.size, max(1, args.size // 128), int(args.size * 2.6875), 2, 256
    full = make_block(d, H, ff, max(T, 64), True, dev)
    blk = TPLlamaBlock(full, world, rank)
    del full
    torch.cuda.empty_cache()
    g = torch.Generator(device=dev).manual_seed(99)
    x = torch.randn((Bt, T, d), device=dev, generator=g)
    chunks = getattr(args, "tp_chunks", None)
    for _ in range(args.warmup):
        blk(x, chunks=chunks)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    from . import _lib
    calls0 = _lib.CALLS["n"]
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            starts[i].record(s)
            y = blk(x, chunks=chunks)
            ends[i].record(s)
        torch.cuda.synchronize()
    launches = _lib.CALLS["n"] - calls0
    barrier(world)
    t_local = statistics.mean(a.elapsed_time(b) for a, b in zip(starts, ends))
    t = max_over_ranks(t_local, world)
    # e2e: pinned host input -> device, forward, result back to the host.  With
    # several ranks each uploads one 1/world slice of the token rows over its own
    # PCIe link, NCCL all-gathers the slices over NVLink, and each rank downloads
    # its slice of the (replicated) output: together they move x in and y out
    # once instead of once per rank.
    rows = Bt * T
    r0, r1 = rows * rank // world, rows * (rank + 1) // world
    even = rows % world == 0
    x2 = x.reshape(rows, d)
    xh = (x2[r0:r1] if (world > 1 and even) else x2).cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    xfull = torch.empty((rows, d), device=dev) if (world > 1 and even) else None
    ts = []
    for _ in range(max(1, min(args.steps, 3))):
        torch.cuda.synchronize()
        barrier(world)
        t0 = time.perf_counter()
        if xfull is not None:
            import torch.distributed as dist
            dist.all_gather_into_tensor(xfull, xh.to(dev, non_blocking=True))
            yd = blk(xfull.view(Bt, T, d), chunks=chunks).reshape(rows, d)[r0:r1]
        else:
            yd = blk(xh.to(dev, non_blocking=True).view(Bt, T, d), chunks=chunks).reshape(rows, d)
        yh.copy_(yd, non_blocking=True)
        torch.cuda.synchronize()
        ts.append(time.perf_counter() - t0)
    te = max_over_ranks(statistics.mean(ts), world)
    if rank != 0:
        return None
    sample = None
    if world == 1:       # batch 0, first 256 tokens: checked and timed on the CPU by bench.py
        ts_ = min(T, 256)
        sample = {"params": blk.full_params(), "x": x[:1, :ts_].cpu(), "y": y[:1, :ts_].cpu(),
                  "heads": H, "mode": args.mode, "iters": args.iters}
    tokens = Bt * T
    macs = tokens * (4 * d * d + 3 * d * ff) // world            # projections, per rank
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    mhz = 1965.0
    peak_mac = sms * 128 * mhz * 1e6 / (2 * args.iters + 2) if args.mode == "cordic" else sms * 128 * mhz * 1e6
    return {
        "metric": "RACLlamaBlock tokens/s", "value": tokens / (t * 1e-3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (random-init weights ~N(0,0.02))",
        "config": {"workload": f"RACLlamaBlock d={d} H={H} ff={ff} SwiGLU, x [{Bt},{T},{d}], causal, "
                               f"{args.mode} {args.iters if args.mode == 'cordic' else ''}",
                   "parallelism": f"tp{world}", "l2": "inputs and weights larger than L2",
                   "tp_batch_pieces": chunks if chunks is not None else 1},
        "roofline": {"bound": "fp32_issue", "achieved": macs / (t_local * 1e-3) / 1e12,
                     "peak": peak_mac / 1e12, "unit": "TMAC/s (projection GEMMs only)",
                     "frac": macs / (t_local * 1e-3) / peak_mac, "traffic": None},
        "e2e": {"value": tokens / te, "unit": "tokens/s", "h2d_bytes_per_step": 4 * x.numel(),
                "d2h_bytes_per_step": 4 * x.numel(),
                "note": "bytes summed over ranks: with N > 1 each rank uploads and downloads "
                        "1/N of the token rows; the input slices are all-gathered over NVLink"},
        "gpu_launches": launches,
        "gpu_launches_note": "librac_b200 entry-point calls in the timed region (projections, "
                             "fused attention, RMSNorm, RoPE)",
        "clocks": clk.summary(),
        "_sample": sample,
    }
