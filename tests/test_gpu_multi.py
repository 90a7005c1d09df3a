"""Two-rank (NCCL) checks of the multi-GPU layouts; skipped with fewer than 2 GPUs.

* N-column sharded rac_matmul: each rank's columns equal the single-GPU
  result bit for bit (the per-output arithmetic is unchanged).
* TPLlamaBlock at world 2 equals the unsharded block (CORDIC 16 and FAST)
  within normwise 1e-4 (the all-reduce changes the summation order), and its
  overlapped two-piece forward equals the one-piece forward bit for bit.
"""
import math
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from rac_b200 import ext, tp
    from rac_b200 import rac_torch as R
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        g = torch.Generator(device="cpu").manual_seed(0)
        A = (torch.rand((512, 1024), generator=g) * 2 - 1).to(dev)
        B = (torch.rand((1024, 768), generator=g) * 2 - 1).to(dev)
        n0, n1 = tp.column_shard(768, world, rank)
        C_loc = tp.sharded_matmul(A, B[:, n0:n1].contiguous(), 16, 1)
        C_full = tp.gather_columns(C_loc, world)
        ref = ext.gemm(A, B, ext.LAYOUT_NN, 16, 1)
        ok_mm = bool(torch.equal(C_full, ref))
        R.rac_set_mode("cordic")
        R.rac_set_precision(16)
        full = tp.make_block(256, 8, 688, 128, True, dev, seed=1)
        x = torch.randn((2, 64, 256), generator=g).to(dev)
        with torch.no_grad():
            y_ref = full(x, is_causal=True)
            blk = tp.TPLlamaBlock(full, world, rank)
            y_tp = blk(x, chunks=2)                         # two batch pieces, overlapped
            y_one = blk(x)
            R.rac_set_mode("fast")
            y_ref_f = full(x, is_causal=True)
            y_tp_f = blk(x)
        err = float((y_tp - y_ref).abs().max() / y_ref.pow(2).mean().sqrt())
        err_f = float((y_tp_f - y_ref_f).abs().max() / y_ref_f.pow(2).mean().sqrt())
        q.put((rank, ok_mm, err, bool(torch.equal(y_tp, y_one)), err_f))
    finally:
        dist.destroy_process_group()


def test_two_rank_matmul_and_tp_block():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=120)
    for rank, ok_mm, err, same_pieces, err_f in res:
        assert ok_mm, rank
        assert err <= 1e-4, (rank, err)
        assert err_f <= 1e-4, (rank, err_f)       # FAST mode: NN on the shards' cached W^T
        assert same_pieces, rank                  # batch pieces: the bits of one piece
