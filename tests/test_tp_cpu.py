"""Host-side logic of the multi-GPU layouts, on CPU with gloo ranks.

The kernels need a GPU; these tests check what does not: the column split,
the head/ff sharding of the Llama block (shard shapes and that concatenating
shards rebuilds the full weights), and the all-gather of column blocks with
world_size 2 over gloo.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from rac_b200 import tp


def test_column_shard_covers_exactly():
    for n in (1, 7, 4096, 11008):
        for w in (1, 2, 3, 4, 8):
            spans = [tp.column_shard(n, w, r) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("world", [1, 2, 4])
def test_tp_shards_rebuild_full_weights(gated, world):
    full = tp.make_block(64, 4, 160, 32, gated, "cpu", seed=3)
    shards = [tp.TPLlamaBlock(full, world, r) for r in range(world)]
    d, hl = 64, 4 // world
    q = torch.cat([s.attn.qkv.weight[: hl * 16] for s in shards], 0)
    assert torch.equal(q, full.attn.qkv.weight[:d])
    v = torch.cat([s.attn.qkv.weight[2 * hl * 16:] for s in shards], 0)
    assert torch.equal(v, full.attn.qkv.weight[2 * d:])
    o = torch.cat([s.attn.out_proj.weight for s in shards], 1)
    assert torch.equal(o, full.attn.out_proj.weight)
    if gated:
        gu = [s.w_gu.weight for s in shards]          # gate row c at 2c, up row c at 2c+1
        assert torch.equal(torch.cat([w[0::2] for w in gu], 0), full.ffn.gate.weight)
        assert torch.equal(torch.cat([w[1::2] for w in gu], 0), full.ffn.up.weight)
        assert torch.equal(torch.cat([s.w_down.weight for s in shards], 1), full.ffn.down.weight)
    else:
        assert torch.equal(torch.cat([s.w_fc1.weight for s in shards], 0), full.ffn.fc1.weight)
        assert torch.equal(torch.cat([s.w_fc2.weight for s in shards], 1), full.ffn.fc2.weight)


def test_tp_rejects_uneven_heads():
    full = tp.make_block(64, 4, 160, 32, True, "cpu")
    with pytest.raises(ValueError):
        tp.TPLlamaBlock(full, 3, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gather_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    n = 10
    n0, n1 = tp.column_shard(n, world, rank)
    full = torch.arange(3 * n, dtype=torch.float32).reshape(3, n)
    got = tp.gather_columns(full[:, n0:n1].contiguous(), world)
    q.put((rank, bool(torch.equal(got, full))))
    dist.destroy_process_group()


def test_gather_columns_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    assert all(ok for _, ok in res)


def _rank_failure_worker(rank, world, port, q):
    """Rank 1 raises before the collective; rank 0 must get an error, not hang."""
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "raised"))
        q.close()
        q.join_thread()
        os._exit(3)
    try:
        tp.gather_columns(torch.zeros(2, 2), world)
        q.put((rank, "no error"))
    except Exception:
        q.put((rank, "error"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_failed_rank_is_detected_on_host():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_failure_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "raised" and res[0] == "error"
