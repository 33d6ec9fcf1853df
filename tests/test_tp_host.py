"""Tensor-parallel host logic on CPU (gloo, world size 2): the NCCL group id
travels from rank 0 to every rank, and the ranks' shards of every sharded
tensor are disjoint and cover it (the geometry lmc_model_load_tp uses)."""
import os
import socket
import types

import torch.multiprocessing as mp

from lmc_b200 import tp

CFG = types.SimpleNamespace(n_heads=32, n_kv_heads=8, head_dim=128, ffn_dim=14336, vocab_size=128256)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nid = tp.exchange_id(dist, lambda: os.urandom(128))
        q.put((rank, nid, tp.shard_plan(CFG, rank, world)))
    finally:
        dist.destroy_process_group()


def _cover(parts, total):
    got = sorted(parts)
    pos = 0
    for b, n in got:
        assert b == pos and n > 0
        pos += n
    assert pos == total


def test_id_exchange_and_shards_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    assert len(res[0][1]) == 128 and res[0][1] == res[1][1]
    plans = [r[2] for r in res]
    _cover([p["q_rows"] for p in plans], CFG.n_heads * CFG.head_dim)
    _cover([p["kv_rows"] for p in plans], CFG.n_kv_heads * CFG.head_dim)
    _cover([p["ffn_rows"] for p in plans], CFG.ffn_dim)
    _cover([p["o_cols"] for p in plans], CFG.n_heads * CFG.head_dim)
    _cover([p["vocab_rows"] for p in plans], CFG.vocab_size)


def test_shard_plan_8_ranks_block_aligned():
    # the column shards (attn_output, ffn_down) must start on 256-column blocks
    for rank in range(8):
        p = tp.shard_plan(CFG, rank, 8)
        assert p["o_cols"][0] % 256 == 0 and p["o_cols"][1] % 256 == 0
        assert p["down_cols"][0] % 256 == 0 and p["down_cols"][1] % 256 == 0
    _cover([tp.shard_plan(CFG, r, 8)["vocab_rows"] for r in range(8)], CFG.vocab_size)


def _failing_worker(rank, world, port, q, mode):
    """Rank 1 fails on the host: it raises before the id exchange
    ("raise"), or exits after one step without a word ("leave").  Rank 0
    must end with an error from the process group's short timeout, not
    hang."""
    import datetime
    import time

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1 and mode == "raise":
        q.put((rank, "raised"))
        raise SystemExit(3)
    t0 = time.time()
    try:
        tp.exchange_id(dist, lambda: os.urandom(128))
        x = torch.ones(4)
        dist.all_reduce(x)  # step 1: every rank takes part
        if rank == 1:
            _put_and_exit(q, (rank, "left"))  # leaves between steps, no collective in flight
        time.sleep(0.5)
        dist.all_reduce(x)  # step 2: the peer is gone
        _put_and_exit(q, (rank, "no error"))
    except Exception as e:  # the bounded collective ends with an error
        _put_and_exit(q, (rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))


def _put_and_exit(q, msg):
    q.put(msg)
    q.close()
    q.join_thread()  # the message is in the pipe before the process ends
    os._exit(0)


def test_rank_failure_ends_peers_with_error():
    import pytest
    ctx = mp.get_context("spawn")
    for mode in ("raise", "leave"):
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q, mode)) for r in range(2)]
        for p in procs:
            p.start()
        res = dict(q.get(timeout=120) for _ in range(2))
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                pytest.fail(f"{mode}: a rank hung")
        assert res[1] in ("raised", "left")
        assert res[0].startswith("error after"), (mode, res[0])
        assert float(res[0].split()[2].rstrip("s:")) < 60
