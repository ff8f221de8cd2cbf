"""Multi-rank host logic on CPU: the request / KV-head plan, max-over-ranks timing and the output
gather, as gloo process groups of world size 2; and a rank that fails before a collective, which the
other rank must see as an error (never a hang).  No GPU is used."""
import datetime
import multiprocessing as mp
import os
import socket
import sys
import time
import traceback

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from openattention_b200 import shard  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_owns_every_pair_once(world):
    for batch in list(range(1, 20)) + [32, 33, 64, 70]:
        if batch < world and 8 % world:
            continue
        owned = {}
        for rank in range(world):
            s = shard.plan(batch, world, rank)
            for r in range(s.req_start, s.req_start + s.req_count):
                for h in range(s.kv_start, s.kv_start + s.kv_count):
                    assert (r, h) not in owned
                    owned[(r, h)] = rank
            assert list(s.q_heads) == list(range(s.kv_start * 4, (s.kv_start + s.kv_count) * 4))
        assert len(owned) == batch * 8
        counts = [shard.plan(batch, world, r).req_count * shard.plan(batch, world, r).kv_count for r in range(world)]
        assert max(counts) - min(counts) <= 8


def test_plan_rejects_bad_arguments():
    with pytest.raises(ValueError):
        shard.plan(0, 2, 0)
    with pytest.raises(ValueError):
        shard.plan(4, 2, 2)
    with pytest.raises(ValueError):
        shard.plan(2, 3, 0)  # 3 ranks cannot split 8 KV heads


def _worker(rank, world, port, mode, q):
    try:
        import torch
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        if mode == "fail" and rank == 1:
            raise RuntimeError("planted failure on rank 1 before the collective")
        B = 6
        s = shard.plan(B, world, rank)
        # this rank's outputs: one (32, 4) row block per request, filled with the request id
        local = torch.arange(s.req_start, s.req_start + s.req_count, dtype=torch.float32)
        local = local.repeat_interleave(32).view(-1, 1).expand(-1, 4).contiguous()
        t0 = time.time()
        try:
            worst = shard.max_over_ranks(10.0 + rank)
            full = shard.gather_rows(local)
        except Exception as e:  # noqa: BLE001
            q.put((rank, "error", f"{type(e).__name__}: {e}", time.time() - t0))
            return
        want = torch.arange(B, dtype=torch.float32).repeat_interleave(32).view(-1, 1).expand(-1, 4)
        q.put((rank, "ok", (worst, bool(torch.equal(full, want))), time.time() - t0))
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        q.put((rank, "raised", traceback.format_exc(limit=2), 0.0))


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    deadline = time.time() + 120
    while len(res) < world and time.time() < deadline:
        try:
            r = q.get(timeout=5)
            res[r[0]] = r[1:]
        except Exception:  # noqa: BLE001
            if not any(p.is_alive() for p in ps):
                break
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
            p.join()
    return res


def test_gloo_two_ranks_timing_and_gather():
    res = _run("ok")
    assert set(res) == {0, 1}, res
    for rank in (0, 1):
        status, val, _ = res[rank]
        assert status == "ok", res
        worst, gathered_ok = val
        assert worst == 11.0
        assert gathered_ok


def test_gloo_failed_rank_is_an_error_not_a_hang():
    res = _run("fail")
    assert res[1][0] == "raised" and "planted failure" in res[1][1]
    status, msg, waited = res[0]
    assert status == "error", res
    assert waited < 60.0
