"""CPU: data-parallel sharding (host logic) and a 2-rank gloo run."""

import os
import random

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from q6w_b200 import dp


def test_shard_range_covers_once():
    for n in (0, 1, 7, 8192):
        for w in (1, 2, 3, 8):
            spans = [dp.shard_range(n, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def test_balance_by_tokens_bound():
    rng = random.Random(0)
    lengths = [rng.randint(8, 256) for _ in range(2048)]
    for w in (1, 2, 4, 8):
        parts = dp.balance_by_tokens(lengths, w)
        assert sorted(i for p in parts for i in p) == list(range(len(lengths)))
        loads = [sum(lengths[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lengths)


def test_requeue_moves_failed_work():
    lengths = [5, 9, 3, 7, 1, 8]
    parts = dp.balance_by_tokens(lengths, 3)
    out = dp.requeue(parts, [1], lengths)
    assert out[1] == []
    assert sorted(i for p in out for i in p) == list(range(6))
    with pytest.raises(RuntimeError):
        dp.requeue(parts, [0, 1, 2])


def _worker(rank, world, port, lengths, fail_rank, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    parts = dp.balance_by_tokens(lengths, world)
    mine = parts[rank]
    # "work": a token checksum per request; rank fail_rank reports failure instead
    result = {"rank": rank, "ok": rank != fail_rank, "done": {i: lengths[i] * 3 for i in mine} if rank != fail_rank else {}}
    got = dp.gather_to_rank0(result, world)
    if rank == 0:
        failed = [g["rank"] for g in got if not g["ok"]]
        parts2 = dp.requeue(parts, failed, lengths)
        done = {}
        for g in got:
            done.update(g["done"])
        for r in failed:  # survivors re-run the orphaned requests (here: rank 0 on their behalf)
            for i in parts2[0]:
                done.setdefault(i, lengths[i] * 3)
        q.put(sorted(done.items()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank", [None, 1])
def test_two_rank_gloo_shard_and_gather(fail_rank):
    lengths = [random.Random(1).randint(8, 256) for _ in range(64)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + random.Random().randint(0, 2000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, lengths, fail_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [i for i, _ in res] == list(range(64))
    assert all(v == lengths[i] * 3 for i, v in res)
