"""The stack's progress hook agreed over ranks (ltx25_b200.watch.RankWatch),
without a GPU.

Failures are made on the host, as processes and threads that stop checking
in: a rank that exits between blocks, a rank that never joins, an abort
request.  The property under test is the one the multi-rank stack needs:
every live rank takes the SAME decision at every check -- all enqueue the
next block (and its collective) or none does -- and a stop names the peer
that caused it, within the bound.
"""
import json
import os
import random
import threading
import time

import pytest

BLOCKS = 8


def _run(watch, steps, exit_at=None, abort_at=None, jitter=None):
    """Drive `watch` like Stack.forward drives its progress hook: one call
    before each block.  Returns the (step, block) pairs that went ahead."""
    went = []
    rng = random.Random(jitter) if jitter is not None else None
    for step in range(steps):
        for b in range(BLOCKS):
            if exit_at == (step, b):
                return went, "exited"
            if abort_at == (step, b):
                watch.abort("cancelled by the caller")
            if rng is not None:
                time.sleep(rng.random() * 0.002)
            if not watch(b, BLOCKS):
                return went, watch.failed
            went.append((step, b))
    return went, None


def _proc(rank, world, path, out_dir, plan):
    import torch.distributed as dist
    import ltx25_b200 as L
    store = dist.FileStore(path, world)
    if plan.get("never_join") == rank:
        return
    # start together: process start-up (imports) must not read as a lagging rank
    store.add("ready", 1)
    joined = world - (1 if plan.get("never_join") is not None else 0)
    t0 = time.monotonic()
    while store.add("ready", 0) < joined and time.monotonic() - t0 < 120:
        time.sleep(0.01)
    w = L.RankWatch(store, rank, world, timeout_s=plan.get("timeout", 1.5))
    went, why = _run(w, plan.get("steps", 3),
                     exit_at=tuple(plan["exit"][1]) if plan.get("exit", [None])[0] == rank
                     else None,
                     abort_at=tuple(plan["abort"][1]) if plan.get("abort", [None])[0] == rank
                     else None)
    with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
        json.dump({"went": went, "why": why if why != "exited" else "exited"}, f)


def _spawn(tmp_path, world, plan):
    import torch.multiprocessing as mp
    mp.start_processes(_proc, args=(world, str(tmp_path / "store"), str(tmp_path), plan),
                       nprocs=world, join=True, start_method="spawn")
    out = {}
    for r in range(world):
        p = tmp_path / f"r{r}.json"
        if p.exists():
            out[r] = json.loads(p.read_text())
    return out


def test_healthy_ranks_all_go(tmp_path):
    out = _spawn(tmp_path, 3, {"steps": 2})
    for r in range(3):
        assert out[r]["why"] is None
        assert len(out[r]["went"]) == 2 * BLOCKS


def test_rank_that_exits_stops_every_other_rank_at_the_same_block(tmp_path):
    t0 = time.monotonic()
    out = _spawn(tmp_path, 3, {"steps": 3, "exit": [2, [1, 4]], "timeout": 1.5})
    assert out[2]["why"] == "exited"
    assert out[2]["went"][-1] == [1, 3]
    for r in (0, 1):
        # both went through step 1 block 3 and stopped before block 4
        assert out[r]["went"] == out[2]["went"], r
        assert out[r]["why"][0] == 2, out[r]["why"]
        assert "no commitment" in out[r]["why"][1]
    assert time.monotonic() - t0 < 60


def test_rank_that_never_joins_stops_the_others_at_the_first_block(tmp_path):
    out = _spawn(tmp_path, 3, {"steps": 1, "never_join": 1, "timeout": 1.0})
    assert 1 not in out
    for r in (0, 2):
        assert out[r]["went"] == []
        assert out[r]["why"][0] == 1


def test_abort_request_stops_every_rank_before_the_next_block(tmp_path):
    out = _spawn(tmp_path, 3, {"steps": 3, "abort": [1, [2, 0]]})
    for r in range(3):
        assert out[r]["went"] == out[0]["went"]
        assert out[r]["why"] == [1, "abort requested: cancelled by the caller"], out[r]["why"]
    # nobody enqueued a block of step 2
    assert all(s < 2 for s, _ in out[0]["went"])


@pytest.mark.parametrize("seed", range(4))
def test_decisions_agree_under_jitter_and_a_late_exit(seed):
    """Threads as ranks over one in-process store: random host delays and one
    rank leaving at a random block; every live rank must have gone through
    exactly the same blocks and name the same culprit."""
    import torch.distributed as dist
    import ltx25_b200 as L
    world = 4
    store = dist.HashStore()
    rng = random.Random(seed)
    leaver = rng.randrange(world)
    exit_at = (rng.randrange(2), rng.randrange(BLOCKS))
    res = {}

    def rank(r):
        w = L.RankWatch(store, r, world, timeout_s=2.0, prefix=f"t{seed}")
        res[r] = _run(w, 2, exit_at=exit_at if r == leaver else None, jitter=seed * 10 + r)

    th = [threading.Thread(target=rank, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=60)
    assert all(not t.is_alive() for t in th)
    live = [r for r in range(world) if r != leaver]
    went = res[live[0]][0]
    for r in live:
        assert res[r][0] == went, (r, res[r][0], went)
        assert res[r][1][0] == leaver
    assert res[leaver][0] == went[:len(res[leaver][0])]
    assert len(went) == exit_at[0] * BLOCKS + exit_at[1]


def test_arguments_are_checked():
    import torch.distributed as dist
    import ltx25_b200 as L
    with pytest.raises(ValueError):
        L.RankWatch(dist.HashStore(), 2, 2)
    with pytest.raises(ValueError):
        L.RankWatch(dist.HashStore(), 0, 1, timeout_s=0)
    # one rank alone always goes ahead, and an abort stops it
    w = L.RankWatch(dist.HashStore(), 0, 1)
    assert all(w(i, 4) for i in range(4))
    w.abort("done")
    assert not w(0, 4) and w.failed == (0, "abort requested: done")


def test_tcp_store_clients_agree():
    """The same protocol over a TCPStore on 127.0.0.1 (the store a multi-node
    run would use), each rank holding its own client: a rank leaving after
    step 0 block 5 stops the others there."""
    import datetime
    import torch.distributed as dist
    import ltx25_b200 as L
    world = 3
    master = dist.TCPStore("127.0.0.1", 0, world, True,
                           timeout=datetime.timedelta(seconds=30), wait_for_workers=False)
    port = master.port
    res = {}

    def rank(r):
        store = dist.TCPStore("127.0.0.1", port, world, False,
                              timeout=datetime.timedelta(seconds=30))
        w = L.RankWatch(store, r, world, timeout_s=2.0, prefix="tcp")
        res[r] = _run(w, 1, exit_at=(0, 5) if r == 2 else None)

    th = [threading.Thread(target=rank, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=60)
    assert all(not t.is_alive() for t in th)
    for r in (0, 1):
        assert res[r][0] == [(0, b) for b in range(5)], res[r][0]
        assert res[r][1][0] == 2
