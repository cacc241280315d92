"""Rank plumbing of the sharded benchmark, exercised with gloo ranks on CPU.

The step itself is stood in for by the CPU oracle (tests only); what is
checked is the product's multi-process logic: shard assignment, the
max-over-ranks reduction, the gather of per-rollout digests and their check
against a single-process run (as the benchmark does after timing), and that
a rank which dies is reported by the others instead of hanging them.
"""

import multiprocessing as mp
import os
import socket
import time

import numpy as np
import pytest

from burn_automata_b200 import multigpu


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("total,world", [(256, 1), (256, 2), (256, 8), (10, 4), (3, 8)])
def test_strong_shards_partition_the_batch(total, world):
    seen = []
    for r in range(world):
        first, count = multigpu.shard(total, world, r, strong=True)
        seen.extend(range(first, first + count))
    assert seen == list(range(total))


def test_weak_shards_are_disjoint_full_batches():
    ranges = [multigpu.shard(256, 4, r, strong=False) for r in range(4)]
    assert [c for _, c in ranges] == [256] * 4
    starts = [f for f, _ in ranges]
    assert starts == [0, 256, 512, 768]


def _rank_main(rank, world, port, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        import oracle
        from burn_automata_b200 import workloads

        oracle.set_threads(1)
        info = multigpu.env_rank()
        multigpu.init("gloo", info, timeout_s=10)
        if mode == "die" and rank == 1:
            raise RuntimeError("rank 1 fails before the barrier")
        first, count = multigpu.shard(4, world, rank, strong=True)
        w = workloads.make("cfg0", batch=count, n=64, first=first)
        t0 = time.perf_counter()
        pos, st, _ = oracle.rollout(w.model, w.weights, w.grid, w.positions, w.states, w.batch,
                                    w.n, 2, w.dt)
        elapsed = time.perf_counter() - t0
        multigpu.barrier_or_fail(timeout_s=5)
        mx = multigpu.max_over_ranks([elapsed, float(rank)])
        times = multigpu.gather_floats(float(rank) + 0.5)
        digests = multigpu.gather_objects(multigpu.rollout_digests(w.batch, first, pos, st))
        plans = multigpu.gather_objects((first, count))
        out.put((rank, "ok", mx, (digests, plans, times)))
        multigpu.finish()
    except Exception as e:  # reported to the parent, never swallowed
        out.put((rank, "error", repr(e), None))


def _run(world, mode, limit=90):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + limit
    while len(results) < world and time.time() < deadline:
        try:
            r = q.get(timeout=1)
            results[r[0]] = r
        except Exception:
            pass
    for p in procs:
        p.join(timeout=max(1, deadline - time.time()))
        if p.is_alive():
            p.kill()
    return results


def test_two_gloo_ranks_match_a_single_process_run():
    import oracle
    from burn_automata_b200 import workloads

    res = _run(2, "ok")
    assert set(res) == {0, 1} and all(r[1] == "ok" for r in res.values()), res
    digests, plans, times = res[0][3]
    assert res[1][3] == (digests, plans, times)
    assert plans == [(0, 2), (2, 2)] and times == [0.5, 1.5]
    assert res[0][2][1] == 1.0  # max over ranks of the rank id
    # the single-process run of all four rollouts, as rank 0 of the benchmark reruns them
    w = workloads.make("cfg0", batch=4, n=64)
    pos, st, _ = oracle.rollout(w.model, w.weights, w.grid, w.positions, w.states, w.batch, w.n,
                                2, w.dt)
    expected = multigpu.rollout_digests(w.batch, 0, pos, st)
    assert multigpu.compare_digests(digests, expected) == (4, [])
    # one changed bit in rollout 3 of the reference run is caught (planted on the CPU side)
    st2 = st.copy()
    st2[3 * 64 * 16 + 5] = np.nextafter(st2[3 * 64 * 16 + 5], np.float32(np.inf))
    assert multigpu.compare_digests(digests, multigpu.rollout_digests(4, 0, pos, st2)) == (4, [3])


def test_a_dead_rank_is_reported_not_waited_on():
    t0 = time.time()
    res = _run(2, "die", limit=90)
    assert time.time() - t0 < 90
    assert res[1][1] == "error"
    assert 0 in res and res[0][1] == "error", res
