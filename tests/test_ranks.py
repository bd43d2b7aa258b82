"""Process-group plumbing of the multi-GPU runs (mlx-flashvsr-swift_b200/ranks.py), on CPU with gloo ranks: the
launcher's rank layout is validated on the host, the per-rank reductions agree on every rank, and a rank that dies
before a collective turns the survivor's collective into an error within the group timeout instead of a hang."""
from __future__ import annotations

import os
import time

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("env,fragment", [
    ({"WORLD_SIZE": "0"}, "WORLD_SIZE"),
    ({"WORLD_SIZE": "2", "RANK": "2"}, "RANK"),
    ({"WORLD_SIZE": "2", "RANK": "-1"}, "RANK"),
    ({"WORLD_SIZE": "4", "RANK": "1", "LOCAL_RANK": "3"}, "LOCAL_RANK"),
    ({"WORLD_SIZE": "two"}, "not an integer"),
])
def test_rank_layout_is_validated(fvsr, env, fragment):
    import importlib
    ranks = importlib.import_module("fvsr_b200.ranks")
    with pytest.raises(ValueError, match=fragment):
        ranks.rank_info(env)


def test_rank_layout_defaults_to_one_process(fvsr):
    import importlib
    ranks = importlib.import_module("fvsr_b200.ranks")
    info = ranks.rank_info({})
    assert (info.rank, info.world, info.local) == (0, 1, 0)
    assert ranks.max_over_ranks(3.5) == 3.5 and ranks.sum_over_ranks(2.0) == 2.0   # no group: the value itself


def _rank_main(rank, world, port, die, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import sys
    sys.path.insert(0, ROOT)
    from __graft_entry__ import _load_package
    _load_package()
    import importlib
    ranks = importlib.import_module("fvsr_b200.ranks")
    info = ranks.rank_info()
    ranks.init(info, "gloo", timeout_s=5)
    ranks.barrier()
    if die and rank == 1:
        os._exit(3)                       # leaves between steps, with no collective in flight
    t0 = time.time()
    try:
        mx = ranks.max_over_ranks(float(rank + 1))
        sm = ranks.sum_over_ranks(float(rank + 1))
        q.put((rank, "ok", mx, sm, time.time() - t0))
        ranks.shutdown()
    except Exception as exc:              # the survivor's collective fails instead of hanging
        q.put((rank, "error", type(exc).__name__, str(exc)[:200], time.time() - t0))


def _run(world, die):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + (os.getpid() + (7 if die else 0)) % 200
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, die, q)) for r in range(world)]
    for p in procs:
        p.start()
    expect = world - (1 if die else 0)
    res = [q.get(timeout=120) for _ in range(expect)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(res), [p.exitcode for p in procs]


def test_reductions_agree_on_every_rank(fvsr):
    res, codes = _run(2, die=False)
    assert [r[1] for r in res] == ["ok", "ok"]
    assert all(r[2] == 2.0 and r[3] == 3.0 for r in res)        # max(1, 2), 1 + 2
    assert codes == [0, 0]


def test_a_dead_rank_ends_the_survivors_collective_with_an_error(fvsr):
    res, codes = _run(2, die=True)
    assert len(res) == 1 and res[0][0] == 0
    assert res[0][1] == "error", res
    assert res[0][4] < 60.0                                      # bounded by the group timeout, not a hang
    assert codes[1] == 3
