"""Failure detection on the host (gloo ranks on CPU, nothing faults a GPU):

* the all-rank agreement that gates every custom transport: when one rank fails its setup, every
  rank falls back (`parallel/symm._agree`);
* a rank that never joins: the others' process-group initialisation ends with an error within its
  timeout instead of hanging;
* a rank that leaves between steps: the others' next collective ends with an error within the
  process-group timeout.
"""

import os
import time

import torch.multiprocessing as mp


def _env(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))


def _agree_worker(rank, world, port, q):
    _env(rank, world, port)
    from vllm_cmp170hx_b200.parallel import state as pstate
    from vllm_cmp170hx_b200.parallel.symm import _agree

    try:
        st = pstate.init(tp_size=world, device="cpu", timeout_s=30)
        ok_all = _agree(True, st.tp_cpu_group)
        one_bad = _agree(rank != 1, st.tp_cpu_group)
        q.put((rank, (ok_all, one_bad)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))
    finally:
        pstate.destroy()


def test_setup_agreement_falls_back_on_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 3
    port = 26100 + os.getpid() % 500
    ps = [ctx.Process(target=_agree_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=30)
    assert all(res[r] == (True, False) for r in range(world)), res


def _late_worker(rank, world, port, q, leave_before_init):
    _env(rank, world, port)
    from vllm_cmp170hx_b200.parallel import state as pstate

    if rank == 1 and leave_before_init:
        q.put((rank, "left"))
        return
    t0 = time.monotonic()
    try:
        st = pstate.init(tp_size=world, device="cpu", timeout_s=4)
        if rank == 1:  # joins, then leaves between steps without taking part in the next collective
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # the message is out before the process ends abruptly
            os._exit(0)
        import torch
        import torch.distributed as dist

        dist.all_reduce(torch.ones(4), group=st.tp_cpu_group)
        q.put((rank, ("no error", time.monotonic() - t0)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, ("error", time.monotonic() - t0, type(e).__name__)))


def _run_late(leave_before_init):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 25600 + os.getpid() % 400 + (7 if leave_before_init else 0)
    ps = [ctx.Process(target=_late_worker, args=(r, 2, port, q, leave_before_init)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=180) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_rank_that_never_joins_is_reported():
    res = _run_late(True)
    assert res[1] == "left"
    kind, elapsed = res[0][0], res[0][1]
    assert kind == "error" and elapsed < 120, res


def test_rank_that_leaves_between_steps_is_reported():
    res = _run_late(False)
    assert res[1] == "left"
    kind, elapsed = res[0][0], res[0][1]
    assert kind == "error" and elapsed < 120, res
