"""Symmetric-memory one-shot all-reduce kernel on 2+ GPUs (NCCL group for the
plumbing): result vs the fp32 sum of every rank's input, repeated calls
(epoch flags, double buffering) and CUDA-graph replay."""

import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _inputs(world, n, it):
    return [torch.randn(n, generator=torch.Generator().manual_seed(1000 * it + r)).to(torch.bfloat16)
            for r in range(world)]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from vllm_cmp170hx_b200 import _ext
    from vllm_cmp170hx_b200.parallel import state as pstate
    from vllm_cmp170hx_b200.parallel.symm import SymmComm

    try:
        st = pstate.init(tp_size=world, timeout_s=60)
        sc = SymmComm(st.tp_group, st.tp_cpu_group, st.device, max_bytes=4 << 20, blocks=32, timeout_s=5.0)
        errs = []
        for it, n in enumerate([8, 1024, 2304 * 128, 2304 * 128, 1 << 20, 4096]):
            xs = _inputs(world, n, it)
            ref = sum(x.float() for x in xs)
            y = sc.all_reduce(xs[rank].cuda())
            torch.cuda.synchronize()
            errs.append(((y.float().cpu() - ref).abs().max() / ref.abs().max()).item())
        # graph capture: three all-reduces replayed twice with new inputs
        x = torch.zeros(2304 * 64, dtype=torch.bfloat16, device="cuda")
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            sc.all_reduce(x)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            y1 = sc.all_reduce(x)
            y2 = sc.all_reduce(y1)
            y3 = sc.all_reduce(y2)
        for it in range(2):
            xs = _inputs(world, x.numel(), 50 + it)
            x.copy_(xs[rank])
            g.replay()
            torch.cuda.synchronize()
            ref = sum(v.float() for v in xs) * world * world
            errs.append(((y3.float().cpu() - ref).abs().max() / ref.abs().max()).item())
        _ext.check_status(st.device)
        del g
        q.put((rank, errs))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))
    finally:
        pstate.destroy()


def test_symm_all_reduce():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    world = min(world, 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 500
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
        assert max(res[r]) < 2e-2, res[r]
