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


def _fused_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from vllm_cmp170hx_b200 import _ext, ops
    from vllm_cmp170hx_b200.parallel import state as pstate
    from vllm_cmp170hx_b200.parallel.symm import FusedComm

    try:
        st = pstate.init(tp_size=world, timeout_s=60)
        fc = FusedComm(st.tp_group, st.tp_cpu_group, st.device, max_ctas=148, tile_cap=64 << 10,
                       combine_bytes=2 << 20, combine_blocks=64, timeout_s=5.0)
        errs = []
        # GEMM + all-reduce: swap (M <= 128) and plain (M in (128, 256]) orientations, with bias
        for it, (M, N, K, bias) in enumerate([(128, 2304, 1024, False), (16, 2304, 512, True), (1, 4096, 256, False),
                                              (200, 2304, 512, False), (128, 2304, 1024, False)]):
            g = torch.Generator().manual_seed(it)
            xs = [torch.randn(M, K, generator=g).to(torch.bfloat16) for _ in range(world)]
            ws = [(torch.randn(N, K, generator=g) * K ** -0.5).to(torch.bfloat16) for _ in range(world)]
            b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16) if bias else None
            ref = sum(x.float() @ w.float().t() for x, w in zip(xs, ws)) + (b.float() if bias else 0)
            y = fc.gemm_all_reduce(xs[rank].cuda(), ws[rank].cuda(), b.cuda() if bias else None)
            assert y is not None, (M, N)
            torch.cuda.synchronize()
            errs.append(((y.float().cpu() - ref).abs().max() / ref.abs().max()).item())
        # combine + all-reduce against combine then a float sum over ranks
        T, H, k, TK = 96, 2304, 8, 96 * 8
        for it in range(3):
            g = torch.Generator().manual_seed(100 + it)
            ys = [torch.randn(TK, 2304 + 64, generator=g) for _ in range(world)]
            slot = torch.randperm(TK, generator=g).int().view(T, k)
            wt = torch.rand(TK, generator=g)
            adds = [torch.randn(T, H, generator=g).to(torch.bfloat16) for _ in range(world)]
            ref = 0
            for r in range(world):
                part = torch.zeros(T, H)
                for t in range(T):
                    for j in range(k):
                        s = int(slot[t, j])
                        part[t] += float(wt[s]) * ys[r][s, :H]
                ref = ref + (part + adds[r].float()).to(torch.bfloat16).float()
            out = fc.combine_all_reduce(ys[rank].cuda(), slot.cuda(), wt.cuda(), k, adds[rank].cuda(), T, H)
            torch.cuda.synchronize()
            errs.append(((out.float().cpu() - ref).abs().max() / ref.abs().max()).item())
        # CUDA graph: GEMM+AR -> combine+AR -> GEMM+AR, replayed with new inputs
        M, N, K = 64, 2304, 1024
        x = torch.zeros(M, K, dtype=torch.bfloat16, device="cuda")
        w = torch.zeros(N, K, dtype=torch.bfloat16, device="cuda")
        w2 = torch.zeros(N, N, dtype=torch.bfloat16, device="cuda")
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fc.gemm_all_reduce(fc.gemm_all_reduce(x, w, None), w2, None)
        torch.cuda.current_stream().wait_stream(s)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            y1 = fc.gemm_all_reduce(x, w, None)
            y2 = fc.gemm_all_reduce(y1, w2, None)
        for it in range(3):
            g = torch.Generator().manual_seed(200 + it)
            xs = [torch.randn(M, K, generator=g).to(torch.bfloat16) for _ in range(world)]
            wsr = [(torch.randn(N, K, generator=g) * K ** -0.5).to(torch.bfloat16) for _ in range(world)]
            w2s = [(torch.randn(N, N, generator=g) * N ** -0.5).to(torch.bfloat16) for _ in range(world)]
            x.copy_(xs[rank])
            w.copy_(wsr[rank])
            w2.copy_(w2s[rank])
            gr.replay()
            torch.cuda.synchronize()
            r1 = sum(a.float() @ b.float().t() for a, b in zip(xs, wsr)).to(torch.bfloat16).float()
            r2 = sum(r1 @ b.float().t() for b in w2s)
            errs.append(((y2.float().cpu() - r2).abs().max() / r2.abs().max()).item())
        _ext.check_status(st.device)
        del gr
        q.put((rank, errs))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))
    finally:
        pstate.destroy()


def test_fused_gemm_and_combine_all_reduce():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    world = min(world, 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29100 + os.getpid() % 400
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
        assert max(res[r]) < 3e-2, res[r]
