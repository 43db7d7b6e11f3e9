"""Fused collective paths of the sequence-parallel layout against their NCCL equivalents (multi-GPU).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m vllm_cmp170hx_b200.bench.collectives [--tokens 128] [--iters 50]

At the config-3 decode shapes (T tokens, hidden 2304, 256 experts top-8, attention heads split over
the N ranks) each path is timed on the device from a CUDA graph of --iters calls (CUDA events, max
over ranks):

  ag_gemm      residual norm + all-gather of the normalised rows, waited inside the KDA input GEMM
               (fused) vs rms_norm + all_gather_into_tensor + GEMM (NCCL)
  gemm_rs      o_proj GEMM pushing each token row to its owner + the owner's sum, residual add and
               norm (fused) vs GEMM + reduce_scatter_tensor + fused_add_rms_norm (NCCL)
  dispatch     router top-k + dispatch of each row to the ranks holding its experts, received by the
               assignment builder (fused) vs top-k + all-gather of rows, ids and weights + the builder
               (NCCL, the reference's expert-parallel dispatch)
  combine      weighted expert sum pushed to the owners + their sum, residual add and norm (fused) vs
               combine + reduce_scatter_tensor + add + norm (NCCL)

Each line gives the bytes one rank sends over NVLink, the HBM bytes the GEMM streams, the FLOPs, and
the roofline time max(FLOPs / bf16 peak, HBM bytes / HBM peak, NVLink bytes / 770 GB/s) with the
achieved fraction of it (peaks from MEASURED_PEAKS.json; 770 GB/s is the measured peer-copy rate per
direction of this pool's B200s).
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from .. import _ext, ops
from ..parallel import state as pstate
from ..parallel.sp import FusedSP, TorchSP, scope
from .kernels import _peaks

NVLINK_GBS = 770.0


def _graph_time_us(fn, iters: int) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    multi = dist.is_initialized()
    if multi:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) * 1e3 / iters], dtype=torch.float64, device="cuda")
    if multi:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    return float(t.item())


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=128)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--profile", action="store_true",
                    help="rank 0 prints a per-kernel table of five eager calls of each path (guidance only)")
    a = ap.parse_args(argv)
    st = pstate.init(tp_size=int(os.environ.get("WORLD_SIZE", "1")), timeout_s=120)
    N, r = st.tp_size, st.tp_rank
    dev = st.device
    T, H, E, k = a.tokens, 2304, 256, 8
    Tr = T // N
    heads_local = 32 // N
    Kin = 3 * heads_local * 128 + 2 * 128 + heads_local  # KDA fused input projection rows of one rank
    Kin += (-Kin) % 8
    Ko = heads_local * 128
    peaks = _peaks()
    g = torch.Generator(device=dev).manual_seed(r)
    bf = torch.bfloat16
    W_in = (torch.randn(Kin, H, device=dev, generator=g) * H ** -0.5).to(bf)
    W_o = (torch.randn(H, Ko, device=dev, generator=g) * Ko ** -0.5).to(bf)
    wn = torch.ones(H, dtype=bf, device=dev)
    x_loc = torch.randn(Tr, H, device=dev, generator=g).to(bf)
    a_full = torch.randn(T, Ko, device=dev, generator=g).to(bf)
    logits = torch.randn(Tr, E, device=dev, generator=g)
    res = torch.zeros(Tr, H, dtype=bf, device=dev)
    h = torch.empty(Tr, H, dtype=bf, device=dev)
    out_in = torch.empty(T, Kin, dtype=bf, device=dev)
    fsp = FusedSP(st.tp_group, st.tp_cpu_group, dev, H, k, max_tokens=max(256, T), timeout_s=10.0)
    tsp = TorchSP(st.tp_group, H, k)
    for sp in (fsp, tsp):
        sp.begin(T)
    TK = T * k
    i32 = dict(dtype=torch.int32, device=dev)
    E_loc = E // N
    bufs = dict(sorted_token=torch.empty(TK, **i32), sorted_weight=torch.empty(TK, dtype=torch.float32, device=dev),
                slot_of=torch.empty(TK, **i32), items=torch.empty(E_loc + TK, 4, **i32),
                num_items=torch.empty(1, **i32), offsets=torch.empty(E_loc + 1, **i32))
    emap = torch.full((E,), -1, dtype=torch.int32)
    emap[r * E_loc:(r + 1) * E_loc] = torch.arange(E_loc, dtype=torch.int32)
    emap = emap.to(dev)
    y = torch.randn(TK, H, device=dev, generator=g)
    add = torch.randn(Tr, H, device=dev, generator=g).to(bf)

    def build(sp):
        ids, w = sp.dispatch_recv()[1:]
        b = bufs
        if sp.fused:
            sp.build_assignments(ids, w, emap, E_loc, 16, b["sorted_token"], b["sorted_weight"], b["slot_of"],
                                 b["items"], b["num_items"], b["offsets"])
        else:
            _ext.ops().moe_build_assignments(ids, w, emap, E_loc, 16, b["sorted_token"], b["sorted_weight"],
                                             b["slot_of"], b["items"], b["num_items"], b["offsets"])

    # a routing to set up slot_of for the combine timing
    for sp in (fsp, tsp):
        sp.route_dispatch(logits, x_loc, k, 0, None, 1.0, True, E_loc)
        build(sp)
    torch.cuda.synchronize()

    def ag_gemm(sp):
        def f():
            sp.norm("local", res, wn, 1e-6, x=x_loc, ag=True)
            with scope(sp):
                ops.gemm(sp.gathered(), W_in, out=out_in)
        return f

    def gemm_rs(sp):
        def f():
            with scope(sp):
                sp.gemm_rs(a_full, W_o)
            sp.norm("rs", res, wn, 1e-6, out=h)
        return f

    def dispatch(sp):
        def f():
            sp.route_dispatch(logits, x_loc, k, 0, None, 1.0, True, E_loc)
            build(sp)
        return f

    def combine(sp):
        def f():
            if sp.fused:
                sp.combine_push(y, bufs["slot_of"], bufs["sorted_weight"], k)
            else:
                part = torch.empty(T, H, dtype=bf, device=dev)
                _ext.ops().moe_combine(y, bufs["slot_of"], bufs["sorted_weight"], k, None, part)
                sp.combine_partial(part)
            sp.norm("comb", res, wn, 1e-6, add=add, out=h)
        return f

    row = H * 2
    # bytes this rank sends over NVLink per call (average routing for the dispatch / combine: a token's 8
    # experts fall on min(N, ~8) ranks; the measured routing is used below)
    dm = fsp.dmask[:Tr].cpu()
    dests = sum(bin(int(v)).count("1") - ((int(v) >> r) & 1) for v in dm.tolist())
    paths = {
        "ag_gemm": (ag_gemm, Tr * row * (N - 1), Kin * H * 2, 2.0 * T * Kin * H),
        "gemm_rs": (gemm_rs, Tr * row * (N - 1), H * Ko * 2, 2.0 * T * H * Ko),
        "dispatch": (dispatch, dests * (row + 8 * k) + (N - 1) * Tr * 8 * k, 0, 0.0),
        "combine": (combine, dests * row, 0, 2.0 * TK * H),
    }
    for name, (mk, nv_bytes, hbm_bytes, flops) in paths.items():
        if a.profile:
            from torch.profiler import ProfilerActivity, profile

            for tag, sp in (("fused", fsp), ("nccl", tsp)):
                f = mk(sp)
                f()
                torch.cuda.synchronize()
                with profile(activities=[ProfilerActivity.CUDA]) as prof:
                    for _ in range(5):
                        f()
                    torch.cuda.synchronize()
                if r == 0:
                    print(f"== {name} ({tag}), 5 calls", flush=True)
                    print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=12, max_name_column_width=60),
                          flush=True)
        t_f = _graph_time_us(mk(fsp), a.iters)
        t_n = _graph_time_us(mk(tsp), a.iters)
        roof_us = max(flops / (peaks["bf16_tflops"] * 1e12), hbm_bytes / (peaks["hbm_gbs"] * 1e9),
                      nv_bytes / (NVLINK_GBS * 1e9)) * 1e6
        _ext.check_status(dev)
        if r == 0:
            print(json.dumps({"path": name, "n_gpus": N, "tokens": T, "fused_us": round(t_f, 2),
                              "nccl_us": round(t_n, 2), "speedup_vs_nccl": round(t_n / t_f, 2),
                              "nvlink_bytes_per_rank": int(nv_bytes), "hbm_bytes": int(hbm_bytes),
                              "flops": flops, "roofline_us": round(roof_us, 3),
                              "fraction_of_roofline": round(roof_us / t_f, 3),
                              "peaks": {"hbm_gbs": peaks["hbm_gbs"], "bf16_tflops": peaks["bf16_tflops"],
                                        "nvlink_gbs": NVLINK_GBS, "source": peaks.get("source")}}), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    pstate.destroy()


if __name__ == "__main__":
    main()
