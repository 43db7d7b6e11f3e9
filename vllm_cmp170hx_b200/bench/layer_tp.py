"""BASELINE config 2 at TP = N: one sparse-MLA decode layer (128 heads, kv_lora 512, indexer 64 heads
x 128 picking top-2048 of a 32768-position paged cache, batch 64), heads split over the N ranks.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m vllm_cmp170hx_b200.bench.layer_tp [--batch 64] [--ctx 32768] [--iters 20]

The timed unit is the layer as it runs inside the sequence-parallel layout: the input RMSNorm of this
rank's rows with the all-gather of the normalised rows, the attention on all tokens with this rank's
heads, and the row-parallel o_proj reduce-scattered to the token owners plus the owners' residual add
and norm.  Two transports: this package's fused kernels (the all-gather waited inside the input GEMM,
the reduce-scatter in the o_proj GEMM's epilogue) and torch.distributed (NCCL all_gather / GEMM /
reduce_scatter).  At N = 1 the layer runs alone.  Device time from a CUDA graph of --iters layers
(CUDA events, max over ranks); one JSON line per transport.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from .. import _ext
from ..config import config2_layer
from ..models.hybrid import MLAAttention
from ..models.layers import WeightInit
from ..parallel import state as pstate
from ..parallel.sp import FusedSP, TorchSP, scope
from .collectives import NVLINK_GBS, _graph_time_us
from .kernels import _paged_ctx, _peaks


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args(argv)
    N = int(os.environ.get("WORLD_SIZE", "1"))
    st = pstate.init(tp_size=N, timeout_s=120)
    st.expert_parallel = False  # config 2 splits the heads (tensor parallel)
    r, dev = st.tp_rank, st.device
    c = config2_layer()
    H = c.hidden_size
    layer = MLAAttention(c, WeightInit(0, dev, "local"), N, r)
    ctx = _paged_ctx(a.batch, a.ctx, dev, mla_layer=layer)
    B = a.batch
    Tr = B // N
    g = torch.Generator(device=dev).manual_seed(7 + r)
    x_loc = torch.randn(Tr, H, device=dev, generator=g).to(torch.bfloat16)
    wn = torch.ones(H, dtype=torch.bfloat16, device=dev)
    res = torch.empty(Tr, H, dtype=torch.bfloat16, device=dev)
    h = torch.empty(Tr, H, dtype=torch.bfloat16, device=dev)
    peaks = _peaks()
    topk = c.mla.index_topk
    wbytes = sum(p.numel() * p.element_size() for p in layer.parameters())
    kv_bytes = B * (min(topk, a.ctx) * 576 * 2 + a.ctx * (128 + 4))
    # this rank's HBM traffic: its weights, the selected rows of its heads' queries (every rank gathers
    # the rows for its heads) and the indexer keys (replicated indexer)
    hbm = wbytes + kv_bytes
    results = []
    with torch.inference_mode():
        if N == 1:
            x = torch.randn(B, H, device=dev, dtype=torch.bfloat16)
            t = _graph_time_us(lambda: layer(x, ctx, 0), a.iters)
            results.append(("none", t, 0))
        else:
            transports = [("fused", FusedSP(st.tp_group, st.tp_cpu_group, dev, H, 8, max_tokens=max(256, B))),
                          ("nccl", TorchSP(st.tp_group, H, 8))]
            for name, sp in transports:
                sp.begin(B)

                def step(sp=sp):
                    sp.norm("local", res, wn, 1e-6, x=x_loc, ag=True)
                    with scope(sp):
                        layer(sp.gathered(), ctx, 0)
                    sp.norm("rs", res, wn, 1e-6, out=h)

                t = _graph_time_us(step, a.iters)
                results.append((name, t, 2 * Tr * H * 2 * (N - 1)))
    _ext.check_status(dev)
    if r == 0:
        for name, t, nv in results:
            roof = max(hbm / (peaks["hbm_gbs"] * 1e9), nv / (NVLINK_GBS * 1e9)) * 1e6
            print(json.dumps({"config": 2, "layer": "sparse-MLA decode, 128 heads, top-2048 of ctx", "n_gpus": N,
                              "parallelism": f"tp{N}", "transport": name, "batch": B, "ctx": a.ctx,
                              "us_per_layer": round(t, 2), "tokens_per_s_per_layer": round(B / (t * 1e-6), 1),
                              "hbm_bytes_per_rank": int(hbm), "nvlink_bytes_per_rank": int(nv),
                              "roofline_us": round(roof, 2), "fraction_of_roofline": round(roof / t, 3),
                              "peaks": {"hbm_gbs": peaks["hbm_gbs"], "nvlink_gbs": NVLINK_GBS,
                                        "source": peaks.get("source")}}), flush=True)
    if N > 1:
        dist.barrier()
    pstate.destroy()


if __name__ == "__main__":
    main()
