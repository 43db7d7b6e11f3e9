"""Kernel micro-benchmarks at the shapes of the BASELINE configs.

    python -m vllm_cmp170hx_b200.bench.kernels <op> [--tokens T] [--iters N] ...

ops:
  gemm        bf16 GEMM y = x W^T (ours vs cuBLAS), --m --n --k
  exl3_moe    config-3 routed experts (256 x [2304 -> 1024 -> 2304], top-8, EXL3 4-bit), --tokens
  marlin_moe  config-4 routed experts (256 x [4096 -> 1536 -> 4096], top-8, Marlin int4 g128), --tokens
  fp8_linear  fp8 128x128 block-scaled linear, --m --n --k
  mla_decode  config-2 sparse-MLA decode layer (128 heads, top-2048 of --ctx positions), --tokens = batch
  kda_decode  config-3 KDA layer decode step (32 heads x 128), --tokens = sequences
  kda_prefill config-3 KDA layer core over --seqs prompts of --tokens tokens (32 heads x 128), the
              chunked tensor-core path and the token recurrence (--mode chunked | recurrent)
  attn        the sparse-attention kernel alone, --tokens --heads --topk --ctx --splits

Each op prints one JSON line: mean device time per call over --iters calls
timed with CUDA events after warm-up (inputs larger than L2 where the op
streams weights), the algorithmic bytes / FLOPs and their fraction of the
measured machine peaks (HBM copy bandwidth and cuBLAS bf16 throughput read
from MEASURED_PEAKS.json at the repository root when present).
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from .. import _ext, ops
from ..config import config2_layer, config3, config4
from ..models.hybrid import KDAAttention, MLAAttention, StepContext
from ..models.layers import WeightInit
from ..parallel import state as pstate

_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def _peaks() -> dict:
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d.get("hbm_gbs", _PEAKS["hbm_gbs"]), "bf16_tflops": d.get("bf16_tflops", _PEAKS["bf16_tflops"]),
                "source": "measured"}
    return dict(_PEAKS, source="fallback")


_PROFILE = False
_GRAPH = False


def time_us(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    if _PROFILE:  # per-kernel breakdown of one call (guidance only; times under the profiler are not reported)
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=25, max_name_column_width=70))
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if _GRAPH:  # the calls replayed from one CUDA graph: device time without host launch gaps
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) * 1e3 / iters
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / iters


def _report(op: str, us: float, nbytes: float = 0.0, flops: float = 0.0, **extra) -> dict:
    pk = _peaks()
    out = {"op": op, "us": round(us, 2)}
    if nbytes:
        gbs = nbytes / us / 1e3
        out.update(bytes=int(nbytes), gbs=round(gbs, 1), frac_hbm=round(gbs / pk["hbm_gbs"], 3))
    if flops:
        tf = flops / us / 1e6
        out.update(flops=int(flops), tflops=round(tf, 1), frac_bf16=round(tf / pk["bf16_tflops"], 3))
    out["peaks"] = pk["source"]
    out.update(extra)
    print(json.dumps(out), flush=True)
    return out


def bench_gemm(a):
    x = torch.randn(a.m, a.k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(a.n, a.k, device="cuda", dtype=torch.bfloat16)
    nbytes = 2 * (a.m * a.k + a.n * a.k + a.m * a.n)
    ours = time_us(lambda: ops.gemm(x, w), a.iters)
    ref = time_us(lambda: torch.nn.functional.linear(x, w), a.iters)
    return _report("gemm", ours, nbytes, 2.0 * a.m * a.n * a.k, m=a.m, n=a.n, k=a.k, cublas_us=round(ref, 2))


def _route(T, E, k, dev):
    from ..ops import moe as moe_ops

    g = torch.Generator(device=dev).manual_seed(0)
    return moe_ops.topk(torch.randn(T, E, device=dev, generator=g), k, 0)


def bench_exl3_moe(a):
    from ..models.hybrid import random_exl3_experts
    from ..ops import moe as moe_ops

    c = config3()
    E, H, I, k = c.moe.num_experts, c.hidden_size, c.moe.intermediate, c.moe.top_k
    # one rank's share: --tp splits every expert's intermediate, --ep keeps E / tp whole experts
    E_loc, I_loc = (E // a.tp, I) if a.ep else (E, I // a.tp)
    ex = random_exl3_experts(E_loc, H, I_loc, c.moe.exl3_bits_x2, c.moe.exl3_codebook,
                             WeightInit(0, "cuda", "local"), 1, 0, 0.0)
    if a.ep and a.tp > 1:
        emap = torch.full((E,), -1, dtype=torch.int32)
        emap[:E_loc] = torch.arange(E_loc, dtype=torch.int32)
        ex.expert_map = emap.cuda()
    x = torch.randn(a.tokens, H, device="cuda", dtype=torch.bfloat16)
    ids, w = _route(a.tokens, E, k, "cuda")
    used = int(torch.unique(ids[ids < E_loc] if a.ep else ids).numel())
    nbytes = used * 3 * H * I_loc * c.moe.exl3_bits_x2 / 16  # trellis bits of the touched experts
    pairs = int((ids < E_loc).sum()) if a.ep else a.tokens * k
    us = time_us(lambda: moe_ops.exl3_moe(x, ids, w, ex), a.iters)
    return _report("exl3_moe", us, nbytes, 2.0 * pairs * 3 * H * I_loc, tokens=a.tokens, experts_touched=used,
                   tp=a.tp, ep=a.ep)


def bench_marlin_moe(a):
    from ..models.marlin_experts import random_marlin_experts
    from ..ops.dequant import marlin_moe

    c = config4()
    E, H, I, k = c.moe.num_experts, c.hidden_size, c.moe.intermediate, c.moe.top_k
    ex = random_marlin_experts(E, H, I, WeightInit(0, "cuda", "local"), 1, 0)
    x = torch.randn(a.tokens, H, device="cuda", dtype=torch.bfloat16)
    ids, w = _route(a.tokens, E, k, "cuda")
    used = int(torch.unique(ids).numel())
    nbytes = used * 3 * H * I * (0.5 + 2 / 128)  # int4 codes + bf16 group scales
    us = time_us(lambda: marlin_moe(x, ids, w, ex), a.iters)
    return _report("marlin_moe", us, nbytes, 2.0 * a.tokens * k * 3 * H * I, tokens=a.tokens, experts_touched=used)


def bench_fp8_linear(a):
    from ..formats import fp8 as f8
    from ..ops.dequant import Fp8Linear, fp8_linear

    w = torch.randn(a.n, a.k) * a.k ** -0.5
    q, s = f8.quantize(w)
    lin = Fp8Linear(q.cuda(), s.cuda())
    x = torch.randn(a.m, a.k, device="cuda", dtype=torch.bfloat16)
    us = time_us(lambda: fp8_linear(x, lin), a.iters)
    return _report("fp8_linear", us, a.n * a.k + 2 * (a.m * a.k + a.m * a.n), 2.0 * a.m * a.n * a.k, m=a.m, n=a.n,
                   k=a.k)


def _paged_ctx(B, ctx, dev, mla_layer=None, kda_layer=None, kda_shapes=None):
    nb = (ctx + 63) // 64
    bt = torch.arange(B * nb, dtype=torch.int32, device=dev).view(B, nb) + 1
    pos = torch.full((B,), ctx - 1, dtype=torch.int32, device=dev)
    slots = (bt[:, -1].long() * 64 + (ctx - 1) % 64)
    caches, states = {}, {}
    rows = (B * nb + 1) * 64
    if mla_layer is not None:
        g = torch.Generator(device=dev).manual_seed(1)
        lat = torch.randn(rows, 576, device=dev, dtype=torch.bfloat16, generator=g)
        idx_k = torch.randint(0, 120, (rows, 128), dtype=torch.uint8, device=dev, generator=g)  # finite e4m3 codes
        idx_s = torch.rand(rows, device=dev, generator=g) * 0.1 + 0.01
        caches[0] = (lat, idx_k, idx_s)
    if kda_shapes is not None:
        rec_shape, conv_shape = kda_shapes
        states[0] = (torch.zeros(B + 1, *rec_shape, device=dev), torch.zeros(B + 1, *conv_shape, device=dev,
                                                                              dtype=torch.bfloat16))
    return StepContext(positions=pos, num_tokens=B, slot_mapping=slots, token_seq=torch.arange(B, dtype=torch.int32,
                                                                                                 device=dev),
                       ctx_lens=pos + 1, block_table=bt, max_ctx=ctx,
                       cu_seqlens=torch.arange(B + 1, dtype=torch.int32, device=dev),
                       kda_slots=torch.arange(1, B + 1, dtype=torch.int32, device=dev),
                       has_init=torch.ones(B, dtype=torch.int32, device=dev), mla_caches=caches, kda_states=states,
                       scores_buf=torch.empty(B, ctx, device=dev))


def bench_mla_decode(a):
    c = config2_layer()
    layer = MLAAttention(c, WeightInit(0, "cuda", "local"), 1, 0)
    ctx = _paged_ctx(a.tokens, a.ctx, "cuda", mla_layer=layer)
    x = torch.randn(a.tokens, c.hidden_size, device="cuda", dtype=torch.bfloat16)
    topk = c.mla.index_topk
    # bytes: selected latent rows + indexer keys over the context + the layer's weights
    wbytes = sum(p.numel() * p.element_size() for p in layer.parameters())
    nbytes = a.tokens * (min(topk, a.ctx) * 576 * 2 + a.ctx * (128 + 4)) + wbytes
    with torch.inference_mode():
        us = time_us(lambda: layer(x, ctx, 0), a.iters)
    return _report("mla_decode", us, nbytes, tokens=a.tokens, ctx=a.ctx, topk=topk, heads=c.mla.num_heads)


def bench_attn(a):
    """The sparse-attention kernel alone: --tokens queries of --heads heads, each attending to --topk
    gathered rows of a --ctx-row cache (random rows, so every gather is a separate line).  --dim 576:
    MLA latent + RoPE rows; 512: DeepSeek-V4.1 rows (K = V) with per-head sinks (--sink)."""
    from ..ops import mla as mla_ops

    T, nh, cnt, D = a.tokens, a.heads, min(a.topk, a.ctx), a.dim
    g = torch.Generator(device="cuda").manual_seed(0)
    q = (torch.randn(T, nh, D, device="cuda", generator=g) * 0.3).to(torch.bfloat16)
    cache = torch.randn(a.ctx, D, device="cuda", generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(a.ctx, device="cuda", generator=g)[:a.topk] for _ in range(T)]).int()
    counts = torch.full((T,), cnt, dtype=torch.int32, device="cuda")
    splits = a.splits or mla_ops.pick_splits(T, nh, a.topk)
    out = torch.empty(T, nh, 512, dtype=torch.bfloat16, device="cuda")
    sink = torch.randn(nh, device="cuda", generator=g) if a.sink else None
    status = _ext.status_word(q.device)

    def call():
        _ext.ops().mla_sparse_attention(q, cache, idx, counts, D ** -0.5, splits, out, None, status, sink)

    us = time_us(call, a.iters)
    nbytes = T * cnt * D * 2 + T * nh * (D + 512) * 2
    flops = 2.0 * T * nh * cnt * (D + 512)
    return _report("attn", us, nbytes, flops, tokens=T, heads=nh, count=cnt, splits=splits, dim=D)


def bench_ple_decode(a):
    """EXL3 PLE row decode: --tokens rows of --dim channels at --bits bits, 4 heads."""
    from ..formats import ple as fple

    n, dim, bits = a.tokens, a.dim, a.bits
    t = fple.random_table(heads=4, vocab=max(n, 64), dim=dim, bits=bits)
    rows = t["trellis"][:n].cuda()
    ids = torch.arange(n, device="cuda")
    args = [t[k].cuda() for k in ("head_bias", "head_offsets", "head_vocab_sizes")]
    out = torch.empty(n, dim, dtype=torch.bfloat16, device="cuda")
    us = time_us(lambda: _ext.ops().ple_decode(rows, ids, *args, 0, 1 << 40, bits, None, out), a.iters)
    nbytes = rows.numel() * 2 + out.numel() * 2
    return _report("ple_decode", us, nbytes, rows=n, dim=dim, bits=bits)


def bench_kda_decode(a):
    c = config3()
    layer = KDAAttention(c, WeightInit(0, "cuda", "local"), 1, 0)
    H, D = c.kda.num_heads, c.kda.head_dim
    shapes = ((H, D, D), (3 * H * D, 3))
    ctx = _paged_ctx(a.tokens, 64, "cuda", kda_shapes=shapes)
    x = torch.randn(a.tokens, c.hidden_size, device="cuda", dtype=torch.bfloat16)
    wbytes = sum(p.numel() * p.element_size() for p in layer.parameters())
    nbytes = a.tokens * H * D * D * 4 * 2 + wbytes  # fp32 state read + written, weights
    with torch.inference_mode():
        us = time_us(lambda: layer(x, ctx, 0), a.iters)
    return _report("kda_decode", us, nbytes, seqs=a.tokens, heads=H)


def bench_kda_prefill(a):
    """The KDA layer core (conv, gates, recurrence, gated norm) over a prefill batch of --seqs prompts of
    --tokens tokens: the kernel time of `ops.kda.kda_forward` in the mode --mode.  FLOPs are those of the
    chunked form (per 64-token chunk: the decayed key/query products, the state products, the inverse
    application, the output and state updates, in bf16 MMA passes)."""
    from .. import envs
    from ..ops import kda as kda_ops

    os.environ["VLLM_B200_KDA_PREFILL"] = a.mode
    envs._cache.clear()
    c = config3()
    H, D = c.kda.num_heads, c.kda.head_dim
    S, L = a.seqs, a.tokens
    T = S * L
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = torch.randn(T, 3 * H * D, device=dev, generator=g).bfloat16()
    g_raw = torch.randn(T, H * D, device=dev, generator=g).bfloat16()
    beta = torch.randn(T, H, device=dev, generator=g).bfloat16()
    g2 = torch.randn(T, H * D, device=dev, generator=g).bfloat16()
    conv_w = (torch.randn(3 * H * D, 4, device=dev, generator=g) * 0.5).bfloat16()
    a_log = torch.randn(H, device=dev, generator=g) * 0.5
    norm_w = torch.ones(D, device=dev, dtype=torch.bfloat16)
    state = torch.zeros(S + 1, H, D, D, device=dev)
    conv = torch.zeros(S + 1, 3 * H * D, 3, device=dev, dtype=torch.bfloat16)
    cu = torch.arange(0, T + 1, L, dtype=torch.int32, device=dev)
    idx = torch.arange(1, S + 1, dtype=torch.int32, device=dev)
    init = torch.zeros(S, dtype=torch.int32, device=dev)
    out = torch.empty(T, H * D, device=dev, dtype=torch.bfloat16)

    def call():
        kda_ops.kda_forward(qkv, g_raw, beta, g2, cu, idx, init, conv, conv_w, None, a_log, None, c.kda.lower_bound,
                            norm_w, state, out=out)

    us = time_us(call, a.iters)
    chunks = S * H * ((L + 63) // 64)
    flops = chunks * 2.0 * (128 * 160 * 128 + 2 * 128 * 128 * 128 + 3 * 128 * 128 * 64 + 2 * 128 * 128 * 64
                            + 3 * 128 * 128 * 64)
    nbytes = T * (3 * H * D * 2 + H * D * 2 * 2 + H * 2) + T * H * D * 2 + S * H * D * D * 4
    return _report("kda_prefill", us, nbytes, flops, mode=a.mode, seqs=S, tokens=L, heads=H,
                   us_per_token_head=round(us / (T * H), 5))


def bench_mhc(a):
    """One mHC boundary (post + Sinkhorn coefficients + collapse + RMSNorm): --tokens tokens, 4
    streams of --dim hidden."""
    from ..ops import mhc as mhc_ops

    T, n, d = a.tokens, 4, a.dim
    g = torch.Generator(device="cuda").manual_seed(0)
    N = 2 * n + n * n
    x = torch.randn(T, d, device="cuda", generator=g).bfloat16()
    H = torch.randn(T, n, d, device="cuda", generator=g).bfloat16()
    post = torch.rand(T, n, device="cuda", generator=g)
    comb = torch.rand(T, n, n, device="cuda", generator=g)
    fn = torch.randn(N, n * d, device="cuda", generator=g) * (n * d) ** -0.5
    scale = torch.ones(3, device="cuda")
    base = torch.zeros(N, device="cuda")
    w = torch.ones(d, device="cuda", dtype=torch.bfloat16)

    def call():
        mhc_ops.post_pre(x, H, post, comb, fn, scale, base, w, rms_eps=1e-6, eps=1e-6, post_mult=2.0, iters=20,
                         norm_eps=1e-6)

    us = time_us(call, a.iters)
    nbytes = T * d * 2 + 2 * T * n * d * 2 + N * n * d * 4 + T * d * 2
    return _report("mhc", us, nbytes, tokens=T, dim=d)


OPS = {"gemm": bench_gemm, "exl3_moe": bench_exl3_moe, "marlin_moe": bench_marlin_moe, "fp8_linear": bench_fp8_linear,
       "mla_decode": bench_mla_decode, "kda_decode": bench_kda_decode, "kda_prefill": bench_kda_prefill,
       "attn": bench_attn,
       "ple_decode": bench_ple_decode, "mhc": bench_mhc}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("op", choices=sorted(OPS))
    ap.add_argument("--tokens", type=int, default=128)
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--m", type=int, default=128)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--heads", type=int, default=128, help="attn: query heads")
    ap.add_argument("--tp", type=int, default=1, help="exl3_moe: the share of one rank of a group this size")
    ap.add_argument("--ep", action="store_true", help="exl3_moe: experts split whole (expert parallel)")
    ap.add_argument("--topk", type=int, default=2048, help="attn: gathered rows per query")
    ap.add_argument("--splits", type=int, default=0, help="attn: position splits (0: the launcher's choice)")
    ap.add_argument("--dim", type=int, default=576, help="attn: row width (576 MLA, 512 DeepSeek-V4.1); "
                                                         "ple_decode: channels")
    ap.add_argument("--sink", action="store_true", help="attn: per-head softmax sinks")
    ap.add_argument("--bits", type=int, default=4, help="ple_decode: bits per channel")
    ap.add_argument("--profile", action="store_true", help="print a per-kernel table of one call (torch profiler)")
    ap.add_argument("--graph", action="store_true", help="time --iters calls replayed from one CUDA graph")
    ap.add_argument("--seqs", type=int, default=8, help="kda_prefill: prompts")
    ap.add_argument("--mode", default="chunked", choices=["chunked", "recurrent"], help="kda_prefill: path")
    a = ap.parse_args(argv)
    global _PROFILE, _GRAPH
    _PROFILE = a.profile
    _GRAPH = a.graph
    pstate.set_state(pstate.ParallelState())
    OPS[a.op](a)
    _ext.check_status(torch.device("cuda"))


if __name__ == "__main__":
    main()
