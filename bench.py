"""Headline benchmark: decode output tokens/s and p50 TPOT of the hybrid
KDA/sparse-MLA MoE model (48 layers, hidden 2304, 32 heads,
256 experts top-8 + 1 shared, EXL3 4-bit experts) serving 128 concurrent
requests of 2048-token prompts, tensor parallel over N GPUs of one node.

    python bench.py --gpus N --steps K --warmup W            # this framework
    python bench.py --impl reference ...                      # the reference arm
    torchrun --nproc-per-node N bench.py --gpus N ...         # N > 1

Protocol: random-init weights and random token ids (no checkpoints, no
datasets); all 128 prompts are prefilled through the engine (untimed), then
W decode steps warm up (CUDA graphs captured) and K decode steps are timed.
Each decode step reads every expert weight (~43.5 GB at TP1), far more than
the 126 MB L2, so no flush is needed between steps.

* value       = 128 * K / (sum of per-step device time) -- CUDA events around
                each step's graph replay on the launching stream, max over ranks;
* e2e.value   = 128 * K / (wall time of K `LLMEngine.step()` calls): includes
                scheduling, the pinned host->device copy of the step inputs and
                the device->host read of the sampled tokens, barrier + sync on
                both sides, max over ranks;
* p50_tpot_ms = median per-step e2e time (every running request gets one
                token per step).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode output tok/s (box, max over ranks) at 1/2/4/8 B200; p50 TPOT"
MODEL_DESC = {
    3: "hybrid KDA/sparse-MLA MoE, 48 layers (36 KDA : 12 MLA), hidden 2304, 32 heads, 256 experts top-8 + 1 shared, "
       "expert intermediate 1024, EXL3 4-bit experts, vocab 163840",
    4: "DeepSeek-style sparse-MLA MoE, 43 layers (3 dense FFN 12288), hidden 4096, 128 heads, 256 experts top-8 + 1 "
       "shared, expert intermediate 1536, Marlin int4 g128 experts, fp8 128x128 block-scaled attention, vocab 129280",
    5: "config 4's model with a 1-layer MTP head drafting 3 tokens, rejection sampling at temperature 0.7",
}


def reference_unavailable(args, reason: str) -> None:
    if int(os.environ.get("RANK", "0")) != 0:  # one line per job (rank 0), as the product arm
        return
    print(json.dumps({"impl": "reference", "unavailable": reason, "metric": METRIC, "n_gpus": args.gpus}))


def sample_clocks_start(index: int):
    try:
        return subprocess.Popen(
            ["nvidia-smi", f"--id={index}",
             "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap",
             "--format=csv,noheader,nounits", "-lms", "200"],
            stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except OSError:
        return None


def sample_clocks_stop(proc) -> dict:
    if proc is None:
        return {}
    proc.terminate()
    try:
        out, _ = proc.communicate(timeout=5)
    except subprocess.TimeoutExpired:
        proc.kill()
        out, _ = proc.communicate()
    sm, mx, reasons = [], 0.0, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in out.strip().splitlines():
        f = [x.strip() for x in line.split(",")]
        if len(f) < 7:
            continue
        try:
            sm.append(float(f[0]))
            mx = max(mx, float(f[1]))
        except ValueError:
            continue
        for n, v in zip(names, f[3:7]):
            if v.lower() == "active":
                reasons.add(n)
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None, "reasons": sorted(reasons),
            "samples": len(sm)}


def count_own_kernels(engine, steps: int, table: bool = False) -> int:
    """Kernels of this package's extension (namespace b200) launched by one
    eager decode step, times the timed steps (graph replays run the same set).
    With `table`, print that step's per-kernel device times to stderr (a
    profiler view for guidance, never a reported number)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    r = engine.runner
    saved = r.cfg.enforce_eager
    r.cfg.enforce_eager = True
    try:
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            engine.step()
            torch.cuda.synchronize()
    finally:
        r.cfg.enforce_eager = saved
    n = sum(1 for e in prof.events() if e.device_type.name == "CUDA" and "b200" in e.name)
    if table:
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=30, max_name_column_width=90),
              file=sys.stderr, flush=True)
    return n * steps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--output", type=int, default=512)
    ap.add_argument("--prefill-chunk", type=int, default=16384)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--nccl-baseline", action="store_true", help="TP collectives on NCCL only (baseline path)")
    ap.add_argument("--synthetic-context", action="store_true",
                    help="no prefill: every request starts decoding at position --prompt over cache rows and "
                         "recurrent states filled with random values (N(0,1) KV rows), so long contexts and "
                         "large batches are measurable")
    ap.add_argument("--no-sp", action="store_true", help="expert parallel with replicated tokens and all-reduces "
                                                        "instead of the sequence-parallel layout")
    ap.add_argument("--profile", action="store_true", help="print rank 0's per-kernel times of one eager step")
    ap.add_argument("--eager", action="store_true", help="no CUDA graphs (debugging)")
    ap.add_argument("--sync-scheduling", action="store_true", help="read every step's tokens back before "
                    "scheduling the next (default: decode steps are scheduled and launched one step ahead)")
    ap.add_argument("--ep", action="store_true", help="(default for N > 1) routed experts split whole over the "
                                                      "ranks (EP=N)")
    ap.add_argument("--moe-tp", action="store_true", help="config 3 at N > 1: split every routed expert by "
                                                          "intermediate columns instead (tensor-parallel MoE)")
    ap.add_argument("--emulate-tp", type=int, default=0,
                    help="1 GPU standing in for rank 0 of a TP group of this size (collectives return local data): "
                         "prints the per-rank step time of the compute kernels only, never a bench line")
    ap.add_argument("--config", type=int, default=3, choices=[3, 4, 5],
                    help="BASELINE config: 3 = hybrid KDA/MLA EXL3 MoE at TP=N (headline); "
                         "4 = DeepSeek-style Marlin MoE, experts EP=N, attention TP=N; "
                         "5 = config 4's model at PP2 x TP(N/2) with MTP speculative decoding (3 drafts, "
                         "temperature 0.7), 512 requests with context lengths uniform in [512, 8192], output 1024 "
                         "(synthetic context: decoding starts at each request's context length)")
    args = ap.parse_args()
    if args.config == 5:
        # the BASELINE workload of config 5 unless given explicitly
        if "--batch" not in sys.argv:
            args.batch = 512
        if "--output" not in sys.argv:
            args.output = 1024
        if "--prompt" not in sys.argv:
            args.prompt = 8192  # the longest context; each request draws its own in [512, 8192]
        args.synthetic_context = True

    if args.impl == "reference":
        ref = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref, "vllm_sm80")):
            reference_unavailable(args, "reference not installed under baseline/_ref")
            return
        # the reference's own entry to the config-3 model: its GLM-5.3 model class (a vLLM plugin class)
        sys.path.insert(0, ref)
        mod = "vllm_sm80.models.glm5next.sm80_model" if args.config == 3 else "vllm_sm80.models.deepseek_v41.sm80_model"
        try:
            import importlib

            importlib.import_module(mod)
        except Exception as e:  # noqa: BLE001 -- whatever stops the reference is the reason
            reference_unavailable(args, f"import {mod} fails ({type(e).__name__}: {str(e)[:120]}): the reference "
                                        "is a vLLM plugin whose model classes subclass upstream vLLM packages "
                                        "(vllm/models/glm5next, deepseek_v41, qwen4_exp, model-runner V2) that the "
                                        "image's vLLM 0.22 does not ship, and its native kernels build for sm_80 only")
            return
        reference_unavailable(args, "the reference imports but has no sm_100 kernels (its extensions build for "
                                    "sm_80 only)")
        return

    import torch
    import torch.distributed as dist

    from vllm_cmp170hx_b200.config import (CacheConfig, EngineConfig, ParallelConfig, SchedulerConfig, config3,
                                           config4)
    from vllm_cmp170hx_b200.engine.llm_engine import LLMEngine
    from vllm_cmp170hx_b200.engine.request import SamplingParams
    from vllm_cmp170hx_b200.parallel import state as pstate

    world = int(os.environ.get("WORLD_SIZE", "1"))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    if args.emulate_tp:
        assert world == 1, "--emulate-tp runs in one process"
        st = pstate.emulate(args.emulate_tp)
        args.gpus = args.emulate_tp
        args.nccl_baseline = True  # no symmetric-memory kernels without peers
    else:
        pp = 2 if (args.config == 5 and args.gpus >= 2) else 1
        st = pstate.init(tp_size=args.gpus // pp, pp_size=pp, timeout_s=600)
    # routed experts: whole experts per rank (EP) unless asked otherwise; attention stays tensor parallel
    args.ep = args.config in (4, 5) or args.ep or (args.gpus > 1 and not args.moe_tp)
    dev = st.device
    model_cfg = config3() if args.config == 3 else config4()
    total_len = args.prompt + args.output + 64
    g_len = torch.Generator().manual_seed(args.seed + 1)
    ctx_lens = ([int(x) for x in torch.randint(512, args.prompt + 1, (args.batch,), generator=g_len)]
                if args.config == 5 else [args.prompt] * args.batch)
    spec_k = 3 if args.config == 5 else 0
    blocks = sum((L + args.output + 64 + 63) // 64 for L in ctx_lens) + 1
    cfg = EngineConfig(model=model_cfg,
                       parallel=ParallelConfig(tensor_parallel_size=st.tp_size, pipeline_parallel_size=st.pp_size,
                                               fused_comm=not args.nccl_baseline,
                                               expert_parallel=args.ep, sequence_parallel=not args.no_sp),
                       scheduler=SchedulerConfig(max_num_seqs=args.batch, max_num_batched_tokens=args.prefill_chunk,
                                                 max_model_len=total_len, max_num_partial_prefills=args.batch,
                                                 num_speculative_tokens=spec_k, spec_method="mtp",
                                                 async_scheduling=not args.sync_scheduling),
                       cache=CacheConfig(num_blocks=blocks),
                       seed=args.seed, device="cuda", enforce_eager=args.eager,
                       cuda_graph_batch_sizes=[args.batch])
    t0 = time.time()
    engine = LLMEngine(cfg)
    fused = False
    if args.gpus > 1 and not args.nccl_baseline and not args.emulate_tp:
        try:
            from vllm_cmp170hx_b200.parallel import symm
            fused = symm.enable_for_engine(engine)
        except ImportError:
            fused = False
    from vllm_cmp170hx_b200.parallel import comm as pcomm

    spt = pcomm._FUSED["sp"]
    layout = ("sequence-parallel (all-gather + reduce-scatter around attention, dispatch / combine around the "
              "experts)" if spt is not None else "replicated tokens (all-reduce)")
    transport = ("fused NVLink peer-store kernels" if (fused and (spt is None or spt.fused)) else "NCCL")
    torch.cuda.synchronize()
    t_load = time.time() - t0
    g = torch.Generator().manual_seed(args.seed)
    V = model_cfg.vocab_size
    if args.synthetic_context:
        engine.runner.fill_caches_random(args.seed)
    temperature = 0.7 if args.config == 5 else 0.0
    for i in range(args.batch):
        prompt = torch.randint(0, V, (ctx_lens[i],), generator=g).tolist()
        engine.add_request(prompt, SamplingParams(max_tokens=args.output, ignore_eos=True, temperature=temperature,
                                                  seed=args.seed + i), f"bench-{i}",
                           synthetic_prefix=ctx_lens[i] - 1 if args.synthetic_context else 0)
    # prefill (untimed): until every request has its first token
    t1 = time.time()
    while any(r.num_computed_tokens < r.num_prompt_tokens for r in engine.scheduler.running) or engine.scheduler.waiting:
        engine.step()
    torch.cuda.synchronize()
    t_prefill = time.time() - t1
    # device timing on from the warm-up on: with asynchronous scheduling the first timed call finishes the
    # step the last warm-up call launched
    engine.runner.time_device = True
    launches = count_own_kernels(engine, args.steps, table=args.profile and st.rank == 0)
    for _ in range(args.warmup):
        engine.step()
    clk = sample_clocks_start(dev.index or 0) if st.rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    dev_ms, e2e_ms = [], []
    h2d = d2h = 0
    reqs = list(engine.requests.values())
    emitted0 = sum(len(r.output_token_ids) for r in reqs)
    t_start = time.perf_counter()
    sync_each = engine.cfg.scheduler.async_scheduling is False
    for _ in range(args.steps):
        a = time.perf_counter()
        engine.step()
        if sync_each:
            torch.cuda.synchronize()
        # asynchronous scheduling: one call launches step n + 1 and returns step n's tokens, so the
        # interval between returns is the per-token time; the synchronize before the loop has finished
        # the step in flight from the warm-up, the one after it the step the last call launched, so the
        # region holds exactly `steps` steps of device work and emits `steps` tokens per request
        e2e_ms.append((time.perf_counter() - a) * 1e3)
        s = engine.runner.last_stats
        dev_ms.append(s.device_ms)
        h2d, d2h = s.h2d_bytes, s.d2h_bytes
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    wall = time.perf_counter() - t_start
    clocks = sample_clocks_stop(clk)
    tot = torch.tensor([sum(dev_ms), wall * 1e3], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    dev_total_ms, wall_ms = tot.tolist()
    # tokens actually emitted in the timed steps (a request that finished early, e.g. on a failed
    # input row, emits none, and the number says so)
    emitted = sum(len(r.output_token_ids) for r in reqs) - emitted0
    failed = sum(1 for r in reqs if r.status.name == "FINISHED_ERROR")
    toks = emitted
    value = toks / (dev_total_ms / 1e3)
    e2e_value = toks / (wall_ms / 1e3)
    if args.emulate_tp:
        print(json.dumps({"emulated_tp": args.emulate_tp, "config": args.config, "batch": args.batch,
                          "tokens_emitted": emitted, "requests_failed": failed,
                          "per_rank_compute_ms_per_step": round(dev_total_ms / args.steps, 3),
                          "p50_step_ms": round(statistics.median(e2e_ms), 3), "clocks": clocks}), flush=True)
        engine.runner.release_graphs()
        return
    if st.rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dev_total_ms / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "impl": "ours",
            "data": (f"synthetic: random token ids, random-init weights of the config-{args.config} architecture"
                     + ("; context rows and recurrent states random (no prefill)" if args.synthetic_context
                        else "; prompts prefilled through the engine")),
            "config": {"model": MODEL_DESC[args.config],
                       "global_batch": args.batch, "seq_len": args.prompt, "output_len": args.output,
                       "parallelism": (f"pp{st.pp_size}+tp{st.tp_size}" + (f"+ep{st.tp_size}" if args.ep else "")
                                       if st.pp_size > 1 else
                                       f"ep{args.gpus}+attn-tp{args.gpus}" if args.ep and args.gpus > 1
                                       else f"tp{args.gpus}"),
                       **({"speculative": "MTP, 3 drafts, temperature 0.7",
                           "context_lens": "uniform [512, %d]" % args.prompt} if args.config == 5 else {}),
                       "collectives": ("none" if args.gpus == 1 else f"{transport}; {layout}"),
                       "l2": "no flush: each step streams the expert weights (GBs per GPU) >> 126 MB L2"},
            "p50_tpot_ms": round(statistics.median(e2e_ms), 3),
            "clocks": clocks,
            "e2e": {"value": round(e2e_value, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "api": "LLMEngine.step()"},
            "gpu_launches": launches,
            "tokens_emitted": emitted, "requests_failed": failed,
            "timing": {"load_s": round(t_load, 1), "prefill_s": round(t_prefill, 1)},
        }), flush=True)
    engine.runner.release_graphs()
    if world > 1:
        dist.barrier()
        pstate.destroy()


if __name__ == "__main__":
    main()
