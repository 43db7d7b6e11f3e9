"""Offline generation with the engine's public API, on CPU (fp32 oracle path) or one B200.

    python examples/offline_generate.py                      # tiny hybrid KDA/MLA model, CPU
    python examples/offline_generate.py --device cuda        # the same on a GPU (CUDA graphs)
    python examples/offline_generate.py --model dsv4         # DeepSeek-V4.1-style attention + mHC
    python examples/offline_generate.py --spec dflash -k 3   # DFlash block drafts, greedy verification
    python examples/offline_generate.py --spec mtp -k 2 --temperature 0.7

Weights are random (no checkpoint is read), so the tokens are meaningless; the point is the call
sequence a user makes: build an EngineConfig, construct LLM, call generate.
"""

import argparse

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny, tiny_deepseek, tiny_dsv4
from vllm_cmp170hx_b200.engine.llm_engine import LLM
from vllm_cmp170hx_b200.engine.request import SamplingParams


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--model", choices=["hybrid", "deepseek", "dsv4"], default="hybrid")
    ap.add_argument("--spec", choices=["none", "mtp", "dflash"], default="none")
    ap.add_argument("-k", type=int, default=2, help="drafts per step")
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--depth-policy", default="", help="dspark-depth-policy/1 file (per-request verify depth)")
    a = ap.parse_args()
    model = {"hybrid": lambda: tiny(layers=4, experts=8, expert_format="exl3"),
             "deepseek": lambda: tiny_deepseek(layers=3),
             "dsv4": lambda: tiny_dsv4(layers=3)}[a.model]()
    k = 0 if a.spec == "none" else a.k
    if a.spec == "mtp":
        model.num_mtp_layers = 1
    cfg = EngineConfig(model=model,
                       scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=256, max_model_len=512,
                                                 num_speculative_tokens=k,
                                                 spec_method=a.spec if a.spec != "none" else "mtp",
                                                 depth_policy=a.depth_policy),
                       cache=CacheConfig(num_blocks=64), device=a.device, enforce_eager=a.device == "cpu")
    llm = LLM(cfg)
    prompts = [[1, 2, 3, 4, 5], list(range(100, 160))]
    for out in llm.generate(prompts, SamplingParams(max_tokens=8, temperature=a.temperature)):
        print(out.request_id, out.output_token_ids, out.finish_reason)
    spec = llm.engine.runner.spec
    if spec is not None:
        print(f"drafts proposed {spec.stats['proposed']}, accepted {spec.stats['accepted']}")


if __name__ == "__main__":
    main()
