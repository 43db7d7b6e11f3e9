"""Loading by upstream tensor names: a model exported under Hugging Face names and loaded into a
model drawn from another seed decodes exactly like the original, at TP1 and (gloo) TP2, for the
hybrid KDA / MLA model with EXL3 experts and for the DeepSeek-style model with fp8 attention."""

import json
import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from vllm_cmp170hx_b200.config import (CacheConfig, EngineConfig, ParallelConfig, SchedulerConfig, tiny, tiny_deepseek,
                                       tiny_dsv4)

PROMPTS = [[(7 * i + 3 * j) % 500 for j in range(6 + 11 * i)] for i in range(3)]


def _cfg(kind, tp=1):
    if kind == "dsv4":
        m = tiny_dsv4(layers=3, experts=4, hidden=256, vocab=512)
        m.moe.expert_format = "bf16"
    elif kind == "deepseek":
        m = tiny_deepseek(layers=2, experts=4, hidden=256, vocab=512)
        m.mla.num_heads = 4
        m.moe.expert_format = "bf16"
    else:
        m = tiny(layers=4, experts=4, hidden=256, expert_format="exl3")
        m.moe.intermediate = 256
        m.moe.shared_intermediate = 256
    return EngineConfig(model=m, parallel=ParallelConfig(tensor_parallel_size=tp),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=256),
                        cache=CacheConfig(num_blocks=32), device="cpu", enforce_eager=True)


def _gen(cfg, model):
    from vllm_cmp170hx_b200.engine.llm_engine import LLM
    from vllm_cmp170hx_b200.engine.request import SamplingParams

    return [o.output_token_ids for o in LLM(cfg, model).generate(PROMPTS, SamplingParams(max_tokens=4))]


@pytest.mark.parametrize("kind", ["hybrid", "deepseek", "dsv4"])
def test_export_then_load_by_upstream_names(kind, tmp_path):
    from safetensors.torch import save_file

    from vllm_cmp170hx_b200 import hf_loader
    from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    cfg = _cfg(kind)
    src = HybridForCausalLM(cfg.model, "cpu", seed=1)
    ref = _gen(cfg, src)
    tensors = hf_loader.export_hf(src)
    first = {"hybrid": "self_attn.q_proj.weight", "deepseek": "self_attn.q_a_proj.weight", "dsv4": "attn.wq_a.weight"}
    assert "model.layers.0." + first[kind] in tensors
    if kind == "dsv4":
        assert "model.layers.0.hc_attn_fn" in tensors and "model.hc_head_fn" in tensors
        assert "model.layers.1.attn.compressor.wgate.weight" in tensors  # the ratio-2 layer
    save_file({k: v.contiguous() for k, v in tensors.items()}, str(tmp_path / "model.safetensors"))
    dst = HybridForCausalLM(cfg.model, "cpu", seed=2)
    assert _gen(cfg, dst) != ref
    hf_loader.load_hf(dst, str(tmp_path))
    assert _gen(cfg, dst) == ref
    with pytest.raises(hf_loader.MissingTensor):
        hf_loader.load_hf(dst, {k: v for k, v in tensors.items() if "lm_head" not in k})


def _worker(rank, world, port, path, kind, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from vllm_cmp170hx_b200 import hf_loader
    from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.init(tp_size=world, device="cpu", timeout_s=120)
    cfg = _cfg(kind, world)
    model = HybridForCausalLM(cfg.model, "cpu", seed=3)
    hf_loader.load_hf(model, path)
    toks = _gen(cfg, model)
    if rank == 0:
        with open(out, "w") as f:
            json.dump(toks, f)
    pstate.destroy()


@pytest.mark.parametrize("kind", ["hybrid", "deepseek", "dsv4"])
def test_tp2_load_matches_tp1(kind, tmp_path):
    from safetensors.torch import save_file

    from vllm_cmp170hx_b200 import hf_loader
    from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    cfg = _cfg(kind)
    src = HybridForCausalLM(cfg.model, "cpu", seed=1)
    ref = _gen(cfg, src)
    save_file({k: v.contiguous() for k, v in hf_loader.export_hf(src).items()}, str(tmp_path / "model.safetensors"))
    out = str(tmp_path / "toks.json")
    port = 29800 + os.getpid() % 150
    mp.start_processes(_worker, args=(2, port, str(tmp_path), kind, out), nprocs=2, join=True, start_method="spawn")
    with open(out) as f:
        assert json.load(f) == ref
