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


def _fresh(cfg, seed):
    from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    return HybridForCausalLM(cfg, "cpu", seed=seed, init_mode="sliced")


@pytest.mark.parametrize("which", ["qwen", "dsv4_engram"])
def test_roundtrip_new_families_strict(which):
    """The Qwen-style family (gated delta net under linear_attn with rows grouped per key head, gated
    attention, shared_expert, PLE projection) and the Engram layers export under upstream names and load
    back exactly, with every tensor consumed (strict inventory)."""
    from vllm_cmp170hx_b200.config import tiny_dsv4, tiny_qwen
    from vllm_cmp170hx_b200.hf_loader import export_hf, load_hf

    cfg = tiny_qwen(layers=4) if which == "qwen" else tiny_dsv4(layers=3, engram=True)
    a = _fresh(cfg, 1)
    tensors = export_hf(a)
    if which == "qwen":  # the upstream name of the singular shared expert
        tensors = {k.replace("shared_experts.", "shared_expert."): v for k, v in tensors.items()}
    b = _fresh(cfg, 2)
    inv = load_hf(b, tensors, strict=True)
    assert inv["unused"] == [] and inv["consumed"] == len(tensors)
    for (n, x), (_, y) in zip(a.named_parameters(), b.named_parameters()):
        assert torch.equal(x, y), n


def test_unused_tensor_is_refused_and_hybrid_exl3_projection_decodes():
    from vllm_cmp170hx_b200.config import tiny_qwen
    from vllm_cmp170hx_b200.formats import exl3 as fx
    from vllm_cmp170hx_b200.hf_loader import UnusedTensors, export_hf, load_hf

    cfg = tiny_qwen(layers=4, ple=False)
    a = _fresh(cfg, 1)
    t = export_hf(a)
    with pytest.raises(UnusedTensors):
        load_hf(_fresh(cfg, 2), {**t, "model.layers.0.mystery.weight": torch.zeros(2)}, strict=True)
    # hybrid checkpoint: layer 0's out projection stored as an EXL3 matrix, selected by a module rule
    name = "model.layers.0.linear_attn.out_proj"
    w = t.pop(name + ".weight")
    m = fx.random_matrix(w.shape[1], w.shape[0], generator=torch.Generator().manual_seed(3))
    for part in ("trellis", "suh", "svh"):
        t[f"{name}.{part}"] = getattr(m, part)
    rules = {"rules": [{"match": r"^model\.layers\.0\.linear_attn\.out_proj$", "method": "exl3"}],
             "default": "unquantized"}
    b = _fresh(cfg, 2)
    inv = load_hf(b, t, strict=True, quantization_config={"module_quantization": rules, "codebook": "mul1"})
    assert inv["unused"] == []
    x = torch.randn(3, w.shape[1])
    got = x @ b.layer(0).attn.o_proj.weight.float().t()
    ref = fx.linear(x, m)
    assert ((got - ref).norm() / ref.norm()).item() < 1e-2
    # a module no rule covers, without a default, is refused
    with pytest.raises(ValueError, match="no module_quantization rule"):
        load_hf(_fresh(cfg, 2), t, quantization_config={"module_quantization": {"rules": rules["rules"]}})
