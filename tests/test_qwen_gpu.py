"""Qwen3-Next-style family on the GPU: the gated delta net (KDA recurrence kernel, gate mode 1) and the
gated attention kernels (prep, the dense mode of the block attention kernel, output gate) against the
fp32 definitions of the same ops on the CPU, and the model in the engine (logits against the CPU oracle
path, CUDA-graph decode equal to eager decode, greedy MTP speculative decoding equal to plain decoding)."""

import pytest
import torch

from vllm_cmp170hx_b200 import _ext
from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny_qwen
from vllm_cmp170hx_b200.engine.llm_engine import LLM, LLMEngine
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.ops import gqa as gqa_ops
from vllm_cmp170hx_b200.ops import kda as kda_ops
from vllm_cmp170hx_b200.oracle import kda as kda_ref
from vllm_cmp170hx_b200.oracle.mla import rope_cos_sin
from vllm_cmp170hx_b200.parallel import state as pstate

pytestmark = pytest.mark.gpu


def test_gdn_kernel_matches_oracle():
    g = torch.Generator().manual_seed(5)
    H, D = 3, 128
    HD = H * D
    lens = [9, 1, 70]
    T = sum(lens)
    cu = torch.tensor([0, 9, 10, 80], dtype=torch.int32)
    qkv = torch.randn(T, 3 * HD, generator=g).to(torch.bfloat16)
    a = torch.randn(T, H, generator=g).to(torch.bfloat16)
    b = torch.randn(T, H, generator=g).to(torch.bfloat16)
    z = torch.randn(T, HD, generator=g).to(torch.bfloat16)
    conv_w = (torch.randn(3 * HD, 4, generator=g) * 0.5).to(torch.bfloat16)
    a_log = torch.randn(H, generator=g) * 0.5
    dt_bias = torch.randn(H, generator=g) * 0.3
    norm_w = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    state = torch.randn(4, H, D, D, generator=g) * 0.05
    conv_state = torch.randn(4, 3 * HD, 3, generator=g).to(torch.bfloat16)
    idx = torch.tensor([3, 1, 0], dtype=torch.int32)
    has_init = torch.tensor([1, 0, 1], dtype=torch.int32)
    st_r, cs_r = state.clone(), conv_state.clone()
    ref = kda_ref.kda_layer(qkv, a, b, z, cu, st_r, cs_r, idx, has_init, conv_w, None, a_log, dt_bias, 0.0, norm_w,
                            eps=1e-6, gate_mode=1)
    st, cs = state.cuda(), conv_state.cuda()
    out = kda_ops.kda_forward(qkv.cuda(), a.cuda(), b.cuda(), z.cuda(), cu.cuda(), idx.cuda(), has_init.cuda(), cs,
                              conv_w.cuda(), None, a_log.cuda(), dt_bias.cuda(), 0.0, norm_w.cuda(), st, eps=1e-6,
                              gate_mode=1)
    torch.cuda.synchronize()
    _ext.check_status(torch.device("cuda"))
    rel = ((out.cpu().float() - ref).norm() / ref.norm()).item()
    print(f"gdn rel {rel:.2e}")
    assert rel < 1e-2, rel
    for slot in (3, 1, 0):
        assert (st[slot].cpu() - st_r[slot]).abs().max() < 1e-3
        assert torch.equal(cs[slot].cpu(), cs_r[slot])


@pytest.mark.parametrize("nh,nkv,lens,splits", [(4, 2, [5, 300], None), (8, 1, [1, 1, 129], 3),
                                                (16, 2, [700], 1), (2, 2, [64, 65], 2)])
def test_gqa_kernels_match_cpu(nh, nkv, lens, splits):
    g = torch.Generator().manual_seed(7)
    T = sum(lens)
    nb = sum((n + 63) // 64 for n in lens) + 2
    proj = (torch.randn(T, nh * 512 + nkv * 512, generator=g) * 0.5).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(256, generator=g)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(256, generator=g)).to(torch.bfloat16)
    cs = rope_cos_sin(2048, 64, 1e7)
    # sequences on shuffled blocks
    perm = torch.randperm(nb, generator=g).tolist()
    maxb = max((n + 63) // 64 for n in lens)
    bt = torch.zeros(len(lens), maxb, dtype=torch.int32)
    pos, tseq, k = [], [], 0
    for s, n in enumerate(lens):
        for j in range((n + 63) // 64):
            bt[s, j] = perm[k]
            k += 1
        pos += list(range(n))
        tseq += [s] * n
    pos = torch.tensor(pos, dtype=torch.int32)
    tseq = torch.tensor(tseq, dtype=torch.int32)
    slots = bt[tseq.long(), (pos // 64).long()].long() * 64 + (pos % 64).long()
    G = nh // nkv
    res = {}
    for dev in ("cpu", "cuda"):
        cache = torch.zeros(nb * 64 * nkv, 512, dtype=torch.bfloat16, device=dev)
        q = torch.empty(T * nkv, G, 512, dtype=torch.bfloat16, device=dev)
        d = lambda x: x.to(dev)  # noqa: E731
        gqa_ops.prep(d(proj), nh, nkv, d(qw), d(kw), 1e-6, d(pos), d(cs), d(slots), q, cache)
        o = gqa_ops.attention(q, cache, d(pos + 1), d(tseq), d(bt), nkv, max(lens), splits=splits)
        y = gqa_ops.gate(o, d(proj), nh)
        if dev == "cuda":
            torch.cuda.synchronize()
            _ext.check_status(torch.device("cuda"))
        res[dev] = (q.cpu(), cache.cpu(), o.cpu()[..., 256:].float(), y.cpu().float())
    qc, cc, oc, yc = res["cpu"]
    qg, cg, og, yg = res["cuda"]
    assert (qg.float() - qc.float()).abs().max() < 2e-2
    used = (slots[:, None] * nkv + torch.arange(nkv)[None]).reshape(-1)
    assert (cg[used].float() - cc[used].float()).abs().max() < 2e-2
    err = (og - oc).abs().max().item()
    print(f"gqa attention max err {err:.2e}")
    assert err < 3e-2, err
    rel = ((yg - yc).norm() / yc.norm()).item()
    assert rel < 1e-2, rel


def _cfg(device, eager=True, k=0, budget=512):
    m = tiny_qwen(layers=4)
    m.num_mtp_layers = 1 if k else 0
    return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=budget,
                                                           max_model_len=512, num_speculative_tokens=k),
                        cache=CacheConfig(num_blocks=32), device=device, enforce_eager=eager,
                        cuda_graph_batch_sizes=[1, 2, 4])


def test_qwen_forward_matches_cpu_oracle():
    pstate.set_state(pstate.ParallelState())
    prompts = [list(range(3, 3 + 90)), [5, 9, 11]]
    hs = {}
    for dev in ("cpu", "cuda"):
        model = HybridForCausalLM(_cfg(dev).model, dev, seed=3, init_mode="sliced")
        eng = LLMEngine(_cfg(dev), model)
        for p in prompts:
            eng.add_request(p, SamplingParams(max_tokens=1))
        out = eng.scheduler.schedule()
        h = eng.runner._host_inputs(out)
        d, ctx, _ = eng.runner._context(h)
        with torch.inference_mode():
            hidden = eng.runner.model(d["ids"], ctx)
            hs[dev] = eng.runner.model.compute_logits(hidden).float().cpu()
    rel = ((hs["cuda"] - hs["cpu"]).norm() / hs["cpu"].norm()).item()
    print(f"qwen logits rel {rel:.2e}")
    assert rel < 5e-2, rel


def test_qwen_graph_decode_and_spec_match_eager():
    pstate.set_state(pstate.ParallelState())
    model = HybridForCausalLM(_cfg("cuda", k=2).model, "cuda", seed=4, init_mode="local")
    prompts = [list(range(10, 10 + n)) for n in (7, 66, 130)]
    p = SamplingParams(max_tokens=6)
    eager = [o.output_token_ids for o in LLM(_cfg("cuda", eager=True), model).generate(prompts, p)]
    graph = [o.output_token_ids for o in LLM(_cfg("cuda", eager=False), model).generate(prompts, p)]
    assert eager == graph
    llm = LLM(_cfg("cuda", eager=False, k=2), model)
    spec = [o.output_token_ids for o in llm.generate(prompts, p)]
    assert spec == eager
    assert llm.engine.runner.spec.stats["proposed"] > 0
