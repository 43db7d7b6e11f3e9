"""DFlash block attention on the GPU: the block-sparse attention kernel over the fused [k | v | 0] rows
(context rows through the request's slots, the block's own rows in scratch rows, only the value half
computed) against the dense attention of the CPU path on the same keys / values."""

import pytest
import torch

from vllm_cmp170hx_b200.models.dflash import DFlashCache, DFlashConfig, DFlashLayer
from vllm_cmp170hx_b200.models.layers import WeightInit

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nh,nkv,hd,lens", [(8, 2, 128, [5, 130, 1]), (16, 4, 128, [300, 64]), (4, 4, 256, [70, 9])])
def test_block_attention_kernel_matches_dense(nh, nkv, hd, lens):
    g = torch.Generator().manual_seed(nh + hd)
    dc = DFlashConfig(num_heads=nh, num_kv_heads=nkv, head_dim=hd, intermediate=256)
    A, B = len(lens), 4
    C = max(lens)
    slots = 1024
    layer_g = DFlashLayer(256, dc, 1e-6, WeightInit(1, "cuda", "sliced"))
    layer_c = DFlashLayer(256, dc, 1e-6, WeightInit(1, "cpu", "sliced"))
    kctx = (torch.randn(slots, nkv, hd, generator=g) * 0.5).bfloat16()
    vctx = torch.randn(slots, nkv, hd, generator=g).bfloat16()
    cg = DFlashCache(slots, nkv, hd, "cuda", scratch=A * B)
    cc = DFlashCache(slots, nkv, hd, "cpu")
    every = torch.arange(slots)
    cg.write(every.cuda(), kctx.cuda(), vctx.cuda())
    cc.write(every, kctx, vctx)
    perm = torch.randperm(slots, generator=g)
    ctx_slots = torch.full((A, C), -1, dtype=torch.int64)
    k0 = 0
    for a, n in enumerate(lens):
        ctx_slots[a, :n] = perm[k0:k0 + n]
        k0 += n
    valid = ctx_slots >= 0
    last = torch.tensor(lens) - 1
    pos = (last[:, None] + 1 + torch.arange(B)[None]).reshape(-1)
    qn = (torch.randn(A * B, nh, hd, generator=g) * 0.5).bfloat16()
    k = (torch.randn(A * B, nkv, hd, generator=g) * 0.5).bfloat16()
    v = torch.randn(A * B, nkv, hd, generator=g).bfloat16()
    ref = layer_c._attend_dense(qn, k, v, pos, cc, ctx_slots, valid, A, B).float()
    got = layer_g._attend_kernel(qn.cuda(), k.cuda(), v.cuda(), pos.cuda(), cg, ctx_slots.cuda(), valid.cuda(), A, B)
    torch.cuda.synchronize()
    err = (got.float().cpu() - ref).abs().max().item()
    print(f"dflash block attention max err {err:.2e}")
    assert err < 3e-2, err
