"""Fused mHC boundary kernel (csrc/mhc.cu) against the fp32 oracle: post into the streams, the
Sinkhorn coefficients and the normalised collapsed input, for the immediate, carried-pre and
stream-0 collapses, with and without a pending sublayer output."""

import pytest
import torch

from vllm_cmp170hx_b200 import _ext
from vllm_cmp170hx_b200.ops import mhc as mhc_ops
from vllm_cmp170hx_b200.oracle import mhc as ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,n,d", [(1, 4, 256), (7, 4, 2304), (64, 4, 4096), (5, 2, 512), (3, 8, 1024)])
@pytest.mark.parametrize("with_post", [False, True])
@pytest.mark.parametrize("mode", ["fresh", "carried", "stream0"])
def test_post_pre_matches_oracle(T, n, d, with_post, mode):
    g = torch.Generator().manual_seed(T * 100 + n * 10 + d % 7)
    N = 2 * n + n * n
    H = torch.randn(T, n, d, generator=g).to(torch.bfloat16)
    fn = torch.randn(N, n * d, generator=g) * (n * d) ** -0.5
    scale = torch.rand(3, generator=g) + 0.5
    base = torch.rand(N, generator=g) - 0.5
    w = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    x = post = comb = None
    if with_post:
        x = torch.randn(T, d, generator=g).to(torch.bfloat16)
        post = torch.rand(T, n, generator=g) * 2
        comb = torch.softmax(torch.randn(T, n, n, generator=g), -1)
    delayed = mode != "fresh"
    pre_mix = torch.rand(T, n, generator=g) if mode == "carried" else None
    kw = dict(rms_eps=1e-6, eps=1e-6, post_mult=2.0, iters=20, norm_eps=1e-5, delayed=delayed, pre_mix=pre_mix)
    r = ref.post_pre(x, H, post, comb, fn, scale, base, w, **kw)
    cu = lambda t: None if t is None else t.cuda()  # noqa: E731
    kw["pre_mix"] = cu(pre_mix)
    o = mhc_ops.post_pre(cu(x), H.cuda().clone(), cu(post), cu(comb), fn.cuda(), scale.cuda(), base.cuda(), w.cuda(), **kw)
    torch.cuda.synchronize()
    _ext.check_status(torch.device("cuda"))
    Hr, yr, postr, combr, prer = r
    Ho, yo, posto, combo, preo = (t.cpu() for t in o)
    # bf16 outputs: sums taken in another order may round one ulp apart
    assert (Ho.float() - Hr.float()).abs().max() <= 2e-2 * Hr.float().abs().max() + 1e-3
    assert torch.allclose(posto, postr, atol=2e-4, rtol=1e-3)
    assert torch.allclose(combo, combr, atol=2e-4, rtol=1e-3)
    assert torch.allclose(preo, prer, atol=2e-4, rtol=1e-3)
    assert ((yo.float() - yr.float()).norm() / yr.float().norm()).item() < 1e-2
