"""The EXL3 PLE row decoder (csrc/rows.cu::ple_decode_kernel) against the fp32 oracle, bit for
bit: several ring widths, ids of other ranks, ids in no head's vocabulary, failed rows, and the
table lookup end to end on the GPU (reference kernel: csrc/exl3/ple.cu:91)."""

import os

import pytest
import torch

from vllm_cmp170hx_b200 import _ext
from vllm_cmp170hx_b200.formats import ple as fple

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dim,bits,n", [(256, 4, 3000), (128, 3, 64), (512, 8, 200), (64, 16, 33), (1024, 2, 7),
                                        (4096, 5, 40)])
def test_ple_decode_matches_oracle(dim, bits, n):
    t = fple.random_table(heads=3, vocab=1000, dim=dim, bits=bits, seed=bits, padding=20)
    g = torch.Generator().manual_seed(dim)
    ids = torch.randint(0, 3020, (n,), generator=g)
    ids[: min(n, 4)] = torch.tensor([0, 2999, 3005, 1500])[: min(n, 4)]  # first, last, padding, middle
    failed = (torch.rand(n, generator=g) < 0.05).to(torch.uint8)
    lo, hi = 700, 2600  # this rank's rows
    packed = t["trellis"][ids]
    exp = fple.decode_rows(packed, ids, t["head_bias"], t["head_offsets"], t["head_vocab_sizes"], lo, hi, bits, failed)
    dev = "cuda"
    out = torch.full((n, dim), 7.0, dtype=torch.bfloat16, device=dev)
    _ext.ops().ple_decode(packed.to(dev), ids.to(dev), t["head_bias"].to(dev), t["head_offsets"].to(dev),
                          t["head_vocab_sizes"].to(dev), lo, hi, bits, failed.to(dev), out)
    torch.cuda.synchronize()
    got = out.cpu()
    nan = exp.isnan()
    assert torch.equal(got.isnan(), nan)
    assert torch.equal(got[~nan], exp[~nan])


def test_ple_table_lookup_on_gpu(tmp_path):
    from vllm_cmp170hx_b200.storage.ple import PleTable

    t = fple.random_table(heads=4, vocab=500, dim=256, bits=4, padding=12)
    path = os.path.join(tmp_path, "ngram_embedding.safetensors")
    fple.write_table(path, "model.ngram_embedding", t, 4)
    tab = PleTable(path, "model.ngram_embedding", device="cuda", threads=4)
    g = torch.Generator().manual_seed(1)
    for step in range(3):
        ids = torch.stack([torch.randint(0, 500, (37,), generator=g) + 500 * h for h in range(4)], 1)
        rows, failed = tab.lookup(ids)
        torch.cuda.synchronize()
        flat = ids.reshape(-1)
        exp = fple.decode_rows(t["trellis"][flat], flat, t["head_bias"], t["head_offsets"], t["head_vocab_sizes"], 0,
                               2012, 4).view(37, -1)
        assert not failed.any()
        assert torch.equal(rows.cpu(), exp), step
