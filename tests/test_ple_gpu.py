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


def test_ple_lookup_async_matches_sync_and_replays(tmp_path):
    """The host-function PLE lookup (no host wait) equals the synchronous one, keeps failed rows
    NaN for the caller's mask, and replays in a CUDA graph with each replay's ids."""
    from vllm_cmp170hx_b200.storage.ple import PleTable

    t = fple.random_table(heads=2, vocab=300, dim=128, bits=4, padding=6)
    path = os.path.join(tmp_path, "p.safetensors")
    fple.write_table(path, "p", t, 4)
    tab = PleTable(path, "p", 100, 550, device="cuda", threads=4)  # this rank owns rows [100, 550)
    g = torch.Generator().manual_seed(3)
    for step in range(3):
        ids = torch.stack([torch.randint(0, 300, (50,), generator=g), torch.randint(300, 606, (50,), generator=g)], 1)
        flat = ids.reshape(-1)
        exp = fple.decode_rows(t["trellis"][flat], flat, t["head_bias"], t["head_offsets"], t["head_vocab_sizes"],
                               100, 550, 4).view(50, -1)
        got = tab.lookup_async(ids.cuda()).cpu()
        assert torch.equal(got, exp), step
    tab.reader.fail_rows_for_test([101])
    ids = torch.tensor([[101, 400], [5, 301]])
    rows, bad = PleTable.mask_failed(tab.lookup_async(ids.cuda()), 2)
    assert bad.cpu().tolist() == [True, False] and (rows[0] == 0).all()
    ids_dev = torch.full((16, 2), 200, dtype=torch.int64, device="cuda")
    tab.lookup_async(ids_dev, fixed=True)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            out = tab.lookup_async(ids_dev, fixed=True)
    for rep in range(2):
        ids = torch.stack([torch.randint(150, 300, (16,), generator=g), torch.randint(300, 540, (16,), generator=g)], 1)
        ids_dev.copy_(ids)
        graph.replay()
        torch.cuda.synchronize()
        flat = ids.reshape(-1)
        exp = fple.decode_rows(t["trellis"][flat], flat, t["head_bias"], t["head_offsets"], t["head_vocab_sizes"],
                               100, 550, 4).view(16, -1)
        assert torch.equal(out.cpu(), exp), rep
    del graph
