"""Row-table dequant kernel on the GPU (e4m3 codes with E8M0 block scales, NaN for failed rows)
against the CPU reference."""

import pytest
import torch

from vllm_cmp170hx_b200.storage import tables

pytestmark = pytest.mark.gpu


def test_row_table_on_gpu(tmp_path):
    x = torch.randn(500, 512, generator=torch.Generator().manual_seed(3)) * 5
    path = str(tmp_path / "t.bin")
    tables.write_table(path, x)
    t = tables.RowTable(path, 500, 512, cache_rows=128, device="cuda")
    t.reader.fail_rows_for_test([42])
    ids = torch.tensor([1, 42, 499, 3, 1])
    y = t.lookup(ids).float().cpu()
    ref = tables.dequantize_rows(torch.from_numpy(tables.quantize_rows(x)), 512)[ids].to(torch.bfloat16).float()
    ok = torch.tensor([True, False, True, True, True])
    assert torch.equal(y[ok], ref[ok]) and torch.isnan(y[1]).all()


def _ref_rows(x, ids):
    r = tables.dequantize_rows(torch.from_numpy(tables.quantize_rows(x)), x.shape[1])
    out = r[ids.clamp_min(0)].to(torch.bfloat16).float()
    out[ids < 0] = 0
    return out


def test_stream_ordered_lookup_matches_sync(tmp_path):
    """The host-function lookup (no host wait) returns the rows of the synchronous one, for device
    ids, repeats, rows of other ranks (-1: zeros) and a failed read (NaN)."""
    x = torch.randn(700, 256, generator=torch.Generator().manual_seed(4)) * 3
    path = str(tmp_path / "t.bin")
    tables.write_table(path, x)
    t = tables.RowTable(path, 700, 256, cache_rows=256, ways=4, threads=4, device="cuda")
    g = torch.Generator().manual_seed(5)
    for step in range(4):
        ids = torch.randint(-1, 600, (300,), generator=g)  # rows 600.. stay out of the host cache
        y = t.lookup_async(ids.cuda()).float().cpu()
        assert torch.equal(y, _ref_rows(x, ids)), step
    t.reader.fail_rows_for_test([650])  # never read before, so the read (and its retries) fails
    ids = torch.tensor([650, 5, 699])
    y = t.lookup_async(ids.cuda()).float().cpu()
    assert torch.isnan(y[0]).all() and torch.equal(y[1:], _ref_rows(x, ids)[1:])
    assert t.cache.host_errors() == 0


def test_stream_ordered_lookup_replays_in_a_cuda_graph(tmp_path):
    """A fixed-job lookup captured once fetches each replay's ids (the host function runs on every
    replay), like the reference's fixed staging under full graphs."""
    x = torch.randn(400, 256, generator=torch.Generator().manual_seed(6)) * 2
    path = str(tmp_path / "t.bin")
    tables.write_table(path, x)
    t = tables.RowTable(path, 400, 256, cache_rows=128, ways=4, threads=4, device="cuda")
    n = 96
    ids_dev = torch.zeros(n, dtype=torch.int64, device="cuda")
    t.lookup_async(ids_dev, fixed=True)  # staging and job made outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            out = t.lookup_async(ids_dev, fixed=True)
    g = torch.Generator().manual_seed(7)
    for rep in range(3):
        ids = torch.randint(0, 400, (n,), generator=g)
        ids_dev.copy_(ids)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.float().cpu(), _ref_rows(x, ids)), rep
    del graph
