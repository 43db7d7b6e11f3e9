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
