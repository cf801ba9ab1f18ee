"""Row gather (msg = feats[idx]) against torch indexing, through the Python wrapper and so
through the C ABI: bf16 and f32 rows, rows that take the 16-byte and the 4-byte path, and
out-of-range indices (zero rows)."""

import pytest
import torch

from gdl_b200 import csrc

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


@pytest.mark.parametrize("dtype,C", [(torch.bfloat16, 64), (torch.bfloat16, 256), (torch.float32, 6),
                                     (torch.float32, 128), (torch.bfloat16, 2)])
def test_gather_rows_matches_index_select(dtype, C):
    g = torch.Generator().manual_seed(C)
    src = torch.randn(5000, C, generator=g).to(dtype).cuda()
    idx = torch.randint(0, 5000, (70001,), generator=g).cuda()
    got = csrc.gather_rows(src, idx)
    want = src.index_select(0, idx)
    assert torch.equal(got.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                       want.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))


def test_gather_rows_out_of_range_gives_zero_rows():
    src = torch.randn(10, 8).cuda()
    idx = torch.tensor([0, -1, 9, 10, 3], device="cuda")
    got = csrc.gather_rows(src, idx)
    assert torch.equal(got[[0, 2, 4]], src[[0, 9, 3]])
    assert torch.equal(got[[1, 3]], torch.zeros(2, 8, device="cuda"))


def test_gather_rows_into_given_output_and_empty():
    src = torch.randn(100, 16, dtype=torch.bfloat16).cuda()
    idx = torch.arange(99, -1, -1).cuda()
    out = torch.empty(100, 16, dtype=torch.bfloat16, device="cuda")
    assert csrc.gather_rows(src, idx, out=out) is out
    assert torch.equal(out, src.flip(0))
    assert csrc.gather_rows(src, idx[:0]).shape == (0, 16)
