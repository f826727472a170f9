"""Writer kernels for the 288-byte rope-free row and the V4 Pro cells against the torch oracles."""
import pytest
import torch

from inference_optimizations_b200.ops import formats as F

pytestmark = pytest.mark.gpu


def test_glmflash_writer_bitexact(cuda):
    from inference_optimizations_b200._ext import ext
    torch.manual_seed(0)
    x = (torch.randn(50, 512) * torch.exp2(torch.randint(-6, 6, (50, 1)).float())).to(torch.bfloat16)
    slot = torch.randperm(64)[:50].int()
    slot[3] = -1
    pool = torch.zeros(64, 288, dtype=torch.uint8, device=cuda)
    ext().glmflash_write(x.to(cuda), slot.to(cuda), pool)
    want = F.glmflash_row_quantize(x.float())
    got = pool.cpu()
    keep = slot >= 0
    assert torch.equal(got[slot[keep].long()], want[keep])
    assert torch.all(got[int(torch.tensor([i for i in range(64) if i not in slot.tolist()])[0])] == 0)


@pytest.mark.parametrize("rope", ["fp8", "bf16"])
def test_v4pro_writer_matches_oracle(cuda, rope):
    from inference_optimizations_b200._ext import ext
    torch.manual_seed(1)
    x = (torch.randn(300, 512) * torch.exp2(torch.randint(-5, 5, (300, 1)).float())).to(torch.bfloat16)
    slot = torch.arange(300, dtype=torch.int32)
    pool = torch.zeros(300, F.v4pro_cell_bytes(rope), dtype=torch.uint8, device=cuda)
    ext().v4pro_write(x.to(cuda), slot.to(cuda), pool, int(rope == "bf16"))
    got, want = pool.cpu(), F.v4pro_cell_quantize(x.float(), rope)
    same_rows = (got == want).all(1).float().mean().item()
    assert same_rows > 0.995, same_rows           # a search tie may pick another equal-error scale
    d_got, d_want = F.v4pro_cell_dequantize(got, rope), F.v4pro_cell_dequantize(want, rope)
    e_got = (d_got[:, :448] - x.float()[:, :448]).pow(2).sum()
    e_want = (d_want[:, :448] - x.float()[:, :448]).pow(2).sum()
    assert abs(e_got - e_want) <= 1e-4 * e_want
