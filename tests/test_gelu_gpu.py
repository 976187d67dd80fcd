"""The feed-forward activation of the depth and Mimi MLPs (F.gelu, erf form, on bf16 tensors) as the stages apply
it: every bf16 bit pattern goes through m3_gelu_bf16 and is compared with PyTorch's own GELU in fp32, rounded to
bf16 (the reference computes F.gelu on bf16 tensors the same way)."""
import pytest
import torch

from maya2_native_b200 import _lib as L

pytestmark = pytest.mark.gpu


def test_gelu_on_every_bf16_input(cuda):
    x = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).to(cuda)
    y = x.clone()
    L.check(L.load().m3_gelu_bf16(y.data_ptr(), x.numel() // 8, L.stream_ptr()), "m3_gelu_bf16")
    ref = torch.nn.functional.gelu(x.float()).to(torch.bfloat16)
    torch.cuda.synchronize()
    nan_y, nan_r = torch.isnan(y), torch.isnan(ref)
    assert torch.equal(nan_y, nan_r)
    yb = y[~nan_y].view(torch.int16).int()
    rb = ref[~nan_r].view(torch.int16).int()
    diff = (yb - rb).abs()
    assert int((diff != 0).sum()) <= 16 and int(diff.max()) <= 1, (int((diff != 0).sum()), int(diff.max()))
