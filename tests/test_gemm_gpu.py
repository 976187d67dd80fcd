"""GPU parity of m3_gemm_bf16, the linear layer every stage calls: this library's GEMV kernel for M <= 8 and cuBLAS
above, against an fp32 PyTorch reference of the same op, over the tick's shapes and ragged ones (M, N, K tails)."""
import pytest
import torch

from maya2_native_b200 import _lib as L

pytestmark = pytest.mark.gpu


def run(x, w, y_f32=False):
    M, K = x.shape
    N = w.shape[0]
    y = torch.empty(M, N, device=x.device, dtype=torch.float32 if y_f32 else torch.bfloat16)
    L.check(L.load().m3_gemm_bf16(x.data_ptr(), K, w.data_ptr(), K, y.data_ptr(), N, M, N, K, int(y_f32),
                                  L.stream_ptr()), "m3_gemm_bf16")
    return y


SHAPES = [(1, 64, 64), (3, 2056, 1024), (7, 1024, 1024), (8, 3072, 3072), (64, 4096, 1024), (128, 1024, 2048),
          (200, 2048, 1000), (256, 6144, 1024), (256, 1024, 3072), (513, 3072, 1024), (2048, 1024, 3072),
          (300, 520, 136), (129, 64, 4096)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_matches_fp32(cuda, M, N, K):
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    ref = x.float() @ w.float().T
    scale = max(1.0, ref.abs().max().item())
    y = run(x, w)
    torch.cuda.synchronize()
    assert (y.float() - ref).abs().max().item() <= 1e-2 * scale        # one bf16 rounding of an fp32 accumulation
    yf = run(x, w, y_f32=True)
    assert (yf - ref).abs().max().item() <= 1e-3 * scale
