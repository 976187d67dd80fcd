"""GPU parity of the linear-layer implementations behind m3_gemm_bf16: the tcgen05 tensor-core kernel and the GEMV
kernel against an fp32 PyTorch reference of the same op (and cuBLAS), over ragged shapes (M, N, K tails)."""
import pytest
import torch

from maya2_native_b200 import _lib as L

pytestmark = pytest.mark.gpu
GEMV, CUBLAS, UMMA, UMMA_GELU, UMMA_SMALL = 1, 2, 3, 4, 5


def run(impl, x, w, y_f32=False):
    M, K = x.shape
    N = w.shape[0]
    y = torch.empty(M, N, device=x.device, dtype=torch.float32 if y_f32 else torch.bfloat16)
    L.check(L.load().m3_gemm_bf16_impl(x.data_ptr(), K, w.data_ptr(), K, y.data_ptr(), N, M, N, K, int(y_f32), impl,
                                       L.stream_ptr()), "m3_gemm_bf16_impl")
    return y


SHAPES = [(1, 64, 64), (7, 1024, 1024), (64, 4096, 1024), (128, 1024, 2048), (200, 2048, 1000), (256, 6144, 1024),
          (256, 1024, 3072), (513, 3072, 1024), (2048, 1024, 3072), (300, 520, 136), (129, 64, 4096)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_tensor_core_gemm_matches_fp32(cuda, M, N, K):
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    ref = x.float() @ w.float().T
    y = run(UMMA, x, w)
    torch.cuda.synchronize()
    err = (y.float() - ref).abs().max().item()
    assert err <= 1e-2 * max(1.0, ref.abs().max().item()), err        # one bf16 rounding of an fp32 accumulation
    yf = run(UMMA, x, w, y_f32=True)
    assert (yf - ref).abs().max().item() <= 1e-3 * max(1.0, ref.abs().max().item())
    yc = run(CUBLAS, x, w, y_f32=True)
    assert (yf - yc).abs().max().item() <= 1e-3 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_gemv_matches_fp32(cuda, M):
    x = torch.randn(M, 3072, device=cuda).to(torch.bfloat16)
    w = (torch.randn(1000, 3072, device=cuda) / 3072 ** 0.5).to(torch.bfloat16)
    ref = x.float() @ w.float().T
    y = run(GEMV, x, w, y_f32=True)
    assert (y - ref).abs().max().item() <= 1e-3 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("M,N,K", [(256, 3072, 1024), (2048, 3072, 1024), (300, 520, 136)])
def test_tensor_core_gemm_gelu_epilogue(cuda, M, N, K):
    """The fused feed-forward activation: bf16(GELU_erf(bf16(x w^T))), the rounding points of the depth / Mimi MLPs."""
    g = torch.Generator(device=cuda).manual_seed(M + N + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    z = (x.float() @ w.float().T).to(torch.bfloat16).float()
    ref = torch.nn.functional.gelu(z)
    y = run(UMMA_GELU, x, w)
    torch.cuda.synchronize()
    assert (y.float() - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("M,N,K", [(1, 64, 64), (37, 1024, 2048), (128, 4096, 1024), (160, 6144, 1024),
                                   (256, 1024, 3072), (256, 4096, 1024), (200, 520, 136), (256, 64, 4096),
                                   (256, 3072, 1024), (96, 2048, 1000)])
def test_small_m_cluster_gemm_matches_fp32(cuda, M, N, K):
    """The cluster split-K kernel for decode-sized batches (M <= 256): K-slices summed across the cluster through
    distributed shared memory, one bf16 rounding; ragged M (rows past M read as zeros), N and K tails."""
    g = torch.Generator(device=cuda).manual_seed(M * 5 + N + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    ref = x.float() @ w.float().T
    y = run(UMMA_SMALL, x, w)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    err = (y.float() - ref).abs().max().item()
    assert err <= 1e-2 * max(1.0, ref.abs().max().item()), err
    y2 = run(UMMA_SMALL, x, w)                    # fixed summation order: bit-identical on a rerun
    assert torch.equal(y, y2)
