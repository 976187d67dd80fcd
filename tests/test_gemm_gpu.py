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


def run_act(x, w, act, n_out):
    M, K = x.shape
    N = w.shape[0]
    y = torch.empty(M, n_out, device=x.device, dtype=torch.bfloat16)
    L.check(L.load().m3_gemm_bf16_act(x.data_ptr(), K, w.data_ptr(), K, y.data_ptr(), n_out, M, N, K, act,
                                      L.stream_ptr()), "m3_gemm_bf16_act")
    return y


@pytest.mark.parametrize("M,N,K", [(1, 3072, 1024), (2, 2048, 512), (5, 3072, 1024), (8, 2048, 512), (8, 520, 136)])
def test_gemv_gelu_epilogue_equals_gemm_then_gelu(cuda, M, N, K):
    """The GEMV kernel's GELU epilogue (depth f1, Mimi fc1 at a few seats) gives the bits of the layer followed by the
    separate GELU pass."""
    g = torch.Generator(device=cuda).manual_seed(M + N + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5 * 3).to(torch.bfloat16)
    fused = run_act(x, w, 1, N)
    ref = run(x, w)
    L.check(L.load().m3_gelu_bf16(ref.data_ptr(), M * N // 8, L.stream_ptr()), "m3_gelu_bf16")
    torch.cuda.synchronize()
    assert torch.equal(fused, ref)
    exact = torch.nn.functional.gelu(x.float() @ w.float().T)
    assert (fused.float() - exact).abs().max().item() <= 1e-2 * max(1.0, exact.abs().max().item())


@pytest.mark.parametrize("M,F,K", [(1, 3072, 1024), (3, 3072, 1024), (8, 3072, 1024), (4, 260, 64)])
def test_gemv_swiglu_epilogue(cuda, M, F, K):
    """The GEMV kernel's SwiGLU epilogue (backbone gate|up at a few seats): each output from the bf16 gate and up
    outputs of the same kernel as bf16(bf16(silu(g)) * u), against that formula applied to the unfused layer's output
    (PyTorch's exp / division in fp32: equal but for rare one-ulp differences of silu) and to fp32."""
    g = torch.Generator(device=cuda).manual_seed(M + F + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * F, K, device=cuda, generator=g) / K ** 0.5 * 3).to(torch.bfloat16)
    fused = run_act(x, w, 2, F)
    gu = run(x, w).float()
    gate, up = gu[:, :F], gu[:, F:]
    ref = ((gate / (1 + torch.exp(-gate))).to(torch.bfloat16).float() * up).to(torch.bfloat16)
    torch.cuda.synchronize()
    same = (fused == ref).float().mean().item()
    assert same >= 0.999, same
    assert (fused.float() - ref.float()).abs().max().item() <= 2 ** -6 * max(1.0, ref.float().abs().max().item())
    full = x.float() @ w.float().T
    exact = torch.nn.functional.silu(full[:, :F]) * full[:, F:]
    assert (fused.float() - exact).abs().max().item() <= 2e-2 * max(1.0, exact.abs().max().item())


def test_activation_outside_the_gemv_path_is_rejected(cuda):
    x = torch.zeros(16, 64, device=cuda, dtype=torch.bfloat16)
    w = torch.zeros(64, 64, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(L.M3Error):
        run_act(x, w, 1, 64)
