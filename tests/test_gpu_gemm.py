"""GEMM engine (s2b_linear) against a plain PyTorch fp32 matmul.

bf16 contexts run the tcgen05 kernel on bf16-rounded operands: compared with
torch fp32 on the same rounded operands, only the fp32 accumulation order
differs (max|d|/max|ref| <= 1e-3).  fp32 contexts: <= 1e-5."""
import numpy as np
import pytest

import s2b

pytestmark = pytest.mark.gpu
# (2750, 2560, 2560) and (700, 2560, 2560) take the 128-wide pair tiles (the 256-wide ones would
# leave most of a last wave idle); the others the 256-wide or single-CTA kernels.
SHAPES = [(128, 256, 64), (5498, 7680, 2560), (58, 2560, 2560), (300, 13824, 2560), (1000, 2560, 6912),
          (77, 64, 2560), (640, 2560, 136), (200, 2560, 132), (1, 2560, 256), (129, 288, 72),
          (2750, 2560, 2560), (700, 2560, 2560)]


@pytest.fixture(scope="module", params=[s2b.PREC_FP32, s2b.PREC_BF16], ids=["fp32", "bf16"])
def ctx(request):
    c = s2b.DitB200(0, request.param)
    yield c
    c.close()


def linear(ctx, x, W, b=None):
    import ctypes
    M, K = x.shape
    N = W.shape[0]
    y = np.zeros((M, N), np.float32)
    F = ctypes.POINTER(ctypes.c_float)
    L = s2b.lib()
    L.s2b_linear.argtypes = [ctypes.c_void_p, F, ctypes.c_int, ctypes.c_int, F, ctypes.c_int, F, F]
    rc = L.s2b_linear(ctx._ctx, x.ctypes.data_as(F), M, K, W.ctypes.data_as(F), N,
                      None if b is None else b.ctypes.data_as(F), y.ctypes.data_as(F))
    assert rc == 0, L.s2b_last_error(ctx._ctx)
    return y


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_vs_torch_fp32(ctx, M, N, K):
    import torch
    x = s2b.synth_normal((M, K), 1, f"x{M}{K}")
    W = s2b.synth_normal((N, K), 2, f"w{N}{K}", 0.0, 0.02)
    b = s2b.synth_normal((N,), 3, f"b{N}", 0.0, 0.02)
    y = linear(ctx, x, W, b)
    xt, wt = torch.from_numpy(x).cuda(), torch.from_numpy(W).cuda()
    if ctx.precision == s2b.PREC_BF16:
        xt, wt = xt.bfloat16().float(), wt.bfloat16().float()
    with torch.no_grad():
        torch.backends.cuda.matmul.allow_tf32 = False
        ref = (xt @ wt.T + torch.from_numpy(b).cuda()).cpu().numpy()
    rel = np.abs(y - ref).max() / np.abs(ref).max()
    assert rel <= (1e-3 if ctx.precision == s2b.PREC_BF16 else 1e-5), rel


@pytest.mark.parametrize("M,N,K", [(5498, 2560, 2560), (300, 13824, 2560), (58, 256, 128), (129, 288, 64)])
def test_linear_bf16_dev_vs_torch_fp32(M, N, K):
    """s2b_linear_bf16_dev on device bf16 buffers, on the caller's stream:
    against torch fp32 on the same bf16 operands, bf16 output rounding
    (max|d|/max|ref| <= 8e-3, two bf16 ulps at the top of the range)."""
    import torch
    c = s2b.DitB200(0, s2b.PREC_BF16)
    try:
        dev = torch.device("cuda", 0)
        x = torch.from_numpy(s2b.synth_normal((M, K), 4, f"dx{M}{K}")).to(dev).bfloat16()
        w = torch.from_numpy(s2b.synth_normal((N, K), 5, f"dw{N}{K}", 0.0, 0.02)).to(dev).bfloat16()
        b = torch.from_numpy(s2b.synth_normal((N,), 6, f"db{N}", 0.0, 0.02)).to(dev)
        y = torch.full((M, N), float("nan"), device=dev, dtype=torch.bfloat16)
        st = torch.cuda.current_stream(dev)
        c.linear_bf16_dev(x.data_ptr(), M, K, w.data_ptr(), N, b.data_ptr(), y.data_ptr(), st.cuda_stream)
        torch.cuda.synchronize(dev)
        torch.backends.cuda.matmul.allow_tf32 = False
        ref = x.float() @ w.float().T + b
        rel = ((y.float() - ref).abs().max() / ref.abs().max()).item()
        assert rel <= 8e-3, rel
        # shapes the kernel cannot take are refused with an argument error
        with pytest.raises(s2b.S2BError):
            c.linear_bf16_dev(x.data_ptr(), M, K - 1, w.data_ptr(), N, None, y.data_ptr(), st.cuda_stream)
    finally:
        c.close()


@pytest.mark.parametrize("K", [2560, 6912])
def test_fp32_linear_rounding_error_vs_cpu_fp32(K):
    """The fp32 context's 3xTF32 Linear against float64: its rounding error is
    a small multiple of a CPU fp32 GEMM's (numpy's blocked sgemm) -- measured
    2.4x at K=2560 and 4x at K=6912, from the tensor core's fp32 accumulation
    along K -- and far below the fp32 parity bar."""
    c = s2b.DitB200(0, s2b.PREC_FP32)
    try:
        rs = np.random.RandomState(0)
        x = rs.randn(512, K).astype(np.float32)
        W = (rs.randn(512, K) * 0.02).astype(np.float32)
        y = linear(c, x, W, None).astype(np.float64)
    finally:
        c.close()
    ref = x.astype(np.float64) @ W.astype(np.float64).T
    cpu = (x @ W.T).astype(np.float64)
    rms = lambda a: float(np.sqrt(((a - ref) ** 2).mean() / (ref ** 2).mean()))
    print(f"K={K}: gpu rms rel {rms(y):.2e}, cpu fp32 {rms(cpu):.2e}")
    assert rms(y) <= 3e-6 and rms(y) <= 6 * max(rms(cpu), 1e-7)
