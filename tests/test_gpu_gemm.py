"""Tile-engine GEMM parity on the B200: Y = X·W^T against a torch fp32 matmul of
the same 16-bit inputs (tolerance: normwise max|err|/max|ref| < 2e-3 for fp16,
8e-3 for bf16 outputs stored in 16 bit). b2p_gemm runs up to 1024 rows on the
cluster split-K kernel (gemm_sk.cu), above on the persistent single-CTA engine;
b2p_gemm_pair on the CTA-pair engine."""
import pytest
import torch

from autoane_b200 import _lib

pytestmark = pytest.mark.gpu

SHAPES = [
    (128, 128, 64), (256, 960, 960), (256, 320, 960), (384, 1600, 960), (256, 2560, 960),
    (256, 960, 2560), (200, 1000, 72), (1024, 16893, 960), (8192, 960, 960), (130, 48, 40),
    (100, 320, 2560), (1000, 2560, 960), (1025, 960, 960),
]


def run_gemm(x, w, out_f32, dtype_code):
    M, K = x.shape
    N = w.shape[0]
    ldy = N if out_f32 else N
    pad = (4 if out_f32 else 8)
    ldy = (N + pad - 1) // pad * pad
    y = torch.zeros(M, ldy, device=x.device, dtype=torch.float32 if out_f32 else x.dtype)
    _lib.call("b2p_gemm", x.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, K, ldy, dtype_code, int(out_f32), None)
    torch.cuda.synchronize()
    _lib.call("b2p_device_status", None)
    return y[:, :N].float()


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("out_f32", [1, 0])
def test_gemm_matches_fp32(b2p, M, N, K, dt, out_f32):
    torch.manual_seed(M * 7 + N * 3 + K)
    dtype = torch.float16 if dt == "f16" else torch.bfloat16
    x = torch.randn(M, K, device="cuda").to(dtype)
    w = (0.02 * torch.randn(N, K, device="cuda")).to(dtype)
    ref = x.float() @ w.float().t()
    y = run_gemm(x, w, out_f32, 0 if dt == "f16" else 1)
    err = (y - ref).abs().max().item() / max(ref.abs().max().item(), 1e-30)
    tol = 2e-3 if (out_f32 or dt == "f16") else 8e-3
    assert err < tol, f"normwise error {err:.3e} (M={M} N={N} K={K} {dt} out_f32={out_f32})"


PAIR_SHAPES = [(256, 960, 960), (512, 1600, 960), (384, 2560, 960), (1024, 16893, 960), (8192, 960, 2560),
               (300, 100, 64), (16384, 5120, 960), (16384, 960, 2560), (16384, 1600, 960)]


@pytest.mark.parametrize("M,N,K", PAIR_SHAPES)
@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("out_f32", [1, 0])
def test_pair_gemm_matches_fp32(b2p, M, N, K, dt, out_f32):
    torch.manual_seed(M * 5 + N * 11 + K)
    dtype = torch.float16 if dt == "f16" else torch.bfloat16
    x = torch.randn(M, K, device="cuda").to(dtype)
    w = (0.02 * torch.randn(N, K, device="cuda")).to(dtype)
    ref = x.float() @ w.float().t()
    pad = 4 if out_f32 else 8
    ldy = (N + pad - 1) // pad * pad
    y = torch.zeros(M, ldy, device="cuda", dtype=torch.float32 if out_f32 else dtype)
    _lib.call("b2p_gemm_pair", x.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, K, ldy, 0 if dt == "f16" else 1,
              out_f32, None)
    torch.cuda.synchronize()
    _lib.call("b2p_device_status", None)
    y = y[:, :N].float()
    err = (y - ref).abs().max().item() / max(ref.abs().max().item(), 1e-30)
    tol = 2e-3 if (out_f32 or dt == "f16") else 8e-3
    assert err < tol, f"normwise error {err:.3e} (M={M} N={N} K={K} {dt} out_f32={out_f32})"


@pytest.mark.parametrize("M,N,K", [(256, 960, 960), (100, 320, 2560), (128, 2560, 960)])
def test_split_k_is_repeatable(b2p, M, N, K):
    """The cluster split-K kernel adds its partial sums in a fixed rank order: two calls give
    the same bits (and so do the fp32 and 16-bit paths after rounding the fp32 result)."""
    torch.manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda").half()
    w = (0.02 * torch.randn(N, K, device="cuda")).half()
    a = run_gemm(x, w, 1, 0)
    b = run_gemm(x, w, 1, 0)
    assert torch.equal(a, b)
    h = run_gemm(x, w, 0, 0)
    assert torch.equal(h, a.half().float())


@pytest.mark.parametrize("M,N,K,x_mn", [(256, 960, 960, 0), (8192, 960, 2560, 0), (8192, 2560, 960, 0),
                                         (4096, 960, 16893, 0), (1024, 960, 1920, 0), (300, 200, 72, 0),
                                         (512, 512, 4096, 1), (1408, 512, 4096, 1), (16893, 512, 4096, 1),
                                         (384, 300, 520, 1)])
@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("out_f32", [1, 0])
def test_pair_gemm_mn_major_operands(b2p, M, N, K, x_mn, dt, out_f32):
    """The backward's GEMMs read W as stored ([out][in]: dX = dY·W, W MN-major) and, for weight
    gradients, dY and X as stored ([tokens][features]: dW = dY^T·X, both MN-major). The same product
    through K-major copies: within the pair engine's tolerance of the fp32 product, and bit-identical to
    the K-major launch on the transposed operands (same tiles, same K order)."""
    if x_mn and not out_f32:
        pytest.skip("MN-major X is built for fp32 (weight-gradient) outputs")
    torch.manual_seed(M + 3 * N + 5 * K + x_mn)
    dtype = torch.float16 if dt == "f16" else torch.bfloat16
    xk = torch.randn(M, K, device="cuda").to(dtype)            # [M][K]
    wk = (0.02 * torch.randn(N, K, device="cuda")).to(dtype)   # [N][K]
    ldw = (N + 7) // 8 * 8
    wmn = torch.zeros(K, ldw, device="cuda", dtype=dtype)
    wmn[:, :N] = wk.t()
    if x_mn:
        ldx = (M + 7) // 8 * 8
        xop = torch.zeros(K, ldx, device="cuda", dtype=dtype)
        xop[:, :M] = xk.t()
    else:
        ldx = (K + 7) // 8 * 8
        xop = torch.zeros(M, ldx, device="cuda", dtype=dtype)
        xop[:, :K] = xk
    ldk = (K + 7) // 8 * 8
    xkp = torch.zeros(M, ldk, device="cuda", dtype=dtype)
    xkp[:, :K] = xk
    wkp = torch.zeros(N, ldk, device="cuda", dtype=dtype)
    wkp[:, :K] = wk
    ref = xk.float() @ wk.float().t()
    pad = 4 if out_f32 else 8
    ldy = (N + pad - 1) // pad * pad
    code = 0 if dt == "f16" else 1
    odt = torch.float32 if out_f32 else dtype
    y_mn = torch.zeros(M, ldy, device="cuda", dtype=odt)
    y_k = torch.zeros(M, ldy, device="cuda", dtype=odt)
    _lib.call("b2p_gemm_pair_mn", xop.data_ptr(), ldx, x_mn, wmn.data_ptr(), ldw, 1, y_mn.data_ptr(), M, N, K, ldy, code,
              out_f32, None)
    _lib.call("b2p_gemm_pair_mn", xkp.data_ptr(), ldk, 0, wkp.data_ptr(), ldk, 0, y_k.data_ptr(), M, N, K, ldy, code,
              out_f32, None)
    torch.cuda.synchronize()
    _lib.call("b2p_device_status", None)
    y_mn, y_k = y_mn[:, :N].float(), y_k[:, :N].float()
    err = (y_mn - ref).abs().max().item() / max(ref.abs().max().item(), 1e-30)
    tol = 2e-3 if (out_f32 or dt == "f16") else 8e-3
    assert err < tol, f"normwise error {err:.3e}"
    assert torch.equal(y_mn, y_k)


@pytest.mark.parametrize("M,N,K", [(128, 960, 960), (256, 320, 960), (1024, 2560, 960), (128, 960, 2560), (100, 200, 72),
                                   (1000, 960, 24), (300, 5000, 960)])
@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("out_f32", [1, 0])
def test_multi_issuer_gemm(b2p, M, N, K, dt, out_f32):
    """b2p_gemm_mi (128 x 64 tiles, four MMA issuers with an accumulator each, summed in issuer order):
    within the engines' tolerance of the fp32 product, including ragged M / N / K, K shorter than one
    64-wide block per issuer and more tiles than SMs; bit-identical on repeat."""
    torch.manual_seed(M + 7 * N + 3 * K)
    dtype = torch.float16 if dt == "f16" else torch.bfloat16
    x = torch.randn(M, K, device="cuda").to(dtype)
    w = (0.02 * torch.randn(N, K, device="cuda")).to(dtype)
    ref = x.float() @ w.float().t()
    pad = 4 if out_f32 else 8
    ldy = (N + pad - 1) // pad * pad
    outs = []
    for _ in range(2):
        y = torch.zeros(M, ldy, device="cuda", dtype=torch.float32 if out_f32 else dtype)
        _lib.call("b2p_gemm_mi", x.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, K, ldy, 0 if dt == "f16" else 1,
                  out_f32, None)
        torch.cuda.synchronize()
        _lib.call("b2p_device_status", None)
        outs.append(y[:, :N].float())
    assert torch.equal(outs[0], outs[1])
    err = (outs[0] - ref).abs().max().item() / max(ref.abs().max().item(), 1e-30)
    tol = 2e-3 if (out_f32 or dt == "f16") else 8e-3
    assert err < tol, f"normwise error {err:.3e}"
