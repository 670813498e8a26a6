"""pk_gemm_bf16 (tcgen05 tensor cores, TMEM accumulator; through the C ABI;
the CTA-pair form (256 x 256 tiles over two SMs) takes the shapes whose pair
tiles fill a wave, the persistent one-CTA form other shapes with more than two
waves of 128 x 256 tiles)
against an fp32 matmul of the same bf16 operands: the output is the fp32
result rounded once to bf16, so each element is within 2^-8 relative (plus
the accumulation-order difference, far below that) of the reference."""
import pytest
import torch

from parakeet_b200.ops import gemm, gemm_error_word

pytestmark = pytest.mark.gpu


def operands(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device="cuda") / K ** 0.5).to(torch.bfloat16)
    r = torch.randn(M, N, generator=g, device="cuda").to(torch.bfloat16)
    return a, w, r


def check_close(out, ref):
    err = (out.float() - ref).abs()
    tol = ref.abs() * 2 ** -8 + 1e-3 * ref.abs().max() + 1e-6
    bad = err > tol
    assert not bool(bad.any()), (f"{int(bad.sum())} of {bad.numel()} elements off; "
                                 f"max err {float(err.max()):.3g}")


@pytest.mark.parametrize("M,N,K", [(1, 64, 64), (7, 512, 512), (128, 128, 64), (320, 2048, 512),
                                   (320, 512, 2048), (320, 1536, 512), (1000, 1024, 1024),
                                   (6720, 4096, 1024), (6720, 1024, 4096), (6720, 3072, 1024),
                                   (6720, 2048, 1024), (6700, 2048, 128), (4096, 2048, 512),
                                   (4096, 1536, 512), (4000, 1024, 512)])
def test_gemm_store(M, N, K):
    a, w, _ = operands(M, N, K, M + N + K)
    ref = a.float() @ w.float().t()
    check_close(gemm(a, w), ref)
    assert gemm_error_word("cuda") == 0


@pytest.mark.parametrize("M,N,K", [(320, 2048, 512), (6720, 4096, 1024), (33, 192, 128),
                                   (4096, 2048, 512)])
def test_gemm_silu(M, N, K):
    a, w, _ = operands(M, N, K, 7 * M + N)
    acc = a.float() @ w.float().t()
    check_close(gemm(a, w, "silu"), acc * torch.sigmoid(acc))


@pytest.mark.parametrize("M,N,K", [(320, 512, 2048), (6720, 1024, 4096), (5, 64, 64),
                                   (6720, 3072, 1024), (6720, 1024, 1024), (4096, 512, 2048)])
def test_gemm_residual(M, N, K):
    a, w, r = operands(M, N, K, 3 * M + K)
    ref = r.float() + 0.5 * (a.float() @ w.float().t())
    check_close(gemm(a, w, "residual", residual=r, alpha=0.5), ref)


def test_gemm_strided_operand_and_graph():
    """A taken from a wider buffer (row stride > K); the call captured in a
    CUDA graph and replayed."""
    M, N, K = 300, 256, 512
    base, w, _ = operands(M, N, 3 * K, 11)
    w = w[:, :K].contiguous()
    a = base[:, K:2 * K]
    ref = a.float() @ w.float().t()
    check_close(gemm(a, w), ref)
    static_a = a.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        out = gemm(static_a, w)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    check_close(out, ref)


@pytest.mark.parametrize("M", [1, 160, 480])
def test_gemm_residual_relu_strided_rows(M):
    """The joint network's hidden: relu(enc[:, t] + h W_pred^T), the residual
    rows taken from a [B, T, 640] tensor (row stride T * 640)."""
    T, D = 14, 640
    a, w, _ = operands(M, D, D, 5 * M)
    g = torch.Generator(device="cuda").manual_seed(M)
    enc = torch.randn(M, T, D, generator=g, device="cuda").to(torch.bfloat16)
    for t in (0, 5, T - 1):
        ref = torch.relu(enc[:, t].float() + a.float() @ w.float().t())
        check_close(gemm(a, w, "residual_relu", residual=enc[:, t]), ref)


@pytest.mark.parametrize("M,classes", [(160, 1026), (480, 1025)])
def test_gemm_bias_padded_classes(M, classes):
    """The joint output layer with its classes padded to a multiple of 64
    (zero weight rows): the real classes equal z W_out^T + b."""
    K = 640
    a, w, _ = operands(M, classes, K, classes)
    g = torch.Generator(device="cuda").manual_seed(classes)
    b = torch.randn(classes, generator=g, device="cuda").to(torch.bfloat16)
    pad = (-classes) % 64
    wp = torch.nn.functional.pad(w, (0, 0, 0, pad)).contiguous()
    bp = torch.nn.functional.pad(b, (0, pad)).contiguous()
    out = gemm(a, wp, "bias", bias=bp)
    ref = a.float() @ w.float().t() + b.float()
    check_close(out[:, :classes], ref)
