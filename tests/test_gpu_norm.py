"""pk_layer_norm (through the C ABI, parakeet_b200.ops.layer_norm) against
torch.nn.functional.layer_norm: fp32 within 1e-5 relative, bf16 within one
bf16 rounding of the fp32 result; the two-in-one form equals two separate
LayerNorms with the first output rounded as stored."""
import pytest
import torch
import torch.nn.functional as F
from torch import nn

from parakeet_b200.ops import layer_norm

pytestmark = pytest.mark.gpu


def make_ln(D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    ln = nn.LayerNorm(D)
    with torch.no_grad():
        ln.weight.copy_(1 + 0.1 * torch.randn(D, generator=g))
        ln.bias.copy_(0.1 * torch.randn(D, generator=g))
    return ln.to("cuda", dtype)


@pytest.mark.parametrize("D", [256, 512, 1024])
@pytest.mark.parametrize("rows", [1, 7, 320, 6720])
def test_layer_norm_fp32(D, rows):
    g = torch.Generator(device="cuda").manual_seed(D + rows)
    x = torch.randn(rows, D, generator=g, device="cuda") * 3 + 0.5
    ln = make_ln(D, torch.float32, 1)
    y = layer_norm(x, ln)
    ref = F.layer_norm(x, (D,), ln.weight, ln.bias, ln.eps)
    assert (y - ref).norm() / ref.norm() < 1e-5
    assert (y - ref).abs().max() < 1e-4


@pytest.mark.parametrize("D", [512, 1024])
def test_layer_norm_bf16_and_double(D):
    g = torch.Generator(device="cuda").manual_seed(D)
    x32 = torch.randn(160, 2, D, generator=g, device="cuda") * 2
    x = x32.to(torch.bfloat16)
    ln1, ln2 = make_ln(D, torch.bfloat16, 2), make_ln(D, torch.bfloat16, 3)
    y = layer_norm(x, ln1)
    ref = F.layer_norm(x.float(), (D,), ln1.weight.float(), ln1.bias.float(), ln1.eps)
    err = (y.float() - ref).abs()
    assert bool((err <= ref.abs() * 2 ** -8 + 1e-2).all())
    a, b = layer_norm(x, ln1, ln2)
    assert torch.equal(a, y)
    b_sep = layer_norm(a, ln2)
    assert torch.equal(b, b_sep)


def test_layer_norm_strided_rows():
    """Rows taken from a wider buffer (row stride > width)."""
    D = 512
    base = torch.randn(64, 3 * D, device="cuda")
    x = base[:, D:2 * D]
    ln = make_ln(D, torch.float32, 4)
    y = layer_norm(x, ln)
    ref = F.layer_norm(x, (D,), ln.weight, ln.bias, ln.eps)
    assert (y - ref).abs().max() < 1e-4
