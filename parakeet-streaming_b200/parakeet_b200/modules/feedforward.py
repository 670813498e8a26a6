"""``ConformerFeedForward`` (parakeet/modules/feedforward.py): Linear, SiLU,
Linear; plain cuBLAS GEMMs, kept for state_dict compatibility.
``forward_residual`` gives the layer's ``x + scale * FF(h)`` with the scale
and the residual add folded into the second GEMM (alpha/beta of one addmm)."""
import torch
from torch import nn

from ..ops import gemm, gemm_supported


class ConformerFeedForward(nn.Module):
    def __init__(self, hidden_size: int, d_ff: int, dropout: float = 0.0, use_bias: bool = False):
        super().__init__()
        self.d_model, self.d_ff, self.use_bias = hidden_size, d_ff, use_bias
        self.linear1 = nn.Linear(hidden_size, d_ff, bias=use_bias)
        self.activation = nn.SiLU()
        self.dropout = nn.Dropout(dropout)
        self.linear2 = nn.Linear(d_ff, hidden_size, bias=use_bias)

    def forward(self, x):
        return self.linear2(self.dropout(self.activation(self.linear1(x))))

    def forward_residual(self, res, x, scale: float):
        """res + scale * forward(x) (encoder.py:63,76) in two GEMM launches:
        in bf16 the first is the tcgen05 GEMM with SiLU on the accumulator;
        the second is cuBLAS with the residual in its epilogue (addmm)."""
        if (self.linear1.bias is None and not self.training
                and gemm_supported(x, self.linear1.weight)):
            a = gemm(x, self.linear1.weight, "silu")
        else:
            a = self.dropout(self.activation(self.linear1(x)))
        return residual_linear(res, a, self.linear2, scale)


def residual_linear(res, a, linear: nn.Linear, scale: float = 1.0, weight=None):
    """res + scale * linear(a) as one cuBLAS GEMM with the epilogue
    res + alpha * acc (addmm)."""
    w = linear.weight if weight is None else weight
    bias = None if linear is None else linear.bias
    shape = res.shape
    r = res.reshape(-1, shape[-1])
    if bias is not None:
        r = r + scale * bias
    return torch.addmm(r, a.reshape(-1, a.shape[-1]), w.t(), beta=1, alpha=scale).reshape(shape)


__all__ = ["ConformerFeedForward", "residual_linear"]
