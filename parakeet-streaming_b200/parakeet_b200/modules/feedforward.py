"""``ConformerFeedForward`` (parakeet/modules/feedforward.py): Linear, SiLU,
Linear, kept for state_dict compatibility.  ``forward_residual`` gives the
layer's ``x + scale * FF(h)`` with the scale and the residual add folded into
the second GEMM's epilogue (``residual_linear``)."""
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
    """res + scale * linear(a) as one GEMM with the epilogue res + alpha * acc:
    in bf16 inference with K <= 512 (the small model's D x D attention output
    and pointwise conv 2) the tcgen05 GEMM, measured ahead of cuBLAS's addmm
    there at 320 to 6720 rows (4.7 vs 6.2 us at 320, 6.1 vs 8.1 at 4096);
    otherwise cuBLAS with the residual in its epilogue (addmm)."""
    w = linear.weight if weight is None else weight
    bias = None if linear is None else linear.bias
    shape = res.shape
    if (bias is None and w.shape[1] <= 512 and res.dtype == torch.bfloat16
            and not (res.requires_grad or a.requires_grad or w.requires_grad)
            and gemm_supported(a, w)):
        return gemm(a, w, "residual", residual=res, alpha=scale).reshape(shape)
    r = res.reshape(-1, shape[-1])
    if bias is not None:
        r = r + scale * bias
    return torch.addmm(r, a.reshape(-1, a.shape[-1]), w.t(), beta=1, alpha=scale).reshape(shape)


__all__ = ["ConformerFeedForward", "residual_linear"]
