"""``ConformerFeedForward`` (parakeet/modules/feedforward.py): Linear, SiLU,
Linear; plain cuBLAS GEMMs, kept for state_dict compatibility."""
from torch import nn


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


__all__ = ["ConformerFeedForward"]
