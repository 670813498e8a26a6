"""Rel-pos multi-head self-attention over the paged window.

Drop-in for ``PositionalEncoding`` and ``ConformerAttention``
(parakeet/modules/attention.py:23-125): same constructor arguments, same
parameter names (``qkv``, ``linear_pos``, ``linear_out``, ``pos_bias_u``,
``pos_bias_v``) so reference state_dicts load unchanged, same
``forward(x, pos_emb, attn_mask, cache)`` signature.

The forward keeps the two projections on cuBLAS (``qkv`` and ``linear_out``)
and replaces everything between them - cache append, ``linear_pos``,
``rel_shift``, the -1e5 mask fill and SDPA - with one libpk call that
appends the chunk's K/V rows to the pages and runs the paged attention with
the streaming mask of the step's window descriptors.  ``linear_pos(pos_emb)`` depends only on the
fixed left context, so it is computed once per layer and reused.
"""
from __future__ import annotations

import math

import torch
from torch import Tensor, nn

from .cache import PagedModelCache
from .feedforward import residual_linear


class PositionalEncoding(nn.Module):
    """Sinusoid table over relative positions max_len-1 ... -(max_len-1)
    (attention.py:23-62): even columns sin(pos * f_k), odd columns
    cos(pos * f_k), f_k = 10000^(-2k / hidden)."""

    def __init__(self, hidden_size: int, dropout: float, max_len: int, dropout_rate_emb: float):
        super().__init__()
        self.hidden_size = hidden_size
        self.max_len = max_len
        self.dropout = nn.Dropout(dropout)
        self.dropout_emb = nn.Dropout(dropout_rate_emb)

    def extend_pe(self, length: int, device) -> None:
        pos = torch.arange(length - 1, -length, -1, dtype=torch.float32, device=device)[:, None]
        freq = torch.exp(torch.arange(0, self.hidden_size, 2, dtype=torch.float32, device=device)
                         * -(math.log(10000.0) / self.hidden_size))
        pe = torch.zeros(pos.shape[0], self.hidden_size, device=device)
        pe[:, 0::2] = torch.sin(pos * freq)
        pe[:, 1::2] = torch.cos(pos * freq)
        self.register_buffer("pe", pe[None], persistent=False)

    def forward(self, x: Tensor, cache_len: int = 0):
        """Rows for relative positions (T+cache_len-1) ... -(T+cache_len-1)."""
        n = x.size(1) + cache_len
        center = self.pe.size(1) // 2 + 1
        return self.dropout(x), self.dropout_emb(self.pe[:, center - n:center + n - 1])


class ConformerAttention(nn.Module):
    def __init__(self, layer_idx, num_heads, hidden_size: int, use_bias: bool = False):
        super().__init__()
        if use_bias:
            raise NotImplementedError("biased projections are not used by the streaming models")
        self.layer_idx = layer_idx
        self.num_heads = num_heads
        self.d_k = hidden_size // num_heads
        self.s_d_k = math.sqrt(self.d_k)
        self.linear_out = nn.Linear(hidden_size, hidden_size, bias=False)
        self.linear_pos = nn.Linear(hidden_size, hidden_size, bias=False)
        self.qkv = nn.Linear(hidden_size, 3 * hidden_size, bias=False)
        self.pos_bias_u = nn.Parameter(torch.zeros(num_heads, self.d_k))
        self.pos_bias_v = nn.Parameter(torch.zeros(num_heads, self.d_k))
        self._pos_key = None
        self._pos_proj = None

    def pos_projection(self, pos_emb: Tensor) -> Tensor:
        """linear_pos(pos_emb) as [P, D], cached while pos_emb and the weight
        are unchanged (attention.py:102-106 recomputes it every call)."""
        w = self.linear_pos.weight
        try:
            version = w._version
        except RuntimeError:   # an inference-mode tensor has no version counter
            version = None
        key = (pos_emb.data_ptr(), tuple(pos_emb.shape), pos_emb.dtype, w.data_ptr(), version)
        if self._pos_key != key:
            self._pos_proj = self.linear_pos(pos_emb.to(w.dtype)).reshape(-1, w.shape[0]).contiguous()
            self._pos_key = key
        return self._pos_proj

    def _context(self, x: Tensor, pos_emb: Tensor, cache: PagedModelCache) -> Tensor:
        if not isinstance(cache, PagedModelCache):
            raise TypeError("ConformerAttention needs the paged streaming cache")
        D = x.shape[-1]
        qkv = self.qkv(x)                                             # attention.py:94
        query, key, value = qkv[..., :D], qkv[..., D:2 * D], qkv[..., 2 * D:]
        pool, pos = cache.pool, self.pos_projection(pos_emb)
        # cache append (attention.py:98) fused into the paged attention call
        if pool.relpos_bd_cols:
            # shapes with the all-stream pre-pass (bf16, 4 heads x chunk <= 16): the
            # rel-pos term of every stream in one pass over the layer's pos rows,
            # then attention over it (the same output, bit for bit)
            bd = pool.relpos_bd(self.layer_idx, query, pos, self.pos_bias_v)
            return pool.attention(self.layer_idx, query, None, self.pos_bias_u, None, cache.slots,
                                  cache.lengths, key=key, value=value, bd=bd)
        return pool.attention(self.layer_idx, query, pos, self.pos_bias_u, self.pos_bias_v,
                              cache.slots, cache.lengths, key=key, value=value)

    def forward(self, x: Tensor, pos_emb: Tensor, attn_mask=None, cache: PagedModelCache = None):
        return self.linear_out(self._context(x, pos_emb, cache))      # attention.py:123

    def forward_residual(self, res: Tensor, x: Tensor, pos_emb: Tensor,
                         cache: PagedModelCache = None) -> Tensor:
        """res + forward(x) with the residual add in the output projection's
        GEMM (encoder.py:66)."""
        return residual_linear(res, self._context(x, pos_emb, cache), self.linear_out)


__all__ = ["ConformerAttention", "PositionalEncoding"]
