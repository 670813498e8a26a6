"""Batched greedy RNNT decode with the prediction-network state in a device
pool: a drop-in for ``ModelRunner._decode_batch`` (parakeet/engine/
model_runner.py:347-447).

The reference sorts the batch by chunk length, copies each row's frame and
prediction state into batch tensors every frame (``_stack_states``), and per
symbol reads ``bool(blank_mask.all())`` and ``ids.tolist()`` on the host.  Here
each slot's LSTM state lives in a pool indexed by the encoder slot id, the
chunk's frames are one [B, T, D] tensor, and every (frame, symbol) step is
joint GEMMs -> ``pk_rnnt_pick`` (argmax, blank mask, token lists, row
bookkeeping) -> prediction GEMMs -> ``pk_lstm_cell`` (cell update fused with the
keep-state-on-blank select).  The first LSTM layer's input half of the gates
(embedding x W_ih + biases) is a per-token table computed once, which the cell
kernel adds by token id, so no embedding lookup or input GEMM runs per step.
In bf16 the joint is two tcgen05 GEMMs: relu(enc + pred_out W_pred) in the
first one's epilogue, the output bias in the second's (the classes padded to
a multiple of 64 with zero rows that the argmax never reads).  Nothing is read back until the chunk's tokens are
complete, so the whole decode of a chunk is one stream of launches (and can be
captured in a CUDA graph).  The prediction network's output is the last LSTM
layer's h, so no separate ``pred_out`` is kept.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .._lib import check, lib
from ..ops import DTYPES, _ptr, _stream, gemm, gemm_supported


class BatchedGreedyDecoder:
    def __init__(self, predictor, joiner, blank_id: int, num_slots: int, max_symbols: int = 5):
        p = next(predictor.parameters())
        self.device, self.dtype = p.device, p.dtype
        if self.dtype not in DTYPES:
            raise ValueError(f"dtype {self.dtype} not handled")
        rnn = predictor.prediction["dec_rnn"]
        self.layers, self.hidden = rnn.num_layers, rnn.hidden_size
        self.blank, self.max_symbols = int(blank_id), int(max_symbols)
        self.emb = predictor.prediction["embed"].weight.detach()
        self.w_ih = [getattr(rnn, f"weight_ih_l{k}").detach() for k in range(self.layers)]
        self.w_hh = [getattr(rnn, f"weight_hh_l{k}").detach() for k in range(self.layers)]
        self.b = [(getattr(rnn, f"bias_ih_l{k}") + getattr(rnn, f"bias_hh_l{k}")).detach()
                  for k in range(self.layers)]
        self.w_enc = joiner.enc.weight.detach()
        self.b_enc = (joiner.enc.bias + joiner.pred.bias).detach()   # both joint biases, once
        self.w_pred = joiner.pred.weight.detach()
        out = joiner.joint_net[2]
        self.w_out, self.b_out = out.weight.detach(), out.bias.detach()
        self.classes = self.w_out.shape[0]
        L, H = self.layers, self.hidden
        # first layer's input half of the gates for every token id (the blank
        # id's embedding row is the padding row)
        self.xtab = torch.addmm(self.b[0], self.emb, self.w_ih[0].t()).contiguous()
        # bf16: the joint and the recurrent GEMM on the tcgen05 kernel (its K
        # and N must be multiples of 64: joint width, hidden, 4 x hidden)
        probe = self.w_pred.new_empty(0, H)
        self.fast = (self.dtype == torch.bfloat16 and gemm_supported(probe, self.w_pred)
                     and self.w_out.shape[1] % 64 == 0
                     and gemm_supported(probe, self.w_hh[0]))
        pad = (-self.classes) % 64
        self.w_out_p = F.pad(self.w_out, (0, 0, 0, pad)).contiguous()
        self.b_out_p = F.pad(self.b_out, (0, pad)).contiguous()
        self.h = torch.zeros(L, num_slots, H, device=self.device, dtype=self.dtype)
        self.c = torch.zeros_like(self.h)
        # create_sequence (model_runner.py:66-80): zero state, one step on blank
        h0 = torch.zeros(L, 1, H, device=self.device, dtype=self.dtype)
        c0 = torch.zeros_like(h0)
        ids = torch.full((1,), self.blank, dtype=torch.int64, device=self.device)
        ones = torch.ones(1, dtype=torch.int32, device=self.device)
        self._predict(ids, h0, c0, ones)
        self._h0, self._c0 = h0, c0

    def reset_slots(self, slots) -> None:
        """A new stream in each of ``slots``: the state after the blank start step."""
        idx = torch.as_tensor(slots, dtype=torch.int64, device=self.device).reshape(-1)
        n = idx.numel()
        self.h.index_copy_(1, idx, self._h0.expand(-1, n, -1).contiguous())
        self.c.index_copy_(1, idx, self._c0.expand(-1, n, -1).contiguous())

    def _predict(self, ids, h, c, emit) -> None:
        """One prediction step for rows with emit != 0 (decoder.py:44-50)."""
        B, H = ids.numel(), self.hidden
        dt = DTYPES[self.dtype]
        x = None
        for k in range(self.layers):
            if k == 0:   # the token's half comes from the table, in the cell kernel
                # (cuBLAS: at 2048 rows 8.9 us against the tcgen05 kernel's 12.8)
                gates = torch.mm(h[0], self.w_hh[0].t())
                xtab, xld = self.xtab, 4 * H
            else:
                gates = torch.addmm(self.b[k], x, self.w_ih[k].t())
                gates.addmm_(h[k], self.w_hh[k].t())
                xtab, xld = None, 0
            check(lib().pk_lstm_cell(gates.data_ptr(), 4 * H, _ptr(xtab), xld, ids.data_ptr(),
                                     h[k].data_ptr(), c[k].data_ptr(), H, emit.data_ptr(), B, H,
                                     dt, _stream(self.device)), "pk_lstm_cell")
            x = h[k]

    def decode(self, enc: torch.Tensor, lengths: torch.Tensor, slots: torch.Tensor):
        """Greedy tokens of one chunk per stream.  enc [B, T, enc_dim] (frames
        at t >= lengths[b] are ignored), slots [B] pool rows.  Returns device
        tensors tokens int32 [B, T, max_symbols] (-1 = none) and counts int32
        [B, T]; the slots' states advance."""
        B, T, Denc = enc.shape
        S, L, H = self.max_symbols, self.layers, self.hidden
        idx = slots.to(device=self.device, dtype=torch.int64)
        lengths = lengths.to(device=self.device, dtype=torch.int32).contiguous()
        h = self.h.index_select(1, idx)
        c = self.c.index_select(1, idx)
        encp = torch.addmm(self.b_enc, enc.reshape(B * T, Denc).to(self.dtype), self.w_enc.t())
        encp = encp.view(B, T, -1)
        tokens = torch.empty(B, T, S, dtype=torch.int32, device=self.device)
        counts = torch.empty(B, T, dtype=torch.int32, device=self.device)
        done = torch.empty(B, dtype=torch.int32, device=self.device)
        emit = torch.empty(B, dtype=torch.int32, device=self.device)
        ids = torch.empty(B, dtype=torch.int64, device=self.device)
        dt, st = DTYPES[self.dtype], _stream(self.device)
        ld = self.w_out_p.shape[0] if self.fast else self.classes
        for t in range(T):
            for s in range(S):
                if self.fast:
                    z = gemm(h[L - 1], self.w_pred, "residual_relu", residual=encp[:, t])
                    logits = gemm(z, self.w_out_p, "bias", bias=self.b_out_p)
                else:
                    z = torch.addmm(encp[:, t], h[L - 1], self.w_pred.t()).relu_()
                    logits = torch.addmm(self.b_out, z, self.w_out.t())
                check(lib().pk_rnnt_pick(logits.data_ptr(), ld, dt, B, self.classes,
                                         self.blank, lengths.data_ptr(), t, s, S, T,
                                         done.data_ptr(), emit.data_ptr(), ids.data_ptr(),
                                         tokens.data_ptr(), counts.data_ptr(), st), "pk_rnnt_pick")
                self._predict(ids, h, c, emit)
        self.h.index_copy_(1, idx, h)
        self.c.index_copy_(1, idx, c)
        return tokens, counts

    def decode_batch(self, seqs, chunks) -> list[list[int]]:
        """``ModelRunner._decode_batch(seqs, chunks)``: chunks[i] is stream i's
        encoder output [1, enc_dim, len_i]; seqs[i].encoder_state its slot.
        Returns each stream's token ids, in ``seqs`` order."""
        if not seqs:
            return []
        lens = [int(ch.shape[2]) for ch in chunks]
        T, Denc = max(lens), int(chunks[0].shape[1])
        enc = torch.zeros(len(seqs), T, Denc, dtype=self.dtype, device=self.device)
        for i, ch in enumerate(chunks):
            enc[i, : lens[i]] = ch[0].transpose(0, 1).to(device=self.device, dtype=self.dtype)
        lengths = torch.tensor(lens, dtype=torch.int32, device=self.device)
        slots = torch.tensor([s.encoder_state for s in seqs], dtype=torch.int64, device=self.device)
        tokens, counts = self.decode(enc, lengths, slots)
        tokens, counts = tokens.cpu(), counts.cpu()   # the one read-back of the chunk
        out = []
        for i in range(len(seqs)):
            row = []
            for t in range(lens[i]):
                row.extend(tokens[i, t, : int(counts[i, t])].tolist())
            out.append(row)
        return out


__all__ = ["BatchedGreedyDecoder"]
