"""RNNT prediction and joint networks: drop-ins for ``Predictor`` and
``Joiner`` (parakeet/modules/decoder.py:5-86) with the same constructor
arguments, submodule names (so reference state_dicts load unchanged) and
``forward`` semantics.  The batched greedy decode in
``parakeet_b200.engine.decoding`` uses their weights directly."""
from __future__ import annotations

import torch
from torch import Tensor, nn


class Predictor(nn.Module):
    def __init__(self, pred_dim: int, hidden_dim: int, num_layers: int, vocab_size: int):
        super().__init__()
        self.prediction = nn.ModuleDict({
            "embed": nn.Embedding(vocab_size + 1, pred_dim, padding_idx=vocab_size),
            "dec_rnn": nn.LSTM(input_size=pred_dim, hidden_size=hidden_dim, num_layers=num_layers),
        })
        self.pred_dim = pred_dim
        self.num_layers = num_layers

    def init_state(self, batch_size: int):
        p = next(self.parameters())
        z = torch.zeros(self.num_layers, batch_size, self.pred_dim, device=p.device, dtype=p.dtype)
        return z, z.clone()

    def forward(self, input_ids: Tensor, state):
        y = self.prediction["embed"](input_ids.reshape(-1, 1)).transpose(0, 1)
        g, hidden = self.prediction["dec_rnn"](y, state)
        return g.transpose(0, 1)[:, -1, :], hidden


class Joiner(nn.Module):
    def __init__(self, encoder_dim, pred_dim, joint_dim, dropout: float = 0.2,
                 num_classes: int = 1024):
        super().__init__()
        self._vocab_size = num_classes
        self._num_classes = num_classes + 1
        self.encoder_dim, self.pred_dim, self.joint_dim = encoder_dim, pred_dim, joint_dim
        self.dropout = dropout
        self.pred = nn.Linear(pred_dim, joint_dim)
        self.enc = nn.Linear(encoder_dim, joint_dim)
        self.joint_net = nn.Sequential(nn.ReLU(inplace=True), nn.Dropout(p=dropout),
                                       nn.Linear(joint_dim, num_classes + 1))

    def forward(self, encoder_frame: Tensor, predictor_out: Tensor) -> Tensor:
        joined = self.enc(encoder_frame) + self.pred(predictor_out).unsqueeze(1)
        return self.joint_net(joined).squeeze(1)


__all__ = ["Predictor", "Joiner"]
