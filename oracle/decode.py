"""float64 numpy restatement of the reference's batched greedy RNNT decode.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Restates, per stream:

* ``Predictor`` (parakeet/modules/decoder.py:5-50): embedding of vocab + 1 rows
  (blank = padding row) -> ``num_layers``-layer LSTM, gates in PyTorch's
  (input, forget, cell, output) order; the step output is the last layer's h;
* ``Joiner`` (decoder.py:53-86): enc(frame) + pred(pred_out) -> ReLU -> output
  layer over vocab + 1 classes (dropout is the identity in eval mode);
* ``ModelRunner._decode_batch`` / ``_decode_frame_batch``
  (parakeet/engine/model_runner.py:347-447): for every frame t < the stream's
  chunk length, emit argmax tokens while they are not blank, at most
  ``max_symbols`` per frame, advancing the prediction network after every
  emitted token.  Batching in the reference only groups rows: a row's tokens and
  state depend on that row alone (the blank rows' states are restored by
  ``torch.where``, model_runner.py:433-445), which this restatement keeps per row;
* ``create_sequence`` (model_runner.py:66-80): a stream starts from zero state
  and one prediction step on the blank id.
"""
from __future__ import annotations

import numpy as np

F64 = np.float64


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


class GreedyDecoderModel:
    def __init__(self, sd: dict, pred_layers: int, blank: int, max_symbols: int):
        g = lambda k: np.asarray(sd[k], F64)  # noqa: E731
        self.embed = g("predictor.prediction.embed.weight")
        self.lstm = [(g(f"predictor.prediction.dec_rnn.weight_ih_l{k}"),
                      g(f"predictor.prediction.dec_rnn.weight_hh_l{k}"),
                      g(f"predictor.prediction.dec_rnn.bias_ih_l{k}")
                      + g(f"predictor.prediction.dec_rnn.bias_hh_l{k}"))
                     for k in range(pred_layers)]
        self.w_pred, self.b_pred = g("joiner.pred.weight"), g("joiner.pred.bias")
        self.w_enc, self.b_enc = g("joiner.enc.weight"), g("joiner.enc.bias")
        self.w_out, self.b_out = g("joiner.joint_net.2.weight"), g("joiner.joint_net.2.bias")
        self.blank, self.max_symbols = blank, max_symbols
        self.hidden = self.lstm[0][1].shape[1]

    def predict(self, token: int, state):
        """One ``Predictor.forward`` step (decoder.py:44-50) on a single token."""
        h, c = state
        x = self.embed[token]
        nh, nc = [], []
        for k, (w_ih, w_hh, b) in enumerate(self.lstm):
            gates = w_ih @ x + w_hh @ h[k] + b
            i, f, gg, o = np.split(gates, 4)
            ck = _sigmoid(f) * c[k] + _sigmoid(i) * np.tanh(gg)
            hk = _sigmoid(o) * np.tanh(ck)
            nh.append(hk)
            nc.append(ck)
            x = hk
        return x, (nh, nc)

    def new_stream(self):
        """``create_sequence``: zero state, then one step on the blank id."""
        L, H = len(self.lstm), self.hidden
        return self.predict(self.blank, ([np.zeros(H)] * L, [np.zeros(H)] * L))

    def logits(self, frame, pred_out):
        """``Joiner.forward`` (decoder.py:82-86) for one frame [enc_dim]."""
        z = self.w_enc @ frame + self.b_enc + self.w_pred @ pred_out + self.b_pred
        return self.w_out @ np.maximum(z, 0.0) + self.b_out

    def decode_chunk(self, chunk, pred_out, state):
        """Greedy tokens of one stream's chunk [enc_dim, length]; returns
        (tokens, pred_out, state) like one row of ``_decode_batch``."""
        toks = []
        for t in range(chunk.shape[1]):
            frame = np.asarray(chunk[:, t], F64)
            for _ in range(self.max_symbols):
                k = int(np.argmax(self.logits(frame, pred_out)))
                if k == self.blank:
                    break
                toks.append(k)
                pred_out, state = self.predict(k, state)
        return toks, pred_out, state
