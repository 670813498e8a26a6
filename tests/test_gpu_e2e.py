"""configs[0] end to end: audio -> tokens against the reference engine's own
token ids and encoder outputs (golden ``e2e_<size>.npz`` from
tests/golden/make_golden_e2e.py: the reference's ``ModelRunner.step()`` on the
CPU in fp32, seeded weights, 10 s of pcm16 white noise pushed in 160 ms
pieces, full encoder depth: 17 layers small, 24 large).

* ``StreamingPipeline`` (GPU log-mel -> batched pre-encode -> paged encoder ->
  batched greedy decode) in fp32 with TF32 off: for every chunk of whole
  audio, the encoder output within rel-L2 1e-5 of the reference's and the
  token ids identical;
* the reference's own ``ModelRunner`` driving this package's ``Scheduler``,
  ``ConformerEncoder``, ``FeatureExtractor`` and ``BatchedGreedyDecoder`` (the
  swaps a maintainer makes) on the GPU: every chunk,
  the final partial one included, identical token ids.  It needs the
  reference install under ``baseline/_ref`` (``bench.py --install-reference``)
  and is skipped without it.
"""
import os
import sys

import numpy as np
import pytest
import torch

from engine_drive import drive, pcm16_noise
from replay import load, rel_l2

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "baseline"))
import harness  # noqa: E402

pytestmark = pytest.mark.gpu

ATT = {"small": (70, 1), "large": (70, 13)}
ENC_TOL = 1e-5          # fp32 encoder output, rel-L2 over the chunk


def build_modules(size, dtype=torch.float32):
    """This package's encoder (with its pre-encoder), prediction and joint
    networks, loaded with the golden run's seeded weights."""
    from parakeet_b200.modules import ConformerEncoder, Joiner, Predictor
    c = harness.MODEL_WEIGHTS[size]
    sd = {k: torch.from_numpy(v) for k, v in harness.model_state_dict(size).items()}
    enc = ConformerEncoder(feat_in=128, hidden_size=c["dim"], ff_expansion_factor=4,
                           num_layers=c["layers"], num_heads=c["heads"], subsampling_factor=8,
                           pos_emb_max_len=5000, conv_kernel_size=9, att_context_size=ATT[size],
                           subsampling_conv_channels=256, use_bias=False)
    pred = Predictor(640, 640, c["pred_layers"], c["vocab"])
    join = Joiner(c["dim"], 640, 640, num_classes=c["vocab"])
    for prefix, m in (("encoder.", enc), ("predictor.", pred), ("joiner.", join)):
        m.load_state_dict({k[len(prefix):]: v for k, v in sd.items() if k.startswith(prefix)},
                          strict=True)
    return [m.to("cuda", dtype).eval() for m in (enc, pred, join)]


def chunks_of(g):
    """Golden per-chunk (tokens, frames, encoder output [D, frames])."""
    off, fr = g["offsets"], g["frames"]
    starts = np.concatenate([[0], np.cumsum(fr)])
    return [(g["tokens"][off[i]:off[i + 1]].tolist(), int(fr[i]),
             g["enc"][:, starts[i]:starts[i + 1]]) for i in range(len(fr))]


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


@pytest.mark.parametrize("size", ["small", "large"])
def test_pipeline_matches_reference_engine_fp32(size):
    from parakeet_b200.engine import StreamingPipeline
    g = load(f"e2e_{size}.npz")
    want = chunks_of(g)
    enc, pred, join = build_modules(size)
    V = harness.MODEL_WEIGHTS[size]["vocab"]
    B = 2                                    # two streams with the same audio
    pipe = StreamingPipeline(enc, enc.pre_encode, pred, join, blank_id=V, num_slots=B,
                             feature_kw={"dither": 0.0})
    slots = torch.arange(B, dtype=torch.int32, device="cuda")
    pipe.start_streams(slots)
    la = ATT[size][1]
    first, nxt = (1 + 8 * la) * 160, (8 + 8 * la) * 160       # model_runner.py:53-56
    audio = pcm16_noise(0, 10.0)
    bounds = [(0, first)]
    while bounds[-1][1] + nxt <= len(audio):
        bounds.append((bounds[-1][1], bounds[-1][1] + nxt))
    assert len(bounds) < len(want)           # the rest is the final partial chunk
    errs = []
    for k, (a, b) in enumerate(bounds):
        x = torch.from_numpy(audio[a:b]).cuda().expand(B, -1).contiguous()
        y, lengths = pipe.encode_audio(x, slots, k)
        tokens, counts = pipe.dec.decode(y, lengths, slots)
        tok, frames, ref_enc = want[k]
        assert y.shape[1] == frames
        tokens, counts, yh = tokens.cpu(), counts.cpu(), y.float().cpu().numpy()
        for r in range(B):
            got = [int(t) for f in range(frames) for t in tokens[r, f, :int(counts[r, f])]]
            assert got == tok, (size, k, r, got, tok)
            errs.append(rel_l2(yh[r].T, ref_enc))
    assert pipe.pool.read_error() == 0 and pipe.fe.error_bits() == 0
    assert max(errs) <= ENC_TOL, (size, max(errs))


@pytest.mark.skipif(not harness.available(), reason="no reference install under baseline/_ref")
@pytest.mark.parametrize("size", ["small", "large"])
def test_reference_engine_over_dropins_fp32(size):
    """The reference's unmodified ModelRunner.step() (model_runner.py:103-107)
    with the drop-ins: token ids of every chunk equal the reference's own run."""
    harness.import_reference()
    from parakeet.config import Config
    from parakeet.engine.model_runner import ModelRunner

    from parakeet_b200.engine import BatchedGreedyDecoder, Scheduler
    from parakeet_b200.modules import FeatureExtractor

    g = load(f"e2e_{size}.npz")
    want = chunks_of(g)
    pool = 2
    model = harness.seeded_parakeet(size)            # the reference's Parakeet
    enc, _, _ = build_modules(size)
    model.encoder = enc                               # paged encoder (+ pre-encoder)
    model._feature_extractor = FeatureExtractor(dither=0.0, num_slots=pool, device="cuda")
    harness.patch_from_pretrained(model)

    class Runner(ModelRunner):
        """The decode swap: prediction state in a slot pool on the device."""

        def _init_model(self):
            super()._init_model()
            self._b200 = BatchedGreedyDecoder(self.decoder, self.joiner, self.blank_id,
                                              num_slots=pool,
                                              max_symbols=self._max_symbols_per_frame)

        def create_sequence(self):
            seq = super().create_sequence()
            if seq is not None:
                self._b200.reset_slots([seq.encoder_state])
            return seq

        def _decode_batch(self, seqs, chunks):
            return self._b200.decode_batch(seqs, chunks)

    runner = Runner(Config(size=size, max_num_streams=pool), torch.device("cuda"),
                    Scheduler(max_active=pool))
    rec = drive(runner, pcm16_noise(0, 10.0))
    assert len(rec) == len(want)
    errs = []
    for k, ((chunk, toks), (tok, frames, ref_enc)) in enumerate(zip(rec, want)):
        assert chunk.shape[1] == frames
        assert toks == tok, (size, k, toks, tok)
        errs.append(rel_l2(chunk, ref_enc))
    assert max(errs) <= ENC_TOL, (size, max(errs))
    assert runner.scheduler.pool.read_error() == 0
