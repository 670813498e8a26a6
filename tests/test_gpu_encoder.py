"""The paged encoder (drop-in modules + scheduler) against the reference's
own outputs: the golden stream schedules of tests/golden/make_golden.py,
replayed through Scheduler.pack_states -> ConformerEncoder.forward ->
unpack_states, on valid frames.  fp32: rel-L2 <= 1e-5 at every depth.  bf16:
rel-L2 <= 1e-2 over 2 layers (small) / 1 layer (large); over the whole stack
(17 / 24 layers) bf16 rounding alone moves the reference's own bf16 run 2-3 %
from its fp32 run (recorded per step in the fixture), so there the bound is
1e-2 or 1.25 x the reference's own bf16 error, whichever is larger."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from parakeet_b200.engine.scheduler import Scheduler
from parakeet_b200.modules import ConformerEncoder
from parakeet_b200.weights import random_encoder_layers
from replay import LARGE, LARGE_FULL, SMALL, SMALL_FULL, load, rel_l2, schedule, valid_rows

pytestmark = pytest.mark.gpu


def build_encoder(cfg, dtype):
    enc = ConformerEncoder(feat_in=128, hidden_size=cfg["dim"], ff_expansion_factor=4,
                           num_layers=cfg["layers"], num_heads=cfg["heads"], subsampling_factor=8,
                           pos_emb_max_len=5000, conv_kernel_size=9, att_context_size=cfg["att"],
                           subsampling_conv_channels=256, use_bias=False)
    sd = random_encoder_layers(cfg["seed"], cfg["layers"], cfg["dim"], cfg["heads"])
    missing, unexpected = enc.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()},
                                              strict=False)
    assert not unexpected and all(k.startswith("pre_encode.") for k in missing)
    return enc.to(device="cuda", dtype=dtype).eval()


def replay_encoder(cfg, dtype, page_size=16):
    enc = build_encoder(cfg, dtype)
    sched = Scheduler(max_active=cfg["pool"])
    sched.init_state_pool(enc, torch.device("cuda"), dtype, cfg["pool"], page_size=page_size)
    slot_of, outs = {}, {}
    for s, rel, acq, names, x, length in schedule(cfg):
        for n in rel:
            sched.release_state_slot(slot_of[n])
        for n in acq:
            slot_of[n] = sched.acquire_state_slot()
        seqs = [SimpleNamespace(encoder_state=slot_of[n]) for n in names]
        st, idx = sched.pack_states(seqs)
        with torch.inference_mode():
            y, st = enc(torch.from_numpy(x).to("cuda", dtype), st,
                        length=torch.from_numpy(length).cuda(), bypass_pre_encode=True)
        sched.unpack_states(st, idx)
        outs[s] = (y.float().cpu().numpy(), idx.cpu().numpy())
    return outs, sched


@pytest.mark.parametrize("cfg,name", [(SMALL, "encoder_small.npz"), (LARGE, "encoder_large.npz"),
                                      (SMALL_FULL, "encoder_small_full.npz"),
                                      (LARGE_FULL, "encoder_large_full.npz")])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_paged_encoder_matches_reference(cfg, name, dtype, page_size=16):
    torch.backends.cuda.matmul.allow_tf32 = False
    g = load(name)
    outs, sched = replay_encoder(cfg, dtype, page_size)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    for s in g["keep_steps"]:
        y, idx = outs[int(s)]
        assert np.array_equal(idx, g[f"slots_{s}"])
        lens = g[f"len_{s}"]
        err = rel_l2(valid_rows(y, lens), valid_rows(g[f"out_{s}"], lens))
        bound = tol
        if dtype == torch.bfloat16 and f"ref_bf16_err_{s}" in g:
            bound = max(tol, 1.25 * float(g[f"ref_bf16_err_{s}"]))
        assert err <= bound, (int(s), err, bound)
    pool = sched.pool
    assert pool.read_error() == 0
    slots = torch.arange(cfg["pool"], dtype=torch.int32, device="cuda")
    proc, clen = pool.counters(slots)
    assert np.array_equal(proc.cpu().numpy(), g["final_processed"])
    assert np.array_equal(clen.cpu().numpy(), g["final_cache_len"])


@pytest.mark.parametrize("cfg,name", [(SMALL, "encoder_small.npz"),
                                      (SMALL_FULL, "encoder_small_full.npz"),
                                      (LARGE, "encoder_large.npz"),
                                      (LARGE_FULL, "encoder_large_full.npz")])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_paged_encoder_8_frame_pages_matches_reference(cfg, name, dtype):
    """The same replay over pages of 8 frames (the small serving engine's pool)."""
    test_paged_encoder_matches_reference(cfg, name, dtype, page_size=8)
