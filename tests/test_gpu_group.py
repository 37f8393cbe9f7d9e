"""Frame-sequence mode from one process (s2b_group_*): frame k runs on member
k mod N; every frame equals the single-context forward of the same inputs
bit for bit (deterministic kernels, no communication)."""
import numpy as np
import pytest

import s2b

pytestmark = pytest.mark.gpu


def test_group_frames_equal_single_context():
    import torch
    ngpu = min(2, torch.cuda.device_count())
    T, H, W, TXT = 1, 24, 28, 58
    Lv = T * H * W
    ns, sh = s2b.make_win(T, H, W, (4, 3, 3), TXT, False), s2b.make_win(T, H, W, (4, 3, 3), TXT, True)
    frames = np.stack([s2b.patchify_grid(s2b.synth_vid_grid(T, 2 * H, 2 * W, 42 + k)) for k in range(3)])
    txt = s2b.synth_txt(TXT, 42)
    g = s2b.FrameGroup(ngpu, s2b.PREC_BF16)
    try:
        g.init_synth(1234)
        g.set_windows(ns, sh)
        out = g.forward_frames(frames, Lv, txt, TXT)
    finally:
        g.close()
    c = s2b.DitB200(0, s2b.PREC_BF16)
    try:
        c.init_synth(1234)
        c.set_windows(ns, sh)
        for k in range(3):
            np.testing.assert_array_equal(out[k], c.forward(frames[k], Lv, txt, TXT))
    finally:
        c.close()


def test_group_rejects_bad_arguments():
    with pytest.raises(s2b.S2BError):
        s2b.FrameGroup(0)
