"""Device-side data formats around the DiT: patchify / unpatchify
(src/dit_vk.cpp:717-750), the engine's vid_grid assembly and latent decode
(src/seedvr2_engine.cpp:154-168, 298-305) and the device grid forward.
All are data movement plus one IEEE operation per element, so results are
compared bit for bit."""
import ctypes

import numpy as np
import pytest

import s2b

pytestmark = pytest.mark.gpu
SCALING = 0.9152


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def test_patchify_unpatchify_dev_match_host():
    import torch
    T, H, W = 2, 10, 12
    grid = s2b.synth_normal((T, H, W, 33), 5, "grid")
    ref_patch = s2b.patchify_grid(grid)
    d_grid = _dev(grid)
    d_patch = torch.empty(T * (H // 2) * (W // 2), 132, device="cuda")
    assert s2b.lib().s2b_patchify_grid_dev(d_grid.data_ptr(), T, H, W, d_patch.data_ptr(), _stream()) == 0
    np.testing.assert_array_equal(d_patch.cpu().numpy(), ref_patch)
    sr = s2b.synth_normal((T * (H // 2) * (W // 2), 64), 6, "sr")
    ref_grid = s2b.unpatchify_latent(sr, T, H, W)
    d_out = torch.empty(T, H, W, 16, device="cuda")
    assert s2b.lib().s2b_unpatchify_latent_dev(_dev(sr).data_ptr(), T, H, W, d_out.data_ptr(), _stream()) == 0
    np.testing.assert_array_equal(d_out.cpu().numpy().reshape(ref_grid.shape), ref_grid)
    # odd sizes are rejected
    assert s2b.lib().s2b_patchify_grid_dev(d_grid.data_ptr(), T, 9, W, d_patch.data_ptr(), _stream()) == 1  # S2B_ERR_ARG


def test_engine_assembly_and_decode_match_reference_loops():
    import torch
    H8, W8 = 14, 18
    noise = s2b.synth_normal((16, H8, W8), 7, "noise")
    latent = s2b.synth_normal((16, H8, W8), 7, "latent")
    sr = s2b.synth_normal((H8, W8, 16), 7, "sr")
    sc = np.float32(SCALING)
    # the engine's loops (src/seedvr2_engine.cpp:159-168, 299-305) in float32
    ref_grid = np.empty((H8, W8, 33), np.float32)
    ref_grid[:, :, :16] = noise.transpose(1, 2, 0)
    ref_grid[:, :, 16:32] = (latent * sc).transpose(1, 2, 0)
    ref_grid[:, :, 32] = 1.0
    ref_z = ((noise - sr.transpose(2, 0, 1)) / sc).astype(np.float32)
    d_grid = torch.empty(H8, W8, 33, device="cuda")
    L = s2b.lib()
    assert L.s2b_assemble_vid_grid_dev(_dev(noise).data_ptr(), _dev(latent).data_ptr(), SCALING, H8, W8,
                                       d_grid.data_ptr(), _stream()) == 0
    np.testing.assert_array_equal(d_grid.cpu().numpy(), ref_grid)
    d_z = torch.empty(16, H8, W8, device="cuda")
    assert L.s2b_decode_latent_dev(_dev(noise).data_ptr(), _dev(sr).data_ptr(), SCALING, H8, W8, d_z.data_ptr(),
                                   _stream()) == 0
    np.testing.assert_array_equal(d_z.cpu().numpy(), ref_z)


def test_forward_grid_dev_matches_forward_grid():
    import torch
    T, H, W, TXT = 1, 48, 56, 58
    c = s2b.DitB200(0, s2b.PREC_BF16)
    try:
        c.init_synth(1234)
        c.set_windows(s2b.make_win(T, H // 2, W // 2, (4, 3, 3), TXT, False),
                      s2b.make_win(T, H // 2, W // 2, (4, 3, 3), TXT, True))
        grid = s2b.synth_vid_grid(T, H, W, 42)
        txt = s2b.synth_txt(TXT, 42)
        ref = c.forward_grid(grid, txt, TXT, 1000.0)
        d_out = torch.empty(T, H, W, 16, device="cuda")
        c.forward_grid_dev(_dev(grid).data_ptr(), T, H, W, _dev(txt).data_ptr(), TXT, 1000.0, d_out.data_ptr(),
                           _stream())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(d_out.cpu().numpy().reshape(ref.shape), ref)
    finally:
        c.close()
