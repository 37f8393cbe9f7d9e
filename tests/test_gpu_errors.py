"""Kernel error reporting: an expired bounded wait inside a kernel must turn
into S2B_ERR_TIMEOUT at the API, once, and the context must stay usable.

The expiry is simulated with the test hook s2b_debug_raise_kernel_error,
which raises the same device flags an expired wait raises (no kernel is made
to fault, trap or hang)."""
import numpy as np
import pytest

import s2b

pytestmark = pytest.mark.gpu
ERR_TIMEOUT = 7
T, H, W, TXT, TS = 1, 8, 10, 58, 1000.0
Lv = T * H * W


@pytest.fixture(scope="module")
def ctx_and_inputs():
    c = s2b.DitB200(0, s2b.PREC_BF16)
    c.init_synth(5, 0, 32)
    c.set_windows(s2b.make_win(T, H, W, (4, 3, 3), TXT, False), s2b.make_win(T, H, W, (4, 3, 3), TXT, True))
    vp = s2b.patchify_grid(s2b.synth_vid_grid(T, 2 * H, 2 * W, 1))
    txt = s2b.synth_txt(TXT, 1)
    yield c, vp, txt
    c.close()


@pytest.mark.parametrize("mask", [1, 2, 4, 7], ids=["gemm", "attention", "exchange", "all"])
def test_host_calls_report_expired_wait_once(ctx_and_inputs, mask):
    c, vp, txt = ctx_and_inputs
    ref = c.forward(vp, Lv, txt, TXT, TS)
    c.debug_raise_kernel_error(mask)
    with pytest.raises(s2b.S2BError) as ei:
        c.forward(vp, Lv, txt, TXT, TS)
    assert ei.value.code == ERR_TIMEOUT and "bounded wait expired" in str(ei.value)
    # reported once: the next call is clean and computes the same result
    np.testing.assert_array_equal(c.forward(vp, Lv, txt, TXT, TS), ref)
    c.debug_raise_kernel_error(mask)
    with pytest.raises(s2b.S2BError) as ei:
        c.forward_latent(vp, Lv, txt, TXT, TS, 0, 1, True, False)
    assert ei.value.code == ERR_TIMEOUT
    c.forward_latent(vp, Lv, txt, TXT, TS, 0, 1, True, False)


def test_dev_calls_report_through_check_errors(ctx_and_inputs):
    import torch
    c, vp, txt = ctx_and_inputs
    dev = torch.device("cuda", 0)
    st = torch.cuda.current_stream(dev)
    d_vid, d_txt = torch.from_numpy(vp).to(dev), torch.from_numpy(txt).to(dev)
    d_sr = torch.empty(Lv, 64, device=dev)
    c.forward_dev(d_vid.data_ptr(), Lv, d_txt.data_ptr(), TXT, TS, d_sr.data_ptr(), st.cuda_stream)
    st.synchronize()
    c.check_errors()                       # clean
    ref = d_sr.cpu().numpy().copy()
    c.debug_raise_kernel_error(2)
    c.forward_dev(d_vid.data_ptr(), Lv, d_txt.data_ptr(), TXT, TS, d_sr.data_ptr(), st.cuda_stream)   # enqueue only
    st.synchronize()
    with pytest.raises(s2b.S2BError) as ei:
        c.check_errors()
    assert ei.value.code == ERR_TIMEOUT
    c.check_errors()                       # reported once
    c.forward_dev(d_vid.data_ptr(), Lv, d_txt.data_ptr(), TXT, TS, d_sr.data_ptr(), st.cuda_stream)
    st.synchronize()
    c.check_errors()
    np.testing.assert_array_equal(d_sr.cpu().numpy(), ref)


def test_awa_and_linear_report_expired_wait():
    c = s2b.DitB200(0, s2b.PREC_BF16)
    try:
        win = s2b.make_win(1, 8, 10, (4, 3, 3), TXT, False)
        vq = s2b.synth_normal((80, 7680), 3, "vq")
        tq = s2b.synth_normal((TXT, 7680), 3, "tq")
        nq = [np.ones(128, np.float32)] * 4
        c.awa_forward(vq, tq, win, *nq, 80, TXT, 1e-5)
        c.debug_raise_kernel_error(2)
        with pytest.raises(s2b.S2BError) as ei:
            c.awa_forward(vq, tq, win, *nq, 80, TXT, 1e-5)
        assert ei.value.code == ERR_TIMEOUT
        c.awa_forward(vq, tq, win, *nq, 80, TXT, 1e-5)
        with pytest.raises(s2b.S2BError):
            c.debug_raise_kernel_error(8)          # not a flag
    finally:
        c.close()
