"""The C-ABI library: loads, exports every declared symbol, validates
arguments and fails loudly (no CPU fallback) when no B200 is present."""
import ctypes
import os

import numpy as np
import pytest

import s2b


def test_library_exports_every_declared_symbol():
    L = s2b.lib()
    names = s2b.exported_symbols()
    assert len(names) >= 29
    for n in names:
        assert hasattr(L, n), n


def test_header_cites_reference_for_each_forward_entry():
    import os
    hdr = open(os.path.join(os.path.dirname(s2b._PKG), "include", "seedvr2_b200.h")).read()
    for needle in ("src/dit_vk.cpp:486-699", "src/awa_vk.h:39-44", "src/awa_layer.cpp:284-453",
                   "src/awa_window.cpp:161-178", "src/ada_compose.cpp:166-235"):
        assert needle in hdr


def test_ctx_create_without_gpu_fails_loudly():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(s2b.S2BError):
        s2b.DitB200(0, s2b.PREC_FP32)


def test_unknown_precision_is_rejected_before_device_work():
    for prec in (-1, 3, 7):
        ctx = ctypes.c_void_p()
        rc = s2b.lib().s2b_ctx_create(0, prec, ctypes.byref(ctx))
        assert rc == 1 and not ctx          # S2B_ERR_ARG, whether or not a GPU is present


def test_make_win_argument_validation():
    L = s2b.lib()
    nw = (ctypes.c_int * 3)(4, 0, 3)
    n = ctypes.c_int()
    assert L.s2b_make_win_size(1, 8, 8, nw, 58, 0, ctypes.byref(n), None, None) == 1
    assert L.s2b_make_win_size(0, 8, 8, (ctypes.c_int * 3)(4, 3, 3), 58, 0, ctypes.byref(n), None, None) == 1


def test_synth_is_deterministic_and_seeded():
    a = s2b.synth_normal((1000,), 5, "x")
    b = s2b.synth_normal((1000,), 5, "x")
    c = s2b.synth_normal((1000,), 6, "x")
    d = s2b.synth_normal((1000,), 5, "y")
    assert np.array_equal(a, b) and not np.array_equal(a, c) and not np.array_equal(a, d)
    big = s2b.synth_normal((200000,), 1, "stat")
    assert abs(big.mean()) < 0.01 and abs(big.std() - 1) < 0.01


def test_synth_m5_layout_matches_reference_loader(tmp_path):
    s2b.synth_write_m5(str(tmp_path), 1, 10, 11)
    p = open(tmp_path / "b10_all_qkv.param").read().split("\n")
    assert p[0] == "7767517" and "InnerProduct" in p[3] and "0=7680" in p[3] and "1=0" in p[3] and "2=19660800" in p[3]
    blob = (tmp_path / "b10_all_out.bin").read_bytes()
    assert int.from_bytes(blob[:4], "little") == 0x01306B47 and len(blob) == 4 + 2560 * 2560 * 2 + 2560 * 4
    raw = (tmp_path / "b3_txt_attn_gate.bin").read_bytes()
    assert int.from_bytes(raw[:8], "little") == 1 and int.from_bytes(raw[8:16], "little") == 2560
    g = np.frombuffer(raw[16:], np.float32)
    assert abs(g.mean() - 1) < 0.01 and abs(g.std() - 0.02) < 0.005


def _has_gpu() -> bool:
    import torch
    return torch.cuda.is_available()


def _build_dropin(tmpdir):
    """Compiles tests/cpp/dropin_engine.cpp against include/seedvr2_b200.hpp and
    links it with the library (returns the binary path)."""
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    lib_dir = os.path.join(root, "seedvr2-2b-ncnn_b200", "lib")
    exe = os.path.join(str(tmpdir), "dropin_engine")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(root, "include"),
           os.path.join(root, "tests", "cpp", "dropin_engine.cpp"), "-L", lib_dir, "-ls2b",
           f"-Wl,-rpath,{lib_dir}", "-o", exe]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_cpp_dropin_header_compiles_and_links(tmp_path):
    import subprocess
    exe = _build_dropin(tmp_path)
    if not _has_gpu():
        # without a GPU the wrapper fails loudly (bool + message), never silently
        r = subprocess.run([exe, str(tmp_path), str(tmp_path / "out.bin")], capture_output=True, text=True)
        assert r.returncode == 1 and "[DitB200]" in r.stderr


def test_nccl_watchdog_host_logic():
    """The NCCL-path watchdog on simulated work (host only): it returns when
    the work finishes, aborts the communicator once on an asynchronous error
    or after its bound, and reports a failed stream without aborting."""
    L = s2b.lib()
    polls, aborted = ctypes.c_int(), ctypes.c_int()
    import time
    # 0: finishes after a few polls
    assert L.s2b_debug_watchdog_selftest(0, 1000, ctypes.byref(polls), ctypes.byref(aborted)) == 0
    assert polls.value == 4 and aborted.value == 0
    # 1: never finishes -> expires after ~timeout, aborts exactly once
    t0 = time.monotonic()
    assert L.s2b_debug_watchdog_selftest(1, 50, ctypes.byref(polls), ctypes.byref(aborted)) == 2
    dt = time.monotonic() - t0
    assert aborted.value == 1 and 0.04 <= dt < 2.0, dt
    # 2: the communicator reports an asynchronous error -> abort at once
    assert L.s2b_debug_watchdog_selftest(2, 10000, ctypes.byref(polls), ctypes.byref(aborted)) == 1
    assert aborted.value == 1 and polls.value == 2
    # 3: the stream itself failed -> reported, no abort
    assert L.s2b_debug_watchdog_selftest(3, 10000, ctypes.byref(polls), ctypes.byref(aborted)) == 3
    assert aborted.value == 0
    assert L.s2b_debug_watchdog_selftest(7, 10, None, None) == -1


def test_forward_output_buffer_validation():
    ok = np.zeros((3, 64), np.float32)
    assert s2b._out(ok, 3) is ok
    assert s2b._out(None, 3).shape == (3, 64)
    for bad in (np.zeros((3, 64), np.float64), np.zeros((4, 64), np.float32), np.zeros((64, 3), np.float32).T):
        with pytest.raises(ValueError):
            s2b._out(bad, 3)
