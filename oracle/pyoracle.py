"""pyoracle -- ctypes access to the CPU checkers.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this module; the product never does.

  Port(): oracle/_build/liboracle.so, this repository's C restatement of the
          reference algorithm (oracle/oracle.c).
  Ref():  oracle/_ref/libref_dit.so, the reference's own src/dit_vk.cpp,
          src/awa_window.cpp and src/test_awa_unit.cpp compiled unchanged
          against the CPU ncnn stand-in (oracle/ncnn_shim).  Built only where
          the reference tree exists; the .so travels with the repository.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_LIB = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_dit.so")

_F = ctypes.POINTER(ctypes.c_float)
_I = ctypes.POINTER(ctypes.c_int)


def _p(a):
    return None if a is None else a.ctypes.data_as(_F)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class or_win(ctypes.Structure):
    _fields_ = [("t", ctypes.c_int), ("h", ctypes.c_int), ("w", ctypes.c_int), ("nwin", ctypes.c_int),
                ("txt_len", ctypes.c_int), ("sl6", _I), ("vf", _F), ("tf", _F)]


def have_port() -> bool:
    return os.path.exists(PORT_LIB)


def have_ref() -> bool:
    return os.path.exists(REF_LIB)


class Port:
    """oracle/oracle.c through ctypes."""

    def __init__(self):
        L = ctypes.CDLL(PORT_LIB)
        L.or_make_windows.argtypes = [ctypes.c_int] * 7 + [_I, ctypes.c_int]
        L.or_make_windows.restype = ctypes.c_int
        L.or_build_freqs.argtypes = [_I, ctypes.c_int, ctypes.c_int, _F, _F]
        L.or_awa.argtypes = [_F, _F, ctypes.c_int, ctypes.c_int, ctypes.POINTER(or_win), _F, _F, _F, _F,
                             ctypes.c_float, _F, _F]
        L.or_linear.argtypes = [_F, ctypes.c_int, ctypes.c_int, _F, ctypes.c_int, _F, _F]
        L.or_model_load.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int]
        L.or_model_load.restype = ctypes.c_void_p
        L.or_model_free.argtypes = [ctypes.c_void_p]
        L.or_time_embedding.argtypes = [ctypes.c_void_p, ctypes.c_float, _F]
        L.or_model_set_graph_last_layer.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.or_set_operand_rounding.argtypes = [ctypes.c_int]
        L.or_forward_latent.argtypes = [ctypes.c_void_p, ctypes.POINTER(or_win), ctypes.POINTER(or_win), _F,
                                        ctypes.c_int, _F, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, _F, _F, _F]
        L.or_forward_latent.restype = ctypes.c_int
        L.or_patchify.argtypes = [_F, ctypes.c_int, ctypes.c_int, ctypes.c_int, _F]
        L.or_synth_normal.argtypes = [_F, ctypes.c_long, ctypes.c_uint64, ctypes.c_char_p, ctypes.c_float,
                                      ctypes.c_float]
        L.or_synth_write_m5.argtypes = [ctypes.c_char_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_int]
        L.or_synth_write_m5.restype = ctypes.c_int
        L.or_synth_vid_grid.argtypes = [_F, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64]
        L.or_synth_txt.argtypes = [_F, ctypes.c_int, ctypes.c_uint64]
        self.L = L
        self._model = None

    # synthetic model and inputs (the product's generator, restated) ------
    def synth_normal(self, shape, seed, stream, mean=0.0, std=1.0):
        out = np.zeros(int(np.prod(shape)), np.float32)
        self.L.or_synth_normal(_p(out), out.size, seed, stream.encode(), mean, std)
        return out.reshape(shape)

    def synth_write_m5(self, path, seed, lo=0, hi=32):
        rc = self.L.or_synth_write_m5(path.encode(), seed, lo, hi)
        assert rc == 0, f"could not write the synthetic model to {path}"

    def synth_vid_grid(self, T, H, W, seed):
        g = np.zeros((T, H, W, 33), np.float32)
        self.L.or_synth_vid_grid(_p(g), T, H, W, seed)
        return g

    def synth_txt(self, TXT, seed):
        t = np.zeros((TXT, 5120), np.float32)
        self.L.or_synth_txt(_p(t), TXT, seed)
        return t

    def patchify_grid(self, grid):
        g = _f32(grid)
        T, H, W, C = g.shape
        assert C == 33 and H % 2 == 0 and W % 2 == 0
        out = np.zeros((T * (H // 2) * (W // 2), 132), np.float32)
        self.L.or_patchify(_p(g), T, H, W, _p(out))
        return out

    # geometry -----------------------------------------------------------
    def make_win(self, t, h, w, nw=(4, 3, 3), txt_len=58, shifted=False):
        cap = 4096
        sl = np.zeros(cap * 6, np.int32)
        n = self.L.or_make_windows(t, h, w, nw[0], nw[1], nw[2], int(shifted), sl.ctypes.data_as(_I), cap)
        assert n >= 0
        sl = sl[: n * 6].reshape(n, 6).copy()
        sizes = (sl[:, 1] - sl[:, 0]) * (sl[:, 3] - sl[:, 2]) * (sl[:, 5] - sl[:, 4])
        vf = np.zeros(int(sizes.sum()) * 126, np.float32)
        tf = np.zeros(n * txt_len * 126, np.float32)
        self.L.or_build_freqs(sl.ctypes.data_as(_I), n, txt_len, _p(vf), _p(tf))
        return sl, vf, tf

    @staticmethod
    def _cwin(t, h, w, txt_len, sl, vf, tf, keep):
        sl = np.ascontiguousarray(sl, np.int32).reshape(-1)
        vf, tf = _f32(vf), _f32(tf)
        keep += [sl, vf, tf]
        return or_win(t, h, w, len(sl) // 6, txt_len, sl.ctypes.data_as(_I), _p(vf), _p(tf))

    def awa(self, vqkv, tqkv, t, h, w, txt_len, sl, vf, tf, nqv, nkv, nqt, nkt, eps):
        keep = []
        cw = self._cwin(t, h, w, txt_len, sl, vf, tf, keep)
        a = [_f32(x) for x in (vqkv, tqkv, nqv, nkv, nqt, nkt)]
        Lv, TXT = a[0].shape[0], a[1].shape[0]
        vo, to = np.zeros((Lv, 2560), np.float32), np.zeros((TXT, 2560), np.float32)
        self.L.or_awa(_p(a[0]), _p(a[1]), Lv, TXT, ctypes.byref(cw), _p(a[2]), _p(a[3]), _p(a[4]), _p(a[5]),
                      eps, _p(vo), _p(to))
        return vo, to

    def linear(self, x, W, b=None):
        x, W = _f32(x), _f32(W)
        b = None if b is None else _f32(b)
        y = np.zeros((x.shape[0], W.shape[0]), np.float32)
        self.L.or_linear(_p(x), x.shape[0], x.shape[1], _p(W), W.shape[0], _p(b), _p(y))
        return y

    # model ---------------------------------------------------------------
    def load(self, m5_dir, l0, l1):
        if self._model:
            self.L.or_model_free(self._model)
        self._model = self.L.or_model_load(m5_dir.encode(), l0, l1)
        assert self._model, f"oracle could not load {m5_dir}"

    def set_operand_rounding(self, mode: int):
        """0 fp32, 1 bf16, 2 fp16 operands (emulation; process-wide)."""
        self.L.or_set_operand_rounding(int(mode))

    def set_graph_last_layer(self, on: bool):
        """Layer 31 with the chunked graph's txt semantics (see oracle.h)."""
        self.L.or_model_set_graph_last_layer(self._model, int(on))

    def time_embedding(self, t):
        e = np.zeros(15360, np.float32)
        self.L.or_time_embedding(self._model, t, _p(e))
        return e

    def forward_latent(self, geo_ns, geo_sh, vid_in, txt_in, t, l0, l1, do_init, do_final):
        """geo_*: (T, H, W, txt_len, slices, vid_freq, txt_freq)."""
        keep = []
        ns = self._cwin(*geo_ns, keep)
        sh = self._cwin(*geo_sh, keep)
        v, x = _f32(vid_in), _f32(txt_in)
        Lv, TXT = v.shape[0], x.shape[0]
        vl = np.zeros((Lv, 2560), np.float32)
        tl = np.zeros((TXT, 2560), np.float32)
        sr = np.zeros((Lv, 64), np.float32)
        rc = self.L.or_forward_latent(self._model, ctypes.byref(ns), ctypes.byref(sh), _p(v), Lv, _p(x), TXT, t,
                                      l0, l1, int(do_init), int(do_final), _p(vl), _p(tl), _p(sr))
        assert rc == 0
        return (None, None, sr) if do_final else (vl, tl, None)

    def close(self):
        if self._model:
            self.L.or_model_free(self._model)
            self._model = None


class Ref:
    """The reference's own CPU code (oracle/_ref/libref_dit.so)."""

    def __init__(self):
        L = ctypes.CDLL(REF_LIB)
        vp = ctypes.c_void_p
        L.ref_win_new.argtypes = [ctypes.c_int] * 8
        L.ref_win_new.restype = vp
        L.ref_win_from.argtypes = [ctypes.c_int] * 5 + [_I, _F, ctypes.c_long, _F, ctypes.c_long]
        L.ref_win_from.restype = vp
        L.ref_win_nwin.argtypes = [vp]
        L.ref_win_nvf.argtypes = [vp]
        L.ref_win_nvf.restype = ctypes.c_long
        L.ref_win_ntf.argtypes = [vp]
        L.ref_win_ntf.restype = ctypes.c_long
        L.ref_win_get.argtypes = [vp, _I, _F, _F]
        L.ref_win_free.argtypes = [vp]
        L.ref_dit_new.argtypes = [ctypes.c_char_p]
        L.ref_dit_new.restype = vp
        L.ref_dit_set_windows.argtypes = [vp, vp, vp]
        L.ref_dit_forward_latent.argtypes = [vp, _F, ctypes.c_int, ctypes.c_int, _F, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             _F, _F, _F]
        L.ref_dit_free.argtypes = [vp]
        L.ref_cpu_awa.argtypes = [_F, _F, vp, _F, _F, _F, _F, ctypes.c_int, ctypes.c_int, _F, _F]
        self.L = L
        self._dit = None

    def make_win(self, t, h, w, nw=(4, 3, 3), txt_len=58, shifted=False):
        p = self.L.ref_win_new(t, h, w, nw[0], nw[1], nw[2], txt_len, int(shifted))
        n = self.L.ref_win_nwin(p)
        sl = np.zeros(n * 6, np.int32)
        vf = np.zeros(self.L.ref_win_nvf(p), np.float32)
        tf = np.zeros(self.L.ref_win_ntf(p), np.float32)
        self.L.ref_win_get(p, sl.ctypes.data_as(_I), _p(vf), _p(tf))
        self.L.ref_win_free(p)
        return sl.reshape(n, 6), vf, tf

    def _win(self, t, h, w, txt_len, sl, vf, tf):
        sl = np.ascontiguousarray(sl, np.int32).reshape(-1)
        vf, tf = _f32(vf), _f32(tf)
        return self.L.ref_win_from(t, h, w, len(sl) // 6, txt_len, sl.ctypes.data_as(_I), _p(vf), vf.size,
                                   _p(tf), tf.size)

    def cpu_awa(self, vqkv, tqkv, t, h, w, txt_len, sl, vf, tf, nqv, nkv, nqt, nkt):
        """src/test_awa_unit.cpp:27-70 (qk_norm eps fixed at 1e-5 there)."""
        wp = self._win(t, h, w, txt_len, sl, vf, tf)
        a = [_f32(x) for x in (vqkv, tqkv, nqv, nkv, nqt, nkt)]
        Lv, TXT = a[0].shape[0], a[1].shape[0]
        vo, to = np.zeros((Lv, 2560), np.float32), np.zeros((TXT, 2560), np.float32)
        self.L.ref_cpu_awa(_p(a[0]), _p(a[1]), wp, _p(a[2]), _p(a[3]), _p(a[4]), _p(a[5]), Lv, TXT, _p(vo), _p(to))
        self.L.ref_win_free(wp)
        return vo, to

    def load(self, m5_dir):
        if self._dit:
            self.L.ref_dit_free(self._dit)
        self._dit = self.L.ref_dit_new(m5_dir.encode())
        assert self._dit

    def forward_latent(self, geo_ns, geo_sh, vid_in, txt_in, t, l0, l1, do_init, do_final):
        ns = self._win(*geo_ns)
        sh = self._win(*geo_sh)
        self.L.ref_dit_set_windows(self._dit, ns, sh)
        self.L.ref_win_free(ns)
        self.L.ref_win_free(sh)
        v, x = _f32(vid_in), _f32(txt_in)
        Lv, TXT = v.shape[0], x.shape[0]
        vl = np.zeros((Lv, 2560), np.float32)
        tl = np.zeros((TXT, 2560), np.float32)
        sr = np.zeros((Lv, 64), np.float32)
        rc = self.L.ref_dit_forward_latent(self._dit, _p(v), Lv, v.shape[1], _p(x), TXT, x.shape[1], t, l0, l1,
                                           int(do_init), int(do_final), _p(vl), _p(tl), _p(sr))
        assert rc == 0
        return (None, None, sr) if do_final else (vl, tl, None)

    def close(self):
        if self._dit:
            self.L.ref_dit_free(self._dit)
            self._dit = None
