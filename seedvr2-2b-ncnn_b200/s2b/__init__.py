"""s2b -- Python mirror of the B200 NaDiT/AWA C ABI (include/seedvr2_b200.h).

The product is lib/libs2b.so (sm_100a kernels + C++ host engine); this module
binds it with ctypes and mirrors the reference engine's operator interfaces
(DitVk::forward_latent / forward / forward_grid, AwaVk::forward,
awa::make_win, AdaCompose) with the same argument meaning and error
behaviour (a non-zero status raises S2BError carrying s2b_last_error).
There is no CPU fallback: without the library or without a B200 the calls
fail loudly.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

HEADS, HEAD_D, DIM, QKV = 20, 128, 2560, 7680
NUM_LAYERS, MM_LAYERS, MLP_DIM, ROPE_ROT = 32, 10, 6912, 126
PATCH_IN, TXT_IN, OUT_CH, EMB_DIM = 132, 5120, 64, 15360
PREC_FP32, PREC_FP16, PREC_BF16 = 0, 1, 2

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG, "lib", "libs2b.so")

_F32P = ctypes.POINTER(ctypes.c_float)
_I32P = ctypes.POINTER(ctypes.c_int)


class S2BError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"s2b status {code}: {msg}")
        self.code = code


class s2b_weight_file(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.c_void_p), ("bytes", ctypes.c_size_t)]


class s2b_win(ctypes.Structure):
    _fields_ = [("t", ctypes.c_int), ("h", ctypes.c_int), ("w", ctypes.c_int), ("nwin", ctypes.c_int),
                ("txt_len", ctypes.c_int),
                ("st", _I32P), ("en", _I32P), ("sh", _I32P), ("eh", _I32P), ("sw", _I32P), ("ew", _I32P),
                ("vid_freq", _F32P), ("n_vid_freq", ctypes.c_long),
                ("txt_freq", _F32P), ("n_txt_freq", ctypes.c_long)]


_lib = None


def lib() -> ctypes.CDLL:
    """Load lib/libs2b.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(f"{LIB_PATH} is missing: build it with __graft_entry__.build()")
    L = ctypes.CDLL(LIB_PATH)
    vp, ip, u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64
    sig = {
        "s2b_ctx_create": [ip, ip, ctypes.POINTER(vp)],
        "s2b_ctx_destroy": [vp],
        "s2b_ctx_precision": [vp],
        "s2b_ctx_device_bytes": [vp, ctypes.POINTER(u64)],
        "s2b_ctx_last_launches": [vp, ctypes.POINTER(ip)],
        "s2b_load_weights_dir": [vp, ctypes.c_char_p, ip, ip],
        "s2b_load_weights_synth": [vp, u64, ip, ip],
        "s2b_make_win_size": [ip, ip, ip, _I32P, ip, ip, _I32P, ctypes.POINTER(ctypes.c_long), ctypes.POINTER(ctypes.c_long)],
        "s2b_make_win_fill": [ip, ip, ip, _I32P, ip, ip, _I32P, _I32P, _I32P, _I32P, _I32P, _I32P, _F32P, _F32P],
        "s2b_set_windows": [vp, ctypes.POINTER(s2b_win), ctypes.POINTER(s2b_win)],
        "s2b_forward_latent": [vp, _F32P, ip, _F32P, ip, ctypes.c_float, ip, ip, ip, ip, _F32P, _F32P, _F32P],
        "s2b_forward": [vp, _F32P, ip, _F32P, ip, ctypes.c_float, _F32P],
        "s2b_forward_dev": [vp, vp, ip, vp, ip, ctypes.c_float, vp, vp],
        "s2b_forward_grid": [vp, _F32P, ip, ip, ip, _F32P, ip, ctypes.c_float, _F32P],
        "s2b_forward_grid_dev": [vp, vp, ip, ip, ip, vp, ip, ctypes.c_float, vp, vp],
        "s2b_load_weights_mem": [vp, ctypes.POINTER(s2b_weight_file), ip, ip, ip],
        "s2b_group_create": [ip, _I32P, ip, ctypes.POINTER(vp)],
        "s2b_group_destroy": [vp],
        "s2b_group_load_weights_dir": [vp, ctypes.c_char_p],
        "s2b_group_load_weights_synth": [vp, u64],
        "s2b_group_set_windows": [vp, ctypes.POINTER(s2b_win), ctypes.POINTER(s2b_win)],
        "s2b_group_forward_frames": [vp, _F32P, ip, ip, _F32P, ip, ctypes.c_float, _F32P],
        "s2b_patchify_grid_dev": [vp, ip, ip, ip, vp, vp],
        "s2b_unpatchify_latent_dev": [vp, ip, ip, ip, vp, vp],
        "s2b_assemble_vid_grid_dev": [vp, vp, ctypes.c_float, ip, ip, vp, vp],
        "s2b_decode_latent_dev": [vp, vp, ctypes.c_float, ip, ip, vp, vp],
        "s2b_patchify_grid": [_F32P, ip, ip, ip, _F32P],
        "s2b_unpatchify_latent": [_F32P, ip, ip, ip, _F32P],
        "s2b_awa_forward": [vp, _F32P, _F32P, ctypes.POINTER(s2b_win), _F32P, _F32P, _F32P, _F32P, ip, ip,
                            ctypes.c_float, _F32P, _F32P],
        "s2b_awa_set_geometry": [vp, ip, ctypes.POINTER(s2b_win)],
        "s2b_awa_forward_dev": [vp, ip, vp, vp, vp, vp, vp, vp, ip, ip, ctypes.c_float, vp, vp, vp],
        "s2b_time_embedding": [vp, ctypes.c_float, _F32P],
        "s2b_ada_compose": [vp, _F32P, _F32P],
        "s2b_linear": [vp, _F32P, ip, ip, _F32P, ip, _F32P, _F32P],
        "s2b_forward_profile": [vp, _F32P, ip, _F32P, ip, ctypes.c_float, ctypes.POINTER(ctypes.c_double),
                                ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double), _I32P],
        "s2b_linear_bf16_dev": [vp, vp, ip, ip, vp, ip, vp, vp, vp],
        "s2b_synth_write_m5": [ctypes.c_char_p, u64, ip, ip],
        "s2b_synth_vid_grid": [_F32P, ip, ip, ip, u64],
        "s2b_synth_txt": [_F32P, ip, u64],
        "s2b_synth_normal": [_F32P, ctypes.c_long, u64, ctypes.c_char_p, ctypes.c_float, ctypes.c_float],
        "s2b_nccl_unique_id": [ctypes.POINTER(ctypes.c_uint8)],
        "s2b_shard_init": [vp, ctypes.POINTER(ctypes.c_uint8), ip, ip],
        "s2b_shard_forward": [vp, _F32P, ip, _F32P, ip, ctypes.c_float, _F32P],
        "s2b_shard_forward_dev": [vp, vp, ip, vp, ip, ctypes.c_float, vp, vp],
        "s2b_shard_forward_profile": [vp, _F32P, ip, _F32P, ip, ctypes.c_float, ctypes.POINTER(ctypes.c_double),
                                      ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double), _I32P],
        "s2b_shard_plan": [ctypes.POINTER(s2b_win), ctypes.POINTER(s2b_win), ip, ip, _I32P, _I32P, _I32P, _I32P,
                           _I32P, _I32P, _I32P],
        "s2b_shard_resync": [vp],
        "s2b_set_last_layer_semantics": [vp, ip],
        "s2b_check_errors": [vp],
        "s2b_debug_raise_kernel_error": [vp, ip],
        "s2b_debug_watchdog_selftest": [ip, ip, _I32P, _I32P],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    L.s2b_last_error.argtypes = [vp]
    L.s2b_last_error.restype = ctypes.c_char_p
    L.s2b_group_last_error.argtypes = [vp]
    L.s2b_group_last_error.restype = ctypes.c_char_p
    _lib = L
    return L


def exported_symbols() -> list[str]:
    """Names of every function include/seedvr2_b200.h declares."""
    import re
    hdr = os.path.join(os.path.dirname(_PKG), "include", "seedvr2_b200.h")
    txt = open(hdr).read()
    return sorted(set(re.findall(r"^(?:int|const char\*)\s+(s2b_\w+)\(", txt, flags=re.M)))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _out(out, Lv: int) -> np.ndarray:
    if out is None:
        return np.zeros((Lv, OUT_CH), np.float32)
    if out.dtype != np.float32 or out.shape != (Lv, OUT_CH) or not out.flags["C_CONTIGUOUS"]:
        raise ValueError(f"out must be a C-contiguous float32 array of shape ({Lv}, {OUT_CH})")
    return out


def _p(a: np.ndarray):
    return a.ctypes.data_as(_F32P) if a is not None else None


def _check(ctx, rc: int):
    if rc != 0:
        msg = lib().s2b_last_error(ctx)
        raise S2BError(rc, msg.decode() if msg else "")


# ---------------------------------------------------------------- geometry
@dataclass
class Win:
    """Python mirror of the reference `Win` (src/dit_vk.h:17-22)."""
    t: int
    h: int
    w: int
    txt_len: int
    slices: np.ndarray                 # (nwin, 6) int32: st, en, sh, eh, sw, ew
    vid_freq: np.ndarray               # (sum f_i * 126,) float32
    txt_freq: np.ndarray               # (nwin * txt_len * 126,) float32
    _keep: list = field(default_factory=list, repr=False)

    @property
    def nwin(self) -> int:
        return int(self.slices.shape[0])

    @property
    def sizes(self) -> np.ndarray:
        s = self.slices
        return (s[:, 1] - s[:, 0]) * (s[:, 3] - s[:, 2]) * (s[:, 5] - s[:, 4])

    def as_c(self) -> s2b_win:
        cols = [np.ascontiguousarray(self.slices[:, k], dtype=np.int32) for k in range(6)]
        vf, tf = _f32(self.vid_freq), _f32(self.txt_freq)
        self._keep = cols + [vf, tf]
        ip = [c.ctypes.data_as(_I32P) for c in cols]
        return s2b_win(self.t, self.h, self.w, self.nwin, self.txt_len, *ip, _p(vf), vf.size, _p(tf), tf.size)


def make_win(t: int, h: int, w: int, num_windows=(4, 3, 3), txt_len: int = 58, shifted: bool = False) -> Win:
    """awa::make_win (src/awa_window.cpp:161-178), computed by the library."""
    L = lib()
    nw = (ctypes.c_int * 3)(*num_windows)
    n, nvf, ntf = ctypes.c_int(), ctypes.c_long(), ctypes.c_long()
    rc = L.s2b_make_win_size(t, h, w, nw, txt_len, int(shifted), ctypes.byref(n), ctypes.byref(nvf), ctypes.byref(ntf))
    _check(None, rc)
    cols = [np.zeros(n.value, np.int32) for _ in range(6)]
    vf, tf = np.zeros(nvf.value, np.float32), np.zeros(ntf.value, np.float32)
    rc = L.s2b_make_win_fill(t, h, w, nw, txt_len, int(shifted), *[c.ctypes.data_as(_I32P) for c in cols], _p(vf), _p(tf))
    _check(None, rc)
    return Win(t, h, w, txt_len, np.stack(cols, axis=1).astype(np.int32), vf, tf)


# ---------------------------------------------------------------- synthetic data
def _same_nccl_as_torch():
    """The library resolves libnccl.so.2 at run time; importing torch first
    makes that the copy torch.distributed uses, so every process of a job
    (and torch's own process group) runs one NCCL version."""
    try:
        import torch  # noqa: F401
    except ImportError:
        pass


class FrameGroup:
    """Frame-sequence mode on several GPUs from one process (s2b_group_*)."""

    def __init__(self, ngpu: int, precision: int = PREC_BF16, devices=None):
        self._g = ctypes.c_void_p()
        dev = None if devices is None else (ctypes.c_int * ngpu)(*devices)
        rc = lib().s2b_group_create(ngpu, dev, precision, ctypes.byref(self._g))
        if rc != 0:
            raise S2BError(rc, (lib().s2b_last_error(None) or b"").decode())
        self.ngpu = ngpu

    def _c(self, rc):
        if rc != 0:
            raise S2BError(rc, (lib().s2b_group_last_error(self._g) or b"").decode())

    def init_synth(self, seed: int):
        self._c(lib().s2b_group_load_weights_synth(self._g, seed))

    def init(self, model_dir: str):
        self._c(lib().s2b_group_load_weights_dir(self._g, model_dir.encode()))

    def set_windows(self, ns: "Win", sh: "Win"):
        a, b = ns.as_c(), sh.as_c()
        self._c(lib().s2b_group_set_windows(self._g, ctypes.byref(a), ctypes.byref(b)))

    def forward_frames(self, vid_patches, Lv, txt, TXT, timestep=1000.0):
        v, t = _f32(vid_patches), _f32(txt)
        n = v.shape[0]
        out = np.zeros((n, Lv, OUT_CH), np.float32)
        self._c(lib().s2b_group_forward_frames(self._g, _p(v), n, Lv, _p(t), TXT, timestep, _p(out)))
        return out

    def close(self):
        if self._g:
            lib().s2b_group_destroy(self._g)
            self._g = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def nccl_unique_id() -> bytes:
    """A fresh ncclUniqueId (rank 0 creates it and shares it with the others)."""
    _same_nccl_as_torch()
    buf = (ctypes.c_uint8 * 128)()
    rc = lib().s2b_nccl_unique_id(buf)
    if rc != 0:
        raise S2BError(rc, "ncclGetUniqueId failed (is libnccl.so.2 loadable?)")
    return bytes(buf)


@dataclass
class ShardPlan:
    """Window ownership / residual exchange plan of one rank (s2b_shard_plan)."""
    bounds: list        # [2] arrays of world+1 window boundaries
    tokens: list        # [2] grid token of every local row
    send_off: list
    send_idx: list
    recv_off: list
    recv_idx: list


def shard_plan(ns: Win, sh: Win, world: int, rank: int) -> ShardPlan:
    Lv = ns.t * ns.h * ns.w
    a, b = ns.as_c(), sh.as_c()
    bounds = np.zeros((2, world + 1), np.int32)
    n_local = np.zeros(2, np.int32)
    tokens = np.zeros((2, Lv), np.int32)
    soff, roff = np.zeros((2, world + 1), np.int32), np.zeros((2, world + 1), np.int32)
    sidx, ridx = np.zeros((2, Lv), np.int32), np.zeros((2, Lv), np.int32)
    P = lambda x: x.ctypes.data_as(_I32P)
    rc = lib().s2b_shard_plan(ctypes.byref(a), ctypes.byref(b), world, rank, P(bounds), P(n_local), P(tokens),
                              P(soff), P(sidx), P(roff), P(ridx))
    if rc != 0:
        raise S2BError(rc, "s2b_shard_plan rejected the geometry")
    n = [int(n_local[0]), int(n_local[1])]
    return ShardPlan(bounds=[bounds[p].copy() for p in range(2)], tokens=[tokens[p, :n[p]].copy() for p in range(2)],
                     send_off=[soff[p].copy() for p in range(2)],
                     send_idx=[sidx[p, :soff[p, -1]].copy() for p in range(2)],
                     recv_off=[roff[p].copy() for p in range(2)],
                     recv_idx=[ridx[p, :roff[p, -1]].copy() for p in range(2)])


def synth_write_m5(path: str, seed: int, layer_lo: int = 0, layer_hi: int = NUM_LAYERS):
    _check(None, lib().s2b_synth_write_m5(path.encode(), seed, layer_lo, layer_hi))


def synth_vid_grid(T: int, H: int, W: int, seed: int) -> np.ndarray:
    g = np.zeros((T, H, W, 33), np.float32)
    _check(None, lib().s2b_synth_vid_grid(_p(g), T, H, W, seed))
    return g


def synth_txt(TXT: int, seed: int) -> np.ndarray:
    x = np.zeros((TXT, TXT_IN), np.float32)
    _check(None, lib().s2b_synth_txt(_p(x), TXT, seed))
    return x


def synth_normal(shape, seed: int, stream: str, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    x = np.zeros(shape, np.float32)
    _check(None, lib().s2b_synth_normal(_p(x), x.size, seed, stream.encode(), mean, std))
    return x


def patchify_grid(grid: np.ndarray) -> np.ndarray:
    T, H, W, _ = grid.shape
    g = _f32(grid)
    out = np.zeros((T * (H // 2) * (W // 2), PATCH_IN), np.float32)
    _check(None, lib().s2b_patchify_grid(_p(g), T, H, W, _p(out)))
    return out


def unpatchify_latent(sr: np.ndarray, T: int, H: int, W: int) -> np.ndarray:
    s = _f32(sr)
    out = np.zeros((T, H, W, 16), np.float32)
    _check(None, lib().s2b_unpatchify_latent(_p(s), T, H, W, _p(out)))
    return out


# ---------------------------------------------------------------- engine
class DitB200:
    """The reference DitVk method set (src/dit_vk.h:24-121) on one B200."""

    def __init__(self, device: int = 0, precision: int = PREC_BF16):
        self._ctx = ctypes.c_void_p()
        rc = lib().s2b_ctx_create(device, precision, ctypes.byref(self._ctx))
        _check(None, rc)
        self.precision = precision

    def close(self):
        if self._ctx:
            lib().s2b_ctx_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _c(self, rc):
        _check(self._ctx, rc)

    def init(self, model_dir: str, layer_lo: int = 0, layer_hi: int = NUM_LAYERS):
        """DitVk::init weight half: the m5 directory layout."""
        self._c(lib().s2b_load_weights_dir(self._ctx, model_dir.encode(), layer_lo, layer_hi))

    def init_mem(self, files: dict, layer_lo: int = 0, layer_hi: int = NUM_LAYERS):
        """s2b_load_weights_mem: files maps m5 file names to their bytes."""
        bufs = {k: ctypes.create_string_buffer(v, len(v)) for k, v in files.items()}
        arr = (s2b_weight_file * len(files))()
        for i, (k, b) in enumerate(bufs.items()):
            arr[i].name = k.encode()
            arr[i].data = ctypes.cast(b, ctypes.c_void_p)
            arr[i].bytes = len(files[k])
        self._c(lib().s2b_load_weights_mem(self._ctx, arr, len(files), layer_lo, layer_hi))

    def init_synth(self, seed: int, layer_lo: int = 0, layer_hi: int = NUM_LAYERS):
        self._c(lib().s2b_load_weights_synth(self._ctx, seed, layer_lo, layer_hi))

    def set_windows(self, ns: Win, sh: Win):
        a, b = ns.as_c(), sh.as_c()
        self._c(lib().s2b_set_windows(self._ctx, ctypes.byref(a), ctypes.byref(b)))

    def forward_latent(self, vid_in, Lv, txt_in, TXT, timestep, l0, l1, do_init, do_final):
        v, t = _f32(vid_in), _f32(txt_in)
        if do_final:
            sr = np.zeros((Lv, OUT_CH), np.float32)
            self._c(lib().s2b_forward_latent(self._ctx, _p(v), Lv, _p(t), TXT, timestep, l0, l1, int(do_init), 1,
                                             None, None, _p(sr)))
            return None, None, sr
        vl, tl = np.zeros((Lv, DIM), np.float32), np.zeros((TXT, DIM), np.float32)
        self._c(lib().s2b_forward_latent(self._ctx, _p(v), Lv, _p(t), TXT, timestep, l0, l1, int(do_init), 0,
                                         _p(vl), _p(tl), None))
        return vl, tl, None

    def forward(self, vid_patch, Lv, txt, TXT, timestep=1000.0, out=None):
        """sr (Lv, 64); `out`, when given, is the float32 C-contiguous array written
        (a page-locked one makes the device-to-host copy direct)."""
        v, t = _f32(vid_patch), _f32(txt)
        sr = _out(out, Lv)
        self._c(lib().s2b_forward(self._ctx, _p(v), Lv, _p(t), TXT, timestep, _p(sr)))
        return sr

    def forward_dev(self, d_vid: int, Lv: int, d_txt: int, TXT: int, timestep: float, d_sr: int, stream: int):
        self._c(lib().s2b_forward_dev(self._ctx, d_vid, Lv, d_txt, TXT, timestep, d_sr, stream))

    def linear_bf16_dev(self, d_x: int, M: int, K: int, d_w: int, N: int, d_bias, d_y: int, stream: int):
        """y = x W^T (+ bias) on device bf16 buffers (pointers as ints), enqueued on `stream`."""
        self._c(lib().s2b_linear_bf16_dev(self._ctx, d_x, M, K, d_w, N, d_bias, d_y, stream))

    def forward_grid(self, vid_grid, txt, TXT, timestep=1000.0):
        T, H, W, _ = vid_grid.shape
        g, t = _f32(vid_grid), _f32(txt)
        out = np.zeros((T, H, W, 16), np.float32)
        self._c(lib().s2b_forward_grid(self._ctx, _p(g), T, H, W, _p(t), TXT, timestep, _p(out)))
        return out

    def forward_grid_dev(self, d_grid: int, T: int, H: int, W: int, d_txt: int, TXT: int, timestep: float,
                         d_sr_grid: int, stream: int):
        self._c(lib().s2b_forward_grid_dev(self._ctx, d_grid, T, H, W, d_txt, TXT, timestep, d_sr_grid, stream))

    def awa_forward(self, vqkv, tqkv, win: Win, nq_v, nk_v, nq_t, nk_t, Lv, TXT, eps=1e-5):
        """AwaVk::forward (src/awa_vk.h:39-44)."""
        a = [_f32(x) for x in (vqkv, tqkv, nq_v, nk_v, nq_t, nk_t)]
        cw = win.as_c()
        vo, to = np.zeros((Lv, DIM), np.float32), np.zeros((TXT, DIM), np.float32)
        self._c(lib().s2b_awa_forward(self._ctx, _p(a[0]), _p(a[1]), ctypes.byref(cw), _p(a[2]), _p(a[3]),
                                      _p(a[4]), _p(a[5]), Lv, TXT, eps, _p(vo), _p(to)))
        return vo, to

    def awa_set_geometry(self, win_type: int, win: Win):
        cw = win.as_c()
        self._c(lib().s2b_awa_set_geometry(self._ctx, win_type, ctypes.byref(cw)))

    def awa_forward_dev(self, win_type, d_vqkv, d_tqkv, d_nqv, d_nkv, d_nqt, d_nkt, Lv, TXT, eps, d_vout, d_tout,
                        stream):
        self._c(lib().s2b_awa_forward_dev(self._ctx, win_type, d_vqkv, d_tqkv, d_nqv, d_nkv, d_nqt, d_nkt, Lv, TXT,
                                          eps, d_vout, d_tout, stream))

    def time_embedding(self, timestep: float) -> np.ndarray:
        e = np.zeros(EMB_DIM, np.float32)
        self._c(lib().s2b_time_embedding(self._ctx, timestep, _p(e)))
        return e

    def ada_compose(self, emb) -> np.ndarray:
        e = _f32(emb)
        out = np.zeros((NUM_LAYERS * 12 + 2, DIM), np.float32)
        self._c(lib().s2b_ada_compose(self._ctx, _p(e), _p(out)))
        return out

    KERNEL_KINDS = ("gemm_tcgen05", "gemm_fp32", "attention", "awa_pack", "norm_convert", "other", "exchange")

    def forward_profile(self, vid_patch, Lv, txt, TXT, timestep=1000.0, sharded=False) -> dict:
        """Per kernel class: device ms, algorithmic FLOPs / bytes, launches (CUDA events).
        sharded: this rank's part of the window-sharded forward."""
        v, t = _f32(vid_patch), _f32(txt)
        D7 = ctypes.c_double * 7
        ms, fl, by, n = D7(), D7(), D7(), (ctypes.c_int * 7)()
        fn = lib().s2b_shard_forward_profile if sharded else lib().s2b_forward_profile
        self._c(fn(self._ctx, _p(v), Lv, _p(t), TXT, timestep, ms, fl, by, n))
        return {k: dict(ms=ms[i], flops=fl[i], bytes=by[i], launches=n[i]) for i, k in enumerate(self.KERNEL_KINDS)}

    # ---- window-sharded image mode (one rank per GPU, NCCL)
    def shard_init(self, nccl_id: bytes, world: int, rank: int):
        """Joins the window-sharded group (every rank calls it together)."""
        if len(nccl_id) != 128:
            raise ValueError("nccl_id must be 128 bytes")
        _same_nccl_as_torch()
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(nccl_id)
        self._c(lib().s2b_shard_init(self._ctx, buf, world, rank))

    def shard_forward(self, vid_patch, Lv, txt, TXT, timestep=1000.0, out=None):
        v, t = _f32(vid_patch), _f32(txt)
        sr = _out(out, Lv)
        self._c(lib().s2b_shard_forward(self._ctx, _p(v), Lv, _p(t), TXT, timestep, _p(sr)))
        return sr

    def shard_forward_dev(self, d_vid: int, Lv: int, d_txt: int, TXT: int, timestep: float, d_sr: int, stream: int):
        self._c(lib().s2b_shard_forward_dev(self._ctx, d_vid, Lv, d_txt, TXT, timestep, d_sr, stream))

    def set_last_layer_semantics(self, graph: bool):
        """Layer 31 txt: False = forward_latent's vid_only (default), True = the chunked graph's."""
        self._c(lib().s2b_set_last_layer_semantics(self._ctx, int(graph)))

    def shard_resync(self):
        """Collective: after a failed shard call on any rank, every rank calls
        this before the next shard forward."""
        self._c(lib().s2b_shard_resync(self._ctx))

    def check_errors(self):
        """Raises S2BError(S2B_ERR_TIMEOUT) if a bounded kernel wait expired in
        a stream-ordered (_dev) call since the last report."""
        self._c(lib().s2b_check_errors(self._ctx))

    def debug_raise_kernel_error(self, mask: int):
        """Test hook: raise the device's kernel error flags (1 GEMM, 2 attention, 4 exchange)."""
        self._c(lib().s2b_debug_raise_kernel_error(self._ctx, mask))

    def last_launches(self) -> int:
        n = ctypes.c_int()
        self._c(lib().s2b_ctx_last_launches(self._ctx, ctypes.byref(n)))
        return n.value

    def device_bytes(self) -> int:
        n = ctypes.c_uint64()
        self._c(lib().s2b_ctx_device_bytes(self._ctx, ctypes.byref(n)))
        return n.value
