"""Seeded inputs of the parity cases (shared by make_golden.py and tests).

Everything is generated from seeds, so only outputs need to be stored:
  * awa_unit: the reference's own AWA unit case (src/test_awa_unit.cpp:77-88):
    T=1 H=2 W=6 (Lv=12), two windows split along W, TXT=4, unit qk-norm
    weights, every value drawn as (float)mt19937()/mt19937::max()*2-1 scaled
    by 0.1, in the order vid_freq, txt_freq, vqkv, tqkv.  numpy's legacy
    RandomState(seed) runs the same MT19937 with the same integer seeding.
  * awa_cfg: the BASELINE single-op configuration: one frame with a 24x28
    token grid, TXT=58, q/k/v ~ N(0,1), qk-norm weights 1+N(0,0.02), eps 1e-6,
    windows from awa::make_win (4 windows) or the literal 3x3 split (9).
  * dit_small: full-width DiT layers on a 24x28 token grid (Lv=672, TXT=58)
    with the synthetic m5 weights of seed 1234 and inputs of seed 42.
"""
from __future__ import annotations

import numpy as np

HEAD_D, DIM, QKV, ROT = 128, 2560, 7680, 126


def mt_uniform_pm1(rs: np.random.RandomState, n: int) -> np.ndarray:
    """(float)rng()/rng.max()*2-1 in float32, as src/test_awa_unit.cpp:77."""
    u = rs.randint(0, 2 ** 32, size=n, dtype=np.uint64).astype(np.uint32)
    f = u.astype(np.float32) / np.float32(4294967295.0)
    return (f * np.float32(2.0) - np.float32(1.0)).astype(np.float32)


def awa_unit_case():
    """Inputs of src/test_awa_unit.cpp:77-88."""
    rs = np.random.RandomState(123)
    Lv, TXT = 12, 4
    slices = np.array([[0, 1, 0, 2, 0, 3], [0, 1, 0, 2, 3, 6]], np.int32)
    vf = mt_uniform_pm1(rs, 12 * ROT) * np.float32(0.1)
    tf = mt_uniform_pm1(rs, 2 * TXT * ROT) * np.float32(0.1)
    ones = np.ones(HEAD_D, np.float32)
    vqkv = (mt_uniform_pm1(rs, Lv * QKV) * np.float32(0.1)).reshape(Lv, QKV)
    tqkv = (mt_uniform_pm1(rs, TXT * QKV) * np.float32(0.1)).reshape(TXT, QKV)
    return dict(t=1, h=2, w=6, txt_len=TXT, slices=slices, vf=vf, tf=tf, vqkv=vqkv, tqkv=tqkv,
                nqv=ones, nkv=ones, nqt=ones, nkt=ones)


def normal(shape, seed, stream, mean=0.0, std=1.0):
    """Seeded N(mean, std) from the product's generator (Philox4x32-10)."""
    import s2b
    return s2b.synth_normal(shape, seed, stream, mean, std)


def awa_cfg_inputs(Lv: int, TXT: int, seed: int = 7):
    vqkv = normal((Lv, QKV), seed, "awa_vqkv")
    tqkv = normal((TXT, QKV), seed, "awa_tqkv")
    nq = [normal((HEAD_D,), seed, s, 1.0, 0.02) for s in ("nqv", "nkv", "nqt", "nkt")]
    return vqkv, tqkv, nq


def literal_3x3(t: int, h: int, w: int):
    """BASELINE config 1's literal 3x3 split of the H and W axes."""
    hs = np.linspace(0, h, 4).round().astype(int)
    ws = np.linspace(0, w, 4).round().astype(int)
    return np.array([[0, t, hs[i], hs[i + 1], ws[j], ws[j + 1]] for j in range(3) for i in range(3)], np.int32)


def freqs_for(slices: np.ndarray, txt_len: int):
    """RoPE tables for arbitrary slices (src/awa_window.cpp:109-159) via the port."""
    from oracle import pyoracle as po
    import ctypes
    P = po.Port()
    sl = np.ascontiguousarray(slices, np.int32)
    sizes = (sl[:, 1] - sl[:, 0]) * (sl[:, 3] - sl[:, 2]) * (sl[:, 5] - sl[:, 4])
    vf = np.zeros(int(sizes.sum()) * ROT, np.float32)
    tf = np.zeros(len(sl) * txt_len * ROT, np.float32)
    P.L.or_build_freqs(sl.reshape(-1).ctypes.data_as(ctypes.POINTER(ctypes.c_int)), len(sl), txt_len,
                       vf.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), tf.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return vf, tf


DIT_SMALL = dict(T=1, H=24, W=28, TXT=58, wseed=1234, iseed=42, t=1000.0)
GRIDS = [(1, 24, 28), (1, 45, 53), (1, 68, 80), (1, 135, 159), (1, 8, 10), (1, 2, 6), (3, 30, 40), (1, 1, 1),
         (1, 5, 97), (31, 20, 20), (1, 90, 160)]
SPLITS = [(4, 3, 3), (1, 1, 1), (2, 2, 5)]


def sample_index(n: int, k: int = 16384, seed: int = 99) -> np.ndarray:
    """A fixed subset of flat indices used to store large outputs compactly."""
    rs = np.random.RandomState(seed)
    return np.sort(rs.choice(n, size=min(k, n), replace=False))


def stats(a: np.ndarray) -> np.ndarray:
    a = np.asarray(a, np.float64)
    return np.array([a.sum(), (a * a).sum(), np.abs(a).max()])


def compare(a, b):
    """(cosine, max |a-b| / max |b|) in float64."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))
    return cos, float(np.abs(a - b).max() / (np.abs(b).max() + 1e-300))


# Full 32-layer forwards at BASELINE's grids (reference CPU forward_latent,
# run layer by layer so every layer boundary is stored).  Weights: synthetic
# m5 seed 1234; inputs: seed 42; t = 1000; windows (4,3,3).
#   cfg2  720p  (45x53 tokens, windows 9/9)    all 32 layers, fp32 bar per layer
#   cfg3  1080p (68x80 tokens, windows 16/25)  all 32 layers, bf16 vs fp32 sr
#   cfg5  2160p (135x159 tokens, windows 64/64, ragged edge windows) layers [0,2)
DIT_FULL = {
    "cfg2": dict(T=1, H=45, W=53, l1=32, full_sr=True),
    "cfg3": dict(T=1, H=68, W=80, l1=32, full_sr=True),
    "cfg5": dict(T=1, H=135, W=159, l1=2, full_sr=False),
}
DIT_FULL_SEEDS = dict(wseed=1234, iseed=42, t=1000.0, TXT=58)
N_VID_SAMPLES, N_TXT_SAMPLES, N_SR_SAMPLES = 8192, 2048, 65536


def full_golden_path(name: str) -> str:
    import os
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), f"dit_{name}.npz")
