"""Regenerate the golden fixtures in tests/golden/ from the REFERENCE itself.

Runs the reference's own CPU code, compiled unchanged into
oracle/_ref/libref_dit.so (build it with `make -C oracle ref`), on the seeded
cases of cases.py and stores its outputs:
  geometry.json     awa::make_win slices + SHA-256 of the float angle tables
  awa_unit.npz      cpu_awa (src/test_awa_unit.cpp:27-70) on its own unit case
  awa_cfg1_ref.npz  cpu_awa on the 24x28 / TXT=58 case (reference eps 1e-5),
                    sampled outputs + stats
  dit_small.npz     DitVk::forward_latent (CPU mode) on the 24x28 grid with
                    synthetic weights: layers [0,2) init+final (sr), layers
                    [0,2) latents (sampled), layers [30,32) final from the
                    [0,2) latent (sr)
Usage: python tests/golden/make_golden.py   (takes a few minutes)
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "seedvr2-2b-ncnn_b200"))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import cases  # noqa: E402
import s2b  # noqa: E402
from oracle import pyoracle as po  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    R = po.Ref()
    geo = []
    for (t, h, w) in cases.GRIDS:
        for nw in cases.SPLITS:
            for shf in (0, 1):
                sl, vf, tf = R.make_win(t, h, w, nw, 58, shf)
                geo.append(dict(grid=[t, h, w], split=list(nw), shifted=shf, slices=sl.tolist(),
                                vf_sha=sha(vf), tf_sha=sha(tf), nvf=int(vf.size), ntf=int(tf.size)))
    json.dump(geo, open(os.path.join(HERE, "geometry.json"), "w"))

    c = cases.awa_unit_case()
    vo, to = R.cpu_awa(c["vqkv"], c["tqkv"], c["t"], c["h"], c["w"], c["txt_len"], c["slices"], c["vf"], c["tf"],
                       c["nqv"], c["nkv"], c["nqt"], c["nkt"])
    np.savez_compressed(os.path.join(HERE, "awa_unit.npz"), vid_out=vo, txt_out=to)

    Lv, TXT = 24 * 28, 58
    vqkv, tqkv, nq = cases.awa_cfg_inputs(Lv, TXT)
    sl, vf, tf = R.make_win(1, 24, 28, (4, 3, 3), TXT, 0)
    vo, to = R.cpu_awa(vqkv, tqkv, 1, 24, 28, TXT, sl, vf, tf, *nq)
    iv, it = cases.sample_index(vo.size), cases.sample_index(to.size)
    np.savez_compressed(os.path.join(HERE, "awa_cfg1_ref.npz"), vid_idx=iv, vid_val=vo.ravel()[iv], txt_idx=it,
                        txt_val=to.ravel()[it], vid_stats=cases.stats(vo), txt_stats=cases.stats(to))

    D = cases.DIT_SMALL
    T, H, W = D["T"], D["H"], D["W"]
    with tempfile.TemporaryDirectory() as md:
        s2b.synth_write_m5(md, D["wseed"], 0, 2)
        s2b.synth_write_m5(md, D["wseed"], 30, 32)
        grid = s2b.synth_vid_grid(T, 2 * H, 2 * W, D["iseed"])
        vp = s2b.patchify_grid(grid)
        txt = s2b.synth_txt(D["TXT"], D["iseed"])
        gns = (T, H, W, D["TXT"]) + R.make_win(T, H, W, (4, 3, 3), D["TXT"], 0)
        gsh = (T, H, W, D["TXT"]) + R.make_win(T, H, W, (4, 3, 3), D["TXT"], 1)
        R.load(md)
        _, _, sr01 = R.forward_latent(gns, gsh, vp, txt, D["t"], 0, 2, 1, 1)
        vl, tl, _ = R.forward_latent(gns, gsh, vp, txt, D["t"], 0, 2, 1, 0)
        _, _, sr3031 = R.forward_latent(gns, gsh, vl, tl, D["t"], 30, 32, 0, 1)
        R.close()
    iv, it = cases.sample_index(vl.size), cases.sample_index(tl.size)
    np.savez_compressed(os.path.join(HERE, "dit_small.npz"), sr01=sr01, sr3031=sr3031, vl_idx=iv,
                        vl_val=vl.ravel()[iv], tl_idx=it, tl_val=tl.ravel()[it], vl_stats=cases.stats(vl),
                        tl_stats=cases.stats(tl))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
