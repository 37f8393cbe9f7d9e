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
  dit_cfg2.npz / dit_cfg3.npz / dit_cfg5.npz  (`full` mode)
                    DitVk::forward_latent (CPU mode) over the BASELINE grids
                    (720p, 1080p, 2160p; cases.DIT_FULL) with the seed-1234
                    synthetic m5 weights, run one layer at a time: per layer
                    boundary a fixed sample of the vid / txt latents plus
                    their stats, and the final sr (full, or sampled for
                    2160p).  The sampled indices come from cases.sample_index.
Usage: python tests/golden/make_golden.py          (small fixtures, a few minutes)
       python tests/golden/make_golden.py full [cfg2 cfg3 cfg5]
                                                   (reference CPU forwards of
                                                    the full grids: ~15 min on 8 cores)
       python tests/golden/make_golden.py emul [cfg2 cfg3]
                                                   (the oracle port's own fp32 /
                                                    bf16- / fp16-operand forwards,
                                                    stored as sr_port_*: ~30 min)
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile
import time

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


def full(names):
    """Reference forward_latent over cases.DIT_FULL, one layer per call."""
    S = cases.DIT_FULL_SEEDS
    TXT = S["TXT"]
    R = po.Ref()
    with tempfile.TemporaryDirectory() as md:
        s2b.synth_write_m5(md, S["wseed"], 0, 32)
        R.load(md)
        for name in names:
            D = cases.DIT_FULL[name]
            T, H, W = D["T"], D["H"], D["W"]
            Lv = T * H * W
            gns = (T, H, W, TXT) + R.make_win(T, H, W, (4, 3, 3), TXT, 0)
            gsh = (T, H, W, TXT) + R.make_win(T, H, W, (4, 3, 3), TXT, 1)
            vp = s2b.patchify_grid(s2b.synth_vid_grid(T, 2 * H, 2 * W, S["iseed"]))
            txt = s2b.synth_txt(TXT, S["iseed"])
            iv = cases.sample_index(Lv * 2560, cases.N_VID_SAMPLES)
            it = cases.sample_index(TXT * 2560, cases.N_TXT_SAMPLES)
            vs, ts, vst, tst = [], [], [], []
            vl, tl, _ = R.forward_latent(gns, gsh, vp, txt, S["t"], 0, 0, True, False)
            for layer in range(D["l1"] + 1):
                vs.append(vl.ravel()[iv]); ts.append(tl.ravel()[it])
                vst.append(cases.stats(vl)); tst.append(cases.stats(tl))
                if layer == D["l1"]:
                    break
                t0 = time.time()
                vl, tl, _ = R.forward_latent(gns, gsh, vl, tl, S["t"], layer, layer + 1, False, False)
                print(f"{name} layer {layer} {time.time() - t0:.1f} s", flush=True)
            _, _, sr = R.forward_latent(gns, gsh, vl, tl, S["t"], D["l1"], D["l1"], False, True)
            out = dict(vid_idx=iv, txt_idx=it, vid_val=np.stack(vs), txt_val=np.stack(ts),
                       vid_stats=np.stack(vst), txt_stats=np.stack(tst), sr_stats=cases.stats(sr))
            if D["full_sr"]:
                out["sr"] = sr
            else:
                isr = cases.sample_index(sr.size, cases.N_SR_SAMPLES)
                out.update(sr_idx=isr, sr_val=sr.ravel()[isr])
            np.savez_compressed(cases.full_golden_path(name), **out)
            print("written", cases.full_golden_path(name), flush=True)
        R.close()


def emul(names, modes):
    """The oracle port's own 32-layer forwards of cases.DIT_FULL (fp32, and
    with bf16 / fp16 operand rounding emulated), added to the goldens as
    sr_port_<mode>: the drift two correct fp32 implementations show after 32
    layers, and the error that rounding every operand to bf16 / fp16 costs by
    itself (the floor for any path with those operands)."""
    S = cases.DIT_FULL_SEEDS
    TXT = S["TXT"]
    P = po.Port()
    with tempfile.TemporaryDirectory() as md:
        P.synth_write_m5(md, S["wseed"], 0, 32)
        P.load(md, 0, 32)
        for name in names:
            D = cases.DIT_FULL[name]
            T, H, W = D["T"], D["H"], D["W"]
            gns = (T, H, W, TXT) + P.make_win(T, H, W, (4, 3, 3), TXT, False)
            gsh = (T, H, W, TXT) + P.make_win(T, H, W, (4, 3, 3), TXT, True)
            vp = P.patchify_grid(P.synth_vid_grid(T, 2 * H, 2 * W, S["iseed"]))
            txt = P.synth_txt(TXT, S["iseed"])
            path = cases.full_golden_path(name)
            out = dict(np.load(path))
            ref = out["sr"] if D["full_sr"] else out["sr_val"]
            for mode in modes:
                P.set_operand_rounding({"fp32": 0, "bf16": 1, "fp16": 2}[mode])
                t0 = time.time()
                _, _, sr = P.forward_latent(gns, gsh, vp, txt, S["t"], 0, D["l1"], True, True)
                P.set_operand_rounding(0)
                out[f"sr_port_{mode}"] = sr if D["full_sr"] else sr.ravel()[out["sr_idx"]]
                print(f"{name} {mode}: {time.time() - t0:.0f} s, vs reference",
                      cases.compare(out[f"sr_port_{mode}"], ref), flush=True)
                np.savez_compressed(path, **out)
        P.close()


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "emul":
        emul(sys.argv[2:] or ["cfg2", "cfg3"], ["fp32", "bf16", "fp16"])
    elif len(sys.argv) > 1 and sys.argv[1] == "full":
        full(sys.argv[2:] or list(cases.DIT_FULL))
    else:
        main()
