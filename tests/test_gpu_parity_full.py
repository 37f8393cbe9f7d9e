"""The whole 32-layer forward against the reference at BASELINE's grids.

Goldens (tests/golden/dit_cfg{2,3,5}.npz, made by make_golden.py `full` from
the reference's own CPU DitVk::forward_latent, src/dit_vk.cpp:486-699, run one
layer per call) hold, per layer boundary, a fixed sample of the vid / txt
residual latents and their stats, and the final sr.

Bars (north star): fp32 path cos >= 0.99999 and max|d|/max|ref| <= 1e-4 per
layer; bf16 path cos >= 0.9999 against the reference fp32.  "max rel err" is
max|d| / max|ref| over the compared values (a normalised absolute error).

Two measured limits, asserted as such:
  * 32 layers chained in fp32 drift to max rel err ~1.5e-4 (cos 0.99999999):
    each layer meets the 1e-4 bar on the reference's own input, but the
    tensor-core fp32 accumulation of the 3xTF32 GEMMs carries 2.4-4x the
    rounding error of a CPU fp32 GEMM per Linear (test_gpu_gemm.py), and 32
    layers compound it; chained checks use 2e-4.
  * bf16 operands cannot reach cos 0.9999 after 32 layers: the oracle port
    with only its GEMM / attention operands rounded to bf16 (sr_port_bf16,
    make_golden.py emul) lands at cos 0.9996 against the reference.  The bf16
    path is held to within 1e-4 of that floor.  fp16 operands (the
    reference's precision 1, same tcgen05 kernels) keep 3 more mantissa bits:
    their floor (sr_port_fp16) is cos 0.999997, and the fp16 path meets the
    0.9999 bar outright."""
import os
import tempfile

import numpy as np
import pytest

import cases
import s2b

pytestmark = pytest.mark.gpu
S = cases.DIT_FULL_SEEDS
TXT, TS = S["TXT"], S["t"]


CHAINED_REL = 2e-4          # fp32, 32 layers chained (see the module docstring)
BF16_FLOOR_MARGIN = 1e-4    # bf16: cos within this of the bf16-operand floor


def bf16_floor(g):
    """cos of the oracle port with bf16 operands against the reference."""
    if "sr_port_bf16" not in g.files:
        pytest.fail("golden lacks sr_port_bf16: python tests/golden/make_golden.py emul")
    return cases.compare(g["sr_port_bf16"], g["sr"])[0]


def gold(name):
    return np.load(cases.full_golden_path(name))


def geom(name):
    D = cases.DIT_FULL[name]
    return D["T"], D["H"], D["W"]


def inputs(name):
    T, H, W = geom(name)
    vp = s2b.patchify_grid(s2b.synth_vid_grid(T, 2 * H, 2 * W, S["iseed"]))
    return vp, s2b.synth_txt(TXT, S["iseed"])


def ctx_for(name, prec, lo=0, hi=32):
    T, H, W = geom(name)
    c = s2b.DitB200(0, prec)
    c.init_synth(S["wseed"], lo, hi)
    c.set_windows(s2b.make_win(T, H, W, (4, 3, 3), TXT, False), s2b.make_win(T, H, W, (4, 3, 3), TXT, True))
    return c


def bar_fp32(a, b, what):
    cos, rel = cases.compare(a, b)
    assert cos >= 0.99999 and rel <= 1e-4, (what, cos, rel)
    return cos, rel


def test_cfg2_fp32_chained_every_layer_and_sr():
    """720p fp32: the GPU's own 32-layer chain, checked at every layer
    boundary against the reference's sampled latents, and the final sr."""
    g = gold("cfg2")
    vp, txt = inputs("cfg2")
    T, H, W = geom("cfg2")
    Lv = T * H * W
    c = ctx_for("cfg2", s2b.PREC_FP32)
    try:
        vl, tl, _ = c.forward_latent(vp, Lv, txt, TXT, TS, 0, 0, True, False)
        rows = []
        for layer in range(33):
            cv = cases.compare(vl.ravel()[g["vid_idx"]], g["vid_val"][layer])
            ct = cases.compare(tl.ravel()[g["txt_idx"]], g["txt_val"][layer])
            rows.append((layer,) + cv + ct)
            if layer < 32:
                vl, tl, _ = c.forward_latent(vl, Lv, tl, TXT, TS, layer, layer + 1, False, False)
        _, _, sr = c.forward_latent(vl, Lv, tl, TXT, TS, 32, 32, False, True)
        sr_graph = c.forward(vp, Lv, txt, TXT, TS)
    finally:
        c.close()
    for r in rows:
        print("after %2d layers: vid cos %.9f rel %.2e | txt cos %.9f rel %.2e" % r)
    print("sr:", cases.compare(sr, g["sr"]), "sr (graph):", cases.compare(sr_graph, g["sr"]))
    for r in rows:
        assert r[1] >= 0.99999 and r[2] <= CHAINED_REL and r[3] >= 0.99999 and r[4] <= CHAINED_REL, r
    for what, a in (("sr", sr), ("sr (graph)", sr_graph)):
        cos, rel = cases.compare(a, g["sr"])
        assert cos >= 0.99999 and rel <= CHAINED_REL, (what, cos, rel)


def test_cfg2_fp32_each_layer_fed_reference_input(ref):
    """720p fp32: every layer run on the REFERENCE's own input for that layer
    (the reference's CPU forward_latent, run here one layer at a time), its
    output compared with the reference's output of the same layer.  The
    reference run itself is checked against the committed golden samples."""
    g = gold("cfg2")
    vp, txt = inputs("cfg2")
    T, H, W = geom("cfg2")
    Lv = T * H * W
    gns = (T, H, W, TXT) + ref.make_win(T, H, W, (4, 3, 3), TXT, 0)
    gsh = (T, H, W, TXT) + ref.make_win(T, H, W, (4, 3, 3), TXT, 1)
    c = ctx_for("cfg2", s2b.PREC_FP32)
    worst = (1.0, 0.0)
    try:
        with tempfile.TemporaryDirectory() as md:
            s2b.synth_write_m5(md, S["wseed"], 0, 32)
            ref.load(md)
            rv, rt, _ = ref.forward_latent(gns, gsh, vp, txt, TS, 0, 0, True, False)
            for layer in range(32):
                np.testing.assert_allclose(rv.ravel()[g["vid_idx"]], g["vid_val"][layer], rtol=1e-5, atol=1e-5)
                gv, gt, _ = c.forward_latent(rv, Lv, rt, TXT, TS, layer, layer + 1, False, False)
                rv, rt, _ = ref.forward_latent(gns, gsh, rv, rt, TS, layer, layer + 1, False, False)
                cv = bar_fp32(gv, rv, f"layer {layer} vid")
                ct = bar_fp32(gt, rt, f"layer {layer} txt")
                worst = (min(worst[0], cv[0], ct[0]), max(worst[1], cv[1], ct[1]))
            ref.close()
        print(f"cfg2 fp32 per layer: worst cos {worst[0]:.8f} worst rel {worst[1]:.2e}")
    finally:
        c.close()


@pytest.mark.parametrize("prec", [s2b.PREC_BF16, s2b.PREC_FP16, s2b.PREC_FP32], ids=["bf16", "fp16", "fp32"])
def test_cfg3_1080p_full_forward_vs_reference_fp32(prec):
    """1080p: the captured 32-layer forward (the path bench.py times) against
    the reference fp32 sr; fp16 at cos >= 0.9999, bf16 at its operand floor,
    fp32 at the fp32 bar."""
    g = gold("cfg3")
    vp, txt = inputs("cfg3")
    T, H, W = geom("cfg3")
    c = ctx_for("cfg3", prec)
    try:
        sr = c.forward(vp, T * H * W, txt, TXT, TS)
    finally:
        c.close()
    cos, rel = cases.compare(sr, g["sr"])
    print(f"cfg3 prec={prec}: cos {cos:.8f} rel {rel:.2e}")
    if prec == s2b.PREC_FP32:
        assert cos >= 0.99999 and rel <= CHAINED_REL, (cos, rel)
    elif prec == s2b.PREC_FP16:
        print(f"cfg3 fp16-operand floor: cos {cases.compare(g['sr_port_fp16'], g['sr'])[0]:.8f}")
        assert cos >= 0.9999, (cos, rel)
    else:
        floor = bf16_floor(g)
        print(f"cfg3 bf16-operand floor: cos {floor:.8f}")
        assert cos >= min(0.9999, floor - BF16_FLOOR_MARGIN), (cos, rel, floor)


@pytest.mark.parametrize("prec", [s2b.PREC_FP32, s2b.PREC_BF16, s2b.PREC_FP16], ids=["fp32", "bf16", "fp16"])
def test_cfg5_2160p_layer_pair_vs_reference(prec):
    """2160p (135x159 tokens, 64/64 windows with ragged edge windows): input
    projections, layers 0 and 1 and the final projection."""
    g = gold("cfg5")
    vp, txt = inputs("cfg5")
    T, H, W = geom("cfg5")
    Lv = T * H * W
    c = ctx_for("cfg5", prec, 0, 2)
    try:
        vl, tl, _ = c.forward_latent(vp, Lv, txt, TXT, TS, 0, 2, True, False)
        _, _, sr = c.forward_latent(vl, Lv, tl, TXT, TS, 2, 2, False, True)
    finally:
        c.close()
    pairs = [(vl.ravel()[g["vid_idx"]], g["vid_val"][2], "vid after 2 layers"),
             (tl.ravel()[g["txt_idx"]], g["txt_val"][2], "txt after 2 layers"),
             (sr.ravel()[g["sr_idx"]], g["sr_val"], "sr")]
    for a, b, what in pairs:
        cos, rel = cases.compare(a, b)
        if prec == s2b.PREC_FP32:
            assert cos >= 0.99999 and rel <= 1e-4, (what, cos, rel)
        else:
            assert cos >= 0.9999, (what, cos, rel)


def test_cfg2_fp16_full_forward_meets_the_bar():
    """720p, fp16 operands: the captured 32-layer forward and the layer-wise
    forward_latent chain both reach cos >= 0.9999 against the reference fp32
    sr, at every sampled layer boundary too."""
    g = gold("cfg2")
    vp, txt = inputs("cfg2")
    T, H, W = geom("cfg2")
    Lv = T * H * W
    c = ctx_for("cfg2", s2b.PREC_FP16)
    try:
        sr_graph = c.forward(vp, Lv, txt, TXT, TS)
        vl, tl, _ = c.forward_latent(vp, Lv, txt, TXT, TS, 0, 0, True, False)
        worst = 1.0
        for layer in range(32):
            vl, tl, _ = c.forward_latent(vl, Lv, tl, TXT, TS, layer, layer + 1, False, False)
            cv = cases.compare(vl.ravel()[g["vid_idx"]], g["vid_val"][layer + 1])
            ct = cases.compare(tl.ravel()[g["txt_idx"]], g["txt_val"][layer + 1])
            worst = min(worst, cv[0], ct[0])
            assert cv[0] >= 0.9999 and ct[0] >= 0.9999, (layer, cv, ct)
        _, _, sr = c.forward_latent(vl, Lv, tl, TXT, TS, 32, 32, False, True)
    finally:
        c.close()
    floor = cases.compare(g["sr_port_fp16"], g["sr"])[0]
    print(f"cfg2 fp16: graph {cases.compare(sr_graph, g['sr'])} chain {cases.compare(sr, g['sr'])} "
          f"worst layer cos {worst:.8f} floor {floor:.8f}")
    for what, a in (("sr", sr), ("sr (graph)", sr_graph)):
        cos, rel = cases.compare(a, g["sr"])
        assert cos >= 0.9999, (what, cos, rel)


def test_cfg2_bf16_folded_norms_vs_standalone_norms():
    """bf16, 720p, all 32 layers: the RMSNorm + adaLN modulate folded into the
    neighbouring GEMMs (S2B_NORM_FUSE=1: operand written by the gate/residual
    epilogue, row factor and shift applied by the next GEMM) is as close to
    the reference fp32 output as the standalone norm kernels (the default)."""
    g = gold("cfg2")
    vp, txt = inputs("cfg2")
    T, H, W = geom("cfg2")
    res = {}
    for fuse in ("1", "0"):
        os.environ["S2B_NORM_FUSE"] = fuse
        try:
            c = ctx_for("cfg2", s2b.PREC_BF16)
            try:
                res[fuse] = cases.compare(c.forward(vp, T * H * W, txt, TXT, TS), g["sr"])
            finally:
                c.close()
        finally:
            os.environ.pop("S2B_NORM_FUSE", None)
    print("folded", res["1"], "standalone", res["0"])
    assert res["1"][0] >= res["0"][0] - 5e-5, res
    assert res["1"][0] >= min(0.9999, bf16_floor(g) - BF16_FLOOR_MARGIN), res
