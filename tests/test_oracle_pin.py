"""Pin the oracle: the C restatement (oracle/oracle.c) and the product's
host geometry against the reference's own outputs (tests/golden/, produced
by tests/golden/make_golden.py from the reference sources compiled unchanged)
and, where the reference library is present, against it live."""
import hashlib
import json
import os

import numpy as np
import pytest

import cases
import s2b

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_geometry_golden_port_and_product(port):
    geo = json.load(open(os.path.join(GOLD, "geometry.json")))
    assert len(geo) == len(cases.GRIDS) * len(cases.SPLITS) * 2
    for g in geo:
        t, h, w = g["grid"]
        sl, vf, tf = port.make_win(t, h, w, tuple(g["split"]), 58, g["shifted"])
        assert sl.tolist() == g["slices"], g["grid"]
        assert sha(vf) == g["vf_sha"] and sha(tf) == g["tf_sha"], g["grid"]
        win = s2b.make_win(t, h, w, tuple(g["split"]), 58, bool(g["shifted"]))
        assert win.slices.tolist() == g["slices"], g["grid"]
        assert sha(win.vid_freq) == g["vf_sha"] and sha(win.txt_freq) == g["tf_sha"], g["grid"]


def test_geometry_windows_tile_grid():
    # every DiT geometry is a partition of the token grid (both parities)
    for (t, h, w) in cases.GRIDS:
        for shf in (False, True):
            win = s2b.make_win(t, h, w, (4, 3, 3), 58, shf)
            cover = np.zeros((t, h, w), np.int32)
            for s in win.slices:
                cover[s[0]:s[1], s[2]:s[3], s[4]:s[5]] += 1
            assert (cover == 1).all(), (t, h, w, shf)


def test_awa_unit_case_port_vs_reference_golden(port):
    c = cases.awa_unit_case()
    g = np.load(os.path.join(GOLD, "awa_unit.npz"))
    vo, to = port.awa(c["vqkv"], c["tqkv"], c["t"], c["h"], c["w"], c["txt_len"], c["slices"], c["vf"], c["tf"],
                      c["nqv"], c["nkv"], c["nqt"], c["nkt"], 1e-5)
    for a, b in ((vo, g["vid_out"]), (to, g["txt_out"])):
        cos, rel = cases.compare(a, b)
        assert cos > 1 - 1e-9 and rel < 1e-6, (cos, rel)


def test_awa_unit_case_inputs_match_reference_generator(ref):
    # The golden outputs can only be reproduced if cases.awa_unit_case
    # regenerates the reference's mt19937 inputs exactly.
    c = cases.awa_unit_case()
    vo, to = ref.cpu_awa(c["vqkv"], c["tqkv"], c["t"], c["h"], c["w"], c["txt_len"], c["slices"], c["vf"], c["tf"],
                         c["nqv"], c["nkv"], c["nqt"], c["nkt"])
    g = np.load(os.path.join(GOLD, "awa_unit.npz"))
    assert np.array_equal(vo, g["vid_out"]) and np.array_equal(to, g["txt_out"])


def test_awa_cfg1_port_vs_reference_golden(port):
    Lv, TXT = 24 * 28, 58
    vqkv, tqkv, nq = cases.awa_cfg_inputs(Lv, TXT)
    sl, vf, tf = port.make_win(1, 24, 28, (4, 3, 3), TXT, False)
    vo, to = port.awa(vqkv, tqkv, 1, 24, 28, TXT, sl, vf, tf, *nq, 1e-5)
    g = np.load(os.path.join(GOLD, "awa_cfg1_ref.npz"))
    for a, idx, val, st in ((vo, g["vid_idx"], g["vid_val"], g["vid_stats"]), (to, g["txt_idx"], g["txt_val"], g["txt_stats"])):
        cos, rel = cases.compare(a.ravel()[idx], val)
        assert cos > 1 - 1e-9 and rel < 1e-5, (cos, rel)
        np.testing.assert_allclose(cases.stats(a), st, rtol=1e-5)


def test_dit_small_port_vs_reference_golden(port, m5_small):
    D = cases.DIT_SMALL
    T, H, W, TXT = D["T"], D["H"], D["W"], D["TXT"]
    grid = s2b.synth_vid_grid(T, 2 * H, 2 * W, D["iseed"])
    vp = s2b.patchify_grid(grid)
    txt = s2b.synth_txt(TXT, D["iseed"])
    gns = (T, H, W, TXT) + port.make_win(T, H, W, (4, 3, 3), TXT, False)
    gsh = (T, H, W, TXT) + port.make_win(T, H, W, (4, 3, 3), TXT, True)
    g = np.load(os.path.join(GOLD, "dit_small.npz"))
    port.load(m5_small, 0, 2)
    _, _, sr = port.forward_latent(gns, gsh, vp, txt, D["t"], 0, 2, True, True)
    cos, rel = cases.compare(sr, g["sr01"])
    assert cos > 1 - 1e-9 and rel < 1e-5, (cos, rel)
    vl, tl, _ = port.forward_latent(gns, gsh, vp, txt, D["t"], 0, 2, True, False)
    for a, idx, val in ((vl, g["vl_idx"], g["vl_val"]), (tl, g["tl_idx"], g["tl_val"])):
        cos, rel = cases.compare(a.ravel()[idx], val)
        assert cos > 1 - 1e-9 and rel < 1e-5, (cos, rel)
    port.load(m5_small, 30, 32)
    _, _, sr2 = port.forward_latent(gns, gsh, vl, tl, D["t"], 30, 32, False, True)
    cos, rel = cases.compare(sr2, g["sr3031"])
    assert cos > 1 - 1e-9 and rel < 1e-4, (cos, rel)


def test_patchify_roundtrip_matches_port():
    from oracle import pyoracle as po
    import ctypes
    P = po.Port()
    grid = s2b.synth_vid_grid(1, 6, 10, 5)
    ours = s2b.patchify_grid(grid)
    theirs = np.zeros_like(ours)
    F = ctypes.POINTER(ctypes.c_float)
    P.L.or_patchify.argtypes = [F, ctypes.c_int, ctypes.c_int, ctypes.c_int, F]
    P.L.or_patchify(grid.ctypes.data_as(F), 1, 6, 10, theirs.ctypes.data_as(F))
    assert np.array_equal(ours, theirs)
    lat = s2b.synth_normal((15, 64), 3, "lat")
    back = s2b.unpatchify_latent(lat, 1, 6, 10)
    theirs = np.zeros_like(back)
    P.L.or_unpatchify.argtypes = [F, ctypes.c_int, ctypes.c_int, ctypes.c_int, F]
    P.L.or_unpatchify(lat.ctypes.data_as(F), 1, 6, 10, theirs.ctypes.data_as(F))
    assert np.array_equal(back, theirs)


def test_full_forward_goldens_are_consistent():
    """dit_cfg{2,3,5}.npz (reference forward_latent at the BASELINE grids): one
    sample row per layer boundary, finite, within the stored absolute maxima."""
    for name in cases.DIT_FULL:
        path = cases.full_golden_path(name)
        if not os.path.exists(path):
            pytest.fail(f"{path} missing: python tests/golden/make_golden.py full {name}")
        g = np.load(path)
        assert g["vid_val"].shape == (cases.DIT_FULL[name]["l1"] + 1, cases.N_VID_SAMPLES)
        assert g["txt_val"].shape == (cases.DIT_FULL[name]["l1"] + 1, cases.N_TXT_SAMPLES)
        assert np.isfinite(g["vid_val"]).all() and np.isfinite(g["txt_val"]).all()
        assert np.all(np.abs(g["vid_val"]).max(1) <= g["vid_stats"][:, 2])
        assert np.all(np.abs(g["txt_val"]).max(1) <= g["txt_stats"][:, 2])


def test_port_pinned_to_cfg2_layer0_golden(port, tmp_path):
    """The C restatement's input projections and layer 0 at 720p (45x53
    tokens, 9 windows) against the reference's golden samples."""
    S = cases.DIT_FULL_SEEDS
    D = cases.DIT_FULL["cfg2"]
    T, H, W, TXT = D["T"], D["H"], D["W"], S["TXT"]
    g = np.load(cases.full_golden_path("cfg2"))
    s2b.synth_write_m5(str(tmp_path), S["wseed"], 0, 1)
    vp = s2b.patchify_grid(s2b.synth_vid_grid(T, 2 * H, 2 * W, S["iseed"]))
    txt = s2b.synth_txt(TXT, S["iseed"])
    gns = (T, H, W, TXT) + port.make_win(T, H, W, (4, 3, 3), TXT, False)
    gsh = (T, H, W, TXT) + port.make_win(T, H, W, (4, 3, 3), TXT, True)
    port.load(str(tmp_path), 0, 1)
    vl, tl, _ = port.forward_latent(gns, gsh, vp, txt, S["t"], 0, 0, True, False)
    for layer in (0, 1):
        for a, b in ((vl.ravel()[g["vid_idx"]], g["vid_val"][layer]), (tl.ravel()[g["txt_idx"]], g["txt_val"][layer])):
            cos, rel = cases.compare(a, b)
            assert cos > 1 - 1e-9 and rel < 1e-5, (layer, cos, rel)
        if layer == 0:
            vl, tl, _ = port.forward_latent(gns, gsh, vl, tl, S["t"], 0, 1, False, False)
    port.close()


def test_oracle_synth_matches_product_generator(port, tmp_path):
    """The oracle's restated generator (used by bench.py's reference arm so
    that it never loads the product library) writes the same model files and
    inputs as the product's, bit for bit."""
    for shape, seed, stream, mean, std in (((1001,), 5, "x", 0.0, 1.0), ((7, 33), 42, "vid_noise", 1.0, 0.02)):
        np.testing.assert_array_equal(port.synth_normal(shape, seed, stream, mean, std),
                                      s2b.synth_normal(shape, seed, stream, mean, std))
    np.testing.assert_array_equal(port.synth_vid_grid(1, 6, 8, 42), s2b.synth_vid_grid(1, 6, 8, 42))
    np.testing.assert_array_equal(port.synth_txt(5, 42), s2b.synth_txt(5, 42))
    g = s2b.synth_vid_grid(2, 6, 8, 3)
    np.testing.assert_array_equal(port.patchify_grid(g), s2b.patchify_grid(g))
    a, b = tmp_path / "oracle", tmp_path / "product"
    port.synth_write_m5(str(a), 1234, 9, 11)      # layer 9 (vid/txt weights) and 10 (shared)
    s2b.synth_write_m5(str(b), 1234, 9, 11)
    names = sorted(os.listdir(b))
    assert sorted(os.listdir(a)) == names and len(names) > 300
    for n in names:
        assert (a / n).read_bytes() == (b / n).read_bytes(), n
