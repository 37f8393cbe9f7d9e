// Drives the B200 path through the reference-shaped C++ interface
// (include/seedvr2_b200.hpp) the way the engine drives DitVk
// (src/seedvr2_engine.cpp:215-272): init, make_win + set_windows, then a
// chunked forward_latent over [0, 2) with synthetic inputs.  (The full
// reference call, init(dir, false, precision, false), loads all 32 layers.)  Writes the
// vid / txt latents to argv[2] as raw fp32.
#include "seedvr2_b200.hpp"

#include <cstdio>
#include <vector>

int main(int argc, char** argv) {
    if (argc < 3) {
        std::fprintf(stderr, "usage: %s <m5 dir> <out file>\n", argv[0]);
        return 2;
    }
    using seedvr2_b200::DitB200;
    const int T = 1, H = 24, W = 28, TXT = 58;
    const int Lv = T * H * W;
    const int split[3] = {4, 3, 3};
    DitB200 dit(0);
    // the test model directory holds layers 0..1 (and 30..31) only
    if (!dit.init(argv[1], S2B_PREC_BF16, 0, 2)) return 1;
    dit.set_windows(seedvr2_b200::make_win(T, H, W, split, TXT, false), seedvr2_b200::make_win(T, H, W, split, TXT, true));
    std::vector<float> grid((size_t)T * 2 * H * 2 * W * 33), txt((size_t)TXT * 5120);
    s2b_synth_vid_grid(grid.data(), T, 2 * H, 2 * W, 42);
    s2b_synth_txt(txt.data(), TXT, 42);
    const std::vector<float> patch = DitB200::patchify_grid(grid, T, 2 * H, 2 * W);
    std::vector<float> vl, tl, sr;
    if (!dit.forward_latent(patch, Lv, txt, TXT, 1000.f, 0, 2, true, false, vl, tl, sr)) return 1;
    std::FILE* f = std::fopen(argv[2], "wb");
    if (!f) return 1;
    std::fwrite(vl.data(), sizeof(float), vl.size(), f);
    std::fwrite(tl.data(), sizeof(float), tl.size(), f);
    std::fclose(f);
    return 0;
}
