// ref_awa_unit.cpp -- exposes the reference's pure-C++ AWA checker
// `cpu_awa` from src/test_awa_unit.cpp:27-70 (qk_norm eps 1e-5, RoPE on 126
// dims, per-window SDPA, txt mean, reverse partition) through a C entry point.
// TEST INFRASTRUCTURE ONLY.  The reference file is compiled unchanged: it is
// #included by path from the reference tree (its `main` renamed so it does
// not clash), and this wrapper, living in the same translation unit, can
// reach its file-static functions.
#define main s2b_ref_test_awa_unit_main
#include "test_awa_unit.cpp"
#undef main

extern "C" int ref_cpu_awa(const float* vqkv, const float* tqkv, void* win,
                           const float* nqv, const float* nkv, const float* nqt, const float* nkt,
                           int Lv, int TXT, float* vid_out, float* txt_out) {
    const Win& w = *(const Win*)win;
    std::vector<float> vq(vqkv, vqkv + (size_t)Lv * QKV), tq(tqkv, tqkv + (size_t)TXT * QKV);
    std::vector<float> a(nqv, nqv + HEAD_D), b(nkv, nkv + HEAD_D), c(nqt, nqt + HEAD_D), d(nkt, nkt + HEAD_D);
    std::vector<float> vo, to;
    cpu_awa(vq, tq, w, a, b, c, d, Lv, TXT, vo, to);
    std::memcpy(vid_out, vo.data(), vo.size() * 4);
    std::memcpy(txt_out, to.data(), to.size() * 4);
    return 0;
}
