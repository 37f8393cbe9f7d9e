// ref_capi.cpp -- extern "C" handles onto the reference's own CPU code so
// Python tests can drive it through ctypes.  TEST INFRASTRUCTURE ONLY: this
// file is compiled together with the UNCHANGED reference sources
// src/dit_vk.cpp and src/awa_window.cpp into oracle/_ref/libref_dit.so.
//   ref_win_*   -> awa::make_win            (src/awa_window.cpp:161-178)
//   ref_dit_*   -> DitVk::init(use_cpu=true) (src/dit_vk.cpp:140-202),
//                  DitVk::set_windows        (src/dit_vk.h:58),
//                  DitVk::forward_latent     (src/dit_vk.cpp:486-699),
#include "dit_vk.h"
#include "awa_window.h"
#include <cstring>

extern "C" {

void* ref_win_new(int t, int h, int w, int n0, int n1, int n2, int txt_len, int shifted) {
    const int nw[3] = {n0, n1, n2};
    return new Win(awa::make_win(t, h, w, nw, txt_len, shifted != 0));
}
// Build a Win from explicit slices + freqs (the form test_awa_unit.cpp:79-84 uses).
void* ref_win_from(int t, int h, int w, int nwin, int txt_len, const int* sl6,
                   const float* vf, long nvf, const float* tf, long ntf) {
    Win* x = new Win; x->t = t; x->h = h; x->w = w; x->nwin = nwin; x->txt_len = txt_len;
    for (int i = 0; i < nwin; i++) {
        x->st.push_back(sl6[6*i+0]); x->en.push_back(sl6[6*i+1]);
        x->sh.push_back(sl6[6*i+2]); x->eh.push_back(sl6[6*i+3]);
        x->sw.push_back(sl6[6*i+4]); x->ew.push_back(sl6[6*i+5]);
    }
    x->vid_freq.assign(vf, vf + nvf); x->txt_freq.assign(tf, tf + ntf);
    return x;
}
int  ref_win_nwin(void* p) { return ((Win*)p)->nwin; }
long ref_win_nvf(void* p) { return (long)((Win*)p)->vid_freq.size(); }
long ref_win_ntf(void* p) { return (long)((Win*)p)->txt_freq.size(); }
void ref_win_get(void* p, int* sl6, float* vf, float* tf) {
    Win* x = (Win*)p;
    for (int i = 0; i < x->nwin; i++) {
        sl6[6*i+0] = x->st[i]; sl6[6*i+1] = x->en[i]; sl6[6*i+2] = x->sh[i];
        sl6[6*i+3] = x->eh[i]; sl6[6*i+4] = x->sw[i]; sl6[6*i+5] = x->ew[i];
    }
    if (vf) std::memcpy(vf, x->vid_freq.data(), x->vid_freq.size() * 4);
    if (tf) std::memcpy(tf, x->txt_freq.data(), x->txt_freq.size() * 4);
}
void ref_win_free(void* p) { delete (Win*)p; }

void* ref_dit_new(const char* model_dir) {
    DitVk* d = new DitVk;
    if (!d->init(model_dir, false, 0, /*use_cpu=*/true)) { delete d; return nullptr; }
    return d;
}
void ref_dit_set_windows(void* d, void* ns, void* sh) { ((DitVk*)d)->set_windows(*(Win*)ns, *(Win*)sh); }
int ref_dit_forward_latent(void* d, const float* vid, int Lv, int vid_cols, const float* txt, int TXT,
                           int txt_cols, float t, int l0, int l1, int do_init, int do_final,
                           float* vid_lat, float* txt_lat, float* sr) {
    std::vector<float> v(vid, vid + (size_t)Lv * vid_cols), tx(txt, txt + (size_t)TXT * txt_cols);
    std::vector<float> vo, to, so;
    if (!((DitVk*)d)->forward_latent(v, Lv, tx, TXT, t, l0, l1, do_init != 0, do_final != 0, vo, to, so))
        return -1;
    if (vid_lat && !vo.empty()) std::memcpy(vid_lat, vo.data(), vo.size() * 4);
    if (txt_lat && !to.empty()) std::memcpy(txt_lat, to.data(), to.size() * 4);
    if (sr && !so.empty()) std::memcpy(sr, so.data(), so.size() * 4);
    return 0;
}
void ref_dit_free(void* d) { delete (DitVk*)d; }

}  // extern "C"
