// awa_geometry.h -- Adaptive Window Attention window slices and 3-axis
// RoPE angle tables (host side, built once per resolution).
//
// Mirrors the reference's `Win` (src/dit_vk.h:17-22) and `awa::make_win`
// (src/awa_window.cpp:161-178): windows are resolution-mapped onto a 45x80
// proxy split {nt,nh,nw} ways, shifted windows are offset by half a window.
#pragma once
#include <vector>
#include <cstdint>

namespace s2b {

struct Window { int t0, t1, h0, h1, w0, w1; int size() const { return (t1 - t0) * (h1 - h0) * (w1 - w0); } };

struct WinGeom {
    int t = 0, h = 0, w = 0, txt_len = 0;
    std::vector<Window> win;          // nwin windows
    std::vector<float> vid_freq;      // sum(f_i) x 126 angles, window-packed token order
    std::vector<float> txt_freq;      // nwin x txt_len x 126 angles
    int nwin() const { return (int)win.size(); }
    int tokens() const { return t * h * w; }
};

// Window slices of a (t,h,w) token grid (src/awa_window.cpp:43-106).
std::vector<Window> make_windows(int t, int h, int w, const int num_windows[3], bool shifted);
// Angle tables for a window list (src/awa_window.cpp:109-159).
void build_freqs(const std::vector<Window>& win, int txt_len, std::vector<float>& vid_freq,
                 std::vector<float>& txt_freq);
WinGeom make_win(int t, int h, int w, const int num_windows[3], int txt_len, bool shifted);

// Device-side window tables derived from a WinGeom: the token index of every
// window-packed vid row (a permutation of [0, Lv) when the windows tile the
// grid), the window start offsets and the packed row offsets including the
// txt rows each window appends.
struct WinTables {
    std::vector<int> vidx;        // sumf: grid token of packed vid row
    std::vector<int> cumf;        // nwin+1: start of window i among packed vid rows
    std::vector<int> cums;        // nwin+1: start of window i among packed [vid | txt] rows
    int sumf = 0, maxS = 0;
    bool covers_all = false;      // every grid token appears exactly once
};
bool build_tables(const WinGeom& g, WinTables& out, const char** why);

}  // namespace s2b
