// awa_geometry.cpp -- window slices + RoPE angle tables (see awa_geometry.h).
//
// The arithmetic must match the reference bit for bit (the window list and
// the float angles feed parity), so the steps are the reference's:
//   scale = sqrt(45*80 / (h*w)); wh = ceil(round(h*scale)/nh);
//   ww = ceil(round(w*scale)/nw); wt = ceil(min(t,30)/nt)
//   (src/awa_window.cpp:49-54), windows enumerated w-outer, h, t-inner
//   (:58-67); shifted windows offset by 0.5 window where a window is
//   smaller than the grid (:83-105); angles base_j = 1/10000^(2j/42) in
//   double, vid axes (txt_len + t, local h, local w), txt axis tiled x3
//   (:121-158), stored as float.
#include "awa_geometry.h"
#include <cmath>
#include <algorithm>

namespace s2b {

namespace {
struct Extent { int wt, wh, ww; };
Extent window_extent(int t, int h, int w, const int nwin[3]) {
    const double scale = std::sqrt((45.0 * 80.0) / ((double)h * w));
    const int rh = (int)std::round(h * scale), rw = (int)std::round(w * scale);
    Extent e;
    e.wh = (rh + nwin[1] - 1) / nwin[1];
    e.ww = (rw + nwin[2] - 1) / nwin[2];
    e.wt = (std::min(t, 30) + nwin[0] - 1) / nwin[0];
    return e;
}
}  // namespace

std::vector<Window> make_windows(int t, int h, int w, const int num_windows[3], bool shifted) {
    std::vector<Window> out;
    if (t <= 0 || h <= 0 || w <= 0) return out;
    const Extent e = window_extent(t, h, w, num_windows);
    if (!shifted) {
        const int nt = (t + e.wt - 1) / e.wt, nh = (h + e.wh - 1) / e.wh, nw = (w + e.ww - 1) / e.ww;
        for (int iw = 0; iw < nw; iw++) {
            const int w0 = iw * e.ww, w1 = std::min((iw + 1) * e.ww, w);
            if (w1 <= w0) continue;
            for (int ih = 0; ih < nh; ih++) {
                const int h0 = ih * e.wh, h1 = std::min((ih + 1) * e.wh, h);
                if (h1 <= h0) continue;
                for (int it = 0; it < nt; it++) {
                    const int t0 = it * e.wt, t1 = std::min((it + 1) * e.wt, t);
                    if (t1 <= t0) continue;
                    out.push_back({t0, t1, h0, h1, w0, w1});
                }
            }
        }
        return out;
    }
    // Shifted: half-window offset along every axis the window does not span.
    const double st = (e.wt < t) ? 0.5 : 0.0, sh = (e.wh < h) ? 0.5 : 0.0, sw = (e.ww < w) ? 0.5 : 0.0;
    const int nt = (st > 0) ? (int)std::ceil((t - st) / e.wt) + 1 : 1;
    const int nh = (sh > 0) ? (int)std::ceil((h - sh) / e.wh) + 1 : 1;
    const int nw = (sw > 0) ? (int)std::ceil((w - sw) / e.ww) + 1 : 1;
    // Bounds are truncated toward zero after the half offset (int cast), then clamped.
    auto lo = [](int i, double s, int sz) { return std::max((int)((i - s) * sz), 0); };
    auto hi = [](int i, double s, int sz, int lim) { return std::min((int)((i - s + 1) * sz), lim); };
    for (int iw = 0; iw < nw; iw++) {
        const int w0 = lo(iw, sw, e.ww), w1 = hi(iw, sw, e.ww, w);
        if (w1 <= w0) continue;
        for (int ih = 0; ih < nh; ih++) {
            const int h0 = lo(ih, sh, e.wh), h1 = hi(ih, sh, e.wh, h);
            if (h1 <= h0) continue;
            for (int it = 0; it < nt; it++) {
                const int t0 = lo(it, st, e.wt), t1 = hi(it, st, e.wt, t);
                if (t1 <= t0) continue;
                out.push_back({t0, t1, h0, h1, w0, w1});
            }
        }
    }
    return out;
}

void build_freqs(const std::vector<Window>& win, int txt_len, std::vector<float>& vid_freq,
                 std::vector<float>& txt_freq) {
    constexpr int AX = 42, ROT = 3 * AX;   // 42 rotated dims per axis, 126 in total
    double base[AX / 2];
    for (int j = 0; j < AX / 2; j++) base[j] = 1.0 / std::pow(10000.0, (double)(2 * j) / AX);
    size_t total = 0;
    for (const auto& w : win) total += (size_t)w.size();
    vid_freq.resize(total * ROT);
    size_t off = 0;
    for (const auto& w : win) {
        const int lt = w.t1 - w.t0, lh = w.h1 - w.h0, lw = w.w1 - w.w0;
        for (int it = 0; it < lt; it++)
            for (int ih = 0; ih < lh; ih++)
                for (int iw = 0; iw < lw; iw++) {
                    const double pos[3] = {(double)(txt_len + it), (double)ih, (double)iw};
                    for (int k = 0; k < ROT; k++) vid_freq[off++] = (float)(pos[k / AX] * base[(k % AX) / 2]);
                }
    }
    txt_freq.resize(win.size() * (size_t)txt_len * ROT);
    off = 0;
    for (size_t i = 0; i < win.size(); i++)
        for (int p = 0; p < txt_len; p++)
            for (int k = 0; k < ROT; k++) txt_freq[off++] = (float)((double)p * base[(k % AX) / 2]);
}

WinGeom make_win(int t, int h, int w, const int num_windows[3], int txt_len, bool shifted) {
    WinGeom g;
    g.t = t; g.h = h; g.w = w; g.txt_len = txt_len;
    g.win = make_windows(t, h, w, num_windows, shifted);
    build_freqs(g.win, txt_len, g.vid_freq, g.txt_freq);
    return g;
}

bool build_tables(const WinGeom& g, WinTables& o, const char** why) {
    const int nwin = g.nwin(), Lv = g.tokens();
    o.vidx.clear(); o.cumf.assign(nwin + 1, 0); o.cums.assign(nwin + 1, 0);
    o.maxS = 0;
    std::vector<unsigned char> seen((size_t)std::max(Lv, 0), 0);
    bool dup = false;
    for (int i = 0; i < nwin; i++) {
        const Window& w = g.win[i];
        if (w.t0 < 0 || w.h0 < 0 || w.w0 < 0 || w.t1 > g.t || w.h1 > g.h || w.w1 > g.w ||
            w.t1 <= w.t0 || w.h1 <= w.h0 || w.w1 <= w.w0) {
            if (why) *why = "window slice outside the token grid or empty";
            return false;
        }
        for (int a = w.t0; a < w.t1; a++)
            for (int b = w.h0; b < w.h1; b++)
                for (int c = w.w0; c < w.w1; c++) {
                    const int tok = (a * g.h + b) * g.w + c;
                    if (seen[tok]) dup = true;
                    seen[tok] = 1;
                    o.vidx.push_back(tok);
                }
        o.cumf[i + 1] = o.cumf[i] + w.size();
        o.cums[i + 1] = o.cums[i] + w.size() + g.txt_len;
        o.maxS = std::max(o.maxS, w.size() + g.txt_len);
    }
    o.sumf = o.cumf[nwin];
    if (dup) { if (why) *why = "a grid token belongs to two windows"; return false; }
    if ((long)g.vid_freq.size() != (long)o.sumf * 126 || (long)g.txt_freq.size() != (long)nwin * g.txt_len * 126) {
        if (why) *why = "freq table sizes do not match the windows";
        return false;
    }
    o.covers_all = (o.sumf == Lv);
    return true;
}

}  // namespace s2b
