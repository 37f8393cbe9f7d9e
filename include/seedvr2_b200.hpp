// seedvr2_b200.hpp -- header-only C++ drop-in over the C ABI (seedvr2_b200.h)
// with the reference engine's class interfaces, so its call sites compile
// against the B200 path by swapping the type:
//
//   Win                   mirrors struct Win          (src/dit_vk.h:17-22)
//   make_win              mirrors awa::make_win       (src/awa_window.cpp:161-178)
//   DitB200               mirrors class DitVk         (src/dit_vk.h:24-204)
//   AwaB200               mirrors class AwaVk         (src/awa_vk.h:14-52)
//
// Methods keep the reference's names, arguments and bool-plus-stderr error
// behaviour.  The Vulkan-only housekeeping (reclaim_vram, reset_vulkan_device,
// release_graph, load_graph) has nothing to do here: weights stay resident in
// HBM and the 32-layer forward is one captured CUDA graph.  The reference's
// CPU mode (use_cpu) is not offered: init then fails with a message, as the
// reference does for a missing model.  Its fp16 arithmetic switch maps to
// fp16 operands (precision 1) when no storage precision is given.
#ifndef SEEDVR2_B200_HPP
#define SEEDVR2_B200_HPP

#include "seedvr2_b200.h"

#include <cstdio>
#include <string>
#include <vector>

namespace seedvr2_b200 {

struct Win {
    int t = 0, h = 0, w = 0, nwin = 0;
    int txt_len = 8;
    std::vector<int> st, en, sh, eh, sw, ew;
    std::vector<float> vid_freq, txt_freq;
};

// C view of a Win (the vectors must outlive it).
inline s2b_win to_c(const Win& w) {
    s2b_win c;
    c.t = w.t; c.h = w.h; c.w = w.w; c.nwin = w.nwin; c.txt_len = w.txt_len;
    c.st = w.st.data(); c.en = w.en.data(); c.sh = w.sh.data(); c.eh = w.eh.data(); c.sw = w.sw.data();
    c.ew = w.ew.data();
    c.vid_freq = w.vid_freq.data(); c.n_vid_freq = (long)w.vid_freq.size();
    c.txt_freq = w.txt_freq.data(); c.n_txt_freq = (long)w.txt_freq.size();
    return c;
}

inline Win make_win(int t, int h, int w, const int num_windows[3], int txt_len, bool shifted) {
    Win out;
    long nvf = 0, ntf = 0;
    if (s2b_make_win_size(t, h, w, num_windows, txt_len, shifted ? 1 : 0, &out.nwin, &nvf, &ntf) != S2B_OK) return out;
    out.t = t; out.h = h; out.w = w; out.txt_len = txt_len;
    for (auto* v : {&out.st, &out.en, &out.sh, &out.eh, &out.sw, &out.ew}) v->resize(out.nwin);
    out.vid_freq.resize(nvf);
    out.txt_freq.resize(ntf);
    s2b_make_win_fill(t, h, w, num_windows, txt_len, shifted ? 1 : 0, out.st.data(), out.en.data(), out.sh.data(),
                      out.eh.data(), out.sw.data(), out.ew.data(), out.vid_freq.data(), out.txt_freq.data());
    return out;
}

class DitB200 {
public:
    explicit DitB200(int device = 0) : device_(device) {}
    ~DitB200() { if (ctx_) s2b_ctx_destroy(ctx_); }
    DitB200(const DitB200&) = delete;
    DitB200& operator=(const DitB200&) = delete;

    // DitVk::init(model_dir, fp16_arith, precision{0 fp32, 1 fp16, 2 bf16}, use_cpu)
    bool init(const std::string& model_dir, bool fp16_arith = false, int precision = 0, bool use_cpu = false) {
        if (use_cpu) return fail("DitB200: CPU mode is not offered (B200 only)");
        if (fp16_arith && precision == 0) precision = S2B_PREC_FP16;   // fp16 arithmetic asked for
        if (ctx_) { s2b_ctx_destroy(ctx_); ctx_ = nullptr; }
        if (s2b_ctx_create(device_, precision, &ctx_) != S2B_OK) {
            ctx_ = nullptr;
            return fail(s2b_last_error(nullptr));
        }
        return ok(s2b_load_weights_dir(ctx_, model_dir.c_str(), 0, 32));
    }
    // Loads only layers [layer_lo, layer_hi) (plus the input / output
    // projections): enough for forward_latent over that range, as the
    // reference's chunked path uses one chunk at a time.
    bool init(const std::string& model_dir, int precision, int layer_lo, int layer_hi) {
        if (ctx_) { s2b_ctx_destroy(ctx_); ctx_ = nullptr; }
        if (s2b_ctx_create(device_, precision, &ctx_) != S2B_OK) {
            ctx_ = nullptr;
            return fail(s2b_last_error(nullptr));
        }
        return ok(s2b_load_weights_dir(ctx_, model_dir.c_str(), layer_lo, layer_hi));
    }

    bool forward(const std::vector<float>& vid_patch, int Lv, const std::vector<float>& txt, int TXT,
                 float timestep, std::vector<float>& out_sr) {
        if (!ctx_) return fail("DitB200: init has not run");
        if (!windows()) return false;
        out_sr.assign((size_t)Lv * 64, 0.f);
        return ok(s2b_forward(ctx_, vid_patch.data(), Lv, txt.data(), TXT, timestep, out_sr.data()));
    }

    bool forward_grid(const std::vector<float>& vid_grid, int T, int H, int W, const std::vector<float>& txt,
                      int TXT, float timestep, std::vector<float>& sr_latent) {
        if (!ctx_) return fail("DitB200: init has not run");
        if (!windows()) return false;
        sr_latent.assign((size_t)T * H * W * 16, 0.f);
        return ok(s2b_forward_grid(ctx_, vid_grid.data(), T, H, W, txt.data(), TXT, timestep, sr_latent.data()));
    }

    void set_windows(const Win& ns, const Win& sh) { win_ns_ = ns; win_sh_ = sh; win_dirty_ = true; }
    bool awa_ready() const { return ctx_ != nullptr; }
    void reclaim_vram() {}
    void reset_vulkan_device() {}

    static std::vector<float> patchify_grid(const std::vector<float>& vid_grid, int T, int H, int W) {
        std::vector<float> out((size_t)T * (H / 2) * (W / 2) * 132);
        s2b_patchify_grid(vid_grid.data(), T, H, W, out.data());
        return out;
    }
    static std::vector<float> unpatchify_latent(const std::vector<float>& sr_latent, int T, int H, int W) {
        std::vector<float> out((size_t)T * H * W * 16);
        s2b_unpatchify_latent(sr_latent.data(), T, H, W, out.data());
        return out;
    }

    bool forward_latent(const std::vector<float>& vid_patch, int Lv, const std::vector<float>& txt, int TXT,
                        float timestep, int l0, int l1, bool do_init, bool do_final,
                        std::vector<float>& vid_out_latent, std::vector<float>& txt_out_latent,
                        std::vector<float>& sr_out) {
        if (!ctx_) return fail("DitB200: init has not run");
        if (!windows()) return false;
        if (do_final) {
            sr_out.assign((size_t)Lv * 64, 0.f);
            return ok(s2b_forward_latent(ctx_, vid_patch.data(), Lv, txt.data(), TXT, timestep, l0, l1,
                                         do_init ? 1 : 0, 1, nullptr, nullptr, sr_out.data()));
        }
        vid_out_latent.assign((size_t)Lv * 2560, 0.f);
        txt_out_latent.assign((size_t)TXT * 2560, 0.f);
        return ok(s2b_forward_latent(ctx_, vid_patch.data(), Lv, txt.data(), TXT, timestep, l0, l1, do_init ? 1 : 0,
                                     0, vid_out_latent.data(), txt_out_latent.data(), nullptr));
    }

    // Stage-3 graph API: the weights are already resident and the 32-layer
    // forward is captured on first use, whatever the chunking asked for.
    bool load_graph(const std::string&, int = 4) { return ctx_ != nullptr; }
    bool load_single(const std::string&, const std::string& = "dit_graph", int = 32) { return ctx_ != nullptr; }
    bool graph_ready() const { return ctx_ != nullptr; }
    bool forward_graph(const std::vector<float>& vid_patch, int Lv, const std::vector<float>& txt, int TXT,
                       float timestep, std::vector<float>& out_sr) {
        return forward(vid_patch, Lv, txt, TXT, timestep, out_sr);
    }
    void release_graph() {}
    int get_precision() const { return ctx_ ? s2b_ctx_precision(ctx_) : -1; }

    std::vector<float> time_embedding(float t) {
        std::vector<float> e(15360, 0.f);
        if (ctx_) s2b_time_embedding(ctx_, t, e.data());
        return e;
    }

    s2b_ctx* handle() const { return ctx_; }
    const char* last_error() const { return ctx_ ? s2b_last_error(ctx_) : s2b_last_error(nullptr); }

private:
    bool fail(const char* msg) {
        std::fprintf(stderr, "[DitB200] %s\n", msg ? msg : "error");
        return false;
    }
    bool ok(int rc) { return rc == S2B_OK ? true : fail(s2b_last_error(ctx_)); }
    bool windows() {
        if (!win_dirty_) return true;
        const s2b_win a = to_c(win_ns_), b = to_c(win_sh_);
        if (!ok(s2b_set_windows(ctx_, &a, &b))) return false;
        win_dirty_ = false;
        return true;
    }

    int device_ = 0;
    s2b_ctx* ctx_ = nullptr;
    Win win_ns_, win_sh_;
    bool win_dirty_ = false;
};

class AwaB200 {
public:
    ~AwaB200() { if (ctx_) s2b_ctx_destroy(ctx_); }
    // AwaVk::init(vkdev, spv_path) -> a device index; bf16 tensor-core or fp32 arithmetic.
    bool init(int device = 0, int precision = S2B_PREC_FP32) {
        if (ctx_) { s2b_ctx_destroy(ctx_); ctx_ = nullptr; }
        if (s2b_ctx_create(device, precision, &ctx_) != S2B_OK) {
            ctx_ = nullptr;
            std::fprintf(stderr, "[AwaB200] %s\n", s2b_last_error(nullptr));
            return false;
        }
        return true;
    }
    bool ready() const { return ctx_ != nullptr; }
    // AwaVk::forward: the txt output is already averaged over the windows.
    bool forward(const std::vector<float>& vqkv, const std::vector<float>& tqkv, const Win& win,
                 const std::vector<float>& nq_v, const std::vector<float>& nk_v, const std::vector<float>& nq_t,
                 const std::vector<float>& nk_t, int Lv, int TXT, std::vector<float>& vid_out,
                 std::vector<float>& txt_out) {
        if (!ctx_) return false;
        vid_out.assign((size_t)Lv * 2560, 0.f);
        txt_out.assign((size_t)TXT * 2560, 0.f);
        const s2b_win w = to_c(win);
        if (s2b_awa_forward(ctx_, vqkv.data(), tqkv.data(), &w, nq_v.data(), nk_v.data(), nq_t.data(), nk_t.data(),
                            Lv, TXT, eps, vid_out.data(), txt_out.data()) != S2B_OK) {
            std::fprintf(stderr, "[AwaB200] %s\n", s2b_last_error(ctx_));
            return false;
        }
        return true;
    }
    float eps = 1e-5f;   // the qk-norm epsilon the reference's push constant carries

private:
    s2b_ctx* ctx_ = nullptr;
};

}  // namespace seedvr2_b200

#endif  // SEEDVR2_B200_HPP
