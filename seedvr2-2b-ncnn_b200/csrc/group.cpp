// group.cpp -- frame-sequence mode on several GPUs from one process.
//
// The engine processes a video frame by frame (src/main.cpp:126-147,
// src/seedvr2_engine.cpp:96: each frame has its own noise seed), and frames
// are independent.  A group holds one context per GPU, each with the whole
// model resident; frame k runs on GPU k mod N, every GPU driven by its own
// host thread, with no communication between GPUs.
#include "../../include/seedvr2_b200.h"

#include <string>
#include <thread>
#include <vector>

struct s2b_group {
    std::vector<s2b_ctx*> ctx;
    std::string err;
};

namespace {

// Runs fn(i) for every member on its own thread; the first failure's status
// and message are kept.
template <typename F>
int for_each_member(s2b_group* g, F fn) {
    const int n = (int)g->ctx.size();
    std::vector<int> rc(n, S2B_OK);
    std::vector<std::thread> th;
    for (int i = 0; i < n; i++) th.emplace_back([&, i] { rc[i] = fn(i); });
    for (auto& t : th) t.join();
    for (int i = 0; i < n; i++)
        if (rc[i] != S2B_OK) {
            const char* m = s2b_last_error(g->ctx[i]);
            g->err = "GPU member " + std::to_string(i) + ": " + (m ? m : "error");
            return rc[i];
        }
    return S2B_OK;
}

}  // namespace

extern "C" {

int s2b_group_create(int ngpu, const int* devices, int precision, s2b_group** out) {
    if (!out || ngpu <= 0) return S2B_ERR_ARG;
    *out = nullptr;
    auto* g = new s2b_group();
    for (int i = 0; i < ngpu; i++) {
        s2b_ctx* c = nullptr;
        const int rc = s2b_ctx_create(devices ? devices[i] : i, precision, &c);
        if (rc != S2B_OK) {
            for (auto* x : g->ctx) s2b_ctx_destroy(x);
            delete g;
            return rc;
        }
        g->ctx.push_back(c);
    }
    *out = g;
    return S2B_OK;
}

int s2b_group_destroy(s2b_group* g) {
    if (!g) return S2B_ERR_ARG;
    for (auto* c : g->ctx) s2b_ctx_destroy(c);
    delete g;
    return S2B_OK;
}

const char* s2b_group_last_error(const s2b_group* g) { return g ? g->err.c_str() : "null group"; }

int s2b_group_load_weights_dir(s2b_group* g, const char* m5_dir) {
    if (!g || !m5_dir) return S2B_ERR_ARG;
    return for_each_member(g, [&](int i) { return s2b_load_weights_dir(g->ctx[i], m5_dir, 0, 32); });
}

int s2b_group_load_weights_synth(s2b_group* g, uint64_t seed) {
    if (!g) return S2B_ERR_ARG;
    return for_each_member(g, [&](int i) { return s2b_load_weights_synth(g->ctx[i], seed, 0, 32); });
}

int s2b_group_set_windows(s2b_group* g, const s2b_win* ns, const s2b_win* sh) {
    if (!g || !ns || !sh) return S2B_ERR_ARG;
    return for_each_member(g, [&](int i) { return s2b_set_windows(g->ctx[i], ns, sh); });
}

int s2b_group_forward_frames(s2b_group* g, const float* vid_patches, int nframes, int Lv, const float* txt, int TXT,
                             float timestep, float* sr_out) {
    if (!g || !vid_patches || !txt || !sr_out || nframes < 0 || Lv <= 0 || TXT <= 0) return S2B_ERR_ARG;
    const int n = (int)g->ctx.size();
    const size_t in_stride = (size_t)Lv * 132, out_stride = (size_t)Lv * 64;
    return for_each_member(g, [&](int i) {
        for (int k = i; k < nframes; k += n) {
            const int rc = s2b_forward(g->ctx[i], vid_patches + k * in_stride, Lv, txt, TXT, timestep,
                                       sr_out + k * out_stride);
            if (rc != S2B_OK) return rc;
        }
        return (int)S2B_OK;
    });
}

}  // extern "C"
