// capi.cpp -- extern "C" boundary (include/seedvr2_b200.h) over DitB200.
#include "../../include/seedvr2_b200.h"
#include "dit_b200.h"
#include "dit_shard.h"
#include "synth.h"
#include "shard_plan.h"
#include <cstring>
#include <mutex>
#include <new>
#include <string>

struct s2b_ctx {
    s2b::DitB200 dit;
};

namespace {
thread_local std::string g_create_err;

int to_geom(const s2b_win* w, s2b::WinGeom& g, std::string& err) {
    if (!w) { err = "null window"; return S2B_ERR_ARG; }
    if (w->t <= 0 || w->h <= 0 || w->w <= 0 || w->nwin < 0 || w->txt_len < 0) { err = "bad window grid"; return S2B_ERR_ARG; }
    if (w->nwin > 0 && (!w->st || !w->en || !w->sh || !w->eh || !w->sw || !w->ew)) { err = "null window slices"; return S2B_ERR_ARG; }
    g.t = w->t; g.h = w->h; g.w = w->w; g.txt_len = w->txt_len;
    g.win.resize(w->nwin);
    long sumf = 0;
    for (int i = 0; i < w->nwin; i++) {
        g.win[i] = {w->st[i], w->en[i], w->sh[i], w->eh[i], w->sw[i], w->ew[i]};
        const int a = w->en[i] - w->st[i], b = w->eh[i] - w->sh[i], c = w->ew[i] - w->sw[i];
        if (a > 0 && b > 0 && c > 0) sumf += (long)a * b * c;
    }
    if (w->n_vid_freq != sumf * s2b::ROPE_ROT || w->n_txt_freq != (long)w->nwin * w->txt_len * s2b::ROPE_ROT) {
        err = "freq table sizes do not match the windows"; return S2B_ERR_ARG;
    }
    if ((w->n_vid_freq && !w->vid_freq) || (w->n_txt_freq && !w->txt_freq)) { err = "null freq tables"; return S2B_ERR_ARG; }
    g.vid_freq.assign(w->vid_freq, w->vid_freq + w->n_vid_freq);
    g.txt_freq.assign(w->txt_freq, w->txt_freq + w->n_txt_freq);
    return S2B_OK;
}
}  // namespace

extern "C" {

int s2b_ctx_create(int device, int precision, s2b_ctx** out) {
    if (!out) return S2B_ERR_ARG;
    *out = nullptr;
    s2b_ctx* c = new (std::nothrow) s2b_ctx;
    if (!c) return S2B_ERR_NOMEM;
    const int rc = c->dit.create(device, precision);
    if (rc) { g_create_err = c->dit.err; delete c; return rc; }
    *out = c;
    return S2B_OK;
}

int s2b_ctx_destroy(s2b_ctx* ctx) { delete ctx; return S2B_OK; }

const char* s2b_last_error(const s2b_ctx* ctx) { return ctx ? ctx->dit.err.c_str() : g_create_err.c_str(); }

int s2b_ctx_precision(const s2b_ctx* ctx) { return ctx ? ctx->dit.precision() : -1; }

int s2b_ctx_device_bytes(const s2b_ctx* ctx, uint64_t* bytes) {
    if (!ctx || !bytes) return S2B_ERR_ARG;
    *bytes = ctx->dit.device_bytes();
    return S2B_OK;
}

int s2b_ctx_last_launches(const s2b_ctx* ctx, int* launches) {
    if (!ctx || !launches) return S2B_ERR_ARG;
    *launches = ctx->dit.last_launches();
    return S2B_OK;
}

int s2b_load_weights_dir(s2b_ctx* ctx, const char* dir, int lo, int hi) {
    if (!ctx || !dir) return S2B_ERR_ARG;
    return ctx->dit.load_weights(dir, false, 0, lo, hi);
}

int s2b_load_weights_synth(s2b_ctx* ctx, uint64_t seed, int lo, int hi) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.load_weights(nullptr, true, seed, lo, hi);
}

int s2b_make_win_size(int t, int h, int w, const int nw[3], int txt_len, int shifted, int* nwin, long* nvf, long* ntf) {
    if (!nw || t <= 0 || h <= 0 || w <= 0 || txt_len < 0 || nw[0] <= 0 || nw[1] <= 0 || nw[2] <= 0) return S2B_ERR_ARG;
    const s2b::WinGeom g = s2b::make_win(t, h, w, nw, txt_len, shifted != 0);
    if (nwin) *nwin = g.nwin();
    if (nvf) *nvf = (long)g.vid_freq.size();
    if (ntf) *ntf = (long)g.txt_freq.size();
    return S2B_OK;
}

int s2b_make_win_fill(int t, int h, int w, const int nw[3], int txt_len, int shifted, int* st, int* en, int* sh,
                      int* eh, int* sw, int* ew, float* vf, float* tf) {
    if (!nw || t <= 0 || h <= 0 || w <= 0 || txt_len < 0 || nw[0] <= 0 || nw[1] <= 0 || nw[2] <= 0) return S2B_ERR_ARG;
    const s2b::WinGeom g = s2b::make_win(t, h, w, nw, txt_len, shifted != 0);
    for (int i = 0; i < g.nwin(); i++) {
        if (st) st[i] = g.win[i].t0;
        if (en) en[i] = g.win[i].t1;
        if (sh) sh[i] = g.win[i].h0;
        if (eh) eh[i] = g.win[i].h1;
        if (sw) sw[i] = g.win[i].w0;
        if (ew) ew[i] = g.win[i].w1;
    }
    if (vf) std::memcpy(vf, g.vid_freq.data(), g.vid_freq.size() * 4);
    if (tf) std::memcpy(tf, g.txt_freq.data(), g.txt_freq.size() * 4);
    return S2B_OK;
}

int s2b_set_windows(s2b_ctx* ctx, const s2b_win* ns, const s2b_win* sh) {
    if (!ctx) return S2B_ERR_ARG;
    s2b::WinGeom a, b;
    if (int rc = to_geom(ns, a, ctx->dit.err)) return rc;
    if (int rc = to_geom(sh, b, ctx->dit.err)) return rc;
    return ctx->dit.set_windows(a, b);
}

int s2b_forward_latent(s2b_ctx* ctx, const float* vid_in, int Lv, const float* txt_in, int TXT, float t, int l0, int l1,
                       int do_init, int do_final, float* vid_lat, float* txt_lat, float* sr_out) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.forward_latent(vid_in, Lv, txt_in, TXT, t, l0, l1, do_init != 0, do_final != 0, vid_lat, txt_lat, sr_out);
}

int s2b_forward(s2b_ctx* ctx, const float* vid_patch, int Lv, const float* txt, int TXT, float t, float* sr_out) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.forward(vid_patch, Lv, txt, TXT, t, sr_out);
}

int s2b_forward_dev(s2b_ctx* ctx, const float* d_vid, int Lv, const float* d_txt, int TXT, float t, float* d_sr,
                    void* stream) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.forward_dev(d_vid, Lv, d_txt, TXT, t, d_sr, (cudaStream_t)stream);
}

int s2b_patchify_grid(const float* g, int T, int H, int W, float* out) {   // src/dit_vk.cpp:717-733
    if (!g || !out || T <= 0 || H <= 0 || W <= 0) return S2B_ERR_ARG;
    const int H2 = H / 2, W2 = W / 2;
    for (int t = 0; t < T; t++)
        for (int hh = 0; hh < H2; hh++)
            for (int ww = 0; ww < W2; ww++)
                for (int ph = 0; ph < 2; ph++)
                    for (int pw = 0; pw < 2; pw++)
                        std::memcpy(out + ((size_t)(t * H2 + hh) * W2 + ww) * 132 + (ph * 2 + pw) * 33,
                                    g + ((size_t)(t * H + hh * 2 + ph) * W + (ww * 2 + pw)) * 33, 33 * 4);
    return S2B_OK;
}

int s2b_unpatchify_latent(const float* sr, int T, int H, int W, float* out) {   // src/dit_vk.cpp:735-750
    if (!sr || !out || T <= 0 || H <= 0 || W <= 0) return S2B_ERR_ARG;
    const int H2 = H / 2, W2 = W / 2;
    std::memset(out, 0, sizeof(float) * (size_t)T * H * W * 16);
    for (int t = 0; t < T; t++)
        for (int hh = 0; hh < H2; hh++)
            for (int ww = 0; ww < W2; ww++)
                for (int ph = 0; ph < 2; ph++)
                    for (int pw = 0; pw < 2; pw++)
                        std::memcpy(out + ((size_t)(t * H + hh * 2 + ph) * W + (ww * 2 + pw)) * 16,
                                    sr + ((size_t)(t * H2 + hh) * W2 + ww) * 64 + (ph * 2 + pw) * 16, 16 * 4);
    return S2B_OK;
}

int s2b_forward_grid(s2b_ctx* ctx, const float* grid, int T, int H, int W, const float* txt, int TXT, float t,
                     float* sr_latent) {
    if (!ctx || !grid || !txt || !sr_latent || T <= 0 || H <= 1 || W <= 1) return S2B_ERR_ARG;
    const int Lv = T * (H / 2) * (W / 2);
    std::vector<float> patch((size_t)Lv * 132), sr((size_t)Lv * 64);
    s2b_patchify_grid(grid, T, H, W, patch.data());
    if (int rc = ctx->dit.forward(patch.data(), Lv, txt, TXT, t, sr.data())) return rc;
    return s2b_unpatchify_latent(sr.data(), T, H, W, sr_latent);
}

int s2b_load_weights_mem(s2b_ctx* ctx, const s2b_weight_file* files, int nfiles, int layer_lo, int layer_hi) {
    if (!ctx || (nfiles > 0 && !files) || nfiles < 0) return S2B_ERR_ARG;
    s2b::WeightFiles table;
    for (int i = 0; i < nfiles; i++) {
        if (!files[i].name || (!files[i].data && files[i].bytes)) return S2B_ERR_ARG;
        table[files[i].name] = {files[i].data, files[i].bytes};
    }
    static std::mutex mem_load_mutex;   // the in-memory table is a process-wide hook during a load
    std::lock_guard<std::mutex> lk(mem_load_mutex);
    return ctx->dit.load_weights_mem(table, layer_lo, layer_hi);
}

int s2b_forward_grid_dev(s2b_ctx* ctx, const float* d_vid_grid, int T, int H, int W, const float* d_txt, int TXT,
                         float t, float* d_sr_grid, void* stream) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.forward_grid_dev(d_vid_grid, T, H, W, d_txt, TXT, t, d_sr_grid, (cudaStream_t)stream);
}

static int launch_status(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return S2B_OK;
    g_create_err = std::string(what) + ": " + cudaGetErrorString(e);
    return S2B_ERR_CUDA;
}

int s2b_patchify_grid_dev(const float* d_vid_grid, int T, int H, int W, float* d_vid_patch, void* stream) {
    if (!d_vid_grid || !d_vid_patch || T <= 0 || H <= 0 || W <= 0 || H % 2 || W % 2) return S2B_ERR_ARG;
    s2b::patchify_dev(d_vid_grid, T, H, W, d_vid_patch, (cudaStream_t)stream);
    return launch_status("patchify");
}

int s2b_unpatchify_latent_dev(const float* d_sr, int T, int H, int W, float* d_sr_grid, void* stream) {
    if (!d_sr || !d_sr_grid || T <= 0 || H <= 0 || W <= 0 || H % 2 || W % 2) return S2B_ERR_ARG;
    s2b::unpatchify_dev(d_sr, T, H, W, d_sr_grid, (cudaStream_t)stream);
    return launch_status("unpatchify");
}

int s2b_assemble_vid_grid_dev(const float* d_noise, const float* d_latent, float scaling, int H8, int W8,
                              float* d_vid_grid, void* stream) {
    if (!d_noise || !d_latent || !d_vid_grid || H8 <= 0 || W8 <= 0) return S2B_ERR_ARG;
    s2b::assemble_grid_dev(d_noise, d_latent, scaling, H8, W8, d_vid_grid, (cudaStream_t)stream);
    return launch_status("assemble vid_grid");
}

int s2b_decode_latent_dev(const float* d_noise, const float* d_sr_grid, float scaling, int H8, int W8,
                          float* d_z, void* stream) {
    if (!d_noise || !d_sr_grid || !d_z || H8 <= 0 || W8 <= 0 || scaling == 0.f) return S2B_ERR_ARG;
    s2b::decode_latent_dev(d_noise, d_sr_grid, scaling, H8, W8, d_z, (cudaStream_t)stream);
    return launch_status("decode latent");
}

int s2b_awa_forward(s2b_ctx* ctx, const float* vqkv, const float* tqkv, const s2b_win* win, const float* nq_v,
                    const float* nk_v, const float* nq_t, const float* nk_t, int Lv, int TXT, float eps,
                    float* vid_out, float* txt_out) {
    if (!ctx) return S2B_ERR_ARG;
    s2b::WinGeom g;
    if (int rc = to_geom(win, g, ctx->dit.err)) return rc;
    return ctx->dit.awa_forward(vqkv, tqkv, g, nq_v, nk_v, nq_t, nk_t, Lv, TXT, eps, vid_out, txt_out);
}

int s2b_awa_set_geometry(s2b_ctx* ctx, int win_type, const s2b_win* win) {
    if (!ctx) return S2B_ERR_ARG;
    s2b::WinGeom g;
    if (int rc = to_geom(win, g, ctx->dit.err)) return rc;
    return ctx->dit.awa_set_geometry(win_type, g);
}

int s2b_awa_forward_dev(s2b_ctx* ctx, int win_type, const float* vqkv, const float* tqkv, const float* nqv,
                        const float* nkv, const float* nqt, const float* nkt, int Lv, int TXT, float eps,
                        float* vid_out, float* txt_out, void* stream) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.awa_forward_dev(win_type, vqkv, tqkv, nqv, nkv, nqt, nkt, Lv, TXT, eps, vid_out, txt_out,
                                    (cudaStream_t)stream);
}

int s2b_awa_forward_dev_static(s2b_ctx* ctx, int win_type, const float* vqkv, const float* tqkv, const float* nqv,
                               const float* nkv, const float* nqt, const float* nkt, int Lv, int TXT, float eps,
                               float* vid_out, float* txt_out, void* stream) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.awa_forward_dev_static(win_type, vqkv, tqkv, nqv, nkv, nqt, nkt, Lv, TXT, eps, vid_out, txt_out,
                                           (cudaStream_t)stream);
}

int s2b_time_embedding(s2b_ctx* ctx, float t, float* emb) {
    if (!ctx || !emb) return S2B_ERR_ARG;
    return ctx->dit.time_embedding(t, emb);
}

int s2b_ada_compose(s2b_ctx* ctx, const float* emb, float* out) {
    if (!ctx || !emb || !out) return S2B_ERR_ARG;
    return ctx->dit.ada_compose(emb, out);
}

int s2b_forward_profile(s2b_ctx* ctx, const float* vid_patch, int Lv, const float* txt, int TXT, float t, double* ms,
                        double* flops, double* bytes, int* launches) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.forward_profile(vid_patch, Lv, txt, TXT, t, ms, flops, bytes, launches);
}

int s2b_shard_forward_profile(s2b_ctx* ctx, const float* vid_patch, int Lv, const float* txt, int TXT, float t, double* ms,
                        double* flops, double* bytes, int* launches) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.forward_profile(vid_patch, Lv, txt, TXT, t, ms, flops, bytes, launches, true);
}

int s2b_linear(s2b_ctx* ctx, const float* x, int M, int K, const float* W, int N, const float* bias, float* y) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.linear(x, M, K, W, N, bias, y);
}

int s2b_linear_bf16_dev(s2b_ctx* ctx, const void* d_x, int M, int K, const void* d_w, int N, const float* d_bias,
                        void* d_y, void* stream) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.linear_bf16_dev(d_x, M, K, d_w, N, d_bias, d_y, (cudaStream_t)stream);
}

int s2b_synth_write_m5(const char* dir, uint64_t seed, int lo, int hi) {
    if (!dir) return S2B_ERR_ARG;
    std::string err;
    return s2b::write_m5(dir, seed, lo, hi, err);
}

int s2b_synth_vid_grid(float* g, int T, int H, int W, uint64_t seed) {
    if (!g || T <= 0 || H <= 0 || W <= 0) return S2B_ERR_ARG;
    s2b::synth_vid_grid(g, T, H, W, seed);
    return S2B_OK;
}

int s2b_synth_txt(float* txt, int TXT, uint64_t seed) {
    if (!txt || TXT < 0) return S2B_ERR_ARG;
    s2b::synth_txt(txt, TXT, seed);
    return S2B_OK;
}

int s2b_synth_normal(float* out, long n, uint64_t seed, const char* stream, float mean, float stdv) {
    if (!out || n < 0 || !stream) return S2B_ERR_ARG;
    s2b::fill_normal_f32(out, (size_t)n, seed, s2b::fnv1a(stream), mean, stdv);
    return S2B_OK;
}

int s2b_nccl_unique_id(uint8_t id[128]);   // dit_shard.cpp

int s2b_shard_init(s2b_ctx* ctx, const uint8_t id[128], int world, int rank) {
    if (!ctx || !id) return S2B_ERR_ARG;
    return ctx->dit.shard_init(id, world, rank);
}

int s2b_shard_forward(s2b_ctx* ctx, const float* vid_patch, int Lv, const float* txt, int TXT, float t, float* sr_out) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.shard_forward(vid_patch, Lv, txt, TXT, t, sr_out);
}

int s2b_shard_forward_dev(s2b_ctx* ctx, const float* d_vid_patch, int Lv, const float* d_txt, int TXT, float t,
                          float* d_sr, void* stream) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.shard_forward_dev(d_vid_patch, Lv, d_txt, TXT, t, d_sr, (cudaStream_t)stream);
}

int s2b_shard_resync(s2b_ctx* ctx) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.shard_resync();
}

int s2b_set_last_layer_semantics(s2b_ctx* ctx, int graph) {
    if (!ctx || (graph != 0 && graph != 1)) return S2B_ERR_ARG;
    return ctx->dit.set_graph_last_layer(graph == 1);
}

int s2b_check_errors(s2b_ctx* ctx) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.check_errors();
}

int s2b_debug_raise_kernel_error(s2b_ctx* ctx, int mask) {
    if (!ctx) return S2B_ERR_ARG;
    return ctx->dit.debug_raise_kernel_error(mask);
}

int s2b_debug_watchdog_selftest(int scenario, int timeout_ms, int* polls, int* aborted) {
    if (scenario < 0 || scenario > 3 || timeout_ms <= 0) return -1;
    int n = 0, ab = 0;
    const int r = s2b::watch_completion(
        [&] {
            n++;
            if (scenario == 0 && n >= 4) return (int)s2b::WATCH_Q_DONE;
            if (scenario == 3 && n >= 3) return (int)s2b::WATCH_Q_ERROR;
            return (int)s2b::WATCH_Q_PENDING;
        },
        [&] { return scenario == 2 && n >= 2; },
        [&] { ab++; },
        (uint64_t)timeout_ms * 1000000ull, 1000000ull);
    if (polls) *polls = n;
    if (aborted) *aborted = ab;
    return r;
}

int s2b_shard_plan(const s2b_win* ns, const s2b_win* sh, int world, int rank, int* bounds, int* n_local,
                   int* tokens, int* send_off, int* send_idx, int* recv_off, int* recv_idx) {
    s2b::WinGeom a, b;
    std::string err;
    if (to_geom(ns, a, err) || to_geom(sh, b, err)) return S2B_ERR_ARG;
    s2b::WinTables ta, tb;
    const char* why = nullptr;
    if (!s2b::build_tables(a, ta, &why) || !s2b::build_tables(b, tb, &why)) return S2B_ERR_ARG;
    s2b::ShardPlan P;
    if (!s2b::make_shard_plan(a, ta, b, tb, world, rank, P, &why)) return S2B_ERR_ARG;
    const int Lv = P.Lv;
    for (int p = 0; p < 2; p++) {
        auto put = [](int* dst, const std::vector<int>& v) { if (dst) std::memcpy(dst, v.data(), v.size() * sizeof(int)); };
        put(bounds ? bounds + p * (world + 1) : nullptr, P.bounds[p]);
        if (n_local) n_local[p] = P.n_local(p);
        put(tokens ? tokens + (size_t)p * Lv : nullptr, P.tokens[p]);
        put(send_off ? send_off + p * (world + 1) : nullptr, P.send_off[p]);
        put(send_idx ? send_idx + (size_t)p * Lv : nullptr, P.send_idx[p]);
        put(recv_off ? recv_off + p * (world + 1) : nullptr, P.recv_off[p]);
        put(recv_idx ? recv_idx + (size_t)p * Lv : nullptr, P.recv_idx[p]);
    }
    return S2B_OK;
}

}  // extern "C"
