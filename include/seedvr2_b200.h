/*
 * seedvr2_b200.h -- C ABI of the B200 (sm_100a) NaDiT DiT forward and its
 * Adaptive Window Attention (AWA).
 *
 * This is the drop-in boundary for the reference's DiT hot path
 * (AiChiTuDouPian/SeedVR2-2b-ncnn).  Every entry point names the reference
 * interface it replaces (file:line in that project).  Conventions:
 *   - every call returns an int status, 0 = S2B_OK; on failure the context's
 *     message is available from s2b_last_error(ctx) (the reference prints to
 *     stderr and returns false / -1);
 *   - a context owns one CUDA device, its weights (resident in HBM) and all
 *     scratch; it is not thread-safe: one context per host thread and device;
 *   - host-buffer entry points copy in, run, copy out and return when the
 *     result is on the host (the reference's submit_and_wait semantics);
 *     "_dev" entry points take device pointers and a cudaStream_t (passed as
 *     void*) and only enqueue (the ncnn custom-layer semantics: record on the
 *     caller's command stream);
 *   - inputs are never retained; outputs are caller-owned;
 *   - S2B_ERR_TIMEOUT: every wait inside the tensor-core kernels and the
 *     multi-GPU exchanges is bounded; one that expires makes its kernel return
 *     early (the output of that call is incomplete) and raises a device flag.
 *     The last kernel of every call folds those flags into the context's
 *     status word.  Host-buffer calls read it after their final
 *     synchronisation and return S2B_ERR_TIMEOUT; "_dev" calls cannot report
 *     at return, so read it with s2b_check_errors after the work finished
 *     (the next host-buffer call on the context reports it too).  The flags
 *     are per device: a context may see an expiry of another context's
 *     kernels on the same device.
 * Layouts are the reference's: fp32, row-major, token index ((t*H)+h)*W+w,
 * qkv rows [q(20x128) | k | v] (src/awa_vk.h:36), patches (ph,pw,c).
 */
#ifndef SEEDVR2_B200_H
#define SEEDVR2_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define S2B_OK 0
#define S2B_ERR_ARG 1
#define S2B_ERR_CUDA 2
#define S2B_ERR_IO 3
#define S2B_ERR_STATE 4
#define S2B_ERR_UNSUPPORTED 5
#define S2B_ERR_NCCL 6
#define S2B_ERR_TIMEOUT 7
#define S2B_ERR_NOMEM 8

/* precision: GEMM/attention operand type (reference DitVk::init `precision`,
 * src/dit_vk.h:37-39: 0 fp32, 1 fp16, 2 bf16).  fp16 and bf16 run the same
 * tcgen05 kernels (kind::f16, fp32 accumulation) with IEEE binary16 or bf16
 * operands; fp16 keeps 3 more mantissa bits, so a 32-layer forward stays
 * within cos 0.99999 of fp32 where bf16 sits near 0.9996.  The residual
 * stream is fp32 in every mode. */
#define S2B_PREC_FP32 0
#define S2B_PREC_FP16 1
#define S2B_PREC_BF16 2

typedef struct s2b_ctx s2b_ctx;

/* C mirror of the reference `Win` (src/dit_vk.h:17-22): grid (t,h,w), window
 * slices [st,en) x [sh,eh) x [sw,ew) and the RoPE angle tables
 * vid_freq[sum(f_i) x 126] (window-packed order) and
 * txt_freq[nwin x txt_len x 126]. */
typedef struct s2b_win {
    int t, h, w, nwin, txt_len;
    const int *st, *en, *sh, *eh, *sw, *ew;
    const float* vid_freq;
    long n_vid_freq;
    const float* txt_freq;
    long n_txt_freq;
} s2b_win;

/* ---- context --------------------------------------------------------- */
/* Replaces DitVk::DitVk + the device half of DitVk::init (src/dit_vk.cpp:140-155). */
int s2b_ctx_create(int device, int precision, s2b_ctx** out);
/* Replaces DitVk::~DitVk (src/dit_vk.cpp:97-107). */
int s2b_ctx_destroy(s2b_ctx* ctx);
const char* s2b_last_error(const s2b_ctx* ctx);
int s2b_ctx_precision(const s2b_ctx* ctx);
/* Device bytes held by the context (weights + activations + scratch). */
int s2b_ctx_device_bytes(const s2b_ctx* ctx, uint64_t* bytes);
/* Number of kernels the last forward enqueued (for launch accounting). */
int s2b_ctx_last_launches(const s2b_ctx* ctx, int* launches);

/* ---- weights --------------------------------------------------------- */
/* Replaces the weight half of DitVk::init (src/dit_vk.cpp:156-177) and the
 * per-Linear ncnn Net loads of DitVk::lin/get_net (src/dit_vk.cpp:204-293):
 * reads the m5 directory layout (<base>.param/.bin fp16 Linear blobs, raw
 * fp32 vectors) for layers [layer_lo, layer_hi) plus the top-level modules,
 * and keeps everything resident in HBM. */
int s2b_load_weights_dir(s2b_ctx* ctx, const char* m5_dir, int layer_lo, int layer_hi);
/* Same tensors as s2b_synth_write_m5(seed) would write, generated in host
 * memory and uploaded without touching the disk. */
int s2b_load_weights_synth(s2b_ctx* ctx, uint64_t seed, int layer_lo, int layer_hi);

/* ---- geometry -------------------------------------------------------- */
/* Replaces awa::make_win (src/awa_window.cpp:161-178).  Two-step: query the
 * sizes, then fill caller buffers (st..ew: nwin ints each). */
int s2b_make_win_size(int t, int h, int w, const int num_windows[3], int txt_len, int shifted,
                      int* nwin, long* n_vid_freq, long* n_txt_freq);
int s2b_make_win_fill(int t, int h, int w, const int num_windows[3], int txt_len, int shifted,
                      int* st, int* en, int* sh, int* eh, int* sw, int* ew, float* vid_freq, float* txt_freq);
/* Replaces DitVk::set_windows (src/dit_vk.h:58) and the AWA layers'
 * set_window_geometry injection (src/dit_graph.cpp:221-262): even layers use
 * `ns`, odd layers `sh` (src/dit_vk.cpp:518). */
int s2b_set_windows(s2b_ctx* ctx, const s2b_win* ns, const s2b_win* sh);

/* ---- DiT forward ----------------------------------------------------- */
/* Replaces DitVk::forward_latent (src/dit_vk.cpp:486-699).  Runs layers
 * [l0, l1).  do_init: vid_in is the (Lv,132) patch input and txt_in (TXT,5120);
 * else they are the (Lv,2560)/(TXT,2560) residual latents of a previous chunk.
 * do_final: writes sr_out (Lv,64) (vid_lat/txt_lat untouched); else writes
 * vid_lat (Lv,2560) and txt_lat (TXT,2560). */
int s2b_forward_latent(s2b_ctx* ctx, const float* vid_in, int Lv, const float* txt_in, int TXT,
                       float timestep, int l0, int l1, int do_init, int do_final,
                       float* vid_lat, float* txt_lat, float* sr_out);
/* Semantics of the last layer (31) for the txt rows.  0 (default):
 * DitVk::forward_latent's vid_only block -- txt is not modulated, not gated
 * and skips its MLP (src/dit_vk.cpp:523-625).  1: the chunked graph that
 * DitVk::forward_graph runs (export/export_dit_graph.py:155-226) -- txt is
 * treated as in every other layer, which changes the txt K/V of the last
 * attention and so the vid output.  Applies to every forward entry point. */
int s2b_set_last_layer_semantics(s2b_ctx* ctx, int graph);
/* Replaces DitVk::forward (src/dit_vk.cpp:710-715) and DitVk::forward_graph
 * (src/dit_graph.cpp:264-549): all 32 layers, replayed from one captured CUDA
 * graph per (Lv, TXT) with weights resident. */
int s2b_forward(s2b_ctx* ctx, const float* vid_patch, int Lv, const float* txt, int TXT,
                float timestep, float* sr_out);
/* Device-pointer form of s2b_forward; enqueues on `stream` (cudaStream_t).
 * d_vid_patch (Lv,132) fp32, d_txt (TXT,5120) fp32, d_sr_out (Lv,64) fp32. */
int s2b_forward_dev(s2b_ctx* ctx, const float* d_vid_patch, int Lv, const float* d_txt, int TXT,
                    float timestep, float* d_sr_out, void* stream);
/* Replaces DitVk::forward_grid (src/dit_vk.cpp:752-763). */
int s2b_forward_grid(s2b_ctx* ctx, const float* vid_grid, int T, int H, int W, const float* txt, int TXT,
                     float timestep, float* sr_latent);
/* Replace DitVk::patchify_grid / unpatchify_latent (src/dit_vk.cpp:717-750). */
int s2b_patchify_grid(const float* vid_grid, int T, int H, int W, float* vid_patch);
int s2b_unpatchify_latent(const float* sr, int T, int H, int W, float* sr_latent);

/* One file of the m5 model directory held in memory (name as in the
 * directory, e.g. "b0_vid_qkv.param", "b0_vid_qkv.bin", "b0_vid_nq.bin"). */
typedef struct s2b_weight_file {
    const char* name;
    const void* data;
    size_t bytes;
} s2b_weight_file;
/* s2b_load_weights_dir with the directory's files supplied in memory (for a
 * host that already holds the model, e.g. from an archive); the same layout
 * and checks (src/dit_vk.cpp:140-177 reads these files one by one). */
int s2b_load_weights_mem(s2b_ctx* ctx, const s2b_weight_file* files, int nfiles, int layer_lo, int layer_hi);

/* ---- device-side data formats around the DiT --------------------------- */
/* DitVk::forward_grid (src/dit_vk.cpp:752-763) on device buffers, ordered on
 * `stream` (cudaStream_t): patchify, the captured 32-layer forward and
 * unpatchify run on the GPU.  d_vid_grid (T, H, W, 33), d_txt (TXT, 5120),
 * d_sr_grid (T, H, W, 16), all fp32; H and W even. */
int s2b_forward_grid_dev(s2b_ctx* ctx, const float* d_vid_grid, int T, int H, int W, const float* d_txt, int TXT,
                         float timestep, float* d_sr_grid, void* stream);
/* patchify_grid / unpatchify_latent (src/dit_vk.cpp:717-750) as kernels on
 * device buffers; no context needed. */
int s2b_patchify_grid_dev(const float* d_vid_grid, int T, int H, int W, float* d_vid_patch, void* stream);
int s2b_unpatchify_latent_dev(const float* d_sr, int T, int H, int W, float* d_sr_grid, void* stream);
/* The engine's DiT input assembly (src/seedvr2_engine.cpp:154-168): vid_grid
 * (H8, W8, 33) = [noise | latent * scaling | 1] from channel-first (16, H8,
 * W8) noise and condition latent (the engine passes scaling 0.9152,
 * src/seedvr2_engine.cpp:22). */
int s2b_assemble_vid_grid_dev(const float* d_noise, const float* d_latent, float scaling, int H8, int W8,
                              float* d_vid_grid, void* stream);
/* The engine's step after the DiT (src/seedvr2_engine.cpp:298-305): z
 * (16, H8, W8) = (noise - sr) / scaling with sr channel-last (H8, W8, 16). */
int s2b_decode_latent_dev(const float* d_noise, const float* d_sr_grid, float scaling, int H8, int W8, float* d_z,
                          void* stream);

/* ---- AWA operator ---------------------------------------------------- */
/* Replaces AwaVk::forward (src/awa_vk.h:39-44, src/awa_vk.cpp:114-251) and
 * the CPU attention branch of DitVk::awa_forward (src/dit_vk.cpp:344-455):
 * qk RMSNorm (eps), 3-axis RoPE, per-window SDPA over [window vid | txt],
 * reverse partition (tokens outside every window get 0), txt mean over
 * windows.  vqkv (Lv,7680), tqkv (TXT,7680), nq_v/nk_v/nq_t/nk_t (128) fp32 host;
 * vid_out (Lv,2560), txt_out (TXT,2560). */
int s2b_awa_forward(s2b_ctx* ctx, const float* vqkv, const float* tqkv, const s2b_win* win,
                    const float* nq_v, const float* nk_v, const float* nq_t, const float* nk_t,
                    int Lv, int TXT, float eps, float* vid_out, float* txt_out);
/* Replaces AwaLayer::forward (src/awa_layer.cpp:284-453): same op on device
 * buffers, enqueued on `stream`; the geometry is the one last passed to
 * s2b_awa_set_geometry for `win_type` (0 non-shifted, 1 shifted), like
 * AwaLayer::set_window_geometry (src/awa_layer.cpp:73-91).  Every device
 * buffer must be 16-byte aligned (S2B_ERR_ARG otherwise; cudaMalloc'ed
 * buffers are). */
int s2b_awa_set_geometry(s2b_ctx* ctx, int win_type, const s2b_win* win);
int s2b_awa_forward_dev(s2b_ctx* ctx, int win_type, const float* d_vqkv, const float* d_tqkv,
                        const float* d_nq_v, const float* d_nk_v, const float* d_nq_t, const float* d_nk_t,
                        int Lv, int TXT, float eps, float* d_vid_out, float* d_txt_out, void* stream);

/* No counterpart in the reference.  s2b_awa_forward_dev without any device
 * allocation, for callers that cannot allocate device memory while they run
 * (a host framework that owns all device memory and hands a plugin only its
 * inputs and outputs, or a latency-critical loop where cudaMalloc/cudaFree
 * would synchronise the device).  Its scratch (packed Q/K/V and the per-window
 * txt partials) lives in one fixed 32 MiB device array inside the library
 * that every device loading the library holds until exit; a geometry needing
 * more (3 * sumS * 2560 * (4 fp32 | 2 bf16) + nwin * TXT * 2560 * 4 bytes,
 * sumS = sum over windows of (f_i + TXT)) is rejected with S2B_ERR_ARG.  The
 * geometry comes from s2b_awa_set_geometry, which does allocate: call it at
 * set-up time.  The first call on a device also resolves the array's device
 * address: make it before any stream capture.  Calls share the array, so
 * calls whose GPU work overlaps race; serialise them.  Device buffers
 * 16-byte aligned, as for s2b_awa_forward_dev.  Enqueues on `stream` and
 * returns without waiting. */
int s2b_awa_forward_dev_static(s2b_ctx* ctx, int win_type, const float* d_vqkv, const float* d_tqkv,
                               const float* d_nq_v, const float* d_nk_v, const float* d_nq_t, const float* d_nk_t,
                               int Lv, int TXT, float eps, float* d_vid_out, float* d_txt_out, void* stream);

/* ---- adaLN ----------------------------------------------------------- */
/* Replaces DitVk::time_embedding (src/dit_vk.cpp:295-309): emb[15360]. */
int s2b_time_embedding(s2b_ctx* ctx, float timestep, float* emb);
/* Replaces AdaComposeLayer::forward (src/ada_compose.cpp:166-235) and
 * DitVk::compute_ada (src/dit_graph.cpp:196-216): from emb[15360] writes the
 * 32*12 + 2 modulation vectors of 2560 in the layer's output order
 * [layer][flow vid,txt][a_sc,a_sh,a_g,m_sc,m_sh,m_g], then fin_sc, fin_sh. */
int s2b_ada_compose(s2b_ctx* ctx, const float* emb, float* out);

/* ---- tracing ---------------------------------------------------------- */
/* The reference accumulates a GEMM / AWA / host-loop time split per chunk
 * (g_lin_time / g_awa_time, src/dit_vk.cpp:23-24, 688-697).  This runs the
 * 32-layer forward_latent with CUDA events around every kernel on the launch
 * stream and returns, per kernel class (0 tcgen05 GEMM, 1 fp32 GEMM,
 * 2 attention, 3 qk-norm/RoPE pack, 4 norm/convert, 5 other, 6 multi-GPU
 * exchange: always 0 here), the summed device milliseconds, algorithmic FLOPs
 * and bytes, and launch counts (arrays of 7). */
int s2b_forward_profile(s2b_ctx* ctx, const float* vid_patch, int Lv, const float* txt, int TXT, float timestep,
                        double* ms, double* flops, double* bytes, int* launches);

/* ---- GEMM engine ----------------------------------------------------- */
/* One Linear y = x W^T (+ bias) on the context's GEMM engine (the ncnn
 * InnerProduct that DitVk::lin runs, src/dit_vk.cpp:270-293): bf16 contexts
 * round x and W to bf16 and run the tcgen05 kernel (fp32 accumulate); fp32
 * contexts run the fp32 kernel.  x (M,K), W (N,K), bias (N) or NULL, y (M,N),
 * fp32 host buffers. */
int s2b_linear(s2b_ctx* ctx, const float* x, int M, int K, const float* W, int N, const float* bias, float* y);
/* The same Linear on device buffers, the form the engine's GEMMs take inside
 * the forward (DitVk::lin, src/dit_vk.cpp:270-293, with x and W already
 * resident): x (M,K) and W (N,K) bf16 row-major, bias (N) fp32 or NULL,
 * y (M,N) bf16, fp32 accumulation on the tcgen05 tensor cores, enqueued on
 * `stream` (a cudaStream_t; NULL = legacy default stream) without
 * synchronising.  K % 64 == 0, N % 32 == 0, 16-byte aligned buffers; else
 * S2B_ERR_ARG.  Works in contexts of either precision. */
int s2b_linear_bf16_dev(s2b_ctx* ctx, const void* d_x, int M, int K, const void* d_w, int N, const float* d_bias,
                        void* d_y, void* stream);

/* ---- synthetic data (no checkpoint ships with this build) ------------- */
/* Writes the m5 directory layout for layers [layer_lo, layer_hi) with
 * seeded random-init weights (Linear N(0,0.02) stored fp16; biases and
 * shifts N(0,0.02); norm weights, scales, gates 1+N(0,0.02)). */
int s2b_synth_write_m5(const char* dir, uint64_t seed, int layer_lo, int layer_hi);
/* Seeded inputs: vid_grid (T,H,W,33) = [noise N(0,1) x16 | condition N(0,1)
 * x16 | mask 1], txt (TXT,5120) N(0,1); fp32 normals of a named stream. */
int s2b_synth_vid_grid(float* vid_grid, int T, int H, int W, uint64_t seed);
int s2b_synth_txt(float* txt, int TXT, uint64_t seed);
int s2b_synth_normal(float* out, long n, uint64_t seed, const char* stream, float mean, float stdv);

/* ---- multi-GPU ------------------------------------------------------- */
/* Frame-sequence mode from one process: one context per GPU (devices, or
 * 0..ngpu-1 when null), each holding the whole model; frame k of a batch
 * runs on member k mod ngpu, each member on its own host thread, with no
 * communication (the engine's frame loop, src/main.cpp:126-147, dealt out;
 * no counterpart in the reference, which runs one device). */
typedef struct s2b_group s2b_group;
int s2b_group_create(int ngpu, const int* devices, int precision, s2b_group** out);
int s2b_group_destroy(s2b_group* group);
const char* s2b_group_last_error(const s2b_group* group);
int s2b_group_load_weights_dir(s2b_group* group, const char* m5_dir);
int s2b_group_load_weights_synth(s2b_group* group, uint64_t seed);
int s2b_group_set_windows(s2b_group* group, const s2b_win* ns, const s2b_win* sh);
/* vid_patches: nframes x (Lv, 132); txt (TXT, 5120) shared by the frames;
 * sr_out: nframes x (Lv, 64). */
int s2b_group_forward_frames(s2b_group* group, const float* vid_patches, int nframes, int Lv, const float* txt,
                             int TXT, float timestep, float* sr_out);

/* Window-sharded image mode: one rank per GPU; each rank owns a subset of
 * the windows of every layer, txt rows are replicated, and per layer the txt
 * partial sums of the attention and the residual rows that change owner are
 * exchanged over NVLink peer memory by this library's kernels (NCCL calls
 * when peers cannot map each other's memory, or S2B_SHARD_P2P=0).
 * `nccl_id` is the 128-byte ncclUniqueId created by rank 0 and shared over
 * any host channel.  Every rank calls every shard entry point in the same
 * order.  Peer waits are bounded by S2B_SHARD_WAIT_MS (default 4000): a rank
 * that waits longer, or that sees a peer running a later call, returns
 * S2B_ERR_TIMEOUT; on the NCCL path a host watchdog aborts the communicator
 * after the same bound (then s2b_shard_init must run again).  After a failed
 * shard call on ANY rank, every rank calls s2b_shard_resync before the next
 * forward. */
int s2b_nccl_unique_id(uint8_t nccl_id[128]);
int s2b_shard_init(s2b_ctx* ctx, const uint8_t nccl_id[128], int world, int rank);
int s2b_shard_forward(s2b_ctx* ctx, const float* vid_patch, int Lv, const float* txt, int TXT,
                      float timestep, float* sr_out);
/* s2b_shard_forward on device buffers, ordered on `stream` (cudaStream_t);
 * every rank passes the whole vid_patch / txt and receives the whole sr. */
int s2b_shard_forward_dev(s2b_ctx* ctx, const float* d_vid_patch, int Lv, const float* d_txt, int TXT,
                          float timestep, float* d_sr, void* stream);
/* Collective over the ranks of s2b_shard_init: agree on the number of the
 * next shard forward (the highest any rank has used), so that the flag values
 * of the peer exchanges match again after a call failed on some rank.  No
 * reference counterpart (the reference is single-device). */
int s2b_shard_resync(s2b_ctx* ctx);
/* The ownership and exchange plan rank `rank` of `world` uses (host only, no
 * context).  Parity p = 0 is the non-shifted windows (even layers), p = 1 the
 * shifted ones (odd layers).  Outputs (any may be null):
 *   bounds[p*(world+1) + r]: first window of rank r (last entry = nwin);
 *   n_local[p]: this rank's residual rows; tokens[p*Lv + j]: grid token of
 *   local row j;
 *   after a layer of parity p this rank sends its local rows
 *   send_idx[p*Lv + send_off[p*(world+1)+q] ..] to rank q and stores rank q's
 *   rows at its new local rows recv_idx[p*Lv + recv_off[p*(world+1)+q] ..],
 *   in ascending grid-token order per pair.
 * No reference counterpart (the reference runs a frame on one device,
 * src/dit_vk.cpp:481-676). */
/* s2b_forward_profile over this rank's part of s2b_shard_forward (arrays of
 * 7; class 6 is the exchanges: the cross-rank txt combine, the residual row
 * exchange and the output assembly, including time spent waiting for peers). */
int s2b_shard_forward_profile(s2b_ctx* ctx, const float* vid_patch, int Lv, const float* txt, int TXT,
                              float timestep, double* ms, double* flops, double* bytes, int* launches);
int s2b_shard_plan(const s2b_win* ns, const s2b_win* sh, int world, int rank, int* bounds, int* n_local,
                   int* tokens, int* send_off, int* send_idx, int* recv_off, int* recv_idx);

/* Status of the "_dev" calls enqueued so far: waits for the context's own
 * stream, then returns S2B_ERR_TIMEOUT (and clears the status) if a bounded
 * wait expired in any of them since the last report, else S2B_OK.  Calls that
 * run on the caller's stream (s2b_awa_forward_dev, s2b_awa_forward_dev_static,
 * s2b_linear_bf16_dev) must be complete first (synchronise that stream).  The
 * reference reports failures of its GPU work through the return value of each
 * synchronous call (src/awa_vk.cpp:182, src/dit_vk.cpp:27-45); this is the
 * same report for the stream-ordered form. */
int s2b_check_errors(s2b_ctx* ctx);

/* Test hooks (no reference counterpart).  s2b_debug_raise_kernel_error raises
 * the device flags an expired wait raises (mask: 1 GEMM, 2 attention, 4 peer
 * exchange) from a one-thread kernel; the next call on the device reports
 * S2B_ERR_TIMEOUT.  s2b_debug_watchdog_selftest runs the NCCL-path watchdog
 * against simulated work on the host only (scenario 0: finishes after a few
 * polls; 1: never finishes; 2: the communicator reports an asynchronous error;
 * 3: the stream fails), with `timeout_ms`; it returns the watchdog's result
 * (0 done, 1 async error, 2 expired, 3 stream error) and reports the polls
 * made and whether the communicator would have been aborted. */
int s2b_debug_raise_kernel_error(s2b_ctx* ctx, int mask);
int s2b_debug_watchdog_selftest(int scenario, int timeout_ms, int* polls, int* aborted);

#ifdef __cplusplus
}
#endif
#endif /* SEEDVR2_B200_H */
