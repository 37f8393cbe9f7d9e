// dit_b200.h -- B200 NaDiT DiT host engine (the DitVk / AwaVk / AwaLayer /
// AdaComposeLayer method set of the reference, src/dit_vk.h:24-204,
// src/awa_vk.h:14-52, backed by sm_100a kernels with weights resident in HBM).
#pragma once
#include "s2b_common.h"
#include "awa_geometry.h"
#include "kernels.h"
#include "shard_plan.h"
#include "watchdog.h"
#include <cuda_runtime.h>
#include <string>
#include <vector>
#include <memory>
#include <map>
#include <utility>

namespace s2b {

// m5 weight files held in memory: file name -> (bytes, size).
using WeightFiles = std::map<std::string, std::pair<const void*, size_t>>;

// Owning device allocation (move-only).
struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() {}
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        if (this != &o) { release(); p = o.p; bytes = o.bytes; o.p = nullptr; o.bytes = 0; }
        return *this;
    }
    ~DevBuf() { release(); }
    void release() { if (p) cudaFree(p); p = nullptr; bytes = 0; }
    cudaError_t ensure(size_t n) {
        if (n <= bytes) return cudaSuccess;
        if (p) { cudaFree(p); p = nullptr; bytes = 0; }
        cudaError_t e = cudaMalloc(&p, n);
        if (e == cudaSuccess) bytes = n;
        return e;
    }
    template <typename T> T* as() const { return (T*)p; }
};

// Device copy of one window geometry (see AwaDev in kernels.h).
struct GeomDev {
    WinGeom host;
    WinTables tab;
    DevBuf vidx, cumf, cums, row_win, vcos, vsin, tcos, tsin, tokpos, cs;
    AwaDev view;
    bool ready = false;
    bool structured = false;    // RoPE angles follow make_win (fused QKV epilogue allowed)
    std::vector<int> tokpos_host;   // host copy of tokpos (int4 per row)
    int npos = 0;                   // rows of the cs table
};

struct Linear {
    DevBuf w;          // [out][ld] in `t`
    DevBuf w2;         // fp32 contexts: [out][2*in] = [tf32 hi | lo] halves for the tensor-core fp32 GEMM
    DevBuf b;          // [out] fp32 or empty
    ActT t = ACT_F32;
    int out = 0, in = 0, ld = 0;
    const float* bias() const { return b.bytes ? b.as<const float>() : nullptr; }
};

struct Block {
    Linear qkv, out, mlp_hg, mlp_out;   // mlp_hg: proj_in | proj_in_gate interleaved in 128-row blocks
    bool loaded = false;
};

// Buffers and geometry one block runs on: the context's own (single GPU) or a
// window shard's local ones (dit_shard.cpp).
struct LayerBufs {
    float* X = nullptr;
    void *Xn = nullptr, *QKV = nullptr, *ATT = nullptr, *Hs = nullptr;
    void *Qp = nullptr, *Kp = nullptr, *Vp = nullptr;
    float* TOUTW = nullptr;
    GeomDev* geom[2] = {nullptr, nullptr};
    // sharded only: where this rank's txt partial sum of layer i goes, and the
    // step that combines all ranks' partials into the mean over all windows
    // (written to att_txt)
    float* (*txt_partial)(void* ctx, int layer) = nullptr;
    int (*txt_finish)(void* ctx, int layer, void* att_txt, cudaStream_t s) = nullptr;
    void* shard_ctx = nullptr;
    // RMSNorm + adaLN folded into the neighbouring GEMMs (bf16 contexts): the
    // gate/residual epilogue before a norm writes Xn = resid * scale and per-row
    // partial sums of squares (SQ, [rows][SQ_SLOTS]); the GEMM after it applies
    // the row factor and the shift (as a bias through its weights).
    float* SQ = nullptr;
    bool fuse_attn_in = false;    // this layer's attention-norm operand came from the previous layer
    bool fuse_attn_out = false;   // this layer's last GEMM writes the next layer's attention-norm operand
    bool fuse_mlp = false;        // the out-projection writes the MLP-norm operand
};

// 256-wide sinusoidal timestep features (src/dit_vk.cpp:295-302).
void sinusoidal256(float t, float* e);

// Kernel classes of the per-kernel profile (s2b_forward_profile).
enum KernelKind { KK_GEMM_TC = 0, KK_GEMM_SIMT = 1, KK_ATTN = 2, KK_PACK = 3, KK_NORM = 4, KK_OTHER = 5,
                  KK_EXCHANGE = 6, KK_COUNT = 7 };

class DitB200 {
public:
    DitB200() {}
    ~DitB200();
    int create(int device, int precision);
    int load_weights(const char* m5_dir, bool synth, uint64_t seed, int layer_lo, int layer_hi);
    // The same from the m5 directory's files supplied in memory (not thread-safe
    // against a concurrent load in another context).
    int load_weights_mem(const WeightFiles& files, int layer_lo, int layer_hi);
    int set_windows(const WinGeom& ns, const WinGeom& sh);

    // DitVk::forward_latent (host buffers)
    int forward_latent(const float* vid_in, int Lv, const float* txt_in, int TXT, float t, int l0, int l1,
                       bool do_init, bool do_final, float* vid_lat, float* txt_lat, float* sr_out);
    // DitVk::forward / forward_graph: all 32 layers, CUDA-graph replay.
    int forward(const float* vid_patch, int Lv, const float* txt, int TXT, float t, float* sr_out);
    int forward_dev(const float* d_vid_patch, int Lv, const float* d_txt, int TXT, float t, float* d_sr,
                    cudaStream_t user);
    // DitVk::forward_grid on device buffers: patchify, the captured forward and
    // unpatchify, all on the caller's stream.
    int forward_grid_dev(const float* d_grid, int T, int H, int W, const float* d_txt, int TXT, float t,
                         float* d_sr_grid, cudaStream_t user);
    int time_embedding(float t, float* emb_host);
    // forward_latent(0, 32, init, final) with CUDA events around every kernel:
    // per KernelKind the summed device ms, algorithmic FLOPs / bytes, launches.
    // sharded: profile this rank's part of shard_forward instead.
    int forward_profile(const float* vid_patch, int Lv, const float* txt, int TXT, float t, double* ms,
                        double* flops, double* bytes, int* count, bool sharded = false);
    // One Linear on the context's GEMM engine (host buffers).
    int linear(const float* x, int M, int K, const float* W, int N, const float* bias, float* y);
    // y = x W^T (+ bias) on device bf16 buffers, bf16 out, on stream s (any precision context)
    int linear_bf16_dev(const void* x, int M, int K, const void* W, int N, const float* bias, void* y, cudaStream_t s);
    int ada_compose(const float* emb_host, float* out_host);
    // AwaVk::forward (host) / AwaLayer::forward (device, stored geometry)
    int awa_forward(const float* vqkv, const float* tqkv, const WinGeom& win, const float* nqv, const float* nkv,
                    const float* nqt, const float* nkt, int Lv, int TXT, float eps, float* vid_out, float* txt_out);
    int awa_set_geometry(int win_type, const WinGeom& win);
    int awa_forward_dev(int win_type, const float* vqkv, const float* tqkv, const float* nqv, const float* nkv,
                        const float* nqt, const float* nkt, int Lv, int TXT, float eps, float* vid_out,
                        float* txt_out, cudaStream_t user);

    // awa_forward_dev with its scratch in the library's fixed device array
    // (k_awa_static.cu): no device allocation, enqueue only.
    int awa_forward_dev_static(int win_type, const float* vqkv, const float* tqkv, const float* nqv,
                               const float* nkv, const float* nqt, const float* nkt, int Lv, int TXT, float eps,
                               float* vid_out, float* txt_out, cudaStream_t user);

    // Status of the stream-ordered (*_dev) calls: synchronises the context's
    // stream, then reports (and clears) the kernel error bits that the
    // forwards folded into the context's status word since the last report.
    int check_errors();
    // Test hook: raises the kernel error flags named by mask (KernelErrBit)
    // on the device, as an expired bounded wait would.
    int debug_raise_kernel_error(int mask);

    // Last layer (31) txt semantics: false = forward_latent's vid_only (the
    // default, the oracle's), true = the chunked graph's (txt modulated, gated
    // and through its MLP as in every other layer).  Recaptures the graphs.
    int set_graph_last_layer(bool on);

    int precision() const { return prec_; }
    uint64_t device_bytes() const;
    int last_launches() const { return last_launches_; }
    std::string err;

    // Multi-GPU window sharding (dit_shard.cpp).
    int shard_init(const uint8_t id[128], int world, int rank);
    int shard_forward(const float* vid_patch, int Lv, const float* txt, int TXT, float t, float* sr_out);
    int shard_forward_dev(const float* d_vid_patch, int Lv, const float* d_txt, int TXT, float t, float* d_sr,
                          cudaStream_t user);
    // Collective (every rank calls it): agree on the shard-forward call number
    // after a failed call on any rank, so the ranks' flag values match again.
    int shard_resync();

private:
    int fail(int code, const std::string& m) { err = m; return code; }
    // Enqueue the fold of the device's kernel error flags into status_ (after
    // the kernels it covers, on the same stream).
    void fold_status(cudaStream_t s) { status_fold(kflags_, status_.as<int>(), s); launches_++; }
    // With s idle: read and clear status_; ERR_TIMEOUT naming the kernel
    // classes whose bounded waits expired, else OK.
    int take_status(cudaStream_t s, const char* what);
    int cuda_check(cudaError_t e, const char* what);
    int sync_check(cudaStream_t s, const char* what);
    int upload_linear(Linear& L, const void* w_src, bool src_f16, const float* bias, int out, int in, ActT t,
                      int ld, int interleave_role);
    int ensure_acts(int Lv, int TXT);
    int capture_full(int Lv, int TXT);
    int awa_run(GeomDev& G, const float* vqkv, const float* tqkv, const float* nqv, const float* nkv,
                const float* nqt, const float* nkt, int Lv, int TXT, float eps, float* vid_out, float* txt_out,
                cudaStream_t user);
    int upload_geom(GeomDev& g, const WinGeom& w, int TXT_expected);
    int upload_geom_with(GeomDev& g, const WinGeom& w, const WinTables& tab, const std::vector<int>& tokpos4,
                         bool structured, int npos, int Lv);
    void gemm(const void* A, int lda, const Linear& L, int M, const GemmEpi& e, cudaStream_t s);
    void gemm2(const void* A0, int lda0, const Linear& L0, int M0, const GemmEpi& e0, const void* A1, int lda1,
               const Linear& L1, int M1, const GemmEpi& e1, cudaStream_t s);
    // Enqueue the pieces of forward_latent on stream s (device inputs already staged).
    int enqueue_init(int Lv, int TXT, cudaStream_t s);
    int enqueue_temb(cudaStream_t s);
    int enqueue_layer(int i, int Lv, int TXT, cudaStream_t s, int l0, int l1);
    // the shift biases of the folded norms for timestep t (recomputed only when t changes)
    int prepare_shift(float t, cudaStream_t s);
    // layer j's attention norm can take its operand from layer j - 1 (txt is
    // modulated there and the QKV GEMM runs the fused pack epilogue)
    bool attn_norm_foldable(int j) const;
    int enqueue_layer_on(int i, int Lv, int TXT, cudaStream_t s, const LayerBufs& B);
    LayerBufs default_bufs();
    int enqueue_final(int Lv, cudaStream_t s);
    int shard_prepare(int Lv, int TXT);
    int shard_enqueue(cudaStream_t s);
    int shard_exchange(int p, cudaStream_t s);
    int shard_capture();
    int shard_begin_call();
    void shard_invalidate_graph();
    int shard_wait(const char* what, bool nccl_in_flight);
    int shard_setup_peers(const ShardPlan& plan, int n0, int n1, int TXT);
    cudaStream_t capture_stream() const { return stream_; }
    const float* ada(int layer, int flow, int k) const {
        return ada_.as<float>() + ((size_t)(layer * 12 + flow * 6 + k)) * DIM;
    }
    const float* shift_qkv(int layer, int flow) const {
        return shift_.as<float>() + ((size_t)(layer * 2 + flow)) * (QKV + 2 * MLP_DIM);
    }
    const float* shift_hg(int layer, int flow) const { return shift_qkv(layer, flow) + QKV; }
    const float* normw(int layer, int flow, int which) const {
        return qknorm_.as<float>() + ((size_t)((layer * 2 + flow) * 2 + which)) * HEAD_D;
    }

    int dev_ = -1, prec_ = PREC_FP32;
    // folded norms (bf16, S2B_NORM_FUSE=1; off by default, see load_weights)
    bool norm_fuse_ = false;
    DevBuf shift_;          // [32][2 flows][qkv 7680 | hg 13824] shift biases (W . adaLN shift)
    DevBuf SQ_;             // [rows][SQ_SLOTS] partial sums of squares
    bool shift_ok_ = false;
    float shift_t_ = 0.f;
    DevBuf status_;         // int: KernelErrBit of every expired wait not yet reported
    KernelFlags kflags_;    // this device's kernel error flags
    ActT act_ = ACT_F32;
    cudaStream_t stream_ = nullptr;
    bool weights_ = false;
    int layer_lo_ = 0, layer_hi_ = 0;
    bool graph_last_ = false;

    Linear vid_in_, txt_in_, emb_in_, emb_hid_, emb_out_, vid_out_;
    Block blk_[NUM_LAYERS][2];
    DevBuf branch_;     // [32*12+2][2560] branch vectors in AdaCompose output order
    DevBuf qknorm_;     // [32][2 flows][2 (q,k)][128]
    DevBuf von_w_;      // [2560] final norm affine
    DevBuf ada_;        // [32*12+2][2560] composed modulation vectors
    DevBuf emb_;        // [15360]
    DevBuf temb_in_, temb_h1_, temb_h2_;   // [256], [2560], [2560]

    GeomDev geom_[2];   // non-shifted (even layers), shifted (odd layers)
    int geom_gen_ = 0;  // bumped by set_windows (shard plans follow it)
    GeomDev awa_geom_[2];

    // activations
    int cap_Lv_ = 0, cap_TXT_ = 0;
    DevBuf X_, Xn_, QKV_, ATT_, Qp_, Kp_, Vp_, TOUTW_, HG_, Hs_, VPIN_, TIN_, SR_, VIDIN_F_, TXTIN_F_;
    DevBuf A2_;         // fp32 contexts: [M][2K] split activations of the tensor-core fp32 GEMM
    bool tf32x3_ = false;
    int prepare_tf32x3();
    // fp32 contexts: attention on the tensor cores from split3 operands
    // (awa_pack_split3 / awa_attend_split3) unless S2B_FP32_ATTN=simt
    bool attn_split3_ = false;
    // bytes per element of the packed Q/K/V buffers (three bf16 parts under split3)
    size_t attn_elem_bytes() const { return attn_split3_ ? 6 : act_bytes(act_); }
    size_t qkv_pack_rows_ = 0;

    // captured full forward
    cudaGraphExec_t gexec_ = nullptr;
    int graph_Lv_ = -1, graph_TXT_ = -1;
    int graph_launches_ = 0;
    int last_launches_ = 0;
    int launches_ = 0;

    // per-kernel CUDA-event profile
    struct ProfMark { int kind; double flops, bytes; cudaEvent_t a, b; };
    bool prof_on_ = false;
    std::vector<ProfMark> marks_;
    std::vector<cudaEvent_t> ev_pool_;
    void pbeg(int kind, double flops, double bytes, cudaStream_t s);
    void pend(cudaStream_t s);

public:
    struct ShardState;
    std::unique_ptr<ShardState> shard_;
};

}  // namespace s2b
