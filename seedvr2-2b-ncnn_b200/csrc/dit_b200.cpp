// dit_b200.cpp -- B200 NaDiT DiT host engine (see dit_b200.h).
//
// One forward is the reference's DitVk::forward_latent (src/dit_vk.cpp:486-699)
// laid out for the GPU:
//   * one fp32 residual buffer X of (Lv + TXT) rows: vid rows first, txt rows
//     after, so layers 10..31 (vid/txt share weights, src/dit_vk.cpp:163-164)
//     run each Linear as ONE GEMM over both streams, and layers 0..9 run two;
//   * every Linear's operands in the context precision (fp32 or bf16), fp32
//     accumulation, and the adaLN gate + residual add fused in the GEMM
//     epilogue; proj_in / proj_in_gate are one GEMM over interleaved weights;
//   * AWA = pack (qk-norm + RoPE into window-packed Q/K/V) -> attention ->
//     txt coalesce;
//   * the 32*12+2 modulation vectors are composed once per timestep
//     (AdaComposeLayer semantics, src/ada_compose.cpp:166-235);
//   * s2b_forward replays the whole forward from one captured CUDA graph.
#include "dit_b200.h"
#include "dit_shard.h"
#include "synth.h"
#include <cmath>
#include <cstdint>
#include <initializer_list>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>

namespace s2b {

DitB200::~DitB200() {
    if (dev_ >= 0) cudaSetDevice(dev_);
    for (cudaEvent_t e : ev_pool_) cudaEventDestroy(e);
    shard_.reset();
    if (gexec_) cudaGraphExecDestroy(gexec_);
    if (stream_) cudaStreamDestroy(stream_);
}

int DitB200::cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return OK;
    err = std::string(what) + ": " + cudaGetErrorString(e);
    return e == cudaErrorMemoryAllocation ? ERR_NOMEM : ERR_CUDA;
}

// Status of everything enqueued on s: a launch-time error of an async call
// (reported once, by cudaGetLastError) or an execution error (by the sync).
int DitB200::sync_check(cudaStream_t s, const char* what) {
    const cudaError_t launch = cudaGetLastError();
    const cudaError_t exec = cudaStreamSynchronize(s);
    return cuda_check(launch != cudaSuccess ? launch : exec, what);
}

int DitB200::create(int device, int precision) {
    if (precision != PREC_FP32 && precision != PREC_FP16 && precision != PREC_BF16)
        return fail(ERR_ARG, "precision must be 0 (fp32), 1 (fp16) or 2 (bf16)");
    int n = 0;
    if (int rc = cuda_check(cudaGetDeviceCount(&n), "cudaGetDeviceCount")) return rc;
    if (device < 0 || device >= n) return fail(ERR_ARG, "device index out of range");
    dev_ = device;
    if (int rc = cuda_check(cudaSetDevice(dev_), "cudaSetDevice")) return rc;
    cudaDeviceProp prop;
    if (int rc = cuda_check(cudaGetDeviceProperties(&prop, dev_), "cudaGetDeviceProperties")) return rc;
    if (prop.major != 10) return fail(ERR_UNSUPPORTED, std::string("sm_100a kernels need a B200-class GPU, found ") + prop.name);
    prec_ = precision;
    act_ = precision == PREC_BF16 ? ACT_BF16 : precision == PREC_FP16 ? ACT_F16 : ACT_F32;
    // fp32 attention on the tensor cores (split3 operands) unless S2B_FP32_ATTN=simt
    const char* aenv = std::getenv("S2B_FP32_ATTN");
    attn_split3_ = act_ == ACT_F32 && !(aenv && aenv[0] == 's');
    if (int rc = cuda_check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate")) return rc;
    if (kernels_init_device() != 0) return fail(ERR_CUDA, "kernel attribute setup failed");
    if (int rc = cuda_check((cudaError_t)kernel_flags_get(&kflags_), "kernel error flags")) return rc;
    if (int rc = cuda_check(status_.ensure(16), "cudaMalloc(status)")) return rc;
    return cuda_check(cudaMemset(status_.p, 0, 16), "status init");
}

int DitB200::take_status(cudaStream_t s, const char* what) {
    int st = 0;
    cudaError_t e = cudaMemcpyAsync(&st, status_.p, sizeof st, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && st) {
        e = cudaMemsetAsync(status_.p, 0, sizeof st, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    if (int rc = cuda_check(e, "kernel status read")) return rc;
    if (!st) return OK;
    std::string m = std::string(what) + ": a bounded wait expired in";
    if (st & KERR_GEMM) m += " the tcgen05 GEMM";
    if (st & KERR_ATTN) m += (st & KERR_GEMM) ? ", the tcgen05 attention" : " the tcgen05 attention";
    if (st & KERR_SHARD) m += (st & (KERR_GEMM | KERR_ATTN)) ? ", a peer-memory exchange" : " a peer-memory exchange";
    return fail(ERR_TIMEOUT, m + "; the output of that call is incomplete");
}

int DitB200::check_errors() {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    cudaSetDevice(dev_);
    if (int rc = shard_wait("check_errors", shard_ != nullptr)) return rc;
    return take_status(stream_, "an earlier stream-ordered call");
}

int DitB200::set_graph_last_layer(bool on) {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    if (graph_last_ == on) return OK;
    graph_last_ = on;
    cudaSetDevice(dev_);
    if (gexec_) { cudaGraphExecDestroy(gexec_); gexec_ = nullptr; graph_Lv_ = -1; }
    shard_invalidate_graph();
    return OK;
}

int DitB200::debug_raise_kernel_error(int mask) {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    if (mask & ~(KERR_GEMM | KERR_ATTN | KERR_SHARD)) return fail(ERR_ARG, "mask must combine 1 (GEMM), 2 (attention), 4 (exchange)");
    cudaSetDevice(dev_);
    status_raise(kflags_, mask, stream_);
    return sync_check(stream_, "debug_raise_kernel_error");
}

uint64_t DitB200::device_bytes() const {
    uint64_t t = 0;
    auto lin = [&](const Linear& L) { t += L.w.bytes + L.b.bytes; };
    lin(vid_in_); lin(txt_in_); lin(emb_in_); lin(emb_hid_); lin(emb_out_); lin(vid_out_);
    for (int i = 0; i < NUM_LAYERS; i++)
        for (int f = 0; f < (i < MM_LAYERS ? 2 : 1); f++) {
            const Block& B = blk_[i][f];
            lin(B.qkv); lin(B.out); lin(B.mlp_hg); lin(B.mlp_out);
        }
    for (const DevBuf* b : {&branch_, &qknorm_, &von_w_, &ada_, &emb_, &X_, &Xn_, &QKV_, &ATT_, &Qp_, &Kp_, &Vp_,
                            &TOUTW_, &HG_, &Hs_, &VPIN_, &TIN_, &SR_, &VIDIN_F_, &TXTIN_F_})
        t += b->bytes;
    return t;
}

// ------------------------------------------------------------------ weights
int DitB200::upload_linear(Linear& L, const void* w_src, bool src_f16, const float* bias, int out, int in, ActT t,
                           int ld, int interleave_role) {
    // interleave_role: -1 plain; 0 / 1: proj_in / proj_in_gate into the [h|g]
    // 128-row block layout of mlp_hg (destination already sized 2*out rows).
    DevBuf stage;
    const size_t src_bytes = (size_t)out * in * (src_f16 ? 2 : 4);
    if (int rc = cuda_check(stage.ensure(src_bytes), "cudaMalloc(weight staging)")) return rc;
    if (int rc = cuda_check(cudaMemcpy(stage.p, w_src, src_bytes, cudaMemcpyHostToDevice), "upload weight")) return rc;
    if (interleave_role < 0) {
        L.t = t; L.out = out; L.in = in; L.ld = ld;
        if (int rc = cuda_check(L.w.ensure((size_t)out * ld * act_bytes(t)), "cudaMalloc(weight)")) return rc;
        ingest_weight(stage.p, src_f16, out, in, L.w.p, t, ld, 0, 0, 0, stream_);
    } else {
        if (!L.w.p) {
            L.t = t; L.out = 2 * out; L.in = in; L.ld = ld;
            if (int rc = cuda_check(L.w.ensure((size_t)2 * out * ld * act_bytes(t)), "cudaMalloc(weight)")) return rc;
        }
        ingest_weight(stage.p, src_f16, out, in, L.w.p, t, ld, 128, 256, interleave_role * 128, stream_);
    }
    if (bias) {
        if (int rc = cuda_check(L.b.ensure((size_t)out * 4), "cudaMalloc(bias)")) return rc;
        if (int rc = cuda_check(cudaMemcpy(L.b.p, bias, (size_t)out * 4, cudaMemcpyHostToDevice), "upload bias")) return rc;
    }
    return sync_check(stream_, "weight ingest");
}

namespace {
// Weights as stored: fp16 bits (ncnn tag 0x01306B47) or fp32 (tag 0).
struct HostLinear {
    int out = 0, in = 0; bool has_bias = false; bool f16 = true;
    std::vector<uint16_t> w; std::vector<float> wf; std::vector<float> b;
    const void* data() const { return f16 ? (const void*)w.data() : (const void*)wf.data(); }
};

// Files of the m5 layout come from a directory or, when `mem` is set, from
// an in-memory table keyed by file name.
const WeightFiles* g_mem_files = nullptr;   // set for the duration of one load (context-local call)

bool read_file(const std::string& p, std::vector<unsigned char>& out) {
    if (g_mem_files) {
        const size_t slash = p.find_last_of('/');
        const std::string name = slash == std::string::npos ? p : p.substr(slash + 1);
        auto it = g_mem_files->find(name);
        if (it == g_mem_files->end()) return false;
        out.assign((const unsigned char*)it->second.first, (const unsigned char*)it->second.first + it->second.second);
        return true;
    }
    std::ifstream f(p, std::ios::binary);
    if (!f) return false;
    f.seekg(0, std::ios::end);
    out.resize((size_t)f.tellg());
    f.seekg(0);
    f.read((char*)out.data(), (std::streamsize)out.size());
    return (bool)f;
}

// ncnn InnerProduct .param/.bin pair (format: src/verify_dit.cpp:62-104).
bool load_host_linear(const std::string& dir, const std::string& base, HostLinear& L, std::string& err) {
    std::vector<unsigned char> ptxt;
    if (!read_file(dir + base + ".param", ptxt)) { err = "missing " + dir + base + ".param"; return false; }
    std::istringstream pf(std::string(ptxt.begin(), ptxt.end()));
    std::string line;
    int nout = 0, bias = 0, wsz = 0;
    while (std::getline(pf, line)) {
        if (line.find("InnerProduct") == std::string::npos) continue;
        std::istringstream ss(line);
        std::string tok;
        while (ss >> tok) {
            if (tok.rfind("0=", 0) == 0) nout = std::atoi(tok.c_str() + 2);
            else if (tok.rfind("1=", 0) == 0) bias = std::atoi(tok.c_str() + 2);
            else if (tok.rfind("2=", 0) == 0) wsz = std::atoi(tok.c_str() + 2);
        }
    }
    if (nout <= 0 || wsz <= 0 || wsz % nout) { err = "bad InnerProduct param in " + base; return false; }
    std::vector<unsigned char> blob;
    if (!read_file(dir + base + ".bin", blob)) { err = "missing " + dir + base + ".bin"; return false; }
    L.out = nout; L.in = wsz / nout; L.has_bias = bias != 0;
    if (blob.size() < 4) { err = "short " + base + ".bin"; return false; }
    uint32_t tag; std::memcpy(&tag, blob.data(), 4);
    size_t off = 4;
    if (tag == 0x01306B47u) {
        if (blob.size() < off + 2 * (size_t)wsz) { err = "short " + base + ".bin"; return false; }
        L.f16 = true;
        L.w.resize((size_t)wsz);
        std::memcpy(L.w.data(), blob.data() + off, 2 * (size_t)wsz);
        off += 2 * (size_t)wsz;
    } else if (tag == 0u) {
        if (blob.size() < off + 4 * (size_t)wsz) { err = "short " + base + ".bin"; return false; }
        L.f16 = false;
        L.wf.resize((size_t)wsz);
        std::memcpy(L.wf.data(), blob.data() + off, 4 * (size_t)wsz);
        off += 4 * (size_t)wsz;
    } else { err = "unsupported weight tag in " + base; return false; }
    if (L.has_bias) {
        if (blob.size() < off + 4 * (size_t)nout) { err = "short bias in " + base; return false; }
        L.b.resize(nout);
        std::memcpy(L.b.data(), blob.data() + off, 4 * (size_t)nout);
    }
    return true;
}

bool load_host_vector(const std::string& dir, const std::string& base, std::vector<float>& v, std::string& err) {
    std::vector<unsigned char> blob;
    if (!read_file(dir + base + ".bin", blob) || blob.size() < 8) { err = "missing " + dir + base + ".bin"; return false; }
    int64_t nd; std::memcpy(&nd, blob.data(), 8);
    if (nd < 0 || nd > 8 || blob.size() < 8 + 8 * (size_t)nd) { err = "bad header " + base; return false; }
    int64_t total = 1;
    for (int64_t i = 0; i < nd; i++) { int64_t d; std::memcpy(&d, blob.data() + 8 + 8 * i, 8); total *= d; }
    const size_t off = 8 + 8 * (size_t)nd;
    if (total < 0 || blob.size() < off + 4 * (size_t)total) { err = "short " + base; return false; }
    v.resize((size_t)total);
    std::memcpy(v.data(), blob.data() + off, 4 * (size_t)total);
    return true;
}
}  // namespace

int DitB200::load_weights_mem(const WeightFiles& files, int lo, int hi) {
    g_mem_files = &files;
    const int rc = load_weights("mem/", false, 0, lo, hi);
    g_mem_files = nullptr;
    return rc;
}

int DitB200::load_weights(const char* dir_c, bool synth, uint64_t seed, int lo, int hi) {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    lo = std::max(0, lo); hi = std::min(NUM_LAYERS, hi);
    cudaSetDevice(dev_);
    std::string dir = dir_c ? dir_c : "";
    if (!synth && (dir.empty())) return fail(ERR_ARG, "empty model directory");
    if (!synth && dir.back() != '/') dir += '/';
    if (gexec_) { cudaGraphExecDestroy(gexec_); gexec_ = nullptr; graph_Lv_ = -1; }
    for (auto& row : blk_) for (auto& b : row) b = Block();

    auto get_lin = [&](const SynthLinear& S, HostLinear& H) -> bool {
        if (synth) {
            H.out = S.out; H.in = S.in; H.has_bias = S.has_bias;
            H.w.resize((size_t)S.out * S.in);
            H.b.resize(S.has_bias ? S.out : 0);
            synth_linear(S, seed, H.w.data(), S.has_bias ? H.b.data() : nullptr);
            return true;
        }
        if (!load_host_linear(dir, S.name, H, err)) return false;
        if (H.out != S.out || H.in != S.in) { err = "shape mismatch for " + S.name; return false; }
        return true;
    };
    const ActT wt = act_;
    for (const auto& S : model_linears(lo, hi)) {
        HostLinear H;
        if (!get_lin(S, H)) return ERR_IO;
        const float* b = H.has_bias ? H.b.data() : nullptr;
        int rc = OK;
        const std::string& n = S.name;
        if (n == "vid_in_proj") rc = upload_linear(vid_in_, H.data(), H.f16, b, H.out, H.in, wt, PATCH_IN_PAD, -1);
        else if (n == "txt_in") rc = upload_linear(txt_in_, H.data(), H.f16, b, H.out, H.in, wt, H.in, -1);
        else if (n == "emb_proj_in") rc = upload_linear(emb_in_, H.data(), H.f16, b, H.out, H.in, ACT_F32, H.in, -1);
        else if (n == "emb_proj_hid") rc = upload_linear(emb_hid_, H.data(), H.f16, b, H.out, H.in, ACT_F32, H.in, -1);
        else if (n == "emb_proj_out") rc = upload_linear(emb_out_, H.data(), H.f16, b, H.out, H.in, ACT_F32, H.in, -1);
        else if (n == "vid_out_proj") rc = upload_linear(vid_out_, H.data(), H.f16, b, H.out, H.in, wt, H.in, -1);
        else {
            // b{i}_{vid|txt|all}_{qkv,out,mlp_in,mlp_g,mlp_out}
            int i = 0; char tag[8] = {0}, what[16] = {0};
            if (std::sscanf(n.c_str(), "b%d_%3[a-z]_%15s", &i, tag, what) != 3) return fail(ERR_IO, "bad weight name " + n);
            const int fl = (std::strcmp(tag, "txt") == 0) ? 1 : 0;
            Block& B = blk_[i][fl];
            const std::string w = what;
            if (w == "qkv") rc = upload_linear(B.qkv, H.data(), H.f16, b, H.out, H.in, wt, H.in, -1);
            else if (w == "out") rc = upload_linear(B.out, H.data(), H.f16, b, H.out, H.in, wt, H.in, -1);
            else if (w == "mlp_in") rc = upload_linear(B.mlp_hg, H.data(), H.f16, b, H.out, H.in, wt, H.in, 0);
            else if (w == "mlp_g") rc = upload_linear(B.mlp_hg, H.data(), H.f16, b, H.out, H.in, wt, H.in, 1);
            else if (w == "mlp_out") { rc = upload_linear(B.mlp_out, H.data(), H.f16, b, H.out, H.in, wt, H.in, -1); B.loaded = true; }
            else return fail(ERR_IO, "bad weight name " + n);
        }
        if (rc) return rc;
    }
    // raw vectors
    std::vector<float> branch((size_t)(NUM_LAYERS * 12 + 2) * DIM), qkn((size_t)NUM_LAYERS * 2 * 2 * HEAD_D), von;
    auto get_vec = [&](const std::string& name, int n, float mean, std::vector<float>& v) -> bool {
        if (synth) { v.resize(n); synth_vector({name, n, mean}, seed, v.data()); return true; }
        if (!load_host_vector(dir, name, v, err)) return false;
        if ((int)v.size() != n) { err = "size mismatch for " + name; return false; }
        return true;
    };
    std::vector<float> v;
    if (!get_vec("vid_out_norm_w", DIM, 1.f, von)) return ERR_IO;
    if (!get_vec("vid_out_ada_scale", DIM, 1.f, v)) return ERR_IO;
    std::memcpy(&branch[(size_t)(NUM_LAYERS * 12) * DIM], v.data(), DIM * 4);
    if (!get_vec("vid_out_ada_shift", DIM, 0.f, v)) return ERR_IO;
    std::memcpy(&branch[(size_t)(NUM_LAYERS * 12 + 1) * DIM], v.data(), DIM * 4);
    static const char* bnames[6] = {"attn_scale", "attn_shift", "attn_gate", "mlp_scale", "mlp_shift", "mlp_gate"};
    static const float bmeans[6] = {1.f, 0.f, 1.f, 1.f, 0.f, 1.f};
    for (int i = 0; i < NUM_LAYERS; i++)
        for (int fl = 0; fl < 2; fl++) {
            const std::string base = "b" + std::to_string(i) + "_" + (i < MM_LAYERS ? (fl ? "txt" : "vid") : "all") + "_";
            for (int k = 0; k < 6; k++) {
                if (!get_vec(base + bnames[k], DIM, bmeans[k], v)) return ERR_IO;
                std::memcpy(&branch[((size_t)(i * 12 + fl * 6 + k)) * DIM], v.data(), DIM * 4);
            }
            if (!get_vec(base + "nq", HEAD_D, 1.f, v)) return ERR_IO;
            std::memcpy(&qkn[((size_t)((i * 2 + fl) * 2 + 0)) * HEAD_D], v.data(), HEAD_D * 4);
            if (!get_vec(base + "nk", HEAD_D, 1.f, v)) return ERR_IO;
            std::memcpy(&qkn[((size_t)((i * 2 + fl) * 2 + 1)) * HEAD_D], v.data(), HEAD_D * 4);
        }
    if (int rc = cuda_check(branch_.ensure(branch.size() * 4), "cudaMalloc")) return rc;
    if (int rc = cuda_check(qknorm_.ensure(qkn.size() * 4), "cudaMalloc")) return rc;
    if (int rc = cuda_check(von_w_.ensure(DIM * 4), "cudaMalloc")) return rc;
    if (int rc = cuda_check(ada_.ensure(branch.size() * 4), "cudaMalloc")) return rc;
    if (int rc = cuda_check(emb_.ensure(EMB_DIM * 4), "cudaMalloc")) return rc;
    if (int rc = cuda_check(temb_in_.ensure(TEMB_IN * 4), "cudaMalloc")) return rc;
    if (int rc = cuda_check(temb_h1_.ensure(DIM * 4), "cudaMalloc")) return rc;
    if (int rc = cuda_check(temb_h2_.ensure(DIM * 4), "cudaMalloc")) return rc;
    if (int rc = cuda_check(cudaMemcpy(branch_.p, branch.data(), branch.size() * 4, cudaMemcpyHostToDevice), "upload vectors")) return rc;
    if (int rc = cuda_check(cudaMemcpy(qknorm_.p, qkn.data(), qkn.size() * 4, cudaMemcpyHostToDevice), "upload vectors")) return rc;
    if (int rc = cuda_check(cudaMemcpy(von_w_.p, von.data(), DIM * 4, cudaMemcpyHostToDevice), "upload vectors")) return rc;
    // folded norms (S2B_NORM_FUSE=1): bf16 contexts whose shared layers
    // modulate vid and txt alike (one GEMM serves both flows there).  Off by
    // default: measured per 1080p forward, the extra work in the gate/residual
    // and consumer epilogues (+4-6 % per GEMM launch) costs what the 62
    // removed norm kernels saved (~1.1 ms), so the standalone kernels stay.
    {
        const char* fe = std::getenv("S2B_NORM_FUSE");
        bool same = true;
        for (int i = MM_LAYERS; i < NUM_LAYERS && same; i++)
            for (int k : {0, 1, 3, 4})
                same = same && std::memcmp(&branch[((size_t)(i * 12 + k)) * DIM], &branch[((size_t)(i * 12 + 6 + k)) * DIM],
                                           DIM * 4) == 0;
        norm_fuse_ = act_ == ACT_BF16 && same && fe && fe[0] == '1';
        shift_ok_ = false;
        if (norm_fuse_)
            if (int rc = cuda_check(shift_.ensure((size_t)NUM_LAYERS * 2 * (QKV + 2 * MLP_DIM) * 4), "cudaMalloc(shift)"))
                return rc;
    }
    // shared layers: the txt flow uses the same Linear objects
    layer_lo_ = lo; layer_hi_ = hi;
    weights_ = true;
    if (act_ == ACT_F32) return prepare_tf32x3();
    return OK;
}

// fp32 contexts: the [hi | lo] tf32 halves of every Linear the tensor-core
// fp32 GEMM serves (input width a multiple of 32), unless S2B_FP32_TC=0.
int DitB200::prepare_tf32x3() {
    const char* env = std::getenv("S2B_FP32_TC");
    tf32x3_ = !(env && env[0] == '0');
    if (!tf32x3_) return OK;
    auto split = [&](Linear& L) -> int {
        if (!L.w.bytes || L.t != ACT_F32 || L.in % 32) return OK;
        if (int rc = cuda_check(L.w2.ensure((size_t)L.out * 2 * L.in * 4), "cudaMalloc(tf32 weights)")) return rc;
        split_tf32(L.w.as<float>(), L.ld, L.out, L.in, L.w2.as<float>(), 2 * L.in, stream_);
        return OK;
    };
    if (int rc = split(txt_in_)) return rc;
    if (int rc = split(vid_out_)) return rc;
    for (auto& row : blk_)
        for (auto& B : row)
            for (Linear* L : {&B.qkv, &B.out, &B.mlp_hg, &B.mlp_out})
                if (int rc = split(*L)) return rc;
    return sync_check(stream_, "tf32 weight split");
}

// ------------------------------------------------------------------ geometry
static void rope_base(double base[21]) {   // src/awa_window.cpp:122-123
    for (int j = 0; j < 21; j++) base[j] = 1.0 / std::pow(10000.0, (double)(2 * j) / 42);
}

int DitB200::upload_geom(GeomDev& g, const WinGeom& w, int TXT_expected) {
    const char* why = nullptr;
    WinTables tab;
    if (!build_tables(w, tab, &why)) return fail(ERR_ARG, std::string("window geometry: ") + why);
    if (TXT_expected >= 0 && w.txt_len != TXT_expected) return fail(ERR_ARG, "window txt_len differs from TXT");
    const int nwin = w.nwin(), TXT = w.txt_len;
    // grid token -> (packed vid index, window, RoPE positions); gi = -1 for
    // tokens outside every window.  The fused QKV epilogue also needs the
    // angle tables to have the make_win structure (angle of pair i =
    // pos[i / 21] * base[i % 21], vid pos = (txt_len + t, local h, local w),
    // txt pos = (p, p, p)); that is checked bit for bit here, and geometries
    // that fail it keep the separate pack kernel.
    double base[21];
    rope_base(base);
    std::vector<int> tokpos(4 * (size_t)std::max(w.tokens(), 1), -1);
    bool structured = true;
    int npos = TXT + 1;
    for (int i = 0; i < nwin; i++) {
        const Window& win = w.win[i];
        int gi = tab.cumf[i];
        for (int a = win.t0; a < win.t1; a++)
            for (int b = win.h0; b < win.h1; b++)
                for (int c = win.w0; c < win.w1; c++, gi++) {
                    const int pos[3] = {TXT + a - win.t0, b - win.h0, c - win.w0};
                    const int tok = (a * w.h + b) * w.w + c;
                    tokpos[4 * (size_t)tok] = gi;
                    tokpos[4 * (size_t)tok + 1] = i;
                    tokpos[4 * (size_t)tok + 2] = pos[0] | (pos[1] << 16);
                    tokpos[4 * (size_t)tok + 3] = pos[2];
                    npos = std::max(npos, std::max(pos[0], std::max(pos[1], pos[2])) + 1);
                    for (int k = 0; k < ROPE_ROT && structured; k++)
                        if (w.vid_freq[(size_t)gi * ROPE_ROT + k] != (float)((double)pos[k / 42] * base[(k % 42) / 2]))
                            structured = false;
                }
        for (int p = 0; p < TXT && structured; p++)
            for (int k = 0; k < ROPE_ROT; k++)
                if (w.txt_freq[((size_t)i * TXT + p) * ROPE_ROT + k] != (float)((double)p * base[(k % 42) / 2])) {
                    structured = false;
                    break;
                }
    }
    if (npos >= 65536) structured = false;
    return upload_geom_with(g, w, tab, tokpos, structured, npos, w.tokens());
}

int DitB200::upload_geom_with(GeomDev& g, const WinGeom& w, const WinTables& tab, const std::vector<int>& tokpos,
                              bool structured, int npos, int Lv) {
    const int nwin = (int)tab.cumf.size() - 1, TXT = w.txt_len;
    std::vector<int> row_win((size_t)tab.cums[nwin]);
    for (int i = 0; i < nwin; i++)
        for (int p = tab.cums[i]; p < tab.cums[i + 1]; p++) row_win[p] = i;
    // cos/sin of every element's own angle, in float as the reference
    // evaluates them (src/dit_vk.cpp:66).
    std::vector<float> vc(w.vid_freq.size()), vs(w.vid_freq.size()), tc(w.txt_freq.size()), ts(w.txt_freq.size());
    for (size_t i = 0; i < vc.size(); i++) { vc[i] = cosf(w.vid_freq[i]); vs[i] = sinf(w.vid_freq[i]); }
    for (size_t i = 0; i < tc.size(); i++) { tc[i] = cosf(w.txt_freq[i]); ts[i] = sinf(w.txt_freq[i]); }
    double base[21];
    rope_base(base);
    std::vector<float> cs((size_t)npos * 21 * 2);
    for (int p = 0; p < npos; p++)
        for (int j = 0; j < 21; j++) {
            const float ang = (float)((double)p * base[j]);
            cs[((size_t)p * 21 + j) * 2] = cosf(ang);
            cs[((size_t)p * 21 + j) * 2 + 1] = sinf(ang);
        }
    auto up = [&](DevBuf& d, const void* src, size_t n) -> int {
        if (int rc = cuda_check(d.ensure(std::max<size_t>(n, 16)), "cudaMalloc(geometry)")) return rc;
        if (n) return cuda_check(cudaMemcpy(d.p, src, n, cudaMemcpyHostToDevice), "upload geometry");
        return OK;
    };
    if (int rc = up(g.vidx, tab.vidx.data(), tab.vidx.size() * 4)) return rc;
    if (int rc = up(g.cumf, tab.cumf.data(), tab.cumf.size() * 4)) return rc;
    if (int rc = up(g.cums, tab.cums.data(), tab.cums.size() * 4)) return rc;
    if (int rc = up(g.row_win, row_win.data(), row_win.size() * 4)) return rc;
    if (int rc = up(g.vcos, vc.data(), vc.size() * 4)) return rc;
    if (int rc = up(g.vsin, vs.data(), vs.size() * 4)) return rc;
    if (int rc = up(g.tcos, tc.data(), tc.size() * 4)) return rc;
    if (int rc = up(g.tsin, ts.data(), ts.size() * 4)) return rc;
    if (int rc = up(g.tokpos, tokpos.data(), tokpos.size() * 4)) return rc;
    if (int rc = up(g.cs, cs.data(), cs.size() * 4)) return rc;
    g.structured = structured;
    g.tokpos_host = tokpos;
    g.npos = npos;
    g.host = w;
    g.tab = tab;
    AwaDev& v = g.view;
    v.nwin = nwin; v.TXT = TXT; v.sumf = tab.sumf; v.sumS = tab.cums[nwin]; v.maxS = tab.maxS; v.Lv = Lv;
    v.vidx = g.vidx.as<int>(); v.cumf = g.cumf.as<int>(); v.cums = g.cums.as<int>(); v.row_win = g.row_win.as<int>();
    v.vcos = g.vcos.as<float>(); v.vsin = g.vsin.as<float>(); v.tcos = g.tcos.as<float>(); v.tsin = g.tsin.as<float>();
    g.ready = true;
    return OK;
}

int DitB200::set_windows(const WinGeom& ns, const WinGeom& sh) {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    cudaSetDevice(dev_);
    if (ns.tokens() != sh.tokens() || ns.txt_len != sh.txt_len) return fail(ERR_ARG, "non-shifted and shifted windows disagree on the grid");
    if (int rc = upload_geom(geom_[0], ns, -1)) return rc;
    if (int rc = upload_geom(geom_[1], sh, -1)) return rc;
    if (!geom_[0].tab.covers_all || !geom_[1].tab.covers_all)
        return fail(ERR_ARG, "DiT windows must tile the token grid exactly");
    if (gexec_) { cudaGraphExecDestroy(gexec_); gexec_ = nullptr; graph_Lv_ = -1; }
    geom_gen_++;
    return OK;
}

// ------------------------------------------------------------------ activations
int DitB200::ensure_acts(int Lv, int TXT) {
    const size_t M = (size_t)Lv + TXT, ab = act_bytes(act_);
    size_t sumS = 0, nwinTXT = 0;
    for (auto& g : geom_)
        if (g.ready) { sumS = std::max(sumS, (size_t)g.view.sumS); nwinTXT = std::max(nwinTXT, (size_t)g.view.nwin * g.view.TXT); }
    int rc;
    if ((rc = cuda_check(X_.ensure(M * DIM * 4), "cudaMalloc(X)"))) return rc;
    if ((rc = cuda_check(Xn_.ensure(M * DIM * ab), "cudaMalloc(Xn)"))) return rc;
    if ((rc = cuda_check(QKV_.ensure(M * QKV * ab), "cudaMalloc(QKV)"))) return rc;
    if ((rc = cuda_check(ATT_.ensure(M * DIM * ab), "cudaMalloc(ATT)"))) return rc;
    const size_t pb = attn_elem_bytes();
    if ((rc = cuda_check(Qp_.ensure(std::max<size_t>(sumS, 1) * DIM * pb), "cudaMalloc(Qp)"))) return rc;
    if ((rc = cuda_check(Kp_.ensure(std::max<size_t>(sumS, 1) * DIM * pb), "cudaMalloc(Kp)"))) return rc;
    if ((rc = cuda_check(Vp_.ensure(std::max<size_t>(sumS, 1) * DIM * pb), "cudaMalloc(Vp)"))) return rc;
    if ((rc = cuda_check(TOUTW_.ensure(std::max<size_t>(nwinTXT, 1) * DIM * 4), "cudaMalloc(TOUTW)"))) return rc;
    // [h | g] fp32 staging of the SIMT SwiGLU path (the tcgen05 path fuses it)
    const bool need_hg = act_ == ACT_F32 || !gemm_tc_supported((int)M, 2 * MLP_DIM, DIM, DIM, DIM);
    if (need_hg && (rc = cuda_check(HG_.ensure(M * 2 * MLP_DIM * 4), "cudaMalloc(HG)"))) return rc;
    if (act_ == ACT_F32 && tf32x3_ && (rc = cuda_check(A2_.ensure(M * 2 * MLP_DIM * 4), "cudaMalloc(A2)"))) return rc;
    if ((rc = cuda_check(Hs_.ensure(M * MLP_DIM * ab), "cudaMalloc(Hs)"))) return rc;
    if (norm_fuse_ && (rc = cuda_check(SQ_.ensure(M * SQ_SLOTS * 4), "cudaMalloc(SQ)"))) return rc;
    if ((rc = cuda_check(VPIN_.ensure((size_t)Lv * PATCH_IN_PAD * ab), "cudaMalloc(VPIN)"))) return rc;
    if ((rc = cuda_check(TIN_.ensure((size_t)TXT * TXT_IN * ab), "cudaMalloc(TIN)"))) return rc;
    if ((rc = cuda_check(SR_.ensure((size_t)Lv * OUT_CH * 4), "cudaMalloc(SR)"))) return rc;
    if ((rc = cuda_check(VIDIN_F_.ensure((size_t)Lv * DIM * 4), "cudaMalloc(VIDIN)"))) return rc;
    if ((rc = cuda_check(TXTIN_F_.ensure((size_t)TXT * TXT_IN * 4), "cudaMalloc(TXTIN)"))) return rc;
    cap_Lv_ = std::max(cap_Lv_, Lv); cap_TXT_ = std::max(cap_TXT_, TXT);
    return OK;
}

// ------------------------------------------------------------------ enqueue
void DitB200::gemm(const void* A, int lda, const Linear& L, int M, const GemmEpi& e, cudaStream_t s) {
    if (M <= 0) return;
    if (act_ == ACT_F32 && L.w2.bytes && e.mode != EPI_QKV_PACK && A2_.bytes >= (size_t)M * 2 * L.in * 4 &&
        gemm_tf32x3_supported(M, L.out, L.in, 2 * L.in, 2 * L.in)) {
        // fp32 path on the tensor cores: split the activations, then hi*hi + hi*lo + lo*hi
        pbeg(KK_GEMM_SIMT, 2.0 * M * L.out * L.in,
             (double)M * L.in * 12 + (double)L.out * L.in * 8 + (double)M * L.out * (e.mode == EPI_GATE_RESID ? 8 : 4), s);
        split_tf32((const float*)A, lda, M, L.in, A2_.as<float>(), 2 * L.in, s);
        const int rc = gemm_tf32x3(A2_.p, 2 * L.in, L.w2.p, 2 * L.in, M, L.out, L.in, e, s, &launches_);
        launches_++;
        pend(s);
        if (rc == 0) return;
    }
    const double flops = 2.0 * M * L.out * L.in;
    const double bytes = (double)M * L.in * act_bytes(act_) + (double)L.out * L.in * act_bytes(L.t) +
                         (double)M * L.out * (e.mode == EPI_GATE_RESID ? 8 : e.mode == EPI_SWIGLU ? act_bytes(e.out_t) / 2.0 : act_bytes(e.out_t));
    if (act_half(act_) && L.t == act_ && gemm_tc_supported(M, L.out, L.in, lda, L.ld)) {
        // 16-bit operands on tcgen05: A and W are both of the context's type
        pbeg(KK_GEMM_TC, flops, bytes, s);
        GemmEpi et = e;
        et.op_t = act_;
        gemm_tc(A, lda, L.w.p, L.ld, M, L.out, L.in, et, s, &launches_);
        pend(s);
        return;
    }
    pbeg(KK_GEMM_SIMT, flops, bytes, s);
    if (e.mode == EPI_SWIGLU) {
        // SIMT path: materialise [h | g] in fp32, then combine.
        GemmEpi st; st.mode = EPI_STORE; st.out = HG_.p; st.ldo = 2 * MLP_DIM; st.out_t = ACT_F32;
        gemm_simt(A, act_, lda, L.w.p, L.t, L.ld, M, L.out, L.in, st, s);
        swiglu_rows(HG_.as<float>(), M, 2 * MLP_DIM, e.out, e.ldo, e.out_t, s);
        launches_ += 2;
    } else {
        gemm_simt(A, act_, lda, L.w.p, L.t, L.ld, M, L.out, L.in, e, s);
        launches_++;
    }
    pend(s);
}

// The vid and txt GEMMs of an MM-DiT block (separate weights, same shape and
// epilogue) as one launch when both suit the tcgen05 pair kernel; otherwise
// two launches.
void DitB200::gemm2(const void* A0, int lda0, const Linear& L0, int M0, const GemmEpi& e0, const void* A1, int lda1,
                    const Linear& L1, int M1, const GemmEpi& e1, cudaStream_t s) {
    if (act_half(act_) && L0.t == act_ && L1.t == act_ && M0 > 128 && M1 > 0 && L0.out == L1.out &&
        L0.in == L1.in && gemm_tc_supported(M0, L0.out, L0.in, lda0, L0.ld) &&
        gemm_tc_supported(M1, L1.out, L1.in, lda1, L1.ld)) {
        const double flops = 2.0 * (M0 + M1) * L0.out * L0.in;
        const double bytes = (double)(M0 + M1) * L0.in * act_bytes(act_) + 2.0 * L0.out * L0.in * act_bytes(L0.t) +
                             (double)(M0 + M1) * L0.out * (e0.mode == EPI_GATE_RESID ? 8 : e0.mode == EPI_SWIGLU ? act_bytes(e0.out_t) / 2.0 : act_bytes(e0.out_t));
        pbeg(KK_GEMM_TC, flops, bytes, s);
        GemmEpi f0 = e0, f1 = e1;
        f0.op_t = f1.op_t = act_;
        const int rc = gemm_tc_grouped(A0, lda0, L0.w.p, L0.ld, M0, f0, A1, lda1, L1.w.p, L1.ld, M1, f1, L0.out,
                                       L0.in, s, &launches_);
        pend(s);
        if (rc == 0) return;
    }
    gemm(A0, lda0, L0, M0, e0, s);
    gemm(A1, lda1, L1, M1, e1, s);
}

void sinusoidal256(float t, float* e) {   // src/dit_vk.cpp:295-302
    const int half = 128;
    for (int j = 0; j < 256; j++) {
        float freq = (j < half) ? (float)std::exp(-logf(10000.f) * j / half) : (float)std::exp(-logf(10000.f) * (j - half) / half);
        e[j] = (j < half) ? sinf(t * freq) : cosf(t * freq);
    }
}

int DitB200::enqueue_temb(cudaStream_t s) {
    // time embedding (src/dit_vk.cpp:303-309) in fp32, then AdaCompose.
    pbeg(KK_OTHER, 2.0 * (TEMB_IN * DIM + DIM * DIM + (double)DIM * EMB_DIM), 4.0 * (TEMB_IN * DIM + DIM * DIM + (double)DIM * EMB_DIM), s);
    // one-row GEMVs (bias and SiLU fused) when the fp32 weights allow float4 rows
    const bool gv = gemv_f32(temb_in_.as<float>(), TEMB_IN, emb_in_.w.as<float>(), emb_in_.ld, DIM, emb_in_.bias(),
                             temb_h1_.as<float>(), true, s);
    if (gv) {
        gemv_f32(temb_h1_.as<float>(), DIM, emb_hid_.w.as<float>(), emb_hid_.ld, DIM, emb_hid_.bias(),
                 temb_h2_.as<float>(), true, s);
        gemv_f32(temb_h2_.as<float>(), DIM, emb_out_.w.as<float>(), emb_out_.ld, EMB_DIM, emb_out_.bias(),
                 emb_.as<float>(), false, s);
        launches_ += 3;
    } else {
        GemmEpi e; e.mode = EPI_STORE; e.out_t = ACT_F32;
        e.bias = emb_in_.bias(); e.out = temb_h1_.p; e.ldo = DIM;
        gemm_simt(temb_in_.p, ACT_F32, TEMB_IN, emb_in_.w.p, ACT_F32, emb_in_.ld, 1, DIM, TEMB_IN, e, s);
        silu_inplace(temb_h1_.as<float>(), DIM, s);
        e.bias = emb_hid_.bias(); e.out = temb_h2_.p;
        gemm_simt(temb_h1_.p, ACT_F32, DIM, emb_hid_.w.p, ACT_F32, emb_hid_.ld, 1, DIM, DIM, e, s);
        silu_inplace(temb_h2_.as<float>(), DIM, s);
        e.bias = emb_out_.bias(); e.out = emb_.p; e.ldo = EMB_DIM;
        gemm_simt(temb_h2_.p, ACT_F32, DIM, emb_out_.w.p, ACT_F32, emb_out_.ld, 1, EMB_DIM, DIM, e, s);
        launches_ += 5;
    }
    s2b::ada_compose(emb_.as<float>(), branch_.as<float>(), NUM_LAYERS * 12 + 2, ada_.as<float>(), s);
    launches_ += 1;
    pend(s);
    return OK;
}

int DitB200::enqueue_init(int Lv, int TXT, cudaStream_t s) {
    // vid_in_proj (132 -> 2560) and txt_in (5120 -> 2560), src/dit_vk.cpp:494-497
    pbeg(KK_NORM, 0, (double)Lv * PATCH_IN * 4 + (double)TXT * TXT_IN * 4 + ((double)Lv * PATCH_IN_PAD + (double)TXT * TXT_IN) * act_bytes(act_), s);
    pad_convert_rows(VIDIN_F_.as<float>(), Lv, PATCH_IN, VPIN_.p, PATCH_IN_PAD, act_, s);
    pad_convert_rows(TXTIN_F_.as<float>(), TXT, TXT_IN, TIN_.p, TXT_IN, act_, s);
    launches_ += 2;
    pend(s);
    GemmEpi e; e.mode = EPI_STORE; e.out_t = ACT_F32; e.ldo = DIM;
    e.bias = vid_in_.bias(); e.out = X_.p;
    gemm(VPIN_.p, PATCH_IN_PAD, vid_in_, Lv, e, s);
    e.bias = txt_in_.bias(); e.out = X_.as<float>() + (size_t)Lv * DIM;
    gemm(TIN_.p, TXT_IN, txt_in_, TXT, e, s);
    return OK;
}

LayerBufs DitB200::default_bufs() {
    LayerBufs b;
    b.X = X_.as<float>(); b.Xn = Xn_.p; b.QKV = QKV_.p; b.ATT = ATT_.p; b.Hs = Hs_.p;
    b.Qp = Qp_.p; b.Kp = Kp_.p; b.Vp = Vp_.p; b.TOUTW = TOUTW_.as<float>();
    b.geom[0] = &geom_[0]; b.geom[1] = &geom_[1];
    return b;
}

bool DitB200::attn_norm_foldable(int j) const {
    // layer 0 reads the input projections; layer 31 leaves txt unmodulated
    // (forward_latent's vid_only block); the fused QKV pack applies the fold
    const GeomDev& G = geom_[j % 2];
    return norm_fuse_ && shift_ok_ && j >= 1 && j <= NUM_LAYERS - 2 && G.structured &&
           G.cs.bytes >= (size_t)G.npos * 21 * sizeof(float2);
}

int DitB200::enqueue_layer(int i, int Lv, int TXT, cudaStream_t s, int l0, int l1) {
    LayerBufs b = default_bufs();
    b.SQ = SQ_.as<float>();
    b.fuse_mlp = norm_fuse_ && shift_ok_;
    b.fuse_attn_in = i > l0 && attn_norm_foldable(i);
    b.fuse_attn_out = i + 1 < l1 && attn_norm_foldable(i + 1);
    return enqueue_layer_on(i, Lv, TXT, s, b);
}

// The folded norms need, per layer and flow, the adaLN shift carried through
// the following Linear: c = W . shift (the norm's output is rs * (x * scale) +
// shift, so its GEMM is rs * ((x * scale) W^T) + W . shift).  The shifts depend
// only on the timestep, so c is computed once per timestep: the time
// embedding and AdaCompose for t, then one bf16 GEMV per Linear.
int DitB200::prepare_shift(float t, cudaStream_t s) {
    if (!norm_fuse_ || (shift_ok_ && t == shift_t_)) return OK;
    float temb[TEMB_IN];
    sinusoidal256(t, temb);
    cudaMemcpyAsync(temb_in_.p, temb, sizeof temb, cudaMemcpyHostToDevice, s);
    enqueue_temb(s);
    for (int i = layer_lo_; i < layer_hi_; i++)
        for (int f = 0; f < (i < MM_LAYERS ? 2 : 1); f++) {
            const Block& B = blk_[i][f];
            gemv_bf16(B.qkv.w.p, B.qkv.ld, QKV, DIM, ada(i, f, 1), const_cast<float*>(shift_qkv(i, f)), s);
            gemv_bf16(B.mlp_hg.w.p, B.mlp_hg.ld, 2 * MLP_DIM, DIM, ada(i, f, 4), const_cast<float*>(shift_hg(i, f)), s);
            launches_ += 2;
        }
    if (int rc = cuda_check(cudaGetLastError(), "shift biases")) return rc;
    shift_ok_ = true;
    shift_t_ = t;
    return OK;
}

int DitB200::enqueue_layer_on(int i, int Lv, int TXT, cudaStream_t s, const LayerBufs& B) {
    // the last layer is vid_only as forward_latent runs it (src/dit_vk.cpp:523-625), unless the
    // chunked graph's semantics were selected (export/export_dit_graph.py:155-226: txt as in every layer)
    const bool dual = i < MM_LAYERS, last = (i == NUM_LAYERS - 1) && !graph_last_;
    const int M = Lv + TXT;
    const size_t ab = act_bytes(act_);
    GeomDev& G = *B.geom[i % 2];
    const Block& BV = blk_[i][0];
    const Block& BT = dual ? blk_[i][1] : blk_[i][0];
    char* xn = (char*)B.Xn;
    char* qkv = (char*)B.QKV;
    char* att = (char*)B.ATT;
    char* hs = (char*)B.Hs;
    float* X = B.X;

    const double norm_bytes = (double)DIM * (4 + ab);
    // 1. attention norm + modulate (txt unmodulated on the last layer, src/dit_vk.cpp:538); folded into
    //    the previous layer's last GEMM (operand) and this layer's QKV GEMM (row factor, shift) when
    //    B.fuse_attn_in
    if (!B.fuse_attn_in) {
        pbeg(KK_NORM, 0, norm_bytes * M, s);
        rmsnorm_mod(X, DIM, M, Lv, ada(i, 0, 0), ada(i, 0, 1), last ? nullptr : ada(i, 1, 0), ada(i, 1, 1), nullptr,
                    NORM_EPS, B.Xn, DIM, act_, s);
        launches_++;
        pend(s);
    }
    // the folded-norm fields of a GEMM consuming a fused operand (rows from row0)
    auto fold_in = [&](GemmEpi& e, const float* shift, int row0) {
        e.sq_in = B.SQ + (size_t)row0 * SQ_SLOTS; e.sq_n = SQ_SLOTS; e.rs_dim = (float)DIM; e.rs_eps = NORM_EPS;
        e.bias = shift;
    };
    // ... and of a gate/residual GEMM producing one for the next norm (scale sc0 for rows < split)
    auto fold_out = [&](GemmEpi& e, const float* sc0, const float* sc1, int split, int row0) {
        e.mod_out = (char*)B.Xn + (size_t)row0 * DIM * ab; e.ldm = DIM;
        e.mod_sc0 = sc0; e.mod_sc1 = sc1; e.mod_split = split;
        e.sq_out = B.SQ + (size_t)row0 * SQ_SLOTS;
    };
    // 2. qkv projection (no bias), then qk-norm + RoPE + window packing
    const bool fused_pack = act_half(act_) && BV.qkv.t == act_ && G.structured &&
                            G.cs.bytes >= (size_t)G.npos * 21 * sizeof(float2) &&
                            gemm_tc_supported(M, QKV, DIM, DIM, DIM);
    if (fused_pack) {
        // one tcgen05 GEMM epilogue writes the packed Q/K/V directly (no qkv buffer)
        GemmEpi e; e.mode = EPI_QKV_PACK;
        PackEpi& k = e.pk;
        k.tokpos = G.tokpos.as<const int4>(); k.cums = G.view.cums; k.cs = G.cs.as<const float2>(); k.npos = G.npos;
        k.nq0 = normw(i, 0, 0); k.nk0 = normw(i, 0, 1); k.nq1 = normw(i, 1, 0); k.nk1 = normw(i, 1, 1);
        k.eps = NORM_EPS; k.Lv = Lv; k.TXT = TXT; k.nwin = G.view.nwin; k.sumS = G.view.sumS;
        k.Qp = B.Qp; k.Kp = B.Kp; k.Vp = B.Vp; k.qkv_t = act_;
        if (dual) {
            GemmEpi et = e;
            k.row_base = 0; et.pk.row_base = Lv;
            if (B.fuse_attn_in) { fold_in(e, shift_qkv(i, 0), 0); fold_in(et, shift_qkv(i, 1), Lv); }
            gemm2(xn, DIM, BV.qkv, Lv, e, xn + (size_t)Lv * DIM * ab, DIM, BT.qkv, TXT, et, s);
        } else {
            k.row_base = 0;
            if (B.fuse_attn_in) fold_in(e, shift_qkv(i, 0), 0);
            gemm(xn, DIM, BV.qkv, M, e, s);
        }
    } else {
        GemmEpi e; e.mode = EPI_STORE; e.out_t = act_; e.ldo = QKV;
        if (dual) {
            e.out = qkv; gemm(xn, DIM, BV.qkv, Lv, e, s);
            e.out = qkv + (size_t)Lv * QKV * ab; gemm(xn + (size_t)Lv * DIM * ab, DIM, BT.qkv, TXT, e, s);
        } else {
            e.out = qkv; gemm(xn, DIM, BV.qkv, M, e, s);
        }
        pbeg(KK_PACK, 0, (double)G.view.sumS * QKV * (ab + attn_elem_bytes()), s);
        if (attn_split3_)
            awa_pack_split3(qkv, qkv + (size_t)Lv * QKV * ab, act_, QKV, G.view, normw(i, 0, 0), normw(i, 0, 1),
                            normw(i, 1, 0), normw(i, 1, 1), NORM_EPS, B.Qp, B.Kp, B.Vp, s);
        else
            awa_pack(qkv, qkv + (size_t)Lv * QKV * ab, act_, QKV, G.view, normw(i, 0, 0), normw(i, 0, 1),
                     normw(i, 1, 0), normw(i, 1, 1), NORM_EPS, B.Qp, B.Kp, B.Vp, act_, s);
        launches_++;
        pend(s);
    }
    // 3. AWA
    double attn_flops = 0;
    for (int w = 0; w < G.view.nwin; w++) {
        const double S = G.tab.cums[w + 1] - G.tab.cums[w];
        attn_flops += 4.0 * S * S * HEAD_D * HEADS;
    }
    pbeg(KK_ATTN, attn_flops, (double)G.view.sumS * QKV * attn_elem_bytes() + (double)Lv * DIM * ab + (double)G.view.nwin * TXT * DIM * 4, s);
    if (attn_split3_) {
        if (awa_attend_split3(B.Qp, B.Kp, B.Vp, G.view, 1.0f / sqrtf((float)HEAD_D), att, DIM, act_, B.TOUTW, s))
            return fail(ERR_CUDA, "fp32 tensor-core attention: tensor maps could not be encoded");
        launches_++;
    } else if (awa_attend(B.Qp, B.Kp, B.Vp, act_, G.view, 1.0f / sqrtf((float)HEAD_D), att, DIM, act_, B.TOUTW, s,
                          &launches_)) {
        return fail(ERR_CUDA, "bf16 tensor-core attention: tensor maps could not be encoded");
    }
    pend(s);
    pbeg(KK_OTHER, 0, (double)G.view.nwin * TXT * DIM * 4 + (double)TXT * DIM * ab, s);
    if (B.txt_partial) {
        // window-sharded: sum this rank's windows, then combine the ranks'
        // partials and divide by the global window count
        awa_coalesce_div(B.TOUTW, G.view.nwin, TXT, B.txt_partial(B.shard_ctx, i), DIM, ACT_F32, 0.f, s);
        pend(s);
        pbeg(KK_EXCHANGE, 0, (double)TXT * DIM * 4, s);
        if (int rc = B.txt_finish(B.shard_ctx, i, att + (size_t)Lv * DIM * ab, s)) return rc;
        launches_ += 2;
    } else {
        awa_coalesce(B.TOUTW, G.view.nwin, TXT, att + (size_t)Lv * DIM * ab, DIM, act_, s);
        launches_++;
    }
    pend(s);
    // 4. out projection (+bias), gate, residual (src/dit_vk.cpp:461-462, 558-575)
    GemmEpi g; g.mode = EPI_GATE_RESID; g.ldr = DIM;
    if (dual) {
        GemmEpi gt = g;
        g.resid = X; g.bias = BV.out.bias(); g.gate0 = ada(i, 0, 2); g.gate_split = M;
        gt.resid = X + (size_t)Lv * DIM; gt.bias = BT.out.bias(); gt.gate0 = last ? nullptr : ada(i, 1, 2);
        gt.gate_split = M;
        if (B.fuse_mlp) { fold_out(g, ada(i, 0, 3), nullptr, M, 0); fold_out(gt, ada(i, 1, 3), nullptr, M, Lv); }
        gemm2(att, DIM, BV.out, Lv, g, att + (size_t)Lv * DIM * ab, DIM, BT.out, TXT, gt, s);
    } else {
        g.resid = X; g.bias = BV.out.bias(); g.gate0 = ada(i, 0, 2); g.gate1 = last ? nullptr : ada(i, 1, 2);
        g.gate_split = Lv;
        if (B.fuse_mlp) fold_out(g, ada(i, 0, 3), ada(i, 1, 3), Lv, 0);
        gemm(att, DIM, BV.out, M, g, s);
    }
    // 5. MLP norm + modulate; txt skips the MLP on the last layer (src/dit_vk.cpp:579-620); folded
    //    into the out-projection (operand) and the SwiGLU GEMM (row factor, shift) when B.fuse_mlp
    const int Mm = last ? Lv : M;
    if (!B.fuse_mlp) {
        pbeg(KK_NORM, 0, norm_bytes * Mm, s);
        rmsnorm_mod(X, DIM, Mm, Lv, ada(i, 0, 3), ada(i, 0, 4), ada(i, 1, 3), ada(i, 1, 4), nullptr, NORM_EPS, B.Xn,
                    DIM, act_, s);
        launches_++;
        pend(s);
    }
    // 6. SwiGLU: proj_out(silu(proj_in_gate x) * proj_in x)
    GemmEpi sw; sw.mode = EPI_SWIGLU; sw.out_t = act_; sw.ldo = MLP_DIM;
    GemmEpi mo; mo.mode = EPI_GATE_RESID; mo.ldr = DIM;
    // the next layer's attention-norm operand (scale a_sc of layer i + 1) from the last GEMM
    const int nx = i + 1 < NUM_LAYERS ? i + 1 : i;
    if (dual && !last) {
        GemmEpi swt = sw, mot = mo;
        sw.out = hs;
        swt.out = hs + (size_t)Lv * MLP_DIM * ab;
        if (B.fuse_mlp) { fold_in(sw, shift_hg(i, 0), 0); fold_in(swt, shift_hg(i, 1), Lv); }
        gemm2(xn, DIM, BV.mlp_hg, Lv, sw, xn + (size_t)Lv * DIM * ab, DIM, BT.mlp_hg, TXT, swt, s);
        mo.resid = X; mo.gate0 = ada(i, 0, 5); mo.gate_split = M;
        mot.resid = X + (size_t)Lv * DIM; mot.gate0 = ada(i, 1, 5); mot.gate_split = M;
        if (B.fuse_attn_out) { fold_out(mo, ada(nx, 0, 0), nullptr, M, 0); fold_out(mot, ada(nx, 1, 0), nullptr, M, Lv); }
        gemm2(hs, MLP_DIM, BV.mlp_out, Lv, mo, hs + (size_t)Lv * MLP_DIM * ab, MLP_DIM, BT.mlp_out, TXT, mot, s);
    } else if (dual) {
        sw.out = hs;
        if (B.fuse_mlp) fold_in(sw, shift_hg(i, 0), 0);
        gemm(xn, DIM, BV.mlp_hg, Lv, sw, s);
        mo.resid = X; mo.gate0 = ada(i, 0, 5); mo.gate_split = M;
        gemm(hs, MLP_DIM, BV.mlp_out, Lv, mo, s);
    } else {
        sw.out = hs;
        if (B.fuse_mlp) fold_in(sw, shift_hg(i, 0), 0);
        gemm(xn, DIM, BV.mlp_hg, Mm, sw, s);
        mo.resid = X; mo.gate0 = ada(i, 0, 5); mo.gate1 = ada(i, 1, 5); mo.gate_split = Lv;
        if (B.fuse_attn_out) fold_out(mo, ada(nx, 0, 0), ada(nx, 1, 0), Lv, 0);
        gemm(hs, MLP_DIM, BV.mlp_out, Mm, mo, s);
    }
    return OK;
}

int DitB200::enqueue_final(int Lv, cudaStream_t s) {
    // final RMSNorm (affine) + modulate (fin_sc, fin_sh) + vid_out_proj (src/dit_vk.cpp:657-675)
    const float* fin_sc = ada_.as<float>() + (size_t)(NUM_LAYERS * 12) * DIM;
    const float* fin_sh = fin_sc + DIM;
    pbeg(KK_NORM, 0, (double)Lv * DIM * (4 + act_bytes(act_)), s);
    rmsnorm_mod(X_.as<float>(), DIM, Lv, Lv, fin_sc, fin_sh, nullptr, nullptr, von_w_.as<float>(), NORM_EPS, Xn_.p,
                DIM, act_, s);
    launches_++;
    pend(s);
    GemmEpi e; e.mode = EPI_STORE; e.out_t = ACT_F32; e.ldo = OUT_CH; e.bias = vid_out_.bias(); e.out = SR_.p;
    gemm(Xn_.p, DIM, vid_out_, Lv, e, s);
    return OK;
}

// ------------------------------------------------------------------ profiling
void DitB200::pbeg(int kind, double flops, double bytes, cudaStream_t s) {
    if (!prof_on_) return;
    while (ev_pool_.size() < 2 * (marks_.size() + 1)) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        ev_pool_.push_back(e);
    }
    ProfMark m;
    m.kind = kind; m.flops = flops; m.bytes = bytes;
    m.a = ev_pool_[2 * marks_.size()];
    m.b = ev_pool_[2 * marks_.size() + 1];
    cudaEventRecord(m.a, s);
    marks_.push_back(m);
}

void DitB200::pend(cudaStream_t s) {
    if (!prof_on_ || marks_.empty()) return;
    cudaEventRecord(marks_.back().b, s);
}

int DitB200::forward_profile(const float* vid_patch, int Lv, const float* txt, int TXT, float t, double* ms,
                             double* flops, double* bytes, int* count, bool sharded) {
    if (!ms || !flops || !bytes || !count) return fail(ERR_ARG, "null profile arrays");
    if (layer_lo_ != 0 || layer_hi_ != NUM_LAYERS) return fail(ERR_STATE, "profiling needs all 32 layers loaded");
    std::vector<float> sr((size_t)std::max(Lv, 0) * OUT_CH);
    marks_.clear();
    prof_on_ = true;
    const int rc = sharded ? shard_forward(vid_patch, Lv, txt, TXT, t, sr.data())
                           : forward_latent(vid_patch, Lv, txt, TXT, t, 0, NUM_LAYERS, true, true, nullptr, nullptr, sr.data());
    prof_on_ = false;
    if (rc) return rc;
    for (int k = 0; k < KK_COUNT; k++) { ms[k] = 0; flops[k] = 0; bytes[k] = 0; count[k] = 0; }
    for (const auto& m : marks_) {
        float e = 0;
        cudaEventElapsedTime(&e, m.a, m.b);
        ms[m.kind] += e; flops[m.kind] += m.flops; bytes[m.kind] += m.bytes; count[m.kind]++;
    }
    marks_.clear();
    return OK;
}

// ------------------------------------------------------------------ public forwards
int DitB200::forward_latent(const float* vid_in, int Lv, const float* txt_in, int TXT, float t, int l0, int l1,
                            bool do_init, bool do_final, float* vid_lat, float* txt_lat, float* sr_out) {
    if (!weights_) return fail(ERR_STATE, "weights not loaded");
    if (!geom_[0].ready || !geom_[1].ready) return fail(ERR_STATE, "windows not set");
    if (Lv != geom_[0].view.Lv) return fail(ERR_ARG, "Lv does not match the window grid");
    if (TXT != geom_[0].view.TXT || TXT <= 0) return fail(ERR_ARG, "TXT does not match the windows' txt_len");
    if (l0 < 0 || l1 > NUM_LAYERS || l0 > l1) return fail(ERR_ARG, "layer range out of [0, 32]");
    if (l0 < l1 && (l0 < layer_lo_ || l1 > layer_hi_)) return fail(ERR_STATE, "layers outside the loaded weight range");
    if (!vid_in || !txt_in || (do_final && !sr_out) || (!do_final && (!vid_lat || !txt_lat)))
        return fail(ERR_ARG, "null buffer");
    cudaSetDevice(dev_);
    if (int rc = ensure_acts(Lv, TXT)) return rc;
    cudaStream_t s = stream_;
    launches_ = 0;
    float temb[TEMB_IN];
    sinusoidal256(t, temb);
    cudaMemcpyAsync(temb_in_.p, temb, sizeof temb, cudaMemcpyHostToDevice, s);
    if (do_init) {
        cudaMemcpyAsync(VIDIN_F_.p, vid_in, (size_t)Lv * PATCH_IN * 4, cudaMemcpyHostToDevice, s);
        cudaMemcpyAsync(TXTIN_F_.p, txt_in, (size_t)TXT * TXT_IN * 4, cudaMemcpyHostToDevice, s);
        enqueue_init(Lv, TXT, s);
    } else {
        cudaMemcpyAsync(X_.p, vid_in, (size_t)Lv * DIM * 4, cudaMemcpyHostToDevice, s);
        cudaMemcpyAsync(X_.as<float>() + (size_t)Lv * DIM, txt_in, (size_t)TXT * DIM * 4, cudaMemcpyHostToDevice, s);
    }
    enqueue_temb(s);
    if (int rc = prepare_shift(t, s)) return rc;
    for (int i = l0; i < l1; i++) enqueue_layer(i, Lv, TXT, s, l0, l1);
    if (do_final) enqueue_final(Lv, s);
    fold_status(s);
    if (do_final) {
        cudaMemcpyAsync(sr_out, SR_.p, (size_t)Lv * OUT_CH * 4, cudaMemcpyDeviceToHost, s);
    } else {
        cudaMemcpyAsync(vid_lat, X_.p, (size_t)Lv * DIM * 4, cudaMemcpyDeviceToHost, s);
        cudaMemcpyAsync(txt_lat, X_.as<float>() + (size_t)Lv * DIM, (size_t)TXT * DIM * 4, cudaMemcpyDeviceToHost, s);
    }
    last_launches_ = launches_;
    if (int rc = cuda_check(cudaGetLastError(), "kernel launch")) return rc;
    if (int rc = sync_check(s, "forward_latent")) return rc;
    return take_status(s, "forward_latent");
}

int DitB200::capture_full(int Lv, int TXT) {
    if (gexec_ && graph_Lv_ == Lv && graph_TXT_ == TXT) return OK;
    if (gexec_) { cudaGraphExecDestroy(gexec_); gexec_ = nullptr; }
    cudaGraph_t graph = nullptr;
    launches_ = 0;
    if (int rc = cuda_check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "begin capture")) return rc;
    enqueue_init(Lv, TXT, stream_);
    enqueue_temb(stream_);
    for (int i = 0; i < NUM_LAYERS; i++) enqueue_layer(i, Lv, TXT, stream_, 0, NUM_LAYERS);
    enqueue_final(Lv, stream_);
    fold_status(stream_);
    cudaError_t ce = cudaStreamEndCapture(stream_, &graph);
    if (int rc = cuda_check(ce, "end capture")) return rc;
    ce = cudaGraphInstantiate(&gexec_, graph, 0);
    cudaGraphDestroy(graph);
    if (int rc = cuda_check(ce, "graph instantiate")) { gexec_ = nullptr; return rc; }
    graph_Lv_ = Lv; graph_TXT_ = TXT; graph_launches_ = launches_;
    return OK;
}

int DitB200::forward_dev(const float* d_vid, int Lv, const float* d_txt, int TXT, float t, float* d_sr,
                         cudaStream_t user) {
    if (!weights_) return fail(ERR_STATE, "weights not loaded");
    if (layer_lo_ != 0 || layer_hi_ != NUM_LAYERS) return fail(ERR_STATE, "full forward needs all 32 layers loaded");
    if (!geom_[0].ready || !geom_[1].ready) return fail(ERR_STATE, "windows not set");
    if (Lv != geom_[0].view.Lv || TXT != geom_[0].view.TXT || TXT <= 0) return fail(ERR_ARG, "Lv/TXT do not match the windows");
    if (!d_vid || !d_txt || !d_sr) return fail(ERR_ARG, "null buffer");
    cudaSetDevice(dev_);
    if (int rc = ensure_acts(Lv, TXT)) return rc;
    if (int rc = prepare_shift(t, stream_)) return rc;
    if (int rc = capture_full(Lv, TXT)) return rc;
    // Order the internal stream after the caller's work, run, then order the
    // caller after us.
    cudaEvent_t ev_in, ev_out;
    cudaEventCreateWithFlags(&ev_in, cudaEventDisableTiming);
    cudaEventCreateWithFlags(&ev_out, cudaEventDisableTiming);
    cudaEventRecord(ev_in, user);
    cudaStreamWaitEvent(stream_, ev_in, 0);
    float temb[TEMB_IN];
    sinusoidal256(t, temb);
    cudaMemcpyAsync(temb_in_.p, temb, sizeof temb, cudaMemcpyHostToDevice, stream_);
    cudaMemcpyAsync(VIDIN_F_.p, d_vid, (size_t)Lv * PATCH_IN * 4, cudaMemcpyDeviceToDevice, stream_);
    cudaMemcpyAsync(TXTIN_F_.p, d_txt, (size_t)TXT * TXT_IN * 4, cudaMemcpyDeviceToDevice, stream_);
    cudaGraphLaunch(gexec_, stream_);
    cudaMemcpyAsync(d_sr, SR_.p, (size_t)Lv * OUT_CH * 4, cudaMemcpyDeviceToDevice, stream_);
    cudaEventRecord(ev_out, stream_);
    cudaStreamWaitEvent(user, ev_out, 0);
    cudaEventDestroy(ev_in);
    cudaEventDestroy(ev_out);
    last_launches_ = graph_launches_;
    return cuda_check(cudaGetLastError(), "forward_dev");
}

int DitB200::forward_grid_dev(const float* d_grid, int T, int H, int W, const float* d_txt, int TXT, float t,
                              float* d_sr_grid, cudaStream_t user) {
    if (!d_grid || !d_txt || !d_sr_grid) return fail(ERR_ARG, "null buffer");
    if (T <= 0 || H <= 0 || W <= 0 || H % 2 || W % 2) return fail(ERR_ARG, "grid H and W must be positive and even");
    if (!weights_) return fail(ERR_STATE, "weights not loaded");
    if (layer_lo_ != 0 || layer_hi_ != NUM_LAYERS) return fail(ERR_STATE, "full forward needs all 32 layers loaded");
    if (!geom_[0].ready || !geom_[1].ready) return fail(ERR_STATE, "windows not set");
    const int Lv = T * (H / 2) * (W / 2);
    if (Lv != geom_[0].view.Lv || TXT != geom_[0].view.TXT || TXT <= 0) return fail(ERR_ARG, "grid / TXT do not match the windows");
    cudaSetDevice(dev_);
    if (int rc = ensure_acts(Lv, TXT)) return rc;
    if (int rc = prepare_shift(t, stream_)) return rc;
    if (int rc = capture_full(Lv, TXT)) return rc;
    cudaEvent_t ev_in, ev_out;
    cudaEventCreateWithFlags(&ev_in, cudaEventDisableTiming);
    cudaEventCreateWithFlags(&ev_out, cudaEventDisableTiming);
    cudaEventRecord(ev_in, user);
    cudaStreamWaitEvent(stream_, ev_in, 0);
    float temb[TEMB_IN];
    sinusoidal256(t, temb);
    cudaMemcpyAsync(temb_in_.p, temb, sizeof temb, cudaMemcpyHostToDevice, stream_);
    patchify_dev(d_grid, T, H, W, VIDIN_F_.as<float>(), stream_);
    cudaMemcpyAsync(TXTIN_F_.p, d_txt, (size_t)TXT * TXT_IN * 4, cudaMemcpyDeviceToDevice, stream_);
    cudaGraphLaunch(gexec_, stream_);
    unpatchify_dev(SR_.as<float>(), T, H, W, d_sr_grid, stream_);
    cudaEventRecord(ev_out, stream_);
    cudaStreamWaitEvent(user, ev_out, 0);
    cudaEventDestroy(ev_in);
    cudaEventDestroy(ev_out);
    last_launches_ = graph_launches_ + 2;
    return cuda_check(cudaGetLastError(), "forward_grid_dev");
}

int DitB200::forward(const float* vid_patch, int Lv, const float* txt, int TXT, float t, float* sr_out) {
    if (!vid_patch || !txt || !sr_out) return fail(ERR_ARG, "null buffer");
    if (!weights_) return fail(ERR_STATE, "weights not loaded");
    if (layer_lo_ != 0 || layer_hi_ != NUM_LAYERS) return fail(ERR_STATE, "full forward needs all 32 layers loaded");
    if (!geom_[0].ready || !geom_[1].ready) return fail(ERR_STATE, "windows not set");
    if (Lv != geom_[0].view.Lv || TXT != geom_[0].view.TXT || TXT <= 0) return fail(ERR_ARG, "Lv/TXT do not match the windows");
    cudaSetDevice(dev_);
    if (int rc = ensure_acts(Lv, TXT)) return rc;
    if (int rc = prepare_shift(t, stream_)) return rc;
    if (int rc = capture_full(Lv, TXT)) return rc;
    // the graph reads its inputs from VIDIN_F_/TXTIN_F_/temb_in_ and leaves sr in SR_
    float temb[TEMB_IN];
    sinusoidal256(t, temb);
    cudaMemcpyAsync(temb_in_.p, temb, sizeof temb, cudaMemcpyHostToDevice, stream_);
    cudaMemcpyAsync(VIDIN_F_.p, vid_patch, (size_t)Lv * PATCH_IN * 4, cudaMemcpyHostToDevice, stream_);
    cudaMemcpyAsync(TXTIN_F_.p, txt, (size_t)TXT * TXT_IN * 4, cudaMemcpyHostToDevice, stream_);
    cudaGraphLaunch(gexec_, stream_);
    cudaMemcpyAsync(sr_out, SR_.p, (size_t)Lv * OUT_CH * 4, cudaMemcpyDeviceToHost, stream_);
    last_launches_ = graph_launches_;
    if (int rc = sync_check(stream_, "forward")) return rc;
    return take_status(stream_, "forward");
}

int DitB200::time_embedding(float t, float* emb_host) {
    if (!weights_) return fail(ERR_STATE, "weights not loaded");
    cudaSetDevice(dev_);
    float temb[TEMB_IN];
    sinusoidal256(t, temb);
    cudaMemcpyAsync(temb_in_.p, temb, sizeof temb, cudaMemcpyHostToDevice, stream_);
    enqueue_temb(stream_);
    cudaMemcpyAsync(emb_host, emb_.p, EMB_DIM * 4, cudaMemcpyDeviceToHost, stream_);
    return sync_check(stream_, "time_embedding");
}

int DitB200::linear(const float* x, int M, int K, const float* W, int N, const float* bias, float* y) {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    if (!x || !W || !y || M <= 0 || K <= 0 || N <= 0) return fail(ERR_ARG, "bad linear arguments");
    cudaSetDevice(dev_);
    const int ld = (K + 7) / 8 * 8;   // row stride padded to 16 bytes for TMA
    const size_t ab = act_bytes(act_);
    DevBuf dx, dw, dxa, dwa, db, dy;
    int rc;
    if ((rc = cuda_check(dx.ensure((size_t)M * K * 4), "cudaMalloc"))) return rc;
    if ((rc = cuda_check(dw.ensure((size_t)N * K * 4), "cudaMalloc"))) return rc;
    if ((rc = cuda_check(dxa.ensure((size_t)M * ld * ab), "cudaMalloc"))) return rc;
    if ((rc = cuda_check(dwa.ensure((size_t)N * ld * ab), "cudaMalloc"))) return rc;
    if ((rc = cuda_check(dy.ensure((size_t)M * N * 4), "cudaMalloc"))) return rc;
    cudaMemcpyAsync(dx.p, x, (size_t)M * K * 4, cudaMemcpyHostToDevice, stream_);
    cudaMemcpyAsync(dw.p, W, (size_t)N * K * 4, cudaMemcpyHostToDevice, stream_);
    if (bias) {
        if ((rc = cuda_check(db.ensure((size_t)N * 4), "cudaMalloc"))) return rc;
        cudaMemcpyAsync(db.p, bias, (size_t)N * 4, cudaMemcpyHostToDevice, stream_);
    }
    pad_convert_rows(dx.as<float>(), M, K, dxa.p, ld, act_, stream_);
    pad_convert_rows(dw.as<float>(), N, K, dwa.p, ld, act_, stream_);
    Linear L;
    L.t = act_; L.out = N; L.in = K; L.ld = ld;
    L.w = std::move(dwa);
    L.b = std::move(db);
    if (act_ == ACT_F32 && tf32x3_ && K % 32 == 0) {
        if ((rc = cuda_check(L.w2.ensure((size_t)N * 2 * K * 4), "cudaMalloc"))) return rc;
        split_tf32(L.w.as<float>(), ld, N, K, L.w2.as<float>(), 2 * K, stream_);
        if ((rc = cuda_check(A2_.ensure((size_t)M * 2 * K * 4), "cudaMalloc"))) return rc;
    }
    GemmEpi e; e.mode = EPI_STORE; e.bias = L.bias(); e.out = dy.p; e.ldo = N; e.out_t = ACT_F32;
    gemm(dxa.p, ld, L, M, e, stream_);
    fold_status(stream_);
    cudaMemcpyAsync(y, dy.p, (size_t)M * N * 4, cudaMemcpyDeviceToHost, stream_);
    if ((rc = sync_check(stream_, "linear"))) return rc;
    return take_status(stream_, "linear");
}

int DitB200::linear_bf16_dev(const void* x, int M, int K, const void* W, int N, const float* bias, void* y,
                             cudaStream_t s) {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    if (!x || !W || !y || M <= 0 || K <= 0 || N <= 0) return fail(ERR_ARG, "bad linear arguments");
    if (K % 64 || N % 32 || ((uintptr_t)x & 15) || ((uintptr_t)W & 15) || ((uintptr_t)y & 15) || ((uintptr_t)bias & 15))
        return fail(ERR_ARG, "the device bf16 Linear needs K % 64 == 0, N % 32 == 0 and 16-byte aligned buffers");
    if (!gemm_tc_supported(M, N, K, K, K)) return fail(ERR_UNSUPPORTED, "shape not supported by the tcgen05 GEMM");
    cudaSetDevice(dev_);
    GemmEpi e;
    e.mode = EPI_STORE; e.bias = bias; e.out = y; e.ldo = N; e.out_t = ACT_BF16;
    if (gemm_tc(x, K, W, K, M, N, K, e, s, &launches_)) return fail(ERR_UNSUPPORTED, "tcgen05 GEMM launch rejected");
    fold_status(s);
    return cuda_check(cudaGetLastError(), "linear_bf16_dev");
}

int DitB200::ada_compose(const float* emb_host, float* out_host) {
    if (!weights_) return fail(ERR_STATE, "weights not loaded");
    cudaSetDevice(dev_);
    cudaMemcpyAsync(emb_.p, emb_host, EMB_DIM * 4, cudaMemcpyHostToDevice, stream_);
    s2b::ada_compose(emb_.as<float>(), branch_.as<float>(), NUM_LAYERS * 12 + 2, ada_.as<float>(), stream_);
    cudaMemcpyAsync(out_host, ada_.p, (size_t)(NUM_LAYERS * 12 + 2) * DIM * 4, cudaMemcpyDeviceToHost, stream_);
    return sync_check(stream_, "ada_compose");
}

// ------------------------------------------------------------------ AWA operator
int DitB200::awa_set_geometry(int win_type, const WinGeom& win) {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    if (win_type != 0 && win_type != 1) return fail(ERR_ARG, "win_type must be 0 or 1");
    cudaSetDevice(dev_);
    return upload_geom(awa_geom_[win_type], win, -1);
}

int DitB200::awa_run(GeomDev& G, const float* vqkv, const float* tqkv, const float* nqv, const float* nkv,
                     const float* nqt, const float* nkt, int Lv, int TXT, float eps, float* vid_out, float* txt_out,
                     cudaStream_t user) {
    if (!G.ready) return fail(ERR_STATE, "AWA geometry not set");
    if (Lv != G.view.Lv || TXT != G.view.TXT || TXT <= 0) return fail(ERR_ARG, "Lv/TXT do not match the geometry");
    if (G.view.nwin <= 0) return fail(ERR_ARG, "no windows");
    const size_t pb = attn_elem_bytes(), sumS = (size_t)G.view.sumS;
    DevBuf q, k, v, tw;
    int rc;
    if ((rc = cuda_check(q.ensure(sumS * DIM * pb), "cudaMalloc"))) return rc;
    if ((rc = cuda_check(k.ensure(sumS * DIM * pb), "cudaMalloc"))) return rc;
    if ((rc = cuda_check(v.ensure(sumS * DIM * pb), "cudaMalloc"))) return rc;
    if ((rc = cuda_check(tw.ensure((size_t)G.view.nwin * TXT * DIM * 4), "cudaMalloc"))) return rc;
    // tokens outside every window read 0 (reference awa_init.comp)
    if (!G.tab.covers_all) cudaMemsetAsync(vid_out, 0, (size_t)Lv * DIM * 4, user);
    if (attn_split3_) {
        awa_pack_split3(vqkv, tqkv, ACT_F32, QKV, G.view, nqv, nkv, nqt, nkt, eps, q.p, k.p, v.p, user);
        if (awa_attend_split3(q.p, k.p, v.p, G.view, 1.0f / sqrtf((float)HEAD_D), vid_out, DIM, ACT_F32,
                              tw.as<float>(), user))
            return fail(ERR_CUDA, "fp32 tensor-core attention: tensor maps could not be encoded");
    } else {
        awa_pack(vqkv, tqkv, ACT_F32, QKV, G.view, nqv, nkv, nqt, nkt, eps, q.p, k.p, v.p, act_, user);
        if (awa_attend(q.p, k.p, v.p, act_, G.view, 1.0f / sqrtf((float)HEAD_D), vid_out, DIM, ACT_F32, tw.as<float>(),
                       user, nullptr))
            return fail(ERR_CUDA, "bf16 tensor-core attention: tensor maps could not be encoded");
    }
    awa_coalesce(tw.as<float>(), G.view.nwin, TXT, txt_out, DIM, ACT_F32, user);
    fold_status(user);
    if ((rc = cuda_check(cudaGetLastError(), "awa launch"))) return rc;
    // the scratch buffers above must outlive the enqueued kernels
    if ((rc = sync_check(user, "awa"))) return rc;
    return take_status(user, "awa");
}

int DitB200::awa_forward_dev(int win_type, const float* vqkv, const float* tqkv, const float* nqv, const float* nkv,
                             const float* nqt, const float* nkt, int Lv, int TXT, float eps, float* vid_out,
                             float* txt_out, cudaStream_t user) {
    if (win_type != 0 && win_type != 1) return fail(ERR_ARG, "win_type must be 0 or 1");
    if (!vqkv || !tqkv || !nqv || !nkv || !nqt || !nkt || !vid_out || !txt_out) return fail(ERR_ARG, "null buffer");
    for (const void* b : {(const void*)vqkv, (const void*)tqkv, (const void*)nqv, (const void*)nkv, (const void*)nqt,
                          (const void*)nkt, (const void*)vid_out, (const void*)txt_out})
        if ((uintptr_t)b & 15) return fail(ERR_ARG, "device buffers must be 16-byte aligned");
    cudaSetDevice(dev_);
    return awa_run(awa_geom_[win_type], vqkv, tqkv, nqv, nkv, nqt, nkt, Lv, TXT, eps, vid_out, txt_out, user);
}

size_t awa_static_bytes_needed(const AwaDev& g, ActT pt);
size_t awa_static_capacity();
int awa_forward_static(const float* vqkv, const float* tqkv, const AwaDev& g, const float* nqv, const float* nkv,
                       const float* nqt, const float* nkt, float eps, float scale, ActT pt, float* vid_out,
                       float* txt_out, cudaStream_t s);

int DitB200::awa_forward_dev_static(int win_type, const float* vqkv, const float* tqkv, const float* nqv,
                                    const float* nkv, const float* nqt, const float* nkt, int Lv, int TXT, float eps,
                                    float* vid_out, float* txt_out, cudaStream_t user) {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    if (win_type != 0 && win_type != 1) return fail(ERR_ARG, "win_type must be 0 or 1");
    if (!vqkv || !tqkv || !nqv || !nkv || !nqt || !nkt || !vid_out || !txt_out) return fail(ERR_ARG, "null buffer");
    for (const void* b : {(const void*)vqkv, (const void*)tqkv, (const void*)nqv, (const void*)nkv, (const void*)nqt,
                          (const void*)nkt, (const void*)vid_out, (const void*)txt_out})
        if ((uintptr_t)b & 15) return fail(ERR_ARG, "device buffers must be 16-byte aligned");
    const GeomDev& G = awa_geom_[win_type];
    if (!G.ready) return fail(ERR_STATE, "AWA geometry not set (s2b_awa_set_geometry)");
    if (Lv != G.view.Lv || TXT != G.view.TXT || TXT <= 0) return fail(ERR_ARG, "Lv/TXT do not match the geometry");
    if (G.view.nwin <= 0) return fail(ERR_ARG, "no windows");
    const size_t need = awa_static_bytes_needed(G.view, act_), cap = awa_static_capacity();
    if (need > cap)
        return fail(ERR_ARG, "geometry needs " + std::to_string(need) + " bytes of scratch; the static scratch holds " +
                                 std::to_string(cap) + " bytes");
    cudaSetDevice(dev_);
    if (!G.tab.covers_all) cudaMemsetAsync(vid_out, 0, (size_t)Lv * DIM * 4, user);
    const int rc = awa_forward_static(vqkv, tqkv, G.view, nqv, nkv, nqt, nkt, eps, 1.0f / sqrtf((float)HEAD_D), act_,
                                      vid_out, txt_out, user);
    if (rc == -1) return fail(ERR_ARG, "geometry does not fit the static scratch");
    if (rc == -2) return fail(ERR_CUDA, "bf16 tensor-core attention: tensor maps could not be encoded");
    if (rc) return cuda_check((cudaError_t)rc, "static scratch address");
    fold_status(user);
    return cuda_check(cudaGetLastError(), "awa_forward_dev_static");
}

int DitB200::awa_forward(const float* vqkv, const float* tqkv, const WinGeom& win, const float* nqv, const float* nkv,
                         const float* nqt, const float* nkt, int Lv, int TXT, float eps, float* vid_out,
                         float* txt_out) {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    if (!vqkv || !tqkv || !nqv || !nkv || !nqt || !nkt || !vid_out || !txt_out) return fail(ERR_ARG, "null buffer");
    if (Lv != win.tokens()) return fail(ERR_ARG, "Lv does not match the window grid");
    if (TXT != win.txt_len || TXT <= 0) return fail(ERR_ARG, "TXT does not match win.txt_len");
    cudaSetDevice(dev_);
    GeomDev g;
    if (int rc = upload_geom(g, win, TXT)) return rc;
    DevBuf dvq, dtq, dn, dvo, dto;
    int rc;
    if ((rc = cuda_check(dvq.ensure((size_t)Lv * QKV * 4), "cudaMalloc"))) return rc;
    if ((rc = cuda_check(dtq.ensure((size_t)TXT * QKV * 4), "cudaMalloc"))) return rc;
    if ((rc = cuda_check(dn.ensure(4 * HEAD_D * 4), "cudaMalloc"))) return rc;
    if ((rc = cuda_check(dvo.ensure((size_t)Lv * DIM * 4), "cudaMalloc"))) return rc;
    if ((rc = cuda_check(dto.ensure((size_t)TXT * DIM * 4), "cudaMalloc"))) return rc;
    cudaMemcpyAsync(dvq.p, vqkv, (size_t)Lv * QKV * 4, cudaMemcpyHostToDevice, stream_);
    cudaMemcpyAsync(dtq.p, tqkv, (size_t)TXT * QKV * 4, cudaMemcpyHostToDevice, stream_);
    const float* norms[4] = {nqv, nkv, nqt, nkt};
    for (int i = 0; i < 4; i++)
        cudaMemcpyAsync(dn.as<float>() + i * HEAD_D, norms[i], HEAD_D * 4, cudaMemcpyHostToDevice, stream_);
    rc = awa_run(g, dvq.as<float>(), dtq.as<float>(), dn.as<float>(), dn.as<float>() + HEAD_D,
                 dn.as<float>() + 2 * HEAD_D, dn.as<float>() + 3 * HEAD_D, Lv, TXT, eps, dvo.as<float>(),
                 dto.as<float>(), stream_);
    if (rc) return rc;
    cudaMemcpyAsync(vid_out, dvo.p, (size_t)Lv * DIM * 4, cudaMemcpyDeviceToHost, stream_);
    cudaMemcpyAsync(txt_out, dto.p, (size_t)TXT * DIM * 4, cudaMemcpyDeviceToHost, stream_);
    return sync_check(stream_, "awa_forward");
}

}  // namespace s2b
