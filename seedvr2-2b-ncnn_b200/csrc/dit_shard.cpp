// dit_shard.cpp -- multi-GPU window-sharded forward (NCCL over NVLink).
//
// One process and one context per GPU.  Every rank holds all weights and
// runs the per-token work (norms, GEMMs, gates) only for the grid tokens of
// the windows it owns in the current layer's parity (shard_plan.h); the 58
// txt rows are replicated.  Per layer there are two exchanges:
//   * the txt outputs of the attention: each rank sums its windows' txt
//     outputs, one ncclAllReduce(sum) of [TXT, 2560] fp32 adds the ranks'
//     partial sums, and the total is divided by the global window count
//     (the cross-window mean of src/dit_vk.cpp:435-437);
//   * the residual rows whose owner changes between the non-shifted and the
//     shifted windows: grouped ncclSend / ncclRecv between the ranks that
//     exchange rows, with gather / scatter kernels on either side.
// The vid input patches are replicated on every rank (each gathers its own
// rows) and the [Lv, 64] output is assembled by an all-reduce of zero-filled
// full-size buffers, so every rank returns the whole result.
#include "dit_shard.h"
#include <dlfcn.h>
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

namespace s2b {

const NcclLib* nccl_lib(std::string* err) {
    static NcclLib lib;
    static std::once_flag once;
    static std::string load_err;
    std::call_once(once, [] {
        const char* name = std::getenv("S2B_NCCL_LIB");
        void* h = dlopen(name && *name ? name : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* e = dlerror();
            load_err = std::string("cannot load NCCL: ") + (e ? e : "unknown dlopen error");
            return;
        }
        bool ok = true;
        auto sym = [&](auto& fn, const char* n) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, n));
            if (!fn) ok = false;
        };
        sym(lib.GetUniqueId, "ncclGetUniqueId");
        sym(lib.CommInitRank, "ncclCommInitRank");
        sym(lib.CommDestroy, "ncclCommDestroy");
        sym(lib.AllReduce, "ncclAllReduce");
        sym(lib.Send, "ncclSend");
        sym(lib.Recv, "ncclRecv");
        sym(lib.GroupStart, "ncclGroupStart");
        sym(lib.GroupEnd, "ncclGroupEnd");
        sym(lib.AllGather, "ncclAllGather");
        sym(lib.GetErrorString, "ncclGetErrorString");
        sym(lib.CommGetAsyncError, "ncclCommGetAsyncError");
        sym(lib.CommAbort, "ncclCommAbort");
        if (!ok) {
            load_err = "the NCCL library lacks an entry point this build needs";
            dlclose(h);
            return;
        }
        lib.handle = h;
    });
    if (!lib.handle) {
        if (err) *err = load_err;
        return nullptr;
    }
    return &lib;
}

int DitB200::ShardState::nccl_check(ncclResult_t r, const char* what, std::string& err) const {
    if (r == ncclSuccess) return OK;
    err = std::string(what) + ": " + (nl && nl->GetErrorString ? nl->GetErrorString(r) : "NCCL error");
    return ERR_NCCL;
}

void DitB200::ShardState::close_peers() {
    for (void* ptr : opened) cudaIpcCloseMemHandle(ptr);
    opened.clear();
    p2p = false;
}

DitB200::ShardState::~ShardState() {
    if (dev >= 0) cudaSetDevice(dev);
    // a graph holding NCCL calls goes before its communicator
    if (gexec) cudaGraphExecDestroy(gexec);
    close_peers();
    if (comm && nl) nl->CommDestroy(comm);
}

int DitB200::shard_init(const uint8_t id[128], int world, int rank) {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    if (!weights_ || layer_lo_ != 0 || layer_hi_ != NUM_LAYERS)
        return fail(ERR_STATE, "window-sharded mode needs all 32 layers loaded");
    if (!id || world < 1 || rank < 0 || rank >= world) return fail(ERR_ARG, "rank outside [0, world)");
    std::string e;
    const NcclLib* nl = nccl_lib(&e);
    if (!nl) return fail(ERR_NCCL, e);
    cudaSetDevice(dev_);
    shard_.reset();
    auto S = std::make_unique<ShardState>();
    S->world = world; S->rank = rank; S->nl = nl; S->dev = dev_;
    // S2B_SHARD_WAIT_MS: bound of every peer-flag wait and of the NCCL-path
    // watchdog (default 4000 ms; a 1080p forward takes ~20 ms)
    if (const char* w = std::getenv("S2B_SHARD_WAIT_MS")) {
        const long ms = std::strtol(w, nullptr, 10);
        if (ms > 0) S->wait_ns = (uint64_t)ms * 1000000ull;
    }
    ncclUniqueId uid;
    static_assert(sizeof(uid.internal) == 128, "ncclUniqueId is 128 bytes");
    std::memcpy(uid.internal, id, 128);
    if (int rc = S->nccl_check(nl->CommInitRank(&S->comm, world, uid, rank), "ncclCommInitRank", err)) {
        S->comm = nullptr;
        return rc;
    }
    shard_ = std::move(S);
    return OK;
}

int DitB200::shard_prepare(int Lv, int TXT) {
    if (!shard_) return fail(ERR_STATE, "shard_init has not run");
    if (!weights_) return fail(ERR_STATE, "weights not loaded");
    if (!geom_[0].ready || !geom_[1].ready) return fail(ERR_STATE, "windows not set");
    if (Lv != geom_[0].view.Lv || TXT != geom_[0].view.TXT || TXT <= 0) return fail(ERR_ARG, "Lv/TXT do not match the windows");
    ShardState& S = *shard_;
    if (S.plan_gen == geom_gen_) return OK;
    const char* why = nullptr;
    ShardPlan plan;
    if (!make_shard_plan(geom_[0].host, geom_[0].tab, geom_[1].host, geom_[1].tab, S.world, S.rank, plan, &why))
        return fail(ERR_ARG, std::string("window sharding: ") + why);
    // local geometries: this rank's windows, vid rows numbered in local packed order
    for (int p = 0; p < 2; p++) {
        const GeomDev& G = geom_[p];
        const int a = plan.bounds[p][S.rank], b = plan.bounds[p][S.rank + 1];
        const int f0 = G.tab.cumf[a], f1 = G.tab.cumf[b], n = f1 - f0;
        WinGeom lw;
        lw.t = G.host.t; lw.h = G.host.h; lw.w = G.host.w; lw.txt_len = TXT;
        lw.win.assign(G.host.win.begin() + a, G.host.win.begin() + b);
        lw.vid_freq.assign(G.host.vid_freq.begin() + (size_t)f0 * ROPE_ROT, G.host.vid_freq.begin() + (size_t)f1 * ROPE_ROT);
        lw.txt_freq.assign(G.host.txt_freq.begin() + (size_t)a * TXT * ROPE_ROT,
                           G.host.txt_freq.begin() + (size_t)b * TXT * ROPE_ROT);
        WinTables lt;
        lt.sumf = n;
        lt.covers_all = true;
        lt.vidx.resize(n);
        for (int j = 0; j < n; j++) lt.vidx[j] = j;
        std::vector<int> tp(4 * (size_t)std::max(n, 1), -1);
        for (int w = a; w <= b; w++) {
            lt.cumf.push_back(G.tab.cumf[w] - f0);
            lt.cums.push_back(G.tab.cums[w] - G.tab.cums[a]);
        }
        for (int w = a; w < b; w++) {
            lt.maxS = std::max(lt.maxS, G.tab.cums[w + 1] - G.tab.cums[w]);
            for (int gi = G.tab.cumf[w]; gi < G.tab.cumf[w + 1]; gi++) {
                const int j = gi - f0, tok = G.tab.vidx[gi];
                tp[4 * (size_t)j] = j;
                tp[4 * (size_t)j + 1] = w - a;
                tp[4 * (size_t)j + 2] = G.tokpos_host[4 * (size_t)tok + 2];
                tp[4 * (size_t)j + 3] = G.tokpos_host[4 * (size_t)tok + 3];
            }
        }
        if (int rc = upload_geom_with(S.geom[p], lw, lt, tp, G.structured, G.npos, n)) return rc;
        S.nwin_global[p] = G.view.nwin;
    }
    const int n0 = plan.n_local(0), n1 = plan.n_local(1), nmax = std::max(n0, n1);
    const size_t Mmax = (size_t)nmax + TXT, ab = act_bytes(act_);
    size_t sumS = 0, nwT = 0;
    for (int p = 0; p < 2; p++) {
        sumS = std::max(sumS, (size_t)S.geom[p].view.sumS);
        nwT = std::max(nwT, (size_t)S.geom[p].view.nwin * TXT);
    }
    // exchange index lists
    size_t nsend = 0, nrecv = 0;
    std::vector<int> snd[2], rcv[2], ssrc[2], sdst[2];
    for (int p = 0; p < 2; p++) {
        const int me = S.rank;
        S.send_ns_off[p].assign(S.world + 1, 0);
        S.recv_ns_off[p].assign(S.world + 1, 0);
        for (int q = 0; q < S.world; q++) {
            const int s0 = plan.send_off[p][q], s1 = plan.send_off[p][q + 1];
            const int r0 = plan.recv_off[p][q], r1 = plan.recv_off[p][q + 1];
            if (q == me) {
                ssrc[p].assign(plan.send_idx[p].begin() + s0, plan.send_idx[p].begin() + s1);
                sdst[p].assign(plan.recv_idx[p].begin() + r0, plan.recv_idx[p].begin() + r1);
            } else {
                snd[p].insert(snd[p].end(), plan.send_idx[p].begin() + s0, plan.send_idx[p].begin() + s1);
                rcv[p].insert(rcv[p].end(), plan.recv_idx[p].begin() + r0, plan.recv_idx[p].begin() + r1);
            }
            S.send_ns_off[p][q + 1] = (int)snd[p].size();
            S.recv_ns_off[p][q + 1] = (int)rcv[p].size();
        }
        if (ssrc[p].size() != sdst[p].size()) return fail(ERR_STATE, "inconsistent local exchange plan");
        S.n_self[p] = (int)ssrc[p].size();
        nsend = std::max(nsend, snd[p].size());
        nrecv = std::max(nrecv, rcv[p].size());
    }
    auto alloc = [&](DevBuf& d, size_t n, const char* what) { return cuda_check(d.ensure(std::max<size_t>(n, 16)), what); };
    auto up = [&](DevBuf& d, const std::vector<int>& v) -> int {
        if (int rc = alloc(d, v.size() * 4, "cudaMalloc(shard index)")) return rc;
        if (v.empty()) return OK;
        return cuda_check(cudaMemcpy(d.p, v.data(), v.size() * 4, cudaMemcpyHostToDevice), "upload shard index");
    };
    int rc;
    if ((rc = alloc(S.X[0], ((size_t)n0 + TXT) * DIM * 4, "cudaMalloc(shard X)"))) return rc;
    if ((rc = alloc(S.X[1], ((size_t)n1 + TXT) * DIM * 4, "cudaMalloc(shard X)"))) return rc;
    if ((rc = alloc(S.Xn, Mmax * DIM * ab, "cudaMalloc(shard Xn)"))) return rc;
    if ((rc = alloc(S.QKV, Mmax * QKV * ab, "cudaMalloc(shard QKV)"))) return rc;
    if ((rc = alloc(S.ATT, Mmax * DIM * ab, "cudaMalloc(shard ATT)"))) return rc;
    if ((rc = alloc(S.Hs, Mmax * MLP_DIM * ab, "cudaMalloc(shard Hs)"))) return rc;
    if ((rc = alloc(S.SQ, Mmax * SQ_SLOTS * 4, "cudaMalloc(shard SQ)"))) return rc;
    if ((rc = alloc(S.Qp, sumS * DIM * attn_elem_bytes(), "cudaMalloc(shard Qp)"))) return rc;
    if ((rc = alloc(S.Kp, sumS * DIM * attn_elem_bytes(), "cudaMalloc(shard Kp)"))) return rc;
    if ((rc = alloc(S.Vp, sumS * DIM * attn_elem_bytes(), "cudaMalloc(shard Vp)"))) return rc;
    if ((rc = alloc(S.TOUTW, nwT * DIM * 4, "cudaMalloc(shard TOUTW)"))) return rc;
    if ((rc = alloc(S.TXTSUM, (size_t)TXT * DIM * 4, "cudaMalloc(shard TXTSUM)"))) return rc;
    if ((rc = alloc(S.VIDIN, (size_t)Lv * PATCH_IN * 4, "cudaMalloc(shard VIDIN)"))) return rc;
    if ((rc = alloc(S.VIDLOC, (size_t)n0 * PATCH_IN * 4, "cudaMalloc(shard VIDLOC)"))) return rc;
    if ((rc = alloc(S.VPIN, (size_t)n0 * PATCH_IN_PAD * ab, "cudaMalloc(shard VPIN)"))) return rc;
    if ((rc = alloc(S.TXTIN, (size_t)TXT * TXT_IN * 4, "cudaMalloc(shard TXTIN)"))) return rc;
    if ((rc = alloc(S.TIN, (size_t)TXT * TXT_IN * ab, "cudaMalloc(shard TIN)"))) return rc;
    if ((rc = alloc(S.SRLOC, (size_t)n1 * OUT_CH * 4, "cudaMalloc(shard SRLOC)"))) return rc;
    if ((rc = alloc(S.SRFULL, (size_t)Lv * OUT_CH * 4, "cudaMalloc(shard SRFULL)"))) return rc;
    if ((rc = alloc(S.XSEND, nsend * DIM * 4, "cudaMalloc(shard XSEND)"))) return rc;
    if ((rc = alloc(S.XRECV, nrecv * DIM * 4, "cudaMalloc(shard XRECV)"))) return rc;
    // [h | g] fp32 staging of the SIMT SwiGLU path (the tcgen05 path fuses it)
    if ((act_ == ACT_F32 || !gemm_tc_supported((int)Mmax, 2 * MLP_DIM, DIM, DIM, DIM)) &&
        (rc = alloc(HG_, Mmax * 2 * MLP_DIM * 4, "cudaMalloc(HG)")))
        return rc;
    if (act_ == ACT_F32 && tf32x3_ && (rc = alloc(A2_, Mmax * 2 * MLP_DIM * 4, "cudaMalloc(A2)"))) return rc;
    if ((rc = up(S.tok0, plan.tokens[0]))) return rc;
    if ((rc = up(S.tok1, plan.tokens[(NUM_LAYERS - 1) % 2]))) return rc;
    for (int p = 0; p < 2; p++) {
        if ((rc = up(S.send_ns[p], snd[p]))) return rc;
        if ((rc = up(S.recv_ns[p], rcv[p]))) return rc;
        if ((rc = up(S.self_src[p], ssrc[p]))) return rc;
        if ((rc = up(S.self_dst[p], sdst[p]))) return rc;
    }
    if ((rc = shard_setup_peers(plan, n0, n1, TXT))) return rc;
    S.plan = std::move(plan);
    S.Lv = Lv; S.TXT = TXT;
    S.plan_gen = geom_gen_;
    return OK;
}

// Maps every rank's txt partials, flags and residual buffers into this rank
// (CUDA IPC handles swapped with one NCCL all-gather) and builds the
// peer-store exchange lists.  All ranks agree on the outcome: if any rank
// cannot map its peers, every rank keeps the NCCL exchanges.
int DitB200::shard_setup_peers(const ShardPlan& plan, int n0, int n1, int TXT) {
    ShardState& S = *shard_;
    S.close_peers();
    const char* env = std::getenv("S2B_SHARD_P2P");
    const bool want = S.world <= 8 && !(env && env[0] == '0');
    int rc;
    if ((rc = cuda_check(S.TXTP.ensure((size_t)2 * TXT * DIM * 4), "cudaMalloc(shard TXTP)"))) return rc;
    if ((rc = cuda_check(S.FLAGS.ensure((size_t)2 * 2 * 8 * 4), "cudaMalloc(shard flags)"))) return rc;
    if ((rc = cuda_check(S.EPOCH.ensure(16), "cudaMalloc(shard epoch)"))) return rc;
    cudaMemset(S.FLAGS.p, 0, S.FLAGS.bytes);
    cudaMemset(S.EPOCH.p, 0, S.EPOCH.bytes);
    // this rank's 5 handles (TXTP, FLAGS, X[0], X[1], SRFULL) + whether it wants peer mode
    constexpr int NH = 5;
    struct Rec { cudaIpcMemHandle_t h[NH]; int want; int pad[15]; };
    static_assert(sizeof(Rec) % 16 == 0, "record size");
    Rec mine;
    std::memset(&mine, 0, sizeof mine);
    mine.want = want ? 1 : 0;
    void* bases[NH] = {S.TXTP.p, S.FLAGS.p, S.X[0].p, S.X[1].p, S.SRFULL.p};
    for (int k = 0; k < NH && mine.want; k++)
        if (cudaIpcGetMemHandle(&mine.h[k], bases[k]) != cudaSuccess) mine.want = 0;
    cudaGetLastError();
    DevBuf dev_recs;
    if ((rc = cuda_check(dev_recs.ensure(sizeof(Rec) * (S.world + 1)), "cudaMalloc(shard handles)"))) return rc;
    cudaMemcpy(dev_recs.as<char>() + sizeof(Rec) * S.world, &mine, sizeof mine, cudaMemcpyHostToDevice);
    if ((rc = S.nccl_check(S.nl->AllGather(dev_recs.as<char>() + sizeof(Rec) * S.world, dev_recs.p, sizeof(Rec),
                                           ncclUint8, S.comm, stream_), "ncclAllGather(handles)", err)))
        return rc;
    std::vector<Rec> recs(S.world);
    if ((rc = cuda_check(cudaMemcpyAsync(recs.data(), dev_recs.p, sizeof(Rec) * S.world, cudaMemcpyDeviceToHost, stream_),
                         "copy handles")))
        return rc;
    cudaStreamSynchronize(stream_);
    bool all = true;
    for (const Rec& r : recs) all = all && r.want;
    int ok = all ? 1 : 0;
    ShardPeers P;
    P.world = S.world; P.rank = S.rank; P.wait_ns = S.wait_ns;
    for (int q = 0; q < S.world && ok; q++) {
        void* ptr[NH];
        for (int k = 0; k < NH; k++) {
            if (q == S.rank) { ptr[k] = bases[k]; continue; }
            if (cudaIpcOpenMemHandle(&ptr[k], recs[q].h[k], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = 0;
                break;
            }
            S.opened.push_back(ptr[k]);
        }
        if (!ok) break;
        P.txtp[q] = (float*)ptr[0]; P.flags[q] = (uint32_t*)ptr[1];
        P.x[0][q] = (float*)ptr[2]; P.x[1][q] = (float*)ptr[3];
        P.sr[q] = (float*)ptr[4];
    }
    // every rank must have mapped every peer
    DevBuf dev_ok;
    if ((rc = cuda_check(dev_ok.ensure(4 * (S.world + 1)), "cudaMalloc(shard ok)"))) return rc;
    cudaMemcpy(dev_ok.as<int>() + S.world, &ok, 4, cudaMemcpyHostToDevice);
    if ((rc = S.nccl_check(S.nl->AllGather(dev_ok.as<int>() + S.world, dev_ok.p, 1, ncclInt32, S.comm, stream_),
                           "ncclAllGather(peer status)", err)))
        return rc;
    std::vector<int> oks(S.world);
    cudaMemcpyAsync(oks.data(), dev_ok.p, 4 * S.world, cudaMemcpyDeviceToHost, stream_);
    if ((rc = cuda_check(cudaStreamSynchronize(stream_), "peer status"))) return rc;
    for (int v : oks) ok = ok && v;
    if (!ok) { S.close_peers(); return OK; }
    S.peers = P;
    // peer-store exchange lists: every local row (vid rows of this rank's
    // windows, then the replicated txt rows) to its owner's row in the next layout
    const int nl[2] = {n0, n1};
    for (int p = 0; p < 2; p++) {
        std::vector<int> src, rnk, dst;
        for (int j = 0; j < nl[p]; j++) {
            const int tok = plan.tokens[p][j];
            src.push_back(j);
            rnk.push_back(plan.owner[1 - p][tok]);
            dst.push_back(plan.lrow[1 - p][tok]);
        }
        for (int t = 0; t < TXT; t++) { src.push_back(nl[p] + t); rnk.push_back(S.rank); dst.push_back(nl[1 - p] + t); }
        S.n_xr[p] = (int)src.size();
        DevBuf* bufs[3] = {&S.xr_src[p], &S.xr_rank[p], &S.xr_dst[p]};
        const std::vector<int>* vals[3] = {&src, &rnk, &dst};
        for (int k = 0; k < 3; k++) {
            if ((rc = cuda_check(bufs[k]->ensure(vals[k]->size() * 4), "cudaMalloc(exchange list)"))) return rc;
            cudaMemcpy(bufs[k]->p, vals[k]->data(), vals[k]->size() * 4, cudaMemcpyHostToDevice);
        }
    }
    S.p2p = true;
    return cuda_check(cudaGetLastError(), "peer setup");
}

// Where layer i's txt partial sum goes: a slot of the peer-visible buffer, or
// the NCCL all-reduce buffer.
static float* shard_txt_partial(void* ctx, int layer) {
    auto* S = static_cast<DitB200::ShardState*>(ctx);
    return S->p2p ? S->TXTP.as<float>() + (size_t)(layer & 1) * S->TXT * DIM : S->TXTSUM.as<float>();
}

// All ranks' partials -> the mean over all windows in att_txt.
static int shard_txt_finish(void* ctx, int layer, void* att_txt, cudaStream_t s) {
    auto* S = static_cast<DitB200::ShardState*>(ctx);
    const float div = (float)S->nwin_global[layer & 1];
    if (S->p2p) {
        shard_txt_reduce(S->peers, S->EPOCH.as<uint32_t>(), layer, S->TXT, div, att_txt, DIM, S->act, s);
        return OK;
    }
    const ncclResult_t r = S->nl->AllReduce(S->TXTSUM.p, S->TXTSUM.p, (size_t)S->TXT * DIM, ncclFloat32, ncclSum,
                                            S->comm, s);
    if (r != ncclSuccess) return ERR_NCCL;
    awa_coalesce_div(S->TXTSUM.as<float>(), 1, S->TXT, att_txt, DIM, S->act, div, s);
    return OK;
}

int DitB200::shard_exchange(int p, cudaStream_t s) {
    ShardState& S = *shard_;
    const int q1 = 1 - p, me = S.rank, TXT = S.TXT;
    float* src = S.X[p].as<float>();
    float* dst = S.X[q1].as<float>();
    const int np = S.plan.n_local(p), nq = S.plan.n_local(q1);
    const int nsend = S.send_ns_off[p][S.world], nrecv = S.recv_ns_off[p][S.world];
    float* xs = S.XSEND.as<float>();
    float* xr = S.XRECV.as<float>();
    copy_rows_f32(src, DIM, S.send_ns[p].as<int>(), xs, DIM, nullptr, nsend, DIM, s);
    copy_rows_f32(src, DIM, S.self_src[p].as<int>(), dst, DIM, S.self_dst[p].as<int>(), S.n_self[p], DIM, s);
    copy_rows_f32(src + (size_t)np * DIM, DIM, nullptr, dst + (size_t)nq * DIM, DIM, nullptr, TXT, DIM, s);
    launches_ += 3;
    if (nsend || nrecv) {
        int rc = S.nccl_check(S.nl->GroupStart(), "ncclGroupStart", err);
        for (int q = 0; q < S.world && !rc; q++) {
            if (q == me) continue;
            const int so = S.send_ns_off[p][q], sc = S.send_ns_off[p][q + 1] - so;
            const int ro = S.recv_ns_off[p][q], rcnt = S.recv_ns_off[p][q + 1] - ro;
            if (sc) rc = S.nccl_check(S.nl->Send(xs + (size_t)so * DIM, (size_t)sc * DIM, ncclFloat32, q, S.comm, s), "ncclSend", err);
            if (!rc && rcnt) rc = S.nccl_check(S.nl->Recv(xr + (size_t)ro * DIM, (size_t)rcnt * DIM, ncclFloat32, q, S.comm, s), "ncclRecv", err);
        }
        const int rc_end = S.nccl_check(S.nl->GroupEnd(), "ncclGroupEnd", err);
        if (rc || rc_end) return ERR_NCCL;
        copy_rows_f32(xr, DIM, nullptr, dst, DIM, S.recv_ns[p].as<int>(), nrecv, DIM, s);
        launches_++;
    }
    return OK;
}

int DitB200::shard_enqueue(cudaStream_t s) {
    ShardState& S = *shard_;
    const int TXT = S.TXT, n0 = S.plan.n_local(0);
    launches_ = 0;
    S.act = act_;
    // vid_in (this rank's patches of the layer-0 layout) and txt_in, src/dit_vk.cpp:494-497
    copy_rows_f32(S.VIDIN.as<float>(), PATCH_IN, S.tok0.as<int>(), S.VIDLOC.as<float>(), PATCH_IN, nullptr, n0,
                  PATCH_IN, s);
    pad_convert_rows(S.VIDLOC.as<float>(), n0, PATCH_IN, S.VPIN.p, PATCH_IN_PAD, act_, s);
    pad_convert_rows(S.TXTIN.as<float>(), TXT, TXT_IN, S.TIN.p, TXT_IN, act_, s);
    launches_ += 3;
    GemmEpi e; e.mode = EPI_STORE; e.out_t = ACT_F32; e.ldo = DIM;
    e.bias = vid_in_.bias(); e.out = S.X[0].p;
    gemm(S.VPIN.p, PATCH_IN_PAD, vid_in_, n0, e, s);
    e.bias = txt_in_.bias(); e.out = S.X[0].as<float>() + (size_t)n0 * DIM;
    gemm(S.TIN.p, TXT_IN, txt_in_, TXT, e, s);
    enqueue_temb(s);
    for (int i = 0; i < NUM_LAYERS; i++) {
        const int p = i % 2;
        LayerBufs B;
        B.X = S.X[p].as<float>(); B.Xn = S.Xn.p; B.QKV = S.QKV.p; B.ATT = S.ATT.p; B.Hs = S.Hs.p;
        B.Qp = S.Qp.p; B.Kp = S.Kp.p; B.Vp = S.Vp.p; B.TOUTW = S.TOUTW.as<float>();
        B.geom[0] = &S.geom[0]; B.geom[1] = &S.geom[1];
        B.txt_partial = shard_txt_partial; B.txt_finish = shard_txt_finish; B.shard_ctx = &S;
        // the MLP norm folds within a layer; the attention norm's operand would have to
        // follow the residual rows through the exchange between layers, so it stays a kernel
        B.SQ = S.SQ.as<float>();
        B.fuse_mlp = norm_fuse_ && shift_ok_;
        if (int rc = enqueue_layer_on(i, S.plan.n_local(p), TXT, s, B)) {
            if (rc == ERR_NCCL) err = "ncclAllReduce of the txt attention sums failed";
            return rc;
        }
        if (i + 1 < NUM_LAYERS) {
            pbeg(KK_EXCHANGE, 0, (double)S.n_xr[p] * DIM * 4, s);
            if (S.p2p) {
                shard_exchange_rows(S.peers, p, S.xr_src[p].as<int>(), S.xr_rank[p].as<int>(), S.xr_dst[p].as<int>(),
                                    S.n_xr[p], S.EPOCH.as<uint32_t>(), i, s);
                launches_ += 2;
            } else if (int rc = shard_exchange(p, s)) {
                return rc;
            }
            pend(s);
        }
    }
    // final norm + vid_out_proj on this rank's rows (src/dit_vk.cpp:657-675),
    // then every rank assembles the whole [Lv, 64] output
    const int pl = (NUM_LAYERS - 1) % 2, nl = S.plan.n_local(pl);
    const float* fin_sc = ada_.as<float>() + (size_t)(NUM_LAYERS * 12) * DIM;
    rmsnorm_mod(S.X[pl].as<float>(), DIM, nl, nl, fin_sc, fin_sc + DIM, nullptr, nullptr, von_w_.as<float>(),
                NORM_EPS, S.Xn.p, DIM, act_, s);
    launches_++;
    GemmEpi f; f.mode = EPI_STORE; f.out_t = ACT_F32; f.ldo = OUT_CH; f.bias = vid_out_.bias(); f.out = S.SRLOC.p;
    gemm(S.Xn.p, DIM, vid_out_, nl, f, s);
    if (S.p2p) {
        // every rank stores its rows into every rank's output (bounded flag wait)
        pbeg(KK_EXCHANGE, 0, (double)nl * OUT_CH * 4 * S.world, s);
        shard_gather_sr(S.peers, S.SRLOC.as<float>(), S.tok1.as<int>(), nl, S.EPOCH.as<uint32_t>(), s);
        pend(s);
        launches_ += 2;
        fold_status(s);
        return OK;
    }
    cudaMemsetAsync(S.SRFULL.p, 0, (size_t)S.Lv * OUT_CH * 4, s);
    copy_rows_f32(S.SRLOC.as<float>(), OUT_CH, nullptr, S.SRFULL.as<float>(), OUT_CH, S.tok1.as<int>(), nl, OUT_CH, s);
    launches_++;
    const int rc = S.nccl_check(S.nl->AllReduce(S.SRFULL.p, S.SRFULL.p, (size_t)S.Lv * OUT_CH, ncclFloat32, ncclSum,
                                                S.comm, s), "ncclAllReduce(sr)", err);
    fold_status(s);
    return rc;
}

// Waits for the context's stream.  On the NCCL path a peer that stops leaves
// an NCCL kernel waiting for good, so the wait is a watchdog: it polls the
// stream and the communicator's asynchronous error, and after S.wait_ns (or on
// an NCCL error) aborts the communicator, which ends the NCCL kernels; the
// shard state then needs shard_init again.
int DitB200::shard_wait(const char* what, bool nccl_in_flight) {
    ShardState* S = shard_.get();
    if (!S || !nccl_in_flight || !S->comm) return sync_check(stream_, what);
    ncclResult_t async_r = ncclSuccess;
    const int r = watch_completion(
        [&] {
            const cudaError_t e = cudaStreamQuery(stream_);
            return e == cudaSuccess ? WATCH_Q_DONE : e == cudaErrorNotReady ? WATCH_Q_PENDING : WATCH_Q_ERROR;
        },
        [&] { return S->nl->CommGetAsyncError(S->comm, &async_r) == ncclSuccess && async_r != ncclSuccess; },
        [&] {
            S->nl->CommAbort(S->comm);
            S->comm = nullptr;
            S->aborted = true;
        },
        S->wait_ns, 200000ull);
    if (r == WATCH_DONE) return sync_check(stream_, what);
    if (r == WATCH_STREAM_ERROR) return sync_check(stream_, what);
    cudaStreamSynchronize(stream_);   // the abort ended the NCCL kernels
    cudaGetLastError();
    return fail(r == WATCH_ASYNC_ERROR ? ERR_NCCL : ERR_TIMEOUT,
                std::string(what) + (r == WATCH_ASYNC_ERROR ? ": NCCL reported an asynchronous error"
                                                            : ": the NCCL exchange did not finish in time") +
                    "; the communicator was aborted (call shard_init again)");
}

void DitB200::shard_invalidate_graph() {
    if (!shard_) return;
    if (shard_->gexec) { cudaGraphExecDestroy(shard_->gexec); shard_->gexec = nullptr; }
    shard_->graph_gen = -1;
}

int DitB200::shard_begin_call() {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    if (!shard_) return fail(ERR_STATE, "shard_init has not run");
    shard_->calls++;     // counted before any check: a failed call still uses its number
    if (shard_->aborted) return fail(ERR_STATE, "the communicator was aborted by the watchdog: call shard_init again");
    return OK;
}

int DitB200::shard_resync() {
    if (dev_ < 0) return fail(ERR_STATE, "context not created");
    if (!shard_ || !shard_->comm) return fail(ERR_STATE, "shard_init has not run (or the communicator was aborted)");
    cudaSetDevice(dev_);
    ShardState& S = *shard_;
    if (int rc = cuda_check(S.EPOCH.ensure(16), "cudaMalloc(shard epoch)")) return rc;
    uint32_t* d = S.EPOCH.as<uint32_t>() + 1;
    set_u32(d, S.calls, stream_);
    if (int rc = S.nccl_check(S.nl->AllReduce(d, d, 1, ncclUint32, ncclMax, S.comm, stream_), "ncclAllReduce(resync)", err))
        return rc;
    uint32_t mx = 0;
    cudaMemcpyAsync(&mx, d, 4, cudaMemcpyDeviceToHost, stream_);
    if (int rc = shard_wait("shard_resync", true)) return rc;
    S.calls = mx;
    return OK;
}

int DitB200::shard_forward(const float* vid_patch, int Lv, const float* txt, int TXT, float t, float* sr_out) {
    if (int rc = shard_begin_call()) return rc;
    if (!vid_patch || !txt || !sr_out) return fail(ERR_ARG, "null buffer");
    cudaSetDevice(dev_);
    if (int rc = shard_prepare(Lv, TXT)) return rc;
    ShardState& S = *shard_;
    if (S.p2p) set_u32(S.EPOCH.as<uint32_t>(), S.calls, stream_);
    float temb[TEMB_IN];
    sinusoidal256(t, temb);
    cudaMemcpyAsync(temb_in_.p, temb, sizeof temb, cudaMemcpyHostToDevice, stream_);
    cudaMemcpyAsync(S.VIDIN.p, vid_patch, (size_t)Lv * PATCH_IN * 4, cudaMemcpyHostToDevice, stream_);
    cudaMemcpyAsync(S.TXTIN.p, txt, (size_t)TXT * TXT_IN * 4, cudaMemcpyHostToDevice, stream_);
    // the per-kernel profile records events around each launch: no graph then
    int rc = prepare_shift(t, stream_);
    if (!rc) rc = prof_on_ ? shard_enqueue(stream_) : shard_capture();
    if (!rc && !prof_on_) rc = cuda_check(cudaGraphLaunch(S.gexec, stream_), "shard graph launch");
    if (rc) {
        shard_wait("shard_forward", !S.p2p);
        return rc;
    }
    cudaMemcpyAsync(sr_out, S.SRFULL.p, (size_t)Lv * OUT_CH * 4, cudaMemcpyDeviceToHost, stream_);
    last_launches_ = (prof_on_ ? launches_ : S.graph_launches) + (S.p2p ? 1 : 0);
    if (int rc = cuda_check(cudaGetLastError(), "kernel launch")) return rc;
    if (int rc = shard_wait("shard_forward", !S.p2p)) return rc;
    return take_status(stream_, "shard_forward");
}

int DitB200::shard_forward_dev(const float* d_vid, int Lv, const float* d_txt, int TXT, float t, float* d_sr,
                               cudaStream_t user) {
    if (int rc = shard_begin_call()) return rc;
    if (!d_vid || !d_txt || !d_sr) return fail(ERR_ARG, "null buffer");
    cudaSetDevice(dev_);
    if (int rc = shard_prepare(Lv, TXT)) return rc;
    ShardState& S = *shard_;
    cudaEvent_t ev_in, ev_out;
    cudaEventCreateWithFlags(&ev_in, cudaEventDisableTiming);
    cudaEventCreateWithFlags(&ev_out, cudaEventDisableTiming);
    cudaEventRecord(ev_in, user);
    cudaStreamWaitEvent(stream_, ev_in, 0);
    float temb[TEMB_IN];
    sinusoidal256(t, temb);
    cudaMemcpyAsync(temb_in_.p, temb, sizeof temb, cudaMemcpyHostToDevice, stream_);
    cudaMemcpyAsync(S.VIDIN.p, d_vid, (size_t)Lv * PATCH_IN * 4, cudaMemcpyDeviceToDevice, stream_);
    cudaMemcpyAsync(S.TXTIN.p, d_txt, (size_t)TXT * TXT_IN * 4, cudaMemcpyDeviceToDevice, stream_);
    int rc = prepare_shift(t, stream_);
    if (!rc) rc = shard_capture();
    if (!rc && S.p2p) set_u32(S.EPOCH.as<uint32_t>(), S.calls, stream_);
    if (!rc) rc = cuda_check(cudaGraphLaunch(S.gexec, stream_), "shard graph launch");
    if (!rc) cudaMemcpyAsync(d_sr, S.SRFULL.p, (size_t)Lv * OUT_CH * 4, cudaMemcpyDeviceToDevice, stream_);
    cudaEventRecord(ev_out, stream_);
    cudaStreamWaitEvent(user, ev_out, 0);
    cudaEventDestroy(ev_in);
    cudaEventDestroy(ev_out);
    last_launches_ = S.graph_launches + (S.p2p ? 1 : 0);
    if (rc) return rc;
    return cuda_check(cudaGetLastError(), "shard_forward_dev");
}

// Captures shard_enqueue (kernels and NCCL calls) once per plan; every rank
// captures the same sequence, so replays stay in step across ranks.
int DitB200::shard_capture() {
    ShardState& S = *shard_;
    if (S.gexec && S.graph_gen == S.plan_gen) return OK;
    if (S.gexec) { cudaGraphExecDestroy(S.gexec); S.gexec = nullptr; }
    cudaGraph_t graph = nullptr;
    if (int rc = cuda_check(cudaStreamBeginCapture(capture_stream(), cudaStreamCaptureModeRelaxed), "begin capture"))
        return rc;
    const int rc = shard_enqueue(capture_stream());
    cudaError_t ce = cudaStreamEndCapture(capture_stream(), &graph);
    if (rc) { if (graph) cudaGraphDestroy(graph); return rc; }
    if (int r = cuda_check(ce, "end capture")) return r;
    ce = cudaGraphInstantiate(&S.gexec, graph, 0);
    cudaGraphDestroy(graph);
    if (int r = cuda_check(ce, "graph instantiate")) { S.gexec = nullptr; return r; }
    S.graph_gen = S.plan_gen;
    S.graph_launches = launches_;
    return OK;
}

}  // namespace s2b

extern "C" int s2b_nccl_unique_id(uint8_t id[128]) {
    if (!id) return s2b::ERR_ARG;
    const s2b::NcclLib* nl = s2b::nccl_lib(nullptr);
    if (!nl) return s2b::ERR_NCCL;
    ncclUniqueId uid;
    if (nl->GetUniqueId(&uid) != ncclSuccess) return s2b::ERR_NCCL;
    std::memcpy(id, uid.internal, 128);
    return s2b::OK;
}
