// dit_shard.h -- per-context state of the multi-GPU window-sharded forward.
#pragma once
#include "dit_b200.h"
#include "shard_plan.h"
#include <nccl.h>

namespace s2b {

// NCCL entry points, resolved at run time from libnccl.so.2 (the copy the
// process already has loaded, if any) so the library itself does not link
// NCCL and single-GPU use never needs it.
struct NcclLib {
    void* handle = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
};
// Loads the library once per process; null (and *err set) when it is missing.
const NcclLib* nccl_lib(std::string* err);

struct DitB200::ShardState {
    int world = 1, rank = 0;
    const NcclLib* nl = nullptr;
    ncclComm_t comm = nullptr;
    int dev = -1;

    // plan of the current window geometry (rebuilt when set_windows runs)
    int plan_gen = -1, Lv = 0, TXT = 0;
    ShardPlan plan;
    GeomDev geom[2];            // this rank's windows, local packed rows
    int nwin_global[2] = {0, 0};

    // residual of parity p's layout: [n_local(p) vid rows | TXT txt rows] x 2560 fp32
    DevBuf X[2];
    DevBuf Xn, QKV, ATT, Hs, Qp, Kp, Vp, TOUTW, TXTSUM, SQ;
    DevBuf VIDIN, VIDLOC, VPIN, TXTIN, TIN, SRLOC, SRFULL;
    DevBuf tok0, tok1;          // init gather / final scatter token lists
    // exchange after a layer of parity p: rows to other ranks (gathered into
    // XSEND in rank order), rows from other ranks (XRECV, scattered), and this
    // rank's own rows that only change position
    DevBuf send_ns[2], recv_ns[2], self_src[2], self_dst[2];
    std::vector<int> send_ns_off[2], recv_ns_off[2];
    int n_self[2] = {0, 0};
    DevBuf XSEND, XRECV;

    // Exchanges over NVLink peer memory (k_shard.cu) instead of NCCL calls,
    // when every pair of ranks can map each other's memory.
    bool p2p = false;
    ActT act = ACT_BF16;            // activation type of the context
    DevBuf TXTP, FLAGS, EPOCH;      // [2][TXT*2560] partials, flags, this forward's call number
    uint32_t calls = 0;             // shard-forward calls on this rank, failed ones included
    uint64_t wait_ns = 4000000000ull;   // bound of every flag wait and of the NCCL watchdog
    bool aborted = false;           // the watchdog aborted the communicator: shard_init again
    ShardPeers peers;
    std::vector<void*> opened;      // IPC mappings of the other ranks' buffers
    DevBuf xr_src[2], xr_rank[2], xr_dst[2];   // peer-store exchange lists per parity
    int n_xr[2] = {0, 0};
    void close_peers();

    // the captured shard forward (kernels + NCCL calls) of the current plan
    cudaGraphExec_t gexec = nullptr;
    int graph_gen = -1, graph_launches = 0;

    int nccl_check(ncclResult_t r, const char* what, std::string& err) const;
    ~ShardState();
};

}  // namespace s2b
