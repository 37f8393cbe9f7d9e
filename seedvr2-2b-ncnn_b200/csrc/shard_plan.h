// shard_plan.h -- window ownership and residual exchange plan of the
// window-sharded (image mode) forward.  Pure host code.
//
// The reference runs a frame on one device (src/dit_vk.cpp:481-676, one
// DitVk::forward_latent per frame).  Window sharding is this library's
// multi-GPU mode: every rank owns a contiguous run of windows per layer
// parity (non-shifted windows on even layers, shifted ones on odd layers,
// src/dit_vk.cpp:512-513), keeps the residual rows of the grid tokens in
// its windows in window-packed order, and replicates the txt rows.  Between
// two layers the ownership changes from one parity to the other, so the
// rows whose owner changes move between ranks.
#pragma once
#include "awa_geometry.h"
#include <vector>

namespace s2b {

struct ShardPlan {
    int world = 1, rank = 0, Lv = 0;
    // bounds[p][r] .. bounds[p][r+1]: windows of rank r for parity p
    std::vector<int> bounds[2];
    // tokens[p][j]: grid token of this rank's local residual row j in parity
    // p's layout (window-packed order of its windows)
    std::vector<int> tokens[2];
    // transition from parity p's layout to parity 1-p's (after a layer of
    // parity p): this rank sends its local rows send_idx[p][send_off[p][q] ..
    // send_off[p][q+1]) to rank q and writes what rank q sends into its new
    // local rows recv_idx[p][recv_off[p][q] .. recv_off[p][q+1]).  Within a
    // (sender, receiver) pair rows go in ascending grid-token order, which
    // both sides derive independently.  q == rank is the local move.
    std::vector<int> send_idx[2], send_off[2], recv_idx[2], recv_off[2];
    // every rank's view: owner[p][tok] = rank holding grid token tok in parity
    // p's layout, lrow[p][tok] = its local row there
    std::vector<int> owner[2], lrow[2];
    int n_local(int p) const { return (int)tokens[p].size(); }
};

// Splits each parity's windows into `world` contiguous runs minimising the
// largest per-rank cost (GEMM work per vid token plus the window's attention
// work) and derives the exchange plan of rank `rank`.  Both geometries must
// tile the same grid (tables built by build_tables with covers_all) and have
// at least `world` windows.
bool make_shard_plan(const WinGeom& ns, const WinTables& tns, const WinGeom& sh, const WinTables& tsh, int world,
                     int rank, ShardPlan& out, const char** why);

}  // namespace s2b
