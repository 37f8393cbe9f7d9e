// shard_plan.cpp -- window ownership and residual exchange plan (see shard_plan.h).
#include "shard_plan.h"
#include "s2b_common.h"
#include <algorithm>
#include <limits>

namespace s2b {

// Contiguous split of costs c[0..n) into k non-empty runs minimising the
// largest run sum (exact dynamic programme; n is at most a few hundred).
static std::vector<int> split_runs(const std::vector<double>& c, int k) {
    const int n = (int)c.size();
    std::vector<double> pre(n + 1, 0.0);
    for (int i = 0; i < n; i++) pre[i + 1] = pre[i] + c[i];
    const double INF = std::numeric_limits<double>::infinity();
    // best[j][i]: first i items in j runs; arg[j][i]: start of the last run
    std::vector<std::vector<double>> best(k + 1, std::vector<double>(n + 1, INF));
    std::vector<std::vector<int>> arg(k + 1, std::vector<int>(n + 1, 0));
    best[0][0] = 0.0;
    for (int j = 1; j <= k; j++)
        for (int i = j; i <= n - (k - j); i++)
            for (int m = j - 1; m < i; m++) {
                const double v = std::max(best[j - 1][m], pre[i] - pre[m]);
                if (v < best[j][i]) { best[j][i] = v; arg[j][i] = m; }
            }
    std::vector<int> b(k + 1);
    b[k] = n;
    for (int j = k, i = n; j > 0; j--) { i = arg[j][i]; b[j - 1] = i; }
    return b;
}

bool make_shard_plan(const WinGeom& ns, const WinTables& tns, const WinGeom& sh, const WinTables& tsh, int world,
                     int rank, ShardPlan& out, const char** why) {
    auto bad = [&](const char* m) { if (why) *why = m; return false; };
    if (world < 1 || rank < 0 || rank >= world) return bad("rank outside [0, world)");
    if (ns.tokens() != sh.tokens() || ns.txt_len != sh.txt_len) return bad("geometries disagree on the grid");
    if (!tns.covers_all || !tsh.covers_all) return bad("windows must tile the token grid exactly");
    if (ns.nwin() < world || sh.nwin() < world) return bad("fewer windows than ranks");
    const int Lv = ns.tokens(), TXT = ns.txt_len;
    const WinGeom* g[2] = {&ns, &sh};
    const WinTables* tb[2] = {&tns, &tsh};
    // per vid token and layer: qkv + out + SwiGLU in + out projections
    const double gemm_per_tok = 2.0 * (QKV + DIM + 2.0 * MLP_DIM + MLP_DIM) * DIM;
    out = ShardPlan();
    out.world = world; out.rank = rank; out.Lv = Lv;
    std::vector<int> owner[2], lrow[2];
    for (int p = 0; p < 2; p++) {
        const int nwin = g[p]->nwin();
        std::vector<double> cost(nwin);
        for (int w = 0; w < nwin; w++) {
            const double f = tb[p]->cumf[w + 1] - tb[p]->cumf[w], S = f + TXT;
            cost[w] = f * gemm_per_tok + 4.0 * S * S * HEAD_D * HEADS;
        }
        out.bounds[p] = split_runs(cost, world);
        owner[p].assign(Lv, -1);
        lrow[p].assign(Lv, -1);
        for (int r = 0; r < world; r++) {
            const int f0 = tb[p]->cumf[out.bounds[p][r]], f1 = tb[p]->cumf[out.bounds[p][r + 1]];
            for (int gi = f0; gi < f1; gi++) {
                const int tok = tb[p]->vidx[gi];
                owner[p][tok] = r;
                lrow[p][tok] = gi - f0;
                if (r == rank) out.tokens[p].push_back(tok);
            }
        }
    }
    out.owner[0] = owner[0]; out.owner[1] = owner[1];
    out.lrow[0] = lrow[0]; out.lrow[1] = lrow[1];
    for (int p = 0; p < 2; p++) {
        const int q1 = 1 - p;
        std::vector<std::vector<int>> snd(world), rcv(world);
        for (int tok = 0; tok < Lv; tok++) {
            if (owner[p][tok] == rank) snd[owner[q1][tok]].push_back(lrow[p][tok]);
            if (owner[q1][tok] == rank) rcv[owner[p][tok]].push_back(lrow[q1][tok]);
        }
        out.send_off[p].assign(world + 1, 0);
        out.recv_off[p].assign(world + 1, 0);
        for (int q = 0; q < world; q++) {
            out.send_idx[p].insert(out.send_idx[p].end(), snd[q].begin(), snd[q].end());
            out.recv_idx[p].insert(out.recv_idx[p].end(), rcv[q].begin(), rcv[q].end());
            out.send_off[p][q + 1] = (int)out.send_idx[p].size();
            out.recv_off[p][q + 1] = (int)out.recv_idx[p].size();
        }
    }
    return true;
}

}  // namespace s2b
