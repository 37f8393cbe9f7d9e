"""Per-rank bodies of the window-sharded tests (run in spawned processes).

gloo_exchange: replays the residual exchange of the library's shard plan
(s2b_shard_plan) between CPU ranks over gloo, for both layer-parity
transitions, plus the txt partial-sum all-reduce, and records what each rank
ends up holding.

nccl_forward: one rank per GPU, the library's own window-sharded forward
(s2b_shard_init / s2b_shard_forward) on synthetic weights; rank 0 also runs
the single-GPU forward of the same inputs for comparison.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for _p in (os.path.join(ROOT, "seedvr2-2b-ncnn_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)


def gloo_exchange(rank: int, world: int, port: int, grid, out_dir: str):
    import torch
    import torch.distributed as dist
    import s2b
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        T, H, W = grid
        Lv, width = T * H * W, 8
        ns = s2b.make_win(T, H, W, (4, 3, 3), 58, False)
        sh = s2b.make_win(T, H, W, (4, 3, 3), 58, True)
        plan = s2b.shard_plan(ns, sh, world, rank)
        # global residual: row tok holds (tok, tok * 0.5, ...) so misplaced rows show
        glob = (np.arange(Lv, dtype=np.float32)[:, None] * np.linspace(1, 2, width, dtype=np.float32)[None, :])
        cur = torch.from_numpy(glob[plan.tokens[0]].copy())
        held = []
        for p in (0, 1):
            q1 = 1 - p
            nxt = torch.full((len(plan.tokens[q1]), width), -1.0)
            so, si, ro, ri = plan.send_off[p], plan.send_idx[p], plan.recv_off[p], plan.recv_idx[p]
            reqs = []
            for q in range(world):
                rows = torch.from_numpy(si[so[q]:so[q + 1]].astype(np.int64))
                dst = torch.from_numpy(ri[ro[q]:ro[q + 1]].astype(np.int64))
                if q == rank:
                    nxt[dst] = cur[rows]
                    continue
                if len(rows):
                    reqs.append(dist.isend(cur[rows].contiguous(), q))
            for q in range(world):
                if q == rank:
                    continue
                dst = torch.from_numpy(ri[ro[q]:ro[q + 1]].astype(np.int64))
                if len(dst):
                    buf = torch.empty((len(dst), width))
                    dist.recv(buf, q)
                    nxt[dst] = buf
            for r in reqs:
                r.wait()
            held.append(nxt.numpy().copy())
            cur = nxt
        # txt partial sums: each rank sums its windows' contributions, one all-reduce
        nwin0 = int(plan.bounds[0][-1])
        contrib = np.stack([np.full((4,), w + 1.0, np.float32) for w in range(nwin0)])
        a, b = int(plan.bounds[0][rank]), int(plan.bounds[0][rank + 1])
        part = torch.from_numpy(contrib[a:b].sum(0))
        dist.all_reduce(part)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), after0=held[0], after1=held[1],
                 tok0=plan.tokens[0], tok1=plan.tokens[1], txt=part.numpy(), glob=glob)
    finally:
        dist.destroy_process_group()


def nccl_forward(rank: int, world: int, uid: bytes, prec: int, grid, out_dir: str, p2p: bool = True):
    # p2p: the per-layer exchanges through peer-memory kernels (default), else NCCL calls
    os.environ["S2B_SHARD_P2P"] = "1" if p2p else "0"
    import s2b
    T, H, W = grid
    Lv, TXT = T * H * W, 58
    ctx = s2b.DitB200(rank, prec)
    try:
        ctx.init_synth(1234)
        ns = s2b.make_win(T, H, W, (4, 3, 3), TXT, False)
        sh = s2b.make_win(T, H, W, (4, 3, 3), TXT, True)
        ctx.set_windows(ns, sh)
        vid = s2b.patchify_grid(s2b.synth_vid_grid(T, 2 * H, 2 * W, 42))
        txt = s2b.synth_txt(TXT, 7)
        ctx.shard_init(uid, world, rank)
        sr = ctx.shard_forward(vid, Lv, txt, TXT, 1000.0)
        sr2 = ctx.shard_forward(vid, Lv, txt, TXT, 1000.0)
        out = dict(sr=sr, sr2=sr2)
        if rank == 0:
            out["single"] = ctx.forward(vid, Lv, txt, TXT, 1000.0)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **out)
    finally:
        ctx.close()


def timeout_recover(rank: int, world: int, uid: bytes, port: int, grid, out_dir: str):
    """A rank that skips a shard call between steps: its peer's bounded flag
    waits run out (S2B_SHARD_WAIT_MS), the peer's call returns S2B_ERR_TIMEOUT
    (host call) or reports it through s2b_check_errors (_dev call), a call
    made with diverged call numbers fails on both ranks, and after
    s2b_shard_resync on every rank the forward is clean again.  The ranks
    agree on what happened over a gloo group on the host; no rank leaves with
    kernels in flight, NVLS is off and the exchanges use plain peer stores."""
    os.environ["S2B_SHARD_P2P"] = "1"
    os.environ["S2B_SHARD_WAIT_MS"] = "500"
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import time
    import torch
    import torch.distributed as dist
    import s2b
    dist.init_process_group("gloo", rank=rank, world_size=world)
    T, H, W = grid
    Lv, TXT = T * H * W, 58
    ctx = s2b.DitB200(rank, s2b.PREC_BF16)
    rec = {}

    def call(fn):
        t0 = time.monotonic()
        try:
            out = fn()
            return 0, out, time.monotonic() - t0
        except s2b.S2BError as e:
            return e.code, None, time.monotonic() - t0

    def any_failed(code):
        t = torch.tensor([1 if code else 0])
        dist.all_reduce(t)
        return int(t.item()) > 0

    try:
        ctx.init_synth(1234)
        ctx.set_windows(s2b.make_win(T, H, W, (4, 3, 3), TXT, False), s2b.make_win(T, H, W, (4, 3, 3), TXT, True))
        vid = s2b.patchify_grid(s2b.synth_vid_grid(T, 2 * H, 2 * W, 42))
        txt = s2b.synth_txt(TXT, 7)
        ctx.shard_init(uid, world, rank)
        fwd = lambda: ctx.shard_forward(vid, Lv, txt, TXT, 1000.0)
        rc, sr_a, _ = call(fwd)
        rec["clean"] = rc
        # 1) host call: rank 1 skips, rank 0's call times out
        if rank == 0:
            rc, _, dt = call(fwd)
            rec["skip_rc"], rec["skip_s"] = rc, dt
        dist.barrier()
        if any_failed(rec.get("skip_rc", 0)):
            ctx.shard_resync()
        rc, sr_b, _ = call(fwd)
        rec["after_resync"] = rc
        # 2) _dev call: rank 1 skips, rank 0 learns it from check_errors
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        st = torch.cuda.current_stream(dev)
        d_vid, d_txt = torch.from_numpy(vid).to(dev), torch.from_numpy(txt).to(dev)
        d_sr = torch.zeros(Lv, 64, device=dev)
        fwd_dev = lambda: ctx.shard_forward_dev(d_vid.data_ptr(), Lv, d_txt.data_ptr(), TXT, 1000.0, d_sr.data_ptr(),
                                                st.cuda_stream)
        code = 0
        if rank == 0:
            rc, _, _ = call(fwd_dev)
            rec["dev_enqueue_rc"] = rc
            st.synchronize()
            code, _, _ = call(ctx.check_errors)
            rec["dev_check_rc"] = code
        dist.barrier()
        if any_failed(code):
            ctx.shard_resync()
        rc, _, _ = call(fwd_dev)
        st.synchronize()
        rc2, _, _ = call(ctx.check_errors)
        rec["dev_after_resync"] = rc or rc2
        sr_c = d_sr.cpu().numpy()
        # 3) rank 0 makes one extra failed call and nobody resyncs: the ranks'
        #    call numbers differ, so the next call fails on BOTH ranks (rank 1
        #    sees a newer flag at once, rank 0 waits out its bound)
        if rank == 0:
            call(fwd)
        dist.barrier()
        rc, _, dt = call(fwd)
        rec["diverged_rc"], rec["diverged_s"] = rc, dt
        if any_failed(rc):
            ctx.shard_resync()
        rc, sr_d, _ = call(fwd)
        rec["final"] = rc
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), sr_a=sr_a, sr_b=sr_b, sr_c=sr_c, sr_d=sr_d,
                 **{k: np.array(v) for k, v in rec.items()})
    finally:
        ctx.close()
        dist.destroy_process_group()
