// k_shard.cu -- the window-sharded forward's two per-layer exchanges done by
// kernels over NVLink peer memory (CUDA IPC mappings of the other ranks'
// buffers), instead of NCCL calls:
//   * txt mean: every rank publishes its windows' txt partial sum, raises a
//     flag in every peer, waits for all peers' flags, and sums all ranks'
//     partials in rank order (the same order on every rank, so all ranks get
//     bit-identical rows), divided by the global window count;
//   * residual exchange: every rank writes the rows it owns in the next
//     layout straight into the owner's residual buffer (peer stores), then
//     raises flags and waits for all peers' before the next layer reads it.
// Flags hold the value (call number * 64 + layer + 1) of the forward that
// raised them; the call number is the host's count of shard-forward calls on
// this rank (failed calls included), written to device memory before each
// forward.  A wait succeeds only on the exact value: an older value means the
// peer is behind (keep waiting), a newer one that this rank is behind (the
// ranks' call sequences have diverged; give up at once).  Every wait is
// bounded in time (ShardPeers::wait_ns): on expiry or divergence the kernel
// records g_shard_err and returns (no trap, no hang).  Once g_shard_err is set
// the rest of the forward neither waits, nor raises flags, nor stores into a
// peer's memory, so a peer that arrives late cannot run past the failed layer
// on stale signals; the forward's last kernel folds the flag into the
// context's status and clears it (status_fold), so the next forward starts
// clean.
#include "kernels.h"
#include "kcommon.cuh"

namespace s2b {

__device__ int g_shard_err;

namespace {

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool forward_failed() { return *(volatile int*)&g_shard_err != 0; }

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Value of the flags for `layer` of the current forward.
__device__ __forceinline__ uint32_t flag_value(const uint32_t* epoch, int layer) {
    return (*epoch) * 64u + (uint32_t)layer + 1u;
}

// Thread 0 of the block: raise this rank's flag in every rank's flag array
// (nothing once the forward has failed).
__device__ __forceinline__ void signal_all(const ShardPeers& P, int kind, int slot, uint32_t v) {
    if (forward_failed()) return;
    __threadfence_system();
    for (int q = 0; q < P.world; q++)
        st_release_sys(P.flags[q] + (kind * 2 + slot) * P.world + P.rank, v);
}

// Thread 0 of the block: wait until every rank's flag in this rank's array
// holds exactly v.  Returns false on expiry (P.wait_ns), on a flag newer than
// v (diverged call sequences), or when the forward has already failed.
__device__ __forceinline__ bool wait_all(const ShardPeers& P, int kind, int slot, uint32_t v) {
    const uint32_t* f = P.flags[P.rank] + (kind * 2 + slot) * P.world;
    const uint64_t t0 = globaltimer_ns();
    // a second bound that does not depend on the timer: 256 ns sleeps at most
    // (a sleep can be shorter, so this bound is the looser one)
    const uint64_t max_iter = P.wait_ns / 16 + 1024;
    for (int q = 0; q < P.world; q++) {
        uint64_t n = 0;
        for (;;) {
            const uint32_t x = ld_acquire_sys(f + q);
            if (x == v) break;
            if (x > v || forward_failed() || ++n > max_iter || globaltimer_ns() - t0 > P.wait_ns) {
                atomicExch(&g_shard_err, 1);
                return false;
            }
            __nanosleep(256);
        }
    }
    return true;
}

// Block 0 publishes this rank's partial (written by the previous kernel);
// every block then waits for all ranks and reduces its share of the rows.
template <typename TO>
__global__ void k_txt_reduce(const ShardPeers P, const uint32_t* epoch, int layer, int n, float divisor, TO* out,
                             int ld) {
    const int slot = layer & 1;
    __shared__ int ok;
    if (threadIdx.x == 0) {
        const uint32_t v = flag_value(epoch, layer);
        if (blockIdx.x == 0) signal_all(P, 0, slot, v);
        ok = wait_all(P, 0, slot, v) ? 1 : 0;
    }
    __syncthreads();
    if (!ok) return;
    for (int i4 = blockIdx.x * blockDim.x + threadIdx.x; i4 < n / 4; i4 += gridDim.x * blockDim.x) {
        float a[4] = {0.f, 0.f, 0.f, 0.f};
        for (int q = 0; q < P.world; q++) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(P.txtp[q] + (size_t)slot * n) + i4);
            a[0] = __fadd_rn(a[0], v.x); a[1] = __fadd_rn(a[1], v.y);
            a[2] = __fadd_rn(a[2], v.z); a[3] = __fadd_rn(a[3], v.w);
        }
        #pragma unroll
        for (int k = 0; k < 4; k++) a[k] = __fdiv_rn(a[k], divisor);
        const int i = i4 * 4;
        store4(out + (size_t)(i / 2560) * ld + (i % 2560), a);
    }
}

// Row k: local row src[k] of X[p] -> row dst[k] of rank rank_of[k]'s X[1-p].
__global__ void k_exchange_rows(const ShardPeers P, int p, const int* __restrict__ src, const int* __restrict__ rank_of,
                                const int* __restrict__ dst, int n) {
    const int k = blockIdx.x;
    if (k >= n || forward_failed()) return;
    const float4* a = reinterpret_cast<const float4*>(P.x[p][P.rank] + (size_t)src[k] * 2560);
    float4* b = reinterpret_cast<float4*>(P.x[1 - p][rank_of[k]] + (size_t)dst[k] * 2560);
    for (int c = threadIdx.x; c < 640; c += blockDim.x) b[c] = a[c];
}

// Row k of the local output -> row tok[k] of every rank's assembled output.
__global__ void k_sr_rows(const ShardPeers P, const float* __restrict__ src, const int* __restrict__ tok, int n) {
    const int k = blockIdx.x * 4 + (threadIdx.x >> 4), c = threadIdx.x & 15;
    if (k >= n || forward_failed()) return;
    const float4 v = reinterpret_cast<const float4*>(src + (size_t)k * 64)[c];
    for (int q = 0; q < P.world; q++) reinterpret_cast<float4*>(P.sr[q] + (size_t)tok[k] * 64)[c] = v;
}

__global__ void k_signal_wait(const ShardPeers P, const uint32_t* epoch, int layer) {
    const uint32_t v = flag_value(epoch, layer);
    signal_all(P, 1, layer & 1, v);
    wait_all(P, 1, layer & 1, v);
}

}  // namespace

void shard_txt_reduce(const ShardPeers& P, const uint32_t* epoch, int layer, int TXT, float divisor, void* out, int ld,
                      ActT t, cudaStream_t s) {
    const int n = TXT * 2560;
    const int blocks = 64;
    if (t == ACT_F32) k_txt_reduce<float><<<blocks, 256, 0, s>>>(P, epoch, layer, n, divisor, (float*)out, ld);
    else if (t == ACT_F16) k_txt_reduce<f16><<<blocks, 256, 0, s>>>(P, epoch, layer, n, divisor, (f16*)out, ld);
    else k_txt_reduce<bf16><<<blocks, 256, 0, s>>>(P, epoch, layer, n, divisor, (bf16*)out, ld);
}

void shard_exchange_rows(const ShardPeers& P, int p, const int* src, const int* rank_of, const int* dst, int n,
                         const uint32_t* epoch, int layer, cudaStream_t s) {
    if (n > 0) k_exchange_rows<<<n, 160, 0, s>>>(P, p, src, rank_of, dst, n);
    k_signal_wait<<<1, 1, 0, s>>>(P, epoch, layer);
}

// The output assembly uses the residual-exchange flags (kind 1) of layer 31,
// a layer after which no residual exchange runs.
void shard_gather_sr(const ShardPeers& P, const float* sr_local, const int* tok, int n, const uint32_t* epoch,
                     cudaStream_t s) {
    if (n > 0) k_sr_rows<<<(n + 3) / 4, 64, 0, s>>>(P, sr_local, tok, n);
    k_signal_wait<<<1, 1, 0, s>>>(P, epoch, 31);
}

int shard_flag_ptr(int** p) { return (int)cudaGetSymbolAddress((void**)p, g_shard_err); }

}  // namespace s2b
