// k_awa_static.cu -- the AWA operator with its scratch in a fixed,
// module-scope device array, for callers that cannot allocate device memory
// while they run: a host framework that owns every device allocation (an
// inference runtime whose plugin API hands the plugin only its input and
// output buffers), or code running where cudaMalloc/cudaFree would block or
// synchronise the device (a latency-critical serving loop).
//
// Scratch: window-packed Q/K/V ([20][sumS][128] in the context precision)
// followed by the per-window txt partial sums ([nwin][TXT][2560] fp32), all
// carved out of ONE array of S2B_AWA_STATIC_BYTES (32 MiB) that every device
// loading this library holds until the process exits.  Calls whose geometry
// needs more are rejected.  No element of the scratch has to start at zero:
// every element a call reads was written earlier in the same call.  All calls
// on a device share the array and it keeps the last call's contents, so
// calls whose GPU work overlaps (different streams, different host threads)
// race on it and must be serialised by the caller.
#include "kernels.h"
#include <mutex>

namespace s2b {

constexpr size_t AWA_STATIC_BYTES = 32ull << 20;

namespace {

static __device__ __align__(256) unsigned char g_awa_scratch[AWA_STATIC_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
void* g_ptr[MAX_DEVICES];

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace

size_t awa_static_bytes_needed(const AwaDev& g, ActT pt) {
    const size_t qkv = align256((size_t)g.sumS * 2560 * act_bytes(pt));
    return 3 * qkv + align256((size_t)g.nwin * g.TXT * 2560 * 4);
}

size_t awa_static_capacity() { return AWA_STATIC_BYTES; }

// Device address of the scratch array on the current device.  The first call
// on a device resolves it with cudaGetSymbolAddress (which may load the
// module on that device, so it must not happen during stream capture).
int awa_static_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= MAX_DEVICES) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_awa_scratch);
        if (e != cudaSuccess) return (int)e;
        g_ptr[dev] = p;
    }
    *out = g_ptr[dev];
    return 0;
}

// pack -> attention -> txt coalesce on the caller's stream, scratch in
// g_awa_scratch.  Returns 0, -1 when the geometry does not fit, -2 when the
// bf16 attention's tensor maps cannot be encoded (the pack was enqueued, the
// attention was not), or a cudaError_t value.
int awa_forward_static(const float* vqkv, const float* tqkv, const AwaDev& g, const float* nqv, const float* nkv,
                       const float* nqt, const float* nkt, float eps, float scale, ActT pt, float* vid_out,
                       float* txt_out, cudaStream_t s) {
    if (awa_static_bytes_needed(g, pt) > AWA_STATIC_BYTES) return -1;
    void* base = nullptr;
    if (int rc = awa_static_scratch(&base)) return rc;
    unsigned char* p = static_cast<unsigned char*>(base);
    const size_t qkv = align256((size_t)g.sumS * 2560 * act_bytes(pt));
    void* Qp = p;
    void* Kp = p + qkv;
    void* Vp = p + 2 * qkv;
    float* toutw = reinterpret_cast<float*>(p + 3 * qkv);
    awa_pack(vqkv, tqkv, ACT_F32, 3 * 2560, g, nqv, nkv, nqt, nkt, eps, Qp, Kp, Vp, pt, s);
    if (awa_attend(Qp, Kp, Vp, pt, g, scale, vid_out, 2560, ACT_F32, toutw, s, nullptr)) return -2;
    awa_coalesce(toutw, g.nwin, g.TXT, txt_out, 2560, ACT_F32, s);
    return 0;
}

}  // namespace s2b
