// k_engine.cu -- the DiT's data formats on either side of the forward, on
// the device: patchify / unpatchify of the latent grid (src/dit_vk.cpp:
// 717-750) and the engine's vid_grid assembly and latent decode step
// (src/seedvr2_engine.cpp:154-168, 298-305).  Pure data movement plus one
// multiply or subtract-divide per element: HBM-bound, one thread per output
// element, consecutive threads on consecutive output addresses.
#include "kernels.h"

namespace s2b {
namespace {

// (T, H, W, 33) channel-last -> (T * H/2 * W/2, 132), element (ph, pw, c) of
// token (t, hh, ww) at column (ph * 2 + pw) * 33 + c.
__global__ void k_patchify(const float* __restrict__ grid, int T, int H, int W, float* __restrict__ patch) {
    const int H2 = H / 2, W2 = W / 2;
    const size_t n = (size_t)T * H2 * W2 * 132;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int col = (int)(i % 132);
    const size_t tok = i / 132;
    const int ww = (int)(tok % W2), hh = (int)((tok / W2) % H2), t = (int)(tok / ((size_t)W2 * H2));
    const int pp = col / 33, c = col % 33, ph = pp >> 1, pw = pp & 1;
    patch[i] = grid[(((size_t)t * H + (hh * 2 + ph)) * W + (ww * 2 + pw)) * 33 + c];
}

// (T * H/2 * W/2, 64) -> (T, H, W, 16) channel-last.
__global__ void k_unpatchify(const float* __restrict__ sr, int T, int H, int W, float* __restrict__ out) {
    const int H2 = H / 2, W2 = W / 2;
    const size_t n = (size_t)T * H * W * 16;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int c = (int)(i % 16);
    const size_t pix = i / 16;
    const int x = (int)(pix % W), y = (int)((pix / W) % H), t = (int)(pix / ((size_t)W * H));
    const int hh = y >> 1, ph = y & 1, ww = x >> 1, pw = x & 1;
    out[i] = sr[(((size_t)t * H2 + hh) * W2 + ww) * 64 + (ph * 2 + pw) * 16 + c];
}

// vid_grid[h][w] = [noise c=0..15 | latent c=0..15 * scale | 1] from
// channel-first (16, H8, W8) noise and condition latent.
__global__ void k_assemble_grid(const float* __restrict__ noise, const float* __restrict__ latent, float scale,
                                int H8, int W8, float* __restrict__ grid) {
    const size_t n = (size_t)H8 * W8 * 33;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int c = (int)(i % 33);
    const size_t hw = i / 33;
    float v;
    if (c < 16) v = noise[(size_t)c * H8 * W8 + hw];
    else if (c < 32) v = __fmul_rn(latent[(size_t)(c - 16) * H8 * W8 + hw], scale);
    else v = 1.0f;
    grid[i] = v;
}

// z[c][h][w] = (noise[c][h][w] - sr[h][w][c]) / scale.
__global__ void k_decode_latent(const float* __restrict__ noise, const float* __restrict__ sr, float scale, int H8,
                                int W8, float* __restrict__ z) {
    const size_t hw_n = (size_t)H8 * W8;
    const size_t n = hw_n * 16;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int c = (int)(i / hw_n);
    const size_t hw = i % hw_n;
    z[i] = __fdiv_rn(__fsub_rn(noise[i], sr[hw * 16 + c]), scale);
}

inline int blocks(size_t n) { return (int)((n + 255) / 256); }

}  // namespace

void patchify_dev(const float* grid, int T, int H, int W, float* patch, cudaStream_t s) {
    const size_t n = (size_t)T * (H / 2) * (W / 2) * 132;
    if (n) k_patchify<<<blocks(n), 256, 0, s>>>(grid, T, H, W, patch);
}

void unpatchify_dev(const float* sr, int T, int H, int W, float* out, cudaStream_t s) {
    const size_t n = (size_t)T * H * W * 16;
    if (n) k_unpatchify<<<blocks(n), 256, 0, s>>>(sr, T, H, W, out);
}

void assemble_grid_dev(const float* noise, const float* latent, float scale, int H8, int W8, float* grid,
                       cudaStream_t s) {
    const size_t n = (size_t)H8 * W8 * 33;
    if (n) k_assemble_grid<<<blocks(n), 256, 0, s>>>(noise, latent, scale, H8, W8, grid);
}

void decode_latent_dev(const float* noise, const float* sr, float scale, int H8, int W8, float* z, cudaStream_t s) {
    const size_t n = (size_t)H8 * W8 * 16;
    if (n) k_decode_latent<<<blocks(n), 256, 0, s>>>(noise, sr, scale, H8, W8, z);
}

}  // namespace s2b
