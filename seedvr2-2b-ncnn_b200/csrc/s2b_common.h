// s2b_common.h -- shared constants and helpers for the B200 NaDiT/AWA path.
//
// Model constants follow the reference DiT host (src/dit_vk.cpp:16-20):
// 20 heads x 128, hidden 2560, qkv 7680, 32 layers of which the first 10
// have separate vid/txt weights, SwiGLU hidden 6912, RoPE on 126 of 128 dims.
#pragma once
#include <cstdint>
#include <cstddef>
#include <string>

namespace s2b {

constexpr int HEADS = 20, HEAD_D = 128, DIM = 2560, QKV = 3 * DIM;
constexpr int NUM_LAYERS = 32, MM_LAYERS = 10;
constexpr int MLP_DIM = 6912;
constexpr int ROPE_ROT = 126;
constexpr int PATCH_IN = 33 * 4;        // 132: (ph,pw,c) patch of the 33-channel grid
constexpr int PATCH_IN_PAD = 136;       // row stride padded to 16 B multiples for TMA
constexpr int TXT_IN = 5120;
constexpr int OUT_CH = 64;              // 2x2 patch x 16 latent channels
constexpr int EMB_DIM = 6 * DIM;        // 15360
constexpr int TEMB_IN = 256;
constexpr float NORM_EPS = 1e-5f;       // src/dit_vk.cpp:17

enum Status {
    OK = 0, ERR_ARG = 1, ERR_CUDA = 2, ERR_IO = 3, ERR_STATE = 4,
    ERR_UNSUPPORTED = 5, ERR_NCCL = 6, ERR_TIMEOUT = 7, ERR_NOMEM = 8,
};

enum Precision { PREC_FP32 = 0, PREC_FP16 = 1, PREC_BF16 = 2 };

// 64-bit FNV-1a: names a tensor's random stream independently of load order.
inline uint64_t fnv1a(const std::string& s) {
    uint64_t h = 1469598103934665603ull;
    for (unsigned char c : s) { h ^= c; h *= 1099511628211ull; }
    return h;
}

}  // namespace s2b
