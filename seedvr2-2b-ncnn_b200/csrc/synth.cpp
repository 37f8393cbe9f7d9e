// synth.cpp -- seeded synthetic weights and inputs for the NaDiT DiT.
//
// There is no checkpoint on this box, so every parity test and benchmark runs
// on random-init weights of the real architecture and seeded inputs of the
// real shapes.  The generator is Philox4x32-10 (Salmon, Moraes, Dror, Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC'11), keyed by the seed,
// counting over (element block, tensor stream), with the Box-Muller transform
// evaluated in double precision.  Every tensor has its own stream (FNV-1a of
// its file name), so values do not depend on which tensors are generated or
// in what order.  Output is deterministic for a given (seed, name).
//
// write_m5 lays weights out exactly as the reference loader reads them
// (names: src/dit_vk.cpp:156-177 and the lin() bases; Linear blob
// [u32 0x01306B47][fp16 W out x in][fp32 bias], raw vector
// [i64 ndim][i64 shape...][f32 data]: src/dit_vk.cpp:38-45).
#include "synth.h"
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>
#include <algorithm>
#include <sys/stat.h>

namespace s2b {

static inline void philox_round(uint32_t c[4], const uint32_t k[2]) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k[0], n2 = hi0 ^ c[3] ^ k[1];
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
}

void philox4x32_10(const uint32_t ctr[4], uint64_t seed, uint32_t out[4]) {
    uint32_t c[4] = {ctr[0], ctr[1], ctr[2], ctr[3]};
    uint32_t k[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    for (int r = 0; r < 10; r++) {
        philox_round(c, k);
        k[0] += 0x9E3779B9u; k[1] += 0xBB67AE85u;
    }
    out[0] = c[0]; out[1] = c[1]; out[2] = c[2]; out[3] = c[3];
}

// Four standard normals from one Philox block: (x0,x1) and (x2,x3) feed two
// Box-Muller pairs, cos first.
static inline void normals4(uint64_t seed, uint64_t stream, uint64_t block, double z[4]) {
    const uint32_t ctr[4] = {(uint32_t)block, (uint32_t)(block >> 32), (uint32_t)stream, (uint32_t)(stream >> 32)};
    uint32_t x[4];
    philox4x32_10(ctr, seed, x);
    const double twopi = 6.283185307179586476925286766559;
    for (int p = 0; p < 2; p++) {
        const double u1 = ((double)x[2 * p] + 0.5) * (1.0 / 4294967296.0);
        const double u2 = ((double)x[2 * p + 1] + 0.5) * (1.0 / 4294967296.0);
        const double r = std::sqrt(-2.0 * std::log(u1));
        z[2 * p] = r * std::cos(twopi * u2);
        z[2 * p + 1] = r * std::sin(twopi * u2);
    }
}

template <typename F>
static void parallel_blocks(size_t nblocks, F&& fn) {
    unsigned nt = std::max(1u, std::min(64u, std::thread::hardware_concurrency()));
    if (nblocks < 4096) nt = 1;
    std::vector<std::thread> th;
    const size_t per = (nblocks + nt - 1) / nt;
    for (unsigned t = 0; t < nt; t++) {
        const size_t b0 = t * per, b1 = std::min(nblocks, b0 + per);
        if (b0 >= b1) break;
        th.emplace_back([=, &fn] { for (size_t b = b0; b < b1; b++) fn(b); });
    }
    for (auto& x : th) x.join();
}

void fill_normal_f32(float* out, size_t n, uint64_t seed, uint64_t stream, float mean, float stdv) {
    parallel_blocks((n + 3) / 4, [&](size_t b) {
        double z[4]; normals4(seed, stream, b, z);
        for (int j = 0; j < 4 && 4 * b + j < n; j++) out[4 * b + j] = (float)(mean + stdv * z[j]);
    });
}

// IEEE binary16 from binary32, round to nearest even (with subnormals).
uint16_t f32_to_f16_bits(float f) {
    uint32_t x; std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);           // overflow -> inf
    if (ax < 0x38800000u) {                                              // subnormal or zero
        if (ax < 0x33000000u) return (uint16_t)sign;                     // below half the min subnormal
        const uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e;                                   // 14..24
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((ax - 0x38000000u) >> 13);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
    return (uint16_t)(sign | h);
}

float f16_bits_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ffu, f;
    if (e == 0) {
        if (m == 0) f = sign;
        else { int ee = 113; while (!(m & 0x400u)) { m <<= 1; ee--; } f = sign | ((uint32_t)ee << 23) | ((m & 0x3ffu) << 13); }
    } else if (e == 31) f = sign | 0x7f800000u | (m << 13);
    else f = sign | ((e + 112) << 23) | (m << 13);
    float out; std::memcpy(&out, &f, 4); return out;
}

void fill_normal_f16(uint16_t* out, size_t n, uint64_t seed, uint64_t stream, float mean, float stdv) {
    parallel_blocks((n + 3) / 4, [&](size_t b) {
        double z[4]; normals4(seed, stream, b, z);
        for (int j = 0; j < 4 && 4 * b + j < n; j++) out[4 * b + j] = f32_to_f16_bits((float)(mean + stdv * z[j]));
    });
}

// ---------------------------------------------------------------- m5 layout
std::vector<SynthLinear> model_linears(int layer_lo, int layer_hi) {
    std::vector<SynthLinear> v = {
        {"vid_in_proj", DIM, PATCH_IN, true},
        {"txt_in", DIM, TXT_IN, true},
        {"emb_proj_in", DIM, TEMB_IN, true},
        {"emb_proj_hid", DIM, DIM, true},
        {"emb_proj_out", EMB_DIM, DIM, true},
        {"vid_out_proj", OUT_CH, DIM, true},
    };
    for (int i = std::max(0, layer_lo); i < std::min(NUM_LAYERS, layer_hi); i++) {
        std::vector<std::string> tags;
        if (i < MM_LAYERS) tags = {"vid", "txt"}; else tags = {"all"};
        for (auto& t : tags) {
            const std::string b = "b" + std::to_string(i) + "_" + t;
            v.push_back({b + "_qkv", QKV, DIM, false});
            v.push_back({b + "_out", DIM, DIM, true});
            v.push_back({b + "_mlp_in", MLP_DIM, DIM, false});
            v.push_back({b + "_mlp_g", MLP_DIM, DIM, false});
            v.push_back({b + "_mlp_out", DIM, MLP_DIM, false});
        }
    }
    return v;
}

// Raw fp32 vectors: (name, length, mean).  Norm weights, scales and gates are
// drawn around 1 (1+N(0,0.02)), shifts around 0 (N(0,0.02)), so every
// modulation path is exercised and the residual updates stay O(1).
std::vector<SynthVector> model_vectors() {
    std::vector<SynthVector> v = {
        {"vid_out_norm_w", DIM, 1.f}, {"vid_out_ada_shift", DIM, 0.f}, {"vid_out_ada_scale", DIM, 1.f},
    };
    for (int i = 0; i < NUM_LAYERS; i++) {
        std::vector<std::string> tags;
        if (i < MM_LAYERS) tags = {"vid", "txt"}; else tags = {"all"};
        for (auto& t : tags) {
            const std::string b = "b" + std::to_string(i) + "_" + t;
            v.push_back({b + "_nq", HEAD_D, 1.f});
            v.push_back({b + "_nk", HEAD_D, 1.f});
            v.push_back({b + "_attn_shift", DIM, 0.f});
            v.push_back({b + "_attn_scale", DIM, 1.f});
            v.push_back({b + "_attn_gate", DIM, 1.f});
            v.push_back({b + "_mlp_shift", DIM, 0.f});
            v.push_back({b + "_mlp_scale", DIM, 1.f});
            v.push_back({b + "_mlp_gate", DIM, 1.f});
        }
    }
    return v;
}

void synth_linear(const SynthLinear& L, uint64_t seed, uint16_t* w_f16, float* bias) {
    fill_normal_f16(w_f16, (size_t)L.out * L.in, seed, fnv1a(L.name + ".weight"), 0.f, SYNTH_STD);
    if (L.has_bias && bias) fill_normal_f32(bias, (size_t)L.out, seed, fnv1a(L.name + ".bias"), 0.f, SYNTH_STD);
}

void synth_vector(const SynthVector& V, uint64_t seed, float* out) {
    fill_normal_f32(out, (size_t)V.n, seed, fnv1a(V.name), V.mean, SYNTH_STD);
}

static bool write_file(const std::string& path, const void* p, size_t n, std::string& err) {
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) { err = "cannot open " + path; return false; }
    const bool ok = std::fwrite(p, 1, n, f) == n;
    std::fclose(f);
    if (!ok) err = "short write " + path;
    return ok;
}

int write_m5(const char* dir_c, uint64_t seed, int layer_lo, int layer_hi, std::string& err) {
    std::string dir = dir_c;
    if (dir.empty()) { err = "empty dir"; return ERR_ARG; }
    if (dir.back() != '/') dir += '/';
    ::mkdir(dir.c_str(), 0755);
    for (const auto& L : model_linears(layer_lo, layer_hi)) {
        char param[512];
        std::snprintf(param, sizeof param,
                      "7767517\n2 2\nInput                    in0                      0 1 in0\n"
                      "InnerProduct             linear_0                 1 1 in0 out0 0=%d 1=%d 2=%d\n",
                      L.out, L.has_bias ? 1 : 0, L.out * L.in);
        if (!write_file(dir + L.name + ".param", param, std::strlen(param), err)) return ERR_IO;
        const size_t nw = (size_t)L.out * L.in;
        std::vector<unsigned char> blob(4 + 2 * nw + (L.has_bias ? 4 * (size_t)L.out : 0));
        const uint32_t tag = 0x01306B47u;
        std::memcpy(blob.data(), &tag, 4);
        std::vector<float> bias(L.has_bias ? L.out : 0);
        synth_linear(L, seed, (uint16_t*)(blob.data() + 4), L.has_bias ? bias.data() : nullptr);
        if (L.has_bias) std::memcpy(blob.data() + 4 + 2 * nw, bias.data(), 4 * (size_t)L.out);
        if (!write_file(dir + L.name + ".bin", blob.data(), blob.size(), err)) return ERR_IO;
    }
    for (const auto& V : model_vectors()) {
        std::vector<unsigned char> blob(16 + 4 * (size_t)V.n);
        const int64_t ndim = 1, len = V.n;
        std::memcpy(blob.data(), &ndim, 8);
        std::memcpy(blob.data() + 8, &len, 8);
        synth_vector(V, seed, (float*)(blob.data() + 16));
        if (!write_file(dir + V.name + ".bin", blob.data(), blob.size(), err)) return ERR_IO;
    }
    return OK;
}

// Seeded DiT inputs: vid_grid (T,H,W,33) = [noise(16) | condition(16) | mask 1]
// with noise and condition N(0,1) (the layout src/seedvr2_engine.cpp:159-168
// builds), and txt (TXT,5120) N(0,1).
void synth_vid_grid(float* grid, int T, int H, int W, uint64_t seed) {
    const size_t n = (size_t)T * H * W;
    std::vector<float> noise(n * 16), cond(n * 16);
    fill_normal_f32(noise.data(), noise.size(), seed, fnv1a("vid_noise"), 0.f, 1.f);
    fill_normal_f32(cond.data(), cond.size(), seed, fnv1a("vid_cond"), 0.f, 1.f);
    for (size_t p = 0; p < n; p++) {
        float* g = grid + p * 33;
        for (int c = 0; c < 16; c++) { g[c] = noise[p * 16 + c]; g[16 + c] = cond[p * 16 + c]; }
        g[32] = 1.f;
    }
}

void synth_txt(float* txt, int TXT, uint64_t seed) {
    fill_normal_f32(txt, (size_t)TXT * TXT_IN, seed, fnv1a("txt"), 0.f, 1.f);
}

}  // namespace s2b
