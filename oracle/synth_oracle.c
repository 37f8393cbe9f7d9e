/* synth_oracle.c -- seeded synthetic weights and inputs for the CPU
 * reference legs.  TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * bench.py's reference arm runs the reference's CPU forward_latent on the
 * same synthetic model and inputs as the product, without loading the
 * product library; this file writes them.  It restates the generator the
 * product documents: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel
 * random numbers: as easy as 1, 2, 3", SC'11) keyed by the seed, counter =
 * (element block of 4, FNV-1a hash of the tensor name), Box-Muller in double
 * (cos, sin pairs), fp16 weights rounded to nearest even (here by the
 * compiler's _Float16 conversion), and the m5 file layout the reference
 * loader reads (src/dit_vk.cpp:38-45, 156-177: Linear blob
 * [u32 0x01306B47][fp16 W out x in][fp32 bias], raw vector
 * [i64 ndim][i64 len][f32]).  tests/test_oracle_pin.py checks it bit for bit
 * against the product's generator.
 */
#define _GNU_SOURCE
#include "oracle.h"
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

enum { DIM = 2560, QKV = 7680, MLP_DIM = 6912, HEAD_D = 128, PATCH_IN = 132, TXT_IN = 5120, TEMB_IN = 256,
       EMB_DIM = 15360, OUT_CH = 64, NUM_LAYERS = 32, MM_LAYERS = 10 };
static const float STD = 0.02f;

static uint64_t fnv1a(const char* s) {
    uint64_t h = 1469598103934665603ull;
    for (; *s; s++) { h ^= (unsigned char)*s; h *= 1099511628211ull; }
    return h;
}

static void philox(const uint32_t ctr[4], uint64_t key, uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
    uint32_t k0 = (uint32_t)key, k1 = (uint32_t)(key >> 32);
    for (int r = 0; r < 10; r++) {
        const uint64_t a = (uint64_t)0xD2511F53u * c0, b = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t)(b >> 32) ^ c1 ^ k0, n2 = (uint32_t)(a >> 32) ^ c3 ^ k1;
        c0 = n0; c1 = (uint32_t)b; c2 = n2; c3 = (uint32_t)a;
        k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* four N(0,1) values of block `blk` of stream `st` */
static void normals4(uint64_t seed, uint64_t st, uint64_t blk, double z[4]) {
    const uint32_t ctr[4] = {(uint32_t)blk, (uint32_t)(blk >> 32), (uint32_t)st, (uint32_t)(st >> 32)};
    uint32_t x[4];
    philox(ctr, seed, x);
    for (int p = 0; p < 2; p++) {
        const double u1 = ((double)x[2 * p] + 0.5) / 4294967296.0;
        const double u2 = ((double)x[2 * p + 1] + 0.5) / 4294967296.0;
        const double r = sqrt(-2.0 * log(u1)), th = 6.283185307179586476925286766559 * u2;
        z[2 * p] = r * cos(th);
        z[2 * p + 1] = r * sin(th);
    }
}

void or_synth_normal(float* out, long n, uint64_t seed, const char* stream, float mean, float stdv) {
    const uint64_t st = fnv1a(stream);
    const long nb = (n + 3) / 4;
    #pragma omp parallel for schedule(static)
    for (long b = 0; b < nb; b++) {
        double z[4];
        normals4(seed, st, (uint64_t)b, z);
        for (int j = 0; j < 4 && 4 * b + j < n; j++) out[4 * b + j] = (float)(mean + stdv * z[j]);
    }
}

static void synth_f16(uint16_t* out, long n, uint64_t seed, const char* stream) {
    const uint64_t st = fnv1a(stream);
    const long nb = (n + 3) / 4;
    #pragma omp parallel for schedule(static)
    for (long b = 0; b < nb; b++) {
        double z[4];
        normals4(seed, st, (uint64_t)b, z);
        for (int j = 0; j < 4 && 4 * b + j < n; j++) {
            const _Float16 h = (_Float16)(float)(0.0 + STD * z[j]);
            memcpy(out + 4 * b + j, &h, 2);
        }
    }
}

static int write_all(const char* path, const void* p, size_t n) {
    FILE* f = fopen(path, "wb");
    if (!f) return -1;
    const int ok = fwrite(p, 1, n, f) == n;
    fclose(f);
    return ok ? 0 : -1;
}

static int write_linear(const char* dir, const char* name, int out, int in, int bias, uint64_t seed) {
    char path[4096], param[512], stream[256];
    snprintf(param, sizeof param,
             "7767517\n2 2\nInput                    in0                      0 1 in0\n"
             "InnerProduct             linear_0                 1 1 in0 out0 0=%d 1=%d 2=%d\n",
             out, bias, out * in);
    snprintf(path, sizeof path, "%s/%s.param", dir, name);
    if (write_all(path, param, strlen(param))) return -1;
    const size_t nw = (size_t)out * in, bytes = 4 + 2 * nw + (bias ? 4 * (size_t)out : 0);
    unsigned char* blob = malloc(bytes);
    if (!blob) return -1;
    const uint32_t tag = 0x01306B47u;
    memcpy(blob, &tag, 4);
    snprintf(stream, sizeof stream, "%s.weight", name);
    synth_f16((uint16_t*)(blob + 4), (long)nw, seed, stream);
    if (bias) {
        snprintf(stream, sizeof stream, "%s.bias", name);
        or_synth_normal((float*)(blob + 4 + 2 * nw), out, seed, stream, 0.f, STD);
    }
    snprintf(path, sizeof path, "%s/%s.bin", dir, name);
    const int rc = write_all(path, blob, bytes);
    free(blob);
    return rc;
}

static int write_vector(const char* dir, const char* name, int n, float mean, uint64_t seed) {
    char path[4096];
    unsigned char* blob = malloc(16 + 4 * (size_t)n);
    if (!blob) return -1;
    const int64_t nd = 1, len = n;
    memcpy(blob, &nd, 8);
    memcpy(blob + 8, &len, 8);
    or_synth_normal((float*)(blob + 16), n, seed, name, mean, STD);
    snprintf(path, sizeof path, "%s/%s.bin", dir, name);
    const int rc = write_all(path, blob, 16 + 4 * (size_t)n);
    free(blob);
    return rc;
}

int or_synth_write_m5(const char* dir, uint64_t seed, int lo, int hi) {
    mkdir(dir, 0755);
    struct { const char* n; int out, in; } top[] = {
        {"vid_in_proj", DIM, PATCH_IN}, {"txt_in", DIM, TXT_IN}, {"emb_proj_in", DIM, TEMB_IN},
        {"emb_proj_hid", DIM, DIM}, {"emb_proj_out", EMB_DIM, DIM}, {"vid_out_proj", OUT_CH, DIM}};
    for (int i = 0; i < 6; i++)
        if (write_linear(dir, top[i].n, top[i].out, top[i].in, 1, seed)) return -1;
    const char* tags[2][2] = {{"vid", "txt"}, {"all", NULL}};
    char b[64], name[96];
    for (int i = lo < 0 ? 0 : lo; i < (hi > NUM_LAYERS ? NUM_LAYERS : hi); i++)
        for (int f = 0; f < 2; f++) {
            const char* t = tags[i < MM_LAYERS ? 0 : 1][f];
            if (!t) continue;
            snprintf(b, sizeof b, "b%d_%s", i, t);
            struct { const char* s; int out, in, bias; } L[] = {
                {"_qkv", QKV, DIM, 0}, {"_out", DIM, DIM, 1}, {"_mlp_in", MLP_DIM, DIM, 0},
                {"_mlp_g", MLP_DIM, DIM, 0}, {"_mlp_out", DIM, MLP_DIM, 0}};
            for (int k = 0; k < 5; k++) {
                snprintf(name, sizeof name, "%s%s", b, L[k].s);
                if (write_linear(dir, name, L[k].out, L[k].in, L[k].bias, seed)) return -1;
            }
        }
    /* every layer's raw vectors (the loader reads all of them) */
    if (write_vector(dir, "vid_out_norm_w", DIM, 1.f, seed) || write_vector(dir, "vid_out_ada_shift", DIM, 0.f, seed) ||
        write_vector(dir, "vid_out_ada_scale", DIM, 1.f, seed))
        return -1;
    for (int i = 0; i < NUM_LAYERS; i++)
        for (int f = 0; f < 2; f++) {
            const char* t = tags[i < MM_LAYERS ? 0 : 1][f];
            if (!t) continue;
            struct { const char* s; int n; float mean; } V[] = {
                {"_nq", HEAD_D, 1.f}, {"_nk", HEAD_D, 1.f}, {"_attn_shift", DIM, 0.f}, {"_attn_scale", DIM, 1.f},
                {"_attn_gate", DIM, 1.f}, {"_mlp_shift", DIM, 0.f}, {"_mlp_scale", DIM, 1.f}, {"_mlp_gate", DIM, 1.f}};
            for (int k = 0; k < 8; k++) {
                snprintf(name, sizeof name, "b%d_%s%s", i, t, V[k].s);
                if (write_vector(dir, name, V[k].n, V[k].mean, seed)) return -1;
            }
        }
    return 0;
}

/* vid_grid (T,H,W,33) = [noise(16) | condition(16) | 1], src/seedvr2_engine.cpp:159-168 */
void or_synth_vid_grid(float* grid, int T, int H, int W, uint64_t seed) {
    const long n = (long)T * H * W;
    float* noise = malloc(sizeof(float) * n * 16);
    float* cond = malloc(sizeof(float) * n * 16);
    or_synth_normal(noise, n * 16, seed, "vid_noise", 0.f, 1.f);
    or_synth_normal(cond, n * 16, seed, "vid_cond", 0.f, 1.f);
    for (long p = 0; p < n; p++) {
        float* g = grid + p * 33;
        for (int c = 0; c < 16; c++) { g[c] = noise[p * 16 + c]; g[16 + c] = cond[p * 16 + c]; }
        g[32] = 1.f;
    }
    free(noise);
    free(cond);
}

void or_synth_txt(float* txt, int TXT, uint64_t seed) { or_synth_normal(txt, (long)TXT * TXT_IN, seed, "txt", 0.f, 1.f); }
