// shim.cpp -- implementation of the CPU-only ncnn stand-in (see ncnn/shim_all.h)
// plus link stubs for the reference classes whose sources are Vulkan-only
// (AwaVk in src/awa_vk.cpp, DitVk's graph methods in src/dit_graph.cpp).
// TEST INFRASTRUCTURE ONLY: built into oracle/_ref/ as the parity checker.
#include "ncnn/shim_all.h"
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <sstream>
#include <string>
#include <algorithm>

#include "awa_vk.h"
#include "dit_vk.h"

namespace ncnn {

int create_gpu_instance(int) { return -1; }
void destroy_gpu_instance() {}
VulkanDevice* get_gpu_device(int) { return nullptr; }
int get_gpu_count() { return 0; }

static float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, f;
    if (e == 0) {
        if (m == 0) f = sign;
        else {  // subnormal: renormalise
            int ee = 113;
            while (!(m & 0x400)) { m <<= 1; ee--; }
            f = sign | ((uint32_t)ee << 23) | ((m & 0x3ff) << 13);
        }
    } else if (e == 31) f = sign | 0x7f800000u | (m << 13);
    else f = sign | ((e + 112) << 23) | (m << 13);
    float out; std::memcpy(&out, &f, 4); return out;
}

int Net::load_param_mem(const char* mem) {
    std::istringstream ss(mem);
    std::string line;
    while (std::getline(ss, line)) {
        if (line.find("InnerProduct") == std::string::npos) continue;
        std::istringstream ls(line);
        std::string tok;
        while (ls >> tok) {
            if (tok.rfind("0=", 0) == 0) num_output = std::atoi(tok.c_str() + 2);
            else if (tok.rfind("1=", 0) == 0) bias_term = std::atoi(tok.c_str() + 2);
            else if (tok.rfind("2=", 0) == 0) weight_data_size = std::atoi(tok.c_str() + 2);
        }
    }
    if (num_output <= 0 || weight_data_size <= 0 || weight_data_size % num_output) {
        fprintf(stderr, "[ncnn-shim] unsupported param (InnerProduct expected)\n");
        return -1;
    }
    return 0;
}

int Net::load_model(const unsigned char* mem) {
    const int out = num_output, in = weight_data_size / num_output;
    uint32_t tag; std::memcpy(&tag, mem, 4);
    const unsigned char* p = mem + 4;
    std::vector<float> w((size_t)out * in);
    if (tag == 0x01306B47u) {
        for (size_t i = 0; i < w.size(); i++) {
            uint16_t hv; std::memcpy(&hv, p + 2 * i, 2); w[i] = half_to_float(hv);
        }
        p += 2 * w.size();
    } else if (tag == 0u) {
        std::memcpy(w.data(), p, 4 * w.size());
        p += 4 * w.size();
    } else {
        fprintf(stderr, "[ncnn-shim] unsupported weight tag 0x%08x\n", tag);
        return -1;
    }
    weight_t.assign((size_t)in * out, 0.f);
    for (int o = 0; o < out; o++)
        for (int i = 0; i < in; i++) weight_t[(size_t)i * out + o] = w[(size_t)o * in + i];
    if (bias_term) { bias.resize(out); std::memcpy(bias.data(), p, 4 * out); p += 4 * out; }
    return (int)(p - mem);
}

int Extractor::input(const char*, const Mat& in) { in_ = in; return 0; }

// y[M,N] = x[M,K] * wt[K,N] + b : register-blocked 4x16, fp32 accumulate.
static void sgemm(const float* x, int M, int K, const float* wt, int N, const float* b, float* y) {
    const int MB = 4, NB = 16;
    const int mt = (M + MB - 1) / MB, nt = N / NB;
    #pragma omp parallel for schedule(dynamic, 4)
    for (long t = 0; t < (long)mt * nt; t++) {
        const int m0 = (int)(t / nt) * MB, n0 = (int)(t % nt) * NB;
        const int mr = std::min(MB, M - m0);
        float acc[MB][NB] = {};
        for (int k = 0; k < K; k++) {
            const float* w = wt + (size_t)k * N + n0;
            for (int r = 0; r < MB; r++) {
                const float xv = (r < mr) ? x[(size_t)(m0 + r) * K + k] : 0.f;
                for (int j = 0; j < NB; j++) acc[r][j] += xv * w[j];
            }
        }
        for (int r = 0; r < mr; r++)
            for (int j = 0; j < NB; j++) y[(size_t)(m0 + r) * N + n0 + j] = acc[r][j] + (b ? b[n0 + j] : 0.f);
    }
    for (int n = nt * NB; n < N; n++)  // ragged N tail
        for (int m = 0; m < M; m++) {
            float a = 0.f;
            for (int k = 0; k < K; k++) a += x[(size_t)m * K + k] * wt[(size_t)k * N + n];
            y[(size_t)m * N + n] = a + (b ? b[n] : 0.f);
        }
}

int Extractor::extract(const char*, Mat& out) {
    const int K = net->weight_data_size / net->num_output, N = net->num_output;
    if (in_.empty() || in_.w != K) {
        fprintf(stderr, "[ncnn-shim] InnerProduct input w=%d, expected %d\n", in_.w, K);
        return -1;
    }
    const int M = in_.h;
    out.create(N, M, 4u);
    sgemm((const float*)in_.data, M, K, net->weight_t.data(), N,
          net->bias_term ? net->bias.data() : nullptr, (float*)out.data);
    return 0;
}

}  // namespace ncnn

// ---- link stubs: Vulkan-only reference classes (never used in CPU mode) ----
AwaVk::AwaVk() {}
AwaVk::~AwaVk() {}
bool AwaVk::init(ncnn::VulkanDevice*, const std::string&) { return false; }
bool AwaVk::forward(const std::vector<float>&, const std::vector<float>&, const Win&,
                    const std::vector<float>&, const std::vector<float>&,
                    const std::vector<float>&, const std::vector<float>&, int, int,
                    std::vector<float>&, std::vector<float>&) { return false; }
void DitVk::release_graph() {}
