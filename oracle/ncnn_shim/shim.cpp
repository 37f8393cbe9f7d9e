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
#include <immintrin.h>

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
    weight.resize((size_t)out * in);
    const long n = (long)weight.size();
    if (tag == 0x01306B47u) {
        const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
        #pragma omp parallel for schedule(static)
        for (long i = 0; i < n; i++) { uint16_t hv; std::memcpy(&hv, h + i, 2); weight[i] = half_to_float(hv); }
        p += 2 * weight.size();
    } else if (tag == 0u) {
        std::memcpy(weight.data(), p, 4 * weight.size());
        p += 4 * weight.size();
    } else {
        fprintf(stderr, "[ncnn-shim] unsupported weight tag 0x%08x\n", tag);
        return -1;
    }
    if (bias_term) { bias.resize(out); std::memcpy(bias.data(), p, 4 * out); p += 4 * out; }
    return (int)(p - mem);
}

int Extractor::input(const char*, const Mat& in) { in_ = in; return 0; }

// y[M,N] = x[M,K] W[N,K]^T + b, fp32.  Tasks = (128-column panel, 480-row
// chunk); each task packs its W panel K-major once, then runs a 6x16 AVX2/FMA
// register micro-kernel over its rows.
static void sgemm(const float* x, int M, int K, const float* W, int N, const float* b, float* y) {
    constexpr int NB = 128, MC = 480, MR = 6;
    const int nbn = (N + NB - 1) / NB, nbm = (M + MC - 1) / MC;
    #pragma omp parallel
    {
        std::vector<float> Bp((size_t)K * NB);
        #pragma omp for schedule(dynamic, 1)
        for (long t = 0; t < (long)nbn * nbm; t++) {
            const int n0 = (int)(t % nbn) * NB, m0 = (int)(t / nbn) * MC;
            const int nw = std::min(NB, N - n0), m1 = std::min(M, m0 + MC);
            for (int j = 0; j < NB; j++) {
                if (j < nw) { const float* wr = W + (size_t)(n0 + j) * K; for (int k = 0; k < K; k++) Bp[(size_t)k * NB + j] = wr[k]; }
                else for (int k = 0; k < K; k++) Bp[(size_t)k * NB + j] = 0.f;
            }
            for (int r0 = m0; r0 < m1; r0 += MR) {
                const int mr = std::min(MR, m1 - r0);
                const float* xr[MR];
                for (int r = 0; r < MR; r++) xr[r] = x + (size_t)(r0 + (r < mr ? r : 0)) * K;
                for (int c0 = 0; c0 < nw; c0 += 16) {
                    __m256 acc[MR][2];
                    for (int r = 0; r < MR; r++) { acc[r][0] = _mm256_setzero_ps(); acc[r][1] = _mm256_setzero_ps(); }
                    const float* bp = Bp.data() + c0;
                    for (int k = 0; k < K; k++) {
                        const __m256 b0 = _mm256_loadu_ps(bp + (size_t)k * NB), b1 = _mm256_loadu_ps(bp + (size_t)k * NB + 8);
                        for (int r = 0; r < MR; r++) {
                            const __m256 xv = _mm256_broadcast_ss(xr[r] + k);
                            acc[r][0] = _mm256_fmadd_ps(xv, b0, acc[r][0]);
                            acc[r][1] = _mm256_fmadd_ps(xv, b1, acc[r][1]);
                        }
                    }
                    for (int r = 0; r < mr; r++) {
                        float tmp[16];
                        _mm256_storeu_ps(tmp, acc[r][0]); _mm256_storeu_ps(tmp + 8, acc[r][1]);
                        for (int j = 0; j < 16 && c0 + j < nw; j++)
                            y[(size_t)(r0 + r) * N + n0 + c0 + j] = tmp[j] + (b ? b[n0 + c0 + j] : 0.f);
                    }
                }
            }
        }
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
    sgemm((const float*)in_.data, M, K, net->weight.data(), N,
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
