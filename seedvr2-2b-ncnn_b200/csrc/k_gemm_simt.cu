// k_gemm_simt.cu -- fp32-accumulate SIMT GEMM with the DiT's fused epilogues.
//
// y = A[M,K] W[N,K]^T (the ncnn InnerProduct the reference runs per Linear,
// src/dit_vk.cpp:270-293).  This kernel carries the fp32 precision path and
// the ragged shapes (K = 132 of vid_in_proj, M = 1 of the time embedding);
// the bf16 path's large GEMMs run on tcgen05 (k_gemm_tc.cu).
// Tile 128x128x16, 256 threads, 8x8 outputs per thread, register-staged
// double buffering.  Epilogue order mirrors the reference host loops:
// (acc + bias) * gate + residual, each a separately rounded op.
#include "kernels.h"
#include "kcommon.cuh"

namespace s2b {
namespace {

constexpr int BM = 128, BN = 128, BK = 16, PAD = 4;

template <typename T>
__device__ __forceinline__ float ldg_f(const T* p) { return Cvt<T>::to_f(*p); }

template <typename TA, typename TW>
__global__ void __launch_bounds__(256)
k_gemm(const TA* __restrict__ A, int lda, const TW* __restrict__ W, int ldw, int M, int N, int K, GemmEpi e) {
    __shared__ float As[2][BK][BM + PAD];
    __shared__ float Bs[2][BK][BN + PAD];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    // loader mapping: element e = tid + 256*i -> (row e/16, k e%16)
    float ra[8], rb[8];
    auto gload = [&](int k0) {
        #pragma unroll
        for (int i = 0; i < 8; i++) {
            const int el = tid + 256 * i, r = el >> 4, k = el & 15;
            const int gm = m0 + r, gn = n0 + r, gk = k0 + k;
            ra[i] = (gm < M && gk < K) ? ldg_f(A + (size_t)gm * lda + gk) : 0.f;
            rb[i] = (gn < N && gk < K) ? ldg_f(W + (size_t)gn * ldw + gk) : 0.f;
        }
    };
    auto sstore = [&](int buf) {
        #pragma unroll
        for (int i = 0; i < 8; i++) {
            const int el = tid + 256 * i, r = el >> 4, k = el & 15;
            As[buf][k][r] = ra[i];
            Bs[buf][k][r] = rb[i];
        }
    };
    float acc[8][8];
    #pragma unroll
    for (int i = 0; i < 8; i++)
        #pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

    const int nk = (K + BK - 1) / BK;
    gload(0);
    sstore(0);
    __syncthreads();
    for (int kt = 0; kt < nk; kt++) {
        const int buf = kt & 1;
        if (kt + 1 < nk) gload((kt + 1) * BK);
        #pragma unroll
        for (int k = 0; k < BK; k++) {
            float a[8], b[8];
            load4(&As[buf][k][ty * 4], a);
            load4(&As[buf][k][64 + ty * 4], a + 4);
            load4(&Bs[buf][k][tx * 4], b);
            load4(&Bs[buf][k][64 + tx * 4], b + 4);
            #pragma unroll
            for (int i = 0; i < 8; i++)
                #pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (kt + 1 < nk) sstore(buf ^ 1);
        __syncthreads();
    }
    // epilogue
    #pragma unroll
    for (int i = 0; i < 8; i++) {
        const int r = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (r >= M) continue;
        const float* gate = (r < e.gate_split) ? e.gate0 : e.gate1;
        #pragma unroll
        for (int j = 0; j < 8; j++) {
            const int c = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (c >= N) continue;
            float v = acc[i][j];
            if (e.bias) v = __fadd_rn(v, e.bias[c]);
            if (e.mode == EPI_GATE_RESID) {
                if (gate) v = __fmul_rn(v, gate[c]);
                float* dst = e.resid + (size_t)r * e.ldr + c;
                *dst = __fadd_rn(v, *dst);
            } else if (e.out_t == ACT_F32) {
                ((float*)e.out)[(size_t)r * e.ldo + c] = v;
            } else if (e.out_t == ACT_F16) {
                ((f16*)e.out)[(size_t)r * e.ldo + c] = __float2half_rn(v);
            } else {
                ((bf16*)e.out)[(size_t)r * e.ldo + c] = __float2bfloat16_rn(v);
            }
        }
    }
}

// y[n] = act(sum_k x[k] W[n][k] + b[n]) for one input row (the time-embedding
// MLP): one warp per output, float4 loads of the weight row, x staged in
// shared memory, a fixed-order shuffle reduction.
constexpr int GEMV_WARPS = 8;
__global__ void __launch_bounds__(GEMV_WARPS * 32)
k_gemv_f32(const float* __restrict__ x, int K, const float* __restrict__ W, int ldw, int N,
           const float* __restrict__ bias, float* __restrict__ y, int silu) {
    extern __shared__ float xs[];
    for (int k = threadIdx.x; k < K; k += blockDim.x) xs[k] = x[k];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * GEMV_WARPS + (threadIdx.x >> 5);
    if (n >= N) return;
    const float4* w = reinterpret_cast<const float4*>(W + (size_t)n * ldw);
    float acc = 0.f;
    for (int c = lane; c < K / 4; c += 32) {
        const float4 a = __ldcs(w + c);
        const float4 b = *reinterpret_cast<const float4*>(xs + 4 * c);
        acc = fmaf(a.x, b.x, acc); acc = fmaf(a.y, b.y, acc);
        acc = fmaf(a.z, b.z, acc); acc = fmaf(a.w, b.w, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) {
        float v = bias ? __fadd_rn(acc, bias[n]) : acc;
        y[n] = silu ? silu_f(v) : v;
    }
}

}  // namespace

bool gemv_f32(const float* x, int K, const float* W, int ldw, int N, const float* bias, float* y, bool silu,
              cudaStream_t s) {
    if (K % 4 || ldw % 4 || ((uintptr_t)W & 15) || ((uintptr_t)x & 15) || K > 12288) return false;
    k_gemv_f32<<<(N + GEMV_WARPS - 1) / GEMV_WARPS, GEMV_WARPS * 32, K * sizeof(float), s>>>(x, K, W, ldw, N, bias, y,
                                                                                             silu ? 1 : 0);
    return true;
}

void gemm_simt(const void* A, ActT at, int lda, const void* W, ActT wt, int ldw, int M, int N, int K,
               const GemmEpi& e, cudaStream_t s) {
    if (M <= 0 || N <= 0) return;
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    if (at == ACT_F32 && wt == ACT_F32)
        k_gemm<float, float><<<grid, 256, 0, s>>>((const float*)A, lda, (const float*)W, ldw, M, N, K, e);
    else if (at == ACT_BF16 && wt == ACT_BF16)
        k_gemm<bf16, bf16><<<grid, 256, 0, s>>>((const bf16*)A, lda, (const bf16*)W, ldw, M, N, K, e);
    else if (at == ACT_F16 && wt == ACT_F16)
        k_gemm<f16, f16><<<grid, 256, 0, s>>>((const f16*)A, lda, (const f16*)W, ldw, M, N, K, e);
    else if (at == ACT_F32 && wt == ACT_BF16)
        k_gemm<float, bf16><<<grid, 256, 0, s>>>((const float*)A, lda, (const bf16*)W, ldw, M, N, K, e);
    else
        k_gemm<bf16, float><<<grid, 256, 0, s>>>((const bf16*)A, lda, (const float*)W, ldw, M, N, K, e);
}

}  // namespace s2b
