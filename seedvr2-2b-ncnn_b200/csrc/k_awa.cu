// k_awa.cu -- Adaptive Window Attention: pack (qk-norm + RoPE), SIMT
// attention, txt coalesce.
//
// Semantics (the reference CPU attention, src/dit_vk.cpp:345-455, and
// awa.comp): per head, q and k rows get RMSNorm over the 128 head dims
// (x / sqrt(mean(x^2)+eps) * w, a 128-vector shared by all heads), then RoPE
// on dims 0..125 with the element's own angle:
//   out[k] = q[k]*cos(f[k]) + (k even ? -q[k+1] : q[k-1]) * sin(f[k]).
// Window i attends over S_i = f_i + TXT keys [its vid tokens | all txt
// tokens] with softmax(q k^T / sqrt(128)).  vid outputs return to their grid
// token; each window's txt outputs are kept and averaged over windows.
//
// Layout: the pack kernel writes Q/K/V window-packed and head-major,
// P[h][p][128] with p = cums[i] + s (s < f_i: vid, else txt), so a window's
// keys are one contiguous [S_i x 128] slab per head -- the tile shape the
// tensor-core attention streams with TMA.
#include "kernels.h"
#include "kcommon.cuh"
#include <math_constants.h>

namespace s2b {
namespace {

// fp32 x as three bf16 parts with x == hi + mid + lo to fp32 precision:
// hi = rn(x), mid = rn(x - hi), lo = rn(x - hi - mid).  Both differences are
// exact in fp32 (each drops the leading 8 significant bits), so the parts
// carry x's 24-bit significand.
__device__ __forceinline__ void split3_bf16(float x, bf16& hi, bf16& mid, bf16& lo) {
    hi = __float2bfloat16_rn(x);
    const float r = __fsub_rn(x, __bfloat162float(hi));
    mid = __float2bfloat16_rn(r);
    lo = __float2bfloat16_rn(__fsub_rn(r, __bfloat162float(mid)));
}

// Four consecutive values as their three bf16 parts, part k at p + k * part.
__device__ __forceinline__ void store4_split3(bf16* p, size_t part, const float v[4]) {
    uint32_t w[3][2];
    #pragma unroll
    for (int j = 0; j < 4; j += 2) {
        bf16 a[3], b[3];
        split3_bf16(v[j], a[0], a[1], a[2]);
        split3_bf16(v[j + 1], b[0], b[1], b[2]);
        #pragma unroll
        for (int k = 0; k < 3; k++)
            w[k][j >> 1] = (uint32_t)__bfloat16_as_ushort(a[k]) | ((uint32_t)__bfloat16_as_ushort(b[k]) << 16);
    }
    #pragma unroll
    for (int k = 0; k < 3; k++) *reinterpret_cast<uint2*>(p + k * part) = make_uint2(w[k][0], w[k][1]);
}

// SPLIT3: TP is bf16 and each of Qp/Kp/Vp holds three parts of
// [HEADS][sumS][128] (hi, mid, lo), 20 * sumS * 128 elements apart.
template <typename TI, typename TP, bool SPLIT3 = false>
__global__ void __launch_bounds__(640)
k_awa_pack(const TI* __restrict__ vqkv, const TI* __restrict__ tqkv, int ldq, AwaDev g,
           const float* __restrict__ nqv, const float* __restrict__ nkv, const float* __restrict__ nqt,
           const float* __restrict__ nkt, float eps, TP* __restrict__ Qp, TP* __restrict__ Kp, TP* __restrict__ Vp) {
    const int p = blockIdx.x;            // packed row
    const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wi = g.row_win[p];
    const int s = p - g.cums[wi];
    const int f = g.cumf[wi + 1] - g.cumf[wi];
    const TI* row;
    const float *cs, *sn, *wq, *wk;
    if (s < f) {
        const int gi = g.cumf[wi] + s;
        row = vqkv + (size_t)g.vidx[gi] * ldq;
        cs = g.vcos + (size_t)gi * 126; sn = g.vsin + (size_t)gi * 126;
        wq = nqv; wk = nkv;
    } else {
        const int ti = s - f;
        row = tqkv + (size_t)ti * ldq;
        cs = g.tcos + (size_t)(wi * g.TXT + ti) * 126; sn = g.tsin + (size_t)(wi * g.TXT + ti) * 126;
        wq = nqt; wk = nkt;
    }
    const int d0 = lane * 4;
    const size_t dst = ((size_t)h * g.sumS + p) * 128 + d0;
    #pragma unroll
    for (int which = 0; which < 2; which++) {
        float x[4], w[4], o[4];
        load4(row + which * 2560 + h * 128 + d0, x);
        load4(which == 0 ? wq + d0 : wk + d0, w);
        float sq = 0.f;
        #pragma unroll
        for (int j = 0; j < 4; j++) sq = fmaf(x[j], x[j], sq);
        sq = warp_sum(sq);
        const float r = sqrtf(__fadd_rn(__fdiv_rn(sq, 128.f), eps));
        #pragma unroll
        for (int j = 0; j < 4; j++) x[j] = __fmul_rn(__fdiv_rn(x[j], r), w[j]);
        #pragma unroll
        for (int j = 0; j < 4; j++) {
            const int k = d0 + j;
            if (k < 126) {
                const float rh = (j & 1) ? x[j - 1] : -x[j + 1];
                o[j] = __fadd_rn(__fmul_rn(x[j], cs[k]), __fmul_rn(rh, sn[k]));
            } else {
                o[j] = x[j];
            }
        }
        if constexpr (SPLIT3) store4_split3((which == 0 ? Qp : Kp) + dst, (size_t)20 * g.sumS * 128, o);
        else store4((which == 0 ? Qp : Kp) + dst, o);
    }
    float v[4];
    load4(row + 2 * 2560 + h * 128 + d0, v);
    if constexpr (SPLIT3) store4_split3(Vp + dst, (size_t)20 * g.sumS * 128, v);
    else store4(Vp + dst, v);
}

// SIMT flash attention: CTA = 64 queries of one (window, head); 4 threads per
// query, each owning 32 of the 128 dims (interleaved in float4 chunks).
constexpr int QT = 64, KT = 64;

template <typename TP, typename TO>
__global__ void __launch_bounds__(256)
k_awa_attn_simt(const TP* __restrict__ Qp, const TP* __restrict__ Kp, const TP* __restrict__ Vp, AwaDev g,
                float scale, TO* __restrict__ att, int ld_att, float* __restrict__ toutw) {
    extern __shared__ float sm[];
    float* Ks = sm;               // [KT][128]
    float* Vs = sm + KT * 128;    // [KT][128]
    const int wi = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * QT;
    const int f = g.cumf[wi + 1] - g.cumf[wi];
    const int S = f + g.TXT;
    if (q0 >= S) return;
    const int base = g.cums[wi];
    const int tid = threadIdx.x, qi = tid >> 2, qq = tid & 3;
    const int qrow = q0 + qi;
    const bool qvalid = qrow < S;
    float q[32], o[32];
    const TP* qp = Qp + ((size_t)h * g.sumS + base + (qvalid ? qrow : 0)) * 128;
    #pragma unroll
    for (int c = 0; c < 8; c++) load4(qp + c * 16 + qq * 4, q + c * 4);
    #pragma unroll
    for (int j = 0; j < 32; j++) o[j] = 0.f;
    float m = -CUDART_INF_F, l = 0.f;
    for (int k0 = 0; k0 < S; k0 += KT) {
        const int nk = min(KT, S - k0);
        __syncthreads();
        for (int e = tid; e < KT * 32; e += 256) {   // float4 units
            const int r = e >> 5, c4 = (e & 31) * 4;
            float kv[4] = {0, 0, 0, 0}, vv[4] = {0, 0, 0, 0};
            if (r < nk) {
                const size_t src = ((size_t)h * g.sumS + base + k0 + r) * 128 + c4;
                load4(Kp + src, kv);
                load4(Vp + src, vv);
            }
            store4(Ks + r * 128 + c4, kv);
            store4(Vs + r * 128 + c4, vv);
        }
        __syncthreads();
        for (int j0 = 0; j0 < nk; j0 += 16) {
            float sc[16];
            float cmax = -CUDART_INF_F;
            #pragma unroll
            for (int jj = 0; jj < 16; jj++) {
                const int j = j0 + jj;
                float part = 0.f;
                if (j < nk) {
                    #pragma unroll
                    for (int c = 0; c < 8; c++) {
                        float kv[4];
                        load4(Ks + j * 128 + c * 16 + qq * 4, kv);
                        part = fmaf(q[c * 4 + 0], kv[0], part);
                        part = fmaf(q[c * 4 + 1], kv[1], part);
                        part = fmaf(q[c * 4 + 2], kv[2], part);
                        part = fmaf(q[c * 4 + 3], kv[3], part);
                    }
                }
                part += __shfl_xor_sync(0xffffffffu, part, 1);
                part += __shfl_xor_sync(0xffffffffu, part, 2);
                sc[jj] = (j < nk) ? part * scale : -CUDART_INF_F;
                cmax = fmaxf(cmax, sc[jj]);
            }
            const float mn = fmaxf(m, cmax);
            const float corr = expf(m - mn);   // m = -inf on the first chunk -> 0
            l *= corr;
            #pragma unroll
            for (int d = 0; d < 32; d++) o[d] *= corr;
            #pragma unroll
            for (int jj = 0; jj < 16; jj++) {
                const int j = j0 + jj;
                if (j >= nk) break;
                const float pj = expf(sc[jj] - mn);
                l += pj;
                #pragma unroll
                for (int c = 0; c < 8; c++) {
                    float vv[4];
                    load4(Vs + j * 128 + c * 16 + qq * 4, vv);
                    o[c * 4 + 0] = fmaf(pj, vv[0], o[c * 4 + 0]);
                    o[c * 4 + 1] = fmaf(pj, vv[1], o[c * 4 + 1]);
                    o[c * 4 + 2] = fmaf(pj, vv[2], o[c * 4 + 2]);
                    o[c * 4 + 3] = fmaf(pj, vv[3], o[c * 4 + 3]);
                }
            }
            m = mn;
        }
    }
    if (!qvalid) return;
    const float inv = 1.f / l;
    #pragma unroll
    for (int d = 0; d < 32; d++) o[d] *= inv;
    if (qrow < f) {
        TO* dst = att + (size_t)g.vidx[g.cumf[wi] + qrow] * ld_att + h * 128;
        #pragma unroll
        for (int c = 0; c < 8; c++) store4(dst + c * 16 + qq * 4, o + c * 4);
    } else {
        float* dst = toutw + ((size_t)wi * g.TXT + (qrow - f)) * 2560 + h * 128;
        #pragma unroll
        for (int c = 0; c < 8; c++) store4(dst + c * 16 + qq * 4, o + c * 4);
    }
}

// One thread per 4 consecutive outputs; the windows are added in window
// order (as the reference's loop, src/dit_vk.cpp:440-444) with the loads of
// 8 windows issued together ahead of their adds.
template <typename TO>
__global__ void k_coalesce(const float* __restrict__ toutw, int nwin, int TXT, TO* __restrict__ out, int ld,
                           float divisor) {
    const int i4 = blockIdx.x * blockDim.x + threadIdx.x;
    if (i4 >= TXT * 640) return;
    const float4* src = reinterpret_cast<const float4*>(toutw) + i4;
    const size_t ws = (size_t)TXT * 640;
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    int w = 0;
    for (; w + 8 <= nwin; w += 8) {
        float4 v[8];
        #pragma unroll
        for (int k = 0; k < 8; k++) v[k] = __ldcs(src + (size_t)(w + k) * ws);
        #pragma unroll
        for (int k = 0; k < 8; k++) {
            a[0] = __fadd_rn(a[0], v[k].x); a[1] = __fadd_rn(a[1], v[k].y);
            a[2] = __fadd_rn(a[2], v[k].z); a[3] = __fadd_rn(a[3], v[k].w);
        }
    }
    for (; w < nwin; w++) {
        const float4 v = __ldcs(src + (size_t)w * ws);
        a[0] = __fadd_rn(a[0], v.x); a[1] = __fadd_rn(a[1], v.y);
        a[2] = __fadd_rn(a[2], v.z); a[3] = __fadd_rn(a[3], v.w);
    }
    if (divisor > 0.f) {
        #pragma unroll
        for (int k = 0; k < 4; k++) a[k] = __fdiv_rn(a[k], divisor);
    }
    const int i = i4 * 4;
    store4(out + (size_t)(i / 2560) * ld + (i % 2560), a);
}

}  // namespace

void awa_pack(const void* vqkv, const void* tqkv, ActT in_t, int ldq, const AwaDev& g, const float* nqv,
              const float* nkv, const float* nqt, const float* nkt, float eps, void* Qp, void* Kp, void* Vp,
              ActT pt, cudaStream_t s) {
    if (g.sumS <= 0) return;
    if (in_t == ACT_F32 && pt == ACT_F32)
        k_awa_pack<float, float><<<g.sumS, 640, 0, s>>>((const float*)vqkv, (const float*)tqkv, ldq, g, nqv, nkv,
                                                        nqt, nkt, eps, (float*)Qp, (float*)Kp, (float*)Vp);
    else if (in_t == ACT_BF16 && pt == ACT_BF16)
        k_awa_pack<bf16, bf16><<<g.sumS, 640, 0, s>>>((const bf16*)vqkv, (const bf16*)tqkv, ldq, g, nqv, nkv,
                                                      nqt, nkt, eps, (bf16*)Qp, (bf16*)Kp, (bf16*)Vp);
    else if (in_t == ACT_F32 && pt == ACT_BF16)
        k_awa_pack<float, bf16><<<g.sumS, 640, 0, s>>>((const float*)vqkv, (const float*)tqkv, ldq, g, nqv, nkv,
                                                       nqt, nkt, eps, (bf16*)Qp, (bf16*)Kp, (bf16*)Vp);
    else if (in_t == ACT_F16 && pt == ACT_F16)
        k_awa_pack<f16, f16><<<g.sumS, 640, 0, s>>>((const f16*)vqkv, (const f16*)tqkv, ldq, g, nqv, nkv,
                                                    nqt, nkt, eps, (f16*)Qp, (f16*)Kp, (f16*)Vp);
    else if (in_t == ACT_F32 && pt == ACT_F16)
        k_awa_pack<float, f16><<<g.sumS, 640, 0, s>>>((const float*)vqkv, (const float*)tqkv, ldq, g, nqv, nkv,
                                                      nqt, nkt, eps, (f16*)Qp, (f16*)Kp, (f16*)Vp);
    else
        k_awa_pack<bf16, float><<<g.sumS, 640, 0, s>>>((const bf16*)vqkv, (const bf16*)tqkv, ldq, g, nqv, nkv,
                                                       nqt, nkt, eps, (float*)Qp, (float*)Kp, (float*)Vp);
}

void awa_pack_split3(const void* vqkv, const void* tqkv, ActT in_t, int ldq, const AwaDev& g, const float* nqv,
                     const float* nkv, const float* nqt, const float* nkt, float eps, void* Q3, void* K3, void* V3,
                     cudaStream_t s) {
    if (g.sumS <= 0) return;
    if (in_t == ACT_F32)
        k_awa_pack<float, bf16, true><<<g.sumS, 640, 0, s>>>((const float*)vqkv, (const float*)tqkv, ldq, g, nqv, nkv,
                                                             nqt, nkt, eps, (bf16*)Q3, (bf16*)K3, (bf16*)V3);
    else
        k_awa_pack<bf16, bf16, true><<<g.sumS, 640, 0, s>>>((const bf16*)vqkv, (const bf16*)tqkv, ldq, g, nqv, nkv,
                                                            nqt, nkt, eps, (bf16*)Q3, (bf16*)K3, (bf16*)V3);
}

int awa_attend_tc(const void* Qp, const void* Kp, const void* Vp, ActT qkv_t, const AwaDev& g, float scale, void* att,
                  int ld_att, ActT at, float* toutw, cudaStream_t s);

int awa_attend(const void* Qp, const void* Kp, const void* Vp, ActT pt, const AwaDev& g, float scale,
               void* att, int ld_att, ActT at, float* toutw, cudaStream_t s, int* launches) {
    if (g.nwin <= 0) return 0;
    // 16-bit operands (bf16 or f16): the tensor-core kernel (k_awa_tc.cu),
    // and nothing else; fp32 operands: the SIMT kernel below
    if (act_half(pt)) {
        if (awa_attend_tc(Qp, Kp, Vp, pt, g, scale, att, ld_att, at, toutw, s) != 0) return -1;
        if (launches) (*launches)++;
        return 0;
    }
    dim3 grid((g.maxS + QT - 1) / QT, 20, g.nwin);
    const size_t smem = 2 * KT * 128 * sizeof(float);
    if (pt == ACT_F32 && at == ACT_F32)
        k_awa_attn_simt<float, float><<<grid, 256, smem, s>>>((const float*)Qp, (const float*)Kp, (const float*)Vp, g, scale, (float*)att, ld_att, toutw);
    else if (pt == ACT_F32)
        k_awa_attn_simt<float, bf16><<<grid, 256, smem, s>>>((const float*)Qp, (const float*)Kp, (const float*)Vp, g, scale, (bf16*)att, ld_att, toutw);
    else if (at == ACT_F32)
        k_awa_attn_simt<bf16, float><<<grid, 256, smem, s>>>((const bf16*)Qp, (const bf16*)Kp, (const bf16*)Vp, g, scale, (float*)att, ld_att, toutw);
    else
        k_awa_attn_simt<bf16, bf16><<<grid, 256, smem, s>>>((const bf16*)Qp, (const bf16*)Kp, (const bf16*)Vp, g, scale, (bf16*)att, ld_att, toutw);
    if (launches) (*launches)++;
    return 0;
}

int awa_init_device() {
    const int smem = 2 * KT * 128 * sizeof(float);
    cudaError_t e = cudaSuccess;
    e = cudaFuncSetAttribute(k_awa_attn_simt<float, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_awa_attn_simt<float, bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_awa_attn_simt<bf16, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_awa_attn_simt<bf16, bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    return e == cudaSuccess ? 0 : (int)e;
}

void awa_coalesce(const float* toutw, int nwin, int TXT, void* att_txt, int ld_att, ActT at, cudaStream_t s) {
    awa_coalesce_div(toutw, nwin, TXT, att_txt, ld_att, at, (float)nwin, s);
}

void awa_coalesce_div(const float* toutw, int nwin, int TXT, void* att_txt, int ld_att, ActT at, float divisor,
                      cudaStream_t s) {
    const int n = TXT * 2560;
    if (n <= 0 || nwin <= 0) return;
    const int n4 = n / 4;
    if (at == ACT_F32) k_coalesce<float><<<(n4 + 127) / 128, 128, 0, s>>>(toutw, nwin, TXT, (float*)att_txt, ld_att, divisor);
    else if (at == ACT_F16) k_coalesce<f16><<<(n4 + 127) / 128, 128, 0, s>>>(toutw, nwin, TXT, (f16*)att_txt, ld_att, divisor);
    else k_coalesce<bf16><<<(n4 + 127) / 128, 128, 0, s>>>(toutw, nwin, TXT, (bf16*)att_txt, ld_att, divisor);
}

}  // namespace s2b
