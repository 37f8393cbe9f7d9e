// k_elementwise.cu -- HBM-bound row kernels: RMSNorm + adaLN modulate,
// SwiGLU combine, SiLU, AdaCompose, conversions.
//
// Arithmetic follows the reference host loops operation by operation, with
// explicit round-to-nearest intrinsics so the compiler does not fuse a
// multiply and an add the reference keeps separate (it builds with
// -ffp-contract=off, CMakeLists.txt:220-228):
//   RMSNorm  r = 1/sqrtf(mean(x^2 in double) + eps); y = x*r*w   (src/dit_vk.cpp:48-52)
//   modulate y*(emb[6d+ks]+scB) + (emb[6d+kh]+shB)               (src/dit_vk.cpp:532-545)
//   SwiGLU   silu(g)*h                                            (src/dit_vk.cpp:465-471)
#include "kernels.h"
#include "kcommon.cuh"
#include <cuda_fp16.h>

namespace s2b {

namespace {

constexpr int NORM_THREADS = 320;   // 2560 / 320 = 8 elements per thread, 2 x float4

template <typename TO>
__global__ void __launch_bounds__(NORM_THREADS)
k_rmsnorm_mod(const float* __restrict__ X, int ldx, int split, const float* __restrict__ sc0,
              const float* __restrict__ sh0, const float* __restrict__ sc1, const float* __restrict__ sh1,
              const float* __restrict__ affine, float eps, TO* __restrict__ Y, int ldy) {
    constexpr int D = 2560;
    const int r = blockIdx.x;
    const float* x = X + (size_t)r * ldx;
    const int c0 = threadIdx.x * 4, c1 = c0 + D / 2;
    float a[4], b[4];
    load4(x + c0, a);
    load4(x + c1, b);
    double s = 0;
    #pragma unroll
    for (int j = 0; j < 4; j++) s += (double)a[j] * a[j] + (double)b[j] * b[j];
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __shared__ double part[NORM_THREADS / 32];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    double tot = 0;
    #pragma unroll
    for (int w = 0; w < NORM_THREADS / 32; w++) tot += part[w];
    const float rr = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)(tot / D), eps)));
    const float* sc = (r < split) ? sc0 : sc1;
    const float* sh = (r < split) ? sh0 : sh1;
    float ya[4], yb[4];
    #pragma unroll
    for (int j = 0; j < 4; j++) {
        float u = __fmul_rn(a[j], rr), v = __fmul_rn(b[j], rr);
        if (affine) { u = __fmul_rn(u, affine[c0 + j]); v = __fmul_rn(v, affine[c1 + j]); }
        if (sc) {
            u = __fadd_rn(__fmul_rn(u, sc[c0 + j]), sh[c0 + j]);
            v = __fadd_rn(__fmul_rn(v, sc[c1 + j]), sh[c1 + j]);
        }
        ya[j] = u; yb[j] = v;
    }
    store4(Y + (size_t)r * ldy + c0, ya);
    store4(Y + (size_t)r * ldy + c1, yb);
}

// The same arithmetic with one warp per row: every lane keeps 20 float4 of
// its row in registers (80 B of loads in flight per lane before the first
// use), the sum of squares is reduced with warp shuffles only, and the
// modulation vectors are read as float4.
constexpr int NORM_ROWS = 4;   // rows (warps) per block
template <typename TO>
__global__ void __launch_bounds__(NORM_ROWS * 32, 3)
k_rmsnorm_mod_w(const float* __restrict__ X, int ldx, int rows, int split, const float* __restrict__ sc0,
                const float* __restrict__ sh0, const float* __restrict__ sc1, const float* __restrict__ sh1,
                const float* __restrict__ affine, float eps, TO* __restrict__ Y, int ldy) {
    constexpr int D = 2560, V = D / 128;
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * NORM_ROWS + (threadIdx.x >> 5);
    if (r >= rows) return;
    const float4* x = reinterpret_cast<const float4*>(X + (size_t)r * ldx);
    float4 v[V];
    #pragma unroll
    for (int k = 0; k < V; k++) v[k] = x[k * 32 + lane];
    double s = 0;
    #pragma unroll
    for (int k = 0; k < V; k++)
        s += (double)v[k].x * v[k].x + (double)v[k].y * v[k].y + (double)v[k].z * v[k].z + (double)v[k].w * v[k].w;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float rr = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)(s / D), eps)));
    const float* sc = (r < split) ? sc0 : sc1;
    const float* sh = (r < split) ? sh0 : sh1;
    TO* y = Y + (size_t)r * ldy;
    #pragma unroll
    for (int k = 0; k < V; k++) {
        const int c = (k * 32 + lane) * 4;
        float u[4] = {__fmul_rn(v[k].x, rr), __fmul_rn(v[k].y, rr), __fmul_rn(v[k].z, rr), __fmul_rn(v[k].w, rr)};
        if (affine) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(affine + c));
            u[0] = __fmul_rn(u[0], a.x); u[1] = __fmul_rn(u[1], a.y); u[2] = __fmul_rn(u[2], a.z); u[3] = __fmul_rn(u[3], a.w);
        }
        if (sc) {
            const float4 m = __ldg(reinterpret_cast<const float4*>(sc + c));
            const float4 b = __ldg(reinterpret_cast<const float4*>(sh + c));
            u[0] = __fadd_rn(__fmul_rn(u[0], m.x), b.x);
            u[1] = __fadd_rn(__fmul_rn(u[1], m.y), b.y);
            u[2] = __fadd_rn(__fmul_rn(u[2], m.z), b.z);
            u[3] = __fadd_rn(__fmul_rn(u[3], m.w), b.w);
        }
        store4(y + c, u);
    }
}

template <typename TO>
__global__ void k_swiglu(const float* __restrict__ HG, int M, int ldhg, TO* __restrict__ Hs, int ldh) {
    // one thread per 4 outputs; HG column block b holds [h 128 | g 128]
    const size_t per_row = 6912 / 4;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)M * per_row) return;
    const int r = (int)(i / per_row), c = (int)(i % per_row) * 4;
    const int blk = c >> 7, j = c & 127;
    float h[4], g[4], o[4];
    load4(HG + (size_t)r * ldhg + blk * 256 + j, h);
    load4(HG + (size_t)r * ldhg + blk * 256 + 128 + j, g);
    #pragma unroll
    for (int k = 0; k < 4; k++) o[k] = __fmul_rn(silu_f(g[k]), h[k]);
    store4(Hs + (size_t)r * ldh + c, o);
}

__global__ void k_silu(float* x, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = silu_f(x[i]);
}

// AdaCompose output order (src/ada_compose.cpp:16, :180-195): per layer and
// flow [a_sc,a_sh,a_g,m_sc,m_sh,m_g] read emb slots {1,0,2,4,3,5}; the two
// final vectors fin_sc, fin_sh read slots 1, 0.
__global__ void k_ada_compose(const float* __restrict__ emb, const float* __restrict__ branch, int nvec,
                              float* __restrict__ out) {
    const int v = blockIdx.y, d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= 2560 || v >= nvec) return;
    const int nlay = nvec - 2;
    int k;
    if (v < nlay) { const int kmap[6] = {1, 0, 2, 4, 3, 5}; k = kmap[v % 6]; }
    else k = (v == nlay) ? 1 : 0;
    out[(size_t)v * 2560 + d] = __fadd_rn(emb[d * 6 + k], branch[(size_t)v * 2560 + d]);
}

template <typename TO>
__global__ void k_pad_convert(const float* __restrict__ src, int rows, int cols, TO* __restrict__ dst, int ld) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)rows * ld) return;
    const int r = (int)(i / ld), c = (int)(i % ld);
    dst[i] = Cvt<TO>::from_f(c < cols ? src[(size_t)r * cols + c] : 0.f);
}

template <typename TO>
__global__ void k_ingest(const void* __restrict__ src, bool f16, int out, int in, TO* __restrict__ dst, int ld,
                         int blk_rows, int blk_stride, int row_off) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)out * ld) return;
    const int r = (int)(i / ld), c = (int)(i % ld);
    float v = 0.f;
    if (c < in) v = f16 ? __half2float(((const __half*)src)[(size_t)r * in + c]) : ((const float*)src)[(size_t)r * in + c];
    const int dr = blk_rows > 0 ? (r / blk_rows) * blk_stride + row_off + r % blk_rows : r;
    dst[(size_t)dr * ld + c] = Cvt<TO>::from_f(v);
}

__global__ void k_copy_rows(const float* __restrict__ src, int ld_src, const int* __restrict__ src_idx,
                            float* __restrict__ dst, int ld_dst, const int* __restrict__ dst_idx, int n, int width) {
    const int r = blockIdx.x;
    if (r >= n) return;
    const int sr = src_idx ? src_idx[r] : r, dr = dst_idx ? dst_idx[r] : r;
    const float4* a = reinterpret_cast<const float4*>(src + (size_t)sr * ld_src);
    float4* b = reinterpret_cast<float4*>(dst + (size_t)dr * ld_dst);
    for (int c = threadIdx.x; c < width / 4; c += blockDim.x) b[c] = a[c];
}

template <typename TI>
__global__ void k_to_f32(const TI* __restrict__ src, size_t n, float* __restrict__ dst) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = Cvt<TI>::to_f(src[i]);
}

// x rounded to the nearest tf32 (10 explicit mantissa bits, ties to even).
__device__ __forceinline__ float round_tf32(float x) {
    uint32_t b = __float_as_uint(x);
    if ((b & 0x7F800000u) != 0x7F800000u) b = (b + 0xFFFu + ((b >> 13) & 1u)) & 0xFFFFE000u;
    return __uint_as_float(b);
}

// hi = tf32(x), lo = tf32(x - hi) (x - hi is exact in fp32).  Rounding lo to
// tf32 here, rather than leaving the tensor core to drop its low 13 mantissa
// bits, makes hi + lo carry x to within half a unit of its 22nd significant
// bit instead of a whole one.
__global__ void k_split_tf32(const float* __restrict__ src, int ld_src, int rows, int cols, float* __restrict__ dst,
                             int ld_dst) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)rows * cols) return;
    const int r = (int)(i / cols), c = (int)(i % cols);
    const float x = src[(size_t)r * ld_src + c];
    const float hi = round_tf32(x);
    dst[(size_t)r * ld_dst + c] = hi;
    dst[(size_t)r * ld_dst + cols + c] = round_tf32(__fsub_rn(x, hi));
}

}  // namespace

void split_tf32(const float* src, int ld_src, int rows, int cols, float* dst, int ld_dst, cudaStream_t s) {
    const size_t n = (size_t)rows * cols;
    if (n) k_split_tf32<<<(int)((n + 255) / 256), 256, 0, s>>>(src, ld_src, rows, cols, dst, ld_dst);
}

void rmsnorm_mod(const float* X, int ldx, int rows, int split, const float* sc0, const float* sh0,
                 const float* sc1, const float* sh1, const float* affine, float eps, void* Y, int ldy,
                 ActT yt, cudaStream_t s) {
    if (rows <= 0) return;
    // float4 paths need 16-byte aligned rows and vectors (always true for the
    // 2560-wide buffers this library allocates)
    const bool vec = ((uintptr_t)X % 16 == 0) && ldx % 4 == 0 && ldy % 4 == 0 && ((uintptr_t)Y % 16 == 0) &&
                     ((uintptr_t)sc0 % 16 == 0) && ((uintptr_t)sh0 % 16 == 0) && ((uintptr_t)sc1 % 16 == 0) &&
                     ((uintptr_t)sh1 % 16 == 0) && ((uintptr_t)affine % 16 == 0);
    if (vec) {
        const int blocks = (rows + NORM_ROWS - 1) / NORM_ROWS;
        if (yt == ACT_F32)
            k_rmsnorm_mod_w<float><<<blocks, NORM_ROWS * 32, 0, s>>>(X, ldx, rows, split, sc0, sh0, sc1, sh1, affine, eps, (float*)Y, ldy);
        else if (yt == ACT_F16)
            k_rmsnorm_mod_w<f16><<<blocks, NORM_ROWS * 32, 0, s>>>(X, ldx, rows, split, sc0, sh0, sc1, sh1, affine, eps, (f16*)Y, ldy);
        else
            k_rmsnorm_mod_w<bf16><<<blocks, NORM_ROWS * 32, 0, s>>>(X, ldx, rows, split, sc0, sh0, sc1, sh1, affine, eps, (bf16*)Y, ldy);
        return;
    }
    if (yt == ACT_F32)
        k_rmsnorm_mod<float><<<rows, NORM_THREADS, 0, s>>>(X, ldx, split, sc0, sh0, sc1, sh1, affine, eps, (float*)Y, ldy);
    else if (yt == ACT_F16)
        k_rmsnorm_mod<f16><<<rows, NORM_THREADS, 0, s>>>(X, ldx, split, sc0, sh0, sc1, sh1, affine, eps, (f16*)Y, ldy);
    else
        k_rmsnorm_mod<bf16><<<rows, NORM_THREADS, 0, s>>>(X, ldx, split, sc0, sh0, sc1, sh1, affine, eps, (bf16*)Y, ldy);
}

void swiglu_rows(const float* HG, int M, int ldhg, void* Hs, int ldh, ActT ht, cudaStream_t s) {
    if (M <= 0) return;
    const size_t n = (size_t)M * (6912 / 4);
    const int blocks = (int)((n + 255) / 256);
    if (ht == ACT_F32) k_swiglu<float><<<blocks, 256, 0, s>>>(HG, M, ldhg, (float*)Hs, ldh);
    else if (ht == ACT_F16) k_swiglu<f16><<<blocks, 256, 0, s>>>(HG, M, ldhg, (f16*)Hs, ldh);
    else k_swiglu<bf16><<<blocks, 256, 0, s>>>(HG, M, ldhg, (bf16*)Hs, ldh);
}

void silu_inplace(float* x, int n, cudaStream_t s) { k_silu<<<(n + 255) / 256, 256, 0, s>>>(x, n); }

void ada_compose(const float* emb, const float* branch, int nvec, float* out, cudaStream_t s) {
    k_ada_compose<<<dim3(10, nvec), 256, 0, s>>>(emb, branch, nvec, out);
}

void pad_convert_rows(const float* src, int rows, int cols, void* dst, int ld_dst, ActT t, cudaStream_t s) {
    const size_t n = (size_t)rows * ld_dst;
    if (!n) return;
    const int blocks = (int)((n + 255) / 256);
    if (t == ACT_F32) k_pad_convert<float><<<blocks, 256, 0, s>>>(src, rows, cols, (float*)dst, ld_dst);
    else if (t == ACT_F16) k_pad_convert<f16><<<blocks, 256, 0, s>>>(src, rows, cols, (f16*)dst, ld_dst);
    else k_pad_convert<bf16><<<blocks, 256, 0, s>>>(src, rows, cols, (bf16*)dst, ld_dst);
}

void convert_f32(const float* src, size_t n, void* dst, ActT t, cudaStream_t s) {
    pad_convert_rows(src, 1, (int)n, dst, (int)n, t, s);
}

void convert_to_f32(const void* src, ActT t, size_t n, float* dst, cudaStream_t s) {
    if (!n) return;
    const int blocks = (int)((n + 255) / 256);
    if (t == ACT_F32) cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToDevice, s);
    else if (t == ACT_F16) k_to_f32<f16><<<blocks, 256, 0, s>>>((const f16*)src, n, dst);
    else k_to_f32<bf16><<<blocks, 256, 0, s>>>((const bf16*)src, n, dst);
}

void copy_rows_f32(const float* src, int ld_src, const int* src_idx, float* dst, int ld_dst, const int* dst_idx,
                   int n, int width, cudaStream_t s) {
    if (n <= 0) return;
    k_copy_rows<<<n, 160, 0, s>>>(src, ld_src, src_idx, dst, ld_dst, dst_idx, n, width);
}

void ingest_weight(const void* src, bool src_f16, int out, int in, void* dst, ActT t, int ld, int blk_rows,
                   int blk_stride, int row_off, cudaStream_t s) {
    const size_t n = (size_t)out * ld;
    const int blocks = (int)((n + 255) / 256);
    if (t == ACT_F32) k_ingest<float><<<blocks, 256, 0, s>>>(src, src_f16, out, in, (float*)dst, ld, blk_rows, blk_stride, row_off);
    else if (t == ACT_F16) k_ingest<f16><<<blocks, 256, 0, s>>>(src, src_f16, out, in, (f16*)dst, ld, blk_rows, blk_stride, row_off);
    else k_ingest<bf16><<<blocks, 256, 0, s>>>(src, src_f16, out, in, (bf16*)dst, ld, blk_rows, blk_stride, row_off);
}

// ---------------------------------------------------------------- kernel error status
__global__ void k_status_fold(int* status, int* f_gemm, int* f_attn, int* f_shard) {
    const int m = (*f_gemm ? KERR_GEMM : 0) | (*f_attn ? KERR_ATTN : 0) | (*f_shard ? KERR_SHARD : 0);
    if (m) {
        *status |= m;
        *f_gemm = 0; *f_attn = 0; *f_shard = 0;
    }
}

__global__ void k_status_raise(int mask, int* f_gemm, int* f_attn, int* f_shard) {
    if (mask & KERR_GEMM) atomicExch(f_gemm, 1);
    if (mask & KERR_ATTN) atomicExch(f_attn, 1);
    if (mask & KERR_SHARD) atomicExch(f_shard, 1);
}

__global__ void k_set_u32(uint32_t* p, uint32_t v) { *p = v; }

int gemm_tc_flag_ptr(int** p);
int awa_tc_flag_ptr(int** p);
int shard_flag_ptr(int** p);

int kernel_flags_get(KernelFlags* f) {
    if (int e = gemm_tc_flag_ptr(&f->gemm)) return e;
    if (int e = awa_tc_flag_ptr(&f->attn)) return e;
    return shard_flag_ptr(&f->shard);
}

void status_fold(const KernelFlags& f, int* status, cudaStream_t s) {
    k_status_fold<<<1, 1, 0, s>>>(status, f.gemm, f.attn, f.shard);
}

void status_raise(const KernelFlags& f, int mask, cudaStream_t s) {
    k_status_raise<<<1, 1, 0, s>>>(mask, f.gemm, f.attn, f.shard);
}

void set_u32(uint32_t* p, uint32_t v, cudaStream_t s) { k_set_u32<<<1, 1, 0, s>>>(p, v); }

// ---------------------------------------------------------------- bf16 GEMV
// One warp per output row: lanes take 8-element slices of the row in a fixed
// order, then a fixed butterfly sum.
__global__ void k_gemv_bf16(const bf16* __restrict__ W, int ld, int N, int K, const float* __restrict__ x,
                            float* __restrict__ y) {
    const int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (n >= N) return;
    const bf16* w = W + (size_t)n * ld;
    float a = 0.f;
    for (int k = lane * 8; k < K; k += 256) {
        const uint4 u = *reinterpret_cast<const uint4*>(w + k);
        const bf16* wb = reinterpret_cast<const bf16*>(&u);
        #pragma unroll
        for (int j = 0; j < 8; j++) a = fmaf(__bfloat162float(wb[j]), __ldg(x + k + j), a);
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) y[n] = a;
}

void gemv_bf16(const void* W, int ld, int N, int K, const float* x, float* y, cudaStream_t s) {
    if (N <= 0) return;
    k_gemv_bf16<<<(N + 7) / 8, 256, 0, s>>>((const bf16*)W, ld, N, K, x, y);
}

}  // namespace s2b
