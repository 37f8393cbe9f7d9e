// k_gemm_tc.cu -- persistent tcgen05 BF16 GEMM with the DiT's fused epilogues.
//
// C[M,N] = A[M,K] B[N,K]^T, A/B bf16 K-major, fp32 accumulation in TMEM.
// One CTA per SM loops over 128x256 output tiles (m fastest, so the CTAs in
// flight share a few B column blocks and the A panel stays in L2):
//   warp 0      TMA producer: A 128x64 and B 256x64 tiles, 128-byte swizzle,
//               STAGES-deep ring guarded by full/empty mbarriers;
//   warp 1      allocates 512 TMEM columns (two 256-column accumulators) and
//               issues tcgen05.mma (M=128, N=256, K=16) from one thread,
//               releasing smem stages and publishing accumulators with
//               tcgen05.commit;
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns at a time, fused
//               bias / adaLN gate + fp32 residual / SwiGLU, direct stores;
//               the accumulator is handed back once read, so the next
//               tile's MMAs overlap this tile's epilogue.
// Loads are plain (non-multicast) TMA tile loads of this GPU's memory.
// Every mbarrier wait is bounded; on expiry the kernel records an error in
// g_tc_err, waits (bounded) for its own TMA loads, frees TMEM and returns.
#include "kernels.h"
#include "kcommon.cuh"
#include "sm100.cuh"
#include <cuda.h>
#include <mutex>

namespace s2b {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 192;
constexpr int ACC_COLS = 256, NUM_ACC = 2, TMEM_COLS = ACC_COLS * NUM_ACC;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t IDESC = sm100::idesc_bf16_f32(BM, BN);

__device__ int g_tc_err;

struct TcParams {
    int M, N, num_m, num_n, num_kb;
    GemmEpi e;
};

struct Ctl {
    uint64_t full[STAGES], empty[STAGES], tfull[NUM_ACC], tempty[NUM_ACC];
    uint32_t tmem_slot;
    int abort;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    for (uint32_t i = 0; i < sm100::WAIT_LIMIT; i++) {
        if (sm100::mbar_try_wait(bar, parity)) return true;
        if ((i & 1023) == 1023 && *abort_flag) return false;
    }
    *abort_flag = 1;
    atomicExch(&g_tc_err, 1);
    return false;
}

__device__ __forceinline__ void store32(float* dst, const float v[32]) {
    #pragma unroll
    for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
}
__device__ __forceinline__ void store32(bf16* dst, const float v[32]) {
    #pragma unroll
    for (int j = 0; j < 32; j += 8) {
        uint4 u;
        __nv_bfloat162 a = __floats2bfloat162_rn(v[j], v[j + 1]), b = __floats2bfloat162_rn(v[j + 2], v[j + 3]);
        __nv_bfloat162 c = __floats2bfloat162_rn(v[j + 4], v[j + 5]), d = __floats2bfloat162_rn(v[j + 6], v[j + 7]);
        u.x = *reinterpret_cast<uint32_t*>(&a); u.y = *reinterpret_cast<uint32_t*>(&b);
        u.z = *reinterpret_cast<uint32_t*>(&c); u.w = *reinterpret_cast<uint32_t*>(&d);
        *reinterpret_cast<uint4*>(dst + j) = u;
    }
}

__device__ __forceinline__ void epilogue_tile(const TcParams& p, uint32_t taddr, int row, int n0) {
    const GemmEpi& e = p.e;
    const bool row_ok = row < p.M;
    if (e.mode == EPI_SWIGLU) {
        // column block [h 128 | g 128] -> 128 outputs at n0 / 2
        #pragma unroll 1
        for (int jc = 0; jc < 4; jc++) {
            float h[32], g[32];
            sm100::tmem_ld32(taddr + jc * 32, h);
            sm100::tmem_ld32(taddr + 128 + jc * 32, g);
            if (!row_ok) continue;
            #pragma unroll
            for (int j = 0; j < 32; j++) h[j] = __fmul_rn(silu_f(g[j]), h[j]);
            const size_t off = (size_t)row * e.ldo + n0 / 2 + jc * 32;
            if (e.out_t == ACT_BF16) store32((bf16*)e.out + off, h);
            else store32((float*)e.out + off, h);
        }
        return;
    }
    const float* gate = (row < e.gate_split) ? e.gate0 : e.gate1;
    #pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
        if (n0 + c0 >= p.N) break;             // warp-uniform
        float v[32];
        sm100::tmem_ld32(taddr + c0, v);
        if (!row_ok) continue;
        const int col = n0 + c0;
        const bool full = col + 32 <= p.N;
        if (e.bias) {
            #pragma unroll
            for (int j = 0; j < 32; j++) v[j] = __fadd_rn(v[j], (full || col + j < p.N) ? e.bias[col + j] : 0.f);
        }
        if (e.mode == EPI_GATE_RESID) {
            float* dst = e.resid + (size_t)row * e.ldr + col;
            if (full) {
                #pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    float4 r = *reinterpret_cast<const float4*>(dst + j);
                    float g0 = gate ? gate[col + j] : 1.f, g1 = gate ? gate[col + j + 1] : 1.f;
                    float g2 = gate ? gate[col + j + 2] : 1.f, g3 = gate ? gate[col + j + 3] : 1.f;
                    r.x = __fadd_rn(gate ? __fmul_rn(v[j], g0) : v[j], r.x);
                    r.y = __fadd_rn(gate ? __fmul_rn(v[j + 1], g1) : v[j + 1], r.y);
                    r.z = __fadd_rn(gate ? __fmul_rn(v[j + 2], g2) : v[j + 2], r.z);
                    r.w = __fadd_rn(gate ? __fmul_rn(v[j + 3], g3) : v[j + 3], r.w);
                    *reinterpret_cast<float4*>(dst + j) = r;
                }
            } else {
                for (int j = 0; j < 32 && col + j < p.N; j++) {
                    const float t = gate ? __fmul_rn(v[j], gate[col + j]) : v[j];
                    dst[j] = __fadd_rn(t, dst[j]);
                }
            }
        } else {
            const size_t off = (size_t)row * e.ldo + col;
            if (full) {
                if (e.out_t == ACT_BF16) store32((bf16*)e.out + off, v);
                else store32((float*)e.out + off, v);
            } else {
                for (int j = 0; j < 32 && col + j < p.N; j++) {
                    if (e.out_t == ACT_BF16) ((bf16*)e.out)[off + j] = __float2bfloat16_rn(v[j]);
                    else ((float*)e.out)[off + j] = v[j];
                }
            }
        }
    }
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_BYTES;
    Ctl* ctl = reinterpret_cast<Ctl*>(smem + STAGES * STAGE_BYTES);
    volatile int* abort_flag = &ctl->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_tiles = p.num_m * p.num_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) { sm100::mbar_init(&ctl->full[s], 1); sm100::mbar_init(&ctl->empty[s], 1); }
        for (int a = 0; a < NUM_ACC; a++) { sm100::mbar_init(&ctl->tfull[a], 1); sm100::mbar_init(&ctl->tempty[a], 4); }
        ctl->abort = 0;
        sm100::fence_barrier_init();
        sm100::tma_prefetch_desc(&tA);
        sm100::tma_prefetch_desc(&tB);
    }
    if (warp == 1) {
        sm100::tmem_alloc(&ctl->tmem_slot, TMEM_COLS);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem_base = ctl->tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            long issued = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const int mb = tile % p.num_m, nb = tile / p.num_m;
                for (int kb = 0; kb < p.num_kb; kb++) {
                    if (!wait_or_abort(&ctl->empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
                    sm100::mbar_arrive_expect_tx(&ctl->full[stage], STAGE_BYTES);
                    sm100::tma_load_2d(sA + stage * A_BYTES, &tA, &ctl->full[stage], kb * BK, mb * BM);
                    sm100::tma_load_2d(sB + stage * B_BYTES, &tB, &ctl->full[stage], kb * BK, nb * BN);
                    issued++;
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
            }
            if (!ok) {
                // drain our own loads still in flight (bounded) before smem goes away
                const long n = issued < STAGES ? issued : STAGES;
                for (long i = 1; i <= n; i++) {
                    const long k = issued - i;
                    const uint32_t s = (uint32_t)(k % STAGES), ph = (uint32_t)((k / STAGES) & 1);
                    for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->full[s], ph); w++) {}
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, it++) {
                const int acc = it & 1;
                const uint32_t acc_phase = (it >> 1) & 1;
                if (!wait_or_abort(&ctl->tempty[acc], acc_phase ^ 1, abort_flag)) { ok = false; break; }
                sm100::tc_fence_after();
                const uint32_t d = tmem_base + acc * ACC_COLS;
                for (int kb = 0; kb < p.num_kb; kb++) {
                    if (!wait_or_abort(&ctl->full[stage], phase, abort_flag)) { ok = false; break; }
                    sm100::tc_fence_after();
                    const uint8_t* a = sA + stage * A_BYTES;
                    const uint8_t* b = sB + stage * B_BYTES;
                    #pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++)
                        sm100::mma_bf16(d, sm100::desc_kmajor_sw128(a, kk * 32), sm100::desc_kmajor_sw128(b, kk * 32),
                                        IDESC, (kb | kk) != 0);
                    sm100::mma_commit(&ctl->empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
                if (ok) sm100::mma_commit(&ctl->tfull[acc]);
            }
        }
    } else {
        const int q = warp & 3;                 // TMEM lane quadrant this warp may access
        int it = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, it++) {
            const int acc = it & 1;
            const uint32_t acc_phase = (it >> 1) & 1;
            // warp-uniform outcome: the tcgen05.ld below are warp-collective
            if (!__all_sync(0xffffffffu, wait_or_abort(&ctl->tfull[acc], acc_phase, abort_flag))) break;
            sm100::tc_fence_after();
            const int mb = tile % p.num_m, nb = tile / p.num_m;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * ACC_COLS;
            epilogue_tile(p, taddr, mb * BM + q * 32 + lane, nb * BN);
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&ctl->tempty[acc]);
        }
    }
    __syncthreads();
    if (warp == 1) {
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int g_num_sms[64];

}  // namespace

// bf16 [rows][cols] with row stride ld elements; box = box_rows x box_cols
// (box_cols * 2 = 128 bytes: one 128-B swizzle row), 128-B swizzle, zero fill.
bool make_tmap_bf16(CUtensorMap* m, const void* base, int rows, int cols, int ld, int box_rows, int box_cols) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool gemm_tc_supported(int M, int N, int K, int lda, int ldw) {
    return M > 0 && N > 0 && K > 0 && N % 32 == 0 && lda % 8 == 0 && ldw % 8 == 0 && encode_fn() != nullptr;
}

int gemm_tc(const void* A, int lda, const void* W, int ldw, int M, int N, int K, const GemmEpi& e, cudaStream_t s,
            int* launches) {
    if (!gemm_tc_supported(M, N, K, lda, ldw)) return -1;
    if (((uintptr_t)A & 15) || ((uintptr_t)W & 15)) return -1;
    if (e.mode == EPI_SWIGLU && N % BN) return -1;
    CUtensorMap ta, tb;
    if (!make_tmap_bf16(&ta, A, M, K, lda, BM, BK) || !make_tmap_bf16(&tb, W, N, K, ldw, BN, BK)) return -1;
    TcParams p;
    p.M = M; p.N = N;
    p.num_m = (M + BM - 1) / BM;
    p.num_n = (N + BN - 1) / BN;
    p.num_kb = (K + BK - 1) / BK;
    p.e = e;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = (dev < 64 && g_num_sms[dev] > 0) ? g_num_sms[dev] : 148;
    const int tiles = p.num_m * p.num_n;
    const int grid = tiles < sms ? tiles : sms;
    k_gemm_tc<<<grid, NUM_THREADS, SMEM_BYTES, s>>>(ta, tb, p);
    if (launches) (*launches)++;
    return 0;
}

int gemm_tc_error_reset(int* had_error) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_err, sizeof v);
    if (e != cudaSuccess) return (int)e;
    if (had_error) *had_error = v;
    const int zero = 0;
    return (int)cudaMemcpyToSymbol(g_tc_err, &zero, sizeof zero);
}

int awa_init_device();
int awa_tc_init_device();

int kernels_init_device() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64) cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    if (int rc = awa_tc_init_device()) return rc;
    return awa_init_device();
}

}  // namespace s2b
