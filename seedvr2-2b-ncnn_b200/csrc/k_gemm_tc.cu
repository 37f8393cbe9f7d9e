// k_gemm_tc.cu -- persistent tcgen05 16-bit GEMMs with the DiT's fused epilogues.
//
// C[M,N] = A[M,K] B[N,K]^T, A/B K-major and of one 16-bit type (bf16, or IEEE
// binary16 for the fp16 precision: the kind::f16 instruction descriptor's A/B
// format fields come from GemmEpi::op_t at run time), fp32 accumulation in TMEM.
//
// Pair kernel (M > 128, every vid Linear): clusters of two CTAs on two SMs
// share one 256x256 output tile per step through tcgen05 cta_group::2.  Each
// CTA stages only its own 128 A rows and 128 of the 256 B rows per 64-wide
// k-block (32 KB), so per unit of MMA work an SM moves a third less data
// through shared memory than with one CTA per 128x256 tile -- the 1-CTA
// kernel is shared-memory-bandwidth bound (ncu: L1TEX ~80 % busy, tensor
// pipe ~35 %).  Roles per CTA:
//   warp 0      TMA producer: 6-stage ring of [A 128x64 | B 128x64] tiles
//               (128-byte swizzle), two consecutive stages per full / empty
//               barrier (bf16); both CTAs' loads complete on the even CTA's
//               full barrier;
//   warp 1      allocates 512 TMEM columns in both CTAs (two 256-column
//               accumulators); in the even CTA one thread issues
//               tcgen05.mma.cta_group::2 (M=256, N=256, K=16), 8 per barrier
//               group, and signals stage releases / accumulator hand-offs to
//               the same barrier in BOTH CTAs with one tcgen05.commit
//               .multicast::cluster (a barrier arrival, not a data load);
//   warps 2-5   epilogue on this CTA's 128 accumulator rows: tcgen05.ld 32
//               lanes x 32 columns, fused bias / adaLN gate + fp32 residual /
//               SwiGLU, direct stores; then release the accumulator to the
//               even CTA's MMA thread.
// Single kernel (M <= 128: the 58-row txt Linears of layers 0..9): one CTA
// per 128x256 tile, 4-stage ring, same roles within one CTA.
// All loads are plain TMA tile loads of this GPU's memory (no load with
// cluster multicast).  Every mbarrier wait is bounded; on expiry a kernel records
// g_tc_err, drains its own TMA loads (bounded), frees TMEM and returns.
// Warp-collective TMEM instructions run only under warp-uniform control flow.
#include "kernels.h"
#include "kcommon.cuh"
#include "sm100.cuh"
#include <cuda.h>
#include <cstring>
#include <mutex>

namespace s2b {
namespace {

constexpr int BK = 64, NUM_THREADS = 192;
constexpr int ACC_COLS = 256, NUM_ACC = 2, TMEM_COLS = ACC_COLS * NUM_ACC;

// single-CTA kernel
constexpr int BM1 = 128, BN1 = 256, STAGES1 = 4;
constexpr int A1_BYTES = BM1 * BK * 2, B1_BYTES = BN1 * BK * 2, STAGE1_BYTES = A1_BYTES + B1_BYTES;
// gate/residual epilogue staging: per epilogue warp two 32x32 fp32 boxes
constexpr int RBOX_BYTES = 32 * 32 * 4, RES_BYTES = 4 * 2 * RBOX_BYTES;
constexpr int SMEM1_BYTES = STAGES1 * STAGE1_BYTES + RES_BYTES + 1024 + 512;
constexpr uint32_t IDESC1 = sm100::idesc_bf16_f32(BM1, BN1);
// kind::f16 A / B format fields (bits 7-9, 10-12): 1 = bf16, 0 = f16
constexpr uint32_t IDESC_AB_FMT = (7u << 7) | (7u << 10);
__host__ __device__ constexpr uint32_t idesc_for(uint32_t idesc_bf16, int op_f16) {
    return op_f16 ? (idesc_bf16 & ~IDESC_AB_FMT) : idesc_bf16;
}

// CTA-pair kernel: per CTA 128 rows of A and 128 rows of B per stage
// Tiles of BM2 x BN rows per pair (BN = 256, or 128 where 256-wide tiles
// would leave much of the last wave idle); each CTA stages 128 A rows and
// BN / 2 B rows per k-block.
constexpr int BM2 = 256;
// KIND_BF16: 16-bit operands (bf16 or f16, see op_t), 64-element k-blocks.  KIND_TF32X3: the fp32
// path's "3xTF32" split product -- A and B arrive as [hi | lo] halves of fp32
// (hi = x rounded to tf32, lo = x - hi), and every k-step issues
// hi*hi + hi*lo + lo*hi as tcgen05.mma kind::tf32 (fp32 accumulate), which
// keeps the products to about fp32 accuracy; k-blocks of 32 fp32 elements
// (one 128-byte swizzle row), each stage holding the four tiles.
constexpr int KIND_BF16 = 0, KIND_TF32X3 = 1;
constexpr uint32_t idesc_tf32_f32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
template <int BN, int KIND = KIND_BF16>
struct PairCfg {
    static constexpr int KB = KIND == KIND_BF16 ? BK : 32;                 // k elements per stage
    static constexpr int NPART = KIND == KIND_BF16 ? 1 : 2;                // operand parts (hi, lo)
    static constexpr int A_TILE = 128 * 128;                               // bytes of one 128-row, 128-B tile
    static constexpr int B_TILE = (BN / 2) * 128;
    static constexpr int A_BYTES = NPART * A_TILE;
    static constexpr int B_BYTES = NPART * B_TILE;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = KIND == KIND_TF32X3 ? 3 : (BN == 256 ? 6 : 8);
    static constexpr int SMEM = STAGES * STAGE_BYTES + RES_BYTES + 1024 + 512;
    static constexpr uint32_t IDESC = KIND == KIND_BF16 ? sm100::idesc_bf16_f32(BM2, BN) : idesc_tf32_f32(BM2, BN);
};

__device__ int g_tc_err;

struct TcParams {
    int M, N, num_m, num_n, num_kb;
    int kdim;            // K (the column offset of the lo half in the tf32x3 kind)
    int resid_tma;       // EPI_GATE_RESID through TMA-staged residual boxes
    GemmEpi e;
};

template <int STAGES>
struct Ctl {
    uint64_t full[STAGES], empty[STAGES], tfull[NUM_ACC], tempty[NUM_ACC];
    uint64_t rfull[4][2];      // residual boxes, per epilogue warp
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
__device__ __forceinline__ void store32(f16* dst, const float v[32]) {
    #pragma unroll
    for (int j = 0; j < 32; j += 8) {
        uint4 u;
        __half2 a = __floats2half2_rn(v[j], v[j + 1]), b = __floats2half2_rn(v[j + 2], v[j + 3]);
        __half2 c = __floats2half2_rn(v[j + 4], v[j + 5]), d = __floats2half2_rn(v[j + 6], v[j + 7]);
        u.x = *reinterpret_cast<uint32_t*>(&a); u.y = *reinterpret_cast<uint32_t*>(&b);
        u.z = *reinterpret_cast<uint32_t*>(&c); u.w = *reinterpret_cast<uint32_t*>(&d);
        *reinterpret_cast<uint4*>(dst + j) = u;
    }
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
// 32 values to a row of the 16-bit operand type t (bf16 or f16)
__device__ __forceinline__ void store32h(void* dst, ActT t, const float v[32]) {
    if (t == ACT_F16) store32((f16*)dst, v);
    else store32((bf16*)dst, v);
}

// Pull this thread's residual row segment of a tile into L2 ahead of its
// epilogue (8 x 128-B lines of fp32).
template <int MODE>
__device__ __forceinline__ void prefetch_resid(const TcParams& p, int row, int n0) {
    if (MODE != EPI_GATE_RESID || row >= p.M) return;
    const float* base = p.e.resid + (size_t)row * p.e.ldr + n0;
    #pragma unroll
    for (int j = 0; j < 8; j++)
        if (n0 + 32 * j < p.N) asm volatile("prefetch.global.L2 [%0];" ::"l"(base + 32 * j));
}

// RoPE in place on dims [d0, d0 + 64) of one normalised head: dims 0..125
// rotate in adjacent pairs (src/dit_vk.cpp:62-71), pair i with the angle of
// position pos[i / 21] and frequency i % 21 (cos/sin from the [pos][21]
// table); dims 126..127 pass through.
__device__ __forceinline__ void rope64(float* x, int d0, const float2* cs, int p0, int p1, int p2) {
    #pragma unroll
    for (int j = 0; j < 64; j += 2) {
        const int kd = d0 + j;
        if (kd < 126) {
            const int i = kd >> 1, ax = i / 21, f = i % 21;
            const int pos = ax == 0 ? p0 : (ax == 1 ? p1 : p2);
            const float2 t = cs[pos * 21 + f];          // shared or global (generic load)
            const float a = x[j], b = x[j + 1];
            x[j] = __fadd_rn(__fmul_rn(a, t.x), __fmul_rn(-b, t.y));
            x[j + 1] = __fadd_rn(__fmul_rn(b, t.x), __fmul_rn(a, t.y));
        }
    }
}

// 32 lanes x 32 consecutive fp32 columns back into TMEM (pair with wait::st).
__device__ __forceinline__ void tmem_st32f(uint32_t taddr, const float v[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        ::"r"(taddr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
          "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]),
          "f"(v[16]), "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]),
          "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
        : "memory");
}

// Row factor of an RMSNorm folded behind the GEMM (GemmEpi::sq_in): the
// partial sums of squares the producing epilogue wrote (fp32 over 128
// columns each), summed in a fixed order.  fp32 throughout: FP64 arithmetic
// here throttled the epilogue warps on the narrow FP64 pipe.
__device__ __forceinline__ float row_rs(const GemmEpi& e, int row, bool row_ok) {
    if (!e.sq_in || !row_ok) return 1.f;
    const float4* sq = reinterpret_cast<const float4*>(e.sq_in + (size_t)row * SQ_SLOTS);
    float4 q[SQ_SLOTS / 4];
    #pragma unroll
    for (int b = 0; b < SQ_SLOTS / 4; b++) q[b] = __ldg(sq + b);
    float t = 0.f;
    #pragma unroll
    for (int b = 0; b < SQ_SLOTS / 4; b++) t += (q[b].x + q[b].y) + (q[b].z + q[b].w);
    return 1.f / sqrtf(t / e.rs_dim + e.rs_eps);
}

// EPI_QKV_PACK: the tile's 256 columns are two heads of one of q / k / v.
// q and k heads get RMSNorm over their 128 dims (x / sqrt(mean(x^2)+eps) * w,
// the division as a reciprocal multiply: this epilogue serves the 16-bit paths)
// and RoPE, v heads pass through; each row lands in its window-packed slot(s)
// (a txt row in every window, with the same angles in each).
template <int BN>
__device__ __forceinline__ void epilogue_qkv_pack(const TcParams& p, uint32_t taddr, int row, int n0,
                                                  const float2* __restrict__ cs) {
    const PackEpi& k = p.e.pk;
    bool row_ok = row < p.M;
    const int gr = k.row_base + row;
    const bool vid = gr < k.Lv;
    const int sec = n0 / 2560;                     // 0 q, 1 k, 2 v
    const int h0 = (n0 % 2560) / 128;
    uint16_t* base = (uint16_t*)(sec == 0 ? k.Qp : sec == 1 ? k.Kp : k.Vp);   // 16-bit elements of k.qkv_t
    int gi = 0, wi = 0, ti = 0, p0 = 0, p1 = 0, p2 = 0;
    if (row_ok && vid) {
        const int4 tp = k.tokpos[gr];
        gi = tp.x; wi = tp.y; p0 = tp.z & 0xFFFF; p1 = tp.z >> 16; p2 = tp.w;
        if (gi < 0) row_ok = false;                // token outside every window: no packed slot
    }
    if (!vid) { ti = gr - k.Lv; p0 = p1 = p2 = ti; }
    const float* w = nullptr;
    if (sec < 2) w = vid ? (sec == 0 ? k.nq0 : k.nk0) : (sec == 0 ? k.nq1 : k.nk1);
    // folded RMSNorm (row factor) and adaLN shift (bias) of a fused operand
    const float rs = row_rs(p.e, row, row_ok);
    const float* cb = p.e.bias;
    // two passes over each head's 128 TMEM columns (sum of squares, then
    // normalise + rotate + store 64 dims at a time) keep 64 values live
    #pragma unroll 1
    for (int hh = 0; hh < BN / 128; hh++) {
        const uint32_t th = taddr + hh * 128;
        float inv = 1.f;
        if (sec < 2 || cb) {
            // pass 1, 32 columns at a time: a folded operand's values become
            // rs * acc + shift in TMEM (the shift loaded before the TMEM read,
            // so its latency is hidden), and q / k heads sum their squares
            float sq = 0.f;
            #pragma unroll 1
            for (int c = 0; c < 4; c++) {
                float4 c4[8];
                if (cb) {
                    const float4* cc = reinterpret_cast<const float4*>(cb + n0 + hh * 128 + c * 32);
                    #pragma unroll
                    for (int j = 0; j < 8; j++) c4[j] = __ldg(cc + j);
                }
                float x[32];
                sm100::tmem_ld32(th + c * 32, x);
                if (cb) {
                    #pragma unroll
                    for (int j = 0; j < 8; j++) {
                        x[4 * j] = fmaf(x[4 * j], rs, c4[j].x); x[4 * j + 1] = fmaf(x[4 * j + 1], rs, c4[j].y);
                        x[4 * j + 2] = fmaf(x[4 * j + 2], rs, c4[j].z); x[4 * j + 3] = fmaf(x[4 * j + 3], rs, c4[j].w);
                    }
                    tmem_st32f(th + c * 32, x);
                }
                if (sec < 2) {
                    #pragma unroll
                    for (int d = 0; d < 32; d++) sq = fmaf(x[d], x[d], sq);
                }
            }
            if (cb) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            if (sec < 2) inv = 1.f / sqrtf(__fadd_rn(sq * (1.f / 128.f), k.eps));
        }
        const int h = h0 + hh;
        // destination of this row: one packed slot (vid) or the first window's (txt)
        uint16_t* dst0 = nullptr;
        if (vid) dst0 = base + ((size_t)h * k.sumS + gi + (size_t)wi * k.TXT) * 128;
        else dst0 = base + ((size_t)h * k.sumS + k.cums[1] - k.TXT + ti) * 128;
        #pragma unroll 1
        for (int c = 0; c < 2; c++) {
            float x[64];
            sm100::tmem_ld64(th + c * 64, x);
            if (!row_ok) continue;
            if (sec < 2) {
                #pragma unroll
                for (int d = 0; d < 64; d += 4) {
                    const float4 w4 = __ldg(reinterpret_cast<const float4*>(w + c * 64 + d));
                    x[d] = x[d] * inv * w4.x; x[d + 1] = x[d + 1] * inv * w4.y;
                    x[d + 2] = x[d + 2] * inv * w4.z; x[d + 3] = x[d + 3] * inv * w4.w;
                }
                rope64(x, c * 64, cs, p0, p1, p2);
            }
            store32h(dst0 + c * 64, k.qkv_t, x);
            store32h(dst0 + c * 64 + 32, k.qkv_t, x + 32);
        }
        if (!row_ok || vid) continue;
        // txt row: the same rotated head in every window's slot
        #pragma unroll 1
        for (int wj = 1; wj < k.nwin; wj++) {
            uint16_t* dst = base + ((size_t)h * k.sumS + k.cums[wj + 1] - k.TXT + ti) * 128;
            #pragma unroll
            for (int c = 0; c < 16; c++)
                reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(dst0)[c];
        }
    }
}

// Epilogue of one accumulator row (thread = TMEM lane = output row) over the
// tile's 256 columns starting at n0.  The tcgen05.ld are warp-collective and
// executed by every lane; only the stores depend on the row.
template <int MODE, int BN = 256>
__device__ __forceinline__ void epilogue_row(const TcParams& p, uint32_t taddr, int row, int n0,
                                             const float2* cs = nullptr) {
    const GemmEpi& e = p.e;
    if constexpr (MODE == EPI_QKV_PACK) { epilogue_qkv_pack<BN>(p, taddr, row, n0, cs); return; }
    const bool row_ok = row < p.M;
    if constexpr (MODE == EPI_SWIGLU) {
        // column block [h 128 | g 128] -> 128 outputs at n0 / 2
        const float rs = row_rs(e, row, row_ok);
        const float* bias = e.bias;
        #pragma unroll 1
        for (int jc = 0; jc < 4; jc++) {
            // folded RMSNorm (row factor) and adaLN shift (bias) of a fused
            // operand; the shifts are loaded before the TMEM reads so their
            // latency is hidden
            float4 bh4[8], bg4[8];
            if (bias) {
                const float4* bh = reinterpret_cast<const float4*>(bias + n0 + jc * 32);
                const float4* bg = reinterpret_cast<const float4*>(bias + n0 + 128 + jc * 32);
                #pragma unroll
                for (int j = 0; j < 8; j++) { bh4[j] = __ldg(bh + j); bg4[j] = __ldg(bg + j); }
            }
            float h[32], g[32];
            sm100::tmem_ld32(taddr + jc * 32, h);
            sm100::tmem_ld32(taddr + 128 + jc * 32, g);
            if (!row_ok) continue;
            if (bias) {
                #pragma unroll
                for (int j = 0; j < 8; j++) {
                    h[4 * j] = fmaf(h[4 * j], rs, bh4[j].x); h[4 * j + 1] = fmaf(h[4 * j + 1], rs, bh4[j].y);
                    h[4 * j + 2] = fmaf(h[4 * j + 2], rs, bh4[j].z); h[4 * j + 3] = fmaf(h[4 * j + 3], rs, bh4[j].w);
                    g[4 * j] = fmaf(g[4 * j], rs, bg4[j].x); g[4 * j + 1] = fmaf(g[4 * j + 1], rs, bg4[j].y);
                    g[4 * j + 2] = fmaf(g[4 * j + 2], rs, bg4[j].z); g[4 * j + 3] = fmaf(g[4 * j + 3], rs, bg4[j].w);
                }
            }
            #pragma unroll
            for (int j = 0; j < 32; j++) h[j] = __fmul_rn(silu_f(g[j]), h[j]);
            const size_t off = (size_t)row * e.ldo + n0 / 2 + jc * 32;
            if (act_half(e.out_t)) store32h((uint16_t*)e.out + off, e.out_t, h);
            else store32((float*)e.out + off, h);
        }
        return;
    }
    const float* gate = (row < e.gate_split) ? e.gate0 : e.gate1;
    if constexpr (MODE == EPI_GATE_RESID) {
        // residual read-modify-write: the chunk's 8 residual loads are issued
        // together, before the TMEM load, so their latency overlaps it and the
        // loads never queue behind the previous chunk's stores.
        float* __restrict__ rrow = e.resid + (size_t)row * e.ldr;
        const float* msc = (row < e.mod_split) ? e.mod_sc0 : e.mod_sc1;
        float sq = 0.f;
        #pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
            if (n0 + c0 >= p.N) break;         // warp-uniform
            const int col = n0 + c0;
            const bool full = col + 32 <= p.N;
            float4 r[8];
            if (row_ok && full) {
                #pragma unroll
                for (int j = 0; j < 8; j++) r[j] = __ldcg(reinterpret_cast<const float4*>(rrow + col) + j);
            }
            float v[32];
            sm100::tmem_ld32(taddr + c0, v);
            if (!row_ok) continue;
            if (full) {
                #pragma unroll
                for (int j = 0; j < 8; j++) {
                    float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f), g4 = make_float4(1.f, 1.f, 1.f, 1.f);
                    if (e.bias) b4 = __ldg(reinterpret_cast<const float4*>(e.bias + col) + j);
                    if (gate) g4 = __ldg(reinterpret_cast<const float4*>(gate + col) + j);
                    float t0 = __fadd_rn(v[4 * j], b4.x), t1 = __fadd_rn(v[4 * j + 1], b4.y);
                    float t2 = __fadd_rn(v[4 * j + 2], b4.z), t3 = __fadd_rn(v[4 * j + 3], b4.w);
                    if (gate) { t0 = __fmul_rn(t0, g4.x); t1 = __fmul_rn(t1, g4.y); t2 = __fmul_rn(t2, g4.z); t3 = __fmul_rn(t3, g4.w); }
                    r[j].x = __fadd_rn(t0, r[j].x); r[j].y = __fadd_rn(t1, r[j].y);
                    r[j].z = __fadd_rn(t2, r[j].z); r[j].w = __fadd_rn(t3, r[j].w);
                }
                #pragma unroll
                for (int j = 0; j < 8; j++) __stcg(reinterpret_cast<float4*>(rrow + col) + j, r[j]);
                if (e.mod_out) {
                    float m[32];
                    #pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float4 s4 = msc ? __ldg(reinterpret_cast<const float4*>(msc + col) + j)
                                              : make_float4(1.f, 1.f, 1.f, 1.f);
                        sq = fmaf(r[j].x, r[j].x, sq); sq = fmaf(r[j].y, r[j].y, sq);
                        sq = fmaf(r[j].z, r[j].z, sq); sq = fmaf(r[j].w, r[j].w, sq);
                        m[4 * j] = r[j].x * s4.x; m[4 * j + 1] = r[j].y * s4.y;
                        m[4 * j + 2] = r[j].z * s4.z; m[4 * j + 3] = r[j].w * s4.w;
                    }
                    store32((bf16*)e.mod_out + (size_t)row * e.ldm + col, m);
                    if (((col + 32) & 127) == 0) { e.sq_out[(size_t)row * SQ_SLOTS + col / 128] = sq; sq = 0.f; }
                }
            } else {
                for (int j = 0; j < 32 && col + j < p.N; j++) {
                    float t = v[j];
                    if (e.bias) t = __fadd_rn(t, e.bias[col + j]);
                    if (gate) t = __fmul_rn(t, gate[col + j]);
                    rrow[col + j] = __fadd_rn(t, rrow[col + j]);
                }
            }
        }
        return;
    } else {
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
            {
                const size_t off = (size_t)row * e.ldo + col;
                if (full) {
                    if (act_half(e.out_t)) store32h((uint16_t*)e.out + off, e.out_t, v);
                    else store32((float*)e.out + off, v);
                } else {
                    for (int j = 0; j < 32 && col + j < p.N; j++) {
                        if (e.out_t == ACT_BF16) ((bf16*)e.out)[off + j] = __float2bfloat16_rn(v[j]);
                        else if (e.out_t == ACT_F16) ((f16*)e.out)[off + j] = __float2half_rn(v[j]);
                        else ((float*)e.out)[off + j] = v[j];
                    }
                }
            }
        }
    }
}

// EPI_GATE_RESID with the residual moved by TMA: for each 32-column chunk of
// the warp's 32 rows, the residual box (32 x 32 fp32, 128-B swizzle) is
// loaded one chunk ahead into one of two shared-memory buffers, each lane
// updates its row in place (resid += (acc + bias) * gate, the same rounding
// steps as epilogue_row), and one TMA store writes the box back.  Global
// traffic is whole 128-B lines instead of 16-B pieces of 32 rows per
// instruction.  Lane 0 issues every TMA operation of the warp.
struct ResidPipe {
    uint8_t* buf;        // this warp's two 4 KB boxes
    uint64_t* full;      // their barriers
    uint32_t k;          // chunks consumed so far (all lanes)
    uint32_t issued;     // box loads issued so far (lane 0)
};

// Lane 0: load the residual box of chunk `issued` into its buffer.
__device__ __forceinline__ void resid_load(const CUtensorMap* tR, ResidPipe& rp, int col, int row) {
    uint64_t* b = &rp.full[rp.issued & 1];
    sm100::mbar_arrive_expect_tx(b, RBOX_BYTES);
    sm100::tma_load_2d(rp.buf + (rp.issued & 1) * RBOX_BYTES, tR, b, col, row);
    rp.issued++;
}

// One tile's 32 rows x up to 256 columns.  next_n0 < 0: no tile follows.
// Returns false when a wait expired (the tile is abandoned).
__device__ __forceinline__ bool epilogue_resid_tma(const TcParams& p, const CUtensorMap* tR, uint32_t taddr, int r0,
                                                   int n0, const CUtensorMap* tR_next, int next_r0, int next_n0,
                                                   ResidPipe& rp, volatile int* abort_flag, int bn = 256) {
    const GemmEpi& e = p.e;
    const int lane = threadIdx.x & 31;
    const int row = r0 + lane;
    const float* gate = (row < e.gate_split) ? e.gate0 : e.gate1;
    const int nch = min(bn / 32, (p.N - n0) / 32);
    const bool mod = e.mod_out != nullptr && row < p.M;
    const float* msc = (row < e.mod_split) ? e.mod_sc0 : e.mod_sc1;
    float sq = 0.f;
    // the box ring runs one chunk ahead; pull the next tile's boxes into L2
    // now, a whole mainloop before they are loaded (groups share N)
    if (lane == 0 && next_n0 >= 0) {
        const int nn = min(bn / 32, (p.N - next_n0) / 32);
        for (int c = 0; c < nn; c++) sm100::tma_prefetch_l2_2d(tR_next, next_n0 + 32 * c, next_r0);
    }
    for (int c = 0; c < nch; c++) {
        const int col = n0 + 32 * c;
        // the next norm's scale, loaded ahead of the TMEM read and the box wait
        float4 s4[8];
        if (mod) {
            #pragma unroll
            for (int j = 0; j < 8; j++)
                s4[j] = msc ? __ldg(reinterpret_cast<const float4*>(msc + col) + j) : make_float4(1.f, 1.f, 1.f, 1.f);
        }
        float v[32];
        sm100::tmem_ld32(taddr + 32 * c, v);
        if (lane == 0) {
            // the other buffer was last stored from one chunk ago
            sm100::bulk_wait_read_all();
            if (c + 1 < nch) resid_load(tR, rp, col + 32, r0);
            else if (next_n0 >= 0) resid_load(tR_next, rp, next_n0, next_r0);
        }
        __syncwarp();
        if (!__all_sync(0xffffffffu, wait_or_abort(&rp.full[rp.k & 1], (rp.k >> 1) & 1, abort_flag))) return false;
        uint8_t* box = rp.buf + (rp.k & 1) * RBOX_BYTES + lane * 128;
        #pragma unroll
        for (int j = 0; j < 8; j++) {
            float4* q = reinterpret_cast<float4*>(box + ((j ^ (lane & 7)) << 4));
            float4 r = *q;
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f), g4 = make_float4(1.f, 1.f, 1.f, 1.f);
            if (e.bias) b4 = __ldg(reinterpret_cast<const float4*>(e.bias + col) + j);
            if (gate) g4 = __ldg(reinterpret_cast<const float4*>(gate + col) + j);
            float t0 = __fadd_rn(v[4 * j], b4.x), t1 = __fadd_rn(v[4 * j + 1], b4.y);
            float t2 = __fadd_rn(v[4 * j + 2], b4.z), t3 = __fadd_rn(v[4 * j + 3], b4.w);
            if (gate) { t0 = __fmul_rn(t0, g4.x); t1 = __fmul_rn(t1, g4.y); t2 = __fmul_rn(t2, g4.z); t3 = __fmul_rn(t3, g4.w); }
            r.x = __fadd_rn(t0, r.x); r.y = __fadd_rn(t1, r.y); r.z = __fadd_rn(t2, r.z); r.w = __fadd_rn(t3, r.w);
            *q = r;
            if (mod) {
                // the next RMSNorm's operand: resid * adaLN scale, and the row's sum of squares
                sq = fmaf(r.x, r.x, sq); sq = fmaf(r.y, r.y, sq); sq = fmaf(r.z, r.z, sq); sq = fmaf(r.w, r.w, sq);
                v[4 * j] = r.x * s4[j].x; v[4 * j + 1] = r.y * s4[j].y;
                v[4 * j + 2] = r.z * s4[j].z; v[4 * j + 3] = r.w * s4[j].w;
            }
        }
        if (mod) {
            store32((bf16*)e.mod_out + (size_t)row * e.ldm + col, v);
            if (((col + 32) & 127) == 0) { e.sq_out[(size_t)row * SQ_SLOTS + col / 128] = sq; sq = 0.f; }
        }
        sm100::fence_proxy_async_smem();      // generic-proxy writes -> the TMA store's reads
        __syncwarp();
        if (lane == 0) {
            sm100::tma_store_2d(tR, rp.buf + (rp.k & 1) * RBOX_BYTES, col, r0);
            sm100::bulk_commit_group();
        }
        rp.k++;
    }
    return true;
}

// Lane 0: let every issued box load land (bounded) and the warp's stores
// complete before the CTA's shared memory goes away.
__device__ __forceinline__ void resid_finish(ResidPipe& rp) {
    if ((threadIdx.x & 31) != 0) return;
    for (uint32_t kk = rp.k; kk < rp.issued; kk++)
        for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&rp.full[kk & 1], (kk >> 1) & 1); w++) {}
    sm100::bulk_wait_all();
}

// EPI_QKV_PACK: the epilogue warps (128 threads) copy the (cos, sin) table
// into the shared-memory area the residual boxes use in the gate/residual
// mode, when it fits; per-row table reads then gather from shared memory
// instead of issuing 32 distinct L1 lines per warp load.  Returns the table
// the epilogue reads.
__device__ __forceinline__ const float2* stage_rope_table(const PackEpi& k, uint8_t* sR) {
    const int n = k.npos * 21;
    if (n <= 0 || n * (int)sizeof(float2) > RES_BYTES) return k.cs;
    float2* t = reinterpret_cast<float2*>(sR);
    for (int i = (int)threadIdx.x - 64; i < n; i += 128) t[i] = __ldg(k.cs + i);
    asm volatile("bar.sync 1, 128;" ::: "memory");     // the 4 epilogue warps (threads 64..191)
    return t;
}

// ------------------------------------------------------------ single CTA
template <int MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB,
          const __grid_constant__ CUtensorMap tR, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES1 * A1_BYTES;
    uint8_t* sR = smem + STAGES1 * STAGE1_BYTES;            // residual boxes (1024-B aligned)
    Ctl<STAGES1>* ctl = reinterpret_cast<Ctl<STAGES1>*>(sR + RES_BYTES);
    volatile int* abort_flag = &ctl->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_tiles = p.num_m * p.num_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES1; s++) { sm100::mbar_init(&ctl->full[s], 1); sm100::mbar_init(&ctl->empty[s], 1); }
        for (int a = 0; a < NUM_ACC; a++) { sm100::mbar_init(&ctl->tfull[a], 1); sm100::mbar_init(&ctl->tempty[a], 4); }
        for (int w = 0; w < 4; w++) { sm100::mbar_init(&ctl->rfull[w][0], 1); sm100::mbar_init(&ctl->rfull[w][1], 1); }
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
                    sm100::mbar_arrive_expect_tx(&ctl->full[stage], STAGE1_BYTES);
                    sm100::tma_load_2d(sA + stage * A1_BYTES, &tA, &ctl->full[stage], kb * BK, mb * BM1);
                    sm100::tma_load_2d(sB + stage * B1_BYTES, &tB, &ctl->full[stage], kb * BK, nb * BN1);
                    issued++;
                    if (++stage == STAGES1) { stage = 0; phase ^= 1; }
                }
            }
            if (!ok) {
                const long n = issued < STAGES1 ? issued : STAGES1;
                for (long i = 1; i <= n; i++) {
                    const long k = issued - i;
                    const uint32_t s = (uint32_t)(k % STAGES1), ph = (uint32_t)((k / STAGES1) & 1);
                    for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->full[s], ph); w++) {}
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc1 = idesc_for(IDESC1, p.e.op_t == ACT_F16);
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
                    const uint8_t* a = sA + stage * A1_BYTES;
                    const uint8_t* b = sB + stage * B1_BYTES;
                    #pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++)
                        sm100::mma_bf16(d, sm100::desc_kmajor_sw128(a, kk * 32), sm100::desc_kmajor_sw128(b, kk * 32),
                                        idesc1, (kb | kk) != 0);
                    sm100::mma_commit(&ctl->empty[stage]);
                    if (++stage == STAGES1) { stage = 0; phase ^= 1; }
                }
                if (ok) sm100::mma_commit(&ctl->tfull[acc]);
            }
        }
    } else {
        const int q = warp & 3;                 // TMEM lane quadrant this warp may access
        ResidPipe rp{sR + q * 2 * RBOX_BYTES, ctl->rfull[q], 0u, 0u};
        const bool rt = MODE == EPI_GATE_RESID && p.resid_tma;
        const float2* cs = nullptr;
        if constexpr (MODE == EPI_QKV_PACK) cs = stage_rope_table(p.e.pk, sR);
        if (rt && lane == 0 && (int)blockIdx.x < num_tiles)
            resid_load(&tR, rp, ((int)blockIdx.x / p.num_m) * BN1, ((int)blockIdx.x % p.num_m) * BM1 + q * 32);
        int it = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, it++) {
            const int acc = it & 1;
            const uint32_t acc_phase = (it >> 1) & 1;
            // warp-uniform outcome: the tcgen05.ld below are warp-collective
            if (!__all_sync(0xffffffffu, wait_or_abort(&ctl->tfull[acc], acc_phase, abort_flag))) break;
            sm100::tc_fence_after();
            const int mb = tile % p.num_m, nb = tile / p.num_m;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * ACC_COLS;
            const int nt = tile + gridDim.x;
            if (rt) {
                const bool more = nt < num_tiles;
                if (!epilogue_resid_tma(p, &tR, taddr, mb * BM1 + q * 32, nb * BN1, &tR,
                                        more ? (nt % p.num_m) * BM1 + q * 32 : 0, more ? (nt / p.num_m) * BN1 : -1,
                                        rp, abort_flag))
                    break;
            } else {
                if (nt < num_tiles) prefetch_resid<MODE>(p, (nt % p.num_m) * BM1 + q * 32 + lane, (nt / p.num_m) * BN1);
                epilogue_row<MODE>(p, taddr, mb * BM1 + q * 32 + lane, nb * BN1, cs);
            }
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&ctl->tempty[acc]);
        }
        if (rt) resid_finish(rp);
    }
    __syncthreads();
    if (warp == 1) {
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ------------------------------------------------------------ CTA pair
// Tensor maps of up to two GEMM groups that share N, K and the epilogue mode
// (the vid and txt Linears of layers 0..9): A, B and the residual boxes.
struct PairMaps {
    CUtensorMap a[2], b[2], r[2];
};

// Tiles of group 0 come first, then group 1's; a tile's group picks its
// maps and epilogue parameters.
struct TileRef {
    int grp, mb, nb;
};
__device__ __forceinline__ TileRef tile_ref(const TcParams& p0, const TcParams& p1, int tiles0, int tile) {
    TileRef t;
    t.grp = tile >= tiles0;
    const int lt = t.grp ? tile - tiles0 : tile;
    const int nm = t.grp ? p1.num_m : p0.num_m;
    t.mb = lt % nm;
    t.nb = lt / nm;
    return t;
}

template <int MODE, int BN, int KIND = KIND_BF16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
k_gemm_tc_pair(const __grid_constant__ PairMaps maps, const __grid_constant__ TcParams p0,
               const __grid_constant__ TcParams p1, int ngroups) {
    using C = PairCfg<BN, KIND>;
    constexpr int STAGES2 = C::STAGES, A2_BYTES = C::A_BYTES, B2_BYTES = C::B_BYTES, STAGE2_BYTES = C::STAGE_BYTES;
    // bf16: two consecutive 64-deep k-blocks share one full / empty barrier
    // pair, so the MMA thread waits and commits once per 8 MMAs
    constexpr int GRP = KIND == KIND_BF16 ? 2 : 1, NBAR = STAGES2 / GRP;
    static_assert(STAGES2 % GRP == 0, "stage groups must tile the ring");
    constexpr int ACC = BN;                                 // TMEM columns per accumulator
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES2 * A2_BYTES;
    uint8_t* sR = smem + STAGES2 * STAGE2_BYTES;            // residual boxes (1024-B aligned)
    Ctl<STAGES2>* ctl = reinterpret_cast<Ctl<STAGES2>*>(sR + RES_BYTES);
    volatile int* abort_flag = &ctl->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = sm100::cluster_ctarank();        // 0: issues the MMAs
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int tiles0 = p0.num_m * p0.num_n;
    const int num_tiles = tiles0 + (ngroups > 1 ? p1.num_m * p1.num_n : 0);
    const int num_kb = p0.num_kb;                           // groups share K

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES2; s++) { sm100::mbar_init(&ctl->full[s], 1); sm100::mbar_init(&ctl->empty[s], 1); }
        for (int a = 0; a < NUM_ACC; a++) { sm100::mbar_init(&ctl->tfull[a], 1); sm100::mbar_init(&ctl->tempty[a], 8); }
        for (int w = 0; w < 4; w++) { sm100::mbar_init(&ctl->rfull[w][0], 1); sm100::mbar_init(&ctl->rfull[w][1], 1); }
        ctl->abort = 0;
        sm100::fence_barrier_init();
        for (int g = 0; g < ngroups; g++) {
            sm100::tma_prefetch_desc(&maps.a[g]);
            sm100::tma_prefetch_desc(&maps.b[g]);
        }
    }
    if (warp == 1) {
        sm100::tmem_alloc_pair(&ctl->tmem_slot, TMEM_COLS);
        sm100::tmem_relinquish_pair();
    }
    sm100::tc_fence_before();
    sm100::cluster_sync();                 // both CTAs' barriers initialised before any remote use
    sm100::tc_fence_after();
    const uint32_t tmem_base = ctl->tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t bs = 0, phase = 0;        // barrier stage (GRP consecutive k-blocks each)
            long issued = 0;                   // barrier stages filled
            bool ok = true;
            for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
                const TileRef t = tile_ref(p0, p1, tiles0, tile);
                const CUtensorMap* ta = &maps.a[t.grp];
                const CUtensorMap* tb = &maps.b[t.grp];
                for (int kb0 = 0; kb0 < num_kb; kb0 += GRP) {
                    const int nsub = min(GRP, num_kb - kb0);
                    if (!wait_or_abort(&ctl->empty[bs], phase ^ 1, abort_flag)) { ok = false; break; }
                    // both CTAs' bytes complete on the even CTA's full barrier
                    if (rank == 0) sm100::mbar_arrive_expect_tx(&ctl->full[bs], nsub * 2 * STAGE2_BYTES);
                    const uint32_t fb = sm100::map_to_rank(&ctl->full[bs], 0);
                    #pragma unroll
                    for (int sub = 0; sub < GRP; sub++) {
                        if (sub >= nsub) break;
                        const int slot = (int)bs * GRP + sub;
                        #pragma unroll
                        for (int part = 0; part < C::NPART; part++) {
                            // part 1 (lo) sits K elements to the right of part 0 (hi)
                            const int x = part * p0.kdim + (kb0 + sub) * C::KB;
                            sm100::tma_load_2d_pair(sA + slot * A2_BYTES + part * C::A_TILE, ta, fb, x,
                                                    t.mb * BM2 + (int)rank * 128);
                            sm100::tma_load_2d_pair(sB + slot * B2_BYTES + part * C::B_TILE, tb, fb, x,
                                                    t.nb * BN + (int)rank * (BN / 2));
                        }
                    }
                    issued++;
                    if (++bs == NBAR) { bs = 0; phase ^= 1; }
                }
            }
            if (!ok && rank == 0) {
                // drain this CTA pair's loads (bounded) before shared memory goes away
                const long n = issued < NBAR ? issued : NBAR;
                for (long i = 1; i <= n; i++) {
                    const long k = issued - i;
                    const uint32_t b = (uint32_t)(k % NBAR), ph = (uint32_t)((k / NBAR) & 1);
                    for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->full[b], ph); w++) {}
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            const uint32_t idesc16 = idesc_for(C::IDESC, p0.e.op_t == ACT_F16);   // groups share the operand type
            uint32_t bs = 0, phase = 0;
            int it = 0;
            bool ok = true;
            for (int tile = pair; tile < num_tiles && ok; tile += npairs, it++) {
                const int acc = it & 1;
                const uint32_t acc_phase = (it >> 1) & 1;
                if (!wait_or_abort(&ctl->tempty[acc], acc_phase ^ 1, abort_flag)) { ok = false; break; }
                sm100::tc_fence_after();
                const uint32_t d = tmem_base + acc * ACC;
                for (int kb0 = 0; kb0 < num_kb; kb0 += GRP) {
                    const int nsub = min(GRP, num_kb - kb0);
                    if (!wait_or_abort(&ctl->full[bs], phase, abort_flag)) { ok = false; break; }
                    sm100::tc_fence_after();
                    #pragma unroll
                    for (int sub = 0; sub < GRP; sub++) {
                        if (sub >= nsub) break;
                        const int kb = kb0 + sub;
                        const uint8_t* a = sA + ((int)bs * GRP + sub) * A2_BYTES;
                        const uint8_t* b = sB + ((int)bs * GRP + sub) * B2_BYTES;
                        if constexpr (KIND == KIND_BF16) {
                            #pragma unroll
                            for (int kk = 0; kk < BK / 16; kk++)
                                sm100::mma_bf16_pair(d, sm100::desc_kmajor_sw128(a, kk * 32),
                                                     sm100::desc_kmajor_sw128(b, kk * 32), idesc16, (kb | kk) != 0);
                        } else {
                            const uint8_t* al = a + C::A_TILE;
                            const uint8_t* bl = b + C::B_TILE;
                            #pragma unroll
                            for (int kk = 0; kk < C::KB / 8; kk++) {      // 8 tf32 = 32 bytes per k-step
                                const uint64_t ah = sm100::desc_kmajor_sw128(a, kk * 32);
                                const uint64_t bh = sm100::desc_kmajor_sw128(b, kk * 32);
                                sm100::mma_tf32_pair(d, ah, bh, C::IDESC, (kb | kk) != 0);
                                sm100::mma_tf32_pair(d, ah, sm100::desc_kmajor_sw128(bl, kk * 32), C::IDESC, 1);
                                sm100::mma_tf32_pair(d, sm100::desc_kmajor_sw128(al, kk * 32), bh, C::IDESC, 1);
                            }
                        }
                    }
                    // release these stages in both CTAs (one multicast commit)
                    sm100::mma_commit_pair_mc(&ctl->empty[bs], 0x3);
                    if (++bs == NBAR) { bs = 0; phase ^= 1; }
                }
                if (ok) {
                    sm100::mma_commit_pair_mc(&ctl->tfull[acc], 0x3);
                }
            }
        }
    } else {
        const int q = warp & 3;
        const int rbase = (int)rank * 128 + q * 32;           // this warp's rows within a 256-row tile
        ResidPipe rp{sR + q * 2 * RBOX_BYTES, ctl->rfull[q], 0u, 0u};
        // TMA residual boxes only when every group has them (checked on the host)
        const bool rt = MODE == EPI_GATE_RESID && p0.resid_tma;
        const float2* cs = nullptr;
        if constexpr (MODE == EPI_QKV_PACK) cs = stage_rope_table(p0.e.pk, sR);   // both groups share the geometry
        if (rt && lane == 0 && pair < num_tiles) {
            const TileRef t = tile_ref(p0, p1, tiles0, pair);
            resid_load(&maps.r[t.grp], rp, t.nb * BN, t.mb * BM2 + rbase);
            const int nn = min(BN / 32, (p0.N - t.nb * BN) / 32);
            for (int c = 1; c < nn; c++) sm100::tma_prefetch_l2_2d(&maps.r[t.grp], t.nb * BN + 32 * c, t.mb * BM2 + rbase);
        }
        int it = 0;
        for (int tile = pair; tile < num_tiles; tile += npairs, it++) {
            const int acc = it & 1;
            const uint32_t acc_phase = (it >> 1) & 1;
            if (!__all_sync(0xffffffffu, wait_or_abort(&ctl->tfull[acc], acc_phase, abort_flag))) break;
            sm100::tc_fence_after();
            const TileRef t = tile_ref(p0, p1, tiles0, tile);
            const TcParams& p = t.grp ? p1 : p0;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * ACC;
            const int nt = tile + npairs;
            const bool more = nt < num_tiles;
            const TileRef u = tile_ref(p0, p1, tiles0, more ? nt : tile);
            if (rt) {
                if (!epilogue_resid_tma(p, &maps.r[t.grp], taddr, t.mb * BM2 + rbase, t.nb * BN, &maps.r[u.grp],
                                        u.mb * BM2 + rbase, more ? u.nb * BN : -1, rp, abort_flag, BN))
                    break;
            } else {
                if (more) prefetch_resid<MODE>(u.grp ? p1 : p0, u.mb * BM2 + rbase + lane, u.nb * BN);
                epilogue_row<MODE, BN>(p, taddr, t.mb * BM2 + rbase + lane, t.nb * BN, cs);
            }
            sm100::tc_fence_before();
            __syncwarp();
            // the accumulator is free once both CTAs' epilogue warps are done with it
            if (lane == 0) sm100::mbar_arrive_cluster(sm100::map_to_rank(&ctl->tempty[acc], 0));
        }
        if (rt) resid_finish(rp);
    }
    sm100::tc_fence_before();
    sm100::cluster_sync();                 // no CTA leaves while its pair still signals it
    if (warp == 1) {
        sm100::tc_fence_after();
        sm100::tmem_dealloc_pair(tmem_base, TMEM_COLS);
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

// fp32 [rows][cols] (row stride ld elements), 32 x 32 boxes, 128-B swizzle:
// the residual boxes of the gate/residual epilogue.
static bool make_tmap_resid(CUtensorMap* m, const float* base, int rows, int cols, int ld) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    const cuuint32_t box[2] = {32, 32};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool gemm_tc_supported(int M, int N, int K, int lda, int ldw) {
    return M > 0 && N > 0 && K > 0 && N % 32 == 0 && lda % 8 == 0 && ldw % 8 == 0 && encode_fn() != nullptr;
}

static int num_sms() {
    int dev = 0;
    cudaGetDevice(&dev);
    return (dev < 64 && g_num_sms[dev] > 0) ? g_num_sms[dev] : 148;
}

static bool gemm_args_ok(const void* A, int lda, const void* W, int ldw, int M, int N, int K, const GemmEpi& e) {
    if (!gemm_tc_supported(M, N, K, lda, ldw)) return false;
    if (((uintptr_t)A & 15) || ((uintptr_t)W & 15)) return false;
    if (e.mode == EPI_SWIGLU && N % 256) return false;
    if (e.mode == EPI_QKV_PACK && N != 3 * 2560) return false;
    if (e.op_t != ACT_BF16 && e.op_t != ACT_F16) return false;
    if (e.mode == EPI_QKV_PACK && e.pk.qkv_t != ACT_BF16 && e.pk.qkv_t != ACT_F16) return false;
    return true;
}

// Parameters and tensor maps of one pair-kernel group (256-row A boxes).
static bool pair_group(const void* A, int lda, const void* W, int ldw, int M, int N, int K, const GemmEpi& e, int bn,
                       TcParams& p, CUtensorMap& ta, CUtensorMap& tb, CUtensorMap& tr) {
    p.M = M; p.N = N;
    p.num_kb = (K + BK - 1) / BK;
    p.kdim = K;
    p.e = e;
    // gate/residual epilogue through TMA boxes when the residual is 16-B aligned
    p.resid_tma = e.mode == EPI_GATE_RESID && e.resid && ((uintptr_t)e.resid & 15) == 0 && e.ldr % 4 == 0 &&
                  make_tmap_resid(&tr, e.resid, M, N, e.ldr);
    if (!p.resid_tma) std::memset(&tr, 0, sizeof tr);
    if (!make_tmap_bf16(&ta, A, M, K, lda, 128, BK) || !make_tmap_bf16(&tb, W, N, K, ldw, bn / 2, BK)) return false;
    p.num_m = (M + BM2 - 1) / BM2;
    p.num_n = (N + bn - 1) / bn;
    return true;
}

// Tile width of the pair kernel: 128 when 256-wide tiles would leave much of
// the GPU idle, never for SwiGLU (its tiles hold matching [h | g] halves).  A
// 128-wide tile takes about 2/3 of a 256-wide one's time (half the FLOPs, but
// TMA writes plus MMA reads of the A tile then exceed the shared-memory
// bandwidth), so it pays only when it removes whole waves.
static int pick_bn(int tiles_m, int N, EpiMode mode, int pairs) {
    if (mode == EPI_SWIGLU || N % 128) return 256;
    const long t256 = (long)tiles_m * ((N + 255) / 256), t128 = (long)tiles_m * ((N + 127) / 128);
    const double w256 = (double)((t256 + pairs - 1) / pairs), w128 = (double)((t128 + pairs - 1) / pairs);
    return (0.67 * w128 < 0.95 * w256) ? 128 : 256;
}

template <int BN>
static void launch_pair_bn(const PairMaps& maps, const TcParams& p0, const TcParams& p1, int ngroups, int pairs,
                           cudaStream_t s) {
    constexpr int SM = PairCfg<BN>::SMEM;
    switch (p0.e.mode) {
        case EPI_STORE: k_gemm_tc_pair<EPI_STORE, BN><<<2 * pairs, NUM_THREADS, SM, s>>>(maps, p0, p1, ngroups); break;
        case EPI_GATE_RESID: k_gemm_tc_pair<EPI_GATE_RESID, BN><<<2 * pairs, NUM_THREADS, SM, s>>>(maps, p0, p1, ngroups); break;
        case EPI_SWIGLU:
            if constexpr (BN == 256) k_gemm_tc_pair<EPI_SWIGLU, 256><<<2 * pairs, NUM_THREADS, SM, s>>>(maps, p0, p1, ngroups);
            break;
        case EPI_QKV_PACK: k_gemm_tc_pair<EPI_QKV_PACK, BN><<<2 * pairs, NUM_THREADS, SM, s>>>(maps, p0, p1, ngroups); break;
    }
}

static void launch_pair(const PairMaps& maps, const TcParams& p0, const TcParams& p1, int ngroups, int bn,
                        cudaStream_t s) {
    const int tiles = p0.num_m * p0.num_n + (ngroups > 1 ? p1.num_m * p1.num_n : 0);
    int pairs = num_sms() / 2;
    if (tiles < pairs) pairs = tiles;
    if (bn == 128) launch_pair_bn<128>(maps, p0, p1, ngroups, pairs, s);
    else launch_pair_bn<256>(maps, p0, p1, ngroups, pairs, s);
}

int gemm_tc(const void* A, int lda, const void* W, int ldw, int M, int N, int K, const GemmEpi& e, cudaStream_t s,
            int* launches) {
    if (!gemm_args_ok(A, lda, W, ldw, M, N, K, e)) return -1;
    if (M > 128) {
        // CTA pairs: 256 x 256 tiles, grid = one cluster of 2 per SM pair
        PairMaps maps;
        TcParams p;
        const int bn = pick_bn((M + BM2 - 1) / BM2, N, e.mode, num_sms() / 2);
        if (!pair_group(A, lda, W, ldw, M, N, K, e, bn, p, maps.a[0], maps.b[0], maps.r[0])) return -1;
        launch_pair(maps, p, p, 1, bn, s);
    } else {
        TcParams p;
        p.M = M; p.N = N;
        p.num_kb = (K + BK - 1) / BK;
        p.kdim = K;
        p.e = e;
        CUtensorMap ta, tb, tr;
        p.resid_tma = e.mode == EPI_GATE_RESID && e.resid && ((uintptr_t)e.resid & 15) == 0 && e.ldr % 4 == 0 &&
                      make_tmap_resid(&tr, e.resid, M, N, e.ldr);
        if (!p.resid_tma) std::memset(&tr, 0, sizeof tr);
        if (!make_tmap_bf16(&ta, A, M, K, lda, BM1, BK) || !make_tmap_bf16(&tb, W, N, K, ldw, BN1, BK)) return -1;
        p.num_m = (M + BM1 - 1) / BM1;
        p.num_n = (N + BN1 - 1) / BN1;
        const int tiles = p.num_m * p.num_n;
        const int sms = num_sms();
        const int grid = tiles < sms ? tiles : sms;
        switch (e.mode) {
            case EPI_STORE: k_gemm_tc<EPI_STORE><<<grid, NUM_THREADS, SMEM1_BYTES, s>>>(ta, tb, tr, p); break;
            case EPI_GATE_RESID: k_gemm_tc<EPI_GATE_RESID><<<grid, NUM_THREADS, SMEM1_BYTES, s>>>(ta, tb, tr, p); break;
            case EPI_SWIGLU: k_gemm_tc<EPI_SWIGLU><<<grid, NUM_THREADS, SMEM1_BYTES, s>>>(ta, tb, tr, p); break;
            case EPI_QKV_PACK: k_gemm_tc<EPI_QKV_PACK><<<grid, NUM_THREADS, SMEM1_BYTES, s>>>(ta, tb, tr, p); break;
        }
    }
    if (launches) (*launches)++;
    return 0;
}

// fp32 [rows][cols] (row stride ld elements) for the tf32x3 kind: boxes of
// box_rows x 32 elements (one 128-byte swizzle row), zero fill.
static bool make_tmap_f32(CUtensorMap* m, const void* base, int rows, int cols, int ld, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    const cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool gemm_tf32x3_supported(int M, int N, int K, int lda2, int ldw2) {
    return M > 0 && N > 0 && K > 0 && K % 32 == 0 && N % 32 == 0 && lda2 % 4 == 0 && ldw2 % 4 == 0 &&
           lda2 >= 2 * K && ldw2 >= 2 * K && encode_fn() != nullptr;
}

int gemm_tf32x3(const void* A2, int lda2, const void* W2, int ldw2, int M, int N, int K, const GemmEpi& e,
                cudaStream_t s, int* launches) {
    if (!gemm_tf32x3_supported(M, N, K, lda2, ldw2)) return -1;
    if (((uintptr_t)A2 & 15) || ((uintptr_t)W2 & 15)) return -1;
    if (e.mode == EPI_SWIGLU && N % 256) return -1;
    if (e.mode == EPI_QKV_PACK) return -1;            // the fused pack writes 16-bit operands
    using C = PairCfg<256, KIND_TF32X3>;
    PairMaps maps;
    TcParams p;
    p.M = M; p.N = N;
    p.num_kb = K / C::KB;
    p.kdim = K;
    p.e = e;
    p.resid_tma = e.mode == EPI_GATE_RESID && e.resid && ((uintptr_t)e.resid & 15) == 0 && e.ldr % 4 == 0 &&
                  make_tmap_resid(&maps.r[0], e.resid, M, N, e.ldr);
    if (!p.resid_tma) std::memset(&maps.r[0], 0, sizeof maps.r[0]);
    if (!make_tmap_f32(&maps.a[0], A2, M, 2 * K, lda2, 128) || !make_tmap_f32(&maps.b[0], W2, N, 2 * K, ldw2, 128))
        return -1;
    p.num_m = (M + BM2 - 1) / BM2;
    p.num_n = (N + 255) / 256;
    const int tiles = p.num_m * p.num_n;
    int pairs = num_sms() / 2;
    if (tiles < pairs) pairs = tiles;
    switch (e.mode) {
        case EPI_STORE: k_gemm_tc_pair<EPI_STORE, 256, KIND_TF32X3><<<2 * pairs, NUM_THREADS, C::SMEM, s>>>(maps, p, p, 1); break;
        case EPI_GATE_RESID: k_gemm_tc_pair<EPI_GATE_RESID, 256, KIND_TF32X3><<<2 * pairs, NUM_THREADS, C::SMEM, s>>>(maps, p, p, 1); break;
        case EPI_SWIGLU: k_gemm_tc_pair<EPI_SWIGLU, 256, KIND_TF32X3><<<2 * pairs, NUM_THREADS, C::SMEM, s>>>(maps, p, p, 1); break;
        default: return -1;
    }
    if (launches) (*launches)++;
    return 0;
}

int gemm_tc_grouped(const void* A0, int lda0, const void* W0, int ldw0, int M0, const GemmEpi& e0, const void* A1,
                    int lda1, const void* W1, int ldw1, int M1, const GemmEpi& e1, int N, int K, cudaStream_t s,
                    int* launches) {
    if (e0.mode != e1.mode || e0.op_t != e1.op_t || M0 <= 0 || M1 <= 0) return -1;
    if (!gemm_args_ok(A0, lda0, W0, ldw0, M0, N, K, e0) || !gemm_args_ok(A1, lda1, W1, ldw1, M1, N, K, e1)) return -1;
    PairMaps maps;
    TcParams p0, p1;
    const int bn = pick_bn((M0 + BM2 - 1) / BM2 + (M1 + BM2 - 1) / BM2, N, e0.mode, num_sms() / 2);
    if (!pair_group(A0, lda0, W0, ldw0, M0, N, K, e0, bn, p0, maps.a[0], maps.b[0], maps.r[0]) ||
        !pair_group(A1, lda1, W1, ldw1, M1, N, K, e1, bn, p1, maps.a[1], maps.b[1], maps.r[1]))
        return -1;
    if (p0.resid_tma != p1.resid_tma) return -1;    // one residual path for the whole launch
    launch_pair(maps, p0, p1, 2, bn, s);
    if (launches) (*launches)++;
    return 0;
}

int gemm_tc_flag_ptr(int** p) { return (int)cudaGetSymbolAddress((void**)p, g_tc_err); }

int awa_init_device();
int awa_tc_init_device();

int kernels_init_device() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64) cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    const void* single[4] = {(const void*)k_gemm_tc<EPI_STORE>, (const void*)k_gemm_tc<EPI_GATE_RESID>,
                             (const void*)k_gemm_tc<EPI_SWIGLU>, (const void*)k_gemm_tc<EPI_QKV_PACK>};
    const void* pairk[4] = {(const void*)k_gemm_tc_pair<EPI_STORE, 256>, (const void*)k_gemm_tc_pair<EPI_GATE_RESID, 256>,
                            (const void*)k_gemm_tc_pair<EPI_SWIGLU, 256>, (const void*)k_gemm_tc_pair<EPI_QKV_PACK, 256>};
    const void* pairn[3] = {(const void*)k_gemm_tc_pair<EPI_STORE, 128>, (const void*)k_gemm_tc_pair<EPI_GATE_RESID, 128>,
                            (const void*)k_gemm_tc_pair<EPI_QKV_PACK, 128>};
    const void* tf32k[3] = {(const void*)k_gemm_tc_pair<EPI_STORE, 256, KIND_TF32X3>,
                            (const void*)k_gemm_tc_pair<EPI_GATE_RESID, 256, KIND_TF32X3>,
                            (const void*)k_gemm_tc_pair<EPI_SWIGLU, 256, KIND_TF32X3>};
    for (const void* k : tf32k)
        if (cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg<256, KIND_TF32X3>::SMEM))
            return (int)e;
    for (int i = 0; i < 4; i++) {
        cudaError_t e = cudaFuncSetAttribute(single[i], cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM1_BYTES);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(pairk[i], cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg<256>::SMEM);
        if (e == cudaSuccess && i < 3) e = cudaFuncSetAttribute(pairn[i], cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg<128>::SMEM);
        if (e != cudaSuccess) return (int)e;
    }
    if (int rc = awa_tc_init_device()) return rc;
    return awa_init_device();
}

}  // namespace s2b
