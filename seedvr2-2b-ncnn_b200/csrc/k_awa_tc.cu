// k_awa_tc.cu -- AWA window attention on the 5th-gen tensor cores.
//
// All operands come from the window-packed, head-major Q/K/V slabs the QKV
// GEMM epilogue (or the pack kernel, k_awa.cu) writes, so every tile is a
// plain 2-D TMA box; vid outputs go back to their grid token, txt outputs to
// the per-window partials averaged later.  Keys past the window's end are
// masked (their shared-memory rows hold the neighbouring window's finite data
// or TMA zero fill).  Two kernels:
//   k_awa_attn_tc4   16-bit operands (bf16, or f16 for the fp16 precision; P
//                    in the same type): one CTA per (window, head, 128-query
//                    tile), two CTAs per SM, 64-key K/V tiles double-
//                    buffered; S in two TMEM slots, P written back into TMEM
//                    and used as the A operand of O += P V.
//   k_awa_attn_x3    fp32 path: the same tiles from three bf16 parts per
//                    fp32 value (six part products), one CTA per SM.
// Softmax: one query row per thread, ex2.approx, lazy O rescale (only when a
// row's max grows by more than 2^8, so P <= 2^8).  Every mbarrier wait is
// bounded (error flag g_attn_err on expiry); warp-collective TMEM
// instructions run under warp-uniform control.
#include "kernels.h"
#include "kcommon.cuh"
#include "sm100.cuh"
#include <cuda.h>
#include <cstdlib>

namespace s2b {

bool make_tmap_bf16(CUtensorMap* m, const void* base, int rows, int cols, int ld, int box_rows, int box_cols);
int awa_tc_poly_exp();

namespace {

constexpr int QT = 128, D = 128;
constexpr int TILE_BYTES = QT * D * 2;            // 32 KB: two 64-column swizzled halves
constexpr int HALF_BYTES = TILE_BYTES / 2;
constexpr int TMEM_COLS = 256;                     // 64-key kernel: S slots [0,128), O [128,256)
constexpr uint32_t IDESC_PV = sm100::idesc_bf16_f32(QT, D) | (1u << 16);   // B (V) MN-major
constexpr float T_RESCALE = 8.f;

__device__ int g_attn_err;

struct AttnParams {
    AwaDev g;
    float scale_log2;     // softmax scale * log2(e)
    void* att;            // vid rows: [Lv][ld_att] in att_t
    int ld_att;
    ActT att_t;           // ACT_F32, ACT_BF16 or ACT_F16
    float* toutw;         // txt rows: [nwin][TXT][2560] fp32
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    for (uint32_t i = 0; i < sm100::WAIT_LIMIT; i++) {
        if (sm100::mbar_try_wait(bar, parity)) return true;
        if ((i & 1023) == 1023 && *abort_flag) return false;
    }
    *abort_flag = 1;
    atomicExch(&g_attn_err, 1);
    return false;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float v[32]) {
    uint32_t r[32];
    #pragma unroll
    for (int i = 0; i < 32; i++) r[i] = __float_as_uint(v[i]);
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// 2^x with the hardware approximation (MUFU, flush-to-zero).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Two floats rounded to nearest-even bf16 and packed (a in the low half).
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}
// The same in IEEE binary16 (the fp16 operand mode's P).
__device__ __forceinline__ uint32_t pack_f16x2_rn(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}
// kind::f16 A / B format fields (bits 7-9, 10-12): 1 = bf16, 0 = f16
constexpr uint32_t idesc_f16(uint32_t idesc_bf16) { return idesc_bf16 & ~((7u << 7) | (7u << 10)); }

// Max of n (<= 64) leading values of v, -inf for the rest, through 8
// independent accumulators (a chain of 8 instead of 64 dependent fmaxf).
template <bool MASK>
__device__ __forceinline__ float max64_t(const float* v, int nvalid) {
    float a[8];
    #pragma unroll
    for (int i = 0; i < 8; i++) a[i] = -INFINITY;
    #pragma unroll
    for (int u = 0; u < 64; u++) a[u & 7] = fmaxf(a[u & 7], (!MASK || u < nvalid) ? v[u] : -INFINITY);
    return fmaxf(fmaxf(fmaxf(a[0], a[1]), fmaxf(a[2], a[3])), fmaxf(fmaxf(a[4], a[5]), fmaxf(a[6], a[7])));
}
__device__ __forceinline__ float sum8(const float* a) {
    return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}

// 32 lanes x 32 consecutive columns of packed values (tcgen05.st; pair with wait::st).
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t r[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// ---------------------------------------------------------------- 64-key kernel
// One CTA = one (window, head, 128-query tile), two CTAs per SM, keys in
// 64-key tiles through two-stage K and V rings.  TMEM per CTA (256 columns):
// S in two 64-column slots (S_{j+1} is computed while the softmax reads
// S_j), O in 128 columns.  The softmax writes P_j back into its S slot as
// packed bf16 pairs, and P_j is the TMEM A operand of O += P_j V_j.  Roles:
//   warps 0-3  softmax + epilogue (thread = query row)
//   warp 4     TMEM allocation; lane 0 issues the MMAs:
//                S_0; per j: S_{j+1} (once K_{j+1} is in and PV_{j-1} has
//                read the slot), then PV_j (once P_j is ready)
//   warp 5     lane 0 issues the TMA loads: Q, then K one tile ahead of V
//              (K_0, K_1, V_0, K_2, V_1, ...), since K_{j+1} gates S_{j+1}
//              while V_j is needed only after the softmax of step j
// The softmax rescales O only when a row's max grows by more than 2^8, and
// then waits for the PV in flight first.  A warp whose 32 rows all lie past
// the window's end (the tail query tile) keeps the barrier protocol but does
// no arithmetic: its O rows are never stored.  The epilogue stages each
// warp's 32 normalised O rows in shared memory (the spent Q/K/V tiles) and
// writes them back one row per warp instruction (256 B bf16 / 512 B fp32),
// instead of 32 rows per instruction.
constexpr int KT4 = 64;
constexpr int KV4_BYTES = KT4 * D * 2;             // 16 KB: two 64-column halves of 8 KB
constexpr int KV4_HALF = KV4_BYTES / 2;
constexpr int T4_THREADS = 192;
constexpr int T4_SMEM = TILE_BYTES + 4 * KV4_BYTES + 1024 + 256;
constexpr uint32_t IDESC_QK4 = sm100::idesc_bf16_f32(QT, KT4);
constexpr int STG_LD = D + 4;                      // staging row stride in floats (528 B: 4-way, not 32-way, banks)
static_assert(4 * 32 * STG_LD * 4 <= TILE_BYTES + 4 * KV4_BYTES, "epilogue staging must fit in the Q/K/V tiles");

struct Attn4Ctl {
    uint64_t q_full, k_full[2], k_empty[2], v_full[2], v_empty[2];
    uint64_t s_full[2], p_ready[2], pv_done, o_full, drain;
    uint32_t tmem_slot;
    int abort;
};

// MN-major V tile of 64 keys: two 64-dim halves KV4_HALF apart, 8-key groups 1 KB apart.
__device__ __forceinline__ uint64_t desc_v64(const void* tile, uint32_t k_group_bytes) {
    const uint32_t addr = sm100::smem_u32(tile) + k_group_bytes;
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)(KV4_HALF >> 4) << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Packed fp32 pairs (Blackwell f32x2 arithmetic: one instruction per pair).
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2unpack(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// 2^x for a pair on the FMA pipe (f32x2 arithmetic), for softmax exponents
// x <= ~8: clamp at -125 so the exponent field stays normal; Cody-Waite split
// x = j + f with j = round(x) (adding 1.5 * 2^23 rounds to an integer in the
// low mantissa bits) and |f| <= 1/2; 2^f by a cubic fitted in this repository
// by relative least squares on Chebyshev nodes of [-1/2, 1/2] (max relative
// error 7.7e-5, below bf16's 2^-9 rounding of P); then j added to the
// exponent field (the rounded sum's low bits are j, and its remaining bits
// vanish in the shift by 23).
__device__ __forceinline__ void ex2_poly2(uint64_t x2, float& ra, float& rb) {
    float xa, xb;
    f2unpack(x2, xa, xb);
    const uint64_t xc = f2pack(fmaxf(xa, -125.f), fmaxf(xb, -125.f));
    const uint64_t magic = f2pack(12582912.f, 12582912.f);
    const uint64_t t = fadd2(xc, magic);
    const uint64_t fr = fsub2(xc, fsub2(t, magic));
    uint64_t p = ffma2(fr, f2pack(0.05508868396282196f, 0.05508868396282196f),
                       f2pack(0.24260404706001282f, 0.24260404706001282f));
    p = ffma2(fr, p, f2pack(0.6932762265205383f, 0.6932762265205383f));
    p = ffma2(fr, p, f2pack(0.9999289512634277f, 0.9999289512634277f));
    float pa, pb, ta, tb;
    f2unpack(p, pa, pb);
    f2unpack(t, ta, tb);
    ra = __int_as_float(__float_as_int(pa) + (__float_as_int(ta) << 23));
    rb = __int_as_float(__float_as_int(pb) + (__float_as_int(tb) << 23));
}

// Max of the 64 values (three-input max, 8 independent chains).
__device__ __forceinline__ float max64_full(const float* v) {
    float a[8];
    #pragma unroll
    for (int i = 0; i < 8; i++) a[i] = fmaxf(v[2 * i], v[2 * i + 1]);
    #pragma unroll
    for (int u = 16; u < 64; u += 2) a[(u >> 1) & 7] = fmax3(a[(u >> 1) & 7], v[u], v[u + 1]);
    return fmax3(fmax3(a[0], a[1], a[2]), fmax3(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
}

// NP of every 4 exponential pairs on the FMA pipe (ex2_poly2), the rest on MUFU.
template <int NP, bool F16>
__global__ void __launch_bounds__(T4_THREADS, 2)
k_awa_attn_tc4(const __grid_constant__ CUtensorMap tQ, const __grid_constant__ CUtensorMap tK,
               const __grid_constant__ CUtensorMap tV, const AttnParams p) {
    const int wi = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * QT;
    const int f = p.g.cumf[wi + 1] - p.g.cumf[wi];
    const int S = f + p.g.TXT;
    if (q0 >= S) return;                       // uniform across the CTA, before any barrier
    const int nkt = (S + KT4 - 1) / KT4;
    const int row_base = h * p.g.sumS + p.g.cums[wi];

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = smem + TILE_BYTES;                 // [2] stages
    uint8_t* sV = smem + TILE_BYTES + 2 * KV4_BYTES; // [2] stages
    Attn4Ctl* ctl = reinterpret_cast<Attn4Ctl*>(smem + TILE_BYTES + 4 * KV4_BYTES);
    volatile int* abort_flag = &ctl->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // the producer initialises the barriers and starts the Q / K_0 loads
    // before the CTA-wide barrier, so their latency overlaps the TMEM
    // allocation; the softmax threads fetch their rows' grid tokens now,
    // long before the epilogue needs them
    const int tid_prod = 5 * 32;
    if (threadIdx.x == tid_prod) {
        sm100::tma_prefetch_desc(&tQ);
        sm100::tma_prefetch_desc(&tK);
        sm100::tma_prefetch_desc(&tV);
        sm100::mbar_init(&ctl->q_full, 1);
        for (int i = 0; i < 2; i++) {
            sm100::mbar_init(&ctl->k_full[i], 1);
            sm100::mbar_init(&ctl->k_empty[i], 1);
            sm100::mbar_init(&ctl->v_full[i], 1);
            sm100::mbar_init(&ctl->v_empty[i], 1);
            sm100::mbar_init(&ctl->s_full[i], 1);
            sm100::mbar_init(&ctl->p_ready[i], 4);
        }
        sm100::mbar_init(&ctl->pv_done, 1);
        sm100::mbar_init(&ctl->o_full, 1);
        sm100::mbar_init(&ctl->drain, 1);
        ctl->abort = 0;
        sm100::fence_barrier_init();
        sm100::mbar_arrive_expect_tx(&ctl->q_full, TILE_BYTES);
        sm100::tma_load_2d(sQ, &tQ, &ctl->q_full, 0, row_base + q0);
        sm100::tma_load_2d(sQ + HALF_BYTES, &tQ, &ctl->q_full, 64, row_base + q0);
        sm100::mbar_arrive_expect_tx(&ctl->k_full[0], KV4_BYTES);
        sm100::tma_load_2d(sK, &tK, &ctl->k_full[0], 0, row_base);
        sm100::tma_load_2d(sK + KV4_HALF, &tK, &ctl->k_full[0], 64, row_base);
        // the two-stage rings run only one tile ahead: bring every later K/V
        // tile of this (window, head) into L2 now, so each ring load is an
        // L2 hit rather than a DRAM round trip
        for (int j = 1; j < nkt; j++) {
            sm100::tma_prefetch_l2_2d(&tK, 0, row_base + j * KT4);
            sm100::tma_prefetch_l2_2d(&tK, 64, row_base + j * KT4);
        }
        for (int j = 0; j < nkt; j++) {
            sm100::tma_prefetch_l2_2d(&tV, 0, row_base + j * KT4);
            sm100::tma_prefetch_l2_2d(&tV, 64, row_base + j * KT4);
        }
    }
    const int my_q = q0 + (threadIdx.x & 127);
    const int my_tok = (warp < 4 && my_q < f) ? p.g.vidx[p.g.cumf[wi] + my_q] : 0;
    if (warp == 4) {
        sm100::tmem_alloc(&ctl->tmem_slot, TMEM_COLS);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = ctl->tmem_slot;
    const uint32_t tO = tmem + 128;            // S slots at [0, 64) and [64, 128)

    if (warp == 5) {
        if (lane == 0) {
            // ---- TMA producer
            bool ok = true;
            int kq = 1, vq = 0;                // K / V tiles issued (Q and K_0 above)
            // stage j & 1 held tile j - 2: its S (K) or PV (V) must be done
            auto load_k = [&](int j) -> bool {
                const int st = j & 1, r = row_base + j * KT4;
                if (j >= 2 && !wait_bar(&ctl->k_empty[st], (uint32_t)((j >> 1) - 1) & 1, abort_flag)) return false;
                sm100::mbar_arrive_expect_tx(&ctl->k_full[st], KV4_BYTES);
                sm100::tma_load_2d(sK + st * KV4_BYTES, &tK, &ctl->k_full[st], 0, r);
                sm100::tma_load_2d(sK + st * KV4_BYTES + KV4_HALF, &tK, &ctl->k_full[st], 64, r);
                kq++;
                return true;
            };
            auto load_v = [&](int j) -> bool {
                const int st = j & 1, r = row_base + j * KT4;
                if (j >= 2 && !wait_bar(&ctl->v_empty[st], (uint32_t)((j >> 1) - 1) & 1, abort_flag)) return false;
                sm100::mbar_arrive_expect_tx(&ctl->v_full[st], KV4_BYTES);
                sm100::tma_load_2d(sV + st * KV4_BYTES, &tV, &ctl->v_full[st], 0, r);
                sm100::tma_load_2d(sV + st * KV4_BYTES + KV4_HALF, &tV, &ctl->v_full[st], 64, r);
                vq++;
                return true;
            };
            for (int j = 0; j < nkt && ok; j++) {
                if (j + 1 < nkt && !(ok = load_k(j + 1))) break;
                ok = load_v(j);
            }
            if (!ok) {
                // drain this thread's own TMA loads (bounded) before shared memory is released
                for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->q_full, 0); w++) {}
                for (int k = (kq > 2 ? kq - 2 : 0); k < kq; k++)
                    for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->k_full[k & 1], (uint32_t)(k >> 1) & 1); w++) {}
                for (int k = (vq > 2 ? vq - 2 : 0); k < vq; k++)
                    for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->v_full[k & 1], (uint32_t)(k >> 1) & 1); w++) {}
            }
        }
    } else if (warp == 4) {
        if (lane == 0) {
            // ---- MMA issuer
            auto issue_s = [&](int j) {
                const uint8_t* k = sK + (j & 1) * KV4_BYTES;
                #pragma unroll
                for (int kk = 0; kk < D / 16; kk++) {
                    const uint32_t aoff = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
                    const uint32_t boff = (kk >> 2) * KV4_HALF + (kk & 3) * 32;
                    sm100::mma_bf16(tmem + (j & 1) * 64, sm100::desc_kmajor_sw128(sQ, aoff),
                                    sm100::desc_kmajor_sw128(k, boff), F16 ? idesc_f16(IDESC_QK4) : IDESC_QK4,
                                    kk != 0);
                }
                sm100::mma_commit(&ctl->s_full[j & 1]);
                sm100::mma_commit(&ctl->k_empty[j & 1]);
            };
            bool ok = wait_bar(&ctl->q_full, 0, abort_flag);
            if (ok && (ok = wait_bar(&ctl->k_full[0], 0, abort_flag))) {
                sm100::tc_fence_after();
                issue_s(0);
            }
            for (int j = 0; j < nkt && ok; j++) {
                const int st = j & 1;
                if (j + 1 < nkt) {
                    if (!(ok = wait_bar(&ctl->k_full[st ^ 1], (uint32_t)((j + 1) >> 1) & 1, abort_flag))) break;
                    // slot (j+1)&1 held P_{j-1}: its PV must be done
                    if (j >= 1 && !(ok = wait_bar(&ctl->pv_done, (uint32_t)(j - 1) & 1, abort_flag))) break;
                    sm100::tc_fence_after();
                    issue_s(j + 1);
                }
                if (!(ok = wait_bar(&ctl->p_ready[st], (uint32_t)(j >> 1) & 1, abort_flag))) break;
                if (!(ok = wait_bar(&ctl->v_full[st], (uint32_t)(j >> 1) & 1, abort_flag))) break;
                sm100::tc_fence_after();
                const uint8_t* v = sV + st * KV4_BYTES;
                #pragma unroll
                for (int kk = 0; kk < KT4 / 16; kk++)
                    sm100::mma_bf16_tmem_a(tO, tmem + st * 64 + kk * 8, desc_v64(v, kk * 2048),
                                           F16 ? idesc_f16(IDESC_PV) : IDESC_PV, (j | kk) != 0);
                sm100::mma_commit(&ctl->pv_done);
                sm100::mma_commit(&ctl->v_empty[st]);
                if (j + 1 == nkt) sm100::mma_commit(&ctl->o_full);
            }
            // all of this thread's MMAs done before TMEM / shared memory go away
            sm100::mma_commit(&ctl->drain);
            for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->drain, 0); w++) {}
        }
    } else {
        // ---- softmax + epilogue: thread = query row q0 + r; TMEM lane quadrant = warp
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const float sl = p.scale_log2;
        const bool live = q0 + warp * 32 < S;  // warp-uniform: any of this warp's rows is a query
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        // tcgen05.ld / st are warp-collective: control flow stays warp-uniform
        for (int j = 0; j < nkt; j++) {
            const int st = j & 1;
            ok = __all_sync(0xffffffffu, wait_bar(&ctl->s_full[st], (uint32_t)(j >> 1) & 1, abort_flag));
            if (!ok) break;
            if (live) {
                sm100::tc_fence_after();
                const int kvalid = S - j * KT4;
                const bool full = kvalid >= KT4;           // CTA-uniform
                float v[64];
                sm100::tmem_ld64(tmem + lane_off + st * 64, v);
                const float mx = (full ? max64_full(v) : max64_t<true>(v, kvalid)) * sl;
                if (j == 0) {
                    m = mx;
                } else {
                    const bool grow = mx > m + T_RESCALE;
                    if (__any_sync(0xffffffffu, grow)) {
                        // the previous PV accumulates into O: wait for it first
                        ok = __all_sync(0xffffffffu, wait_bar(&ctl->pv_done, (uint32_t)(j - 1) & 1, abort_flag));
                        if (!ok) break;
                        sm100::tc_fence_after();
                        const float mn = grow ? mx : m;
                        const float corr = exp2f(m - mn);
                        #pragma unroll 1
                        for (int c = 0; c < 4; c++) {
                            float o[32];
                            sm100::tmem_ld32(tO + lane_off + c * 32, o);
                            #pragma unroll
                            for (int u = 0; u < 32; u++) o[u] *= corr;
                            tmem_st32(tO + lane_off + c * 32, o);
                        }
                        l *= corr;
                        m = mn;
                    }
                }
                // P_j as packed 16-bit pairs (the operand type) over the slot's columns [0, 32)
                const uint64_t sl2 = f2pack(sl, sl), nm2 = f2pack(-m, -m);
                uint32_t pk[32];
                uint64_t ls[4];
                #pragma unroll
                for (int i = 0; i < 4; i++) ls[i] = f2pack(0.f, 0.f);
                #pragma unroll
                for (int u = 0; u < 32; u++) {
                    const uint64_t x2 = ffma2(f2pack(v[2 * u], v[2 * u + 1]), sl2, nm2);
                    float a, b;
                    if ((u & 3) < NP) {
                        ex2_poly2(x2, a, b);
                    } else {
                        float xa, xb;
                        f2unpack(x2, xa, xb);
                        a = ex2_approx(xa);
                        b = ex2_approx(xb);
                    }
                    if (!full) { a = (2 * u < kvalid) ? a : 0.f; b = (2 * u + 1 < kvalid) ? b : 0.f; }
                    ls[u & 3] = fadd2(ls[u & 3], f2pack(a, b));
                    pk[u] = F16 ? pack_f16x2_rn(a, b) : pack_bf16x2_rn(a, b);
                }
                float s8[8];
                #pragma unroll
                for (int i = 0; i < 4; i++) f2unpack(ls[i], s8[2 * i], s8[2 * i + 1]);
                l += sum8(s8);
                tmem_st32u(tmem + lane_off + st * 64, pk);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            }
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&ctl->p_ready[st]);
        }
        // O is final once every PV is done (a barrier of its own: pv_done may
        // still be two phases behind here, which its parity cannot tell apart)
        if (ok) ok = __all_sync(0xffffffffu, wait_bar(&ctl->o_full, 0, abort_flag));
        if (ok && live) {
            sm100::tc_fence_after();
            // every MMA and TMA load of the CTA is complete: the Q/K/V tiles
            // are free to stage this warp's 32 rows
            const float inv = 1.f / l;
            float* stage = reinterpret_cast<float*>(smem) + (size_t)warp * 32 * STG_LD;
            float* mine = stage + lane * STG_LD;
            #pragma unroll 1
            for (int c = 0; c < 2; c++) {
                float o[64];
                sm100::tmem_ld64(tO + lane_off + c * 64, o);
                #pragma unroll
                for (int u = 0; u < 64; u += 4)
                    *reinterpret_cast<float4*>(mine + c * 64 + u) =
                        make_float4(o[u] * inv, o[u + 1] * inv, o[u + 2] * inv, o[u + 3] * inv);
            }
            const int qw = q0 + warp * 32;
            const int nrows = min(32, S - qw);
            __syncwarp();
            #pragma unroll 4
            for (int rr = 0; rr < nrows; rr++) {
                const int q = qw + rr;
                const int tok = __shfl_sync(0xffffffffu, my_tok, rr);
                const float4 x = *reinterpret_cast<const float4*>(stage + rr * STG_LD + lane * 4);
                const float xv[4] = {x.x, x.y, x.z, x.w};
                if (q < f) {
                    if (p.att_t == ACT_BF16)
                        store4((bf16*)p.att + (size_t)tok * p.ld_att + h * D + lane * 4, xv);
                    else if (p.att_t == ACT_F16)
                        store4((f16*)p.att + (size_t)tok * p.ld_att + h * D + lane * 4, xv);
                    else
                        store4((float*)p.att + (size_t)tok * p.ld_att + h * D + lane * 4, xv);
                } else {
                    store4(p.toutw + ((size_t)wi * p.g.TXT + (q - f)) * 2560 + h * D + lane * 4, xv);
                }
            }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ---------------------------------------------------------------- fp32 attention on the tensor cores
// The fp32 path's attention from split3 operands (awa_pack_split3): every
// fp32 value of Q, K, V and P is hi + mid + lo in bf16, and QK^T and PV are
// the six part products of order <= 2 -- (1,1), (2,0), (0,2), (1,0), (0,1),
// (0,0) with 0 = hi, 1 = mid, 2 = lo, smallest first -- accumulated in fp32
// in TMEM; the dropped terms are below 2^-24 of the product.  Structure of
// k_awa_attn_tc4, one CTA per SM (192 KB of part tiles, all 512 TMEM
// columns): Q parts 3 x 32 KB, one K and one V tile (3 x 16 KB each, 64
// keys), S in one 64-column slot, P as three 32-column parts of packed bf16
// pairs, O in 128 columns.  The S slot is released (s_free) as soon as the
// softmax has S_j in registers, so S_{j+1} runs on the tensor pipe during
// the softmax of step j; the softmax waits for PV_{j-1} only before it
// overwrites the P parts.  The loads run one tile ahead: K_{j+1} once S_j is
// done, V_{j+1} once PV_j is done.
constexpr int X3_TILES = 3 * TILE_BYTES + 6 * KV4_BYTES;   // 192 KB
constexpr int X3_SMEM = X3_TILES + 1024 + 256;
constexpr int X3_TMEM = 512;
constexpr int X3_NTERM = 6;
__device__ __constant__ int8_t c_x3_terms[X3_NTERM][2] = {{1, 1}, {2, 0}, {0, 2}, {1, 0}, {0, 1}, {0, 0}};

struct AttnX3Ctl {
    uint64_t q_full, k_full, k_empty, v_full, v_empty;
    uint64_t s_full, s_free, p_ready, pv_done, o_full, drain;
    uint32_t tmem_slot;
    int abort;
};

// fp32 P as three bf16 parts of a pair (a in the low halves).
__device__ __forceinline__ void split3_pair(float a, float b, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const float ra = __fsub_rn(a, hf.x), rb = __fsub_rn(b, hf.y);
    const __nv_bfloat162 m = __floats2bfloat162_rn(ra, rb);
    const float2 mf = __bfloat1622float2(m);
    const __nv_bfloat162 l = __floats2bfloat162_rn(__fsub_rn(ra, mf.x), __fsub_rn(rb, mf.y));
    hi = *reinterpret_cast<const uint32_t*>(&h);
    mid = *reinterpret_cast<const uint32_t*>(&m);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

__global__ void __launch_bounds__(T4_THREADS, 1)
k_awa_attn_x3(const __grid_constant__ CUtensorMap tQ, const __grid_constant__ CUtensorMap tK,
              const __grid_constant__ CUtensorMap tV, const AttnParams p) {
    const int wi = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * QT;
    const int f = p.g.cumf[wi + 1] - p.g.cumf[wi];
    const int S = f + p.g.TXT;
    if (q0 >= S) return;                       // uniform across the CTA, before any barrier
    const int nkt = (S + KT4 - 1) / KT4;
    const int row_base = h * p.g.sumS + p.g.cums[wi];
    const int part_rows = 20 * p.g.sumS;       // rows between the parts of one operand

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                              // 3 parts x 32 KB
    uint8_t* sK = smem + 3 * TILE_BYTES;             // 3 parts x 16 KB
    uint8_t* sV = sK + 3 * KV4_BYTES;                // 3 parts x 16 KB
    AttnX3Ctl* ctl = reinterpret_cast<AttnX3Ctl*>(smem + X3_TILES);
    volatile int* abort_flag = &ctl->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    auto load_kv = [&](const CUtensorMap* tm, uint8_t* dst, uint64_t* bar, int j) {
        sm100::mbar_arrive_expect_tx(bar, 3 * KV4_BYTES);
        #pragma unroll
        for (int a = 0; a < 3; a++) {
            const int r = a * part_rows + row_base + j * KT4;
            sm100::tma_load_2d(dst + a * KV4_BYTES, tm, bar, 0, r);
            sm100::tma_load_2d(dst + a * KV4_BYTES + KV4_HALF, tm, bar, 64, r);
        }
    };
    if (threadIdx.x == 5 * 32) {
        sm100::tma_prefetch_desc(&tQ);
        sm100::tma_prefetch_desc(&tK);
        sm100::tma_prefetch_desc(&tV);
        sm100::mbar_init(&ctl->q_full, 1);
        sm100::mbar_init(&ctl->k_full, 1);
        sm100::mbar_init(&ctl->k_empty, 1);
        sm100::mbar_init(&ctl->v_full, 1);
        sm100::mbar_init(&ctl->v_empty, 1);
        sm100::mbar_init(&ctl->s_full, 1);
        sm100::mbar_init(&ctl->s_free, 4);
        sm100::mbar_init(&ctl->p_ready, 4);
        sm100::mbar_init(&ctl->pv_done, 1);
        sm100::mbar_init(&ctl->o_full, 1);
        sm100::mbar_init(&ctl->drain, 1);
        ctl->abort = 0;
        sm100::fence_barrier_init();
        sm100::mbar_arrive_expect_tx(&ctl->q_full, 3 * TILE_BYTES);
        #pragma unroll
        for (int a = 0; a < 3; a++) {
            const int r = a * part_rows + row_base + q0;
            sm100::tma_load_2d(sQ + a * TILE_BYTES, &tQ, &ctl->q_full, 0, r);
            sm100::tma_load_2d(sQ + a * TILE_BYTES + HALF_BYTES, &tQ, &ctl->q_full, 64, r);
        }
        load_kv(&tK, sK, &ctl->k_full, 0);
        load_kv(&tV, sV, &ctl->v_full, 0);
    }
    const int my_q = q0 + (threadIdx.x & 127);
    const int my_tok = (warp < 4 && my_q < f) ? p.g.vidx[p.g.cumf[wi] + my_q] : 0;
    if (warp == 4) {
        sm100::tmem_alloc(&ctl->tmem_slot, X3_TMEM);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = ctl->tmem_slot;
    const uint32_t tS = tmem, tP = tmem + 64, tO = tmem + 256;   // P parts at tP + 32 * part

    if (warp == 5) {
        if (lane == 0) {
            // ---- TMA producer: K_{j+1} once S_j is done, V_{j+1} once PV_j is done
            bool ok = true;
            int kq = 1, vq = 1;
            for (int j = 0; j + 1 < nkt && ok; j++) {
                if (!(ok = wait_bar(&ctl->k_empty, (uint32_t)j & 1, abort_flag))) break;
                load_kv(&tK, sK, &ctl->k_full, j + 1);
                kq++;
                if (!(ok = wait_bar(&ctl->v_empty, (uint32_t)j & 1, abort_flag))) break;
                load_kv(&tV, sV, &ctl->v_full, j + 1);
                vq++;
            }
            if (!ok) {
                // drain this thread's own TMA loads (bounded) before shared memory is released
                for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->q_full, 0); w++) {}
                for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->k_full, (uint32_t)(kq - 1) & 1); w++) {}
                for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->v_full, (uint32_t)(vq - 1) & 1); w++) {}
            }
        }
    } else if (warp == 4) {
        if (lane == 0) {
            // ---- MMA issuer
            auto issue_s = [&]() {
                #pragma unroll 1
                for (int t = 0; t < X3_NTERM; t++) {
                    const uint8_t* qa = sQ + c_x3_terms[t][0] * TILE_BYTES;
                    const uint8_t* kb = sK + c_x3_terms[t][1] * KV4_BYTES;
                    #pragma unroll
                    for (int kk = 0; kk < D / 16; kk++) {
                        const uint32_t aoff = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
                        const uint32_t boff = (kk >> 2) * KV4_HALF + (kk & 3) * 32;
                        sm100::mma_bf16(tS, sm100::desc_kmajor_sw128(qa, aoff), sm100::desc_kmajor_sw128(kb, boff),
                                        IDESC_QK4, (t | kk) != 0);
                    }
                }
                sm100::mma_commit(&ctl->s_full);
                sm100::mma_commit(&ctl->k_empty);
            };
            bool ok = wait_bar(&ctl->q_full, 0, abort_flag);
            if (ok && (ok = wait_bar(&ctl->k_full, 0, abort_flag))) {
                sm100::tc_fence_after();
                issue_s();
            }
            for (int j = 0; j < nkt && ok; j++) {
                if (j + 1 < nkt) {
                    // the softmax has S_j in registers and K_{j+1} is in
                    if (!(ok = wait_bar(&ctl->s_free, (uint32_t)j & 1, abort_flag))) break;
                    if (!(ok = wait_bar(&ctl->k_full, (uint32_t)(j + 1) & 1, abort_flag))) break;
                    sm100::tc_fence_after();
                    issue_s();
                }
                if (!(ok = wait_bar(&ctl->p_ready, (uint32_t)j & 1, abort_flag))) break;
                if (!(ok = wait_bar(&ctl->v_full, (uint32_t)j & 1, abort_flag))) break;
                sm100::tc_fence_after();
                #pragma unroll 1
                for (int t = 0; t < X3_NTERM; t++) {
                    const uint32_t pa = tP + 32 * c_x3_terms[t][0];
                    const uint8_t* vb = sV + c_x3_terms[t][1] * KV4_BYTES;
                    #pragma unroll
                    for (int kk = 0; kk < KT4 / 16; kk++)
                        sm100::mma_bf16_tmem_a(tO, pa + kk * 8, desc_v64(vb, kk * 2048), IDESC_PV, (j | t | kk) != 0);
                }
                sm100::mma_commit(&ctl->pv_done);
                sm100::mma_commit(&ctl->v_empty);
                if (j + 1 == nkt) sm100::mma_commit(&ctl->o_full);
            }
            sm100::mma_commit(&ctl->drain);
            for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->drain, 0); w++) {}
        }
    } else {
        // ---- softmax + epilogue: thread = query row q0 + r; TMEM lane quadrant = warp
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const float sl = p.scale_log2;
        const bool live = q0 + warp * 32 < S;  // warp-uniform: any of this warp's rows is a query
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkt; j++) {
            ok = __all_sync(0xffffffffu, wait_bar(&ctl->s_full, (uint32_t)j & 1, abort_flag));
            if (!ok) break;
            float v[64];
            if (live) {
                sm100::tc_fence_after();
                sm100::tmem_ld64(tS + lane_off, v);
            }
            // S_j is in registers: the slot may take S_{j+1}
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&ctl->s_free);
            bool pv_waited = (j == 0);                 // warp-uniform
            uint32_t ph[32], pm[32], pl[32];
            if (live) {
                const int kvalid = S - j * KT4;
                const bool full = kvalid >= KT4;           // CTA-uniform
                const float mx = (full ? max64_full(v) : max64_t<true>(v, kvalid)) * sl;
                if (j == 0) {
                    m = mx;
                } else {
                    const bool grow = mx > m + T_RESCALE;
                    if (__any_sync(0xffffffffu, grow)) {
                        ok = __all_sync(0xffffffffu, wait_bar(&ctl->pv_done, (uint32_t)(j - 1) & 1, abort_flag));
                        if (!ok) break;
                        pv_waited = true;
                        sm100::tc_fence_after();
                        const float mn = grow ? mx : m;
                        const float corr = exp2f(m - mn);
                        #pragma unroll 1
                        for (int c = 0; c < 4; c++) {
                            float o[32];
                            sm100::tmem_ld32(tO + lane_off + c * 32, o);
                            #pragma unroll
                            for (int u = 0; u < 32; u++) o[u] *= corr;
                            tmem_st32(tO + lane_off + c * 32, o);
                        }
                        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                        l *= corr;
                        m = mn;
                    }
                }
                const float nm = -m;
                float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                #pragma unroll
                for (int u = 0; u < 32; u++) {
                    float a = ex2_approx(fmaf(v[2 * u], sl, nm)), b = ex2_approx(fmaf(v[2 * u + 1], sl, nm));
                    if (!full) { a = (2 * u < kvalid) ? a : 0.f; b = (2 * u + 1 < kvalid) ? b : 0.f; }
                    ls[u & 7] += a + b;
                    split3_pair(a, b, ph[u], pm[u], pl[u]);
                }
                l += sum8(ls);
            }
            // every warp waits for PV_{j-1} before its p_ready of step j: the
            // P parts are free, and no arrival of step j lands in step j-1's phase
            if (!pv_waited) {
                ok = __all_sync(0xffffffffu, wait_bar(&ctl->pv_done, (uint32_t)(j - 1) & 1, abort_flag));
                if (!ok) break;
            }
            if (live) {
                tmem_st32u(tP + lane_off, ph);
                tmem_st32u(tP + lane_off + 32, pm);
                tmem_st32u(tP + lane_off + 64, pl);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            }
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&ctl->p_ready);
        }
        if (ok) ok = __all_sync(0xffffffffu, wait_bar(&ctl->o_full, 0, abort_flag));
        if (ok && live) {
            sm100::tc_fence_after();
            const float inv = 1.f / l;
            float* stage = reinterpret_cast<float*>(smem) + (size_t)warp * 32 * STG_LD;
            float* mine = stage + lane * STG_LD;
            #pragma unroll 1
            for (int c = 0; c < 2; c++) {
                float o[64];
                sm100::tmem_ld64(tO + lane_off + c * 64, o);
                #pragma unroll
                for (int u = 0; u < 64; u += 4)
                    *reinterpret_cast<float4*>(mine + c * 64 + u) =
                        make_float4(o[u] * inv, o[u + 1] * inv, o[u + 2] * inv, o[u + 3] * inv);
            }
            const int qw = q0 + warp * 32;
            const int nrows = min(32, S - qw);
            __syncwarp();
            #pragma unroll 4
            for (int rr = 0; rr < nrows; rr++) {
                const int q = qw + rr;
                const int tok = __shfl_sync(0xffffffffu, my_tok, rr);
                const float4 x = *reinterpret_cast<const float4*>(stage + rr * STG_LD + lane * 4);
                const float xv[4] = {x.x, x.y, x.z, x.w};
                if (q < f) {
                    if (p.att_t == ACT_BF16)
                        store4((bf16*)p.att + (size_t)tok * p.ld_att + h * D + lane * 4, xv);
                    else if (p.att_t == ACT_F16)
                        store4((f16*)p.att + (size_t)tok * p.ld_att + h * D + lane * 4, xv);
                    else
                        store4((float*)p.att + (size_t)tok * p.ld_att + h * D + lane * 4, xv);
                } else {
                    store4(p.toutw + ((size_t)wi * p.g.TXT + (q - f)) * 2560 + h * D + lane * 4, xv);
                }
            }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem, X3_TMEM);
    }
}

}  // namespace

bool awa_tc_available() { return true; }

int awa_attend_tc(const void* Qp, const void* Kp, const void* Vp, ActT qkv_t, const AwaDev& g, float scale, void* att,
                  int ld_att, ActT at, float* toutw, cudaStream_t s) {
    if (qkv_t != ACT_BF16 && qkv_t != ACT_F16) return -1;
    const int rows = 20 * g.sumS;
    CUtensorMap tq, tk, tv;
    if (!make_tmap_bf16(&tq, Qp, rows, D, D, QT, 64) || !make_tmap_bf16(&tk, Kp, rows, D, D, KT4, 64) ||
        !make_tmap_bf16(&tv, Vp, rows, D, D, KT4, 64))
        return -1;
    AttnParams p;
    p.g = g;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.att = att;
    p.ld_att = ld_att;
    p.att_t = at;
    p.toutw = toutw;
    {
        dim3 grid((g.maxS + QT - 1) / QT, 20, g.nwin);
        const int np = awa_tc_poly_exp();
        if (qkv_t == ACT_F16) {
            if (np == 2) k_awa_attn_tc4<2, true><<<grid, T4_THREADS, T4_SMEM, s>>>(tq, tk, tv, p);
            else if (np == 1) k_awa_attn_tc4<1, true><<<grid, T4_THREADS, T4_SMEM, s>>>(tq, tk, tv, p);
            else k_awa_attn_tc4<0, true><<<grid, T4_THREADS, T4_SMEM, s>>>(tq, tk, tv, p);
        } else {
            if (np == 2) k_awa_attn_tc4<2, false><<<grid, T4_THREADS, T4_SMEM, s>>>(tq, tk, tv, p);
            else if (np == 1) k_awa_attn_tc4<1, false><<<grid, T4_THREADS, T4_SMEM, s>>>(tq, tk, tv, p);
            else k_awa_attn_tc4<0, false><<<grid, T4_THREADS, T4_SMEM, s>>>(tq, tk, tv, p);
        }
    }
    return 0;
}

int awa_attend_split3(const void* Q3, const void* K3, const void* V3, const AwaDev& g, float scale, void* att,
                      int ld_att, ActT at, float* toutw, cudaStream_t s) {
    const int rows = 3 * 20 * g.sumS;       // the three parts stacked
    CUtensorMap tq, tk, tv;
    if (!make_tmap_bf16(&tq, Q3, rows, D, D, QT, 64) || !make_tmap_bf16(&tk, K3, rows, D, D, KT4, 64) ||
        !make_tmap_bf16(&tv, V3, rows, D, D, KT4, 64))
        return -1;
    AttnParams p;
    p.g = g;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.att = att;
    p.ld_att = ld_att;
    p.att_t = at;
    p.toutw = toutw;
    dim3 grid((g.maxS + QT - 1) / QT, 20, g.nwin);
    k_awa_attn_x3<<<grid, T4_THREADS, X3_SMEM, s>>>(tq, tk, tv, p);
    return 0;
}

int awa_tc_init_device() {
    if (cudaError_t e = cudaFuncSetAttribute(k_awa_attn_x3, cudaFuncAttributeMaxDynamicSharedMemorySize, X3_SMEM))
        return (int)e;
    const void* v4[6] = {(const void*)k_awa_attn_tc4<0, false>, (const void*)k_awa_attn_tc4<1, false>,
                         (const void*)k_awa_attn_tc4<2, false>, (const void*)k_awa_attn_tc4<0, true>,
                         (const void*)k_awa_attn_tc4<1, true>, (const void*)k_awa_attn_tc4<2, true>};
    for (const void* k : v4)
        if (cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, T4_SMEM)) return (int)e;
    return 0;
}

// S2B_ATTN_POLY=n (0, 1, 2): n of every 4 softmax exponential pairs of the
// 64-key kernel on the FMA pipe (ex2_poly2).
int awa_tc_poly_exp() {
    const char* e = std::getenv("S2B_ATTN_POLY");
    return (e && e[0] == '2') ? 2 : (e && e[0] == '1') ? 1 : 0;
}

int awa_tc_flag_ptr(int** p) { return (int)cudaGetSymbolAddress((void**)p, g_attn_err); }

}  // namespace s2b
