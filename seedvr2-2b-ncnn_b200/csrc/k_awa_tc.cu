// k_awa_tc.cu -- AWA window attention on the 5th-gen tensor cores (bf16).
//
// One CTA = one (window, head, 128-query tile).  Keys of the window are
// streamed in 128-key tiles; all operands come from the window-packed,
// head-major Q/K/V slabs the pack kernel writes (k_awa.cu), so every tile is
// a plain 2-D TMA box.
//   S_j  = Q K_j^T        tcgen05.mma, A = Q, B = K_j (both K-major, 128-B
//                         swizzle), fp32 accumulator in TMEM (128 columns)
//   softmax (warps 0-3)   thread = query row: tcgen05.ld of its S row,
//                         online max / sum in fp32 (exp2), O rescaled in
//                         TMEM when the running max grows, P_j rounded to
//                         bf16 and written to shared memory in the K-major
//                         swizzled layout, over K_j's spent tile
//   O   += P_j V_j        tcgen05.mma, A = P_j (K-major), B = V_j
//                         (MN-major: head dims contiguous), TMEM 128 columns
//   epilogue              O / l; vid rows go back to their grid token, txt
//                         rows to the per-window partials averaged later.
// Warp 4 lane 0 issues the TMA loads and the MMAs.  Keys past the window's
// end are masked to -inf (their smem rows hold the neighbouring window's
// finite data or TMA zero fill).  96 KB shared memory and 256 TMEM columns
// per CTA, so two CTAs share an SM and one's softmax overlaps the other's
// MMAs.  Every mbarrier wait is bounded (error flag g_attn_err on expiry).
#include "kernels.h"
#include "kcommon.cuh"
#include "sm100.cuh"
#include <cuda.h>

namespace s2b {

bool make_tmap_bf16(CUtensorMap* m, const void* base, int rows, int cols, int ld, int box_rows, int box_cols);

namespace {

constexpr int QT = 128, KT = 128, D = 128;
constexpr int TILE_BYTES = QT * D * 2;            // 32 KB: two 64-column swizzled halves
constexpr int HALF_BYTES = TILE_BYTES / 2;
constexpr int NUM_THREADS = 160;
constexpr int TMEM_COLS = 256;                     // S: [0,128), O: [128,256)
constexpr int SMEM_BYTES = 3 * TILE_BYTES + 1024 + 256;
constexpr uint32_t IDESC_QK = sm100::idesc_bf16_f32(QT, KT);
constexpr uint32_t IDESC_PV = sm100::idesc_bf16_f32(QT, D) | (1u << 16);   // B (V) MN-major

__device__ int g_attn_err;

struct AttnCtl {
    uint64_t q_full, k_full, v_full, s_full, p_ready, pv_done;
    uint32_t tmem_slot;
    int abort;
};

struct AttnParams {
    AwaDev g;
    float scale_log2;     // softmax scale * log2(e)
    void* att;            // vid rows: [Lv][ld_att] in att_t
    int ld_att;
    int att_bf16;
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

// MN-major operand (V: rows = keys, 64 head dims per 128-B row, two 64-dim
// halves 16 KB apart): leading byte offset = distance between 64-wide MN
// blocks, stride byte offset = distance between 8-key groups.
__device__ __forceinline__ uint64_t desc_mnmajor_sw128(const void* tile, uint32_t k_group_bytes) {
    const uint32_t addr = sm100::smem_u32(tile) + k_group_bytes;
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)(HALF_BYTES >> 4) << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
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

__global__ void __launch_bounds__(NUM_THREADS, 2)
k_awa_attn_tc(const __grid_constant__ CUtensorMap tQ, const __grid_constant__ CUtensorMap tK,
              const __grid_constant__ CUtensorMap tV, const AttnParams p) {
    const int wi = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * QT;
    const int f = p.g.cumf[wi + 1] - p.g.cumf[wi];
    const int S = f + p.g.TXT;
    if (q0 >= S) return;                       // uniform across the CTA, before any barrier
    const int nkt = (S + KT - 1) / KT;
    const int row_base = h * p.g.sumS + p.g.cums[wi];

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = smem + TILE_BYTES;          // K_j, then P_j
    uint8_t* sV = smem + 2 * TILE_BYTES;
    AttnCtl* ctl = reinterpret_cast<AttnCtl*>(smem + 3 * TILE_BYTES);
    volatile int* abort_flag = &ctl->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        sm100::mbar_init(&ctl->q_full, 1);
        sm100::mbar_init(&ctl->k_full, 1);
        sm100::mbar_init(&ctl->v_full, 1);
        sm100::mbar_init(&ctl->s_full, 1);
        sm100::mbar_init(&ctl->p_ready, 4);
        sm100::mbar_init(&ctl->pv_done, 1);
        ctl->abort = 0;
        sm100::fence_barrier_init();
    }
    if (warp == 4) {
        sm100::tmem_alloc(&ctl->tmem_slot, TMEM_COLS);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = ctl->tmem_slot;
    const uint32_t tS = tmem, tO = tmem + 128;

    if (warp == 4) {
        if (lane == 0) {
            bool ok = true;
            sm100::mbar_arrive_expect_tx(&ctl->q_full, TILE_BYTES);
            sm100::tma_load_2d(sQ, &tQ, &ctl->q_full, 0, row_base + q0);
            sm100::tma_load_2d(sQ + HALF_BYTES, &tQ, &ctl->q_full, 64, row_base + q0);
            sm100::mbar_arrive_expect_tx(&ctl->k_full, TILE_BYTES);
            sm100::tma_load_2d(sK, &tK, &ctl->k_full, 0, row_base);
            sm100::tma_load_2d(sK + HALF_BYTES, &tK, &ctl->k_full, 64, row_base);
            sm100::mbar_arrive_expect_tx(&ctl->v_full, TILE_BYTES);
            sm100::tma_load_2d(sV, &tV, &ctl->v_full, 0, row_base);
            sm100::tma_load_2d(sV + HALF_BYTES, &tV, &ctl->v_full, 64, row_base);
            int kv_issued = 1;        // K/V tile loads issued so far
            ok = wait_bar(&ctl->q_full, 0, abort_flag);
            for (int j = 0; j < nkt && ok; j++) {
                const uint32_t ph = j & 1;
                if (!(ok = wait_bar(&ctl->k_full, ph, abort_flag))) break;
                sm100::tc_fence_after();
                #pragma unroll
                for (int kk = 0; kk < D / 16; kk++) {
                    const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
                    sm100::mma_bf16(tS, sm100::desc_kmajor_sw128(sQ, off), sm100::desc_kmajor_sw128(sK, off),
                                    IDESC_QK, kk != 0);
                }
                sm100::mma_commit(&ctl->s_full);
                if (!(ok = wait_bar(&ctl->v_full, ph, abort_flag))) break;
                if (!(ok = wait_bar(&ctl->p_ready, ph, abort_flag))) break;
                sm100::tc_fence_after();
                #pragma unroll
                for (int kk = 0; kk < KT / 16; kk++) {
                    const uint32_t aoff = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
                    sm100::mma_bf16(tO, sm100::desc_kmajor_sw128(sK, aoff), desc_mnmajor_sw128(sV, kk * 2048),
                                    IDESC_PV, (j | kk) != 0);
                }
                sm100::mma_commit(&ctl->pv_done);
                if (j + 1 < nkt) {
                    // P_j (in the K buffer) and V_j are read by the PV MMAs: wait, then refill
                    if (!(ok = wait_bar(&ctl->pv_done, ph, abort_flag))) break;
                    const int r = row_base + (j + 1) * KT;
                    sm100::mbar_arrive_expect_tx(&ctl->k_full, TILE_BYTES);
                    sm100::tma_load_2d(sK, &tK, &ctl->k_full, 0, r);
                    sm100::tma_load_2d(sK + HALF_BYTES, &tK, &ctl->k_full, 64, r);
                    sm100::mbar_arrive_expect_tx(&ctl->v_full, TILE_BYTES);
                    sm100::tma_load_2d(sV, &tV, &ctl->v_full, 0, r);
                    sm100::tma_load_2d(sV + HALF_BYTES, &tV, &ctl->v_full, 64, r);
                    kv_issued++;
                }
            }
            if (!ok) {
                // drain this thread's own TMA loads (bounded) before shared memory is released
                const uint32_t ph = (uint32_t)(kv_issued - 1) & 1;
                for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->q_full, 0); w++) {}
                for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->k_full, ph); w++) {}
                for (uint32_t w = 0; w < sm100::WAIT_LIMIT && !sm100::mbar_try_wait(&ctl->v_full, ph); w++) {}
            }
        }
    } else {
        // softmax / epilogue: thread = query row q0 + r; TMEM lane quadrant = warp
        const int r = warp * 32 + lane;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        // Every tcgen05.ld / tcgen05.st below is warp-collective (.sync.aligned):
        // all 32 lanes execute each one, with warp-uniform control flow; the
        // per-row differences only select values and stores.
        for (int j = 0; j < nkt; j++) {
            ok = __all_sync(0xffffffffu, wait_bar(&ctl->s_full, j & 1, abort_flag));
            if (!ok) break;
            sm100::tc_fence_after();
            const int kvalid = S - j * KT;           // keys [0, kvalid) of this tile are real
            float s[128];
            #pragma unroll
            for (int c = 0; c < 4; c++) sm100::tmem_ld32(tS + lane_off + c * 32, s + c * 32);
            float mx = -INFINITY;
            #pragma unroll
            for (int c = 0; c < 128; c++) {
                s[c] = (c < kvalid) ? s[c] * p.scale_log2 : -INFINITY;
                mx = fmaxf(mx, s[c]);
            }
            const float mn = fmaxf(m, mx);
            // rescale the running O rows when any row's max grew (the previous
            // PV is complete: its commit preceded this S tile's)
            const bool grow = (j > 0) && (mn > m);
            if (__any_sync(0xffffffffu, grow)) {
                const float corr = grow ? exp2f(m - mn) : 1.f;
                #pragma unroll 1
                for (int c = 0; c < 4; c++) {
                    float o[32];
                    sm100::tmem_ld32(tO + lane_off + c * 32, o);
                    #pragma unroll
                    for (int t = 0; t < 32; t++) o[t] *= corr;
                    tmem_st32(tO + lane_off + c * 32, o);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                l *= corr;
            }
            m = mn;
            // P row -> shared memory, K-major 128-B swizzled [128 rows x 128 keys]
            #pragma unroll
            for (int c8 = 0; c8 < 16; c8++) {
                float pv[8];
                #pragma unroll
                for (int t = 0; t < 8; t++) { pv[t] = exp2f(s[c8 * 8 + t] - mn); l += pv[t]; }
                uint4 u;
                __nv_bfloat162 a = __floats2bfloat162_rn(pv[0], pv[1]), b = __floats2bfloat162_rn(pv[2], pv[3]);
                __nv_bfloat162 cc = __floats2bfloat162_rn(pv[4], pv[5]), d = __floats2bfloat162_rn(pv[6], pv[7]);
                u.x = *reinterpret_cast<uint32_t*>(&a); u.y = *reinterpret_cast<uint32_t*>(&b);
                u.z = *reinterpret_cast<uint32_t*>(&cc); u.w = *reinterpret_cast<uint32_t*>(&d);
                const int half = c8 >> 3, chunk = c8 & 7;
                uint8_t* dst = sK + half * HALF_BYTES + r * 128 + ((chunk ^ (r & 7)) << 4);
                *reinterpret_cast<uint4*>(dst) = u;
            }
            sm100::fence_proxy_async_smem();      // generic-proxy smem writes -> tensor-core reads
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&ctl->p_ready);
        }
        if (ok) ok = __all_sync(0xffffffffu, wait_bar(&ctl->pv_done, (nkt - 1) & 1, abort_flag));
        if (ok) {
            sm100::tc_fence_after();
            const int q = q0 + r;
            const float inv = 1.f / l;
            const bool is_vid = q < f, is_txt = (q >= f) && (q < S);
            float* tdst = p.toutw + ((size_t)wi * p.g.TXT + (is_txt ? q - f : 0)) * 2560 + h * D;
            const size_t tok = is_vid ? (size_t)p.g.vidx[p.g.cumf[wi] + q] : 0;
            #pragma unroll 1
            for (int c = 0; c < 4; c++) {
                float o[32];
                sm100::tmem_ld32(tO + lane_off + c * 32, o);
                #pragma unroll
                for (int t = 0; t < 32; t++) o[t] *= inv;
                if (is_vid) {
                    if (p.att_bf16) {
                        bf16* dst = (bf16*)p.att + tok * p.ld_att + h * D + c * 32;
                        #pragma unroll
                        for (int t = 0; t < 32; t += 4) store4(dst + t, o + t);
                    } else {
                        float* dst = (float*)p.att + tok * p.ld_att + h * D + c * 32;
                        #pragma unroll
                        for (int t = 0; t < 32; t += 4) store4(dst + t, o + t);
                    }
                } else if (is_txt) {
                    #pragma unroll
                    for (int t = 0; t < 32; t += 4) store4(tdst + c * 32 + t, o + t);
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

}  // namespace

bool awa_tc_available() { return true; }

int awa_attend_tc(const void* Qp, const void* Kp, const void* Vp, const AwaDev& g, float scale, void* att, int ld_att,
                  ActT at, float* toutw, cudaStream_t s) {
    const int rows = 20 * g.sumS;
    CUtensorMap tq, tk, tv;
    if (!make_tmap_bf16(&tq, Qp, rows, D, D, QT, 64) || !make_tmap_bf16(&tk, Kp, rows, D, D, KT, 64) ||
        !make_tmap_bf16(&tv, Vp, rows, D, D, KT, 64))
        return -1;
    AttnParams p;
    p.g = g;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.att = att;
    p.ld_att = ld_att;
    p.att_bf16 = (at == ACT_BF16);
    p.toutw = toutw;
    dim3 grid((g.maxS + QT - 1) / QT, 20, g.nwin);
    k_awa_attn_tc<<<grid, NUM_THREADS, SMEM_BYTES, s>>>(tq, tk, tv, p);
    return 0;
}

int awa_tc_init_device() {
    return (int)cudaFuncSetAttribute(k_awa_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
}

int awa_tc_error_reset(int* had_error) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_attn_err, sizeof v);
    if (e != cudaSuccess) return (int)e;
    if (had_error) *had_error = v;
    const int zero = 0;
    return (int)cudaMemcpyToSymbol(g_attn_err, &zero, sizeof zero);
}

}  // namespace s2b
