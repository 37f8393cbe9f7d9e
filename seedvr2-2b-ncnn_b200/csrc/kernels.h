// kernels.h -- host-side launchers of the sm_100a kernels (no torch types).
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace s2b {

// Operand types: fp32, and the two 16-bit types of the tensor cores' kind::f16
// (bf16 for the bf16 precision, IEEE binary16 for the fp16 precision).
enum ActT { ACT_F32 = 0, ACT_BF16 = 1, ACT_F16 = 2 };
__host__ __device__ inline size_t act_bytes(ActT t) { return t == ACT_F32 ? 4 : 2; }
__host__ __device__ inline bool act_half(ActT t) { return t != ACT_F32; }

// ---------------------------------------------------------------- GEMM
enum EpiMode {
    EPI_STORE = 0,       // out[r,c] = acc + bias[c]
    EPI_GATE_RESID = 1,  // resid[r,c] = (acc + bias[c]) * gate[c] + resid[r,c]
    EPI_SWIGLU = 2,      // 256-wide column blocks [h 128 | g 128]: out[r, blk*128+j] = silu(g_j) * h_j
    EPI_QKV_PACK = 3,    // qkv projection -> qk RMSNorm + RoPE -> window-packed Q/K/V (tcgen05 kernel only)
};

// Window geometry + per-flow qk-norm weights for EPI_QKV_PACK.  Rows of the
// GEMM are rows row_base.. of the [vid | txt] residual: row < Lv is grid
// token `row` (one packed destination), row >= Lv is txt row row - Lv (one
// destination per window).
// RoPE angles must follow the make_win structure (checked on the host): the
// angle of pair i of a row is pos[i / 21] * base[i % 21] with pos = (txt_len +
// t, local h, local w) for vid rows and (p, p, p) for txt row p, so one
// (cos, sin) table indexed [pos][21] reproduces the per-element tables.
struct PackEpi {
    const int4* tokpos = nullptr;   // [Lv] (vid packed index gi, window, pos0 | pos1 << 16, pos2)
    const int* cums = nullptr;      // [nwin+1] packed row offsets of windows
    const float2* cs = nullptr;     // [npos][21] (cos, sin)
    int npos = 0;
    const float *nq0 = nullptr, *nk0 = nullptr;     // vid flow qk-norm weights [128]
    const float *nq1 = nullptr, *nk1 = nullptr;     // txt flow
    float eps = 1e-5f;
    int Lv = 0, TXT = 0, nwin = 0, sumS = 0, row_base = 0;
    void *Qp = nullptr, *Kp = nullptr, *Vp = nullptr;   // [20][sumS][128] in qkv_t
    ActT qkv_t = ACT_BF16;                              // ACT_BF16 or ACT_F16
};

struct GemmEpi {
    PackEpi pk;
    EpiMode mode = EPI_STORE;
    ActT op_t = ACT_BF16;            // tcgen05 kernels: the 16-bit type of A and W (both the same)
    const float* bias = nullptr;     // [N] or null
    void* out = nullptr;             // STORE / SWIGLU output
    int ldo = 0;
    ActT out_t = ACT_F32;
    float* resid = nullptr;          // GATE_RESID target (fp32 residual stream)
    int ldr = 0;
    const float* gate0 = nullptr;    // rows < gate_split (null: gate 1)
    const float* gate1 = nullptr;    // rows >= gate_split (null: gate 1)
    int gate_split = 0;
    // EPI_GATE_RESID fused with the next RMSNorm + adaLN scale (bf16 operand):
    // also mod_out[r][c] = bf16(resid_new[r][c] * sc[c]) (sc = mod_sc0 for rows
    // < mod_split, else mod_sc1; null: 1) and per row the sum of squares of
    // resid_new over every 128-column block: sq_out[r * SQ_SLOTS + c / 128].
    void* mod_out = nullptr;
    int ldm = 0;
    const float* mod_sc0 = nullptr;
    const float* mod_sc1 = nullptr;
    int mod_split = 0;
    float* sq_out = nullptr;
    // EPI_QKV_PACK / EPI_SWIGLU on such an operand: acc is first scaled per row
    // by rs = 1 / sqrt(sum_b sq_in[r * SQ_SLOTS + b] / rs_dim + rs_eps) (the
    // RMSNorm, applied after the GEMM since it is one factor per row), then the
    // bias (there: the adaLN shift folded through the weights) is added.
    const float* sq_in = nullptr;
    int sq_n = 0;
    float rs_dim = 2560.f;
    float rs_eps = 1e-5f;
};
// Row slots of the fused-norm partial sums of squares (2560 / 128).
constexpr int SQ_SLOTS = 20;

// C = A[M,K] (row stride lda) x W[N,K]^T (row stride ldw), fp32 accumulate,
// fused epilogue.  SIMT kernel; any M, N, K.
void gemm_simt(const void* A, ActT at, int lda, const void* W, ActT wt, int ldw, int M, int N, int K,
               const GemmEpi& e, cudaStream_t s);

// One-row fp32 GEMV y = act(x W^T + b) (act = SiLU when silu); false when
// the shapes do not suit it (K and ldw multiples of 4, 16-B aligned x / W).
bool gemv_f32(const float* x, int K, const float* W, int ldw, int N, const float* bias, float* y, bool silu,
              cudaStream_t s);

// tcgen05 (5th-gen tensor core) BF16 GEMM, TMA-staged, TMEM accumulators.
// Requirements: A, W bf16, K % 64 == 0 (the TMA maps zero-fill ragged M/N),
// lda/ldw multiples of 8 elements, 16-byte aligned bases.
bool gemm_tc_supported(int M, int N, int K, int lda, int ldw);
int gemm_tc(const void* A, int lda, const void* W, int ldw, int M, int N, int K, const GemmEpi& e,
            cudaStream_t s, int* launches);
// Two GEMMs with the same N, K and epilogue mode (the vid and txt Linears of
// an MM-DiT block) in one launch of the CTA-pair kernel; their tiles share
// the persistent grid.  Returns -1 when either does not suit the kernel.
int gemm_tc_grouped(const void* A0, int lda0, const void* W0, int ldw0, int M0, const GemmEpi& e0, const void* A1,
                    int lda1, const void* W1, int ldw1, int M1, const GemmEpi& e1, int N, int K, cudaStream_t s,
                    int* launches);
// fp32 GEMM on the tensor cores ("3xTF32"): A2 [M][2K] and W2 [N][2K] hold
// [hi | lo] halves (split_tf32); C = A_hi W_hi^T + A_hi W_lo^T + A_lo W_hi^T
// with fp32 accumulation.  K % 32 == 0; lda2 / ldw2 multiples of 4.
bool gemm_tf32x3_supported(int M, int N, int K, int lda2, int ldw2);
int gemm_tf32x3(const void* A2, int lda2, const void* W2, int ldw2, int M, int N, int K, const GemmEpi& e,
                cudaStream_t s, int* launches);
// dst[r][0..cols) = tf32(src[r][c]) (round to nearest), dst[r][cols..2cols) = src - that.
void split_tf32(const float* src, int ld_src, int rows, int cols, float* dst, int ld_dst, cudaStream_t s);

// ---------------------------------------------------------------- elementwise
// Row RMSNorm (eps, optional affine weight) + adaLN modulate.  Rows < split
// use (sc0, sh0), the rest (sc1, sh1); a null scale means "norm only".
// Output y[r*ldy + d] in type yt.
void rmsnorm_mod(const float* X, int ldx, int rows, int split, const float* sc0, const float* sh0,
                 const float* sc1, const float* sh1, const float* affine, float eps, void* Y, int ldy,
                 ActT yt, cudaStream_t s);
// HG rows hold 54 column blocks [h 128 | g 128]; Hs[r, b*128+j] = silu(g) * h.
void swiglu_rows(const float* HG, int M, int ldhg, void* Hs, int ldh, ActT ht, cudaStream_t s);
// out[i] = silu(x[i]) (time embedding MLP)
void silu_inplace(float* x, int n, cudaStream_t s);
// out[v][d] = emb[d*6 + k(v)] + branch[v][d] for the 32*12+2 modulation vectors.
void ada_compose(const float* emb, const float* branch, int nvec, float* out, cudaStream_t s);
// dst[r*ld_dst + c] = src[r*cols + c] for c < cols, 0 for cols <= c < ld_dst.
void pad_convert_rows(const float* src, int rows, int cols, void* dst, int ld_dst, ActT t, cudaStream_t s);
void convert_f32(const float* src, size_t n, void* dst, ActT t, cudaStream_t s);
void convert_to_f32(const void* src, ActT t, size_t n, float* dst, cudaStream_t s);
// Weight ingest: src [out][in] (fp16 bits or fp32) -> dst rows of `ld` elements
// in type t, zero-padded past `in`.  With blk_rows > 0, source row r lands on
// destination row (r / blk_rows) * blk_stride + row_off + r % blk_rows.
void ingest_weight(const void* src, bool src_f16, int out, int in, void* dst, ActT t, int ld, int blk_rows,
                   int blk_stride, int row_off, cudaStream_t s);
// y[n] = sum_k W[n][k] x[k] for bf16 W (row stride ld) and fp32 x, fp32
// accumulate in a fixed order (one warp per row).
void gemv_bf16(const void* W, int ld, int N, int K, const float* x, float* y, cudaStream_t s);
// Per-device one-time kernel attributes (dynamic shared memory opt-ins).
int kernels_init_device();
// *p = v on stream s (one thread; the value travels as a kernel argument).
void set_u32(uint32_t* p, uint32_t v, cudaStream_t s);

// ---------------------------------------------------------------- kernel error status
// Every bounded wait of the tcgen05 GEMM, the tcgen05 attention and the
// peer-memory exchanges sets its kernel class's device flag when it expires
// (the kernel then returns early, leaving its output incomplete).  The flags
// are module globals of the device, shared by every context on it.
enum KernelErrBit { KERR_GEMM = 1, KERR_ATTN = 2, KERR_SHARD = 4 };
struct KernelFlags { int* gemm = nullptr; int* attn = nullptr; int* shard = nullptr; };
// Device addresses of the three flags on the current device (cudaError_t value).
int kernel_flags_get(KernelFlags* f);
// One thread, stream-ordered after the kernels it covers: *status |= the
// KernelErrBit of every raised flag, then the flags are cleared.
void status_fold(const KernelFlags& f, int* status, cudaStream_t s);
// Test hook: raise the flags named by mask (KernelErrBit) from one thread.
void status_raise(const KernelFlags& f, int mask, cudaStream_t s);

// ---------------------------------------------------------------- AWA
struct AwaDev {
    int nwin = 0, TXT = 0, sumf = 0, sumS = 0, maxS = 0, Lv = 0;
    const int* vidx = nullptr;      // [sumf]
    const int* cumf = nullptr;      // [nwin+1]
    const int* cums = nullptr;      // [nwin+1]
    const int* row_win = nullptr;   // [sumS] window of each packed row
    const float* vcos = nullptr;    // [sumf][126]
    const float* vsin = nullptr;
    const float* tcos = nullptr;    // [nwin*TXT][126]
    const float* tsin = nullptr;
};
// qk RMSNorm + RoPE + window packing: Qp/Kp/Vp [HEADS][sumS][128].
void awa_pack(const void* vqkv, const void* tqkv, ActT in_t, int ldq, const AwaDev& g, const float* nqv,
              const float* nkv, const float* nqt, const float* nkt, float eps, void* Qp, void* Kp, void* Vp,
              ActT pt, cudaStream_t s);
// The same packing for the fp32 tensor-core attention: Q3/K3/V3 each hold
// three bf16 parts [3][HEADS][sumS][128] (hi, mid, lo; hi + mid + lo equals
// the fp32 value to fp32 precision).
void awa_pack_split3(const void* vqkv, const void* tqkv, ActT in_t, int ldq, const AwaDev& g, const float* nqv,
                     const float* nkv, const float* nqt, const float* nkt, float eps, void* Q3, void* K3, void* V3,
                     cudaStream_t s);
// fp32 attention on the tcgen05 tensor cores from split3 operands: QK^T and
// PV as the six bf16 part products of order <= 2 (hi.hi, hi.mid, mid.hi,
// hi.lo, lo.hi, mid.mid), fp32 accumulation in TMEM.  Returns -1 when the
// kernel cannot run (no tensor-map encoder); then nothing was launched.
int awa_attend_split3(const void* Q3, const void* K3, const void* V3, const AwaDev& g, float scale, void* att,
                      int ld_att, ActT at, float* toutw, cudaStream_t s);
// Per-window SDPA.  vid rows scattered to att[vidx]; txt rows to toutw[wi][i].
// 16-bit operands (bf16 / f16) run the tcgen05 kernel only: -1 (nothing launched) when its
// tensor maps cannot be encoded.  fp32 operands run the SIMT kernel.
int awa_attend(const void* Qp, const void* Kp, const void* Vp, ActT pt, const AwaDev& g, float scale,
                void* att, int ld_att, ActT at, float* toutw, cudaStream_t s, int* launches);
// att_txt[i, d] = sum_w toutw[w][i][d] / nwin
void awa_coalesce(const float* toutw, int nwin, int TXT, void* att_txt, int ld_att, ActT at, cudaStream_t s);
// att_txt = sum_w toutw[w] / divisor (divisor <= 0: the plain sum)
void awa_coalesce_div(const float* toutw, int nwin, int TXT, void* att_txt, int ld_att, ActT at, float divisor,
                      cudaStream_t s);
// dst rows (stride ld_dst) = src rows (stride ld_src), element gather/scatter of
// whole 2560-wide fp32 rows: dst[dst_idx[i]] = src[src_idx[i]] for i < n
// (a null index array means the identity).
void copy_rows_f32(const float* src, int ld_src, const int* src_idx, float* dst, int ld_dst, const int* dst_idx,
                   int n, int width, cudaStream_t s);

// ---------------------------------------------------------------- sharded exchanges over peer memory (k_shard.cu)
// Every rank's buffers, mapped into this rank (own entries are local).
struct ShardPeers {
    float* txtp[8] = {};          // [2 slots][TXT * 2560] txt partial sums
    uint32_t* flags[8] = {};      // [2 kinds][2 slots][world] ready flags
    float* x[2][8] = {};          // residual of each layout parity, [rows][2560]
    float* sr[8] = {};            // assembled [Lv][64] output
    int world = 1, rank = 0;
    uint64_t wait_ns = 4000000000ull;   // bound of every flag wait
};
// Publish this rank's partial of `layer`, wait for all ranks', write their
// rank-ordered sum / divisor to the TXT rows at out (stride ld).
void shard_txt_reduce(const ShardPeers& P, const uint32_t* epoch, int layer, int TXT, float divisor, void* out, int ld,
                      ActT t, cudaStream_t s);
// Rows src[k] of X[p] -> rows dst[k] of rank rank_of[k]'s X[1-p]; then flags
// and a wait until every rank's rows of this exchange have arrived.
void shard_exchange_rows(const ShardPeers& P, int p, const int* src, const int* rank_of, const int* dst, int n,
                         const uint32_t* epoch, int layer, cudaStream_t s);
// Rows k < n of sr_local (64 wide) -> row tok[k] of every rank's sr buffer;
// then flags and a wait until every rank's rows have arrived.
void shard_gather_sr(const ShardPeers& P, const float* sr_local, const int* tok, int n, const uint32_t* epoch,
                     cudaStream_t s);

// ---------------------------------------------------------------- grid / engine formats (k_engine.cu)
// (T, H, W, 33) -> (T*H/2*W/2, 132) and (T*H/2*W/2, 64) -> (T, H, W, 16), src/dit_vk.cpp:717-750.
void patchify_dev(const float* grid, int T, int H, int W, float* patch, cudaStream_t s);
void unpatchify_dev(const float* sr, int T, int H, int W, float* out, cudaStream_t s);
// vid_grid (H8, W8, 33) from channel-first noise and latent, src/seedvr2_engine.cpp:154-168.
void assemble_grid_dev(const float* noise, const float* latent, float scale, int H8, int W8, float* grid,
                       cudaStream_t s);
// z (16, H8, W8) = (noise - sr) / scale with sr channel-last (H8, W8, 16), src/seedvr2_engine.cpp:298-305.
void decode_latent_dev(const float* noise, const float* sr, float scale, int H8, int W8, float* z, cudaStream_t s);

}  // namespace s2b
