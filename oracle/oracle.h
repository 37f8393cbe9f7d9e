/* oracle.h -- CPU restatement of the reference NaDiT DiT / AWA path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the parity checker: tests/, the
 * smoke() entry and bench.py's cpu_baseline leg may call it; the product
 * never links, imports or falls back to it.
 *
 * Parity pinning: every function here is checked (tests/test_oracle_pin.py)
 * against the reference's own sources compiled unchanged into
 * oracle/_ref/libref_dit.so (src/dit_vk.cpp, src/awa_window.cpp,
 * src/test_awa_unit.cpp against a CPU ncnn stand-in) and against the golden
 * vectors in tests/golden/ that the same library produced.
 */
#ifndef S2B_ORACLE_H
#define S2B_ORACLE_H
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int t, h, w, nwin, txt_len;
    const int* sl6;      /* nwin x [t0,t1,h0,h1,w0,w1] */
    const float* vf;     /* sum(f_i) x 126 */
    const float* tf;     /* nwin x txt_len x 126 */
} or_win;

typedef struct or_model or_model;

/* src/awa_window.cpp:43-106; returns nwin (or -needed when cap is short). */
int or_make_windows(int t, int h, int w, int n0, int n1, int n2, int shifted, int* sl6, int cap);
/* src/awa_window.cpp:109-159 */
void or_build_freqs(const int* sl6, int nwin, int txt_len, float* vf, float* tf);
/* Attention core of src/dit_vk.cpp:345-455 (qk_norm with eps, RoPE,
 * per-window SDPA over [window vid | txt], txt mean, reverse partition). */
void or_awa(const float* vqkv, const float* tqkv, int Lv, int TXT, const or_win* win,
            const float* nqv, const float* nkv, const float* nqt, const float* nkt, float eps,
            float* vid_out, float* txt_out);
/* Operand rounding emulation for every later call (process-wide): 0 fp32
 * (the reference's arithmetic), 1 bf16, 2 fp16 -- GEMM operands and the
 * attention's q, k, v, p rounded to that type, arithmetic in fp32. */
void or_set_operand_rounding(int mode);
/* y[M,N] = x[M,K] W[N,K]^T + b (fp32 accumulate). */
void or_linear(const float* x, int M, int K, const float* W, int N, const float* b, float* y);

or_model* or_model_load(const char* m5_dir, int l0, int l1);
void or_model_free(or_model* m);
/* Last layer (31): 0 = forward_latent's vid_only semantics (txt unmodulated,
 * ungated, no txt MLP; src/dit_vk.cpp:523-623, the default); 1 = the chunked
 * graph's (export/export_dit_graph.py:155-226: txt like every other layer). */
void or_model_set_graph_last_layer(or_model* m, int on);
/* src/dit_vk.cpp:295-309 */
int or_time_embedding(or_model* m, float t, float* emb);
/* src/dit_vk.cpp:486-699 */
int or_forward_latent(or_model* m, const or_win* ns, const or_win* sh, const float* vid_in, int Lv,
                      const float* txt_in, int TXT, float t, int l0, int l1, int do_init, int do_final,
                      float* vid_lat, float* txt_lat, float* sr);
/* src/dit_vk.cpp:717-750 */
void or_patchify(const float* grid, int T, int H, int W, float* out);
void or_unpatchify(const float* lat, int T, int H, int W, float* out);

/* Seeded synthetic model and inputs (synth_oracle.c): the product's
 * generator restated, so CPU reference runs need no product library. */
#include <stdint.h>
void or_synth_normal(float* out, long n, uint64_t seed, const char* stream, float mean, float stdv);
int or_synth_write_m5(const char* dir, uint64_t seed, int lo, int hi);
void or_synth_vid_grid(float* grid, int T, int H, int W, uint64_t seed);
void or_synth_txt(float* txt, int TXT, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif
