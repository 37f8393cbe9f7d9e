/* oracle.c -- CPU restatement of the reference NaDiT DiT / AWA path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Each function cites the
 * reference lines it restates.  Arithmetic is fp32 like the reference
 * (RMSNorm sums squares in double as src/dit_vk.cpp:48-52 does); GEMMs
 * accumulate in fp32; softmax uses one max over the whole S x S block of a
 * (window, head) exactly as src/dit_vk.cpp:420-427.
 */
#define _GNU_SOURCE
#include "oracle.h"
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

enum { HEADS = 20, HEAD_D = 128, DIM = 2560, QKV = 7680, NUM_LAYERS = 32, MM_LAYERS = 10,
       MLP_DIM = 6912, ROPE_ROT = 126 };
static const float EPS = 1e-5f; /* src/dit_vk.cpp:17 */

static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

/* ------------------------------------------------------------ geometry */
static void extent(int t, int h, int w, int n0, int n1, int n2, int* wt, int* wh, int* ww) {
    double scale = sqrt((45.0 * 80.0) / ((double)h * w));   /* src/awa_window.cpp:49 */
    int rh = (int)round(h * scale), rw = (int)round(w * scale);
    *wh = (rh + n1 - 1) / n1;
    *ww = (rw + n2 - 1) / n2;
    *wt = (imin(t, 30) + n0 - 1) / n0;
}

int or_make_windows(int t, int h, int w, int n0, int n1, int n2, int shifted, int* sl6, int cap) {
    int wt, wh, ww, n = 0;
    extent(t, h, w, n0, n1, n2, &wt, &wh, &ww);
    if (!shifted) { /* src/awa_window.cpp:55-67 */
        int nt = (t + wt - 1) / wt, nh = (h + wh - 1) / wh, nw = (w + ww - 1) / ww;
        for (int iw = 0; iw < nw; iw++) {
            int w0 = iw * ww, w1 = imin((iw + 1) * ww, w);
            if (w1 <= w0) continue;
            for (int ih = 0; ih < nh; ih++) {
                int h0 = ih * wh, h1 = imin((ih + 1) * wh, h);
                if (h1 <= h0) continue;
                for (int it = 0; it < nt; it++) {
                    int t0 = it * wt, t1 = imin((it + 1) * wt, t);
                    if (t1 <= t0) continue;
                    if (n < cap) { int* s = sl6 + 6 * n; s[0]=t0; s[1]=t1; s[2]=h0; s[3]=h1; s[4]=w0; s[5]=w1; }
                    n++;
                }
            }
        }
    } else { /* src/awa_window.cpp:83-105 */
        double st = (wt < t) ? 0.5 : 0.0, sh = (wh < h) ? 0.5 : 0.0, sw = (ww < w) ? 0.5 : 0.0;
        int nt = (int)ceil((t - st) / wt), nh = (int)ceil((h - sh) / wh), nw = (int)ceil((w - sw) / ww);
        nt = (st > 0) ? nt + 1 : 1; nh = (sh > 0) ? nh + 1 : 1; nw = (sw > 0) ? nw + 1 : 1;
        for (int iw = 0; iw < nw; iw++) {
            int w0 = imax((int)((iw - sw) * ww), 0), w1 = imin((int)((iw - sw + 1) * ww), w);
            if (w1 <= w0) continue;
            for (int ih = 0; ih < nh; ih++) {
                int h0 = imax((int)((ih - sh) * wh), 0), h1 = imin((int)((ih - sh + 1) * wh), h);
                if (h1 <= h0) continue;
                for (int it = 0; it < nt; it++) {
                    int t0 = imax((int)((it - st) * wt), 0), t1 = imin((int)((it - st + 1) * wt), t);
                    if (t1 <= t0) continue;
                    if (n < cap) { int* s = sl6 + 6 * n; s[0]=t0; s[1]=t1; s[2]=h0; s[3]=h1; s[4]=w0; s[5]=w1; }
                    n++;
                }
            }
        }
    }
    return n <= cap ? n : -n;
}

void or_build_freqs(const int* sl6, int nwin, int txt_len, float* vf, float* tf) {
    double base[21];                                          /* src/awa_window.cpp:122-123 */
    for (int j = 0; j < 21; j++) base[j] = 1.0 / pow(10000.0, (double)(j * 2) / 42);
    size_t off = 0;
    for (int i = 0; i < nwin; i++) {                          /* :126-145 */
        const int* s = sl6 + 6 * i;
        for (int it = 0; it < s[1] - s[0]; it++)
            for (int ih = 0; ih < s[3] - s[2]; ih++)
                for (int iw = 0; iw < s[5] - s[4]; iw++)
                    for (int k = 0; k < 126; k++) {
                        double v;
                        if (k < 42) v = (double)(txt_len + it) * base[k / 2];
                        else if (k < 84) v = (double)ih * base[(k - 42) / 2];
                        else v = (double)iw * base[(k - 84) / 2];
                        vf[off++] = (float)v;
                    }
    }
    off = 0;
    for (int i = 0; i < nwin; i++)                            /* :148-158 */
        for (int p = 0; p < txt_len; p++)
            for (int k = 0; k < 126; k++) tf[off++] = (float)((double)p * base[(k % 42) / 2]);
}

/* ------------------------------------------------------------ small ops */
static void rmsnorm(const float* x, int n, const float* w, float* out, float eps) { /* src/dit_vk.cpp:48-52 */
    double s = 0;
    for (int i = 0; i < n; i++) s += (double)x[i] * x[i];
    float r = 1.0f / sqrtf((float)(s / n) + eps);
    for (int i = 0; i < n; i++) out[i] = x[i] * r * (w ? w[i] : 1.f);
}
static void qk_norm(const float* x, const float* w, float* out, float eps) { /* src/dit_vk.cpp:54-61 */
    for (int h = 0; h < HEADS; h++) {
        const float* xp = x + h * HEAD_D; float* op = out + h * HEAD_D;
        float sq = 0;
        for (int d = 0; d < HEAD_D; d++) sq += xp[d] * xp[d];
        float r = sqrtf(sq / HEAD_D + eps);
        for (int d = 0; d < HEAD_D; d++) op[d] = xp[d] / r * w[d];
    }
}
static void rope(const float* fr, const float* q, float* out) { /* src/dit_vk.cpp:62-71 */
    for (int k = 0; k < ROPE_ROT; k++) {
        float c = cosf(fr[k]), s = sinf(fr[k]);
        float rh = (k % 2 == 0) ? -q[k + 1] : q[k - 1];
        out[k] = q[k] * c + rh * s;
    }
    for (int k = ROPE_ROT; k < HEAD_D; k++) out[k] = q[k];
}

/* ------------------------------------------------------------ operand rounding (emulation) */
/* 0: fp32 (the reference).  1 / 2: every GEMM operand and every attention
 * operand (q, k, v, p) rounded to bf16 / fp16 (nearest even) before use, the
 * arithmetic itself fp32 -- an emulation of a reduced-precision operand path,
 * used to tell the rounding a bf16 path cannot avoid from errors of its own. */
static int g_round = 0;
void or_set_operand_rounding(int mode) { g_round = (mode == 1 || mode == 2) ? mode : 0; }

static float round_operand(float x) {
    if (g_round == 1) {
        uint32_t b; memcpy(&b, &x, 4);
        if ((b & 0x7F800000u) != 0x7F800000u) b = (b + 0x7FFFu + ((b >> 16) & 1u)) & 0xFFFF0000u;
        memcpy(&x, &b, 4);
        return x;
    }
    if (g_round == 2) return (float)(_Float16)x;
    return x;
}
static void round_rows(float* x, size_t n) {
    if (!g_round) return;
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < (long)n; i++) x[i] = round_operand(x[i]);
}

static void linear_f32(const float* x, int M, int K, const float* W, int N, const float* b, float* y);

void or_linear(const float* x, int M, int K, const float* W, int N, const float* b, float* y) {
    if (!g_round) { linear_f32(x, M, K, W, N, b, y); return; }
    float* xr = (float*)malloc(sizeof(float) * (size_t)M * K);
    float* wr = (float*)malloc(sizeof(float) * (size_t)N * K);
    memcpy(xr, x, sizeof(float) * (size_t)M * K);
    memcpy(wr, W, sizeof(float) * (size_t)N * K);
    round_rows(xr, (size_t)M * K);
    round_rows(wr, (size_t)N * K);
    linear_f32(xr, M, K, wr, N, b, y);
    free(xr); free(wr);
}

static void linear_f32(const float* x, int M, int K, const float* W, int N, const float* b, float* y) {
    /* ncnn InnerProduct semantics (src/dit_vk.cpp:270-293): y = x W^T + b, fp32. */
    const int MB = 4, NB = 64;
    const int mt = (M + MB - 1) / MB, nt = (N + NB - 1) / NB;
    #pragma omp parallel for schedule(dynamic, 2)
    for (long t = 0; t < (long)mt * nt; t++) {
        int m0 = (int)(t / nt) * MB, n0 = (int)(t % nt) * NB;
        int mr = imin(MB, M - m0), nr = imin(NB, N - n0);
        for (int r = 0; r < mr; r++) {
            const float* xr = x + (size_t)(m0 + r) * K;
            for (int j = 0; j < nr; j++) {
                const float* wr = W + (size_t)(n0 + j) * K;
                float a0 = 0, a1 = 0, a2 = 0, a3 = 0, a4 = 0, a5 = 0, a6 = 0, a7 = 0;
                int k = 0;
                for (; k + 8 <= K; k += 8) {
                    a0 += xr[k] * wr[k];         a1 += xr[k + 1] * wr[k + 1];
                    a2 += xr[k + 2] * wr[k + 2]; a3 += xr[k + 3] * wr[k + 3];
                    a4 += xr[k + 4] * wr[k + 4]; a5 += xr[k + 5] * wr[k + 5];
                    a6 += xr[k + 6] * wr[k + 6]; a7 += xr[k + 7] * wr[k + 7];
                }
                for (; k < K; k++) a0 += xr[k] * wr[k];
                y[(size_t)(m0 + r) * N + n0 + j] = ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7)) + (b ? b[n0 + j] : 0.f);
            }
        }
    }
}

/* ------------------------------------------------------------ attention */
void or_awa(const float* vqkv, const float* tqkv, int Lv, int TXT, const or_win* win,
            const float* nqv, const float* nkv, const float* nqt, const float* nkt, float eps,
            float* vid_out, float* txt_out) {
    const int nwin = win->nwin, H = win->h, Wd = win->w;
    int* cumf = (int*)calloc(nwin + 1, sizeof(int));
    for (int wi = 0; wi < nwin; wi++) {                       /* src/dit_vk.cpp:360-364 */
        const int* s = win->sl6 + 6 * wi;
        cumf[wi + 1] = cumf[wi] + (s[1] - s[0]) * (s[3] - s[2]) * (s[5] - s[4]);
    }
    const int sumf = cumf[nwin];
    int* vidx = (int*)malloc(sizeof(int) * (sumf > 0 ? sumf : 1));
    for (int wi = 0, g = 0; wi < nwin; wi++) {                /* partition order :367-378 */
        const int* s = win->sl6 + 6 * wi;
        for (int lt = s[0]; lt < s[1]; lt++)
            for (int lh = s[2]; lh < s[3]; lh++)
                for (int lw = s[4]; lw < s[5]; lw++) vidx[g++] = ((lt * H) + lh) * Wd + lw;
    }
    float* tout_win = (float*)calloc((size_t)nwin * TXT * DIM, sizeof(float));
    memset(vid_out, 0, sizeof(float) * (size_t)Lv * DIM);    /* uncovered tokens stay 0 (:445) */
    const float scale = 1.0f / sqrtf((float)HEAD_D);
    #pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int wi = 0; wi < nwin; wi++)
        for (int hh = 0; hh < HEADS; hh++) {
            const int f = cumf[wi + 1] - cumf[wi], S = f + TXT;
            float* q = (float*)malloc(sizeof(float) * (size_t)S * HEAD_D);
            float* k = (float*)malloc(sizeof(float) * (size_t)S * HEAD_D);
            float* v = (float*)malloc(sizeof(float) * (size_t)S * HEAD_D);
            float* sc = (float*)malloc(sizeof(float) * (size_t)S * S);
            float* p = (float*)malloc(sizeof(float) * (size_t)S);
            float nrm[HEAD_D];
            for (int a = 0; a < S; a++) {
                const float* row; const float* fr; const float *wq, *wk;
                if (a < f) { row = vqkv + (size_t)vidx[cumf[wi] + a] * QKV; fr = win->vf + (size_t)(cumf[wi] + a) * ROPE_ROT; wq = nqv; wk = nkv; }
                else { row = tqkv + (size_t)(a - f) * QKV; fr = win->tf + (size_t)(wi * TXT + a - f) * ROPE_ROT; wq = nqt; wk = nkt; }
                /* qk_norm is per head, so norming only head hh equals slicing the full qk_norm */
                {
                    const float* xp = row + hh * HEAD_D; float sq = 0;
                    for (int d = 0; d < HEAD_D; d++) sq += xp[d] * xp[d];
                    float r = sqrtf(sq / HEAD_D + eps);
                    for (int d = 0; d < HEAD_D; d++) nrm[d] = xp[d] / r * wq[d];
                    rope(fr, nrm, q + (size_t)a * HEAD_D);
                }
                {
                    const float* xp = row + DIM + hh * HEAD_D; float sq = 0;
                    for (int d = 0; d < HEAD_D; d++) sq += xp[d] * xp[d];
                    float r = sqrtf(sq / HEAD_D + eps);
                    for (int d = 0; d < HEAD_D; d++) nrm[d] = xp[d] / r * wk[d];
                    rope(fr, nrm, k + (size_t)a * HEAD_D);
                }
                memcpy(v + (size_t)a * HEAD_D, row + 2 * DIM + hh * HEAD_D, HEAD_D * sizeof(float));
                if (g_round)
                    for (int d = 0; d < HEAD_D; d++) {
                        q[(size_t)a * HEAD_D + d] = round_operand(q[(size_t)a * HEAD_D + d]);
                        k[(size_t)a * HEAD_D + d] = round_operand(k[(size_t)a * HEAD_D + d]);
                        v[(size_t)a * HEAD_D + d] = round_operand(v[(size_t)a * HEAD_D + d]);
                    }
            }
            float mx = -1e30f;                                 /* :420-428 */
            for (int a = 0; a < S; a++)
                for (int b = 0; b < S; b++) {
                    float dot = 0;
                    for (int d = 0; d < HEAD_D; d++) dot += q[(size_t)a * HEAD_D + d] * k[(size_t)b * HEAD_D + d];
                    dot *= scale; sc[(size_t)a * S + b] = dot; if (dot > mx) mx = dot;
                }
            for (int a = 0; a < S; a++) {                      /* :429-437 */
                float sm = 0, o[HEAD_D];
                for (int b = 0; b < S; b++) { float e = expf(sc[(size_t)a * S + b] - mx); p[b] = e; sm += e; }
                for (int b = 0; b < S; b++) p[b] = round_operand(p[b] / sm);
                for (int d = 0; d < HEAD_D; d++) o[d] = 0;
                for (int b = 0; b < S; b++) for (int d = 0; d < HEAD_D; d++) o[d] += p[b] * v[(size_t)b * HEAD_D + d];
                if (a < f) memcpy(vid_out + (size_t)vidx[cumf[wi] + a] * DIM + hh * HEAD_D, o, sizeof o);
                else memcpy(tout_win + ((size_t)(wi * TXT + a - f)) * DIM + hh * HEAD_D, o, sizeof o);
            }
            free(q); free(k); free(v); free(sc); free(p);
        }
    memset(txt_out, 0, sizeof(float) * (size_t)TXT * DIM);    /* txt mean over windows :440-444 */
    for (int wi = 0; wi < nwin; wi++)
        for (size_t i = 0; i < (size_t)TXT * DIM; i++) txt_out[i] += tout_win[(size_t)wi * TXT * DIM + i];
    for (size_t i = 0; i < (size_t)TXT * DIM; i++) txt_out[i] /= (float)nwin;
    free(tout_win); free(vidx); free(cumf);
}

/* ------------------------------------------------------------ model */
typedef struct { int out, in; float* W; float* b; } lin_t;
typedef struct { float *nq, *nk, *a_shift, *a_scale, *a_gate, *m_shift, *m_scale, *m_gate; } branch_t;
typedef struct { lin_t qkv, out, mlp_in, mlp_g, mlp_out; int loaded; } block_t;
struct or_model {
    char dir[1024];
    lin_t vid_in, txt_in, emb_in, emb_hid, emb_out, vid_out;
    float *von_w, *voa_shift, *voa_scale;
    branch_t br[NUM_LAYERS][2];
    block_t blk[NUM_LAYERS][2];   /* [i][0]=vid or all, [i][1]=txt or all (aliases for shared) */
    int graph_last;               /* last layer with the chunked graph's txt semantics */
};

void or_model_set_graph_last_layer(or_model* m, int on) { if (m) m->graph_last = on != 0; }

static float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff, f;
    if (e == 0) {
        if (!m) f = sign;
        else { int ee = 113; while (!(m & 0x400)) { m <<= 1; ee--; } f = sign | ((uint32_t)ee << 23) | ((m & 0x3ff) << 13); }
    } else if (e == 31) f = sign | 0x7f800000u | (m << 13);
    else f = sign | ((e + 112) << 23) | (m << 13);
    float o; memcpy(&o, &f, 4); return o;
}

static int load_linear(const char* dir, const char* base, lin_t* L) {
    char path[1200]; int nout = 0, bias = 0, wsz = 0;
    snprintf(path, sizeof path, "%s/%s.param", dir, base);
    FILE* f = fopen(path, "r");
    if (!f) { fprintf(stderr, "[oracle] missing %s\n", path); return -1; }
    char line[1024];
    while (fgets(line, sizeof line, f)) {
        if (!strstr(line, "InnerProduct")) continue;
        char* tok = strtok(line, " \t\n");
        while (tok) {
            if (!strncmp(tok, "0=", 2)) nout = atoi(tok + 2);
            else if (!strncmp(tok, "1=", 2)) bias = atoi(tok + 2);
            else if (!strncmp(tok, "2=", 2)) wsz = atoi(tok + 2);
            tok = strtok(NULL, " \t\n");
        }
    }
    fclose(f);
    if (nout <= 0 || wsz % nout) return -1;
    L->out = nout; L->in = wsz / nout;
    snprintf(path, sizeof path, "%s/%s.bin", dir, base);
    f = fopen(path, "rb");
    if (!f) { fprintf(stderr, "[oracle] missing %s\n", path); return -1; }
    uint32_t tag = 0;
    if (fread(&tag, 4, 1, f) != 1) { fclose(f); return -1; }
    L->W = (float*)malloc(sizeof(float) * (size_t)wsz);
    if (tag == 0x01306B47u) {
        uint16_t* hb = (uint16_t*)malloc(2 * (size_t)wsz);
        if (fread(hb, 2, wsz, f) != (size_t)wsz) { free(hb); fclose(f); return -1; }
        for (size_t i = 0; i < (size_t)wsz; i++) L->W[i] = h2f(hb[i]);
        free(hb);
    } else if (fread(L->W, 4, wsz, f) != (size_t)wsz) { fclose(f); return -1; }
    L->b = NULL;
    if (bias) {
        L->b = (float*)malloc(sizeof(float) * nout);
        if (fread(L->b, 4, nout, f) != (size_t)nout) { fclose(f); return -1; }
    }
    fclose(f);
    return 0;
}
static void free_linear(lin_t* L) { free(L->W); free(L->b); L->W = L->b = NULL; }

static float* load_raw(const char* dir, const char* base) { /* src/dit_vk.cpp:38-45 */
    char path[1200]; snprintf(path, sizeof path, "%s/%s.bin", dir, base);
    FILE* f = fopen(path, "rb");
    if (!f) { fprintf(stderr, "[oracle] missing %s\n", path); return NULL; }
    int64_t nd = 0, total = 1;
    if (fread(&nd, 8, 1, f) != 1) { fclose(f); return NULL; }
    for (int64_t i = 0; i < nd; i++) { int64_t d; if (fread(&d, 8, 1, f) != 1) { fclose(f); return NULL; } total *= d; }
    float* v = (float*)malloc(sizeof(float) * (size_t)total);
    if (fread(v, 4, total, f) != (size_t)total) { free(v); fclose(f); return NULL; }
    fclose(f);
    return v;
}

or_model* or_model_load(const char* dir, int l0, int l1) {
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    snprintf(m->dir, sizeof m->dir, "%s", dir);
    int bad = 0;
    bad |= load_linear(dir, "vid_in_proj", &m->vid_in);
    bad |= load_linear(dir, "txt_in", &m->txt_in);
    bad |= load_linear(dir, "emb_proj_in", &m->emb_in);
    bad |= load_linear(dir, "emb_proj_hid", &m->emb_hid);
    bad |= load_linear(dir, "emb_proj_out", &m->emb_out);
    bad |= load_linear(dir, "vid_out_proj", &m->vid_out);
    m->von_w = load_raw(dir, "vid_out_norm_w");
    m->voa_shift = load_raw(dir, "vid_out_ada_shift");
    m->voa_scale = load_raw(dir, "vid_out_ada_scale");
    static const char* names[8] = {"nq", "nk", "attn_shift", "attn_scale", "attn_gate", "mlp_shift", "mlp_scale", "mlp_gate"};
    for (int i = 0; i < NUM_LAYERS; i++)                     /* src/dit_vk.cpp:161-177 */
        for (int fl = 0; fl < 2; fl++) {
            char base[256];
            const char* tag = (i < MM_LAYERS) ? (fl == 0 ? "vid" : "txt") : "all";
            float** dst[8] = {&m->br[i][fl].nq, &m->br[i][fl].nk, &m->br[i][fl].a_shift, &m->br[i][fl].a_scale,
                              &m->br[i][fl].a_gate, &m->br[i][fl].m_shift, &m->br[i][fl].m_scale, &m->br[i][fl].m_gate};
            for (int k = 0; k < 8; k++) {
                snprintf(base, sizeof base, "b%d_%s_%s", i, tag, names[k]);
                *dst[k] = load_raw(dir, base);
                if (!*dst[k]) bad = 1;
            }
        }
    for (int i = imax(l0, 0); i < imin(l1, NUM_LAYERS); i++)
        for (int fl = 0; fl < (i < MM_LAYERS ? 2 : 1); fl++) {
            const char* tag = (i < MM_LAYERS) ? (fl == 0 ? "vid" : "txt") : "all";
            char base[256]; block_t* B = &m->blk[i][fl];
            snprintf(base, sizeof base, "b%d_%s_qkv", i, tag); bad |= load_linear(dir, base, &B->qkv);
            snprintf(base, sizeof base, "b%d_%s_out", i, tag); bad |= load_linear(dir, base, &B->out);
            snprintf(base, sizeof base, "b%d_%s_mlp_in", i, tag); bad |= load_linear(dir, base, &B->mlp_in);
            snprintf(base, sizeof base, "b%d_%s_mlp_g", i, tag); bad |= load_linear(dir, base, &B->mlp_g);
            snprintf(base, sizeof base, "b%d_%s_mlp_out", i, tag); bad |= load_linear(dir, base, &B->mlp_out);
            B->loaded = 1;
            if (i >= MM_LAYERS) m->blk[i][1] = *B;
        }
    if (bad || !m->von_w || !m->voa_shift || !m->voa_scale) { or_model_free(m); return NULL; }
    return m;
}

void or_model_free(or_model* m) {
    if (!m) return;
    free_linear(&m->vid_in); free_linear(&m->txt_in); free_linear(&m->emb_in);
    free_linear(&m->emb_hid); free_linear(&m->emb_out); free_linear(&m->vid_out);
    free(m->von_w); free(m->voa_shift); free(m->voa_scale);
    for (int i = 0; i < NUM_LAYERS; i++) {
        for (int fl = 0; fl < 2; fl++) {
            branch_t* b = &m->br[i][fl];
            free(b->nq); free(b->nk); free(b->a_shift); free(b->a_scale); free(b->a_gate);
            free(b->m_shift); free(b->m_scale); free(b->m_gate);
        }
        if (m->blk[i][0].loaded) {
            block_t* B = &m->blk[i][0];
            free_linear(&B->qkv); free_linear(&B->out); free_linear(&B->mlp_in); free_linear(&B->mlp_g); free_linear(&B->mlp_out);
        }
        if (i < MM_LAYERS && m->blk[i][1].loaded) {
            block_t* B = &m->blk[i][1];
            free_linear(&B->qkv); free_linear(&B->out); free_linear(&B->mlp_in); free_linear(&B->mlp_g); free_linear(&B->mlp_out);
        }
    }
    free(m);
}

static void silu_inplace(float* x, int n) { for (int i = 0; i < n; i++) x[i] = x[i] / (1.f + expf(-x[i])); }

int or_time_embedding(or_model* m, float t, float* emb) {    /* src/dit_vk.cpp:295-309 */
    float e[256], h1[DIM], h2[DIM];
    const int half = 128;
    for (int j = 0; j < 256; j++) {
        float freq = (j < half) ? (float)exp(-logf(10000.f) * j / half) : (float)exp(-logf(10000.f) * (j - half) / half);
        e[j] = (j < half) ? sinf(t * freq) : cosf(t * freq);
    }
    /* the timestep MLP stays fp32 in every operand mode (the product keeps it fp32) */
    linear_f32(e, 1, 256, m->emb_in.W, DIM, m->emb_in.b, h1); silu_inplace(h1, DIM);
    linear_f32(h1, 1, DIM, m->emb_hid.W, DIM, m->emb_hid.b, h2); silu_inplace(h2, DIM);
    linear_f32(h2, 1, DIM, m->emb_out.W, 6 * DIM, m->emb_out.b, emb);
    return 0;
}

/* norm + adaLN modulate of rows: y = rms(x) * (emb[6d+ks] + sc[d]) + (emb[6d+kh] + sh[d]) */
static void norm_mod(const float* x, int rows, const float* emb, int ks, int kh, const float* sc, const float* sh,
                     int modulate, float* y) {
    #pragma omp parallel for
    for (int t = 0; t < rows; t++) {
        rmsnorm(x + (size_t)t * DIM, DIM, NULL, y + (size_t)t * DIM, EPS);
        if (modulate)
            for (int d = 0; d < DIM; d++)
                y[(size_t)t * DIM + d] = y[(size_t)t * DIM + d] * (emb[d * 6 + ks] + sc[d]) + (emb[d * 6 + kh] + sh[d]);
    }
}

static void swiglu(const block_t* B, const float* x, int n, float* out) { /* src/dit_vk.cpp:465-472 */
    float* h = (float*)malloc(sizeof(float) * (size_t)n * MLP_DIM);
    float* g = (float*)malloc(sizeof(float) * (size_t)n * MLP_DIM);
    or_linear(x, n, DIM, B->mlp_in.W, MLP_DIM, NULL, h);
    or_linear(x, n, DIM, B->mlp_g.W, MLP_DIM, NULL, g);
    for (size_t k = 0; k < (size_t)n * MLP_DIM; k++) g[k] = (g[k] / (1.f + expf(-g[k]))) * h[k];
    or_linear(g, n, MLP_DIM, B->mlp_out.W, DIM, NULL, out);
    free(h); free(g);
}

int or_forward_latent(or_model* m, const or_win* ns, const or_win* shw, const float* vid_in, int Lv,
                      const float* txt_in, int TXT, float t, int l0, int l1, int do_init, int do_final,
                      float* vid_lat, float* txt_lat, float* sr) {
    const size_t nv = (size_t)Lv * DIM, nt = (size_t)TXT * DIM;
    float* vid = (float*)malloc(sizeof(float) * nv);
    float* txt = (float*)malloc(sizeof(float) * nt);
    if (do_init) {                                            /* :494-497 */
        or_linear(vid_in, Lv, 132, m->vid_in.W, DIM, m->vid_in.b, vid);
        or_linear(txt_in, TXT, 5120, m->txt_in.W, DIM, m->txt_in.b, txt);
    } else { memcpy(vid, vid_in, sizeof(float) * nv); memcpy(txt, txt_in, sizeof(float) * nt); }
    float emb[6 * DIM];
    or_time_embedding(m, t, emb);                             /* :511 */
    float* van = (float*)malloc(sizeof(float) * nv);
    float* tan_ = (float*)malloc(sizeof(float) * nt);
    float* vqkv = (float*)malloc(sizeof(float) * (size_t)Lv * QKV);
    float* tqkv = (float*)malloc(sizeof(float) * (size_t)TXT * QKV);
    float* vat = (float*)malloc(sizeof(float) * nv);
    float* tat = (float*)malloc(sizeof(float) * nt);
    float* vo = (float*)malloc(sizeof(float) * nv);
    float* to = (float*)malloc(sizeof(float) * nt);
    int rc = 0;
    for (int i = l0; i < imin(l1, NUM_LAYERS); i++) {         /* :517-655 */
        const or_win* win = (i % 2 == 0) ? ns : shw;
        const branch_t* vR = &m->br[i][0]; const branch_t* tR = &m->br[i][1];
        const block_t* bv = &m->blk[i][0]; const block_t* bt = &m->blk[i][1];
        if (!bv->loaded) { rc = -1; break; }
        /* forward_latent's vid_only last layer (:523-525); with graph_last the
         * chunked graph's semantics (export/export_dit_graph.py:155-226): txt
         * is modulated, gated and runs its MLP in every layer */
        const int last = (i == NUM_LAYERS - 1) && !m->graph_last;
        norm_mod(vid, Lv, emb, 1, 0, vR->a_scale, vR->a_shift, 1, van);          /* :529-537 */
        norm_mod(txt, TXT, emb, 1, 0, tR->a_scale, tR->a_shift, !last, tan_);    /* :538-545 */
        or_linear(van, Lv, DIM, bv->qkv.W, QKV, NULL, vqkv);                    /* :321-322 */
        or_linear(tan_, TXT, DIM, bt->qkv.W, QKV, NULL, tqkv);
        or_awa(vqkv, tqkv, Lv, TXT, win, vR->nq, vR->nk, tR->nq, tR->nk, EPS, vat, tat);
        or_linear(vat, Lv, DIM, bv->out.W, DIM, bv->out.b, vo);                 /* :461-462 */
        or_linear(tat, TXT, DIM, bt->out.W, DIM, bt->out.b, to);
        for (size_t k = 0; k < nv; k++) { int d = (int)(k % DIM); vo[k] *= (emb[d * 6 + 2] + vR->a_gate[d]); }  /* :558-559 */
        if (!last) for (size_t k = 0; k < nt; k++) { int d = (int)(k % DIM); to[k] *= (emb[d * 6 + 2] + tR->a_gate[d]); }
        for (size_t k = 0; k < nv; k++) vid[k] = vo[k] + vid[k];                /* :574-575 */
        for (size_t k = 0; k < nt; k++) txt[k] = to[k] + txt[k];
        norm_mod(vid, Lv, emb, 4, 3, vR->m_scale, vR->m_shift, 1, van);         /* :577-589 */
        if (!last) norm_mod(txt, TXT, emb, 4, 3, tR->m_scale, tR->m_shift, 1, tan_);
        swiglu(bv, van, Lv, vo);                                                 /* :608 */
        for (size_t k = 0; k < nv; k++) { int d = (int)(k % DIM); vo[k] *= (emb[d * 6 + 5] + vR->m_gate[d]); }  /* :615-616 */
        for (size_t k = 0; k < nv; k++) vid[k] = vo[k] + vid[k];                /* :631 */
        if (!last) {                                                             /* :610-620, 632 */
            swiglu(bt, tan_, TXT, to);
            for (size_t k = 0; k < nt; k++) { int d = (int)(k % DIM); to[k] *= (emb[d * 6 + 5] + tR->m_gate[d]); }
            for (size_t k = 0; k < nt; k++) txt[k] = to[k] + txt[k];
        }
    }
    if (rc == 0) {
        if (do_final) {                                       /* :657-675 */
            #pragma omp parallel for
            for (int r = 0; r < Lv; r++) {
                float* y = van + (size_t)r * DIM;
                rmsnorm(vid + (size_t)r * DIM, DIM, m->von_w, y, EPS);
                for (int d = 0; d < DIM; d++) y[d] = y[d] * (emb[d * 6 + 1] + m->voa_scale[d]) + (emb[d * 6 + 0] + m->voa_shift[d]);
            }
            or_linear(van, Lv, DIM, m->vid_out.W, 64, m->vid_out.b, sr);
        } else {
            if (vid_lat) memcpy(vid_lat, vid, sizeof(float) * nv);
            if (txt_lat) memcpy(txt_lat, txt, sizeof(float) * nt);
        }
    }
    free(vid); free(txt); free(van); free(tan_); free(vqkv); free(tqkv); free(vat); free(tat); free(vo); free(to);
    return rc;
}

void or_patchify(const float* grid, int T, int H, int W, float* out) { /* src/dit_vk.cpp:717-733 */
    int H2 = H / 2, W2 = W / 2;
    for (int t = 0; t < T; t++) for (int hh = 0; hh < H2; hh++) for (int ww = 0; ww < W2; ww++)
        for (int ph = 0; ph < 2; ph++) for (int pw = 0; pw < 2; pw++) for (int c = 0; c < 33; c++)
            out[((size_t)(t * H2 + hh) * W2 + ww) * 132 + (ph * 2 + pw) * 33 + c] =
                grid[((size_t)(t * H + hh * 2 + ph) * W + (ww * 2 + pw)) * 33 + c];
}
void or_unpatchify(const float* lat, int T, int H, int W, float* out) { /* src/dit_vk.cpp:735-750 */
    int H2 = H / 2, W2 = W / 2;
    memset(out, 0, sizeof(float) * (size_t)T * H * W * 16);
    for (int t = 0; t < T; t++) for (int hh = 0; hh < H2; hh++) for (int ww = 0; ww < W2; ww++)
        for (int ph = 0; ph < 2; ph++) for (int pw = 0; pw < 2; pw++) for (int c = 0; c < 16; c++)
            out[((size_t)(t * H + hh * 2 + ph) * W + (ww * 2 + pw)) * 16 + c] =
                lat[((size_t)(t * H2 + hh) * W2 + ww) * 64 + (ph * 2 + pw) * 16 + c];
}
