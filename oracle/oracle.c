/* oracle.c -- CPU restatement of the cohere-transcribe reference (checker only).
 *
 * TEST INFRASTRUCTURE: loaded by tests/, __graft_entry__.smoke() and bench.py's
 * CPU legs, never by libct_b200.so.  See oracle.h for the contract.
 *
 * Arithmetic order follows the reference CPU backend statement by statement
 * (sequential fp32 sums, the same expression shapes, libm expf/sqrtf/sinf/cosf)
 * so that, compiled with the same flags, results are bit-identical to
 * backends/cpu/backend.c.  Independent outputs are spread over OpenMP threads;
 * each output is still produced by one thread in the reference order.
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define XMALLOC(n) xmalloc_((size_t)(n))
static void *xmalloc_(size_t bytes) {
    void *p = malloc(bytes ? bytes : 1);
    if (!p) { fputs("oracle: out of memory\n", stderr); abort(); }
    return p;
}

void orc_dims_full(ct_dims *d) {
    /* backends/model_types.h:14-30 */
    d->enc_d = 1280; d->enc_ff = 5120; d->enc_h = 8; d->enc_dk = 160; d->enc_n = 48;
    d->enc_ck = 9; d->sub_ch = 256;
    d->dec_d = 1024; d->dec_ff = 4096; d->dec_h = 8; d->dec_dk = 128; d->dec_n = 8;
    d->vocab = 16384; d->max_seq = 1024; d->n_mels = 128;
}

/* bf16 -> fp32 widening, backends/model_types.h:42-47 */
static inline float bf16_widen(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
float orc_bf16(uint16_t b) { return bf16_widen(b); }
#define BF(x) bf16_widen(x)

/* ------------------------------------------------------------------ */
/* primitives                                                          */
/* ------------------------------------------------------------------ */

/* backends/cpu/backend.c:109-122 -- eps 1e-5, biased variance. */
void orc_layernorm(float *dst, const float *src, const uint16_t *w, const uint16_t *b, int T, int D) {
    const float eps = 1e-5f;
    #pragma omp parallel for schedule(static) if (T > 8)
    for (int t = 0; t < T; t++) {
        const float *row = src + (size_t)t * D;
        float *out = dst + (size_t)t * D;
        float mean = 0, var = 0;
        for (int i = 0; i < D; i++) mean += row[i];
        mean /= D;
        for (int i = 0; i < D; i++) { float c = row[i] - mean; var += c * c; }
        float inv = 1.0f / sqrtf(var / D + eps);
        for (int i = 0; i < D; i++) out[i] = (row[i]-mean)*inv*BF(w[i]) + BF(b[i]);
    }
}

/* backends/cpu/backend.c:124-182: one sequential dot product per output,
 * seeded with the bias; epilogue store / SiLU / ReLU / acc += scale*s. */
void orc_linear(float *y, const float *x, const uint16_t *W, const uint16_t *b,
                int T, int in_d, int out_d, int ep, float scale) {
    #pragma omp parallel for collapse(2) schedule(static) if ((long)T * out_d > 4096)
    for (int t = 0; t < T; t++) {
        for (int j = 0; j < out_d; j++) {
            const float *xr = x + (size_t)t * in_d;
            const uint16_t *wr = W + (size_t)j * in_d;
            float s = b ? BF(b[j]) : 0.0f;
            for (int k = 0; k < in_d; k++) s += xr[k] * BF(wr[k]);
            float *yo = y + (size_t)t * out_d + j;
            switch (ep) {
            case ORC_EP_SILU:  *yo = s / (1.0f + expf(-s)); break;
            case ORC_EP_RELU:  *yo = s > 0.0f ? s : 0.0f; break;
            case ORC_EP_FMADD: *yo += scale * s; break;
            default:           *yo = s; break;
            }
        }
    }
}

/* backends/cpu/backend.c:184-186 */
void orc_add_inplace(float *dst, const float *src, int n) {
    for (int i = 0; i < n; i++) dst[i] += src[i];
}

/* backends/cpu/backend.c:75-103: grouped 2-D convolution, NCHW, zero padding. */
static void conv2d(float *out, const float *in, const uint16_t *Wf, const uint16_t *bf,
                   int in_c, int in_h, int in_w, int out_c, int kH, int kW,
                   int stride, int pad, int groups) {
    const int out_h = (in_h + 2*pad - kH) / stride + 1;
    const int out_w = (in_w + 2*pad - kW) / stride + 1;
    const int icg = in_c / groups, ocg = out_c / groups;
    #pragma omp parallel for schedule(static)
    for (int oc = 0; oc < out_c; oc++) {
        const int g = oc / ocg;
        for (int oh = 0; oh < out_h; oh++)
        for (int ow = 0; ow < out_w; ow++) {
            float s = bf ? BF(bf[oc]) : 0.0f;
            for (int ic = 0; ic < icg; ic++) {
                const int icx = g*icg + ic;
                for (int kh = 0; kh < kH; kh++) {
                    const int ih = oh*stride - pad + kh;
                    if (ih < 0 || ih >= in_h) continue;
                    for (int kw = 0; kw < kW; kw++) {
                        const int iw = ow*stride - pad + kw;
                        if (iw < 0 || iw >= in_w) continue;
                        s += in[icx*(in_h*in_w) + ih*in_w + iw]
                           * BF(Wf[(oc*icg + ic)*kH*kW + kh*kW + kw]);
                    }
                }
            }
            out[oc*(out_h*out_w) + oh*out_w + ow] = s;
        }
    }
}

static void relu_inplace(float *x, size_t n) {
    for (size_t i = 0; i < n; i++) if (x[i] < 0.0f) x[i] = 0.0f;
}

/* backends/cpu/backend.c:188-229: 8x time/frequency subsampling.
 * conv0 3x3/s2 (1->C) + ReLU, dw 3x3/s2, pw 1x1 + ReLU, dw 3x3/s2, pw 1x1 + ReLU,
 * flatten to [T_enc, C*F3] (channel-major inside a row), linear C*F3 -> enc_d. */
void orc_encoder_subsampling(const ct_dims *d, const float *mel, int T_mel, int T_mel_stride,
                             float *x_enc, int T_enc, const Weights *W) {
    const int C = d->sub_ch;
    const int F0 = d->n_mels, F1 = (F0 + 1) / 2, F2 = (F1 + 1) / 2, F3 = (F2 + 1) / 2;
    const int T1 = (T_mel + 1) / 2, T2 = (T1 + 1) / 2;
    float *mel_t = XMALLOC(sizeof(float) * (size_t)T_mel * F0);
    float *a = XMALLOC(sizeof(float) * (size_t)C * T1 * F1);
    float *bb = XMALLOC(sizeof(float) * (size_t)C * T1 * F1);
    for (int t = 0; t < T_mel; t++)
        for (int m = 0; m < F0; m++)
            mel_t[(size_t)t * F0 + m] = mel[(size_t)m * T_mel_stride + t];
    conv2d(a, mel_t, W->s0w, W->s0b, 1, T_mel, F0, C, 3, 3, 2, 1, 1);
    relu_inplace(a, (size_t)C * T1 * F1);
    conv2d(bb, a, W->s2w, W->s2b, C, T1, F1, C, 3, 3, 2, 1, C);
    conv2d(a, bb, W->s3w, W->s3b, C, T2, F2, C, 1, 1, 1, 0, 1);
    relu_inplace(a, (size_t)C * T2 * F2);
    conv2d(bb, a, W->s5w, W->s5b, C, T2, F2, C, 3, 3, 2, 1, C);
    conv2d(a, bb, W->s6w, W->s6b, C, T_enc, F3, C, 1, 1, 1, 0, 1);
    relu_inplace(a, (size_t)C * T_enc * F3);
    const int feat = C * F3;
    float *flat = XMALLOC(sizeof(float) * (size_t)T_enc * feat);
    for (int t = 0; t < T_enc; t++)
        for (int c = 0; c < C; c++)
            for (int f = 0; f < F3; f++)
                flat[(size_t)t * feat + c * F3 + f] = a[((size_t)c * T_enc + t) * F3 + f];
    orc_linear(x_enc, flat, W->sow, W->sob, T_enc, feat, d->enc_d, ORC_EP_STORE, 0.0f);
    free(flat); free(a); free(bb); free(mel_t);
}

/* backends/cpu/backend.c:231-242: row p encodes relative position T-1-p;
 * even columns sin, odd columns cos, frequency 10000^(-2k/enc_d). */
void orc_make_rel_pos_emb(const ct_dims *d, float *pe, int T) {
    const int D = d->enc_d, L = 2 * T - 1;
    const float log10k = logf(10000.0f);
    for (int p = 0; p < L; p++) {
        const float pos = (float)(T - 1 - p);
        for (int k = 0; k < D / 2; k++) {
            const float freq = expf(-(float)(2*k) * log10k / D);
            pe[(size_t)p * D + 2*k]     = sinf(pos * freq);
            pe[(size_t)p * D + 2*k + 1] = cosf(pos * freq);
        }
    }
}

/* backends/cpu/backend.c:67-73 */
static void softmax_row(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float s = 0;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); s += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= s;
}

/* backends/cpu/backend.c:244-298: Transformer-XL style relative attention.
 * score[q,k] = ((Q+u)·K[k] + (Q+v)·P[k+T-1-q]) / sqrt(dk), softmax over k,
 * weighted sum of V, output projection.  P = pos_emb · W_pos (no bias). */
void orc_rel_pos_mhsa(const ct_dims *d, float *x, const float *pos_emb, int T, const ELayer *L) {
    const int D = d->enc_d, H = d->enc_h, DK = d->enc_dk, PL = 2 * T - 1;
    float *Q = XMALLOC(sizeof(float) * (size_t)T * D);
    float *K = XMALLOC(sizeof(float) * (size_t)T * D);
    float *V = XMALLOC(sizeof(float) * (size_t)T * D);
    float *P = XMALLOC(sizeof(float) * (size_t)PL * D);
    float *att = XMALLOC(sizeof(float) * (size_t)T * D);
    orc_linear(Q, x, L->sa_qw, L->sa_qb, T, D, D, ORC_EP_STORE, 0.f);
    orc_linear(K, x, L->sa_kw, L->sa_kb, T, D, D, ORC_EP_STORE, 0.f);
    orc_linear(V, x, L->sa_vw, L->sa_vb, T, D, D, ORC_EP_STORE, 0.f);
    orc_linear(P, pos_emb, L->sa_pw, NULL, PL, D, D, ORC_EP_STORE, 0.f);
    const float scale = 1.0f / sqrtf((float)DK);
    #pragma omp parallel
    {
        float *sc = XMALLOC(sizeof(float) * (size_t)T);
        float *bd = XMALLOC(sizeof(float) * (size_t)PL);
        #pragma omp for collapse(2) schedule(static)
        for (int h = 0; h < H; h++)
        for (int q = 0; q < T; q++) {
            const float *qr = Q + (size_t)q * D + h * DK;
            for (int k = 0; k < T; k++) {
                float s = 0;
                for (int i = 0; i < DK; i++)
                    s += (qr[i] + BF(L->sa_pbu[h*DK + i])) * K[(size_t)k * D + h * DK + i];
                sc[k] = s * scale;
            }
            /* only the P rows k+T-1-q for k in [0,T) are used: p in [T-1-q, 2T-2-q] */
            for (int p = T - 1 - q; p <= 2 * T - 2 - q; p++) {
                float s = 0;
                for (int i = 0; i < DK; i++)
                    s += (qr[i] + BF(L->sa_pbv[h*DK + i])) * P[(size_t)p * D + h * DK + i];
                bd[p] = s;
            }
            for (int k = 0; k < T; k++) sc[k] += bd[k + (T - 1) - q] * scale;
            softmax_row(sc, T);
            for (int i = 0; i < DK; i++) {
                float s = 0;
                for (int k = 0; k < T; k++) s += sc[k] * V[(size_t)k * D + h * DK + i];
                att[(size_t)q * D + h * DK + i] = s;
            }
        }
        free(sc); free(bd);
    }
    orc_linear(x, att, L->sa_ow, L->sa_ob, T, D, D, ORC_EP_STORE, 0.f);
    free(Q); free(K); free(V); free(P); free(att);
}

/* backends/cpu/backend.c:300-337: pw1 (D->2D), GLU a*sigmoid(b), depthwise conv
 * (kernel ck, "same" zero padding), eval BatchNorm (eps 1e-5), SiLU, pw2. */
void orc_conformer_conv(const ct_dims *d, float *x, int T, const ELayer *L) {
    const int D = d->enc_d, CK = d->enc_ck, pad = (CK - 1) / 2;
    float *pw1 = XMALLOC(sizeof(float) * (size_t)T * 2 * D);
    float *glu = XMALLOC(sizeof(float) * (size_t)T * D);
    float *dw  = XMALLOC(sizeof(float) * (size_t)T * D);
    orc_linear(pw1, x, L->cv_pw1w, L->cv_pw1b, T, D, 2 * D, ORC_EP_STORE, 0.f);
    for (int t = 0; t < T; t++)
        for (int c = 0; c < D; c++) {
            float a = pw1[(size_t)t*2*D + c];
            float g = pw1[(size_t)t*2*D + c + D];
            glu[(size_t)t*D + c] = a / (1.0f + expf(-g));
        }
    for (int t = 0; t < T; t++)
        for (int c = 0; c < D; c++) {
            float s = BF(L->cv_dwb[c]);
            for (int k = 0; k < CK; k++) {
                int ti = t - pad + k;
                if (ti < 0 || ti >= T) continue;
                s += BF(L->cv_dww[c * CK + k]) * glu[(size_t)ti * D + c];
            }
            dw[(size_t)t * D + c] = s;
        }
    const float bn_eps = 1e-5f;
    for (int t = 0; t < T; t++)
        for (int c = 0; c < D; c++) {
            float v = dw[(size_t)t*D + c];
            v = (v - BF(L->cv_bnmean[c])) / sqrtf(BF(L->cv_bnvar[c]) + bn_eps)
                * BF(L->cv_bnw[c]) + BF(L->cv_bnb[c]);
            dw[(size_t)t*D + c] = v;
        }
    for (size_t i = 0; i < (size_t)T * D; i++) dw[i] = dw[i] / (1.0f + expf(-dw[i]));
    orc_linear(x, dw, L->cv_pw2w, L->cv_pw2b, T, D, D, ORC_EP_STORE, 0.f);
    free(pw1); free(glu); free(dw);
}

/* backends/cpu/backend.c:339-360: per head softmax(q·k/sqrt(dk) + mask)·v. */
void orc_sdp_attn(const ct_dims *d, float *out, const float *q, const float *k, const float *v,
                  const float *mask, int T_q, int T_k) {
    const int D = d->dec_d, H = d->dec_h, DK = d->dec_dk;
    const float scale = 1.0f / sqrtf((float)DK);
    #pragma omp parallel if ((long)T_q * T_k > 2048)
    {
        float *sc = XMALLOC(sizeof(float) * (size_t)(T_k > 0 ? T_k : 1));
        #pragma omp for collapse(2) schedule(static)
        for (int h = 0; h < H; h++)
        for (int qi = 0; qi < T_q; qi++) {
            for (int ki = 0; ki < T_k; ki++) {
                float s = 0;
                for (int i = 0; i < DK; i++)
                    s += q[(size_t)qi*D + h*DK + i] * k[(size_t)ki*D + h*DK + i];
                sc[ki] = s * scale + (mask ? mask[(size_t)qi*T_k + ki] : 0.0f);
            }
            softmax_row(sc, T_k);
            for (int i = 0; i < DK; i++) {
                float s = 0;
                for (int ki = 0; ki < T_k; ki++) s += sc[ki] * v[(size_t)ki*D + h*DK + i];
                out[(size_t)qi*D + h*DK + i] = s;
            }
        }
        free(sc);
    }
}

/* backends/cpu/backend.c:362-371 */
void orc_embed(const ct_dims *d, float *h, const int *tokens, int S, int pos_start,
               const uint16_t *etw, const uint16_t *epw, const uint16_t *elnw, const uint16_t *elnb) {
    const int D = d->dec_d;
    for (int t = 0; t < S; t++) {
        const int id = tokens[t];
        for (int i = 0; i < D; i++)
            h[(size_t)t*D + i] = BF(etw[(size_t)id*D + i]) + BF(epw[(size_t)(pos_start + t)*D + i]);
    }
    orc_layernorm(h, h, elnw, elnb, S, D);
}

/* backends/cpu/backend.c:373-377 */
void orc_fill_causal_mask(float *mask, int S) {
    for (int qi = 0; qi < S; qi++)
        for (int ki = 0; ki < S; ki++)
            mask[(size_t)qi*S + ki] = (ki > qi) ? -1e9f : 0.0f;
}

/* backends/cpu/backend.c:379-387: tied LM head, logits = hdb + last · etw^T */
void orc_lm_head(const ct_dims *d, float *logits, const float *last,
                 const uint16_t *etw, const uint16_t *hdb) {
    orc_linear(logits, last, etw, hdb, 1, d->dec_d, d->vocab, ORC_EP_STORE, 0.f);
}

/* backends/cpu/backend.c:451-453: first index of the maximum (strict >). */
int orc_argmax(const float *lg, int n) {
    int best = 0; float bv = lg[0];
    for (int i = 1; i < n; i++) if (lg[i] > bv) { bv = lg[i]; best = i; }
    return best;
}

void orc_top2(const float *lg, int n, int *idx, float *margin) {
    int best = orc_argmax(lg, n);
    float second = -INFINITY;
    for (int i = 0; i < n; i++) if (i != best && lg[i] > second) second = lg[i];
    *idx = best;
    *margin = lg[best] - second;
}

/* ------------------------------------------------------------------ */
/* batched decode helpers                                              */
/* ------------------------------------------------------------------ */

/* backends/cpu/backend.c:425-435 */
void orc_embed_decode_batch(const ct_dims *d, float *h, const int *tokens, const int *S_dev,
                            const int *active, int B, const uint16_t *etw, const uint16_t *epw,
                            const uint16_t *elnw, const uint16_t *elnb) {
    for (int b = 0; b < B; b++) {
        if (!active[b]) continue;
        orc_embed(d, h + (size_t)b * d->dec_d, &tokens[b], 1, S_dev[b] - 1, etw, epw, elnw, elnb);
    }
}

/* backends/cpu/backend.c:437-444 */
void orc_lm_head_batch(const ct_dims *d, float *logits, const float *h, const uint16_t *etw,
                       const uint16_t *hdb, const int *active, int B) {
    for (int b = 0; b < B; b++) {
        if (!active[b]) continue;
        orc_lm_head(d, logits + (size_t)b * d->vocab, h + (size_t)b * d->dec_d, etw, hdb);
    }
}

/* backends/cpu/backend.c:446-456 */
void orc_argmax_batch(const ct_dims *d, int *out, const float *logits, const int *active, int B) {
    for (int b = 0; b < B; b++)
        if (active[b]) out[b] = orc_argmax(logits + (size_t)b * d->vocab, d->vocab);
}

/* backends/cpu/backend.c:466-476: row b goes to slot S_dev[b]-1 of item b. */
void orc_linear_to_kvcache_batch(float *cache, const float *x, const uint16_t *W, const uint16_t *b,
                                 int B, int cache_seq_stride, int in_d, int out_d, const int *S_dev) {
    for (int i = 0; i < B; i++) {
        const int slot = S_dev[i] - 1;
        orc_linear(cache + ((size_t)i * cache_seq_stride + slot) * out_d, x + (size_t)i * in_d,
                   W, b, 1, in_d, out_d, ORC_EP_STORE, 0.f);
    }
}

/* backends/cpu/backend.c:478-500: one query per item over T_k[b] keys. */
void orc_sdp_attn_batch_decode(const ct_dims *d, float *out, const float *Q, const float *K,
                               const float *V, int T_k_stride, int B, const int *T_k) {
    const size_t D = (size_t)d->dec_d;
    for (int b = 0; b < B; b++)
        orc_sdp_attn(d, out + b * D, Q + b * D, K + (size_t)b * T_k_stride * D,
                     V + (size_t)b * T_k_stride * D, NULL, 1, T_k[b]);
}

/* ------------------------------------------------------------------ */
/* model level                                                         */
/* ------------------------------------------------------------------ */

/* model.h:276-314: macaron FFN/2, rel-pos MHSA, conv module, FFN/2, LN. */
void orc_conformer_layer(const ct_dims *d, float *x, const float *pos_emb, int T, const ELayer *L) {
    const int D = d->enc_d, FF = d->enc_ff;
    float *ln  = XMALLOC(sizeof(float) * (size_t)T * D);
    float *tmp = XMALLOC(sizeof(float) * (size_t)T * FF);
    orc_layernorm(ln, x, L->ff1_lnw, L->ff1_lnb, T, D);
    orc_linear(tmp, ln, L->ff1_w1, L->ff1_b1, T, D, FF, ORC_EP_SILU, 0.f);
    orc_linear(x, tmp, L->ff1_w2, L->ff1_b2, T, FF, D, ORC_EP_FMADD, 0.5f);
    orc_layernorm(ln, x, L->sa_lnw, L->sa_lnb, T, D);
    orc_rel_pos_mhsa(d, ln, pos_emb, T, L);
    orc_add_inplace(x, ln, T * D);
    orc_layernorm(ln, x, L->cv_lnw, L->cv_lnb, T, D);
    orc_conformer_conv(d, ln, T, L);
    orc_add_inplace(x, ln, T * D);
    orc_layernorm(ln, x, L->ff2_lnw, L->ff2_lnb, T, D);
    orc_linear(tmp, ln, L->ff2_w1, L->ff2_b1, T, D, FF, ORC_EP_SILU, 0.f);
    orc_linear(x, tmp, L->ff2_w2, L->ff2_b2, T, FF, D, ORC_EP_FMADD, 0.5f);
    orc_layernorm(x, x, L->out_lnw, L->out_lnb, T, D);
    free(ln); free(tmp);
}

/* model.h:573-609: per item subsampling, enc_n Conformer layers over its own
 * T_enc[b] rows with the T_enc_max position table shifted by T_enc_max-T_enc[b],
 * then the encoder->decoder projection.  enc_h_batch is [B, T_enc_max, dec_d]. */
void orc_encoder_forward_batch(const ct_dims *d, const Weights *W, const float *mel_batch, int B,
                               int T_mel_max, const int *T_mel, const int *T_enc, int T_enc_max,
                               float *enc_h_batch) {
    const int D = d->enc_d;
    float *pe = XMALLOC(sizeof(float) * (size_t)(2 * T_enc_max - 1) * D);
    float *x = XMALLOC(sizeof(float) * (size_t)T_enc_max * D);
    orc_make_rel_pos_emb(d, pe, T_enc_max);
    for (int b = 0; b < B; b++) {
        const int Te = T_enc[b];
        const float *pe_b = pe + (size_t)(T_enc_max - Te) * D;
        orc_encoder_subsampling(d, mel_batch + (size_t)b * d->n_mels * T_mel_max, T_mel[b],
                                T_mel_max, x, Te, W);
        for (int l = 0; l < d->enc_n; l++) orc_conformer_layer(d, x, pe_b, Te, &W->enc[l]);
        orc_linear(enc_h_batch + (size_t)b * T_enc_max * d->dec_d, x, W->prw, W->prb, Te, D,
                   d->dec_d, ORC_EP_STORE, 0.f);
    }
    free(pe); free(x);
}

/* model.h:349-364 / :620-635 */
void orc_precompute_ca_kv(const ct_dims *d, const Weights *W, const float *enc_h, int T_enc,
                          float **ca_k, float **ca_v) {
    for (int l = 0; l < d->dec_n; l++) {
        orc_linear(ca_k[l], enc_h, W->dec[l].ca_kw, W->dec[l].ca_kb, T_enc, d->dec_d, d->dec_d, ORC_EP_STORE, 0.f);
        orc_linear(ca_v[l], enc_h, W->dec[l].ca_vw, W->dec[l].ca_vb, T_enc, d->dec_d, d->dec_d, ORC_EP_STORE, 0.f);
    }
}

/* model.h:376-409: pre-LN self-attention over the KV cache (new rows written
 * at [S_kv-S_q, S_kv)), cross-attention, ReLU FFN, all with residual adds. */
static void decoder_layer(const ct_dims *d, float *h, const float *ca_k, const float *ca_v,
                          const float *mask, int S_q, int S_kv, int T_enc,
                          float *sa_k, float *sa_v, const DLayer *L) {
    const int D = d->dec_d, FF = d->dec_ff;
    float *ln = XMALLOC(sizeof(float) * (size_t)S_q * D);
    float *Q  = XMALLOC(sizeof(float) * (size_t)S_q * (FF > D ? FF : D));
    float *ao = XMALLOC(sizeof(float) * (size_t)S_q * D);
    float *Kn = sa_k + (size_t)(S_kv - S_q) * D;
    float *Vn = sa_v + (size_t)(S_kv - S_q) * D;
    orc_layernorm(ln, h, L->sa_lnw, L->sa_lnb, S_q, D);
    orc_linear(Q, ln, L->sa_qw, L->sa_qb, S_q, D, D, ORC_EP_STORE, 0.f);
    orc_linear(Kn, ln, L->sa_kw, L->sa_kb, S_q, D, D, ORC_EP_STORE, 0.f);
    orc_linear(Vn, ln, L->sa_vw, L->sa_vb, S_q, D, D, ORC_EP_STORE, 0.f);
    orc_sdp_attn(d, ao, Q, sa_k, sa_v, mask, S_q, S_kv);
    orc_linear(h, ao, L->sa_ow, L->sa_ob, S_q, D, D, ORC_EP_FMADD, 1.0f);
    orc_layernorm(ln, h, L->ca_lnw, L->ca_lnb, S_q, D);
    orc_linear(Q, ln, L->ca_qw, L->ca_qb, S_q, D, D, ORC_EP_STORE, 0.f);
    orc_sdp_attn(d, ao, Q, ca_k, ca_v, NULL, S_q, T_enc);
    orc_linear(h, ao, L->ca_ow, L->ca_ob, S_q, D, D, ORC_EP_FMADD, 1.0f);
    orc_layernorm(ln, h, L->ffn_lnw, L->ffn_lnb, S_q, D);
    orc_linear(Q, ln, L->ffn_w1, L->ffn_b1, S_q, D, FF, ORC_EP_RELU, 0.f);
    orc_linear(h, Q, L->ffn_w2, L->ffn_b2, S_q, FF, D, ORC_EP_FMADD, 1.0f);
    free(ln); free(Q); free(ao);
}

/* model.h:461-503 with S_q == S (prefill of the whole prompt): causal mask,
 * dec_n layers, final LN, LM head on the last row, host argmax. */
int orc_decoder_prefill(const ct_dims *d, const Weights *W, const int *tokens, int S, int T_enc,
                        float **ca_k, float **ca_v, float **sa_k, float **sa_v, float *logits_out) {
    const int D = d->dec_d;
    float *h = XMALLOC(sizeof(float) * (size_t)S * D);
    float *mask = XMALLOC(sizeof(float) * (size_t)S * S);
    float *lg = logits_out ? logits_out : XMALLOC(sizeof(float) * (size_t)d->vocab);
    orc_embed(d, h, tokens, S, 0, W->etw, W->epw, W->elnw, W->elnb);
    if (S > 1) orc_fill_causal_mask(mask, S);
    for (int l = 0; l < d->dec_n; l++)
        decoder_layer(d, h, ca_k[l], ca_v[l], S > 1 ? mask : NULL, S, S, T_enc, sa_k[l], sa_v[l],
                      &W->dec[l]);
    orc_layernorm(h, h, W->dlnw, W->dlnb, S, D);
    orc_lm_head(d, lg, h + (size_t)(S - 1) * D, W->etw, W->hdb);
    int best = orc_argmax(lg, d->vocab);
    if (!logits_out) free(lg);
    free(h); free(mask);
    return best;
}

/* model.h:666-744: one batched decode step (inactive rows computed, discarded). */
void orc_decoder_step_decode_batch(const ct_dims *d, const Weights *W,
                                   const int *tokens_cur, const int *S_dev, const int *active,
                                   const int *T_enc, int T_enc_stride,
                                   float **ca_k_batch, float **ca_v_batch,
                                   float **sa_k_batch, float **sa_v_batch,
                                   float *h_dec, float *logits, int B, int *next_tokens) {
    const int D = d->dec_d, FF = d->dec_ff;
    float *ln = XMALLOC(sizeof(float) * (size_t)B * D);
    float *Q  = XMALLOC(sizeof(float) * (size_t)B * (FF > D ? FF : D));
    float *ao = XMALLOC(sizeof(float) * (size_t)B * D);
    orc_embed_decode_batch(d, h_dec, tokens_cur, S_dev, active, B, W->etw, W->epw, W->elnw, W->elnb);
    for (int l = 0; l < d->dec_n; l++) {
        const DLayer *L = &W->dec[l];
        orc_layernorm(ln, h_dec, L->sa_lnw, L->sa_lnb, B, D);
        orc_linear(Q, ln, L->sa_qw, L->sa_qb, B, D, D, ORC_EP_STORE, 0.f);
        orc_linear_to_kvcache_batch(sa_k_batch[l], ln, L->sa_kw, L->sa_kb, B, d->max_seq, D, D, S_dev);
        orc_linear_to_kvcache_batch(sa_v_batch[l], ln, L->sa_vw, L->sa_vb, B, d->max_seq, D, D, S_dev);
        orc_sdp_attn_batch_decode(d, ao, Q, sa_k_batch[l], sa_v_batch[l], d->max_seq, B, S_dev);
        orc_linear(h_dec, ao, L->sa_ow, L->sa_ob, B, D, D, ORC_EP_FMADD, 1.0f);
        orc_layernorm(ln, h_dec, L->ca_lnw, L->ca_lnb, B, D);
        orc_linear(Q, ln, L->ca_qw, L->ca_qb, B, D, D, ORC_EP_STORE, 0.f);
        orc_sdp_attn_batch_decode(d, ao, Q, ca_k_batch[l], ca_v_batch[l], T_enc_stride, B, T_enc);
        orc_linear(h_dec, ao, L->ca_ow, L->ca_ob, B, D, D, ORC_EP_FMADD, 1.0f);
        orc_layernorm(ln, h_dec, L->ffn_lnw, L->ffn_lnb, B, D);
        orc_linear(Q, ln, L->ffn_w1, L->ffn_b1, B, D, FF, ORC_EP_RELU, 0.f);
        orc_linear(h_dec, Q, L->ffn_w2, L->ffn_b2, B, FF, D, ORC_EP_FMADD, 1.0f);
    }
    orc_layernorm(h_dec, h_dec, W->dlnw, W->dlnb, B, D);
    orc_lm_head_batch(d, logits, h_dec, W->etw, W->hdb, active, B);
    orc_argmax_batch(d, next_tokens, logits, active, B);
    free(ln); free(Q); free(ao);
}

/* transcribe.c:686-795 (per-item prefill then the joint decode loop), driven
 * from encoder outputs, with forced-EOS lengths and optional teacher forcing.
 * logits_out (optional, [B][logits_cap][V]) receives the logits that chose
 * generated token g of sequence b, for g < logits_cap (g = 0: the prefill's). */
int orc_decode_batch_logits(const ct_dims *d, const Weights *W, int B, const int *T_enc, int T_enc_stride,
                            const float *enc_h_batch, const int *prompt, int n_prompt,
                            const int *forced_len, const int *force_tokens,
                            int *tokens, int *n_tok, int *am, float *margin,
                            float *logits_out, int logits_cap) {
    const int D = d->dec_d, L = d->dec_n, MS = d->max_seq, V = d->vocab;
    float **ca_k = XMALLOC(sizeof(float *) * L), **ca_v = XMALLOC(sizeof(float *) * L);
    float **sa_k = XMALLOC(sizeof(float *) * L), **sa_v = XMALLOC(sizeof(float *) * L);
    for (int l = 0; l < L; l++) {
        ca_k[l] = XMALLOC(sizeof(float) * (size_t)B * T_enc_stride * D);
        ca_v[l] = XMALLOC(sizeof(float) * (size_t)B * T_enc_stride * D);
        sa_k[l] = XMALLOC(sizeof(float) * (size_t)B * MS * D);
        sa_v[l] = XMALLOC(sizeof(float) * (size_t)B * MS * D);
    }
    float *lg = XMALLOC(sizeof(float) * (size_t)B * V);
    float *h = XMALLOC(sizeof(float) * (size_t)B * D);
    int *S = XMALLOC(sizeof(int) * B), *S_dev = XMALLOC(sizeof(int) * B);
    int *active = XMALLOC(sizeof(int) * B), *cur = XMALLOC(sizeof(int) * B);
    int *next = XMALLOC(sizeof(int) * B), *gen = XMALLOC(sizeof(int) * B);
    float **cak_b = XMALLOC(sizeof(float *) * L), **cav_b = XMALLOC(sizeof(float *) * L);
    float **sak_b = XMALLOC(sizeof(float *) * L), **sav_b = XMALLOC(sizeof(float *) * L);

    for (int b = 0; b < B; b++) {
        const float *eh = enc_h_batch + (size_t)b * T_enc_stride * D;
        for (int l = 0; l < L; l++) {
            cak_b[l] = ca_k[l] + (size_t)b * T_enc_stride * D;
            cav_b[l] = ca_v[l] + (size_t)b * T_enc_stride * D;
            sak_b[l] = sa_k[l] + (size_t)b * MS * D;
            sav_b[l] = sa_v[l] + (size_t)b * MS * D;
        }
        orc_precompute_ca_kv(d, W, eh, T_enc[b], cak_b, cav_b);
        int *tb = tokens + (size_t)b * MS;
        memcpy(tb, prompt, sizeof(int) * n_prompt);
        int id;
        float mg;
        orc_decoder_prefill(d, W, tb, n_prompt, T_enc[b], cak_b, cav_b, sak_b, sav_b, lg);
        orc_top2(lg, V, &id, &mg);
        if (am) am[(size_t)b * MS + n_prompt] = id;
        if (margin) margin[(size_t)b * MS + n_prompt] = mg;
        if (logits_out && logits_cap > 0) memcpy(logits_out + (size_t)b * logits_cap * V, lg, sizeof(float) * V);
        gen[b] = 1;
        if (force_tokens) id = force_tokens[(size_t)b * MS + n_prompt];
        if (gen[b] >= forced_len[b]) id = CT_TOK_EOS;
        tb[n_prompt] = id;
        S[b] = n_prompt + 1;
        active[b] = (gen[b] < forced_len[b]) && S[b] < MS;
        S_dev[b] = S[b] - 1;
    }
    int n_active = 0;
    for (int b = 0; b < B; b++) n_active += active[b];
    while (n_active > 0) {
        for (int b = 0; b < B; b++) {
            cur[b] = active[b] ? tokens[(size_t)b * MS + S[b] - 1] : 0;
            if (active[b]) S_dev[b]++;
        }
        orc_decoder_step_decode_batch(d, W, cur, S_dev, active, T_enc, T_enc_stride,
                                      ca_k, ca_v, sa_k, sa_v, h, lg, B, next);
        for (int b = 0; b < B; b++) {
            if (!active[b]) continue;
            int id; float mg;
            orc_top2(lg + (size_t)b * V, V, &id, &mg);
            if (am) am[(size_t)b * MS + S[b]] = id;
            if (margin) margin[(size_t)b * MS + S[b]] = mg;
            if (logits_out && gen[b] < logits_cap)
                memcpy(logits_out + ((size_t)b * logits_cap + gen[b]) * V, lg + (size_t)b * V, sizeof(float) * V);
            gen[b]++;
            if (force_tokens) id = force_tokens[(size_t)b * MS + S[b]];
            if (gen[b] >= forced_len[b]) id = CT_TOK_EOS;
            tokens[(size_t)b * MS + S[b]] = id;
            S[b]++;
            if (gen[b] >= forced_len[b] || S[b] >= MS) { active[b] = 0; n_active--; }
        }
    }
    for (int b = 0; b < B; b++) n_tok[b] = S[b];
    for (int l = 0; l < L; l++) { free(ca_k[l]); free(ca_v[l]); free(sa_k[l]); free(sa_v[l]); }
    free(ca_k); free(ca_v); free(sa_k); free(sa_v); free(lg); free(h); free(S); free(S_dev);
    free(active); free(cur); free(next); free(gen); free(cak_b); free(cav_b); free(sak_b); free(sav_b);
    return 0;
}

int orc_decode_batch(const ct_dims *d, const Weights *W, int B, const int *T_enc, int T_enc_stride,
                     const float *enc_h_batch, const int *prompt, int n_prompt,
                     const int *forced_len, const int *force_tokens,
                     int *tokens, int *n_tok, int *am, float *margin) {
    return orc_decode_batch_logits(d, W, B, T_enc, T_enc_stride, enc_h_batch, prompt, n_prompt, forced_len,
                                   force_tokens, tokens, n_tok, am, margin, NULL, 0);
}

/* ------------------------------------------------------------------ */
/* log-mel front-end                                                   */
/* ------------------------------------------------------------------ */

/* transcribe.c:45-50: symmetric Hann window of ORC_WIN points. */
void orc_hann(float *w) {
    for (int i = 0; i < ORC_WIN; i++)
        w[i] = 0.5f * (1.0f - cosf(2.0f * (float)M_PI * i / (ORC_WIN - 1)));
}

/* transcribe.c:56-70: Slaney mel scale (linear below 1 kHz, log above). */
static double slaney_hz_to_mel(double f) {
    const double f_sp = 200.0 / 3.0, brk = 1000.0, brk_mel = brk / f_sp, step = log(6.4) / 27.0;
    return f < brk ? f / f_sp : brk_mel + log(f / brk) / step;
}
static double slaney_mel_to_hz(double m) {
    const double f_sp = 200.0 / 3.0, brk = 1000.0, brk_mel = brk / f_sp, step = log(6.4) / 27.0;
    return m < brk_mel ? f_sp * m : brk * exp(step * (m - brk_mel));
}

/* transcribe.c:72-97: triangular filters between ORC_N_MELS + 2 points equally
 * spaced in mel from 0 to SR/2, area-normalised (librosa norm='slaney'). */
void orc_mel_filterbank(float *fb) {
    double pts[ORC_N_MELS + 2], gap[ORC_N_MELS + 1];
    const double lo = slaney_hz_to_mel(0.0), hi = slaney_hz_to_mel(ORC_SR / 2.0);
    for (int i = 0; i < ORC_N_MELS + 2; i++)
        pts[i] = slaney_mel_to_hz(lo + (hi - lo) * i / (ORC_N_MELS + 1));
    for (int i = 0; i < ORC_N_MELS + 1; i++) gap[i] = pts[i + 1] - pts[i];
    for (int m = 0; m < ORC_N_MELS; m++) {
        const double norm = 2.0 / (pts[m + 2] - pts[m]);
        for (int k = 0; k < ORC_N_BINS; k++) {
            const double f = (ORC_SR / 2.0) * k / (ORC_N_BINS - 1);
            const double up = (f - pts[m]) / gap[m], down = (pts[m + 2] - f) / gap[m + 1];
            const double w = up < down ? up : down;
            fb[m * ORC_N_BINS + k] = (float)(w > 0.0 ? w * norm : 0.0);
        }
    }
}

/* transcribe.c:99-123: iterative radix-2 decimation-in-time FFT, bit-reversal
 * permutation first, twiddles advanced by complex multiplication per stage. */
static void orc_fft(float *re, float *im, int n) {
    for (int i = 1, j = 0; i < n; i++) {
        int bit = n >> 1;
        for (; j & bit; bit >>= 1) j ^= bit;
        j ^= bit;
        if (i < j) {
            float t = re[i]; re[i] = re[j]; re[j] = t;
            t = im[i]; im[i] = im[j]; im[j] = t;
        }
    }
    for (int len = 2; len <= n; len <<= 1) {
        const float ang = -2.0f * (float)M_PI / len;
        const float wr = cosf(ang), wi = sinf(ang);
        for (int i = 0; i < n; i += len) {
            float cr = 1, ci = 0;
            for (int k = 0; k < len / 2; k++) {
                const int a = i + k, b = i + k + len / 2;
                const float ur = re[a], ui = im[a];
                const float vr = re[b] * cr - im[b] * ci;
                const float vi = re[b] * ci + im[b] * cr;
                re[a] = ur + vr; im[a] = ui + vi;
                re[b] = ur - vr; im[b] = ui - vi;
                const float nc = cr * wr - ci * wi;
                ci = cr * wi + ci * wr;
                cr = nc;
            }
        }
    }
}

/* transcribe.c:177-214: zero-pad WIN/2 on both sides, pre-emphasis 0.97,
 * Hann-windowed 512-point power spectra every HOP samples, mel projection,
 * log(x + 2^-24), then per-mel-bin normalisation over time (mean, unbiased
 * variance, eps 1e-5). */
void orc_compute_mel(const float *samples, int N, float *mel) {
    static float hann[ORC_WIN], fb[ORC_N_MELS * ORC_N_BINS];
    static int ready = 0;
    if (!ready) { orc_hann(hann); orc_mel_filterbank(fb); ready = 1; }
    const int T = 1 + N / ORC_HOP, pad = ORC_WIN / 2, Np = N + 2 * pad;
    float *s = XMALLOC(sizeof(float) * (size_t)Np);
    memset(s, 0, sizeof(float) * (size_t)Np);
    memcpy(s + pad, samples, sizeof(float) * (size_t)N);
    for (int i = Np - 1; i > 0; i--) s[i] -= 0.97f * s[i - 1];
    float re[ORC_N_FFT], im[ORC_N_FFT], ps[ORC_N_BINS];
    for (int t = 0; t < T; t++) {
        const int off = t * ORC_HOP;
        for (int i = 0; i < ORC_N_FFT; i++) re[i] = im[i] = 0.0f;
        for (int i = 0; i < ORC_WIN && off + i < Np; i++) re[i] = s[off + i] * hann[i];
        orc_fft(re, im, ORC_N_FFT);
        for (int k = 0; k < ORC_N_BINS; k++) ps[k] = re[k] * re[k] + im[k] * im[k];
        for (int m = 0; m < ORC_N_MELS; m++) {
            float v = 0;
            for (int k = 0; k < ORC_N_BINS; k++) v += fb[m * ORC_N_BINS + k] * ps[k];
            mel[(size_t)m * T + t] = v;
        }
    }
    const float guard = powf(2.0f, -24.0f);
    for (int m = 0; m < ORC_N_MELS; m++) {
        float *row = mel + (size_t)m * T;
        float mean = 0, var = 0;
        for (int t = 0; t < T; t++) { row[t] = logf(row[t] + guard); mean += row[t]; }
        mean /= T;
        for (int t = 0; t < T; t++) { const float d = row[t] - mean; var += d * d; }
        var /= (T - 1);
        const float inv = 1.0f / sqrtf(var + 1e-5f);
        for (int t = 0; t < T; t++) row[t] = (row[t] - mean) * inv;
    }
    free(s);
}
