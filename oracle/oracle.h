/* oracle.h -- CPU restatement of the cohere-transcribe reference algorithm.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the B200 backend:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * legs may load it.  The product (libct_b200.so) never links or calls it.
 *
 * Every function restates a reference function (cited file:line, paths within
 * the apaz-cli/cohere-transcribe project) in the same arithmetic order, with
 * the model dimensions taken from a runtime `ct_dims` (the reference fixes them
 * at compile time in backends/model_types.h:14-30), so one build serves both
 * the full-size model and the tiny test configuration.
 *
 * Parity pin: tests/test_oracle_golden.py checks these functions against the
 * reference's own test vectors (tests/test_kernels.c run on the reference CPU
 * backend, committed as tests/golden/test_kernels_ref_cpu.bin) and, where the
 * reference CPU backend has been built into oracle/_ref/, against it directly.
 */
#ifndef CT_ORACLE_H
#define CT_ORACLE_H

#include <stdint.h>
#include <stddef.h>
#include "../include/ct_model_types.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ct_dims {
    int enc_d, enc_ff, enc_h, enc_dk, enc_n, enc_ck, sub_ch;
    int dec_d, dec_ff, dec_h, dec_dk, dec_n;
    int vocab, max_seq, n_mels;
} ct_dims;

/* epilogues of the linear family, backend.h:56-64 */
enum { ORC_EP_STORE = 0, ORC_EP_SILU = 1, ORC_EP_RELU = 2, ORC_EP_FMADD = 3 };

void  orc_dims_full(ct_dims *d);
float orc_bf16(uint16_t b);

/* ---- primitives (backends/cpu/backend.c) ---- */
void orc_layernorm(float *dst, const float *src, const uint16_t *w, const uint16_t *b, int T, int D);
void orc_linear(float *y, const float *x, const uint16_t *W, const uint16_t *b,
                int T, int in_d, int out_d, int ep, float scale);
void orc_add_inplace(float *dst, const float *src, int n);
void orc_encoder_subsampling(const ct_dims *d, const float *mel, int T_mel, int T_mel_stride,
                             float *x_enc, int T_enc, const Weights *W);
void orc_make_rel_pos_emb(const ct_dims *d, float *pe, int T);
void orc_rel_pos_mhsa(const ct_dims *d, float *x, const float *pos_emb, int T, const ELayer *L);
void orc_conformer_conv(const ct_dims *d, float *x, int T, const ELayer *L);
void orc_sdp_attn(const ct_dims *d, float *out, const float *q, const float *k, const float *v,
                  const float *mask, int T_q, int T_k);
void orc_embed(const ct_dims *d, float *h, const int *tokens, int S, int pos_start,
               const uint16_t *etw, const uint16_t *epw, const uint16_t *elnw, const uint16_t *elnb);
void orc_fill_causal_mask(float *mask, int S);
void orc_lm_head(const ct_dims *d, float *logits, const float *last,
                 const uint16_t *etw, const uint16_t *hdb);
int  orc_argmax(const float *lg, int n);

/* ---- batched decode helpers (backends/cpu/backend.c:425-500) ---- */
void orc_embed_decode_batch(const ct_dims *d, float *h, const int *tokens, const int *S_dev,
                            const int *active, int B, const uint16_t *etw, const uint16_t *epw,
                            const uint16_t *elnw, const uint16_t *elnb);
void orc_lm_head_batch(const ct_dims *d, float *logits, const float *h, const uint16_t *etw,
                       const uint16_t *hdb, const int *active, int B);
void orc_argmax_batch(const ct_dims *d, int *out, const float *logits, const int *active, int B);
void orc_linear_to_kvcache_batch(float *cache, const float *x, const uint16_t *W, const uint16_t *b,
                                 int B, int cache_seq_stride, int in_d, int out_d, const int *S_dev);
void orc_sdp_attn_batch_decode(const ct_dims *d, float *out, const float *Q, const float *K,
                               const float *V, int T_k_stride, int B, const int *T_k);

/* ---- model level (model.h) ---- */
void orc_conformer_layer(const ct_dims *d, float *x, const float *pos_emb, int T, const ELayer *L);
void orc_encoder_forward_batch(const ct_dims *d, const Weights *W, const float *mel_batch, int B,
                               int T_mel_max, const int *T_mel, const int *T_enc, int T_enc_max,
                               float *enc_h_batch);
void orc_precompute_ca_kv(const ct_dims *d, const Weights *W, const float *enc_h, int T_enc,
                          float **ca_k, float **ca_v);
int  orc_decoder_prefill(const ct_dims *d, const Weights *W, const int *tokens, int S, int T_enc,
                         float **ca_k, float **ca_v, float **sa_k, float **sa_v, float *logits_out);
void orc_decoder_step_decode_batch(const ct_dims *d, const Weights *W,
                                   const int *tokens_cur, const int *S_dev, const int *active,
                                   const int *T_enc, int T_enc_stride,
                                   float **ca_k_batch, float **ca_v_batch,
                                   float **sa_k_batch, float **sa_v_batch,
                                   float *h_dec, float *logits, int B, int *next_tokens);

/* Static ragged batch decode: the per-item prefill + joint decode loop of
 * transcribe.c:686-795, from precomputed encoder outputs, with the harness's
 * forced-EOS lengths.  forced_len[b] = number of generated tokens (the last one
 * is forced to EOS; a natural EOS before it is kept and decoding continues).
 * force_tokens (optional, [B, max_seq]): teacher forcing -- the token appended
 * at every position is taken from it instead of the oracle's own argmax.
 * Outputs: tokens [B, max_seq] (prompt included), n_tok[b] = total length;
 * optional am[B, max_seq] = the oracle's argmax at each generated position and
 * margin[B, max_seq] = its top-1 minus top-2 logit.  Returns 0. */
int orc_decode_batch(const ct_dims *d, const Weights *W, int B, const int *T_enc, int T_enc_stride,
                     const float *enc_h_batch, const int *prompt, int n_prompt,
                     const int *forced_len, const int *force_tokens,
                     int *tokens, int *n_tok, int *am, float *margin);

/* orc_decode_batch that also returns logits: logits_out [B, logits_cap, vocab]
 * holds the logits that chose generated token g of sequence b, for
 * g < logits_cap (g = 0 is the prefill's token). */
int orc_decode_batch_logits(const ct_dims *d, const Weights *W, int B, const int *T_enc, int T_enc_stride,
                            const float *enc_h_batch, const int *prompt, int n_prompt,
                            const int *forced_len, const int *force_tokens,
                            int *tokens, int *n_tok, int *am, float *margin,
                            float *logits_out, int logits_cap);

/* top-1 index and (top1 - top2) over n logits */
void orc_top2(const float *lg, int n, int *idx, float *margin);

/* ---- log-mel front-end (transcribe.c:45-123, :177-214) -------------------
 * 16 kHz mono samples -> normalised log-mel [ORC_N_MELS][T_mel], T_mel = 1 + N / 160. */
#define ORC_SR 16000
#define ORC_N_FFT 512
#define ORC_WIN 400
#define ORC_HOP 160
#define ORC_N_MELS 128
#define ORC_N_BINS (ORC_N_FFT / 2 + 1)
void orc_mel_filterbank(float *fb /* [ORC_N_MELS * ORC_N_BINS] */);
void orc_hann(float *w /* [ORC_WIN] */);
void orc_compute_mel(const float *samples, int N, float *mel /* [ORC_N_MELS][1 + N / ORC_HOP] */);

#ifdef __cplusplus
}
#endif
#endif
