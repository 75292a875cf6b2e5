/* ct_engine.h -- continuous-batching decode engine of libct_b200.so.
 *
 * Additive to the drop-in ABI of ct_backend.h: that ABI cannot express a
 * paged KV cache or admission of new sequences into a running batch (its KV
 * cache is a dense fp32 [B, MAX_SEQ, DEC_D] arena region, backends/backend.h:214-217,
 * and transcribe_batch admits nothing mid-flight, transcribe.c:752-795).  The
 * engine replaces the per-item prefill + joint decode loop of transcribe_batch
 * (transcribe.c:692-795) and decoder_step_decode_batch (model.h:721-744):
 *
 *   - one engine per GPU, driven by one host thread;
 *   - sequences are admitted into slots; every step packs the query rows of all
 *     live slots (10 prompt rows for a slot's first step, then 1 row) with
 *     prefix sums on the GPU, so prefill and decode share one batched pass;
 *   - self-attention K/V and cross-attention K/V live in a bf16 page pool
 *     (16 token rows per page, all layers); cross K/V are projected once at
 *     admission (model.h:620-635) straight into pages;
 *   - greedy argmax, EOS / forced-length retirement and token append happen on
 *     the GPU; the host only admits, launches the captured step graph and
 *     harvests finished sequences.
 *
 * All functions return 0 on success or a negative CT_E* code; none exits.
 */
#ifndef CT_ENGINE_H
#define CT_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#include "ct_model_types.h"

#ifdef __cplusplus
extern "C" {
#endif

#define CT_OK 0
#define CT_EINVAL (-1)      /* bad argument */
#define CT_ENOMEM (-2)      /* device or page-pool allocation failed */
#define CT_EBUSY (-3)       /* no free slot / pages: retry after harvesting */
#define CT_EDEVICE (-4)     /* a CUDA call failed */
#define CT_ETIMEDOUT (-5)   /* a bounded device wait gave up (status word set) */

typedef struct ct_engine ct_engine;

typedef struct {
    int max_slots;       /* concurrent sequences (default 256, max 1024) */
    int max_rows;        /* packed query rows per step (default and maximum 1024) */
    int kv_pages;        /* pages in the pool; 0 = size for max_slots full-length sequences */
    int precision;       /* 1 = activations as bf16 hi+lo planes (near fp32, default), 0 = bf16 */
    int n_prompt;        /* default prompt length (default 10, at most 96) */
    const int *prompt;   /* prompt tokens (default: transcribe.c:1320-1330 with a synthetic language id) */
    int profile;         /* 1 = capture CUDA event nodes around the attention and FFN launches of
                            every layer (per-kernel-class device times in ct_engine_stats); the
                            event nodes serialise their neighbours, so timed runs leave this 0 */
    int no_pdl;          /* 1 = launch step kernels without programmatic dependent launch */
    int enc_max_utts;    /* encoder batch: utterances (default 64; < 0 = no encoder) */
    int enc_max_frames;  /* encoder batch: log-mel frames in total (default 64 x 3001, 30 s each) */
    int keep_logits;     /* 1 = also store every step's fp32 logits for ct_engine_last_logits; 0 (default):
                            the LM head hands only per-tile maxima to the greedy argmax in its epilogue */
    int fused_step;      /* 1 = run each decode step as one persistent kernel (one CTA per SM, grid
                            barriers between its phases) instead of ~70 separate launches; same
                            results bit for bit.  Needs the whole GPU: one such engine per device */
} ct_engine_config;

typedef struct {
    long long utt_id;
    int n_tokens;        /* generated tokens, EOS included */
    int status;          /* 0 ok */
} ct_result;

/* w_host: the reference weight table (host pointers into host_blob). */
int ct_engine_create(ct_engine **out, int device, const void *host_blob, size_t bytes, const Weights *w_host,
                     const ct_engine_config *cfg);
void ct_engine_destroy(ct_engine *e);

/* Prompt of the utterances submitted from now on (any of the submit calls):
 * 1 to 96 tokens -- the reference's 10 (transcribe.c:1320-1330: language,
 * punctuation, ITN, timestamp and diarisation variants), or its long-form
 * prompts with up to 64 tokens carried over from the previous chunk inserted
 * after the first two (transcribe.c:484-532).  prompt == NULL restores the
 * engine's default.  Utterances with different prompts, of any lengths,
 * decode together in one packed batch. */
int ct_engine_set_prompt(ct_engine *e, const int *prompt, int n_prompt);

/* Queue one utterance from its encoder output enc_h (host, fp32 [T_enc, DEC_D],
 * the rows model.h's encoder_forward_batch produces).  forced_len > 0 forces EOS
 * as the forced_len-th generated token (natural EOS before it is ignored);
 * forced_len == 0 decodes until EOS or MAX_SEQ. */
int ct_engine_submit_encoded(ct_engine *e, long long utt_id, const float *enc_h, int T_enc, int forced_len);

/* Encode n utterances (host log-mel mel[b] = [N_MELS][T_mel[b]], the layout
 * compute_mel writes, transcribe.c:177-214) with the packed Conformer encoder
 * (model.h:573-609).  enc_h (host) receives the encoder outputs of all
 * utterances back to back, fp32 [sum T_enc, DEC_D]; T_enc[b] their lengths
 * (transcribe.c:268-271).  At most enc_max_utts / enc_max_frames per call. */
int ct_engine_encode(ct_engine *e, int n, const float *const *mel, const int *T_mel, float *enc_h, int *T_enc);

/* Queue one utterance from its log-mel [N_MELS][T_mel] (host).  Queued
 * utterances are encoded in packed batches by ct_engine_step / ct_engine_run
 * and then decoded like ct_engine_submit_encoded ones. */
int ct_engine_submit_mel(ct_engine *e, long long utt_id, const float *mel, int T_mel, int forced_len);

/* Queue one utterance from 16 kHz mono samples (host, n_samples >= 160): the
 * engine computes its log-mel on the GPU (the front-end of transcribe.c:177-214)
 * and then encodes and decodes it like ct_engine_submit_mel input. */
int ct_engine_submit_audio(ct_engine *e, long long utt_id, const float *samples, int n_samples, int forced_len);

/* The GPU log-mel front-end alone: n utterances of 16 kHz samples (host) ->
 * mel_out (host), utterance b's [N_MELS][T_mel[b]] block after those of
 * utterances 0 .. b-1, T_mel = 1 + n_samples / 160 (transcribe.c:268). */
int ct_engine_log_mel(ct_engine *e, int n, const float *const *samples, const int *n_samples, float *mel_out);

/* Run up to n_steps packed steps (admitting queued utterances when slots and
 * pages allow).  Step graphs are queued back to back and the host synchronises
 * every 32 steps (every 8 while utterances wait for admission, and after the
 * last), harvesting finished sequences and admitting new ones at those points.
 * Returns the number of sequences still queued or live, or a negative error. */
int ct_engine_step(ct_engine *e, int n_steps);

/* Run until every submitted utterance has finished. */
int ct_engine_run(ct_engine *e);

/* Finished utterances (up to max), oldest first.  tokens (optional) receives
 * each result's generated tokens at tokens + i * tok_stride. */
int ct_engine_poll(ct_engine *e, ct_result *out, int max, int *tokens, int tok_stride);

/* Counters since creation.  Device times come from CUDA events on the engine's
 * stream; the per-kernel-class times from event nodes captured inside the step
 * graphs around those launches. */
typedef struct {
    long long steps, rows, tokens, admitted;
    double step_ms;          /* step graphs */
    double admit_ms;         /* admission compute: cross K/V projection into pages */
    double self_attn_ms;     /* paged self-attention kernels (all layers; profile = 1 only) */
    double cross_attn_ms;    /* paged cross-attention kernels (all layers; profile = 1 only) */
    double ffn_ms;           /* FFN1 + FFN2 GEMMs (all layers; profile = 1 only) */
    double self_kv_bytes;    /* algorithmic K/V bytes the self-attention launches read */
    double cross_kv_bytes;   /* algorithmic K/V bytes the cross-attention launches read */
    double ffn_bytes;        /* algorithmic bytes of the FFN GEMMs (weights + activations) */
    long long attn_launches; /* self + cross attention launches (main kernel, per layer) */
    long long ffn_launches;
    long long kernel_launches; /* kernels of this library launched (graph kernel nodes + admission) */
    double enc_ms;           /* encoder batches (subsampling + 48 Conformer layers + projection) */
    long long enc_utts, enc_frames;
} ct_engine_stats_t;
int ct_engine_stats(ct_engine *e, ct_engine_stats_t *out);

/* Device time (ms) of each packed step run since the previous call, oldest
 * first: up to max values are copied to out, the log is cleared, and the number
 * copied is returned. */
int ct_engine_step_times(ct_engine *e, float *out, int max);

/* Profile mode: JSON object {label: [total device ms, launches]} of every
 * launch group of the step graph, from the event nodes between them.
 * Returns the JSON length (written truncated to cap - 1 bytes). */
int ct_engine_profile_report(ct_engine *e, char *buf, int cap);

/* Logits of the most recent packed step, for checking them against a
 * reference (model.h:721-744 computes the same [B, VOCAB] logits before its
 * argmax, backend_lm_head_batch, backends/backend.h:192-194).  For each
 * sequence of that step, up to max: its VOCAB fp32 logits at
 * logits + i * VOCAB (the row the greedy argmax chose from), its utterance id
 * in utt_ids[i] and, in gen_index[i], which generated token they chose (0 =
 * the token after the prompt).  Call it after ct_engine_step(e, 1), before the
 * next step.  Needs keep_logits = 1 in the configuration (else CT_EINVAL).
 * Returns the number of sequences written. */
int ct_engine_last_logits(ct_engine *e, float *logits, long long *utt_ids, int *gen_index, int max);

/* Read (and clear) the device status word; 0 when no kernel reported a problem. */
int ct_engine_status(ct_engine *e);

#ifdef __cplusplus
}
#endif
#endif
