/* ref_harness.c -- drives the REFERENCE model graph (model.h of
 * apaz-cli/cohere-transcribe, included from the reference tree at build time)
 * through whatever library provides the backend_* ABI it is linked with:
 *
 *   oracle/_ref/libref_decode_cpu.so   : + reference backends/cpu/backend.c
 *                                        (the reference's own CPU path; the
 *                                        `bench.py --impl reference` arm)
 *   tests/bin/libref_decode_b200.so    : + libct_b200.so (drop-in check: the
 *                                        unmodified reference caller on the
 *                                        B200 backend)
 *
 * TEST / BENCH INFRASTRUCTURE.  The call sequence restates the host driver of
 * transcribe.c (transcribe_batch, transcribe.c:572-808): arena layout with the
 * same sizing formulas (:597-661), batched encoder (:684-686), CA-KV
 * precompute (:689-690), per-item prefill (:692-728), T_enc upload (:731) and
 * the joint decode loop (:752-795).  Two harness additions, both outside the
 * reference: forced EOS at a per-sequence generated length (the benchmark's
 * deterministic ragged shape) and optional teacher forcing for parity.
 */
#define _GNU_SOURCE
#include <pthread.h>
#include <time.h>

int verbose = 0;

#include "model.h"

/* Copy a table of host weight pointers (same struct as model.h's W). */
void refh_bind_weights(const Weights *w) { W = *w; }

/* Optional logits capture of the next decode calls on this thread: buf
 * [count][cap][VOCAB] receives the logits that chose generated token g of item
 * b for g < cap (g = 0: the prefill's token).  Needs am or margin (the logits
 * are read back only then).  cap = 0 switches it off. */
static __thread float *g_lg_buf = NULL;
static __thread int g_lg_cap = 0;
void refh_capture_logits(float *buf, int cap) { g_lg_buf = buf; g_lg_cap = buf ? cap : 0; }

#ifndef EMBEDDED_MODEL
#include <unistd.h>
/* The reference's own model-file loader (model.h load_weights: sf_load of
 * model_files/model.safetensors, then sf_get of every tensor by its Hugging
 * Face name) run in directory `dir`; the resulting weight table is copied to
 * *out.  A missing tensor makes the reference loader exit(1). */
int refh_load_model_file(const char *dir, Weights *out) {
    char cwd[4096];
    if (!getcwd(cwd, sizeof cwd) || chdir(dir) != 0) return -1;
    load_weights();
    const int rc = chdir(cwd);
    *out = W;
    return rc;
}
#endif

static int t_enc_of(int T_mel) {
    int T1 = (T_mel + 1) / 2, T2 = (T1 + 1) / 2;
    return (T2 + 1) / 2;
}

/* Arena sizing of transcribe.c:597-627 for `count` items. */
static size_t arena_floats_for(int count, int T_mel_max, int T_enc_max) {
    int T1_max = (T_mel_max + 1) / 2, T2_max = (T1_max + 1) / 2;
    size_t n_mel_b  = (size_t)count * N_MELS * T_mel_max;
    size_t n_xenc_b = (size_t)count * T_enc_max * ENC_D;
    size_t n_posemb = (size_t)(2 * T_enc_max - 1) * ENC_D;
    size_t n_ench_b = (size_t)count * T_enc_max * DEC_D;
    size_t n_cakv_b = (size_t)count * DEC_N * T_enc_max * DEC_D;
    size_t n_sakv_b = (size_t)count * DEC_N * MAX_SEQ * DEC_D;
    size_t n_hdec = (size_t)MAX_SEQ * DEC_D, n_mask = (size_t)MAX_SEQ * MAX_SEQ;
    size_t n_logits = (size_t)count * VOCAB, n_h_dec_b = (size_t)count * DEC_D;
    size_t work_sub = (size_t)SUB_CH * ((size_t)T1_max * 64 + (size_t)T2_max * 32);
    size_t mhsa_scores = (size_t)T_enc_max * ((size_t)3 * T_enc_max - 1);
    size_t mhsa_attn = (size_t)2 * T_enc_max * ENC_D;
    size_t mhsa_shared = mhsa_scores > mhsa_attn ? mhsa_scores : mhsa_attn;
    size_t wc_mhsa = (size_t)T_enc_max * ENC_FF + (size_t)T_enc_max * ENC_D
                   + (size_t)(5 * (size_t)T_enc_max - 1) * ENC_D + mhsa_shared;
    size_t wc_conv = (size_t)T_enc_max * (ENC_FF + 4 * ENC_D);
    size_t work_conf = wc_mhsa > wc_conv ? wc_mhsa : wc_conv;
    size_t work_dec = (size_t)5 * MAX_SEQ * DEC_D + (size_t)MAX_SEQ * MAX_SEQ;
    /* the batched decode step puts B*DEC_H*max(MAX_SEQ,T_enc_max) scores in work */
    size_t work_bat = (size_t)3 * count * DEC_D
                    + (size_t)count * DEC_H * (MAX_SEQ > T_enc_max ? MAX_SEQ : T_enc_max);
    size_t work = work_sub;
    if (work_conf > work) work = work_conf;
    if (work_dec > work) work = work_dec;
    if (work_bat > work) work = work_bat;
    return n_mel_b + n_xenc_b + n_posemb + n_ench_b + 2 * n_cakv_b + 2 * n_sakv_b
         + n_hdec + n_mask + n_logits + n_h_dec_b + work;
}

typedef struct {
    float *mel, *x_enc, *pos_emb, *enc_h, *ca_k[DEC_N], *ca_v[DEC_N], *sa_k[DEC_N], *sa_v[DEC_N];
    float *h_dec, *mask, *logits, *h_dec_b, *work;
} Arena;

static void arena_layout(Arena *a, float *base, int count, int T_mel_max, int T_enc_max) {
    size_t off = 0;
    a->mel = base + off;     off += (size_t)count * N_MELS * T_mel_max;
    a->x_enc = base + off;   off += (size_t)count * T_enc_max * ENC_D;
    a->pos_emb = base + off; off += (size_t)(2 * T_enc_max - 1) * ENC_D;
    a->enc_h = base + off;   off += (size_t)count * T_enc_max * DEC_D;
    for (int l = 0; l < DEC_N; l++) { a->ca_k[l] = base + off; off += (size_t)count * T_enc_max * DEC_D; }
    for (int l = 0; l < DEC_N; l++) { a->ca_v[l] = base + off; off += (size_t)count * T_enc_max * DEC_D; }
    for (int l = 0; l < DEC_N; l++) { a->sa_k[l] = base + off; off += (size_t)count * MAX_SEQ * DEC_D; }
    for (int l = 0; l < DEC_N; l++) { a->sa_v[l] = base + off; off += (size_t)count * MAX_SEQ * DEC_D; }
    a->h_dec = base + off;   off += (size_t)MAX_SEQ * DEC_D;
    a->mask = base + off;    off += (size_t)MAX_SEQ * MAX_SEQ;
    a->logits = base + off;  off += (size_t)count * VOCAB;
    a->h_dec_b = base + off; off += (size_t)count * DEC_D;
    a->work = base + off;
}

static void top2(const float *lg, int *idx, float *mg) {
    int best = 0; float bv = lg[0];
    for (int v = 1; v < VOCAB; v++) if (lg[v] > bv) { bv = lg[v]; best = v; }
    float sec = -INFINITY;
    for (int v = 0; v < VOCAB; v++) if (v != best && lg[v] > sec) sec = lg[v];
    *idx = best; *mg = bv - sec;
}

/* Prefill + joint decode from encoder outputs already in the arena (enc_h).
 * am/margin (optional) receive the backend's argmax and top-2 margin per
 * generated position; they require a logits readback each step. */
static void decode_loop(Arena *a, int count, const int *T_mel, const int *T_enc, int T_enc_max,
                        const int *prompt, int n_prompt, const int *forced_len,
                        const int *force_tokens, int *tokens, int *n_tok, int *am, float *margin) {
    int *S = malloc(sizeof(int) * count), *S_dev = malloc(sizeof(int) * count);
    int *active = malloc(sizeof(int) * count), *cur = malloc(sizeof(int) * count);
    int *next = malloc(sizeof(int) * count), *gen = malloc(sizeof(int) * count);
    float *lg_host = (am || margin) ? malloc(sizeof(float) * (size_t)count * VOCAB) : NULL;

    precompute_ca_kv_batch(a->enc_h, count, T_enc, T_enc_max, a->ca_k, a->ca_v);
    for (int b = 0; b < count; b++) {
        int *tb = tokens + (size_t)b * MAX_SEQ;
        for (int i = 0; i < n_prompt; i++) tb[i] = prompt[i];
        float *cak[DEC_N], *cav[DEC_N], *sak[DEC_N], *sav[DEC_N];
        for (int l = 0; l < DEC_N; l++) {
            cak[l] = a->ca_k[l] + (size_t)b * T_enc_max * DEC_D;
            cav[l] = a->ca_v[l] + (size_t)b * T_enc_max * DEC_D;
            sak[l] = a->sa_k[l] + (size_t)b * MAX_SEQ * DEC_D;
            sav[l] = a->sa_v[l] + (size_t)b * MAX_SEQ * DEC_D;
        }
        backend_decode_set_S(n_prompt);
        int id = decoder_step(tb, n_prompt, n_prompt, T_mel[b] + (b + 1) * 100000, T_enc[b],
                              cak, cav, sak, sav, a->h_dec, a->mask, a->work);
        if (am || margin) {
            float mg; int i2;
            backend_dtoh(lg_host, a->work, VOCAB * sizeof(float));
            if (g_lg_cap > 0) memcpy(g_lg_buf + (size_t)b * g_lg_cap * VOCAB, lg_host, sizeof(float) * VOCAB);
            top2(lg_host, &i2, &mg);
            if (am) am[(size_t)b * MAX_SEQ + n_prompt] = i2;
            if (margin) margin[(size_t)b * MAX_SEQ + n_prompt] = mg;
        }
        gen[b] = 1;
        if (force_tokens) id = force_tokens[(size_t)b * MAX_SEQ + n_prompt];
        if (gen[b] >= forced_len[b]) id = TOK_EOS;
        tb[n_prompt] = id;
        S[b] = n_prompt + 1;
    }
    backend_upload_T_enc(T_enc, count);
    int n_active = 0;
    for (int b = 0; b < count; b++) {
        active[b] = gen[b] < forced_len[b] && S[b] < MAX_SEQ;
        n_active += active[b];
        S_dev[b] = S[b] - 1;
    }
    while (n_active > 0) {
        for (int b = 0; b < count; b++) {
            cur[b] = active[b] ? tokens[(size_t)b * MAX_SEQ + S[b] - 1] : 0;
            if (active[b]) S_dev[b]++;
        }
        decoder_step_decode_batch(cur, S_dev, active, T_enc_max, a->ca_k, a->ca_v, a->sa_k,
                                  a->sa_v, a->h_dec_b, a->logits, a->work, count, next);
        if (am || margin)
            backend_dtoh(lg_host, a->logits, (size_t)count * VOCAB * sizeof(float));
        for (int b = 0; b < count; b++) {
            if (!active[b]) continue;
            int id = next[b];
            if (am || margin) {
                float mg; int i2;
                top2(lg_host + (size_t)b * VOCAB, &i2, &mg);
                if (gen[b] < g_lg_cap)
                    memcpy(g_lg_buf + ((size_t)b * g_lg_cap + gen[b]) * VOCAB, lg_host + (size_t)b * VOCAB,
                           sizeof(float) * VOCAB);
                if (am) am[(size_t)b * MAX_SEQ + S[b]] = id;
                if (margin) margin[(size_t)b * MAX_SEQ + S[b]] = mg;
            }
            gen[b]++;
            if (force_tokens) id = force_tokens[(size_t)b * MAX_SEQ + S[b]];
            if (gen[b] >= forced_len[b]) id = TOK_EOS;
            tokens[(size_t)b * MAX_SEQ + S[b]] = id;
            S[b]++;
            if (gen[b] >= forced_len[b] || S[b] >= MAX_SEQ) { active[b] = 0; n_active--; }
        }
    }
    for (int b = 0; b < count; b++) n_tok[b] = S[b];
    free(S); free(S_dev); free(active); free(cur); free(next); free(gen); free(lg_host);
}

/* Decode `count` sequences from host encoder outputs enc_h [count, T_enc_max, DEC_D].
 * The caller has called backend_weights_upload_blob + backend_init on this thread.
 * Returns the elapsed wall seconds of the whole call (upload included). */
double refh_decode_from_enc(int count, const float *enc_h, const int *T_enc, int T_enc_max,
                            const int *prompt, int n_prompt, const int *forced_len,
                            const int *force_tokens, int *tokens, int *n_tok,
                            int *am, float *margin) {
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    int *T_mel = malloc(sizeof(int) * count);
    for (int b = 0; b < count; b++) T_mel[b] = 8 * T_enc[b];   /* graph keys only */
    float *base = backend_arena_alloc(arena_floats_for(count, 8 * T_enc_max, T_enc_max));
    Arena a;
    arena_layout(&a, base, count, 8 * T_enc_max, T_enc_max);
    backend_htod(a.enc_h, enc_h, (size_t)count * T_enc_max * DEC_D);
    decode_loop(&a, count, T_mel, T_enc, T_enc_max, prompt, n_prompt, forced_len, force_tokens,
                tokens, n_tok, am, margin);
    backend_arena_free(base);
    free(T_mel);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    return (t1.tv_sec - t0.tv_sec) + 1e-9 * (t1.tv_nsec - t0.tv_nsec);
}

/* Full pipeline from host log-mel [count, N_MELS, T_mel_max] (zero padded):
 * batched encoder, CA-KV, prefill, decode.  enc_h_out (optional, host
 * [count, T_enc_max, DEC_D]) receives the encoder output.  Returns seconds. */
double refh_transcribe_batch(int count, const float *mel, int T_mel_max, const int *T_mel,
                             const int *prompt, int n_prompt, const int *forced_len,
                             const int *force_tokens, int *tokens, int *n_tok,
                             int *am, float *margin, float *enc_h_out) {
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    int *T_enc = malloc(sizeof(int) * count);
    int T_enc_max = t_enc_of(T_mel_max);
    for (int b = 0; b < count; b++) T_enc[b] = t_enc_of(T_mel[b]);
    float *base = backend_arena_alloc(arena_floats_for(count, T_mel_max, T_enc_max));
    Arena a;
    arena_layout(&a, base, count, T_mel_max, T_enc_max);
    backend_htod(a.mel, mel, (size_t)count * N_MELS * T_mel_max);
    encoder_forward_batch(a.mel, count, T_mel_max, T_mel, T_enc, T_enc_max, a.x_enc, a.pos_emb,
                          a.enc_h, a.work);
    if (enc_h_out)
        backend_dtoh(enc_h_out, a.enc_h, sizeof(float) * (size_t)count * T_enc_max * DEC_D);
    decode_loop(&a, count, T_mel, T_enc, T_enc_max, prompt, n_prompt, forced_len, force_tokens,
                tokens, n_tok, am, margin);
    backend_arena_free(base);
    free(T_enc);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    return (t1.tv_sec - t0.tv_sec) + 1e-9 * (t1.tv_nsec - t0.tv_nsec);
}

/* ---- multi-threaded CPU timing: one host thread per group of sequences,
 * mirroring run_files_parallel (transcribe.c:947-984) with one "device" per
 * core.  Each thread decodes its own slice of the batch. */
typedef struct {
    int dev, count, T_enc_max, n_prompt;
    const float *enc_h; const int *T_enc, *prompt, *forced_len;
    int *tokens, *n_tok;
} Job;

static void *job_main(void *p) {
    Job *j = (Job *)p;
    backend_init(j->dev);
    refh_decode_from_enc(j->count, j->enc_h, j->T_enc, j->T_enc_max, j->prompt, j->n_prompt,
                         j->forced_len, NULL, j->tokens, j->n_tok, NULL, NULL);
    backend_thread_cleanup();
    return NULL;
}

double refh_parallel_decode(int n_threads, int count, const float *enc_h, const int *T_enc,
                            int T_enc_max, const int *prompt, int n_prompt,
                            const int *forced_len, int *tokens, int *n_tok) {
    struct timespec t0, t1;
    if (n_threads > count) n_threads = count;
    pthread_t *th = malloc(sizeof(pthread_t) * n_threads);
    Job *jobs = malloc(sizeof(Job) * n_threads);
    clock_gettime(CLOCK_MONOTONIC, &t0);
    int start = 0;
    for (int i = 0; i < n_threads; i++) {
        int n = count / n_threads + (i < count % n_threads);
        Job *j = &jobs[i];
        j->dev = i; j->count = n; j->T_enc_max = T_enc_max; j->n_prompt = n_prompt;
        j->enc_h = enc_h + (size_t)start * T_enc_max * DEC_D;
        j->T_enc = T_enc + start; j->prompt = prompt; j->forced_len = forced_len + start;
        j->tokens = tokens + (size_t)start * MAX_SEQ; j->n_tok = n_tok + start;
        pthread_create(&th[i], NULL, job_main, j);
        start += n;
    }
    for (int i = 0; i < n_threads; i++) pthread_join(th[i], NULL);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    free(th); free(jobs);
    return (t1.tv_sec - t0.tv_sec) + 1e-9 * (t1.tv_nsec - t0.tv_nsec);
}

/* ---- multi-threaded CPU transcription (encoder + decode): one host thread
 * per group of utterances, as refh_parallel_decode, each thread running
 * refh_transcribe_batch on its slice of the log-mel batch
 * ([count][N_MELS][T_mel_max], zero padded). */
typedef struct {
    int dev, count, T_mel_max, n_prompt;
    const float *mel; const int *T_mel, *prompt, *forced_len;
    int *tokens, *n_tok;
} TJob;

static void *tjob_main(void *p) {
    TJob *j = (TJob *)p;
    backend_init(j->dev);
    refh_transcribe_batch(j->count, j->mel, j->T_mel_max, j->T_mel, j->prompt, j->n_prompt, j->forced_len, NULL,
                          j->tokens, j->n_tok, NULL, NULL, NULL);
    backend_thread_cleanup();
    return NULL;
}

double refh_parallel_transcribe(int n_threads, int count, const float *mel, int T_mel_max, const int *T_mel,
                                const int *prompt, int n_prompt, const int *forced_len, int *tokens, int *n_tok) {
    struct timespec t0, t1;
    if (n_threads > count) n_threads = count;
    pthread_t *th = malloc(sizeof(pthread_t) * n_threads);
    TJob *jobs = malloc(sizeof(TJob) * n_threads);
    clock_gettime(CLOCK_MONOTONIC, &t0);
    int start = 0;
    for (int i = 0; i < n_threads; i++) {
        int n = count / n_threads + (i < count % n_threads);
        TJob *j = &jobs[i];
        j->dev = i; j->count = n; j->T_mel_max = T_mel_max; j->n_prompt = n_prompt;
        j->mel = mel + (size_t)start * N_MELS * T_mel_max;
        j->T_mel = T_mel + start; j->prompt = prompt; j->forced_len = forced_len + start;
        j->tokens = tokens + (size_t)start * MAX_SEQ; j->n_tok = n_tok + start;
        pthread_create(&th[i], NULL, tjob_main, j);
        start += n;
    }
    for (int i = 0; i < n_threads; i++) pthread_join(th[i], NULL);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    free(th); free(jobs);
    return (t1.tv_sec - t0.tv_sec) + 1e-9 * (t1.tv_nsec - t0.tv_nsec);
}
