/* ct_backend.h -- the drop-in C ABI exported by libct_b200.so.
 *
 * libct_b200.so exports exactly the 40 `backend_*` symbols that the reference
 * engine's host code (transcribe.c, model.h, tests/test_kernels.c) calls, with
 * identical signatures and semantics.  Each declaration cites the reference
 * declaration it replaces (backends/backend.h:<line>) and the reference CPU
 * implementation whose results it must reproduce (backends/cpu/backend.c:<line>).
 *
 * Conventions (same as the reference CUDA backend, backends/cuda/backend.cu):
 *   - weight pointers are HOST pointers into the blob handed to
 *     backend_weights_upload_blob; the library maps them by byte offset onto
 *     its device copy (one copy per visible GPU);
 *   - activation pointers are device pointers inside the arena returned by
 *     backend_arena_alloc (fp32);
 *   - `tokens`, `S_dev`, `active`, `T_enc` and argmax `out` are host arrays;
 *   - all mutable state (stream, arena, graph cache, per-item counters) is
 *     per host thread; one host thread drives one GPU;
 *   - functions return void; a CUDA failure prints to stderr and exits(1).
 *
 * All compute runs on sm_100a kernels of this library; there is no CPU path.
 */
#ifndef CT_BACKEND_H
#define CT_BACKEND_H

#include "ct_model_types.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- lifecycle / memory (backend.h:20-46) ---------------------------- */
void  backend_init(int device_id);                                  /* backend.h:20 */
void  backend_destroy(void);                                        /* backend.h:21 */
int   backend_num_devices(void);                                    /* backend.h:25 */
void  backend_thread_cleanup(void);                                 /* backend.h:30 */
void  backend_weights_upload_blob(const void *host_base, size_t bytes); /* backend.h:34 */
void *backend_device_ptr(const void *host_ptr);                     /* backend.h:38 */
float *backend_arena_alloc(size_t floats);                          /* backend.h:41 */
void   backend_arena_free(float *arena);                            /* backend.h:42 */
void backend_htod(float *dev_dst, const float *host_src, size_t floats); /* backend.h:45 */
void backend_dtoh(void *host_dst, const void *dev_src, size_t bytes);    /* backend.h:46 */

/* ---- compute primitives (backend.h:52-106; cpu/backend.c:109-387) ----- */
void backend_layernorm(float *dst, const float *src,
                       const uint16_t *w, const uint16_t *b, int T, int D);        /* backend.h:52 */
void backend_linear(float *y, const float *x,
                    const uint16_t *W, const uint16_t *b, int T, int in_d, int out_d); /* backend.h:56 */
void backend_linear_silu(float *y, const float *x,
                         const uint16_t *W, const uint16_t *b, int T, int in_d, int out_d); /* backend.h:58 */
void backend_linear_relu(float *y, const float *x,
                         const uint16_t *W, const uint16_t *b, int T, int in_d, int out_d); /* backend.h:60 */
void backend_linear_fmadd(float *acc, float scale, const float *x,
                          const uint16_t *W, const uint16_t *b, int T, int in_d, int out_d); /* backend.h:63 */
void backend_add_inplace(float *dst, const float *src, int n);                       /* backend.h:67 */
void backend_encoder_subsampling(const float *mel, int T_mel, int T_mel_stride,
                                 float *x_enc, int T_enc, float *work,
                                 const Weights *W);                                    /* backend.h:72 */
void backend_make_rel_pos_emb(float *pe, int T);                                      /* backend.h:77 */
void backend_rel_pos_mhsa(float *x, const float *pos_emb,
                          int T, const ELayer *L, float *work);                        /* backend.h:81 */
void backend_conformer_conv(float *x, int T, const ELayer *L, float *work);           /* backend.h:86 */
void backend_sdp_attn(float *out, const float *q, const float *k, const float *v,
                      const float *mask, int T_q, int T_k, float *work);               /* backend.h:90 */
void backend_embed(float *h, const int *tokens, int S, int pos_start,
                   const uint16_t *etw, const uint16_t *epw,
                   const uint16_t *elnw, const uint16_t *elnb);                       /* backend.h:96 */
void backend_fill_causal_mask(float *mask, int S);                                    /* backend.h:101 */
void backend_lm_head(float *logits_out, const float *last,
                     const uint16_t *etw, const uint16_t *hdb);                       /* backend.h:105 */

/* ---- graph hooks (backend.h:113-138) ---------------------------------- */
#define GRAPH_TAG_ENCODER    0
#define GRAPH_TAG_PRECOMPUTE 1
#define GRAPH_TAG_DECODER    2
void backend_upload_tokens(const int *host_tokens, int S);                            /* backend.h:121 */
int  backend_graph_replay(int tag, int T_enc, int S, int B);                          /* backend.h:128 */
void backend_graph_begin_capture(int tag);                                            /* backend.h:133 */
void backend_graph_end_capture(int tag, int T_enc, int S, int B);                     /* backend.h:138 */

/* ---- device-side sequence counter, B=1 decode (backend.h:147-175) ----- */
void backend_decode_set_S(int n);                                                     /* backend.h:147 */
void backend_decode_inc_S(void);                                                      /* backend.h:152 */
void backend_linear_to_kvcache(float *cache, const float *x,
                               const uint16_t *W, const uint16_t *b,
                               int in_d, int out_d);                                   /* backend.h:159 */
void backend_sdp_attn_devS(float *out, const float *q,
                           const float *k, const float *v, float *work);               /* backend.h:166 */
void backend_embed_decode(float *h,
                          const uint16_t *etw, const uint16_t *epw,
                          const uint16_t *elnw, const uint16_t *elnb);                 /* backend.h:173 */

/* ---- batched decode step (backend.h:185-228; cpu/backend.c:425-500) --- */
void backend_embed_decode_batch(float *h, const int *tokens,
                                const int *S_dev, const int *active, int B,
                                const uint16_t *etw, const uint16_t *epw,
                                const uint16_t *elnw, const uint16_t *elnb);           /* backend.h:185 */
void backend_lm_head_batch(float *logits, const float *h,
                           const uint16_t *etw, const uint16_t *hdb,
                           const int *active, int B);                                  /* backend.h:192 */
void backend_argmax_batch(int *out, const float *logits,
                          const int *active, int B);                                   /* backend.h:198 */
void backend_upload_T_enc(const int *T_enc, int B);                                   /* backend.h:207 */
void backend_linear_to_kvcache_batch(float *cache, const float *x,
                                     const uint16_t *W, const uint16_t *b,
                                     int B, int cache_seq_stride,
                                     int in_d, int out_d);                             /* backend.h:214 */
void backend_sdp_attn_batch_decode_sa(float *out, const float *Q,
                                      const float *K, const float *V,
                                      int T_k_stride, int B, float *work);             /* backend.h:223 */
void backend_sdp_attn_batch_decode_ca(float *out, const float *Q,
                                      const float *K, const float *V,
                                      int T_k_stride, int B, float *work);             /* backend.h:226 */

/* ---- extensions (no counterpart in the reference ABI) -------------------- */

/* Read and clear the device status word that this library's bounded waits and
 * index checks set instead of trapping (0 = nothing reported).  No counterpart
 * in the reference. */
int ct_device_status(void);

/* Self-test of the bounded device waits.  No counterpart in the reference
 * (its kernels never wait on one another).  Launches one small kernel on the
 * current device that waits, through the same bounded mbarrier wait every
 * pipeline of this library uses, on a barrier phase that nothing ever
 * completes; after limit_us microseconds (1 .. 1000000) the wait gives up,
 * records `code` (1 .. 255) in the device status word and the kernel returns.
 * The call synchronises, then reads and clears the status word and returns
 * it, so a caller sees `code` when the wait expired as designed; -1 for bad
 * arguments, -4 when a CUDA call failed.  Needs no backend_init and leaves the
 * context usable. */
int ct_selftest_bounded_wait(int limit_us, int code);

/* Batched decode attention that allocates nothing.  No counterpart in the
 * reference: it is the no-allocation form of backend_sdp_attn_batch_decode_sa
 * / _ca for callers that cannot call cudaMalloc -- code running under CUDA
 * graph stream capture (allocation is rejected in global / thread-local
 * capture mode), real-time threads and callbacks that must not take the device
 * synchronisation an allocation can imply, and hosts with a fixed memory
 * budget.  Every argument is caller memory: out/Q [B, DEC_D], K/V
 * [B, T_k_stride, DEC_D] (fp32, device), lens [B] (int, device) = keys per
 * item; stream is a cudaStream_t (NULL = the default stream).  Does not need
 * backend_init.  Its split-KV scratch is a static device array of
 * CT_NOALLOC_ATTN_SCRATCH_FLOATS floats (2 MiB, held by every GPU that loads
 * the library until exit); B * DEC_H * ceil(T_k_stride / 128) * (DEC_DK + 2)
 * must fit in it (e.g. B <= 64 with T_k_stride <= MAX_SEQ), else the call
 * returns CT_NOALLOC_ETOOBIG and launches nothing.  The first call on a device
 * looks up the array's device address (once per device, with that device
 * current) and loads both of its kernels, so make that first call before any
 * stream capture.  Calls share the array: calls that overlap on the GPU race
 * and must be serialised.  A lens[b] above T_k_stride is clamped to it; one of
 * zero or less gives item b an all-zero output row; both set the library's
 * device status word, which ct_device_status reads and clears (that reader
 * needs backend_init on the calling thread).  Returns 0, CT_NOALLOC_EINVAL,
 * CT_NOALLOC_ETOOBIG or CT_NOALLOC_ECUDA; ECUDA is also returned, with nothing
 * launched, when an earlier CUDA error is already pending on the calling
 * thread (that error is left in place for the code that caused it). */
#define CT_NOALLOC_ATTN_SCRATCH_FLOATS (64 * DEC_H * ((MAX_SEQ + 127) / 128) * (DEC_DK + 2))
#define CT_NOALLOC_EINVAL (-1)
#define CT_NOALLOC_ETOOBIG (-2)
#define CT_NOALLOC_ECUDA (-4)
int ct_sdp_attn_batch_decode_noalloc(float *out, const float *Q, const float *K, const float *V,
                                     const int *lens, int T_k_stride, int B, void *stream);

/* The library's tensor-core GEMM on caller-held bf16 activations.  No
 * counterpart in the reference (its linears take fp32 activations,
 * backends/backend.h:56-64): for callers that keep activations as bf16 planes.
 * Y [T, N] fp32 (row stride ldy) = act(X W^T + b) with X = X_hi + X_lo
 * (bf16 [T, K] each; X_lo may be NULL), W bf16 [N, K], b bf16 [N] or NULL;
 * act 0 none, 1 SiLU, 2 ReLU.  All pointers device, 16-byte aligned; K a
 * multiple of 8.  Launches on `stream` (a cudaStream_t, NULL = default) and
 * returns 0, -1 (bad argument) or -4 (launch failed). */
int ct_linear_bf16(float *Y, int ldy, const uint16_t *X_hi, const uint16_t *X_lo, const uint16_t *W,
                   const uint16_t *bias, int T, int K, int N, int act, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* CT_BACKEND_H */
