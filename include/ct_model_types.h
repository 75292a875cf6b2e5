/* ct_model_types.h -- model dimensions and weight-table structs shared by the
 * B200 backend library (libct_b200.so), the CPU oracle and the host drivers.
 *
 * ABI contract: the three structs below are passed by pointer across the
 * backend boundary (backend_encoder_subsampling takes `const Weights *`,
 * backend_rel_pos_mhsa / backend_conformer_conv take `const ELayer *`), so
 * their field order and types must equal the reference's
 * backends/model_types.h:52-77 exactly.  tests/test_abi_layout.py checks every
 * field offset against a table generated from the reference header.
 *
 * Dimensions follow backends/model_types.h:14-37 (cohere-transcribe-03-2026).
 * They are compile-time constants there; here every macro is guarded so a
 * build may override them (the CPU oracle additionally takes a runtime
 * dimension struct, which is how the tiny configuration is run).
 */
#ifndef CT_MODEL_TYPES_H
#define CT_MODEL_TYPES_H

#include <stdint.h>
#include <stddef.h>

/* encoder (Conformer) */
#ifndef ENC_D
#define ENC_D    1280   /* model width */
#endif
#ifndef ENC_FF
#define ENC_FF   5120   /* macaron FFN hidden width */
#endif
#ifndef ENC_H
#define ENC_H    8      /* attention heads */
#endif
#ifndef ENC_DK
#define ENC_DK   160    /* head width */
#endif
#ifndef ENC_N
#define ENC_N    48     /* layers */
#endif
#ifndef ENC_CK
#define ENC_CK   9      /* depthwise conv kernel */
#endif
#ifndef SUB_CH
#define SUB_CH   256    /* subsampling conv channels */
#endif

/* decoder (Transformer with cross-attention) */
#ifndef DEC_D
#define DEC_D    1024
#endif
#ifndef DEC_FF
#define DEC_FF   4096
#endif
#ifndef DEC_H
#define DEC_H    8
#endif
#ifndef DEC_DK
#define DEC_DK   128
#endif
#ifndef DEC_N
#define DEC_N    8
#endif

#ifndef VOCAB
#define VOCAB    16384
#endif
#ifndef MAX_SEQ
#define MAX_SEQ  1024   /* decoder positions (rows of the position table) */
#endif

/* audio front-end (only N_MELS is used on the device path) */
#ifndef N_MELS
#define N_MELS   128
#endif

/* Greedy-decoding special tokens, model.h:24-36. */
#define CT_TOK_EOS 3

/* One Conformer layer: bf16 tensors, pointers into the weight blob. */
typedef struct {
    const uint16_t *ff1_lnw, *ff1_lnb, *ff1_w1, *ff1_b1, *ff1_w2, *ff1_b2;
    const uint16_t *sa_lnw, *sa_lnb, *sa_qw, *sa_qb, *sa_kw, *sa_kb,
                   *sa_vw, *sa_vb, *sa_pw, *sa_ow, *sa_ob, *sa_pbu, *sa_pbv;
    const uint16_t *cv_lnw, *cv_lnb, *cv_pw1w, *cv_pw1b, *cv_dww, *cv_dwb,
                   *cv_bnw, *cv_bnb, *cv_bnmean, *cv_bnvar, *cv_pw2w, *cv_pw2b;
    const uint16_t *ff2_lnw, *ff2_lnb, *ff2_w1, *ff2_b1, *ff2_w2, *ff2_b2;
    const uint16_t *out_lnw, *out_lnb;
} ELayer;

/* One decoder layer: self-attention, cross-attention, ReLU FFN. */
typedef struct {
    const uint16_t *sa_lnw, *sa_lnb, *sa_qw, *sa_qb, *sa_kw, *sa_kb,
                   *sa_vw, *sa_vb, *sa_ow, *sa_ob;
    const uint16_t *ca_lnw, *ca_lnb, *ca_qw, *ca_qb, *ca_kw, *ca_kb,
                   *ca_vw, *ca_vb, *ca_ow, *ca_ob;
    const uint16_t *ffn_lnw, *ffn_lnb, *ffn_w1, *ffn_b1, *ffn_w2, *ffn_b2;
} DLayer;

/* Whole model.  s0..s6 / so = subsampling convs and output linear,
 * pr = encoder->decoder projection, et/ep = token / position embedding
 * (et doubles as the LM head, tied), eln = embedding LayerNorm,
 * dln = final decoder LayerNorm, hdb = LM-head bias. */
typedef struct {
    const uint16_t *s0w, *s0b, *s2w, *s2b, *s3w, *s3b, *s5w, *s5b, *s6w, *s6b, *sow, *sob;
    ELayer enc[ENC_N];
    const uint16_t *prw, *prb;
    const uint16_t *etw, *epw, *elnw, *elnb;
    DLayer dec[DEC_N];
    const uint16_t *dlnw, *dlnb, *hdb;
} Weights;

#endif /* CT_MODEL_TYPES_H */
