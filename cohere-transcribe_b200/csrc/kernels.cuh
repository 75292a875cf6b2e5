// kernels.cuh -- non-GEMM kernels of libct_b200.so (host launchers).
#pragma once
#include "ct_common.cuh"

namespace ct {

// ---- LayerNorm (eps 1e-5, biased variance; backends/cpu/backend.c:109-122) --
// dst may alias src.  Optional bf16 copy of the result (dst_bf, same layout).
void layernorm(cudaStream_t st, float *dst, const float *src, const bf16 *w, const bf16 *b, int T, int D,
               bf16 *dst_bf = nullptr);

// h[r] = LN(etw[tok[r]] + epw[p(r)]) for rows r < R, p(r) = pos[r] + pos_off
// (pos a device array) or pos_off + r (pos null).  active (device, optional):
// rows with active[r] == 0 are left untouched.
void embed_ln(cudaStream_t st, float *h, const int *tok, const int *pos, int pos_off, const int *active, int R,
              const bf16 *etw, const bf16 *epw, const bf16 *lnw, const bf16 *lnb, int D, int vocab, int max_pos,
              bf16 *h_bf = nullptr);

void add_inplace(cudaStream_t st, float *dst, const float *src, size_t n);
void fill_causal_mask(cudaStream_t st, float *mask, int S);
void make_rel_pos_emb(cudaStream_t st, float *pe, int T, int D);

// ---- attention over fp32 K/V rows (decoder; backends/cpu/backend.c:339-360) --
// For query row r: out[r] = softmax(Q[r].K^T * scale + mask[r]) . V over the
// first L(r) key rows of item r, per head (H heads of width DK, row width D).
// Key rows of item r start at K + r * kv_item (kv_item = 0: all rows share
// K/V).  L(r) = len_arr ? len_arr[r] : (len_dev ? *len_dev : len_const).
// Split-KV (flash-decoding): fixed 128-key chunks, deterministic combine.
struct AttnRows {
    const float *Q; int ldq;
    const float *K, *V; long kv_item; int ldkv;
    const int *len_arr; const int *len_dev; int len_const; int len_max;
    const float *mask; int mask_ld;   // additive, [R, mask_ld] or null
    float *out; int ldo;
    int R, H, DK;
    float scale;
};
void attn_rows_f32(cudaStream_t st, const AttnRows &a, float *ws, size_t ws_floats);
size_t attn_ws_floats(int R, int H, int DK, int len_max);

// ---- encoder relative-position attention core (backends/cpu/backend.c:262-295)
// out[q] = sum_k softmax_k(((Q[q]+u).K[k] + (Q[q]+v).P[k+T-1-q]) * scale) V[k]
void relpos_attn_f32(cudaStream_t st, const float *Q, const float *K, const float *V, const float *P,
                     const bf16 *pbu, const bf16 *pbv, float *out, int T, int H, int DK, int D);

// ---- conformer conv core: GLU + depthwise conv (same padding) + eval BN + SiLU
// (backends/cpu/backend.c:304-334).  pw1 [T, 2D] -> y [T, D].
void glu_dwconv_bn_silu(cudaStream_t st, const float *pw1, float *y, int T, int D, int CK, const bf16 *dww,
                        const bf16 *dwb, const bf16 *bnw, const bf16 *bnb, const bf16 *bnm, const bf16 *bnv);

// ---- subsampling convs, channels-last activations [T, F, C] ----------------
// conv0: 3x3 stride 2 pad 1, 1 -> C channels, input mel [n_mels, stride] (mel
// bins x frames), + ReLU; output [T1, F1, C].
void sub_conv0(cudaStream_t st, const float *mel, int T_mel, int mel_stride, int n_mels, const bf16 *w,
               const bf16 *b, float *out, int C);
// depthwise 3x3 stride 2 pad 1 on [Ti, Fi, C] -> [To, Fo, C]
void sub_dwconv(cudaStream_t st, const float *in, int Ti, int Fi, int C, const bf16 *w, const bf16 *b, float *out);

// ---- greedy argmax: first index of the row maximum (strict >) -------------
void argmax_rows(cudaStream_t st, const float *logits, int R, int V, const int *active, int *out);

}  // namespace ct
