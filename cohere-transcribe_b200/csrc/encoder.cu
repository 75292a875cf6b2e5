// encoder.cu -- packed ragged Conformer encoder of the engine.
//
// Restates encoder_forward_batch / conformer_layer (model.h:276-314, :573-609)
// for a batch of utterances packed along one row axis: utterance b owns rows
// [off[b], off[b] + T[b]) of every activation.  Row-wise work (LayerNorm, all
// linear layers, 1x1 convolutions) runs once over all packed rows; the three
// operations that mix rows -- the subsampling convolutions, the relative-
// position attention and the depthwise convolution -- take a row -> utterance
// table and never cross an utterance boundary, so each utterance's result is
// the same as encoding it alone.
//
// Relative positions: the reference builds the position table for T_max and
// gives utterance b the slice starting at row T_max - T[b] (model.h:584-592);
// its score term P[k + T[b] - 1 - q] then reads table row k - q + T_max - 1,
// which no longer depends on T[b].  The projected table P = pos_emb . W_pos is
// therefore computed once per layer for the whole batch.
#include <algorithm>
#include <string.h>
#include <vector>

#include "gemm.cuh"
#include "kernels.cuh"

namespace ct {
namespace enc {

constexpr int D = ENC_D, FF = ENC_FF, H = ENC_H, DK = ENC_DK, NL = ENC_N, CK = ENC_CK, C = SUB_CH;
constexpr int F0 = N_MELS, F1 = (F0 + 1) / 2, F2 = (F1 + 1) / 2, F3 = (F2 + 1) / 2;

struct Layer {
    const bf16 *ff1_lnw, *ff1_lnb, *ff1_w1, *ff1_b1, *ff1_w2, *ff1_b2;
    const bf16 *sa_lnw, *sa_lnb, *sa_pw, *sa_ow, *sa_ob, *sa_pbu, *sa_pbv;
    bf16 *qkv_w, *qkv_b;   // [3D, D] concatenation of linear_q/k/v
    const bf16 *cv_lnw, *cv_lnb, *cv_pw1w, *cv_pw1b, *cv_dww, *cv_dwb, *cv_bnw, *cv_bnb, *cv_bnm, *cv_bnv;
    const bf16 *cv_pw2w, *cv_pw2b;
    const bf16 *ff2_lnw, *ff2_lnb, *ff2_w1, *ff2_b1, *ff2_w2, *ff2_b2;
    const bf16 *out_lnw, *out_lnb;
};

struct Weights_ {
    const bf16 *s0w, *s0b, *s2w, *s2b, *s3w, *s3b, *s5w, *s5b, *s6w, *s6b, *sow, *sob, *prw, *prb;
    Layer L[NL];
};

// Utterance tables of one encoder batch (device arrays, n utterances).
struct Batch {
    int n;
    int *T_mel, *mel_off;          // mel block of utterance b at mel + mel_off[b], [N_MELS][T_mel[b]]
    int *r1_off, *r2_off, *r3_off; // packed row offsets after each stride-2 stage (T1, T2, T_enc), n+1 each
    int *row_utt1, *row_utt2, *row_utt3;   // packed row -> utterance, per stage
    int R1, R2, R3;                // total rows per stage
    int T_max;                     // max T_enc of the batch
};

// ------------------------------------------------------------ kernels -----
// conv0 3x3 stride 2 pad 1 on the (time, mel) plane of each utterance, 1 -> C
// channels, ReLU; output rows packed by utterance, channels last [R1][F1][C].
__global__ void conv0_packed(const float *mel, Batch b, const bf16 *w, const bf16 *bias, float *out) {
    const size_t n = (size_t)b.R1 * F1 * C;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % C), f = (int)((i / C) % F1);
        const int row = (int)(i / ((size_t)C * F1));
        const int u = b.row_utt1[row];
        const int t = row - b.r1_off[u], Tm = b.T_mel[u];
        const float *m = mel + b.mel_off[u];
        float s = bf2f(bias[c]);
        for (int kh = 0; kh < 3; ++kh) {
            const int ih = 2 * t - 1 + kh;
            if (ih < 0 || ih >= Tm) continue;
            for (int kw = 0; kw < 3; ++kw) {
                const int iw = 2 * f - 1 + kw;
                if (iw < 0 || iw >= F0) continue;
                s += m[(size_t)iw * Tm + ih] * bf2f(w[c * 9 + kh * 3 + kw]);
            }
        }
        out[i] = s > 0.0f ? s : 0.0f;
    }
}

// depthwise 3x3 stride 2 pad 1, channels last, per utterance: input rows of
// utterance u are [in_off[u], in_off[u+1]) with Fi bins, output rows
// [out_off[u], out_off[u+1]) with (Fi+1)/2 bins.
__global__ void dw_packed(const float *in, int Fi, const int *in_off, const int *out_off, const int *row_utt_out,
                          int R_out, const bf16 *w, const bf16 *bias, float *out) {
    const int Fo = (Fi + 1) / 2;
    const size_t n = (size_t)R_out * Fo * C;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % C), f = (int)((i / C) % Fo);
        const int row = (int)(i / ((size_t)C * Fo));
        const int u = row_utt_out[row];
        const int t = row - out_off[u];
        const int base = in_off[u], Ti = in_off[u + 1] - base;
        float s = bf2f(bias[c]);
        for (int kh = 0; kh < 3; ++kh) {
            const int ih = 2 * t - 1 + kh;
            if (ih < 0 || ih >= Ti) continue;
            for (int kw = 0; kw < 3; ++kw) {
                const int iw = 2 * f - 1 + kw;
                if (iw < 0 || iw >= Fi) continue;
                s += in[((size_t)(base + ih) * Fi + iw) * C + c] * bf2f(w[c * 9 + kh * 3 + kw]);
            }
        }
        out[i] = s;
    }
}

// LayerNorm (eps 1e-5) of packed rows of width D: optional fp32 output (may
// alias x) and bf16 hi/lo planes.
__global__ void __launch_bounds__(256) ln_enc(const float *x, int R, const bf16 *w, const bf16 *b, float *y,
                                              bf16 *hi, bf16 *lo) {
    __shared__ float red[8];
    const int r = blockIdx.x;
    if (r >= R) return;
    const float *xr = x + (size_t)r * D;
    float v[D / 256];
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < D / 256; ++j) { v[j] = xr[threadIdx.x + 256 * j]; s += v[j]; }
    auto bsum = [&](float a) {
        a = warp_sum(a);
        __syncthreads();
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
        __syncthreads();
        float t = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) t += red[k];
        return t;
    };
    const float mean = bsum(s) / D;
    float var = 0.0f;
#pragma unroll
    for (int j = 0; j < D / 256; ++j) { const float c = v[j] - mean; var += c * c; }
    const float inv = 1.0f / sqrtf(bsum(var) / D + 1e-5f);
#pragma unroll
    for (int j = 0; j < D / 256; ++j) {
        const int k = threadIdx.x + 256 * j;
        const float o = (v[j] - mean) * inv * bf2f(w[k]) + bf2f(b[k]);
        if (y) y[(size_t)r * D + k] = o;
        if (hi) {
            const bf16 h = __float2bfloat16_rn(o);
            hi[(size_t)r * D + k] = h;
            if (lo) lo[(size_t)r * D + k] = __float2bfloat16_rn(o - __bfloat162float(h));
        }
    }
}

// Relative-position attention over packed rows (backends/cpu/backend.c:262-295):
// one warp per (row, head), online softmax over 32-key chunks of the row's own
// utterance.  QKV rows hold [Q | K | V] (stride 3D); P is the projected table
// of 2*T_max - 1 rows; the key k / query q term reads P[k - q + T_max - 1].
// Output: bf16 hi/lo planes [R, D].
__global__ void __launch_bounds__(128) relpos_packed(const float *QKV, const float *P, Batch b, const bf16 *pbu,
                                                     const bf16 *pbv, bf16 *hi, bf16 *lo) {
    __shared__ __align__(16) float qu_s[4][DK];
    __shared__ __align__(16) float qv_s[4][DK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 4 + warp, h = blockIdx.y;
    if (row >= b.R3) return;
    const int u = b.row_utt3[row];
    const int base = b.r3_off[u];
    const int T = b.r3_off[u + 1] - base;
    const int q = row - base;
    float *qu = qu_s[warp], *qv = qv_s[warp];
    for (int d = lane; d < DK; d += 32) {
        const float x = QKV[(size_t)row * 3 * D + h * DK + d];
        qu[d] = x + bf2f(pbu[h * DK + d]);
        qv[d] = x + bf2f(pbv[h * DK + d]);
    }
    __syncwarp();
    const float scale = 1.0f / sqrtf((float)DK);
    float m = -INFINITY, l = 0.0f, o[DK / 32];
#pragma unroll
    for (int j = 0; j < DK / 32; ++j) o[j] = 0.0f;
    for (int k0 = 0; k0 < T; k0 += 32) {
        const int k = k0 + lane;
        float sc = -INFINITY;
        if (k < T) {
            const float4 *kp = reinterpret_cast<const float4 *>(QKV + (size_t)(base + k) * 3 * D + D + h * DK);
            const float4 *pp = reinterpret_cast<const float4 *>(P + (size_t)(k - q + b.T_max - 1) * D + h * DK);
            const float4 *up = reinterpret_cast<const float4 *>(qu);
            const float4 *vp = reinterpret_cast<const float4 *>(qv);
            float ac = 0.0f, bd = 0.0f;
#pragma unroll 8
            for (int i = 0; i < DK / 4; ++i) {
                const float4 kv = kp[i], pv = pp[i], a = up[i], c = vp[i];
                ac += a.x * kv.x; ac += a.y * kv.y; ac += a.z * kv.z; ac += a.w * kv.w;
                bd += c.x * pv.x; bd += c.y * pv.y; bd += c.z * pv.z; bd += c.w * pv.w;
            }
            sc = ac * scale + bd * scale;
        }
        const float mn = fmaxf(m, warp_max(sc));
        const float corr = expf(m - mn);
        const float p = k < T ? expf(sc - mn) : 0.0f;
        l = l * corr + warp_sum(p);
#pragma unroll
        for (int j = 0; j < DK / 32; ++j) o[j] *= corr;
        const int kn = min(32, T - k0);
        for (int kk0 = 0; kk0 < kn; kk0 += 8) {
            float vv[8][DK / 32];
#pragma unroll
            for (int t8 = 0; t8 < 8; ++t8) {
                const int kk = kk0 + t8;
                const float *vrow = QKV + (size_t)(base + k0 + (kk < kn ? kk : 0)) * 3 * D + 2 * D + h * DK;
#pragma unroll
                for (int j = 0; j < DK / 32; ++j) vv[t8][j] = vrow[lane + 32 * j];
            }
#pragma unroll
            for (int t8 = 0; t8 < 8; ++t8) {
                const int kk = kk0 + t8;
                const float pk = __shfl_sync(0xffffffffu, p, kk < 32 ? kk : 0);
                if (kk < kn) {
#pragma unroll
                    for (int j = 0; j < DK / 32; ++j) o[j] += pk * vv[t8][j];
                }
            }
        }
        m = mn;
    }
#pragma unroll
    for (int j = 0; j < DK / 32; ++j) {
        const float v = o[j] / l;
        const size_t idx = (size_t)row * D + h * DK + lane + 32 * j;
        const bf16 hb = __float2bfloat16_rn(v);
        hi[idx] = hb;
        if (lo) lo[idx] = __float2bfloat16_rn(v - __bfloat162float(hb));
    }
}

// GLU(pw1) -> depthwise conv (kernel CK, same padding inside the utterance) ->
// eval BatchNorm -> SiLU (backends/cpu/backend.c:304-334); output bf16 planes.
__global__ void glu_dw_packed(const float *pw1, Batch b, const bf16 *dww, const bf16 *dwb, const bf16 *bnw,
                              const bf16 *bnb, const bf16 *bnm, const bf16 *bnv, bf16 *hi, bf16 *lo) {
    const size_t n = (size_t)b.R3 * D;
    const int pad = (CK - 1) / 2;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(i / D), c = (int)(i % D);
        const int u = b.row_utt3[row];
        const int base = b.r3_off[u];
        const int T = b.r3_off[u + 1] - base;
        const int t = row - base;
        float s = bf2f(dwb[c]);
        for (int k = 0; k < CK; ++k) {
            const int ti = t - pad + k;
            if (ti < 0 || ti >= T) continue;
            const float a = pw1[(size_t)(base + ti) * 2 * D + c];
            const float g = pw1[(size_t)(base + ti) * 2 * D + D + c];
            s += bf2f(dww[c * CK + k]) * (a / (1.0f + expf(-g)));
        }
        float v = (s - bf2f(bnm[c])) / sqrtf(bf2f(bnv[c]) + 1e-5f) * bf2f(bnw[c]) + bf2f(bnb[c]);
        v = v / (1.0f + expf(-v));
        const bf16 hb = __float2bfloat16_rn(v);
        hi[i] = hb;
        if (lo) lo[i] = __float2bfloat16_rn(v - __bfloat162float(hb));
    }
}

// ------------------------------------------------------------ host ------
struct State {
    Weights_ w;
    int max_utts = 0, max_frames = 0;     // capacity: utterances and log-mel frames per batch
    int R1_max = 0, R2_max = 0, R3_max = 0, T_cap = 0;
    bool two = true;                       // activations as hi+lo bf16 planes
    float *mel = nullptr, *s1 = nullptr, *s2 = nullptr, *x = nullptr, *qkv = nullptr, *pos = nullptr, *P = nullptr;
    float *enc_h = nullptr;
    bf16 *xa[2] = {nullptr, nullptr}, *hid[2] = {nullptr, nullptr}, *ap[2] = {nullptr, nullptr};
    bf16 *posp[2] = {nullptr, nullptr};
    int *tab = nullptr;                    // device tables
    std::vector<int> htab;
    std::vector<void *> owned;
};

static int t1_of(int t) { return (t + 1) / 2; }

template <typename T>
static bool ealloc(State &st, T **p, size_t n) {
    if (cudaMalloc(reinterpret_cast<void **>(p), sizeof(T) * (n ? n : 1)) != cudaSuccess) return false;
    st.owned.push_back(*p);
    return true;
}

// Sizes every buffer for `max_utts` utterances of at most `max_frames` log-mel
// frames in total (at most 2^19 frames, about 87 minutes of audio).
static bool state_alloc(State &st, int max_utts, int max_frames, bool two) {
    // the first 1x1 subsampling GEMM tiles R2 * F2 rows in 128-row CTAs along grid.y (<= 65535)
    if (max_utts <= 0 || max_frames <= 0 || max_frames > (1 << 19) || max_utts > (1 << 14)) return false;
    st.max_utts = max_utts;
    st.max_frames = max_frames;
    st.two = two;
    st.R1_max = max_frames / 2 + max_utts;
    st.R2_max = st.R1_max / 2 + max_utts;
    st.R3_max = st.R2_max / 2 + max_utts;
    st.T_cap = st.R3_max;
    const size_t s1 = std::max({(size_t)st.R1_max * F1 * C, (size_t)st.R2_max * F2 * C, (size_t)st.R3_max * C * F3});
    const size_t s2 = std::max((size_t)st.R2_max * F2 * C, (size_t)st.R3_max * F3 * C);
    const size_t R = st.R3_max;
    bool ok = ealloc(st, &st.mel, (size_t)max_frames * F0) && ealloc(st, &st.s1, s1) && ealloc(st, &st.s2, s2) &&
              ealloc(st, &st.x, R * D) && ealloc(st, &st.qkv, R * 3 * D) && ealloc(st, &st.enc_h, R * DEC_D) &&
              ealloc(st, &st.pos, (size_t)(2 * st.T_cap) * D) && ealloc(st, &st.P, (size_t)(2 * st.T_cap) * D) &&
              ealloc(st, &st.tab, (size_t)8 * max_utts + 8 + st.R1_max + st.R2_max + st.R3_max);
    const size_t hidn = std::max((size_t)R * FF, (size_t)st.R2_max * F2 * C);
    for (int k = 0; k < (two ? 2 : 1); ++k)
        ok = ok && ealloc(st, &st.xa[k], R * D) && ealloc(st, &st.hid[k], hidn) && ealloc(st, &st.ap[k], R * D) &&
             ealloc(st, &st.posp[k], (size_t)(2 * st.T_cap) * D);
    return ok;
}

static void state_free(State &st) {
    for (void *p : st.owned) cudaFree(p);
    st.owned.clear();
}

static inline int grid_of(size_t n) {
    size_t b = (n + 255) / 256;
    return (int)std::min<size_t>(std::max<size_t>(b, 1), 148 * 16);
}

static void egemm_enc(cudaStream_t s, const State &st, const bf16 *W, int N, int K, bf16 *const *xp, int T, long x_rows,
                      GemmEpilogue ep) {
    ep.x_rows = x_rows;
    gemm_bf16(s, W, N, K, xp[0], st.two ? xp[1] : nullptr, T, ep, false);
}

// Encode n utterances (host log-mel, mel[b] = [N_MELS][T_mel[b]]) into
// st.enc_h: packed rows [R3, DEC_D], utterance b at rows r3_off[b] ..
// r3_off[b+1] - 1 (returned in r3_off_out, n+1 entries).  Returns false when
// the batch exceeds the capacity.
static bool encode(cudaStream_t s, State &st, int n, const float *const *mel, const int *T_mel, int *r3_off_out) {
    if (n <= 0 || n > st.max_utts) return false;
    // ---- tables (host) ----
    std::vector<int> mel_off(n), r1(n + 1), r2(n + 1), r3(n + 1);
    int frames = 0;
    r1[0] = r2[0] = r3[0] = 0;
    int T_max = 0;
    for (int b = 0; b < n; ++b) {
        if (T_mel[b] <= 0) return false;
        mel_off[b] = frames * F0;
        frames += T_mel[b];
        const int t1 = t1_of(T_mel[b]), t2 = t1_of(t1), t3 = t1_of(t2);
        r1[b + 1] = r1[b] + t1;
        r2[b + 1] = r2[b] + t2;
        r3[b + 1] = r3[b] + t3;
        T_max = std::max(T_max, t3);
    }
    if (frames > st.max_frames || r1[n] > st.R1_max || r2[n] > st.R2_max || r3[n] > st.R3_max || T_max > st.T_cap)
        return false;
    const int R1 = r1[n], R2 = r2[n], R3 = r3[n];
    // device table layout: T_mel[n] mel_off[n] r1[n+1] r2[n+1] r3[n+1] utt1[R1] utt2[R2] utt3[R3]
    std::vector<int> &h = st.htab;
    h.assign((size_t)5 * n + 3 + R1 + R2 + R3, 0);
    int *hp = h.data();
    memcpy(hp, T_mel, sizeof(int) * n);
    memcpy(hp + n, mel_off.data(), sizeof(int) * n);
    memcpy(hp + 2 * n, r1.data(), sizeof(int) * (n + 1));
    memcpy(hp + 3 * n + 1, r2.data(), sizeof(int) * (n + 1));
    memcpy(hp + 4 * n + 2, r3.data(), sizeof(int) * (n + 1));
    int *u1 = hp + 5 * n + 3, *u2 = u1 + R1, *u3 = u2 + R2;
    for (int b = 0; b < n; ++b) {
        for (int r = r1[b]; r < r1[b + 1]; ++r) u1[r] = b;
        for (int r = r2[b]; r < r2[b + 1]; ++r) u2[r] = b;
        for (int r = r3[b]; r < r3[b + 1]; ++r) u3[r] = b;
    }
    CT_CHECK(cudaMemcpyAsync(st.tab, hp, sizeof(int) * h.size(), cudaMemcpyHostToDevice, s));
    for (int b = 0; b < n; ++b)
        CT_CHECK(cudaMemcpyAsync(st.mel + mel_off[b], mel[b], sizeof(float) * F0 * T_mel[b], cudaMemcpyHostToDevice, s));
    Batch bt;
    bt.n = n;
    bt.T_mel = st.tab;
    bt.mel_off = st.tab + n;
    bt.r1_off = st.tab + 2 * n;
    bt.r2_off = st.tab + 3 * n + 1;
    bt.r3_off = st.tab + 4 * n + 2;
    bt.row_utt1 = st.tab + 5 * n + 3;
    bt.row_utt2 = bt.row_utt1 + R1;
    bt.row_utt3 = bt.row_utt2 + R2;
    bt.R1 = R1; bt.R2 = R2; bt.R3 = R3;
    bt.T_max = T_max;
    const Weights_ &w = st.w;
    bf16 *hidp[2] = {st.hid[0], st.hid[1]};
    // ---- subsampling (backends/cpu/backend.c:188-229), channels last ----
    conv0_packed<<<grid_of((size_t)R1 * F1 * C), 256, 0, s>>>(st.mel, bt, w.s0w, w.s0b, st.s1);
    dw_packed<<<grid_of((size_t)R2 * F2 * C), 256, 0, s>>>(st.s1, F1, bt.r1_off, bt.r2_off, bt.row_utt2, R2, w.s2w,
                                                           w.s2b, st.s2);
    split_fp32_to_bf16(s, st.s2, R2 * F2, C, C, hidp[0], st.two ? hidp[1] : nullptr, C);
    GemmEpilogue e3;
    e3.epi = EPI_RELU; e3.bias = w.s3b; e3.Y = st.s1; e3.ldy = C;
    egemm_enc(s, st, w.s3w, C, C, hidp, R2 * F2, (long)st.R2_max * F2, e3);
    dw_packed<<<grid_of((size_t)R3 * F3 * C), 256, 0, s>>>(st.s1, F2, bt.r2_off, bt.r3_off, bt.row_utt3, R3, w.s5w,
                                                           w.s5b, st.s2);
    split_fp32_to_bf16(s, st.s2, R3 * F3, C, C, hidp[0], st.two ? hidp[1] : nullptr, C);
    GemmEpilogue e6;
    e6.epi = EPI_RELU_FLAT; e6.bias = w.s6b; e6.Y = st.s1; e6.ldy = C * F3; e6.flat_f = F3;
    egemm_enc(s, st, w.s6w, C, C, hidp, R3 * F3, (long)st.R3_max * F3, e6);
    split_fp32_to_bf16(s, st.s1, R3, C * F3, C * F3, hidp[0], st.two ? hidp[1] : nullptr, C * F3);
    GemmEpilogue eo;
    eo.bias = w.sob; eo.Y = st.x; eo.ldy = D;
    egemm_enc(s, st, w.sow, D, C * F3, hidp, R3, st.R3_max, eo);
    // ---- relative positional table for T_max (backends/cpu/backend.c:231-242) ----
    const int PL = 2 * T_max - 1;
    make_rel_pos_emb(s, st.pos, T_max, D);
    split_fp32_to_bf16(s, st.pos, PL, D, D, st.posp[0], st.two ? st.posp[1] : nullptr, D);
    bf16 *xap[2] = {st.xa[0], st.xa[1]}, *app[2] = {st.ap[0], st.ap[1]};
    bf16 *lo_a = st.two ? st.xa[1] : nullptr, *lo_h = st.two ? st.hid[1] : nullptr, *lo_p = st.two ? st.ap[1] : nullptr;
    const int RT = st.R3_max;
    // ---- Conformer layers (model.h:276-314) ----
    for (int l = 0; l < NL; ++l) {
        const Layer &L = w.L[l];
        // FFN1: x += 0.5 * W2 silu(W1 LN(x) + b1) + b2
        ln_enc<<<R3, 256, 0, s>>>(st.x, R3, L.ff1_lnw, L.ff1_lnb, nullptr, st.xa[0], lo_a);
        GemmEpilogue f1;
        f1.epi = EPI_BF16; f1.act = 1; f1.bias = L.ff1_b1; f1.Ybf = st.hid[0]; f1.Ybf_lo = lo_h; f1.ldy = FF;
        egemm_enc(s, st, L.ff1_w1, FF, D, xap, R3, RT, f1);
        GemmEpilogue f2;
        f2.epi = EPI_FMADD; f2.scale = 0.5f; f2.bias = L.ff1_b2; f2.Y = st.x; f2.ldy = D;
        egemm_enc(s, st, L.ff1_w2, D, FF, hidp, R3, RT, f2);
        // relative-position self-attention: x += Wo attn(LN(x)) + bo
        ln_enc<<<R3, 256, 0, s>>>(st.x, R3, L.sa_lnw, L.sa_lnb, nullptr, st.xa[0], lo_a);
        GemmEpilogue eq;
        eq.bias = L.qkv_b; eq.Y = st.qkv; eq.ldy = 3 * D;
        egemm_enc(s, st, L.qkv_w, 3 * D, D, xap, R3, RT, eq);
        GemmEpilogue ep;
        ep.Y = st.P; ep.ldy = D;
        egemm_enc(s, st, L.sa_pw, D, D, st.posp, PL, 2 * st.T_cap, ep);
        relpos_packed<<<dim3((R3 + 3) / 4, H), 128, 0, s>>>(st.qkv, st.P, bt, L.sa_pbu, L.sa_pbv, st.ap[0], lo_p);
        GemmEpilogue eo2;
        eo2.epi = EPI_FMADD; eo2.scale = 1.0f; eo2.bias = L.sa_ob; eo2.Y = st.x; eo2.ldy = D;
        egemm_enc(s, st, L.sa_ow, D, D, app, R3, RT, eo2);
        // conv module: x += pw2(silu(bn(dw(glu(pw1(LN(x)))))))
        ln_enc<<<R3, 256, 0, s>>>(st.x, R3, L.cv_lnw, L.cv_lnb, nullptr, st.xa[0], lo_a);
        GemmEpilogue e1;
        e1.bias = L.cv_pw1b; e1.Y = st.qkv; e1.ldy = 2 * D;
        egemm_enc(s, st, L.cv_pw1w, 2 * D, D, xap, R3, RT, e1);
        glu_dw_packed<<<grid_of((size_t)R3 * D), 256, 0, s>>>(st.qkv, bt, L.cv_dww, L.cv_dwb, L.cv_bnw, L.cv_bnb,
                                                              L.cv_bnm, L.cv_bnv, st.ap[0], lo_p);
        GemmEpilogue e2;
        e2.epi = EPI_FMADD; e2.scale = 1.0f; e2.bias = L.cv_pw2b; e2.Y = st.x; e2.ldy = D;
        egemm_enc(s, st, L.cv_pw2w, D, D, app, R3, RT, e2);
        // FFN2
        ln_enc<<<R3, 256, 0, s>>>(st.x, R3, L.ff2_lnw, L.ff2_lnb, nullptr, st.xa[0], lo_a);
        GemmEpilogue g1 = f1;
        g1.bias = L.ff2_b1;
        egemm_enc(s, st, L.ff2_w1, FF, D, xap, R3, RT, g1);
        GemmEpilogue g2 = f2;
        g2.bias = L.ff2_b2;
        egemm_enc(s, st, L.ff2_w2, D, FF, hidp, R3, RT, g2);
        // x = LN_out(x); its planes feed the next layer's nothing / the projection
        ln_enc<<<R3, 256, 0, s>>>(st.x, R3, L.out_lnw, L.out_lnb, st.x, st.xa[0], lo_a);
    }
    // ---- encoder -> decoder projection (model.h:607) ----
    GemmEpilogue pj;
    pj.bias = w.prb; pj.Y = st.enc_h; pj.ldy = DEC_D;
    egemm_enc(s, st, w.prw, DEC_D, D, xap, R3, RT, pj);
    CT_CHECK(cudaGetLastError());
    memcpy(r3_off_out, r3.data(), sizeof(int) * (n + 1));
    return true;
}

}  // namespace enc
}  // namespace ct
