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
    const int *qtile;              // relative-position attention work list: utterance << 16 | first query row
    int n_qtiles;
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

// LayerNorm (eps 1e-5, biased variance; backends/cpu/backend.c:109-122) of
// packed rows of width D, one warp per row (40 values per lane in registers):
// optional fp32 output y (may alias x) and bf16 hi/lo planes.
__global__ void __launch_bounds__(256) ln_enc(const float *x, int R, const bf16 *w, const bf16 *b, float *y,
                                              bf16 *hi, bf16 *lo) {
    constexpr int NV = D / 128;   // float4 per lane
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    if (r >= R) return;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)r * D);
    float4 v[NV];
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        v[j] = xr[lane + 32 * j];
        s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
    const float mean = warp_sum(s) / D;
    float var = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const float a = v[j].x - mean, b2 = v[j].y - mean, c = v[j].z - mean, d = v[j].w - mean;
        var += (a * a + b2 * b2) + (c * c + d * d);
    }
    const float inv = 1.0f / sqrtf(warp_sum(var) / D + 1e-5f);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int k = 4 * (lane + 32 * j);
        const float o[4] = {(v[j].x - mean) * inv * bf2f(w[k]) + bf2f(b[k]),
                            (v[j].y - mean) * inv * bf2f(w[k + 1]) + bf2f(b[k + 1]),
                            (v[j].z - mean) * inv * bf2f(w[k + 2]) + bf2f(b[k + 2]),
                            (v[j].w - mean) * inv * bf2f(w[k + 3]) + bf2f(b[k + 3])};
        if (y) *reinterpret_cast<float4 *>(y + (size_t)r * D + k) = make_float4(o[0], o[1], o[2], o[3]);
        if (hi) {
            bf16 h4[4], l4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                h4[e] = __float2bfloat16_rn(o[e]);
                l4[e] = __float2bfloat16_rn(o[e] - __bfloat162float(h4[e]));
            }
            *reinterpret_cast<uint2 *>(hi + (size_t)r * D + k) = *reinterpret_cast<const uint2 *>(h4);
            if (lo) *reinterpret_cast<uint2 *>(lo + (size_t)r * D + k) = *reinterpret_cast<const uint2 *>(l4);
        }
    }
}

// Relative-position attention over packed rows (backends/cpu/backend.c:262-295),
// fp32 throughout.  One CTA per (query tile of RQ rows of one utterance, head);
// key tiles of RQ keys; the DK = 160 dimensions are staged through shared
// memory in chunks of RC.  Thread (ty, tx) of 16 x 16 owns a 4 x 4 block of
// the score tile: queries ty*4 + i, keys tx*4 + j.  Both score terms
//   AC[q][k] = (Q[q] + u) . K[k]          BD[q][k] = (Q[q] + v) . P[k - q + T_max - 1]
// are accumulated together; the P rows a tile needs form a band of 2*RQ - 1
// consecutive rows (relative offset k - q from -(RQ-1) to RQ-1), of which a
// thread's block reads 7 consecutive ones.  Online softmax per query row (the
// 16 threads of a row are 16 consecutive lanes), probabilities to shared
// memory, then O[q][c] += p[q][k] V[k][c] with thread (ty, tx) owning rows
// ty*4 + i and columns tx + 16*jj.  QKV rows hold [Q | K | V] (stride 3D); P
// is the projected table of 2*T_max - 1 rows.  Output: bf16 hi/lo planes.
constexpr int RQ = 64, RC = 32, RPAD = 4;
constexpr int RP_ROWS = 2 * RQ;   // band of 2*RQ - 1 rows, padded to a multiple of 4
struct RelposSmem {
    union {
        struct {
            float qu[RC][RQ + RPAD], qv[RC][RQ + RPAD], k[RC][RQ + RPAD], p[RC][RP_ROWS + RPAD];
        } c;                       // score phase: one chunk of dimensions, transposed (d-major)
        float v[RQ][DK];           // value phase
    } u;
    float pr[RQ][RQ + RPAD];       // probabilities of the key tile
};

__global__ void __launch_bounds__(256) relpos_flash(const float *QKV, const float *P, Batch b, const bf16 *pbu,
                                                    const bf16 *pbv, bf16 *hi, bf16 *lo) {
    extern __shared__ __align__(16) uint8_t relpos_raw[];
    RelposSmem &sm = *reinterpret_cast<RelposSmem *>(relpos_raw);
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int h = blockIdx.y;
    const int wq = b.qtile[blockIdx.x];
    const int u = wq >> 16, q0 = wq & 0xFFFF;
    const int base = b.r3_off[u];
    const int T = b.r3_off[u + 1] - base;
    const int Tm = b.T_max, PL = 2 * Tm - 1;
    const float scale = 1.0f / sqrtf((float)DK);
    const size_t ld = (size_t)3 * D;

    float o[4][DK / 16];
    float m[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int jj = 0; jj < DK / 16; ++jj) o[i][jj] = 0.0f;
    }

    for (int k0 = 0; k0 < T; k0 += RQ) {
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[i][j] = 0.0f;
        // band row m <-> relative offset (k - q) = (k0 - q0) - (RQ - 1) + m
        const int rb = (k0 - q0) - (RQ - 1) + Tm - 1;
        for (int d0 = 0; d0 < DK; d0 += RC) {
            // ---- stage the chunk [d0, d0 + RC) of Q+u, Q+v, K (RQ rows) and the P band
            {
                const int r = tid >> 2, dd = (tid & 3) * 8;   // 64 rows x 4 groups of 8 dims
                const int q = q0 + r, k = k0 + r;
                float4 qa = make_float4(0.f, 0.f, 0.f, 0.f), qb = qa, ka = qa, kb2 = qa;
                if (q < T) {
                    const float4 *src = reinterpret_cast<const float4 *>(QKV + (size_t)(base + q) * ld + h * DK + d0 + dd);
                    qa = src[0]; qb = src[1];
                }
                if (k < T) {
                    const float4 *src = reinterpret_cast<const float4 *>(QKV + (size_t)(base + k) * ld + D + h * DK + d0 + dd);
                    ka = src[0]; kb2 = src[1];
                }
                const float qv8[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                const float kv8[8] = {ka.x, ka.y, ka.z, ka.w, kb2.x, kb2.y, kb2.z, kb2.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int d = dd + e;
                    sm.u.c.qu[d][r] = qv8[e] + bf2f(pbu[h * DK + d0 + d]);
                    sm.u.c.qv[d][r] = qv8[e] + bf2f(pbv[h * DK + d0 + d]);
                    sm.u.c.k[d][r] = kv8[e];
                }
                // P band: 2*RQ - 1 rows; rows outside the table (only reached by
                // padded queries or keys, whose scores are discarded) read as 0
                for (int idx = tid; idx < RP_ROWS * (RC / 4); idx += 256) {
                    const int mrow = idx / (RC / 4), d4 = (idx % (RC / 4)) * 4;
                    const int pr = rb + mrow;
                    float4 pv = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (mrow < 2 * RQ - 1 && pr >= 0 && pr < PL)
                        pv = *reinterpret_cast<const float4 *>(P + (size_t)pr * D + h * DK + d0 + d4);
                    sm.u.c.p[d4 + 0][mrow] = pv.x;
                    sm.u.c.p[d4 + 1][mrow] = pv.y;
                    sm.u.c.p[d4 + 2][mrow] = pv.z;
                    sm.u.c.p[d4 + 3][mrow] = pv.w;
                }
            }
            __syncthreads();
            // ---- scores: block rows ty*4+i, keys tx*4+j; band index
            // (tx*4 + j) - (ty*4 + i) + RQ - 1 = mb + (j - i) + 3
            const int mb = (tx - ty) * 4 + RQ - 4;
#pragma unroll 4
            for (int d = 0; d < RC; ++d) {
                const float4 a = *reinterpret_cast<const float4 *>(&sm.u.c.qu[d][ty * 4]);
                const float4 c = *reinterpret_cast<const float4 *>(&sm.u.c.qv[d][ty * 4]);
                const float4 kk = *reinterpret_cast<const float4 *>(&sm.u.c.k[d][tx * 4]);
                const float4 p0 = *reinterpret_cast<const float4 *>(&sm.u.c.p[d][mb]);
                const float4 p1 = *reinterpret_cast<const float4 *>(&sm.u.c.p[d][mb + 4]);
                const float av[4] = {a.x, a.y, a.z, a.w}, cv[4] = {c.x, c.y, c.z, c.w};
                const float kv[4] = {kk.x, kk.y, kk.z, kk.w};
                const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) sc[i][j] += av[i] * kv[j] + cv[i] * pv[j - i + 3];
            }
            __syncthreads();
        }
        // ---- online softmax over this key tile
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float rmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const bool valid = k0 + tx * 4 + j < T;
                sc[i][j] = valid ? sc[i][j] * scale : -INFINITY;
                rmax = fmaxf(rmax, sc[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
            const float mn = fmaxf(m[i], rmax);   // finite: key k0 is valid
            const float corr = expf(m[i] - mn);
            float rs = 0.0f;
            float pj[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) { pj[j] = expf(sc[i][j] - mn); rs += pj[j]; }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
            l[i] = l[i] * corr + rs;
            m[i] = mn;
#pragma unroll
            for (int jj = 0; jj < DK / 16; ++jj) o[i][jj] *= corr;
            *reinterpret_cast<float4 *>(&sm.pr[ty * 4 + i][tx * 4]) = make_float4(pj[0], pj[1], pj[2], pj[3]);
        }
        // ---- value tile (aliases the chunk buffers, free after the last sync)
        for (int idx = tid; idx < RQ * (DK / 4); idx += 256) {
            const int r = idx / (DK / 4), c4 = (idx % (DK / 4)) * 4;
            float4 vv = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k0 + r < T) vv = *reinterpret_cast<const float4 *>(QKV + (size_t)(base + k0 + r) * ld + 2 * D + h * DK + c4);
            *reinterpret_cast<float4 *>(&sm.u.v[r][c4]) = vv;
        }
        __syncthreads();
        const int kn = min(RQ, T - k0);
        for (int kk = 0; kk < kn; ++kk) {
            float pq[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) pq[i] = sm.pr[ty * 4 + i][kk];
#pragma unroll
            for (int jj = 0; jj < DK / 16; ++jj) {
                const float vv = sm.u.v[kk][tx + 16 * jj];
#pragma unroll
                for (int i = 0; i < 4; ++i) o[i][jj] += pq[i] * vv;
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int q = q0 + ty * 4 + i;
        if (q >= T) continue;
        const float inv = 1.0f / l[i];
#pragma unroll
        for (int jj = 0; jj < DK / 16; ++jj) {
            const float v = o[i][jj] * inv;
            const size_t idx = (size_t)(base + q) * D + h * DK + tx + 16 * jj;
            const bf16 hb = __float2bfloat16_rn(v);
            hi[idx] = hb;
            if (lo) lo[idx] = __float2bfloat16_rn(v - __bfloat162float(hb));
        }
    }
}

// GLU(pw1) -> depthwise conv (kernel CK, same padding inside the utterance) ->
// eval BatchNorm -> SiLU (backends/cpu/backend.c:304-334); output bf16 planes.
// Block = GR packed rows x GC channels: the GLU of rows [r0 - pad, r0 + GR +
// pad) is computed once into shared memory (coalesced along channels), then
// each output sums its CK taps from there, skipping taps outside its own
// utterance.
constexpr int GR = 32, GC = 128;
__global__ void __launch_bounds__(256) glu_dw_packed(const float *pw1, Batch b, const bf16 *dww, const bf16 *dwb,
                                                     const bf16 *bnw, const bf16 *bnb, const bf16 *bnm,
                                                     const bf16 *bnv, bf16 *hi, bf16 *lo) {
    constexpr int pad = (CK - 1) / 2, HR = GR + CK - 1;
    __shared__ float g_s[HR][GC];
    const int r0 = blockIdx.x * GR, c0 = blockIdx.y * GC;
    const int tc = threadIdx.x & (GC - 1), tr = threadIdx.x / GC;   // 2 row lanes x 128 channels
    const int c = c0 + tc;
    for (int hr = tr; hr < HR; hr += 256 / GC) {
        const int row = r0 - pad + hr;
        float gv = 0.0f;
        if (row >= 0 && row < b.R3) {
            const float a = pw1[(size_t)row * 2 * D + c];
            const float g = pw1[(size_t)row * 2 * D + D + c];
            gv = a / (1.0f + expf(-g));
        }
        g_s[hr][tc] = gv;
    }
    float wk[CK];
#pragma unroll
    for (int k = 0; k < CK; ++k) wk[k] = bf2f(dww[c * CK + k]);
    const float bias = bf2f(dwb[c]);
    const float bn_scale = bf2f(bnw[c]) / sqrtf(bf2f(bnv[c]) + 1e-5f), bn_mean = bf2f(bnm[c]), bn_b = bf2f(bnb[c]);
    __syncthreads();
    for (int rr = tr; rr < GR; rr += 256 / GC) {
        const int row = r0 + rr;
        if (row >= b.R3) break;
        const int u = b.row_utt3[row];
        const int lo_row = b.r3_off[u], hi_row = b.r3_off[u + 1];
        float sum = bias;
#pragma unroll
        for (int k = 0; k < CK; ++k) {
            const int ti = row - pad + k;
            if (ti >= lo_row && ti < hi_row) sum += wk[k] * g_s[rr + k][tc];
        }
        float v = (sum - bn_mean) * bn_scale + bn_b;
        v = v / (1.0f + expf(-v));
        const size_t i = (size_t)row * D + c;
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
    // profile mode: events recorded between kernel groups, with the label of
    // the group each closes (labels[0] is unused)
    bool prof = false;
    std::vector<cudaEvent_t> ev;
    std::vector<const char *> labels;
    int n_marks = 0;
};

static void mark(cudaStream_t s, State &st, const char *label) {
    if (!st.prof) return;
    if (st.n_marks >= (int)st.ev.size()) {
        cudaEvent_t e;
        CT_CHECK(cudaEventCreate(&e));
        st.ev.push_back(e);
        st.labels.push_back(nullptr);
    }
    st.labels[st.n_marks] = label;
    CT_CHECK(cudaEventRecord(st.ev[st.n_marks], s));
    ++st.n_marks;
}

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
              ealloc(st, &st.tab, (size_t)9 * max_utts + 8 + st.R1_max + st.R2_max + st.R3_max + st.R3_max / RQ + 1);
    const size_t hidn = std::max((size_t)R * FF, (size_t)st.R2_max * F2 * C);
    for (int k = 0; k < (two ? 2 : 1); ++k)
        ok = ok && ealloc(st, &st.xa[k], R * D) && ealloc(st, &st.hid[k], hidn) && ealloc(st, &st.ap[k], R * D) &&
             ealloc(st, &st.posp[k], (size_t)(2 * st.T_cap) * D);
    return ok;
}

static void state_free(State &st) {
    for (void *p : st.owned) cudaFree(p);
    st.owned.clear();
    for (cudaEvent_t e : st.ev) cudaEventDestroy(e);
    st.ev.clear();
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
    // attention work list: query tiles, longest utterances first
    std::vector<int> qt;
    {
        std::vector<int> order(n);
        for (int b = 0; b < n; ++b) order[b] = b;
        std::stable_sort(order.begin(), order.end(),
                         [&](int a, int c) { return r3[a + 1] - r3[a] > r3[c + 1] - r3[c]; });
        for (int b : order)
            for (int q0 = 0; q0 < r3[b + 1] - r3[b]; q0 += RQ) qt.push_back(b << 16 | q0);
    }
    const int NQ = (int)qt.size();
    std::vector<int> &h = st.htab;
    h.assign((size_t)5 * n + 3 + R1 + R2 + R3 + NQ, 0);
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
    memcpy(u3 + R3, qt.data(), sizeof(int) * NQ);
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
    bt.qtile = bt.row_utt3 + R3;
    bt.n_qtiles = NQ;
    static thread_local int relpos_dev = -1;
    int dev = 0;
    CT_CHECK(cudaGetDevice(&dev));
    if (relpos_dev != dev) {
        CT_CHECK(cudaFuncSetAttribute(relpos_flash, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(RelposSmem)));
        relpos_dev = dev;
    }
    const Weights_ &w = st.w;
    bf16 *hidp[2] = {st.hid[0], st.hid[1]};
    st.n_marks = 0;
    mark(s, st, "");
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
    mark(s, st, "enc_subsampling");
    // ---- relative positional table for T_max (backends/cpu/backend.c:231-242) ----
    const int PL = 2 * T_max - 1;
    make_rel_pos_emb(s, st.pos, T_max, D);
    split_fp32_to_bf16(s, st.pos, PL, D, D, st.posp[0], st.two ? st.posp[1] : nullptr, D);
    mark(s, st, "enc_pos_table");
    bf16 *xap[2] = {st.xa[0], st.xa[1]}, *app[2] = {st.ap[0], st.ap[1]};
    bf16 *lo_a = st.two ? st.xa[1] : nullptr, *lo_h = st.two ? st.hid[1] : nullptr, *lo_p = st.two ? st.ap[1] : nullptr;
    const int RT = st.R3_max;
    // ---- Conformer layers (model.h:276-314) ----
    for (int l = 0; l < NL; ++l) {
        const Layer &L = w.L[l];
        // FFN1: x += 0.5 * W2 silu(W1 LN(x) + b1) + b2
        ln_enc<<<(R3 + 7) / 8, 256, 0, s>>>(st.x, R3, L.ff1_lnw, L.ff1_lnb, nullptr, st.xa[0], lo_a);
        mark(s, st, "enc_layernorm");
        GemmEpilogue f1;
        f1.epi = EPI_BF16; f1.act = 1; f1.bias = L.ff1_b1; f1.Ybf = st.hid[0]; f1.Ybf_lo = lo_h; f1.ldy = FF;
        egemm_enc(s, st, L.ff1_w1, FF, D, xap, R3, RT, f1);
        mark(s, st, "enc_gemm_ffn1");
        GemmEpilogue f2;
        f2.epi = EPI_FMADD; f2.scale = 0.5f; f2.bias = L.ff1_b2; f2.Y = st.x; f2.ldy = D;
        egemm_enc(s, st, L.ff1_w2, D, FF, hidp, R3, RT, f2);
        mark(s, st, "enc_gemm_ffn2");
        // relative-position self-attention: x += Wo attn(LN(x)) + bo
        ln_enc<<<(R3 + 7) / 8, 256, 0, s>>>(st.x, R3, L.sa_lnw, L.sa_lnb, nullptr, st.xa[0], lo_a);
        mark(s, st, "enc_layernorm");
        GemmEpilogue eq;
        eq.bias = L.qkv_b; eq.Y = st.qkv; eq.ldy = 3 * D;
        egemm_enc(s, st, L.qkv_w, 3 * D, D, xap, R3, RT, eq);
        mark(s, st, "enc_gemm_qkv");
        GemmEpilogue ep;
        ep.Y = st.P; ep.ldy = D;
        egemm_enc(s, st, L.sa_pw, D, D, st.posp, PL, 2 * st.T_cap, ep);
        mark(s, st, "enc_gemm_pos");
        relpos_flash<<<dim3(NQ, H), 256, sizeof(RelposSmem), s>>>(st.qkv, st.P, bt, L.sa_pbu, L.sa_pbv, st.ap[0], lo_p);
        mark(s, st, "enc_relpos_attn");
        GemmEpilogue eo2;
        eo2.epi = EPI_FMADD; eo2.scale = 1.0f; eo2.bias = L.sa_ob; eo2.Y = st.x; eo2.ldy = D;
        egemm_enc(s, st, L.sa_ow, D, D, app, R3, RT, eo2);
        mark(s, st, "enc_gemm_o");
        // conv module: x += pw2(silu(bn(dw(glu(pw1(LN(x)))))))
        ln_enc<<<(R3 + 7) / 8, 256, 0, s>>>(st.x, R3, L.cv_lnw, L.cv_lnb, nullptr, st.xa[0], lo_a);
        mark(s, st, "enc_layernorm");
        GemmEpilogue e1;
        e1.bias = L.cv_pw1b; e1.Y = st.qkv; e1.ldy = 2 * D;
        egemm_enc(s, st, L.cv_pw1w, 2 * D, D, xap, R3, RT, e1);
        mark(s, st, "enc_gemm_pw1");
        glu_dw_packed<<<dim3((R3 + GR - 1) / GR, D / GC), 256, 0, s>>>(st.qkv, bt, L.cv_dww, L.cv_dwb, L.cv_bnw, L.cv_bnb,
                                                              L.cv_bnm, L.cv_bnv, st.ap[0], lo_p);
        mark(s, st, "enc_glu_dwconv");
        GemmEpilogue e2;
        e2.epi = EPI_FMADD; e2.scale = 1.0f; e2.bias = L.cv_pw2b; e2.Y = st.x; e2.ldy = D;
        egemm_enc(s, st, L.cv_pw2w, D, D, app, R3, RT, e2);
        mark(s, st, "enc_gemm_pw2");
        // FFN2
        ln_enc<<<(R3 + 7) / 8, 256, 0, s>>>(st.x, R3, L.ff2_lnw, L.ff2_lnb, nullptr, st.xa[0], lo_a);
        mark(s, st, "enc_layernorm");
        GemmEpilogue g1 = f1;
        g1.bias = L.ff2_b1;
        egemm_enc(s, st, L.ff2_w1, FF, D, xap, R3, RT, g1);
        mark(s, st, "enc_gemm_ffn1");
        GemmEpilogue g2 = f2;
        g2.bias = L.ff2_b2;
        egemm_enc(s, st, L.ff2_w2, D, FF, hidp, R3, RT, g2);
        mark(s, st, "enc_gemm_ffn2");
        // x = LN_out(x); its planes feed the next layer's nothing / the projection
        ln_enc<<<(R3 + 7) / 8, 256, 0, s>>>(st.x, R3, L.out_lnw, L.out_lnb, st.x, st.xa[0], lo_a);
        mark(s, st, "enc_layernorm");
    }
    // ---- encoder -> decoder projection (model.h:607) ----
    GemmEpilogue pj;
    pj.bias = w.prb; pj.Y = st.enc_h; pj.ldy = DEC_D;
    egemm_enc(s, st, w.prw, DEC_D, D, xap, R3, RT, pj);
    mark(s, st, "enc_gemm_proj");
    CT_CHECK(cudaGetLastError());
    memcpy(r3_off_out, r3.data(), sizeof(int) * (n + 1));
    return true;
}

}  // namespace enc
}  // namespace ct
