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

#include "frontend.cu"
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
    const int *qtile2;             // the same with 128-row query tiles (tensor-memory kernel)
    int n_qtiles2;
};

// ------------------------------------------------------------ kernels -----
// The first two subsampling convolutions fused (backends/cpu/backend.c:188-229:
// conv0 3x3/s2 1 -> C + ReLU, then the depthwise 3x3/s2), written as the bf16
// planes the following 1x1 GEMM reads: out[r2 * F2 + f2][c].  One CTA per
// stage-2 row r2 (time step t2 of utterance u), thread = channel c.  The conv0
// activations A[t1][f1][c] that the depthwise stencil needs (t1 = 2 t2 - 1 ..
// 2 t2 + 1, all f1) are recomputed from the 7 log-mel frames 4 t2 - 3 .. 4 t2 + 3
// staged in shared memory, walking f2 left to right with a 3 x 3 window of A
// values in registers (two new A columns per step), so the [R1][F1][C]
// intermediate never reaches memory.  Padding: mel outside the utterance or
// the bins is 0 (conv0's), A outside [0, T1) x [0, F1) is 0 (the depthwise's).
// Summation order per output: conv0 taps (kh, kw) row-major, then depthwise
// taps (kh, kw) row-major, each starting from its bias, as the reference.
constexpr int SUB_TH = 7;   // mel frames per stage-2 row (4 t2 - 3 .. 4 t2 + 3)
// staged bins start at -SUB_LP, so the five bins 4 f2 - 1 .. 4 f2 + 3 that step
// f2 reads sit at columns 4 f2 + 4 .. 4 f2 + 8: one aligned float4 and one float
constexpr int SUB_LP = 5, SUB_W = 136;
static_assert(2 * F2 <= F1 && 4 * (F2 - 1) + 8 < SUB_W && SUB_W % 4 == 0, "staged log-mel columns");
__global__ void __launch_bounds__(C) conv0_dw_planes(const float *mel, Batch b, const bf16 *w0, const bf16 *b0,
                                                     const bf16 *w2, const bf16 *b2, bf16 *hi, bf16 *lo) {
    __shared__ __align__(16) float ms[SUB_TH][SUB_W];   // [frame][bin + SUB_LP], zero outside
    const int r2 = blockIdx.x;
    const int c = threadIdx.x;
    const int u = b.row_utt2[r2];
    const int t2 = r2 - b.r2_off[u];
    const int T1 = b.r1_off[u + 1] - b.r1_off[u], Tm = b.T_mel[u];
    const float *m = mel + b.mel_off[u];
    for (int i = threadIdx.x; i < SUB_TH * SUB_W; i += blockDim.x) {   // frames fastest: a bin's 7 are adjacent
        const int fr = i % SUB_TH, bin = i / SUB_TH - SUB_LP;
        const int t = 4 * t2 - 3 + fr;
        ms[fr][bin + SUB_LP] = (t >= 0 && t < Tm && bin >= 0 && bin < F0) ? m[(size_t)bin * Tm + t] : 0.0f;
    }
    float k0[9], k2[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) { k0[i] = bf2f(w0[c * 9 + i]); k2[i] = bf2f(w2[c * 9 + i]); }
    const float bias0 = bf2f(b0[c]), bias2 = bf2f(b2[c]);
    bool rv[3];   // A rows t1 = 2 t2 - 1 + j inside the utterance
#pragma unroll
    for (int j = 0; j < 3; ++j) { const int t1 = 2 * t2 - 1 + j; rv[j] = t1 >= 0 && t1 < T1; }
    __syncthreads();
    // A[j][f1] for row j (t1 = 2 t2 - 1 + j) uses frames 2 j .. 2 j + 2 and bins
    // 2 f1 - 1 .. 2 f1 + 1; at step f2, f1 = 2 f2 takes bins x[0..2] and
    // f1 = 2 f2 + 1 takes x[2..4] of the frame's five bins x = 4 f2 - 1 .. 4 f2 + 3
    float a[3][3];   // A[j][2 f2 - 1 + i]; A[j][-1] = 0 (the depthwise's padding)
#pragma unroll
    for (int j = 0; j < 3; ++j) a[j][2] = 0.0f;
    const size_t row0 = (size_t)r2 * F2;
#pragma unroll 1
    for (int f2 = 0; f2 < F2; ++f2) {
        float x[SUB_TH][5];
#pragma unroll
        for (int fr = 0; fr < SUB_TH; ++fr) {
            const float4 q = *reinterpret_cast<const float4 *>(&ms[fr][4 * f2 + 4]);
            x[fr][0] = q.x; x[fr][1] = q.y; x[fr][2] = q.z; x[fr][3] = q.w;
            x[fr][4] = ms[fr][4 * f2 + 8];
        }
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            float s0 = bias0, s1 = bias0;   // conv0 taps (kh, kw) row-major, from the bias
#pragma unroll
            for (int kh = 0; kh < 3; ++kh)
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) {
                    s0 += x[2 * j + kh][kw] * k0[kh * 3 + kw];
                    s1 += x[2 * j + kh][kw + 2] * k0[kh * 3 + kw];
                }
            a[j][0] = a[j][2];
            a[j][1] = rv[j] && s0 > 0.0f ? s0 : 0.0f;
            a[j][2] = rv[j] && s1 > 0.0f ? s1 : 0.0f;
        }
        float s = bias2;
#pragma unroll
        for (int kh = 0; kh < 3; ++kh)
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) s += a[kh][kw] * k2[kh * 3 + kw];
        const size_t i = (row0 + f2) * C + c;
        const bf16 hb = __float2bfloat16_rn(s);
        hi[i] = hb;
        if (lo) lo[i] = __float2bfloat16_rn(s - __bfloat162float(hb));
    }
}

// depthwise 3x3 stride 2 pad 1 (the second one), channels last, fp32 input
// rows [in_off[u], in_off[u+1]) of utterance u with Fi bins; output as bf16
// planes [R_out * Fo][C] for the following 1x1 GEMM.  One CTA per output row,
// thread = channel.
__global__ void __launch_bounds__(C) dw_planes(const float *in, int Fi, const int *in_off, const int *out_off,
                                               const int *row_utt_out, const bf16 *w, const bf16 *bias, bf16 *hi,
                                               bf16 *lo) {
    const int Fo = (Fi + 1) / 2;
    const int row = blockIdx.x, c = threadIdx.x;
    const int u = row_utt_out[row];
    const int t = row - out_off[u];
    const int base = in_off[u], Ti = in_off[u + 1] - base;
    float k[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) k[i] = bf2f(w[c * 9 + i]);
    const float b0 = bf2f(bias[c]);
#pragma unroll 1
    for (int f = 0; f < Fo; ++f) {
        float s = b0;
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
            const int ih = 2 * t - 1 + kh;
            if (ih < 0 || ih >= Ti) continue;
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) {
                const int iw = 2 * f - 1 + kw;
                if (iw < 0 || iw >= Fi) continue;
                s += in[((size_t)(base + ih) * Fi + iw) * C + c] * k[kh * 3 + kw];
            }
        }
        const size_t i = ((size_t)row * Fo + f) * C + c;
        const bf16 hb = __float2bfloat16_rn(s);
        hi[i] = hb;
        if (lo) lo[i] = __float2bfloat16_rn(s - __bfloat162float(hb));
    }
}

// LayerNorm (eps 1e-5, biased variance; backends/cpu/backend.c:109-122) of
// packed rows of width D, one warp per row (40 values per lane in registers):
// optional fp32 output y (may alias x) and bf16 hi/lo planes.  With w2 the
// planes are those of a second LayerNorm (w2, b2) applied to the first one's
// output (a layer's final LayerNorm followed by the next layer's first): y
// holds the first, the planes the second, from one read of x.
__device__ __forceinline__ void ln_row_stats(const float4 (&v)[D / 128], float &mean, float &inv) {
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < D / 128; ++j) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    mean = warp_sum(s) / D;
    float var = 0.0f;
#pragma unroll
    for (int j = 0; j < D / 128; ++j) {
        const float a = v[j].x - mean, b2 = v[j].y - mean, c = v[j].z - mean, d = v[j].w - mean;
        var += (a * a + b2 * b2) + (c * c + d * d);
    }
    inv = 1.0f / sqrtf(warp_sum(var) / D + 1e-5f);
}
__device__ __forceinline__ void ln_row_apply(float4 (&v)[D / 128], float mean, float inv, const bf16 *w,
                                             const bf16 *b, int lane) {
#pragma unroll
    for (int j = 0; j < D / 128; ++j) {
        const int k = 4 * (lane + 32 * j);
        v[j] = make_float4((v[j].x - mean) * inv * bf2f(w[k]) + bf2f(b[k]),
                           (v[j].y - mean) * inv * bf2f(w[k + 1]) + bf2f(b[k + 1]),
                           (v[j].z - mean) * inv * bf2f(w[k + 2]) + bf2f(b[k + 2]),
                           (v[j].w - mean) * inv * bf2f(w[k + 3]) + bf2f(b[k + 3]));
    }
}
// Persistent over rows: warp w takes rows w, w + W, w + 2W, ... (W = warps in
// the grid) and loads its next row before it reduces and writes the current
// one, so every SM keeps streaming while rows are normalised.
__global__ void __launch_bounds__(256, 2) ln_enc(const float *x, int R, const bf16 *w, const bf16 *b, float *y,
                                                 bf16 *hi, bf16 *lo, const bf16 *w2 = nullptr,
                                                 const bf16 *b2 = nullptr) {
    constexpr int NV = D / 128;   // float4 per lane
    const int lane = threadIdx.x & 31;
    const int W = gridDim.x * 8;
    int r = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (r >= R) return;
    float4 v[NV], nx[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) v[j] = reinterpret_cast<const float4 *>(x + (size_t)r * D)[lane + 32 * j];
    for (; r < R; r += W) {
        const int rn = r + W;
        if (rn < R)
#pragma unroll
            for (int j = 0; j < NV; ++j) nx[j] = reinterpret_cast<const float4 *>(x + (size_t)rn * D)[lane + 32 * j];
        float mean, inv;
        ln_row_stats(v, mean, inv);
        ln_row_apply(v, mean, inv, w, b, lane);
        if (y)
#pragma unroll
            for (int j = 0; j < NV; ++j) reinterpret_cast<float4 *>(y + (size_t)r * D)[lane + 32 * j] = v[j];
        if (w2) {
            ln_row_stats(v, mean, inv);
            ln_row_apply(v, mean, inv, w2, b2, lane);
        }
        if (hi) {
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                const int k = 4 * (lane + 32 * j);
                const float o[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
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
#pragma unroll
        for (int j = 0; j < NV; ++j) v[j] = nx[j];
    }
}

// Relative-position attention over packed rows (backends/cpu/backend.c:262-295)
// on the tensor cores.  One CTA per (query tile of 64 rows of one utterance,
// head); warp w owns queries 16w .. 16w+15 of the tile; key tiles of 64.
//   score[q][k] = ((Q+u).K[k] + (Q+v).P[k - q + T_max - 1]) / sqrt(DK)
// is computed as Q.K^T + u.K[k] + Q.Pb^T + v.Pb[m], the bias terms u.K and v.P
// as fp32 dot products over the staged rows.  Q, K, V and P arrive as bf16
// hi/lo planes (written so by the projection GEMMs' epilogues) and are copied
// to shared memory with asynchronous 16-byte copies.  The products run as
// warp-level bf16 MMAs (m16n8k16, fp32 accumulate) on both planes, three
// passes (hi.hi + hi.lo + lo.hi): about 16 mantissa bits per product, like the
// fp32 reference to ~1e-5 relative.  The BD term: each warp
// multiplies its 16 queries by the 80 consecutive P rows its (query, key)
// pairs can reach (a band GEMM), parks that 16 x 80 tile in shared memory and
// reads it back along the diagonals k - q.  Online softmax per query row over
// the quad of threads that holds it; the probabilities feed the P.V MMA
// directly from the score accumulators.  qkv_h / qkv_l rows hold [Q | K | V]
// (stride 3D); P_h / P_l the projected table of 2*T_max - 1 rows.  Output:
// bf16 hi/lo planes.  With TWO = false (plain bf16 activations) only the hi
// planes are staged and every product is one bf16 MMA (fp32 accumulate); the
// shared-memory footprint then halves and two CTAs share an SM.
constexpr int RQ = 64, RB = 128, RS = DK + 8;   // query/key tile, CTA band rows, smem row stride (bf16)
template <bool TWO>
struct RelposSmem {
    static constexpr int NP = TWO ? 2 : 1;
    bf16 q[NP][RQ][RS];
    bf16 k[NP][RQ][RS];   // K tile, then the V tile of the same keys
    bf16 p[NP][RB][RS];   // P band
    float uk[RQ], vp[RB];          // u.K[k], v.P[m]
    float bd[4][16][84];           // per warp: its 16 x 80 band tile
};

__device__ __forceinline__ void ldsm_x4(const void *p, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(const void *p, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo_col, float hi_col) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo_col, hi_col);
    return *reinterpret_cast<const uint32_t *>(&v);
}
__device__ __forceinline__ float bf_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
// Asynchronously copy N rows of DK bf16 values from the hi and lo planes
// (row i at plane + src_row(i) * ld + col0, or zeros where src_row(i) < 0) into
// padded shared rows; 16-byte pieces spread over the 128 threads.
template <int N, int NP, class RowOf>
__device__ __forceinline__ void stage_planes(RowOf src_row, const bf16 *ph_g, const bf16 *pl_g, size_t ld, int col0,
                                             bf16 (*hi)[RS], bf16 (*lo)[RS]) {
    constexpr int CH = DK / 8;   // 16-byte pieces per row and plane
    for (int id = threadIdx.x; id < N * NP * CH; id += 128) {
        const int row = id / (NP * CH), rem = id % (NP * CH), plane = rem / CH, c = (rem % CH) * 8;
        const int sr = src_row(row);
        const bf16 *g = plane ? pl_g : ph_g;
        const bf16 *src = sr >= 0 ? g + (size_t)sr * ld + col0 + c : g;
        cp_async16(plane ? &lo[row][c] : &hi[row][c], src, sr >= 0);
    }
}
// dot[i] = bias . (hi[i] + lo[i]) (lo null: bias . hi[i]) for N rows, 128 / N threads per row.
template <int N>
__device__ __forceinline__ void row_dots(const bf16 (*hi)[RS], const bf16 (*lo)[RS], const bf16 *bias, float *dot) {
    constexpr int TPR = 128 / N, PER = DK / TPR;
    const int row = threadIdx.x / TPR, part = threadIdx.x % TPR;
    float acc = 0.0f;
    for (int c = part * PER; c < part * PER + PER; ++c)
        acc += bf2f(bias[c]) * (__bfloat162float(hi[row][c]) + (lo ? __bfloat162float(lo[row][c]) : 0.0f));
#pragma unroll
    for (int o = 1; o < TPR; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (part == 0) dot[row] = acc;
}

template <bool TWO>
__global__ void __launch_bounds__(128, TWO ? 1 : 2) relpos_tc(const bf16 *qkv_h, const bf16 *qkv_l, const bf16 *P_h,
                                                              const bf16 *P_l, Batch b, const bf16 *pbu,
                                                              const bf16 *pbv, bf16 *hi, bf16 *lo) {
    extern __shared__ __align__(16) uint8_t relpos_raw[];
    using Smem = RelposSmem<TWO>;
    constexpr int NP = Smem::NP;
    Smem &sm = *reinterpret_cast<Smem *>(relpos_raw);
    // plane views (the lo views alias the hi planes when TWO is false and are never read then)
    bf16 (*sqh)[RS] = sm.q[0], (*sql)[RS] = sm.q[NP - 1];
    bf16 (*skh)[RS] = sm.k[0], (*skl)[RS] = sm.k[NP - 1];
    bf16 (*sph)[RS] = sm.p[0], (*spl)[RS] = sm.p[NP - 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tig = lane & 3;
    const int h = blockIdx.y;
    const int wq = b.qtile[blockIdx.x];
    const int u = wq >> 16, q0 = wq & 0xFFFF;
    const int base = b.r3_off[u];
    const int T = b.r3_off[u + 1] - base;
    const int Tm = b.T_max, PL = 2 * Tm - 1;
    const float scale = 1.0f / sqrtf((float)DK);
    const size_t ld = (size_t)3 * D;
    const bf16 *ub = pbu + h * DK, *vb = pbv + h * DK;

    stage_planes<RQ, NP>([&](int r) { return q0 + r < T ? base + q0 + r : -1; }, qkv_h, qkv_l, ld, h * DK, sqh, sql);

    float o[DK / 8][4];
#pragma unroll
    for (int i = 0; i < DK / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;   // rows g and g + 8
    const int mbw = 48 - 16 * warp;                                // this warp's band start (CTA band rows)
    cp_async_wait_all();   // Q tile (made visible by the loop's first barrier)

    for (int k0 = 0; k0 < T; k0 += RQ) {
        __syncthreads();   // the previous tile's V and band reads are done
        stage_planes<RQ, NP>([&](int r) { return k0 + r < T ? base + k0 + r : -1; }, qkv_h, qkv_l, ld, D + h * DK, skh,
                             skl);
        // CTA band row m <-> relative offset (k - q) = (k0 - q0 - 63) + m
        const int prow0 = (k0 - q0) - (RQ - 1) + Tm - 1;
        stage_planes<RB, NP>([&](int m) {
            const int pr = prow0 + m;
            return (m < 2 * RQ - 1 && pr >= 0 && pr < PL) ? pr : -1;
        }, P_h, P_l, (size_t)D, h * DK, sph, spl);
        cp_async_wait_all();
        __syncthreads();
        row_dots<RQ>(skh, TWO ? skl : nullptr, ub, sm.uk);
        row_dots<RB>(sph, TWO ? spl : nullptr, vb, sm.vp);
        __syncthreads();

        float sc[RQ / 8][4], bnd[10][4];
#pragma unroll
        for (int i = 0; i < RQ / 8; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.0f;
#pragma unroll
        for (int i = 0; i < 10; ++i) bnd[i][0] = bnd[i][1] = bnd[i][2] = bnd[i][3] = 0.0f;
        const int arow = 16 * warp + (lane & 15), acol = (lane >> 4) * 8;
        const int brow = (lane & 7) + ((lane >> 4) << 3), bcol = ((lane >> 3) & 1) * 8;
#pragma unroll 2
        for (int ks = 0; ks < DK / 16; ++ks) {
            uint32_t ah0, ah1, ah2, ah3, al0 = 0, al1 = 0, al2 = 0, al3 = 0;
            ldsm_x4(&sqh[arow][ks * 16 + acol], ah0, ah1, ah2, ah3);
            if (TWO) ldsm_x4(&sql[arow][ks * 16 + acol], al0, al1, al2, al3);
#pragma unroll
            for (int np = 0; np < RQ / 16; ++np) {   // key n8-tile pairs
                uint32_t bh0, bh1, bh2, bh3, bl0 = 0, bl1 = 0, bl2 = 0, bl3 = 0;
                ldsm_x4(&skh[np * 16 + brow][ks * 16 + bcol], bh0, bh1, bh2, bh3);
                if (TWO) ldsm_x4(&skl[np * 16 + brow][ks * 16 + bcol], bl0, bl1, bl2, bl3);
                mma16816(sc[2 * np], ah0, ah1, ah2, ah3, bh0, bh1);
                if (TWO) {
                    mma16816(sc[2 * np], ah0, ah1, ah2, ah3, bl0, bl1);
                    mma16816(sc[2 * np], al0, al1, al2, al3, bh0, bh1);
                }
                mma16816(sc[2 * np + 1], ah0, ah1, ah2, ah3, bh2, bh3);
                if (TWO) {
                    mma16816(sc[2 * np + 1], ah0, ah1, ah2, ah3, bl2, bl3);
                    mma16816(sc[2 * np + 1], al0, al1, al2, al3, bh2, bh3);
                }
            }
#pragma unroll
            for (int np = 0; np < 5; ++np) {         // band n8-tile pairs
                uint32_t bh0, bh1, bh2, bh3, bl0 = 0, bl1 = 0, bl2 = 0, bl3 = 0;
                ldsm_x4(&sph[mbw + np * 16 + brow][ks * 16 + bcol], bh0, bh1, bh2, bh3);
                if (TWO) ldsm_x4(&spl[mbw + np * 16 + brow][ks * 16 + bcol], bl0, bl1, bl2, bl3);
                mma16816(bnd[2 * np], ah0, ah1, ah2, ah3, bh0, bh1);
                if (TWO) {
                    mma16816(bnd[2 * np], ah0, ah1, ah2, ah3, bl0, bl1);
                    mma16816(bnd[2 * np], al0, al1, al2, al3, bh0, bh1);
                }
                mma16816(bnd[2 * np + 1], ah0, ah1, ah2, ah3, bh2, bh3);
                if (TWO) {
                    mma16816(bnd[2 * np + 1], ah0, ah1, ah2, ah3, bl2, bl3);
                    mma16816(bnd[2 * np + 1], al0, al1, al2, al3, bh2, bh3);
                }
            }
        }
        // band tile -> shared memory, read back along the diagonals
        float (*bd)[84] = sm.bd[warp];
#pragma unroll
        for (int bt = 0; bt < 10; ++bt) {
            bd[g][bt * 8 + 2 * tig] = bnd[bt][0];
            bd[g][bt * 8 + 2 * tig + 1] = bnd[bt][1];
            bd[g + 8][bt * 8 + 2 * tig] = bnd[bt][2];
            bd[g + 8][bt * 8 + 2 * tig + 1] = bnd[bt][3];
        }
        __syncwarp();
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int kt = 0; kt < RQ / 8; ++kt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = g + (e >> 1) * 8, j = kt * 8 + 2 * tig + (e & 1);
                const int mm = j - i + 15;   // diagonal index in this warp's band
                float v = (sc[kt][e] + sm.uk[j] + bd[i][mm] + sm.vp[mbw + mm]) * scale;
                if (k0 + j >= T) v = -INFINITY;
                sc[kt][e] = v;
                if (e < 2) mx0 = fmaxf(mx0, v); else mx1 = fmaxf(mx1, v);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);   // finite: key k0 is valid
        const float c0 = expf(m0 - n0), c1 = expf(m1 - n1);
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
        for (int kt = 0; kt < RQ / 8; ++kt) {
            sc[kt][0] = expf(sc[kt][0] - n0); s0 += sc[kt][0];
            sc[kt][1] = expf(sc[kt][1] - n0); s0 += sc[kt][1];
            sc[kt][2] = expf(sc[kt][2] - n1); s1 += sc[kt][2];
            sc[kt][3] = expf(sc[kt][3] - n1); s1 += sc[kt][3];
        }
        s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
        s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
        l0 = l0 * c0 + s0;
        l1 = l1 * c1 + s1;
        m0 = n0;
        m1 = n1;
#pragma unroll
        for (int i = 0; i < DK / 8; ++i) { o[i][0] *= c0; o[i][1] *= c0; o[i][2] *= c1; o[i][3] *= c1; }

        __syncthreads();   // every warp is done with the K tile: stage V over it
        stage_planes<RQ, NP>([&](int r) { return k0 + r < T ? base + k0 + r : -1; }, qkv_h, qkv_l, ld,
                             2 * D + h * DK, skh, skl);
        cp_async_wait_all();
        __syncthreads();
        // O += P.V, P from the score accumulators (16-key blocks)
#pragma unroll
        for (int kk = 0; kk < RQ / 16; ++kk) {
            const float *pa = sc[2 * kk], *pb2 = sc[2 * kk + 1];
            const float hv[8] = {bf_round(pa[0]), bf_round(pa[1]), bf_round(pa[2]), bf_round(pa[3]),
                                 bf_round(pb2[0]), bf_round(pb2[1]), bf_round(pb2[2]), bf_round(pb2[3])};
            const uint32_t ph0 = pack_bf16(hv[0], hv[1]), ph1 = pack_bf16(hv[2], hv[3]);
            const uint32_t ph2 = pack_bf16(hv[4], hv[5]), ph3 = pack_bf16(hv[6], hv[7]);
            const uint32_t pl0 = pack_bf16(pa[0] - hv[0], pa[1] - hv[1]), pl1 = pack_bf16(pa[2] - hv[2], pa[3] - hv[3]);
            const uint32_t pl2 = pack_bf16(pb2[0] - hv[4], pb2[1] - hv[5]),
                           pl3 = pack_bf16(pb2[2] - hv[6], pb2[3] - hv[7]);
#pragma unroll
            for (int dp = 0; dp < DK / 16; ++dp) {   // dim n8-tile pairs
                uint32_t vh0, vh1, vh2, vh3, vl0 = 0, vl1 = 0, vl2 = 0, vl3 = 0;
                ldsm_x4_t(&skh[kk * 16 + (lane & 15)][dp * 16 + (lane >> 4) * 8], vh0, vh1, vh2, vh3);
                if (TWO) ldsm_x4_t(&skl[kk * 16 + (lane & 15)][dp * 16 + (lane >> 4) * 8], vl0, vl1, vl2, vl3);
                mma16816(o[2 * dp], ph0, ph1, ph2, ph3, vh0, vh1);
                if (TWO) {
                    mma16816(o[2 * dp], ph0, ph1, ph2, ph3, vl0, vl1);
                    mma16816(o[2 * dp], pl0, pl1, pl2, pl3, vh0, vh1);
                }
                mma16816(o[2 * dp + 1], ph0, ph1, ph2, ph3, vh2, vh3);
                if (TWO) {
                    mma16816(o[2 * dp + 1], ph0, ph1, ph2, ph3, vl2, vl3);
                    mma16816(o[2 * dp + 1], pl0, pl1, pl2, pl3, vh2, vh3);
                }
            }
        }
    }
    const float i0 = 1.0f / l0, i1 = 1.0f / l1;
    const int qa = q0 + 16 * warp + g, qb = qa + 8;
#pragma unroll
    for (int nt = 0; nt < DK / 8; ++nt) {
        const int c = h * DK + nt * 8 + 2 * tig;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int q = e < 2 ? qa : qb;
            if (q >= T) continue;
            const float v = o[nt][e] * (e < 2 ? i0 : i1);
            const size_t idx = (size_t)(base + q) * D + c + (e & 1);
            const bf16 hb = __float2bfloat16_rn(v);
            hi[idx] = hb;
            if (lo) lo[idx] = __float2bfloat16_rn(v - __bfloat162float(hb));
        }
    }
}

#include "relpos_umma.cuh"

// GLU(pw1) -> depthwise conv (kernel CK, same padding inside the utterance) ->
// eval BatchNorm -> SiLU (backends/cpu/backend.c:304-334); output bf16 planes.
// Block = GR packed rows x GC channels: the GLU of rows [r0 - pad, r0 + GR +
// pad) is computed once into shared memory (coalesced along channels), then
// each output sums its CK taps from there, skipping taps outside its own
// utterance.
constexpr int GR = 32, GC = 128;
// two adjacent channels of a pw1 row as float2 (8 B fp32 or 4 B bf16 loads)
__device__ __forceinline__ float2 ld_act2(const float *p) { return *reinterpret_cast<const float2 *>(p); }
__device__ __forceinline__ float2 ld_act2(const bf16 *p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(p));
}
template <typename TIn>   // the pw1 output: fp32, or bf16 with plain bf16 activations
__global__ void __launch_bounds__(256) glu_dw_packed(const TIn *pw1, Batch b, const bf16 *dww, const bf16 *dwb,
                                                     const bf16 *bnw, const bf16 *bnb, const bf16 *bnm,
                                                     const bf16 *bnv, bf16 *hi, bf16 *lo) {
    constexpr int pad = (CK - 1) / 2, HR = GR + CK - 1;
    constexpr int TC = GC / 2, RL = 256 / TC;   // 64 channel pairs x 4 row lanes
    __shared__ float2 g_s[HR][TC];
    __shared__ int lo_s[GR], hi_s[GR];          // the utterance row range of each output row
    const int r0 = blockIdx.x * GR, c0 = blockIdx.y * GC;
    const int tc = threadIdx.x % TC, tr = threadIdx.x / TC;
    const int c = c0 + 2 * tc;                  // this thread's channels c, c + 1
    // every load of the thread's rows issued before the first use (memory-level
    // parallelism: the kernel streams 2560 values per row)
    constexpr int NH = HR / RL;
    static_assert(HR % RL == 0, "halo rows split evenly over the row lanes");
    float2 av[NH], gw[NH];
#pragma unroll
    for (int k = 0; k < NH; ++k) {
        const int row = r0 - pad + tr + k * RL;
        const bool in = row >= 0 && row < b.R3;
        av[k] = in ? ld_act2(pw1 + (size_t)row * 2 * D + c) : make_float2(0.0f, 0.0f);
        gw[k] = in ? ld_act2(pw1 + (size_t)row * 2 * D + D + c) : make_float2(0.0f, 0.0f);
    }
    // (dependent index loads once per CTA, while the activation loads are in flight)
    if (threadIdx.x < GR) {
        const int row = min(r0 + (int)threadIdx.x, b.R3 - 1);
        const int u = b.row_utt3[row];
        lo_s[threadIdx.x] = b.r3_off[u];
        hi_s[threadIdx.x] = b.r3_off[u + 1];
    }
#pragma unroll
    for (int k = 0; k < NH; ++k) {
        const int row = r0 - pad + tr + k * RL;
        const bool in = row >= 0 && row < b.R3;
        g_s[tr + k * RL][tc] = in ? make_float2(mul_sigmoid(av[k].x, gw[k].x), mul_sigmoid(av[k].y, gw[k].y))
                                  : make_float2(0.0f, 0.0f);
    }
    float wk0[CK], wk1[CK];
#pragma unroll
    for (int k = 0; k < CK; ++k) { wk0[k] = bf2f(dww[c * CK + k]); wk1[k] = bf2f(dww[(c + 1) * CK + k]); }
    const float bias0 = bf2f(dwb[c]), bias1 = bf2f(dwb[c + 1]);
    const float sc0 = bf2f(bnw[c]) / sqrtf(bf2f(bnv[c]) + 1e-5f), sc1 = bf2f(bnw[c + 1]) / sqrtf(bf2f(bnv[c + 1]) + 1e-5f);
    const float mu0 = bf2f(bnm[c]), mu1 = bf2f(bnm[c + 1]), be0 = bf2f(bnb[c]), be1 = bf2f(bnb[c + 1]);
    __syncthreads();
#pragma unroll
    for (int rr = tr; rr < GR; rr += RL) {
        const int row = r0 + rr;
        if (row >= b.R3) break;
        const int lo_row = lo_s[rr], hi_row = hi_s[rr];
        float s0 = bias0, s1 = bias1;
        if (row - pad >= lo_row && row + pad < hi_row) {   // every tap inside the utterance (warp-uniform)
#pragma unroll
            for (int k = 0; k < CK; ++k) {
                const float2 g = g_s[rr + k][tc];
                s0 += wk0[k] * g.x;
                s1 += wk1[k] * g.y;
            }
        } else {
#pragma unroll
            for (int k = 0; k < CK; ++k) {
                const int ti = row - pad + k;
                if (ti >= lo_row && ti < hi_row) {
                    const float2 g = g_s[rr + k][tc];
                    s0 += wk0[k] * g.x;
                    s1 += wk1[k] * g.y;
                }
            }
        }
        const float v0 = silu_fast((s0 - mu0) * sc0 + be0), v1 = silu_fast((s1 - mu1) * sc1 + be1);
        const size_t i = (size_t)row * D + c;
        const __nv_bfloat162 h2 = __floats2bfloat162_rn(v0, v1);
        *reinterpret_cast<__nv_bfloat162 *>(hi + i) = h2;
        if (lo)
            *reinterpret_cast<__nv_bfloat162 *>(lo + i) =
                __floats2bfloat162_rn(v0 - __low2float(h2), v1 - __high2float(h2));
    }
}

// ------------------------------------------------------------ host ------
struct State {
    Weights_ w;
    int max_utts = 0, max_frames = 0;     // capacity: utterances and log-mel frames per batch
    int n_sm = 148;                        // SMs of the device (LayerNorm grid)
    int R1_max = 0, R2_max = 0, R3_max = 0, T_cap = 0;
    bool two = true;                       // activations as hi+lo bf16 planes
    float *mel = nullptr, *s1 = nullptr, *x = nullptr, *qkv = nullptr, *pos = nullptr;
    float *enc_h = nullptr;
    bf16 *xa[2] = {nullptr, nullptr}, *hid[2] = {nullptr, nullptr}, *ap[2] = {nullptr, nullptr};
    bf16 *posp[2] = {nullptr, nullptr};
    bf16 *qkvp[2] = {nullptr, nullptr}, *Pp[2] = {nullptr, nullptr};   // Q|K|V and P as bf16 hi/lo planes
    float *ukg = nullptr, *vpg = nullptr;  // u.K per packed row and head, v.P per table row and head
    int *tab = nullptr;                    // device tables
    std::vector<int> htab;
    std::vector<void *> owned;
    // profile mode: events recorded between kernel groups, with the label of
    // the group each closes (labels[0] is unused)
    fe::Front fe;                          // log-mel front-end (audio input)
    bool prof = false;
    std::vector<cudaEvent_t> ev;
    std::vector<const char *> labels;
    int n_marks = 0;
};

// LayerNorm grid: a warp per row, at most two CTAs of 8 warps per SM (each
// warp then walks several rows)
static int ln_grid(const State &st, int R) { return std::max(1, std::min((R + 7) / 8, 2 * st.n_sm)); }

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
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&st.n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || st.n_sm <= 0)
        return false;
    st.R1_max = max_frames / 2 + max_utts;
    st.R2_max = st.R1_max / 2 + max_utts;
    st.R3_max = st.R2_max / 2 + max_utts;
    st.T_cap = st.R3_max;
    // fp32 outputs of the two 1x1 subsampling GEMMs ([R2 * F2][C], [R3][C * F3])
    const size_t s1 = std::max((size_t)st.R2_max * F2 * C, (size_t)st.R3_max * C * F3);
    const size_t R = st.R3_max;
    bool ok = ealloc(st, &st.mel, (size_t)max_frames * F0) && ealloc(st, &st.s1, s1) &&
              ealloc(st, &st.x, R * D) && ealloc(st, &st.qkv, R * 3 * D) && ealloc(st, &st.enc_h, R * DEC_D) &&
              ealloc(st, &st.pos, (size_t)(2 * st.T_cap) * D) && ealloc(st, &st.qkvp[0], R * 3 * D) &&
              ealloc(st, &st.qkvp[1], R * 3 * D) && ealloc(st, &st.Pp[0], (size_t)(2 * st.T_cap) * D) &&
              ealloc(st, &st.Pp[1], (size_t)(2 * st.T_cap) * D) &&
              ealloc(st, &st.ukg, (size_t)st.R3_max * H) && ealloc(st, &st.vpg, (size_t)(2 * st.T_cap) * H) &&
              ealloc(st, &st.tab, (size_t)9 * max_utts + 8 + st.R1_max + st.R2_max + st.R3_max + st.R3_max / RQ +
                                      st.R3_max / UQ + 2);
    const size_t hidn = std::max((size_t)R * FF, (size_t)st.R2_max * F2 * C);
    for (int k = 0; k < (two ? 2 : 1); ++k)
        ok = ok && ealloc(st, &st.xa[k], R * D) && ealloc(st, &st.hid[k], hidn) && ealloc(st, &st.ap[k], R * D) &&
             ealloc(st, &st.posp[k], (size_t)(2 * st.T_cap) * D);
    return ok && fe::front_alloc(st.fe, max_utts, max_frames);
}

static void state_free(State &st) {
    for (void *p : st.owned) cudaFree(p);
    st.owned.clear();
    fe::front_free(st.fe);
    for (cudaEvent_t e : st.ev) cudaEventDestroy(e);
    st.ev.clear();
}

static void egemm_enc(cudaStream_t s, const State &st, const bf16 *W, int N, int K, bf16 *const *xp, int T, long x_rows,
                      GemmEpilogue ep) {
    ep.x_rows = x_rows;
    gemm_bf16(s, W, N, K, xp[0], st.two ? xp[1] : nullptr, T, ep, false);
}

// Encode n utterances (host log-mel, mel[b] = [N_MELS][T_mel[b]]; mel == null:
// the log-mel is already in st.mel, packed) into st.enc_h: packed rows
// [R3, DEC_D], utterance b at rows r3_off[b] .. r3_off[b+1] - 1 (returned in
// r3_off_out, n+1 entries).  Returns false when the batch exceeds the capacity.
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
    // (64-row tiles for the warp-MMA kernel, then 128-row tiles for the tensor-memory kernel)
    std::vector<int> qt, qt2;
    {
        std::vector<int> order(n);
        for (int b = 0; b < n; ++b) order[b] = b;
        std::stable_sort(order.begin(), order.end(),
                         [&](int a, int c) { return r3[a + 1] - r3[a] > r3[c + 1] - r3[c]; });
        for (int b : order)
            for (int q0 = 0; q0 < r3[b + 1] - r3[b]; q0 += RQ) qt.push_back(b << 16 | q0);
        for (int b : order)
            for (int q0 = 0; q0 < r3[b + 1] - r3[b]; q0 += UQ) qt2.push_back(b << 16 | q0);
    }
    const int NQ = (int)qt.size(), NQ2 = (int)qt2.size();
    std::vector<int> &h = st.htab;
    h.assign((size_t)5 * n + 3 + R1 + R2 + R3 + NQ + NQ2, 0);
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
    memcpy(u3 + R3 + NQ, qt2.data(), sizeof(int) * NQ2);
    CT_CHECK(cudaMemcpyAsync(st.tab, hp, sizeof(int) * h.size(), cudaMemcpyHostToDevice, s));
    if (mel)   // host or device sources (the engine's job-ring mirror)
        for (int b = 0; b < n; ++b)
            CT_CHECK(cudaMemcpyAsync(st.mel + mel_off[b], mel[b], sizeof(float) * F0 * T_mel[b], cudaMemcpyDefault,
                                     s));
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
    bt.qtile2 = bt.qtile + NQ;
    bt.n_qtiles2 = NQ2;
    static thread_local int relpos_dev = -1;
    int dev = 0;
    CT_CHECK(cudaGetDevice(&dev));
    if (relpos_dev != dev) {
        CT_CHECK(cudaFuncSetAttribute(relpos_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)sizeof(RelposSmem<true>)));
        CT_CHECK(cudaFuncSetAttribute(relpos_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)sizeof(RelposSmem<false>)));
        CT_CHECK(cudaFuncSetAttribute(relpos_umma, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)sizeof(RelposUmmaSmem) + 1024));
        relpos_dev = dev;
    }
    const Weights_ &w = st.w;
    bf16 *hidp[2] = {st.hid[0], st.hid[1]};
    if (mel) {
        st.n_marks = 0;
        mark(s, st, "");
    }
    // ---- subsampling (backends/cpu/backend.c:188-229), channels last ----
    conv0_dw_planes<<<R2, C, 0, s>>>(st.mel, bt, w.s0w, w.s0b, w.s2w, w.s2b, hidp[0], st.two ? hidp[1] : nullptr);
    GemmEpilogue e3;
    e3.epi = EPI_RELU; e3.bias = w.s3b; e3.Y = st.s1; e3.ldy = C;
    egemm_enc(s, st, w.s3w, C, C, hidp, R2 * F2, (long)st.R2_max * F2, e3);
    dw_planes<<<R3, C, 0, s>>>(st.s1, F2, bt.r2_off, bt.r3_off, bt.row_utt3, w.s5w, w.s5b, hidp[0],
                               st.two ? hidp[1] : nullptr);
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
    // tensor-memory rel-pos attention (plain bf16): operand maps over this batch's rows
    // (the maps span the buffers' capacity, at least one box: rows past this
    // batch only reach query rows that are not stored and keys that are masked)
    const bool umma = !st.two && st.R3_max >= UQ;
    CUtensorMap tmQ{}, tmK{}, tmP{};
    RelposUmmaArgs ua{};
    if (umma) {
        tmQ = gemm_tmap(st.qkvp[0], st.R3_max, 3 * D, UQ);
        tmK = gemm_tmap(st.qkvp[0], st.R3_max, 3 * D, UK);
        tmP = gemm_tmap(st.Pp[0], 2 * st.T_cap, D, UK);   // 64-row band blocks
        ua.qkv = st.qkvp[0]; ua.ukg = st.ukg; ua.vpg = st.vpg; ua.qtile = bt.qtile2; ua.r3_off = bt.r3_off;
        ua.T_max = T_max; ua.PL = PL; ua.out = st.ap[0];
    }
    // ---- Conformer layers (model.h:276-314) ----
    for (int l = 0; l < NL; ++l) {
        const Layer &L = w.L[l];
        // FFN1: x += 0.5 * W2 silu(W1 LN(x) + b1) + b2
        if (l == 0) {   // later layers get these planes from the previous layer's final LayerNorm
            ln_enc<<<ln_grid(st, R3), 256, 0, s>>>(st.x, R3, L.ff1_lnw, L.ff1_lnb, nullptr, st.xa[0], lo_a);
            mark(s, st, "enc_layernorm");
        }
        GemmEpilogue f1;
        f1.epi = EPI_BF16; f1.act = 1; f1.bias = L.ff1_b1; f1.Ybf = st.hid[0]; f1.Ybf_lo = lo_h; f1.ldy = FF;
        egemm_enc(s, st, L.ff1_w1, FF, D, xap, R3, RT, f1);
        mark(s, st, "enc_gemm_ffn1");
        GemmEpilogue f2;
        f2.epi = EPI_FMADD; f2.scale = 0.5f; f2.bias = L.ff1_b2; f2.Y = st.x; f2.ldy = D;
        egemm_enc(s, st, L.ff1_w2, D, FF, hidp, R3, RT, f2);
        mark(s, st, "enc_gemm_ffn2");
        // relative-position self-attention: x += Wo attn(LN(x)) + bo
        ln_enc<<<ln_grid(st, R3), 256, 0, s>>>(st.x, R3, L.sa_lnw, L.sa_lnb, nullptr, st.xa[0], lo_a);
        mark(s, st, "enc_layernorm");
        GemmEpilogue eq;
        eq.epi = EPI_BF16; eq.bias = L.qkv_b; eq.Ybf = st.qkvp[0]; eq.Ybf_lo = st.two ? st.qkvp[1] : nullptr; eq.ldy = 3 * D;
        egemm_enc(s, st, L.qkv_w, 3 * D, D, xap, R3, RT, eq);
        mark(s, st, "enc_gemm_qkv");
        GemmEpilogue ep;
        ep.epi = EPI_BF16; ep.Ybf = st.Pp[0]; ep.Ybf_lo = st.two ? st.Pp[1] : nullptr; ep.ldy = D;
        egemm_enc(s, st, L.sa_pw, D, D, st.posp, PL, 2 * st.T_cap, ep);
        mark(s, st, "enc_gemm_pos");
        if (st.two)
            relpos_tc<true><<<dim3(NQ, H), 128, sizeof(RelposSmem<true>), s>>>(
                st.qkvp[0], st.qkvp[1], st.Pp[0], st.Pp[1], bt, L.sa_pbu, L.sa_pbv, st.ap[0], lo_p);
        else if (!umma)
            relpos_tc<false><<<dim3(NQ, H), 128, sizeof(RelposSmem<false>), s>>>(
                st.qkvp[0], nullptr, st.Pp[0], nullptr, bt, L.sa_pbu, L.sa_pbv, st.ap[0], nullptr);
        else {
            relpos_bias_dots<<<(R3 + PL + 7) / 8, 256, 0, s>>>(st.qkvp[0], nullptr, st.Pp[0], nullptr, R3, PL,
                                                                        L.sa_pbu, L.sa_pbv, st.ukg, st.vpg);
            relpos_umma<<<dim3(bt.n_qtiles2, H), U_THREADS, sizeof(RelposUmmaSmem) + 1024, s>>>(tmQ, tmK, tmP, ua);
        }
        mark(s, st, "enc_relpos_attn");
        GemmEpilogue eo2;
        eo2.epi = EPI_FMADD; eo2.scale = 1.0f; eo2.bias = L.sa_ob; eo2.Y = st.x; eo2.ldy = D;
        egemm_enc(s, st, L.sa_ow, D, D, app, R3, RT, eo2);
        mark(s, st, "enc_gemm_o");
        // conv module: x += pw2(silu(bn(dw(glu(pw1(LN(x)))))))
        ln_enc<<<ln_grid(st, R3), 256, 0, s>>>(st.x, R3, L.cv_lnw, L.cv_lnb, nullptr, st.xa[0], lo_a);
        mark(s, st, "enc_layernorm");
        // pw1 output: fp32 with hi+lo planes, bf16 with plain bf16 activations
        // (half the bytes written and read back by the GLU)
        GemmEpilogue e1;
        e1.bias = L.cv_pw1b; e1.ldy = 2 * D;
        bf16 *pw1_bf = reinterpret_cast<bf16 *>(st.qkv);
        if (st.two) e1.Y = st.qkv;
        else { e1.epi = EPI_BF16; e1.Ybf = pw1_bf; }
        egemm_enc(s, st, L.cv_pw1w, 2 * D, D, xap, R3, RT, e1);
        mark(s, st, "enc_gemm_pw1");
        const dim3 ggrid((R3 + GR - 1) / GR, D / GC);
        if (st.two)
            glu_dw_packed<float><<<ggrid, 256, 0, s>>>(st.qkv, bt, L.cv_dww, L.cv_dwb, L.cv_bnw, L.cv_bnb, L.cv_bnm,
                                                       L.cv_bnv, st.ap[0], lo_p);
        else
            glu_dw_packed<bf16><<<ggrid, 256, 0, s>>>(pw1_bf, bt, L.cv_dww, L.cv_dwb, L.cv_bnw, L.cv_bnb, L.cv_bnm,
                                                      L.cv_bnv, st.ap[0], lo_p);
        mark(s, st, "enc_glu_dwconv");
        GemmEpilogue e2;
        e2.epi = EPI_FMADD; e2.scale = 1.0f; e2.bias = L.cv_pw2b; e2.Y = st.x; e2.ldy = D;
        egemm_enc(s, st, L.cv_pw2w, D, D, app, R3, RT, e2);
        mark(s, st, "enc_gemm_pw2");
        // FFN2
        ln_enc<<<ln_grid(st, R3), 256, 0, s>>>(st.x, R3, L.ff2_lnw, L.ff2_lnb, nullptr, st.xa[0], lo_a);
        mark(s, st, "enc_layernorm");
        GemmEpilogue g1 = f1;
        g1.bias = L.ff2_b1;
        egemm_enc(s, st, L.ff2_w1, FF, D, xap, R3, RT, g1);
        mark(s, st, "enc_gemm_ffn1");
        GemmEpilogue g2 = f2;
        g2.bias = L.ff2_b2;
        egemm_enc(s, st, L.ff2_w2, D, FF, hidp, R3, RT, g2);
        mark(s, st, "enc_gemm_ffn2");
        // x = LN_out(x), and the planes of the next layer's FFN1 LayerNorm of it
        // (after the last layer: the planes of x itself, for the projection)
        if (l + 1 < NL)
            ln_enc<<<ln_grid(st, R3), 256, 0, s>>>(st.x, R3, L.out_lnw, L.out_lnb, st.x, st.xa[0], lo_a,
                                                 w.L[l + 1].ff1_lnw, w.L[l + 1].ff1_lnb);
        else
            ln_enc<<<ln_grid(st, R3), 256, 0, s>>>(st.x, R3, L.out_lnw, L.out_lnb, st.x, st.xa[0], lo_a);
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

// Encode n utterances from host 16 kHz samples: the log-mel front-end writes
// st.mel, then encode() runs on it.  T_mel[b] = 1 + n_samples[b] / 160.
static bool encode_audio(cudaStream_t s, State &st, int n, const float *const *samples, const int *n_samples,
                         int *T_mel, int *r3_off_out) {
    st.n_marks = 0;
    mark(s, st, "");
    if (!fe::log_mel(s, st.fe, n, samples, n_samples, st.mel, T_mel)) return false;
    mark(s, st, "enc_log_mel");
    return encode(s, st, n, nullptr, T_mel, r3_off_out);
}

}  // namespace enc
}  // namespace ct
