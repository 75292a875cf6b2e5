// kernels.cu -- non-GEMM kernels (see kernels.cuh for the contracts).
#include "kernels.cuh"

namespace ct {

static inline int grid_for(size_t n, int threads, int cap = 148 * 16) {
    size_t b = (n + threads - 1) / threads;
    if (b < 1) b = 1;
    return (int)(b > (size_t)cap ? cap : b);
}

// Block-wide sum over 256 threads (8 warps); all threads get the result.
__device__ __forceinline__ float block_sum256(float v, float *red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += red[i];
    return s;
}

// ---------------------------------------------------------------- LN -------
__global__ void __launch_bounds__(256) layernorm_kernel(float *dst, const float *src, const bf16 *w, const bf16 *b,
                                                        int D, bf16 *dst_bf) {
    __shared__ float red[8];
    const size_t row = blockIdx.x;
    const float *x = src + row * D;
    float s = 0.0f;
    for (int i = threadIdx.x; i < D; i += 256) s += x[i];
    const float mean = block_sum256(s, red) / D;
    float v = 0.0f;
    for (int i = threadIdx.x; i < D; i += 256) { const float c = x[i] - mean; v += c * c; }
    const float inv = 1.0f / sqrtf(block_sum256(v, red) / D + 1e-5f);
    float *y = dst + row * D;
    for (int i = threadIdx.x; i < D; i += 256) {
        const float o = (x[i] - mean) * inv * bf2f(w[i]) + bf2f(b[i]);
        y[i] = o;
        if (dst_bf) dst_bf[row * D + i] = __float2bfloat16_rn(o);
    }
}

void layernorm(cudaStream_t st, float *dst, const float *src, const bf16 *w, const bf16 *b, int T, int D,
               bf16 *dst_bf) {
    if (T <= 0) return;
    layernorm_kernel<<<T, 256, 0, st>>>(dst, src, w, b, D, dst_bf);
    CT_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------- embed ----
__global__ void __launch_bounds__(256) embed_ln_kernel(float *h, const int *tok, const int *pos, int pos_off,
                                                       const int *active, const bf16 *etw, const bf16 *epw,
                                                       const bf16 *lnw, const bf16 *lnb, int D, int vocab,
                                                       int max_pos, bf16 *h_bf) {
    extern __shared__ float row[];
    __shared__ float red[8];
    const int r = blockIdx.x;
    if (active && !active[r]) return;
    const int id = tok[r];
    const int p = pos ? pos[r] + pos_off : pos_off + r;
    if (id < 0 || id >= vocab || p < 0 || p >= max_pos) {
        if (threadIdx.x == 0) set_status(CT_STATUS_BAD_ARG);
        return;
    }
    float s = 0.0f;
    for (int i = threadIdx.x; i < D; i += 256) {
        const float v = bf2f(etw[(size_t)id * D + i]) + bf2f(epw[(size_t)p * D + i]);
        row[i] = v;
        s += v;
    }
    const float mean = block_sum256(s, red) / D;
    float var = 0.0f;
    for (int i = threadIdx.x; i < D; i += 256) { const float c = row[i] - mean; var += c * c; }
    const float inv = 1.0f / sqrtf(block_sum256(var, red) / D + 1e-5f);
    for (int i = threadIdx.x; i < D; i += 256) {
        const float o = (row[i] - mean) * inv * bf2f(lnw[i]) + bf2f(lnb[i]);
        h[(size_t)r * D + i] = o;
        if (h_bf) h_bf[(size_t)r * D + i] = __float2bfloat16_rn(o);
    }
}

void embed_ln(cudaStream_t st, float *h, const int *tok, const int *pos, int pos_off, const int *active, int R,
              const bf16 *etw, const bf16 *epw, const bf16 *lnw, const bf16 *lnb, int D, int vocab, int max_pos,
              bf16 *h_bf) {
    if (R <= 0) return;
    embed_ln_kernel<<<R, 256, D * sizeof(float), st>>>(h, tok, pos, pos_off, active, etw, epw, lnw, lnb, D, vocab,
                                                       max_pos, h_bf);
    CT_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------- misc -----
__global__ void add_kernel(float *dst, const float *src, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] += src[i];
}
void add_inplace(cudaStream_t st, float *dst, const float *src, size_t n) {
    if (!n) return;
    add_kernel<<<grid_for(n, 256), 256, 0, st>>>(dst, src, n);
    CT_CHECK(cudaGetLastError());
}

__global__ void causal_mask_kernel(float *mask, int S) {
    const int n = S * S;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        mask[i] = (i % S) > (i / S) ? -1e9f : 0.0f;
}
void fill_causal_mask(cudaStream_t st, float *mask, int S) {
    if (S <= 0) return;
    causal_mask_kernel<<<grid_for((size_t)S * S, 256), 256, 0, st>>>(mask, S);
    CT_CHECK(cudaGetLastError());
}

// backends/cpu/backend.c:231-242
__global__ void rel_pos_kernel(float *pe, int T, int D) {
    const int L = 2 * T - 1, half = D / 2;
    const float log10k = logf(10000.0f);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < L * half; i += gridDim.x * blockDim.x) {
        const int p = i / half, k = i % half;
        const float pos = (float)(T - 1 - p);
        const float freq = expf(-(float)(2 * k) * log10k / D);
        pe[(size_t)p * D + 2 * k] = sinf(pos * freq);
        pe[(size_t)p * D + 2 * k + 1] = cosf(pos * freq);
    }
}
void make_rel_pos_emb(cudaStream_t st, float *pe, int T, int D) {
    if (T <= 0) return;
    rel_pos_kernel<<<grid_for((size_t)(2 * T - 1) * (D / 2), 256), 256, 0, st>>>(pe, T, D);
    CT_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------- attention
static constexpr int ACH = 128;   // keys per chunk (one per thread)

// Keys of row r.  A length above len_max is clamped to it and one of zero or
// less leaves the row with no keys (attn_chunk_kernel writes zeros); both set
// CT_STATUS_BAD_ARG in the device status word.
__device__ __forceinline__ int attn_len(const AttnRows &a, int r) {
    int L = a.len_arr ? a.len_arr[r] : (a.len_dev ? *a.len_dev : a.len_const);
    if (L > a.len_max) { set_status(CT_STATUS_BAD_ARG); L = a.len_max; }
    if (L <= 0) { set_status(CT_STATUS_BAD_ARG); L = 0; }
    return L;
}

__global__ void __launch_bounds__(ACH) attn_chunk_kernel(const AttnRows a, float *ws, int nchunk_max) {
    __shared__ __align__(16) float qs[256];
    __shared__ float ps[ACH];
    __shared__ float red[4];
    __shared__ float ored[4][256];
    const int r = blockIdx.z, h = blockIdx.y, c = blockIdx.x;
    const int L = attn_len(a, r);
    const int nck = (L + ACH - 1) / ACH;
    if (L == 0 && c == 0) {   // no keys (a bad length): the output row is defined as zero
        for (int d = threadIdx.x; d < a.DK; d += ACH) a.out[(size_t)r * a.ldo + h * a.DK + d] = 0.0f;
        return;
    }
    if (c >= nck) return;
    const int DK = a.DK, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int d = tid; d < DK; d += ACH) qs[d] = a.Q[(size_t)r * a.ldq + h * DK + d];
    __syncthreads();
    const int k = c * ACH + tid;
    const float *Kr = a.K + (size_t)r * a.kv_item;
    const float *Vr = a.V + (size_t)r * a.kv_item;
    float s = -INFINITY;
    if (k < L) {
        const float4 *kp = reinterpret_cast<const float4 *>(Kr + (size_t)k * a.ldkv + h * DK);
        const float4 *qp = reinterpret_cast<const float4 *>(qs);
        float acc = 0.0f;
        for (int i = 0; i < DK / 4; ++i) {
            const float4 kv = kp[i], qv = qp[i];
            acc += qv.x * kv.x; acc += qv.y * kv.y; acc += qv.z * kv.z; acc += qv.w * kv.w;
        }
        s = acc * a.scale + (a.mask ? a.mask[(size_t)r * a.mask_ld + k] : 0.0f);
    }
    float m = warp_max(s);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float p = k < L ? expf(s - m) : 0.0f;
    ps[tid] = p;
    float l = warp_sum(p);
    __syncthreads();
    if (lane == 0) red[warp] = l;
    __syncthreads();
    l = red[0] + red[1] + red[2] + red[3];
    // o[d] = sum_k p_k V[k][d]: warp w owns keys [32w, 32w+32), lane owns dims lane + 32j
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = 0.0f;
    const int kw0 = c * ACH + warp * 32;
    const int kn = min(32, L - kw0);
    for (int kk = 0; kk < kn; ++kk) {
        const float pk = ps[warp * 32 + kk];
        const float *vrow = Vr + (size_t)(kw0 + kk) * a.ldkv + h * DK;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (lane + 32 * j < DK) o[j] += pk * vrow[lane + 32 * j];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (lane + 32 * j < DK) ored[warp][lane + 32 * j] = kn > 0 ? o[j] : 0.0f;
    __syncthreads();
    if (nck == 1) {
        for (int d = tid; d < DK; d += ACH)
            a.out[(size_t)r * a.ldo + h * DK + d] = (ored[0][d] + ored[1][d] + ored[2][d] + ored[3][d]) / l;
    } else {
        float *w = ws + (((size_t)r * a.H + h) * nchunk_max + c) * (DK + 2);
        if (tid == 0) { w[0] = m; w[1] = l; }
        for (int d = tid; d < DK; d += ACH) w[2 + d] = ored[0][d] + ored[1][d] + ored[2][d] + ored[3][d];
    }
}

__global__ void attn_combine_kernel(const AttnRows a, const float *ws, int nchunk_max) {
    const int r = blockIdx.x, h = blockIdx.y;
    const int L = attn_len(a, r);
    const int nck = (L + ACH - 1) / ACH;
    if (nck <= 1) return;
    const float *w = ws + ((size_t)r * a.H + h) * nchunk_max * (a.DK + 2);
    float M = -INFINITY;
    for (int c = 0; c < nck; ++c) M = fmaxf(M, w[(size_t)c * (a.DK + 2)]);
    float Ls = 0.0f;
    for (int c = 0; c < nck; ++c) Ls += w[(size_t)c * (a.DK + 2) + 1] * expf(w[(size_t)c * (a.DK + 2)] - M);
    for (int d = threadIdx.x; d < a.DK; d += blockDim.x) {
        float o = 0.0f;
        for (int c = 0; c < nck; ++c) o += w[(size_t)c * (a.DK + 2) + 2 + d] * expf(w[(size_t)c * (a.DK + 2)] - M);
        a.out[(size_t)r * a.ldo + h * a.DK + d] = o / Ls;
    }
}

size_t attn_ws_floats(int R, int H, int DK, int len_max) {
    const int nck = (len_max + ACH - 1) / ACH;
    return nck > 1 ? (size_t)R * H * nck * (DK + 2) : 0;
}

void attn_rows_f32(cudaStream_t st, const AttnRows &a, float *ws, size_t ws_floats) {
    if (a.R <= 0 || a.len_max <= 0) return;
    if (a.DK > 256 || (a.DK & 3) || (a.ldkv & 3) || (a.kv_item & 3)) CT_FATAL("attention: unsupported head layout");
    const int nck = (a.len_max + ACH - 1) / ACH;
    if (attn_ws_floats(a.R, a.H, a.DK, a.len_max) > ws_floats) CT_FATAL("attention workspace too small");
    dim3 grid(nck, a.H, a.R);
    attn_chunk_kernel<<<grid, ACH, 0, st>>>(a, ws, nck);
    CT_CHECK(cudaGetLastError());
    if (nck > 1) {
        attn_combine_kernel<<<dim3(a.R, a.H), 128, 0, st>>>(a, ws, nck);
        CT_CHECK(cudaGetLastError());
    }
}

// ------------------------------------------------------ rel-pos attention ----
// One warp per (query, head), online softmax over 32-key chunks (lane = key).
__global__ void __launch_bounds__(128) relpos_attn_kernel(const float *Q, const float *K, const float *V,
                                                          const float *P, const bf16 *pbu, const bf16 *pbv,
                                                          float *out, int T, int H, int DK, int D, float scale) {
    __shared__ __align__(16) float qu_s[4][256];
    __shared__ __align__(16) float qv_s[4][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * 4 + warp, h = blockIdx.y;
    if (q >= T) return;
    float *qu = qu_s[warp], *qv = qv_s[warp];
    for (int d = lane; d < DK; d += 32) {
        const float x = Q[(size_t)q * D + h * DK + d];
        qu[d] = x + bf2f(pbu[h * DK + d]);
        qv[d] = x + bf2f(pbv[h * DK + d]);
    }
    __syncwarp();
    float m = -INFINITY, l = 0.0f, o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = 0.0f;
    for (int k0 = 0; k0 < T; k0 += 32) {
        const int k = k0 + lane;
        float s = -INFINITY;
        if (k < T) {
            const float4 *kp = reinterpret_cast<const float4 *>(K + (size_t)k * D + h * DK);
            const float4 *pp = reinterpret_cast<const float4 *>(P + (size_t)(k + T - 1 - q) * D + h * DK);
            const float4 *up = reinterpret_cast<const float4 *>(qu);
            const float4 *vp = reinterpret_cast<const float4 *>(qv);
            float ac = 0.0f, bd = 0.0f;
            for (int i = 0; i < DK / 4; ++i) {
                const float4 kv = kp[i], pv = pp[i], a = up[i], b = vp[i];
                ac += a.x * kv.x; ac += a.y * kv.y; ac += a.z * kv.z; ac += a.w * kv.w;
                bd += b.x * pv.x; bd += b.y * pv.y; bd += b.z * pv.z; bd += b.w * pv.w;
            }
            s = ac * scale + bd * scale;
        }
        const float mn = fmaxf(m, warp_max(s));
        const float corr = expf(m - mn);   // m = -inf on the first chunk -> 0
        const float p = k < T ? expf(s - mn) : 0.0f;
        l = l * corr + warp_sum(p);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] *= corr;
        const int kn = min(32, T - k0);
        for (int kk = 0; kk < kn; ++kk) {
            const float pk = __shfl_sync(0xffffffffu, p, kk);
            const float *vrow = V + (size_t)(k0 + kk) * D + h * DK;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (lane + 32 * j < DK) o[j] += pk * vrow[lane + 32 * j];
        }
        m = mn;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (lane + 32 * j < DK) out[(size_t)q * D + h * DK + lane + 32 * j] = o[j] / l;
}

void relpos_attn_f32(cudaStream_t st, const float *Q, const float *K, const float *V, const float *P,
                     const bf16 *pbu, const bf16 *pbv, float *out, int T, int H, int DK, int D) {
    if (T <= 0) return;
    if (DK > 256 || (DK & 3) || (D & 3)) CT_FATAL("rel-pos attention: unsupported head layout");
    dim3 grid((T + 3) / 4, H);
    relpos_attn_kernel<<<grid, 128, 0, st>>>(Q, K, V, P, pbu, pbv, out, T, H, DK, D, 1.0f / sqrtf((float)DK));
    CT_CHECK(cudaGetLastError());
}

// -------------------------------------------------------- conv module ------
__global__ void glu_dw_kernel(const float *pw1, float *y, int T, int D, int CK, const bf16 *dww, const bf16 *dwb,
                              const bf16 *bnw, const bf16 *bnb, const bf16 *bnm, const bf16 *bnv) {
    const size_t n = (size_t)T * D;
    const int pad = (CK - 1) / 2;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / D), c = (int)(i % D);
        float s = bf2f(dwb[c]);
        for (int k = 0; k < CK; ++k) {
            const int ti = t - pad + k;
            if (ti < 0 || ti >= T) continue;
            const float a = pw1[(size_t)ti * 2 * D + c];
            const float g = pw1[(size_t)ti * 2 * D + D + c];
            s += bf2f(dww[c * CK + k]) * (a / (1.0f + expf(-g)));
        }
        float v = (s - bf2f(bnm[c])) / sqrtf(bf2f(bnv[c]) + 1e-5f) * bf2f(bnw[c]) + bf2f(bnb[c]);
        y[i] = v / (1.0f + expf(-v));
    }
}

void glu_dwconv_bn_silu(cudaStream_t st, const float *pw1, float *y, int T, int D, int CK, const bf16 *dww,
                        const bf16 *dwb, const bf16 *bnw, const bf16 *bnb, const bf16 *bnm, const bf16 *bnv) {
    if (T <= 0) return;
    glu_dw_kernel<<<grid_for((size_t)T * D, 256), 256, 0, st>>>(pw1, y, T, D, CK, dww, dwb, bnw, bnb, bnm, bnv);
    CT_CHECK(cudaGetLastError());
}

// -------------------------------------------------------- subsampling ------
// conv0 of backends/cpu/backend.c:205 on the (time, mel) plane, channels-last out.
__global__ void sub_conv0_kernel(const float *mel, int T_mel, int mel_stride, int n_mels, const bf16 *w,
                                 const bf16 *b, float *out, int C, int T1, int F1) {
    const size_t n = (size_t)T1 * F1 * C;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % C);
        const int f = (int)((i / C) % F1);
        const int t = (int)(i / ((size_t)C * F1));
        float s = bf2f(b[c]);
        for (int kh = 0; kh < 3; ++kh) {
            const int ih = 2 * t - 1 + kh;
            if (ih < 0 || ih >= T_mel) continue;
            for (int kw = 0; kw < 3; ++kw) {
                const int iw = 2 * f - 1 + kw;
                if (iw < 0 || iw >= n_mels) continue;
                s += mel[(size_t)iw * mel_stride + ih] * bf2f(w[c * 9 + kh * 3 + kw]);
            }
        }
        out[i] = s > 0.0f ? s : 0.0f;
    }
}

void sub_conv0(cudaStream_t st, const float *mel, int T_mel, int mel_stride, int n_mels, const bf16 *w,
               const bf16 *b, float *out, int C) {
    const int T1 = (T_mel + 1) / 2, F1 = (n_mels + 1) / 2;
    sub_conv0_kernel<<<grid_for((size_t)T1 * F1 * C, 256), 256, 0, st>>>(mel, T_mel, mel_stride, n_mels, w, b, out,
                                                                        C, T1, F1);
    CT_CHECK(cudaGetLastError());
}

// depthwise 3x3 stride 2 pad 1 (backends/cpu/backend.c:209, :216, groups = C)
__global__ void sub_dw_kernel(const float *in, int Ti, int Fi, int C, const bf16 *w, const bf16 *b, float *out,
                              int To, int Fo) {
    const size_t n = (size_t)To * Fo * C;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % C);
        const int f = (int)((i / C) % Fo);
        const int t = (int)(i / ((size_t)C * Fo));
        float s = bf2f(b[c]);
        for (int kh = 0; kh < 3; ++kh) {
            const int ih = 2 * t - 1 + kh;
            if (ih < 0 || ih >= Ti) continue;
            for (int kw = 0; kw < 3; ++kw) {
                const int iw = 2 * f - 1 + kw;
                if (iw < 0 || iw >= Fi) continue;
                s += in[((size_t)ih * Fi + iw) * C + c] * bf2f(w[c * 9 + kh * 3 + kw]);
            }
        }
        out[i] = s;
    }
}

void sub_dwconv(cudaStream_t st, const float *in, int Ti, int Fi, int C, const bf16 *w, const bf16 *b, float *out) {
    const int To = (Ti + 1) / 2, Fo = (Fi + 1) / 2;
    sub_dw_kernel<<<grid_for((size_t)To * Fo * C, 256), 256, 0, st>>>(in, Ti, Fi, C, w, b, out, To, Fo);
    CT_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------- argmax ---
__global__ void __launch_bounds__(256) argmax_kernel(const float *logits, int V, const int *active, int *out) {
    __shared__ float bv[256];
    __shared__ int bi[256];
    const int r = blockIdx.x;
    if (active && !active[r]) return;
    const float *x = logits + (size_t)r * V;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += 256) {   // ascending indices: strict > keeps the first
        const float v = x[i];
        if (v > best) { best = v; idx = i; }
    }
    bv[threadIdx.x] = best;
    bi[threadIdx.x] = idx;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            const float ov = bv[threadIdx.x + s];
            const int oi = bi[threadIdx.x + s];
            if (ov > bv[threadIdx.x] || (ov == bv[threadIdx.x] && oi < bi[threadIdx.x])) {
                bv[threadIdx.x] = ov;
                bi[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) out[r] = bi[0] == 0x7fffffff ? 0 : bi[0];
}

void argmax_rows(cudaStream_t st, const float *logits, int R, int V, const int *active, int *out) {
    if (R <= 0) return;
    argmax_kernel<<<R, 256, 0, st>>>(logits, V, active, out);
    CT_CHECK(cudaGetLastError());
}

}  // namespace ct
