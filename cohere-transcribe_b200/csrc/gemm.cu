// gemm.cu -- tcgen05 / TMA GEMM (see gemm.cuh).
//
// One CTA computes a 128 (features) x BN (tokens) output tile over a K range:
//   warp 0      TMA producer: W tile [128 x 64] and X tile(s) [BN x 64] per stage
//   warp 1      MMA issuer: 4 (or 8 with X_lo) tcgen05.mma K=16 per stage,
//               TMEM allocation owner
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, bias/activation/
//               residual/scatter, coalesced stores (lanes = consecutive features)
// Stages are released by tcgen05.commit on the stage's "empty" mbarrier.
// Split-K (grid.z) writes fp32 partials that a second kernel sums in split
// order, so the result is deterministic and independent of T.
#include <algorithm>
#include <memory>
#include <unordered_map>

#include "gemm.cuh"

namespace ct {

static constexpr int BM = 128;
static constexpr int BK = 64;
static constexpr int kThreads = 192;
static constexpr int kSmemBudget = 220 * 1024;

struct KernelParams {
    int N, K, T;
    int kbps;      // k-blocks (of 64) per split
    int kb_total;
    int stages;
    int nsplit;    // K splits = cluster size along grid.z (1 = no split)
    int bar_off;   // byte offset of the mbarriers in the aligned shared memory
    GemmEpilogue ep;
};

// Store one output value for the store-only epilogues (no loads).
__device__ __forceinline__ void store_epilogue(const GemmEpilogue &ep, int t, int n, float v) {
    switch (ep.epi) {
    case EPI_STORE: ep.Y[(size_t)t * ep.ldy + n] = v; break;
    case EPI_SILU: ep.Y[(size_t)t * ep.ldy + n] = v / (1.0f + expf(-v)); break;
    case EPI_RELU: ep.Y[(size_t)t * ep.ldy + n] = v > 0.0f ? v : 0.0f; break;
    case EPI_BF16: {
        float a = v;
        if (ep.act == 1) a = silu_fast(v);
        else if (ep.act == 2) a = v > 0.0f ? v : 0.0f;
        const bf16 hb = __float2bfloat16_rn(a);
        ep.Ybf[(size_t)t * ep.ldy + n] = hb;
        if (ep.Ybf_lo) ep.Ybf_lo[(size_t)t * ep.ldy + n] = __float2bfloat16_rn(a - __bfloat162float(hb));
        break;
    }
    case EPI_RELU_FLAT:
        ep.Y[(size_t)(t / ep.flat_f) * ep.ldy + (size_t)n * ep.flat_f + (t % ep.flat_f)] = v > 0.0f ? v : 0.0f;
        break;
    default: break;
    }
}

// Epilogue of feature n for tokens t0 .. t0 + tl - 1 (tl <= 16), values v[j]
// (bias included).  Every load the chunk needs -- row mask, KV positions, page
// offsets, the old values of an FMADD -- is issued before the first store:
// the stores may alias those addresses as far as the compiler knows, so
// interleaving loads and stores would serialise one memory round trip per token.
// E >= 0 fixes the epilogue kind at compile time (the persistent kernel's
// instantiations: one switch arm of code instead of all of them, no dispatch
// per chunk); E = -1 dispatches on ep.epi.
template <int E = -1>
__device__ __forceinline__ void epilogue16(const GemmEpilogue &ep, int t0, int tl, int n, const float *v) {
    bool keep[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) keep[j] = j < tl && (!ep.row_mask || ep.row_mask[t0 + j]);
    switch (E >= 0 ? E : ep.epi) {
    case EPI_FMADD: {
        // Y += scale * v as a reduction into memory: no load round trip per
        // chunk.  Each element has exactly one writer in the launch, so the
        // sum is the load / add / store result (atom and red .add.f32 round to
        // nearest; they also flush subnormals, which these residuals never reach).
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (keep[j]) atomicAdd(ep.Y + (size_t)(t0 + j) * ep.ldy + n, ep.scale * v[j]);
        break;
    }
    case EPI_KVCACHE: {
        int slot[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) slot[j] = keep[j] ? ep.pos[t0 + j] - 1 : 0;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (!keep[j]) continue;
            if (slot[j] < 0 || slot[j] >= ep.kv_stride) { set_status(CT_STATUS_BAD_ARG); continue; }
            ep.Y[((size_t)(t0 + j) * ep.kv_stride + slot[j]) * ep.ldy + n] = v[j];
        }
        break;
    }
    case EPI_QKV_PAGED:
    case EPI_CAKV_PAGED: {
        const bool qpart = ep.epi == EPI_QKV_PAGED && n < ep.qdim;
        if (qpart) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (keep[j]) ep.Y[(size_t)(t0 + j) * ep.ldy + n] = v[j];
            break;
        }
        long long off[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) off[j] = keep[j] ? ep.row_off[t0 + j] : -1;
        // (layer*2 + kv) block of the page and the column inside it
        const int n2 = ep.epi == EPI_QKV_PAGED ? n - ep.qdim : n;
        const int lk = ep.epi == EPI_QKV_PAGED ? ep.layer * 2 + n2 / ep.kv_width : n2 / ep.kv_width;
        const long long col = (long long)lk * kPageRows * ep.kv_width + n2 % ep.kv_width;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (off[j] >= 0) ep.kv_pool[off[j] + col] = __float2bfloat16_rn(v[j]);
        break;
    }
    case EPI_STORE:
    case EPI_SILU:
    case EPI_RELU: {
        // one branch per chunk, not per element
        float *y = ep.Y + (size_t)t0 * ep.ldy + n;
        const size_t ld = (size_t)ep.ldy;
        if (ep.epi == EPI_STORE) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (keep[j]) y[j * ld] = v[j];
        } else if (ep.epi == EPI_SILU) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (keep[j]) y[j * ld] = v[j] / (1.0f + expf(-v[j]));
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (keep[j]) y[j * ld] = fmaxf(v[j], 0.0f);
        }
        break;
    }
    case EPI_BF16: {
        float a[16];
        if (ep.act == 1) {
#pragma unroll
            for (int j = 0; j < 16; ++j) a[j] = silu_fast(v[j]);
        } else if (ep.act == 2) {
#pragma unroll
            for (int j = 0; j < 16; ++j) a[j] = fmaxf(v[j], 0.0f);
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) a[j] = v[j];
        }
        const size_t ld = (size_t)ep.ldy;
        bf16 *yh = ep.Ybf + (size_t)t0 * ld + n;
        if (ep.Ybf_lo) {
            bf16 *yl = ep.Ybf_lo + (size_t)t0 * ld + n;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                if (!keep[j]) continue;
                const bf16 hb = __float2bfloat16_rn(a[j]);
                yh[j * ld] = hb;
                yl[j * ld] = __float2bfloat16_rn(a[j] - __bfloat162float(hb));
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (keep[j]) yh[j * ld] = __float2bfloat16_rn(a[j]);
        }
        break;
    }
    default:
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (keep[j]) store_epilogue(ep, t0 + j, n, v[j]);
        break;
    }
}

// Epilogue of token t for the four features nf .. nf + 3 (split-K path), in
// two halves: epilogue_f4_pre issues every load the stores need (row mask, KV
// slot, page offset, the old values of an FMADD) and epilogue_f4_post stores,
// so that a caller can issue the loads of several tokens, and its own partial
// sums, before the first store.  Four consecutive outputs go out as one
// vector store where they are contiguous and aligned.
struct EpiPre {
    float4 old;        // EPI_FMADD: the previous values
    long long off;     // paged modes: row offset; EPI_KVCACHE: slot
    bool keep;
};

__device__ __forceinline__ EpiPre epilogue_f4_pre(const GemmEpilogue &ep, int t, int nf, int N) {
    EpiPre e;
    e.old = make_float4(0.f, 0.f, 0.f, 0.f);
    e.off = -1;
    e.keep = !ep.row_mask || ep.row_mask[t];
    switch (ep.epi) {
    case EPI_FMADD: {
        const float *y = ep.Y + (size_t)t * ep.ldy + nf;
        if (nf + 3 < N && ((reinterpret_cast<uintptr_t>(y) & 15) == 0)) {
            e.old = *reinterpret_cast<const float4 *>(y);
        } else {
            e.old.x = nf < N ? y[0] : 0.0f;
            e.old.y = nf + 1 < N ? y[1] : 0.0f;
            e.old.z = nf + 2 < N ? y[2] : 0.0f;
            e.old.w = nf + 3 < N ? y[3] : 0.0f;
        }
        break;
    }
    case EPI_KVCACHE: e.off = ep.pos[t] - 1; break;
    case EPI_QKV_PAGED:
    case EPI_CAKV_PAGED: {
        bool any_kv = false;
#pragma unroll
        for (int i = 0; i < 4; ++i) any_kv |= !(ep.epi == EPI_QKV_PAGED && nf + i < ep.qdim);
        if (any_kv) e.off = ep.row_off[t];
        break;
    }
    default: break;
    }
    return e;
}

__device__ __forceinline__ void store_bf16x4(bf16 *dst, const float (&a)[4]) {
    __nv_bfloat162 h01 = __floats2bfloat162_rn(a[0], a[1]), h23 = __floats2bfloat162_rn(a[2], a[3]);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t *>(&h01);
    u.y = *reinterpret_cast<const uint32_t *>(&h23);
    *reinterpret_cast<uint2 *>(dst) = u;
}

// EPI_FMADD leaves the four stored values in `stored` (for the row statistics).
__device__ __forceinline__ void epilogue_f4_post(const GemmEpilogue &ep, int t, int nf, int N, const float (&v)[4],
                                                 const EpiPre &e, float (&stored)[4]) {
    if (!e.keep) return;
    switch (ep.epi) {
    case EPI_FMADD: {
        float *y = ep.Y + (size_t)t * ep.ldy + nf;
        const float o[4] = {e.old.x + ep.scale * v[0], e.old.y + ep.scale * v[1], e.old.z + ep.scale * v[2],
                            e.old.w + ep.scale * v[3]};
#pragma unroll
        for (int i = 0; i < 4; ++i) stored[i] = o[i];
        if (nf + 3 < N && ((reinterpret_cast<uintptr_t>(y) & 15) == 0)) {
            *reinterpret_cast<float4 *>(y) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (nf + i < N) y[i] = o[i];
        }
        break;
    }
    case EPI_KVCACHE: {
        const long long slot = e.off;
        if (slot < 0 || slot >= ep.kv_stride) { set_status(CT_STATUS_BAD_ARG); break; }
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (nf + i < N) ep.Y[((size_t)t * ep.kv_stride + slot) * ep.ldy + nf + i] = v[i];
        break;
    }
    case EPI_BF16: {
        float a[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            a[i] = v[i];
            if (ep.act == 1) a[i] = silu_fast(v[i]);
            else if (ep.act == 2) a[i] = v[i] > 0.0f ? v[i] : 0.0f;
        }
        const size_t idx = (size_t)t * ep.ldy + nf;
        if (nf + 3 < N && (idx & 3) == 0 && ((reinterpret_cast<uintptr_t>(ep.Ybf) & 7) == 0) &&
            (!ep.Ybf_lo || (reinterpret_cast<uintptr_t>(ep.Ybf_lo) & 7) == 0)) {
            float hf[4], lf[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                hf[i] = __bfloat162float(__float2bfloat16_rn(a[i]));
                lf[i] = a[i] - hf[i];
            }
            store_bf16x4(ep.Ybf + idx, hf);
            if (ep.Ybf_lo) store_bf16x4(ep.Ybf_lo + idx, lf);
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (nf + i < N) store_epilogue(ep, t, nf + i, v[i]);
        }
        break;
    }
    case EPI_QKV_PAGED:
    case EPI_CAKV_PAGED: {
        const long long off = e.off;
        const bool qpart = ep.epi == EPI_QKV_PAGED && nf < ep.qdim;
        const int n2 = ep.epi == EPI_QKV_PAGED ? nf - ep.qdim : nf;
        if (!qpart && off >= 0 && nf + 3 < N && (nf + 3 >= ep.qdim || ep.epi != EPI_QKV_PAGED) &&
            n2 % ep.kv_width + 3 < ep.kv_width) {
            // four K/V values of one pool row
            const int lk = ep.epi == EPI_QKV_PAGED ? ep.layer * 2 + n2 / ep.kv_width : n2 / ep.kv_width;
            bf16 *dst = ep.kv_pool + off + (long long)lk * kPageRows * ep.kv_width + n2 % ep.kv_width;
            if ((reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
                store_bf16x4(dst, v);
                break;
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int n = nf + i;
            if (n >= N) continue;
            if (ep.epi == EPI_QKV_PAGED && n < ep.qdim) { ep.Y[(size_t)t * ep.ldy + n] = v[i]; continue; }
            if (off < 0) continue;
            const int m2 = ep.epi == EPI_QKV_PAGED ? n - ep.qdim : n;
            const int lk = ep.epi == EPI_QKV_PAGED ? ep.layer * 2 + m2 / ep.kv_width : m2 / ep.kv_width;
            ep.kv_pool[off + (long long)lk * kPageRows * ep.kv_width + m2 % ep.kv_width] = __float2bfloat16_rn(v[i]);
        }
        break;
    }
    default:
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (nf + i < N) store_epilogue(ep, t, nf + i, v[i]);
        break;
    }
}

// Split-K reduction of one CTA's token slice (CS = cluster size): epilogue
// warp w2 handles tokens tb + w2, tb + w2 + 4, ... of the tile, P = min(2, 16 / CS)
// of them per pass; lane owns features 4*lane .. 4*lane + 3.  Per pass every
// load -- the epilogue's, then one 16-byte remote load per (token, CTA) -- is
// issued before the first sum, and the sums run in CTA rank order.
template <int CS>
__device__ __forceinline__ void splitk_reduce(const KernelParams &p, int t0, int T_eff, int n0, int tb, int slice,
                                              int w2, int lane, uint32_t base, const float (&b4)[4]) {
    constexpr int P = CS >= 16 ? 1 : 2;
    const int f0 = 4 * lane;
    for (int j0 = w2; j0 < slice; j0 += 4 * P) {
        if (t0 + tb + j0 >= T_eff) break;
        bool on[P];
        EpiPre pre[P];
#pragma unroll
        for (int pp = 0; pp < P; ++pp) {
            const int j = j0 + 4 * pp;
            on[pp] = j < slice && t0 + tb + j < T_eff;
            if (on[pp]) pre[pp] = epilogue_f4_pre(p.ep, t0 + tb + j, n0 + f0, p.N);
        }
        float4 part[P][CS];
#pragma unroll
        for (int pp = 0; pp < P; ++pp) {
            const uint32_t off = base + (uint32_t)(((tb + j0 + 4 * pp) * BM + f0) * 4);
#pragma unroll
            for (int r = 0; r < CS; ++r)
                if (on[pp]) part[pp][r] = dsmem_ld4(dsmem_addr(off, (uint32_t)r));
        }
#pragma unroll
        for (int pp = 0; pp < P; ++pp) {
            if (!on[pp]) continue;
            float4 sum = part[pp][0];
#pragma unroll
            for (int r = 1; r < CS; ++r) {
                sum.x += part[pp][r].x; sum.y += part[pp][r].y; sum.z += part[pp][r].z; sum.w += part[pp][r].w;
            }
            const float vals[4] = {sum.x + b4[0], sum.y + b4[1], sum.z + b4[2], sum.w + b4[3]};
            float o[4] = {0.f, 0.f, 0.f, 0.f};
            const int t = t0 + tb + j0 + 4 * pp;
            epilogue_f4_post(p.ep, t, n0 + f0, p.N, vals, pre[pp], o);
            if (p.ep.stats_out) {
                // (mean, M2) of the tile's 128 new values of row t: the warp holds
                // all of them (four per lane); the host allows this only for
                // EPI_FMADD without a row mask and N a multiple of 128
                const float m = warp_sum((o[0] + o[1]) + (o[2] + o[3])) * (1.0f / 128.0f);
                const float d0 = o[0] - m, d1 = o[1] - m, d2 = o[2] - m, d3 = o[3] - m;
                const float q = warp_sum((d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3));
                if (lane == 0) p.ep.stats_out[(size_t)t * (p.N / BM) + blockIdx.x] = make_float2(m, q);
            }
        }
    }
}

// LayerNorm-input mode: the four epilogue warps (et = 0..127) form the CTA's
// activation tiles, LN(x[t]) for t in [t0, t0 + BN) over k-blocks kb0 ..
// kb0 + nkb - 1, as bf16 hi (and lo) planes in the layout a 128-byte-swizzled
// TMA load writes: row r of a [BN x 64] tile at r * 128 bytes, its 16-byte
// chunk c at position c ^ (r & 7).  Tiles sit at xs + (kb * planes + plane) *
// BN * 128.  The row's mean and variance merge the eight (mean, M2) partials
// of its 128-feature tiles in tile order (equal counts of 128); rows past the
// device row count are zero.
template <int BN, bool TWO, int NT = 128>
__device__ __forceinline__ void ln_fill(const GemmEpilogue &ep, uint8_t *xs, int t0, int T_eff, int kb0, int nkb,
                                        int et) {
    constexpr int K = 1024;
    constexpr int TPR = BN >= NT ? 1 : NT / BN;     // threads per row
    static_assert(TPR <= 8, "at most eight threads per row (one 16-byte chunk each)");
    constexpr int CPT = 8 / TPR;                    // 16-byte chunks per thread and k-block
    constexpr int RSTEP = NT / TPR;                 // rows per pass of the NT threads
    constexpr uint32_t TILE = BN * 128;
    for (int r = et / TPR; r < BN; r += RSTEP) {
        const int t = t0 + r;
        const int c0 = (et % TPR) * CPT;
        const bool valid = t < T_eff;
        float mu = 0.0f, rs = 0.0f;
        if (valid) {
            const float4 *sp = reinterpret_cast<const float4 *>(ep.ln_stats + (size_t)t * (K / 128));
            const float4 a0 = sp[0], a1 = sp[1], a2 = sp[2], a3 = sp[3];
            const float m[8] = {a0.x, a0.z, a1.x, a1.z, a2.x, a2.z, a3.x, a3.z};
            const float q[8] = {a0.y, a0.w, a1.y, a1.w, a2.y, a2.w, a3.y, a3.w};
            float ms = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) ms += m[j];
            mu = ms * 0.125f;
            float m2 = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float d = m[j] - mu;
                m2 += q[j] + 128.0f * d * d;
            }
            rs = 1.0f / sqrtf(m2 * (1.0f / K) + 1e-5f);
        }
        for (int kb = 0; kb < nkb; ++kb) {
            uint8_t *tile = xs + (size_t)kb * (TWO ? 2 : 1) * TILE;
#pragma unroll
            for (int cc = 0; cc < CPT; ++cc) {
                const int c = c0 + cc;
                uint4 hv = make_uint4(0u, 0u, 0u, 0u), lv = make_uint4(0u, 0u, 0u, 0u);
                if (valid) {
                    const int k = (kb0 + kb) * BK + c * 8;
                    const float4 x0 = *reinterpret_cast<const float4 *>(ep.ln_x + (size_t)t * K + k);
                    const float4 x1 = *reinterpret_cast<const float4 *>(ep.ln_x + (size_t)t * K + k + 4);
                    const uint4 g = *reinterpret_cast<const uint4 *>(ep.ln_g + k);
                    const uint4 b = *reinterpret_cast<const uint4 *>(ep.ln_b + k);
                    const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, bw[4] = {b.x, b.y, b.z, b.w};
                    uint32_t hw[4], lw[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float v[2];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const float gg = __uint_as_float(((gw[i] >> (16 * h)) & 0xFFFFu) << 16);
                            const float bb = __uint_as_float(((bw[i] >> (16 * h)) & 0xFFFFu) << 16);
                            v[h] = (x[2 * i + h] - mu) * rs * gg + bb;
                        }
                        const __nv_bfloat162 hh = __floats2bfloat162_rn(v[0], v[1]);
                        const __nv_bfloat162 ll = __floats2bfloat162_rn(v[0] - __low2float(hh), v[1] - __high2float(hh));
                        hw[i] = *reinterpret_cast<const uint32_t *>(&hh);
                        lw[i] = *reinterpret_cast<const uint32_t *>(&ll);
                    }
                    hv = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    lv = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                }
                const uint32_t off = (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
                *reinterpret_cast<uint4 *>(tile + off) = hv;
                if (TWO) *reinterpret_cast<uint4 *>(tile + TILE + off) = lv;
            }
        }
    }
}

// Greedy-argmax order of (value, index) candidates: the larger value, and the
// lower index among equal values, so the winner is the first index of the
// maximum.  Candidates that are NaN or -inf never win (index INT_MAX).
__device__ __forceinline__ void amax_take(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

// Transposing warp reduction: on entry lane l holds one candidate per token j
// (v[j], ix[j]) for its own feature; on exit v[0], ix[0] of lane l is the
// best of the warp's 32 features for token l.  Five exchange rounds: in the
// round of distance s each lane keeps the half of its tokens selected by bit
// s of its lane id and folds in the partner's copy of that half.
__device__ __forceinline__ void warp_amax_transpose(float (&v)[32], int (&ix)[32], int lane) {
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const bool upper = (lane & s) != 0;
#pragma unroll
        for (int i = 0; i < s; ++i) {
            const float send_v = upper ? v[i] : v[i + s];
            const int send_i = upper ? ix[i] : ix[i + s];
            float keep_v = upper ? v[i + s] : v[i];
            int keep_i = upper ? ix[i + s] : ix[i];
            const float rv = __shfl_xor_sync(0xffffffffu, send_v, s);
            const int ri = __shfl_xor_sync(0xffffffffu, send_i, s);
            amax_take(keep_v, keep_i, rv, ri);
            v[i] = keep_v;
            ix[i] = keep_i;
        }
    }
}

// Named barrier 1 over the NT epilogue threads (the producer and MMA warps do not take part).
template <int NT = 128>
__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }

// Greedy hand-off of the LM head (ArgmaxSink, no K split): the NT epilogue
// threads (et = 0..NT-1) merge the four TMEM lane quarters' per-token maxima
// (red, quarter order = feature order) into one candidate per token row of
// this CTA's vocabulary tile and fold it into the row's key (atomicMax), then
// take ticket rb (the row block) of `tiles`; the CTA that completes the block
// reads the keys and appends each row's token.  Nothing waits on another CTA.
template <int BN, int NT = 128>
__device__ __forceinline__ void argmax_tail(const ArgmaxSink &sk, const float2 *red, int *flag, int t0, int T_eff,
                                            int et, int tiles, int rb) {
    for (int j = et; j < BN; j += NT) {
        if (t0 + j >= T_eff) break;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float2 c = red[(j >> 5) * 128 + w * 32 + (j & 31)];
            amax_take(bv, bi, c.x, __float_as_int(c.y));
        }
        if (bi != 0x7fffffff) atomicMax(&sk.best[t0 + j], argmax_key(bv, bi));
    }
    __threadfence();
    epi_bar_sync<NT>();
    if (et == 0) *flag = atomicAdd(&sk.ticket[rb], 1u) == (unsigned)(tiles - 1);
    epi_bar_sync<NT>();
    if (!*flag) return;
    __threadfence();
    for (int j = et; j < BN; j += NT) {
        const int t = t0 + j;
        if (t >= T_eff) break;
        const unsigned long long key = __ldcg(&sk.best[t]);
        sk.best[t] = 0ull;   // ready for the next step's launch
        decode_append(sk, t, key ? (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull)) : 0);
    }
    if (et == 0) sk.ticket[rb] = 0u;
}

template <int BN, bool TWO>
__global__ void __launch_bounds__(kThreads) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW,
                                                           const __grid_constant__ CUtensorMap tmXh,
                                                           const __grid_constant__ CUtensorMap tmXl,
                                                           const KernelParams p) {
    constexpr uint32_t A_BYTES = BM * BK * 2;
    constexpr uint32_t B_BYTES = BN * BK * 2;
    constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES * (TWO ? 2 : 1);
    constexpr uint32_t NCOLS = BN < 32 ? 32 : BN;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int stages = p.stages;
    // LayerNorm-input mode: stages hold only weight tiles; the activation
    // tiles of all this CTA's k-blocks follow them (see ln_fill)
    const bool lnx = p.ep.ln_x != nullptr;
    const uint32_t stage_bytes = lnx ? A_BYTES : STAGE_BYTES;
    uint8_t *xs = smem + (size_t)stages * stage_bytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.bar_off);
    uint64_t *empty = full + stages;
    uint64_t *accb = empty + stages;
    uint64_t *xfull = accb + 1;   // LayerNorm-input mode: the 128 epilogue threads filled xs
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accb + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BM, t0 = blockIdx.y * BN, z = blockIdx.z;
    // Rows beyond the device row count: every CTA of a cluster shares (n0, t0),
    // so the whole cluster leaves together, before any TMA or TMEM work.  The
    // count is produced at least two kernels upstream (see gemm.cuh).
    const int T_eff = p.ep.T_dev ? min(p.T, *p.ep.T_dev) : p.T;
    if (t0 >= T_eff) return;
    const int kb0 = z * p.kbps;
    const int kb1 = min(kb0 + p.kbps, p.kb_total);
    const int nkb = kb1 - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(accb, 1);
        mbar_init(xfull, 128);
        fence_mbar_init();
        prefetch_tmap(&tmW);
        if (!lnx) {
            prefetch_tmap(&tmXh);
            if (TWO) prefetch_tmap(&tmXl);
        }
    }
    if (warp == 1) { tmem_alloc(tmem_slot, NCOLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Weights do not depend on the previous kernel: start streaming the first
    // stages of this CTA's weight tiles before waiting for it.
    const int pre = min(stages, nkb);
    if (warp == 0 && lane == 0) {
        for (int i = 0; i < pre; ++i) {
            mbar_expect_tx(&full[i], stage_bytes);
            tma_load_2d(smem + (size_t)i * stage_bytes, &tmW, &full[i], (kb0 + i) * BK, n0);
        }
    }
    pdl_wait();
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < nkb; ++i) {
                const int s = i % stages;
                const uint32_t ph = (uint32_t)(i / stages) & 1u;
                uint8_t *a = smem + (size_t)s * stage_bytes;
                const int kc = (kb0 + i) * BK;
                if (i >= pre) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, CT_STATUS_TIMEOUT_FREE)) break;
                    mbar_expect_tx(&full[s], stage_bytes);
                    tma_load_2d(a, &tmW, &full[s], kc, n0);
                }
                if (!lnx) {
                    tma_load_2d(a + A_BYTES, &tmXh, &full[s], kc, t0);
                    if (TWO) tma_load_2d(a + A_BYTES + B_BYTES, &tmXl, &full[s], kc, t0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(BM, BN);
            const bool xok = !lnx || mbar_wait(xfull, 0, CT_STATUS_TIMEOUT_TMA);
            for (int i = 0; i < nkb && xok; ++i) {
                const int s = i % stages;
                const uint32_t ph = (uint32_t)(i / stages) & 1u;
                if (!mbar_wait(&full[s], ph, CT_STATUS_TIMEOUT_TMA)) break;
                tc_fence_after();
                const uint32_t a = smem_u32(smem + (size_t)s * stage_bytes);
                const uint32_t b = lnx ? smem_u32(xs) + (uint32_t)i * (TWO ? 2u : 1u) * B_BYTES : a + A_BYTES;
                const uint64_t ad = sw128_desc(a);
                const uint64_t bd = sw128_desc(b);
#pragma unroll
                for (int k = 0; k < BK / 16; ++k)
                    mma_bf16(tmem, ad + 2 * k, bd + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
                if (TWO) {
                    const uint64_t ld = sw128_desc(b + B_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) mma_bf16(tmem, ad + 2 * k, ld + 2 * k, idesc, 1u);
                }
                mma_commit(&empty[s]);
            }
            mma_commit(accb);
        }
    }
    // ---------------------------------------------------------------- epilogue
    const bool split = p.nsplit > 1;
    const int q = warp & 3;
    const int n = n0 + q * 32 + lane;
    const bool epi_warp = warp >= 2;
    if (epi_warp && lnx) {
        ln_fill<BN, TWO>(p.ep, xs, t0, T_eff, kb0, nkb, threadIdx.x - 64);
        fence_proxy_async_smem();   // the MMA reads these tiles through the async proxy
        mbar_arrive(xfull);
    }
    bool ok = true;
    if (epi_warp) {
        ok = mbar_wait(accb, 0, CT_STATUS_TIMEOUT_MMA);
        ok = __all_sync(0xffffffffu, ok);
        tc_fence_after();
    }
    const float bias = (epi_warp && n < p.N && p.ep.bias) ? bf2f(p.ep.bias[n]) : 0.0f;
    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
    if (!split) {
        const bool amx = p.ep.amax.best != nullptr;
        // argmax hand-off: per-token maxima of each epilogue warp, [BN/32][4][32],
        // in the stage buffers (idle once the accumulator is complete)
        float2 *red = reinterpret_cast<float2 *>(smem);
        if (epi_warp) {
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                if (t0 + c >= T_eff) break;   // warp-uniform
                float v[32];
                if (ok) tmem_ld32(tbase + (uint32_t)c, v);
                if (ok && n < p.N) {
                    const int tl = min(32, T_eff - (t0 + c));
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] += bias;
                    if (p.ep.Y || p.ep.epi != EPI_STORE) {   // EPI_STORE without Y: argmax hand-off only
                        epilogue16(p.ep, t0 + c, min(16, tl), n, v);
                        if (tl > 16) epilogue16(p.ep, t0 + c + 16, tl - 16, n, v + 16);
                    }
                }
                if (amx) {
                    int ix[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const bool cand = ok && n < p.N && v[j] > -INFINITY;
                        ix[j] = cand ? n : 0x7fffffff;
                        v[j] = cand ? v[j] : -INFINITY;
                    }
                    warp_amax_transpose(v, ix, lane);
                    red[(c >> 5) * 128 + q * 32 + lane] = make_float2(v[0], __int_as_float(ix[0]));
                }
            }
            if (amx) {
                epi_bar_sync();
                argmax_tail<BN>(p.ep.amax, red, reinterpret_cast<int *>(red + BN * 4), t0, T_eff, threadIdx.x - 64,
                                gridDim.x, blockIdx.y);
            }
        }
    } else {
        // Split-K across the CTAs of one cluster (grid.z = cluster size): each
        // CTA parks its fp32 accumulator tile in its own shared memory (the
        // pipeline buffers are idle once the accumulator is complete), then CTA
        // r sums tokens [r*BN/cs, (r+1)*BN/cs) of the tile over all CTAs in
        // rank order through distributed shared memory.
        float *acc_s = reinterpret_cast<float *>(smem);   // [BN][BM], feature fastest
        if (epi_warp) {
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                float v[32];
                if (ok) tmem_ld32(tbase + (uint32_t)c, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) acc_s[(c + j) * BM + q * 32 + lane] = ok ? v[j] : 0.0f;
            }
        }
        cluster_sync();
        if (epi_warp) {
            const int cs = p.nsplit;
            const int slice = BN / cs;
            const int tb = (int)cluster_ctarank() * slice;
            const uint32_t base = smem_u32(acc_s);
            const int f0 = 4 * lane;
            float b4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                b4[i] = (n0 + f0 + i < p.N && p.ep.bias) ? bf2f(p.ep.bias[n0 + f0 + i]) : 0.0f;
            switch (cs) {
            case 2: splitk_reduce<2>(p, t0, T_eff, n0, tb, slice, warp - 2, lane, base, b4); break;
            case 4: splitk_reduce<4>(p, t0, T_eff, n0, tb, slice, warp - 2, lane, base, b4); break;
            case 8: splitk_reduce<8>(p, t0, T_eff, n0, tb, slice, warp - 2, lane, base, b4); break;
            case 16: splitk_reduce<16>(p, t0, T_eff, n0, tb, slice, warp - 2, lane, base, b4); break;
            default: if (lane == 0) set_status(CT_STATUS_BAD_ARG); break;   // the host picks powers of two
            }
        }
        cluster_sync();   // no CTA leaves while another still reads its shared memory
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, NCOLS);
}

// Persistent form for large T (no K split, no device row count): one CTA per
// SM walks output tiles tile = blockIdx.x, blockIdx.x + gridDim.x, ...  The
// TMA producer (warp 0) and the MMA issuer (warp 1) run ahead into the next
// tile while the epilogue warps (2..5) drain the previous one: the TMEM holds
// two BN-column accumulators, handed over through acc_full (MMA commit ->
// epilogue) and acc_empty (4 epilogue warps -> MMA).  Per output element the
// MMA sequence over K is the one of gemm_tc_kernel, so both forms give
// bit-identical results.
static constexpr int kThreadsP = 320;   // persistent kernel: TMA warp, MMA warp, 8 epilogue warps

template <int BN, bool TWO, int EPI>
__global__ void __launch_bounds__(kThreadsP, 1) gemm_pers_kernel(const __grid_constant__ CUtensorMap tmW,
                                                                const __grid_constant__ CUtensorMap tmXh,
                                                                const __grid_constant__ CUtensorMap tmXl,
                                                                const KernelParams p) {
    constexpr uint32_t A_BYTES = BM * BK * 2;
    constexpr uint32_t B_BYTES = BN * BK * 2;
    constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES * (TWO ? 2 : 1);
    constexpr uint32_t NCOLS = 2 * BN;   // two accumulators

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int stages = p.stages;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.bar_off);
    uint64_t *empty = full + stages;
    uint64_t *acc_full = empty + stages;     // [2]
    uint64_t *acc_empty = acc_full + 2;      // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_n = (p.N + BM - 1) / BM;
    const int n_tiles = tiles_n * ((p.T + BN - 1) / BN);
    const int nkb = p.kb_total;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], 8); }
        fence_mbar_init();
        prefetch_tmap(&tmW);
        prefetch_tmap(&tmXh);
        if (TWO) prefetch_tmap(&tmXl);
    }
    if (warp == 1) { tmem_alloc(tmem_slot, NCOLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                const int n0 = (tile % tiles_n) * BM, t0 = (tile / tiles_n) * BN;
                for (int i = 0; i < nkb; ++i, ++it) {
                    const int s = (int)(it % (uint32_t)stages);
                    const uint32_t ph = (it / (uint32_t)stages) & 1u;
                    if (it >= (uint32_t)stages && !mbar_wait(&empty[s], ph ^ 1u, CT_STATUS_TIMEOUT_FREE)) { ok = false; break; }
                    uint8_t *a = smem + (size_t)s * STAGE_BYTES;
                    const int kc = i * BK;
                    mbar_expect_tx(&full[s], STAGE_BYTES);
                    tma_load_2d(a, &tmW, &full[s], kc, n0);
                    tma_load_2d(a + A_BYTES, &tmXh, &full[s], kc, t0);
                    if (TWO) tma_load_2d(a + A_BYTES + B_BYTES, &tmXl, &full[s], kc, t0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(BM, BN);
            uint32_t it = 0, lt = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++lt) {
                const uint32_t buf = lt & 1u, use = lt >> 1;
                if (use > 0 && !mbar_wait(&acc_empty[buf], (use - 1) & 1u, CT_STATUS_TIMEOUT_FREE)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * BN;
                for (int i = 0; i < nkb; ++i, ++it) {
                    const int s = (int)(it % (uint32_t)stages);
                    const uint32_t ph = (it / (uint32_t)stages) & 1u;
                    if (!mbar_wait(&full[s], ph, CT_STATUS_TIMEOUT_TMA)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a = smem_u32(smem + (size_t)s * STAGE_BYTES);
                    const uint64_t ad = sw128_desc(a);
                    const uint64_t bd = sw128_desc(a + A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        mma_bf16(d, ad + 2 * k, bd + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
                    if (TWO) {
                        const uint64_t ld = sw128_desc(a + A_BYTES + B_BYTES);
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k) mma_bf16(d, ad + 2 * k, ld + 2 * k, idesc, 1u);
                    }
                    mma_commit(&empty[s]);
                }
                if (ok) mma_commit(&acc_full[buf]);
            }
        }
    } else {
        // epilogue warps 2..9: warp w reads TMEM lanes 32*(w%4).. (its lane
        // quarter) and half (w-2)/4 of the accumulator's BN columns
        const int q = warp & 3;
        const int c_lo = ((warp - 2) >> 2) * (BN / 2), c_hi = c_lo + BN / 2;
        uint32_t lt = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++lt) {
            const uint32_t buf = lt & 1u, use = lt >> 1;
            const int n0 = (tile % tiles_n) * BM, t0 = (tile / tiles_n) * BN;
            bool ok = mbar_wait(&acc_full[buf], use & 1u, CT_STATUS_TIMEOUT_MMA);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            const int n = n0 + q * 32 + lane;
            const float bias = (n < p.N && p.ep.bias) ? bf2f(p.ep.bias[n]) : 0.0f;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + buf * BN;
#pragma unroll 1
            for (int c = c_lo; c < c_hi; c += 32) {
                if (t0 + c >= p.T) break;   // warp-uniform
                float v[32];
                tmem_ld32(tbase + (uint32_t)c, v);
                if (n < p.N) {
                    const int tl = min(32, p.T - (t0 + c));
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] += bias;
                    epilogue16<EPI>(p.ep, t0 + c, min(16, tl), n, v);
                    if (tl > 16) epilogue16<EPI>(p.ep, t0 + c + 16, tl - 16, n, v + 16);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, NCOLS);
}

__global__ void split_fp32_kernel(const float *__restrict__ x, int T, int K, int ldx, bf16 *__restrict__ hi,
                                  bf16 *__restrict__ lo, int Kp) {
    const size_t total = (size_t)T * Kp;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / Kp), k = (int)(i % Kp);
        const float v = k < K ? x[(size_t)t * ldx + k] : 0.0f;
        const bf16 h = __float2bfloat16_rn(v);
        hi[i] = h;
        if (lo) lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
}

// ---------------------------------------------------------------- host ------

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        CT_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p) CT_FATAL("cuTensorMapEncodeTiled unavailable");
        fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

struct MapKey {
    const void *p;
    long rows, cols, box;
    bool operator==(const MapKey &o) const { return p == o.p && rows == o.rows && cols == o.cols && box == o.box; }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const {
        return std::hash<const void *>()(k.p) ^ (std::hash<long>()(k.rows) * 31) ^ (std::hash<long>()(k.cols) * 131) ^
               (std::hash<long>()(k.box) * 7919);
    }
};

struct WCopy {
    bf16 *p;
    int Kp;
};

struct GemmCtx {
    int device = -1;
    bf16 *xhi = nullptr, *xlo = nullptr;
    size_t x_elems = 0;
    std::unordered_map<MapKey, CUtensorMap, MapKeyHash> maps;
    std::unordered_map<const void *, WCopy> wcopies;
};

static thread_local std::unique_ptr<GemmCtx> t_ctx;

static bool capturing(cudaStream_t st) {
    cudaStreamCaptureStatus s = cudaStreamCaptureStatusNone;
    CT_CHECK(cudaStreamIsCapturing(st, &s));
    return s != cudaStreamCaptureStatusNone;
}

GemmCtx *gemm_ctx() {
    int dev = 0;
    CT_CHECK(cudaGetDevice(&dev));
    if (t_ctx && t_ctx->device != dev) gemm_ctx_release();
    if (!t_ctx) {
        t_ctx.reset(new GemmCtx());
        t_ctx->device = dev;
        t_ctx->x_elems = 16ull << 20;
        CT_CHECK(cudaMalloc(&t_ctx->xhi, t_ctx->x_elems * sizeof(bf16)));
        CT_CHECK(cudaMalloc(&t_ctx->xlo, t_ctx->x_elems * sizeof(bf16)));
    }
    return t_ctx.get();
}

void gemm_ctx_release() {
    if (!t_ctx) return;
    int cur = 0;
    CT_CHECK(cudaGetDevice(&cur));
    CT_CHECK(cudaSetDevice(t_ctx->device));
    CT_CHECK(cudaDeviceSynchronize());
    cudaFree(t_ctx->xhi);
    cudaFree(t_ctx->xlo);
    for (auto &kv : t_ctx->wcopies) cudaFree(kv.second.p);
    t_ctx.reset();
    CT_CHECK(cudaSetDevice(cur));
}

static const CUtensorMap &tmap_bf16(GemmCtx *c, const void *ptr, long rows, long cols, long box_rows) {
    MapKey key{ptr, rows, cols, box_rows};
    auto it = c->maps.find(key);
    if (it != c->maps.end()) return it->second;
    if (((uintptr_t)ptr & 15) || (cols & 7)) CT_FATAL("TMA operand not 16-byte aligned (ptr %p, cols %ld)", ptr, cols);
    CUtensorMap m;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
                             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) CT_FATAL("cuTensorMapEncodeTiled failed (%d) rows %ld cols %ld box %ld", (int)r, rows, cols, box_rows);
    return c->maps.emplace(key, m).first->second;
}

int split_factor(int N, int K) {
    const int tiles = (N + BM - 1) / BM;
    const int kb = (K + BK - 1) / BK;
    if ((long)N * K > 4l * 1024 * 1024) return 1;
    int s = 1;
    while (s < 16 && tiles * s * 2 <= 256 && kb / (s * 2) >= 1) s *= 2;
    return s;
}

int gemm_nsplit(int N, int K, int BN, int requested) {
    const int kb_total = (K + BK - 1) / BK;
    int nsplit = requested > 0 ? std::min(requested, 16) : split_factor(N, K);
    while (nsplit > 1 && BN % nsplit) nsplit >>= 1;
    const int kbps = (kb_total + nsplit - 1) / nsplit;
    if ((kb_total + kbps - 1) / kbps != nsplit) nsplit = 1;   // every split must own >= 1 block
    return nsplit;
}

CUtensorMap gemm_tmap(const void *ptr, long rows, long cols, long box_rows) {
    return tmap_bf16(gemm_ctx(), ptr, rows, cols, box_rows);
}

template <int BN, bool TWO>
static void launch_tc(cudaStream_t st, const CUtensorMap &mw, const CUtensorMap &mh, const CUtensorMap &ml,
                      KernelParams p, bool pdl) {
    // LayerNorm-input mode: weight-only stages, then the activation tiles of
    // all of a CTA's k-blocks
    const bool lnx = p.ep.ln_x != nullptr;
    const int STAGE = lnx ? BM * BK * 2 : BM * BK * 2 + BN * BK * 2 * (TWO ? 2 : 1);
    const int xbytes = lnx ? p.kbps * BN * BK * 2 * (TWO ? 2 : 1) : 0;
    // large clusters: keep two CTAs per SM so a 16-CTA cluster fits in a GPC
    const int budget = p.nsplit > 8 ? 100 * 1024 : kSmemBudget;
    if (xbytes + STAGE + 2048 > budget) CT_FATAL("LayerNorm-input GEMM tile does not fit: %d B of activations", xbytes);
    const int max_stages = std::max(1, (budget - 2048 - xbytes) / STAGE);
    p.stages = std::min(std::min(p.kbps, max_stages), 8);
    size_t body = (size_t)p.stages * STAGE + xbytes;
    if (p.nsplit > 1) body = std::max(body, (size_t)BM * BN * sizeof(float));   // parked accumulator
    p.bar_off = (int)((body + 15) & ~(size_t)15);
    const size_t smem = 1024 + p.bar_off + 16 * (2 * p.stages + 2);
    static thread_local int configured_dev = -1;   // per instantiation and thread
    int dev = 0;
    CT_CHECK(cudaGetDevice(&dev));
    if (configured_dev != dev) {
        CT_CHECK(cudaFuncSetAttribute(gemm_tc_kernel<BN, TWO>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kSmemBudget));
        // K-split clusters of 16 CTAs exceed the portable limit of 8
        CT_CHECK(cudaFuncSetAttribute(gemm_tc_kernel<BN, TWO>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        configured_dev = dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.N + BM - 1) / BM, (p.T + BN - 1) / BN, p.nsplit);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (p.nsplit > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = 1;
        at[na].val.clusterDim.y = 1;
        at[na].val.clusterDim.z = p.nsplit;
        ++na;
    }
    if (pdl) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    if (p.nsplit > 1) {
        // a cluster shape the device cannot schedule would fail the launch
        static thread_local std::unordered_map<long, int> fits;
        const long key = ((long)dev << 40) | ((long)p.nsplit << 32) | (long)smem;
        auto it = fits.find(key);
        if (it == fits.end()) {
            int n = 0;
            cudaLaunchConfig_t q = cfg;
            q.attrs = at;
            q.numAttrs = 1;   // cluster attribute only
            if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<BN, TWO>, &q) != cudaSuccess) n = 0;
            cudaGetLastError();
            it = fits.emplace(key, n).first;
        }
        if (it->second <= 0) CT_FATAL("GEMM cluster of %d CTAs with %zu B shared memory cannot be scheduled", p.nsplit, smem);
    }
    CT_CHECK(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, TWO>, mw, mh, ml, p));
}

template <int BN, bool TWO, int EPI>
static void launch_pers(cudaStream_t st, const CUtensorMap &mw, const CUtensorMap &mh, const CUtensorMap &ml,
                        KernelParams p, bool pdl) {
    constexpr int STAGE = BM * BK * 2 + BN * BK * 2 * (TWO ? 2 : 1);
    p.stages = std::min(std::max(1, (kSmemBudget - 2048) / STAGE), 8);
    p.nsplit = 1;
    p.bar_off = p.stages * STAGE;
    const size_t smem = 1024 + p.bar_off + 8 * (2 * p.stages + 4) + 16;
    static thread_local int configured_dev = -1;
    int dev = 0;
    CT_CHECK(cudaGetDevice(&dev));
    static thread_local int n_sm = 0;
    if (configured_dev != dev) {
        CT_CHECK(cudaFuncSetAttribute(gemm_pers_kernel<BN, TWO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kSmemBudget));
        CT_CHECK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
        configured_dev = dev;
    }
    const int n_tiles = ((p.N + BM - 1) / BM) * ((p.T + BN - 1) / BN);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min(n_tiles, n_sm));
    cfg.blockDim = dim3(kThreadsP);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    CT_CHECK(cudaLaunchKernelEx(&cfg, gemm_pers_kernel<BN, TWO, EPI>, mw, mh, ml, p));
}

// The persistent kernel compiled per epilogue kind the encoder and admission use.
template <int BN, bool TWO>
static void launch_pers_epi(cudaStream_t st, const CUtensorMap &mw, const CUtensorMap &mh, const CUtensorMap &ml,
                            const KernelParams &p, bool pdl) {
    switch (p.ep.epi) {
    case EPI_STORE: launch_pers<BN, TWO, EPI_STORE>(st, mw, mh, ml, p, pdl); break;
    case EPI_RELU: launch_pers<BN, TWO, EPI_RELU>(st, mw, mh, ml, p, pdl); break;
    case EPI_FMADD: launch_pers<BN, TWO, EPI_FMADD>(st, mw, mh, ml, p, pdl); break;
    case EPI_BF16: launch_pers<BN, TWO, EPI_BF16>(st, mw, mh, ml, p, pdl); break;
    case EPI_RELU_FLAT: launch_pers<BN, TWO, EPI_RELU_FLAT>(st, mw, mh, ml, p, pdl); break;
    case EPI_CAKV_PAGED: launch_pers<BN, TWO, EPI_CAKV_PAGED>(st, mw, mh, ml, p, pdl); break;
    default: launch_pers<BN, TWO, -1>(st, mw, mh, ml, p, pdl); break;
    }
}

void gemm_bf16(cudaStream_t st, const bf16 *W, int N, int K, const bf16 *X_hi, const bf16 *X_lo, int T,
               const GemmEpilogue &ep_in, bool allow_split) {
    if (T <= 0 || N <= 0) return;
    GemmCtx *c = gemm_ctx();
    GemmEpilogue ep = ep_in;
    if (ep.ldy == 0) ep.ldy = N;
    const bool two = X_lo != nullptr;
    int BN = T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : (two ? 128 : 256);
    const int kb_total = (K + BK - 1) / BK;
    const int nsplit = allow_split ? gemm_nsplit(N, K, BN, ep.split) : 1;
    const int kbps = (kb_total + nsplit - 1) / nsplit;
    const int kbps_final = nsplit > 1 ? kbps : kb_total;
    // X maps use the scratch capacity (or the caller's buffer rows) as the row count
    const long xrows = (X_hi == c->xhi || X_hi == c->xlo) ? (long)(c->x_elems / K) : (ep.x_rows > 0 ? ep.x_rows : (long)T);
    // large problems without K split or device row count: persistent kernel
    const bool pers = nsplit == 1 && !ep.T_dev && !ep.ln_x && T > (two ? 64 : 128);
    if (pers) BN = two ? 128 : 256;
    if (ep.ln_x && (K != 1024 || !ep.ln_stats || !ep.ln_g || !ep.ln_b || (((uintptr_t)ep.ln_g | (uintptr_t)ep.ln_b) & 15)))
        CT_FATAL("LayerNorm-input GEMM needs K = 1024, row statistics and 16-byte aligned LN weights");
    if (ep.stats_out && (ep.epi != EPI_FMADD || ep.row_mask || N % BM || nsplit < 2))
        CT_FATAL("row statistics need EPI_FMADD with a K split, no row mask and N a multiple of %d", BM);
    if (ep.amax.best && (ep.epi != EPI_STORE || ep.row_mask || nsplit != 1 || pers || ep.ln_x || !ep.amax.ticket ||
                         !ep.amax.next || !ep.T_dev))
        CT_FATAL("the argmax hand-off needs EPI_STORE without a K split, a device row count and its ticket buffers");
    if (ep.epi == EPI_STORE && !ep.Y && !ep.amax.best) CT_FATAL("GEMM without an output");
    const CUtensorMap &mw = tmap_bf16(c, W, N, K, BM);
    const CUtensorMap &mh = tmap_bf16(c, X_hi, xrows, K, BN);
    const CUtensorMap &ml = two ? tmap_bf16(c, X_lo, xrows, K, BN) : mh;
    KernelParams p;
    p.N = N; p.K = K; p.T = T; p.kbps = kbps_final; p.kb_total = kb_total; p.stages = 1;
    p.nsplit = nsplit; p.bar_off = 0;
    p.ep = ep;
    if (pers) {
        two ? launch_pers_epi<128, true>(st, mw, mh, ml, p, ep.pdl) : launch_pers_epi<256, false>(st, mw, mh, ml, p, ep.pdl);
        return;
    }
    switch (BN) {
    case 32: two ? launch_tc<32, true>(st, mw, mh, ml, p, ep.pdl) : launch_tc<32, false>(st, mw, mh, ml, p, ep.pdl); break;
    case 64: two ? launch_tc<64, true>(st, mw, mh, ml, p, ep.pdl) : launch_tc<64, false>(st, mw, mh, ml, p, ep.pdl); break;
    case 128: two ? launch_tc<128, true>(st, mw, mh, ml, p, ep.pdl) : launch_tc<128, false>(st, mw, mh, ml, p, ep.pdl); break;
    default: launch_tc<256, false>(st, mw, mh, ml, p, ep.pdl); break;
    }
}

void split_fp32_to_bf16(cudaStream_t st, const float *x, int T, int K, int ldx, bf16 *hi, bf16 *lo, int Kp) {
    const size_t total = (size_t)T * Kp;
    if (!total) return;
    int blocks = (int)((total + 255) / 256);
    if (blocks > 148 * 16) blocks = 148 * 16;
    split_fp32_kernel<<<blocks, 256, 0, st>>>(x, T, K, ldx, hi, lo, Kp);
    CT_CHECK(cudaGetLastError());
}

static const bf16 *usable_weight(GemmCtx *c, cudaStream_t st, const bf16 *W, int N, int K, int Kp) {
    if (((uintptr_t)W & 15) == 0 && Kp == K) return W;
    auto it = c->wcopies.find(W);
    if (it != c->wcopies.end() && it->second.Kp == Kp) return it->second.p;
    if (capturing(st)) CT_FATAL("weight at %p needs an aligned copy; first use may not be inside graph capture", (const void *)W);
    bf16 *cp = nullptr;
    CT_CHECK(cudaMalloc(&cp, (size_t)N * Kp * sizeof(bf16)));
    CT_CHECK(cudaMemsetAsync(cp, 0, (size_t)N * Kp * sizeof(bf16), st));
    CT_CHECK(cudaMemcpy2DAsync(cp, (size_t)Kp * 2, W, (size_t)K * 2, (size_t)K * 2, N, cudaMemcpyDeviceToDevice, st));
    c->wcopies[W] = WCopy{cp, Kp};
    return cp;
}

void linear_fp32(cudaStream_t st, const bf16 *W, int N, int K, const float *X, int T, int ldx,
                 const GemmEpilogue &ep, bool allow_split, bool two_term) {
    if (T <= 0 || N <= 0) return;
    GemmCtx *c = gemm_ctx();
    const int Kp = (K + 7) & ~7;
    const bf16 *Wu = usable_weight(c, st, W, N, K, Kp);
    if ((size_t)T * Kp > c->x_elems) {
        if (capturing(st)) CT_FATAL("activation scratch too small inside graph capture (T %d, K %d)", T, K);
        CT_CHECK(cudaStreamSynchronize(st));
        scratch_moved();
        cudaFree(c->xhi);
        cudaFree(c->xlo);
        for (auto it = c->maps.begin(); it != c->maps.end();)
            it = (it->first.p == c->xhi || it->first.p == c->xlo) ? c->maps.erase(it) : std::next(it);
        c->x_elems = (size_t)T * Kp * 2;
        CT_CHECK(cudaMalloc(&c->xhi, c->x_elems * sizeof(bf16)));
        CT_CHECK(cudaMalloc(&c->xlo, c->x_elems * sizeof(bf16)));
    }
    split_fp32_to_bf16(st, X, T, K, ldx, c->xhi, two_term ? c->xlo : nullptr, Kp);
    gemm_bf16(st, Wu, N, Kp, c->xhi, two_term ? c->xlo : nullptr, T, ep, allow_split);
}

}  // namespace ct
