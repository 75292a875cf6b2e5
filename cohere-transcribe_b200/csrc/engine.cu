// engine.cu -- continuous-batching decode engine (include/ct_engine.h).
//
// Device state per engine (one GPU, one host thread):
//   slot table (SoA): state, current token, filled KV rows, generated count,
//                     forced length, T_enc, self/cross page tables, output tokens
//   page pool (bf16): [page][DEC_N][K,V][16 rows][DEC_D]
//   step buffers sized for max_rows packed query rows
// One step = build rows (block prefix sum over slots) -> embed+LN ->
// DEC_N x [QKV GEMM (K/V scattered into pages), paged self-attention,
// O GEMM + residual, Q GEMM, paged cross-attention, O GEMM + residual,
// FFN1 (ReLU), FFN2 + residual] -> final LN of each sequence's last row ->
// LM head GEMM -> argmax + retire / append on the GPU.  The pre-LayerNorms of
// the Q, FFN1 and (from layer 1) QKV GEMMs run inside those GEMMs, from row
// statistics the residual GEMMs leave behind.  Kernels read the row and
// sequence counts from device memory, so one captured graph per capacity
// bucket serves every step.
#include <algorithm>
#include <atomic>
#include <sched.h>
#include <stdlib.h>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <map>
#include <mutex>
#include <string>
#include <string.h>
#include <thread>
#include <vector>

#include "../../include/ct_engine.h"
#include "gemm.cuh"
#include "kernels.cuh"
#include "encoder.cu"

namespace ct {
namespace eng {

constexpr int D = DEC_D, FF = DEC_FF, H = DEC_H, DK = DEC_DK, NL = DEC_N, V = VOCAB;
constexpr int PR = kPageRows;
constexpr int SELF_PAGES = MAX_SEQ / PR;     // 64
constexpr int CROSS_PAGES = 64;              // T_enc <= 1024
constexpr long long PAGE_ELEMS = (long long)NL * 2 * PR * D;
constexpr int PROMPT_MAX = 96;                 // longest prompt (the reference's long-form prompts reach 2 + 64 + 16)
constexpr int AW = 8;                          // consumer warps per attention CTA (one per head)
constexpr int ANST = 3;                        // page stages in the attention pipeline
constexpr int GP = 4;                          // pages per attention group: a row's keys are cut into
                                               // fixed groups of GP pages, whatever else is in the batch
constexpr int SEG_MAX = (SELF_PAGES > CROSS_PAGES ? SELF_PAGES : CROSS_PAGES) / GP;   // groups per row

struct DevState {
    int *state, *tok, *pos, *gen, *forced, *tenc;
    int *self_pt, *cross_pt;     // [slots][64]
    int *out_tok;                // [slots][MAX_SEQ]
    int *prompt;                 // [slots][PROMPT_MAX]: each slot's prompt (written at admission)
    int *plen;                   // [slots]: its length
    int *done_map;               // host-mapped [slots]: n_gen when finished (device pointer)
    // per-step rows
    int *r_slot, *r_pos, *r_tok;
    long long *r_off;            // self page offset of each row
    int *q_row, *q_slot;         // per sequence: last row, slot
    int *n_rows, *n_seqs;        // device counts
    // attention page lists of the step (self, cross): one entry per (row, page):
    // meta = row | page-in-row << 10 | (valid keys - 1) << 16 | last-page << 20
    //        | written-this-step << 21
    int *w_self, *w_cross;       // meta, [rows * 64]
    int *pid_self, *pid_cross;   // pool page id, [rows * 64]
    int *rp_self, *rp_cross;     // per row: first entry (prefix sum over rows), [rows + 1]
    int *n_wself, *n_wcross;     // entry counts
    int *grp_self, *grp_cross;   // first entry of each group (rows in order, GP entries per group), [rows * 32 + 1]
    int *n_grp;                  // [2]: group counts (self, cross)
    int *crange;                 // [2][n_cta + 1]: first entry of each attention CTA's range (self, cross)
    int max_slots, max_rows, n_prompt;
    int n_cta;                   // attention grid (one CTA per SM)
};

// ------------------------------------------------------------ kernels -----
// Block-wide exclusive scan of NV values per thread at once (blockDim = 1024):
// out[v] = sum of v-th values of threads < this one, total[v] = block sum.
template <int NV>
__device__ void block_excl_scan_n(const int (&v)[NV], int (&out)[NV], int (&total)[NV], int (*tmp)[64]) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        x[k] = v[k];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x[k], o);
            if (lane >= o) x[k] += y;
        }
        if (lane == 31) tmp[k][w] = x[k];
    }
    __syncthreads();
    if (w < NV) {   // warp k scans the 32 warp totals of value k
        int t = tmp[w][lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        tmp[w][32 + lane] = t;   // inclusive per-warp prefix
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        out[k] = (w > 0 ? tmp[k][32 + w - 1] : 0) + x[k] - v[k];
        total[k] = tmp[k][63];
    }
}

// Packs the step: thread i (slot i) counts its rows, pages and page groups; one
// block scan gives every slot its offsets; the thread writes its rows'
// (slot, position, token, self-page offset).  Then warp w lists the attention
// pages of sequences w, w + 32, ... with the lanes over pages: the slot's page
// ids are loaded once (read-only path), then each row's self entries (causal
// prefix of the slot's pages) and cross entries (all its encoder pages) are
// stored, rows in order, with the group starts and per-row first entries.
// Finally the per-CTA entry ranges of the attention grid.
__global__ void __launch_bounds__(1024) build_rows_kernel(DevState s, int row_cap, int seq_cap) {
    __shared__ int tmp[6][64];
    __shared__ int4 seq_a[1024];   // per sequence: slot, first row, rows, position (-1: prefill)
    __shared__ int4 seq_b[1024];   // per sequence: first self entry, first cross entry, first self / cross group
    __shared__ int seq_te[1024];   // per sequence: encoder rows
    const int i = threadIdx.x;
    const int st = i < s.max_slots ? s.state[i] : SEQ_FREE;
    const int nr = st == SEQ_PREFILL ? s.plen[i] : st == SEQ_DECODE ? 1 : 0;
    const int te = nr > 0 ? s.tenc[i] : 0;
    const int pos = st == SEQ_DECODE ? s.pos[i] : -1;
    const int cross_np = (te + PR - 1) / PR;
    int self_np = 0, self_ng = 0;   // self-attention pages and groups over the slot's rows
    if (st == SEQ_PREFILL) {
        for (int j = 0; j < nr; ++j) {
            const int np = (j + 1 + PR - 1) / PR;
            self_np += np;
            self_ng += (np + GP - 1) / GP;
        }
    } else if (st == SEQ_DECODE) {
        self_np = (pos + 1 + PR - 1) / PR;
        self_ng = (self_np + GP - 1) / GP;
    }
    const int cross_ng = (cross_np + GP - 1) / GP;
    const int cnt[6] = {nr, nr > 0 ? 1 : 0, self_np, nr * cross_np, self_ng, nr * cross_ng};
    int off[6], tot[6];
    block_excl_scan_n<6>(cnt, off, tot, tmp);
    const int base = off[0], sidx = off[1];
    const int total = tot[0], nseq = tot[1], n_ps = tot[2], n_pc = tot[3], n_gs = tot[4], n_gc = tot[5];
    if (total > row_cap || nseq > seq_cap) {   // the host bounds admissions; never expected
        if (i == 0) { set_status(CT_STATUS_BAD_ARG); *s.n_rows = 0; *s.n_seqs = 0; }
        if (i <= s.n_cta) { s.crange[i] = 0; s.crange[s.n_cta + 1 + i] = 0; }
        return;
    }
    for (int j = 0; j < nr; ++j) {
        const int r = base + j;
        const int p = st == SEQ_PREFILL ? j : pos;
        s.r_slot[r] = i;
        s.r_pos[r] = p;
        s.r_tok[r] = st == SEQ_PREFILL ? s.prompt[i * PROMPT_MAX + j] : s.tok[i];
        const int page = (p >= 0 && p < MAX_SEQ) ? s.self_pt[i * SELF_PAGES + p / PR] : -1;
        s.r_off[r] = page >= 0 ? (long long)page * PAGE_ELEMS + (long long)(p % PR) * D : -1;
    }
    if (nr > 0) {
        s.q_row[sidx] = base + nr - 1;
        s.q_slot[sidx] = i;
        seq_a[sidx] = make_int4(i, base, nr, pos);
        seq_b[sidx] = make_int4(off[2], off[3], off[4], off[5]);
        seq_te[sidx] = te;
    }
    if (i == 0) {
        *s.n_rows = total; *s.n_seqs = nseq; *s.n_wself = n_ps; *s.n_wcross = n_pc;
        s.n_grp[0] = n_gs;
        s.n_grp[1] = n_gc;
        s.rp_self[total] = n_ps;
        s.rp_cross[total] = n_pc;
        s.grp_self[n_gs] = n_ps;
        s.grp_cross[n_gc] = n_pc;
    }
    __syncthreads();
    // attention page lists, rows in order: row r's entries are [rp[r], rp[r+1])
    const int lane = i & 31;
    for (int q = i >> 5; q < nseq; q += 32) {
        const int4 a = seq_a[q], b = seq_b[q];
        const int slot = a.x, r0 = a.y, rows = a.z, dpos = a.w;
        const int tq = seq_te[q];
        const int cnp = (tq + PR - 1) / PR, cng = (cnp + GP - 1) / GP;
        // lane k holds page ids k and k + 32 of both tables (64 each)
        const int sp0 = __ldg(s.self_pt + slot * SELF_PAGES + lane), sp1 = __ldg(s.self_pt + slot * SELF_PAGES + 32 + lane);
        const int cp0 = __ldg(s.cross_pt + slot * CROSS_PAGES + lane), cp1 = __ldg(s.cross_pt + slot * CROSS_PAGES + 32 + lane);
        int gs = b.x, gc = b.y, qs = b.z, qc = b.w;
        for (int j = 0; j < rows; ++j) {
            const int r = r0 + j;
            const bool prefill = dpos < 0;
            const int L = (prefill ? j : dpos) + 1;      // causal: keys 0 .. position
            const int np = min((L + PR - 1) / PR, SELF_PAGES);
            const int ng = (np + GP - 1) / GP;
            for (int g = lane; g < ng; g += 32) s.grp_self[qs + g] = gs + g * GP;
            for (int g = lane; g < cng; g += 32) s.grp_cross[qc + g] = gc + g * GP;
            if (lane == 0) { s.rp_self[r] = gs; s.rp_cross[r] = gc; }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int k = lane + 32 * h;
                if (k < np) {
                    int pid = h ? sp1 : sp0;
                    if (pid < 0) { set_status(CT_STATUS_BAD_ARG); pid = 0; }
                    const int nv = min(PR, L - k * PR);
                    // bit 21: written by this step's QKV projection (every page of a
                    // prefill row, the last page of a decode row)
                    const int fresh = prefill || k == np - 1;
                    s.pid_self[gs + k] = pid;
                    s.w_self[gs + k] = r | k << 10 | (nv - 1) << 16 | (k == np - 1) << 20 | fresh << 21;
                }
                if (k < cnp) {
                    int pid = h ? cp1 : cp0;
                    if (pid < 0) { set_status(CT_STATUS_BAD_ARG); pid = 0; }
                    const int nv = min(PR, tq - k * PR);
                    s.pid_cross[gc + k] = pid;
                    s.w_cross[gc + k] = r | k << 10 | (nv - 1) << 16 | (k == cnp - 1) << 20;
                }
            }
            gs += np; gc += cnp; qs += ng; qc += cng;
        }
    }
    // attention CTA b takes groups [b*NG/G, (b+1)*NG/G) of G = min(n_cta, NG)
    // equal shares; CTAs b >= G get an empty range
    __syncthreads();
    if (i <= s.n_cta) {
        for (int c = 0; c < 2; ++c) {
            const int NG = c ? n_gc : n_gs;
            const int *grp = c ? s.grp_cross : s.grp_self;
            const int G = max(1, min(s.n_cta, NG));
            const int b = min(i, G);
            s.crange[c * (s.n_cta + 1) + i] = grp[(int)((long long)b * NG / G)];
        }
    }
}

__device__ __forceinline__ void store_planes(float v, bf16 *hi, bf16 *lo, size_t idx) {
    const bf16 h = __float2bfloat16_rn(v);
    hi[idx] = h;
    if (lo) lo[idx] = __float2bfloat16_rn(v - __bfloat162float(h));
}

__device__ __forceinline__ float block_sum256e(float v, float *red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k];
    return t;
}

// h[r] = LN_e(etw[tok] + epw[pos]) (fp32) and the bf16 planes of LN_1(h[r])
// (the first decoder layer's self-attention LayerNorm); rows r < *n.
__global__ void __launch_bounds__(256) embed_rows_kernel(DevState s, const bf16 *etw, const bf16 *epw,
                                                         const bf16 *lnw, const bf16 *lnb, const bf16 *ln1w,
                                                         const bf16 *ln1b, float *h, bf16 *hi, bf16 *lo) {
    pdl_wait();
    pdl_trigger();
    __shared__ float row[D];
    __shared__ float red[8];
    const int r = blockIdx.x;
    if (r >= *s.n_rows) return;
    const int id = s.r_tok[r], p = s.r_pos[r];
    if (id < 0 || id >= V || p < 0 || p >= MAX_SEQ) { if (threadIdx.x == 0) set_status(CT_STATUS_BAD_ARG); return; }
    float sum = 0.0f;
    for (int k = threadIdx.x; k < D; k += 256) {
        const float v = bf2f(etw[(size_t)id * D + k]) + bf2f(epw[(size_t)p * D + k]);
        row[k] = v;
        sum += v;
    }
    const float mean = block_sum256e(sum, red) / D;
    float var = 0.0f;
    for (int k = threadIdx.x; k < D; k += 256) { const float c = row[k] - mean; var += c * c; }
    const float inv = 1.0f / sqrtf(block_sum256e(var, red) / D + 1e-5f);
    float s2 = 0.0f;
    for (int k = threadIdx.x; k < D; k += 256) {
        const float o = (row[k] - mean) * inv * bf2f(lnw[k]) + bf2f(lnb[k]);
        h[(size_t)r * D + k] = o;
        row[k] = o;
        s2 += o;
    }
    const float mean2 = block_sum256e(s2, red) / D;
    float var2 = 0.0f;
    for (int k = threadIdx.x; k < D; k += 256) { const float c = row[k] - mean2; var2 += c * c; }
    const float inv2 = 1.0f / sqrtf(block_sum256e(var2, red) / D + 1e-5f);
    for (int k = threadIdx.x; k < D; k += 256)
        store_planes((row[k] - mean2) * inv2 * bf2f(ln1w[k]) + bf2f(ln1b[k]), hi, lo, (size_t)r * D + k);
}

// planes[r] = LN(h[src(r)]) for r < *n; src(r) = rows ? rows[r] : r.
__global__ void __launch_bounds__(256) ln_rows_kernel(const int *n, const int *rows, const float *h, const bf16 *w,
                                                      const bf16 *b, bf16 *hi, bf16 *lo) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[8];
    const int r = blockIdx.x;
    if (r >= *n) return;
    const float *x = h + (size_t)(rows ? rows[r] : r) * D;
    float v[D / 256];
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < D / 256; ++j) { v[j] = x[threadIdx.x + 256 * j]; sum += v[j]; }
    const float mean = block_sum256e(sum, red) / D;
    float var = 0.0f;
#pragma unroll
    for (int j = 0; j < D / 256; ++j) { const float c = v[j] - mean; var += c * c; }
    const float inv = 1.0f / sqrtf(block_sum256e(var, red) / D + 1e-5f);
#pragma unroll
    for (int j = 0; j < D / 256; ++j) {
        const int k = threadIdx.x + 256 * j;
        store_planes((v[j] - mean) * inv * bf2f(w[k]) + bf2f(b[k]), hi, lo, (size_t)r * D + k);
    }
}

// Paged attention over bf16 K/V with bulk-copied pages.  The row builder lists
// every (row, 16-key page) entry of the step, rows in order, and cuts each row
// into fixed groups of GP pages; CTA b takes the entry range the builder wrote
// for it (equal shares of the groups).  Row r of slot s attends, in self mode,
// to positions [0, r_pos[r]] of the slot's self pages (the causal prefix; a
// decode row is its last position), in cross mode to rows [0, T_enc[s]) of its
// cross pages.  Warp AW streams each entry's K page (32 KB) and V page (32 KB),
// contiguous in the pool, into a ring of ANST shared-memory stages with
// cp.async.bulk; warps 0..AW-1 (head = warp) read their head's 256-byte slices,
// reduce the 16 scores of a page with a butterfly over the lanes and keep an
// online softmax per group.  A one-group row is written directly; otherwise
// each group leaves (m, l, o) per head in ws and takes a per-(row, head)
// ticket, and the warp holding the last ticket merges the row's groups in
// order (lane c loads group c's (m, l); the o loads go four groups at a time).
struct AttnSmem {
    bf16 kv[ANST][2][PR * D];                  // [stage][K,V][16 rows x 1024]
    float pbuf[AW][PR];                        // per consumer warp: the page's probabilities
    uint64_t full[ANST], empty[ANST];
};
static_assert(SEG_MAX <= 32, "a row's groups are merged one per lane");


__global__ void __launch_bounds__((AW + 1) * 32, 1) attn_paged_kernel(DevState s, const float *Q, const bf16 *pool,
                                                                      int layer, int cross, bf16 *hi, bf16 *lo,
                                                                      float *ws, int *tickets) {
    extern __shared__ __align__(128) uint8_t asmem_raw[];
    AttnSmem &sm = *reinterpret_cast<AttnSmem *>(asmem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < ANST; ++i) { mbar_init(&sm.full[i], 1); mbar_init(&sm.empty[i], AW); }
        fence_mbar_init();
    }
    __syncthreads();
    // The page lists (row builder), the cross pages and the self pages of
    // earlier steps are written at least two kernels upstream, so they may be
    // read before the dependency wait (this kernel's predecessor completes only
    // after every kernel before it has).  Q and the self pages written by this
    // step's QKV projection (flagged by the row builder) need the wait.
    // CTAs take equal shares of the groups (ranges listed by the row builder
    // for a grid of s.n_cta); a group's partial result depends only on the
    // row, never on the split
    const int *cr = s.crange + (cross ? s.n_cta + 1 : 0);
    const int b = blockIdx.x;
    const int g0 = b < s.n_cta ? cr[b] : 0, g1 = b < s.n_cta ? cr[b + 1] : 0;
    const int n = g1 - g0;
    if (n <= 0) {
        pdl_wait();
        pdl_trigger();
        return;
    }
    const int *meta_l = (cross ? s.w_cross : s.w_self) + g0;
    const int *pid_l = (cross ? s.pid_cross : s.pid_self) + g0;
    const int *rp = cross ? s.rp_cross : s.rp_self;
    const long long kvoff = (long long)layer * 2 * PR * D;

    if (warp == AW) {
        // ------------------------------------------------------ producer warp
        // page ids fetched 32 at a time (one round trip), bulk loads by lane 0;
        // the first stages are issued before the dependency wait when allowed
        bool waited = false;
        for (int i0 = 0; i0 < n; i0 += 32) {
            const int pid_v = i0 + lane < n ? pid_l[i0 + lane] : 0;
            const int fresh_v = (!cross && i0 + lane < n) ? (meta_l[i0 + lane] >> 21) & 1 : 0;
            const int cnt = min(32, n - i0);
            for (int j = 0; j < cnt; ++j) {
                const int pid = __shfl_sync(0xffffffffu, pid_v, j);
                const int fresh = __shfl_sync(0xffffffffu, fresh_v, j);
                const int g = i0 + j, st = g % ANST;
                if (!waited && (g >= ANST || fresh)) {
                    pdl_wait();
                    pdl_trigger();
                    waited = true;
                }
                bool ok = true;
                if (lane == 0) {
                    if (g >= ANST) ok = mbar_wait(&sm.empty[st], ((g / ANST) & 1) ^ 1, CT_STATUS_TIMEOUT_FREE);
                    if (ok) {
                        const bf16 *src = pool + (long long)pid * PAGE_ELEMS + kvoff;
                        mbar_expect_tx(&sm.full[st], 2 * PR * D * sizeof(bf16));
                        bulk_load(sm.kv[st][0], src, PR * D * sizeof(bf16), &sm.full[st]);
                        bulk_load(sm.kv[st][1], src + PR * D, PR * D * sizeof(bf16), &sm.full[st]);
                    }
                }
                if (!__shfl_sync(0xffffffffu, (int)ok, 0)) return;
            }
        }
        if (!waited) { pdl_wait(); pdl_trigger(); }
        return;
    }
    // ---------------------------------------------------------- consumer warps
    // the first 32 entries' metadata (row builder output) before the wait
    int meta_v = lane < n ? meta_l[lane] : 0;
    pdl_wait();
    pdl_trigger();
    const int hh = warp;
    const float scale = 1.0f / sqrtf((float)DK);
    float *pb = sm.pbuf[warp];
    float m = -INFINITY, l = 0.0f, o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    float4 qv = make_float4(0.f, 0.f, 0.f, 0.f);
    int rpa = 0, rpb = 0;        // the current row's entry range
    for (int g = 0; g < n; ++g) {
        if ((g & 31) == 0 && g > 0) meta_v = g + lane < n ? meta_l[g + lane] : 0;
        const int meta = __shfl_sync(0xffffffffu, meta_v, g & 31);
        const int r = meta & 1023, pg = (meta >> 10) & 63, nv = ((meta >> 16) & 15) + 1, last = (meta >> 20) & 1;
        if (pg % GP == 0) {   // a group starts (CTA ranges start at group starts)
            qv = *reinterpret_cast<const float4 *>(Q + (size_t)r * D + hh * DK + 4 * lane);
            rpa = rp[r];
            rpb = rp[r + 1];
            m = -INFINITY; l = 0.0f; o0 = o1 = o2 = o3 = 0.0f;
        }
        const int st = g % ANST;
        if (!mbar_wait(&sm.full[st], (g / ANST) & 1, CT_STATUS_TIMEOUT_TMA)) return;
        const bf16 *Ks = sm.kv[st][0] + hh * DK + 4 * lane;
        const bf16 *Vs = sm.kv[st][1] + hh * DK + 4 * lane;
        // partial dot products of the page's 16 keys over this lane's 4 dims
        float sc[PR];
#pragma unroll
        for (int k = 0; k < PR; ++k) {
            const uint2 u = *reinterpret_cast<const uint2 *>(Ks + k * D);
            const bf16 *e = reinterpret_cast<const bf16 *>(&u);
            sc[k] = qv.x * __bfloat162float(e[0]) + qv.y * __bfloat162float(e[1]) +
                    qv.z * __bfloat162float(e[2]) + qv.w * __bfloat162float(e[3]);
        }
        // butterfly reduce-scatter: afterwards lanes 2j', 2j'+1 hold one key's score
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const bool up = lane & 16;
            const float send = up ? sc[k] : sc[k + 8];
            const float keep = up ? sc[k + 8] : sc[k];
            sc[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const bool up = lane & 8;
            const float send = up ? sc[k] : sc[k + 4];
            const float keep = up ? sc[k + 4] : sc[k];
            sc[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const bool up = lane & 4;
            const float send = up ? sc[k] : sc[k + 2];
            const float keep = up ? sc[k + 2] : sc[k];
            sc[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        {
            const bool up = lane & 2;
            const float send = up ? sc[0] : sc[1];
            const float keep = up ? sc[1] : sc[0];
            sc[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
        }
        sc[0] += __shfl_xor_sync(0xffffffffu, sc[0], 1);
        // lane l holds the score of key j: bits 4..1 of l, reversed
        const int j = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
        const bool valid = j < nv;
        const float sj = valid ? sc[0] * scale : -INFINITY;
        const float mn = fmaxf(m, warp_max(sj));       // key 0 of the page is always valid
        const float corr = expf(m - mn);               // m = -inf at a segment start -> 0
        const float pj = valid ? expf(sj - mn) : 0.0f;
        l = l * corr + warp_sum(pj) * 0.5f;            // every key is held by two lanes
        o0 *= corr; o1 *= corr; o2 *= corr; o3 *= corr;
        m = mn;
        if ((lane & 1) == 0) pb[j] = pj;
        __syncwarp();
        // P.V: probabilities broadcast from shared memory; masked keys have p = 0
        // (their V rows are finite: the pool starts zeroed and holds only
        // projected values)
        const float4 *p4 = reinterpret_cast<const float4 *>(pb);
#pragma unroll
        for (int k4 = 0; k4 < PR / 4; ++k4) {
            const float4 pk = p4[k4];
            const float pv[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint2 u = *reinterpret_cast<const uint2 *>(Vs + (4 * k4 + t) * D);
                const bf16 *e = reinterpret_cast<const bf16 *>(&u);
                o0 += pv[t] * __bfloat162float(e[0]);
                o1 += pv[t] * __bfloat162float(e[1]);
                o2 += pv[t] * __bfloat162float(e[2]);
                o3 += pv[t] * __bfloat162float(e[3]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[st]);
        if (!(last || pg % GP == GP - 1)) continue;
        // ---- the group ends here
        const size_t idx = (size_t)r * D + hh * DK + 4 * lane;
        const int nseg = (rpb - rpa + GP - 1) / GP;   // the row's groups
        if (nseg == 1) {
            const float inv = 1.0f / l;
            store_planes(o0 * inv, hi, lo, idx);
            store_planes(o1 * inv, hi, lo, idx + 1);
            store_planes(o2 * inv, hi, lo, idx + 2);
            store_planes(o3 * inv, hi, lo, idx + 3);
            continue;
        }
        const int seg = pg / GP;
        float *wp = ws + ((size_t)r * SEG_MAX + seg) * (2 * H + D);
        if (lane == 0) { wp[hh] = m; wp[H + hh] = l; }
        *reinterpret_cast<float4 *>(wp + 2 * H + hh * DK + 4 * lane) = make_float4(o0, o1, o2, o3);
        // per-(row, head) ticket: the warp that completes the head's last
        // segment combines it (no barrier between the consumer warps)
        __threadfence();
        __syncwarp();
        int tk = 0;
        if (lane == 0) tk = atomicAdd(&tickets[r * H + hh], 1);
        if (__shfl_sync(0xffffffffu, tk, 0) != nseg - 1) continue;
        __threadfence();
        const float *wr = ws + (size_t)r * SEG_MAX * (2 * H + D);
        // merge in group order: lane c loads group c's (m, l); the o loads are
        // issued four groups at a time, so the merge costs a few L2 round trips
        const int cl = min(lane, nseg - 1);
        const float mc = __ldcg(wr + (size_t)cl * (2 * H + D) + hh);
        const float lc = __ldcg(wr + (size_t)cl * (2 * H + D) + H + hh);
        const float Mg = warp_max(mc);                 // lanes >= nseg repeat group nseg - 1
        const float fc = expf(mc - Mg);
        float Lg = 0.0f;
        float4 og = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c0 = 0; c0 < nseg; c0 += 4) {
            float4 v[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int cc = min(c0 + t, nseg - 1);
                v[t] = __ldcg(reinterpret_cast<const float4 *>(wr + (size_t)cc * (2 * H + D) + 2 * H + hh * DK) + lane);
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float f = __shfl_sync(0xffffffffu, fc, min(c0 + t, nseg - 1));
                const float lt = __shfl_sync(0xffffffffu, lc, min(c0 + t, nseg - 1));
                if (c0 + t < nseg) {
                    Lg += lt * f;
                    og.x += v[t].x * f; og.y += v[t].y * f; og.z += v[t].z * f; og.w += v[t].w * f;
                }
            }
        }
        const float inv = 1.0f / Lg;
        store_planes(og.x * inv, hi, lo, idx);
        store_planes(og.y * inv, hi, lo, idx + 1);
        store_planes(og.z * inv, hi, lo, idx + 2);
        store_planes(og.w * inv, hi, lo, idx + 3);
        if (lane == 0) tickets[r * H + hh] = 0;              // ready for the next launch
    }
}

#include "step.cuh"

// ------------------------------------------------------------ host --------
// Pinned host ring: contiguous blocks allocated at submission and released
// in submission order, so inputs are copied once from the caller and uploaded
// asynchronously.  alloc returns the block offset or -1 when no contiguous
// space is free (the caller then keeps a pageable copy).
struct PinnedRing {
    long long cap = 0, head = 0, tail = 0, used = 0;
    long long alloc(long long n) {
        if (n <= 0 || n > cap) return -1;
        if (used == 0) head = tail = 0;
        if (used > 0 && head == tail) return -1;   // full
        long long off = -1;
        if (head >= tail) {                        // free: [head, cap) and [0, tail)
            if (head + n <= cap) off = head;
            else if (n <= tail) off = 0;
        } else if (head + n <= tail) {             // free: [head, tail)
            off = head;
        }
        if (off < 0) return -1;
        head = off + n;
        used += n;
        return off;
    }
    void release(long long off, long long n) {
        tail = off + n;
        used -= n;
        if (used == 0) head = tail = 0;
    }
};

struct Pending {
    long long id;
    std::vector<int> prompt;         // this utterance's prompt (empty: the engine's)
    long long ring_off = -1;         // host encoder rows in the pinned submission ring (row offset) ...
    std::vector<float> enc;          // ... or in pageable memory when the ring was full ...
    const float *dev_rows = nullptr; // ... or device rows (encoded in-engine from log-mel)
    int T_enc, forced;
};

struct Bucket {
    std::vector<std::string> labels;   // profile mode: label of each event node, in order
    int rows = 0;
    int kernels = 0;   // kernel nodes in the captured step graph
    cudaGraphExec_t exec = nullptr;
    cudaGraph_t graph = nullptr;
};

}  // namespace eng
}  // namespace ct

using namespace ct;
using namespace ct::eng;

// Host copies into the pinned staging rings (submissions of encoder rows,
// log-mel or audio): a copy of 256 KB or more is split over a few persistent
// worker threads, since one thread's memcpy into pinned memory (~10 GB/s)
// would otherwise be the longest part of a submission.  copy() returns once
// every part has landed.  Submissions come in bursts of small copies (one
// utterance is ~0.2-2 MB), so a worker keeps polling for the next copy for
// kSpinUs after its last part before it sleeps: a futex wake-up per copy cost
// more than the copy's own parts.
class CopyPool {
  public:
    explicit CopyPool(int n) {
        for (int i = 0; i < n; ++i) workers_.emplace_back([this] { loop(); });
    }
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> g(m_);
            stop_ = true;
            stop_flag_ = true;
        }
        cv_.notify_all();
        for (auto &t : workers_) t.join();
    }
    void copy(void *dst, const void *src, size_t bytes) {
        // parts of at least 128 KB: below that one thread's memcpy beats handing parts out
        const size_t parts = std::min(workers_.size() + 1, bytes / (128u << 10));
        if (parts <= 1) {
            memcpy(dst, src, bytes);
            return;
        }
        const size_t chunk = ((bytes + parts - 1) / parts + 63) & ~(size_t)63;
        const unsigned long long g = gen_.load() + 1;
        dst_ = static_cast<char *>(dst);
        src_ = static_cast<const char *>(src);
        bytes_ = bytes;
        chunk_ = chunk;
        parts_ = parts;
        left_ = parts - 1;
        claim_ = (g << kPartBits) | 1;   // part 0 is the caller's
        gen_ = g;
        if (sleepers_.load() > 0) {
            std::lock_guard<std::mutex> lk(m_);
            cv_.notify_all();
        }
        memcpy(dst, src, std::min(chunk, bytes));
        run_parts(g);   // help with the parts no worker has taken yet
        while (left_.load() != 0) cpu_relax();
    }

  private:
    static constexpr int kSpinUs = 200;
    static constexpr int kPartBits = 16;
    static constexpr unsigned long long kPartMask = (1ull << kPartBits) - 1;
    static void cpu_relax() {
#if defined(__x86_64__) || defined(__i386__)
        __builtin_ia32_pause();
#endif
    }
    // Take and copy parts of copy g until none is left.  A part is claimed by a
    // compare-and-swap on (generation, next part), so a thread still holding an
    // earlier copy's generation can never take a part of a later copy, and a
    // copy's fields stay fixed while any of its parts is being copied (copy()
    // returns only when all are done).
    void run_parts(unsigned long long g) {
        for (;;) {
            unsigned long long v = claim_.load();
            for (;;) {
                if ((v >> kPartBits) != g || (v & kPartMask) >= parts_.load()) return;
                if (claim_.compare_exchange_weak(v, v + 1)) break;
            }
            const size_t part = (size_t)(v & kPartMask);
            const size_t off = part * chunk_.load(), bytes = bytes_.load();
            const size_t n = off < bytes ? std::min(chunk_.load(), bytes - off) : 0;
            if (n) memcpy(dst_.load() + off, src_.load() + off, n);
            left_.fetch_sub(1);
        }
    }
    void loop() {
        unsigned long long seen = 0;
        for (;;) {
            // poll for a new copy for kSpinUs, then sleep until one is posted
            const auto t0 = std::chrono::steady_clock::now();
            unsigned long long g = gen_.load();
            for (int i = 0; g == seen && !stop_flag_.load(); ++i) {
                cpu_relax();
                if ((i & 255) == 255 &&
                    std::chrono::steady_clock::now() - t0 > std::chrono::microseconds(kSpinUs)) {
                    std::unique_lock<std::mutex> lk(m_);
                    sleepers_.fetch_add(1);
                    cv_.wait(lk, [&] { return stop_ || gen_.load() != seen; });
                    sleepers_.fetch_sub(1);
                    if (stop_) return;
                }
                g = gen_.load();
            }
            if (stop_flag_.load()) return;
            seen = g;
            run_parts(g);
        }
    }
    std::vector<std::thread> workers_;
    std::mutex m_;
    std::condition_variable cv_;
    // the current copy (written by copy() before gen_ is bumped, read by the parts' takers)
    std::atomic<char *> dst_{nullptr};
    std::atomic<const char *> src_{nullptr};
    std::atomic<size_t> bytes_{0}, chunk_{0}, parts_{0}, left_{0};
    std::atomic<unsigned long long> claim_{0}, gen_{0};
    std::atomic<int> sleepers_{0};
    std::atomic<bool> stop_flag_{false};
    bool stop_ = false;   // guarded by m_
};

// Copy workers: half the CPUs this process may run on, less the calling
// thread, shared among the engines of one node (torchrun's LOCAL_WORLD_SIZE
// processes, one per GPU), at most 7.  Polling workers on oversubscribed CPUs
// would only delay the threads that launch the GPU work.
static int copy_threads() {
    int cpus = 0;
    cpu_set_t set;
    if (sched_getaffinity(0, sizeof(set), &set) == 0) cpus = CPU_COUNT(&set);
    if (cpus <= 0) cpus = (int)std::thread::hardware_concurrency();
    const char *lw = getenv("LOCAL_WORLD_SIZE");
    const int local = lw ? std::max(1, atoi(lw)) : 1;
    const int share = cpus / local;
    return std::max(0, std::min(7, share / 2 - 1));
}

struct ct_engine {
    int device = -1;
    cudaStream_t st = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    // step graphs in flight between host synchronisations: their start / end events
    static constexpr int kStepRing = 32;    // steps queued before the host synchronises
    static constexpr int kAdmitRing = 8;    // ... while utterances wait for admission
    cudaEvent_t sev0[kStepRing] = {}, sev1[kStepRing] = {};
    std::vector<float> step_log;      // device time of each step since the last ct_engine_step_times
    ct_engine_config cfg;
    std::vector<int> prompt;
    // weights
    void *blob = nullptr;
    size_t blob_bytes = 0;
    const uint8_t *host_base = nullptr;
    const bf16 *etw, *epw, *elnw, *elnb, *dlnw, *dlnb, *hdb;
    struct Layer {
        const bf16 *sa_lnw, *sa_lnb, *sa_ow, *sa_ob, *ca_lnw, *ca_lnb, *ca_qw, *ca_qb, *ca_ow, *ca_ob;
        const bf16 *ffn_lnw, *ffn_lnb, *ffn_w1, *ffn_b1, *ffn_w2, *ffn_b2;
        bf16 *qkv_w, *qkv_b;
    } L[NL];
    bf16 *cakv_w = nullptr, *cakv_b = nullptr;
    // pool
    bf16 *pool = nullptr;
    int n_pages = 0;
    std::vector<int> free_pages;
    // device state
    DevState ds;
    int *h_done = nullptr;   // host view of done_map
    // step buffers
    float *h = nullptr, *q = nullptr, *attn_ws = nullptr, *logits = nullptr;
    float2 *ln_stats = nullptr;   // per row and 128-feature tile of h: (mean, M2), written by the residual GEMMs
    int *tickets = nullptr;          // per (row, head) segment counters of the attention kernel
    int attn_ctas = 148;             // attention grid (one CTA per SM; set from the device)
    bf16 *xa[2], *xb[2], *xm[2], *lm[2];
    int *next = nullptr;
    unsigned long long *amax_best = nullptr;   // LM head -> argmax: each sequence's argmax key
    unsigned *amax_ticket = nullptr; // per 32-sequence block of the LM head: vocabulary tiles finished
    // persistent step kernel (cfg.fused_step): one plan per token tile (32, 64, 128)
    struct StepPlan {
        StepPhase *ph = nullptr;
        StepGemm *gm = nullptr;
        CUtensorMap *maps = nullptr;
        int n_ph = 0, n_gm = 0;
        std::vector<std::string> labels;   // per phase (profile mode)
    } plans[3];
    float *step_part = nullptr;      // split-K partial tiles (shared by the phases)
    unsigned *step_cnt = nullptr;    // per GEMM phase and (token tile, feature tile): arrival counters
    unsigned long long *step_gbar = nullptr;     // grid barrier: arrivals, failed-launch marker
    unsigned long long *step_stamps = nullptr;   // profile mode: per phase and CTA stamps (ns)
    int last_plan = -1;                          // plan of the last fused step launched (profile mode)
    size_t attn_ws_floats = 0;
    // admission staging
    float *enc_dev = nullptr;
    bf16 *enc_pl[2];
    long long *enc_off = nullptr;
    int enc_rows_cap = 0;
    CopyPool copier{copy_threads()}; // host -> pinned-ring staging copies
    float *enc_stage = nullptr;      // pinned submission ring for host encoder rows (enc_rows_cap rows)
    PinnedRing ring;                 // over enc_stage, in rows
    // device mirror of enc_stage (same offsets): a submission's rows are
    // uploaded on the copy stream as soon as they are staged, and admission
    // waits for the uploads (upload_ev, recorded after the latest) before it
    // gathers the admitted rows from the mirror
    float *enc_ring_dev = nullptr;
    cudaStream_t cst = nullptr;
    cudaEvent_t upload_ev = nullptr;
    PinnedRing job_ring;             // over job_stage: queued audio / log-mel inputs, in floats
    float *job_stage = nullptr;
    float *job_ring_dev = nullptr;   // device mirror of job_stage (same offsets), filled at submission
    int *tok_stage = nullptr;        // pinned [max_slots][MAX_SEQ]: harvested tokens
    long long *off_stage = nullptr;  // pinned
    int *slot_stage = nullptr;       // pinned admission records [max_slots][REC_INTS]
    int *rec_dev = nullptr;          // their device copy
    float *mel_rows = nullptr;       // encoder rows of the last in-engine encoder batch, awaiting admission
    // host slot bookkeeping
    std::vector<int> slot_live;      // 0 free, 1 live
    std::vector<int> slot_first;     // 1 until its first (prefill) step has been launched
    std::vector<long long> slot_id;
    std::vector<std::vector<int>> slot_pages;
    std::deque<Pending> pending;
    std::deque<ct_result> results;
    std::deque<std::vector<int>> result_tokens;
    std::vector<Bucket> buckets;
    long long n_steps = 0, n_rows = 0, n_tokens = 0;
    double step_ms = 0.0;
    int n_live = 0;
    ct_engine_stats_t st_acc;
    std::vector<cudaEvent_t> marks;  // profile mode: event nodes between the step's launch groups
    std::vector<std::string> mark_label;
    std::map<std::string, std::pair<double, long long>> mark_ms;   // label -> (total ms, count)
    cudaEvent_t aev0 = nullptr, aev1 = nullptr;
    std::vector<int> slot_steps;     // steps run since admission (host mirror of the KV length)
    std::vector<int> slot_limit;     // steps after which the slot's sequence has certainly finished
    enc::State *enc = nullptr;       // packed encoder (null when the blob has no encoder weights)
    // queued utterance: log-mel [N_MELS][T_mel] or 16 kHz samples (n_samples > 0)
    // input in job_ring (ring_off >= 0, float offset) or in the vector (ring full)
    struct MelJob {
        long long id, ring_off;
        std::vector<float> mel;
        int T_mel, n_samples, forced;
        std::vector<int> prompt;
        size_t count;                // floats of input
    };
    std::vector<int> next_prompt;    // prompt of the utterances submitted next (empty: the engine's)
    std::deque<MelJob> mel_pending;
    cudaEvent_t eev0 = nullptr, eev1 = nullptr;
    std::vector<int> slot_tenc;
    std::vector<int> slot_plen;      // prompt length of each slot's sequence
    std::vector<void *> owned;       // aligned copies of misaligned weights
};

#define EK(x)                                                                                     \
    do {                                                                                          \
        cudaError_t e_ = (x);                                                                     \
        if (e_ != cudaSuccess) {                                                                  \
            fprintf(stderr, "ct_engine: %s: %s\n", #x, cudaGetErrorString(e_));                   \
            return CT_EDEVICE;                                                                    \
        }                                                                                         \
    } while (0)

static const bf16 *ew(ct_engine *e, const uint16_t *hp) {
    if (!hp) return nullptr;
    const uint8_t *p = reinterpret_cast<const uint8_t *>(hp);
    if (p < e->host_base || p >= e->host_base + e->blob_bytes) return nullptr;
    return reinterpret_cast<const bf16 *>(static_cast<uint8_t *>(e->blob) + (p - e->host_base));
}

// A weight matrix used as a TMA operand must start on a 16-byte boundary;
// tensors of a safetensors file need not, so those get an aligned copy.
static const bf16 *ew_matrix(ct_engine *e, const uint16_t *hp, size_t elems) {
    const bf16 *d = ew(e, hp);
    if (!d || ((uintptr_t)d & 15) == 0) return d;
    bf16 *c = nullptr;
    if (cudaMalloc(&c, elems * sizeof(bf16)) != cudaSuccess) return nullptr;
    e->owned.push_back(c);
    if (cudaMemcpy(c, d, elems * sizeof(bf16), cudaMemcpyDeviceToDevice) != cudaSuccess) return nullptr;
    return c;
}

static bool two_planes(const ct_engine *e) { return e->cfg.precision != 0; }

static thread_local bool t_pdl = true;   // set from the engine's config while a step is captured

// Profile mode: record an external event node after a launch group; the time
// from the previous mark is attributed to `label`.
static void mark(ct_engine *e, const char *label) {
    if (!e->cfg.profile) return;
    const size_t i = e->mark_label.size();
    if (i >= e->marks.size()) {
        cudaEvent_t ev;
        CT_CHECK(cudaEventCreate(&ev));
        e->marks.push_back(ev);
    }
    e->mark_label.push_back(label);
    CT_CHECK(cudaEventRecordWithFlags(e->marks[i], e->st, cudaEventRecordExternal));
}

// GEMM on the engine's stream with buffer-capacity tensor maps; step GEMMs use
// programmatic dependent launch.
static void egemm(ct_engine *e, const bf16 *W, int N, int K, const bf16 *xh, const bf16 *xl, int T, long x_rows,
                  GemmEpilogue ep, bool split, bool pdl = true) {
    ep.x_rows = x_rows;
    ep.pdl = pdl && t_pdl;
    gemm_bf16(e->st, W, N, K, xh, xl, T, ep, split);
}

// Launch with programmatic stream serialization (the kernel calls pdl_wait()
// before it reads anything its predecessor writes).
template <typename... KArgs, typename... Args>
static void launch_pdl(cudaStream_t st, dim3 grid, dim3 block, void (*k)(KArgs...), Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = t_pdl ? 1 : 0;
    CT_CHECK(cudaLaunchKernelEx(&cfg, k, args...));
}

static void launch_attn(cudaStream_t st, int ctas, const DevState &s, const float *q, const bf16 *pool, int layer,
                        int cross, bf16 *hi, bf16 *lo, float *ws, int *tickets) {
    static thread_local int configured_dev = -1;
    int dev = 0;
    CT_CHECK(cudaGetDevice(&dev));
    if (configured_dev != dev) {
        CT_CHECK(cudaFuncSetAttribute(attn_paged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)sizeof(AttnSmem)));
        configured_dev = dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3((AW + 1) * 32);
    cfg.dynamicSmemBytes = sizeof(AttnSmem);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = t_pdl ? 1 : 0;
    CT_CHECK(cudaLaunchKernelEx(&cfg, attn_paged_kernel, s, q, pool, layer, cross, hi, lo, ws, tickets));
}

// The GEMMs of a decode step with their epilogues, shared by the
// separate-kernel step (encode_step launches them one by one) and the
// persistent step kernel (which runs them as phases), so both compute the same.
enum StepGemmKind { G_QKV = 0, G_O, G_QC, G_OC, G_F1, G_F2, G_LM };

struct GemmSpec {
    const bf16 *W;
    int N, K;
    const bf16 *xh, *xl;   // activation planes (LayerNorm-input mode: shape of the tensor maps only)
    long x_rows;           // their capacity in rows
    GemmEpilogue ep;
};

static GemmSpec gemm_spec(ct_engine *e, int l, int kind) {
    const DevState &s = e->ds;
    const bool two = two_planes(e);
    GemmSpec g{};
    GemmEpilogue &ep = g.ep;
    // The pre-LayerNorms of the QKV (layers 1..7), cross-query and FFN1
    // projections run inside those GEMMs: each residual GEMM (EPI_FMADD) leaves
    // per-row (mean, M2) partials of its 128-feature tiles in ln_stats, and the
    // next GEMM normalises its own K slice of h into shared memory.  Layer 0's
    // self-attention LayerNorm is fused into the embedding, which writes planes.
    auto ln_input = [&](const bf16 *w, const bf16 *b) {
        ep.ln_x = e->h; ep.ln_stats = e->ln_stats; ep.ln_g = w; ep.ln_b = b;
        g.xh = e->xa[0]; g.xl = two ? e->xa[1] : nullptr;
    };
    g.x_rows = e->cfg.max_rows;
    ep.T_dev = s.n_rows;
    if (kind == G_LM) {
        // LM head with the greedy argmax, the token append and the retirement in
        // its epilogue (logits stored only when the caller keeps them)
        g.W = e->etw; g.N = V; g.K = D;
        g.xh = e->lm[0]; g.xl = two ? e->lm[1] : nullptr; g.x_rows = e->cfg.max_slots;
        ep.bias = e->hdb; ep.Y = e->cfg.keep_logits ? e->logits : nullptr; ep.ldy = V; ep.T_dev = s.n_seqs;
        ep.split = 1;   // 128 vocabulary tiles, one wave: each CTA streams its 128 x 1024 slice of the table
        ArgmaxSink &sk = ep.amax;
        sk.best = e->amax_best; sk.ticket = e->amax_ticket; sk.next = e->next;
        sk.q_slot = s.q_slot; sk.forced = s.forced; sk.plen = s.plen;
        sk.state = s.state; sk.gen = s.gen; sk.pos = s.pos; sk.tok = s.tok; sk.out_tok = s.out_tok;
        sk.done_map = s.done_map; sk.max_seq = MAX_SEQ; sk.eos = CT_TOK_EOS;
        return g;
    }
    const auto &Ly = e->L[l];
    switch (kind) {
    case G_QKV:
        g.W = Ly.qkv_w; g.N = 3 * D; g.K = D;
        g.xh = e->xa[0]; g.xl = two ? e->xa[1] : nullptr;
        ep.epi = EPI_QKV_PAGED; ep.bias = Ly.qkv_b; ep.Y = e->q; ep.ldy = D; ep.qdim = D;
        ep.kv_pool = e->pool; ep.row_off = s.r_off; ep.layer = l;
        if (l > 0) ln_input(Ly.sa_lnw, Ly.sa_lnb);
        break;
    case G_O:
    case G_OC:
        g.W = kind == G_O ? Ly.sa_ow : Ly.ca_ow; g.N = D; g.K = D;
        g.xh = e->xb[0]; g.xl = two ? e->xb[1] : nullptr;
        ep.epi = EPI_FMADD; ep.scale = 1.0f; ep.bias = kind == G_O ? Ly.sa_ob : Ly.ca_ob; ep.Y = e->h; ep.ldy = D;
        ep.stats_out = e->ln_stats;
        break;
    case G_QC:
        g.W = Ly.ca_qw; g.N = D; g.K = D;
        ep.bias = Ly.ca_qb; ep.Y = e->q; ep.ldy = D;
        ln_input(Ly.ca_lnw, Ly.ca_lnb);
        break;
    case G_F1:
        g.W = Ly.ffn_w1; g.N = FF; g.K = D;
        ep.epi = EPI_BF16; ep.act = 2; ep.bias = Ly.ffn_b1; ep.Ybf = e->xm[0]; ep.Ybf_lo = two ? e->xm[1] : nullptr;
        ep.ldy = FF;
        ln_input(Ly.ffn_lnw, Ly.ffn_lnb);
        break;
    case G_F2:
        g.W = Ly.ffn_w2; g.N = D; g.K = FF;
        g.xh = e->xm[0]; g.xl = two ? e->xm[1] : nullptr;
        ep.epi = EPI_FMADD; ep.scale = 1.0f; ep.bias = Ly.ffn_b2; ep.Y = e->h; ep.ldy = D;
        ep.stats_out = e->ln_stats;
        break;
    default: break;
    }
    return g;
}

static void launch_gemm_spec(ct_engine *e, const GemmSpec &g, int T) {
    egemm(e, g.W, g.N, g.K, g.xh, g.xl, T, g.x_rows, g.ep, true);
}

// Token tile of the persistent step kernel for a bucket of `rows` rows.
static int step_bn(int rows) { return rows <= 32 ? 32 : rows <= 64 ? 64 : 128; }

// Encode one step for capacity `rows` (seqs capacity = min(rows, max_slots)) on e->st.
static void encode_step(ct_engine *e, int rows) {
    const int seqs = std::min(rows, e->cfg.max_slots);
    DevState s = e->ds;
    cudaStream_t st = e->st;
    const bool two = two_planes(e);
    bf16 *xa_lo = two ? e->xa[1] : nullptr;
    e->mark_label.clear();
    mark(e, "start");
    build_rows_kernel<<<1, 1024, 0, st>>>(s, rows, seqs);
    mark(e, "build_rows");
    if (e->cfg.fused_step) {
        const int bn = step_bn(rows);
        const int slot = bn == 32 ? 0 : bn == 64 ? 1 : 2;
        const auto &pl = e->plans[slot];
        StepParams sp{};
        sp.s = s; sp.ph = pl.ph; sp.n_ph = pl.n_ph; sp.gm = pl.gm; sp.n_gm = pl.n_gm;
        sp.etw = e->etw; sp.epw = e->epw; sp.elnw = e->elnw; sp.elnb = e->elnb;
        sp.ln1w = e->L[0].sa_lnw; sp.ln1b = e->L[0].sa_lnb; sp.h = e->h; sp.xa_hi = e->xa[0]; sp.xa_lo = xa_lo;
        sp.q = e->q; sp.pool = e->pool; sp.xb_hi = e->xb[0]; sp.xb_lo = two ? e->xb[1] : nullptr;
        sp.attn_ws = e->attn_ws; sp.tickets = e->tickets;
        sp.dlnw = e->dlnw; sp.dlnb = e->dlnb; sp.lm_hi = e->lm[0]; sp.lm_lo = two ? e->lm[1] : nullptr;
        sp.gbar = e->step_gbar;
        sp.stamps = e->cfg.profile ? e->step_stamps : nullptr;
        e->last_plan = slot;
        void (*k)(StepParams) = nullptr;
        if (two) k = bn == 32 ? step_kernel<32, true> : bn == 64 ? step_kernel<64, true> : step_kernel<128, true>;
        else k = bn == 32 ? step_kernel<32, false> : bn == 64 ? step_kernel<64, false> : step_kernel<128, false>;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(e->ds.n_cta);
        cfg.blockDim = dim3(SP_THREADS);
        cfg.dynamicSmemBytes = SP_SMEM;
        cfg.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeCooperative;   // every CTA resident: the grid barriers need it
        at[0].val.cooperative = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        CT_CHECK(cudaLaunchKernelEx(&cfg, k, sp));
        mark(e, "step_fused");
        return;
    }
    launch_pdl(st, dim3(rows), dim3(256), embed_rows_kernel, s, e->etw, e->epw, e->elnw, e->elnb, e->L[0].sa_lnw,
               e->L[0].sa_lnb, e->h, e->xa[0], xa_lo);
    mark(e, "embed_ln");
    static const int kinds[6] = {G_QKV, G_O, G_QC, G_OC, G_F1, G_F2};   // the layer's GEMMs in order
    auto launch_k = [&](int k) { launch_gemm_spec(e, gemm_spec(e, k / 6, kinds[k % 6]), rows); };
    for (int l = 0; l < NL; ++l) {
        launch_k(6 * l + 0);
        mark(e, "gemm_qkv");
        launch_attn(st, e->attn_ctas, s, e->q, e->pool, l, 0, e->xb[0], two ? e->xb[1] : nullptr, e->attn_ws,
                    e->tickets);
        mark(e, "attn_self");
        launch_k(6 * l + 1);
        mark(e, "gemm_o");
        launch_k(6 * l + 2);
        mark(e, "gemm_q_cross");
        launch_attn(st, e->attn_ctas, s, e->q, e->pool, l, 1, e->xb[0], two ? e->xb[1] : nullptr, e->attn_ws,
                    e->tickets);
        mark(e, "attn_cross");
        launch_k(6 * l + 3);
        mark(e, "gemm_o");
        launch_k(6 * l + 4);
        mark(e, "gemm_ffn1");
        launch_k(6 * l + 5);
        mark(e, "gemm_ffn2");
    }
    launch_pdl(st, dim3(seqs), dim3(256), ln_rows_kernel, (const int *)s.n_seqs, (const int *)s.q_row, (const float *)e->h,
               e->dlnw, e->dlnb, e->lm[0], two ? e->lm[1] : nullptr);
    mark(e, "layernorm_final");
    launch_gemm_spec(e, gemm_spec(e, 0, G_LM), seqs);
    mark(e, "gemm_lm_head_argmax");
}

static int dalloc_bytes(void **p, size_t bytes) { return cudaMalloc(p, bytes) == cudaSuccess ? 0 : 1; }

// Phase table and GEMM descriptors of the persistent step kernel for token
// tile bn (written once, at engine creation: no allocation during capture).
static int build_step_plan(ct_engine *e, int slot, int bn) {
    auto &pl = e->plans[slot];
    std::vector<StepPhase> ph;
    std::vector<GemmSpec> specs;
    static const char *gname[] = {"gemm_qkv", "gemm_o", "gemm_q_cross", "gemm_o_cross", "gemm_ffn1", "gemm_ffn2",
                                  "gemm_lm_head_argmax"};
    pl.labels.clear();
    auto add_gemm = [&](int l, int kind) {
        specs.push_back(gemm_spec(e, l, kind));
        ph.push_back({SP_GEMM, (int)specs.size() - 1, -1, -1});
        pl.labels.push_back(std::string("fused:") + gname[kind]);
    };
    auto add = [&](int kind, int arg, const char *label) {
        ph.push_back({kind, arg, -1, -1});
        pl.labels.push_back(label);
    };
    add(SP_EMBED, 0, "fused:embed_ln");
    for (int l = 0; l < NL; ++l) {
        add_gemm(l, G_QKV);
        add(SP_ATTN, l * 2 + 0, "fused:attn_self");
        add_gemm(l, G_O);
        add_gemm(l, G_QC);
        add(SP_ATTN, l * 2 + 1, "fused:attn_cross");
        add_gemm(l, G_OC);
        add_gemm(l, G_F1);
        add_gemm(l, G_F2);
    }
    add(SP_FINAL_LN, 0, "fused:layernorm_final");
    add_gemm(0, G_LM);
    for (size_t i = 0; i < ph.size(); ++i) {
        for (size_t j = i + 1; j < ph.size(); ++j)
            if (ph[j].kind == SP_GEMM) { ph[i].next_gemm = ph[j].arg; break; }
        if (i + 1 < ph.size() && ph[i + 1].kind == SP_ATTN) ph[i].next_attn = ph[i + 1].arg;
    }
    if ((int)ph.size() > SP_MAX_PH || (int)specs.size() > SP_MAX_GEMM) return CT_EINVAL;
    // tensor maps: W (box 128 rows) and X planes (box bn rows) of every GEMM
    std::vector<CUtensorMap> maps(specs.size() * 3);
    std::vector<StepGemm> gm(specs.size());
    const size_t cnt_per = (size_t)(e->cfg.max_rows / 32 + 1) * (V / 128);
    const int planes = two_planes(e) ? 2 : 1;
    for (size_t i = 0; i < specs.size(); ++i) {
        const GemmSpec &g = specs[i];
        maps[3 * i] = gemm_tmap(g.W, g.N, g.K, 128);
        const bool lnx = g.ep.ln_x != nullptr;
        if (!lnx) {
            maps[3 * i + 1] = gemm_tmap(g.xh, g.x_rows, g.K, bn);
            if (g.xl) maps[3 * i + 2] = gemm_tmap(g.xl, g.x_rows, g.K, bn);
        }
        StepGemm &d = gm[i];
        d.W = g.W; d.N = g.N; d.K = g.K;
        d.S = gemm_nsplit(g.N, g.K, bn, g.ep.split);
        if (g.N % 128 || g.K % 64 || (g.K / 64) % d.S || bn % d.S ||
            (d.S > 1 && d.S != 2 && d.S != 4 && d.S != 8 && d.S != 16))
            return CT_EINVAL;
        // two feature tiles per item when one tile per item would take more
        // than one wave of CTAs and the stages still fit
        const int tiles = g.N / 128, kbps = g.K / 64 / d.S;
        const size_t xbytes = lnx ? (size_t)kbps * planes * bn * 128 : 0;
        const size_t stage1 = 16384 + (lnx ? 0 : (size_t)planes * bn * 128);
        const size_t stage2 = 2 * 16384 + (lnx ? 0 : (size_t)planes * bn * 128);
        if (SP_NSTG * stage1 + xbytes > SP_RING) return CT_EINVAL;
        d.TG = (d.S > 1 && tiles % 2 == 0 && tiles * d.S > e->ds.n_cta && SP_NSTG * stage2 + xbytes <= SP_RING) ? 2 : 1;
        d.ep = g.ep;
        d.part = e->step_part;
        d.cnt = e->step_cnt + (size_t)(slot * SP_MAX_GEMM + i) * cnt_per;
    }
    if (dalloc_bytes((void **)&pl.maps, maps.size() * sizeof(CUtensorMap)) ||
        dalloc_bytes((void **)&pl.gm, gm.size() * sizeof(StepGemm)) ||
        dalloc_bytes((void **)&pl.ph, ph.size() * sizeof(StepPhase)))
        return CT_ENOMEM;
    for (size_t i = 0; i < specs.size(); ++i) {
        gm[i].tmW = pl.maps + 3 * i;
        const bool lnx = specs[i].ep.ln_x != nullptr;
        gm[i].tmXh = lnx ? nullptr : pl.maps + 3 * i + 1;
        gm[i].tmXl = (lnx || !specs[i].xl) ? nullptr : pl.maps + 3 * i + 2;
    }
    EK(cudaMemcpy(pl.maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice));
    EK(cudaMemcpy(pl.gm, gm.data(), gm.size() * sizeof(StepGemm), cudaMemcpyHostToDevice));
    EK(cudaMemcpy(pl.ph, ph.data(), ph.size() * sizeof(StepPhase), cudaMemcpyHostToDevice));
    pl.n_ph = (int)ph.size();
    pl.n_gm = (int)gm.size();
    return CT_OK;
}

static Bucket *bucket_for(ct_engine *e, int rows_needed) {
    int cap = 32;
    while (cap < rows_needed) cap *= 2;
    cap = std::min(cap, e->cfg.max_rows);
    for (auto &b : e->buckets)
        if (b.rows == cap) return &b;
    Bucket b;
    b.rows = cap;
    CT_CHECK(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeRelaxed));
    t_pdl = !e->cfg.no_pdl;
    encode_step(e, cap);
    t_pdl = true;
    b.labels = e->mark_label;
    CT_CHECK(cudaStreamEndCapture(e->st, &b.graph));
    CT_CHECK(cudaGraphInstantiate(&b.exec, b.graph, 0));
    size_t nn = 0;
    CT_CHECK(cudaGraphGetNodes(b.graph, nullptr, &nn));
    std::vector<cudaGraphNode_t> nodes(nn);
    CT_CHECK(cudaGraphGetNodes(b.graph, nodes.data(), &nn));
    for (auto nd : nodes) {
        cudaGraphNodeType ty;
        CT_CHECK(cudaGraphNodeGetType(nd, &ty));
        if (ty == cudaGraphNodeTypeKernel) ++b.kernels;
    }
    e->buckets.push_back(b);
    return &e->buckets.back();
}

// Host mirror of the device slot record written at admission.
enum { REC_SLOT, REC_STATE, REC_TOK, REC_POS, REC_GEN, REC_FORCED, REC_TENC, REC_N };
constexpr int REC_PROMPT_MAX = 1 + PROMPT_MAX;   // prompt length, then its tokens
constexpr int REC_INTS = REC_N + SELF_PAGES + CROSS_PAGES + REC_PROMPT_MAX;   // one admission record

// Writes the slot records of k admissions (built on the host, one H2D copy):
// block r takes record r.
__global__ void admit_records_kernel(DevState s, const int *rec) {
    const int *r = rec + (size_t)blockIdx.x * REC_INTS;
    const int slot = r[REC_SLOT];
    if (slot < 0 || slot >= s.max_slots) { if (threadIdx.x == 0) set_status(CT_STATUS_BAD_ARG); return; }
    if (threadIdx.x == 0) {
        s.state[slot] = r[REC_STATE]; s.tok[slot] = r[REC_TOK]; s.pos[slot] = r[REC_POS];
        s.gen[slot] = r[REC_GEN]; s.forced[slot] = r[REC_FORCED]; s.tenc[slot] = r[REC_TENC];
    }
    for (int j = threadIdx.x; j < SELF_PAGES; j += blockDim.x) s.self_pt[(size_t)slot * SELF_PAGES + j] = r[REC_N + j];
    for (int j = threadIdx.x; j < CROSS_PAGES; j += blockDim.x)
        s.cross_pt[(size_t)slot * CROSS_PAGES + j] = r[REC_N + SELF_PAGES + j];
    const int *pr = r + REC_N + SELF_PAGES + CROSS_PAGES;   // length, then tokens
    if (threadIdx.x == 0) s.plen[slot] = pr[0];
    for (int j = threadIdx.x; j < pr[0]; j += blockDim.x) s.prompt[(size_t)slot * PROMPT_MAX + j] = pr[1 + j];
}

static long long ring_alloc(ct_engine *e, int n) { return e->ring.alloc(n); }
static void ring_free(ct_engine *e, long long off, int n) { e->ring.release(off, n); }

static int admit(ct_engine *e) {
    // pick admissions: free slot, pages, rows budget, encoder-row staging budget
    int live_rows = 0;
    for (int i = 0; i < e->cfg.max_slots; ++i) live_rows += e->slot_live[i] ? 1 : 0;
    int enc_rows = 0, n_rec = 0;
    std::vector<std::pair<long long, int>> ring_release;   // ring blocks of the admitted utterances
    if (!e->pending.empty()) EK(cudaStreamWaitEvent(e->st, e->upload_ev, 0));   // submitted rows uploaded
    while (!e->pending.empty()) {
        Pending &p = e->pending.front();
        if (enc_rows + p.T_enc > e->enc_rows_cap) break;
        const std::vector<int> &pr = p.prompt.empty() ? e->prompt : p.prompt;
        const int plen = (int)pr.size();
        if (live_rows + plen > e->cfg.max_rows) break;
        const int gen_max = p.forced > 0 ? p.forced : MAX_SEQ - plen;
        const int self_need = (std::min(MAX_SEQ, plen + gen_max) + PR - 1) / PR;
        const int cross_need = (p.T_enc + PR - 1) / PR;
        if ((int)e->free_pages.size() < self_need + cross_need) break;
        int slot = -1;
        for (int i = 0; i < e->cfg.max_slots; ++i)
            if (!e->slot_live[i]) { slot = i; break; }
        if (slot < 0) break;
        std::vector<int> pages(e->free_pages.end() - (self_need + cross_need), e->free_pages.end());
        e->free_pages.resize(e->free_pages.size() - (self_need + cross_need));
        e->slot_live[slot] = 1;
        e->slot_first[slot] = 1;
        e->slot_id[slot] = p.id;
        e->slot_pages[slot] = pages;
        e->slot_steps[slot] = 0;
        e->slot_limit[slot] = p.forced > 0 ? std::min(p.forced, MAX_SEQ - plen) : MAX_SEQ - plen;
        e->slot_tenc[slot] = p.T_enc;
        ++e->st_acc.admitted;
        // slot record + page tables (copied for all admissions at once below)
        int *rec = e->slot_stage + (size_t)n_rec * REC_INTS;
        ++n_rec;
        rec[REC_SLOT] = slot;
        rec[REC_STATE] = SEQ_PREFILL; rec[REC_TOK] = 0; rec[REC_POS] = 0; rec[REC_GEN] = 0;
        rec[REC_FORCED] = p.forced; rec[REC_TENC] = p.T_enc;
        int *spt = rec + REC_N, *cpt = spt + SELF_PAGES;
        for (int j = 0; j < SELF_PAGES; ++j) spt[j] = j < self_need ? pages[j] : -1;
        for (int j = 0; j < CROSS_PAGES; ++j) cpt[j] = j < cross_need ? pages[self_need + j] : -1;
        cpt[CROSS_PAGES] = plen;
        std::copy(pr.begin(), pr.end(), cpt + CROSS_PAGES + 1);
        e->slot_plen[slot] = plen;
        // encoder rows of this utterance -> contiguous device rows, with their cross page offsets
        float *dst = e->enc_dev + (size_t)enc_rows * D;
        const size_t bytes = sizeof(float) * (size_t)p.T_enc * D;
        if (p.dev_rows) {
            EK(cudaMemcpyAsync(dst, p.dev_rows, bytes, cudaMemcpyDeviceToDevice, e->st));
        } else if (p.ring_off >= 0) {   // uploaded at submission; the ring space is released after the sync below
            EK(cudaMemcpyAsync(dst, e->enc_ring_dev + (size_t)p.ring_off * D, bytes, cudaMemcpyDeviceToDevice, e->st));
            ring_release.push_back({p.ring_off, p.T_enc});
        } else {                        // pageable: the call returns once the source has been staged
            EK(cudaMemcpyAsync(dst, p.enc.data(), bytes, cudaMemcpyHostToDevice, e->st));
        }
        for (int t = 0; t < p.T_enc; ++t)
            e->off_stage[enc_rows + t] = (long long)pages[self_need + t / PR] * PAGE_ELEMS + (long long)(t % PR) * D;
        enc_rows += p.T_enc;
        live_rows += plen;
        ++e->n_live;
        e->pending.pop_front();
    }
    if (enc_rows == 0) return 0;
    EK(cudaMemcpyAsync(e->rec_dev, e->slot_stage, sizeof(int) * (size_t)n_rec * REC_INTS, cudaMemcpyHostToDevice,
                       e->st));
    admit_records_kernel<<<n_rec, 64, 0, e->st>>>(e->ds, e->rec_dev);
    EK(cudaGetLastError());
    // cross-attention K/V of all admitted utterances: one GEMM into their pages
    EK(cudaMemcpyAsync(e->enc_off, e->off_stage, sizeof(long long) * enc_rows, cudaMemcpyHostToDevice, e->st));
    EK(cudaEventRecord(e->aev0, e->st));
    const bool two = two_planes(e);
    split_fp32_to_bf16(e->st, e->enc_dev, enc_rows, D, D, e->enc_pl[0], two ? e->enc_pl[1] : nullptr, D);
    GemmEpilogue ep;
    ep.epi = EPI_CAKV_PAGED; ep.bias = e->cakv_b; ep.kv_pool = e->pool; ep.row_off = e->enc_off;
    egemm(e, e->cakv_w, NL * 2 * D, D, e->enc_pl[0], two ? e->enc_pl[1] : nullptr, enc_rows, e->enc_rows_cap, ep, false,
          false);
    EK(cudaEventRecord(e->aev1, e->st));
    EK(cudaStreamSynchronize(e->st));   // staging reuse
    for (auto &rb : ring_release) ring_free(e, rb.first, rb.second);
    float ams = 0.0f;
    EK(cudaEventElapsedTime(&ams, e->aev0, e->aev1));
    e->st_acc.admit_ms += ams;
    e->st_acc.kernel_launches += 3;   // records + plane split + cross K/V GEMM
    return 0;
}

static int harvest(ct_engine *e) {
    // finished sequences: copy all their tokens out, free their slots, then one sync
    std::vector<std::pair<int, int>> done;   // (slot, generated tokens)
    for (int i = 0; i < e->cfg.max_slots; ++i) {
        if (!e->slot_live[i]) continue;
        const int ng = ((volatile int *)e->h_done)[i];
        if (ng <= 0) continue;
        EK(cudaMemcpyAsync(e->tok_stage + (size_t)i * MAX_SEQ, e->ds.out_tok + (size_t)i * MAX_SEQ, sizeof(int) * ng,
                           cudaMemcpyDeviceToHost, e->st));
        EK(cudaMemsetAsync(e->ds.state + i, 0, sizeof(int), e->st));   // SEQ_FREE
        done.push_back({i, ng});
    }
    if (done.empty()) return 0;
    EK(cudaStreamSynchronize(e->st));
    for (auto &d : done) {
        const int i = d.first, ng = d.second;
        ((volatile int *)e->h_done)[i] = 0;
        ct_result r;
        r.utt_id = e->slot_id[i];
        r.n_tokens = ng;
        r.status = 0;
        e->results.push_back(r);
        e->result_tokens.emplace_back(e->tok_stage + (size_t)i * MAX_SEQ, e->tok_stage + (size_t)i * MAX_SEQ + ng);
        for (int pg : e->slot_pages[i]) e->free_pages.push_back(pg);
        e->slot_pages[i].clear();
        e->slot_live[i] = 0;
        --e->n_live;
        e->n_tokens += ng;
    }
    return 0;
}

// Profile mode: fold the encoder's event marks into the per-label totals.
static void collect_enc_marks(ct_engine *e) {
    enc::State &st = *e->enc;
    if (!st.prof) return;
    for (int i = 1; i < st.n_marks; ++i) {
        float t = 0.f;
        if (cudaEventElapsedTime(&t, st.ev[i - 1], st.ev[i]) != cudaSuccess) continue;
        auto &acc = e->mark_ms[st.labels[i]];
        acc.first += t;
        acc.second += 1;
    }
}

static bool admissible(const ct_engine *e, int T_enc, int forced_len);

// Encode up to one encoder batch of queued log-mel utterances and queue their
// encoder rows for admission.
static int encode_pending(ct_engine *e) {
    if (e->mel_pending.empty()) return 0;
    if (!e->enc) return CT_EINVAL;
    // one batch: a prefix of the queue of one input kind, within capacity
    std::vector<const float *> mels;
    std::vector<int> T_mel, n_samp;
    int frames = 0;
    const bool audio = e->mel_pending.front().n_samples > 0;
    for (auto &j : e->mel_pending) {
        if ((j.n_samples > 0) != audio) break;
        if ((int)mels.size() >= e->enc->max_utts || frames + j.T_mel > e->enc->max_frames) break;
        mels.push_back(j.ring_off >= 0 ? e->job_ring_dev + j.ring_off : j.mel.data());   // device mirror or host
        T_mel.push_back(j.T_mel);
        n_samp.push_back(j.n_samples);
        frames += j.T_mel;
    }
    const int n = (int)mels.size();
    std::vector<int> off(n + 1);
    EK(cudaEventRecord(e->eev0, e->st));
    EK(cudaStreamWaitEvent(e->st, e->upload_ev, 0));   // inputs staged in the job ring are on the device
    const bool ok = audio ? enc::encode_audio(e->st, *e->enc, n, mels.data(), n_samp.data(), T_mel.data(), off.data())
                          : enc::encode(e->st, *e->enc, n, mels.data(), T_mel.data(), off.data());
    if (!ok) return CT_EINVAL;
    EK(cudaEventRecord(e->eev1, e->st));
    // the rows wait in mel_rows until admitted (the next encoder batch runs
    // only once every pending utterance has been admitted)
    EK(cudaMemcpyAsync(e->mel_rows, e->enc->enc_h, sizeof(float) * (size_t)off[n] * D, cudaMemcpyDeviceToDevice,
                       e->st));
    EK(cudaStreamSynchronize(e->st));
    float ms = 0.f;
    EK(cudaEventElapsedTime(&ms, e->eev0, e->eev1));
    collect_enc_marks(e);
    e->st_acc.enc_ms += ms;
    e->st_acc.enc_utts += n;
    e->st_acc.enc_frames += frames;
    e->st_acc.kernel_launches += 5 + 3 + 1 + 2 + NL * (5 + 2 + 2 + 2 + 1 + 2 + 2 + 1 + 3) + 1;
    for (int b = 0; b < n; ++b) {
        const auto &j = e->mel_pending.front();
        if (j.ring_off >= 0) e->job_ring.release(j.ring_off, (long long)j.count);   // uploaded (synchronised above)
        Pending p;
        p.id = j.id;
        p.T_enc = off[b + 1] - off[b];
        p.dev_rows = e->mel_rows + (size_t)off[b] * D;
        p.forced = j.forced;
        p.prompt = j.prompt;
        e->pending.push_back(std::move(p));
        e->mel_pending.pop_front();
    }
    return 0;
}

// Profile mode of the persistent step: per phase, the span from the first
// CTA's start to the last CTA's finish, then the barrier from that finish to
// the first release; for the GEMM phases also the median over the CTAs with
// work of start -> accumulator ready -> split-K partials counted in -> done,
// and the spread of the start times.
static int collect_step_stamps(ct_engine *e) {
    const auto &pl = e->plans[e->last_plan];
    const int G = e->ds.n_cta;
    const int NS = SP_NSTAMP;
    std::vector<unsigned long long> st((size_t)(pl.n_ph + 1) * G * NS);
    EK(cudaMemcpy(st.data(), e->step_stamps, st.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
    // a CTA without a GEMM item in a phase writes no middle stamps next time
    EK(cudaMemset(e->step_stamps, 0, st.size() * sizeof(unsigned long long)));
    auto at = [&](int ph, int c, int k) { return st[((size_t)ph * G + c) * NS + k]; };
    auto lo = [&](int ph, int k) {
        unsigned long long v = ~0ull;
        for (int c = 0; c < G; ++c) v = std::min(v, at(ph, c, k));
        return v;
    };
    auto hi = [&](int ph, int k) {
        unsigned long long v = 0;
        for (int c = 0; c < G; ++c) v = std::max(v, at(ph, c, k));
        return v;
    };
    auto median = [](std::vector<double> v) {
        if (v.empty()) return 0.0;
        std::nth_element(v.begin(), v.begin() + v.size() / 2, v.end());
        return v[v.size() / 2];
    };
    auto add_ms = [&](const std::string &k, double v) {
        auto &x = e->mark_ms[k];
        x.first += v;
        x.second += 1;
    };
    for (int ph = 0; ph < pl.n_ph; ++ph) {
        const unsigned long long s0 = lo(ph, 0), d1 = hi(ph, 3);
        const double work = d1 > s0 ? (d1 - s0) * 1e-6 : 0.0;
        add_ms(pl.labels[ph], work);
        if (pl.labels[ph] == "fused:attn_self") e->st_acc.self_attn_ms += work;
        else if (pl.labels[ph] == "fused:attn_cross") e->st_acc.cross_attn_ms += work;
        else if (pl.labels[ph].rfind("fused:gemm_ffn", 0) == 0) e->st_acc.ffn_ms += work;
        std::vector<double> m1, m2, m3;
        for (int c = 0; c < G; ++c) {
            const unsigned long long t0 = at(ph, c, 0), t1 = at(ph, c, 1), t2 = at(ph, c, 2), t3 = at(ph, c, 3);
            if (t1 > t0) {
                m1.push_back((t1 - t0) * 1e-6);
                if (t2 > t1) m2.push_back((t2 - t1) * 1e-6);
                m3.push_back((t3 - (t2 > t1 ? t2 : t1)) * 1e-6);
            }
        }
        if (!m1.empty()) {
            add_ms(pl.labels[ph] + "/cta_to_accumulator", median(m1));
            add_ms(pl.labels[ph] + "/cta_partials_wait", median(m2));
            add_ms(pl.labels[ph] + "/cta_reduce_epilogue", median(m3));
            add_ms(pl.labels[ph] + "/start_spread", (hi(ph, 0) - s0) * 1e-6);
        }
        if (ph + 1 < pl.n_ph) {
            const unsigned long long s1 = lo(ph + 1, 0);
            add_ms("fused:barrier", s1 > d1 ? (s1 - d1) * 1e-6 : 0.0);
        }
    }
    return 0;
}

extern "C" int ct_engine_step(ct_engine *e, int n_steps) {
    if (!e) return CT_EINVAL;
    EK(cudaSetDevice(e->device));
    int inflight = 0;   // steps launched since the last synchronisation
    auto sync_inflight = [&]() -> int {
        EK(cudaEventSynchronize(e->sev1[inflight - 1]));
        for (int j = 0; j < inflight; ++j) {
            float ms = 0.0f;
            EK(cudaEventElapsedTime(&ms, e->sev0[j], e->sev1[j]));
            e->step_ms += ms;
            e->step_log.push_back(ms);
        }
        inflight = 0;
        return 0;
    };
    for (int it = 0; it < n_steps; ++it) {
        if (inflight == 0) {   // harvest and admit only at synchronisation points
            if (e->pending.empty() && !e->mel_pending.empty()) {
                const int rc = encode_pending(e);
                if (rc) return rc;
            }
            int rc = harvest(e);
            if (rc) return rc;
            rc = admit(e);
            if (rc) return rc;
        }
        if (e->n_live == 0) {
            if (!e->pending.empty()) return CT_EBUSY;   // nothing live and nothing admissible
            break;
        }
        // A sequence has certainly finished on the device once it has run its
        // forced length of steps (or MAX_SEQ minus its prompt).  When every
        // live sequence has, the queued steps already retired them: collect
        // them instead of launching a step over no rows.
        bool any_active = false;
        for (int i = 0; i < e->cfg.max_slots && !any_active; ++i)
            any_active = e->slot_live[i] && e->slot_steps[i] < e->slot_limit[i];
        if (!any_active && inflight > 0) {
            const int rc = sync_inflight();
            if (rc) return rc;
            continue;
        }
        int rows = 0;
        double self_b = 0.0, cross_b = 0.0;
        const double kv_row = 2.0 * D * sizeof(bf16);   // K + V bytes of one cached row, one layer
        for (int i = 0; i < e->cfg.max_slots; ++i) {
            if (!e->slot_live[i]) continue;
            if (e->slot_first[i]) {
                rows += e->slot_plen[i];
                for (int p = 0; p < e->slot_plen[i]; ++p) self_b += (p + 1) * kv_row;
                cross_b += (double)e->slot_plen[i] * e->slot_tenc[i] * kv_row;
            } else {
                rows += 1;
                self_b += (double)(e->slot_plen[i] + e->slot_steps[i]) * kv_row;
                cross_b += (double)e->slot_tenc[i] * kv_row;
            }
        }
        Bucket *b = bucket_for(e, std::max(rows, 1));
        const int k = inflight;
        EK(cudaEventRecord(e->sev0[k], e->st));
        EK(cudaGraphLaunch(b->exec, e->st));
        EK(cudaEventRecord(e->sev1[k], e->st));
        ++inflight;
        // The next step's rows come from the device state (finished sequences
        // drop out there), so further graphs can be queued before this one
        // ends; the host synchronises every kStepRing steps (every kAdmitRing
        // while utterances wait for admission, which happens only at
        // synchronisation points), at the last step, and for every step in
        // profile mode.
        const bool waiting = !e->pending.empty() || !e->mel_pending.empty();
        if (inflight == ct_engine::kStepRing || (waiting && inflight >= ct_engine::kAdmitRing) ||
            it == n_steps - 1 || e->cfg.profile) {
            const int rc = sync_inflight();
            if (rc) return rc;
        }
        e->st_acc.kernel_launches += b->kernels;
        ++e->n_steps;
        e->n_rows += rows;
        if (e->cfg.profile) {
            for (size_t i = 1; i < b->labels.size(); ++i) {
                float t = 0.f;
                EK(cudaEventElapsedTime(&t, e->marks[i - 1], e->marks[i]));
                auto &acc = e->mark_ms[b->labels[i]];
                acc.first += t;
                acc.second += 1;
                if (b->labels[i] == "attn_self") e->st_acc.self_attn_ms += t;
                else if (b->labels[i] == "attn_cross") e->st_acc.cross_attn_ms += t;
                else if (b->labels[i].rfind("gemm_ffn", 0) == 0) e->st_acc.ffn_ms += t;
            }
            if (e->cfg.fused_step && e->step_stamps && e->last_plan >= 0) {
                const int rc = collect_step_stamps(e);
                if (rc) return rc;
            }
        }
        e->st_acc.self_kv_bytes += NL * self_b;
        e->st_acc.cross_kv_bytes += NL * cross_b;
        e->st_acc.ffn_bytes += NL * (2.0 * 2.0 * FF * D + (double)rows * (D + FF) * 2.0 * (two_planes(e) ? 2 : 1));
        e->st_acc.attn_launches += 2 * NL;
        e->st_acc.ffn_launches += 2 * NL;
        for (int i = 0; i < e->cfg.max_slots; ++i) {
            if (e->slot_live[i]) ++e->slot_steps[i];
            e->slot_first[i] = 0;
        }
    }
    int rc = harvest(e);
    if (rc) return rc;
    return (int)e->pending.size() + (int)e->mel_pending.size() + e->n_live;
}

// Copy a queued utterance's input once: into the pinned job ring when it has
// room (and from there at once into the ring's device mirror, on the copy
// stream), else into the job's own (pageable) vector.
static int stage_job(ct_engine *e, ct_engine::MelJob &j, const float *src, size_t count) {
    j.count = count;
    j.ring_off = e->job_ring.alloc((long long)count);
    if (j.ring_off < 0) {
        j.mel.assign(src, src + count);
        return CT_OK;
    }
    e->copier.copy(e->job_stage + j.ring_off, src, sizeof(float) * count);
    EK(cudaSetDevice(e->device));
    EK(cudaMemcpyAsync(e->job_ring_dev + j.ring_off, e->job_stage + j.ring_off, sizeof(float) * count,
                       cudaMemcpyHostToDevice, e->cst));
    EK(cudaEventRecord(e->upload_ev, e->cst));
    return CT_OK;
}

extern "C" int ct_engine_submit_mel(ct_engine *e, long long utt_id, const float *mel, int T_mel, int forced_len) {
    if (!e || !mel || T_mel <= 0 || forced_len < 0) return CT_EINVAL;
    if (!e->enc || T_mel > e->enc->max_frames) return CT_EINVAL;
    const int t1 = (T_mel + 1) / 2, t2 = (t1 + 1) / 2, T_enc = (t2 + 1) / 2;
    if (!admissible(e, T_enc, forced_len)) return CT_EINVAL;
    ct_engine::MelJob j;
    j.id = utt_id;
    if (const int rc = stage_job(e, j, mel, (size_t)N_MELS * T_mel)) return rc;
    j.T_mel = T_mel;
    j.n_samples = 0;
    j.forced = forced_len;
    j.prompt = e->next_prompt;
    e->mel_pending.push_back(std::move(j));
    return CT_OK;
}

extern "C" int ct_engine_submit_audio(ct_engine *e, long long utt_id, const float *samples, int n_samples,
                                      int forced_len) {
    if (!e || !samples || n_samples < fe::HOP || forced_len < 0) return CT_EINVAL;
    const int T_mel = 1 + n_samples / fe::HOP;
    if (!e->enc || T_mel > e->enc->max_frames) return CT_EINVAL;
    const int t1 = (T_mel + 1) / 2, t2 = (t1 + 1) / 2, T_enc = (t2 + 1) / 2;
    if (!admissible(e, T_enc, forced_len)) return CT_EINVAL;
    ct_engine::MelJob j;
    j.id = utt_id;
    if (const int rc = stage_job(e, j, samples, (size_t)n_samples)) return rc;
    j.T_mel = T_mel;
    j.n_samples = n_samples;
    j.forced = forced_len;
    j.prompt = e->next_prompt;
    e->mel_pending.push_back(std::move(j));
    return CT_OK;
}

extern "C" int ct_engine_log_mel(ct_engine *e, int n, const float *const *samples, const int *n_samples,
                                 float *mel_out) {
    if (!e || n <= 0 || !samples || !n_samples || !mel_out) return CT_EINVAL;
    if (!e->enc) return CT_EINVAL;
    EK(cudaSetDevice(e->device));
    std::vector<int> T_mel(n);
    if (!fe::log_mel(e->st, e->enc->fe, n, samples, n_samples, e->enc->mel, T_mel.data())) return CT_EINVAL;
    size_t frames = 0;
    for (int b = 0; b < n; ++b) frames += (size_t)T_mel[b];
    EK(cudaMemcpyAsync(mel_out, e->enc->mel, sizeof(float) * N_MELS * frames, cudaMemcpyDeviceToHost, e->st));
    EK(cudaStreamSynchronize(e->st));
    return CT_OK;
}

extern "C" int ct_engine_encode(ct_engine *e, int n, const float *const *mel, const int *T_mel, float *enc_h, int *T_enc) {
    if (!e || n <= 0 || !mel || !T_mel || !enc_h || !T_enc) return CT_EINVAL;
    if (!e->enc) return CT_EINVAL;
    EK(cudaSetDevice(e->device));
    std::vector<int> off(n + 1);
    EK(cudaEventRecord(e->eev0, e->st));
    if (!enc::encode(e->st, *e->enc, n, mel, T_mel, off.data())) return CT_EINVAL;
    EK(cudaEventRecord(e->eev1, e->st));
    EK(cudaMemcpyAsync(enc_h, e->enc->enc_h, sizeof(float) * (size_t)off[n] * D, cudaMemcpyDeviceToHost, e->st));
    EK(cudaStreamSynchronize(e->st));
    float ms = 0.f;
    EK(cudaEventElapsedTime(&ms, e->eev0, e->eev1));
    collect_enc_marks(e);
    e->st_acc.enc_ms += ms;
    e->st_acc.enc_utts += n;
    for (int b = 0; b < n; ++b) { T_enc[b] = off[b + 1] - off[b]; e->st_acc.enc_frames += T_mel[b]; }
    return CT_OK;
}

extern "C" int ct_engine_run(ct_engine *e) {
    for (;;) {
        const int r = ct_engine_step(e, 64);
        if (r <= 0) return r;
    }
}

// An utterance of T_enc encoder rows that could ever be admitted.
static bool admissible(const ct_engine *e, int T_enc, int forced_len) {
    if (T_enc <= 0 || T_enc > CROSS_PAGES * PR || forced_len < 0 || T_enc > e->enc_rows_cap) return false;
    // with the prompt the utterance is submitted with
    const int plen = e->next_prompt.empty() ? e->cfg.n_prompt : (int)e->next_prompt.size();
    const int gen_max = forced_len > 0 ? forced_len : MAX_SEQ - plen;
    if (plen + 1 > MAX_SEQ) return false;
    const int need = (std::min(MAX_SEQ, plen + gen_max) + PR - 1) / PR + (T_enc + PR - 1) / PR;
    return need <= e->n_pages;
}

extern "C" int ct_engine_submit_encoded(ct_engine *e, long long utt_id, const float *enc_h, int T_enc, int forced_len) {
    if (!e || !enc_h || !admissible(e, T_enc, forced_len)) return CT_EINVAL;
    Pending p;
    p.id = utt_id;
    p.prompt = e->next_prompt;
    p.ring_off = ring_alloc(e, T_enc);
    if (p.ring_off >= 0) {
        const size_t off = (size_t)p.ring_off * D, bytes = sizeof(float) * (size_t)T_enc * D;
        e->copier.copy(e->enc_stage + off, enc_h, bytes);
        EK(cudaSetDevice(e->device));
        EK(cudaMemcpyAsync(e->enc_ring_dev + off, e->enc_stage + off, bytes, cudaMemcpyHostToDevice, e->cst));
        EK(cudaEventRecord(e->upload_ev, e->cst));
    } else {
        p.enc.assign(enc_h, enc_h + (size_t)T_enc * D);
    }
    p.T_enc = T_enc;
    p.forced = forced_len;
    e->pending.push_back(std::move(p));
    return CT_OK;
}

extern "C" int ct_engine_poll(ct_engine *e, ct_result *out, int max, int *tokens, int tok_stride) {
    if (!e || max < 0 || (max > 0 && !out) || (tokens && tok_stride <= 0)) return CT_EINVAL;
    int n = 0;
    while (n < max && !e->results.empty()) {
        out[n] = e->results.front();
        if (tokens) {
            const auto &tk = e->result_tokens.front();
            memcpy(tokens + (size_t)n * tok_stride, tk.data(), sizeof(int) * std::min<size_t>(tk.size(), tok_stride));
        }
        e->results.pop_front();
        e->result_tokens.pop_front();
        ++n;
    }
    return n;
}

extern "C" int ct_engine_stats(ct_engine *e, ct_engine_stats_t *out) {
    if (!e || !out) return CT_EINVAL;
    *out = e->st_acc;
    out->steps = e->n_steps;
    out->rows = e->n_rows;
    out->tokens = e->n_tokens;
    out->step_ms = e->step_ms;
    return CT_OK;
}

extern "C" int ct_engine_profile_report(ct_engine *e, char *buf, int cap) {
    if (!e || !buf || cap <= 0) return CT_EINVAL;
    std::string s = "{";
    bool first = true;
    for (auto &kv : e->mark_ms) {
        char tmp[160];
        snprintf(tmp, sizeof(tmp), "%s\"%s\": [%.6f, %lld]", first ? "" : ", ", kv.first.c_str(), kv.second.first,
                 kv.second.second);
        s += tmp;
        first = false;
    }
    s += "}";
    snprintf(buf, cap, "%s", s.c_str());
    return (int)s.size();
}

extern "C" int ct_engine_set_prompt(ct_engine *e, const int *prompt, int n_prompt) {
    if (!e) return CT_EINVAL;
    if (!prompt) { e->next_prompt.clear(); return CT_OK; }
    if (n_prompt <= 0 || n_prompt > PROMPT_MAX || n_prompt > e->cfg.max_rows) return CT_EINVAL;
    for (int j = 0; j < n_prompt; ++j)
        if (prompt[j] < 0 || prompt[j] >= V) return CT_EINVAL;
    e->next_prompt.assign(prompt, prompt + n_prompt);
    return CT_OK;
}

extern "C" int ct_engine_step_times(ct_engine *e, float *out, int max) {
    if (!e || max < 0 || (!out && max > 0)) return CT_EINVAL;
    const int n = std::min<int>(max, (int)e->step_log.size());
    for (int i = 0; i < n; ++i) out[i] = e->step_log[i];
    e->step_log.clear();
    return n;
}

extern "C" int ct_engine_last_logits(ct_engine *e, float *logits, long long *utt_ids, int *gen_index, int max) {
    if (!e || max < 0 || (max > 0 && (!logits || !utt_ids || !gen_index))) return CT_EINVAL;
    if (!e->cfg.keep_logits) return CT_EINVAL;   // the LM head stored none
    if (e->n_steps == 0 || max == 0) return 0;
    EK(cudaSetDevice(e->device));
    EK(cudaStreamSynchronize(e->st));
    int n = 0;
    EK(cudaMemcpy(&n, e->ds.n_seqs, sizeof(int), cudaMemcpyDeviceToHost));
    n = std::min(n, max);
    if (n <= 0) return 0;
    std::vector<int> qs(n), gen(e->cfg.max_slots);
    EK(cudaMemcpy(qs.data(), e->ds.q_slot, sizeof(int) * n, cudaMemcpyDeviceToHost));
    EK(cudaMemcpy(gen.data(), e->ds.gen, sizeof(int) * e->cfg.max_slots, cudaMemcpyDeviceToHost));
    EK(cudaMemcpy(logits, e->logits, sizeof(float) * (size_t)n * V, cudaMemcpyDeviceToHost));
    for (int i = 0; i < n; ++i) {
        const int slot = qs[i];
        if (slot < 0 || slot >= e->cfg.max_slots) return CT_EDEVICE;
        utt_ids[i] = e->slot_id[slot];
        gen_index[i] = gen[slot] - 1;   // the argmax kernel counted this step's token
    }
    return n;
}

extern "C" int ct_engine_status(ct_engine *e) {
    if (!e) return CT_EINVAL;
    EK(cudaSetDevice(e->device));
    EK(cudaStreamSynchronize(e->st));
    int v = 0, zero = 0;
    EK(cudaMemcpyFromSymbol(&v, g_ct_status, sizeof(int)));
    EK(cudaMemcpyToSymbol(g_ct_status, &zero, sizeof(int)));
    return v;
}

extern "C" void ct_engine_destroy(ct_engine *e) {
    if (!e) return;
    cudaSetDevice(e->device);
    if (e->cst) cudaStreamSynchronize(e->cst);
    cudaStreamSynchronize(e->st);
    for (auto &b : e->buckets) { cudaGraphExecDestroy(b.exec); cudaGraphDestroy(b.graph); }
    void *ptrs[] = {e->blob, e->pool, e->cakv_w, e->cakv_b, e->h, e->q, e->attn_ws, e->logits, e->xa[0], e->xa[1],
                    e->xb[0], e->xb[1], e->xm[0], e->xm[1], e->lm[0], e->lm[1], e->next, e->enc_dev, e->enc_ring_dev, e->job_ring_dev, e->enc_pl[0],
                    e->enc_pl[1], e->enc_off, e->ds.state, e->ds.tok, e->ds.pos, e->ds.gen, e->ds.forced,
                    e->ds.tenc, e->ds.self_pt, e->ds.cross_pt, e->ds.out_tok, e->ds.prompt, e->ds.plen, e->ds.r_slot,
                    e->ds.r_pos, e->ds.r_tok, e->ds.r_off, e->ds.q_row, e->ds.q_slot, e->ds.n_rows, e->ds.n_seqs,
                    e->tickets, e->ds.w_self, e->ds.w_cross, e->ds.pid_self, e->ds.pid_cross, e->ds.rp_self,
                    e->ds.rp_cross, e->ds.n_grp, e->ds.grp_self, e->ds.grp_cross, e->ds.n_wself, e->ds.n_wcross,
                    e->ds.crange, e->rec_dev,
                    e->mel_rows, e->ln_stats, e->amax_best, e->amax_ticket, e->step_part, e->step_cnt,
                    e->step_gbar, e->step_stamps, e->plans[0].ph, e->plans[0].gm, e->plans[0].maps,
                    e->plans[1].ph, e->plans[1].gm, e->plans[1].maps, e->plans[2].ph, e->plans[2].gm,
                    e->plans[2].maps};
    for (void *p : ptrs) cudaFree(p);
    for (int l = 0; l < NL; ++l) { cudaFree(e->L[l].qkv_w); cudaFree(e->L[l].qkv_b); }
    cudaFreeHost(e->h_done);
    cudaFreeHost(e->enc_stage);
    cudaFreeHost(e->tok_stage);
    if (e->job_stage) cudaFreeHost(e->job_stage);
    cudaFreeHost(e->off_stage);
    cudaFreeHost(e->slot_stage);
    cudaEventDestroy(e->ev0);
    for (int j = 0; j < ct_engine::kStepRing; ++j) {
        if (e->sev0[j]) cudaEventDestroy(e->sev0[j]);
        if (e->sev1[j]) cudaEventDestroy(e->sev1[j]);
    }
    cudaEventDestroy(e->ev1);
    cudaEventDestroy(e->aev0);
    cudaEventDestroy(e->aev1);
    for (auto ev : e->marks) cudaEventDestroy(ev);
    if (e->eev0) cudaEventDestroy(e->eev0);
    if (e->eev1) cudaEventDestroy(e->eev1);
    if (e->enc) {
        for (int l = 0; l < ENC_N; ++l) { cudaFree(e->enc->w.L[l].qkv_w); cudaFree(e->enc->w.L[l].qkv_b); }
        enc::state_free(*e->enc);
        delete e->enc;
    }
    cudaStreamDestroy(e->st);
    if (e->cst) cudaStreamDestroy(e->cst);
    if (e->upload_ev) cudaEventDestroy(e->upload_ev);
    for (void *p : e->owned) cudaFree(p);
    delete e;
}

template <typename T>
static int dalloc(T **p, size_t n) {
    if (cudaMalloc(reinterpret_cast<void **>(p), sizeof(T) * (n ? n : 1)) != cudaSuccess) return CT_ENOMEM;
    return CT_OK;
}

extern "C" int ct_engine_create(ct_engine **out, int device, const void *host_blob, size_t bytes, const Weights *w,
                                const ct_engine_config *cfg_in) {
    if (!out || !host_blob || !w) return CT_EINVAL;
    *out = nullptr;
    ct_engine_config cfg;
    memset(&cfg, 0, sizeof(cfg));
    if (cfg_in) cfg = *cfg_in;
    if (cfg.max_slots <= 0) cfg.max_slots = 256;
    if (cfg.max_rows <= 0) cfg.max_rows = 1024;
    if (cfg.n_prompt <= 0) cfg.n_prompt = 10;
    // attention page entries pack the row index in 10 bits
    if (cfg.max_slots > 1024 || cfg.n_prompt > PROMPT_MAX || cfg.max_rows < cfg.n_prompt || cfg.max_rows > 1024)
        return CT_EINVAL;
    static const int kPrompt[10] = {13764, 7, 4, 16, 62, 62, 5, 9, 11, 13};
    if (!cfg.prompt && cfg.n_prompt != 10) return CT_EINVAL;   // the default prompt has 10 tokens
    if (cfg.prompt)
        for (int j = 0; j < cfg.n_prompt; ++j)
            if (cfg.prompt[j] < 0 || cfg.prompt[j] >= V) return CT_EINVAL;
    ct_engine *e = new ct_engine();
    e->cfg = cfg;
    e->prompt.assign(cfg.prompt ? cfg.prompt : kPrompt, (cfg.prompt ? cfg.prompt : kPrompt) + cfg.n_prompt);
    e->device = device;
    if (cudaSetDevice(device) != cudaSuccess) { delete e; return CT_EDEVICE; }
    EK(cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking));
    EK(cudaStreamCreateWithFlags(&e->cst, cudaStreamNonBlocking));
    EK(cudaEventCreateWithFlags(&e->upload_ev, cudaEventDisableTiming));
    EK(cudaEventCreate(&e->ev0));
    for (int j = 0; j < ct_engine::kStepRing; ++j) {
        EK(cudaEventCreate(&e->sev0[j]));
        EK(cudaEventCreate(&e->sev1[j]));
    }
    EK(cudaEventCreate(&e->ev1));
    EK(cudaEventCreate(&e->aev0));
    EK(cudaEventCreate(&e->aev1));
    memset(&e->st_acc, 0, sizeof(e->st_acc));
    // weights: one device copy of the blob, then derived concatenations
    e->host_base = static_cast<const uint8_t *>(host_blob);
    e->blob_bytes = bytes;
    if (dalloc((uint8_t **)&e->blob, bytes)) { ct_engine_destroy(e); return CT_ENOMEM; }
    EK(cudaMemcpy(e->blob, host_blob, bytes, cudaMemcpyHostToDevice));
    e->etw = ew_matrix(e, w->etw, (size_t)V * D); e->epw = ew(e, w->epw); e->elnw = ew(e, w->elnw); e->elnb = ew(e, w->elnb);
    e->dlnw = ew(e, w->dlnw); e->dlnb = ew(e, w->dlnb); e->hdb = ew(e, w->hdb);
    if (!e->etw || !e->epw || !e->elnw || !e->elnb || !e->dlnw || !e->dlnb || !e->hdb) { ct_engine_destroy(e); return CT_EINVAL; }
    if (dalloc(&e->cakv_w, (size_t)NL * 2 * D * D) || dalloc(&e->cakv_b, (size_t)NL * 2 * D)) { ct_engine_destroy(e); return CT_ENOMEM; }
    for (int l = 0; l < NL; ++l) {
        const DLayer &d = w->dec[l];
        auto &Ly = e->L[l];
        // LayerNorm vectors are read 16 bytes at a time by the LayerNorm-input GEMMs
        Ly.sa_lnw = ew_matrix(e, d.sa_lnw, D); Ly.sa_lnb = ew_matrix(e, d.sa_lnb, D); Ly.sa_ob = ew(e, d.sa_ob);
        Ly.sa_ow = ew_matrix(e, d.sa_ow, (size_t)D * D);
        Ly.ca_lnw = ew_matrix(e, d.ca_lnw, D); Ly.ca_lnb = ew_matrix(e, d.ca_lnb, D); Ly.ca_qb = ew(e, d.ca_qb);
        Ly.ca_qw = ew_matrix(e, d.ca_qw, (size_t)D * D);
        Ly.ca_ow = ew_matrix(e, d.ca_ow, (size_t)D * D); Ly.ca_ob = ew(e, d.ca_ob);
        Ly.ffn_lnw = ew_matrix(e, d.ffn_lnw, D); Ly.ffn_lnb = ew_matrix(e, d.ffn_lnb, D);
        Ly.ffn_w1 = ew_matrix(e, d.ffn_w1, (size_t)FF * D);
        Ly.ffn_b1 = ew(e, d.ffn_b1); Ly.ffn_w2 = ew_matrix(e, d.ffn_w2, (size_t)D * FF); Ly.ffn_b2 = ew(e, d.ffn_b2);
        const bf16 *parts[3] = {ew(e, d.sa_qw), ew(e, d.sa_kw), ew(e, d.sa_vw)};
        const bf16 *bparts[3] = {ew(e, d.sa_qb), ew(e, d.sa_kb), ew(e, d.sa_vb)};
        if (dalloc(&Ly.qkv_w, (size_t)3 * D * D) || dalloc(&Ly.qkv_b, (size_t)3 * D)) { ct_engine_destroy(e); return CT_ENOMEM; }
        for (int j = 0; j < 3; ++j) {
            if (!parts[j] || !bparts[j]) { ct_engine_destroy(e); return CT_EINVAL; }
            EK(cudaMemcpy(Ly.qkv_w + (size_t)j * D * D, parts[j], sizeof(bf16) * D * D, cudaMemcpyDeviceToDevice));
            EK(cudaMemcpy(Ly.qkv_b + (size_t)j * D, bparts[j], sizeof(bf16) * D, cudaMemcpyDeviceToDevice));
        }
        const bf16 *ck = ew(e, d.ca_kw), *cv = ew(e, d.ca_vw), *ckb = ew(e, d.ca_kb), *cvb = ew(e, d.ca_vb);
        if (!ck || !cv || !ckb || !cvb || !Ly.sa_ow || !Ly.ca_qw || !Ly.ffn_w1 || !Ly.ffn_w2 || !Ly.sa_lnw ||
            !Ly.sa_lnb || !Ly.ca_lnw || !Ly.ca_lnb || !Ly.ffn_lnw || !Ly.ffn_lnb) { ct_engine_destroy(e); return CT_EINVAL; }
        EK(cudaMemcpy(e->cakv_w + (size_t)(2 * l) * D * D, ck, sizeof(bf16) * D * D, cudaMemcpyDeviceToDevice));
        EK(cudaMemcpy(e->cakv_w + (size_t)(2 * l + 1) * D * D, cv, sizeof(bf16) * D * D, cudaMemcpyDeviceToDevice));
        EK(cudaMemcpy(e->cakv_b + (size_t)(2 * l) * D, ckb, sizeof(bf16) * D, cudaMemcpyDeviceToDevice));
        EK(cudaMemcpy(e->cakv_b + (size_t)(2 * l + 1) * D, cvb, sizeof(bf16) * D, cudaMemcpyDeviceToDevice));
    }
    // page pool
    const int S = cfg.max_slots, R = cfg.max_rows;
    e->n_pages = cfg.kv_pages > 0 ? cfg.kv_pages : S * (SELF_PAGES + 24);
    if (dalloc(&e->pool, (size_t)e->n_pages * PAGE_ELEMS)) { ct_engine_destroy(e); return CT_ENOMEM; }
    EK(cudaMemset(e->pool, 0, (size_t)e->n_pages * PAGE_ELEMS * sizeof(bf16)));   // no NaN bit patterns in unset rows
    for (int i = e->n_pages - 1; i >= 0; --i) e->free_pages.push_back(i);
    // device slot table
    DevState &s = e->ds;
    s.max_slots = S; s.max_rows = R; s.n_prompt = cfg.n_prompt;
    {
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        e->attn_ctas = std::min(sms, 1023);   // the row builder (1024 threads) fills the range table
        s.n_cta = e->attn_ctas;
    }
    if (dalloc(&s.crange, 2 * ((size_t)s.n_cta + 1)) || dalloc(&s.state, S) || dalloc(&s.tok, S) || dalloc(&s.pos, S) || dalloc(&s.gen, S) || dalloc(&s.forced, S) ||
        dalloc(&s.tenc, S) || dalloc(&s.self_pt, (size_t)S * SELF_PAGES) || dalloc(&s.cross_pt, (size_t)S * CROSS_PAGES) ||
        dalloc(&s.out_tok, (size_t)S * MAX_SEQ) || dalloc(&s.prompt, (size_t)S * PROMPT_MAX) ||
        dalloc(&s.plen, S) || dalloc(&s.r_slot, R) ||
        dalloc(&s.r_pos, R) || dalloc(&s.r_tok, R) || dalloc(&s.r_off, R) || dalloc(&s.q_row, S) ||
        dalloc(&s.q_slot, S) || dalloc(&s.n_rows, 1) || dalloc(&s.n_seqs, 1) ||
        dalloc(&s.w_self, (size_t)R * SELF_PAGES) || dalloc(&s.w_cross, (size_t)R * CROSS_PAGES) ||
        dalloc(&s.pid_self, (size_t)R * SELF_PAGES) || dalloc(&s.pid_cross, (size_t)R * CROSS_PAGES) ||
        dalloc(&s.rp_self, (size_t)R + 1) || dalloc(&s.rp_cross, (size_t)R + 1) || dalloc(&s.n_grp, 2) ||
        dalloc(&s.grp_self, (size_t)R * SEG_MAX + 1) || dalloc(&s.grp_cross, (size_t)R * SEG_MAX + 1) ||
        dalloc(&s.n_wself, 1) ||
        dalloc(&s.n_wcross, 1)) { ct_engine_destroy(e); return CT_ENOMEM; }
    EK(cudaMemset(s.crange, 0, sizeof(int) * 2 * ((size_t)s.n_cta + 1)));
    EK(cudaMemset(s.state, 0, sizeof(int) * S));
    EK(cudaMemset(s.n_rows, 0, sizeof(int)));
    EK(cudaMemset(s.n_seqs, 0, sizeof(int)));
    for (int i = 0; i < S; ++i) {
        EK(cudaMemcpy(s.prompt + (size_t)i * PROMPT_MAX, e->prompt.data(), sizeof(int) * cfg.n_prompt,
                      cudaMemcpyHostToDevice));
        EK(cudaMemcpy(s.plen + i, &cfg.n_prompt, sizeof(int), cudaMemcpyHostToDevice));
    }
    EK(cudaHostAlloc(&e->h_done, sizeof(int) * S, cudaHostAllocMapped));
    memset(e->h_done, 0, sizeof(int) * S);
    EK(cudaHostGetDevicePointer(&s.done_map, e->h_done, 0));
    // step buffers
    if (dalloc(&e->h, (size_t)R * D) || dalloc(&e->q, (size_t)R * D) || dalloc(&e->xa[0], (size_t)R * D) ||
        dalloc(&e->xa[1], (size_t)R * D) || dalloc(&e->xb[0], (size_t)R * D) || dalloc(&e->xb[1], (size_t)R * D) ||
        dalloc(&e->xm[0], (size_t)R * FF) || dalloc(&e->xm[1], (size_t)R * FF) || dalloc(&e->lm[0], (size_t)S * D) ||
        dalloc(&e->lm[1], (size_t)S * D) || dalloc(&e->logits, (size_t)S * V) || dalloc(&e->next, S) ||
        dalloc(&e->ln_stats, (size_t)R * (D / 128)) || dalloc(&e->amax_best, S) ||
        dalloc(&e->amax_ticket, S)) { ct_engine_destroy(e); return CT_ENOMEM; }
    EK(cudaMemset(e->ln_stats, 0, sizeof(float2) * (size_t)R * (D / 128)));
    EK(cudaMemset(e->amax_ticket, 0, sizeof(unsigned) * S));
    EK(cudaMemset(e->amax_best, 0, sizeof(unsigned long long) * S));
    e->attn_ws_floats = (size_t)R * SEG_MAX * (2 * H + D);
    if (dalloc(&e->attn_ws, e->attn_ws_floats) || dalloc(&e->tickets, (size_t)R * H)) {
        ct_engine_destroy(e);
        return CT_ENOMEM;
    }
    EK(cudaMemset(e->tickets, 0, sizeof(int) * (size_t)R * H));
    if (cfg.fused_step) {
        // persistent step kernel: split-K partial tiles (the largest phase:
        // rows in whole 128-row tiles x N x S floats), tile counters, grid
        // barrier, profile stamps, phase plans
        const size_t Rp = ((size_t)R + 127) / 128 * 128;
        size_t part = 0;
        for (int kind = G_QKV; kind <= G_F2; ++kind) {
            const GemmSpec g = gemm_spec(e, 0, kind);
            part = std::max(part, Rp * g.N * gemm_nsplit(g.N, g.K, 32, g.ep.split));
        }
        const size_t cnt = (size_t)3 * SP_MAX_GEMM * (R / 32 + 1) * (V / 128);
        if (dalloc(&e->step_part, part) || dalloc(&e->step_cnt, cnt) || dalloc(&e->step_gbar, 2) ||
            (cfg.profile && dalloc(&e->step_stamps, (size_t)(SP_MAX_PH + 1) * e->ds.n_cta * SP_NSTAMP))) {
            ct_engine_destroy(e);
            return CT_ENOMEM;
        }
        EK(cudaMemset(e->step_cnt, 0, sizeof(unsigned) * cnt));
        EK(cudaMemset(e->step_gbar, 0, sizeof(unsigned long long) * 2));
        if (e->step_stamps)
            EK(cudaMemset(e->step_stamps, 0, sizeof(unsigned long long) * (SP_MAX_PH + 1) * e->ds.n_cta * SP_NSTAMP));
        for (auto k : {step_kernel<32, true>, step_kernel<64, true>, step_kernel<128, true>, step_kernel<32, false>,
                       step_kernel<64, false>, step_kernel<128, false>})
            EK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SP_SMEM));
        int per_sm = 0;
        EK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_kernel<128, true>, SP_THREADS, SP_SMEM));
        if (per_sm < 1) { ct_engine_destroy(e); return CT_EDEVICE; }
        const int bns[3] = {32, 64, 128};
        for (int i = 0; i < 3; ++i) {
            const int rc = build_step_plan(e, i, bns[i]);
            if (rc != CT_OK) { ct_engine_destroy(e); return rc; }
        }
    }
    // admission staging: up to 64 utterances of 30 s worth of encoder rows
    e->enc_rows_cap = 64 * 400;
    if (dalloc(&e->enc_dev, (size_t)e->enc_rows_cap * D) || dalloc(&e->enc_ring_dev, (size_t)e->enc_rows_cap * D) ||
        dalloc(&e->enc_pl[0], (size_t)e->enc_rows_cap * D) ||
        dalloc(&e->enc_pl[1], (size_t)e->enc_rows_cap * D) || dalloc(&e->enc_off, e->enc_rows_cap)) { ct_engine_destroy(e); return CT_ENOMEM; }
    EK(cudaHostAlloc(&e->enc_stage, sizeof(float) * (size_t)e->enc_rows_cap * D, cudaHostAllocDefault));
    EK(cudaHostAlloc(&e->tok_stage, sizeof(int) * (size_t)cfg.max_slots * MAX_SEQ, cudaHostAllocDefault));
    e->ring.cap = e->enc_rows_cap;
    EK(cudaHostAlloc(&e->off_stage, sizeof(long long) * e->enc_rows_cap, cudaHostAllocDefault));
    EK(cudaHostAlloc(&e->slot_stage, sizeof(int) * (size_t)cfg.max_slots * REC_INTS, cudaHostAllocDefault));
    if (dalloc(&e->rec_dev, (size_t)cfg.max_slots * REC_INTS)) { ct_engine_destroy(e); return CT_ENOMEM; }
    e->slot_live.assign(S, 0);
    e->slot_first.assign(S, 0);
    e->slot_id.assign(S, -1);
    e->slot_pages.assign(S, {});
    e->slot_steps.assign(S, 0);
    e->slot_limit.assign(S, 0);
    e->slot_tenc.assign(S, 0);
    e->slot_plen.assign(S, cfg.n_prompt);
    EK(cudaEventCreate(&e->eev0));
    EK(cudaEventCreate(&e->eev1));
    // packed encoder, when the blob carries the encoder weights
    if (cfg.enc_max_utts >= 0 && ew(e, w->enc[0].ff1_w1) && ew(e, w->s0w) && ew(e, w->prw)) {
        const int ED = ENC_D, EFF = ENC_FF;
        enc::State *st = new enc::State();
        e->enc = st;
        enc::Weights_ &ww = st->w;
        ww.s0w = ew(e, w->s0w); ww.s0b = ew(e, w->s0b); ww.s2w = ew(e, w->s2w); ww.s2b = ew(e, w->s2b);
        ww.s3w = ew_matrix(e, w->s3w, (size_t)SUB_CH * SUB_CH); ww.s3b = ew(e, w->s3b);
        ww.s5w = ew(e, w->s5w); ww.s5b = ew(e, w->s5b);
        ww.s6w = ew_matrix(e, w->s6w, (size_t)SUB_CH * SUB_CH); ww.s6b = ew(e, w->s6b);
        ww.sow = ew_matrix(e, w->sow, (size_t)ED * SUB_CH * 16); ww.sob = ew(e, w->sob);
        ww.prw = ew_matrix(e, w->prw, (size_t)D * ED); ww.prb = ew(e, w->prb);
        bool ok = ww.s0w && ww.s0b && ww.s2w && ww.s3w && ww.s5w && ww.s6w && ww.sow && ww.prw;
        for (int l = 0; l < ENC_N && ok; ++l) {
            const ELayer &s = w->enc[l];
            enc::Layer &L = ww.L[l];
            L.ff1_lnw = ew(e, s.ff1_lnw); L.ff1_lnb = ew(e, s.ff1_lnb);
            L.ff1_w1 = ew_matrix(e, s.ff1_w1, (size_t)EFF * ED); L.ff1_b1 = ew(e, s.ff1_b1);
            L.ff1_w2 = ew_matrix(e, s.ff1_w2, (size_t)ED * EFF); L.ff1_b2 = ew(e, s.ff1_b2);
            L.sa_lnw = ew(e, s.sa_lnw); L.sa_lnb = ew(e, s.sa_lnb);
            L.sa_pw = ew_matrix(e, s.sa_pw, (size_t)ED * ED);
            L.sa_ow = ew_matrix(e, s.sa_ow, (size_t)ED * ED); L.sa_ob = ew(e, s.sa_ob);
            // 16-byte vector loads in the rel-pos bias dots: aligned copies when the blob's are not
            L.sa_pbu = ew_matrix(e, s.sa_pbu, (size_t)ED); L.sa_pbv = ew_matrix(e, s.sa_pbv, (size_t)ED);
            L.cv_lnw = ew(e, s.cv_lnw); L.cv_lnb = ew(e, s.cv_lnb);
            L.cv_pw1w = ew_matrix(e, s.cv_pw1w, (size_t)2 * ED * ED); L.cv_pw1b = ew(e, s.cv_pw1b);
            L.cv_dww = ew(e, s.cv_dww); L.cv_dwb = ew(e, s.cv_dwb);
            L.cv_bnw = ew(e, s.cv_bnw); L.cv_bnb = ew(e, s.cv_bnb); L.cv_bnm = ew(e, s.cv_bnmean);
            L.cv_bnv = ew(e, s.cv_bnvar);
            L.cv_pw2w = ew_matrix(e, s.cv_pw2w, (size_t)ED * ED); L.cv_pw2b = ew(e, s.cv_pw2b);
            L.ff2_lnw = ew(e, s.ff2_lnw); L.ff2_lnb = ew(e, s.ff2_lnb);
            L.ff2_w1 = ew_matrix(e, s.ff2_w1, (size_t)EFF * ED); L.ff2_b1 = ew(e, s.ff2_b1);
            L.ff2_w2 = ew_matrix(e, s.ff2_w2, (size_t)ED * EFF); L.ff2_b2 = ew(e, s.ff2_b2);
            L.out_lnw = ew(e, s.out_lnw); L.out_lnb = ew(e, s.out_lnb);
            const bf16 *q = ew(e, s.sa_qw), *k = ew(e, s.sa_kw), *v = ew(e, s.sa_vw);
            const bf16 *qb = ew(e, s.sa_qb), *kb = ew(e, s.sa_kb), *vb = ew(e, s.sa_vb);
            ok = q && k && v && qb && kb && vb && L.ff1_w1 && L.ff1_w2 && L.sa_pw && L.sa_ow && L.cv_pw1w &&
                 L.cv_pw2w && L.ff2_w1 && L.ff2_w2 && L.out_lnw && L.cv_dww;
            if (!ok) break;
            if (dalloc(&L.qkv_w, (size_t)3 * ED * ED) || dalloc(&L.qkv_b, (size_t)3 * ED)) { ok = false; break; }
            const bf16 *parts[3] = {q, k, v}, *bparts[3] = {qb, kb, vb};
            for (int j = 0; j < 3; ++j) {
                EK(cudaMemcpy(L.qkv_w + (size_t)j * ED * ED, parts[j], sizeof(bf16) * ED * ED, cudaMemcpyDeviceToDevice));
                EK(cudaMemcpy(L.qkv_b + (size_t)j * ED, bparts[j], sizeof(bf16) * ED, cudaMemcpyDeviceToDevice));
            }
        }
        const int mu = cfg.enc_max_utts > 0 ? cfg.enc_max_utts : 64;
        const int mf = cfg.enc_max_frames > 0 ? cfg.enc_max_frames : 64 * 3001;
        if (!ok || !enc::state_alloc(*st, mu, mf, cfg.precision != 0) || dalloc(&e->mel_rows, (size_t)st->R3_max * D)) {
            ct_engine_destroy(e);
            return CT_ENOMEM;
        }
        st->prof = cfg.profile != 0;
        // one encoder batch of audio input (the larger of samples and log-mel)
        e->job_ring.cap = (long long)mf * fe::HOP;
        EK(cudaHostAlloc(&e->job_stage, sizeof(float) * (size_t)e->job_ring.cap, cudaHostAllocDefault));
        if (dalloc(&e->job_ring_dev, (size_t)e->job_ring.cap)) { ct_engine_destroy(e); return CT_ENOMEM; }
    }
    EK(cudaDeviceSynchronize());
    *out = e;
    return CT_OK;
}
