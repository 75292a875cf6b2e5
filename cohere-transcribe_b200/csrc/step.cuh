// step.cuh -- the decode step as one persistent kernel.  Included by
// engine.cu inside namespace ct::eng, after the step's separate kernels: it
// uses their DevState, page-pool geometry, attention layout and the GEMM
// helpers of gemm.cu.
//
// The separate-kernel step is ~70 dependent launches, and each pays a launch
// gap, a prologue (TMEM allocation, barrier set-up), pipeline fill and, in the
// split-K GEMMs, two cluster barriers around a distributed-shared-memory merge.
// Here one launch of n_cta CTAs (one per SM, all co-resident: a cooperative
// launch) runs the step as phases separated by grid barriers:
//   embedding (+ layer 0's LN_1) -> DEC_N x [QKV (K/V into pages),
//   self-attention, O + residual, cross-Q, cross-attention, cross-O +
//   residual, FFN1, FFN2 + residual] -> final LayerNorm -> LM head with the
//   greedy argmax, token append and retirement.
// Each phase does the arithmetic of its separate kernel in the same order
// (the same K splits, reductions and LayerNorm statistics), so both forms give
// bitwise-identical results.  A split-K GEMM's partial tiles go to global
// memory (they stay in L2) instead of a cluster's shared memory: the S CTAs of
// an output tile count in on a per-tile counter, then CTA z sums token slice z
// of the tile over the S partials in split order.  At the start of every phase
// each CTA prefetches its share of the next GEMM phase's weights into L2, and
// the first pages of the next attention phase.  Every wait -- grid barrier,
// tile counter, mbarrier -- is bounded and ends with a status code.
//
// Warps: 0 = TMA / bulk-copy producer, 1 = MMA issuer (TMEM owner),
// 2..9 = workers (LayerNorm fills, epilogues, split-K sums, attention heads).

constexpr int SP_WARPS = 10;
constexpr int SP_THREADS = SP_WARPS * 32;
constexpr int SP_NW = 256;                       // worker threads
constexpr int SP_NSTG = 4;                       // GEMM ring stages
constexpr int SP_RING = 196 * 1024;              // shared data region (GEMM ring + X tiles | attention ring)
constexpr int SP_CTRL = 26 * 1024;               // control region: barriers, argmax scratch, phase tables
constexpr int SP_MAX_GEMM = 6 * DEC_N + 1;       // GEMM phases of a step
constexpr int SP_MAX_PH = 2 + 8 * DEC_N + 1;     // phases of a step
constexpr int SP_SMEM = 1024 + SP_RING + SP_CTRL;
// profile stamps per phase and CTA: work start, accumulator ready (last GEMM
// item), split-K partials counted in (last item), work done
constexpr int SP_NSTAMP = 4;
static_assert(sizeof(AttnSmem) <= SP_RING, "attention ring exceeds the shared data region");

enum StepPhaseKind : int { SP_EMBED = 0, SP_GEMM = 1, SP_ATTN = 2, SP_FINAL_LN = 3 };

// One GEMM phase.  Tensor maps live in global memory (64-byte aligned).
struct StepGemm {
    const CUtensorMap *tmW;            // weights [N, K], box 64 x 128
    const CUtensorMap *tmXh, *tmXl;    // activation planes [rows, K], box 64 x BN; null in LayerNorm-input mode
    const bf16 *W;                     // the weights (L2 prefetch)
    int N, K, S;                       // K split in S equal k-block ranges (S divides BN); S = 1: no split
    int TG;                            // 128-feature tiles per item (1 or 2: two accumulators, one X tile set)
    GemmEpilogue ep;                   // as the separate kernel's; ep.T_dev = the row count
    float *part;                       // S > 1: [token tiles][N / 128][S][BN][128] fp32 partial tiles
    unsigned *cnt;                     // S > 1: [token tiles][N / 128] arrival counters (monotonic)
};

struct StepPhase {
    int kind;        // StepPhaseKind
    int arg;         // SP_GEMM: index into the GEMM table; SP_ATTN: layer * 2 + cross
    int next_gemm;   // the first GEMM phase after this one (L2 prefetch of its weights), -1 for none
    int next_attn;   // the next phase's attention (layer * 2 + cross) when it is one (L2 prefetch of pages), -1
};

struct StepParams {
    DevState s;
    const StepPhase *ph;
    int n_ph;
    const StepGemm *gm;
    int n_gm;
    // embedding: h = LN_e(etw[tok] + epw[pos]), xa = planes of LN_1(h) (layer 0)
    const bf16 *etw, *epw, *elnw, *elnb, *ln1w, *ln1b;
    float *h;
    bf16 *xa_hi, *xa_lo;
    // attention
    const float *q;
    const bf16 *pool;
    bf16 *xb_hi, *xb_lo;
    float *attn_ws;
    int *tickets;
    // final LayerNorm of each sequence's last row -> LM head planes
    const bf16 *dlnw, *dlnb;
    bf16 *lm_hi, *lm_lo;
    unsigned long long *gbar;     // [2]: grid-barrier arrivals (monotonic), failed-launch marker
    unsigned long long *stamps;   // profile mode: [phase][CTA][SP_NSTAMP] ns stamps; else null
};

// Control region layout.
struct StepCtrl {
    uint64_t full[SP_NSTG], empty[SP_NSTG];   // GEMM ring
    uint64_t accb, acc_free, xfull;           // accumulator ready / read; LayerNorm tiles filled
    uint64_t afull[ANST], aempty[ANST];       // attention ring
    uint32_t tmem_slot;
    unsigned long long gen0;                  // barrier epoch this launch started from (arrivals / grid)
    int flag;
    float red[SP_NW / 32];
    float2 amax[128 / 32 * 128];              // argmax hand-off: [BN / 32][4 lane quarters][32]
    StepPhase ph[SP_MAX_PH];                  // the phase table and the GEMM descriptors, copied once
    StepGemm gm[SP_MAX_GEMM];
};
static_assert(sizeof(StepCtrl) <= SP_CTRL, "control region too small");

// Per-CTA running counters: every mbarrier keeps its phase across items and
// phases, so its parity follows from how often it has been used.
struct StepSeq {
    uint32_t kb_p = 0, kb_m = 0;   // GEMM ring stages filled (producer) / consumed (MMA)
    uint32_t acc_m = 0;            // accumulators committed (MMA warp)
    uint32_t acc_w = 0;            // accumulators drained (workers)
    uint32_t x_m = 0;              // LayerNorm tile sets consumed (MMA warp)
    uint32_t att = 0;              // attention ring stages (every thread)
    uint32_t att_p = 0;            // attention ring stages issued (producer)
};

// Failure handling.  A wait that runs out records its code and marks this
// launch as failed (gbar[1] = the epoch it started from + 1); every other wait
// of the launch then gives up at its next check instead of spending its own
// budget, so a failed step ends within one budget.  The marker of an earlier
// launch never matches a later one (every launch advances the epoch by its
// phase count: each CTA arrives once at every barrier, failed or not).
__device__ __forceinline__ bool sp_failed(const unsigned long long *gbar, unsigned long long gen0) {
    return *reinterpret_cast<const volatile unsigned long long *>(gbar + 1) == gen0 + 1ull;
}
__device__ __forceinline__ void sp_fail(unsigned long long *gbar, unsigned long long gen0, int code) {
    set_status(code);
    atomicExch(gbar + 1, gen0 + 1ull);
}
__device__ __noinline__ bool sp_mbar_wait(uint64_t *bar, uint32_t parity, int code, unsigned long long *gbar,
                                          unsigned long long gen0) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 255u) {
            if (sp_failed(gbar, gen0)) return false;
            if (globaltimer() - t0 > CT_WAIT_NS) { sp_fail(gbar, gen0, code); return false; }
        }
    }
}
// Acquire-spin until a 32-bit counter reaches target (wrap-around order) or a
// 64-bit one reaches target64.
__device__ __noinline__ bool sp_word_wait(const unsigned *p, unsigned target, unsigned long long *gbar,
                                          unsigned long long gen0) {
    if ((int)(ld_acquire_u32(p) - target) >= 0) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
        if ((int)(ld_acquire_u32(p) - target) >= 0) return true;
        if ((it & 63u) == 63u) {
            if (sp_failed(gbar, gen0)) return false;
            if (globaltimer() - t0 > CT_WAIT_NS) { sp_fail(gbar, gen0, CT_STATUS_TIMEOUT_GRID); return false; }
        }
    }
}
__device__ __noinline__ bool sp_word_wait64(const unsigned long long *p, unsigned long long target,
                                            unsigned long long *gbar, unsigned long long gen0) {
    if (ld_acquire_u64(p) >= target) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
        if (ld_acquire_u64(p) >= target) return true;
        if ((it & 63u) == 63u) {
            if (sp_failed(gbar, gen0)) return false;
            if (globaltimer() - t0 > CT_WAIT_NS) { sp_fail(gbar, gen0, CT_STATUS_TIMEOUT_GRID); return false; }
        }
    }
}
// Time-bounded wait that ignores the failure marker (draining copies in flight).
__device__ __forceinline__ void sp_drain_wait(uint64_t *bar, uint32_t parity) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer() - t0 > 20000000ull) return;   // 20 ms
}

__device__ __forceinline__ void sp_wbar() { asm volatile("bar.sync 2, %0;" ::"n"(SP_NW) : "memory"); }

// Grid barrier over all CTAs: one release add per CTA on a monotonic 64-bit
// arrival counter (gbar[0]), then an acquire spin until it reaches the next
// multiple of the grid size.  The release (after the CTA barrier) publishes
// the CTA's writes; the acquire makes the other CTAs' writes visible to this
// SM's later loads.  Bounded (status 5).
__device__ __forceinline__ void sp_grid_sync(unsigned long long *gbar, unsigned long long gen0,
                                             unsigned long long *stamp_done, unsigned long long *stamp_next) {
    __syncthreads();
    if (threadIdx.x == 0) {
        if (stamp_done) *stamp_done = globaltimer();
        const unsigned long long G = gridDim.x;
        const unsigned long long old = atom_add_release_u64(gbar, 1ull);
        sp_word_wait64(gbar, (old / G + 1ull) * G, gbar, gen0);
        if (stamp_next) *stamp_next = globaltimer();
    }
    __syncthreads();
}

// 256-thread sum in the order of block_sum256e (warp sums, then the 8 warp
// totals in warp order) over the worker threads.
__device__ __forceinline__ float sp_sum256(float v, float *red, int et) {
    v = warp_sum(v);
    sp_wbar();
    if ((et & 31) == 0) red[et >> 5] = v;
    sp_wbar();
    float t = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k];
    return t;
}

// ---------------------------------------------------------------- phases --

// Embedding of every packed row (embed_rows_kernel's arithmetic), one row per
// CTA at a time over the worker threads.
__device__ void sp_embed(const StepParams &p, float *row, float *red, int et) {
    const DevState &s = p.s;
    const int n = *s.n_rows;
    for (int r = blockIdx.x; r < n; r += gridDim.x) {
        const int id = s.r_tok[r], ps = s.r_pos[r];
        if (id < 0 || id >= V || ps < 0 || ps >= MAX_SEQ) {
            if (et == 0) set_status(CT_STATUS_BAD_ARG);
            continue;
        }
        float sum = 0.0f;
        for (int k = et; k < D; k += SP_NW) {
            const float v = bf2f(p.etw[(size_t)id * D + k]) + bf2f(p.epw[(size_t)ps * D + k]);
            row[k] = v;
            sum += v;
        }
        const float mean = sp_sum256(sum, red, et) / D;
        float var = 0.0f;
        for (int k = et; k < D; k += SP_NW) { const float c = row[k] - mean; var += c * c; }
        const float inv = 1.0f / sqrtf(sp_sum256(var, red, et) / D + 1e-5f);
        float s2 = 0.0f;
        for (int k = et; k < D; k += SP_NW) {
            const float o = (row[k] - mean) * inv * bf2f(p.elnw[k]) + bf2f(p.elnb[k]);
            p.h[(size_t)r * D + k] = o;
            row[k] = o;
            s2 += o;
        }
        const float mean2 = sp_sum256(s2, red, et) / D;
        float var2 = 0.0f;
        for (int k = et; k < D; k += SP_NW) { const float c = row[k] - mean2; var2 += c * c; }
        const float inv2 = 1.0f / sqrtf(sp_sum256(var2, red, et) / D + 1e-5f);
        for (int k = et; k < D; k += SP_NW)
            store_planes((row[k] - mean2) * inv2 * bf2f(p.ln1w[k]) + bf2f(p.ln1b[k]), p.xa_hi, p.xa_lo,
                         (size_t)r * D + k);
        sp_wbar();   // row[] is reused by the next row
    }
}

// Final LayerNorm of each sequence's last row (ln_rows_kernel's arithmetic).
__device__ void sp_final_ln(const StepParams &p, float *red, int et) {
    const DevState &s = p.s;
    const int n = *s.n_seqs;
    for (int r = blockIdx.x; r < n; r += gridDim.x) {
        const float *x = p.h + (size_t)s.q_row[r] * D;
        float v[D / SP_NW];
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < D / SP_NW; ++j) { v[j] = x[et + SP_NW * j]; sum += v[j]; }
        const float mean = sp_sum256(sum, red, et) / D;
        float var = 0.0f;
#pragma unroll
        for (int j = 0; j < D / SP_NW; ++j) { const float c = v[j] - mean; var += c * c; }
        const float inv = 1.0f / sqrtf(sp_sum256(var, red, et) / D + 1e-5f);
#pragma unroll
        for (int j = 0; j < D / SP_NW; ++j) {
            const int k = et + SP_NW * j;
            store_planes((v[j] - mean) * inv * bf2f(p.dlnw[k]) + bf2f(p.dlnb[k]), p.lm_hi, p.lm_lo, (size_t)r * D + k);
        }
    }
}

// Paged attention of one layer (attn_paged_kernel's arithmetic): warp 0
// streams K/V pages into the ring, worker warp 2 + h is head h's consumer.
__device__ void sp_attention(const StepParams &p, AttnSmem &sm, StepCtrl &c, StepSeq &sq, int layer, int cross,
                             int warp, int lane) {
    const DevState &s = p.s;
    const int *cr = s.crange + (cross ? s.n_cta + 1 : 0);
    const int b = blockIdx.x;
    const int g0 = b < s.n_cta ? cr[b] : 0, g1 = b < s.n_cta ? cr[b + 1] : 0;
    const int n = g1 - g0;
    const uint32_t base = sq.att;
    if (n > 0) sq.att += (uint32_t)n;   // every thread: the ring position after this phase
    if (n <= 0) return;
    const int *meta_l = (cross ? s.w_cross : s.w_self) + g0;
    const int *pid_l = (cross ? s.pid_cross : s.pid_self) + g0;
    const int *rp = cross ? s.rp_cross : s.rp_self;
    const long long kvoff = (long long)layer * 2 * PR * D;
    if (warp == 0) {
        for (int i0 = 0; i0 < n; i0 += 32) {
            const int pid_v = i0 + lane < n ? pid_l[i0 + lane] : 0;
            const int cnt = min(32, n - i0);
            for (int j = 0; j < cnt; ++j) {
                const int pid = __shfl_sync(0xffffffffu, pid_v, j);
                const uint32_t G = base + (uint32_t)(i0 + j);
                const int st = (int)(G % ANST);
                bool ok = true;
                if (lane == 0) {
                    if (G >= (uint32_t)ANST)
                        ok = sp_mbar_wait(&c.aempty[st], ((G / ANST) & 1u) ^ 1u, CT_STATUS_TIMEOUT_FREE, p.gbar, c.gen0);
                    if (ok) {
                        const bf16 *src = p.pool + (long long)pid * PAGE_ELEMS + kvoff;
                        mbar_expect_tx(&c.afull[st], 2 * PR * D * sizeof(bf16));
                        bulk_load(sm.kv[st][0], src, PR * D * sizeof(bf16), &c.afull[st]);
                        bulk_load(sm.kv[st][1], src + PR * D, PR * D * sizeof(bf16), &c.afull[st]);
                        sq.att_p = G + 1u;
                    }
                }
                if (!__shfl_sync(0xffffffffu, (int)ok, 0)) return;
            }
        }
        return;
    }
    if (warp < 2) return;
    const int hh = warp - 2;
    int meta_v = lane < n ? meta_l[lane] : 0;
    const float scale = 1.0f / sqrtf((float)DK);
    float *pb = sm.pbuf[hh];
    float m = -INFINITY, l = 0.0f, o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    float4 qv = make_float4(0.f, 0.f, 0.f, 0.f);
    int rpa = 0, rpb = 0;
    bf16 *hi = p.xb_hi, *lo = p.xb_lo;
    for (int g = 0; g < n; ++g) {
        if ((g & 31) == 0 && g > 0) meta_v = g + lane < n ? meta_l[g + lane] : 0;
        const int meta = __shfl_sync(0xffffffffu, meta_v, g & 31);
        const int r = meta & 1023, pg = (meta >> 10) & 63, nv = ((meta >> 16) & 15) + 1, last = (meta >> 20) & 1;
        if (pg % GP == 0) {
            qv = __ldcg(reinterpret_cast<const float4 *>(p.q + (size_t)r * D + hh * DK + 4 * lane));
            rpa = rp[r];
            rpb = rp[r + 1];
            m = -INFINITY; l = 0.0f; o0 = o1 = o2 = o3 = 0.0f;
        }
        const uint32_t G = base + (uint32_t)g;
        const int st = (int)(G % ANST);
        if (!sp_mbar_wait(&c.afull[st], (G / ANST) & 1u, CT_STATUS_TIMEOUT_TMA, p.gbar, c.gen0)) return;
        const bf16 *Ks = sm.kv[st][0] + hh * DK + 4 * lane;
        const bf16 *Vs = sm.kv[st][1] + hh * DK + 4 * lane;
        float sc[PR];
#pragma unroll
        for (int k = 0; k < PR; ++k) {
            const uint2 u = *reinterpret_cast<const uint2 *>(Ks + k * D);
            const bf16 *e = reinterpret_cast<const bf16 *>(&u);
            sc[k] = qv.x * __bfloat162float(e[0]) + qv.y * __bfloat162float(e[1]) +
                    qv.z * __bfloat162float(e[2]) + qv.w * __bfloat162float(e[3]);
        }
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
        const int j = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
        const bool valid = j < nv;
        const float sj = valid ? sc[0] * scale : -INFINITY;
        const float mn = fmaxf(m, warp_max(sj));
        const float corr = expf(m - mn);
        const float pj = valid ? expf(sj - mn) : 0.0f;
        l = l * corr + warp_sum(pj) * 0.5f;
        o0 *= corr; o1 *= corr; o2 *= corr; o3 *= corr;
        m = mn;
        if ((lane & 1) == 0) pb[j] = pj;
        __syncwarp();
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
        if (lane == 0) mbar_arrive(&c.aempty[st]);
        if (!(last || pg % GP == GP - 1)) continue;
        const size_t idx = (size_t)r * D + hh * DK + 4 * lane;
        const int nseg = (rpb - rpa + GP - 1) / GP;
        if (nseg == 1) {
            const float inv = 1.0f / l;
            store_planes(o0 * inv, hi, lo, idx);
            store_planes(o1 * inv, hi, lo, idx + 1);
            store_planes(o2 * inv, hi, lo, idx + 2);
            store_planes(o3 * inv, hi, lo, idx + 3);
            continue;
        }
        const int seg = pg / GP;
        float *wp = p.attn_ws + ((size_t)r * SEG_MAX + seg) * (2 * H + D);
        if (lane == 0) { wp[hh] = m; wp[H + hh] = l; }
        *reinterpret_cast<float4 *>(wp + 2 * H + hh * DK + 4 * lane) = make_float4(o0, o1, o2, o3);
        __threadfence();
        __syncwarp();
        int tk = 0;
        if (lane == 0) tk = atomicAdd(&p.tickets[r * H + hh], 1);
        if (__shfl_sync(0xffffffffu, tk, 0) != nseg - 1) continue;
        __threadfence();
        const float *wr = p.attn_ws + (size_t)r * SEG_MAX * (2 * H + D);
        const int cl = min(lane, nseg - 1);
        const float mc = __ldcg(wr + (size_t)cl * (2 * H + D) + hh);
        const float lc = __ldcg(wr + (size_t)cl * (2 * H + D) + H + hh);
        const float Mg = warp_max(mc);
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
        if (lane == 0) p.tickets[r * H + hh] = 0;
    }
}

// Sum of CS partial float4s in split order (all loads issued first).
template <int CS>
__device__ __forceinline__ float4 sp_sum_parts(const float *pbase, size_t stride, size_t off) {
    float4 v[CS];
#pragma unroll
    for (int r = 0; r < CS; ++r) v[r] = __ldcg(reinterpret_cast<const float4 *>(pbase + r * stride + off));
    float4 s = v[0];
#pragma unroll
    for (int r = 1; r < CS; ++r) { s.x += v[r].x; s.y += v[r].y; s.z += v[r].z; s.w += v[r].w; }
    return s;
}

// One GEMM phase: items (token tile, group of TG 128-feature tiles, K split z)
// over the CTAs, item i on CTA i mod G (a group's S items are consecutive, so
// the S CTAs of a tile meet at its counter in the same round or in a later
// one, never in a cycle).  With TG = 2 an item keeps two accumulators in TMEM
// and both tiles share the item's activation tiles; each accumulator gets the
// MMA sequence of a TG = 1 item, so results do not depend on TG.
template <int BN, bool TWO>
__device__ void sp_gemm(const StepGemm &g, uint8_t *smem, StepCtrl &c, StepSeq &sq, uint32_t tmem, int warp,
                        int lane, unsigned long long *gbar, unsigned long long *stamp) {
    const unsigned long long gen0 = c.gen0;
    constexpr uint32_t A_BYTES = BM * BK * 2;
    constexpr uint32_t B_BYTES = BN * BK * 2;
    const GemmEpilogue &ep = g.ep;
    const bool lnx = ep.ln_x != nullptr;
    const int TG = g.TG;
    const uint32_t stage_bytes = (uint32_t)TG * A_BYTES + (lnx ? 0u : B_BYTES * (TWO ? 2u : 1u));
    uint8_t *xs = smem + (size_t)SP_NSTG * stage_bytes;   // LayerNorm-input tiles
    const int T_eff = *ep.T_dev;
    const int tiles = g.N / BM;
    const int groups = tiles / TG;
    const int kb_total = g.K / BK;
    const int S = g.S;
    const int kbps = kb_total / S;
    const int ntt = (T_eff + BN - 1) / BN;
    const int n_items = ntt * groups * S;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
        const int tt = it / (groups * S), rem = it % (groups * S);
        const int grp = rem / S, z = rem % S;
        const int t0 = tt * BN;
        const int kb0 = z * kbps;
        if (warp == 0) {
            if (lane == 0) {
                for (int i = 0; i < kbps; ++i) {
                    const uint32_t G = sq.kb_p;
                    const int st = (int)(G % SP_NSTG);
                    if (G >= (uint32_t)SP_NSTG &&
                        !sp_mbar_wait(&c.empty[st], ((G / SP_NSTG) & 1u) ^ 1u, CT_STATUS_TIMEOUT_FREE, gbar, gen0))
                        break;
                    uint8_t *a = smem + (size_t)st * stage_bytes;
                    const int kc = (kb0 + i) * BK;
                    mbar_expect_tx(&c.full[st], stage_bytes);
                    for (int t = 0; t < TG; ++t) tma_load_2d(a + t * A_BYTES, g.tmW, &c.full[st], kc, (grp * TG + t) * BM);
                    if (!lnx) {
                        uint8_t *x = a + TG * A_BYTES;
                        tma_load_2d(x, g.tmXh, &c.full[st], kc, t0);
                        if (TWO) tma_load_2d(x + B_BYTES, g.tmXl, &c.full[st], kc, t0);
                    }
                    sq.kb_p = G + 1u;
                }
            }
            continue;
        }
        if (warp == 1) {
            if (lane == 0) {
                constexpr uint32_t idesc = idesc_bf16(BM, BN);
                bool ok = true;
                if (sq.acc_m > 0) ok = sp_mbar_wait(&c.acc_free, (sq.acc_m - 1) & 1u, CT_STATUS_TIMEOUT_MMA, gbar, gen0);
                if (ok && lnx) ok = sp_mbar_wait(&c.xfull, sq.x_m & 1u, CT_STATUS_TIMEOUT_TMA, gbar, gen0);
                if (lnx) ++sq.x_m;
                tc_fence_after();
                for (int i = 0; i < kbps; ++i) {
                    const uint32_t G = sq.kb_m++;
                    const int st = (int)(G % SP_NSTG);
                    if (!ok) continue;
                    if (!sp_mbar_wait(&c.full[st], (G / SP_NSTG) & 1u, CT_STATUS_TIMEOUT_TMA, gbar, gen0)) {
                        ok = false;
                        continue;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(smem + (size_t)st * stage_bytes);
                    const uint32_t b = lnx ? smem_u32(xs) + (uint32_t)i * (TWO ? 2u : 1u) * B_BYTES
                                           : a + (uint32_t)TG * A_BYTES;
                    const uint64_t bd = sw128_desc(b);
                    for (int t = 0; t < TG; ++t) {
                        const uint64_t ad = sw128_desc(a + (uint32_t)t * A_BYTES);
                        const uint32_t acc = tmem + (uint32_t)(t * BN);
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k)
                            mma_bf16(acc, ad + 2 * k, bd + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
                        if (TWO) {
                            const uint64_t ld = sw128_desc(b + B_BYTES);
#pragma unroll
                            for (int k = 0; k < BK / 16; ++k) mma_bf16(acc, ad + 2 * k, ld + 2 * k, idesc, 1u);
                        }
                    }
                    mma_commit(&c.empty[st]);
                }
                mma_commit(&c.accb);
                ++sq.acc_m;
            }
            continue;
        }
        // ------------------------------------------------------------ workers
        const int et = threadIdx.x - 64;
        const int q = warp & 3;            // TMEM lane quarter: features q*32 .. q*32 + 31
        const int half = (warp - 2) >> 2;  // which 32-column chunks this warp drains
        if (lnx) {
            ln_fill<BN, TWO, SP_NW>(ep, xs, t0, T_eff, kb0, kbps, et);
            fence_proxy_async_smem();
            mbar_arrive(&c.xfull);
        }
        bool ok = sp_mbar_wait(&c.accb, sq.acc_w & 1u, CT_STATUS_TIMEOUT_MMA, gbar, gen0);
        ++sq.acc_w;
        if (stamp && et == 0) stamp[1] = globaltimer();
        ok = __all_sync(0xffffffffu, ok);
        tc_fence_after();
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
        const int f = q * 32 + lane;
        if (S == 1) {
            // no K split (TG = 1): the epilogue of gemm_tc_kernel's non-split path (the LM head)
            const int n0 = grp * BM;
            const int n = n0 + f;
            const float bias = (n < g.N && ep.bias) ? bf2f(ep.bias[n]) : 0.0f;
            const bool amx = ep.amax.best != nullptr;
            for (int cc = half * 32; cc < BN; cc += 64) {
                if (t0 + cc >= T_eff) break;
                float v[32];
                if (ok) tmem_ld32(tbase + (uint32_t)cc, v);
                if (ok && n < g.N) {
                    const int tl = min(32, T_eff - (t0 + cc));
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] += bias;
                    if (ep.Y || ep.epi != EPI_STORE) {
                        epilogue16(ep, t0 + cc, min(16, tl), n, v);
                        if (tl > 16) epilogue16(ep, t0 + cc + 16, tl - 16, n, v + 16);
                    }
                }
                if (amx) {
                    int ix[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const bool cand = ok && n < g.N && v[j] > -INFINITY;
                        ix[j] = cand ? n : 0x7fffffff;
                        v[j] = cand ? v[j] : -INFINITY;
                    }
                    warp_amax_transpose(v, ix, lane);
                    c.amax[(cc >> 5) * 128 + q * 32 + lane] = make_float2(v[0], __int_as_float(ix[0]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&c.acc_free);
            if (amx) {
                sp_wbar();
                argmax_tail<BN, SP_NW>(ep.amax, c.amax, &c.flag, t0, T_eff, et, tiles, tt);
                sp_wbar();   // c.amax and c.flag are reused by the next item
            }
            continue;
        }
        // split-K: park this CTA's partial tiles in global memory (feature fastest)
        for (int t = 0; t < TG; ++t) {
            const int tile = grp * TG + t;
            float *pt = g.part + (((size_t)tt * tiles + tile) * S + z) * (size_t)BN * BM;
            for (int cc = half * 32; cc < BN; cc += 64) {
                if (t0 + cc >= T_eff) break;
                float v[32];
                if (ok) tmem_ld32(tbase + (uint32_t)(t * BN + cc), v);
                const int tl = min(32, T_eff - (t0 + cc));
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j < tl) pt[(size_t)(cc + j) * BM + f] = ok ? v[j] : 0.0f;
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&c.acc_free);
        // count in on the tiles (a release add after the workers' barrier
        // publishes all of this CTA's partial stores), wait for their S partials
        sp_wbar();
        if (et < TG) {
            unsigned *cn = g.cnt + (size_t)tt * tiles + grp * TG + et;
            const unsigned old = atom_add_release_u32(cn, 1u);
            const unsigned target = (old / (unsigned)S + 1u) * (unsigned)S;
            sp_word_wait(cn, target, gbar, gen0);
            if (stamp && et == 0) stamp[2] = globaltimer();
        }
        sp_wbar();
        // token slice z of each tile: sum the S partials in split order (as
        // splitk_reduce), then the epilogue; warp k takes (tile, token) pairs
        // k, k + 8, ... of the TG x slice pairs
        const int slice = BN / S;
        const int tb = z * slice;
        const int wk = warp - 2;
        const int f0 = 4 * lane;
        for (int pi = wk; pi < TG * slice; pi += 8) {
            const int t_ = pi / slice, jj = pi % slice;
            const int tile = grp * TG + t_;
            const int n0 = tile * BM;
            const int t = t0 + tb + jj;
            if (t >= T_eff) continue;
            const EpiPre pre = epilogue_f4_pre(ep, t, n0 + f0, g.N);
            float b4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) b4[i] = (n0 + f0 + i < g.N && ep.bias) ? bf2f(ep.bias[n0 + f0 + i]) : 0.0f;
            const float *pbase = g.part + ((size_t)tt * tiles + tile) * S * (size_t)BN * BM;
            const size_t off = (size_t)(tb + jj) * BM + f0;
            float4 sum;
            switch (S) {
            case 2: sum = sp_sum_parts<2>(pbase, (size_t)BN * BM, off); break;
            case 4: sum = sp_sum_parts<4>(pbase, (size_t)BN * BM, off); break;
            case 8: sum = sp_sum_parts<8>(pbase, (size_t)BN * BM, off); break;
            default: sum = sp_sum_parts<16>(pbase, (size_t)BN * BM, off); break;
            }
            const float vals[4] = {sum.x + b4[0], sum.y + b4[1], sum.z + b4[2], sum.w + b4[3]};
            float o[4] = {0.f, 0.f, 0.f, 0.f};
            epilogue_f4_post(ep, t, n0 + f0, g.N, vals, pre, o);
            if (ep.stats_out) {
                const float mm = warp_sum((o[0] + o[1]) + (o[2] + o[3])) * (1.0f / 128.0f);
                const float d0 = o[0] - mm, d1 = o[1] - mm, d2 = o[2] - mm, d3 = o[3] - mm;
                const float qq = warp_sum((d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3));
                if (lane == 0) ep.stats_out[(size_t)t * (g.N / BM) + tile] = make_float2(mm, qq);
            }
        }
    }
}

// L2 prefetch of this CTA's first pages of an attention phase (cross pages are
// static; self pages are final except the rows this step's QKV phase writes,
// and those writes land in L2 over the prefetched lines).  One ring's worth
// only: more competes with the running phase for HBM.
__device__ __forceinline__ void sp_prefetch_pages(const StepParams &p, int layer, int cross) {
    const DevState &s = p.s;
    const int *cr = s.crange + (cross ? s.n_cta + 1 : 0);
    const int b = blockIdx.x;
    if (b >= s.n_cta) return;
    const int g0 = cr[b], g1 = cr[b + 1];
    const int *pid_l = cross ? s.pid_cross : s.pid_self;
    const long long kvoff = (long long)layer * 2 * PR * D;
    for (int gi = g0; gi < g1 && gi < g0 + ANST; ++gi)
        prefetch_l2(p.pool + (long long)pid_l[gi] * PAGE_ELEMS + kvoff, 2 * PR * D * sizeof(bf16));
}

// L2 prefetch of this CTA's share of a GEMM phase's weights, of its bias and
// LayerNorm vectors (CTA 0; small, but a cold miss on the phase's critical path
// otherwise) and of its tensor maps.
__device__ __forceinline__ void sp_prefetch_weights(const StepGemm &g) {
    prefetch_tmap(g.tmW);
    if (g.tmXh) prefetch_tmap(g.tmXh);
    if (g.tmXl) prefetch_tmap(g.tmXl);
    if (blockIdx.x == 0) {   // (a bulk prefetch needs a 16-byte aligned start; vectors of a file may lack it)
        auto vec = [](const bf16 *v, int n) {
            if (v && ((reinterpret_cast<uintptr_t>(v) & 15) == 0)) prefetch_l2(v, (uint32_t)((n * sizeof(bf16)) & ~15u));
        };
        vec(g.ep.bias, g.N);
        vec(g.ep.ln_g, g.K);
        vec(g.ep.ln_b, g.K);
    }
    const size_t total = (size_t)g.N * g.K * sizeof(bf16);
    size_t chunk = (total + gridDim.x - 1) / gridDim.x;
    chunk = (chunk + 15) & ~(size_t)15;
    const size_t off = (size_t)blockIdx.x * chunk;
    if (off >= total) return;
    size_t bytes = total - off < chunk ? total - off : chunk;
    const uint8_t *w = reinterpret_cast<const uint8_t *>(g.W) + off;
    while (bytes > 0) {   // at most 1 MB per instruction
        const uint32_t b = (uint32_t)(bytes < (1u << 20) ? bytes : (1u << 20));
        prefetch_l2(w, b);
        w += b;
        bytes -= b;
    }
}

template <int BN, bool TWO>
__global__ void __launch_bounds__(SP_THREADS, 1) step_kernel(const __grid_constant__ StepParams p) {
    extern __shared__ __align__(1024) uint8_t sp_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sp_smem_raw) + 1023) & ~(uintptr_t)1023);
    StepCtrl &c = *reinterpret_cast<StepCtrl *>(smem + SP_RING);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int et = threadIdx.x - 64;
    if (threadIdx.x == 0) {
        for (int i = 0; i < SP_NSTG; ++i) { mbar_init(&c.full[i], 1); mbar_init(&c.empty[i], 1); }
        mbar_init(&c.accb, 1);
        mbar_init(&c.acc_free, SP_NW / 32);
        mbar_init(&c.xfull, SP_NW);
        for (int i = 0; i < ANST; ++i) { mbar_init(&c.afull[i], 1); mbar_init(&c.aempty[i], AW); }
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(&c.tmem_slot, 256); tmem_relinquish(); }
    // the barrier epoch: the counter holds a whole number of epochs when the
    // launch starts, and a CTA reads it before its own first arrival, so every
    // CTA reads the same epoch
    if (threadIdx.x == 32) c.gen0 = ld_acquire_u64(p.gbar) / gridDim.x;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = c.tmem_slot;
    // the phase table and GEMM descriptors (fixed per engine) into shared memory
    {
        const int n_gm = min(p.n_gm, SP_MAX_GEMM), n_ph = min(p.n_ph, SP_MAX_PH);
        const uint32_t *src = reinterpret_cast<const uint32_t *>(p.gm);
        uint32_t *dst = reinterpret_cast<uint32_t *>(c.gm);
        for (size_t i = threadIdx.x; i < n_gm * sizeof(StepGemm) / 4; i += SP_THREADS) dst[i] = src[i];
        const uint32_t *src2 = reinterpret_cast<const uint32_t *>(p.ph);
        uint32_t *dst2 = reinterpret_cast<uint32_t *>(c.ph);
        for (size_t i = threadIdx.x; i < n_ph * sizeof(StepPhase) / 4; i += SP_THREADS) dst2[i] = src2[i];
    }
    __syncthreads();
    const int n_ph = min(p.n_ph, SP_MAX_PH);
    // the first phase's weights do not depend on the row builder
    if (threadIdx.x == 0 && n_ph > 0 && c.ph[0].next_gemm >= 0) sp_prefetch_weights(c.gm[c.ph[0].next_gemm]);
    pdl_wait();
    unsigned long long *stamp = p.stamps ? p.stamps + SP_NSTAMP * (size_t)blockIdx.x : nullptr;
    const size_t stamp_ph = SP_NSTAMP * (size_t)gridDim.x;
    if (stamp && threadIdx.x == 0) stamp[0] = globaltimer();
    StepSeq sq;
    for (int ph = 0; ph < n_ph; ++ph) {
        const StepPhase P = c.ph[ph];
        if (ph > 0 && threadIdx.x == 0 && P.next_gemm >= 0) sp_prefetch_weights(c.gm[P.next_gemm]);
        if (threadIdx.x == 0 && P.next_attn >= 0) sp_prefetch_pages(p, P.next_attn >> 1, P.next_attn & 1);
        switch (P.kind) {
        case SP_EMBED:
            if (warp >= 2) sp_embed(p, reinterpret_cast<float *>(smem), c.red, et);
            break;
        case SP_FINAL_LN:
            if (warp >= 2) sp_final_ln(p, c.red, et);
            break;
        case SP_ATTN:
            sp_attention(p, *reinterpret_cast<AttnSmem *>(smem), c, sq, P.arg >> 1, P.arg & 1, warp, lane);
            break;
        case SP_GEMM:
            sp_gemm<BN, TWO>(c.gm[P.arg], smem, c, sq, tmem, warp, lane, p.gbar, stamp ? stamp + ph * stamp_ph : nullptr);
            break;
        default: break;
        }
        // generic writes to the shared data region (row buffer, attention
        // probabilities, LayerNorm tiles) before the next phase's async copies
        fence_proxy_async_smem();
        sp_grid_sync(p.gbar, c.gen0, stamp ? stamp + ph * stamp_ph + 3 : nullptr,
                     stamp ? stamp + (ph + 1) * stamp_ph : nullptr);
    }
    // copies and MMAs still in flight (only after a wait gave up): let them
    // land before the shared memory and the TMEM are released
    if (threadIdx.x == 0) {
        for (uint32_t G = sq.kb_p > SP_NSTG ? sq.kb_p - SP_NSTG : 0u; G < sq.kb_p; ++G)
            sp_drain_wait(&c.full[G % SP_NSTG], (G / SP_NSTG) & 1u);
        for (uint32_t G = sq.att_p > ANST ? sq.att_p - ANST : 0u; G < sq.att_p; ++G)
            sp_drain_wait(&c.afull[G % ANST], (G / ANST) & 1u);
    }
    if (threadIdx.x == 32 && sq.acc_m > 0) sp_drain_wait(&c.accb, (sq.acc_m - 1) & 1u);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, 256);
}
