// gemm.cuh -- tcgen05 GEMM of libct_b200.so: Y[t, n] = epi( X[t, :] . W[n, :] + b[n] ).
//
// W is a bf16 weight matrix [N, K] (row-major, the layout of every linear in
// the model file), X is bf16 activations [T, K].  The kernel tiles the
// weights as the MMA's M side (128 output features per tile) and the tokens as
// the N side (BN = 32..256 tokens per tile), so small decode batches still
// fill the 128-row MMA ("swap-AB").  Optional second activation plane (X_lo)
// carries the bf16 residual of fp32 activations: X ~= X_hi + X_lo to ~2^-17
// relative, which lets fp32 inputs reach near-fp32 accuracy on bf16 tensor
// cores (two MMAs into the same TMEM accumulator).
#pragma once
#include "ct_common.cuh"

namespace ct {

enum Epi : int {
    EPI_STORE = 0,    // Y = acc + b
    EPI_SILU = 1,     // Y = silu(acc + b)
    EPI_RELU = 2,     // Y = relu(acc + b)
    EPI_FMADD = 3,    // Y += scale * (acc + b)
    EPI_KVCACHE = 4,  // Y[(t*kv_stride + pos[t]-1) * ldy + n] = acc + b
    EPI_BF16 = 5,     // Ybf[t * ldy + n] = bf16(act(acc + b)), act = p.act (0 none, 1 silu, 2 relu)
    EPI_RELU_FLAT = 6,  // token t = frame * flat_f + f:  Y[frame * ldy + n * flat_f + f] = relu(acc + b)
    EPI_QKV_PAGED = 7,  // n < qdim: Y[t*ldy+n] = v (fp32 Q); else K/V -> kv_pool at row_off[t] (layer `layer`)
    EPI_CAKV_PAGED = 8, // n = (l*2 + kv)*1024 + c -> kv_pool[row_off[t] + (l*2+kv)*PAGE*1024 + c]
};

// Paged KV pool geometry: page = [DEC_N layers][K,V][kPageRows rows][1024].
constexpr int kPageRows = 16;

// Sequence states of the engine's slot table.
enum SeqState : int { SEQ_FREE = 0, SEQ_PREFILL = 1, SEQ_DECODE = 2, SEQ_DONE = 3 };

// Greedy-decode hand-off of the LM-head GEMM.  With ArgmaxSink::best set, the
// epilogue reduces each token row's logits over the CTA's 128-entry
// vocabulary tile (first index of the maximum, warp shuffles) and folds the
// result into the row's 64-bit key with one atomicMax: the key orders by the
// value, then by the lower index, so the fold is independent of the order in
// which the tiles arrive and the winner is the first index of the maximum over
// the whole vocabulary, as the reference's argmax
// (backends/cpu/backend.c:446-456).  The CTA that takes the last ticket of a
// row block (no waiting) reads the keys, appends each row's token to its
// sequence (decode_append) and clears the keys.
struct ArgmaxSink {
    unsigned long long *best = nullptr;   // [rows]: argmax key (0 = no candidate; cleared after use)
    unsigned *ticket = nullptr;           // [row blocks]: tiles finished (the last one resets it to 0)
    int *next = nullptr;                  // [rows]: chosen token (before the forced-EOS rule)
    // slot table (row q belongs to slot q_slot[q])
    const int *q_slot = nullptr, *forced = nullptr, *plen = nullptr;
    int *state = nullptr, *gen = nullptr, *pos = nullptr, *tok = nullptr, *out_tok = nullptr;
    int *done_map = nullptr;    // host-mapped: generated count of a finished slot
    int max_seq = 0, eos = 0;
};

// Argmax key of a candidate (value v, index i < 2^31): the float's bits mapped
// to an unsigned order (larger value, larger key) in the high word, the
// complement of the index in the low word (lower index, larger key).
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
    const unsigned b = v == 0.0f ? 0u : __float_as_uint(v);   // -0 ties with +0, as the float comparison does
    const unsigned ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)i);
}

// Append the greedy token of row q to its sequence: EOS when the forced length
// is reached, advance the position (the prompt on the prefill step), retire
// on EOS / forced length / max_seq (done_map tells the host).
__device__ __forceinline__ void decode_append(const ArgmaxSink &s, int q, int tok) {
    s.next[q] = tok;
    const int slot = s.q_slot[q];
    const int st = s.state[slot];
    const int gen = s.gen[slot] + 1;
    const int forced = s.forced[slot];
    if (forced > 0 && gen >= forced) tok = s.eos;
    if (gen - 1 < s.max_seq) s.out_tok[(size_t)slot * s.max_seq + gen - 1] = tok;
    s.gen[slot] = gen;
    s.pos[slot] += st == SEQ_PREFILL ? s.plen[slot] : 1;
    s.tok[slot] = tok;
    const bool done = (forced > 0 ? gen >= forced : tok == s.eos) || s.plen[slot] + gen >= s.max_seq;
    if (done) {
        s.state[slot] = SEQ_DONE;
        volatile int *dm = s.done_map;
        dm[slot] = gen;
        __threadfence_system();
    } else {
        s.state[slot] = SEQ_DECODE;
    }
}

struct GemmEpilogue {
    int epi = EPI_STORE;
    float scale = 1.0f;
    const bf16 *bias = nullptr;   // [N] or null
    float *Y = nullptr;           // fp32 output
    bf16 *Ybf = nullptr;          // bf16 output (EPI_BF16)
    int ldy = 0;                  // output row stride in elements (default N)
    const int *pos = nullptr;     // EPI_KVCACHE: per-token sequence length (slot = pos-1)
    int kv_stride = 0;            // EPI_KVCACHE: rows per item
    int act = 0;                  // EPI_BF16 activation
    int flat_f = 0;               // EPI_RELU_FLAT: frequency bins per frame
    const int *row_mask = nullptr;  // optional: rows t with row_mask[t] == 0 are not stored
    bf16 *Ybf_lo = nullptr;       // EPI_BF16: optional residual plane (v - hi), same layout
    bf16 *kv_pool = nullptr;      // EPI_QKV_PAGED / EPI_CAKV_PAGED
    const long long *row_off = nullptr;  // per-row element offset of (page, row-in-page); < 0 skips
    int layer = 0;
    int qdim = 0;
    int kv_width = 1024;          // K/V row width in the pool
    const int *T_dev = nullptr;   // optional device row count (rows >= *T_dev are skipped)
    long x_rows = 0;              // rows of the X buffers (tensor-map extent); 0 = T
    bool pdl = false;             // launch with programmatic stream serialization
    int split = 0;                // K-split factor override (0 = split_factor(N, K)); a fixed
                                  // per-call-site value keeps results independent of T
    // Row statistics of the stored values (EPI_FMADD with a K split): for token t
    // and 128-feature tile j, stats_out[t * (N / 128) + j] = (mean, sum of squared
    // deviations) of the tile's 128 new values -- the partials a following
    // LayerNorm-input GEMM merges into the row's mean and variance.
    float2 *stats_out = nullptr;
    // LayerNorm-input mode: instead of TMA-loading bf16 planes, the kernel forms
    // its activation tiles as LN(ln_x[t]) = (x - mean) * rstd * ln_g + ln_b
    // (eps 1e-5, biased variance), split into hi/lo planes in shared memory.
    // ln_stats holds the (mean, M2) partials of the K / 128 feature tiles of
    // each row, as stats_out writes them; ln_x rows have stride K.  K must be a
    // multiple of 128 and at most 1024; ln_g / ln_b 16-byte aligned.
    const float *ln_x = nullptr;
    const float2 *ln_stats = nullptr;
    const bf16 *ln_g = nullptr;
    const bf16 *ln_b = nullptr;
    // Greedy argmax of each token row over N (EPI_STORE without a K split;
    // Y may then be null, in which case no logits are stored).
    ArgmaxSink amax;
};

// Per-thread GEMM context: stream, workspaces, tensor-map cache.
struct GemmCtx;
GemmCtx *gemm_ctx();   // the calling thread's context (created on first use)
void gemm_ctx_release();

// Launch on `st`.  X_lo may be null (single bf16 plane).  allow_split enables
// the split-K used for decode-sized problems: the K-split CTAs of one output
// tile form a thread-block cluster and reduce through distributed shared
// memory in rank order, so the result is deterministic; the split factor
// depends only on (N, K) (and BN divisibility), never on T.  With ep.T_dev the
// kernel reads a device row count before its dependency wait, so that count
// must come from a kernel at least two launches upstream.
void gemm_bf16(cudaStream_t st, const bf16 *W, int N, int K, const bf16 *X_hi, const bf16 *X_lo, int T,
               const GemmEpilogue &ep, bool allow_split);

// fp32 activations [T, K] (row stride ldx) -> bf16 hi/lo planes [T, Kp], zero-padded to Kp.
void split_fp32_to_bf16(cudaStream_t st, const float *x, int T, int K, int ldx, bf16 *hi, bf16 *lo, int Kp);

// Convenience for the fp32 ABI: converts X into the thread's scratch planes,
// pads K to a multiple of 8 (TMA row pitch) and makes an aligned weight copy
// when the blob pointer is not 16-byte aligned.
void linear_fp32(cudaStream_t st, const bf16 *W, int N, int K, const float *X, int T, int ldx,
                 const GemmEpilogue &ep, bool allow_split = true, bool two_term = true);

int split_factor(int N, int K);

// K-split factor gemm_bf16 uses for an N x K weight at token tile BN
// (`requested` = ep.split: 0 = by shape, 1 = none).
int gemm_nsplit(int N, int K, int BN, int requested);

// Tensor map of a bf16 [rows, cols] operand with a box of 64 x box_rows
// (128-byte swizzle), as the GEMMs load it.
CUtensorMap gemm_tmap(const void *ptr, long rows, long cols, long box_rows);

// Called whenever a per-thread scratch buffer moves, so that cached CUDA graphs
// holding its old address are dropped (defined by the ABI layer).
void scratch_moved();

}  // namespace ct
