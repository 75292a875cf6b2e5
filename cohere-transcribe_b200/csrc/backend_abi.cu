// backend_abi.cu -- the 40 backend_* entry points of include/ct_backend.h.
//
// Same contract as the reference backends (backends/backend.h:20-228): weight
// arguments are host pointers into the blob given to
// backend_weights_upload_blob and are translated by byte offset to this
// thread's device copy; activations are fp32 in the arena; per-thread state.
// fp32 activations reach the bf16 tensor cores as two bf16 planes (hi + lo),
// which keeps the linear family within ~1e-6 relative of the fp32 reference.
#include <string.h>

#include <vector>

#include "../../include/ct_backend.h"
#include "gemm.cuh"
#include "kernels.cuh"

using namespace ct;

#define CT_MAX_DEVICES 8
#define CT_MAX_BATCH 4096

// ---- process-wide weight copies (one per device) ---------------------------
static const uint8_t *g_host_base = nullptr;
static size_t g_blob_bytes = 0;
static void *g_dev_blob[CT_MAX_DEVICES];
static int g_num_devices = 0;

struct GraphEntry {
    int tag, T, S, B;
    const void *arena;
    cudaGraph_t graph;
    cudaGraphExec_t exec;
};

struct Tls {
    int device = -1;
    cudaStream_t st = nullptr;
    cudaStream_t side = nullptr;
    cudaEvent_t staged = nullptr;      // last upload from the pinned staging area
    float *arena = nullptr;
    size_t arena_bytes = 0;
    int *d_tokens = nullptr;           // MAX_SEQ prompt/decode tokens (backend_upload_tokens)
    int *d_S = nullptr;                // device decode counter (B = 1 path)
    int *d_S_batch = nullptr, *d_T_enc = nullptr, *d_active = nullptr, *d_cur = nullptr, *d_out = nullptr;
    int *h_stage = nullptr;            // pinned: 4 x CT_MAX_BATCH ints
    float *attn_ws = nullptr;
    size_t attn_ws_floats = 0;
    std::vector<GraphEntry> graphs;
};
static thread_local Tls t;

static inline const bf16 *W16(const uint16_t *host_ptr) {
    if (!host_ptr) return nullptr;
    const uint8_t *p = reinterpret_cast<const uint8_t *>(host_ptr);
    if (!g_host_base || p < g_host_base || p >= g_host_base + g_blob_bytes)
        CT_FATAL("weight pointer %p is outside the uploaded blob", (const void *)host_ptr);
    if (t.device < 0 || t.device >= g_num_devices || !g_dev_blob[t.device])
        CT_FATAL("backend_init(device) with an uploaded blob must precede compute calls");
    return reinterpret_cast<const bf16 *>(static_cast<uint8_t *>(g_dev_blob[t.device]) + (p - g_host_base));
}

static void require_init() {
    if (t.device < 0) CT_FATAL("backend_init() was not called on this thread");
}

static bool capturing() {
    cudaStreamCaptureStatus s = cudaStreamCaptureStatusNone;
    CT_CHECK(cudaStreamIsCapturing(t.st, &s));
    return s != cudaStreamCaptureStatusNone;
}

static void graphs_clear() {
    for (auto &g : t.graphs) {
        cudaGraphExecDestroy(g.exec);
        cudaGraphDestroy(g.graph);
    }
    t.graphs.clear();
}

void ct::scratch_moved() { graphs_clear(); }

static float *attn_ws(size_t floats) {
    if (floats <= t.attn_ws_floats) return t.attn_ws;
    if (t.st && capturing()) CT_FATAL("attention workspace growth inside graph capture");
    if (t.st) CT_CHECK(cudaStreamSynchronize(t.st));
    graphs_clear();
    cudaFree(t.attn_ws);
    t.attn_ws_floats = floats * 2;
    CT_CHECK(cudaMalloc(&t.attn_ws, t.attn_ws_floats * sizeof(float)));
    return t.attn_ws;
}

// Copy n host ints into the device array `dst` through pinned staging slot `slot`.
static void stage_ints(int *dst, const int *host, int n, int slot) {
    if (n < 0 || n > CT_MAX_BATCH) CT_FATAL("batch of %d exceeds %d", n, CT_MAX_BATCH);
    CT_CHECK(cudaEventSynchronize(t.staged));
    int *h = t.h_stage + (size_t)slot * CT_MAX_BATCH;
    memcpy(h, host, sizeof(int) * n);
    CT_CHECK(cudaMemcpyAsync(dst, h, sizeof(int) * n, cudaMemcpyHostToDevice, t.st));
    CT_CHECK(cudaEventRecord(t.staged, t.st));
}

// ============================================================ lifecycle ====
extern "C" int backend_num_devices(void) { return g_num_devices; }

extern "C" void backend_thread_cleanup(void) {
    if (t.device < 0) return;
    CT_CHECK(cudaSetDevice(t.device));
    CT_CHECK(cudaStreamSynchronize(t.st));
    graphs_clear();
    gemm_ctx_release();
    cudaFree(t.arena);
    cudaFree(t.d_tokens);
    cudaFree(t.d_S);
    cudaFree(t.d_S_batch);
    cudaFree(t.d_T_enc);
    cudaFree(t.d_active);
    cudaFree(t.d_cur);
    cudaFree(t.d_out);
    cudaFree(t.attn_ws);
    cudaFreeHost(t.h_stage);
    cudaEventDestroy(t.staged);
    cudaStreamDestroy(t.side);
    cudaStreamDestroy(t.st);
    t = Tls();
}

extern "C" void backend_init(int device_id) {
    if (t.device >= 0) backend_thread_cleanup();
    int n = 0;
    CT_CHECK(cudaGetDeviceCount(&n));
    if (device_id < 0 || device_id >= n) CT_FATAL("backend_init: device %d of %d", device_id, n);
    t.device = device_id;
    CT_CHECK(cudaSetDevice(device_id));
    int major = 0, minor = 0;
    CT_CHECK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device_id));
    CT_CHECK(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device_id));
    if (major != 10 || minor != 0) CT_FATAL("device %d is sm_%d%d; this library is built for sm_100a (B200)", device_id, major, minor);
    CT_CHECK(cudaStreamCreateWithFlags(&t.st, cudaStreamNonBlocking));
    CT_CHECK(cudaStreamCreateWithFlags(&t.side, cudaStreamNonBlocking));
    CT_CHECK(cudaEventCreateWithFlags(&t.staged, cudaEventDisableTiming));
    CT_CHECK(cudaEventRecord(t.staged, t.st));
    CT_CHECK(cudaMalloc(&t.d_tokens, MAX_SEQ * sizeof(int)));
    CT_CHECK(cudaMalloc(&t.d_S, sizeof(int)));
    CT_CHECK(cudaMalloc(&t.d_S_batch, CT_MAX_BATCH * sizeof(int)));
    CT_CHECK(cudaMalloc(&t.d_T_enc, CT_MAX_BATCH * sizeof(int)));
    CT_CHECK(cudaMalloc(&t.d_active, CT_MAX_BATCH * sizeof(int)));
    CT_CHECK(cudaMalloc(&t.d_cur, CT_MAX_BATCH * sizeof(int)));
    CT_CHECK(cudaMalloc(&t.d_out, CT_MAX_BATCH * sizeof(int)));
    CT_CHECK(cudaMemset(t.d_S, 0, sizeof(int)));
    CT_CHECK(cudaMallocHost(&t.h_stage, 4 * CT_MAX_BATCH * sizeof(int)));
    attn_ws(8u << 20);
    gemm_ctx();
}

extern "C" void backend_destroy(void) {
    backend_thread_cleanup();
    for (int d = 0; d < g_num_devices; ++d) {
        if (!g_dev_blob[d]) continue;
        CT_CHECK(cudaSetDevice(d));
        CT_CHECK(cudaFree(g_dev_blob[d]));
        g_dev_blob[d] = nullptr;
    }
    g_num_devices = 0;
    g_host_base = nullptr;
    g_blob_bytes = 0;
}

// Weight fan-out: host -> device 0 once, then device 0 -> every other device
// over NVLink (cudaMemcpyPeer), instead of one host upload per GPU.
extern "C" void backend_weights_upload_blob(const void *host_base, size_t bytes) {
    int n = 0, cur = 0;
    CT_CHECK(cudaGetDeviceCount(&n));
    CT_CHECK(cudaGetDevice(&cur));
    if (n > CT_MAX_DEVICES) n = CT_MAX_DEVICES;
    for (int d = 0; d < g_num_devices; ++d)
        if (g_dev_blob[d]) { CT_CHECK(cudaSetDevice(d)); cudaFree(g_dev_blob[d]); g_dev_blob[d] = nullptr; }
    g_host_base = static_cast<const uint8_t *>(host_base);
    g_blob_bytes = bytes;
    g_num_devices = n;
    for (int d = 0; d < n; ++d) {
        CT_CHECK(cudaSetDevice(d));
        CT_CHECK(cudaMalloc(&g_dev_blob[d], bytes));
    }
    CT_CHECK(cudaSetDevice(0));
    CT_CHECK(cudaMemcpy(g_dev_blob[0], host_base, bytes, cudaMemcpyHostToDevice));
    for (int d = 1; d < n; ++d) CT_CHECK(cudaMemcpyPeer(g_dev_blob[d], d, g_dev_blob[0], 0, bytes));
    CT_CHECK(cudaDeviceSynchronize());
    CT_CHECK(cudaSetDevice(cur));
}

extern "C" void *backend_device_ptr(const void *host_ptr) {
    return const_cast<bf16 *>(W16(static_cast<const uint16_t *>(host_ptr)));
}

extern "C" float *backend_arena_alloc(size_t floats) {
    require_init();
    const size_t need = floats * sizeof(float);
    graphs_clear();
    if (need > t.arena_bytes) {
        CT_CHECK(cudaStreamSynchronize(t.st));
        cudaFree(t.arena);
        t.arena = nullptr;
        CT_CHECK(cudaMalloc(&t.arena, need));
        t.arena_bytes = need;
    }
    return t.arena;
}

extern "C" void backend_arena_free(float *arena) {
    (void)arena;
    require_init();
    CT_CHECK(cudaStreamSynchronize(t.st));
}

extern "C" void backend_htod(float *dev_dst, const float *host_src, size_t floats) {
    require_init();
    CT_CHECK(cudaMemcpyAsync(dev_dst, host_src, floats * sizeof(float), cudaMemcpyHostToDevice, t.st));
    CT_CHECK(cudaStreamSynchronize(t.st));
}

extern "C" void backend_dtoh(void *host_dst, const void *dev_src, size_t bytes) {
    require_init();
    CT_CHECK(cudaMemcpyAsync(host_dst, dev_src, bytes, cudaMemcpyDeviceToHost, t.st));
    CT_CHECK(cudaStreamSynchronize(t.st));
}

// ============================================================ compute ======
extern "C" void backend_layernorm(float *dst, const float *src, const uint16_t *w, const uint16_t *b, int T, int D) {
    require_init();
    layernorm(t.st, dst, src, W16(w), W16(b), T, D);
}

static void linear_ep(float *y, const float *x, const uint16_t *W, const uint16_t *b, int T, int in_d, int out_d,
                      int epi, float scale) {
    require_init();
    GemmEpilogue ep;
    ep.epi = epi;
    ep.scale = scale;
    ep.bias = W16(b);
    ep.Y = y;
    ep.ldy = out_d;
    linear_fp32(t.st, W16(W), out_d, in_d, x, T, in_d, ep);
}

extern "C" void backend_linear(float *y, const float *x, const uint16_t *W, const uint16_t *b, int T, int in_d,
                               int out_d) {
    linear_ep(y, x, W, b, T, in_d, out_d, EPI_STORE, 1.0f);
}
extern "C" void backend_linear_silu(float *y, const float *x, const uint16_t *W, const uint16_t *b, int T, int in_d,
                                    int out_d) {
    linear_ep(y, x, W, b, T, in_d, out_d, EPI_SILU, 1.0f);
}
extern "C" void backend_linear_relu(float *y, const float *x, const uint16_t *W, const uint16_t *b, int T, int in_d,
                                    int out_d) {
    linear_ep(y, x, W, b, T, in_d, out_d, EPI_RELU, 1.0f);
}
extern "C" void backend_linear_fmadd(float *acc, float scale, const float *x, const uint16_t *W, const uint16_t *b,
                                     int T, int in_d, int out_d) {
    linear_ep(acc, x, W, b, T, in_d, out_d, EPI_FMADD, scale);
}

extern "C" void backend_add_inplace(float *dst, const float *src, int n) {
    require_init();
    add_inplace(t.st, dst, src, n > 0 ? (size_t)n : 0);
}

// backends/cpu/backend.c:188-229 with channels-last activations: the two 1x1
// convolutions are tensor-core GEMMs over (frame, bin) rows, the last one
// stores straight into the flattened [T_enc, C*F3] layout.
extern "C" void backend_encoder_subsampling(const float *mel, int T_mel, int T_mel_stride, float *x_enc, int T_enc,
                                            float *work, const Weights *W) {
    require_init();
    const int C = SUB_CH, F1 = (N_MELS + 1) / 2, F2 = (F1 + 1) / 2, F3 = (F2 + 1) / 2;
    const int T1 = (T_mel + 1) / 2, T2 = (T1 + 1) / 2, T3 = (T2 + 1) / 2;
    if (T3 != T_enc) CT_FATAL("encoder_subsampling: T_enc %d does not match T_mel %d (expected %d)", T_enc, T_mel, T3);
    float *r0 = work, *r1 = work + (size_t)C * T1 * F1;
    sub_conv0(t.st, mel, T_mel, T_mel_stride, N_MELS, W16(W->s0w), W16(W->s0b), r0, C);
    sub_dwconv(t.st, r0, T1, F1, C, W16(W->s2w), W16(W->s2b), r1);
    GemmEpilogue ep;
    ep.epi = EPI_RELU; ep.bias = W16(W->s3b); ep.Y = r0; ep.ldy = C;
    linear_fp32(t.st, W16(W->s3w), C, C, r1, T2 * F2, C, ep);
    sub_dwconv(t.st, r0, T2, F2, C, W16(W->s5w), W16(W->s5b), r1);
    GemmEpilogue ef;
    ef.epi = EPI_RELU_FLAT; ef.bias = W16(W->s6b); ef.Y = r0; ef.ldy = C * F3; ef.flat_f = F3;
    linear_fp32(t.st, W16(W->s6w), C, C, r1, T_enc * F3, C, ef);
    GemmEpilogue eo;
    eo.bias = W16(W->sob); eo.Y = x_enc; eo.ldy = ENC_D;
    linear_fp32(t.st, W16(W->sow), ENC_D, C * F3, r0, T_enc, C * F3, eo);
}

extern "C" void backend_make_rel_pos_emb(float *pe, int T) {
    require_init();
    make_rel_pos_emb(t.st, pe, T, ENC_D);
}

// backends/cpu/backend.c:244-298; scores never leave the SM (online softmax).
extern "C" void backend_rel_pos_mhsa(float *x, const float *pos_emb, int T, const ELayer *L, float *work) {
    require_init();
    const int D = ENC_D, PL = 2 * T - 1;
    float *Q = work, *K = Q + (size_t)T * D, *V = K + (size_t)T * D, *P = V + (size_t)T * D;
    float *att = P + (size_t)PL * D;
    GemmEpilogue e;
    e.ldy = D;
    e.Y = Q; e.bias = W16(L->sa_qb); linear_fp32(t.st, W16(L->sa_qw), D, D, x, T, D, e);
    e.Y = K; e.bias = W16(L->sa_kb); linear_fp32(t.st, W16(L->sa_kw), D, D, x, T, D, e);
    e.Y = V; e.bias = W16(L->sa_vb); linear_fp32(t.st, W16(L->sa_vw), D, D, x, T, D, e);
    e.Y = P; e.bias = nullptr;       linear_fp32(t.st, W16(L->sa_pw), D, D, pos_emb, PL, D, e);
    relpos_attn_f32(t.st, Q, K, V, P, W16(L->sa_pbu), W16(L->sa_pbv), att, T, ENC_H, ENC_DK, D);
    e.Y = x; e.bias = W16(L->sa_ob); linear_fp32(t.st, W16(L->sa_ow), D, D, att, T, D, e);
}

// backends/cpu/backend.c:300-337
extern "C" void backend_conformer_conv(float *x, int T, const ELayer *L, float *work) {
    require_init();
    const int D = ENC_D;
    float *pw1 = work, *y = work + (size_t)T * 2 * D;
    GemmEpilogue e;
    e.Y = pw1; e.ldy = 2 * D; e.bias = W16(L->cv_pw1b);
    linear_fp32(t.st, W16(L->cv_pw1w), 2 * D, D, x, T, D, e);
    glu_dwconv_bn_silu(t.st, pw1, y, T, D, ENC_CK, W16(L->cv_dww), W16(L->cv_dwb), W16(L->cv_bnw), W16(L->cv_bnb),
                       W16(L->cv_bnmean), W16(L->cv_bnvar));
    GemmEpilogue o;
    o.Y = x; o.ldy = D; o.bias = W16(L->cv_pw2b);
    linear_fp32(t.st, W16(L->cv_pw2w), D, D, y, T, D, o);
}

static AttnRows dec_rows(float *out, const float *Q, const float *K, const float *V, int R) {
    AttnRows a;
    a.Q = Q; a.ldq = DEC_D; a.K = K; a.V = V; a.kv_item = 0; a.ldkv = DEC_D;
    a.len_arr = nullptr; a.len_dev = nullptr; a.len_const = 0; a.len_max = 0;
    a.mask = nullptr; a.mask_ld = 0; a.out = out; a.ldo = DEC_D;
    a.R = R; a.H = DEC_H; a.DK = DEC_DK; a.scale = 1.0f / sqrtf((float)DEC_DK);
    return a;
}

static void run_attn(const AttnRows &a) {
    attn_rows_f32(t.st, a, attn_ws(attn_ws_floats(a.R, a.H, a.DK, a.len_max)), t.attn_ws_floats);
}

extern "C" void backend_sdp_attn(float *out, const float *q, const float *k, const float *v, const float *mask,
                                 int T_q, int T_k, float *work) {
    (void)work;
    require_init();
    AttnRows a = dec_rows(out, q, k, v, T_q);
    a.len_const = T_k; a.len_max = T_k; a.mask = mask; a.mask_ld = T_k;
    run_attn(a);
}

extern "C" void backend_embed(float *h, const int *tokens, int S, int pos_start, const uint16_t *etw,
                              const uint16_t *epw, const uint16_t *elnw, const uint16_t *elnb) {
    require_init();
    if (S < 0 || S > MAX_SEQ) CT_FATAL("backend_embed: S %d", S);
    // Outside capture the host tokens are authoritative; inside capture the
    // device token buffer staged by backend_upload_tokens is (as in model.h).
    if (tokens && !capturing())
        CT_CHECK(cudaMemcpyAsync(t.d_tokens, tokens, sizeof(int) * S, cudaMemcpyHostToDevice, t.st));
    embed_ln(t.st, h, t.d_tokens, nullptr, pos_start, nullptr, S, W16(etw), W16(epw), W16(elnw), W16(elnb), DEC_D,
             VOCAB, MAX_SEQ);
    if (tokens && !capturing()) CT_CHECK(cudaStreamSynchronize(t.st));
}

extern "C" void backend_fill_causal_mask(float *mask, int S) {
    require_init();
    fill_causal_mask(t.st, mask, S);
}

extern "C" void backend_lm_head(float *logits_out, const float *last, const uint16_t *etw, const uint16_t *hdb) {
    linear_ep(logits_out, last, etw, hdb, 1, DEC_D, VOCAB, EPI_STORE, 1.0f);
}

// ============================================================ graphs =======
extern "C" void backend_upload_tokens(const int *host_tokens, int S) {
    require_init();
    if (S < 0 || S > MAX_SEQ) CT_FATAL("backend_upload_tokens: S %d", S);
    CT_CHECK(cudaMemcpyAsync(t.d_tokens, host_tokens, sizeof(int) * S, cudaMemcpyHostToDevice, t.st));
    CT_CHECK(cudaStreamSynchronize(t.st));
}

extern "C" int backend_graph_replay(int tag, int T_enc, int S, int B) {
    require_init();
    for (auto &g : t.graphs)
        if (g.tag == tag && g.T == T_enc && g.S == S && g.B == B && g.arena == t.arena) {
            CT_CHECK(cudaGraphLaunch(g.exec, t.st));
            CT_CHECK(cudaStreamSynchronize(t.st));
            return 1;
        }
    return 0;
}

extern "C" void backend_graph_begin_capture(int tag) {
    (void)tag;
    require_init();
    CT_CHECK(cudaStreamBeginCapture(t.st, cudaStreamCaptureModeRelaxed));
}

extern "C" void backend_graph_end_capture(int tag, int T_enc, int S, int B) {
    require_init();
    GraphEntry g{tag, T_enc, S, B, t.arena, nullptr, nullptr};
    CT_CHECK(cudaStreamEndCapture(t.st, &g.graph));
    CT_CHECK(cudaGraphInstantiate(&g.exec, g.graph, 0));
    CT_CHECK(cudaGraphLaunch(g.exec, t.st));
    CT_CHECK(cudaStreamSynchronize(t.st));
    if (t.graphs.size() >= 4096) {   // bounded cache, as the reference's (backends/cuda/backend.cu:834-846)
        cudaGraphExecDestroy(g.exec);
        cudaGraphDestroy(g.graph);
        return;
    }
    t.graphs.push_back(g);
}

// ============================================================ B = 1 decode =
__global__ void inc_counter_kernel(int *s) { *s += 1; }

extern "C" void backend_decode_set_S(int n) {
    require_init();
    CT_CHECK(cudaMemcpyAsync(t.d_S, &n, sizeof(int), cudaMemcpyHostToDevice, t.st));
    CT_CHECK(cudaStreamSynchronize(t.st));
}

extern "C" void backend_decode_inc_S(void) {
    require_init();
    inc_counter_kernel<<<1, 1, 0, t.st>>>(t.d_S);
    CT_CHECK(cudaGetLastError());
}

extern "C" void backend_linear_to_kvcache(float *cache, const float *x, const uint16_t *W, const uint16_t *b,
                                          int in_d, int out_d) {
    require_init();
    GemmEpilogue e;
    e.epi = EPI_KVCACHE; e.bias = W16(b); e.Y = cache; e.ldy = out_d; e.pos = t.d_S; e.kv_stride = MAX_SEQ;
    linear_fp32(t.st, W16(W), out_d, in_d, x, 1, in_d, e);
}

extern "C" void backend_sdp_attn_devS(float *out, const float *q, const float *k, const float *v, float *work) {
    (void)work;
    require_init();
    AttnRows a = dec_rows(out, q, k, v, 1);
    a.len_dev = t.d_S; a.len_max = MAX_SEQ;
    run_attn(a);
}

extern "C" void backend_embed_decode(float *h, const uint16_t *etw, const uint16_t *epw, const uint16_t *elnw,
                                     const uint16_t *elnb) {
    require_init();
    embed_ln(t.st, h, t.d_tokens, t.d_S, -1, nullptr, 1, W16(etw), W16(epw), W16(elnw), W16(elnb), DEC_D, VOCAB,
             MAX_SEQ);
}

// ============================================================ batched ======
extern "C" void backend_embed_decode_batch(float *h, const int *tokens, const int *S_dev, const int *active, int B,
                                           const uint16_t *etw, const uint16_t *epw, const uint16_t *elnw,
                                           const uint16_t *elnb) {
    require_init();
    stage_ints(t.d_cur, tokens, B, 0);
    stage_ints(t.d_S_batch, S_dev, B, 1);
    stage_ints(t.d_active, active, B, 2);
    embed_ln(t.st, h, t.d_cur, t.d_S_batch, -1, t.d_active, B, W16(etw), W16(epw), W16(elnw), W16(elnb), DEC_D,
             VOCAB, MAX_SEQ);
}

extern "C" void backend_lm_head_batch(float *logits, const float *h, const uint16_t *etw, const uint16_t *hdb,
                                      const int *active, int B) {
    require_init();
    stage_ints(t.d_active, active, B, 2);
    GemmEpilogue e;
    e.bias = W16(hdb); e.Y = logits; e.ldy = VOCAB; e.row_mask = t.d_active;
    linear_fp32(t.st, W16(etw), VOCAB, DEC_D, h, B, DEC_D, e);
}

extern "C" void backend_argmax_batch(int *out, const float *logits, const int *active, int B) {
    require_init();
    stage_ints(t.d_active, active, B, 2);
    argmax_rows(t.st, logits, B, VOCAB, t.d_active, t.d_out);
    int *h = t.h_stage + 3 * (size_t)CT_MAX_BATCH;
    CT_CHECK(cudaMemcpyAsync(h, t.d_out, sizeof(int) * B, cudaMemcpyDeviceToHost, t.st));
    CT_CHECK(cudaStreamSynchronize(t.st));
    for (int b = 0; b < B; ++b)
        if (active[b]) out[b] = h[b];
}

extern "C" void backend_upload_T_enc(const int *T_enc, int B) {
    require_init();
    stage_ints(t.d_T_enc, T_enc, B, 0);
    CT_CHECK(cudaStreamSynchronize(t.st));
}

extern "C" void backend_linear_to_kvcache_batch(float *cache, const float *x, const uint16_t *W, const uint16_t *b,
                                                int B, int cache_seq_stride, int in_d, int out_d) {
    require_init();
    GemmEpilogue e;
    e.epi = EPI_KVCACHE; e.bias = W16(b); e.Y = cache; e.ldy = out_d; e.pos = t.d_S_batch;
    e.kv_stride = cache_seq_stride;
    linear_fp32(t.st, W16(W), out_d, in_d, x, B, in_d, e);
}

static void sdp_batch(float *out, const float *Q, const float *K, const float *V, int T_k_stride, int B,
                      const int *lens) {
    require_init();
    AttnRows a = dec_rows(out, Q, K, V, B);
    a.kv_item = (long)T_k_stride * DEC_D;
    a.len_arr = lens;
    a.len_max = T_k_stride;
    run_attn(a);
}

extern "C" void backend_sdp_attn_batch_decode_sa(float *out, const float *Q, const float *K, const float *V,
                                                 int T_k_stride, int B, float *work) {
    (void)work;
    sdp_batch(out, Q, K, V, T_k_stride, B, t.d_S_batch);
}

extern "C" void backend_sdp_attn_batch_decode_ca(float *out, const float *Q, const float *K, const float *V,
                                                 int T_k_stride, int B, float *work) {
    (void)work;
    sdp_batch(out, Q, K, V, T_k_stride, B, t.d_T_enc);
}

// ============================================================ status =======
// Extension (not in the reference ABI): read and clear the device status word
// that bounded waits and index checks write instead of trapping.
extern "C" int ct_device_status(void) {
    require_init();
    int v = 0, zero = 0;
    CT_CHECK(cudaStreamSynchronize(t.st));
    CT_CHECK(cudaMemcpyFromSymbol(&v, g_ct_status, sizeof(int)));
    CT_CHECK(cudaMemcpyToSymbol(g_ct_status, &zero, sizeof(int)));
    return v;
}

// Extension (not in the reference ABI): one thread waits on an mbarrier phase
// that nothing completes, with a budget of limit_ns, through the bounded wait
// the pipelines use; it records `code` and returns when the budget runs out.
__global__ void selftest_wait_kernel(uint64_t limit_ns, int code, unsigned long long *elapsed_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_mbar_init();
    const uint64_t t0 = globaltimer();
    const bool arrived = mbar_wait_for(&bar, 0, code, limit_ns);
    *elapsed_ns = arrived ? 0ull : (unsigned long long)(globaltimer() - t0);
}

extern "C" int ct_selftest_bounded_wait(int limit_us, int code) {
    if (limit_us < 1 || limit_us > 1000000 || code < 1 || code > 255) return -1;
    unsigned long long *el = nullptr;
    if (cudaMallocHost(&el, sizeof(*el)) != cudaSuccess) return -4;
    *el = 0;
    int v = 0, zero = 0;
    cudaError_t e = cudaSuccess;
    selftest_wait_kernel<<<1, 32>>>((uint64_t)limit_us * 1000ull, code, el);
    if ((e = cudaGetLastError()) == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_ct_status, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_ct_status, &zero, sizeof(int));
    // the wait must have lasted its budget (the timer is checked every 256 polls)
    if (e == cudaSuccess && v == code && *el < (unsigned long long)limit_us * 1000ull) v = -4;
    cudaFreeHost(el);
    return e == cudaSuccess ? v : -4;
}

// Extension (not in the reference ABI): the library's tensor-core GEMM on
// caller-held bf16 activation planes; Y = act(X W^T + b), fp32 out.
extern "C" int ct_linear_bf16(float *Y, int ldy, const uint16_t *X_hi, const uint16_t *X_lo, const uint16_t *W,
                              const uint16_t *bias, int T, int K, int N, int act, void *stream) {
    if (!Y || !X_hi || !W || T <= 0 || N <= 0 || K <= 0 || (K & 7) || ldy < N || act < 0 || act > 2) return -1;
    if (((uintptr_t)X_hi | (uintptr_t)X_lo | (uintptr_t)W) & 15) return -1;
    GemmEpilogue ep;
    ep.epi = act == 1 ? EPI_SILU : act == 2 ? EPI_RELU : EPI_STORE;
    ep.bias = reinterpret_cast<const bf16 *>(bias);
    ep.Y = Y;
    ep.ldy = ldy;
    ep.x_rows = T;
    gemm_bf16(static_cast<cudaStream_t>(stream), reinterpret_cast<const bf16 *>(W), N, K,
              reinterpret_cast<const bf16 *>(X_hi), reinterpret_cast<const bf16 *>(X_lo), T, ep, false);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
