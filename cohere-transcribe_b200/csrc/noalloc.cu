// noalloc.cu -- batched decode attention that allocates nothing.
//
// Some callers cannot call cudaMalloc: code that runs while a stream is being
// captured into a CUDA graph in global or thread-local mode (allocation calls
// are rejected there), callbacks and real-time threads that must not take the
// implicit device synchronisation cudaMalloc/cudaFree may perform, and hosts
// that hand this library a fixed memory budget up front.  For them this entry
// point keeps the split-KV partial results of the attention in a fixed-size
// array that is part of the library image (static __device__ storage), so a
// call allocates nothing; the caller passes every input and output buffer.
//
// The array holds CT_NOALLOC_ATTN_SCRATCH_FLOATS floats (2 MiB) on every GPU
// that loads the library, until the process exits.  All calls on a device share
// it: two calls that overlap on the GPU (different streams, or different host
// threads on the same device) race on it and must be serialised by the caller.
// Nothing in it has to start at zero: every partial a call reads was written
// earlier in the same call.
#include <mutex>

#include "../../include/ct_backend.h"
#include "kernels.cuh"

static __device__ __align__(256) float g_noalloc_attn_scratch[CT_NOALLOC_ATTN_SCRATCH_FLOATS];

namespace {
std::mutex g_noalloc_mu;
float *g_noalloc_dev_ptr[64];   // device address of the array, per device ordinal
}  // namespace

extern "C" int ct_sdp_attn_batch_decode_noalloc(float *out, const float *Q, const float *K, const float *V,
                                                const int *lens, int T_k_stride, int B, void *stream) {
    using namespace ct;
    if (!out || !Q || !K || !V || !lens || T_k_stride <= 0 || B <= 0) return CT_NOALLOC_EINVAL;
    if (attn_ws_floats(B, DEC_H, DEC_DK, T_k_stride) > (size_t)CT_NOALLOC_ATTN_SCRATCH_FLOATS)
        return CT_NOALLOC_ETOOBIG;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CT_NOALLOC_ECUDA;
    float *scratch = nullptr;
    {
        // one-time set-up per device, with that device current: the host-side
        // symbol is only a stand-in, the kernels need the device address
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_dev_ptr[dev]) {
            void *p = nullptr;
            if (cudaGetSymbolAddress(&p, g_noalloc_attn_scratch) != cudaSuccess || !p) return CT_NOALLOC_ECUDA;
            // With lazy module loading a kernel is loaded at its first launch,
            // which may allocate or synchronise; querying both kernels here
            // loads them now, so a later call (e.g. the first one long enough
            // to need the combine kernel) loads nothing.
            cudaFuncAttributes fa;
            if (cudaFuncGetAttributes(&fa, attn_chunk_kernel) != cudaSuccess ||
                cudaFuncGetAttributes(&fa, attn_combine_kernel) != cudaSuccess)
                return CT_NOALLOC_ECUDA;
            g_noalloc_dev_ptr[dev] = static_cast<float *>(p);
        }
        scratch = g_noalloc_dev_ptr[dev];
    }
    AttnRows a;
    a.Q = Q; a.ldq = DEC_D; a.K = K; a.V = V; a.kv_item = (long)T_k_stride * DEC_D; a.ldkv = DEC_D;
    a.len_arr = lens; a.len_dev = nullptr; a.len_const = 0; a.len_max = T_k_stride;
    a.mask = nullptr; a.mask_ld = 0; a.out = out; a.ldo = DEC_D;
    a.R = B; a.H = DEC_H; a.DK = DEC_DK; a.scale = 1.0f / sqrtf((float)DEC_DK);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // an error left pending by unrelated earlier work stays for its owner to
    // read; this call launches nothing and reports it
    if (cudaPeekAtLastError() != cudaSuccess) return CT_NOALLOC_ECUDA;
    const int nck = (T_k_stride + 127) / 128;
    attn_chunk_kernel<<<dim3(nck, DEC_H, B), 128, 0, st>>>(a, scratch, nck);
    if (cudaGetLastError() != cudaSuccess) return CT_NOALLOC_ECUDA;
    if (nck > 1) {
        attn_combine_kernel<<<dim3(B, DEC_H), 128, 0, st>>>(a, scratch, nck);
        if (cudaGetLastError() != cudaSuccess) return CT_NOALLOC_ECUDA;
    }
    return 0;
}
