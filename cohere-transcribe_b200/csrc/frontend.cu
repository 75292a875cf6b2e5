// frontend.cu -- log-mel front-end on the GPU (transcribe.c:45-123, :177-214).
//
// 16 kHz mono samples of a batch of utterances -> the normalised log-mel that
// the packed encoder reads: utterance b at mel + mel_off[b], [N_MELS][T_mel[b]],
// T_mel = 1 + N / 160.  Per frame: zero padding of WIN/2 samples on both sides,
// pre-emphasis s[i] - 0.97 s[i-1], symmetric Hann window of 400 points,
// 512-point power spectrum, Slaney mel filterbank (128 filters, area-normalised),
// log(x + 2^-24); then per (utterance, mel bin) normalisation over time with the
// unbiased variance and eps 1e-5.
//
// mel_power_kernel: one warp per frame.  The windowed frame is written into
// shared memory in bit-reversed order, so the radix-2 FFT runs its 9
// butterfly stages in place with a twiddle table (exact cos/sin, computed once
// on the host); the mel projection sums each filter over its nonzero bins only,
// in ascending bin order (the zero weights the reference also adds leave its
// sums unchanged).  mel_norm_kernel: one warp per (utterance, mel bin).
#include <math.h>
#include <vector>

#include "ct_common.cuh"

namespace ct {
namespace fe {

constexpr int NFFT = 512, WIN = 400, HOP = 160, NM = N_MELS, NB = NFFT / 2 + 1, SR = 16000;
constexpr int FW = 8;   // frames (warps) per CTA
// Shared-memory index of FFT element x with one padding float per 32: the
// bit-reversed stores and the power-of-two butterfly strides then fall in
// different banks (the values and the arithmetic are unchanged).
__device__ __forceinline__ int fpad(int x) { return x + (x >> 5); }
constexpr int NFFT_P = NFFT + NFFT / 32;

struct Front {
    float *hann = nullptr, *twr = nullptr, *twi = nullptr, *fb = nullptr;
    int *fb_lo = nullptr, *fb_hi = nullptr;   // nonzero bin range [lo, hi) of each filter
    float *samples = nullptr;
    size_t samples_cap = 0;
    int *tab = nullptr;                       // n_samp[n] samp_off[n] frame_off[n+1] mel_off[n] frame_utt[F]
    size_t tab_cap = 0;
    int max_utts = 0, max_frames = 0;
    std::vector<int> htab;
    std::vector<void *> owned;
};

__global__ void __launch_bounds__(FW * 32) mel_power_kernel(const float *samples, const int *tab, int n, int F,
                                                            const float *hann, const float *twr, const float *twi,
                                                            const float *fb, const int *fb_lo, const int *fb_hi,
                                                            float *mel) {
    __shared__ float re_s[FW][NFFT_P], im_s[FW][NFFT_P];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int f = blockIdx.x * FW + warp;
    if (f >= F) return;
    const int *n_samp = tab, *samp_off = tab + n, *frame_off = tab + 2 * n, *mel_off = tab + 3 * n + 1;
    const int *frame_utt = tab + 4 * n + 1;
    const int u = frame_utt[f];
    const int t = f - frame_off[u], T = frame_off[u + 1] - frame_off[u];
    const int N = n_samp[u], Np = N + WIN;   // padded length
    const float *x = samples + samp_off[u];
    float *re = re_s[warp], *im = im_s[warp];
    // padded sample j (0 <= j < Np) is x[j - WIN/2] inside the signal, else 0;
    // pre-emphasised s[j] = xp[j] - 0.97 xp[j-1] (s[0] = xp[0])
    auto xp = [&](int j) { return (j >= WIN / 2 && j < N + WIN / 2) ? x[j - WIN / 2] : 0.0f; };
    for (int i = lane; i < NFFT; i += 32) {
        float v = 0.0f;
        const int j = t * HOP + i;
        if (i < WIN && j < Np) {
            const float sj = j > 0 ? xp(j) - 0.97f * xp(j - 1) : xp(0);
            v = sj * hann[i];
        }
        const int r = __brev(i) >> (32 - 9);   // 9-bit bit reversal
        re[fpad(r)] = v;
        im[fpad(r)] = 0.0f;
    }
    __syncwarp();
    for (int len = 2; len <= NFFT; len <<= 1) {
        const int half = len >> 1, step = NFFT / len;
        for (int bidx = lane; bidx < NFFT / 2; bidx += 32) {
            const int grp = bidx / half, pos = bidx - grp * half;
            const int a = fpad(grp * len + pos), c = fpad(grp * len + pos + half);
            const float wr = twr[pos * step], wi = twi[pos * step];
            const float vr = re[c] * wr - im[c] * wi;
            const float vi = re[c] * wi + im[c] * wr;
            const float ur = re[a], ui = im[a];
            re[a] = ur + vr; im[a] = ui + vi;
            re[c] = ur - vr; im[c] = ui - vi;
        }
        __syncwarp();
    }
    for (int k = lane; k < NB; k += 32) {   // power spectrum
        const float r = re[fpad(k)], i = im[fpad(k)];
        im[fpad(k)] = r * r + i * i;
    }
    __syncwarp();
    const float guard = 5.9604644775390625e-08f;   // 2^-24
    for (int m = lane; m < NM; m += 32) {
        float v = 0.0f;
        for (int k = fb_lo[m]; k < fb_hi[m]; ++k) v += fb[m * NB + k] * im[fpad(k)];
        mel[mel_off[u] + (size_t)m * T + t] = logf(v + guard);
    }
}

__global__ void __launch_bounds__(256) mel_norm_kernel(const int *tab, int n, float *mel) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wid = blockIdx.x * 8 + warp;
    if (wid >= n * NM) return;
    const int u = wid / NM, m = wid % NM;
    const int *frame_off = tab + 2 * n, *mel_off = tab + 3 * n + 1;
    const int T = frame_off[u + 1] - frame_off[u];
    float *row = mel + mel_off[u] + (size_t)m * T;
    float s = 0.0f;
    for (int t = lane; t < T; t += 32) s += row[t];
    const float mean = warp_sum(s) / T;
    float v = 0.0f;
    for (int t = lane; t < T; t += 32) { const float d = row[t] - mean; v += d * d; }
    const float var = warp_sum(v) / (T - 1);
    const float inv = 1.0f / sqrtf(var + 1e-5f);
    for (int t = lane; t < T; t += 32) row[t] = (row[t] - mean) * inv;
}

// ---------------------------------------------------------------- host ------
static double fe_hz_to_mel(double f) {
    const double f_sp = 200.0 / 3.0, brk = 1000.0, step = log(6.4) / 27.0;
    return f < brk ? f / f_sp : brk / f_sp + log(f / brk) / step;
}
static double fe_mel_to_hz(double m) {
    const double f_sp = 200.0 / 3.0, brk = 1000.0, step = log(6.4) / 27.0;
    return m < brk / f_sp ? f_sp * m : brk * exp(step * (m - brk / f_sp));
}

template <typename T>
static bool fe_alloc(Front &f, T **p, size_t n) {
    if (cudaMalloc(reinterpret_cast<void **>(p), sizeof(T) * (n ? n : 1)) != cudaSuccess) return false;
    f.owned.push_back(*p);
    return true;
}

// Tables (window, twiddles, filterbank) and buffers for batches of up to
// max_utts utterances and max_frames log-mel frames in total.
static bool front_alloc(Front &f, int max_utts, int max_frames) {
    f.max_utts = max_utts;
    f.max_frames = max_frames;
    f.samples_cap = (size_t)max_frames * HOP;
    f.tab_cap = (size_t)5 * max_utts + 2 + max_frames;
    if (!(fe_alloc(f, &f.hann, WIN) && fe_alloc(f, &f.twr, NFFT / 2) && fe_alloc(f, &f.twi, NFFT / 2) &&
          fe_alloc(f, &f.fb, (size_t)NM * NB) && fe_alloc(f, &f.fb_lo, NM) && fe_alloc(f, &f.fb_hi, NM) &&
          fe_alloc(f, &f.samples, f.samples_cap) && fe_alloc(f, &f.tab, f.tab_cap)))
        return false;
    std::vector<float> hann(WIN), twr(NFFT / 2), twi(NFFT / 2), fb((size_t)NM * NB);
    std::vector<int> lo(NM), hi(NM);
    for (int i = 0; i < WIN; ++i) hann[i] = 0.5f * (1.0f - cosf(2.0f * (float)M_PI * i / (WIN - 1)));
    for (int k = 0; k < NFFT / 2; ++k) {   // w^k = exp(-2 pi i k / 512)
        twr[k] = (float)cos(2.0 * M_PI * k / NFFT);
        twi[k] = (float)-sin(2.0 * M_PI * k / NFFT);
    }
    double pts[NM + 2], gap[NM + 1];
    const double mlo = fe_hz_to_mel(0.0), mhi = fe_hz_to_mel(SR / 2.0);
    for (int i = 0; i < NM + 2; ++i) pts[i] = fe_mel_to_hz(mlo + (mhi - mlo) * i / (NM + 1));
    for (int i = 0; i < NM + 1; ++i) gap[i] = pts[i + 1] - pts[i];
    for (int m = 0; m < NM; ++m) {
        const double norm = 2.0 / (pts[m + 2] - pts[m]);
        lo[m] = NB;
        hi[m] = 0;
        for (int k = 0; k < NB; ++k) {
            const double fr = (SR / 2.0) * k / (NB - 1);
            const double up = (fr - pts[m]) / gap[m], down = (pts[m + 2] - fr) / gap[m + 1];
            const double w = up < down ? up : down;
            fb[(size_t)m * NB + k] = (float)(w > 0.0 ? w * norm : 0.0);
            if (fb[(size_t)m * NB + k] != 0.0f) { lo[m] = std::min(lo[m], k); hi[m] = k + 1; }
        }
        if (hi[m] == 0) lo[m] = 0;
    }
    CT_CHECK(cudaMemcpy(f.hann, hann.data(), sizeof(float) * WIN, cudaMemcpyHostToDevice));
    CT_CHECK(cudaMemcpy(f.twr, twr.data(), sizeof(float) * NFFT / 2, cudaMemcpyHostToDevice));
    CT_CHECK(cudaMemcpy(f.twi, twi.data(), sizeof(float) * NFFT / 2, cudaMemcpyHostToDevice));
    CT_CHECK(cudaMemcpy(f.fb, fb.data(), sizeof(float) * fb.size(), cudaMemcpyHostToDevice));
    CT_CHECK(cudaMemcpy(f.fb_lo, lo.data(), sizeof(int) * NM, cudaMemcpyHostToDevice));
    CT_CHECK(cudaMemcpy(f.fb_hi, hi.data(), sizeof(int) * NM, cudaMemcpyHostToDevice));
    return true;
}

static void front_free(Front &f) {
    for (void *p : f.owned) cudaFree(p);
    f.owned.clear();
}

// Log-mel of n utterances (host samples) into mel_dev, packed as the encoder
// reads it; T_mel_out[b] = 1 + n_samples[b] / 160.  Every utterance needs at
// least 160 samples (2 frames: the normalisation divides by T_mel - 1).
// Returns false when the batch exceeds the capacity.
static bool log_mel(cudaStream_t s, Front &f, int n, const float *const *samples, const int *n_samples,
                    float *mel_dev, int *T_mel_out) {
    if (n <= 0 || n > f.max_utts) return false;
    std::vector<int> ns(n), so(n), fo(n + 1), mo(n);
    size_t tot_s = 0;
    int frames = 0;
    fo[0] = 0;
    for (int b = 0; b < n; ++b) {
        if (n_samples[b] < HOP || !samples[b]) return false;
        ns[b] = n_samples[b];
        so[b] = (int)tot_s;
        tot_s += (size_t)n_samples[b];
        const int T = 1 + n_samples[b] / HOP;
        T_mel_out[b] = T;
        mo[b] = frames * NM;
        frames += T;
        fo[b + 1] = frames;
    }
    if (frames > f.max_frames || tot_s > f.samples_cap || tot_s > (size_t)INT32_MAX) return false;
    std::vector<int> &h = f.htab;
    h.assign((size_t)4 * n + 1 + frames, 0);
    std::copy(ns.begin(), ns.end(), h.begin());
    std::copy(so.begin(), so.end(), h.begin() + n);
    std::copy(fo.begin(), fo.end(), h.begin() + 2 * n);
    std::copy(mo.begin(), mo.end(), h.begin() + 3 * n + 1);
    int *fu = h.data() + 4 * n + 1;
    for (int b = 0; b < n; ++b)
        for (int t = fo[b]; t < fo[b + 1]; ++t) fu[t] = b;
    CT_CHECK(cudaMemcpyAsync(f.tab, h.data(), sizeof(int) * h.size(), cudaMemcpyHostToDevice, s));
    for (int b = 0; b < n; ++b)   // host or device sources (the engine's job-ring mirror)
        CT_CHECK(cudaMemcpyAsync(f.samples + so[b], samples[b], sizeof(float) * ns[b], cudaMemcpyDefault, s));
    mel_power_kernel<<<(frames + FW - 1) / FW, FW * 32, 0, s>>>(f.samples, f.tab, n, frames, f.hann, f.twr, f.twi,
                                                                f.fb, f.fb_lo, f.fb_hi, mel_dev);
    mel_norm_kernel<<<(n * NM + 7) / 8, 256, 0, s>>>(f.tab, n, mel_dev);
    CT_CHECK(cudaGetLastError());
    return true;
}

}  // namespace fe
}  // namespace ct
