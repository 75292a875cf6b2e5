/* mel_harness.c -- exposes the REFERENCE log-mel front-end for the oracle's
 * pinning test.  TEST INFRASTRUCTURE: this translation unit includes the
 * reference's transcribe.c from the reference tree at build time (its
 * compute_mel, init_hann and init_mel_filterbank are file-static there), with
 * its main() renamed, and is linked with the reference CPU backend into
 * oracle/_ref/libref_mel.so by oracle/Makefile.  transcribe.c's embedded
 * vocabulary header is generated empty: the front-end does not use it. */
#define main ref_transcribe_main
#include "transcribe.c"
#undef main

/* samples: N mono 16 kHz floats -> mel [N_MELS][1 + N / HOP_LEN] */
void refmel_compute(const float *samples, int N, float *mel) {
    static int ready = 0;
    if (!ready) {
        init_hann();
        init_mel_filterbank();
        ready = 1;
    }
    const int T = 1 + N / HOP_LEN;
    float *work = malloc(sizeof(float) * ((size_t)N + WIN_LEN));
    compute_mel(samples, N, T, mel, work);
    free(work);
}

/* The reference's long-form split points (transcribe.c:484-507): frame RMS,
 * silence threshold (automatic when silence_db is NaN), silence midpoints,
 * merged to the target chunk length.  Writes at most max_out split sample
 * indices and returns how many there are. */
int refsplit(const float *samples, int n_samples, float silence_db, float silence_dur, float target_sec,
             int *splits_out, int max_out) {
    const int n_frames = n_samples / HOP_LEN;
    float *rms = malloc(sizeof(float) * (size_t)(n_frames > 0 ? n_frames : 1));
    compute_frame_rms(samples, n_frames, rms);
    const float thresh = isnan(silence_db) ? estimate_silence_thresh(rms, n_frames)
                                           : powf(10.0f, silence_db / 20.0f);
    int splits[4096];
    int n = find_splits(rms, n_frames, thresh, silence_dur, splits, 4096);
    free(rms);
    n = apply_target(splits, n, (int)(target_sec * SR));
    for (int i = 0; i < n && i < max_out; i++) splits_out[i] = splits[i];
    return n;
}
