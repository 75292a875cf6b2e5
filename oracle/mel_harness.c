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
