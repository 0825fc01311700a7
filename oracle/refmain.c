/* Standalone runner over the reference's model code (TEST INFRASTRUCTURE / CPU BASELINE
 * ONLY).
 *
 *   dcref forward WEIGHTS CONFIG MIX.f32 B C T OUT.f32      one forward, prints seconds
 *   dcref time    WEIGHTS CONFIG MIX.f32 B C T REPEATS      timed forwards, prints JSON
 *   dcref apply   WEIGHTS CONFIG MIX.f32 B C T OUT.f32 SHIFTS BATCH
 *                                                           dc_apply_model (overlap 0.25)
 *
 * MIX.f32 is raw little-endian float32 [B][C][T].  Built twice by oracle/Makefile: over the
 * reference's CPU backend (oracle/_ref/dcref, bench.py's CPU-baseline leg, one process per
 * host core) and over libdc_b200.so (oracle/_ref/abi/dcabi, the reference's model code on
 * the GPU through the backend.h ABI, run by the GPU tests). */
#include "util.h"

#include <stdio.h>
#include <stdlib.h>
#include <time.h>

int dcref_load(const char *weights, const char *config);
int dcref_forward_plain(const float *mix_h, int B, int C, int T, float *out);
int dcref_n_sources(void);
int dcref_apply(const float *mix_h, int B, int C, int T, float *out, int shifts, int split,
                float overlap, float transition_power, int batch_size, unsigned seed,
                int use_seed);

static double now_s(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double)ts.tv_sec + (double)ts.tv_nsec * 1e-9;
}

int main(int argc, char **argv) {
  if (argc < 8) {
    fprintf(stderr, "usage: dcref forward|time WEIGHTS CONFIG MIX.f32 B C T [OUT|REPEATS]\n");
    return 2;
  }
  const char *mode = argv[1];
  int B = atoi(argv[5]), C = atoi(argv[6]), T = atoi(argv[7]);
  size_t n = (size_t)B * C * T;
  float *mix = (float *)malloc(n * sizeof(float));
  FILE *f = fopen(argv[4], "rb");
  if (!f || fread(mix, sizeof(float), n, f) != n) {
    fprintf(stderr, "cannot read %s\n", argv[4]);
    return 1;
  }
  fclose(f);
  dcref_load(argv[2], argv[3]);
  int S = dcref_n_sources();
  float *out = (float *)malloc((size_t)B * S * C * T * sizeof(float) + 16);
  if (mode[0] == 'a') {
    if (argc < 11) {
      fprintf(stderr, "usage: dcref apply WEIGHTS CONFIG MIX.f32 B C T OUT SHIFTS BATCH\n");
      return 2;
    }
    double t0 = now_s();
    dcref_apply(mix, B, C, T, out, atoi(argv[9]), 1, 0.25f, 1.0f, atoi(argv[10]), 1, 0);
    double dt = now_s() - t0;
    FILE *o = fopen(argv[8], "wb");
    if (!o || fwrite(out, sizeof(float), (size_t)B * S * C * T, o) != (size_t)B * S * C * T) {
      fprintf(stderr, "cannot write %s\n", argv[8]);
      return 1;
    }
    fclose(o);
    printf("{\"seconds\": %.6f}\n", dt);
  } else if (mode[0] == 'f') {
    double t0 = now_s();
    int tout = dcref_forward_plain(mix, B, C, T, out);
    double dt = now_s() - t0;
    if (argc > 8) {
      FILE *o = fopen(argv[8], "wb");
      fwrite(out, sizeof(float), (size_t)B * S * C * tout, o);
      fclose(o);
    }
    printf("{\"seconds\": %.6f, \"tout\": %d}\n", dt, tout);
  } else {
    int reps = argc > 8 ? atoi(argv[8]) : 1;
    double best = 1e30, total = 0;
    printf("{\"times_s\": [");
    for (int r = 0; r < reps; r++) {
      double t0 = now_s();
      dcref_forward_plain(mix, B, C, T, out);
      double dt = now_s() - t0;
      total += dt;
      best = dt < best ? dt : best;
      printf("%s%.6f", r ? ", " : "", dt);
      fflush(stdout);
    }
    printf("], \"best_s\": %.6f, \"mean_s\": %.6f, \"repeats\": %d}\n", best, total / reps,
           reps);
  }
  free(out);
  free(mix);
  return 0;
}
