/* Drives the R shim's core (jaxr_b200/r/jxrng_shim.c) through the call sequence its .Call
 * routines make -- key words from R doubles, then random_bits / uniform / normal /
 * bernoulli / split / fold_in with host results -- and writes each result to
 * <outdir>/<name>.bin for tests/test_r_shim.py to compare with the oracle.  Plain C,
 * linked to libjxrng.so and the CUDA runtime; needs a GPU. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "jxrng.h"
#include "jxrng_shim.h"

static const char* g_dir;

static void check(int rc, const char* what) {
  if (rc != JXR_OK) {
    fprintf(stderr, "%s failed (%d): %s\n", what, rc, jxs_error());
    exit(1);
  }
}

static void save(const char* name, const void* p, size_t bytes) {
  char path[4096];
  snprintf(path, sizeof path, "%s/%s.bin", g_dir, name);
  FILE* f = fopen(path, "wb");
  if (!f || fwrite(p, 1, bytes, f) != bytes) {
    fprintf(stderr, "cannot write %s\n", path);
    exit(1);
  }
  fclose(f);
}

int main(int argc, char** argv) {
  if (argc != 2) {
    fprintf(stderr, "usage: %s OUTDIR\n", argv[0]);
    return 2;
  }
  g_dir = argv[1];
  /* two keys as jaxR holds them: random_key(0L), random_key(42L) in x32 mode */
  const double words[4] = {0.0, 0.0, 0.0, 42.0};
  uint32_t keys[4];
  check(jxs_key_words(words, 4, keys), "jxs_key_words");
  uint64_t n = 0;
  check(jxs_count(1001.0, "size", &n), "jxs_count");
  const int64_t nk = 2;
  void* buf = malloc(8 * 2 * 1001 + 64);
  check(jxs_random_bits(keys, nk, n, 1, 32, buf), "bits u32");
  save("bits_p32", buf, 4 * 2 * n);
  check(jxs_random_bits(keys, nk, n, 0, 8, buf), "bits u8 original");
  save("bits_o8", buf, 2 * n);
  check(jxs_random_bits(keys, nk, n, 1, 64, buf), "bits u64");
  save("bits_p64", buf, 8 * 2 * n);
  check(jxs_uniform(keys, nk, n, 1, JXR_F32, -2.0, 3.0, buf), "uniform f32");
  save("unif_f32", buf, 4 * 2 * n);
  check(jxs_uniform(keys, nk, n, 0, JXR_F64, 0.0, 1.0, buf), "uniform f64 original");
  save("unif_o64", buf, 8 * 2 * n);
  check(jxs_uniform(keys, nk, n, 1, JXR_BF16, -1.0, 1.0, buf), "uniform bf16");
  save("unif_bf16", buf, 2 * 2 * n);
  check(jxs_normal(keys, nk, n, 1, JXR_F32, 0, buf), "normal f32");
  save("norm_f32", buf, 4 * 2 * n);
  check(jxs_normal(keys, nk, n, 1, JXR_F64, 0, buf), "normal f64");
  save("norm_f64", buf, 8 * 2 * n);
  check(jxs_normal(keys, nk, n, 1, JXR_F32, 1, buf), "normal f32 accurate");
  save("norm_f32_acc", buf, 4 * 2 * n);
  if (jxr_get_accurate_erf_inv() != 0) {
    fprintf(stderr, "the accurate erf_inv setting leaked out of the call\n");
    return 1;
  }
  check(jxs_bernoulli(keys, nk, n, 1, JXR_F32, 0.3, (uint8_t*)buf), "bernoulli");
  save("bern_f32", buf, 2 * n);
  check(jxs_split(keys, nk, 5, 1, (uint32_t*)buf), "split");
  save("split_p5", buf, 4 * 2 * 5 * 2);
  check(jxs_split(keys, nk, 3, 0, (uint32_t*)buf), "split original");
  save("split_o3", buf, 4 * 2 * 3 * 2);
  const uint32_t data[1] = {17};
  check(jxs_fold_in(keys, nk, data, 1, (uint32_t*)buf), "fold_in");
  save("fold_17", buf, 4 * 2 * 2);
  /* failures come back as statuses with a message, device buffers freed */
  if (jxs_uniform(keys, nk, n, 1, 9, 0.0, 1.0, buf) != JXR_ERR_INVALID_ARGUMENT ||
      strstr(jxs_error(), "dtype") == NULL) {
    fprintf(stderr, "bad dtype not rejected: %s\n", jxs_error());
    return 1;
  }
  if (jxs_normal(keys, nk, n, 7, JXR_F32, 0, buf) != JXR_ERR_INVALID_ARGUMENT ||
      strstr(jxs_error(), "layout") == NULL) {
    fprintf(stderr, "bad layout not rejected: %s\n", jxs_error());
    return 1;
  }
  free(buf);
  printf("R_SHIM_DRIVER_OK\n");
  return 0;
}
