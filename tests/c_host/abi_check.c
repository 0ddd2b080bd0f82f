/* A plain C host of the C ABI (include/pace_b200.h), built and run by
 * tests/test_c_host.py.
 *
 *   abi_check cpu   argument errors, status strings, per-call error messages:
 *                   no device is touched
 *   abi_check gpu   silu_and_mul (fp32) against a double-precision host
 *                   computation, and a KV block gather byte-exact, on device 0
 *
 * Exit status 0 on success; the failing check is printed otherwise. */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "pace_b200.h"

static int failures = 0;
#define CHECK(cond, ...)                                 \
  do {                                                   \
    if (!(cond)) {                                       \
      fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
      fprintf(stderr, __VA_ARGS__);                      \
      fprintf(stderr, "\n");                             \
      ++failures;                                        \
    }                                                    \
  } while (0)

static int cpu_checks(void) {
  CHECK(pace_version() > 0, "version %d", pace_version());
  CHECK(strcmp(pace_status_string(PACE_OK), "PACE_OK") == 0, "status string");
  int rc = pace_rms_norm(NULL, NULL, NULL, 1e-5f, -1, 8, 8, 8, PACE_BF16, NULL);
  CHECK(rc == PACE_ERR_INVALID_ARGUMENT, "rms_norm bad shape rc=%d", rc);
  CHECK(strstr(pace_last_error(), "rms_norm") != NULL, "message: %s", pace_last_error());
  rc = pace_silu_and_mul(NULL, NULL, 4, 8, 8, 8, PACE_BF16, NULL);
  CHECK(rc == PACE_ERR_INVALID_ARGUMENT, "silu row stride rc=%d", rc);
  rc = pace_topk_softmax(NULL, NULL, NULL, NULL, 4, 2048, 2, 0, NULL);
  CHECK(rc == PACE_ERR_TOO_LARGE, "topk E=2048 rc=%d", rc);
  rc = pace_rms_norm(NULL, NULL, NULL, 1e-5f, 0, 8, 8, 8, PACE_BF16, NULL);
  CHECK(rc == PACE_OK, "zero tokens is a no-op, rc=%d", rc);
  return failures;
}

static int gpu_checks(void) {
  const int T = 3, d = 1000;
  float* hx = (float*)malloc(sizeof(float) * T * 2 * d);
  float* hy = (float*)malloc(sizeof(float) * T * d);
  for (int i = 0; i < T * 2 * d; ++i) hx[i] = (float)sin(0.37 * i) * 4.0f;
  float *dx = NULL, *dy = NULL;
  CHECK(cudaMalloc((void**)&dx, sizeof(float) * T * 2 * d) == cudaSuccess, "cudaMalloc x");
  CHECK(cudaMalloc((void**)&dy, sizeof(float) * T * d) == cudaSuccess, "cudaMalloc y");
  if (failures) return failures;
  cudaMemcpy(dx, hx, sizeof(float) * T * 2 * d, cudaMemcpyHostToDevice);
  int rc = pace_silu_and_mul(dy, dx, T, d, 2 * d, d, PACE_F32, NULL);
  CHECK(rc == PACE_OK, "silu_and_mul rc=%d: %s", rc, pace_last_error());
  CHECK(cudaDeviceSynchronize() == cudaSuccess, "sync");
  cudaMemcpy(hy, dy, sizeof(float) * T * d, cudaMemcpyDeviceToHost);
  double worst = 0.0, scale = 0.0;
  for (int t = 0; t < T; ++t)
    for (int j = 0; j < d; ++j) {
      const double a = hx[t * 2 * d + j], b = hx[t * 2 * d + d + j];
      const double want = a / (1.0 + exp(-a)) * b;
      const double err = fabs(hy[t * d + j] - want);
      if (err > worst) worst = err;
      if (fabs(want) > scale) scale = fabs(want);
    }
  CHECK(worst <= 1e-5 * scale, "silu_and_mul max error %g of %g", worst, scale);

  /* KV gather: 2 layers of 6 blocks of 64 bytes; blocks {4, 1, 5} of each layer */
  const int L = 2, nb = 6, bb = 64, n = 3;
  unsigned char host[2][6 * 64];
  for (int l = 0; l < L; ++l)
    for (int i = 0; i < nb * bb; ++i) host[l][i] = (unsigned char)(l * 131 + i * 7);
  void* layers[2];
  for (int l = 0; l < L; ++l) {
    cudaMalloc(&layers[l], nb * bb);
    cudaMemcpy(layers[l], host[l], nb * bb, cudaMemcpyHostToDevice);
  }
  const int32_t ids[3] = {4, 1, 5};
  int32_t* dids = NULL;
  void* dout = NULL;
  cudaMalloc((void**)&dids, sizeof(ids));
  cudaMalloc(&dout, L * n * bb);
  cudaMemcpy(dids, ids, sizeof(ids), cudaMemcpyHostToDevice);
  rc = pace_kv_gather_blocks(layers, L, dids, n, bb, nb, dout, NULL, NULL);
  CHECK(rc == PACE_OK, "gather rc=%d: %s", rc, pace_last_error());
  unsigned char got[2 * 3 * 64];
  CHECK(cudaMemcpy(got, dout, sizeof(got), cudaMemcpyDeviceToHost) == cudaSuccess, "copy back");
  for (int l = 0; l < L; ++l)
    for (int j = 0; j < n; ++j)
      CHECK(memcmp(got + (l * n + j) * bb, host[l] + ids[j] * bb, bb) == 0,
            "gathered block %d of layer %d differs", ids[j], l);
  for (int l = 0; l < L; ++l) cudaFree(layers[l]);
  cudaFree(dids);
  cudaFree(dout);
  cudaFree(dx);
  cudaFree(dy);
  free(hx);
  free(hy);
  return failures;
}

int main(int argc, char** argv) {
  if (argc < 2) {
    fprintf(stderr, "usage: %s cpu|gpu\n", argv[0]);
    return 2;
  }
  const int bad = strcmp(argv[1], "gpu") == 0 ? gpu_checks() : cpu_checks();
  if (!bad) printf("abi_check %s ok\n", argv[1]);
  return bad ? 1 : 0;
}
