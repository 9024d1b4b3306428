/* A plain C (C11) caller of a generated Loom B200 package, as any C program
 * would use the drop-in ABI: the generated header, caller-owned device
 * buffers, a workspace sized by <entry>_workspace_size, status codes.
 * Prints "abi_smoke ok" and exits 0 when saxpy and dot agree with a host
 * computation (saxpy with fmaf, bit for bit; dot to 1e-5 relative). */
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

#include "loom/b200_suite.h"

#define N 100003

static int check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
    return 1;
  }
  return 0;
}

int main(void) {
  float* hx = (float*)malloc(N * sizeof(float));
  float* hy = (float*)malloc(N * sizeof(float));
  float* ho = (float*)malloc(N * sizeof(float));
  unsigned s = 12345u;
  for (int i = 0; i < N; ++i) {
    s = s * 1664525u + 1013904223u;
    hx[i] = (float)(s >> 8) / 16777216.0f * 2.0f - 1.0f;
    s = s * 1664525u + 1013904223u;
    hy[i] = (float)(s >> 8) / 16777216.0f * 2.0f - 1.0f;
  }
  float *dx, *dy, *dout, *dscalar;
  void* ws;
  size_t ws_size = loom_kernels_dot_workspace_size(N);
  if (check(cudaMalloc((void**)&dx, N * sizeof(float)), "malloc x") ||
      check(cudaMalloc((void**)&dy, N * sizeof(float)), "malloc y") ||
      check(cudaMalloc((void**)&dout, N * sizeof(float)), "malloc out") ||
      check(cudaMalloc((void**)&dscalar, sizeof(float)), "malloc scalar") ||
      check(cudaMalloc(&ws, ws_size), "malloc workspace") ||
      check(cudaMemcpy(dx, hx, N * sizeof(float), cudaMemcpyHostToDevice), "copy x") ||
      check(cudaMemcpy(dy, hy, N * sizeof(float), cudaMemcpyHostToDevice), "copy y"))
    return 1;
  if (loom_kernels_saxpy_workspace_size(N) != 0) return 2;
  int st = loom_kernels_saxpy(2.5f, dx, dy, N, dout, NULL, 0);
  if (st != LOOM_STATUS_OK) {
    fprintf(stderr, "saxpy status %d\n", st);
    return 3;
  }
  if (check(cudaMemcpy(ho, dout, N * sizeof(float), cudaMemcpyDeviceToHost), "copy out")) return 1;
  for (int i = 0; i < N; ++i) {
    if (ho[i] != fmaf(2.5f, hx[i], hy[i])) {
      fprintf(stderr, "saxpy mismatch at %d\n", i);
      return 4;
    }
  }
  if (loom_kernels_dot(dx, dy, N, dscalar, ws, 8) != LOOM_STATUS_WORKSPACE_TOO_SMALL) return 5;
  st = loom_kernels_dot(dx, dy, N, dscalar, ws, ws_size);
  if (st != LOOM_STATUS_OK) {
    fprintf(stderr, "dot status %d\n", st);
    return 6;
  }
  float got;
  if (check(cudaMemcpy(&got, dscalar, sizeof(float), cudaMemcpyDeviceToHost), "copy dot")) return 1;
  double ref = 0.0;
  for (int i = 0; i < N; ++i) ref += (double)hx[i] * (double)hy[i];
  if (fabs((double)got - ref) > 1e-5 * fabs(ref) + 1e-3) {
    fprintf(stderr, "dot %.9g vs %.9g\n", got, ref);
    return 7;
  }
  printf("abi_smoke ok\n");
  return 0;
}
