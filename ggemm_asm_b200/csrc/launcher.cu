// launcher.cu - standalone CUDA-event timing launcher for the variable-K grouped FP8 wgrad.
//
// Replaces the reference's HIP launcher (ggemm-asm launcher.cpp:1-192) with the same workload
// and output line: E=32 groups, M_total=131072 tokens split uniformly (launcher.cpp:99-102),
// every LHS/RHS byte 0x38 (launcher.cpp:106-107), scales 0.1 (launcher.cpp:110-112), warmup
// then `iters` back-to-back launches between two events (launcher.cpp:150-176), and
// "  Kernel:  <ms> ms  <TFLOPS> TFLOPS" with flops = 2*M_total*OUT_M*OUT_N (launcher.cpp:76,178).
// Unlike the reference it also checks the result: with e4m3fn 0x38 = 1.0 and e5m2 0x38 = 0.5,
// every C element of a group with K tokens is bf16(0.1f*0.1f*K*0.5).
//
// Usage: ggemm_vark_launcher [--site gate_up_wgrad|down_wgrad] [--warmup N] [--iters N]
//                            [--groups E] [--tokens M] [--path auto|tcgen05|simt]
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "ggemm_vark.h"

#define CK(x)                                                                          \
  do {                                                                                 \
    cudaError_t e_ = (x);                                                              \
    if (e_ != cudaSuccess) {                                                           \
      fprintf(stderr, "CUDA error %d: %s at %s:%d\n", (int)e_, cudaGetErrorString(e_), \
              __FILE__, __LINE__);                                                     \
      return 1;                                                                        \
    }                                                                                  \
  } while (0)

#define VK(x)                                                                                 \
  do {                                                                                        \
    int r_ = (x);                                                                             \
    if (r_ != GGEMM_VARK_OK) {                                                                \
      fprintf(stderr, "ggemm_vark error %d: %s (cuda %d) at %s:%d\n", r_, ggemm_vark_strerror(r_), \
              ggemm_vark_last_cuda_error(), __FILE__, __LINE__);                              \
      return 1;                                                                               \
    }                                                                                         \
  } while (0)

int main(int argc, char** argv) {
  int warmup = 20, iters = 100, E = 32, M_TOTAL = 131072;
  const char* site = "gate_up_wgrad";
  const char* path = "auto";
  for (int i = 1; i < argc; i++) {
    if (!strcmp(argv[i], "--warmup") && i + 1 < argc) warmup = atoi(argv[++i]);
    else if (!strcmp(argv[i], "--iters") && i + 1 < argc) iters = atoi(argv[++i]);
    else if (!strcmp(argv[i], "--site") && i + 1 < argc) site = argv[++i];
    else if (!strcmp(argv[i], "--groups") && i + 1 < argc) E = atoi(argv[++i]);
    else if (!strcmp(argv[i], "--tokens") && i + 1 < argc) M_TOTAL = atoi(argv[++i]);
    else if (!strcmp(argv[i], "--path") && i + 1 < argc) path = argv[++i];
    else {
      fprintf(stderr, "unknown argument %s\n", argv[i]);
      return 1;
    }
  }
  int OUT_M, OUT_N;
  if (!strcmp(site, "gate_up_wgrad")) {
    OUT_M = 2880;
    OUT_N = 5760;
  } else if (!strcmp(site, "down_wgrad")) {
    OUT_M = 2880;
    OUT_N = 2880;
  } else {
    fprintf(stderr, "Unknown site: %s\n", site);
    return 1;
  }
  int path_id = GGEMM_VARK_PATH_AUTO;
  if (!strcmp(path, "tcgen05")) path_id = GGEMM_VARK_PATH_TCGEN05;
  else if (!strcmp(path, "simt")) path_id = GGEMM_VARK_PATH_SIMT;

  const double flops = 2.0 * M_TOTAL * (double)OUT_M * OUT_N;
  cudaDeviceProp props;
  CK(cudaGetDeviceProperties(&props, 0));
  printf("GPU: %s (%d SMs)\n", props.name, props.multiProcessorCount);
  printf("Site: %s  E=%d M=%d OUT_M=%d OUT_N=%d  path=%s\n", site, E, M_TOTAL, OUT_M, OUT_N, path);
  printf("Warmup: %d  Iters: %d\n", warmup, iters);

  void *d_lhs, *d_rhs, *d_out, *d_ls, *d_rs, *d_offs;
  CK(cudaMalloc(&d_lhs, (size_t)M_TOTAL * OUT_M));
  CK(cudaMalloc(&d_rhs, (size_t)M_TOTAL * OUT_N));
  CK(cudaMalloc(&d_out, (size_t)E * OUT_M * OUT_N * 2));
  CK(cudaMalloc(&d_ls, 4));
  CK(cudaMalloc(&d_rs, 4));
  CK(cudaMalloc(&d_offs, (E + 1) * 8));
  std::vector<int64_t> offs(E + 1);
  for (int i = 0; i <= E; i++) offs[i] = (int64_t)M_TOTAL * i / E;
  CK(cudaMemcpy(d_offs, offs.data(), (E + 1) * 8, cudaMemcpyHostToDevice));
  CK(cudaMemset(d_lhs, 0x38, (size_t)M_TOTAL * OUT_M));
  CK(cudaMemset(d_rhs, 0x38, (size_t)M_TOTAL * OUT_N));
  CK(cudaMemset(d_out, 0, (size_t)E * OUT_M * OUT_N * 2));
  const float scale = 0.1f;
  CK(cudaMemcpy(d_ls, &scale, 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(d_rs, &scale, 4, cudaMemcpyHostToDevice));

  auto launch = [&]() {
    return ggemm_vark_fp8_wgrad_ex(d_lhs, d_rhs, d_out, (const float*)d_ls, (const float*)d_rs,
                                   (const int64_t*)d_offs, E, OUT_M, OUT_N, OUT_M, OUT_N,
                                   OUT_M * OUT_N, OUT_N, 1, M_TOTAL, 0, path_id, nullptr, 0,
                                   nullptr);
  };
  for (int i = 0; i < warmup; i++) VK(launch());
  CK(cudaDeviceSynchronize());

  cudaEvent_t start, stop;
  CK(cudaEventCreate(&start));
  CK(cudaEventCreate(&stop));
  CK(cudaEventRecord(start, nullptr));
  for (int i = 0; i < iters; i++) VK(launch());
  CK(cudaEventRecord(stop, nullptr));
  CK(cudaEventSynchronize(stop));
  float total_ms = 0;
  CK(cudaEventElapsedTime(&total_ms, start, stop));
  const double avg_ms = total_ms / iters;
  printf("  Kernel:  %.3f ms  %.1f TFLOPS\n", avg_ms, flops / (avg_ms * 1e-3) / 1e12);

  // Closed-form check of every group's first and last element.
  uint32_t bits = 0;
  VK(ggemm_vark_read_status(nullptr, 1, &bits));
  int bad = 0;
  for (int g = 0; g < E; ++g) {
    const int64_t K = offs[g + 1] - offs[g];
    const float expect = __bfloat162float(__float2bfloat16_rn((float)(K * 0.5) * (scale * scale)));
    for (int which = 0; which < 2; ++which) {
      const size_t idx = (size_t)g * OUT_M * OUT_N + (which ? (size_t)OUT_M * OUT_N - 1 : 0);
      __nv_bfloat16 v;
      CK(cudaMemcpy(&v, (char*)d_out + 2 * idx, 2, cudaMemcpyDeviceToHost));
      if (__bfloat162float(v) != expect) {
        if (bad < 4) fprintf(stderr, "group %d elem %zu: got %g expected %g\n", g, idx, __bfloat162float(v), expect);
        ++bad;
      }
    }
  }
  printf("  Check:   %s (device status 0x%x)\n", bad == 0 && bits == 0 ? "PASS" : "FAIL", bits);

  CK(cudaEventDestroy(start));
  CK(cudaEventDestroy(stop));
  CK(cudaFree(d_lhs));
  CK(cudaFree(d_rhs));
  CK(cudaFree(d_out));
  CK(cudaFree(d_ls));
  CK(cudaFree(d_rs));
  CK(cudaFree(d_offs));
  return bad == 0 && bits == 0 ? 0 : 2;
}
