// loom_b200_launch.cuh -- host-side launchers for the kernels in
// loom_b200_device.cuh, shared by every generated package.
//
// They replace the launch arithmetic of the reference's emitted wrapper
// (src/loom_backend_cuda/cuda_backend.ml:1828-2270 and the support helpers at
// :2344-2422): instead of fixed block-count caps (4096 / 32768 blocks of 256
// threads) and a host loop of combine launches, the grid is sized from the
// device's SM count times the resident CTAs per SM of the kernel actually
// launched, and a reduction is always exactly two launches.
//
// Nothing here allocates device memory and nothing holds device state: the
// caches below hold only device attributes and occupancy numbers.
#pragma once

#include <atomic>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "loom_b200_device.cuh"

#ifndef LOOM_STATUS_OK
#define LOOM_STATUS_OK 0
#define LOOM_STATUS_INVALID_ARGUMENT 1
#define LOOM_STATUS_WORKSPACE_TOO_SMALL 2
#define LOOM_STATUS_CUDA_ERROR 3
#endif

namespace loomb {

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Bytes of workspace region reserved after the CTA partials for the
// multi-GPU path: one local fp64 value at +0 and the rank gather at +64.
constexpr size_t kRankScratchBytes = 256;
constexpr int kMaxRanks = 24;

// Number of CTA partial slots a reduction over n elements may use.  The
// workspace size and every reduction launch use this same bound.
inline int64_t partial_capacity(int64_t n) {
  int64_t c = ceil_div(n, kTileElems);
  if (c < 1) c = 1;
  if (c > kMaxPartials) c = kMaxPartials;
  return c;
}

// Workspace layout, carved from the first 256-byte boundary at or after the
// caller's pointer (the trailing 256 bytes of slack make any base address
// fit): [0, P) CTA partials (fp64 slots), [P, P + kRankScratchBytes) rank
// scratch.
inline size_t rank_scratch_offset(int64_t n) {
  return align_up((size_t)partial_capacity(n) * sizeof(double), 256);
}

inline size_t reduce_workspace_bytes(int64_t n) {
  if (n <= 0) return 0;
  return rank_scratch_offset(n) + kRankScratchBytes + 256;
}

// First 256-byte boundary at or after `workspace`.
inline unsigned char* workspace_base(void* workspace) {
  return reinterpret_cast<unsigned char*>(align_up((size_t)(uintptr_t)workspace, 256));
}

inline int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

inline int sm_count(int dev) {
  static std::atomic<int> cache[kMaxDevices];
  if (dev < 0 || dev >= kMaxDevices) return 148;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
    cudaGetLastError();
    v = 148;
  }
  cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

// Resident CTAs per SM of `kernel` at kThreads threads, cached per device in
// the caller-provided slot array (one array per kernel instantiation).
template <class Kernel>
inline int resident_ctas(std::atomic<int>* cache, int dev, Kernel kernel) {
  if (dev < 0 || dev >= kMaxDevices) return 4;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kernel, kThreads, 0) != cudaSuccess ||
      v <= 0) {
    cudaGetLastError();
    v = 4;
  }
  cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

inline bool aligned4(const void* p) { return ((uintptr_t)p & 3u) == 0; }

template <int K>
inline bool pointers_aligned4(const Ptrs<K>& in, const void* out) {
  for (int k = 0; k < K; ++k)
    if (!aligned4(in.p[k])) return false;
  return out == nullptr || aligned4(out);
}

// True when every pointer has the same address mod 16 as `ref`.
template <int K>
inline bool congruent16(const Ptrs<K>& in, const void* ref) {
  const uintptr_t m = (uintptr_t)ref & 15u;
  for (int k = 0; k < K; ++k)
    if (((uintptr_t)in.p[k] & 15u) != m) return false;
  return true;
}

inline int64_t head_elems(const void* ref, int64_t n) {
  const int64_t h = (int64_t)((16u - ((uintptr_t)ref & 15u)) & 15u) >> 2;
  return h < n ? h : n;
}

inline int launch_status() {
  return cudaGetLastError() == cudaSuccess ? LOOM_STATUS_OK : LOOM_STATUS_CUDA_ERROR;
}

// out[i] = body(in[0][i], ...) for i in [0, n).
template <class Body>
inline int launch_map(float* out, const Ptrs<Body::kInputs>& in, int64_t n, const Body& body,
                      cudaStream_t stream) {
  static std::atomic<int> occ_vec[kMaxDevices];
  static std::atomic<int> occ_scalar[kMaxDevices];
  if (n <= 0) return LOOM_STATUS_OK;
  if (!pointers_aligned4(in, out)) return LOOM_STATUS_INVALID_ARGUMENT;
  const int dev = current_device();
  const int sms = sm_count(dev);
  if (congruent16(in, out)) {
    const int64_t head = head_elems(out, n);
    const int64_t nvec = (n - head) >> 2;
    const int64_t cap = (int64_t)sms * resident_ctas(occ_vec, dev, map_vec_kernel<Body>);
    int64_t grid = ceil_div(nvec, kTileVecs);
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    map_vec_kernel<Body><<<(unsigned)grid, kThreads, 0, stream>>>(out, in, n, head, body);
  } else {
    const int64_t cap = (int64_t)sms * resident_ctas(occ_scalar, dev, map_scalar_kernel<Body>);
    int64_t grid = ceil_div(n, (int64_t)kThreads * kUnroll * 4);
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    map_scalar_kernel<Body><<<(unsigned)grid, kThreads, 0, stream>>>(out, in, n, body);
  }
  return launch_status();
}

// Reduces body(in[...][i]) over [0, n) with Op into out[0] (fp32) and/or
// partial_out[0] (Op::Acc).  `partials` must hold partial_capacity(n) slots.
template <class Op, class Body>
inline int launch_reduce(const Ptrs<Body::kInputs>& in, int64_t n, const Body& body,
                         typename Op::Acc* partials, float* out,
                         typename Op::Acc* partial_out, cudaStream_t stream) {
  static std::atomic<int> occ_vec[kMaxDevices];
  static std::atomic<int> occ_scalar[kMaxDevices];
  if (n <= 0) return LOOM_STATUS_INVALID_ARGUMENT;
  if (!pointers_aligned4(in, nullptr)) return LOOM_STATUS_INVALID_ARGUMENT;
  const int dev = current_device();
  const int sms = sm_count(dev);
  const int64_t capacity = partial_capacity(n);
  int64_t grid;
  if (congruent16(in, in.p[0])) {
    const int64_t head = head_elems(in.p[0], n);
    const int64_t nvec = (n - head) >> 2;
    const int64_t cap = (int64_t)sms * resident_ctas(occ_vec, dev, reduce_vec_kernel<Op, Body>);
    grid = ceil_div(nvec, kTileVecs);
    if (grid > cap) grid = cap;
    if (grid > capacity) grid = capacity;
    if (grid < 1) grid = 1;
    reduce_vec_kernel<Op, Body><<<(unsigned)grid, kThreads, 0, stream>>>(partials, in, n, head, body);
  } else {
    const int64_t cap = (int64_t)sms * resident_ctas(occ_scalar, dev, reduce_scalar_kernel<Op, Body>);
    grid = ceil_div(n, (int64_t)kThreads * kUnroll * 4);
    if (grid > cap) grid = cap;
    if (grid > capacity) grid = capacity;
    if (grid < 1) grid = 1;
    reduce_scalar_kernel<Op, Body><<<(unsigned)grid, kThreads, 0, stream>>>(partials, in, n, body);
  }
  int st = launch_status();
  if (st != LOOM_STATUS_OK) return st;
  reduce_finalize_kernel<Op><<<1, kThreads, 0, stream>>>(partials, (int)grid, out, partial_out);
  return launch_status();
}

// Blocks until the device is idle, mapping the result to a status code (the
// reference wrappers end the same way unless built with
// cuda-async-wrapper-return).
inline int finish_sync() {
  return cudaDeviceSynchronize() == cudaSuccess ? LOOM_STATUS_OK : LOOM_STATUS_CUDA_ERROR;
}

}  // namespace loomb
