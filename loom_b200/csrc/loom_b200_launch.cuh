// loom_b200_launch.cuh -- host-side launchers for the kernels in
// loom_b200_device.cuh, shared by every generated package.
//
// They replace the launch arithmetic of the reference's emitted wrapper
// (src/loom_backend_cuda/cuda_backend.ml:1828-2270 and the support helpers at
// :2344-2422): instead of fixed block-count caps (4096 / 32768 blocks of 256
// threads) and a host loop of combine launches, every kernel gets one CTA per
// tile (a reduction at most kMaxPartials CTAs, or fewer when the caller's
// scratch has fewer partial slots, and one wave of CTAs when its tiles fill
// one to three waves), and a reduction is one launch when its
// grid fits one thread-block cluster (at most 8 CTAs) and two otherwise.
//
// Nothing here allocates device memory and nothing holds device state; the
// only host state is a per-device cache of how many CTAs of each reduction
// kernel fit on the device at once.
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

// Number of CTA partial slots a reduction over n elements may use: one per
// smallest tile, at most kMaxPartials.  The workspace size and every
// workspace-backed reduction launch use this same bound.
inline int64_t partial_capacity(int64_t n) {
  int64_t c = ceil_div(n, kMinTileElems);
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

// The finalize CTA as a programmatic dependent launch of the kernel before
// it on the stream: the hardware may schedule it while that kernel still
// runs, and its griddepcontrol.wait holds it until that grid has completed.
// Where the attribute is refused, a plain launch gives the same result.
template <class Op>
inline int launch_finalize(const typename Op::Acc* partials, int count, float* out,
                           typename Op::Acc* partial_out, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kFinalizeThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, reduce_finalize_kernel<Op>, partials, count, out, partial_out) ==
      cudaSuccess)
    return LOOM_STATUS_OK;
  cudaGetLastError();
  reduce_finalize_kernel<Op><<<1, kFinalizeThreads, 0, stream>>>(partials, count, out,
                                                                  partial_out);
  return launch_status();
}

// A grid of 2..kMaxClusterCtas CTAs launched as one thread-block cluster:
// the CTAs fold their values through distributed shared memory, so the
// reduction needs no finalize launch.  It is launched without the
// programmatic-serialization attribute (its griddepcontrol.wait is then a
// no-op): with both attributes the small-N call measured a full finalize
// launch slower on B200.  Returns false (with the error
// cleared) where the cluster launch is refused; the caller then takes the
// two-launch path.
template <class Op, class Body, int U>
inline bool launch_cluster_reduce(unsigned grid, const Ptrs<Body::kInputs>& in, int64_t n,
                                  int64_t head, const Body& body, float* out,
                                  typename Op::Acc* partial_out, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = grid;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  typename Op::Acc* no_partials = nullptr;
  if (cudaLaunchKernelEx(&cfg, reduce_vec_kernel<Op, Body, U, true>, no_partials, in, n, head,
                         body, out, partial_out) == cudaSuccess)
    return true;
  cudaGetLastError();
  return false;
}

// Every streaming kernel is launched as a programmatic dependent of the
// kernel before it on the stream.  Each kernel first lets its own dependent
// be scheduled (griddepcontrol.launch_dependents) and then waits for its
// prerequisite grid to complete and flush (griddepcontrol.wait) before it
// touches global memory, so stream order is kept; what is gained is that the
// next kernel's first CTAs are already resident when this one ends.  After
// a kernel that does not trigger (a library kernel, a copy) the launch simply
// waits for it.  Where the attribute is refused, a plain launch is made.
template <class Kern, class... Args>
inline void launch_pdl(Kern kernel, unsigned grid, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess) return;
  cudaGetLastError();
  kernel<<<grid, kThreads, 0, stream>>>(args...);
}

inline unsigned clamp_grid(int64_t g, int64_t cap) {
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

// A reduction whose tiles fill more than one but at most kBalanceWaves waves
// of resident CTAs runs as one wave: ceil(tiles / wave) tiles per CTA, so
// every CTA walks the same number of tiles and no ragged second wave runs
// while most SMs idle (measured on a B200: pipeline_sum at 2^22 elements
// 15.4 against 17.4 us a call, dot 7.2 against 8.0 us replayed from a graph;
// no change from 2^26 up, where the grid is many waves deep).  `wave` <= 0
// (unknown) leaves the grid as it is.
constexpr int64_t kBalanceWaves = 3;

inline int64_t balanced_grid(int64_t tiles, int64_t wave) {
  if (wave <= 0 || tiles <= wave || tiles > kBalanceWaves * wave) return tiles;
  const int64_t per_cta = ceil_div(tiles, wave);
  return ceil_div(tiles, per_cta);
}

// CTAs of reduce_vec_kernel<Op, Body, U> (kThreads threads, no dynamic
// shared memory) that the current device holds at once, looked up once per
// device (kMaxDevices of them); 0 when the runtime cannot say.
template <class Op, class Body, int U>
inline int64_t reduce_wave() {
  static std::atomic<int64_t> cache[kMaxDevices];
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return 0;
  }
  int64_t wave = cache[dev].load(std::memory_order_relaxed);
  if (wave > 0) return wave;
  int sms = 0, per_sm = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, reduce_vec_kernel<Op, Body, U>,
                                                    kThreads, 0) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  wave = (int64_t)sms * per_sm;
  cache[dev].store(wave, std::memory_order_relaxed);
  return wave;
}

// out[i] = body(in[0][i], ...) for i in [0, n).
template <class Body>
inline int launch_map(float* out, const Ptrs<Body::kInputs>& in, int64_t n, const Body& body,
                      cudaStream_t stream) {
  if (n <= 0) return LOOM_STATUS_OK;
  if (!pointers_aligned4(in, out)) return LOOM_STATUS_INVALID_ARGUMENT;
  if (congruent16(in, out)) {
    constexpr int U = MapUnroll<Body::kInputs>::value;
    const int64_t head = head_elems(out, n);
    const int64_t nvec = (n - head) >> 2;
    const int64_t tiles = ceil_div(nvec, (int64_t)kThreads * U);
    if (tiles > kMaxGrid) return LOOM_STATUS_INVALID_ARGUMENT;  // > 2^40 elements: no such GPU
    const unsigned grid = clamp_grid(tiles, kMaxGrid);
    launch_pdl(map_vec_kernel<Body, U>, grid, stream, out, in, n, head, body);
  } else {
    const unsigned grid = clamp_grid(ceil_div(n, (int64_t)kThreads * kScalarUnroll), kMaxGrid);
    launch_pdl(map_scalar_kernel<Body>, grid, stream, out, in, n, body);
  }
  return launch_status();
}

// The first stage of a reduction of body(in[...][i]) over [0, n) with Op.
// `partials` must hold `max_partials` slots (at least 1); the kernel uses at
// most that many CTAs.  On return *pending is the number of CTA partials left
// in `partials` for a finalize to fold, or 0 when the stage already wrote
// the result to out[0] (fp32) and/or partial_out[0] (Op::Acc): a one-CTA
// grid, or a grid of at most kMaxClusterCtas launched as one cluster.
template <class Op, class Body>
inline int launch_reduce_stage(const Ptrs<Body::kInputs>& in, int64_t n, const Body& body,
                               typename Op::Acc* partials, int64_t max_partials, float* out,
                               typename Op::Acc* partial_out, cudaStream_t stream,
                               unsigned* pending) {
  *pending = 0;
  if (n <= 0 || max_partials < 1) return LOOM_STATUS_INVALID_ARGUMENT;
  if (!pointers_aligned4(in, nullptr)) return LOOM_STATUS_INVALID_ARGUMENT;
  unsigned grid;
  if (congruent16(in, in.p[0])) {
    constexpr int U = ReduceUnroll<Body::kInputs>::value;
    const int64_t head = head_elems(in.p[0], n);
    const int64_t nvec = (n - head) >> 2;
    int64_t tiles = ceil_div(nvec, (int64_t)kThreads * U);
    if (tiles > kMaxClusterCtas) tiles = balanced_grid(tiles, reduce_wave<Op, Body, U>());
    grid = clamp_grid(tiles, max_partials);
    if (grid > 1 && grid <= (unsigned)kMaxClusterCtas &&
        launch_cluster_reduce<Op, Body, U>(grid, in, n, head, body, out, partial_out, stream))
      return LOOM_STATUS_OK;
    launch_pdl(reduce_vec_kernel<Op, Body, U>, grid, stream, partials, in, n, head, body, out,
               partial_out);
  } else {
    grid = clamp_grid(ceil_div(n, (int64_t)kThreads * kScalarUnroll), max_partials);
    reduce_scalar_kernel<Op, Body><<<grid, kThreads, 0, stream>>>(partials, in, n, body, out,
                                                                  partial_out);
  }
  const int st = launch_status();
  if (st == LOOM_STATUS_OK && grid > 1) *pending = grid;  // one CTA wrote the result itself
  return st;
}

// Reduces body(in[...][i]) over [0, n) with Op into out[0] (fp32) and/or
// partial_out[0] (Op::Acc): the first stage, then the finalize CTA where
// partials are left.
template <class Op, class Body>
inline int launch_reduce(const Ptrs<Body::kInputs>& in, int64_t n, const Body& body,
                         typename Op::Acc* partials, int64_t max_partials, float* out,
                         typename Op::Acc* partial_out, cudaStream_t stream) {
  unsigned pending = 0;
  const int st = launch_reduce_stage<Op>(in, n, body, partials, max_partials, out, partial_out,
                                         stream, &pending);
  if (st != LOOM_STATUS_OK || pending == 0) return st;
  return launch_finalize<Op>(partials, (int)pending, out, partial_out, stream);
}

// Blocks until the device is idle, mapping the result to a status code (the
// reference wrappers end the same way unless built with
// cuda-async-wrapper-return).
inline int finish_sync() {
  return cudaDeviceSynchronize() == cudaSuccess ? LOOM_STATUS_OK : LOOM_STATUS_CUDA_ERROR;
}

}  // namespace loomb
