// loom_b200_device.cuh -- hand-written sm_100a kernels behind every generated
// Loom entry point.
//
// Every Loom entry lowers to ONE streaming kernel (plus, for reductions, a
// one-CTA finalize).  The generated code only supplies a body functor: a
// struct with `static constexpr int kInputs` and
// `__device__ float operator()(const float* in) const`, which evaluates the
// whole fused element-wise DAG of the entry for one element from the values
// of its kInputs distinct tensor parameters.  Intermediates of a fused chain
// live in registers and never reach HBM.
//
// These kernels replace the reference's emitted templates
// (src/loom_backend_cuda/cuda_backend.ml:908-1627): the grid-stride scalar and
// float4 element-wise kernels, the first-stage reduction with its
// shared-memory or shuffle block reduce, and the multi-launch combine tree.
//
// Layout and strategy (B200):
//  * all tensors are 1D contiguous fp32 in HBM; when every pointer of a call
//    has the same address mod 16 the kernel peels a head of 0..3 elements,
//    streams the body as 128-bit float4 loads/stores (ld.global.cs /
//    st.global.cs: each byte is touched once, so it is marked evict-first)
//    and finishes a tail of 0..3 elements; otherwise it streams 32-bit
//    elements;
//  * one tile per CTA: a tile is kThreads x U float4 per input (U by the
//    number of inputs, so every thread keeps 1-4 independent 16-byte loads per
//    input in flight), and the grid has one CTA per tile, so the hardware
//    scheduler hands tiles to SMs as they free up.  Measured on B200 this
//    beats a persistent grid-stride loop (SM count x resident CTAs) by 13-16%
//    for maps and 3-4% for reductions: the static stride leaves the slowest
//    SMs with the tail.  Map kernels have no loop at all; reductions walk
//    whole tiles with a grid stride past kMaxPartials CTAs, and where the
//    launcher folds a grid of one to three waves into one balanced wave;
//  * reductions: sums convert every value to fp64 and accumulate in fp64
//    (a fixed tree per thread and tile, then a per-thread accumulator);
//    CTAs reduce with xor-shuffle butterflies and write one fp64 partial each to the caller's
//    workspace (at most kMaxPartials; past that CTAs take several tiles with
//    a grid stride); the finalize CTA sums the partials in a fixed order.
//    No float atomics anywhere: the result is bit-reproducible for a given
//    grid.  Max keeps fp32 fmaxf throughout (exact in any order).
#pragma once

#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <type_traits>

namespace loomb {

constexpr int kThreads = 256;            // threads per streaming CTA
constexpr int kFinalizeThreads = 1024;   // threads of the one-CTA finalize
constexpr int kScalarUnroll = 8;         // 32-bit elements per thread per tile (scalar path)
constexpr int kMaxPartials = 32768;      // upper bound on reduction CTAs (fp64 partial slots)
constexpr int64_t kMinTileElems = (int64_t)kThreads * 4;  // smallest tile of any kernel
constexpr int64_t kMaxGrid = (int64_t)1 << 30;
constexpr int kMaxDevices = 64;
constexpr int kMaxClusterCtas = 8;       // portable thread-block cluster size

// float4 loads per input per thread per tile (measured best on B200).
template <int K>
struct MapUnroll {
  static constexpr int value = K == 1 ? 2 : 1;
};
template <int K>
struct ReduceUnroll {
  static constexpr int value = K == 1 ? 4 : 2;
};

template <int K>
struct Ptrs {
  const float* p[K];
};

// ---------------------------------------------------------------------------
// streaming memory access

__device__ __forceinline__ float4 load_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ float load_stream(const float* p) { return __ldcs(p); }
__device__ __forceinline__ void store_stream(float4* p, const float4& v) { __stcs(p, v); }
__device__ __forceinline__ void store_stream(float* p, float v) { __stcs(p, v); }

// Programmatic dependent launch.  Every kernel here is launched as a
// programmatic dependent of the kernel before it on the stream.  It first
// lets its own dependent be scheduled (launch_dependents), then waits for
// its prerequisite grid to complete and its writes to become visible
// (wait) before it touches global memory.  Both are no-ops for a kernel
// launched without the attribute.
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void wait_for_prerequisite_grid() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <class Body>
__device__ __forceinline__ float4 apply4(const Body& body, const float4 (&v)[Body::kInputs]) {
  constexpr int K = Body::kInputs;
  float a[K];
  float4 r;
#pragma unroll
  for (int k = 0; k < K; ++k) a[k] = v[k].x;
  r.x = body(a);
#pragma unroll
  for (int k = 0; k < K; ++k) a[k] = v[k].y;
  r.y = body(a);
#pragma unroll
  for (int k = 0; k < K; ++k) a[k] = v[k].z;
  r.z = body(a);
#pragma unroll
  for (int k = 0; k < K; ++k) a[k] = v[k].w;
  r.w = body(a);
  return r;
}

template <class Body>
__device__ __forceinline__ float apply1(const Body& body, const Ptrs<Body::kInputs>& in, int64_t i) {
  constexpr int K = Body::kInputs;
  float a[K];
#pragma unroll
  for (int k = 0; k < K; ++k) a[k] = load_stream(in.p[k] + i);
  return body(a);
}

// ---------------------------------------------------------------------------
// element-wise map: out[i] = body(in_0[i], ..., in_{K-1}[i])

// Vector path, one tile of kThreads x U float4 per CTA and no loop (the grid
// covers every tile, which keeps the kernel at about 20 registers and the SMs
// at full occupancy).  Preconditions (checked by the host launcher): every
// pointer is 4-byte aligned and congruent to `out` mod 16; head = number of
// leading elements before the first 16-byte boundary (0..3, at most n); the
// grid is max(1, number of tiles).
template <class Body, int U>
__global__ void __launch_bounds__(kThreads)
map_vec_kernel(float* __restrict__ out, const Ptrs<Body::kInputs> in, const int64_t n,
               const int64_t head, const Body body) {
  allow_dependent_launch();
  wait_for_prerequisite_grid();
  constexpr int K = Body::kInputs;
  constexpr int kTile = kThreads * U;
  const int64_t nvec = (n - head) >> 2;
  const int64_t t = (int64_t)blockIdx.x * kTile;
  const int64_t left = nvec - t;
  const float4* src[K];
#pragma unroll
  for (int k = 0; k < K; ++k) src[k] = reinterpret_cast<const float4*>(in.p[k] + head) + t;
  float4* dst = reinterpret_cast<float4*>(out + head) + t;
  if (left >= kTile) {
    float4 v[U][K];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int k = 0; k < K; ++k) v[u][k] = load_stream(src[k] + u * kThreads + threadIdx.x);
#pragma unroll
    for (int u = 0; u < U; ++u) store_stream(dst + u * kThreads + threadIdx.x, apply4(body, v[u]));
  } else {
    const int rem = left > 0 ? (int)left : 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = u * kThreads + threadIdx.x;
      if (i < rem) {
        float4 v[K];
#pragma unroll
        for (int k = 0; k < K; ++k) v[k] = load_stream(src[k] + i);
        store_stream(dst + i, apply4(body, v));
      }
    }
  }
  if (blockIdx.x == gridDim.x - 1) {
    const int64_t tail0 = head + (nvec << 2);
    const int r = threadIdx.x;
    int64_t i = -1;
    if (r < head) i = r;
    else if (r >= 4 && (int64_t)(r - 4) < n - tail0) i = tail0 + (r - 4);
    if (i >= 0) store_stream(out + i, apply1(body, in, i));
  }
}

// Scalar path for calls whose pointers disagree mod 16.
template <class Body>
__global__ void __launch_bounds__(kThreads)
map_scalar_kernel(float* __restrict__ out, const Ptrs<Body::kInputs> in, const int64_t n,
                  const Body body) {
  allow_dependent_launch();
  wait_for_prerequisite_grid();
  constexpr int kU = kScalarUnroll;
  constexpr int64_t kTile = (int64_t)kThreads * kU;
  const int64_t stride = (int64_t)gridDim.x * kTile;
  for (int64_t t = (int64_t)blockIdx.x * kTile; t < n; t += stride) {
    if (t + kTile <= n) {
      float v[kU][Body::kInputs];
#pragma unroll
      for (int u = 0; u < kU; ++u)
#pragma unroll
        for (int k = 0; k < Body::kInputs; ++k)
          v[u][k] = load_stream(in.p[k] + t + u * kThreads + threadIdx.x);
#pragma unroll
      for (int u = 0; u < kU; ++u) store_stream(out + t + u * kThreads + threadIdx.x, body(v[u]));
    } else {
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = t + u * kThreads + threadIdx.x;
        if (i < n) store_stream(out + i, apply1(body, in, i));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// reductions

// A reduction op.  Acc is the per-thread and per-CTA accumulator; Chunk is
// what one thread folds a tile's values into before absorbing them.  Sums
// convert every fp32 value to fp64 and add in fp64 (pairwise inside a float4,
// then in a fixed tree over the tile), so the result is the fp64 sum of the
// fp32 values up to fp64 rounding, whatever the data's cancellation: the
// fp64 pipe (64 lanes per SM per clock on B200) and the f32->f64 conversions
// have several times the throughput an HBM-bound stream needs.  Max stays
// fp32 fmaxf, which is exact in any order.
struct SumOp {
  using Acc = double;
  using Chunk = double;
  static __device__ __forceinline__ double init() { return 0.0; }
  static __device__ __forceinline__ double chunk4(const float4& v) {
    return __dadd_rn(__dadd_rn((double)v.x, (double)v.y), __dadd_rn((double)v.z, (double)v.w));
  }
  static __device__ __forceinline__ double chunk2(double a, double b) { return __dadd_rn(a, b); }
  static __device__ __forceinline__ double absorb(double acc, double chunk) {
    return __dadd_rn(acc, chunk);
  }
  static __device__ __forceinline__ double combine(double a, double b) { return __dadd_rn(a, b); }
  static __device__ __forceinline__ float to_float(double a) { return __double2float_rn(a); }
};

struct MaxOp {
  using Acc = float;
  using Chunk = float;
  static __device__ __forceinline__ float init() { return -INFINITY; }
  static __device__ __forceinline__ float chunk4(const float4& v) {
    return fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
  }
  static __device__ __forceinline__ float chunk2(float a, float b) { return fmaxf(a, b); }
  static __device__ __forceinline__ float absorb(float acc, float chunk) { return fmaxf(acc, chunk); }
  static __device__ __forceinline__ float combine(float a, float b) { return fmaxf(a, b); }
  static __device__ __forceinline__ float to_float(float a) { return a; }
};

// Whether a body's values are never negative: the generated body says so
// (`kNonNegative`, for the square families x*x and (a-b)*(a-b)); a body
// without the member counts as signed.
template <class Body, class = void>
struct NonNegative {
  static constexpr bool value = false;
};
template <class Body>
struct NonNegative<Body, std::void_t<decltype(Body::kNonNegative)>> {
  static constexpr bool value = Body::kNonNegative;
};

// How one thread folds a tile's values before absorbing them into its
// accumulator: Op's own chunk type (fp64 for sums), except for sums of
// values that are never negative.  Those add their up to 16 values per tile
// in fp32 (a fixed tree at most 4 levels deep) and convert once: with no
// cancellation possible, each tile's sum errs by at most about 4 fp32 units
// in the last place of that sum, so the whole sum errs by at most about 4
// units of the total, 2.4e-7 relative, inside the 1e-6 * log2(N) bound for
// every N, and the per-value f32->f64 conversions are saved.
template <class Op, bool kNonNeg>
struct Chunking {
  using T = typename Op::Chunk;
  static __device__ __forceinline__ T chunk4(const float4& v) { return Op::chunk4(v); }
  static __device__ __forceinline__ T chunk2(T a, T b) { return Op::chunk2(a, b); }
  static __device__ __forceinline__ typename Op::Acc absorb(typename Op::Acc acc, T c) {
    return Op::absorb(acc, c);
  }
};
template <>
struct Chunking<SumOp, true> {
  using T = float;
  static __device__ __forceinline__ float chunk4(const float4& v) {
    return __fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w));
  }
  static __device__ __forceinline__ float chunk2(float a, float b) { return __fadd_rn(a, b); }
  static __device__ __forceinline__ double absorb(double acc, float c) {
    return __dadd_rn(acc, (double)c);
  }
};

// Deterministic CTA reduce: xor butterflies inside each warp, then warp 0
// folds the per-warp values in warp order.  The result is valid in thread 0.
template <class Op, int T = kThreads>
__device__ __forceinline__ typename Op::Acc block_reduce(typename Op::Acc v) {
  using Acc = typename Op::Acc;
  __shared__ Acc warp_vals[T / 32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = Op::combine(v, __shfl_xor_sync(0xffffffffu, v, off));
  if (lane == 0) warp_vals[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (T / 32) ? warp_vals[lane] : Op::init();
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = Op::combine(v, __shfl_xor_sync(0xffffffffu, v, off));
  }
  return v;
}

// Fixed-order fold of the U per-float4 chunks of one tile.
template <class C, int U>
__device__ __forceinline__ typename C::T fold_chunks(const typename C::T (&c)[U]) {
  if constexpr (U == 1) {
    return c[0];
  } else if constexpr (U == 2) {
    return C::chunk2(c[0], c[1]);
  } else {
    static_assert(U == 4, "tile unroll must be 1, 2 or 4");
    return C::chunk2(C::chunk2(c[0], c[1]), C::chunk2(c[2], c[3]));
  }
}


// A one-CTA reduction is already complete in that CTA: it writes the result
// itself and the launcher skips the finalize kernel.  With kCluster the whole
// grid (at most kMaxClusterCtas CTAs) is one thread-block cluster: each CTA
// leaves its value in its shared memory, and CTA rank 0 folds them in rank
// order through distributed shared memory, so a small reduction is complete
// in one launch.  The second cluster barrier keeps every CTA's shared memory
// alive until rank 0 has read it.  `acc` is valid in thread 0 only.
template <class Op, bool kCluster>
__device__ __forceinline__ void store_reduction(typename Op::Acc acc,
                                                typename Op::Acc* __restrict__ partials,
                                                float* __restrict__ out,
                                                typename Op::Acc* __restrict__ partial_out) {
  using Acc = typename Op::Acc;
  if constexpr (kCluster) {
    namespace cg = cooperative_groups;
    __shared__ Acc cta_value;
    cg::cluster_group cluster = cg::this_cluster();
    if (threadIdx.x == 0) cta_value = acc;
    cluster.sync();
    if (threadIdx.x == 0 && cluster.block_rank() == 0) {
      Acc total = acc;
      const unsigned ctas = cluster.num_blocks();
      for (unsigned r = 1; r < ctas; ++r)
        total = Op::combine(total, *cluster.map_shared_rank(&cta_value, r));
      if (out != nullptr) out[0] = Op::to_float(total);
      if (partial_out != nullptr) partial_out[0] = total;
    }
    cluster.sync();
    return;
  }
  if (threadIdx.x != 0) return;
  if (gridDim.x == 1) {
    if (out != nullptr) out[0] = Op::to_float(acc);
    if (partial_out != nullptr) partial_out[0] = acc;
  } else {
    partials[blockIdx.x] = acc;
  }
}

template <class Op, class Body, int U, bool kCluster = false>
__global__ void __launch_bounds__(kThreads)
reduce_vec_kernel(typename Op::Acc* __restrict__ partials, const Ptrs<Body::kInputs> in,
                  const int64_t n, const int64_t head, const Body body, float* __restrict__ out,
                  typename Op::Acc* __restrict__ partial_out) {
  allow_dependent_launch();
  wait_for_prerequisite_grid();
  constexpr int K = Body::kInputs;
  constexpr int kTile = kThreads * U;
  using Acc = typename Op::Acc;
  using C = Chunking<Op, NonNegative<Body>::value>;
  const int64_t nvec = (n - head) >> 2;
  const int64_t full_tiles = nvec / kTile;
  const int rem_last = (int)(nvec - full_tiles * kTile);
  const int64_t grid = gridDim.x;
  const int64_t b = blockIdx.x;
  const float4* src[K];
#pragma unroll
  for (int k = 0; k < K; ++k)
    src[k] = reinterpret_cast<const float4*>(in.p[k] + head) + b * kTile + threadIdx.x;
  const int iters = b < full_tiles ? (int)((full_tiles - 1 - b) / grid + 1) : 0;
  const int64_t stride = grid * kTile;
  Acc acc = Op::init();
  for (int it = 0; it < iters; ++it) {
    float4 v[U][K];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int k = 0; k < K; ++k) v[u][k] = load_stream(src[k] + u * kThreads);
    typename C::T c[U];
#pragma unroll
    for (int u = 0; u < U; ++u) c[u] = C::chunk4(apply4(body, v[u]));
    acc = C::absorb(acc, fold_chunks<C, U>(c));
#pragma unroll
    for (int k = 0; k < K; ++k) src[k] += stride;
  }
  // The ragged last tile (tile index full_tiles) is the next tile of CTA
  // full_tiles mod grid, whose pointers now stand at its start.
  if (rem_last > 0 && b == full_tiles % grid) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (u * kThreads + (int)threadIdx.x < rem_last) {
        float4 v[K];
#pragma unroll
        for (int k = 0; k < K; ++k) v[k] = load_stream(src[k] + u * kThreads);
        acc = C::absorb(acc, C::chunk4(apply4(body, v)));
      }
    }
  }
  if (b == grid - 1) {
    const int64_t tail0 = head + (nvec << 2);
    const int r = threadIdx.x;
    int64_t i = -1;
    if (r < head) i = r;
    else if (r >= 4 && (int64_t)(r - 4) < n - tail0) i = tail0 + (r - 4);
    if (i >= 0) acc = Op::absorb(acc, apply1(body, in, i));
  }
  acc = block_reduce<Op>(acc);
  store_reduction<Op, kCluster>(acc, partials, out, partial_out);
}

template <class Op, class Body>
__global__ void __launch_bounds__(kThreads)
reduce_scalar_kernel(typename Op::Acc* __restrict__ partials, const Ptrs<Body::kInputs> in,
                     const int64_t n, const Body body, float* __restrict__ out,
                     typename Op::Acc* __restrict__ partial_out) {
  allow_dependent_launch();
  wait_for_prerequisite_grid();
  using Acc = typename Op::Acc;
  constexpr int kU = kScalarUnroll;
  constexpr int64_t kTile = (int64_t)kThreads * kU;
  const int64_t stride = (int64_t)gridDim.x * kTile;
  Acc acc = Op::init();
  for (int64_t t = (int64_t)blockIdx.x * kTile; t < n; t += stride) {
    if (t + kTile <= n) {
      float v[kU][Body::kInputs];
#pragma unroll
      for (int u = 0; u < kU; ++u)
#pragma unroll
        for (int k = 0; k < Body::kInputs; ++k)
          v[u][k] = load_stream(in.p[k] + t + u * kThreads + threadIdx.x);
      using C = Chunking<Op, false>;
      typename C::T c[kU / 4];
#pragma unroll
      for (int q = 0; q < kU / 4; ++q) {
        float4 f;
        f.x = body(v[4 * q + 0]);
        f.y = body(v[4 * q + 1]);
        f.z = body(v[4 * q + 2]);
        f.w = body(v[4 * q + 3]);
        c[q] = C::chunk4(f);
      }
      acc = C::absorb(acc, fold_chunks<C, kU / 4>(c));
    } else {
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = t + u * kThreads + threadIdx.x;
        if (i < n) acc = Op::absorb(acc, apply1(body, in, i));
      }
    }
  }
  acc = block_reduce<Op>(acc);
  store_reduction<Op, false>(acc, partials, out, partial_out);
}

// One CTA of kFinalizeThreads folds `count` CTA partials in a fixed order:
// each thread issues 16 independent loads per round (the partials are in L2,
// so the fold is bound by load latency, not bandwidth) into four interleaved
// accumulators, then the CTA tree.  The result is valid in thread 0.
template <class Op>
__device__ __forceinline__ typename Op::Acc fold_partials(
    const typename Op::Acc* __restrict__ partials, const int count) {
  using Acc = typename Op::Acc;
  constexpr int T = kFinalizeThreads;
  constexpr int kLoads = 16;
  Acc a[4] = {Op::init(), Op::init(), Op::init(), Op::init()};
  int i = threadIdx.x;
  for (; i + (kLoads - 1) * T < count; i += kLoads * T) {
    Acc v[kLoads];
#pragma unroll
    for (int j = 0; j < kLoads; ++j) v[j] = partials[i + j * T];
#pragma unroll
    for (int j = 0; j < kLoads; ++j) a[j & 3] = Op::combine(a[j & 3], v[j]);
  }
  for (; i < count; i += T) a[0] = Op::combine(a[0], partials[i]);
  const Acc acc = Op::combine(Op::combine(a[0], a[1]), Op::combine(a[2], a[3]));
  return block_reduce<Op, T>(acc);
}

// The finalize CTA: folds the partials, writes the fp32 result to `out` (if
// non-null) and the full-precision value to `partial_out` (if non-null; the
// multi-GPU path exchanges it).
template <class Op>
__global__ void __launch_bounds__(kFinalizeThreads)
reduce_finalize_kernel(const typename Op::Acc* __restrict__ partials, const int count,
                       float* __restrict__ out, typename Op::Acc* __restrict__ partial_out) {
  wait_for_prerequisite_grid();
  allow_dependent_launch();
  const typename Op::Acc acc = fold_partials<Op>(partials, count);
  if (threadIdx.x == 0) {
    if (out != nullptr) out[0] = Op::to_float(acc);
    if (partial_out != nullptr) partial_out[0] = acc;
  }
}

// Folds `count` per-rank values (gathered in rank order) into out[0].
template <class Op>
__global__ void rank_combine_kernel(const typename Op::Acc* __restrict__ ranks, const int count,
                                    float* __restrict__ out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    typename Op::Acc acc = Op::init();
    for (int r = 0; r < count; ++r) acc = Op::combine(acc, ranks[r]);
    out[0] = Op::to_float(acc);
  }
}

}  // namespace loomb
