// bulk_sweep.cu -- standalone probe: streaming through the bulk-copy engine
// (cp.async.bulk global -> shared, completion on an mbarrier) against the
// 128-bit register loads that loom_b200_device.cuh uses, for 1-3 input
// reductions and maps over N = 2^28 fp32, one tile per CTA.
// Build and run on a B200:
//   nvcc -std=c++17 -O3 -gencode arch=compute_100a,code=sm_100a \
//        loom_b200/csrc/bulk_sweep.cu -o /tmp/bulk_sweep && /tmp/bulk_sweep
// Prints one JSON line per variant (CUDA events, 3 warm-up + 20 timed launches)
// and the error flag of the bounded waits (0 when every wait completed).
//
// Every copy is 16-byte aligned with a size that is a multiple of 16 bytes
// (tiles of 8-32 KiB at 256-byte aligned bases, N a multiple of every tile).
// Waits on the mbarrier give up after kMaxPolls polls, record the failure in
// g_err and skip the tile's arithmetic; the CTA then still waits (bounded
// again) for its copies before it exits.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>

#define CK(x)                                                                        \
  do {                                                                               \
    cudaError_t e = (x);                                                             \
    if (e != cudaSuccess) {                                                          \
      printf("ERR %s at %d: %s\n", #x, __LINE__, cudaGetErrorString(e));              \
      exit(1);                                                                       \
    }                                                                                \
  } while (0)

constexpr int T = 256;
constexpr long kMaxPolls = 1L << 22;
__device__ int g_err;

struct P3 {
  const float4* p[3];
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Polls phase 0 of the mbarrier; false after kMaxPolls unsuccessful polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar) {
  for (long i = 0; i < kMaxPolls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_addr(bar))
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_addr(src)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_store_drain() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

template <int K>
__device__ __forceinline__ float4 combine(const float4 (&v)[K]) {
  float4 r;
  if constexpr (K == 1) {
    r.x = fmaxf(v[0].x, 0.f); r.y = fmaxf(v[0].y, 0.f);
    r.z = fmaxf(v[0].z, 0.f); r.w = fmaxf(v[0].w, 0.f);
  } else if constexpr (K == 2) {
    r.x = fmaf(2.5f, v[0].x, v[1].x); r.y = fmaf(2.5f, v[0].y, v[1].y);
    r.z = fmaf(2.5f, v[0].z, v[1].z); r.w = fmaf(2.5f, v[0].w, v[1].w);
  } else {
    r.x = fmaf(v[0].x, v[1].x, v[2].x); r.y = fmaf(v[0].y, v[1].y, v[2].y);
    r.z = fmaf(v[0].z, v[1].z, v[2].z); r.w = fmaf(v[0].w, v[1].w, v[2].w);
  }
  return r;
}

__device__ __forceinline__ void block_sum_store(double acc, double* part) {
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  __shared__ double w[T / 32];
  if ((threadIdx.x & 31) == 0) w[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0;
    for (int i = 0; i < T / 32; ++i) s += w[i];
    part[blockIdx.x] = s;
  }
}

// Register path (the product's shape): U float4 per input per thread.
template <int K, int U>
__global__ void __launch_bounds__(T) red_lsu(double* __restrict__ part, P3 in) {
  const int64_t i0 = (int64_t)blockIdx.x * T * U + threadIdx.x;
  float4 v[U][K];
#pragma unroll
  for (int u = 0; u < U; ++u)
#pragma unroll
    for (int k = 0; k < K; ++k) v[u][k] = __ldcs(in.p[k] + i0 + u * T);
  float c = 0.f;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const float4 r = combine<K>(v[u]);
    c += (r.x + r.y) + (r.z + r.w);
  }
  block_sum_store((double)c, part);
}

// Bulk path: thread 0 copies one VEC-float4-per-thread tile of every input
// into shared memory; the CTA then reads it from there.
template <int K, int VEC>
__global__ void __launch_bounds__(T) red_bulk(double* __restrict__ part, P3 in) {
  extern __shared__ __align__(128) float4 buf[];  // K * T * VEC float4
  __shared__ __align__(8) uint64_t bar;
  constexpr uint32_t kBytes = T * VEC * 16;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_expect_tx(&bar, K * kBytes);
    const int64_t base = (int64_t)blockIdx.x * T * VEC;
#pragma unroll
    for (int k = 0; k < K; ++k) bulk_load(buf + k * T * VEC, in.p[k] + base, kBytes, &bar);
  }
  __syncthreads();
  float c = 0.f;
  if (mbar_wait(&bar)) {
#pragma unroll
    for (int u = 0; u < VEC; ++u) {
      float4 v[K];
#pragma unroll
      for (int k = 0; k < K; ++k) v[k] = buf[k * T * VEC + u * T + threadIdx.x];
      const float4 r = combine<K>(v);
      c += (r.x + r.y) + (r.z + r.w);
    }
  } else {
    atomicExch(&g_err, 1);
    mbar_wait(&bar);  // bounded: do not leave copies in flight into freed shared memory
  }
  block_sum_store((double)c, part);
}

template <int K, int U>
__global__ void __launch_bounds__(T) map_lsu(float4* __restrict__ out, P3 in) {
  const int64_t i0 = (int64_t)blockIdx.x * T * U + threadIdx.x;
  float4 v[U][K];
#pragma unroll
  for (int u = 0; u < U; ++u)
#pragma unroll
    for (int k = 0; k < K; ++k) v[u][k] = __ldcs(in.p[k] + i0 + u * T);
#pragma unroll
  for (int u = 0; u < U; ++u) __stcs(out + i0 + u * T, combine<K>(v[u]));
}

// Bulk loads; results stored either from registers (STORE_BULK = 0) or
// staged in shared memory and written by one bulk store (STORE_BULK = 1).
template <int K, int VEC, int STORE_BULK>
__global__ void __launch_bounds__(T) map_bulk(float4* __restrict__ out, P3 in) {
  extern __shared__ __align__(128) float4 buf[];  // (K + 1) * T * VEC float4
  __shared__ __align__(8) uint64_t bar;
  constexpr uint32_t kBytes = T * VEC * 16;
  const int64_t base = (int64_t)blockIdx.x * T * VEC;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_expect_tx(&bar, K * kBytes);
#pragma unroll
    for (int k = 0; k < K; ++k) bulk_load(buf + k * T * VEC, in.p[k] + base, kBytes, &bar);
  }
  __syncthreads();
  bool ok = mbar_wait(&bar);
  if (!ok) {
    atomicExch(&g_err, 1);
    mbar_wait(&bar);  // bounded: do not leave copies in flight into freed shared memory
  }
  float4* res = buf + K * T * VEC;
  if (ok) {
#pragma unroll
    for (int u = 0; u < VEC; ++u) {
      float4 v[K];
#pragma unroll
      for (int k = 0; k < K; ++k) v[k] = buf[k * T * VEC + u * T + threadIdx.x];
      if constexpr (STORE_BULK) res[u * T + threadIdx.x] = combine<K>(v);
      else __stcs(out + base + u * T + threadIdx.x, combine<K>(v));
    }
  }
  if constexpr (STORE_BULK) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    // every thread reaches this barrier; the store runs only if all waits completed
    const bool all_ok = __syncthreads_and(ok);
    if (threadIdx.x == 0 && all_ok) {
      bulk_store(out + base, res, kBytes);
      bulk_store_drain();
    }
  }
}

static float* g_in[3];
static float* g_out;
static double* g_part;
static const int64_t N = (int64_t)1 << 28;

template <typename F>
float time_it(F launch, int reps) {
  cudaEvent_t a, b;
  CK(cudaEventCreate(&a));
  CK(cudaEventCreate(&b));
  for (int i = 0; i < 3; ++i) launch();
  CK(cudaDeviceSynchronize());
  CK(cudaEventRecord(a));
  for (int i = 0; i < reps; ++i) launch();
  CK(cudaEventRecord(b));
  CK(cudaEventSynchronize(b));
  float ms;
  CK(cudaEventElapsedTime(&ms, a, b));
  CK(cudaGetLastError());
  return ms / reps;
}

static int read_err() {
  int e = 0;
  CK(cudaMemcpyFromSymbol(&e, g_err, sizeof(int)));
  return e;
}

static P3 inputs() {
  P3 in;
  for (int k = 0; k < 3; ++k) in.p[k] = reinterpret_cast<const float4*>(g_in[k]);
  return in;
}

static void report(const char* kind, const char* path, int K, int vec, int store_bulk,
                   size_t smem, int occ, int64_t grid, float ms, double bytes) {
  printf("{\"kind\":\"%s\",\"path\":\"%s\",\"K\":%d,\"vec\":%d,\"store_bulk\":%d,"
         "\"smem\":%zu,\"occ\":%d,\"grid\":%lld,\"us\":%.1f,\"gbs\":%.1f,\"err\":%d}\n",
         kind, path, K, vec, store_bulk, smem, occ, (long long)grid, ms * 1e3,
         bytes / (ms * 1e-3) / 1e9, read_err());
  fflush(stdout);
}

template <int K, int U>
void run_red_lsu() {
  int occ = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, red_lsu<K, U>, T, 0));
  const int64_t grid = N / 4 / (T * U);
  P3 in = inputs();
  float ms = time_it([&] { red_lsu<K, U><<<(unsigned)grid, T>>>(g_part, in); }, 20);
  report("red", "lsu", K, U, 0, 0, occ, grid, ms, 4.0 * N * K);
}

template <int K, int VEC>
void run_red_bulk() {
  const size_t smem = (size_t)K * T * VEC * 16;
  CK(cudaFuncSetAttribute(red_bulk<K, VEC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)smem));
  int occ = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, red_bulk<K, VEC>, T, smem));
  const int64_t grid = N / 4 / (T * VEC);
  P3 in = inputs();
  float ms =
      time_it([&] { red_bulk<K, VEC><<<(unsigned)grid, T, smem>>>(g_part, in); }, 20);
  report("red", "bulk", K, VEC, 0, smem, occ, grid, ms, 4.0 * N * K);
}

template <int K, int U>
void run_map_lsu() {
  int occ = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, map_lsu<K, U>, T, 0));
  const int64_t grid = N / 4 / (T * U);
  P3 in = inputs();
  float ms = time_it(
      [&] { map_lsu<K, U><<<(unsigned)grid, T>>>(reinterpret_cast<float4*>(g_out), in); }, 20);
  report("map", "lsu", K, U, 0, 0, occ, grid, ms, 4.0 * N * (K + 1));
}

template <int K, int VEC, int SB>
void run_map_bulk() {
  const size_t smem = (size_t)(K + SB) * T * VEC * 16;
  CK(cudaFuncSetAttribute(map_bulk<K, VEC, SB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)smem));
  int occ = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, map_bulk<K, VEC, SB>, T, smem));
  const int64_t grid = N / 4 / (T * VEC);
  P3 in = inputs();
  float ms = time_it(
      [&] {
        map_bulk<K, VEC, SB><<<(unsigned)grid, T, smem>>>(reinterpret_cast<float4*>(g_out), in);
      },
      20);
  report("map", "bulk", K, VEC, SB, smem, occ, grid, ms, 4.0 * N * (K + 1));
}

__global__ void fill(float* p, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v * (float)(i & 1023) - 3.0f;
}

int main() {
  for (int k = 0; k < 3; ++k) {
    CK(cudaMalloc(&g_in[k], N * 4));
    fill<<<1024, 256>>>(g_in[k], N, 0.001f * (k + 1));
  }
  CK(cudaMalloc(&g_out, N * 4));
  CK(cudaMalloc(&g_part, (N / 4 / T) * sizeof(double)));
  CK(cudaDeviceSynchronize());
  // reductions: the product's register shape, then bulk tiles of 8, 16, 32 KiB per input
  run_red_lsu<1, 4>();
  run_red_bulk<1, 2>();
  run_red_bulk<1, 4>();
  run_red_bulk<1, 8>();
  run_red_lsu<2, 2>();
  run_red_bulk<2, 2>();
  run_red_bulk<2, 4>();
  run_red_bulk<2, 8>();
  run_red_lsu<3, 2>();
  run_red_bulk<3, 2>();
  run_red_bulk<3, 4>();
  // maps: register shape, bulk loads with register stores, bulk loads and bulk store
  run_map_lsu<1, 2>();
  run_map_bulk<1, 2, 0>();
  run_map_bulk<1, 4, 0>();
  run_map_bulk<1, 4, 1>();
  run_map_lsu<2, 1>();
  run_map_bulk<2, 2, 0>();
  run_map_bulk<2, 4, 0>();
  run_map_bulk<2, 4, 1>();
  run_map_lsu<3, 1>();
  run_map_bulk<3, 2, 0>();
  run_map_bulk<3, 2, 1>();
  return 0;
}
