// stream_sweep.cu -- standalone probe of the streaming loop shapes used by
// loom_b200_device.cuh: load/store cache flavours, float4 per thread (U),
// threads per CTA (T) and the grid shape (one tile per CTA vs a persistent
// grid-stride loop), for 1-3 input maps and reductions over N = 2^28 fp32.
// Build and run on a B200:
//   nvcc -std=c++17 -O3 -gencode arch=compute_100a,code=sm_100a \
//        loom_b200/csrc/stream_sweep.cu -o /tmp/stream_sweep && /tmp/stream_sweep
// Prints one JSON line per variant (CUDA events, 3 warm-up + 20 timed launches).
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

// LD: 0 ld.global.cs, 1 ld.global.nc, 2 ld.global, 3 ld.global.lu,
//     4 ld.global.nc.L1::no_allocate.L2::256B
template <int LD>
__device__ __forceinline__ float4 ld4(const float4* p) {
  if constexpr (LD == 0) return __ldcs(p);
  else if constexpr (LD == 1) return __ldg(p);
  else if constexpr (LD == 2) return *p;
  else if constexpr (LD == 3) return __ldlu(p);
  else {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
  }
}

// ST: 0 st.global.cs, 1 st.global, 2 st.global.wb, 3 st.global.L1::no_allocate
template <int ST>
__device__ __forceinline__ void st4(float4* p, float4 v) {
  if constexpr (ST == 0) __stcs(p, v);
  else if constexpr (ST == 1) *p = v;
  else if constexpr (ST == 2) __stwb(p, v);
  else {
    asm volatile("st.global.L1::no_allocate.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x),
                 "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
  }
}

struct P3 {
  const float4* p[3];
};

// Every input feeds the result, so no load is dead.
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

template <int K, int U, int T, int LD, int ST>
__global__ void __launch_bounds__(T) mapk(float4* __restrict__ out, P3 in, int64_t nvec) {
  const int64_t tile = (int64_t)T * U;
  const int64_t stride = (int64_t)gridDim.x * tile;
  for (int64_t t = (int64_t)blockIdx.x * tile; t < nvec; t += stride) {
    const int64_t i0 = t + threadIdx.x;
    if (t + tile <= nvec) {
      float4 v[U][K];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int k = 0; k < K; ++k) v[u][k] = ld4<LD>(in.p[k] + i0 + u * T);
#pragma unroll
      for (int u = 0; u < U; ++u) st4<ST>(out + i0 + u * T, combine<K>(v[u]));
    } else {
      for (int u = 0; u < U; ++u) {
        const int64_t i = i0 + u * T;
        if (i < nvec) {
          float4 v[K];
          for (int k = 0; k < K; ++k) v[k] = ld4<LD>(in.p[k] + i);
          st4<ST>(out + i, combine<K>(v));
        }
      }
    }
  }
}

template <int K, int U, int T, int LD>
__global__ void __launch_bounds__(T) redk(double* __restrict__ part, P3 in, int64_t nvec) {
  const int64_t tile = (int64_t)T * U;
  const int64_t stride = (int64_t)gridDim.x * tile;
  double acc = 0.0;
  for (int64_t t = (int64_t)blockIdx.x * tile; t < nvec; t += stride) {
    const int64_t i0 = t + threadIdx.x;
    if (t + tile <= nvec) {
      float4 v[U][K];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int k = 0; k < K; ++k) v[u][k] = ld4<LD>(in.p[k] + i0 + u * T);
      float c = 0.f;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float4 r = combine<K>(v[u]);
        c += (r.x + r.y) + (r.z + r.w);
      }
      acc += (double)c;
    } else {
      for (int u = 0; u < U; ++u) {
        const int64_t i = i0 + u * T;
        if (i < nvec) {
          float4 v[K];
          for (int k = 0; k < K; ++k) v[k] = ld4<LD>(in.p[k] + i);
          const float4 r = combine<K>(v);
          acc += (double)((r.x + r.y) + (r.z + r.w));
        }
      }
    }
  }
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

static float* g_in[3];
static float* g_out;
static double* g_part;
static int g_sms;
static const int64_t N = (int64_t)1 << 28;
static const int64_t kMaxPart = 262144;

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

// grid_mult 0: one tile per CTA; M > 0: M x (SMs x resident CTAs), grid-stride.
static int64_t pick_grid(int occ, int64_t tiles, int grid_mult) {
  if (grid_mult == 0) return tiles;
  int64_t g = (int64_t)g_sms * occ * grid_mult;
  return g > tiles ? tiles : g;
}

template <int K, int U, int T, int LD, int ST>
void run_map(int grid_mult) {
  int occ = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, mapk<K, U, T, LD, ST>, T, 0));
  const int64_t nvec = N / 4;
  const int64_t tiles = (nvec + (int64_t)T * U - 1) / ((int64_t)T * U);
  const int64_t grid = pick_grid(occ, tiles, grid_mult);
  P3 in;
  for (int k = 0; k < 3; ++k) in.p[k] = reinterpret_cast<const float4*>(g_in[k]);
  float ms = time_it([&] {
    mapk<K, U, T, LD, ST><<<(unsigned)grid, T>>>(reinterpret_cast<float4*>(g_out), in, nvec);
  }, 20);
  printf("{\"kind\":\"map\",\"K\":%d,\"U\":%d,\"T\":%d,\"LD\":%d,\"ST\":%d,\"grid_mult\":%d,"
         "\"occ\":%d,\"grid\":%lld,\"us\":%.1f,\"gbs\":%.1f}\n",
         K, U, T, LD, ST, grid_mult, occ, (long long)grid, ms * 1e3,
         4.0 * N * (K + 1) / (ms * 1e-3) / 1e9);
  fflush(stdout);
}

template <int K, int U, int T, int LD>
void run_red(int grid_mult) {
  int occ = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, redk<K, U, T, LD>, T, 0));
  const int64_t nvec = N / 4;
  const int64_t tiles = (nvec + (int64_t)T * U - 1) / ((int64_t)T * U);
  int64_t grid = pick_grid(occ, tiles, grid_mult);
  if (grid > kMaxPart) grid = kMaxPart;
  P3 in;
  for (int k = 0; k < 3; ++k) in.p[k] = reinterpret_cast<const float4*>(g_in[k]);
  float ms = time_it([&] { redk<K, U, T, LD><<<(unsigned)grid, T>>>(g_part, in, nvec); }, 20);
  printf("{\"kind\":\"red\",\"K\":%d,\"U\":%d,\"T\":%d,\"LD\":%d,\"grid_mult\":%d,\"occ\":%d,"
         "\"grid\":%lld,\"us\":%.1f,\"gbs\":%.1f}\n",
         K, U, T, LD, grid_mult, occ, (long long)grid, ms * 1e3,
         4.0 * N * K / (ms * 1e-3) / 1e9);
  fflush(stdout);
}

__global__ void fill(float* p, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v * (float)(i & 1023) - 3.0f;
}

int main() {
  CK(cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, 0));
  for (int k = 0; k < 3; ++k) {
    CK(cudaMalloc(&g_in[k], N * 4));
    fill<<<1024, 256>>>(g_in[k], N, 0.001f * (k + 1));
  }
  CK(cudaMalloc(&g_out, N * 4));
  CK(cudaMalloc(&g_part, kMaxPart * 8));
  CK(cudaDeviceSynchronize());
  // one-input maps: cache flavours, unroll, threads, grid shape
  run_map<1, 4, 256, 0, 0>(1);
  run_map<1, 4, 256, 1, 0>(1);
  run_map<1, 4, 256, 2, 0>(1);
  run_map<1, 4, 256, 4, 0>(1);
  run_map<1, 4, 256, 0, 1>(1);
  run_map<1, 4, 256, 2, 1>(1);
  run_map<1, 4, 256, 0, 3>(1);
  run_map<1, 4, 256, 3, 0>(1);
  run_map<1, 8, 256, 0, 0>(1);
  run_map<1, 2, 256, 0, 0>(1);
  run_map<1, 4, 128, 0, 0>(1);
  run_map<1, 4, 512, 0, 0>(1);
  run_map<1, 4, 256, 0, 0>(4);
  run_map<1, 4, 256, 0, 0>(16);
  run_map<1, 4, 256, 0, 0>(0);
  run_map<1, 2, 256, 0, 0>(0);
  run_map<1, 1, 256, 0, 0>(0);
  run_map<1, 8, 256, 0, 0>(0);
  run_map<1, 2, 256, 1, 1>(0);
  run_map<1, 2, 128, 0, 0>(0);
  run_map<1, 2, 512, 0, 0>(0);
  // two- and three-input maps
  run_map<2, 4, 256, 0, 0>(1);
  run_map<2, 4, 256, 0, 0>(8);
  run_map<2, 4, 256, 0, 0>(0);
  run_map<2, 2, 256, 0, 0>(0);
  run_map<2, 1, 256, 0, 0>(0);
  run_map<2, 2, 256, 1, 1>(0);
  run_map<2, 2, 512, 0, 0>(0);
  run_map<3, 4, 256, 0, 0>(1);
  run_map<3, 4, 256, 0, 0>(0);
  run_map<3, 2, 256, 0, 0>(0);
  run_map<3, 1, 256, 0, 0>(0);
  // reductions
  run_red<1, 4, 256, 0>(1);
  run_red<1, 4, 256, 1>(1);
  run_red<1, 4, 256, 0>(4);
  run_red<1, 4, 256, 0>(0);
  run_red<1, 2, 256, 0>(0);
  run_red<1, 8, 256, 0>(0);
  run_red<2, 4, 256, 0>(1);
  run_red<2, 4, 256, 0>(4);
  run_red<2, 4, 256, 0>(0);
  run_red<2, 2, 256, 0>(0);
  run_red<3, 4, 256, 0>(1);
  run_red<3, 4, 256, 0>(0);
  run_red<3, 2, 256, 0>(0);
  printf("done\n");
  return 0;
}
