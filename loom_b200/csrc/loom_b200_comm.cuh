// loom_b200_comm.cuh -- multi-GPU support for generated Loom packages.
//
// The reference has no multi-GPU path at all (no NCCL, no device selection;
// its generated code runs on the caller's current device).  This adds the one
// exchange a sharded Loom entry needs: element-wise maps shard with no
// communication, and a reduction combines one scalar per GPU over NVLink /
// NVSwitch with NCCL.
//
//  * sum: every rank reduces its shard to one fp64 value (the same fixed-order
//    kernels as the single-GPU path), the ranks all-gather the fp64 values and
//    every rank folds them in rank order -- bit-identical on every rank and
//    from run to run;
//  * max: fp32 ncclMax all-reduce of the per-rank maxima (exact in any order).
//
// Where every pair of GPUs can reach each other's memory (NVLink / NVSwitch),
// the scalar exchange does not go through NCCL at all: each rank's exchange
// kernel stores its value straight into every peer's exchange buffer (P2P
// stores over NVLink), then reads the nranks values from its own buffer and
// folds them in rank order -- the same values in the same order as the NCCL
// path, so the same bits.  That replaces an NCCL collective and a fold kernel
// by one single-thread kernel (see peer_exchange_kernel).
//
// Communicators are explicit handles created by the caller (one process per
// GPU via comm_init_rank, or one process for several GPUs via comm_init_all)
// and destroyed with comm_destroy; the library keeps no global state.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>
#include <string.h>

#include <new>

#include "loom_b200_launch.cuh"

#ifndef LOOM_STATUS_COMM_ERROR
#define LOOM_STATUS_COMM_ERROR 4
#endif

namespace loomb {

// Every rank's exchange buffer, as addressed from this rank's device.
struct PeerTable {
  unsigned char* buf[kMaxRanks];
};

// Layout of an exchange buffer (kExchangeBytes, zeroed at creation):
//   +0   u64  exchanges this rank has made (its epoch counter)
//   +8   u32  status: 0 ok, 1 a wait for a peer ran out
//   +16  u64  wait statistics of this rank's exchanges: total ns spent from
//   +24  u64  sending its value to holding every rank's (%globaltimer), the
//   +32  u64  largest such wait, and the number of exchanges timed
//   +64  ExchangeSlot[2][kMaxRanks]: the value each rank sent for the
//        exchanges of even / odd epoch.  Two sets suffice: a rank can be at
//        most one exchange ahead of any other, since it cannot finish an
//        exchange before every rank has sent to it.
// A slot holds the value's 64 bits as two words, each carrying 32 bits of it
// (low half in half[0], high half in half[1]) under the low 32 bits of the
// sender's epoch in its upper half.  An aligned 64-bit store is seen whole
// or not at all, so a reader that finds this epoch's tag in both words
// holds the value: the sender needs no release fence (a round trip to the
// peer) and the reader no acquire.  Epochs start at 1, so a slot still
// zeroed from creation never matches, and a used slot holds the tag of the
// exchange two epochs back at worst.
struct ExchangeSlot {
  unsigned long long half[2];
};
constexpr size_t kExchangeSlotsOffset = 64;
constexpr size_t kExchangeBytes = 4096;
static_assert(kExchangeSlotsOffset + 2 * kMaxRanks * sizeof(ExchangeSlot) + 64 +
                      kMaxRanks * sizeof(cudaIpcMemHandle_t) + 64 <=
                  kExchangeBytes,
              "exchange buffer too small for the slots and the setup scratch");

struct Comm {
  ncclComm_t nccl = nullptr;
  int nranks = 0;
  int rank = 0;
  int device = 0;
  unsigned char* xbuf = nullptr;     // this rank's exchange buffer (device memory)
  PeerTable peers = {};              // every rank's buffer, from this device
  bool ipc_opened[kMaxRanks] = {};   // peers mapped with cudaIpcOpenMemHandle
  bool peer_capable = false;         // the buffers are set up on every rank
  bool peer_exchange = false;        // exchange through peer memory (else NCCL)
  unsigned long long timeout_ns = 30000000000ull;  // a peer exchange's wait limit
};

// Restores the caller's current device when it goes out of scope.
struct DeviceGuard {
  int device = -1;
  DeviceGuard() { cudaGetDevice(&device); }
  ~DeviceGuard() {
    if (device >= 0) cudaSetDevice(device);
  }
};

inline void release_exchange(Comm* c) {
  for (int r = 0; r < kMaxRanks; ++r) {
    if (c->ipc_opened[r]) cudaIpcCloseMemHandle(c->peers.buf[r]);
    c->ipc_opened[r] = false;
    c->peers.buf[r] = nullptr;
  }
  if (c->xbuf != nullptr) cudaFree(c->xbuf);
  c->xbuf = nullptr;
  c->peer_capable = c->peer_exchange = false;
}

inline bool alloc_exchange(Comm* c) {
  if (cudaMalloc(&c->xbuf, kExchangeBytes) != cudaSuccess) {
    c->xbuf = nullptr;
    cudaGetLastError();
    return false;
  }
  return cudaMemset(c->xbuf, 0, kExchangeBytes) == cudaSuccess &&
         cudaDeviceSynchronize() == cudaSuccess;
}

// One process per GPU: every rank exports its exchange buffer with a CUDA
// IPC handle, the handles are all-gathered over the new communicator, and
// every rank maps the others' buffers.  The ranks then agree (an NCCL min of
// a success flag) so that either all of them use peer memory or none does.
// A failure to map leaves every rank on the NCCL path.  The setup scratch
// (nranks handles and the flag) sits behind the exchange area of the same
// allocation; a rank that could not make even that allocation would leave
// the others waiting in the collective, as a failure inside
// ncclCommInitRank would.
inline void setup_exchange_ipc(Comm* c) {
  constexpr size_t kH = sizeof(cudaIpcMemHandle_t);
  bool ok = alloc_exchange(c);
  if (!ok) {
    release_exchange(c);
    return;
  }
  unsigned char* scratch = c->xbuf + kExchangeSlotsOffset + 2 * kMaxRanks * sizeof(ExchangeSlot);
  scratch = reinterpret_cast<unsigned char*>(align_up((size_t)(uintptr_t)scratch, 64));
  cudaIpcMemHandle_t own;
  memset(&own, 0, sizeof(own));
  ok = cudaIpcGetMemHandle(&own, c->xbuf) == cudaSuccess;
  unsigned char host[kMaxRanks * kH];
  cudaMemcpy(scratch + (size_t)c->rank * kH, &own, kH, cudaMemcpyHostToDevice);
  const bool gathered =
      ncclAllGather(scratch + (size_t)c->rank * kH, scratch, kH, ncclChar, c->nccl, nullptr) ==
          ncclSuccess &&
      cudaStreamSynchronize(nullptr) == cudaSuccess &&
      cudaMemcpy(host, scratch, c->nranks * kH, cudaMemcpyDeviceToHost) == cudaSuccess;
  ok = ok && gathered;
  for (int r = 0; r < c->nranks && ok; ++r) {
    if (r == c->rank) {
      c->peers.buf[r] = c->xbuf;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, host + (size_t)r * kH, kH);
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = false;
      break;
    }
    c->peers.buf[r] = static_cast<unsigned char*>(p);
    c->ipc_opened[r] = true;
  }
  int flag = ok ? 1 : 0;
  int* dflag = reinterpret_cast<int*>(scratch + (size_t)c->nranks * kH);
  const bool agreed =
      cudaMemcpy(dflag, &flag, sizeof(int), cudaMemcpyHostToDevice) == cudaSuccess &&
      ncclAllReduce(dflag, dflag, 1, ncclInt32, ncclMin, c->nccl, nullptr) == ncclSuccess &&
      cudaStreamSynchronize(nullptr) == cudaSuccess &&
      cudaMemcpy(&flag, dflag, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && flag == 1;
  // the scratch is not part of the exchange area; clear it again
  cudaMemset(scratch, 0, (size_t)c->nranks * kH + sizeof(int));
  cudaDeviceSynchronize();
  if (!agreed) {
    release_exchange(c);
    return;
  }
  c->peer_capable = c->peer_exchange = true;
}

// One process, several GPUs: direct peer access between every pair.
inline void setup_exchange_local(Comm** cs, int ndev) {
  bool ok = true;
  for (int d = 0; d < ndev && ok; ++d) {
    ok = cudaSetDevice(cs[d]->device) == cudaSuccess && alloc_exchange(cs[d]);
  }
  for (int i = 0; i < ndev && ok; ++i) {
    for (int j = 0; j < ndev && ok; ++j) {
      if (i == j) continue;
      int can = 0;
      if (cudaDeviceCanAccessPeer(&can, cs[i]->device, cs[j]->device) != cudaSuccess || !can) {
        ok = false;
        break;
      }
      cudaSetDevice(cs[i]->device);
      const cudaError_t e = cudaDeviceEnablePeerAccess(cs[j]->device, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
      else if (e != cudaSuccess) ok = false;
    }
  }
  for (int d = 0; d < ndev; ++d) {
    cudaSetDevice(cs[d]->device);
    if (!ok) {
      cudaGetLastError();
      release_exchange(cs[d]);
      continue;
    }
    for (int r = 0; r < ndev; ++r) cs[d]->peers.buf[r] = cs[r]->xbuf;
    cs[d]->peer_capable = cs[d]->peer_exchange = true;
  }
}

inline int comm_id_size() { return (int)sizeof(ncclUniqueId); }

inline int comm_unique_id(void* id_out, size_t id_size) {
  if (id_out == nullptr || id_size < sizeof(ncclUniqueId)) return LOOM_STATUS_INVALID_ARGUMENT;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return LOOM_STATUS_COMM_ERROR;
  memcpy(id_out, &id, sizeof(id));
  return LOOM_STATUS_OK;
}

// One rank of a communicator on the caller's current device (collective:
// returns when all nranks have joined).
inline int comm_init_rank(void** comm_out, int nranks, int rank, const void* id, size_t id_size) {
  if (comm_out == nullptr || id == nullptr || id_size < sizeof(ncclUniqueId) || nranks <= 0 ||
      nranks > kMaxRanks || rank < 0 || rank >= nranks)
    return LOOM_STATUS_INVALID_ARGUMENT;
  *comm_out = nullptr;
  Comm* c = new (std::nothrow) Comm();
  if (c == nullptr) return LOOM_STATUS_COMM_ERROR;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  if (cudaGetDevice(&c->device) != cudaSuccess) {
    delete c;
    return LOOM_STATUS_CUDA_ERROR;
  }
  if (ncclCommInitRank(&c->nccl, nranks, uid, rank) != ncclSuccess) {
    delete c;
    return LOOM_STATUS_COMM_ERROR;
  }
  c->nranks = nranks;
  c->rank = rank;
  if (nranks > 1) setup_exchange_ipc(c);
  *comm_out = c;
  return LOOM_STATUS_OK;
}

// One communicator per listed device, all owned by this process.
inline int comm_init_all(void** comms_out, int ndev, const int* devices) {
  if (comms_out == nullptr || devices == nullptr || ndev <= 0 || ndev > kMaxRanks)
    return LOOM_STATUS_INVALID_ARGUMENT;
  ncclComm_t raw[kMaxRanks];
  if (ncclCommInitAll(raw, ndev, devices) != ncclSuccess) return LOOM_STATUS_COMM_ERROR;
  for (int d = 0; d < ndev; ++d) {
    Comm* c = new (std::nothrow) Comm();
    if (c == nullptr) {
      for (int e = 0; e < ndev; ++e) {
        if (e < d) {
          delete static_cast<Comm*>(comms_out[e]);
          comms_out[e] = nullptr;
        }
        ncclCommDestroy(raw[e]);
      }
      return LOOM_STATUS_COMM_ERROR;
    }
    c->nccl = raw[d];
    c->nranks = ndev;
    c->rank = d;
    c->device = devices[d];
    comms_out[d] = c;
  }
  if (ndev > 1) {
    DeviceGuard guard;
    setup_exchange_local(reinterpret_cast<Comm**>(comms_out), ndev);
  }
  return LOOM_STATUS_OK;
}

inline int comm_destroy(void* comm) {
  if (comm == nullptr) return LOOM_STATUS_OK;
  Comm* c = static_cast<Comm*>(comm);
  {
    DeviceGuard guard;
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    release_exchange(c);
  }
  const ncclResult_t r = ncclCommDestroy(c->nccl);
  delete c;
  return r == ncclSuccess ? LOOM_STATUS_OK : LOOM_STATUS_COMM_ERROR;
}

// Choose the exchange path: 1 peer memory (only where it was set up), 0
// NCCL.  Collective in effect: every rank must make the same choice before
// its next reduction, or the ranks wait for values that never come (the
// waits are bounded; see comm_check).
inline int comm_set_peer_exchange(void* comm, int enable) {
  if (comm == nullptr) return LOOM_STATUS_INVALID_ARGUMENT;
  Comm* c = static_cast<Comm*>(comm);
  if (enable && !c->peer_capable) return LOOM_STATUS_INVALID_ARGUMENT;
  c->peer_exchange = enable != 0;
  return LOOM_STATUS_OK;
}

// The wait limit of this rank's peer exchanges, in milliseconds (> 0).
inline int comm_set_timeout_ms(void* comm, int64_t ms) {
  if (comm == nullptr || ms <= 0 || ms > 3600000) return LOOM_STATUS_INVALID_ARGUMENT;
  static_cast<Comm*>(comm)->timeout_ns = (unsigned long long)ms * 1000000ull;
  return LOOM_STATUS_OK;
}

inline int comm_peer_exchange(void* comm) {
  return comm != nullptr && static_cast<Comm*>(comm)->peer_exchange ? 1 : 0;
}

// Waits for this rank's device and reports whether any peer exchange gave up
// waiting for another rank (COMM_ERROR; the affected results were NaN).
inline int comm_check(void* comm) {
  if (comm == nullptr) return LOOM_STATUS_INVALID_ARGUMENT;
  Comm* c = static_cast<Comm*>(comm);
  if (c->xbuf == nullptr) return LOOM_STATUS_OK;
  DeviceGuard guard;
  unsigned int status = 0;
  if (cudaSetDevice(c->device) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(&status, c->xbuf + 8, sizeof(status), cudaMemcpyDeviceToHost) != cudaSuccess)
    return LOOM_STATUS_CUDA_ERROR;
  return status == 0 ? LOOM_STATUS_OK : LOOM_STATUS_COMM_ERROR;
}

// Copies this rank's exchange wait statistics (total ns, largest ns, number
// of exchanges timed, since the communicator was created or the last reset)
// to `out` after waiting for the rank's device, then zeroes them if `reset`.
// All zero on the NCCL path.
inline int comm_exchange_stats(void* comm, unsigned long long* out, int reset) {
  if (comm == nullptr || out == nullptr) return LOOM_STATUS_INVALID_ARGUMENT;
  Comm* c = static_cast<Comm*>(comm);
  out[0] = out[1] = out[2] = 0;
  if (c->xbuf == nullptr) return LOOM_STATUS_OK;
  DeviceGuard guard;
  constexpr size_t kBytes = 3 * sizeof(unsigned long long);
  if (cudaSetDevice(c->device) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(out, c->xbuf + 16, kBytes, cudaMemcpyDeviceToHost) != cudaSuccess)
    return LOOM_STATUS_CUDA_ERROR;
  if (reset && (cudaMemset(c->xbuf + 16, 0, kBytes) != cudaSuccess ||
                cudaDeviceSynchronize() != cudaSuccess))
    return LOOM_STATUS_CUDA_ERROR;
  return LOOM_STATUS_OK;
}

inline int nccl_group_start() { return ncclGroupStart() == ncclSuccess ? 0 : 1; }
inline int nccl_group_end() { return ncclGroupEnd() == ncclSuccess ? 0 : 1; }

// Rank scratch of a shard of n_local elements (see reduce_workspace_bytes).
inline unsigned char* rank_scratch(void* workspace, int64_t n_local) {
  return workspace_base(workspace) + rank_scratch_offset(n_local > 0 ? n_local : 1);
}

template <class Op>
struct RankSlots {
  typename Op::Acc* local;
  typename Op::Acc* gather;
  RankSlots(void* workspace, int64_t n_local) {
    unsigned char* s = rank_scratch(workspace, n_local);
    local = reinterpret_cast<typename Op::Acc*>(s);
    gather = reinterpret_cast<typename Op::Acc*>(s + 64);
  }
};

template <class Op>
inline ncclDataType_t nccl_type();
template <>
inline ncclDataType_t nccl_type<SumOp>() { return ncclDouble; }
template <>
inline ncclDataType_t nccl_type<MaxOp>() { return ncclFloat; }

// Phase 1: this rank's shard -> one Op::Acc value in the rank scratch.
template <class Op, class Body>
inline int dist_local(const Ptrs<Body::kInputs>& in, int64_t n_local, const Body& body,
                      void* workspace, cudaStream_t stream) {
  RankSlots<Op> slots(workspace, n_local);
  auto* partials = reinterpret_cast<typename Op::Acc*>(workspace_base(workspace));
  if (n_local == 0) {
    reduce_finalize_kernel<Op><<<1, kFinalizeThreads, 0, stream>>>(partials, 0, nullptr,
                                                                    slots.local);
    return launch_status();
  }
  return launch_reduce<Op>(in, n_local, body, partials, partial_capacity(n_local), nullptr,
                           slots.local, stream);
}

// Phase 2: the scalar collective (sum: all-gather of fp64; max: all-reduce).
template <class Op>
inline int dist_collective(void* workspace, int64_t n_local, float* out, Comm* comm,
                           cudaStream_t stream);

template <>
inline int dist_collective<SumOp>(void* workspace, int64_t n_local, float* out, Comm* comm,
                                  cudaStream_t stream) {
  (void)out;
  RankSlots<SumOp> slots(workspace, n_local);
  return ncclAllGather(slots.local, slots.gather, 1, ncclDouble, comm->nccl, stream) == ncclSuccess
             ? LOOM_STATUS_OK
             : LOOM_STATUS_COMM_ERROR;
}

template <>
inline int dist_collective<MaxOp>(void* workspace, int64_t n_local, float* out, Comm* comm,
                                  cudaStream_t stream) {
  RankSlots<MaxOp> slots(workspace, n_local);
  return ncclAllReduce(slots.local, out, 1, ncclFloat, ncclMax, comm->nccl, stream) == ncclSuccess
             ? LOOM_STATUS_OK
             : LOOM_STATUS_COMM_ERROR;
}

// Phase 3: fold the gathered values in rank order (sum only).
template <class Op>
inline int dist_finish(void* workspace, int64_t n_local, float* out, Comm* comm,
                       cudaStream_t stream);

template <>
inline int dist_finish<SumOp>(void* workspace, int64_t n_local, float* out, Comm* comm,
                              cudaStream_t stream) {
  RankSlots<SumOp> slots(workspace, n_local);
  rank_combine_kernel<SumOp><<<1, 32, 0, stream>>>(slots.gather, comm->nranks, out);
  return launch_status();
}

template <>
inline int dist_finish<MaxOp>(void*, int64_t, float*, Comm*, cudaStream_t) {
  return LOOM_STATUS_OK;
}

// ---------------------------------------------------------------------------
// peer-memory exchange

__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned long long acc_bits(double v) {
  return (unsigned long long)__double_as_longlong(v);
}
__device__ __forceinline__ unsigned long long acc_bits(float v) { return __float_as_uint(v); }
template <class Acc>
__device__ __forceinline__ Acc bits_acc(unsigned long long b);
template <>
__device__ __forceinline__ double bits_acc<double>(unsigned long long b) {
  return __longlong_as_double((long long)b);
}
template <>
__device__ __forceinline__ float bits_acc<float>(unsigned long long b) {
  return __uint_as_float((unsigned int)b);
}

// What an exchange needs, passed by value to the kernels that do one.
struct PeerArgs {
  PeerTable peers;
  int nranks;
  int rank;
  unsigned char* own;              // this rank's exchange buffer
  float* out;                      // the global result (fp32)
  unsigned long long timeout_ns;
};

inline PeerArgs peer_args(const Comm* c, float* out) {
  PeerArgs a;
  a.peers = c->peers;
  a.nranks = c->nranks;
  a.rank = c->rank;
  a.own = c->xbuf;
  a.out = out;
  a.timeout_ns = c->timeout_ns;
  return a;
}

// The exchange, in every thread of one CTA (`local`, this rank's value, is
// valid in thread 0; the CTA has at least kMaxRanks threads).  Thread r
// stores this rank's value into slot [epoch parity][rank] of rank r's
// exchange buffer (two epoch-tagged words, relaxed stores), then waits until
// both words of rank r's slot in the own buffer carry this epoch's tag and
// copies the value to shared memory; thread 0 folds the nranks values in
// rank order into out[0].  The sends and the waits of the ranks run in
// parallel, one thread per rank: one thread sending to every rank in turn
// paid a remote store's round trip per rank (about 2 us each on NVLink,
// 17-18 us per exchange at 8 GPUs).  The epoch is this rank's own
// exchange count, kept in device memory, so it also works when replayed
// from a graph.  A wait for a peer's value gives up after the
// communicator's timeout (30 s unless set), records status 1 in the rank's
// own exchange buffer and leaves NaN in out[0].  As a backstop that does
// not depend on the clock, it also gives up after timeout / 16 polls: every
// poll is an uncached load of far more than 16 ns.
static_assert(kMaxRanks <= 32, "one sending thread per rank in a warp-sized CTA");

template <class Op>
__device__ __forceinline__ void exchange_and_fold(const typename Op::Acc local,
                                                  const PeerArgs& a) {
  using Acc = typename Op::Acc;
  unsigned long long* counter = reinterpret_cast<unsigned long long*>(a.own);
  unsigned int* status = reinterpret_cast<unsigned int*>(a.own + 8);
  unsigned long long* wait_stats = reinterpret_cast<unsigned long long*>(a.own + 16);
  __shared__ unsigned long long x_bits, x_epoch, x_t_send;
  __shared__ unsigned long long x_vals[kMaxRanks];
  __shared__ int x_failed;
  if (threadIdx.x == 0) {
    x_t_send = global_ns();
    x_epoch = *counter + 1;
    *counter = x_epoch;
    x_bits = acc_bits(local);
    x_failed = 0;
  }
  __syncthreads();
  const unsigned long long epoch = x_epoch;
  const int set = (int)(epoch & 1ull) * kMaxRanks;
  const int r = (int)threadIdx.x;
  if (r < a.nranks) {
    const unsigned long long tag = (epoch & 0xffffffffull) << 32;
    ExchangeSlot* s =
        reinterpret_cast<ExchangeSlot*>(a.peers.buf[r] + kExchangeSlotsOffset) + set + a.rank;
    st_relaxed_sys(&s->half[0], tag | (x_bits & 0xffffffffull));
    st_relaxed_sys(&s->half[1], tag | (x_bits >> 32));
    ExchangeSlot* mine = reinterpret_cast<ExchangeSlot*>(a.own + kExchangeSlotsOffset) + set + r;
    const unsigned long long t0 = global_ns();
    const unsigned long long max_polls = a.timeout_ns / 16 + 1;
    unsigned long long polls = 0;
    unsigned long long lo = ld_relaxed_sys(&mine->half[0]);
    unsigned long long hi = ld_relaxed_sys(&mine->half[1]);
    bool ok = true;
    while ((lo & ~0xffffffffull) != tag || (hi & ~0xffffffffull) != tag) {
      if (++polls > max_polls || global_ns() - t0 > a.timeout_ns) {
        ok = false;
        break;
      }
      __nanosleep(32);
      lo = ld_relaxed_sys(&mine->half[0]);
      hi = ld_relaxed_sys(&mine->half[1]);
    }
    if (ok) x_vals[r] = ((hi & 0xffffffffull) << 32) | (lo & 0xffffffffull);
    else x_failed = 1;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  if (x_failed) {
    atomicExch(status, 1u);
    a.out[0] = __int_as_float(0x7fffffff);  // NaN: no result
    return;
  }
  Acc total = Op::init();
  for (int q = 0; q < a.nranks; ++q) total = Op::combine(total, bits_acc<Acc>(x_vals[q]));
  a.out[0] = Op::to_float(total);
  const unsigned long long waited = global_ns() - x_t_send;
  wait_stats[0] += waited;
  if (waited > wait_stats[1]) wait_stats[1] = waited;
  wait_stats[2] += 1;
}

// The exchange after a first stage that left this rank's value in `local`
// (a one-CTA or one-cluster grid); one CTA of 32 threads.
template <class Op>
__global__ void peer_exchange_kernel(const typename Op::Acc* __restrict__ local,
                                     const PeerArgs a) {
  wait_for_prerequisite_grid();
  exchange_and_fold<Op>(threadIdx.x == 0 ? *local : Op::init(), a);
}

// The finalize and the exchange in one kernel: the CTA folds this rank's
// partials, then exchanges the total with the other ranks over NVLink and
// folds theirs.
template <class Op>
__global__ void __launch_bounds__(kFinalizeThreads)
finalize_exchange_kernel(const typename Op::Acc* __restrict__ partials, const int count,
                         const PeerArgs a) {
  wait_for_prerequisite_grid();
  allow_dependent_launch();
  const typename Op::Acc acc = fold_partials<Op>(partials, count);
  exchange_and_fold<Op>(acc, a);
}

// A one-CTA kernel as a programmatic dependent of the kernel before it on
// the stream (its griddepcontrol.wait holds it until that one has finished);
// a plain launch where the attribute is refused.
template <class Kern, class... Args>
inline int launch_dependent_cta(Kern kernel, int threads, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess) return LOOM_STATUS_OK;
  cudaGetLastError();
  kernel<<<1, threads, 0, stream>>>(args...);
  return launch_status();
}

// This rank's shard reduced and exchanged through peer memory: the first
// stage, then either the fused finalize-and-exchange CTA (when the stage
// left partials) or the exchange kernel alone.  An empty shard exchanges
// Op's identity.
template <class Op, class Body>
inline int dist_local_exchange(const Ptrs<Body::kInputs>& in, int64_t n_local, const Body& body,
                               void* workspace, float* out, const Comm* comm,
                               cudaStream_t stream) {
  RankSlots<Op> slots(workspace, n_local);
  auto* partials = reinterpret_cast<typename Op::Acc*>(workspace_base(workspace));
  const PeerArgs a = peer_args(comm, out);
  if (n_local == 0)
    return launch_dependent_cta(finalize_exchange_kernel<Op>, kFinalizeThreads, stream,
                                static_cast<const typename Op::Acc*>(partials), 0, a);
  unsigned pending = 0;
  const int st = launch_reduce_stage<Op>(in, n_local, body, partials, partial_capacity(n_local),
                                         nullptr, slots.local, stream, &pending);
  if (st != LOOM_STATUS_OK) return st;
  if (pending == 0)
    return launch_dependent_cta(peer_exchange_kernel<Op>, 32, stream,
                                static_cast<const typename Op::Acc*>(slots.local), a);
  return launch_dependent_cta(finalize_exchange_kernel<Op>, kFinalizeThreads, stream,
                              static_cast<const typename Op::Acc*>(partials), (int)pending, a);
}

template <class Op, class Body>
inline int dist_reduce(const Ptrs<Body::kInputs>& in, int64_t n_local, const Body& body,
                       void* workspace, float* out, Comm* comm, cudaStream_t stream) {
  if (comm->peer_exchange)
    return dist_local_exchange<Op>(in, n_local, body, workspace, out, comm, stream);
  int st = dist_local<Op>(in, n_local, body, workspace, stream);
  if (st != LOOM_STATUS_OK) return st;
  st = dist_collective<Op>(workspace, n_local, out, comm, stream);
  if (st != LOOM_STATUS_OK) return st;
  return dist_finish<Op>(workspace, n_local, out, comm, stream);
}

// Whether every communicator of a one-process group exchanges through peer
// memory (else the group uses NCCL).
inline bool all_peer_exchange(int ndev, void* const* comms) {
  for (int d = 0; d < ndev; ++d)
    if (!static_cast<Comm*>(comms[d])->peer_exchange) return false;
  return true;
}

// One process, ndev GPUs, on the NCCL path, after the local phase on every
// device: one grouped NCCL collective and the rank fold on every device.
template <class Op>
inline int multi_nccl_exchange(int ndev, void* const* comms, void* const* workspace,
                               const int64_t* shard_n, float* const* out) {
  if (nccl_group_start() != 0) return LOOM_STATUS_COMM_ERROR;
  int group_status = LOOM_STATUS_OK;
  for (int d = 0; d < ndev && group_status == LOOM_STATUS_OK; ++d) {
    group_status = dist_collective<Op>(workspace[d], shard_n[d], out[d],
                                       static_cast<Comm*>(comms[d]), nullptr);
  }
  if (nccl_group_end() != 0) return LOOM_STATUS_COMM_ERROR;
  if (group_status != LOOM_STATUS_OK) return group_status;
  for (int d = 0; d < ndev; ++d) {
    Comm* c = static_cast<Comm*>(comms[d]);
    if (cudaSetDevice(c->device) != cudaSuccess) return LOOM_STATUS_CUDA_ERROR;
    const int st = dist_finish<Op>(workspace[d], shard_n[d], out[d], c, nullptr);
    if (st != LOOM_STATUS_OK) return st;
  }
  return LOOM_STATUS_OK;
}

}  // namespace loomb
