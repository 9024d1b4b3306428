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

struct Comm {
  ncclComm_t nccl = nullptr;
  int nranks = 0;
  int rank = 0;
  int device = 0;
};

// Restores the caller's current device when it goes out of scope.
struct DeviceGuard {
  int device = -1;
  DeviceGuard() { cudaGetDevice(&device); }
  ~DeviceGuard() {
    if (device >= 0) cudaSetDevice(device);
  }
};

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
  return LOOM_STATUS_OK;
}

inline int comm_destroy(void* comm) {
  if (comm == nullptr) return LOOM_STATUS_OK;
  Comm* c = static_cast<Comm*>(comm);
  const ncclResult_t r = ncclCommDestroy(c->nccl);
  delete c;
  return r == ncclSuccess ? LOOM_STATUS_OK : LOOM_STATUS_COMM_ERROR;
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

template <class Op, class Body>
inline int dist_reduce(const Ptrs<Body::kInputs>& in, int64_t n_local, const Body& body,
                       void* workspace, float* out, Comm* comm, cudaStream_t stream) {
  int st = dist_local<Op>(in, n_local, body, workspace, stream);
  if (st != LOOM_STATUS_OK) return st;
  st = dist_collective<Op>(workspace, n_local, out, comm, stream);
  if (st != LOOM_STATUS_OK) return st;
  return dist_finish<Op>(workspace, n_local, out, comm, stream);
}

}  // namespace loomb
