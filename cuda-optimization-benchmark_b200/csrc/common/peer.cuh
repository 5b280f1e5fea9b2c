// Peer exchange of fixed-size records among the ranks of one node, one process per GPU, over
// NVLink / NVSwitch peer memory (CUDA IPC mappings; plain 16-byte stores and loads, no switch
// reduction, no collective library).
//
// Every rank owns one device buffer of records [2 halves][world][slots], half = epoch & 1.  Records
// travel in LL form (ll.cuh): every 4-byte word with the epoch in one 8-byte value, so a record is
// pushed to a peer the moment it is computed, with no fence and no ready flag.  Rank `rank` stores
// its records for epoch e into half (e & 1), slot range of `rank`, of the other ranks' buffers;
// each rank reads the others' records from its own buffer, waiting (bounded) on words not yet
// arrived.  The two halves keep a peer's records of epoch e + 1 away from the half still being
// read for epoch e, and a peer cannot reach e + 2 before it has read this rank's e + 1 records,
// which this rank stores only after it has finished reading e.  Epochs start at 1 (the buffer
// starts zeroed) and go up by one a step, skipping 0 on wrap-around without repeating a half.
//
// The ranks exchange their 64-byte CUDA IPC handles through the caller's own channel (the Python
// side uses torch.distributed) and open one another's buffers with peer_open().
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "b200_common.cuh"
#include "bulk.cuh"
#include "ll.cuh"

namespace b200 {

constexpr int kMaxPeers = 64;
constexpr size_t kPeerHandleBytes = sizeof(cudaIpcMemHandle_t);  // 64

struct PeerExchange {
  int world = 0, rank = 0, device = 0;
  int64_t slots = 0;      // records per rank
  size_t rec_bytes = 0;   // one record in LL form: 8 bytes per 4-byte payload word
  size_t half_bytes = 0;  // world * slots * rec_bytes
  char* local = nullptr;  // this rank's buffer
  char* base[kMaxPeers] = {};
  bool opened[kMaxPeers] = {};
  char** base_dev = nullptr;  // device copy of base[]
};

inline int peer_create(int world, int rank, int64_t slots, size_t rec_bytes, PeerExchange** out, void* handle_out) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world || slots < 0 || rec_bytes == 0 || rec_bytes % 16 ||
      out == nullptr || handle_out == nullptr)
    return kInvalidArgument;
  PeerExchange* x = new PeerExchange();
  x->world = world;
  x->rank = rank;
  x->slots = slots;
  x->rec_bytes = rec_bytes;
  x->half_bytes = size_t(world) * size_t(slots) * rec_bytes;
  const size_t bytes = 2 * x->half_bytes + 256;  // never a zero-byte allocation
  if (cudaGetDevice(&x->device) != cudaSuccess || cudaMalloc(&x->local, bytes) != cudaSuccess ||
      cudaMemset(x->local, 0, bytes) != cudaSuccess || cudaMalloc(&x->base_dev, sizeof(char*) * world) != cudaSuccess) {
    if (x->local) cudaFree(x->local);
    delete x;
    return kCudaError;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, x->local) != cudaSuccess) {
    cudaFree(x->local);
    cudaFree(x->base_dev);
    delete x;
    return kCudaError;
  }
  memcpy(handle_out, &h, kPeerHandleBytes);
  x->base[rank] = x->local;
  *out = x;
  return kOk;
}

// handles: world * 64 bytes, rank-ordered (this rank's own entry is ignored).
inline int peer_open(PeerExchange* x, const void* handles) {
  if (x == nullptr || handles == nullptr) return kInvalidArgument;
  for (int r = 0; r < x->world; ++r) {
    if (r == x->rank || x->opened[r]) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const char*>(handles) + size_t(r) * kPeerHandleBytes, kPeerHandleBytes);
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return kCudaError;
    x->base[r] = static_cast<char*>(p);
    x->opened[r] = true;
  }
  if (cudaMemcpy(x->base_dev, x->base, sizeof(char*) * x->world, cudaMemcpyHostToDevice) != cudaSuccess)
    return kCudaError;
  return kOk;
}

inline int peer_destroy(PeerExchange* x) {
  if (x == nullptr) return kOk;
  int st = kOk;
  if (cudaDeviceSynchronize() != cudaSuccess) st = kCudaError;
  for (int r = 0; r < x->world; ++r)
    if (x->opened[r] && cudaIpcCloseMemHandle(x->base[r]) != cudaSuccess) st = kCudaError;
  if (x->base_dev) cudaFree(x->base_dev);
  if (x->local) cudaFree(x->local);
  delete x;
  return st;
}

// Device view passed to kernels.
struct PeerView {
  char* const* base;  // every rank's buffer (device array)
  int world, rank;
  int64_t slots;
  size_t rec_bytes, half_bytes;
  unsigned epoch;
};

inline PeerView peer_view(const PeerExchange& x, unsigned epoch) {
  return PeerView{x.base_dev, x.world, x.rank, x.slots, x.rec_bytes, x.half_bytes, epoch};
}

// Record slot `i` of rank `owner` in rank `r`'s buffer, in the half of the view's epoch.
__device__ __forceinline__ ulonglong2* peer_record(const PeerView& v, int r, int owner, int64_t i) {
  return reinterpret_cast<ulonglong2*>(v.base[r] + size_t(v.epoch & 1u) * v.half_bytes +
                                  (size_t(owner) * v.slots + i) * v.rec_bytes);
}

// The epoch after e: e + 1, with 0 (the zeroed buffer's value) skipped by going on to 2, which
// keeps the halves alternating (0xffffffff is odd, 2 is even).
__host__ __device__ __forceinline__ unsigned peer_next_epoch(unsigned e) { return e == 0xffffffffu ? 2u : e + 1u; }

}  // namespace b200
