// Per-device scratch arena for the drop-in (`void reference(...)`-shaped) entry points.
//
// The reference ABI gives a kernel no workspace argument (tasks/FORMAT.md:35), so ops that need
// scratch (grid-reduction partials and their control words) take it from this arena.  The arena is
// allocated with cudaMalloc on the first call on a device, grows when a larger call needs it, and
// is never freed before process exit; after the first call at a given size a call performs no
// allocation.  Fresh memory is zero-filled on the caller's stream before first use.
//
// Each op has its own slot (ArenaClient), because ops keep state in their scratch between calls
// (the reductions' control words carry over from one call to the next).  Calls of one op that share
// its slot must not overlap on the GPU: issue them on one stream, or order them with events.
// The stream forms in the C ABI that take a caller workspace have no such restriction beyond the
// usual one for the workspace they are given.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <mutex>

#include "b200_common.cuh"

namespace b200 {

struct ArenaSlot {
  void* ptr = nullptr;
  size_t bytes = 0;
};

inline std::mutex& arena_mutex() {
  static std::mutex m;
  return m;
}

enum ArenaClient : int { kArenaRobustL1 = 0, kArenaPpo = 1, kArenaKan = 2, kArenaClients = 3 };

inline ArenaSlot* arena_slots() {
  static ArenaSlot slots[64 * kArenaClients];
  return slots;
}

// Returns a zero-initialised-at-allocation device buffer of at least `bytes` bytes for the
// current device and the given client, or nullptr with *status set.  Contents persist between
// calls.
inline void* arena_get(ArenaClient client, size_t bytes, cudaStream_t stream, int* status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = kCudaError;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(arena_mutex());
  ArenaSlot& slot = arena_slots()[dev * kArenaClients + client];
  if (slot.bytes >= bytes && slot.ptr != nullptr) {
    *status = kOk;
    return slot.ptr;
  }
  size_t want = bytes < 4096 ? 4096 : bytes;
  if (slot.ptr != nullptr) {
    // cudaFree waits for the device to finish work that may still use the old buffer.
    cudaFree(slot.ptr);
    slot.ptr = nullptr;
    slot.bytes = 0;
  }
  void* p = nullptr;
  if (cudaMalloc(&p, want) != cudaSuccess) {
    *status = kCudaError;
    return nullptr;
  }
  if (cudaMemsetAsync(p, 0, want, stream) != cudaSuccess) {
    cudaFree(p);
    *status = kCudaError;
    return nullptr;
  }
  slot.ptr = p;
  slot.bytes = want;
  *status = kOk;
  return p;
}

// Round a byte count up to a 256-byte boundary (keeps every workspace sub-buffer aligned).
constexpr size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

}  // namespace b200
