// A small table from a device-context id to a device address, for the
// library-owned scratch arrays of the allocation-free entry points.
//
// A `__device__` array has one address per CUDA context (the module is loaded
// into each context separately).  Keying the cached address by the device
// number alone goes stale when that device's context changes: after
// cudaDeviceReset the primary context is destroyed and a new one is created on
// next use, and a host may make its own driver-API context current on the same
// device.  The key here is the driver's context id (cuCtxGetId), which is
// unique for the life of the process and never reused, so a new context always
// misses and its address is looked up again.
//
// Plain host C++ (no CUDA types): the CPU test suite compiles it on its own.
#pragma once

#include <cstdint>
#include <mutex>

namespace walsh {

template <int kEntries>
class ContextAddressCache {
 public:
  // The address stored for context `id`, or nullptr.
  void* find(uint64_t id) {
    if (id == 0) return nullptr;
    std::lock_guard<std::mutex> lock(mu_);
    for (int i = 0; i < n_; ++i)
      if (ids_[i] == id) return ptrs_[i];
    return nullptr;
  }

  // Store (id, p); replaces an entry with the same id, else takes a free slot,
  // else the oldest entry (contexts that were destroyed are never asked for
  // again, so evicting them is harmless).
  void insert(uint64_t id, void* p) {
    if (id == 0 || p == nullptr) return;
    std::lock_guard<std::mutex> lock(mu_);
    for (int i = 0; i < n_; ++i)
      if (ids_[i] == id) {
        ptrs_[i] = p;
        return;
      }
    int slot;
    if (n_ < kEntries) {
      slot = n_++;
    } else {
      slot = next_evict_;
      next_evict_ = (next_evict_ + 1) % kEntries;
    }
    ids_[slot] = id;
    ptrs_[slot] = p;
  }

  int size() {
    std::lock_guard<std::mutex> lock(mu_);
    return n_;
  }

 private:
  std::mutex mu_;
  uint64_t ids_[kEntries] = {};
  void* ptrs_[kEntries] = {};
  int n_ = 0;
  int next_evict_ = 0;
};

}  // namespace walsh
