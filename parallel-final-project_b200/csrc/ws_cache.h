// ws_cache.h — the per-(device, stream) scratch cache behind the reference-
// signature launchers, which have no workspace argument (reference
// include/attention.h:6-35).  Host-only and header-only, so that its
// threading behaviour is tested on the CPU against a fake allocator.
//
// The launchers are reentrant from any host thread.  A thread takes the
// buffer's address under the mutex and enqueues its kernel after releasing
// it, so a buffer that has been handed out may be used by a launch at any
// later time.  The cache therefore never frees a buffer: when a larger shape
// needs more scratch, the current buffer is retired (kept allocated until the
// process exits) and a new one of at least twice the size replaces it, so the
// retired buffers add up to less than the live one.  Launches on one stream
// run in order, and each buffer starts zeroed and is left zeroed by every
// kernel that uses it, so whichever buffer a launch got is in the state the
// kernels expect.
#pragma once

#include <cstddef>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

namespace tqkv {

// Alloc provides `void* alloc(int device, Stream stream, size_t bytes)`: a
// new buffer, zero-filled in stream order, or nullptr on failure.
template <typename Stream, typename Alloc>
class WorkspaceCache {
  public:
    explicit WorkspaceCache(Alloc alloc) : alloc_(std::move(alloc)) {}
    WorkspaceCache(const WorkspaceCache&) = delete;
    WorkspaceCache& operator=(const WorkspaceCache&) = delete;

    // A buffer of at least `bytes` for (device, stream); nullptr on failure.
    void* get(int device, Stream stream, size_t bytes) {
        if (bytes == 0) return nullptr;
        std::lock_guard<std::mutex> lock(mu_);
        Entry& e = entries_[{device, stream}];
        if (e.bytes >= bytes) return e.ptr;
        size_t grow = e.bytes * 2;
        if (grow < bytes) grow = bytes;
        void* p = alloc_(device, stream, grow);
        if (p == nullptr) return nullptr;
        if (e.ptr != nullptr) retired_.push_back(e.ptr);  // may still be in use: never freed
        e.ptr = p;
        e.bytes = grow;
        return p;
    }

    size_t retired_count() {
        std::lock_guard<std::mutex> lock(mu_);
        return retired_.size();
    }

  private:
    struct Entry {
        void* ptr = nullptr;
        size_t bytes = 0;
    };
    Alloc alloc_;
    std::mutex mu_;
    std::map<std::pair<int, Stream>, Entry> entries_;
    std::vector<void*> retired_;
};

}  // namespace tqkv
