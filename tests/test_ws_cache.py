"""The scratch cache behind the reference-signature launchers
(parallel-final-project_b200/csrc/ws_cache.h), on the CPU with a fake
allocator.

The launchers take no workspace argument and may be called from any host
thread.  A thread takes a buffer from the cache under its mutex and enqueues
its kernel afterwards, so the cache must never free a buffer it has handed
out, even when another thread grows it in between.  Eight threads ask for
growing and shrinking sizes on shared (device, stream) keys; each checks,
after the cache's lock is released and again a little later (where its
kernel would run), that its buffer is still allocated and large enough.  The
retired buffers must add up to less than the live ones (geometric growth)."""
import os
import subprocess
import tempfile

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(REPO, "parallel-final-project_b200", "csrc")

PROG = r'''
#include "ws_cache.h"
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <random>
#include <set>
#include <thread>
#include <vector>

struct Live {
    std::mutex mu;
    std::set<std::pair<char*, size_t>> bufs;
    size_t total = 0;
};
static Live g_live;

struct FakeAlloc {
    void* operator()(int, int, size_t bytes) const {
        char* p = static_cast<char*>(std::calloc(bytes, 1));
        std::lock_guard<std::mutex> lock(g_live.mu);
        g_live.bufs.insert({p, bytes});
        g_live.total += bytes;
        return p;
    }
};

static bool live_and_big(void* p, size_t need) {
    std::lock_guard<std::mutex> lock(g_live.mu);
    for (auto& b : g_live.bufs)
        if (b.first == p) return b.second >= need;
    return false;
}

int main() {
    tqkv::WorkspaceCache<int, FakeAlloc> cache{FakeAlloc{}};
    std::atomic<int> bad{0};
    std::vector<std::thread> ts;
    for (int t = 0; t < 8; ++t) {
        ts.emplace_back([&, t] {
            std::mt19937 rng(1234 + t);
            for (int i = 0; i < 20000; ++i) {
                const int stream = static_cast<int>(rng() % 2);   // two streams, shared
                const size_t need = 1 + rng() % (64 + 64 * static_cast<size_t>(i));
                void* p = cache.get(0, stream, need);
                if (!p || !live_and_big(p, need)) ++bad;
                std::this_thread::yield();          // another thread may grow the cache now
                if (!live_and_big(p, need)) ++bad;  // where the launch would use it
            }
        });
    }
    for (auto& th : ts) th.join();
    size_t live_max = 0;
    for (int s = 0; s < 2; ++s) {
        void* p = cache.get(0, s, 1);
        std::lock_guard<std::mutex> lock(g_live.mu);
        for (auto& b : g_live.bufs)
            if (b.first == p) live_max += b.second;
    }
    std::printf("%d %zu %zu %zu\n", bad.load(), cache.retired_count(), g_live.total, live_max);
    return 0;
}
'''


def test_cache_never_frees_a_buffer_it_handed_out():
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "t.cpp"), os.path.join(d, "t")
        with open(src, "w") as f:
            f.write(PROG)
        subprocess.run(["g++", "-O1", "-std=c++17", "-pthread", "-I", CSRC, src, "-o", exe],
                       check=True)
        r = subprocess.run([exe], capture_output=True, text=True, timeout=120, check=True)
    bad, retired, total, live = (int(x) for x in r.stdout.split())
    assert bad == 0
    assert retired > 0                 # the cache did grow while threads held buffers
    assert total - live < live         # retired buffers add up to less than the live ones
