// TEST INFRASTRUCTURE: the replay driver over this library's host layer, with
// a bookkeeping-only pool (no device storage), so it runs without a GPU.
#include <cstring>

#define REPLAY_MAKE_ALLOCATOR(cfg) \
    new qwenvl_paged::MemoryAllocator((cfg), qwenvl_paged::DevicePoolOptions{-1, false, nullptr})
#include "replay_ops.h"

extern "C" __attribute__((visibility("default"))) int qvp_replay(const char* script, char* out, size_t cap) {
    const std::string t = replay::run(script);
    if (t.size() + 1 > cap) return -static_cast<int>(t.size() + 1);
    std::memcpy(out, t.c_str(), t.size() + 1);
    return static_cast<int>(t.size());
}
