// TEST INFRASTRUCTURE ONLY: the replay driver (tests/native/replay_ops.h)
// over the reference's own classes, compiled into oracle/_ref/libqvp_ref.so.
#include <cstring>

#define REPLAY_MAKE_ALLOCATOR(cfg) new qwenvl_paged::MemoryAllocator((cfg))
#include "replay_ops.h"

extern "C" __attribute__((visibility("default"))) int ref_replay(const char* script, char* out, size_t cap) {
    const std::string t = replay::run(script);
    if (t.size() + 1 > cap) return -static_cast<int>(t.size() + 1);
    std::memcpy(out, t.c_str(), t.size() + 1);
    return static_cast<int>(t.size());
}
