// kv_cache.h — decode shape helper, same members and element counts as the
// reference's AttnShape (reference include/kv_cache.h:4-14), header-only.
#pragma once
#include <cstddef>

struct AttnShape {
    int B;  // batch
    int H;  // heads
    int S;  // cached tokens per head
    int D;  // head dimension

    size_t q_elems() const { return static_cast<size_t>(B) * H * D; }
    size_t k_elems() const { return static_cast<size_t>(B) * H * S * D; }
    size_t v_elems() const { return k_elems(); }
    size_t o_elems() const { return q_elems(); }
};
