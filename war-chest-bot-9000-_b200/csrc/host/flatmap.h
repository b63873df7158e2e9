// A 64-bit key -> 32-bit value table with open addressing (linear probing,
// at most half full), for the builder's lookups on its hot paths. Keys
// never have all 64 bits set: that value marks a free slot.
#pragma once

#include <cstddef>
#include <cstdint>
#include <utility>
#include <vector>

namespace wc {

struct FlatMap {
    static constexpr uint64_t FREE = ~0ull;
    std::vector<uint64_t> keys;
    std::vector<uint32_t> vals;
    size_t used = 0;

    static uint64_t mix(uint64_t x) {  // the splitmix64 finaliser
        x ^= x >> 30;
        x *= 0xbf58476d1ce4e5b9ull;
        x ^= x >> 27;
        x *= 0x94d049bb133111ebull;
        return x ^ (x >> 31);
    }
    // the value of `key`, or nullptr
    const uint32_t* find(uint64_t key) const {
        if (keys.empty()) return nullptr;
        const size_t mask = keys.size() - 1;
        for (size_t i = mix(key) & mask;; i = (i + 1) & mask) {
            if (keys[i] == key) return &vals[i];
            if (keys[i] == FREE) return nullptr;
        }
    }
    void insert(uint64_t key, uint32_t v) {  // key not present
        if (2 * (used + 1) > keys.size()) grow();
        const size_t mask = keys.size() - 1;
        size_t i = mix(key) & mask;
        while (keys[i] != FREE) i = (i + 1) & mask;
        keys[i] = key;
        vals[i] = v;
        ++used;
    }
    void grow() {
        std::vector<uint64_t> ok = std::move(keys);
        std::vector<uint32_t> ov = std::move(vals);
        keys.assign(ok.empty() ? 1024 : 2 * ok.size(), FREE);
        vals.assign(keys.size(), 0);
        used = 0;
        for (size_t i = 0; i < ok.size(); ++i)
            if (ok[i] != FREE) insert(ok[i], ov[i]);
    }
};

}  // namespace wc
