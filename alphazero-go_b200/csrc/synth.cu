// Seeded synthetic networks and positions for benchmarks and tests: the
// same networks and inputs the reference builds from a seed, so a run here
// and a run of the reference's CPU engine evaluate identical bits.
//
//   * xoshiro256** seeded by splitmix64 (Blackman & Vigna; the generator of
//     robominds/alphazero-go src/rng.cpp:19-86), uniform() from the top 53
//     bits, below(n) by Lemire's multiply-shift with rejection, normal() by
//     Box-Muller without a cached second value;
//   * Network(cfg, seed): He-normal conv and linear weights in parameter
//     order, zero biases, identity batch norm (src/network.cpp:77-111);
//   * batch-norm randomisers: kind 0 (benchmark) gamma ~ U(0.5,1.5),
//     beta ~ N(0,0.1), running mean ~ N(0,0.1), running var ~ U(0.5,1.5)
//     from Rng(deriveSeed(seed, 1)); kind 1 (tests) as the reference test
//     suite's randomNetwork (tests/test_cuda.cpp:188-204);
//   * positions: per sample Rng(deriveSeed(seed, 2, index)), side to move,
//     then each point occupied with probability 0.4 and coloured 50/50,
//     encoded as encodePlanes does with one history position
//     (src/encode.cpp:14-43).
#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>

#include "../../include/azb200.h"
#include "engine.hpp"

namespace {

uint64_t splitmix(uint64_t& x) {
    uint64_t z = (x += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

uint64_t derive(uint64_t a, uint64_t b = 0, uint64_t c = 0, uint64_t d = 0) {
    uint64_t h = 0x243F6A8885A308D3ULL;
    for (uint64_t v : {a, b, c, d}) {
        uint64_t x = h ^ v;
        h = splitmix(x);
    }
    return h;
}

class Xoshiro {
public:
    explicit Xoshiro(uint64_t seed) {
        uint64_t x = seed;
        for (uint64_t& w : s_) w = splitmix(x);
    }
    uint64_t next() {
        const uint64_t r = rotl(s_[1] * 5, 7) * 9;
        const uint64_t t = s_[1] << 17;
        s_[2] ^= s_[0];
        s_[3] ^= s_[1];
        s_[1] ^= s_[2];
        s_[0] ^= s_[3];
        s_[2] ^= t;
        s_[3] = rotl(s_[3], 45);
        return r;
    }
    double uniform() { return static_cast<double>(next() >> 11) * 0x1.0p-53; }
    int below(int n) {
        const uint32_t range = static_cast<uint32_t>(n);
        uint64_t m = (next() >> 32) * range;
        uint32_t low = static_cast<uint32_t>(m);
        if (low < range) {
            const uint32_t threshold = (0u - range) % range;
            while (low < threshold) {
                m = (next() >> 32) * range;
                low = static_cast<uint32_t>(m);
            }
        }
        return static_cast<int>(m >> 32);
    }
    double normal() {
        const double u1 = 1.0 - uniform();
        const double u2 = uniform();
        return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586476925286766559 * u2);
    }

private:
    static uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
    uint64_t s_[4];
};

bool ends_with(const std::string& s, const char* tail) {
    const size_t n = std::strlen(tail);
    return s.size() >= n && s.compare(s.size() - n, n, tail) == 0;
}

bool is_weight(const std::string& n) { return ends_with(n, ".w"); }

int fan_in(const azb::NetShape& s, const std::string& n) {
    if (n == "stem.conv.w") return s.planes() * 9;
    if (n.compare(0, 5, "block") == 0) return s.filters * 9;
    if (n == "policy.fc.w") return 2 * s.area();
    if (n == "value.fc1.w") return s.area();
    if (n == "value.fc2.w") return s.value_hidden;
    return s.filters;   // the heads' 1x1 convolutions
}

} // namespace

extern "C" {

int azb_synth_network(const azb_net_desc* desc, uint64_t seed, int kind, float* params, float* buffers) {
    try {
        const azb::NetShape s = azb::NetShape::from(*desc);
        const azb::Layout L = azb::Layout::of(s);
        std::memset(params, 0, L.param_floats * sizeof(float));
        std::memset(buffers, 0, L.buffer_floats * sizeof(float));
        Xoshiro init(seed);
        // Weights in parameter order, which is the reference's init order
        // (the ownership conv, listed last, is also drawn last).
        for (const azb::LayoutEntry& e : L.params) {
            float* v = params + e.offset;
            if (is_weight(e.name)) {
                const double sd = std::sqrt(2.0 / fan_in(s, e.name));
                for (size_t i = 0; i < e.size; ++i) v[i] = static_cast<float>(init.normal() * sd);
            } else if (ends_with(e.name, ".gamma")) {
                for (size_t i = 0; i < e.size; ++i) v[i] = 1.0f;
            }
        }
        for (const azb::LayoutEntry& e : L.buffers)
            if (ends_with(e.name, ".runVar"))
                for (size_t i = 0; i < e.size; ++i) buffers[e.offset + i] = 1.0f;
        if (kind < 0) return 0;
        Xoshiro r(kind == 0 ? derive(seed, 1) : seed + 17);
        for (const azb::LayoutEntry& e : L.params) {
            float* v = params + e.offset;
            if (ends_with(e.name, ".gamma")) {
                for (size_t i = 0; i < e.size; ++i) v[i] = static_cast<float>(0.5 + r.uniform());
            } else if (!is_weight(e.name)) {   // beta and linear biases
                if (kind == 0) {
                    if (ends_with(e.name, ".beta"))
                        for (size_t i = 0; i < e.size; ++i) v[i] = static_cast<float>(0.1 * r.normal());
                } else {
                    for (size_t i = 0; i < e.size; ++i) v[i] = static_cast<float>(0.4 * r.uniform() - 0.2);
                }
            }
        }
        for (const azb::LayoutEntry& e : L.buffers) {
            float* v = buffers + e.offset;
            const bool var = ends_with(e.name, ".runVar");
            for (size_t i = 0; i < e.size; ++i) {
                if (var) v[i] = static_cast<float>(0.5 + r.uniform());
                else v[i] = kind == 0 ? static_cast<float>(0.1 * r.normal()) : static_cast<float>(0.4 * r.uniform() - 0.2);
            }
        }
        return 0;
    } catch (...) {
        return -1;
    }
}

int azb_synth_positions(const azb_net_desc* desc, uint64_t seed, long first, int B, float* out) {
    try {
        const azb::NetShape s = azb::NetShape::from(*desc);
        const int A = s.area(), P = s.planes();
        for (int b = 0; b < B; ++b) {
            Xoshiro r(derive(seed, 2, static_cast<uint64_t>(first + b)));
            float* x = out + size_t(b) * P * A;
            std::memset(x, 0, size_t(P) * A * sizeof(float));
            const int to_move = r.below(2);   // 0 black, 1 white
            for (int p = 0; p < A; ++p)
                if (r.uniform() < 0.4) x[size_t(r.below(2) == to_move ? 0 : 1) * A + p] = 1.0f;
            float* plane = x + size_t(2 * s.history + to_move) * A;
            for (int p = 0; p < A; ++p) plane[p] = 1.0f;
        }
        return 0;
    } catch (...) {
        return -1;
    }
}

int azb_device_pci_bus_id(int device, char* out, size_t cap) {
    char buf[64] = {};
    if (cudaDeviceGetPCIBusId(buf, sizeof buf, device) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    std::strncpy(out, buf, cap);
    if (cap) out[cap - 1] = '\0';
    return 0;
}

} // extern "C"
