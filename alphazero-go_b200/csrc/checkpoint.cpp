// The reference's network checkpoint (.azn) read into the engine's weight
// arenas, for hosts that hold no reference Network (src/checkpoint.cpp,
// include/azgo/checkpoint.hpp:12-23, include/azgo/serialize.hpp).
//
// Format, all little-endian: u32 magic 0x4F475A41 ("AZGO"), u32 version (1,
// or 2 with an ownership flag), five i32 (board, history, blocks, filters,
// value_hidden), in version 2 an i32 ownership flag (0 or 1), u32 tensor
// count, then per tensor: u32 name length, the name's bytes, u64 float
// count, the floats. Tensors come in params() order, then buffers() order,
// i.e. the order of the engine's layout for the same shape.
//
// Errors carry the reference loader's messages (src/checkpoint.cpp:36-143):
// "cannot open checkpoint <path>", "<path>: not an AZGO checkpoint",
// "<path>: unsupported version N", "<path>: invalid ownership flag in header",
// "<path>: invalid network shape in header", "<path>: has N tensors but the
// network needs M", "<path>: tensor I is 'x' but expected 'y'", "<path>:
// tensor 'x' has N values but expected M", "<path>: unexpected data after
// the last tensor", and "<path>: truncated" for a file that ends early.
#include <cstdint>
#include <cstring>
#include <fstream>
#include <iterator>
#include <stdexcept>
#include <string>
#include <vector>

#include "azb200.h"
#include "engine.hpp"

namespace azb {
namespace {

constexpr uint32_t kMagic = 0x4F475A41u;
constexpr uint32_t kVersionPlain = 1, kVersionOwnership = 2;
// The shape limits the reference's loader accepts (include/azgo/config.hpp:20-21,
// src/checkpoint.cpp:52-58).
constexpr int kMaxBlocks = 40, kMaxFilters = 512;

struct FormatError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct Truncated {};

class Reader {
public:
    explicit Reader(const std::vector<uint8_t>& data) : d_(data) {}
    uint32_t u32() {
        need(4);
        uint32_t v = 0;
        for (int k = 3; k >= 0; --k) v = (v << 8) | d_[at_ + size_t(k)];
        at_ += 4;
        return v;
    }
    uint64_t u64() {
        const uint64_t lo = u32();
        return lo | (uint64_t(u32()) << 32);
    }
    int32_t i32() { return static_cast<int32_t>(u32()); }
    std::string str() {
        const uint32_t n = u32();
        need(n);
        std::string s(reinterpret_cast<const char*>(d_.data() + at_), n);
        at_ += n;
        return s;
    }
    void floats(float* dst, size_t n) {
        need(n * 4);
        for (size_t i = 0; i < n; ++i) {
            const uint32_t bits = u32();
            std::memcpy(dst + i, &bits, 4);
        }
    }
    bool at_end() const { return at_ == d_.size(); }

private:
    void need(size_t n) const {
        if (d_.size() - at_ < n) throw Truncated{};
    }
    const std::vector<uint8_t>& d_;
    size_t at_ = 0;
};

std::vector<uint8_t> read_file(const std::string& path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error("cannot open checkpoint " + path);
    return std::vector<uint8_t>(std::istreambuf_iterator<char>(in), std::istreambuf_iterator<char>());
}

azb_net_desc read_header(Reader& r) {
    if (r.u32() != kMagic) throw FormatError("not an AZGO checkpoint");
    const uint32_t version = r.u32();
    if (version != kVersionPlain && version != kVersionOwnership)
        throw FormatError("unsupported version " + std::to_string(version));
    azb_net_desc d{};
    d.board = r.i32();
    d.history = r.i32();
    d.blocks = r.i32();
    d.filters = r.i32();
    d.value_hidden = r.i32();
    d.ownership = 0;
    if (version == kVersionOwnership) {
        const int32_t flag = r.i32();
        if (flag != 0 && flag != 1) throw FormatError("invalid ownership flag in header");
        d.ownership = flag;
    }
    if (d.board < 5 || d.board > 19 || d.history < 1 || d.history > 16 || d.blocks < 0 || d.blocks > kMaxBlocks ||
        d.filters < 1 || d.filters > kMaxFilters || d.value_hidden < 1 || d.value_hidden > 1024)
        throw FormatError("invalid network shape in header");
    return d;
}

// Runs body on the file's reader, turning every failure into the
// reference's message for it.
template <class Body>
void with_checkpoint(const std::string& path, Body body) {
    const std::vector<uint8_t> data = read_file(path);
    Reader r(data);
    try {
        body(r);
    } catch (const FormatError& e) {
        throw std::runtime_error(path + ": " + e.what());
    } catch (const Truncated&) {
        throw std::runtime_error(path + ": truncated");
    }
}

// The names, sizes and offsets for any shape a header can hold; the
// engine's own limits apply when a runner is made.
Layout layout_of(const azb_net_desc& d) {
    return Layout::of(NetShape{d.board, d.history, d.blocks, d.filters, d.value_hidden, d.ownership != 0});
}

void put(char* dst, size_t cap, const std::string& s) {
    if (dst && cap) {
        const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
        std::memcpy(dst, s.data(), n);
        dst[n] = '\0';
    }
}

} // namespace
} // namespace azb

using namespace azb;

extern "C" {

int azb_checkpoint_config(const char* path, azb_net_desc* desc, size_t* n_params, size_t* n_buffers, char* err,
                          size_t err_cap) {
    try {
        if (!path || !desc) throw std::invalid_argument("azb_checkpoint_config: null argument");
        with_checkpoint(path, [&](Reader& r) { *desc = read_header(r); });
        const Layout L = layout_of(*desc);
        if (n_params) *n_params = L.param_floats;
        if (n_buffers) *n_buffers = L.buffer_floats;
        return 0;
    } catch (const std::exception& e) {
        put(err, err_cap, e.what());
        return -1;
    }
}

int azb_checkpoint_read(const char* path, azb_net_desc* desc, float* params, size_t n_params, float* buffers,
                        size_t n_buffers, char* err, size_t err_cap) {
    try {
        if (!path || !desc || !params || !buffers) throw std::invalid_argument("azb_checkpoint_read: null argument");
        with_checkpoint(path, [&](Reader& r) {
            const azb_net_desc d = read_header(r);
            const Layout L = layout_of(d);
            if (n_params != L.param_floats || n_buffers != L.buffer_floats)
                throw std::invalid_argument("azb_checkpoint_read: arenas of " + std::to_string(n_params) + " and " +
                                            std::to_string(n_buffers) + " floats; the checkpoint's layout needs " +
                                            std::to_string(L.param_floats) + " and " +
                                            std::to_string(L.buffer_floats));
            const size_t total = L.params.size() + L.buffers.size();
            const uint32_t count = r.u32();
            if (count != total)
                throw FormatError("has " + std::to_string(count) + " tensors but the network needs " +
                                  std::to_string(total));
            std::memset(params, 0, n_params * sizeof(float));
            std::memset(buffers, 0, n_buffers * sizeof(float));
            for (size_t i = 0; i < total; ++i) {
                const bool is_param = i < L.params.size();
                const LayoutEntry& e = is_param ? L.params[i] : L.buffers[i - L.params.size()];
                const std::string name = r.str();
                if (name != e.name)
                    throw FormatError("tensor " + std::to_string(i) + " is '" + name + "' but expected '" + e.name +
                                      "'");
                const uint64_t size = r.u64();
                if (size != e.size)
                    throw FormatError("tensor '" + name + "' has " + std::to_string(size) + " values but expected " +
                                      std::to_string(e.size));
                r.floats((is_param ? params : buffers) + e.offset, e.size);
            }
            if (!r.at_end()) throw FormatError("unexpected data after the last tensor");
            *desc = d;
        });
        return 0;
    } catch (const std::exception& e) {
        put(err, err_cap, e.what());
        return -1;
    }
}

} // extern "C"
