// The reference's network checkpoint (.azn) read straight into the engine's
// weight arenas, for hosts that hold no reference Network (the format of
// saveNetwork / loadNetwork, include/azgo/checkpoint.hpp:12-23,
// src/checkpoint.cpp:80-133, with include/azgo/serialize.hpp's encoding).
//
// Format, all little-endian: u32 magic 0x4F475A41 ("AZGO"), u32 version (1,
// or 2 with an ownership flag), five i32 (board, history, blocks, filters,
// value_hidden), in version 2 an i32 ownership flag (0 or 1), u32 tensor
// count, then per tensor: u32 name length, the name's bytes, u64 float
// count, the floats. Tensors come in params() order, then buffers() order,
// i.e. the order of the engine's layout for the same shape.
//
// The file is mapped read-only and walked once by a bounds-checked view
// whose reads report a short file instead of throwing; each check returns
// a Verdict, so the first problem in file order decides the message, as
// with the reference loader. Float data is copied from the mapping in one
// memcpy per tensor. Messages are the reference loader's
// (src/checkpoint.cpp:36-143): "cannot open checkpoint <path>", "<path>: not
// an AZGO checkpoint", "<path>: unsupported version N", "<path>: invalid
// ownership flag in header", "<path>: invalid network shape in header",
// "<path>: has N tensors but the network needs M", "<path>: tensor I is 'x'
// but expected 'y'", "<path>: tensor 'x' has N values but expected M",
// "<path>: unexpected data after the last tensor", and "<path>: truncated"
// for a file that ends early.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>

#include "azb200.h"
#include "engine.hpp"

static_assert(__BYTE_ORDER__ == __ORDER_LITTLE_ENDIAN__, "the .azn reader copies little-endian data as is");

namespace azb {
namespace {

constexpr uint32_t kMagic = 0x4F475A41u;
constexpr uint32_t kPlainVersion = 1, kOwnershipVersion = 2;

// The header's shape fields in file order, with the ranges the reference's
// loader accepts (src/checkpoint.cpp:52-58; the block and filter limits are
// include/azgo/config.hpp:20-21).
struct ShapeField {
    int azb_net_desc::*member;
    int lo, hi;
};
constexpr ShapeField kShape[] = {
    {&azb_net_desc::board, 5, 19},     {&azb_net_desc::history, 1, 16},      {&azb_net_desc::blocks, 0, 40},
    {&azb_net_desc::filters, 1, 512},  {&azb_net_desc::value_hidden, 1, 1024},
};

// The outcome of one check: fine, the file ended early, or a format problem
// with its text (the path is prefixed where the message is assembled).
struct Verdict {
    enum Kind { kFine, kShort, kBad } kind = kFine;
    std::string text;
    explicit operator bool() const { return kind != kFine; }
};
Verdict fine() { return {}; }
Verdict short_file() { return {Verdict::kShort, {}}; }
Verdict bad(std::string text) { return {Verdict::kBad, std::move(text)}; }

// A read-only view of the mapped file with a cursor. Every take_* returns
// false, leaving the cursor, when fewer bytes remain than it needs.
class ByteView {
public:
    ByteView(const uint8_t* data, size_t size) : data_(data), size_(size) {}
    size_t left() const { return size_ - at_; }
    template <class T>
    bool take(T* out) {
        if (left() < sizeof(T)) return false;
        std::memcpy(out, data_ + at_, sizeof(T));
        at_ += sizeof(T);
        return true;
    }
    bool take_bytes(size_t n, const uint8_t** out) {
        if (left() < n) return false;
        *out = data_ + at_;
        at_ += n;
        return true;
    }

private:
    const uint8_t* data_;
    size_t size_, at_ = 0;
};

// A read-only mapping of a whole file (an empty file is an empty view).
class MappedFile {
public:
    explicit MappedFile(const std::string& path) {
        const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
        struct stat st {};
        if (fd < 0 || ::fstat(fd, &st) != 0) {
            if (fd >= 0) ::close(fd);
            throw std::runtime_error("cannot open checkpoint " + path);
        }
        // Something that opens but holds no readable bytes (a directory)
        // reads as an empty file, which the reference reports as truncated.
        size_ = S_ISREG(st.st_mode) ? size_t(st.st_size) : 0;
        if (size_ > 0) {
            void* p = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
            if (p == MAP_FAILED) {
                ::close(fd);
                throw std::runtime_error("cannot open checkpoint " + path);
            }
            data_ = static_cast<const uint8_t*>(p);
        }
        ::close(fd);
    }
    ~MappedFile() {
        if (data_) ::munmap(const_cast<uint8_t*>(data_), size_);
    }
    MappedFile(const MappedFile&) = delete;
    MappedFile& operator=(const MappedFile&) = delete;
    ByteView view() const { return ByteView(data_, size_); }

private:
    const uint8_t* data_ = nullptr;
    size_t size_ = 0;
};

Verdict read_header(ByteView& v, azb_net_desc* d) {
    uint32_t magic = 0, version = 0;
    if (!v.take(&magic)) return short_file();
    if (magic != kMagic) return bad("not an AZGO checkpoint");
    if (!v.take(&version)) return short_file();
    if (version != kPlainVersion && version != kOwnershipVersion) return bad("unsupported version " + std::to_string(version));
    *d = azb_net_desc{};
    for (const ShapeField& f : kShape) {
        int32_t x = 0;
        if (!v.take(&x)) return short_file();
        d->*f.member = x;
    }
    if (version == kOwnershipVersion) {
        int32_t flag = 0;
        if (!v.take(&flag)) return short_file();
        if (flag != 0 && flag != 1) return bad("invalid ownership flag in header");
        d->ownership = flag;
    }
    for (const ShapeField& f : kShape)
        if (d->*f.member < f.lo || d->*f.member > f.hi) return bad("invalid network shape in header");
    return fine();
}

// The tensor table after the header: each record's name and size checked
// against the layout in order, its floats copied to the arena offset.
Verdict read_tensors(ByteView& v, const Layout& L, float* params, float* buffers) {
    const size_t want = L.params.size() + L.buffers.size();
    uint32_t count = 0;
    if (!v.take(&count)) return short_file();
    if (count != want)
        return bad("has " + std::to_string(count) + " tensors but the network needs " + std::to_string(want));
    for (size_t i = 0; i < want; ++i) {
        const bool in_params = i < L.params.size();
        const LayoutEntry& e = in_params ? L.params[i] : L.buffers[i - L.params.size()];
        uint32_t name_len = 0;
        const uint8_t* name = nullptr;
        if (!v.take(&name_len) || !v.take_bytes(name_len, &name)) return short_file();
        const std::string got(reinterpret_cast<const char*>(name), name_len);
        if (got != e.name) return bad("tensor " + std::to_string(i) + " is '" + got + "' but expected '" + e.name + "'");
        uint64_t size = 0;
        if (!v.take(&size)) return short_file();
        if (size != e.size)
            return bad("tensor '" + got + "' has " + std::to_string(size) + " values but expected " + std::to_string(e.size));
        const uint8_t* data = nullptr;
        if (!v.take_bytes(size_t(size) * sizeof(float), &data)) return short_file();
        std::memcpy((in_params ? params : buffers) + e.offset, data, size_t(size) * sizeof(float));
    }
    if (v.left() != 0) return bad("unexpected data after the last tensor");
    return fine();
}

void raise(const std::string& path, const Verdict& v) {
    throw std::runtime_error(path + ": " + (v.kind == Verdict::kShort ? std::string("truncated") : v.text));
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

}  // namespace
}  // namespace azb

using namespace azb;

extern "C" {

int azb_checkpoint_config(const char* path, azb_net_desc* desc, size_t* n_params, size_t* n_buffers, char* err,
                          size_t err_cap) {
    try {
        if (!path || !desc) throw std::invalid_argument("azb_checkpoint_config: null argument");
        const MappedFile file(path);
        ByteView v = file.view();
        if (const Verdict h = read_header(v, desc)) raise(path, h);
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
        const MappedFile file(path);
        ByteView v = file.view();
        azb_net_desc d{};
        if (const Verdict h = read_header(v, &d)) raise(path, h);
        const Layout L = layout_of(d);
        if (n_params != L.param_floats || n_buffers != L.buffer_floats)
            throw std::invalid_argument("azb_checkpoint_read: arenas of " + std::to_string(n_params) + " and " +
                                        std::to_string(n_buffers) + " floats; the checkpoint's layout needs " +
                                        std::to_string(L.param_floats) + " and " + std::to_string(L.buffer_floats));
        std::memset(params, 0, n_params * sizeof(float));
        std::memset(buffers, 0, n_buffers * sizeof(float));
        if (const Verdict t = read_tensors(v, L, params, buffers)) raise(path, t);
        *desc = d;
        return 0;
    } catch (const std::exception& e) {
        put(err, err_cap, e.what());
        return -1;
    }
}

}  // extern "C"
