// The engine's host side (engine.hpp). Weights are reordered once per upload
// into the layouts the kernels read; a pass is a fixed sequence of launches
// on one stream: the stem, 2 x blocks fused tensor-core convolutions and the
// fused heads.
#include "engine.hpp"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstring>
#include <stdexcept>

#include "../../include/azb200.h"

#ifndef AZB_KERNEL_HASH
#define AZB_KERNEL_HASH "00000000"
#endif

namespace azb {

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("cuda: ") + what + ": " + cudaGetErrorString(e));
}

NetShape NetShape::from(const azb_net_desc& d) {
    NetShape s{d.board, d.history, d.blocks, d.filters, d.value_hidden, d.ownership != 0};
    if (s.board < 5 || s.board > 19) throw std::invalid_argument("azb: board size must be in 5..19");
    if (s.history < 1 || s.blocks < 0 || s.value_hidden < 1) throw std::invalid_argument("azb: bad network shape");
    if (s.filters < 8 || s.filters > 256 || s.filters % 8 != 0)
        throw std::invalid_argument("azb: filters must be a multiple of 8 in [8, 256]");
    return s;
}

const char* precision_name(int p) {
    switch (p) {
        case kTF32: return "tf32";
        case kTF32x3: return "tf32x3";
        case kBF16: return "bf16";
        default: return "unknown";
    }
}

// ------------------------------------------------------------------ layout

namespace {

size_t align64(size_t f) { return (f + 63) / 64 * 64; }

void push(std::vector<LayoutEntry>& list, size_t& floats, const std::string& name, size_t size) {
    list.push_back({name, size, floats});
    floats = align64(floats + size);
}

} // namespace

Layout Layout::of(const NetShape& s) {
    Layout L;
    const size_t F = size_t(s.filters), P = size_t(s.planes()), A = size_t(s.area()), V = size_t(s.value_hidden);
    auto bn = [&](const std::string& pre, size_t c) {
        push(L.params, L.param_floats, pre + ".gamma", c);
        push(L.params, L.param_floats, pre + ".beta", c);
    };
    auto stats = [&](const std::string& pre, size_t c) {
        push(L.buffers, L.buffer_floats, pre + ".runMean", c);
        push(L.buffers, L.buffer_floats, pre + ".runVar", c);
    };
    push(L.params, L.param_floats, "stem.conv.w", F * P * 9);
    bn("stem.bn", F);
    for (int i = 0; i < s.blocks; ++i) {
        const std::string pre = "block" + std::to_string(i);
        push(L.params, L.param_floats, pre + ".conv1.w", F * F * 9);
        bn(pre + ".bn1", F);
        push(L.params, L.param_floats, pre + ".conv2.w", F * F * 9);
        bn(pre + ".bn2", F);
    }
    push(L.params, L.param_floats, "policy.conv.w", 2 * F);
    bn("policy.bn", 2);
    push(L.params, L.param_floats, "policy.fc.w", (A + 1) * 2 * A);
    push(L.params, L.param_floats, "policy.fc.b", A + 1);
    push(L.params, L.param_floats, "value.conv.w", F);
    bn("value.bn", 1);
    push(L.params, L.param_floats, "value.fc1.w", V * A);
    push(L.params, L.param_floats, "value.fc1.b", V);
    push(L.params, L.param_floats, "value.fc2.w", V);
    push(L.params, L.param_floats, "value.fc2.b", 1);
    if (s.ownership) {
        push(L.params, L.param_floats, "ownership.conv.w", F);
        bn("ownership.bn", 1);
    }
    stats("stem.bn", F);
    for (int i = 0; i < s.blocks; ++i) {
        const std::string pre = "block" + std::to_string(i);
        stats(pre + ".bn1", F);
        stats(pre + ".bn2", F);
    }
    stats("policy.bn", 2);
    stats("value.bn", 1);
    if (s.ownership) stats("ownership.bn", 1);
    return L;
}

const LayoutEntry& Layout::param(const std::string& name) const {
    for (const LayoutEntry& e : params)
        if (e.name == name) return e;
    throw std::logic_error("azb: no parameter '" + name + "'");
}

const LayoutEntry& Layout::buffer(const std::string& name) const {
    for (const LayoutEntry& e : buffers)
        if (e.name == name) return e;
    throw std::logic_error("azb: no buffer '" + name + "'");
}

// ------------------------------------------------------------------ device

namespace {

// "12.9" from the runtime's 12090.
std::string version_text(int v) { return std::to_string(v / 1000) + "." + std::to_string((v % 1000) / 10); }

int attribute(cudaDeviceAttr what, int device) {
    int v = 0;
    check(cudaDeviceGetAttribute(&v, what, device), "cudaDeviceGetAttribute");
    return v;
}

// Device admission, once per device. The checks run in the order in which a
// failure says the most: the runtime sees the device; the device is the
// architecture this library's machine code (sm_100a only, no PTX) was built
// for, which the runtime confirms by finding the code for one of its
// kernels; the device grants the opt-in shared memory and the thread-block
// clusters the tensor-core kernels are built around; and a first kernel
// transforms a pattern copied in from the host, which is copied back and
// checked, so copies in both directions and a launch all work.
void admit(int device, DeviceInfo& d) {
    int count = 0;
    if (const cudaError_t e = cudaGetDeviceCount(&count); e != cudaSuccess)
        throw std::runtime_error(std::string("no CUDA device: ") + cudaGetErrorString(e));
    if (count < 1) throw std::runtime_error("no CUDA device");
    if (device < 0 || device >= count)
        throw std::runtime_error("no CUDA device " + std::to_string(device) + " (" + std::to_string(count) + " present)");
    check(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop{};
    check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    d.name = prop.name;
    d.total_memory = prop.totalGlobalMem;
    d.architecture = 10 * attribute(cudaDevAttrComputeCapabilityMajor, device) +
                     attribute(cudaDevAttrComputeCapabilityMinor, device);
    d.sms = attribute(cudaDevAttrMultiProcessorCount, device);
    const std::string sm = "sm_" + std::to_string(d.architecture);

    cudaFuncAttributes image{};
    if (fill_attributes(&image) != cudaSuccess) {
        cudaGetLastError();   // not sticky: the context stays usable
        throw std::runtime_error("no kernels for this GPU (" + sm + "; built for sm_100a)");
    }
    d.binary_version = image.binaryVersion;
    if (d.binary_version != d.architecture || d.architecture != 100)
        throw std::runtime_error("kernels built for sm_" + std::to_string(d.binary_version) + "; this GPU is " + sm);
    if (attribute(cudaDevAttrMaxSharedMemoryPerBlockOptin, device) < 227 * 1024)
        throw std::runtime_error(sm + " grants less than 227 KB of shared memory per block");
    if (!attribute(cudaDevAttrClusterLaunch, device))
        throw std::runtime_error(sm + " does not launch thread-block clusters");

    constexpr int kWords = 64;
    uint32_t sent[kWords], back[kWords] = {};
    for (int i = 0; i < kWords; ++i) sent[i] = 0x9E3779B9u * uint32_t(i + 1);
    uint32_t* dev = nullptr;
    cudaStream_t stream = nullptr;
    cudaError_t r = cudaMalloc(&dev, sizeof sent);
    if (r == cudaSuccess) r = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
    if (r == cudaSuccess) r = cudaMemcpyAsync(dev, sent, sizeof sent, cudaMemcpyHostToDevice, stream);
    if (r == cudaSuccess) r = launch_admission_probe(dev, kWords, stream);
    if (r == cudaSuccess) r = cudaMemcpyAsync(back, dev, sizeof back, cudaMemcpyDeviceToHost, stream);
    if (r == cudaSuccess) r = cudaStreamSynchronize(stream);
    if (stream) cudaStreamDestroy(stream);
    if (dev) cudaFree(dev);
    check(r, "first kernel");
    for (int i = 0; i < kWords; ++i)
        if (back[i] != admission_probe_value(sent[i], i)) throw std::runtime_error("the first kernel wrote wrong values");

    int driver_api = 0, runtime = 0;
    check(cudaDriverGetVersion(&driver_api), "cudaDriverGetVersion");
    check(cudaRuntimeGetVersion(&runtime), "cudaRuntimeGetVersion");
    // The reference's cudaDescription() format (include/azgo/cuda.hpp:45-49).
    d.description = d.name + " " + sm + ", driver API " + version_text(driver_api) + ", runtime " +
                    version_text(runtime) + ", kernels " + AZB_KERNEL_HASH;
    d.usable = true;
}

} // namespace

const DeviceInfo& device_info(int device) {
    static std::mutex m;
    static std::vector<std::unique_ptr<DeviceInfo>> infos(64);
    if (device < 0 || device >= 64) {
        static DeviceInfo bad;
        bad.why = "device index out of range";
        return bad;
    }
    std::lock_guard<std::mutex> lock(m);
    auto& slot = infos[static_cast<size_t>(device)];
    if (!slot) {
        slot = std::make_unique<DeviceInfo>();
        try {
            admit(device, *slot);
        } catch (const std::exception& e) {
            slot->usable = false;
            slot->why = e.what();
        }
    }
    return *slot;
}

const DeviceInfo& require_device(int device) {
    const DeviceInfo& d = device_info(device);
    if (!d.usable) throw std::runtime_error("cuda: " + d.why);
    check(cudaSetDevice(device), "cudaSetDevice");
    return d;
}

// ----------------------------------------------------------- tensor maps

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_tiled() {
    static EncodeTiled fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiled>(p);
    }();
    if (!fn) throw std::runtime_error("cuda: cuTensorMapEncodeTiled is not available from the driver");
    return fn;
}

// ---------------------------------------------------------- conversions

uint32_t bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}

float from_bits(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// Round to nearest, ties away from zero, keeping 10 mantissa bits (the
// rounding of cvt.rna.tf32.f32); the low 13 bits of the result are zero.
float tf32_rna(float x) {
    const uint32_t u = bits(x);
    if ((u & 0x7F800000u) == 0x7F800000u) return x;
    return from_bits((u + 0x1000u) & 0xFFFFE000u);
}

// Round to nearest even bfloat16.
uint16_t bf16_rne(float x) {
    const uint32_t u = bits(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
    return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// BatchNorm2d::forwardInfer's folding (src/layers.cpp:91-92), as bn_fold
// computes it on the reference's GPU (src/cuda/kernels.cu:37-41): float,
// each operation rounded on its own.
void fold_bn(const float* gamma, const float* beta, const float* mean, const float* var, int C, float* scale,
             float* shift) {
    for (int c = 0; c < C; ++c) {
        const float sd = std::sqrt(var[c] + 1e-5f);
        scale[c] = gamma[c] / sd;
        const float prod = scale[c] * mean[c];
        shift[c] = beta[c] - prod;
    }
}

int round_up(int x, int m) { return (x + m - 1) / m * m; }

int n_out_for(int filters) { return filters <= 32 ? 32 : filters <= 64 ? 64 : filters <= 128 ? 128 : 256; }

int cpad_for(int filters, int precision) {
    return std::max(round_up(filters, chunk_channels(precision)), n_out_for(filters));
}

// Sub-allocation of one device arena, 256-byte aligned pieces.
struct Carver {
    size_t used = 0;
    size_t take(size_t bytes) {
        const size_t off = used;
        used = (used + bytes + 255) / 256 * 256;
        return off;
    }
};

} // namespace

// A row-major [rows][inner] tensor read in boxes of box_inner x box_rows
// with the 128-byte swizzle; rows outside [0, rows) read as zero.
CUtensorMap make_tensor_map(const void* base, int precision, uint64_t inner, uint64_t rows, uint32_t box_inner,
                     uint32_t box_rows, int swizzle_bytes) {
    CUtensorMap m;
    const size_t esz = size_t(elem_bytes(precision));
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {inner * esz};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_tiled()(&m, precision == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                                      2, const_cast<void*>(base), dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                                      swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuda: cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return m;
}


// ---------------------------------------------------------------- weights

int stem_k_for(const NetShape& s, int precision) { return round_up(9 * s.planes(), chunk_channels(precision)); }

size_t Weights::bytes_for(const NetShape& s, int precision) {
    const int F = s.filters, n_out = n_out_for(F), cpad = cpad_for(F, precision), ks = stem_k_for(s, precision);
    const size_t A = size_t(s.area()), V = size_t(s.value_hidden);
    const size_t esz = size_t(elem_bytes(precision)), planes = precision == kTF32x3 ? 2 : 1;
    Carver c;
    for (int i = 0; i < 1 + 2 * s.blocks; ++i) {
        c.take(size_t(n_out) * 4);
        c.take(size_t(n_out) * 4);
        const size_t k = i == 0 ? size_t(ks) : size_t(9) * cpad;
        for (size_t p = 0; p < planes; ++p) c.take(size_t(n_out) * k * esz);
    }
    c.take(2 * size_t(F) * 4);
    c.take(8);
    c.take(8);
    c.take((A + 1) * ((2 * A + 3) / 4 * 4) * 4);   // policy FC rows padded to 4 inputs
    c.take((A + 1) * 4);
    c.take(size_t(F) * 4);
    c.take(4);
    c.take(4);
    c.take(V * ((A + 3) / 4 * 4) * 4);             // value FC1 rows padded to 4 inputs
    c.take(V * 4);
    c.take(V * 4);
    c.take(4);
    c.take(size_t(F) * 4);
    c.take(4);
    c.take(4);
    c.take(size_t(2 * s.blocks + 1) * sizeof(FusedLayer));   // the fused tower's layer table (+ the stem)
    return c.used;
}

Weights::Weights(const NetShape& s, int precision, int device, const float* params, size_t n_params,
                 const float* buffers, size_t n_buffers)
    : shape_(s), precision_(precision), device_(device) {
    if (precision != kTF32 && precision != kTF32x3 && precision != kBF16)
        throw std::invalid_argument("azb: unknown precision " + std::to_string(precision));
    require_device(device);
    const Layout L = Layout::of(s);
    if (n_params != L.param_floats)
        throw std::logic_error("azb: the parameter arena has " + std::to_string(n_params) + " floats, the layout " +
                               std::to_string(L.param_floats));
    if (n_buffers != L.buffer_floats)
        throw std::logic_error("azb: the statistics arena has " + std::to_string(n_buffers) + " floats, the layout " +
                               std::to_string(L.buffer_floats));
    const int F = s.filters, P = s.planes(), A = s.area(), V = s.value_hidden;
    n_out_ = n_out_for(F);
    cpad_ = cpad_for(F, precision);
    kstem_ = stem_k_for(s, precision);
    const int KC = chunk_channels(precision), Kp = 9 * cpad_;
    const size_t esz = size_t(elem_bytes(precision));
    const bool split = precision == kTF32x3;
    auto P_ = [&](const std::string& n) { return params + L.param(n).offset; };
    auto B_ = [&](const std::string& n) { return buffers + L.buffer(n).offset; };

    std::vector<uint8_t> img(bytes_for(s, precision), 0);
    Carver c;
    auto put = [&](const void* src, size_t bytes) {
        const size_t off = c.take(bytes);
        if (off + bytes > img.size()) throw std::logic_error("azb: weight image layout out of step with bytes_for");
        std::memcpy(img.data() + off, src, bytes);
        return off;
    };
    struct ConvOffs {
        size_t scale, shift, w, w_lo, k;
    };
    std::vector<ConvOffs> co(size_t(1 + 2 * s.blocks));
    std::vector<float> sc(size_t(n_out_), 0.0f), sh(sc.size(), 0.0f);
    // One conv in kernel layout: [n_out][k] elements, column col(o, ci, t)
    // for the reference's w[o][ci*9 + t] (src/layers.cpp:44-45); folded BN
    // scale/shift padded with zeros to n_out.
    auto pack = [&](size_t i, const std::string& wname, const std::string& bn, int cin, size_t k, auto col) {
        std::fill(sc.begin(), sc.end(), 0.0f);
        std::fill(sh.begin(), sh.end(), 0.0f);
        fold_bn(P_(bn + ".gamma"), P_(bn + ".beta"), B_(bn + ".runMean"), B_(bn + ".runVar"), F, sc.data(), sh.data());
        co[i].scale = put(sc.data(), size_t(n_out_) * 4);
        co[i].shift = put(sh.data(), size_t(n_out_) * 4);
        co[i].k = k;
        std::vector<uint8_t> wk(size_t(n_out_) * k * esz, 0), wl(split ? size_t(n_out_) * k * 4 : 0, 0);
        const float* w = P_(wname);
        for (int o = 0; o < F; ++o)
            for (int ci = 0; ci < cin; ++ci)
                for (int t = 0; t < 9; ++t) {
                    const float v = w[(size_t(o) * cin + ci) * 9 + t];
                    const size_t at = size_t(o) * k + col(ci, t);
                    if (precision == kBF16) {
                        const uint16_t h = bf16_rne(v);
                        std::memcpy(wk.data() + at * 2, &h, 2);
                    } else {
                        const float hi = tf32_rna(v);
                        std::memcpy(wk.data() + at * 4, &hi, 4);
                        if (split) {
                            const float lo = v - hi;
                            std::memcpy(wl.data() + at * 4, &lo, 4);
                        }
                    }
                }
        co[i].w = put(wk.data(), wk.size());
        co[i].w_lo = split ? put(wl.data(), wl.size()) : 0;
    };
    // The stem as a one-tap GEMM over its packed operand: column t*P + p.
    pack(0, "stem.conv.w", "stem.bn", P, size_t(kstem_), [&](int ci, int t) { return size_t(t) * P + ci; });
    // The tower: K index (chunk*9 + tap)*KC + channel-in-chunk.
    for (int i = 0; i < 2 * s.blocks; ++i) {
        const std::string blk = "block" + std::to_string(i / 2);
        pack(size_t(1 + i), blk + (i % 2 ? ".conv2.w" : ".conv1.w"), blk + (i % 2 ? ".bn2" : ".bn1"), F, size_t(Kp),
             [&](int ci, int t) { return size_t((ci / KC) * 9 + t) * KC + ci % KC; });
    }
    // heads: the FC weights output-major as the reference stores them
    // ([out][in]), each row padded with zeros to a multiple of 4 inputs so
    // the FC kernel reads it in 16-byte pieces.
    auto pad_rows = [](const float* w, int out, int in) {
        const int in4 = (in + 3) / 4 * 4;
        std::vector<float> t(size_t(out) * in4, 0.0f);
        for (int o = 0; o < out; ++o)
            for (int i = 0; i < in; ++i) t[size_t(o) * in4 + i] = w[size_t(o) * in + i];
        return t;
    };
    std::vector<float> hsc(2), hsh(2);
    const size_t o_pw = put(P_("policy.conv.w"), size_t(2) * F * 4);
    fold_bn(P_("policy.bn.gamma"), P_("policy.bn.beta"), B_("policy.bn.runMean"), B_("policy.bn.runVar"), 2, hsc.data(), hsh.data());
    const size_t o_psc = put(hsc.data(), 8), o_psh = put(hsh.data(), 8);
    const std::vector<float> fct = pad_rows(P_("policy.fc.w"), A + 1, 2 * A);
    const size_t o_fcw = put(fct.data(), fct.size() * 4);
    const size_t o_fcb = put(P_("policy.fc.b"), size_t(A + 1) * 4);
    const size_t o_vw = put(P_("value.conv.w"), size_t(F) * 4);
    fold_bn(P_("value.bn.gamma"), P_("value.bn.beta"), B_("value.bn.runMean"), B_("value.bn.runVar"), 1, hsc.data(), hsh.data());
    const size_t o_vsc = put(hsc.data(), 4), o_vsh = put(hsh.data(), 4);
    const std::vector<float> v1t = pad_rows(P_("value.fc1.w"), V, A);
    const size_t o_v1w = put(v1t.data(), v1t.size() * 4);
    const size_t o_v1b = put(P_("value.fc1.b"), size_t(V) * 4);
    const size_t o_v2w = put(P_("value.fc2.w"), size_t(V) * 4);
    const size_t o_v2b = put(P_("value.fc2.b"), 4);
    size_t o_ow = 0, o_osc = 0, o_osh = 0;
    if (s.ownership) {
        o_ow = put(P_("ownership.conv.w"), size_t(F) * 4);
        fold_bn(P_("ownership.bn.gamma"), P_("ownership.bn.beta"), B_("ownership.bn.runMean"), B_("ownership.bn.runVar"),
                1, hsc.data(), hsh.data());
        o_osc = put(hsc.data(), 4);
        o_osh = put(hsh.data(), 4);
    }
    // The fused tower's layer table (tensor maps and batch-norm pointers of
    // the tower convs), filled once the arena's addresses are known.
    const size_t o_fused = c.take(size_t(2 * s.blocks + 1) * sizeof(FusedLayer));
    if (c.used > img.size()) throw std::logic_error("azb: weight image layout out of step with bytes_for");
    bytes_ = img.size();
    check(cudaMalloc(&arena_, bytes_), "cudaMalloc weights");
    const cudaError_t e = cudaMemcpy(arena_, img.data(), bytes_, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(arena_);
        arena_ = nullptr;
        check(e, "upload weights");
    }
    auto at = [&](size_t off) { return reinterpret_cast<float*>(static_cast<uint8_t*>(arena_) + off); };
    convs_.resize(co.size());
    for (size_t i = 0; i < co.size(); ++i) {
        Conv& cv = convs_[i];
        cv.scale = at(co[i].scale);
        cv.shift = at(co[i].shift);
        cv.w = at(co[i].w);
        cv.map_w = make_tensor_map(cv.w, precision, uint64_t(co[i].k), uint64_t(n_out_), uint32_t(KC), uint32_t(n_out_));
        cv.map_w_pair = make_tensor_map(cv.w, precision, uint64_t(co[i].k), uint64_t(n_out_), uint32_t(KC),
                                        uint32_t(n_out_ / 2));
        if (split) {
            cv.w_lo = at(co[i].w_lo);
            cv.map_w_lo = make_tensor_map(cv.w_lo, precision, uint64_t(co[i].k), uint64_t(n_out_), uint32_t(KC),
                                          uint32_t(n_out_));
            cv.map_w_lo_pair = make_tensor_map(cv.w_lo, precision, uint64_t(co[i].k), uint64_t(n_out_), uint32_t(KC),
                                               uint32_t(n_out_ / 2));
        } else {
            cv.map_w_lo = cv.map_w;
            cv.map_w_lo_pair = cv.map_w_pair;
        }
    }
    if (s.blocks > 0) {
        std::vector<FusedLayer> table(size_t(2 * s.blocks + 1));   // the tower's convs, then the stem
        for (size_t i = 0; i < table.size(); ++i) {
            const Conv& cv = convs_[i + 1 < table.size() ? 1 + i : 0];
            table[i].w = cv.map_w;
            table[i].w_lo = cv.map_w_lo;
            table[i].scale = cv.scale;
            table[i].shift = cv.shift;
        }
        fused_ = reinterpret_cast<const FusedLayer*>(static_cast<uint8_t*>(arena_) + o_fused);
        const cudaError_t te = cudaMemcpy(const_cast<FusedLayer*>(fused_), table.data(),
                                          table.size() * sizeof(FusedLayer), cudaMemcpyHostToDevice);
        if (te != cudaSuccess) {
            cudaFree(arena_);
            arena_ = nullptr;
            check(te, "upload the fused tower's layer table");
        }
    }
    head_.ld = cpad_;
    head_.n = s.board;
    head_.S = (s.board + 1) * (s.board + 1);
    head_.A = A;
    head_.F = F;
    head_.V = V;
    head_.ownership = s.ownership;
    head_.pol_w = at(o_pw);
    head_.pol_scale = at(o_psc);
    head_.pol_shift = at(o_psh);
    head_.fc_w = at(o_fcw);
    head_.fc_b = at(o_fcb);
    head_.val_w = at(o_vw);
    head_.val_scale = at(o_vsc);
    head_.val_shift = at(o_vsh);
    head_.v1_w = at(o_v1w);
    head_.v1_b = at(o_v1b);
    head_.v2_w = at(o_v2w);
    head_.v2_b = at(o_v2b);
    if (s.ownership) {
        head_.own_w = at(o_ow);
        head_.own_scale = at(o_osc);
        head_.own_shift = at(o_osh);
    }
}

Weights::~Weights() {
    if (arena_) {
        cudaSetDevice(device_);
        cudaFree(arena_);
    }
}

// -------------------------------------------------------------- workspace

namespace {
std::atomic<int> g_tower_fused{-1};   // -1 default (on where it applies), 0 off, 1 without board pairs, 2 pairs always
}

void set_tower_fused(int mode) { g_tower_fused = mode; }

bool fused_tower_plan(const NetShape& s, int precision, FusedArgs* plan) {
    const Frame fr(s.board);
    const int n_out = n_out_for(s.filters);
    if (s.blocks < 1 || fr.S > 128 || (n_out != 32 && n_out != 64)) return false;
    FusedArgs a{};
    a.n = s.board;
    a.S = fr.S;
    a.group = 128 / fr.S;
    a.layers = 2 * s.blocks;
    a.nch = cpad_for(s.filters, precision) / chunk_channels(precision);
    a.top = round_up(s.board + 2, 8);
    // A sub-buffer holds the rows a group's real points read: the zero halo
    // above, the group's frames and the zero halo below. The rows of a
    // 128-row tile past the group are outputs nobody reads; their taps read
    // on into the next sub-buffer, or past the last into the weight ring.
    const int group_rows = a.group * fr.S;
    a.act_bytes = round_up((a.top + group_rows + s.board + 2) * 128, 1024);
    // The stem joins the launch when its packed operand has as many chunks
    // as a stored row (it is staged in the mid buffer).
    const int stem_nch = stem_k_for(s, precision) / chunk_channels(precision);
    a.stem_nch = stem_nch == a.nch ? stem_nch : 0;
    const size_t smem = fused_tower_smem(n_out, precision, a.nch, a.act_bytes, a.layers, &a.stages);
    if (smem == 0) return false;
    // Those reads stay inside the CTA's shared memory: the furthest, a tap
    // of the tile's last row in the last sub-buffer, ends before the ring
    // does (the ring's smallest: two stages of one tap).
    const size_t over = size_t(a.top + 128 + s.board + 2) * 128 - size_t(a.act_bytes);
    if (over > size_t(2) * n_out * 128) return false;
    *plan = a;
    return true;
}

// Floats per board of the heads' feature buffer: the 2A policy features and
// the A value features, each padded with zeros to a multiple of 4 (16-byte
// rows for the FC kernel's loads).
size_t feat_floats(const NetShape& s) {
    const size_t A = size_t(s.area());
    return (2 * A + 3) / 4 * 4 + (A + 3) / 4 * 4;
}

namespace {
// The persistent tower's counters: one per layer (the stem and the tower
// convs) and 128-row tile of a full batch, and the next-item counter.
size_t tower_flags_for(const NetShape& s, int max_batch) {
    const size_t tiles = (size_t(max_batch) * Frame(s.board).S + 127) / 128;
    return size_t(2 * s.blocks + 1) * tiles + 1;
}
// The head tail kernel's counters: one per tile of 16 boards.
size_t tail_counters_for(int max_batch) { return (size_t(max_batch) + 15) / 16; }
} // namespace

size_t Workspace::bytes_for(const NetShape& s, int precision, int max_batch) {
    const Frame fr(s.board);
    const size_t rows = size_t(max_batch) * fr.S;
    const size_t cpad = size_t(cpad_for(s.filters, precision)), esz = size_t(elem_bytes(precision));
    const size_t A = size_t(s.area()), L = size_t(s.actions()), B = size_t(max_batch);
    Carver c;
    c.take(B * s.planes() * A * 4);
    const size_t ks = size_t(stem_k_for(s, precision));
    c.take(rows * ks * esz);
    if (precision == kTF32x3) c.take(rows * ks * 4);
    for (int i = 0; i < 3; ++i) c.take(rows * cpad * esz);
    if (precision == kTF32x3)
        for (int i = 0; i < 3; ++i) c.take(rows * cpad * 4);
    c.take(B * L * 4);
    c.take(B * 4);
    if (s.ownership) c.take(B * A * 4);
    c.take(B * L * 4);
    c.take(B * feat_floats(s) * 4);
    c.take(B * size_t(s.value_hidden) * 4);
    c.take(B * stones_record_bytes(s.history, s.board));
    c.take(16);
    c.take((tail_counters_for(max_batch) + tower_flags_for(s, max_batch)) * 4);
    return c.used;
}

// The same carving as bytes_for, from `base`.
void Workspace::place(const Weights& w, uint8_t* base) {
    const NetShape& s = w.shape();
    const int precision = w.precision();
    const Frame fr(s.board);
    const size_t rows = size_t(max_batch_) * fr.S;
    const size_t cpad = size_t(w.cpad()), esz = size_t(elem_bytes(precision));
    const size_t A = size_t(s.area()), L = size_t(s.actions()), B = size_t(max_batch_);
    Carver c;
    auto at = [&](size_t off) { return base + off; };
    stage = reinterpret_cast<float*>(at(c.take(B * s.planes() * A * 4)));
    const size_t ks = size_t(w.kstem());
    stem_in = at(c.take(rows * ks * esz));
    if (precision == kTF32x3) stem_in_lo = at(c.take(rows * ks * 4));
    for (int i = 0; i < 3; ++i) trunk[i] = at(c.take(rows * cpad * esz));
    if (precision == kTF32x3)
        for (int i = 0; i < 3; ++i) trunk_lo[i] = at(c.take(rows * cpad * 4));
    logits = reinterpret_cast<float*>(at(c.take(B * L * 4)));
    values = reinterpret_cast<float*>(at(c.take(B * 4)));
    if (s.ownership) ownership = reinterpret_cast<float*>(at(c.take(B * A * 4)));
    probs = reinterpret_cast<float*>(at(c.take(B * L * 4)));
    feat = reinterpret_cast<float*>(at(c.take(B * feat_floats(s) * 4)));
    hid = reinterpret_cast<float*>(at(c.take(B * size_t(s.value_hidden) * 4)));
    records = at(c.take(B * stones_record_bytes(s.history, s.board)));
    err = reinterpret_cast<int*>(at(c.take(16)));
    tail_count_n = tail_counters_for(max_batch_);
    tower_flag_count = tower_flags_for(s, max_batch_);
    tail_count = reinterpret_cast<unsigned*>(at(c.take((tail_count_n + tower_flag_count) * 4)));
    tower_flags = tail_count + tail_count_n;
    const uint32_t KC = uint32_t(chunk_channels(precision));
    map_stem = make_tensor_map(stem_in, precision, ks, rows, KC, uint32_t(fr.halo));
    map_stem_lo = precision == kTF32x3 ? make_tensor_map(stem_in_lo, precision, ks, rows, KC, uint32_t(fr.halo)) : map_stem;
    for (int i = 0; i < 3; ++i) {
        map[i] = make_tensor_map(trunk[i], precision, cpad, rows, KC, uint32_t(fr.halo));
        map_lo[i] = precision == kTF32x3 ? make_tensor_map(trunk_lo[i], precision, cpad, rows, KC, uint32_t(fr.halo)) : map[i];
        // The conv epilogue's boxes: {32 channels, 32 rows}; bf16 64-byte rows
        // with the 64-byte swizzle, fp32 (tf32, and both planes of the split
        // mode) 128-byte rows with the 128-byte swizzle.
        if (precision == kBF16) emap[i] = make_tensor_map(trunk[i], precision, cpad, rows, 32, 32, 64);
        else emap[i] = make_tensor_map(trunk[i], precision, cpad, rows, 32, 32, 128);
        emap_lo[i] = precision == kTF32x3 ? make_tensor_map(trunk_lo[i], precision, cpad, rows, 32, 32, 128) : emap[i];
    }
    fused = fused_tower_plan(s, precision, &fused_plan);
    if (fused) {
        const uint32_t box_rows = uint32_t(fused_plan.group * fr.S);
        fmap = make_tensor_map(trunk[0], precision, cpad, rows, KC, box_rows, 128);
        fmap_lo = precision == kTF32x3 ? make_tensor_map(trunk_lo[0], precision, cpad, rows, KC, box_rows, 128) : fmap;
        smap = fmap;
        smap_lo = fmap_lo;
        if (fused_plan.stem_nch > 0) {
            smap = make_tensor_map(stem_in, precision, ks, rows, KC, box_rows, 128);
            smap_lo = precision == kTF32x3 ? make_tensor_map(stem_in_lo, precision, ks, rows, KC, box_rows, 128) : smap;
        }
    }
}

Workspace::Workspace(const Weights& w, int max_batch) : max_batch_(max_batch) {
    if (max_batch < 1) throw std::invalid_argument("azb: max_batch must be >= 1");
    bytes_ = bytes_for(w.shape(), w.precision(), max_batch);
    check(cudaSetDevice(w.device()), "cudaSetDevice");
    check(cudaMalloc(&arena_, bytes_), "cudaMalloc workspace");
    // Zero once: the frames' padding rows are never written again.
    const cudaError_t z = cudaMemset(arena_, 0, bytes_);
    if (z != cudaSuccess) {
        cudaFree(arena_);
        check(z, "cudaMemset workspace");
    }
    place(w, static_cast<uint8_t*>(arena_));
}

Workspace::Workspace(const Weights& w, int max_batch, void* memory) : max_batch_(max_batch) {
    if (max_batch < 1) throw std::invalid_argument("azb: max_batch must be >= 1");
    bytes_ = bytes_for(w.shape(), w.precision(), max_batch);
    place(w, static_cast<uint8_t*>(memory));
}

Workspace::~Workspace() {
    if (arena_) cudaFree(arena_);
}

// ---------------------------------------------------------------- forward

std::string kernel_error_text(int code) {
    switch (code) {
        case kErrWaitProducer: return "a tensor-core kernel's copy engine waited too long for a free stage";
        case kErrWaitMma: return "a tensor-core kernel's MMA issue waited too long for its operands";
        case kErrWaitEpilogue: return "a tensor-core kernel's epilogue waited too long for its accumulator";
        case kErrWaitDrain: return "a tensor-core kernel timed out draining its copies";
        case kErrProbeTimeout: return "bounded wait ran out";
        case kErrWaitHeadLoad: return "the head kernel's copy thread waited too long for a free stage";
        case kErrWaitHeadData: return "the head kernel waited too long for its trunk rows";
        case kErrWaitLayer: return "the persistent tower waited too long for the previous layer";
        default: return "kernel error " + std::to_string(code);
    }
}

void encode_forward(const Weights& w, Workspace& ws, int B, cudaStream_t s, bool probs, PassTimer* timer) {
    if (B < 1 || B > ws.max_batch()) throw std::invalid_argument("CudaNetwork: batch out of range");
    const NetShape& sh = w.shape();
    const int precision = w.precision();
    const Frame fr(sh.board);
    const DeviceInfo& dev = device_info(w.device());
    check(cudaMemsetAsync(ws.err, 0, sizeof(int), s), "reset error word");
    const bool timed = timer && timer->enabled;
    auto mark_begin = [&](int slot) {
        if (timed) check(cudaEventRecord(timer->begin[size_t(slot)], s), "event");
    };
    auto mark_end = [&](int slot) {
        if (timed) check(cudaEventRecord(timer->end[size_t(slot)], s), "event");
    };

    StemArgs st;
    st.in = ws.stage;
    st.B = B;
    st.P = sh.planes();
    st.n = sh.board;
    st.S = fr.S;
    st.ld = w.kstem();
    st.out = ws.stem_in;
    st.out_lo = ws.stem_in_lo;
    // Small boards run the fused tower; the others, where it applies, the
    // persistent tower (whose counters the stem operand kernel zeroes).
    const bool fused = ws.fused && g_tower_fused.load() != 0;
    const int pass_tiles = (B * fr.S + 127) / 128;
    const bool persistent = !fused && sh.blocks > 0 && ws.tower_flags != nullptr &&
                            size_t(2 * sh.blocks + 1) * size_t(pass_tiles) + 1 <= ws.tower_flag_count &&
                            tower_persistent(w.n_out(), precision);
    // The counters the pass uses start at zero: the head tail kernel's (16
    // boards each), then, with the persistent tower, the tower's.
    st.flags = ws.tail_count;
    st.nflags = int(ws.tail_count_n) + (persistent ? (2 * sh.blocks + 1) * pass_tiles + 1 : 0);
    mark_begin(kSlotStemPack);
    check(launch_stem_pack(st, precision, s), "stem operand");
    mark_end(kSlotStemPack);

    ConvArgs a{};
    a.n = sh.board;
    a.S = fr.S;
    a.rows = B * fr.S;
    a.ntiles = (a.rows + 127) / 128;
    a.ld = w.cpad();
    a.halo_rows = fr.halo;
    a.a_bytes = (fr.halo * 128 + 1023) / 1024 * 1024;
    a.err = ws.err;
    auto conv = [&](int index, const CUtensorMap& in, const CUtensorMap& in_lo, int dst, int skip, int taps,
                    int nchunks, int timer_slot) {
        const Weights::Conv& cv = w.conv(index);
        ConvMaps m{in, in_lo, cv.map_w, cv.map_w_lo, cv.map_w_pair, cv.map_w_lo_pair, ws.emap[dst],
                   ws.emap[skip >= 0 ? skip : dst], ws.emap_lo[dst]};
        a.taps = taps;
        a.nchunks = nchunks;
        a.out = ws.trunk[dst];
        a.out_lo = ws.trunk_lo[dst];
        a.skip = skip >= 0 ? ws.trunk[skip] : nullptr;
        a.skip_lo = skip >= 0 ? ws.trunk_lo[skip] : nullptr;
        a.scale = cv.scale;
        a.shift = cv.shift;
        mark_begin(timer_slot);
        check(launch_conv(m, a, w.n_out(), precision, dev.sms, s), "conv");
        mark_end(timer_slot);
    };
    // The stem: conv -> BN -> ReLU as one tap over the packed operand (in
    // the fused or the persistent tower's launch when that runs it).
    if ((fused && ws.fused_plan.stem_nch > 0) || persistent) {
        mark_begin(kSlotStemGemm);
        mark_end(kSlotStemGemm);
    } else {
        conv(0, ws.map_stem, ws.map_stem_lo, 0, -1, 1, w.kstem() / chunk_channels(precision), kSlotStemGemm);
    }
    // The tower: conv -> BN -> ReLU -> conv -> BN -> + skip -> ReLU per block,
    // rotating through three frame buffers.
    HeadArgs h = w.head_args();
    h.B = B;
    h.logits = ws.logits;
    h.values = ws.values;
    h.ownership_out = ws.ownership;
    h.probs = probs ? ws.probs : nullptr;
    h.feat = ws.feat;
    h.feat_val = int((2 * size_t(sh.area()) + 3) / 4 * 4);
    h.feat_ld = int(feat_floats(sh));
    h.hid = ws.hid;
    h.tail_count = ws.tail_count;
    h.err = ws.err;
    const int tower_chunks = w.cpad() / chunk_channels(precision);
    int x = 0;
    if (fused) {
        // Small boards: the whole tower (and the stem, where it fits) in one
        // launch, in place on trunk[0].
        FusedArgs fa = ws.fused_plan;
        fa.boards = B;
        fa.layer = w.fused_layers();
        fa.stem = w.fused_layers() + 2 * sh.blocks;
        fa.heads = 1;   // the heads' 1x1 convolutions from the resident trunk; no trunk is stored
        fa.pairs = g_tower_fused.load() == 1 ? 0 : g_tower_fused.load() == 2 ? 2 : 1;   // 1, 2: for tests
        fa.head = h;
        fa.err = ws.err;
        const FusedMaps fm{ws.fmap, ws.fmap_lo, ws.fmap, ws.fmap_lo, ws.smap, ws.smap_lo};
        mark_begin(kSlotTower);
        check(launch_fused_tower(fm, fa, w.n_out(), precision, dev.sms, s), "fused tower");
        mark_end(kSlotTower);
        for (int i = 1; i < 2 * sh.blocks; ++i) {   // the per-conv slots, empty
            mark_begin(kSlotTower + i);
            mark_end(kSlotTower + i);
        }
    } else if (persistent) {
        // The stem and every tower conv in one launch: the stem writes
        // trunk[0], conv l reads trunk[l % 3] and writes trunk[(l + 1) % 3],
        // so the trunk ends in trunk[2·blocks % 3] as the per-layer rotation
        // leaves it.
        a.taps = 9;
        a.nchunks = tower_chunks;
        a.out = a.out_lo = nullptr;
        a.skip = a.skip_lo = nullptr;
        a.scale = a.shift = nullptr;
        mark_begin(kSlotTower);
        TowerArgs tf;
        tf.tower = w.fused_layers();
        tf.layers = 2 * sh.blocks + 1;
        tf.flags = ws.tower_flags;
        tf.flag_extra = tower_starve() ? 1u : 0u;
        tf.stem_first = 1;
        tf.stem_nchunks = w.kstem() / chunk_channels(precision);
        tf.stem = ws.map_stem;
        tf.stem_lo = ws.map_stem_lo;
        for (int i = 0; i < 3; ++i) {
            tf.in[i] = ws.map[i];
            tf.in_lo[i] = ws.map_lo[i];
            tf.out[i] = ws.emap[i];
            tf.out_lo[i] = ws.emap_lo[i];
            tf.trunk[i] = ws.trunk[i];
            tf.trunk_lo[i] = ws.trunk_lo[i];
        }
        check(launch_tower_persistent(tf, a, w.n_out(), precision, dev.sms, s), "persistent tower");
        mark_end(kSlotTower);
        for (int i = 1; i < 2 * sh.blocks; ++i) {   // the per-conv slots, empty
            mark_begin(kSlotTower + i);
            mark_end(kSlotTower + i);
        }
        x = (2 * sh.blocks) % 3;
    } else {
        for (int i = 0; i < sh.blocks; ++i) {
            const int mid = (x + 1) % 3, out = (x + 2) % 3;
            conv(1 + 2 * i, ws.map[x], ws.map_lo[x], mid, -1, 9, tower_chunks, kSlotTower + 2 * i);
            conv(2 + 2 * i, ws.map[mid], ws.map_lo[mid], out, x, 9, tower_chunks, kSlotTower + 2 * i + 1);
            x = out;
        }
    }
    h.trunk = ws.trunk[x];
    h.trunk_lo = ws.trunk_lo[x];
    // The heads: the 1x1 convolutions streamed from the trunk, then the FCs
    // and the value's finish in one launch; the fused tower runs all of it.
    mark_begin(kSlotHeadConv);
    if (!fused) check(launch_head_conv(h, precision, dev.sms, s), "head convolutions");
    mark_end(kSlotHeadConv);
    mark_begin(kSlotHeadFc);
    if (!fused) check(launch_head_tail(h, s), "head tail");
    mark_end(kSlotHeadFc);
    mark_begin(kSlotHeadOut);   // (the finish runs in the tail launch)
    mark_end(kSlotHeadOut);
}

// -------------------------------------------------------------- inference

Inference::Inference(const NetShape& s, const float* params, size_t n_params, const float* buffers, size_t n_buffers,
                     int max_batch, int device, int precision)
    : device_(device) {
    require_device(device);
    w_ = std::make_unique<Weights>(s, precision, device, params, n_params, buffers, n_buffers);
    ws_ = std::make_unique<Workspace>(*w_, max_batch);
    check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    check(cudaHostAlloc(reinterpret_cast<void**>(&err_host_), sizeof(int), cudaHostAllocDefault), "cudaHostAlloc");
    *err_host_ = 0;
}

Inference::~Inference() {
    cudaSetDevice(device_);
    if (stream_) {
        cudaStreamSynchronize(stream_);
        cudaStreamDestroy(stream_);
    }
    if (err_host_) cudaFreeHost(err_host_);
    if (pin_in_) cudaFreeHost(pin_in_);
    if (pin_out_) cudaFreeHost(pin_out_);
    ws_.reset();
    w_.reset();
}

void Inference::check_error_word() {
    if (*err_host_ != 0) {
        const int code = *err_host_;
        *err_host_ = 0;
        throw std::runtime_error("cuda: " + kernel_error_text(code));
    }
}

void Inference::infer(const float* input, int B, float* logits, float* values, float* ownership, float* probs) {
    const NetShape& s = w_->shape();
    if (ownership && !s.ownership) throw std::invalid_argument("CudaInference: no ownership head");
    if (B < 1 || B > ws_->max_batch()) throw std::invalid_argument("CudaInference: batch out of range");
    check(cudaSetDevice(device_), "cudaSetDevice");
    const size_t in = size_t(B) * s.planes() * s.area();
    check(cudaMemcpyAsync(ws_->stage, input, in * 4, cudaMemcpyHostToDevice, stream_), "input");
    encode_forward(*w_, *ws_, B, stream_, probs != nullptr);
    check(cudaMemcpyAsync(logits, ws_->logits, size_t(B) * s.actions() * 4, cudaMemcpyDeviceToHost, stream_), "logits");
    check(cudaMemcpyAsync(values, ws_->values, size_t(B) * 4, cudaMemcpyDeviceToHost, stream_), "values");
    if (ownership)
        check(cudaMemcpyAsync(ownership, ws_->ownership, size_t(B) * s.area() * 4, cudaMemcpyDeviceToHost, stream_),
              "ownership");
    if (probs)
        check(cudaMemcpyAsync(probs, ws_->probs, size_t(B) * s.actions() * 4, cudaMemcpyDeviceToHost, stream_), "probs");
    check(cudaMemcpyAsync(err_host_, ws_->err, sizeof(int), cudaMemcpyDeviceToHost, stream_), "error word");
    check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    check_error_word();
}

void Inference::infer_stones(const uint8_t* records, int B, float* logits, float* values, float* ownership) {
    const NetShape& s = w_->shape();
    if (ownership && !s.ownership) throw std::invalid_argument("CudaInference: no ownership head");
    if (B < 1 || B > ws_->max_batch()) throw std::invalid_argument("CudaInference: batch out of range");
    check(cudaSetDevice(device_), "cudaSetDevice");
    check(cudaMemcpyAsync(ws_->records, records, size_t(B) * stones_record_bytes(s.history, s.board),
                          cudaMemcpyHostToDevice, stream_), "records");
    EncodeArgs e{ws_->records, B, s.history, s.board, ws_->stage};
    check(launch_encode_planes(e, stream_), "encode");
    encode_forward(*w_, *ws_, B, stream_, false);
    check(cudaMemcpyAsync(logits, ws_->logits, size_t(B) * s.actions() * 4, cudaMemcpyDeviceToHost, stream_), "logits");
    check(cudaMemcpyAsync(values, ws_->values, size_t(B) * 4, cudaMemcpyDeviceToHost, stream_), "values");
    if (ownership)
        check(cudaMemcpyAsync(ownership, ws_->ownership, size_t(B) * s.area() * 4, cudaMemcpyDeviceToHost, stream_),
              "ownership");
    check(cudaMemcpyAsync(err_host_, ws_->err, sizeof(int), cudaMemcpyDeviceToHost, stream_), "error word");
    check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    check_error_word();
}

void Inference::stage(const float* input, int B) {
    const NetShape& s = w_->shape();
    if (B < 1 || B > ws_->max_batch()) throw std::invalid_argument("CudaInference: batch out of range");
    check(cudaSetDevice(device_), "cudaSetDevice");
    check(cudaMemcpyAsync(ws_->stage, input, size_t(B) * s.planes() * s.area() * 4, cudaMemcpyHostToDevice, stream_),
          "input");
    check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
}

void Inference::enqueue(int B) {
    check(cudaSetDevice(device_), "cudaSetDevice");
    encode_forward(*w_, *ws_, B, stream_, true);
}

void Inference::sync() {
    check(cudaSetDevice(device_), "cudaSetDevice");
    check(cudaMemcpyAsync(err_host_, ws_->err, sizeof(int), cudaMemcpyDeviceToHost, stream_), "error word");
    check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    check_error_word();
}

void Inference::read(int B, float* logits, float* values, float* ownership, float* probs) {
    const NetShape& s = w_->shape();
    check(cudaSetDevice(device_), "cudaSetDevice");
    if (logits) check(cudaMemcpyAsync(logits, ws_->logits, size_t(B) * s.actions() * 4, cudaMemcpyDeviceToHost, stream_), "logits");
    if (values) check(cudaMemcpyAsync(values, ws_->values, size_t(B) * 4, cudaMemcpyDeviceToHost, stream_), "values");
    if (ownership && s.ownership)
        check(cudaMemcpyAsync(ownership, ws_->ownership, size_t(B) * s.area() * 4, cudaMemcpyDeviceToHost, stream_), "ownership");
    if (probs) check(cudaMemcpyAsync(probs, ws_->probs, size_t(B) * s.actions() * 4, cudaMemcpyDeviceToHost, stream_), "probs");
    sync();
}

void Inference::time(int B, int warmup, int steps, bool with_copies, double* ms, double* conv_ms, double* stage_ms) {
    const NetShape& s = w_->shape();
    if (B < 1 || B > ws_->max_batch()) throw std::invalid_argument("CudaInference: batch out of range");
    check(cudaSetDevice(device_), "cudaSetDevice");
    const size_t in_floats = size_t(B) * s.planes() * s.area();
    const size_t out_floats = size_t(B) * s.actions();
    if (with_copies && !pin_in_) {
        check(cudaHostAlloc(reinterpret_cast<void**>(&pin_in_), size_t(ws_->max_batch()) * s.planes() * s.area() * 4,
                            cudaHostAllocDefault), "cudaHostAlloc");
        check(cudaHostAlloc(reinterpret_cast<void**>(&pin_out_), size_t(ws_->max_batch()) * (s.actions() + 1) * 4,
                            cudaHostAllocDefault), "cudaHostAlloc");
        check(cudaMemcpy(pin_in_, ws_->stage, in_floats * 4, cudaMemcpyDeviceToHost), "copy staged input");
    }
    auto pass = [&](PassTimer* t) {
        if (with_copies)
            check(cudaMemcpyAsync(ws_->stage, pin_in_, in_floats * 4, cudaMemcpyHostToDevice, stream_), "input");
        encode_forward(*w_, *ws_, B, stream_, false, t);
        if (with_copies) {
            check(cudaMemcpyAsync(pin_out_, ws_->logits, out_floats * 4, cudaMemcpyDeviceToHost, stream_), "logits");
            check(cudaMemcpyAsync(pin_out_ + out_floats, ws_->values, size_t(B) * 4, cudaMemcpyDeviceToHost, stream_),
                  "values");
        }
    };
    for (int i = 0; i < warmup; ++i) pass(nullptr);
    sync();
    cudaEvent_t e0, e1;
    check(cudaEventCreate(&e0), "cudaEventCreate");
    check(cudaEventCreate(&e1), "cudaEventCreate");
    check(cudaEventRecord(e0, stream_), "cudaEventRecord");
    for (int i = 0; i < steps; ++i) pass(nullptr);
    check(cudaEventRecord(e1, stream_), "cudaEventRecord");
    check(cudaEventSynchronize(e1), "cudaEventSynchronize");
    float total = 0.0f;
    check(cudaEventElapsedTime(&total, e0, e1), "cudaEventElapsedTime");
    *ms = total;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    sync();
    if (conv_ms || stage_ms) {
        PassTimer t;
        t.enabled = true;
        const size_t n = size_t(kSlotTower + 2 * s.blocks);
        t.begin.resize(n);
        t.end.resize(n);
        for (size_t i = 0; i < n; ++i) {
            check(cudaEventCreate(&t.begin[i]), "cudaEventCreate");
            check(cudaEventCreate(&t.end[i]), "cudaEventCreate");
        }
        double stages[kTimedStages] = {};
        for (int k = 0; k < steps; ++k) {
            pass(&t);
            check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
            for (size_t i = 0; i < n; ++i) {
                float d = 0.0f;
                check(cudaEventElapsedTime(&d, t.begin[i], t.end[i]), "cudaEventElapsedTime");
                const int slot = int(i);
                const int stage = slot == kSlotStemPack ? 0 : slot == kSlotStemGemm ? 1 : slot == kSlotHeadConv ? 3
                                : slot == kSlotHeadFc ? 4 : slot == kSlotHeadOut ? 5 : 2;
                stages[stage] += d;
            }
        }
        for (size_t i = 0; i < n; ++i) {
            cudaEventDestroy(t.begin[i]);
            cudaEventDestroy(t.end[i]);
        }
        if (conv_ms) *conv_ms = stages[2];
        if (stage_ms)
            for (int i = 0; i < kTimedStages; ++i) stage_ms[i] = stages[i];
        sync();
    }
}

// ------------------------------------------------------------------ hooks

Hooks& hooks() {
    static Hooks h;
    return h;
}

} // namespace azb
