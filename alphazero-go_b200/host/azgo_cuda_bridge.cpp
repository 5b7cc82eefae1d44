// The reference's CUDA-engine API (robominds/alphazero-go include/azgo/cuda.hpp)
// implemented over this engine's C ABI (include/azb200.h). Built in place of
// the reference's src/cuda/*.cu with -DAZ_USE_CUDA, it makes
// WorkerEvaluators(net, "cuda", ...), InferenceHub, self-play and the arena
// run on the B200 engine without a change to their code: makeCudaRunner
// returns an azgo::BatchRunner whose passes are the engine's runner slots.
//
// Beyond the reference's API (its header has no place for them):
//   azb_host::setDefaults(device, precision) picks the GPU and the arithmetic
//   of the runners and CudaInference objects made afterwards; without it the
//   environment's AZB_DEVICE (default 0) and AZB_PRECISION (tf32x3, tf32 or
//   bf16; default tf32x3, the fp32-class mode that matches the reference's
//   fp32 engine within 1e-4) decide.
//   azb_host::makeCudaRunnerOn(net, maxBatch, slots, device) for one hub per
//   GPU in a multi-GPU process.
// The reference's kernel-level probes of its SIMT design (cuda_probe::gemm,
// im2col3, bnInfer, relu, addInto, policyFlatten, biasAddRows, convBnRelu,
// transposeInput) have no counterpart here: this engine has no such kernels;
// its own kernel checks are the azb_probe_* entry points. tanhInPlace runs
// the tanhf the head kernels use.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "azb200.h"
#include "azb_host.hpp"
#include "azgo/cuda.hpp"
#include "azgo/inference_hub.hpp"
#include "azgo/param_layout.hpp"

namespace azb_host {

namespace {

std::atomic<int> gDevice{-1}, gPrecision{-1};

int envPrecision() {
    const char* p = std::getenv("AZB_PRECISION");
    if (!p) return AZB_TF32X3;
    const std::string s(p);
    if (s == "bf16") return AZB_BF16;
    if (s == "tf32") return AZB_TF32;
    return AZB_TF32X3;
}

int envDevice() {
    const char* d = std::getenv("AZB_DEVICE");
    return d ? std::atoi(d) : 0;
}

} // namespace

void setDefaults(int device, int precision) {
    gDevice = device;
    gPrecision = precision;
}

int defaultDevice() { return gDevice.load() >= 0 ? gDevice.load() : envDevice(); }
int defaultPrecision() { return gPrecision.load() >= 0 ? gPrecision.load() : envPrecision(); }

azb_net_desc describe(const azgo::NetConfig& c) {
    return azb_net_desc{c.boardSize, c.history, c.blocks, c.filters, c.valueHidden, c.ownership ? 1 : 0};
}

Arenas arenas(const azgo::Network& network) { return arenas(network, network.config()); }

Arenas arenas(const azgo::Network& network, const azgo::NetConfig& layout) {
    azgo::Network& net = const_cast<azgo::Network&>(network);   // params() hands out views; nothing is written
    const azb_net_desc d = describe(layout);
    Arenas a;
    a.params.assign(azb_layout_floats(&d, 0), 0.0f);
    a.buffers.assign(azb_layout_floats(&d, 1), 0.0f);
    // Each view checked against the engine's layout at the same position, by
    // name and size, as CudaWeights::upload checks against ParamLayout
    // (src/cuda/cuda_network.cu:24-41): a tensor the engine does not know
    // (a layer without a GPU port) is refused by name.
    auto copy = [&](const auto& views, int which, std::vector<float>& arena) {
        const int n = azb_layout_count(&d, which);
        char name[128];
        size_t size = 0, offset = 0;
        for (size_t i = 0; i < views.size(); ++i) {
            if (static_cast<int>(i) >= n || azb_layout_entry(&d, which, static_cast<int>(i), name, sizeof name, &size, &offset) != 0 ||
                views[i].name != name)
                throw std::logic_error("GPU network: unknown tensor '" + views[i].name + "' (a layer without a GPU port?)");
            if (size != views[i].size)
                throw std::logic_error("GPU network: tensor '" + views[i].name + "' has " + std::to_string(views[i].size) +
                                       " floats, the layout " + std::to_string(size));
            std::memcpy(arena.data() + offset, views[i].value, size * sizeof(float));
        }
        if (static_cast<int>(views.size()) < n) {
            azb_layout_entry(&d, which, static_cast<int>(views.size()), name, sizeof name, &size, &offset);
            throw std::logic_error(std::string("GPU network: the network lacks tensor '") + name + "'");
        }
    };
    copy(net.params(), 0, a.params);
    copy(net.buffers(), 1, a.buffers);
    return a;
}

// The BatchRunner over the engine's runner (one slot = one pass in flight).
class Runner : public azgo::BatchRunner {
public:
    Runner(const azgo::Network& net, int maxBatch, int slots, int device, int precision) {
        const azb_net_desc d = describe(net.config());
        const Arenas a = arenas(net);
        char err[1024] = {};
        if (azb_runner_create(&d, a.params.data(), a.params.size(), a.buffers.data(), a.buffers.size(), maxBatch,
                              slots, device, precision, &r_, err, sizeof err) != 0) {
            const std::string msg(err);
            if (msg.find("must be") != std::string::npos) throw std::invalid_argument(msg);
            throw std::runtime_error(msg);
        }
    }
    ~Runner() override { azb_runner_destroy(r_); }   // drains every pass in flight first

    int slots() const override { return azb_runner_slots(r_); }
    int maxBatch() const override { return azb_runner_max_batch(r_); }
    float* input(int slot) override { return azb_runner_input(r_, slot); }
    const float* logits(int slot) const override { return azb_runner_logits(r_, slot); }
    const float* values(int slot) const override { return azb_runner_values(r_, slot); }

    void begin(int slot, int B, std::function<void(int slot, std::string error)> done) override {
        auto* ctx = new std::function<void(int, std::string)>(std::move(done));
        if (azb_runner_begin(r_, slot, B, &Runner::trampoline, ctx) != 0) {
            delete ctx;
            throw std::out_of_range("runner: slot " + std::to_string(slot) + " out of range");
        }
    }

private:
    static void trampoline(void* ctx, int slot, const char* error) {
        std::unique_ptr<std::function<void(int, std::string)>> fn(static_cast<std::function<void(int, std::string)>*>(ctx));
        (*fn)(slot, std::string(error ? error : ""));
    }
    azb_runner* r_ = nullptr;
};

std::unique_ptr<azgo::BatchRunner> makeCudaRunnerOn(const azgo::Network& net, int maxBatch, int slots, int device,
                                                    int precision) {
    if (maxBatch < 1) throw std::invalid_argument("makeCudaRunner: maxBatch must be >= 1");
    if (slots < 1 || slots > azgo::kInferenceSlots)
        throw std::invalid_argument("makeCudaRunner: slots must be in [1, " + std::to_string(azgo::kInferenceSlots) + "]");
    return std::make_unique<Runner>(net, maxBatch, slots, device, precision < 0 ? defaultPrecision() : precision);
}

namespace {

// The reference's Evaluator (include/azgo/evaluator.hpp) over a hub lane.
class HubEvaluator : public azgo::Evaluator {
public:
    HubEvaluator(azb_hub* hub, int lane, const azgo::NetConfig& cfg, int maxRequest)
        : hub_(hub), lane_(lane), n_(cfg.boardSize), history_(cfg.history), max_request_(maxRequest) {}
    int boardSize() const override { return n_; }
    int history() const override { return history_; }
    int maxBatch() const override { return max_request_; }
    void evaluate(const float* input, int B, float* logits, float* values) override {
        char err[1024] = {};
        if (azb_hub_evaluate(hub_, lane_, input, B, logits, values, err, sizeof err) != 0) {
            const std::string msg(err);
            if (msg.rfind("GPU inference failed", 0) == 0) throw std::runtime_error(msg);
            throw std::invalid_argument(msg);
        }
    }

private:
    azb_hub* hub_;
    int lane_, n_, history_, max_request_;
};

} // namespace

HubEvaluators::HubEvaluators(const azgo::Network& net, const std::vector<int>& devices, int workers, int maxRequest,
                             int inferenceBatch, int slots, int precision, bool records) {
    if (workers < 1) throw std::invalid_argument("HubEvaluators: workers must be >= 1");
    if (devices.empty()) throw std::invalid_argument("HubEvaluators: no devices");
    const azb_net_desc d = describe(net.config());
    const Arenas a = arenas(net);
    char err[1024] = {};
    if (azb_hub_create(&d, a.params.data(), a.params.size(), a.buffers.data(), a.buffers.size(), devices.data(),
                       static_cast<int>(devices.size()), inferenceBatch, slots,
                       precision < 0 ? defaultPrecision() : precision, records ? AZB_HUB_RECORDS : AZB_HUB_PLANES,
                       &hub_, err, sizeof err) != 0)
        throw std::runtime_error(err);
    if (maxRequest < 1 || maxRequest > azb_hub_pass_cap(hub_)) {
        azb_hub_destroy(hub_);
        throw std::invalid_argument("HubEvaluators: maxRequest must be in [1, " + std::to_string(inferenceBatch) + "]");
    }
    for (int w = 0; w < workers; ++w)
        evaluators_.push_back(std::make_unique<HubEvaluator>(hub_, w % static_cast<int>(devices.size()),
                                                             net.config(), maxRequest));
}

HubEvaluators::~HubEvaluators() {
    evaluators_.clear();
    azb_hub_destroy(hub_);   // waits for passes in flight
}

azgo::Evaluator& HubEvaluators::forWorker(int worker) { return *evaluators_.at(static_cast<size_t>(worker)); }

namespace {
long long lane_sum(azb_hub* hub, int which) {
    long long total = 0;
    for (int l = 0; l < azb_hub_lanes(hub); ++l) {
        long long passes = 0, positions = 0, full = 0;
        azb_hub_stats(hub, l, &passes, &positions, &full, nullptr);
        total += which == 0 ? positions : which == 1 ? passes : full;
    }
    return total;
}
} // namespace

long long HubEvaluators::evaluations() const { return lane_sum(hub_, 0); }
long long HubEvaluators::passes() const { return lane_sum(hub_, 1); }
long long HubEvaluators::fullPasses() const { return lane_sum(hub_, 2); }
int HubEvaluators::passCap() const { return azb_hub_pass_cap(hub_); }
int HubEvaluators::lanes() const { return azb_hub_lanes(hub_); }

} // namespace azb_host

namespace azgo {

bool cudaBuilt() { return true; }

bool cudaAvailable(std::string* why) {
    char buf[512] = {};
    const bool ok = azb_cuda_available(azb_host::defaultDevice(), buf, sizeof buf) != 0;
    if (!ok && why) *why = buf;
    return ok;
}

std::string cudaDescription() {
    char buf[512] = {};
    azb_describe(azb_host::defaultDevice(), azb_host::defaultPrecision(), buf, sizeof buf);
    return buf;
}

std::unique_ptr<BatchRunner> makeCudaRunner(const Network& net, int maxBatch, int slots) {
    return azb_host::makeCudaRunnerOn(net, maxBatch, slots, azb_host::defaultDevice(), azb_host::defaultPrecision());
}

void checkCudaInferenceMemory(const NetConfig& cfg, int inferenceBatch, int hubs, int slotsPerHub) {
    if (inferenceBatch < 1 || hubs < 1 || slotsPerHub < 1)
        throw std::invalid_argument("checkCudaInferenceMemory: bad arguments");
    checkCudaInferenceMemory(cfg, std::vector<GpuHubs>{{hubs, slotsPerHub, inferenceBatch}});
}

void checkCudaInferenceMemory(const NetConfig& cfg, const std::vector<GpuHubs>& groups) {
    if (groups.empty()) throw std::invalid_argument("checkCudaInferenceMemory: no hubs");
    const azb_net_desc d = azb_host::describe(cfg);
    const int precision = azb_host::defaultPrecision();
    double need = 0;
    int hubs = 0, batch = 0;
    for (const GpuHubs& g : groups) {
        if (g.inferenceBatch < 1 || g.hubs < 1 || g.slotsPerHub < 1)
            throw std::invalid_argument("checkCudaInferenceMemory: bad arguments");
        need += double(g.hubs) * (double(g.slotsPerHub) * double(azb_workspace_bytes(&d, g.inferenceBatch, precision)) +
                                  double(azb_weights_bytes(&d, precision)));
        hubs += g.hubs;
        batch = std::max(batch, g.inferenceBatch);
    }
    char err[1024] = {};
    if (azb_check_bytes(azb_host::defaultDevice(), need, batch, hubs, err, sizeof err) != 0) throw std::runtime_error(err);
}

struct CudaInference::Impl {
    azb_infer* h = nullptr;
    NetConfig cfg;
    ~Impl() { azb_infer_destroy(h); }
};

CudaInference::CudaInference(const Network& net, int maxBatch) : impl_(std::make_unique<Impl>()) {
    impl_->cfg = net.config();
    const azb_net_desc d = azb_host::describe(net.config());
    const azb_host::Arenas a = azb_host::arenas(net);
    char err[1024] = {};
    if (azb_infer_create(&d, a.params.data(), a.params.size(), a.buffers.data(), a.buffers.size(), maxBatch,
                         azb_host::defaultDevice(), azb_host::defaultPrecision(), &impl_->h, err, sizeof err) != 0)
        throw std::runtime_error(err);
}

CudaInference::~CudaInference() = default;

void CudaInference::infer(const float* input, int B, float* logits, float* values, float* ownership) {
    if (ownership && !impl_->cfg.ownership) throw std::invalid_argument("CudaInference: no ownership head");
    char err[1024] = {};
    if (azb_infer_run(impl_->h, input, B, logits, values, ownership, nullptr, err, sizeof err) != 0) {
        const std::string msg(err);
        if (msg.find("batch out of range") != std::string::npos) throw std::invalid_argument("CudaInference: batch out of range");
        throw std::runtime_error(msg);
    }
}

size_t CudaInference::bytes() const { return azb_infer_bytes(impl_->h); }

namespace cuda_probe {

std::string deviceName() {
    const std::string d = cudaDescription();
    const size_t sm = d.find(" sm_");
    return sm == std::string::npos ? d : d.substr(0, sm);
}
int deviceArchitecture() { return azb_probe_device_architecture(azb_host::defaultDevice()); }
int binaryVersion() { return azb_probe_binary_version(azb_host::defaultDevice()); }
void fill(float* data, size_t n, float value, size_t tail) {
    char err[512] = {};
    if (azb_probe_fill(azb_host::defaultDevice(), data, n, value, tail, err, sizeof err) != 0) throw std::runtime_error(err);
}
void setHubChaosSeed(uint64_t seed) { azb_probe_set_hub_chaos_seed(seed); }
uint64_t hubChaosSeed() { return azb_probe_hub_chaos_seed(); }
void failPassesAfter(int n) { azb_probe_fail_passes_after(n); }
void setMemoryLimit(size_t bytes) { azb_probe_set_memory_limit(bytes); }
long long passesCompleted() { return azb_probe_passes_completed(); }
void setCopyOutDelay(int microseconds) { azb_probe_set_copy_out_delay(microseconds); }
void checkUpload(const Network& layoutNet, const Network& net) { azb_host::arenas(net, layoutNet.config()); }
// The engine's pass for a shape reads exactly that shape's layout: every
// tensor of net the encodeAs layout lacks is one such a pass never reads.
void checkForwardReadsEveryTensor(const Network& network, const NetConfig& encodeAs) {
    Network& net = const_cast<Network&>(network);
    const azb_net_desc d = azb_host::describe(encodeAs);
    std::vector<std::string> known;
    char name[128];
    size_t size = 0, offset = 0;
    for (int which = 0; which < 2; ++which)
        for (int i = 0, n = azb_layout_count(&d, which); i < n; ++i)
            if (azb_layout_entry(&d, which, i, name, sizeof name, &size, &offset) == 0) known.emplace_back(name);
    std::string unread;
    auto scan = [&](const auto& views) {
        for (const auto& v : views)
            if (std::find(known.begin(), known.end(), v.name) == known.end()) unread += (unread.empty() ? "" : ", ") + v.name;
    };
    scan(net.params());
    scan(net.buffers());
    if (!unread.empty()) throw std::logic_error("GPU network: the pass never reads " + unread);
}
void tanhInPlace(float* x, size_t count) {
    char err[512] = {};
    if (azb_probe_tanh(azb_host::defaultDevice(), x, count, err, sizeof err) != 0) throw std::runtime_error(err);
}

} // namespace cuda_probe

} // namespace azgo
