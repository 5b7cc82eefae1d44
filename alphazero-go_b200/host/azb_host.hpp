// The C++ side of the drop-in (azgo_cuda_bridge.cpp): what a reference
// build needs beyond include/azgo/cuda.hpp to place this engine's runners on
// chosen GPUs and in a chosen arithmetic.
#pragma once
#include <memory>
#include <vector>

#include "azb200.h"
#include "azgo/inference_hub.hpp"
#include "azgo/network.hpp"

namespace azb_host {

// Device and precision (AZB_TF32, AZB_TF32X3, AZB_BF16) for the runners and
// CudaInference objects made from now on.
void setDefaults(int device, int precision);
int defaultDevice();
int defaultPrecision();

azb_net_desc describe(const azgo::NetConfig& c);

// The network's two ParamLayout arenas, each tensor checked by name and size
// against the engine's layout (refusing unknown, missing or mis-sized ones).
struct Arenas {
    std::vector<float> params, buffers;
};
Arenas arenas(const azgo::Network& net);
// The same against the layout of another shape (cuda_probe::checkUpload):
// refuses, by name, the first tensor of net that layout does not have.
Arenas arenas(const azgo::Network& net, const azgo::NetConfig& layout);
azb_net_desc describe(const azgo::NetConfig& c);

// makeCudaRunner on a given device (one hub per GPU); precision < 0: the default.
std::unique_ptr<azgo::BatchRunner> makeCudaRunnerOn(const azgo::Network& net, int maxBatch, int slots, int device,
                                                    int precision = -1);

// One evaluator per worker over an azb_hub with a lane per device: the
// counterpart of the reference's WorkerEvaluators(net, "cuda", ...)
// (include/azgo/inference_hub.hpp:151-176) for one or more GPUs in one
// process. Worker w evaluates on lane w % devices.size(), so a slice's
// games are split across the GPUs. records: the hub carries stone records
// (the planes are encoded on the GPU).
class HubEvaluators {
public:
    HubEvaluators(const azgo::Network& net, const std::vector<int>& devices, int workers, int maxRequest,
                  int inferenceBatch, int slots, int precision, bool records);
    ~HubEvaluators();
    HubEvaluators(const HubEvaluators&) = delete;
    HubEvaluators& operator=(const HubEvaluators&) = delete;
    azgo::Evaluator& forWorker(int worker);
    int workers() const { return static_cast<int>(evaluators_.size()); }
    long long evaluations() const;     // positions evaluated, all lanes
    long long passes() const;          // passes run, all lanes
    long long fullPasses() const;      // passes of exactly passCap() positions
    int passCap() const;
    int lanes() const;

private:
    azb_hub* hub_ = nullptr;
    std::vector<std::unique_ptr<azgo::Evaluator>> evaluators_;
};

} // namespace azb_host
