// azb_infer_run_noalloc: the forward pass of azb_infer_run with its scratch
// memory -- the input staging, the stem's packed operand, the three
// activation frames, the output rows and the kernel error word -- taken from
// a static device array instead of a workspace allocated with cudaMalloc.
//
// Who needs it: callers that may not allocate device memory at the moment
// they evaluate. An application that hands the GPU's memory to its own pool
// allocator, or runs under a fixed device-memory budget, forbids
// allocations behind its back; and on a latency-critical path cudaMalloc
// can synchronise the whole device. Such a caller creates its azb_infer
// handle once at set-up (that allocates, and uploads the weights) and then
// evaluates through this entry point, which allocates nothing.
//
// The array holds kScratchBytes on every GPU that loads this library, for as
// long as the process lives. Every call shares it and it keeps the previous
// call's contents, so each call first clears the part it uses (the frames'
// padding rows must read zero). Calls that overlap on the GPU (several host
// threads, or several handles on the same device at once) race on the
// array: serialise them.
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

#include "../../include/azb200.h"
#include "capi_types.hpp"
#include "engine.hpp"

namespace {

constexpr size_t kScratchBytes = size_t(32) << 20;   // 32 MiB

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// The array's device address on `device`. Host code cannot use g_scratch's
// name as a device pointer (on the host it names a stand-in, not device
// memory), so it is looked up once per device with that device current. The
// first call on a device does this set-up: make it before any stream capture.
void* scratch_on(int device) {
    static std::mutex m;
    static void* address[64] = {};
    if (device < 0 || device >= 64) throw std::invalid_argument("azb_infer_run_noalloc: device index out of range");
    std::lock_guard<std::mutex> lock(m);
    if (!address[device]) {
        azb::check(cudaSetDevice(device), "cudaSetDevice");
        void* p = nullptr;
        azb::check(cudaGetSymbolAddress(&p, g_scratch), "cudaGetSymbolAddress");
        address[device] = p;
    }
    return address[device];
}

void put_text(char* dst, size_t cap, const std::string& s) {
    if (!dst || cap == 0) return;
    const size_t n = std::min(cap - 1, s.size());
    std::memcpy(dst, s.data(), n);
    dst[n] = '\0';
}

} // namespace

extern "C" int azb_infer_run_noalloc(azb_infer* h, const float* input, int B, float* logits, float* values,
                                     float* ownership, char* err, size_t err_cap) {
    try {
        if (!h) throw std::invalid_argument("azb_infer_run_noalloc: null handle");
        azb::Inference& inf = *h->impl;
        const azb::Weights& w = inf.weights();
        const azb::NetShape& s = w.shape();
        if (B < 1) throw std::invalid_argument("CudaInference: batch out of range");
        if (ownership && !s.ownership) throw std::invalid_argument("CudaInference: no ownership head");
        const size_t need = azb::Workspace::bytes_for(s, w.precision(), B);
        if (need > kScratchBytes)
            throw std::invalid_argument("azb_infer_run_noalloc: batch " + std::to_string(B) + " of this network needs " +
                                        std::to_string(need) + " bytes of scratch, more than the static array's " +
                                        std::to_string(kScratchBytes) + " (32 MiB); use azb_infer_run");
        void* memory = scratch_on(w.device());
        azb::check(cudaSetDevice(w.device()), "cudaSetDevice");
        const cudaStream_t st = inf.stream();
        azb::check(cudaMemsetAsync(memory, 0, need, st), "clear scratch");
        azb::Workspace ws(w, B, memory);
        azb::check(cudaMemcpyAsync(ws.stage, input, size_t(B) * s.planes() * s.area() * 4, cudaMemcpyHostToDevice, st),
                   "input");
        azb::encode_forward(w, ws, B, st, false);
        azb::check(cudaMemcpyAsync(logits, ws.logits, size_t(B) * s.actions() * 4, cudaMemcpyDeviceToHost, st), "logits");
        azb::check(cudaMemcpyAsync(values, ws.values, size_t(B) * 4, cudaMemcpyDeviceToHost, st), "values");
        if (ownership)
            azb::check(cudaMemcpyAsync(ownership, ws.ownership, size_t(B) * s.area() * 4, cudaMemcpyDeviceToHost, st),
                       "ownership");
        int* err_word = inf.error_host();
        azb::check(cudaMemcpyAsync(err_word, ws.err, sizeof(int), cudaMemcpyDeviceToHost, st), "error word");
        azb::check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        if (*err_word != 0) {
            const int code = *err_word;
            *err_word = 0;
            throw std::runtime_error("cuda: " + azb::kernel_error_text(code));
        }
        return 0;
    } catch (const std::exception& e) {
        put_text(err, err_cap, std::string("GPU inference failed: ") + e.what());
        return -1;
    }
}
