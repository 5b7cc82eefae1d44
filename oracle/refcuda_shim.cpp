// C ABI over the reference's own CUDA engine (robominds/alphazero-go
// src/cuda/*.cu, compiled unmodified for sm_100 by oracle/Makefile's
// `refcuda` target): CudaInference (include/azgo/cuda.hpp:72-84) on a
// network loaded from the two ParamLayout arenas, for the comparison arm
// ("ref-CUDA@sm_100") beside this engine's numbers and for a parity check of
// that build against the CPU oracle.
//
// TEST AND BASELINE INFRASTRUCTURE ONLY: nothing in the product loads it.
#include <chrono>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "azgo/cuda.hpp"
#include "azgo/network.hpp"
#include "azgo/param_layout.hpp"

using namespace azgo;

namespace {

void put(char* dst, size_t cap, const std::string& s) {
    if (dst && cap) {
        std::strncpy(dst, s.c_str(), cap - 1);
        dst[cap - 1] = '\0';
    }
}

struct Handle {
    std::unique_ptr<Network> net;
    std::unique_ptr<CudaInference> inf;
    std::vector<float> logits, values;
};

} // namespace

extern "C" {

int azrefcuda_available(char* why, size_t cap) {
    std::string w;
    const bool ok = cudaAvailable(&w);
    if (!ok) put(why, cap, w);
    return ok ? 1 : 0;
}

int azrefcuda_description(char* out, size_t cap) {
    try {
        put(out, cap, cudaDescription());
        return 0;
    } catch (const std::exception& e) {
        put(out, cap, e.what());
        return -1;
    }
}

void* azrefcuda_create(int board, int history, int blocks, int filters, int vh, const float* params, size_t n_params,
                       const float* buffers, size_t n_buffers, int max_batch, char* err, size_t cap) {
    try {
        NetConfig c;
        c.boardSize = board;
        c.history = history;
        c.blocks = blocks;
        c.filters = filters;
        c.valueHidden = vh;
        auto h = std::make_unique<Handle>();
        h->net = std::make_unique<Network>(c, 0);
        const ParamLayout L = ParamLayout::of(*h->net);
        if (n_params != L.paramFloats || n_buffers != L.bufferFloats)
            throw std::invalid_argument("arena sizes do not match the layout");
        std::vector<ParamView> pv = h->net->params();
        for (size_t i = 0; i < pv.size(); ++i) std::memcpy(pv[i].value, params + L.params[i].offset, pv[i].size * 4);
        std::vector<BufferView> bv = h->net->buffers();
        for (size_t i = 0; i < bv.size(); ++i) std::memcpy(bv[i].value, buffers + L.buffers[i].offset, bv[i].size * 4);
        h->inf = std::make_unique<CudaInference>(*h->net, max_batch);
        return h.release();
    } catch (const std::exception& e) {
        put(err, cap, e.what());
        return nullptr;
    }
}

void azrefcuda_destroy(void* p) { delete static_cast<Handle*>(p); }

int azrefcuda_infer(void* p, const float* input, int B, float* logits, float* values, char* err, size_t cap) {
    try {
        static_cast<Handle*>(p)->inf->infer(input, B, logits, values);
        return 0;
    } catch (const std::exception& e) {
        put(err, cap, e.what());
        return -1;
    }
}

// Wall seconds of `steps` synchronous CudaInference::infer calls on B
// positions (host input copied in, logits and values copied out, as the
// reference's engine does every call), after `warmup` untimed calls.
int azrefcuda_time(void* p, const float* input, int B, int warmup, int steps, double* seconds, char* err, size_t cap) {
    try {
        Handle* h = static_cast<Handle*>(p);
        const size_t L = size_t(h->net->config().actions());
        h->logits.resize(size_t(B) * L);
        h->values.resize(size_t(B));
        for (int i = 0; i < warmup; ++i) h->inf->infer(input, B, h->logits.data(), h->values.data());
        const auto t0 = std::chrono::steady_clock::now();
        for (int i = 0; i < steps; ++i) h->inf->infer(input, B, h->logits.data(), h->values.data());
        *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        return 0;
    } catch (const std::exception& e) {
        put(err, cap, e.what());
        return -1;
    }
}

} // extern "C"
