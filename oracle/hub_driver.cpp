// The reference's own InferenceHub and WorkerEvaluators driving the B200
// engine through alphazero-go_b200/host/azgo_cuda_bridge.cpp: the drop-in,
// exercised the way the reference's tests exercise its CUDA runner
// (tests/test_cuda.cpp:1096-1179).
//
// TEST INFRASTRUCTURE ONLY: built by `make -C oracle hub` from the
// reference's sources (the hub, evaluators, network) plus the bridge into
// oracle/_ref/libazhub.so, loaded by tests/test_gpu_dropin.py.
#include <dirent.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "azb_host.hpp"
#include "azgo/cuda.hpp"
#include "azgo/evaluator.hpp"
#include "azgo/inference_hub.hpp"
#include "azgo/network.hpp"
#include "azgo/rng.hpp"

using namespace azgo;

namespace {

void put(char* dst, size_t cap, const std::string& s) {
    if (dst && cap) {
        std::strncpy(dst, s.c_str(), cap - 1);
        dst[cap - 1] = '\0';
    }
}

NetConfig config(int board, int history, int blocks, int filters, int vh, int own) {
    NetConfig c;
    c.boardSize = board;
    c.history = history;
    c.blocks = blocks;
    c.filters = filters;
    c.valueHidden = vh;
    c.ownership = own != 0;
    return c;
}

// The reference test suite's randomNetwork (tests/test_cuda.cpp:188-204).
void randomize(Network& net, uint64_t seed) {
    Rng rng(seed + 17);
    for (ParamView& p : net.params()) {
        const std::string& n = p.name;
        if (n.size() > 6 && n.compare(n.size() - 6, 6, ".gamma") == 0)
            for (size_t i = 0; i < p.size; ++i) p.value[i] = static_cast<float>(0.5 + rng.uniform());
        else if (!p.decay)
            for (size_t i = 0; i < p.size; ++i) p.value[i] = static_cast<float>(0.4 * rng.uniform() - 0.2);
    }
    for (BufferView& b : net.buffers()) {
        const bool var = b.name.find("runVar") != std::string::npos;
        for (size_t i = 0; i < b.size; ++i)
            b.value[i] = static_cast<float>(var ? 0.5 + rng.uniform() : 0.4 * rng.uniform() - 0.2);
    }
}

} // namespace

extern "C" {

// `clients` worker threads, each sending `requests` requests of 1..8
// positions drawn from a pool, through WorkerEvaluators(net, "cuda", ...)
// with the hub in chaos mode (random batch caps, shuffles, pauses). Every
// row must equal, bit for bit, the same position evaluated alone by
// CudaInference. Returns 0 and the number of mismatching rows, or -1.
int azhub_chaos(int board, int history, int blocks, int filters, int vh, uint64_t seed, int clients, int requests,
                int inference_batch, int slots, uint64_t chaos_seed, int device, int precision, long long* mismatches,
                long long* evaluated, char* err, size_t cap) {
    try {
        azb_host::setDefaults(device, precision);
        Network net(config(board, history, blocks, filters, vh, 0), seed);
        randomize(net, seed);
        const NetConfig& cfg = net.config();
        const int P = cfg.planes(), A = cfg.area(), L = cfg.actions();
        const int pool = 64;
        Rng rng(seed + 1);
        std::vector<float> positions(static_cast<size_t>(pool) * P * A);
        for (float& v : positions) v = static_cast<float>(rng.below(2));
        std::vector<float> refLogits(static_cast<size_t>(pool) * L), refValues(pool);
        {
            CudaInference alone(net, 1);
            for (int i = 0; i < pool; ++i)
                alone.infer(positions.data() + static_cast<size_t>(i) * P * A, 1, refLogits.data() + static_cast<size_t>(i) * L,
                            refValues.data() + i);
        }
        cuda_probe::setHubChaosSeed(chaos_seed);
        std::atomic<long long> bad{0}, done{0};
        std::mutex m;
        std::string firstError;
        {
            WorkerEvaluators evals(net, "cuda", clients, 8, inference_batch, slots);
            std::vector<std::thread> threads;
            for (int w = 0; w < clients; ++w) {
                threads.emplace_back([&, w] {
                    try {
                        Evaluator& ev = evals.forWorker(w);
                        Rng r(seed * 1000 + static_cast<uint64_t>(w));
                        std::vector<float> in(static_cast<size_t>(8) * P * A), lg(static_cast<size_t>(8) * L), val(8);
                        std::vector<int> picks(8);
                        for (int q = 0; q < requests; ++q) {
                            const int B = 1 + r.below(8);
                            for (int b = 0; b < B; ++b) {
                                picks[b] = r.below(pool);
                                std::memcpy(in.data() + static_cast<size_t>(b) * P * A,
                                            positions.data() + static_cast<size_t>(picks[b]) * P * A, sizeof(float) * P * A);
                            }
                            ev.evaluate(in.data(), B, lg.data(), val.data());
                            for (int b = 0; b < B; ++b) {
                                const bool same =
                                    std::memcmp(lg.data() + static_cast<size_t>(b) * L,
                                                refLogits.data() + static_cast<size_t>(picks[b]) * L, sizeof(float) * L) == 0 &&
                                    std::memcmp(&val[b], &refValues[picks[b]], sizeof(float)) == 0;
                                if (!same) ++bad;
                            }
                            done += B;
                        }
                    } catch (const std::exception& e) {
                        std::lock_guard<std::mutex> lock(m);
                        if (firstError.empty()) firstError = e.what();
                    }
                });
            }
            for (std::thread& t : threads) t.join();
        }
        cuda_probe::setHubChaosSeed(0);
        if (!firstError.empty()) throw std::runtime_error(firstError);
        *mismatches = bad.load();
        *evaluated = done.load();
        return 0;
    } catch (const std::exception& e) {
        cuda_probe::setHubChaosSeed(0);
        put(err, cap, e.what());
        return -1;
    }
}

// Failure injection through the normal error path (tests/test_cuda.cpp:1143-1179):
// after `after` passes, one pass fails; every request of it and every later
// request must throw "GPU inference failed: ...". Returns the number of
// requests that threw, and the first message in msg.
int azhub_fail_after(int after, int requests, int device, int precision, char* msg, size_t cap) {
    azb_host::setDefaults(device, precision);
    Network net(config(9, 1, 1, 16, 16, 0), 3);
    const NetConfig& cfg = net.config();
    std::vector<float> in(static_cast<size_t>(cfg.planes()) * cfg.area(), 1.0f), lg(cfg.actions()), val(1);
    int threw = 0;
    std::string first;
    {
        WorkerEvaluators evals(net, "cuda", 1, 1, 8, 2);
        cuda_probe::failPassesAfter(after);
        for (int q = 0; q < requests; ++q) {
            try {
                evals.forWorker(0).evaluate(in.data(), 1, lg.data(), val.data());
            } catch (const std::exception& e) {
                if (first.empty()) first = e.what();
                ++threw;
            }
        }
        cuda_probe::failPassesAfter(0);
    }
    put(msg, cap, first);
    return threw;
}

// makeCudaRunner's memory refusal before allocating (tests/test_cuda.cpp:1184-1217).
int azhub_memory_refusal(size_t limit, int device, char* msg, size_t cap) {
    azb_host::setDefaults(device, AZB_BF16);
    Network net(config(19, 1, 2, 64, 64, 0), 1);
    cuda_probe::setMemoryLimit(limit);
    int refused = 0;
    try {
        auto r = makeCudaRunner(net, 1024, 2);
    } catch (const std::runtime_error& e) {
        put(msg, cap, e.what());
        refused = 1;
    }
    cuda_probe::setMemoryLimit(0);
    return refused;
}

// cuda_probe::checkUpload(layout, net) (tests/test_cuda.cpp:920-930): net of
// shape (board, history, blocks, filters, vh, own_net) uploaded against the
// layout of the same shape with ownership own_layout. 0 accepted, 1 refused
// with a logic_error (its message in msg), -1 any other error.
int azhub_check_upload(int board, int history, int blocks, int filters, int vh, int own_layout, int own_net, char* msg,
                       size_t cap) {
    try {
        const Network layout(config(board, history, blocks, filters, vh, own_layout), 1);
        const Network net(config(board, history, blocks, filters, vh, own_net), 1);
        cuda_probe::checkUpload(layout, net);
        return 0;
    } catch (const std::logic_error& e) {
        put(msg, cap, e.what());
        return 1;
    } catch (const std::exception& e) {
        put(msg, cap, e.what());
        return -1;
    }
}

// cuda_probe::checkForwardReadsEveryTensor(net, encodeAs)
// (tests/test_cuda.cpp:932-949). Same codes as azhub_check_upload.
int azhub_check_reads(int board, int history, int blocks, int filters, int vh, int own_net, int own_encode, char* msg,
                      size_t cap) {
    try {
        const Network net(config(board, history, blocks, filters, vh, own_net), 1);
        cuda_probe::checkForwardReadsEveryTensor(net, config(board, history, blocks, filters, vh, own_encode));
        return 0;
    } catch (const std::logic_error& e) {
        put(msg, cap, e.what());
        return 1;
    } catch (const std::exception& e) {
        put(msg, cap, e.what());
        return -1;
    }
}

// cuda_probe::tanhInPlace over x[0..n) on `device` (tests/test_cuda.cpp:492-512).
int azhub_tanh(float* x, size_t n, int device, char* msg, size_t cap) {
    try {
        azb_host::setDefaults(device, AZB_TF32X3);
        cuda_probe::tanhInPlace(x, n);
        return 0;
    } catch (const std::exception& e) {
        put(msg, cap, e.what());
        return -1;
    }
}

namespace {
int threadCount() {
    int count = 0;
    if (DIR* d = opendir("/proc/self/task")) {
        while (const dirent* e = readdir(d))
            if (e->d_name[0] != '.') ++count;
        closedir(d);
    }
    return count;
}
} // namespace

// makeCudaRunner created and destroyed `cycles` times, every other one with
// a pass in flight, leaves no thread behind (tests/test_cuda.cpp:1220-1238).
// Reports the process's thread count before and after (waiting up to 2 s for
// exiting threads). 0, or -1 with msg.
int azhub_runner_cycles(int cycles, int device, int* before, int* after, char* msg, size_t cap) {
    try {
        azb_host::setDefaults(device, AZB_BF16);
        Network net(config(9, 1, 1, 8, 16, 0), 707);
        randomize(net, 707);
        const NetConfig& cfg = net.config();
        { auto warm = makeCudaRunner(net, 8); }
        *before = threadCount();
        for (int i = 0; i < cycles; ++i) {
            auto runner = makeCudaRunner(net, 8);
            std::fill_n(runner->input(0), static_cast<size_t>(8) * cfg.planes() * cfg.area(), 0.5f);
            if (i % 2) runner->begin(0, 8, [](int, std::string) {});
        }
        int now = threadCount();
        for (int tries = 0; now > *before && tries < 100; ++tries) {
            std::this_thread::sleep_for(std::chrono::milliseconds(20));
            now = threadCount();
        }
        *after = now;
        return 0;
    } catch (const std::exception& e) {
        put(msg, cap, e.what());
        return -1;
    }
}

} // extern "C"
