// A C ABI over the reference's own CPU network, built from the reference's
// sources by oracle/Makefile into oracle/_ref/libazref.so.
//
// TEST INFRASTRUCTURE ONLY: tests use it to pin the C restatement
// (azoracle.c) and to make the golden fixtures; bench.py's reference arm and
// CPU-baseline leg time it. It links robominds/alphazero-go's Network,
// layers, backends (naive and OpenBLAS), ParamLayout, Rng and encodePlanes
// unchanged; this file only adapts their C++ interfaces to C.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "azgo/backend.hpp"
#include "azgo/board.hpp"
#include "azgo/encode.hpp"
#include "azgo/checkpoint.hpp"
#include "azgo/network.hpp"
#include "azgo/param_layout.hpp"
#include "azgo/rng.hpp"

using namespace azgo;

struct azref_net {
    Network net;
    ParamLayout layout;
    azref_net(const NetConfig& cfg, uint64_t seed) : net(cfg, seed), layout(ParamLayout::of(net)) {}
};

namespace {

void fail(char* err, size_t cap, const std::string& what) {
    if (err && cap) {
        std::strncpy(err, what.c_str(), cap - 1);
        err[cap - 1] = '\0';
    }
}

bool endsWith(const std::string& s, const char* tail) {
    const size_t n = std::strlen(tail);
    return s.size() >= n && s.compare(s.size() - n, n, tail) == 0;
}

// Batch-norm statistics that are not the identity. kind 0: the benchmark's
// distributions from Rng(deriveSeed(seed, 1)); kind 1: the reference test
// suite's randomNetwork (tests/test_cuda.cpp:188-204).
void randomize(Network& net, int kind, uint64_t seed) {
    Rng rng(kind == 0 ? deriveSeed(seed, 1) : seed + 17);
    for (ParamView& p : net.params()) {
        if (endsWith(p.name, ".gamma")) {
            for (size_t i = 0; i < p.size; ++i) p.value[i] = static_cast<float>(0.5 + rng.uniform());
        } else if (!p.decay) {
            if (kind == 0) {
                if (endsWith(p.name, ".beta"))
                    for (size_t i = 0; i < p.size; ++i) p.value[i] = static_cast<float>(0.1 * rng.normal());
            } else {
                for (size_t i = 0; i < p.size; ++i) p.value[i] = static_cast<float>(0.4 * rng.uniform() - 0.2);
            }
        }
    }
    for (BufferView& b : net.buffers()) {
        const bool var = b.name.find("runVar") != std::string::npos;
        for (size_t i = 0; i < b.size; ++i) {
            if (var) b.value[i] = static_cast<float>(0.5 + rng.uniform());
            else b.value[i] = kind == 0 ? static_cast<float>(0.1 * rng.normal())
                                        : static_cast<float>(0.4 * rng.uniform() - 0.2);
        }
    }
}

NetConfig config(int board, int history, int blocks, int filters, int valueHidden, int ownership) {
    NetConfig c;
    c.boardSize = board;
    c.history = history;
    c.blocks = blocks;
    c.filters = filters;
    c.valueHidden = valueHidden;
    c.ownership = ownership != 0;
    return c;
}

} // namespace

extern "C" {

azref_net* azref_net_create(int board, int history, int blocks, int filters, int value_hidden, int ownership,
                            uint64_t seed, int randomize_kind) {
    try {
        auto* h = new azref_net(config(board, history, blocks, filters, value_hidden, ownership), seed);
        if (randomize_kind >= 0) randomize(h->net, randomize_kind, seed);
        return h;
    } catch (...) {
        return nullptr;
    }
}

void azref_net_destroy(azref_net* h) { delete h; }

// saveNetwork (src/checkpoint.cpp:80-100) of the shim's network. 0, or -1 with err.
int azref_save_checkpoint(azref_net* h, const char* path, char* err, size_t cap) {
    try {
        saveNetwork(h->net, path);
        return 0;
    } catch (const std::exception& e) {
        fail(err, cap, e.what());
        return -1;
    }
}

// loadNetwork (src/checkpoint.cpp:102-133) of `path`: 0 when it loads (its
// two arenas written when params/buffers are non-null and of the right
// sizes, *shape = board, history, blocks, filters, value_hidden, ownership),
// 1 with the loader's message when it throws.
int azref_load_checkpoint(const char* path, int* shape, float* params, size_t n_params, float* buffers,
                          size_t n_buffers, char* err, size_t cap) {
    try {
        Network net = loadNetwork(path);
        const NetConfig& c = net.config();
        const int v[6] = {c.boardSize, c.history, c.blocks, c.filters, c.valueHidden, c.ownership ? 1 : 0};
        if (shape) std::memcpy(shape, v, sizeof v);
        const ParamLayout L = ParamLayout::of(net);
        if (params && buffers && n_params == L.paramFloats && n_buffers == L.bufferFloats) {
            std::fill(params, params + n_params, 0.0f);
            std::fill(buffers, buffers + n_buffers, 0.0f);
            const auto views = net.params();
            for (size_t i = 0; i < views.size(); ++i)
                std::memcpy(params + L.params[i].offset, views[i].value, views[i].size * sizeof(float));
            const auto bufs = net.buffers();
            for (size_t i = 0; i < bufs.size(); ++i)
                std::memcpy(buffers + L.buffers[i].offset, bufs[i].value, bufs[i].size * sizeof(float));
        }
        return 0;
    } catch (const std::exception& e) {
        fail(err, cap, e.what());
        return 1;
    }
}

size_t azref_floats(azref_net* h, int which) { return which == 0 ? h->layout.paramFloats : h->layout.bufferFloats; }

int azref_layout_count(azref_net* h, int which) {
    return static_cast<int>(which == 0 ? h->layout.params.size() : h->layout.buffers.size());
}

int azref_layout_entry(azref_net* h, int which, int index, char* name, size_t cap, size_t* size, size_t* offset) {
    const auto& list = which == 0 ? h->layout.params : h->layout.buffers;
    if (index < 0 || static_cast<size_t>(index) >= list.size()) return -1;
    const ParamLayout::Entry& e = list[static_cast<size_t>(index)];
    fail(name, cap, e.name);
    if (size) *size = e.size;
    if (offset) *offset = e.offset;
    return 0;
}

// The two arenas, params() then buffers() at ParamLayout offsets, zero between tensors.
void azref_export(azref_net* h, float* params, float* buffers) {
    std::fill(params, params + h->layout.paramFloats, 0.0f);
    std::fill(buffers, buffers + h->layout.bufferFloats, 0.0f);
    const auto views = h->net.params();
    for (size_t i = 0; i < views.size(); ++i)
        std::memcpy(params + h->layout.params[i].offset, views[i].value, views[i].size * sizeof(float));
    const auto bufs = h->net.buffers();
    for (size_t i = 0; i < bufs.size(); ++i)
        std::memcpy(buffers + h->layout.buffers[i].offset, bufs[i].value, bufs[i].size * sizeof(float));
}

int azref_infer(azref_net* h, const char* backend, const float* input, int B, float* logits, float* values,
                float* ownership, char* err, size_t cap) {
    try {
        std::unique_ptr<Backend> be = makeBackend(backend, 1);
        Workspace ws(h->net.config(), B, *be);
        h->net.infer(ws, input, B, logits, values, ownership);
        return 0;
    } catch (const std::exception& e) {
        fail(err, cap, e.what());
        return -1;
    }
}

// Network::infer over B positions split into `threads` contiguous slices,
// each slice on its own thread with its own single-threaded backend and
// Workspace, as the reference's workers share one read-only Network
// (include/azgo/evaluator.hpp's LocalEvaluator). Each position's outputs
// are those of infer alone: the reference's forward is batch independent.
int azref_infer_threads(azref_net* h, const char* backend, const float* input, int B, float* logits, float* values,
                        float* ownership, int threads, char* err, size_t cap) {
    try {
        const NetConfig& cfg = h->net.config();
        const size_t P = static_cast<size_t>(cfg.planes()) * cfg.area();
        threads = std::max(1, std::min(threads, B));
        const int per = (B + threads - 1) / threads;
        std::vector<std::thread> pool;
        std::mutex m;
        std::string first_error;
        for (int t = 0; t < threads; ++t) {
            const int lo = t * per, n = std::min(B, lo + per) - lo;
            if (n <= 0) break;
            pool.emplace_back([&, lo, n] {
                try {
                    std::unique_ptr<Backend> be = makeBackend(backend, 1);
                    Workspace ws(cfg, n, *be);
                    h->net.infer(ws, input + lo * P, n, logits + static_cast<size_t>(lo) * cfg.actions(), values + lo,
                                 ownership ? ownership + static_cast<size_t>(lo) * cfg.area() : nullptr);
                } catch (const std::exception& e) {
                    std::lock_guard<std::mutex> lock(m);
                    if (first_error.empty()) first_error = e.what();
                }
            });
        }
        for (auto& th : pool) th.join();
        if (!first_error.empty()) throw std::runtime_error(first_error);
        return 0;
    } catch (const std::exception& e) {
        fail(err, cap, e.what());
        return -1;
    }
}

// Replaces the network's tensors with the two ParamLayout arenas
// (params() then buffers() at their offsets), e.g. to run the reference
// forward on weights made or changed outside it.
void azref_import(azref_net* h, const float* params, const float* buffers) {
    const auto views = h->net.params();
    for (size_t i = 0; i < views.size(); ++i)
        std::memcpy(views[i].value, params + h->layout.params[i].offset, views[i].size * sizeof(float));
    const auto bufs = h->net.buffers();
    for (size_t i = 0; i < bufs.size(); ++i)
        std::memcpy(bufs[i].value, buffers + h->layout.buffers[i].offset, bufs[i].size * sizeof(float));
}

// Positions with one history position, encoded by the reference's
// encodePlanes (src/encode.cpp:14-43); the stones are drawn exactly as
// azoracle.c's az_inputs_positions draws them.
void azref_inputs_positions(int board, int history, uint64_t seed, long first, int B, float* out) {
    const int A = board * board, P = numPlanes(history);
    std::vector<uint8_t> stones(static_cast<size_t>(A));
    for (int b = 0; b < B; ++b) {
        Rng rng(deriveSeed(seed, 2, static_cast<uint64_t>(first + b)));
        const Color toMove = rng.below(2) == 0 ? Color::Black : Color::White;
        for (int p = 0; p < A; ++p) {
            stones[static_cast<size_t>(p)] = static_cast<uint8_t>(Color::Empty);
            if (rng.uniform() < 0.4)
                stones[static_cast<size_t>(p)] =
                    static_cast<uint8_t>(rng.below(2) == 0 ? Color::Black : Color::White);
        }
        std::vector<const uint8_t*> history1{stones.data()};
        encodePlanes(history1, board, toMove, history, 0, out + static_cast<size_t>(b) * P * A);
    }
}

// The reference's encodePlanes (src/encode.cpp:15-43) on position records:
// per position, stones[H][A] Color bytes (k plies ago), then toMove (1
// Black, 2 White), the number of history positions present, the symmetry.
void azref_encode_records(int board, int history, int B, const uint8_t* records, size_t record_bytes, float* out) {
    const int A = board * board, P = numPlanes(history);
    for (int b = 0; b < B; ++b) {
        const uint8_t* r = records + static_cast<size_t>(b) * record_bytes;
        const uint8_t* head = r + static_cast<size_t>(history) * A;
        std::vector<const uint8_t*> stones;
        for (int k = 0; k < head[1]; ++k) stones.push_back(r + static_cast<size_t>(k) * A);
        encodePlanes(stones, board, static_cast<Color>(head[0]), history, head[2], out + static_cast<size_t>(b) * P * A);
    }
}

void azref_inputs_planes(uint64_t seed, size_t count, float* out) {
    Rng rng(seed);
    for (size_t i = 0; i < count; ++i) out[i] = static_cast<float>(rng.below(2));
}

// The reference's CPU engine at full load, as apps/bench.cpp's
// measureCpuWorkers runs it (apps/bench.cpp:455-476): `workers` threads,
// each with its own single-threaded backend and workspace, evaluating
// `batch` positions per Network::infer call until `seconds` have passed
// (or `max_calls` calls per worker, when > 0). Returns positions per
// second; *positions gets the count. input holds `batch` positions.
double azref_bench_workers(azref_net* h, const char* backend, int workers, int batch, const float* input,
                           double seconds, long long max_calls, long long* positions, char* err, size_t cap) {
    try {
        const NetConfig& cfg = h->net.config();
        std::atomic<bool> stop{false};
        std::atomic<long long> done{0};
        std::mutex m;
        std::string firstError;
        std::vector<std::thread> threads;
        const auto start = std::chrono::steady_clock::now();
        for (int w = 0; w < workers; ++w) {
            threads.emplace_back([&] {
                try {
                    std::unique_ptr<Backend> be = makeBackend(backend, 1);
                    Workspace ws(cfg, batch, *be);
                    std::vector<float> logits(static_cast<size_t>(batch) * cfg.actions()), values(batch);
                    long long calls = 0;
                    while (!stop.load(std::memory_order_relaxed)) {
                        h->net.infer(ws, input, batch, logits.data(), values.data());
                        done += batch;
                        if (max_calls > 0 && ++calls >= max_calls) break;
                    }
                } catch (const std::exception& e) {
                    std::lock_guard<std::mutex> lock(m);
                    if (firstError.empty()) firstError = e.what();
                    stop = true;
                }
            });
        }
        if (max_calls <= 0) {
            while (!stop.load() &&
                   std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count() < seconds)
                std::this_thread::sleep_for(std::chrono::milliseconds(2));
            stop = true;
        }
        for (std::thread& t : threads) t.join();
        const double elapsed = std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
        if (!firstError.empty()) throw std::runtime_error(firstError);
        if (positions) *positions = done.load();
        return static_cast<double>(done.load()) / elapsed;
    } catch (const std::exception& e) {
        fail(err, cap, e.what());
        return -1.0;
    }
}

// Raw generator outputs (src/rng.cpp), for the oracle's known-answer pins:
// what = 0 next() (as two 32-bit halves in doubles: hi, lo), 1 uniform(),
// 2 below(n), 3 normal().
void azref_rng_sample(uint64_t seed, int what, int n, int count, double* out) {
    Rng rng(seed);
    for (int i = 0; i < count; ++i) {
        switch (what) {
            case 0: {
                const uint64_t v = rng.next();
                out[2 * i] = static_cast<double>(v >> 32);
                out[2 * i + 1] = static_cast<double>(v & 0xFFFFFFFFull);
                break;
            }
            case 1: out[i] = rng.uniform(); break;
            case 2: out[i] = rng.below(n); break;
            default: out[i] = rng.normal(); break;
        }
    }
}

uint64_t azref_derive_seed(uint64_t a, uint64_t b, uint64_t c, uint64_t d) { return deriveSeed(a, b, c, d); }

const char* azref_blas_description() {
    static std::string d = blasAvailable() ? blasDescription() : std::string("naive only (built without BLAS)");
    return d.c_str();
}

} // extern "C"
