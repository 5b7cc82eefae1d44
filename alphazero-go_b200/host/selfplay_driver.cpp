// Self-play with the reference's own search and game code on a chosen
// engine: the way the reference plays a generation's slice
// (playSelfPlayQueue, src/selfplay_slice.cpp:93-149), restated as a C entry
// point so a benchmark or a test can drive it without the reference's job
// files, checkpoints or run state.
//
// Game i of the slice [first, first + count) is playSelfPlayGame
// (src/selfplay.cpp:50) with Rng(deriveSeed(seed, generation, kPhaseSelfPlay,
// i)), played by one of `workers` threads (capped at count), each with its
// evaluator from one WorkerEvaluators(net, backend, workers, mcts_batch,
// inference_batch) (src/inference_hub.cpp:273-287). backend "cuda" is this
// engine behind the reference's InferenceHub, through azgo_cuda_bridge.cpp
// (the reference's include/azgo/cuda.hpp over include/azb200.h); "naive" and
// "blas" are the reference's CPU engines where the build has them.
//
// Statistics as SliceStats (include/azgo/selfplay_slice.hpp:78-81): wall
// seconds, positions recorded, and network evaluations; playouts/s is
// positions x simulations / seconds (each search adds exactly `simulations`
// playouts, src/mcts.cpp:224-258). The records' bytes go into an FNV-1a hash
// in index order, so callers can check that the games do not depend on the
// number of workers, the batch cap or the hub's chaos mode.
//
// azsp_arena plays an arena wave the same way: the reference's
// playArenaGames (src/arena.cpp) on waveSlice(wave, first, count), with one
// evaluator set (one hub, for cuda) per network, the games hashed in order.
//
// Built by alphazero-go_b200/host/Makefile from the reference's sources.
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

#include "azgo/arena.hpp"
#include "azgo/evaluator.hpp"
#include "azgo/inference_hub.hpp"
#include "azgo/mcts.hpp"
#include "azgo/network.hpp"
#include "azgo/param_layout.hpp"
#include "azgo/rng.hpp"
#include "azgo/selfplay.hpp"

#ifdef AZSP_WITH_ENGINE
#include "azb_host.hpp"
#endif

using namespace azgo;

namespace {

// The phase constant game seeds are derived with (include/azgo/run_state.hpp:118).
constexpr uint64_t kPhaseSelfPlay = 1;

void put(char* dst, size_t cap, const std::string& s) {
    if (dst && cap) {
        std::strncpy(dst, s.c_str(), cap - 1);
        dst[cap - 1] = '\0';
    }
}

struct Fnv {
    uint64_t h = 1469598103934665603ull;
    void bytes(const void* p, size_t n) {
        const unsigned char* c = static_cast<const unsigned char*>(p);
        for (size_t i = 0; i < n; ++i) {
            h ^= c[i];
            h *= 1099511628211ull;
        }
    }
    template <class T>
    void value(const T& v) {
        bytes(&v, sizeof v);
    }
};

void hash_record(Fnv& f, const GameRecord& g) {
    f.value(g.boardSize);
    f.value(g.komi);
    f.value(g.resultForBlack);
    f.value(static_cast<uint8_t>(g.resigned));
    f.value(g.moves.size());
    f.bytes(g.moves.data(), g.moves.size() * sizeof(int));
    f.bytes(g.stones.data(), g.stones.size());
    for (const auto& ply : g.visits) {
        f.value(ply.size());
        for (const auto& v : ply) {
            f.value(v.first);
            f.value(v.second);
        }
    }
    f.bytes(g.finalOwnership.data(), g.finalOwnership.size());
}

// Counts the positions a worker's evaluator evaluated, as the reference's
// EngineEvaluator (src/selfplay_slice.cpp:49-68) does.
class CountingEvaluator : public Evaluator {
public:
    explicit CountingEvaluator(Evaluator& inner) : inner_(inner) {}
    int boardSize() const override { return inner_.boardSize(); }
    int history() const override { return inner_.history(); }
    int maxBatch() const override { return inner_.maxBatch(); }
    void evaluate(const float* input, int B, float* logits, float* values) override {
        inner_.evaluate(input, B, logits, values);
        count_ += B;
    }
    long long count() const { return count_; }

private:
    Evaluator& inner_;
    long long count_ = 0;
};

// Copies the two ParamLayout arenas into the network's tensors.
void load_arenas(Network& net, const float* params, size_t n_params, const float* buffers, size_t n_buffers) {
    const ParamLayout L = ParamLayout::of(net);
    if (n_params != L.paramFloats || n_buffers != L.bufferFloats)
        throw std::invalid_argument("azsp: arena sizes do not match the network's layout");
    std::vector<ParamView> pv = net.params();
    for (size_t i = 0; i < pv.size(); ++i) std::memcpy(pv[i].value, params + L.params[i].offset, pv[i].size * 4);
    std::vector<BufferView> bv = net.buffers();
    for (size_t i = 0; i < bv.size(); ++i) std::memcpy(bv[i].value, buffers + L.buffers[i].offset, bv[i].size * 4);
}

NetConfig make_config(int board, int history, int blocks, int filters, int value_hidden) {
    NetConfig cfg;
    cfg.boardSize = board;
    cfg.history = history;
    cfg.blocks = blocks;
    cfg.filters = filters;
    cfg.valueHidden = value_hidden;
    return cfg;
}

} // namespace

// The reference's setThreadQos (src/selfplay_slice.cpp:34-40) asks macOS to
// schedule a worker at a QoS class and does nothing elsewhere; arena.cpp
// calls it, and selfplay_slice.cpp (which defines it) is not linked here.
void azgo::setThreadQos(CpuQos) {}

namespace {

struct SliceOutcome {
    double seconds = 0;
    long long positions = 0;
    uint64_t hash = 0;
};

// Games [first, first + count) of `generation` on `nw` worker threads, each
// with evaluators.forWorker(w): playSelfPlayGame with the game's own seed,
// the records hashed in index order.
template <class Evaluators>
SliceOutcome play_slice(Evaluators& evaluators, int nw, const SelfPlayConfig& sp, uint64_t seed, int generation,
                       int first, int count, std::chrono::steady_clock::time_point start) {
    std::vector<GameRecord> records(static_cast<size_t>(std::max(0, count)));
    std::atomic<int> next{0};
    std::atomic<bool> stop{false};
    std::atomic<long long> pos{0};
    std::mutex error_mutex;
    std::exception_ptr first_error;
    auto work = [&](int w) {
        try {
            CountingEvaluator ev(evaluators.forWorker(w));
            while (!stop) {
                const int k = next++;
                if (k >= count) break;
                const int i = first + k;
                Rng rng(deriveSeed(seed, static_cast<uint64_t>(generation), kPhaseSelfPlay, static_cast<uint64_t>(i)));
                GameRecord record = playSelfPlayGame(ev, sp, rng);
                pos += record.positions();
                records[static_cast<size_t>(k)] = std::move(record);
            }
        } catch (...) {
            std::lock_guard<std::mutex> lock(error_mutex);
            if (!first_error) first_error = std::current_exception();
            stop = true;
        }
    };
    std::vector<std::thread> threads;
    for (int w = 0; w < nw; ++w) threads.emplace_back(work, w);
    for (std::thread& t : threads) t.join();
    if (first_error) std::rethrow_exception(first_error);
    SliceOutcome r;
    r.seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
    r.positions = pos;
    Fnv f;
    for (const GameRecord& g : records) hash_record(f, g);
    r.hash = f.h;
    return r;
}

SelfPlayConfig selfplay_config(int simulations, int mcts_batch, float c_puct, int temperature_moves, float komi,
                               int max_moves) {
    SelfPlayConfig sp;
    sp.mcts.simulations = simulations;
    sp.mcts.batchSize = mcts_batch;
    sp.mcts.cPuct = c_puct;
    sp.temperatureMoves = temperature_moves;
    sp.komi = komi;
    sp.maxMoves = max_moves;
    sp.resignation = false;
    return sp;
}

} // namespace

extern "C" {

// Plays games [first, first + count) of `generation` and reports the slice's
// statistics and record hash. Returns 0, or -1 with the reason in err.
int azsp_play(int board, int history, int blocks, int filters, int value_hidden, const float* params,
              size_t n_params, const float* buffers, size_t n_buffers, const char* backend, int workers,
              int inference_batch, int device, int precision, int simulations, int mcts_batch, float c_puct,
              int temperature_moves, float komi, int max_moves, uint64_t seed, int generation, int first, int count,
              double* seconds, long long* positions, long long* evaluations, uint64_t* record_hash, char* err,
              size_t cap) {
    try {
#ifdef AZSP_WITH_ENGINE
        azb_host::setDefaults(device, precision);
#else
        (void)device;
        (void)precision;
#endif
        Network net(make_config(board, history, blocks, filters, value_hidden), 0);
        load_arenas(net, params, n_params, buffers, n_buffers);
        const SelfPlayConfig sp = selfplay_config(simulations, mcts_batch, c_puct, temperature_moves, komi, max_moves);
        const auto start = std::chrono::steady_clock::now();
        const int nw = std::max(1, std::min(workers, count));
        WorkerEvaluators evaluators(net, backend, nw, mcts_batch, inference_batch);
        const SliceOutcome r = play_slice(evaluators, nw, sp, seed, generation, first, count, start);
        if (seconds) *seconds = r.seconds;
        if (positions) *positions = r.positions;
        if (evaluations) *evaluations = evaluators.evaluations();
        if (record_hash) *record_hash = r.hash;
        return 0;
    } catch (const std::exception& e) {
        put(err, cap, e.what());
        return -1;
    }
}

#ifdef AZSP_WITH_ENGINE
// The same slice on the engine's own hub (azb_hub) with a lane per device
// in `devices` (worker w on lane w % n_devices) instead of the reference's
// InferenceHub: records != 0 carries stone records to the GPU. Also reports
// the hub's passes, those of exactly its pass cap, and the cap.
int azsp_play_hub(int board, int history, int blocks, int filters, int value_hidden, const float* params,
                  size_t n_params, const float* buffers, size_t n_buffers, const int* devices, int n_devices,
                  int records, int workers, int inference_batch, int precision, int simulations, int mcts_batch,
                  float c_puct, int temperature_moves, float komi, int max_moves, uint64_t seed, int generation,
                  int first, int count, double* seconds, long long* positions, long long* evaluations,
                  uint64_t* record_hash, long long* passes, long long* full_passes, int* pass_cap, char* err,
                  size_t cap) {
    try {
        Network net(make_config(board, history, blocks, filters, value_hidden), 0);
        load_arenas(net, params, n_params, buffers, n_buffers);
        const SelfPlayConfig sp = selfplay_config(simulations, mcts_batch, c_puct, temperature_moves, komi, max_moves);
        const auto start = std::chrono::steady_clock::now();
        const int nw = std::max(1, std::min(workers, count));
        azb_host::HubEvaluators evaluators(net, std::vector<int>(devices, devices + n_devices), nw, mcts_batch,
                                           inference_batch, 2, precision, records != 0);
        const SliceOutcome r = play_slice(evaluators, nw, sp, seed, generation, first, count, start);
        if (seconds) *seconds = r.seconds;
        if (positions) *positions = r.positions;
        if (evaluations) *evaluations = evaluators.evaluations();
        if (record_hash) *record_hash = r.hash;
        if (passes) *passes = evaluators.passes();
        if (full_passes) *full_passes = evaluators.fullPasses();
        if (pass_cap) *pass_cap = evaluators.passCap();
        return 0;
    } catch (const std::exception& e) {
        put(err, cap, e.what());
        return -1;
    }
}
#endif

// An arena wave: matches m = 0 .. n_matches-1 between network a_net[m] and
// network b_net[m] (or, when b_net[m] < 0, a uniform bot searching
// bot_sims[m] playouts), games[m] games seeded seeds[m]; games [first, first
// + count) of the wave (numbered match-major) are played with
// playArenaGames(waveSlice(wave, first, count), cfg, run) on the networks
// loaded from their arenas. Reports A's total score, the evaluations, an
// FNV-1a hash of every game's (score, moves) in order, and (game_hashes, when
// not null: `count` entries) each game's own hash. 0, or -1 with err.
int azsp_arena(int board, int history, int blocks, int filters, int value_hidden, int n_nets,
               const float* const* params, const size_t* n_params, const float* const* buffers,
               const size_t* n_buffers, int n_matches, const int* a_net, const int* b_net, const int* bot_sims,
               const int* games, const uint64_t* seeds, int first, int count, int simulations, int mcts_batch,
               int temperature_moves, const char* backend, int workers, int inference_batch, int device,
               int precision, double* score_a, long long* evaluations, uint64_t* record_hash, uint64_t* game_hashes,
               char* err, size_t cap) {
    try {
#ifdef AZSP_WITH_ENGINE
        azb_host::setDefaults(device, precision);
#else
        (void)device;
        (void)precision;
#endif
        const NetConfig cfg = make_config(board, history, blocks, filters, value_hidden);
        std::vector<std::unique_ptr<Network>> nets;
        for (int i = 0; i < n_nets; ++i) {
            nets.push_back(std::make_unique<Network>(cfg, 0));
            load_arenas(*nets.back(), params[i], n_params[i], buffers[i], n_buffers[i]);
        }
        auto net_at = [&](int i) -> const Network& {
            if (i < 0 || i >= n_nets) throw std::invalid_argument("azsp_arena: no network " + std::to_string(i));
            return *nets[static_cast<size_t>(i)];
        };
        std::vector<ArenaMatchSpec> wave;
        for (int m = 0; m < n_matches; ++m) {
            ArenaMatchSpec spec;
            spec.a = ArenaPlayer::network(net_at(a_net[m]));
            spec.b = b_net[m] >= 0 ? ArenaPlayer::network(net_at(b_net[m])) : ArenaPlayer::bot(bot_sims[m]);
            spec.games = games[m];
            spec.seed = seeds[m];
            wave.push_back(spec);
        }
        ArenaConfig ac;
        ac.simulations = simulations;
        ac.mctsBatch = mcts_batch;
        ac.temperatureMoves = temperature_moves;
        EngineRun run;
        run.backend = backend;
        run.workers = workers;
        run.inferenceBatch = inference_batch;
        SliceStats stats;
        const std::vector<ArenaGameResult> played = playArenaGames(waveSlice(wave, first, count), ac, run, &stats);
        Fnv f;
        double total = 0;
        for (size_t i = 0; i < played.size(); ++i) {
            const ArenaGameResult& g = played[i];
            Fnv one;
            for (Fnv* h : {&f, &one}) {
                h->value(g.scoreA);
                h->value(g.moves.size());
                h->bytes(g.moves.data(), g.moves.size() * sizeof(int));
            }
            if (game_hashes && i < static_cast<size_t>(count)) game_hashes[i] = one.h;
            total += g.scoreA;
        }
        if (score_a) *score_a = total;
        if (evaluations) *evaluations = stats.evaluations;
        if (record_hash) *record_hash = f.h;
        return 0;
    } catch (const std::exception& e) {
        put(err, cap, e.what());
        return -1;
    }
}

} // extern "C"
