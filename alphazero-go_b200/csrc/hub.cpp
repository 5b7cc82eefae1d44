// azb_hub: leaf batching for many search threads over one runner per GPU,
// in one process. It serves the role of the reference's InferenceHub and
// WorkerEvaluators for the "cuda" backend (include/azgo/inference_hub.hpp:
// 83-150, src/inference_hub.cpp:95-295), designed differently:
//
//  * No dispatcher thread. A request is given rows in its lane's filling
//    pass under the lane's lock, by whichever thread has room to give: the
//    arriving thread itself, or the thread that frees or launches a pass
//    (the runner's completion thread, or a worker). Small requests are
//    copied into the pass's page-locked staging by that thread, outside the
//    lock, so a waiting worker blocks once, for its results; large ones
//    (over 64 KB of input, e.g. 19x19 boards with history 8) are woken to
//    copy their own rows, in parallel. The completion thread scatters each
//    pass's results straight into the waiting requests' arrays and frees
//    the pass at once, so the next pass can fill while the requests of the
//    last one are still waking up.
//  * A pass's size is capped at the largest whole number of the engine's
//    tiles that fits the batch limit (a 128-row tile of frame rows holds 8
//    19x19 boards, 32 9x9 boards in the per-layer kernels; the small-board
//    tower takes whole groups of boards), so a full pass has no ragged tile.
//  * One lane (runner, device) per GPU in the process: a caller binds each
//    of its workers to a lane, e.g. games partitioned across GPUs.
//
// The flush policy is the reference's: a pass launches as soon as it is full
// or as soon as its GPU has nothing in flight (once every row given in it has
// been copied in); with two passes per lane one computes while the next
// fills. Waiting requests are given rows oldest first. A failed pass fails
// its requests and every later one (the failure is sticky, as in the
// reference's hub); destroying a hub refuses requests that have no rows yet
// ("inference hub shut down"), lets the filling and in-flight passes finish
// and waits for every thread still inside evaluate.
//
// Input: float planes as the reference's Evaluator takes them ([B][2H+2][n*n],
// encodePlanes' layout) or position records (azb_stones_record_bytes). A
// records-mode hub converts planes to records as it copies them (exact: the
// planes of a position are 0/1 stone and side-to-move indicators) and the
// GPU encodes them back, so ~H*n*n bytes per position cross to the device
// instead of (2H+2)*n*n floats.
#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <numeric>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../../include/azb200.h"
#include "engine.hpp"

namespace azb {
namespace {

using Clock = std::chrono::steady_clock;

// What a lane needs from the thing that runs its passes: the engine's
// Runner on a GPU, or a CPU stand-in for the host-logic tests.
class PassEngine {
public:
    using Done = std::function<void(int slot, const std::string& error)>;
    virtual ~PassEngine() = default;
    virtual int slots() const = 0;
    virtual float* planes(int slot) = 0;
    virtual uint8_t* records(int slot) = 0;
    virtual const float* logits(int slot) const = 0;
    virtual const float* values(int slot) const = 0;
    virtual void begin(int slot, int B, bool records, Done done) = 0;
};

class RunnerEngine final : public PassEngine {
public:
    explicit RunnerEngine(std::unique_ptr<Runner> r) : r_(std::move(r)) {}
    int slots() const override { return r_->slots(); }
    float* planes(int slot) override { return r_->input(slot); }
    uint8_t* records(int slot) override { return r_->records(slot); }
    const float* logits(int slot) const override { return r_->logits(slot); }
    const float* values(int slot) const override { return r_->values(slot); }
    void begin(int slot, int B, bool records, Done done) override {
        r_->begin(slot, B, std::move(done), records ? Runner::Input::kRecords : Runner::Input::kPlanes);
    }

private:
    std::unique_ptr<Runner> r_;
};

// A CPU stand-in for a GPU pass, for testing the hub's host logic without a
// GPU: after `delay_us` on its own thread it writes, for each position, the
// planes it describes (records decoded as the device encoder decodes them)
// hashed with FNV-1a: value = the hash's top 24 bits / 2^24, logit a = value
// + a. After `fail_after` passes (when > 0) one pass fails.
class FakeEngine final : public PassEngine {
public:
    FakeEngine(int board, int history, int max_batch, int slots, int delay_us, int fail_after)
        : n_(board), H_(history), delay_us_(delay_us), fail_after_(fail_after) {
        const size_t A = size_t(n_) * n_, P = size_t(2 * H_ + 2);
        for (int i = 0; i < slots; ++i) {
            Slot s;
            s.planes.assign(size_t(max_batch) * P * A, 0.0f);
            s.records.assign(size_t(max_batch) * stones_record_bytes(H_, n_), 0);
            s.logits.assign(size_t(max_batch) * (A + 1), 0.0f);
            s.values.assign(size_t(max_batch), 0.0f);
            slots_.push_back(std::move(s));
        }
        worker_ = std::thread([this] { work(); });
    }
    ~FakeEngine() override {
        {
            std::lock_guard<std::mutex> lock(mu_);
            stop_ = true;
        }
        wake_.notify_all();
        worker_.join();
    }
    int slots() const override { return int(slots_.size()); }
    float* planes(int slot) override { return slots_[size_t(slot)].planes.data(); }
    uint8_t* records(int slot) override { return slots_[size_t(slot)].records.data(); }
    const float* logits(int slot) const override { return slots_[size_t(slot)].logits.data(); }
    const float* values(int slot) const override { return slots_[size_t(slot)].values.data(); }
    void begin(int slot, int B, bool records, Done done) override {
        {
            std::lock_guard<std::mutex> lock(mu_);
            jobs_.push_back(Job{slot, B, records, std::move(done)});
        }
        wake_.notify_all();
    }

private:
    struct Slot {
        std::vector<float> planes, logits, values;
        std::vector<uint8_t> records;
    };
    struct Job {
        int slot, B;
        bool records;
        Done done;
    };
    void work() {
        std::unique_lock<std::mutex> lock(mu_);
        for (;;) {
            wake_.wait(lock, [&] { return stop_ || !jobs_.empty(); });
            if (jobs_.empty()) return;
            Job j = std::move(jobs_.front());
            jobs_.pop_front();
            lock.unlock();
            std::this_thread::sleep_for(std::chrono::microseconds(delay_us_));
            run(j);
            const int pass = ++done_;
            j.done(j.slot, fail_after_ > 0 && pass == fail_after_ + 1 ? "fake: injected failure" : "");
            lock.lock();
        }
    }
    void run(const Job& j) {
        Slot& s = slots_[size_t(j.slot)];
        const size_t A = size_t(n_) * n_, P = size_t(2 * H_ + 2), rec = stones_record_bytes(H_, n_);
        std::vector<float> row(P * A);
        for (int b = 0; b < j.B; ++b) {
            const float* x = s.planes.data() + size_t(b) * P * A;
            if (j.records) {
                decode(s.records.data() + size_t(b) * rec, row.data());
                x = row.data();
            }
            uint64_t h = 1469598103934665603ull;
            const unsigned char* c = reinterpret_cast<const unsigned char*>(x);
            for (size_t i = 0; i < P * A * sizeof(float); ++i) h = (h ^ c[i]) * 1099511628211ull;
            const float v = float(h >> 40) / 16777216.0f;
            s.values[size_t(b)] = v;
            for (size_t a = 0; a <= A; ++a) s.logits[size_t(b) * (A + 1) + a] = v + float(a);
        }
    }
    // The device encoder's planes for a record whose symmetry is 0.
    void decode(const uint8_t* r, float* out) const {
        const int A = n_ * n_;
        const uint8_t* head = r + size_t(H_) * A;
        const int to_move = head[0], avail = std::min(int(head[1]), H_), opp = to_move == 1 ? 2 : 1;
        for (int k = 0; k < H_; ++k)
            for (int p = 0; p < A; ++p) {
                const int stone = k < avail ? r[size_t(k) * A + p] : 0;
                out[size_t(2 * k) * A + p] = stone == to_move ? 1.0f : 0.0f;
                out[size_t(2 * k + 1) * A + p] = stone == opp ? 1.0f : 0.0f;
            }
        for (int p = 0; p < A; ++p) {
            out[size_t(2 * H_) * A + p] = to_move == 1 ? 1.0f : 0.0f;
            out[size_t(2 * H_ + 1) * A + p] = to_move == 1 ? 0.0f : 1.0f;
        }
    }
    int n_, H_, delay_us_, fail_after_;
    std::vector<Slot> slots_;
    std::mutex mu_;
    std::condition_variable wake_;
    std::deque<Job> jobs_;
    bool stop_ = false;
    int done_ = 0;
    std::thread worker_;
};

// Planes -> a record with symmetry 0 and all H history positions present
// (an absent position's planes are zero, as an empty board's are). False
// when the planes are not 0/1 stone indicators with one side to move.
bool planes_to_record(const float* x, int n, int H, uint8_t* rec) {
    const int A = n * n;
    const float black = x[size_t(2 * H) * A];
    if (black != 0.0f && black != 1.0f) return false;
    const uint8_t to_move = black == 1.0f ? 1 : 2, opp = to_move == 1 ? 2 : 1;
    for (int p = 0; p < A; ++p)
        if (x[size_t(2 * H) * A + p] != black || x[size_t(2 * H + 1) * A + p] != 1.0f - black) return false;
    for (int k = 0; k < H; ++k) {
        const float* own = x + size_t(2 * k) * A;
        const float* oth = own + A;
        uint8_t* row = rec + size_t(k) * A;
        for (int p = 0; p < A; ++p) {
            const float o = own[p], t = oth[p];
            if ((o != 0.0f && o != 1.0f) || (t != 0.0f && t != 1.0f) || (o == 1.0f && t == 1.0f)) return false;
            row[p] = o == 1.0f ? to_move : t == 1.0f ? opp : 0;
        }
    }
    uint8_t* head = rec + size_t(H) * A;
    head[0] = to_move;
    head[1] = uint8_t(H);
    head[2] = 0;
    for (size_t i = size_t(H) * A + 3; i < stones_record_bytes(H, n); ++i) rec[i] = 0;
    return true;
}

// Boards per whole tile of frame rows: the small-board tower's group, else
// the boards whose frames fill 128-row tiles exactly.
int tile_quantum(const NetShape& s, int precision) {
    FusedArgs plan{};
    if (fused_tower_plan(s, precision, &plan)) return plan.group;
    const int S = (s.board + 1) * (s.board + 1);
    return 128 / std::gcd(S, 128);
}

}  // namespace

class Lane {
public:
    Lane(std::unique_ptr<PassEngine> engine, int cap, bool records, int board, int history)
        : engine_(std::move(engine)), cap_(cap), records_(records), n_(board), H_(history),
          passes_(size_t(engine_->slots())) {}

    ~Lane() {
        std::unique_lock<std::mutex> lock(mu_);
        closing_ = true;
        admit_waiting(lock);   // refuses the requests still waiting for rows (gives none)
        // A filling pass goes once its rows are in (its requests finish, as
        // a reference hub's packed batch does); an empty one is dropped.
        if (filling_ >= 0) {
            Pass& f = passes_[size_t(filling_)];
            const int s = filling_;
            filling_ = -1;
            if (f.reserved == 0) {
                f = Pass{};
            } else {
                f.full = true;
                if (f.written == f.reserved) launch(s, lock);
            }
        }
        drained_.wait(lock, [&] { return inside_ == 0 && in_flight_ == 0; });
        lock.unlock();
        engine_.reset();   // every pass has returned
    }

    int cap() const { return cap_; }

    void evaluate(const float* planes, const uint8_t* records, int B, float* logits, float* values) {
        if (B < 1 || B > cap_)
            throw std::invalid_argument("azb_hub: a request of " + std::to_string(B) + " positions (1.." +
                                        std::to_string(cap_) + ")");
        if (records && !records_)
            throw std::invalid_argument("azb_hub: this hub takes planes; make it with AZB_HUB_RECORDS to pass records");
        {
            std::lock_guard<std::mutex> lock(mu_);
            if (!failed_.empty()) throw std::runtime_error("GPU inference failed: " + failed_);
            if (closing_) throw std::logic_error("azb_hub: evaluate after shutdown");
            ++inside_;
        }
        try {
            run_request(planes, records, B, logits, values);
        } catch (...) {
            leave();
            throw;
        }
        leave();
    }

    void stats(long long* passes, long long* positions, long long* full, double* gpu_seconds) const {
        std::lock_guard<std::mutex> lock(mu_);
        if (passes) *passes = stats_passes_;
        if (positions) *positions = stats_positions_;
        if (full) *full = stats_full_;
        if (gpu_seconds) *gpu_seconds = stats_seconds_;
    }

private:
    enum State { kFree, kFilling, kFlight };
    static constexpr const char* kShutDown = "inference hub shut down";

    // One evaluate call, on its caller's stack while it waits.
    struct Request {
        int B = 0;
        const float* planes = nullptr;     // its input: planes, or
        const uint8_t* records = nullptr;  // records
        float* logits = nullptr;
        float* values = nullptr;
        int slot = -1, off = 0;   // its rows, once given
        bool self_copy = false;   // given rows, it copies its input itself (a large request)
        bool done = false;        // its results are in its arrays (or error is set)
        bool discard = false;     // its rows hold stand-ins: no results to copy
        std::string bad;          // why its input was refused (records mode)
        std::string error;        // why it got no rows, or why its pass failed
        std::condition_variable wake;
    };
    // Requests of up to this many input bytes are copied in by the thread
    // that gives them rows (the one that frees or launches a pass), so a
    // waiting worker wakes once, for its results; larger ones are woken to
    // copy their own rows, in parallel with each other.
    static constexpr size_t kAdmitterCopyBytes = size_t(64) << 10;
    struct Pass {
        State state = kFree;
        int reserved = 0, written = 0;   // rows given to requests / copied in by them
        bool full = false;               // launch once every reserved row is written
        std::vector<Request*> members;
        Clock::time_point started{};
    };

    // The last thread out of evaluate lets a waiting destructor go on.
    void leave() {
        std::lock_guard<std::mutex> lock(mu_);
        if (--inside_ == 0) drained_.notify_all();
    }

    void run_request(const float* planes, const uint8_t* records, int B, float* logits, float* values) {
        std::unique_lock<std::mutex> lock(mu_);
        Request r;
        r.B = B;
        r.planes = planes;
        r.records = records;
        r.logits = logits;
        r.values = values;
        waiting_.push_back(&r);
        deliver(admit_waiting(lock), lock);
        r.wake.wait(lock, [&] { return r.done || r.self_copy; });
        if (!r.done) {   // a large request: its rows are copied here
            lock.unlock();
            copy_rows(r);
            lock.lock();
            wrote(r, lock);
            r.wake.wait(lock, [&] { return r.done; });
        }
        lock.unlock();
        if (r.slot < 0) {   // refused before it got rows
            if (r.error == kShutDown) throw std::logic_error("azb_hub: evaluate after shutdown");
            throw std::runtime_error("GPU inference failed: " + r.error);
        }
        if (!r.error.empty()) throw std::runtime_error("GPU inference failed: " + r.error);
        if (!r.bad.empty()) throw std::invalid_argument(r.bad);
    }

    // A request's input into its rows of its pass's staging (no lock: the
    // rows are its own until the pass launches, which waits for them).
    void copy_rows(Request& r) {
        const int A = n_ * n_, P = 2 * H_ + 2;
        const size_t rec = stones_record_bytes(H_, n_);
        if (records_) {
            uint8_t* dst = engine_->records(r.slot) + size_t(r.off) * rec;
            for (int b = 0; b < r.B; ++b) {
                uint8_t* row = dst + size_t(b) * rec;
                if (r.records) {
                    std::memcpy(row, r.records + size_t(b) * rec, rec);
                } else if (!planes_to_record(r.planes + size_t(b) * P * A, n_, H_, row)) {
                    if (r.bad.empty())
                        r.bad = "azb_hub: position " + std::to_string(b) + "'s planes are not stone planes (records mode)";
                    std::memset(row, 0, rec);
                    row[size_t(H_) * A] = 1;   // a valid record in its place (its results are not used)
                }
            }
        } else {
            std::memcpy(engine_->planes(r.slot) + size_t(r.off) * P * A, r.planes, size_t(r.B) * P * A * sizeof(float));
        }
    }

    // A request's rows are in: count them, and launch its pass when it is
    // complete and full or its GPU idle. Under the lock.
    void wrote(Request& r, std::unique_lock<std::mutex>& lock) {
        r.discard = !r.bad.empty();
        Pass& p = passes_[size_t(r.slot)];
        p.written += r.B;
        if (p.written == p.reserved && (p.full || in_flight_ == 0)) {
            launch(r.slot, lock);
            deliver(admit_waiting(lock), lock);   // requests waiting for rows take the next pass
        }
    }

    // Copies in the small requests this thread gave rows to, then counts
    // them (which may launch passes and give more requests rows). Under the
    // lock; dropped for the copies.
    void deliver(std::vector<Request*> mine, std::unique_lock<std::mutex>& lock) {
        while (!mine.empty()) {
            lock.unlock();
            for (Request* q : mine) copy_rows(*q);
            lock.lock();
            std::vector<Request*> next;
            for (Request* q : mine) {
                q->discard = !q->bad.empty();
                Pass& p = passes_[size_t(q->slot)];
                p.written += q->B;
                if (p.written == p.reserved && (p.full || in_flight_ == 0)) {
                    launch(q->slot, lock);
                    std::vector<Request*> more = admit_waiting(lock);
                    next.insert(next.end(), more.begin(), more.end());
                }
            }
            mine = std::move(next);
        }
    }

    // Requests waiting for rows, oldest first: each is given rows in the
    // filling pass (a free pass becomes the filling pass when there is none)
    // and woken alone, so a freed pass wakes only the requests it takes. A
    // filling pass that cannot take the next request is closed: it goes as
    // soon as its rows are in. After a failure or at shutdown the waiting
    // requests are refused. Under the lock (dropped while a pass launches).
    std::vector<Request*> admit_waiting(std::unique_lock<std::mutex>& lock) {
        std::vector<Request*> mine;
        const size_t row_bytes = records_ ? stones_record_bytes(H_, n_) : size_t(2 * H_ + 2) * n_ * n_ * sizeof(float);
        while (!waiting_.empty()) {
            if (!failed_.empty() || closing_) {
                for (Request* q : waiting_) {
                    q->error = failed_.empty() ? kShutDown : failed_;
                    q->done = true;
                    q->wake.notify_one();
                }
                waiting_.clear();
                break;
            }
            if (filling_ < 0) {
                for (size_t i = 0; i < passes_.size() && filling_ < 0; ++i)
                    if (passes_[i].state == kFree) {
                        passes_[i].state = kFilling;
                        filling_ = int(i);
                    }
                if (filling_ < 0) break;   // every pass is busy: the next one to return admits
            }
            Pass& f = passes_[size_t(filling_)];
            Request* q = waiting_.front();
            if (f.reserved + q->B > cap_) {
                f.full = true;
                const int s = filling_;
                filling_ = -1;
                if (f.written == f.reserved) launch(s, lock);
                continue;
            }
            waiting_.pop_front();
            q->slot = filling_;
            q->off = f.reserved;
            f.reserved += q->B;
            f.members.push_back(q);
            if (size_t(q->B) * row_bytes <= kAdmitterCopyBytes) {
                mine.push_back(q);
            } else {
                q->self_copy = true;
                q->wake.notify_one();
            }
        }
        return mine;
    }

    // Starts pass `slot` (every reserved row written). Under the lock; drops
    // it while the engine enqueues. After a failure nothing new runs: the
    // pass's requests fail at once.
    void launch(int slot, std::unique_lock<std::mutex>& lock) {
        Pass& p = passes_[size_t(slot)];
        if (filling_ == slot) filling_ = -1;
        if (!failed_.empty()) {
            finish(slot, failed_);
            return;
        }
        p.state = kFlight;
        p.started = Clock::now();
        ++in_flight_;
        const int rows = p.reserved;
        lock.unlock();
        engine_->begin(slot, rows, records_, [this](int s, const std::string& e) { on_done(s, e); });
        lock.lock();
    }

    // Wakes every request of a pass with `error` (results already copied
    // when it is empty) and frees the pass. Under the lock.
    void finish(int slot, const std::string& error) {
        Pass& p = passes_[size_t(slot)];
        if (!error.empty() && failed_.empty()) failed_ = error;
        for (Request* q : p.members) {
            q->error = error;
            q->done = true;
            q->wake.notify_one();
        }
        p = Pass{};
    }

    // The engine's done(slot, error), on its completion thread: scatters the
    // results into the waiting requests' arrays (outputs are A+2 floats a
    // position, smaller than its input), frees the pass, launches the
    // filling pass if the GPU went idle, and admits waiting requests.
    void on_done(int slot, const std::string& error) {
        std::unique_lock<std::mutex> lock(mu_);
        Pass& p = passes_[size_t(slot)];
        --in_flight_;
        if (error.empty()) {
            ++stats_passes_;
            stats_positions_ += p.reserved;
            if (p.reserved == cap_) ++stats_full_;
            stats_seconds_ += std::chrono::duration<double>(Clock::now() - p.started).count();
            // The pass stays in flight for everyone else while it is copied out.
            const std::vector<Request*> members = p.members;
            lock.unlock();
            const size_t L = size_t(n_) * n_ + 1;
            const float* lg = engine_->logits(slot);
            const float* v = engine_->values(slot);
            for (Request* q : members) {
                if (q->discard) continue;
                std::memcpy(q->logits, lg + size_t(q->off) * L, size_t(q->B) * L * sizeof(float));
                std::memcpy(q->values, v + size_t(q->off), size_t(q->B) * sizeof(float));
            }
            lock.lock();
        }
        finish(slot, error);
        // The GPU is idle: the filling pass goes if its rows are all in.
        if (in_flight_ == 0 && filling_ >= 0) {
            Pass& f = passes_[size_t(filling_)];
            if (f.reserved > 0 && f.written == f.reserved) launch(filling_, lock);
        }
        deliver(admit_waiting(lock), lock);
        if (in_flight_ == 0) drained_.notify_all();
    }

    std::unique_ptr<PassEngine> engine_;
    const int cap_;
    const bool records_;
    const int n_, H_;
    mutable std::mutex mu_;
    std::condition_variable drained_;
    std::deque<Request*> waiting_;
    std::vector<Pass> passes_;
    int filling_ = -1, in_flight_ = 0, inside_ = 0;
    bool closing_ = false;
    std::string failed_;
    long long stats_passes_ = 0, stats_positions_ = 0, stats_full_ = 0;
    double stats_seconds_ = 0.0;
};

}  // namespace azb

struct azb_hub {
    std::vector<std::unique_ptr<azb::Lane>> lanes;
    int cap = 0;
};

using namespace azb;

namespace {

void put_text(char* dst, size_t cap, const std::string& s) {
    if (!dst || cap == 0) return;
    const size_t n = std::min(cap - 1, s.size());
    std::memcpy(dst, s.data(), n);
    dst[n] = '\0';
}

template <class Fn>
int guarded(char* err, size_t cap, Fn fn) {
    try {
        fn();
        return 0;
    } catch (const std::exception& e) {
        put_text(err, cap, e.what());
    } catch (...) {
        put_text(err, cap, "unknown error");
    }
    return -1;
}

}  // namespace

extern "C" {

int azb_hub_create(const azb_net_desc* desc, const float* params, size_t n_params, const float* buffers,
                   size_t n_buffers, const int* devices, int n_devices, int max_batch, int slots, int precision,
                   int input_mode, azb_hub** out, char* err, size_t err_cap) {
    if (out) *out = nullptr;
    return guarded(err, err_cap, [&] {
        if (!desc || !out || !devices || n_devices < 1) throw std::invalid_argument("azb_hub_create: bad arguments");
        if (input_mode != AZB_HUB_PLANES && input_mode != AZB_HUB_RECORDS)
            throw std::invalid_argument("azb_hub_create: input_mode must be AZB_HUB_PLANES or AZB_HUB_RECORDS");
        const NetShape s = NetShape::from(*desc);
        const int q = tile_quantum(s, precision);
        const int cap = max_batch >= q ? max_batch / q * q : max_batch;
        auto hub = std::make_unique<azb_hub>();
        hub->cap = cap;
        for (int i = 0; i < n_devices; ++i) {
            auto runner = std::make_unique<Runner>(s, params, n_params, buffers, n_buffers, cap, slots, devices[i],
                                                   precision);
            hub->lanes.push_back(std::make_unique<Lane>(std::make_unique<RunnerEngine>(std::move(runner)), cap,
                                                        input_mode == AZB_HUB_RECORDS, s.board, s.history));
        }
        *out = hub.release();
    });
}

int azb_hub_create_fake(int board, int history, int lanes, int max_batch, int slots, int quantum, int input_mode,
                        int delay_us, int fail_after, azb_hub** out, char* err, size_t err_cap) {
    if (out) *out = nullptr;
    return guarded(err, err_cap, [&] {
        if (!out || lanes < 1 || max_batch < 1 || slots < 1 || quantum < 1 || board < 5 || board > 19 || history < 1)
            throw std::invalid_argument("azb_hub_create_fake: bad arguments");
        const int cap = max_batch >= quantum ? max_batch / quantum * quantum : max_batch;
        auto hub = std::make_unique<azb_hub>();
        hub->cap = cap;
        for (int i = 0; i < lanes; ++i)
            hub->lanes.push_back(std::make_unique<Lane>(
                std::make_unique<FakeEngine>(board, history, cap, slots, delay_us, fail_after), cap,
                input_mode == AZB_HUB_RECORDS, board, history));
        *out = hub.release();
    });
}

void azb_hub_destroy(azb_hub* h) { delete h; }

int azb_hub_lanes(const azb_hub* h) { return h ? int(h->lanes.size()) : 0; }
int azb_hub_pass_cap(const azb_hub* h) { return h ? h->cap : 0; }

int azb_hub_evaluate(azb_hub* h, int lane, const float* input, int B, float* logits, float* values, char* err,
                     size_t err_cap) {
    return guarded(err, err_cap, [&] {
        if (!h || lane < 0 || lane >= int(h->lanes.size()) || !input || !logits || !values)
            throw std::invalid_argument("azb_hub_evaluate: bad arguments");
        h->lanes[size_t(lane)]->evaluate(input, nullptr, B, logits, values);
    });
}

int azb_hub_evaluate_records(azb_hub* h, int lane, const uint8_t* records, int B, float* logits, float* values,
                             char* err, size_t err_cap) {
    return guarded(err, err_cap, [&] {
        if (!h || lane < 0 || lane >= int(h->lanes.size()) || !records || !logits || !values)
            throw std::invalid_argument("azb_hub_evaluate_records: bad arguments");
        h->lanes[size_t(lane)]->evaluate(nullptr, records, B, logits, values);
    });
}

int azb_hub_stats(const azb_hub* h, int lane, long long* passes, long long* positions, long long* full_passes,
                  double* gpu_seconds) {
    if (!h || lane < 0 || lane >= int(h->lanes.size())) return -1;
    h->lanes[size_t(lane)]->stats(passes, positions, full_passes, gpu_seconds);
    return 0;
}

}  // extern "C"
