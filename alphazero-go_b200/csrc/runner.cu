// The asynchronous batch runner: the drop-in behind the reference's
// BatchRunner seam (include/azgo/inference_hub.hpp:41-53, made by
// makeCudaRunner, include/azgo/cuda.hpp:58), and the memory admission that
// guards its creation (checkCudaInferenceMemory, include/azgo/cuda.hpp:63).
//
// A slot is a workspace, a stream, an event and page-locked staging (float
// planes, or position records for the device encoder). begin() enqueues the
// slot's copy-in, forward pass and copy-out, records the slot's event after
// the copies, and files a ticket in the slot: the callback, any error met
// while enqueueing, and the issue time.
//
// One reporter thread makes every done() call. Self-play is bound by the
// host's cores, so the reporter should neither spin through a pass nor
// learn of its end late: it keeps a running estimate of how long the GPU
// takes per pass (its service time), predicts when the earliest live ticket
// finishes, sleeps until shortly before that, and then polls every live
// slot's event with yields for a short window, so a pass is reported within
// a few microseconds of its copy-out and whichever slot finishes first is
// reported first. A pass that overruns its prediction by more than the
// window is polled with sleeps that grow from 50 to 200 us, so a long or
// stalled pass costs no core.
#include "engine.hpp"

#include <algorithm>
#include <cstdio>
#include <stdexcept>

namespace azb {

namespace {

using Clock = std::chrono::steady_clock;
using Micros = std::chrono::microseconds;

// Memory the admission check leaves free for the CUDA runtime and the rest
// of the machine (the reference's margin, src/cuda/cuda_runner.cu:51).
constexpr double kReserveBytes = double(size_t(512) << 20);

// Reporter timing: wake this long before a predicted finish (at least the
// kernel's timer slack, so the sleep does not overshoot the finish), poll
// with yields this long past it, then back off between these sleeps.
constexpr Micros kMinLead{60}, kMinWindow{100}, kBackoffFirst{50}, kBackoffLast{200};

}  // namespace

bool Hooks::pass_marked_to_fail() {
    int left = fail_countdown.load();
    do {
        if (left <= 0) return false;
    } while (!fail_countdown.compare_exchange_weak(left, left - 1));
    return left == 1;
}

struct Runner::Slot {
    std::unique_ptr<Workspace> ws;
    cudaStream_t stream = nullptr;
    cudaEvent_t done_event = nullptr;
    float* planes = nullptr;     // pinned [max_batch][planes][area]
    uint8_t* records = nullptr;  // pinned [max_batch][stones_record_bytes]
    float* logits = nullptr;     // pinned [max_batch][actions]
    float* values = nullptr;     // pinned [max_batch]
    float* ownership = nullptr;  // pinned [max_batch][area], with the head
    int* err_word = nullptr;     // pinned: the pass's kernel error word
    // The pass in flight: written by begin() before `live` is raised, read
    // and cleared by the reporter after it sees `live`.
    std::atomic<bool> live{false};
    Done done;
    std::string enqueue_error;
    Clock::time_point issued;
};

namespace {

template <class T>
T* pinned(size_t count) {
    void* p = nullptr;
    check(cudaHostAlloc(&p, count * sizeof(T), cudaHostAllocDefault), "cudaHostAlloc");
    return static_cast<T*>(p);
}

}  // namespace

Runner::Runner(const NetShape& s, const float* params, size_t n_params, const float* buffers, size_t n_buffers,
               int max_batch, int slots, int device, int precision)
    : shape_(s), device_(device), max_batch_(max_batch) {
    if (max_batch < 1) throw std::invalid_argument("makeCudaRunner: maxBatch must be >= 1");
    if (slots < 1 || slots > 2) throw std::invalid_argument("makeCudaRunner: slots must be in [1, 2]");
    require_device(device);
    check_fits(device, hub_bytes(s, precision, max_batch, slots), max_batch, 1);
    w_ = std::make_unique<Weights>(s, precision, device, params, n_params, buffers, n_buffers);
    const size_t B = size_t(max_batch);
    try {
        for (int i = 0; i < slots; ++i) {
            slots_.push_back(std::make_unique<Slot>());
            Slot& sl = *slots_.back();
            sl.ws = std::make_unique<Workspace>(*w_, max_batch);
            check(cudaStreamCreateWithFlags(&sl.stream, cudaStreamNonBlocking), "cudaStreamCreate");
            check(cudaEventCreateWithFlags(&sl.done_event, cudaEventDisableTiming), "cudaEventCreate");
            sl.planes = pinned<float>(B * s.planes() * s.area());
            sl.records = pinned<uint8_t>(B * stones_record_bytes(s.history, s.board));
            sl.logits = pinned<float>(B * s.actions());
            sl.values = pinned<float>(B);
            if (s.ownership) sl.ownership = pinned<float>(B * s.area());
            sl.err_word = pinned<int>(1);
            *sl.err_word = 0;
        }
    } catch (...) {
        release_slots();
        throw;
    }
    reporter_ = std::thread([this] { report_loop(); });
}

void Runner::release_slots() {
    cudaSetDevice(device_);
    for (auto& sl : slots_) {
        if (sl->stream) cudaStreamSynchronize(sl->stream);
        for (void* p : {static_cast<void*>(sl->planes), static_cast<void*>(sl->records), static_cast<void*>(sl->logits),
                        static_cast<void*>(sl->values), static_cast<void*>(sl->ownership),
                        static_cast<void*>(sl->err_word)})
            if (p) cudaFreeHost(p);
        if (sl->done_event) cudaEventDestroy(sl->done_event);
        if (sl->stream) cudaStreamDestroy(sl->stream);
        sl->ws.reset();
    }
    slots_.clear();
}

Runner::~Runner() {
    {
        std::lock_guard<std::mutex> lock(mu_);
        closing_ = true;
    }
    wake_.notify_all();
    // The reporter returns once every live ticket and every refusal has had its done() call.
    if (reporter_.joinable()) reporter_.join();
    release_slots();
}

int Runner::slots() const { return int(slots_.size()); }
float* Runner::input(int slot) { return slots_.at(size_t(slot))->planes; }
uint8_t* Runner::records(int slot) { return slots_.at(size_t(slot))->records; }
const float* Runner::logits(int slot) const { return slots_.at(size_t(slot))->logits; }
const float* Runner::values(int slot) const { return slots_.at(size_t(slot))->values; }
const float* Runner::ownership(int slot) const { return slots_.at(size_t(slot))->ownership; }

void Runner::enqueue(Slot& sl, int B, Input from) {
    if (B < 1 || B > max_batch_)
        throw std::invalid_argument("runner: batch out of range (" + std::to_string(B) + " positions, at most " +
                                    std::to_string(max_batch_) + ")");
    check(cudaSetDevice(device_), "cudaSetDevice");
    Workspace& ws = *sl.ws;
    if (from == Input::kRecords) {
        const size_t bytes = size_t(B) * stones_record_bytes(shape_.history, shape_.board);
        check(cudaMemcpyAsync(ws.records, sl.records, bytes, cudaMemcpyHostToDevice, sl.stream), "records");
        const EncodeArgs e{ws.records, B, shape_.history, shape_.board, ws.stage};
        check(launch_encode_planes(e, sl.stream), "encode");
    } else {
        check(cudaMemcpyAsync(ws.stage, sl.planes, size_t(B) * shape_.planes() * shape_.area() * 4,
                              cudaMemcpyHostToDevice, sl.stream), "input");
    }
    encode_forward(*w_, ws, B, sl.stream, false);
    if (const int delay_us = hooks().copy_out_delay_us.load(); delay_us > 0)
        check(launch_spin(1000ull * unsigned(delay_us), sl.stream), "copy-out delay");
    check(cudaMemcpyAsync(sl.logits, ws.logits, size_t(B) * shape_.actions() * 4, cudaMemcpyDeviceToHost, sl.stream),
          "logits");
    check(cudaMemcpyAsync(sl.values, ws.values, size_t(B) * 4, cudaMemcpyDeviceToHost, sl.stream), "values");
    if (shape_.ownership)
        check(cudaMemcpyAsync(sl.ownership, ws.ownership, size_t(B) * shape_.area() * 4, cudaMemcpyDeviceToHost,
                              sl.stream), "ownership");
    check(cudaMemcpyAsync(sl.err_word, ws.err, sizeof(int), cudaMemcpyDeviceToHost, sl.stream), "error word");
}

void Runner::begin(int slot, int B, Done done, Input from) {
    if (slot < 0 || slot >= slots()) {
        refuse(slot, std::move(done), "runner: slot out of range");
        return;
    }
    Slot& sl = *slots_[size_t(slot)];
    if (sl.live.load(std::memory_order_acquire)) {
        refuse(slot, std::move(done), "runner: slot " + std::to_string(slot) + " already has a pass in flight");
        return;
    }
    std::string error;
    try {
        enqueue(sl, B, from);
    } catch (const std::exception& e) {
        error = e.what();
    }
    // The event marks the end of everything enqueued above (all of it when
    // enqueueing failed part way), so the slot's staging is not reused
    // while a copy may still touch it.
    if (const cudaError_t e = cudaEventRecord(sl.done_event, sl.stream); e != cudaSuccess) {
        cudaGetLastError();
        if (error.empty()) error = std::string("cuda: cudaEventRecord: ") + cudaGetErrorString(e);
    }
    sl.done = std::move(done);
    sl.enqueue_error = std::move(error);
    sl.issued = Clock::now();
    {
        std::lock_guard<std::mutex> lock(mu_);
        sl.live.store(true, std::memory_order_release);
    }
    wake_.notify_all();
}

void Runner::refuse(int slot, Done done, std::string error) {
    {
        std::lock_guard<std::mutex> lock(mu_);
        refused_.push_back(Refusal{slot, std::move(done), std::move(error)});
    }
    wake_.notify_all();
}

bool Runner::any_live() const {
    for (const auto& sl : slots_)
        if (sl->live.load(std::memory_order_acquire)) return true;
    return false;
}

Clock::time_point Runner::predicted_finish(const Slot& sl) const {
    // The GPU runs the slots' passes one after another, so a pass issued
    // while another ran starts when that one was reported, not when issued.
    const Clock::time_point start = std::max(sl.issued, last_finish_);
    return start + std::chrono::duration_cast<Clock::duration>(std::chrono::duration<double, std::micro>(service_us_));
}

int Runner::await_first(cudaError_t* status) {
    Micros backoff = kBackoffFirst;
    for (;;) {
        Clock::time_point due = Clock::time_point::max();
        bool any = false;
        for (size_t i = 0; i < slots_.size(); ++i) {
            const Slot& sl = *slots_[i];
            if (!sl.live.load(std::memory_order_acquire)) continue;
            any = true;
            const cudaError_t q = cudaEventQuery(sl.done_event);
            if (q != cudaErrorNotReady) {
                *status = q;
                return int(i);
            }
            due = std::min(due, predicted_finish(sl));
        }
        if (!any) return -1;
        const Micros lead = std::max(kMinLead, Micros(int64_t(service_us_ / 8)));
        const Micros window = std::max(kMinWindow, Micros(int64_t(service_us_ / 4)));
        const Clock::time_point now = Clock::now();
        if (now + lead < due) {
            std::this_thread::sleep_until(due - lead);
        } else if (now < due + window) {
            std::this_thread::yield();
        } else {
            std::this_thread::sleep_for(backoff);
            backoff = std::min(kBackoffLast, 2 * backoff);
        }
    }
}

void Runner::report_loop() {
    cudaSetDevice(device_);
    std::unique_lock<std::mutex> lock(mu_);
    for (;;) {
        wake_.wait(lock, [&] { return closing_ || !refused_.empty() || any_live(); });
        if (!refused_.empty()) {
            Refusal r = std::move(refused_.front());
            refused_.pop_front();
            lock.unlock();
            ++hooks().passes_completed;
            if (r.done) r.done(r.slot, r.error);
            lock.lock();
            continue;
        }
        if (!any_live()) {
            if (closing_) return;
            continue;
        }
        lock.unlock();
        cudaError_t status = cudaSuccess;
        const int slot = await_first(&status);
        if (slot >= 0) report(slot, status);
        lock.lock();
    }
}

void Runner::report(int slot, cudaError_t status) {
    Slot& sl = *slots_[size_t(slot)];
    const Clock::time_point now = Clock::now();
    // Service time of this pass: from when the GPU could start it to now.
    const double took = std::chrono::duration<double, std::micro>(now - std::max(sl.issued, last_finish_)).count();
    service_us_ = service_us_ <= 0.0 ? took : service_us_ + 0.25 * (took - service_us_);
    last_finish_ = now;

    std::string error = std::move(sl.enqueue_error);
    if (error.empty() && status != cudaSuccess) error = std::string("cuda: ") + cudaGetErrorString(status);
    if (error.empty() && *sl.err_word != 0) error = "cuda: " + kernel_error_text(*sl.err_word);
    *sl.err_word = 0;
    const bool injected = hooks().pass_marked_to_fail();
    if (injected && error.empty()) error = "cuda: injected failure (a test hook)";
    Done done = std::move(sl.done);
    sl.done = nullptr;
    sl.enqueue_error.clear();
    ++hooks().passes_completed;
    // Lowered before done(): the hub may begin this slot again from its callback.
    sl.live.store(false, std::memory_order_release);
    if (done) done(slot, error);
}

// -------------------------------------------------------------- memory

double hub_bytes(const NetShape& s, int precision, int max_batch, int slots) {
    return double(slots) * double(Workspace::bytes_for(s, precision, max_batch)) +
           double(Weights::bytes_for(s, precision));
}

namespace {

// Bytes a new allocation may take on the current device: the test hook's
// stand-in limit when set, else the free memory less the reserve.
double headroom_bytes() {
    if (const size_t limit = hooks().memory_limit.load(); limit > 0) return double(limit);
    size_t free_bytes = 0, total_bytes = 0;
    check(cudaMemGetInfo(&free_bytes, &total_bytes), "cudaMemGetInfo");
    return std::max(0.0, double(free_bytes) - kReserveBytes);
}

// The reference's refusal text (src/cuda/cuda_runner.cu:218-222), which
// callers and tests match.
std::string refusal_text(double need, double have, int max_batch, int hubs) {
    char hubs_note[32] = "";
    if (hubs > 1) std::snprintf(hubs_note, sizeof hubs_note, " (%d hubs)", hubs);
    char text[256];
    std::snprintf(text, sizeof text,
                  "cuda: inference needs %lld MB of GPU memory at inference_batch %d%s, more than the %lld MB the GPU "
                  "has free; lower inference_batch",
                  static_cast<long long>(need / 1e6), max_batch, hubs_note, static_cast<long long>(have / 1e6));
    return text;
}

}  // namespace

void check_fits(int device, double need, int max_batch, int hubs) {
    require_device(device);
    const double have = headroom_bytes();
    if (need > have) throw std::runtime_error(refusal_text(need, have, max_batch, hubs));
}

}  // namespace azb
