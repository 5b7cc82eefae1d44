// The engine's host side: device context, weights in kernel layout,
// workspaces, the forward pass, the synchronous inference object and the
// asynchronous batch runner. Plain C++17 over the CUDA runtime; the C ABI
// (include/azb200.h) is a thin layer over these classes (capi.cu).
#pragma once
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstddef>
#include <cstdint>
#include <deque>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "kernels.hpp"

struct azb_net_desc;

namespace azb {

// Throws std::runtime_error("cuda: <what>: <error string>") unless cudaSuccess.
void check(cudaError_t e, const char* what);

// NetConfig with the engine's derived shapes.
struct NetShape {
    int board, history, blocks, filters, value_hidden, ownership;
    int planes() const { return 2 * history + 2; }
    int area() const { return board * board; }
    int actions() const { return area() + 1; }
    static NetShape from(const azb_net_desc& d);
};

// ParamLayout::of (include/azgo/param_layout.hpp:18-34; src/param_layout.cpp:18-29):
// params() then buffers() order, each tensor at a 64-float offset.
struct LayoutEntry {
    std::string name;
    size_t size, offset;
};
struct Layout {
    std::vector<LayoutEntry> params, buffers;
    size_t param_floats = 0, buffer_floats = 0;
    static Layout of(const NetShape& s);
    const LayoutEntry& param(const std::string& name) const;
    const LayoutEntry& buffer(const std::string& name) const;
};

// Validates a device, checks the machine code matches it, runs a first kernel.
struct DeviceInfo {
    bool usable = false;
    std::string why, name, description;   // description without the precision
    int architecture = 0, binary_version = 0, sms = 0;
    size_t total_memory = 0;
};
const DeviceInfo& device_info(int device);   // set up once per device (thread-safe)
const DeviceInfo& require_device(int device);   // throws the reason when unusable

const char* precision_name(int precision);

// The fused tower's plan for a shape (boards whose frame rows fit one
// 128-row tile, 32 or 64 output channels, at least one block; its shared
// memory fits): false when the per-layer kernels run the tower.
bool fused_tower_plan(const NetShape& s, int precision, FusedArgs* plan);
// Test hook: -1 the default (fused where it applies), 0 per-layer kernels always.
void set_tower_fused(int mode);

// One network's weights on one device, in the kernels' layouts.
class Weights {
public:
    Weights(const NetShape& s, int precision, int device, const float* params, size_t n_params, const float* buffers,
            size_t n_buffers);
    ~Weights();
    Weights(const Weights&) = delete;
    Weights& operator=(const Weights&) = delete;

    struct Conv {
        const float* scale = nullptr;   // [n_out] folded batch norm
        const float* shift = nullptr;
        const void* w = nullptr;        // [n_out][9*cpad] kernel layout (split: tf32 high part)
        const void* w_lo = nullptr;     // split: low part
        CUtensorMap map_w{}, map_w_lo{};
        CUtensorMap map_w_pair{}, map_w_lo_pair{};   // boxes of n_out/2 rows, for the CTA-pair form
    };
    const NetShape& shape() const { return shape_; }
    int precision() const { return precision_; }
    int device() const { return device_; }
    int cpad() const { return cpad_; }      // channels per stored pixel row
    int n_out() const { return n_out_; }    // MMA N (filters rounded up)
    size_t bytes() const { return bytes_; }
    int kstem() const { return kstem_; }    // the stem operand's K: 9*planes rounded up to whole chunks
    // 0: the stem (one-tap GEMM over the packed operand); 1 + 2*block + (0|1): the tower.
    const Conv& conv(int i) const { return convs_[static_cast<size_t>(i)]; }
    HeadArgs head_args() const { return head_; }   // weights only
    // The tower convs' table for the fused tower (device memory; null without blocks).
    const FusedLayer* fused_layers() const { return fused_; }

    // Bytes of the device arena for these shapes (the memory checks).
    static size_t bytes_for(const NetShape& s, int precision);

private:
    NetShape shape_;
    int precision_, device_, cpad_, n_out_, kstem_;
    size_t bytes_ = 0;
    void* arena_ = nullptr;
    std::vector<Conv> convs_;
    HeadArgs head_{};
    const FusedLayer* fused_ = nullptr;
};

// Activations and outputs for up to max_batch positions.
class Workspace {
public:
    Workspace(const Weights& w, int max_batch);
    // The same layout placed in caller-provided device memory of at least
    // bytes_for(shape, precision, max_batch) bytes, 256-byte aligned: nothing
    // is allocated, cleared or freed (the caller zeroes it first, since the
    // frames' padding rows must read zero).
    Workspace(const Weights& w, int max_batch, void* memory);
    ~Workspace();
    Workspace(const Workspace&) = delete;
    Workspace& operator=(const Workspace&) = delete;
    int max_batch() const { return max_batch_; }
    size_t bytes() const { return bytes_; }
    static size_t bytes_for(const NetShape& s, int precision, int max_batch);

    float* stage = nullptr;       // [max_batch][planes][area] fp32 input
    void* stem_in = nullptr;      // frame rows x kstem: the stem's packed operand
    void* stem_in_lo = nullptr;   // split mode
    void* trunk[3] = {};          // frame rows x cpad
    void* trunk_lo[3] = {};       // split mode
    float* logits = nullptr;      // [max_batch][actions]
    float* values = nullptr;      // [max_batch]
    float* ownership = nullptr;   // [max_batch][area] when the head exists
    float* probs = nullptr;       // [max_batch][actions]
    float* feat = nullptr;        // [max_batch][feat_floats]: the heads' 1x1 conv features
    float* hid = nullptr;         // [max_batch][value_hidden]: value FC1 output
    uint8_t* records = nullptr;   // [max_batch][stones_record_bytes]: encoder input (infer_stones)
    int* err = nullptr;           // kernel error word
    // The persistent tower's counters: per tower conv and tile group (up to
    // the tiles of max_batch), then the pass's next-item counter.
    unsigned* tower_flags = nullptr;
    size_t tower_flag_count = 0;
    // The head tail kernel's counters (one per 16 boards), just before the
    // tower's: the stem operand kernel zeroes both at a pass's start.
    unsigned* tail_count = nullptr;
    size_t tail_count_n = 0;
    CUtensorMap map[3]{}, map_lo[3]{};
    CUtensorMap emap[3]{};        // the frames in the conv epilogue's {32, 32} boxes (split mode: high planes)
    CUtensorMap emap_lo[3]{};     // split mode: the low planes in the same boxes
    // The fused tower (small boards): its plan and trunk[0] (its input and
    // output, in place) in boxes of {chunk, group * S} rows.
    bool fused = false;
    FusedArgs fused_plan{};
    CUtensorMap fmap{}, fmap_lo{};
    CUtensorMap smap{}, smap_lo{};   // the stem's packed operand in the same boxes (when the stem runs there)
    CUtensorMap map_stem{}, map_stem_lo{};

private:
    void place(const Weights& w, uint8_t* base);   // carves the buffers and builds the tensor maps
    int max_batch_;
    size_t bytes_ = 0;
    void* arena_ = nullptr;
};

// Per-launch timing, for the rooflines: events around each launch of a
// pass. Slots: the stem operand, the stem GEMM, the three head launches,
// then the tower convs (kSlotTower + i for conv i of 2 x blocks).
struct PassTimer {
    std::vector<cudaEvent_t> begin, end;
    bool enabled = false;
};
enum TimerSlot : int { kSlotStemPack = 0, kSlotStemGemm, kSlotHeadConv, kSlotHeadFc, kSlotHeadOut, kSlotTower };
// Stage totals Inference::time reports: these six, in this order.
constexpr int kTimedStages = 6;   // stem operand, stem GEMM, tower, head conv, head tail, (0: no finish launch)

// Network::forward (src/network.cpp:228-309) on the GPU: stem, the tower's
// fused convolutions, the fused heads; all on one stream.
size_t feat_floats(const NetShape& s);   // floats per board of the heads' feature buffer
void encode_forward(const Weights& w, Workspace& ws, int B, cudaStream_t s, bool probs, PassTimer* timer = nullptr);

// A row-major [rows][inner] tensor read by TMA in boxes of box_inner x
// box_rows with the 128-byte (or 64-byte) swizzle; rows outside [0, rows)
// read as zero and are not written.
CUtensorMap make_tensor_map(const void* base, int precision, uint64_t inner, uint64_t rows, uint32_t box_inner,
                            uint32_t box_rows, int swizzle_bytes = 128);

// Turns a nonzero kernel error word into the message a pass reports.
std::string kernel_error_text(int code);

// CudaInference (include/azgo/cuda.hpp:72-84).
class Inference {
public:
    Inference(const NetShape& s, const float* params, size_t n_params, const float* buffers, size_t n_buffers,
              int max_batch, int device, int precision);
    ~Inference();
    void infer(const float* input, int B, float* logits, float* values, float* ownership, float* probs);
    // The same from position records (kernels.hpp's EncodeArgs): the planes
    // are encoded on the device, so only the records cross to it.
    void infer_stones(const uint8_t* records, int B, float* logits, float* values, float* ownership);
    size_t bytes() const { return ws_->bytes(); }
    void stage(const float* input, int B);
    void enqueue(int B);
    void sync();
    void read(int B, float* logits, float* values, float* ownership, float* probs);
    cudaStream_t stream() const { return stream_; }
    const Weights& weights() const { return *w_; }
    int* error_host() const { return err_host_; }   // pinned, one int
    // (total ms of K passes, summed conv-kernel ms)
    // `steps` passes after `warmup`: their total ms; with conv_ms or
    // stage_ms, `steps` more passes with an event around every launch give
    // the summed tower-conv ms and the kTimedStages stage totals.
    void time(int B, int warmup, int steps, bool with_copies, double* ms, double* conv_ms, double* stage_ms = nullptr);

private:
    void check_error_word();
    int device_;
    std::unique_ptr<Weights> w_;
    std::unique_ptr<Workspace> ws_;
    cudaStream_t stream_ = nullptr;
    int* err_host_ = nullptr;    // pinned
    float* pin_in_ = nullptr;    // pinned staging for the end-to-end timing
    float* pin_out_ = nullptr;
};

// The BatchRunner (include/azgo/inference_hub.hpp:41-53): slots of pinned
// staging and a workspace each, one reporter thread for every done() call
// (runner.cu).
class Runner {
public:
    using Done = std::function<void(int slot, const std::string& error)>;
    // What begin() reads from the slot's staging: float planes (input()) or
    // position records for the device encoder (records()).
    enum class Input { kPlanes, kRecords };
    Runner(const NetShape& s, const float* params, size_t n_params, const float* buffers, size_t n_buffers,
           int max_batch, int slots, int device, int precision);
    ~Runner();
    Runner(const Runner&) = delete;
    Runner& operator=(const Runner&) = delete;
    int slots() const;
    int max_batch() const { return max_batch_; }
    float* input(int slot);       // [max_batch][planes][area]
    uint8_t* records(int slot);   // [max_batch][stones_record_bytes(history, board)]
    const float* logits(int slot) const;
    const float* values(int slot) const;
    const float* ownership(int slot) const;
    // Returns at once; done(slot, error) follows exactly once, from the
    // reporter thread, after the outputs reached the slot's staging.
    void begin(int slot, int B, Done done, Input from = Input::kPlanes);

private:
    struct Slot;
    struct Refusal {
        int slot;
        Done done;
        std::string error;
    };
    void enqueue(Slot& sl, int B, Input from);
    void refuse(int slot, Done done, std::string error);
    bool any_live() const;
    std::chrono::steady_clock::time_point predicted_finish(const Slot& sl) const;
    int await_first(cudaError_t* status);
    void report(int slot, cudaError_t status);
    void report_loop();
    void release_slots();

    NetShape shape_;
    int device_, max_batch_;
    std::unique_ptr<Weights> w_;
    std::vector<std::unique_ptr<Slot>> slots_;
    std::mutex mu_;
    std::condition_variable wake_;
    std::deque<Refusal> refused_;
    bool closing_ = false;
    // The reporter's own state: its estimate of a pass's GPU time and when it last reported one.
    double service_us_ = 0.0;
    std::chrono::steady_clock::time_point last_finish_{};
    std::thread reporter_;
};

// Device memory of `slots` workspaces and one weight replica, and the
// admission check before allocating it (checkCudaInferenceMemory,
// include/azgo/cuda.hpp:63): throws the reference's "cuda: inference needs
// N MB ... lower inference_batch" when `need` exceeds the free memory less a
// 512 MB reserve (or the test hook's limit).
double hub_bytes(const NetShape& s, int precision, int max_batch, int slots);
void check_fits(int device, double need, int max_batch, int hubs);

// Test hooks (src/cuda/cuda_runner.cu:39-45, 258-267).
struct Hooks {
    std::atomic<uint64_t> chaos_seed{0};
    std::atomic<int> fail_countdown{0};
    std::atomic<size_t> memory_limit{0};
    std::atomic<long long> passes_completed{0};
    std::atomic<int> copy_out_delay_us{0};
    // Steps the failure countdown for one reported pass; true for the pass it marks.
    bool pass_marked_to_fail();
};
Hooks& hooks();

} // namespace azb
