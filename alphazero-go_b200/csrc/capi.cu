// The C ABI (include/azb200.h) over the engine's classes: every entry point
// catches exceptions and turns them into a negative return and a message.
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/azb200.h"
#include "capi_types.hpp"
#include "engine.hpp"

using namespace azb;

struct azb_runner {
    std::unique_ptr<Runner> impl;
};

namespace {

void put_text(char* dst, size_t cap, const std::string& s) {
    if (!dst || cap == 0) return;
    const size_t n = std::min(cap - 1, s.size());
    std::memcpy(dst, s.data(), n);
    dst[n] = '\0';
}

template <class Fn>
int guarded(char* err, size_t cap, const char* prefix, Fn fn) {
    try {
        fn();
        return 0;
    } catch (const std::exception& e) {
        put_text(err, cap, std::string(prefix) + e.what());
    } catch (...) {
        put_text(err, cap, std::string(prefix) + "unknown error");
    }
    return -1;
}

} // namespace

extern "C" {

int azb_cuda_built(void) { return 1; }

int azb_cuda_available(int device, char* why, size_t why_cap) {
    const DeviceInfo& d = device_info(device);
    if (!d.usable) put_text(why, why_cap, d.why);
    return d.usable ? 1 : 0;
}

int azb_describe(int device, int precision, char* out, size_t cap) {
    const DeviceInfo& d = device_info(device);
    if (!d.usable) {
        put_text(out, cap, d.why);
        return -1;
    }
    put_text(out, cap, d.description + ", " + precision_name(precision));
    return 0;
}

int azb_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

// ------------------------------------------------------------ sync infer

int azb_infer_create(const azb_net_desc* desc, const float* params, size_t n_params, const float* buffers,
                     size_t n_buffers, int max_batch, int device, int precision, azb_infer** out, char* err,
                     size_t err_cap) {
    if (out) *out = nullptr;
    return guarded(err, err_cap, "", [&] {
        if (!desc || !out) throw std::invalid_argument("azb_infer_create: null argument");
        auto h = std::make_unique<azb_infer>();
        h->impl = std::make_unique<Inference>(NetShape::from(*desc), params, n_params, buffers, n_buffers, max_batch,
                                              device, precision);
        *out = h.release();
    });
}

void azb_infer_destroy(azb_infer* h) { delete h; }

int azb_infer_run(azb_infer* h, const float* input, int B, float* logits, float* values, float* ownership,
                  float* probs, char* err, size_t err_cap) {
    return guarded(err, err_cap, "GPU inference failed: ",
                   [&] { h->impl->infer(input, B, logits, values, ownership, probs); });
}

size_t azb_infer_bytes(const azb_infer* h) { return h ? h->impl->bytes() : 0; }

int azb_infer_stage(azb_infer* h, const float* input, int B, char* err, size_t err_cap) {
    return guarded(err, err_cap, "", [&] { h->impl->stage(input, B); });
}

int azb_infer_enqueue(azb_infer* h, int B) {
    try {
        h->impl->enqueue(B);
        return 0;
    } catch (...) {
        return -1;
    }
}

int azb_infer_sync(azb_infer* h, char* err, size_t err_cap) {
    return guarded(err, err_cap, "GPU inference failed: ", [&] { h->impl->sync(); });
}

void* azb_infer_stream(azb_infer* h) { return h ? static_cast<void*>(h->impl->stream()) : nullptr; }

int azb_infer_time(azb_infer* h, int B, int warmup, int steps, int with_copies, double* ms, double* conv_ms,
                   char* err, size_t err_cap) {
    return guarded(err, err_cap, "GPU inference failed: ",
                   [&] { h->impl->time(B, warmup, steps, with_copies != 0, ms, conv_ms); });
}

size_t azb_stones_record_bytes(int history, int board) {
    return history < 1 || board < 1 ? 0 : stones_record_bytes(history, board);
}

int azb_infer_run_stones(azb_infer* h, const uint8_t* records, int B, float* logits, float* values, float* ownership,
                         char* err, size_t err_cap) {
    return guarded(err, err_cap, "GPU inference failed: ", [&] {
        if (!h || !records || !logits || !values) throw std::invalid_argument("azb_infer_run_stones: null argument");
        h->impl->infer_stones(records, B, logits, values, ownership);
    });
}

int azb_infer_time_stages(azb_infer* h, int B, int steps, double* stage_ms, char* err, size_t err_cap) {
    return guarded(err, err_cap, "GPU inference failed: ", [&] {
        if (!stage_ms) throw std::invalid_argument("azb_infer_time_stages: null stage_ms");
        double ms = 0.0;
        h->impl->time(B, 0, steps, false, &ms, nullptr, stage_ms);
    });
}

int azb_infer_read(azb_infer* h, int B, float* logits, float* values, float* ownership, float* probs, char* err,
                   size_t err_cap) {
    return guarded(err, err_cap, "GPU inference failed: ",
                   [&] { h->impl->read(B, logits, values, ownership, probs); });
}

// ---------------------------------------------------------------- runner

int azb_runner_create(const azb_net_desc* desc, const float* params, size_t n_params, const float* buffers,
                      size_t n_buffers, int max_batch, int slots, int device, int precision, azb_runner** out,
                      char* err, size_t err_cap) {
    if (out) *out = nullptr;
    return guarded(err, err_cap, "", [&] {
        if (!desc || !out) throw std::invalid_argument("azb_runner_create: null argument");
        auto r = std::make_unique<azb_runner>();
        r->impl = std::make_unique<Runner>(NetShape::from(*desc), params, n_params, buffers, n_buffers, max_batch,
                                           slots, device, precision);
        *out = r.release();
    });
}

void azb_runner_destroy(azb_runner* r) { delete r; }

int azb_runner_slots(const azb_runner* r) { return r ? r->impl->slots() : 0; }
int azb_runner_max_batch(const azb_runner* r) { return r ? r->impl->max_batch() : 0; }

float* azb_runner_input(azb_runner* r, int slot) {
    if (!r || slot < 0 || slot >= r->impl->slots()) return nullptr;
    return r->impl->input(slot);
}

namespace {
int begin_pass(azb_runner* r, int slot, int B, azb_done_fn done, void* ctx, Runner::Input from) {
    if (!r || slot < 0 || slot >= r->impl->slots()) return -1;
    r->impl->begin(slot, B, [done, ctx](int s, const std::string& error) {
        if (done) done(ctx, s, error.c_str());
    }, from);
    return 0;
}
}  // namespace

int azb_runner_begin(azb_runner* r, int slot, int B, azb_done_fn done, void* ctx) {
    return begin_pass(r, slot, B, done, ctx, Runner::Input::kPlanes);
}

uint8_t* azb_runner_records(azb_runner* r, int slot) {
    if (!r || slot < 0 || slot >= r->impl->slots()) return nullptr;
    return r->impl->records(slot);
}

int azb_runner_begin_stones(azb_runner* r, int slot, int B, azb_done_fn done, void* ctx) {
    return begin_pass(r, slot, B, done, ctx, Runner::Input::kRecords);
}

const float* azb_runner_logits(const azb_runner* r, int slot) {
    return r && slot >= 0 && slot < r->impl->slots() ? r->impl->logits(slot) : nullptr;
}
const float* azb_runner_values(const azb_runner* r, int slot) {
    return r && slot >= 0 && slot < r->impl->slots() ? r->impl->values(slot) : nullptr;
}
const float* azb_runner_ownership(const azb_runner* r, int slot) {
    return r && slot >= 0 && slot < r->impl->slots() ? r->impl->ownership(slot) : nullptr;
}

// ---------------------------------------------------------------- memory

size_t azb_workspace_bytes(const azb_net_desc* desc, int max_batch, int precision) {
    try {
        return Workspace::bytes_for(NetShape::from(*desc), precision, max_batch);
    } catch (...) {
        return 0;
    }
}

int azb_check_memory(const azb_net_desc* desc, int inference_batch, int hubs, int slots_per_hub, int device,
                     int precision, char* err, size_t err_cap) {
    return guarded(err, err_cap, "", [&] {
        if (inference_batch < 1 || hubs < 1 || slots_per_hub < 1)
            throw std::invalid_argument("checkCudaInferenceMemory: bad arguments");
        const NetShape s = NetShape::from(*desc);
        check_fits(device, hubs * hub_bytes(s, precision, inference_batch, slots_per_hub), inference_batch, hubs);
    });
}

size_t azb_weights_bytes(const azb_net_desc* desc, int precision) {
    try {
        return Weights::bytes_for(NetShape::from(*desc), precision);
    } catch (...) {
        return 0;
    }
}

int azb_check_bytes(int device, double bytes, int inference_batch, int hubs, char* err, size_t err_cap) {
    return guarded(err, err_cap, "", [&] { check_fits(device, bytes, inference_batch, hubs); });
}

// ------------------------------------------------------------ test hooks

void azb_probe_set_hub_chaos_seed(uint64_t seed) { hooks().chaos_seed = seed; }
uint64_t azb_probe_hub_chaos_seed(void) { return hooks().chaos_seed.load(); }
void azb_probe_fail_passes_after(int n) { hooks().fail_countdown = n > 0 ? n + 1 : 0; }
void azb_probe_set_memory_limit(size_t bytes) { hooks().memory_limit = bytes; }
long long azb_probe_passes_completed(void) { return hooks().passes_completed.load(); }
void azb_probe_set_copy_out_delay(int us) { hooks().copy_out_delay_us = us > 0 ? us : 0; }
void azb_probe_set_conv_path(int path) { set_conv_path(path); }
void azb_probe_set_conv_segment(int steps) { set_conv_segment(steps); }
void azb_probe_set_tower_fused(int mode) { set_tower_fused(mode); }
void azb_probe_set_tower_persistent(int mode) { set_tower_persistent(mode); }
void azb_probe_starve_tower(int on) { set_tower_starve(on); }

int azb_probe_binary_version(int device) { return device_info(device).binary_version; }
int azb_probe_device_architecture(int device) { return device_info(device).architecture; }

int azb_probe_fill(int device, float* data, size_t n, float value, size_t tail, char* err, size_t err_cap) {
    return guarded(err, err_cap, "", [&] {
        require_device(device);
        float* d = nullptr;
        check(cudaMalloc(&d, (n + tail + 1) * sizeof(float)), "cudaMalloc");
        cudaError_t e = cudaMemcpy(d, data, (n + tail) * sizeof(float), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = launch_fill(d, n, value, nullptr);
        if (e == cudaSuccess) e = cudaMemcpy(data, d, (n + tail) * sizeof(float), cudaMemcpyDeviceToHost);
        cudaFree(d);
        check(e, "fill");
    });
}

int azb_probe_tanh(int device, float* data, size_t n, char* err, size_t err_cap) {
    return guarded(err, err_cap, "", [&] {
        require_device(device);
        if (n == 0) return;
        float* d = nullptr;
        check(cudaMalloc(&d, n * sizeof(float)), "cudaMalloc");
        cudaError_t e = cudaMemcpy(d, data, n * sizeof(float), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = launch_tanh(d, n, nullptr);
        if (e == cudaSuccess) e = cudaMemcpy(data, d, n * sizeof(float), cudaMemcpyDeviceToHost);
        cudaFree(d);
        check(e, "tanh");
    });
}

int azb_probe_bounded_wait(int device, unsigned long long limit_ns, char* err, size_t err_cap) {
    int code = -1;
    const int rc = guarded(err, err_cap, "", [&] {
        require_device(device);
        int* d = nullptr;
        check(cudaMalloc(&d, sizeof(int)), "cudaMalloc");
        cudaError_t e = cudaMemset(d, 0, sizeof(int));
        if (e == cudaSuccess) e = launch_bounded_wait_probe(d, limit_ns, nullptr);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        int host = -1;
        if (e == cudaSuccess) e = cudaMemcpy(&host, d, sizeof(int), cudaMemcpyDeviceToHost);
        cudaFree(d);
        check(e, "bounded wait probe");
        code = host;
    });
    return rc == 0 ? code : -1;
}

int azb_probe_umma(int device, int precision, int n_out, int halo_rows, int shift_rows, int k_chunks,
                   int base_offset_mode, const float* a, const float* w, float* d, char* err, size_t err_cap) {
    return guarded(err, err_cap, "", [&] {
        require_device(device);
        if (halo_rows < 128 || halo_rows > 256 || k_chunks < 1) throw std::invalid_argument("azb_probe_umma: bad shape");
        const int KC = chunk_channels(precision);
        const size_t esz = size_t(elem_bytes(precision));
        const size_t inner_a = size_t(KC) * k_chunks, inner_w = size_t(KC) * 9 * k_chunks;
        std::vector<uint8_t> ha(size_t(halo_rows) * inner_a * esz), hw(size_t(n_out) * inner_w * esz);
        auto conv = [&](const float* src, size_t n, uint8_t* dst) {
            for (size_t i = 0; i < n; ++i) {
                if (precision == kBF16) {
                    uint32_t u;
                    std::memcpy(&u, &src[i], 4);
                    const uint16_t h = static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
                    std::memcpy(dst + i * 2, &h, 2);
                } else {
                    std::memcpy(dst + i * 4, &src[i], 4);
                }
            }
        };
        conv(a, size_t(halo_rows) * inner_a, ha.data());
        conv(w, size_t(n_out) * inner_w, hw.data());
        void *da = nullptr, *dw = nullptr;
        float* dd = nullptr;
        int* de = nullptr;
        check(cudaMalloc(&da, ha.size()), "cudaMalloc");
        check(cudaMalloc(&dw, hw.size()), "cudaMalloc");
        check(cudaMalloc(&dd, size_t(128) * n_out * 4), "cudaMalloc");
        check(cudaMalloc(&de, 4), "cudaMalloc");
        cudaError_t e = cudaMemcpy(da, ha.data(), ha.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(dw, hw.data(), hw.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemset(de, 0, 4);
        std::string fail;
        if (e == cudaSuccess) {
            try {
                ConvMaps m;
                m.a = m.a_lo = make_tensor_map(da, precision, inner_a, uint64_t(halo_rows), uint32_t(KC), uint32_t(halo_rows));
                m.w = m.w_lo = make_tensor_map(dw, precision, inner_w, uint64_t(n_out), uint32_t(KC), uint32_t(n_out));
                e = launch_umma_probe(m, n_out, precision, halo_rows, shift_rows, k_chunks, base_offset_mode, dd, de, nullptr);
            } catch (const std::exception& ex) {
                fail = ex.what();
            }
        }
        if (e == cudaSuccess && fail.empty()) e = cudaDeviceSynchronize();
        int code = 0;
        if (e == cudaSuccess && fail.empty()) e = cudaMemcpy(d, dd, size_t(128) * n_out * 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && fail.empty()) e = cudaMemcpy(&code, de, 4, cudaMemcpyDeviceToHost);
        cudaFree(da);
        cudaFree(dw);
        cudaFree(dd);
        cudaFree(de);
        if (!fail.empty()) throw std::runtime_error(fail);
        check(e, "umma probe");
        if (code) throw std::runtime_error("umma probe: " + kernel_error_text(code));
    });
}

// ---------------------------------------------------------------- layout

int azb_layout_count(const azb_net_desc* desc, int which) {
    try {
        const Layout L = Layout::of(NetShape::from(*desc));
        return static_cast<int>(which == 0 ? L.params.size() : L.buffers.size());
    } catch (...) {
        return -1;
    }
}

int azb_layout_entry(const azb_net_desc* desc, int which, int index, char* name, size_t name_cap, size_t* size,
                     size_t* offset) {
    try {
        const Layout L = Layout::of(NetShape::from(*desc));
        const auto& list = which == 0 ? L.params : L.buffers;
        if (index < 0 || size_t(index) >= list.size()) return -1;
        const LayoutEntry& e = list[size_t(index)];
        put_text(name, name_cap, e.name);
        if (size) *size = e.size;
        if (offset) *offset = e.offset;
        return 0;
    } catch (...) {
        return -1;
    }
}

size_t azb_layout_floats(const azb_net_desc* desc, int which) {
    try {
        const Layout L = Layout::of(NetShape::from(*desc));
        return which == 0 ? L.param_floats : L.buffer_floats;
    } catch (...) {
        return 0;
    }
}

} // extern "C"
