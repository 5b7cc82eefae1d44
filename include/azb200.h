/* azb200: a B200 (sm_100a) engine for the AlphaZero network evaluation of
 * robominds/alphazero-go, behind a plain C ABI.
 *
 * The engine runs Network::infer's inference forward (residual tower +
 * policy/value/ownership heads) on the GPU: tcgen05 tensor-core implicit-GEMM
 * 3x3 convolutions with batch norm, skip and ReLU fused into the epilogue,
 * and one fused head kernel. It is the drop-in for the reference's CUDA
 * engine (include/azgo/cuda.hpp) and BatchRunner (include/azgo/inference_hub.hpp):
 * the C++ bridge alphazero-go_b200/host/azgo_cuda_bridge.cpp maps these calls
 * onto those interfaces.
 *
 * Conventions: functions return 0 on success and a negative value on
 * failure, with a message in err[0..err_cap) when err is not null. No C++
 * exception crosses this boundary. Host arrays are plain float arrays in the
 * reference's layouts: input [B][planes][area], logits [B][area+1], values
 * [B], ownership [B][area]. Weights come as the two ParamLayout arenas
 * (include/azgo/param_layout.hpp:18-34): params() then buffers(), each
 * tensor at its 64-float offset.
 */
#ifndef AZB200_H
#define AZB200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* NetConfig (include/azgo/network.hpp:23-36). */
typedef struct azb_net_desc {
    int board;         /* 5..19 */
    int history;       /* planes = 2*history + 2 */
    int blocks;        /* residual blocks */
    int filters;       /* a multiple of 8, at most 256 */
    int value_hidden;
    int ownership;     /* 0/1 */
} azb_net_desc;

/* The arithmetic of a pass. TF32: fp32 activations, tf32 tensor-core
 * products, fp32 accumulation. TF32X3: the products split into tf32 high and
 * low parts (three MMAs), fp32-class results. BF16: bf16 weights and
 * activations, fp32 accumulation. */
enum { AZB_TF32 = 0, AZB_TF32X3 = 1, AZB_BF16 = 2 };

/* ---------------------------------------------------------------- layout */

/* ParamLayout::of (include/azgo/param_layout.hpp:18-34, src/param_layout.cpp:18-29)
 * for this shape: which = 0 params() order, 1 buffers() order. An adapter
 * holding the reference Network checks its tensors against these names,
 * sizes and offsets before upload, as CudaWeights::upload does
 * (src/cuda/cuda_network.cu:24-41). */
int azb_layout_count(const azb_net_desc* desc, int which);
int azb_layout_entry(const azb_net_desc* desc, int which, int index, char* name, size_t name_cap, size_t* size,
                     size_t* offset);
size_t azb_layout_floats(const azb_net_desc* desc, int which);

/* ------------------------------------------------------------ checkpoint */

/* The reference's network checkpoint (.azn: saveNetwork / loadNetwork /
 * readCheckpointConfig, include/azgo/checkpoint.hpp:12-23, src/checkpoint.cpp)
 * for hosts without the reference's Network. azb_checkpoint_config reads the
 * header's NetConfig (readCheckpointConfig) and the two arenas' sizes in
 * floats (either pointer may be null); azb_checkpoint_read reads every
 * tensor into arenas of those sizes at their layout offsets (zero between
 * tensors), checking each
 * tensor's name and size against the layout in params() then buffers()
 * order, as loadNetwork does, and sets *desc. Both return 0, or -1 with the
 * reference loader's message in err ("cannot open checkpoint <path>",
 * "<path>: truncated", "<path>: unsupported version 7", ...). Any shape the
 * reference accepts loads; the engine's own limits apply at creation. */
int azb_checkpoint_config(const char* path, azb_net_desc* desc, size_t* n_params, size_t* n_buffers, char* err,
                          size_t err_cap);
int azb_checkpoint_read(const char* path, azb_net_desc* desc, float* params, size_t n_params, float* buffers,
                        size_t n_buffers, char* err, size_t err_cap);

/* ---------------------------------------------------------------- device */

/* cudaBuilt() (include/azgo/cuda.hpp:30): 1 in this library. */
int azb_cuda_built(void);
/* cudaAvailable(&why) (include/azgo/cuda.hpp:39): 1 when device `device` is a
 * usable sm_100 GPU for this library's machine code; else 0 and the reason. */
int azb_cuda_available(int device, char* why, size_t why_cap);
/* cudaDescription() (include/azgo/cuda.hpp:49), with the precision added:
 * "<GPU> sm_100, driver API x.y, runtime x.y, kernels <8 hex>, <precision>". */
int azb_describe(int device, int precision, char* out, size_t cap);
int azb_device_count(void);
/* The device's PCI bus id ("0000:1b:00.0"), to match it with nvidia-smi. */
int azb_device_pci_bus_id(int device, char* out, size_t cap);

/* ---------------------------------------------------------- synthetic data */
/* No reference counterpart as an API: these restate the reference's seeded
 * construction so benchmarks can build the reference's own networks and
 * inputs without it. azb_synth_network = Network(cfg, seed)
 * (src/network.cpp:77-111) then a batch-norm randomiser (kind 0: gamma
 * U(0.5,1.5), beta N(0,0.1), mean N(0,0.1), var U(0.5,1.5) from
 * Rng(deriveSeed(seed,1)); kind 1: tests/test_cuda.cpp:188-204; kind -1:
 * none). azb_synth_positions: sample first+b from Rng(deriveSeed(seed, 2,
 * first+b)), encoded as encodePlanes (src/encode.cpp:14-43). */
int azb_synth_network(const azb_net_desc* desc, uint64_t seed, int kind, float* params, float* buffers);
int azb_synth_positions(const azb_net_desc* desc, uint64_t seed, long first, int B, float* out);

/* ------------------------------------------------------------ sync infer */

typedef struct azb_infer azb_infer;

/* CudaInference(net, maxBatch) (include/azgo/cuda.hpp:72-84): uploads the
 * weights once (checked against the layout: an unknown, missing or
 * mis-sized tensor is refused by name) and holds one workspace. */
int azb_infer_create(const azb_net_desc* desc, const float* params, size_t n_params, const float* buffers,
                     size_t n_buffers, int max_batch, int device, int precision, azb_infer** out, char* err,
                     size_t err_cap);
void azb_infer_destroy(azb_infer* h);
/* CudaInference::infer: copy in, forward, copy out, wait. ownership may be
 * null (needs the head otherwise); probs (softmax over area+1, may be null). */
int azb_infer_run(azb_infer* h, const float* input, int B, float* logits, float* values, float* ownership,
                  float* probs, char* err, size_t err_cap);
/* CudaInference::bytes(): GPU memory of the activations. */
size_t azb_infer_bytes(const azb_infer* h);

/* azb_infer_run without allocating: no counterpart in the reference. For
 * callers that may not allocate device memory when they evaluate -- hosts
 * whose own pool allocator owns the GPU's memory or that run under a fixed
 * device-memory budget, latency-critical paths where cudaMalloc may
 * synchronise the device. The handle is created once at set-up (that
 * allocates, and uploads the weights); this call then runs the same forward
 * pass with all its scratch (input staging, stem operand, activation frames,
 * outputs, error word) in a static 32 MiB device array that every GPU
 * loading this library holds until exit: enough, e.g., for batch 32 of the
 * 19x19 20x256 network in bf16. A batch whose scratch exceeds it is refused
 * with an error naming the size. The first call on a device looks the
 * array's address up (make it before any stream capture). Every call shares
 * the array and clears the part it uses; calls that overlap on the GPU race
 * on it and must be serialised by the caller. */
int azb_infer_run_noalloc(azb_infer* h, const float* input, int B, float* logits, float* values, float* ownership,
                          char* err, size_t err_cap);

/* Device-resident use, for timing the kernels alone: copy B positions into
 * the workspace once, then enqueue forward passes on it (no host copies). */
int azb_infer_stage(azb_infer* h, const float* input, int B, char* err, size_t err_cap);
int azb_infer_enqueue(azb_infer* h, int B);
/* Synchronizes and reports any error (CUDA or a kernel's error word). */
int azb_infer_sync(azb_infer* h, char* err, size_t err_cap);
/* The stream passes run on (a cudaStream_t), for events recorded on it. */
void* azb_infer_stream(azb_infer* h);
/* K passes of batch B after W warm-ups, timed with CUDA events on the
 * engine's stream; *ms = total milliseconds of the K passes. with_copies:
 * each pass also copies the input in from pinned host memory and the
 * outputs back (the end-to-end path). The conv kernels' own time (the sum
 * of their event-bracketed durations over the K passes) goes to *conv_ms
 * when not null. */
int azb_infer_time(azb_infer* h, int B, int warmup, int steps, int with_copies, double* ms, double* conv_ms,
                   char* err, size_t err_cap);
/* Position records for azb_infer_run_stones: per position, stones[H][n*n]
 * Color bytes (0 empty, 1 Black, 2 White; row k is the position k plies
 * ago), then toMove (1 Black, 2 White), the number of history positions
 * present (0..H), the symmetry (0..7, the reference's transformPoint
 * numbering), and zero padding: azb_stones_record_bytes(H, n) bytes. */
size_t azb_stones_record_bytes(int history, int board);
/* CudaInference::infer from position records: the reference's encodePlanes
 * (src/encode.cpp:15-43) runs on the device, so ~n*n*H bytes per position
 * cross to it instead of (2H+2)*n*n floats. No reference counterpart (the
 * reference encodes on the host: src/mcts.cpp:117-132). */
int azb_infer_run_stones(azb_infer* h, const uint8_t* records, int B, float* logits, float* values, float* ownership,
                         char* err, size_t err_cap);
/* Per-stage device time of `steps` passes (CUDA events around every launch,
 * summed over the passes): stage_ms[0..5] = stem operand, stem GEMM, tower
 * convs, head 1x1 convs, head tail (FCs, value tanh, softmax: one launch),
 * and 0 (the finish has no launch of its own). Small boards run the stem GEMM
 * and every head stage inside the tower launch.
 * Measurement only; no reference counterpart. */
int azb_infer_time_stages(azb_infer* h, int B, int steps, double* stage_ms, char* err, size_t err_cap);
/* Read back the device outputs of the last enqueued pass. */
int azb_infer_read(azb_infer* h, int B, float* logits, float* values, float* ownership, float* probs, char* err,
                   size_t err_cap);

/* --------------------------------------------------------------- runner */

typedef struct azb_runner azb_runner;
/* BatchRunner::begin's done(slot, error): error is "" on success. Called
 * exactly once per begin, from the runner's completion thread. */
typedef void (*azb_done_fn)(void* ctx, int slot, const char* error);

/* makeCudaRunner(net, maxBatch, slots) (include/azgo/cuda.hpp:58,
 * src/cuda/cuda_runner.cu:227-234): slots in [1, 2]; refuses with "cuda:
 * inference needs N MB ...; lower inference_batch" before allocating when
 * the slots would not fit the device's free memory. */
int azb_runner_create(const azb_net_desc* desc, const float* params, size_t n_params, const float* buffers,
                      size_t n_buffers, int max_batch, int slots, int device, int precision, azb_runner** out,
                      char* err, size_t err_cap);
/* Drains every pass in flight (each still gets its done call), then frees. */
void azb_runner_destroy(azb_runner* r);
int azb_runner_slots(const azb_runner* r);
int azb_runner_max_batch(const azb_runner* r);
/* BatchRunner::input(slot): pinned [max_batch][planes][area] staging. */
float* azb_runner_input(azb_runner* r, int slot);
/* BatchRunner::begin (include/azgo/inference_hub.hpp:41-53): enqueues copy
 * in, forward, copy out and returns at once. A batch out of range or an
 * enqueue error is reported through done (never by returning). */
int azb_runner_begin(azb_runner* r, int slot, int B, azb_done_fn done, void* ctx);
/* The same pass from position records instead of planes (the record
 * format of azb_stones_record_bytes): azb_runner_records(slot) is pinned
 * [max_batch][azb_stones_record_bytes(history, board)] staging, and
 * azb_runner_begin_stones encodes its first B records on the device (the
 * reference's encodePlanes, src/encode.cpp:15-43) before the forward pass,
 * so ~H*n*n bytes per position cross to the GPU instead of (2H+2)*n*n
 * floats. No reference counterpart: the reference's BatchRunner takes
 * planes only, encoded on the host (src/mcts.cpp:117-132). */
uint8_t* azb_runner_records(azb_runner* r, int slot);
int azb_runner_begin_stones(azb_runner* r, int slot, int B, azb_done_fn done, void* ctx);
const float* azb_runner_logits(const azb_runner* r, int slot);
const float* azb_runner_values(const azb_runner* r, int slot);
const float* azb_runner_ownership(const azb_runner* r, int slot);

/* ------------------------------------------------------------------ hub */

/* Leaf batching for many search threads over one runner per GPU, in one
 * process: the role of the reference's InferenceHub + WorkerEvaluators for
 * the "cuda" backend (include/azgo/inference_hub.hpp:83-150,
 * src/inference_hub.cpp:95-295), with one lane (runner) per device, so one
 * process drives several GPUs (the reference pins device 0,
 * src/cuda/cuda_context.cu:51). Each worker thread is bound to a lane and
 * calls azb_hub_evaluate, which blocks until its positions are evaluated.
 * There is no dispatcher thread: the thread that gives a request rows in the
 * filling pass copies it into the pass's pinned staging (large requests copy
 * themselves, in parallel), and the runner's completion thread copies the
 * results back; a pass launches when full or when its GPU is idle; its size
 * is capped at the largest whole number of the engine's tiles within
 * max_batch (azb_hub_pass_cap). A failed pass fails every later request
 * ("GPU inference failed: ..."); destroying the hub refuses requests that
 * have no rows yet and waits for the passes that have. Outputs are those of
 * the runner: a position's results do not depend on its pass.
 * input_mode AZB_HUB_RECORDS: passes carry position records and the GPU
 * encodes them (azb_runner_begin_stones); planes given to azb_hub_evaluate
 * are turned into records on the calling thread (0/1 stone planes only). */
typedef struct azb_hub azb_hub;
enum { AZB_HUB_PLANES = 0, AZB_HUB_RECORDS = 1 };
int azb_hub_create(const azb_net_desc* desc, const float* params, size_t n_params, const float* buffers,
                   size_t n_buffers, const int* devices, int n_devices, int max_batch, int slots, int precision,
                   int input_mode, azb_hub** out, char* err, size_t err_cap);
/* The same hub logic over a CPU stand-in for the GPU passes (no GPU): after
 * delay_us, each position's value is the FNV-1a hash of its planes' bytes,
 * top 24 bits / 2^24, and logit a is value + a; after fail_after passes
 * (when > 0) one pass fails. quantum: the boards of a whole tile. For tests. */
int azb_hub_create_fake(int board, int history, int lanes, int max_batch, int slots, int quantum, int input_mode,
                        int delay_us, int fail_after, azb_hub** out, char* err, size_t err_cap);
void azb_hub_destroy(azb_hub* h);
int azb_hub_lanes(const azb_hub* h);
int azb_hub_pass_cap(const azb_hub* h);
/* B positions ([B][planes][area] floats, or records) on lane `lane`; logits
 * [B][area+1], values [B]. Thread-safe. 0, or -1 with err. */
int azb_hub_evaluate(azb_hub* h, int lane, const float* input, int B, float* logits, float* values, char* err,
                     size_t err_cap);
int azb_hub_evaluate_records(azb_hub* h, int lane, const uint8_t* records, int B, float* logits, float* values,
                             char* err, size_t err_cap);
/* A lane's completed passes, their positions, the passes that were full
 * (exactly azb_hub_pass_cap positions) and their summed begin-to-done seconds. */
int azb_hub_stats(const azb_hub* h, int lane, long long* passes, long long* positions, long long* full_passes,
                  double* gpu_seconds);

/* ------------------------------------------------------- memory checks */

/* CudaWorkspace::bytesFor (src/cuda/cuda_network.cu:199-201): device bytes
 * of one slot's workspace at max_batch. */
size_t azb_workspace_bytes(const azb_net_desc* desc, int max_batch, int precision);
/* checkCudaInferenceMemory (include/azgo/cuda.hpp:63): 0 when `hubs` hubs of
 * `slots_per_hub` slots at inference_batch fit on `device`, else -1 and the
 * reference's message. */
int azb_check_memory(const azb_net_desc* desc, int inference_batch, int hubs, int slots_per_hub, int device,
                     int precision, char* err, size_t err_cap);

/* The engine's weight bytes on a device, and the reference's one combined
 * check (src/cuda/cuda_runner.cu:203-223): 0 when `bytes` fit in the
 * device's free memory less a 512 MB margin (or the test hook's limit),
 * else -1 and "cuda: inference needs N MB ...; lower inference_batch". */
size_t azb_weights_bytes(const azb_net_desc* desc, int precision);
int azb_check_bytes(int device, double bytes, int inference_batch, int hubs, char* err, size_t err_cap);

/* ------------------------------------------------ test hooks (cuda_probe) */
/* include/azgo/cuda.hpp:138-155 */
void azb_probe_set_hub_chaos_seed(uint64_t seed);
uint64_t azb_probe_hub_chaos_seed(void);
void azb_probe_fail_passes_after(int n);
void azb_probe_set_memory_limit(size_t bytes);
long long azb_probe_passes_completed(void);
void azb_probe_set_copy_out_delay(int microseconds);
/* Which tensor-core conv form passes use: 0 the default (CTA pairs, i.e.
 * 2-CTA clusters with M = 256 per MMA via tcgen05 cta_group::2, for layers
 * of 256 output channels; two 128-row tiles per CTA sharing each weight
 * tile for layers of 128 or fewer with at least two tiles per SM; one tile
 * per CTA otherwise), 1 always one tile per CTA, 2 always CTA pairs, 3 two
 * tiles per CTA where N <= 128. For tests and measurements. */
void azb_probe_set_conv_path(int path);
/* tf32x3 at 128 output channels or fewer accumulates each tile in segments
 * (three taps at 128 channels, nine at 64 or fewer; a one-tap pass: one
 * chunk), summed in fp32 round-to-nearest by the epilogue (tcgen05's fp32
 * accumulation rounds toward zero at every MMA). -1 the default, 0 one
 * accumulator run per tile (for measurements). */
void azb_probe_set_conv_segment(int steps);
/* Boards whose frame rows fit one 128-row tile (n <= 10) with 32 or 64
 * output channels run the residual tower as one launch, each CTA keeping a
 * group of boards' activations in shared memory through every block (the
 * same arithmetic as the per-layer kernels, bit for bit). -1 the default
 * (the split mode at 64 channels with two groups of boards per CTA where that
 * saves a round of CTAs), 0 the per-layer kernels always, 1 the fused launch
 * with one group per CTA, 2 with two wherever the shape allows. For tests and
 * measurements. */
void azb_probe_set_tower_fused(int mode);
/* Towers that do not fuse run every tower conv in one persistent launch:
 * CTAs take (layer, tile group) items in order, each waiting for the
 * previous layer's groups its halo reads (bounded waits; the same
 * arithmetic as the per-layer kernels, bit for bit). -1 the default (128
 * or fewer channels, every precision), 0 per layer always, 1 at any width
 * (bf16 and tf32; TF32X3 only up to 128 channels, in its default
 * accumulation segments). For tests and measurements. */
void azb_probe_set_tower_persistent(int mode);
/* Nonzero: the persistent tower waits for one counter step more than its
 * epilogue warps add, so its first wait for a previous layer runs out (after
 * its bound of half a second, before the pipeline waits it starves) and the
 * pass fails with "cuda: the persistent tower waited too long for the
 * previous layer"; the next pass runs normally. For the failure-detection
 * test. */
void azb_probe_starve_tower(int on);
/* cuda_probe::binaryVersion / deviceArchitecture / fill (include/azgo/cuda.hpp:93-103). */
int azb_probe_binary_version(int device);
int azb_probe_device_architecture(int device);
int azb_probe_fill(int device, float* data, size_t n, float value, size_t tail, char* err, size_t err_cap);
/* cuda_probe::tanhInPlace (include/azgo/cuda.hpp:112): data[0..n) = tanh(data) on the device, with the
 * tanhf the head kernels use for the value and ownership outputs. */
int azb_probe_tanh(int device, float* data, size_t n, char* err, size_t err_cap);
/* A kernel that waits on a barrier nothing arrives on: returns the kernel's
 * error word (5: its wait ran out after limit_ns) with the context intact. */
int azb_probe_bounded_wait(int device, unsigned long long limit_ns, char* err, size_t err_cap);
/* The tensor-core path alone on one CTA: D[128][n_out] = A[shift .. shift+127]
 * . W^T over k_chunks 128-byte chunks, A [halo_rows][chunk*k_chunks] and W
 * [n_out][9*chunk*k_chunks] given as host fp32 (converted per precision);
 * D written to host fp32 [128][n_out]. */
int azb_probe_umma(int device, int precision, int n_out, int halo_rows, int shift_rows, int k_chunks,
                   int base_offset_mode, const float* a, const float* w, float* d, char* err, size_t err_cap);

#ifdef __cplusplus
}
#endif
#endif
