// The engine's kernels as the host code launches them.
//
// Activation layout in HBM ("board frames"): NHWC rows of `ld` channels,
// one row per pixel of a padded board. Board b occupies frame rows
// [b*S, (b+1)*S) with S = (n+1)^2: frame row 0 is all padding, then n rows
// of n+1 pixels whose last pixel is padding. Point (y, x) of board b is row
//     q = b*S + (y+1)*(n+1) + x,
// so the 3x3 neighbour (y+dy, x+dx) is row q + dy*(n+1) + dx for every point
// of the board, and a neighbour off the board is always a padding row. The
// padding rows are zeroed once when a buffer is allocated and no kernel ever
// writes them, so a 3x3 convolution reads its 'same' padding as plain rows.
#pragma once
#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace azb {

// Launches `kernel` on `s` with programmatic stream serialization: it may
// begin while the previous kernel on the stream finishes, and waits for it
// with grid_dependency_wait (sm100.cuh) before using that kernel's output.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Lets `Kernel` use `bytes` of dynamic shared memory on the current device.
// The attribute belongs to the device, so each device is opened once (and
// again for a larger size): one process may launch on several GPUs.
constexpr int kMaxDevices = 64;
template <auto Kernel>
cudaError_t open_smem(size_t bytes) {
    static std::atomic<size_t> opened[kMaxDevices];
    int dev = 0;
    if (const cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return e;
    if (dev >= 0 && dev < kMaxDevices && bytes <= opened[dev].load()) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
    if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
        size_t seen = opened[dev].load();
        while (seen < bytes && !opened[dev].compare_exchange_weak(seen, bytes)) {
        }
    }
    return e;
}

// Error codes a kernel leaves in its error word (0: none).
enum KernelError : int {
    kErrNone = 0,
    kErrWaitProducer = 1,   // the TMA warp waited too long for a free stage
    kErrWaitMma = 2,        // the MMA warp waited too long for data or a free accumulator
    kErrWaitEpilogue = 3,   // the epilogue waited too long for an accumulator
    kErrWaitDrain = 4,      // draining in-flight copies after an error timed out
    kErrProbeTimeout = 5,   // the bounded-wait probe's wait ran out (expected by its test)
    kErrWaitHeadLoad = 6,   // the head kernel's copy thread waited too long for a free stage
    kErrWaitHeadData = 7,   // the head kernel's readers waited too long for a board row
    kErrWaitLayer = 8,      // the persistent tower waited too long for the previous layer's tile groups
};


// The arithmetic a pass runs in (also the operand storage of the trunk).
enum Precision : int {
    kTF32 = 0,     // fp32 activations, tf32 tensor-core products, fp32 accumulate
    kTF32x3 = 1,   // split tf32 (a_hi*b_hi + a_hi*b_lo + a_lo*b_hi): fp32-class accuracy
    kBF16 = 2,     // bf16 activations and weights, fp32 accumulate
};

inline int elem_bytes(int precision) { return precision == kBF16 ? 2 : 4; }
// Channels in one 128-byte K chunk of the implicit GEMM.
inline int chunk_channels(int precision) { return 128 / elem_bytes(precision); }

struct Frame {
    int n;      // board size
    int S;      // rows per board, (n+1)^2
    int halo;   // rows a 128-row tile reads: 128 + 2(n+2)
    explicit Frame(int board) : n(board), S((board + 1) * (board + 1)), halo(128 + 2 * (board + 2)) {}
    size_t row(int b, int y, int x) const { return size_t(b) * S + size_t(y + 1) * (n + 1) + x; }
};

struct FusedLayer;

// One fused 3x3 convolution + folded batch norm (+ skip) + ReLU.
struct ConvArgs {
    int n, S;          // board, frame rows per board
    int rows;          // B * S: frame rows of this pass
    int ntiles;        // ceil(rows / 128)
    int nchunks;       // input channels / chunk_channels
    int taps;          // 9: the 3x3 views of the halo; 1: the centre view only (a plain GEMM over K)
    int ld;            // channels per stored pixel row (input, output and skip)
    int halo_rows;     // 128 + 2(n+2)
    int a_bytes;       // one halo buffer, rounded up to 1024
    int sa, sb;        // pipeline depths: halo buffers, weight buffers
    int seg;           // stacked split mode: 0 one accumulator run per tile, else segments (3 or 9 taps by width)
    void* out;         // [rows][ld] bf16 or f32 (split: the tf32 high part)
    void* out_lo;      // split: f32 low part
    const void* skip;  // null, or the residual input (same layout as out)
    const void* skip_lo;
    const float* scale;   // [N] folded batch norm (0 for padded channels)
    const float* shift;   // [N]
    int* err;          // kernel error word (KernelError)
};

// The persistent tower's own parameters (a separate kernel parameter, so
// the per-layer kernels' ConvArgs stay as they are): the stem's packed
// operand and the three frame buffers as it addresses them, the layer
// table, and per (layer, tile group) the count of epilogue warps that have
// stored their part of it, zeroed by the pass's stem operand kernel.
struct TowerArgs {
    CUtensorMap stem, stem_lo;       // the stem's packed operand in halo boxes
    CUtensorMap in[3], in_lo[3];     // halo boxes {chunk, halo_rows} (in_lo: the split mode's low planes)
    CUtensorMap out[3], out_lo[3];   // the epilogue's {32, 32} boxes
    const void* trunk[3];            // the frames (the split mode reads its residual directly)
    const void* trunk_lo[3];
    const FusedLayer* tower;         // the layers' weight maps and batch norms (tower convs, then the stem)
    int layers;
    unsigned* flags;
    unsigned flag_extra;   // 0; the failure-detection test's 1 makes every wait for a previous layer run out
    // 1: layer 0 is the stem, one tap over its packed operand of
    // stem_nchunks chunks (its weights the table's last entry), writing
    // buffer 0; tower conv l is then layer l + 1.
    int stem_first;
    int stem_nchunks;
};

struct ConvMaps {
    CUtensorMap a, a_lo;             // input activations: box {chunk, halo_rows}
    CUtensorMap w, w_lo;             // weights [N][9*Cin]: box {chunk, N}
    CUtensorMap w_pair, w_lo_pair;   // the same weights in boxes of {chunk, N/2}: one half per CTA of a pair
    CUtensorMap out, skip;           // bf16/tf32: the output and residual frames in boxes of {32, 32} (epilogue)
    CUtensorMap out_lo;              // split mode: the output's low plane in boxes of {32, 32} (out: the high plane)
};

// Shared memory a conv launch needs, and its pipeline depths (pair: the
// CTA-pair form, which stages half of each weight tile per CTA).
size_t conv_smem_bytes(int n_out, int precision, int halo_rows, int* sa, int* sb, bool pair = false, int tiles = 1);

// Enqueues the conv on `s` in one of three forms: 2-CTA pairs (M = 256 per
// MMA, tcgen05 cta_group::2) for 256 output channels; for 128 or fewer, two
// tiles per CTA sharing each weight tile when there are at least two tiles
// per SM, else one tile per CTA; unless the test hook selects a form. The
// pipeline depths in `a` are chosen here.
cudaError_t launch_conv(const ConvMaps& maps, const ConvArgs& a, int n_out, int precision, int sms, cudaStream_t s);
// Test hook: 0 by width, 1 one tile per CTA, 2 CTA pairs, 3 two tiles per CTA (N <= 128).
void set_conv_path(int path);
// Test hook for the stacked split mode's accumulation: -1 the default
// (segments of three taps at 128 channels, nine at 64 or fewer), 0 one
// accumulator run per tile.
void set_conv_segment(int steps);

// The persistent tower: every tower conv (a.layers of them, a.tower's
// entries) in one launch of at most one CTA per SM (bf16 and tf32 at any
// width, the split mode at 128 channels or fewer). CTAs take (layer, tile
// group) items in layer-major order from a counter; an item's halo loads
// wait for the three groups of the previous layer whose rows they read.
// Tower conv l reads frame buffer l mod 3 and writes (l+1) mod 3; a block's
// second conv adds (l-1) mod 3, the block's input.
// Returns cudaErrorNotSupported where it does not apply (the caller then
// launches per layer).
cudaError_t launch_tower_persistent(const TowerArgs& t, const ConvArgs& a, int n_out, int precision, int sms,
                                    cudaStream_t s);
// Whether the persistent tower runs for n_out channels in `precision` (and
// the test hook's choice: -1 the default, 0 per layer, 1 persistent where
// it applies). The split mode needs its default accumulation segments.
bool tower_persistent(int n_out, int precision);
void set_tower_persistent(int mode);
// Test hook: nonzero makes the persistent tower wait for one counter step
// more than its epilogue warps add, so its first wait for a previous layer
// runs out (bounded) and the pass reports kErrWaitLayer.
void set_tower_starve(int on);
bool tower_starve();

// The stem's packed operand: the [B][P][A] fp32 input unfolded into frame
// rows of K = 9*P values (column t*P + p), ld elements apart. The stem conv
// itself then runs as a one-tap GEMM on the tensor-core kernel.
struct StemArgs {
    const float* in;    // [B][P][A]
    int B, P, n, S, ld;
    void* out; void* out_lo;
    unsigned* flags;    // the pass's counters (the head tail's, then the persistent tower's), zeroed here
    int nflags;
};
cudaError_t launch_stem_pack(const StemArgs& a, int precision, cudaStream_t s);

// Positions as the reference's encoder takes them (src/encode.cpp:15-43), one
// record of stones_record_bytes(H, n) bytes each: stones[H][n*n] Color bytes
// (0 empty, 1 Black, 2 White; row k is the position k plies ago), then
// toMove (1 Black, 2 White), the number of history positions present
// (0..H), the symmetry (0..7, as transformPoint numbers them), and zero
// padding to a multiple of 4 bytes. The kernel writes the [B][2H+2][n*n]
// fp32 planes encodePlanes writes, into the stage buffer.
__host__ __device__ inline size_t stones_record_bytes(int H, int n) { return (size_t(H) * n * n + 3 + 3) / 4 * 4; }
struct EncodeArgs {
    const uint8_t* records;
    int B, H, n;
    float* out;
};
cudaError_t launch_encode_planes(const EncodeArgs& a, cudaStream_t s);

// The heads: policy 1x1 conv + BN + ReLU + FC, value 1x1 conv + BN + ReLU +
// FC + ReLU + FC + tanh, ownership 1x1 conv + BN + tanh, and the softmax
// over the A+1 moves, in three launches (trunk stream, FC tiles, per-board
// finish) through the small feat/hid scratch buffers.
struct HeadArgs {
    const void* trunk; const void* trunk_lo;
    int ld, n, S, A, F, V, B, ownership;
    const float* pol_w;     // [2][F]
    const float* pol_scale; const float* pol_shift;   // [2]
    const float* fc_w; const float* fc_b;             // [A+1][2A rounded up to 4], [A+1]
    const float* val_w;     // [F]
    const float* val_scale; const float* val_shift;   // [1]
    const float* v1_w; const float* v1_b;             // [V][A rounded up to 4], [V]
    const float* v2_w; const float* v2_b;             // [V], [1]
    const float* own_w; const float* own_scale; const float* own_shift;
    float* logits;      // [B][A+1]
    float* values;      // [B]
    float* ownership_out;   // [B][A] or null
    float* probs;       // [B][A+1] or null
    float* feat;        // scratch [B][feat_ld]: policy features (c*A + p), zeros to a multiple of 4,
                        // then value features from feat_val, zeros to a multiple of 4
    int feat_ld, feat_val;
    float* hid;         // scratch [B][V]: value FC1 after ReLU
    unsigned* tail_count;   // per 16-board tile: the head tail kernel's finished CTAs (zero at a pass's start)
    int* err;           // kernel error word (a bounded wait that ran out)
};
cudaError_t launch_head_conv(const HeadArgs& a, int precision, int sms, cudaStream_t s);   // 1x1 convs -> feat

// The residual tower of a small board in one launch (tower_fused.cu): each
// CTA keeps a group of whole boards' activations in shared memory through
// every block. One conv's weights and folded batch norm, in device memory
// (the kernel reads the tensor maps from there).
struct FusedLayer {
    CUtensorMap w, w_lo;   // weight tiles, box {chunk, n_out} (w_lo: the split mode's low plane)
    const float* scale;    // [n_out]
    const float* shift;
    uint8_t pad[48];
};
static_assert(sizeof(FusedLayer) % 64 == 0, "tensor maps in device memory are 64-byte aligned");

struct FusedArgs {
    int n, S;            // board, frame rows per board
    int boards;          // B
    int group;           // boards per CTA group: group * S <= 128
    int layers;          // 2 * blocks
    int nch;             // 128-byte channel chunks per stored row (cpad / chunk)
    int top;             // the group's first row in an activation buffer: >= n + 2, a multiple of 8
    int act_bytes;       // one (plane, chunk) buffer: 1024-aligned, top + group * S + n + 2 rows of 128 bytes
    int stages;          // weight ring depth (set by the launcher)
    int stem_nch;        // > 0: the stem runs here too, over its packed operand of stem_nch (== nch) chunks
    const FusedLayer* layer;   // [layers]
    const FusedLayer* stem;    // the stem conv (one tap), when stem_nch > 0
    int heads;           // 1: the heads' 1x1 convolutions run here too (into head.feat), and no trunk is stored
    int pairs;           // the split mode at two input chunks, two groups per CTA at once: 0 never, 1 where it pays, 2 always
    HeadArgs head;
    int* err;
};

// The tower's input (the stem's output) and output frames, boxes of
// {chunk, group * S} rows, 128-byte swizzle (lo: the split mode's low planes);
// with the stem in the kernel, its packed operand instead of the input.
struct FusedMaps {
    CUtensorMap in, in_lo, out, out_lo;
    CUtensorMap stem, stem_lo;   // the stem's packed operand in the same boxes (stem_nch > 0)
};

// Shared memory of a fused launch (0 when it does not fit), and its weight
// ring depth.
size_t fused_tower_smem(int n_out, int precision, int nch, int act_bytes, int layers, int* stages, int ctas = 1,
                        int taps_per_stage = 1);
cudaError_t launch_fused_tower(const FusedMaps& maps, const FusedArgs& a, int n_out, int precision, int sms,
                               cudaStream_t s);

// feat -> logits, hid -> values (and probs): the FCs and the value's finish in one launch.
cudaError_t launch_head_tail(const HeadArgs& a, cudaStream_t s);

// Test hooks and context checks.
cudaError_t launch_fill(float* data, size_t n, float value, cudaStream_t s);
cudaError_t launch_tanh(float* data, size_t n, cudaStream_t s);   // data = tanhf(data), as the heads compute it
cudaError_t fill_attributes(cudaFuncAttributes* attr);
cudaError_t launch_spin(unsigned long long ns, cudaStream_t s);
// Device admission's first kernel: data[i] = admission_probe_value(data[i], i).
__host__ __device__ inline uint32_t admission_probe_value(uint32_t x, int i) {
    return (x ^ (x >> 13)) * 5u + uint32_t(i);
}
cudaError_t launch_admission_probe(uint32_t* data, int n, cudaStream_t s);
// A kernel that waits on an mbarrier nothing arrives on, with a limit of
// `limit_ns`; it leaves kErrProbeTimeout in *err and returns.
cudaError_t launch_bounded_wait_probe(int* err, unsigned long long limit_ns, cudaStream_t s);

// A single-CTA check of the tensor-core path: D[128][N] = A[s .. s+127][K] .
// W[N][K]^T for a shifted view s of a staged halo tile (conv's tap views).
cudaError_t launch_umma_probe(const ConvMaps& maps, int n_out, int precision, int halo_rows, int shift_rows,
                              int k_chunks, int base_offset_mode, float* d_out, int* err, cudaStream_t s);

} // namespace azb
