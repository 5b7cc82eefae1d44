// The stem convolution, the fused heads, and the small kernels the runner's
// checks and test hooks use.
#include <algorithm>
#include <atomic>

#include "head_rows.cuh"
#include "kernels.hpp"
#include "sm100.cuh"

namespace azb {

namespace {

// Blocks for a grid-stride loop over `count` items: at most 8 waves of the
// GPU's SMs, so the grid depends only on the count.
unsigned blocks_for(size_t count, int threads) {
    const size_t b = (count + threads - 1) / threads;
    return static_cast<unsigned>(std::max<size_t>(1, std::min<size_t>(b, 148 * 8)));
}

// ---------------------------------------------------------------- the stem

// The stem's input as a packed GEMM operand: for every board point, the
// 9*P values its 3x3 window reads (tap-major: column t*P + p, t = ky*3 + kx,
// 0 off the board), in the point's frame row. The stem then runs on the
// tensor cores as a one-tap GEMM with K = 9*P (rounded up to whole 128-byte
// chunks), instead of a 3x3 convolution over P channels padded to a chunk.
// One CTA per board (grid-stride): the board's P planes are staged in shared
// memory, then consecutive threads write consecutive 16-byte pieces of the
// frame rows (whole rows, the zero columns past 9*P included), so the stores
// are coalesced. Frame padding rows are never written (zero since the
// buffer was allocated).
template <int kMode>
__global__ void __launch_bounds__(256) stem_pack_kernel(const StemArgs a) {
    extern __shared__ float planes[];   // [P][A], then the column table
    constexpr int W = kMode == kBF16 ? 8 : 4;   // values per 16-byte piece
    const int A = a.n * a.n, K = 9 * a.P, pieces = a.ld / W;
    // Column k of a row reads plane k % P at tap t = k / P: table[e][j] for
    // k = j*W + e holds (plane * A) << 4 | (dy+1) << 2 | (dx+1), or -1 past
    // K (laid out by e so that the lanes, consecutive j, read consecutive
    // words).
    int* table = reinterpret_cast<int*>(planes + size_t(a.P) * A);
    grid_dependency_wait();
    grid_launch_dependents();
    if (a.flags)   // the persistent tower's counters start each pass at zero
        for (int i = int(blockIdx.x * blockDim.x + threadIdx.x); i < a.nflags; i += int(gridDim.x * blockDim.x))
            a.flags[i] = 0u;
    for (int i = threadIdx.x; i < W * pieces; i += blockDim.x) {
        const int e = i / pieces, j = i % pieces, k = j * W + e;
        int code = -1;
        if (k < K) {
            const int t = k / a.P, pl = k % a.P;
            code = ((pl * A) << 4) | ((t / 3) << 2) | (t % 3);
        }
        table[i] = code;
    }
    for (int b = blockIdx.x; b < a.B; b += gridDim.x) {
        __syncthreads();
        for (int i = threadIdx.x; i < a.P * A; i += blockDim.x) planes[i] = __ldg(a.in + size_t(b) * a.P * A + i);
        __syncthreads();
        // Thread t keeps piece j = t % pieces of every row it writes (its W
        // column codes in registers) and steps through the points t / pieces,
        // + per_step, ...: no division per piece. Consecutive threads write
        // consecutive pieces of a row, then the next point's row.
        const int per_step = int(blockDim.x) / pieces;
        if (int(threadIdx.x) >= per_step * pieces) continue;
        const int j = int(threadIdx.x) % pieces, first = int(threadIdx.x) / pieces;
        int codes[W];
#pragma unroll
        for (int e = 0; e < W; ++e) codes[e] = table[e * pieces + j];
        int py = first / a.n, px = first - py * a.n;
        for (int pt = first; pt < A; pt += per_step) {
            float v[W];
#pragma unroll
            for (int e = 0; e < W; ++e) {
                const int code = codes[e];
                v[e] = 0.0f;
                if (code >= 0) {
                    const int y = py + ((code >> 2) & 3) - 1, x = px + (code & 3) - 1;
                    if (y >= 0 && y < a.n && x >= 0 && x < a.n) v[e] = planes[(code >> 4) + y * a.n + x];
                }
            }
            const size_t off = (size_t(b) * a.S + size_t(py + 1) * (a.n + 1) + px) * a.ld + size_t(j) * W;
            if (kMode == kBF16) {
                uint4 w4;
                __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&w4);
#pragma unroll
                for (int e = 0; e < 4; ++e) h2[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
                *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + off) = w4;
            } else if (kMode == kTF32x3) {
                float4 h, l;
                h.x = to_tf32(v[0]); l.x = __fsub_rn(v[0], h.x);
                h.y = to_tf32(v[1]); l.y = __fsub_rn(v[1], h.y);
                h.z = to_tf32(v[2]); l.z = __fsub_rn(v[2], h.z);
                h.w = to_tf32(v[3]); l.w = __fsub_rn(v[3], h.w);
                *reinterpret_cast<float4*>(static_cast<float*>(a.out) + off) = h;
                *reinterpret_cast<float4*>(static_cast<float*>(a.out_lo) + off) = l;
            } else {
                *reinterpret_cast<float4*>(static_cast<float*>(a.out) + off) = make_float4(v[0], v[1], v[2], v[3]);
            }
            px += per_step;
            while (px >= a.n) {
                px -= a.n;
                ++py;
            }
        }
    }
}

// ------------------------------------------------------------- the encoder

// One thread per (position, point q): q's value in every plane. The
// symmetry sends point p to transformPoint(sym, p), so q reads point
// p = transformPoint(inverse(sym), q): mirror left-right (sym & 4) first,
// then (sym & 3) clockwise quarter turns (src/symmetry.cpp:6-19); mirrored
// symmetries are their own inverse, k turns are undone by 4 - k.
__device__ __forceinline__ int transform_point(int sym, int point, int n) {
    int row = point / n, col = point % n;
    if (sym & 4) col = n - 1 - col;
    for (int t = 0; t < (sym & 3); ++t) {
        const int r = col, c = n - 1 - row;
        row = r;
        col = c;
    }
    return row * n + col;
}

__global__ void __launch_bounds__(256) encode_planes_kernel(const EncodeArgs a) {
    grid_dependency_wait();
    grid_launch_dependents();
    const int A = a.n * a.n, P = 2 * a.H + 2;
    const size_t rec = stones_record_bytes(a.H, a.n);
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < size_t(a.B) * A;
         i += size_t(gridDim.x) * blockDim.x) {
        const int b = int(i / A), q = int(i % A);
        const uint8_t* r = a.records + size_t(b) * rec;
        const uint8_t* head = r + size_t(a.H) * A;
        const int to_move = head[0], avail = min(int(head[1]), a.H), sym = head[2] & 7;
        const int inv = (sym & 4) ? sym : (4 - sym) & 3;
        const int p = transform_point(inv, q, a.n);
        const int opp = to_move == 1 ? 2 : 1;
        float* out = a.out + size_t(b) * P * A + q;
        for (int k = 0; k < a.H; ++k) {
            const int stone = k < avail ? r[size_t(k) * A + p] : 0;
            out[size_t(2 * k) * A] = stone == to_move ? 1.0f : 0.0f;
            out[size_t(2 * k + 1) * A] = stone == opp ? 1.0f : 0.0f;
        }
        out[size_t(2 * a.H) * A] = to_move == 1 ? 1.0f : 0.0f;
        out[size_t(2 * a.H + 1) * A] = to_move == 1 ? 0.0f : 1.0f;
    }
}

// --------------------------------------------------------------- the heads
//
// Two launches (the small-board fused tower runs all of it in its own):
//  1. head_conv_kernel streams the trunk once through shared memory
//     (bulk copies; HBM-bound): the policy (2),
//     value (1) and ownership (1) 1x1 convolutions of every board point,
//     their batch norms and ReLU (ownership: tanh, straight to its output);
//     features land in a small [B][3A] buffer, the policy part in the
//     reference's flatten order c*A + p (src/network.cpp:278-285).
//  2. head_tail_kernel: the policy FC (2A -> A+1, + bias) and value FC1
//     (A -> V, + bias, ReLU) for tiles of 16 boards x 32 outputs, each FC
//     weight read once per tile, the tile's inputs in shared memory; the
//     last CTA of a board tile then runs the value FC2 and tanh, and the
//     softmax over the A+1 logits, a warp per board.
// Every output is a fixed-order sum over its own board's data: the results
// do not depend on the batch or on where a board sits in it.

constexpr int kHeadThreads = 256;
constexpr int kFcBoards = 16;    // boards per FC tile: each weight is read once per 16 boards

// The trunk streamed once through shared memory. A copy thread (warp 8)
// stages `kbr` board rows at a time into a ring of `stages` buffers: the n
// real points of a board row are n consecutive frame rows, one bulk copy
// each, so padding rows are never read. 16 reader warps take the staged rows
// four "slots" at a time: kLpr lanes share one row (kLpr x kNch 16-byte
// pieces, lane l reading pieces l, l + kLpr, ...: consecutive lanes,
// consecutive pieces), each lane summing its channels into 4 slots x 4
// heads = 16 partial sums with the 1x1 weights of its channels held in
// registers. A reduce-scatter over the kLpr lanes (at the step over lane
// bit b a lane keeps the half of its sums that bit selects and adds its
// partner's copy; once one sum is left, a butterfly) leaves each lane its
// finished sums, which it applies the batch norm to and stores. Every sum is the same tree of
// additions whatever its slot: outputs do not depend on the batch.
// Persistent CTAs, one per SM; every wait is bounded.
constexpr int kHcReaders = 16;
constexpr int kHcThreads = 32 * (kHcReaders + 1);


template <int kMode, int kLpr, int kNch>
__global__ void __launch_bounds__(kHcThreads, 1)
    head_conv_kernel(const HeadArgs a, int stages, int kbr, uint32_t row_bytes) {
    extern __shared__ uint8_t hc_raw[];
    constexpr uint32_t kPlanes = kMode == kTF32x3 ? 2u : 1u;
    const int n = a.n, board_rows = a.B * n;
    const int nblk = (board_rows + kbr - 1) / kbr;
    const uint32_t br_bytes = uint32_t(n) * row_bytes;              // one board row, one plane
    const uint32_t plane_bytes = uint32_t(kbr) * br_bytes;          // one stage, one plane
    uint8_t* buf = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(hc_raw) + 127) & ~uintptr_t(127));
    uint64_t* full = reinterpret_cast<uint64_t*>(buf + size_t(stages) * kPlanes * plane_bytes);
    uint64_t* empty = full + stages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < stages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kHcReaders);
        }
        fence_barrier_init();
    }
    __syncthreads();
    grid_dependency_wait();
    grid_launch_dependents();

    if (warp == kHcReaders) {
        // ------------------------------------------------------- copy thread
        if (lane == 0) {
            Ring r;
            uint32_t issued = 0;
            const uint8_t* hi = static_cast<const uint8_t*>(a.trunk);
            const uint8_t* lo = static_cast<const uint8_t*>(a.trunk_lo);
            for (int blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
                if (!mbar_wait(&empty[r.idx], r.phase ^ 1u, a.err, kErrWaitHeadLoad)) break;
                const int first = blk * kbr, cnt = min(kbr, board_rows - first);
                mbar_arrive_expect_tx(&full[r.idx], kPlanes * uint32_t(cnt) * br_bytes);
                uint8_t* dst = buf + size_t(r.idx) * kPlanes * plane_bytes;
                for (int i = 0; i < cnt; ++i) {
                    const int b = (first + i) / n, y = (first + i) % n;
                    const size_t row0 = size_t(b) * a.S + size_t(y + 1) * (n + 1);
                    bulk_load(dst + i * br_bytes, hi + row0 * row_bytes, br_bytes, &full[r.idx]);
                    if (kMode == kTF32x3)
                        bulk_load(dst + plane_bytes + i * br_bytes, lo + row0 * row_bytes, br_bytes, &full[r.idx]);
                }
                r.next(uint32_t(stages));
                ++issued;
            }
            // Every copy has landed before the CTA may exit.
            for (uint32_t st = 0; st < uint32_t(stages) && st < issued; ++st) {
                const uint32_t uses = (issued - st + stages - 1) / stages;
                mbar_wait(&full[st], (uses - 1) & 1, a.err, kErrWaitDrain);
            }
        }
        return;
    }

    // ----------------------------------------------------------- readers
    HeadLane<kMode, kLpr, kNch> hl;
    hl.load(a, lane);
    const float inv_n = 1.0f / float(n);
    Ring r;
    for (int blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
        if (!mbar_wait(&full[r.idx], r.phase, a.err, kErrWaitHeadData)) break;
        const uint8_t* stage = buf + size_t(r.idx) * kPlanes * plane_bytes;
        const int first = blk * kbr, rows = min(kbr, board_rows - first) * n;
        // Staged row `row` (the points of board rows first.., n per board row).
        auto piece = [&](int row, int j) {
            TrunkPiece<kMode> pc;
            const uint32_t off = uint32_t(row) * row_bytes + uint32_t(j) * 16u;
            pc.hi = *reinterpret_cast<const uint4*>(stage + off);
            if (kMode == kTF32x3) pc.lo = *reinterpret_cast<const uint4*>(stage + plane_bytes + off);
            return pc;
        };
        auto where = [&](int row, int* b, int* p) {
            const int rq = div_small(row, n, inv_n), br = first + rq, x = row - rq * n;
            *b = div_small(br, n, inv_n);
            *p = (br - *b * n) * n + x;
        };
        for (int base = warp * HeadLane<kMode, kLpr, kNch>::kStepRows; base < rows;
             base += kHcReaders * HeadLane<kMode, kLpr, kNch>::kStepRows)
            hl.step(a, base, rows, piece, where, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[r.idx]);
        r.next(uint32_t(stages));
    }
}

// The heads after their 1x1 convolutions, in one launch: a CTA takes a tile
// of kFcBoards (16) boards x 32 outputs of the policy FC (output tiles 0 ..
// ceil((A+1)/32) - 1 of gridDim.y) or of the value FC1 (the rest), with the
// tile's inputs, [16][n rounded up to 4], in shared memory; each warp takes
// kFcOuts (4) outputs for the 16 boards (head_fc_quads: every weight read
// once per 16 boards). The last CTA of a board tile to finish (a counter per
// board tile, zeroed by the pass's stem operand kernel) then runs the value
// FC2 + tanh and, when asked for, the softmax over A+1 for the tile's boards,
// a warp per board, reading the other CTAs' hidden layers and logits through
// L2. One launch instead of an FC launch and a finishing launch.
constexpr int kFcOuts = 4;
__global__ void __launch_bounds__(kHeadThreads) head_tail_kernel(const HeadArgs a) {
    extern __shared__ float4 xs[];
    __shared__ unsigned last_cta;
    grid_dependency_wait();
    grid_launch_dependents();
    const int A = a.A, L = A + 1, V = a.V;
    constexpr int kWarps = kHeadThreads / 32, outs_per_cta = kWarps * kFcOuts;
    const int pol_tiles = (L + outs_per_cta - 1) / outs_per_cta;
    const bool policy = int(blockIdx.y) < pol_tiles;
    const int n_in = policy ? 2 * A : A, n4 = (n_in + 3) / 4;
    const int foff = policy ? 0 : a.feat_val;   // multiples of 4 floats, as is feat_ld
    const int b0 = blockIdx.x * kFcBoards, G = min(kFcBoards, a.B - b0);
    const float4* feat4 = reinterpret_cast<const float4*>(a.feat);
    for (int idx = threadIdx.x; idx < kFcBoards * n4; idx += kHeadThreads) {
        const int g = idx / n4, j = idx - g * n4;
        xs[idx] = g < G ? feat4[(size_t(b0 + g) * a.feat_ld + foff) / 4 + j] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // This CTA's quads: the policy quads of its policy tile, or the value
    // quads of its value tile (quads are numbered policy first).
    const int pol_quads = (L + kFcOuts - 1) / kFcOuts;
    const int tile_quad0 = policy ? int(blockIdx.y) * outs_per_cta / kFcOuts
                                  : pol_quads + (int(blockIdx.y) - pol_tiles) * outs_per_cta / kFcOuts;
    const int tile_quads = policy ? min(kWarps, pol_quads - tile_quad0)
                                  : min(kWarps, pol_quads + (V + kFcOuts - 1) / kFcOuts - tile_quad0);
    if (warp < tile_quads) {
        auto x = [&](int g, int j) { return xs[g * n4 + j]; };
        head_fc_quads<kFcOuts, kFcBoards>(a, b0, G, tile_quad0 + warp, 1 << 30, x, x,
                                          [&](int g) { return a.hid + size_t(b0 + g) * V; }, lane);
    }
    // The board tile's last CTA finishes it.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_cta = atomicAdd(a.tail_count + blockIdx.x, 1u) + 1u == gridDim.y;
    __syncthreads();
    if (!last_cta) return;
    __threadfence();
    for (int g = warp; g < G; g += kWarps) head_finish_board(a, b0 + g, a.hid + size_t(b0 + g) * V, lane);
}

// ------------------------------------------------------------ small kernels

__global__ void fill_kernel(float* data, size_t n, float value) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
        data[i] = value;
}

__global__ void tanh_kernel(float* data, size_t n) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
        data[i] = tanhf(data[i]);
}

// Holds the GPU for `ns` nanoseconds of %globaltimer (a test hook; bounded).
__global__ void spin_kernel(unsigned long long ns) {
    const uint64_t start = global_timer();
    while (global_timer() - start < ns) {
    }
}

// Waits on a barrier that nothing arrives on; the wait's own limit ends it.
__global__ void bounded_wait_probe(int* err, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint64_t start = global_timer();
        bool done = false;
        while (!done && global_timer() - start < limit_ns) done = mbar_try_wait(&bar, 0);
        if (!done) atomicCAS(err, 0, kErrProbeTimeout);
    }
}

} // namespace

cudaError_t launch_stem_pack(const StemArgs& a, int precision, cudaStream_t s) {
    if (a.B <= 0) return cudaSuccess;
    const int W = precision == kBF16 ? 8 : 4;
    if (a.ld % W != 0) return cudaErrorInvalidValue;
    const size_t smem = size_t(a.P) * a.n * a.n * sizeof(float) + size_t(a.ld) * sizeof(int);
    const unsigned grid = static_cast<unsigned>(std::min(a.B, 148 * 8));
    switch (precision) {
        case kTF32: return launch_pdl(stem_pack_kernel<kTF32>, dim3(grid), dim3(256), smem, s, a);
        case kTF32x3: return launch_pdl(stem_pack_kernel<kTF32x3>, dim3(grid), dim3(256), smem, s, a);
        case kBF16: return launch_pdl(stem_pack_kernel<kBF16>, dim3(grid), dim3(256), smem, s, a);
        default: return cudaErrorInvalidValue;
    }
}

namespace {

// One persistent CTA per SM (fewer for small batches). A stage holds as
// many board rows as about three reader steps cover (16 warps x 4 slots x
// rows per slot each), capped so that at least two stages fit in 200 KB;
// as many stages as fit, at most 8 (C4 bf16: 2 stages of 10 board rows).
template <int kMode, int kLpr, int kNch>
cudaError_t launch_head_conv_as(const HeadArgs& a, int sms, cudaStream_t s) {
    const uint32_t row_bytes = uint32_t(a.ld) * (kMode == kBF16 ? 2u : 4u);
    const size_t planes = kMode == kTF32x3 ? 2 : 1, br_bytes = size_t(a.n) * row_bytes * planes;
    constexpr size_t kBudget = 200u << 10;
    const int step_rows = kHcReaders * kHcSlots * (32 / kLpr);
    int kbr = std::max(1, (step_rows * 3) / a.n);   // about three reader steps per stage, if two stages fit
    kbr = int(std::max<size_t>(1, std::min<size_t>(size_t(kbr), kBudget / 2 / br_bytes)));
    kbr = std::min(kbr, a.B * a.n);
    const size_t stage = size_t(kbr) * br_bytes;
    const int stages = int(std::max<size_t>(2, std::min<size_t>(8, kBudget / stage)));
    const size_t smem = 128 + size_t(stages) * stage + size_t(stages) * 16;
    if (const cudaError_t e = open_smem<head_conv_kernel<kMode, kLpr, kNch>>(smem); e != cudaSuccess) return e;
    const int nblk = (a.B * a.n + kbr - 1) / kbr;
    const unsigned grid = static_cast<unsigned>(std::max(1, std::min(nblk, sms)));
    return launch_pdl(head_conv_kernel<kMode, kLpr, kNch>, dim3(grid), dim3(kHcThreads), smem, s, a, stages, kbr,
                      row_bytes);
}

template <int kMode>
cudaError_t launch_head_conv_mode(const HeadArgs& a, int sms, cudaStream_t s) {
    switch (a.ld / TrunkPiece<kMode>::kWidth) {   // 16-byte pieces per trunk row
        case 8: return launch_head_conv_as<kMode, 8, 1>(a, sms, s);
        case 16: return launch_head_conv_as<kMode, 16, 1>(a, sms, s);
        case 32: return launch_head_conv_as<kMode, 32, 1>(a, sms, s);
        case 64: return launch_head_conv_as<kMode, 32, 2>(a, sms, s);
        default: return cudaErrorInvalidValue;
    }
}

} // namespace

cudaError_t launch_encode_planes(const EncodeArgs& a, cudaStream_t s) {
    if (a.B <= 0) return cudaSuccess;
    return launch_pdl(encode_planes_kernel, dim3(blocks_for(size_t(a.B) * a.n * a.n, 256)), dim3(256), 0, s, a);
}

cudaError_t launch_head_conv(const HeadArgs& a, int precision, int sms, cudaStream_t s) {
    if (a.B <= 0) return cudaSuccess;
    if ((a.ld * (precision == kBF16 ? 2 : 4)) % 16 != 0) return cudaErrorInvalidValue;
    switch (precision) {
        case kTF32: return launch_head_conv_mode<kTF32>(a, sms, s);
        case kTF32x3: return launch_head_conv_mode<kTF32x3>(a, sms, s);
        case kBF16: return launch_head_conv_mode<kBF16>(a, sms, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_head_tail(const HeadArgs& a, cudaStream_t s) {
    if (a.B <= 0) return cudaSuccess;
    if (a.tail_count == nullptr) return cudaErrorInvalidValue;
    const int L = a.A + 1, outs = (kHeadThreads / 32) * kFcOuts;
    const dim3 grid((a.B + kFcBoards - 1) / kFcBoards, (L + outs - 1) / outs + (a.V + outs - 1) / outs);
    const size_t smem = size_t((2 * a.A + 3) / 4) * 4 * kFcBoards * sizeof(float);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(head_tail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(head_tail_kernel, grid, dim3(kHeadThreads), smem, s, a);
}

cudaError_t launch_fill(float* data, size_t n, float value, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    fill_kernel<<<blocks_for(n, 256), 256, 0, s>>>(data, n, value);
    return cudaGetLastError();
}

cudaError_t launch_tanh(float* data, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    tanh_kernel<<<blocks_for(n, 256), 256, 0, s>>>(data, n);
    return cudaGetLastError();
}

cudaError_t fill_attributes(cudaFuncAttributes* attr) { return cudaFuncGetAttributes(attr, fill_kernel); }

cudaError_t launch_spin(unsigned long long ns, cudaStream_t s) {
    if (ns == 0) return cudaSuccess;
    spin_kernel<<<1, 1, 0, s>>>(ns);
    return cudaGetLastError();
}

namespace {
__global__ void admission_probe_kernel(uint32_t* data, int n) {
    const int i = int(blockIdx.x * blockDim.x + threadIdx.x);
    if (i < n) data[i] = admission_probe_value(data[i], i);
}
}  // namespace

cudaError_t launch_admission_probe(uint32_t* data, int n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    admission_probe_kernel<<<(n + 127) / 128, 128, 0, s>>>(data, n);
    return cudaGetLastError();
}

cudaError_t launch_bounded_wait_probe(int* err, unsigned long long limit_ns, cudaStream_t s) {
    bounded_wait_probe<<<1, 32, 0, s>>>(err, limit_ns);
    return cudaGetLastError();
}

} // namespace azb
