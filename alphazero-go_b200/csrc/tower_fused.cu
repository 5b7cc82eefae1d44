// The residual tower of a small board (n <= 10, a board's frame rows fit one
// 128-row tile) in one launch: each CTA takes a group of whole boards, loads
// their stem operand (or, where it does not fit, the stem's output) into
// shared memory once, runs the stem and every conv of every residual block
// on the resident activations (tcgen05, operands straight from shared
// memory, accumulators in TMEM), then the heads' 1x1 convolutions on the
// resident trunk (or stores the trunk, for the head kernel). A 3x3 conv of a
// board reads only that board's rows and zero padding, so no CTA waits for
// another, and nothing goes back to HBM between layers: at these sizes the
// per-layer launch and round trip, not the MMAs, are what a pass costs.
//
// The arithmetic is the per-layer kernel's (conv_tc.cu) in the same order:
// the same K order per MMA accumulator, the split mode's stacked
// [a_hi.b_hi | a_hi.b_lo + a_lo.b_hi] accumulator per input chunk (its
// segments), the same epilogue roundings; the outputs are the same bits.
//
// Shared memory: activation buffers of [plane][chunk] sub-buffers of frame
// rows x 128 bytes in the 128-byte swizzle, the group's rows from row `top`
// (a multiple of 8, at least n + 2: the zero halo above), then n + 2 zero
// rows; then a ring of weight tiles (one (chunk, tap) tile per stage, both
// planes), as deep as the room left. A 128-row tile's rows past the group
// are outputs nothing reads: their taps read on into the next sub-buffer (or
// the ring), which costs no room.
//
// The split mode keeps one activation buffer: every step writes its output
// over its input in place (its MMAs have all read it), and a block's input,
// which its second conv adds back, waits in TMEM beside the accumulators,
// put there by the epilogue warps while the block's first conv is on the
// tensor core (and read back with the accumulators). The other modes, two
// CTAs to an SM with half the registers, keep two (x: a block's input and
// output, the output written in place over the residual it reads; mid: the
// block's middle activation).
//
// Warps: 0 loads (the group's input, then every layer's weight tiles), 1
// issues the MMAs and owns TMEM, 2-9 the epilogue (warp w reads TMEM lanes
// 32(w % 4)...; the two warps of a lane quarter split the output columns).
// The split mode at 64 channels (two input chunks, each with its own
// stacked accumulator) adds warp 10 as a second MMA issuer: each thread
// issues one chunk's MMAs, in the order one thread would, so every
// accumulator sees the same MMAs in the same order (the same bits). One
// thread cannot issue that mode's 144 MMAs per layer as fast as the tensor
// core runs them; two can. The producer then interleaves the two chunks'
// weight stages, so both issuers find their next stage loaded.
#include <algorithm>
#include <atomic>

#include "head_rows.cuh"
#include "kernels.hpp"
#include "sm100.cuh"

namespace azb {

namespace {

constexpr int kFusedEpiWarps = 8;
constexpr int kFusedFcBoards = 4;   // boards per group at most (5x5: three frames per 128-row tile)

// Threads per CTA: the loader, the MMA issuer and eight epilogue warps; the
// split mode adds the second issuer's warp (warp 10).
template <bool kSplit>
constexpr int kFusedThreads = kSplit ? 352 : 320;

template <int N, bool kBf16, bool kSplit, int kTps = 1>
struct FusedCfg {
    static constexpr int kEsz = kBf16 ? 2 : 4;
    static constexpr int kKc = 128 / kEsz;        // channels per 128-byte chunk
    static constexpr int kSteps = 4;              // MMAs per chunk and tap (32 bytes of K each)
    static constexpr int kOps = kSplit ? 2 : 1;   // operand planes
    static constexpr uint32_t kWTile = uint32_t(N) * 128u;   // one plane of a weight tile
    static constexpr uint32_t kTap = kOps * kWTile;     // one tap's weight tile, both planes
    // A ring stage holds kTps consecutive taps' tiles: one wait and one
    // commit of the MMA thread per kTps taps (each costs the issue loop
    // about as much as an MMA).
    static constexpr uint32_t kStage = uint32_t(kTps) * kTap;
    static_assert(9 % kTps == 0, "taps per stage divide 9");
    // Output columns per epilogue warp: halves of N (N = 32: one warp per
    // lane quarter, the other idle).
    static constexpr int kWarpCols = N >= 64 ? N / 2 : N;
    static_assert(N == 32 || N == 64, "the fused tower runs 32 or 64 output channels");
    static_assert(kWarpCols == 32, "an epilogue warp takes 32 output columns");
};

// The TMEM columns a configuration needs: the split mode one stacked
// accumulator (2N columns) per input chunk, then N columns of the block
// input (fp32, the residual); else one accumulator of N.
__host__ __device__ constexpr uint32_t fused_acc_cols(int n_out, bool split, int nch) {
    return uint32_t(split ? 2 * n_out * nch : n_out);
}
__host__ __device__ constexpr uint32_t fused_tmem_cols(int n_out, bool split, int nch) {
    const int cols = int(fused_acc_cols(n_out, split, nch)) + (split ? n_out : 0);
    return cols <= 32 ? 32u : cols <= 64 ? 64u : cols <= 128 ? 128u : cols <= 256 ? 256u : 512u;
}

// Activation buffers: one in the split mode, else two.
__host__ __device__ constexpr int fused_act_bufs(bool split) { return split ? 1 : 2; }

struct FusedSmem {
    uint8_t* act[2];   // x, mid (the split mode: both the one buffer)
    uint8_t* ring;
    float* bn;         // every layer's folded batch norm: layer l's scale at l * 2N, shift at l * 2N + N
    uint64_t *wfull, *wempty, *in_full, *acc_full, *act_ready, *out_done, *done;
    uint64_t* epi;     // the epilogue warps' own barrier (one arrival per warp)
    uint32_t* tmem_slot;
};

__device__ __forceinline__ FusedSmem fused_carve(uint8_t* raw, const FusedArgs& p, int ops, uint32_t stage_bytes,
                                             int n_out, int bufs) {
    FusedSmem s;
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    const size_t buf = size_t(ops) * p.nch * p.act_bytes;
    s.act[0] = base;
    s.act[1] = base + (bufs - 1) * buf;
    s.ring = base + bufs * buf;
    s.bn = reinterpret_cast<float*>(s.ring + size_t(p.stages) * stage_bytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(s.bn + size_t(p.layers + 1) * 2 * n_out);
    s.wfull = bars;
    s.wempty = bars + p.stages;
    s.in_full = s.wempty + p.stages;
    s.acc_full = s.in_full + 1;
    s.act_ready = s.acc_full + 1;
    s.out_done = s.act_ready + 1;
    s.done = s.out_done + 1;
    s.epi = s.done + 1;
    s.tmem_slot = reinterpret_cast<uint32_t*>(s.epi + 1);
    return s;
}

// Byte offset of 16-byte piece u of `row` in a 128-byte-swizzled sub-buffer
// (as TMA's 128-byte swizzle and the MMA descriptors lay it out; the
// sub-buffers are 1024-byte aligned).
__device__ __forceinline__ uint32_t swz(int row, int u) {
    return uint32_t(row) * 128u + ((uint32_t(u) ^ uint32_t(row & 7)) << 4);
}

// CTAs per SM: two where the configuration's registers and shared memory
// allow (one CTA's epilogue then overlaps the other's MMAs), else one.
template <bool kSplit>
constexpr int kFusedCtas = kSplit ? 1 : 2;

template <int N, bool kBf16, bool kSplit, int kTps>
__global__ void __launch_bounds__(kFusedThreads<kSplit>, kFusedCtas<kSplit>)
    tower_fused(const __grid_constant__ CUtensorMap mIn, const __grid_constant__ CUtensorMap mInLo,
                const __grid_constant__ CUtensorMap mOut, const __grid_constant__ CUtensorMap mOutLo,
                const __grid_constant__ CUtensorMap mStem, const __grid_constant__ CUtensorMap mStemLo,
                const __grid_constant__ FusedArgs p) {
    using C = FusedCfg<N, kBf16, kSplit, kTps>;
    extern __shared__ uint8_t smem_raw[];
    constexpr int kBufs = fused_act_bufs(kSplit);
    const FusedSmem sm = fused_carve(smem_raw, p, C::kOps, C::kStage, N, kBufs);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ngroups = (p.boards + p.group - 1) / p.group;
    const int group_rows = p.group * p.S;
    const uint32_t tmem_cols = fused_tmem_cols(N, kSplit, p.nch);
    // Two issuers where each input chunk has its own accumulator and there
    // are two chunks; issuer i then owns chunk i's stages.
    const int issuers = kSplit && p.nch == 2 ? 2 : 1;

    // Zero the activation buffers: the halos and the rows past the group
    // stay zero for the whole launch.
    {
        const size_t words = size_t(kBufs) * C::kOps * p.nch * p.act_bytes / 16;
        uint4* w = reinterpret_cast<uint4*>(sm.act[0]);
        for (size_t i = threadIdx.x; i < words; i += blockDim.x) w[i] = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
        // Every layer's batch norm into shared memory: the epilogue reads it
        // on each layer's critical path. (Weights, not activations: no wait
        // for the previous kernel is needed.)
        // (the stem's, when it runs here, after the tower's: entry `layers`)
        const int nbn = (p.layers + (p.stem_nch > 0 ? 1 : 0)) * 2 * N;
        for (int i = threadIdx.x; i < nbn; i += blockDim.x) {
            const int l = i / (2 * N), j = i % (2 * N);
            const FusedLayer& L = l < p.layers ? p.layer[l] : *p.stem;
            sm.bn[i] = j < N ? L.scale[j] : L.shift[j - N];
        }
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.stages; ++i) {
            mbar_init(&sm.wfull[i], 1);
            mbar_init(&sm.wempty[i], 1);
        }
        mbar_init(sm.in_full, 1);
        mbar_init(sm.acc_full, uint32_t(issuers));
        mbar_init(sm.act_ready, kFusedEpiWarps);
        mbar_init(sm.out_done, p.heads ? kFusedEpiWarps : 1);   // heads: every epilogue warp reads x
        mbar_init(sm.done, uint32_t(issuers));
        mbar_init(sm.epi, kFusedEpiWarps);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&mIn);
        tma_prefetch_map(&mOut);
        if (kSplit) {
            tma_prefetch_map(&mInLo);
            tma_prefetch_map(&mOutLo);
        }
    }
    if (warp == 1) tmem_alloc(sm.tmem_slot, tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *sm.tmem_slot;
    grid_dependency_wait();   // the stem's output is read from here on
    grid_launch_dependents();

    // With the stem here, the input is the stem's packed operand (stem_nch
    // chunks, into mid) and step 0 is the stem (one tap); else the stem's
    // output (into x). Steps 1.. (or 0..) are the tower's convs.
    const int first = p.stem_nch > 0 ? 1 : 0, steps = p.layers + first;
    const uint32_t in_tx = uint32_t(group_rows) * 128u * C::kOps * (first ? p.stem_nch : p.nch);
    if (warp == 0) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            Ring rw;
            uint32_t nw = 0;
            bool ok = true;
            uint32_t k = 0;   // groups of this CTA so far
            for (int g = blockIdx.x; g < ngroups && ok; g += gridDim.x, ++k) {
                // The previous group's output has been stored (read out of x).
                if (k > 0 && !(ok = mbar_wait(sm.out_done, (k - 1) & 1, p.err, kErrWaitProducer))) break;
                mbar_arrive_expect_tx(sm.in_full, in_tx);
                for (int pl = 0; pl < C::kOps; ++pl)
                    for (int c = 0; c < (first ? p.stem_nch : p.nch); ++c)
                        tma_load_2d(first ? (pl ? &mStemLo : &mStem) : (pl ? &mInLo : &mIn),
                                    sm.act[first] + (size_t(pl) * p.nch + c) * p.act_bytes + size_t(p.top) * 128,
                                    sm.in_full, c * C::kKc, g * group_rows);
                for (int st_ = 0; st_ < steps && ok; ++st_) {
                    const bool stem = st_ < first;
                    const FusedLayer& L = stem ? *p.stem : p.layer[st_ - first];
                    // The stem: one tile per chunk (its stage otherwise empty).
                    // With two issuers the chunks' stages alternate (tap
                    // groups outer); else chunk-major, one issuer's order.
                    const int taps = stem ? 1 : 9, per_stage = stem ? 1 : kTps;
                    const int nch = stem ? p.stem_nch : p.nch, groups = taps / per_stage;
                    for (int i = 0; i < nch * groups && ok; ++i) {
                        const int c = issuers == 2 ? i % nch : i / groups;
                        const int t0 = (issuers == 2 ? i / nch : i % groups) * per_stage;
                        if (!(ok = mbar_wait(&sm.wempty[rw.idx], rw.phase ^ 1u, p.err, kErrWaitProducer))) break;
                        mbar_arrive_expect_tx(&sm.wfull[rw.idx], uint32_t(per_stage) * C::kTap);
                        for (int j = 0; j < per_stage; ++j) {
                            uint8_t* st = sm.ring + size_t(rw.idx) * C::kStage + size_t(j) * C::kTap;
                            const int x = (c * taps + t0 + j) * C::kKc;
                            tma_load_2d(&L.w, st, &sm.wfull[rw.idx], x, 0);
                            if (kSplit) tma_load_2d(&L.w_lo, st + C::kWTile, &sm.wfull[rw.idx], x, 0);
                        }
                        rw.next(p.stages);
                        ++nw;
                    }
                }
            }
            // Every copy issued has landed before the CTA may exit.
            for (uint32_t s = 0; s < uint32_t(p.stages) && s < nw; ++s) {
                const uint32_t uses = (nw - s + p.stages - 1) / p.stages;
                mbar_wait(&sm.wfull[s], (uses - 1) & 1, p.err, kErrWaitDrain);
            }
            if (k > 0) mbar_wait(sm.in_full, (k - 1) & 1, p.err, kErrWaitDrain);
        }
    } else if (warp == 1 || (kSplit && warp == 2 + kFusedEpiWarps)) {
        // -------------------------------------------------------- MMA issue
        // Issuer `me` issues the MMAs of the stages it owns and walks past
        // the others; with one issuer it owns them all.
        const int me = warp == 1 ? 0 : 1;
        if (lane == 0 && me < issuers) {
            Ring rw;
            bool ok = true;
            uint32_t k = 0, layers_done = 0;
            const uint32_t a0 = smem_u32(sm.act[0]), a1 = smem_u32(sm.act[1]);
            const uint64_t ring_desc = sw128_desc(smem_u32(sm.ring));
            constexpr uint32_t kStage16 = C::kStage >> 4, kTap16 = C::kTap >> 4;
            const uint32_t plane16 = (uint32_t(p.nch) * uint32_t(p.act_bytes)) >> 4, chunk16 = uint32_t(p.act_bytes) >> 4;
            // Tap t's view starts (top + dy(n+1) + dx) rows into the buffer
            // (descriptor units of 16 bytes: 8 per row).
            const uint32_t centre16 = uint32_t(p.top) * 8u, row16 = uint32_t(p.n + 1) * 8u;
            for (int g = blockIdx.x; g < ngroups && ok; g += gridDim.x, ++k) {
                for (int st_ = 0; st_ < steps && ok; ++st_) {
                    // The previous layer's epilogue has read TMEM and written
                    // this layer's input; the first layer's input is loaded.
                    if (layers_done > 0 &&
                        !(ok = mbar_wait(sm.act_ready, (layers_done - 1) & 1, p.err, kErrWaitMma)))
                        break;
                    if (st_ == 0 && !(ok = mbar_wait(sm.in_full, k & 1, p.err, kErrWaitMma))) break;
                    tc_fence_after();
                    if (st_ < first) {
                        // The stem: a one-tap GEMM over the packed operand in mid.
                        for (int c = 0; c < p.stem_nch && ok; ++c) {
                            if (c % issuers == me) {
                                if (!(ok = mbar_wait(&sm.wfull[rw.idx], rw.phase, p.err, kErrWaitMma))) break;
                                tc_fence_after();
                                const uint64_t at = sw128_desc(a1) + c * chunk16 + centre16,
                                               bt = ring_desc + rw.idx * kStage16;
#pragma unroll
                                for (int kk = 0; kk < C::kSteps; ++kk) {
                                    if constexpr (kSplit) {
                                        const uint32_t d = tmem + uint32_t(c) * 2u * N;
                                        constexpr uint32_t kIdescStack = umma_idesc(2 * N, kBf16);
                                        umma<kBf16>(d, at + 2 * kk, bt + 2 * kk, kIdescStack, kk != 0);
                                        umma<kBf16>(d + N, at + plane16 + 2 * kk, bt + 2 * kk, umma_idesc(N, kBf16), 1);
                                    } else {
                                        umma<kBf16>(tmem, at + 2 * kk, bt + 2 * kk, umma_idesc(N, kBf16), (c | kk) != 0);
                                    }
                                }
                                umma_commit(&sm.wempty[rw.idx]);
                            }
                            rw.next(p.stages);
                        }
                        if (!ok) break;
                        umma_commit(sm.acc_full);
                        ++layers_done;
                        continue;
                    }
                    const int l = st_ - first;
                    const uint64_t a_desc = sw128_desc((l & 1) ? a1 : a0);
                    if (issuers == 2) {
                        // Tap groups outer, the two chunks' stages alternating;
                        // this issuer's chunk is `me`, its own accumulator.
                        const uint64_t ac = a_desc + me * chunk16;
                        const uint32_t d = tmem + uint32_t(me) * 2u * N;
#pragma unroll
                        for (int t0 = 0; t0 < 9; t0 += kTps) {
#pragma unroll
                            for (int c = 0; c < 2; ++c) {
                                if (c == me) {
                                    if (!(ok = mbar_wait(&sm.wfull[rw.idx], rw.phase, p.err, kErrWaitMma))) break;
                                    tc_fence_after();
                                    const uint64_t bs = ring_desc + rw.idx * kStage16;
#pragma unroll
                                    for (int j = 0; j < kTps; ++j) {
                                        const int t = t0 + j;
                                        const uint64_t at = ac + centre16 + (t / 3 - 1) * int(row16) + (t % 3 - 1) * 8,
                                                       bt = bs + j * kTap16;
#pragma unroll
                                        for (int kk = 0; kk < C::kSteps; ++kk) {
                                            constexpr uint32_t kIdescStack = umma_idesc(2 * N, kBf16);
                                            umma<kBf16>(d, at + 2 * kk, bt + 2 * kk, kIdescStack, (t | kk) != 0);
                                            umma<kBf16>(d + N, at + plane16 + 2 * kk, bt + 2 * kk,
                                                        umma_idesc(N, kBf16), 1);
                                        }
                                    }
                                    umma_commit(&sm.wempty[rw.idx]);
                                }
                                rw.next(p.stages);
                            }
                            if (!ok) break;
                        }
                    } else {
                        for (int c = 0; c < p.nch && ok; ++c) {
                            const uint64_t ac = a_desc + c * chunk16;
                            uint64_t bs = 0;   // the current stage's descriptor
#pragma unroll
                            for (int t = 0; t < 9; ++t) {
                                if (t % kTps == 0) {
                                    if (!(ok = mbar_wait(&sm.wfull[rw.idx], rw.phase, p.err, kErrWaitMma))) break;
                                    tc_fence_after();
                                    bs = ring_desc + rw.idx * kStage16;
                                }
                                const uint64_t at = ac + centre16 + (t / 3 - 1) * int(row16) + (t % 3 - 1) * 8,
                                               bt = bs + (t % kTps) * kTap16;
#pragma unroll
                                for (int kk = 0; kk < C::kSteps; ++kk) {
                                    if constexpr (kSplit) {
                                        // Per input chunk its own stacked accumulator:
                                        // [0, N) a_hi.b_hi, [N, 2N) a_hi.b_lo + a_lo.b_hi.
                                        const uint32_t d = tmem + uint32_t(c) * 2u * N;
                                        constexpr uint32_t kIdescStack = umma_idesc(2 * N, kBf16);
                                        umma<kBf16>(d, at + 2 * kk, bt + 2 * kk, kIdescStack, (t | kk) != 0);
                                        umma<kBf16>(d + N, at + plane16 + 2 * kk, bt + 2 * kk, umma_idesc(N, kBf16), 1);
                                    } else {
                                        umma<kBf16>(tmem, at + 2 * kk, bt + 2 * kk, umma_idesc(N, kBf16),
                                                    (c | t | kk) != 0);
                                    }
                                }
                                if (t % kTps == kTps - 1) {
                                    umma_commit(&sm.wempty[rw.idx]);
                                    rw.next(p.stages);
                                }
                            }
                        }
                    }
                    if (!ok) break;
                    umma_commit(sm.acc_full);
                    ++layers_done;
                }
            }
            // Every MMA issued is complete before TMEM is freed (also after an error).
            umma_commit(sm.done);
            mbar_wait(sm.done, 0, p.err, kErrWaitDrain);
        }
    } else if (warp < 2 + kFusedEpiWarps) {
        // ---------------------------------------------------------- epilogue
        const int e = warp - 2, quarter = warp & 3, half = e >> 2;
        const bool active = N >= 64 || half == 0;
        const int col0 = half * C::kWarpCols;   // this warp's first output column
        const int row = quarter * 32 + lane;    // row of the tile (and TMEM lane)
        const int brow = p.top + row;           // its row in the activation buffers
        const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16);
        // This warp's residual columns: the block input at its rows and
        // output columns, fp32 (the split mode's hi + lo, as added).
        const uint32_t tres = taddr + fused_acc_cols(N, kSplit, p.nch) + uint32_t(col0);
        uint32_t k = 0, layers_done = 0, epi_uses = 0;
        bool ok = true;
        // The epilogue warps' barrier (bounded, where a named barrier would
        // wait forever for a warp that gave up): global writes before it are
        // visible to every epilogue warp after it.
        auto epi_sync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(sm.epi);
            const bool fine = mbar_wait(sm.epi, epi_uses & 1, p.err, kErrWaitEpilogue);
            ++epi_uses;
            __syncwarp();
            return fine;
        };
        // The heads' FCs of a group (policy FC and value FC1, the head tail
        // kernel's lane split and tree: the same bits) run while the next
        // group's layers are on the tensor core, a slice of this warp's quads
        // (e, e + 8, ...) per step; a warp per board then finishes the value
        // (FC2, tanh) and, when asked for, the softmax. The last group's run
        // after its own heads.
        int pend = -1, pend_boards = 0;   // the group whose FCs are pending: its first board
        const float4* feat4 = reinterpret_cast<const float4*>(p.head.feat);
        const size_t ld4 = size_t(p.head.feat_ld) / 4, val4 = size_t(p.head.feat_val) / 4;
        auto xpol = [&](int gb, int j) { return feat4[size_t(pend + gb) * ld4 + j]; };
        auto xval = [&](int gb, int j) { return feat4[size_t(pend + gb) * ld4 + val4 + j]; };
        auto hid_at = [&](int gb) { return p.head.hid + size_t(pend + gb) * p.head.V; };
        const int fc_quads = p.heads ? head_fc_quad_count<4>(p.head) : 0;
        const int warp_quads = (fc_quads + kFusedEpiWarps - 1) / kFusedEpiWarps;
        const int slice = (warp_quads + steps - 2) / (steps - 1);   // quads per step, the last step left for the finish
        auto fc_slice = [&](int i0, int i1) {
            for (int i = i0; i < i1; ++i) {
                const int q = e + i * kFusedEpiWarps;
                if (q >= fc_quads) break;
                head_fc_quad<4, kFusedFcBoards, true>(p.head, pend, pend_boards, q, xpol, xval, hid_at, lane);
            }
        };
        auto fc_finish = [&]() -> bool {
            if (!epi_sync()) return false;   // every warp's FC outputs are in
            for (int gb = e; gb < pend_boards; gb += kFusedEpiWarps) head_finish_board(p.head, pend + gb, hid_at(gb), lane);
            pend = -1;
            return true;
        };
        for (int g = blockIdx.x; g < ngroups && ok; g += gridDim.x, ++k) {
            const int boards = min(p.group, p.boards - g * p.group);
            bool valid = row < boards * p.S;
            if (valid) {
                const int r = row % p.S;
                valid = r >= p.n + 1 && (r % (p.n + 1)) != p.n;
            }
            for (int st_ = 0; st_ < steps && ok; ++st_) {
                const bool stem = st_ < first;
                const int l = stem ? p.layers : st_ - first;   // the batch norm's entry
                const bool skip = !stem && (l & 1) != 0;   // the block's second conv adds the block input
                if (kSplit && !stem && !skip && active) {
                    // A block's first conv: while its MMAs read the block input,
                    // this warp copies its part (every lane its row, 32
                    // columns) into TMEM, where the second conv's epilogue
                    // reads it back: the buffer then takes each output in place.
                    // The group's first step reads the loaded input.
                    if (st_ == 0 && !(ok = mbar_wait(sm.in_full, k & 1, p.err, kErrWaitEpilogue))) break;
                    uint32_t r[32];
                    const uint8_t* hi = sm.act[0] + size_t(col0 / 32) * p.act_bytes;
                    const uint8_t* lo = sm.act[0] + (size_t(p.nch) + col0 / 32) * p.act_bytes;
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const float4 h = *reinterpret_cast<const float4*>(hi + swz(brow, u));
                        const float4 l4 = *reinterpret_cast<const float4*>(lo + swz(brow, u));
                        r[4 * u] = __float_as_uint(__fadd_rn(h.x, l4.x));
                        r[4 * u + 1] = __float_as_uint(__fadd_rn(h.y, l4.y));
                        r[4 * u + 2] = __float_as_uint(__fadd_rn(h.z, l4.z));
                        r[4 * u + 3] = __float_as_uint(__fadd_rn(h.w, l4.w));
                    }
                    tmem_st32(tres, r);
                    tmem_wait_st();
                }
                if (pend >= 0) {
                    if (st_ < steps - 1)
                        fc_slice(st_ * slice, (st_ + 1) * slice);
                    else if (!(ok = fc_finish()))
                        break;
                }
                if (!(ok = mbar_wait(sm.acc_full, layers_done & 1, p.err, kErrWaitEpilogue))) break;
                tc_fence_after();
                uint8_t* out = stem || (l & 1) ? sm.act[0] : sm.act[1];
                if (active && kSplit) {
                    // The split mode, its 32 columns in two halves of 16: the
                    // second half's TMEM loads fly while the first half's
                    // pieces are computed. Per column the accumulator is
                    // (hh + mixed) of chunk 0, then + (hh + mixed) of chunk 1.
                    const float4* sc4 = reinterpret_cast<const float4*>(sm.bn + size_t(l) * 2 * N + col0);
                    const float4* sh4 = reinterpret_cast<const float4*>(sm.bn + size_t(l) * 2 * N + N + col0);
                    uint8_t* hi = out + size_t(col0 / 32) * p.act_bytes;
                    uint8_t* lo = out + (size_t(p.nch) + col0 / 32) * p.act_bytes;
                    const bool two = p.nch == 2;
                    uint32_t rv[32];   // the block input, at the block's second conv
                    uint32_t v0[16], w0[16], v1[16], w1[16];
                    float acc[16];
                    auto load = [&](int h) {
                        const uint32_t at = taddr + uint32_t(col0 + 16 * h);
                        tmem_ld16(at, v0);
                        tmem_ld16(at + N, w0);
                        if (two) {
                            tmem_ld16(at + 2 * N, v1);
                            tmem_ld16(at + 3 * N, w1);
                        }
                    };
                    auto combine = [&]() {
#pragma unroll
                        for (int i = 0; i < 16; i += 2) {
                            float2 s2 = fadd2_rn(make_float2(__uint_as_float(v0[i]), __uint_as_float(v0[i + 1])),
                                                 make_float2(__uint_as_float(w0[i]), __uint_as_float(w0[i + 1])));
                            if (two)
                                s2 = fadd2_rn(s2, fadd2_rn(make_float2(__uint_as_float(v1[i]), __uint_as_float(v1[i + 1])),
                                                           make_float2(__uint_as_float(w1[i]), __uint_as_float(w1[i + 1]))));
                            acc[i] = s2.x;
                            acc[i + 1] = s2.y;
                        }
                    };
                    // Pieces 4h..4h+3: the batch norm, the residual, ReLU, the
                    // tf32 split, the stores (the reference's separate
                    // roundings, src/cuda/kernels.cu:172-176).
                    auto pieces = [&](int h) {
                        if (!valid) return;
#pragma unroll
                        for (int uu = 0; uu < 4; ++uu) {
                            const int u = 4 * h + uu;
                            const float4 a = sc4[u], b = sh4[u];
                            // (The batch norm stays scalar: a packed multiply
                            // feeding a packed add is fused into one rounding.)
                            float2 y01 = make_float2(__fadd_rn(__fmul_rn(a.x, acc[4 * uu]), b.x),
                                                     __fadd_rn(__fmul_rn(a.y, acc[4 * uu + 1]), b.y));
                            float2 y23 = make_float2(__fadd_rn(__fmul_rn(a.z, acc[4 * uu + 2]), b.z),
                                                     __fadd_rn(__fmul_rn(a.w, acc[4 * uu + 3]), b.w));
                            if (skip) {
                                y01 = fadd2_rn(y01, make_float2(__uint_as_float(rv[4 * u]), __uint_as_float(rv[4 * u + 1])));
                                y23 = fadd2_rn(y23, make_float2(__uint_as_float(rv[4 * u + 2]), __uint_as_float(rv[4 * u + 3])));
                            }
                            y01.x = y01.x > 0.0f ? y01.x : 0.0f;
                            y01.y = y01.y > 0.0f ? y01.y : 0.0f;
                            y23.x = y23.x > 0.0f ? y23.x : 0.0f;
                            y23.y = y23.y > 0.0f ? y23.y : 0.0f;
                            const float4 hv = make_float4(to_tf32(y01.x), to_tf32(y01.y), to_tf32(y23.x), to_tf32(y23.y));
                            const float2 l01 = fsub2_rn(y01, make_float2(hv.x, hv.y));
                            const float2 l23 = fsub2_rn(y23, make_float2(hv.z, hv.w));
                            *reinterpret_cast<float4*>(hi + swz(brow, u)) = hv;
                            *reinterpret_cast<float4*>(lo + swz(brow, u)) = make_float4(l01.x, l01.y, l23.x, l23.y);
                        }
                    };
                    auto hold = [&]() {
                        tmem_hold(v0);
                        tmem_hold(w0);
                        if (two) {
                            tmem_hold(v1);
                            tmem_hold(w1);
                        }
                    };
                    if (skip) tmem_ld32(tres, rv);
                    load(0);
                    tmem_wait_ld();
                    hold();
                    if (skip) tmem_hold(rv);
                    combine();
                    load(1);   // in flight during the first half's pieces
                    pieces(0);
                    tmem_wait_ld();
                    hold();
                    combine();
                    pieces(1);
                } else if (active) {
#pragma unroll
                    for (int cb = 0; cb < C::kWarpCols / 32; ++cb) {
                        const int c0 = col0 + cb * 32;   // 32 output channels
                        float acc[32];
                        {
                            uint32_t v[32];
                            tmem_ld32(taddr + uint32_t(c0), v);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(v[i]);
                        }
                        if (valid) {
                            // Per 16-byte piece: the batch norm, the residual, ReLU, the store
                            // (the reference's separate roundings, src/cuda/kernels.cu:172-176).
                            const float4* sc4 = reinterpret_cast<const float4*>(sm.bn + size_t(l) * 2 * N + c0);
                            const float4* sh4 = reinterpret_cast<const float4*>(sm.bn + size_t(l) * 2 * N + N + c0);
                            if constexpr (kBf16) {
                                const int u0 = c0 / 8;   // one 128-byte chunk of 64 channels, 8 per piece
#pragma unroll
                                for (int u = 0; u < 4; ++u) {
                                    float y[8];
#pragma unroll
                                    for (int h = 0; h < 2; ++h) {
                                        const float4 a = sc4[2 * u + h], b = sh4[2 * u + h];
                                        y[4 * h] = __fadd_rn(__fmul_rn(a.x, acc[8 * u + 4 * h]), b.x);
                                        y[4 * h + 1] = __fadd_rn(__fmul_rn(a.y, acc[8 * u + 4 * h + 1]), b.y);
                                        y[4 * h + 2] = __fadd_rn(__fmul_rn(a.z, acc[8 * u + 4 * h + 2]), b.z);
                                        y[4 * h + 3] = __fadd_rn(__fmul_rn(a.w, acc[8 * u + 4 * h + 3]), b.w);
                                    }
                                    uint8_t* at = out + swz(brow, u0 + u);
                                    if (skip) {
                                        const uint4 w4 = *reinterpret_cast<const uint4*>(at);
                                        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w4);
#pragma unroll
                                        for (int q = 0; q < 4; ++q) {
                                            const float2 f = __bfloat1622float2(h2[q]);
                                            y[2 * q] = __fadd_rn(y[2 * q], f.x);
                                            y[2 * q + 1] = __fadd_rn(y[2 * q + 1], f.y);
                                        }
                                    }
                                    uint4 o;
                                    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                                    for (int q = 0; q < 4; ++q)
                                        o2[q] = __floats2bfloat162_rn(y[2 * q] > 0.0f ? y[2 * q] : 0.0f,
                                                                      y[2 * q + 1] > 0.0f ? y[2 * q + 1] : 0.0f);
                                    *reinterpret_cast<uint4*>(at) = o;
                                }
                            } else {
                                // fp32 (tf32 mode): channel block c0 is chunk c0 / 32.
                                uint8_t* hi = out + size_t(c0 / 32) * p.act_bytes;
#pragma unroll
                                for (int u = 0; u < 8; ++u) {
                                    const float4 a = sc4[u], b = sh4[u];
                                    float y[4] = {__fadd_rn(__fmul_rn(a.x, acc[4 * u]), b.x),
                                                  __fadd_rn(__fmul_rn(a.y, acc[4 * u + 1]), b.y),
                                                  __fadd_rn(__fmul_rn(a.z, acc[4 * u + 2]), b.z),
                                                  __fadd_rn(__fmul_rn(a.w, acc[4 * u + 3]), b.w)};
                                    if (skip) {
                                        const float4 h = *reinterpret_cast<const float4*>(hi + swz(brow, u));
                                        y[0] = __fadd_rn(y[0], h.x);
                                        y[1] = __fadd_rn(y[1], h.y);
                                        y[2] = __fadd_rn(y[2], h.z);
                                        y[3] = __fadd_rn(y[3], h.w);
                                    }
#pragma unroll
                                    for (int q = 0; q < 4; ++q) y[q] = y[q] > 0.0f ? y[q] : 0.0f;
                                    *reinterpret_cast<float4*>(hi + swz(brow, u)) = make_float4(y[0], y[1], y[2], y[3]);
                                }
                            }
                        }
                    }
                }
                fence_proxy_async_smem();   // the writes, visible to the next layer's MMAs and the store
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(sm.act_ready);
                ++layers_done;
            }
            if (!ok) break;
            if (p.heads) {
                // The heads' 1x1 convolutions straight from x, with the head
                // kernel's lane split and reduction tree (the same bits),
                // once every epilogue warp has written the last layer.
                if (!(ok = mbar_wait(sm.act_ready, (layers_done - 1) & 1, p.err, kErrWaitEpilogue))) break;
                constexpr int kMode = kBf16 ? kBF16 : (kSplit ? kTF32x3 : kTF32);
                constexpr int kLpr = kBf16 || N == 32 ? 8 : 16;   // 16-byte pieces per stored row
                using H = HeadLane<kMode, kLpr, 1>;
                H hl;
                hl.load(p.head, lane);
                const int A = p.n * p.n, pts = boards * A, n = p.n, S = p.S, top = p.top;
                const int first_board = g * p.group;
                const size_t act_bytes = size_t(p.act_bytes), lo_off = size_t(p.nch) * act_bytes;
                const uint8_t* xbuf = sm.act[0];
                auto piece = [=](int pt, int j) {   // point pt of the group: its row in x
                    const int b = pt / A, q = pt - b * A, y = q / n, xx = q - y * n;
                    const int brow = top + b * S + (y + 1) * (n + 1) + xx, c = j >> 3, u = j & 7;
                    TrunkPiece<kMode> pc;
                    pc.hi = *reinterpret_cast<const uint4*>(xbuf + size_t(c) * act_bytes + swz(brow, u));
                    if (kSplit) pc.lo = *reinterpret_cast<const uint4*>(xbuf + lo_off + size_t(c) * act_bytes + swz(brow, u));
                    return pc;
                };
                auto where = [=](int pt, int* b, int* q) {
                    *b = first_board + pt / A;
                    *q = pt % A;
                };
                for (int base = e * H::kStepRows; base < pts; base += kFusedEpiWarps * H::kStepRows)
                    hl.step(p.head, base, pts, piece, where, lane);
                __syncwarp();
                if (lane == 0) mbar_arrive(sm.out_done);   // x may be overwritten by the next group's input
                // The features every epilogue warp wrote are visible to all;
                // the group's FCs wait for the next group's steps.
                if (!(ok = epi_sync())) break;
                pend = first_board;
                pend_boards = boards;
            } else if (e == 0 && lane == 0) {
                // The tower's output (x) leaves once every epilogue warp has
                // written the last layer.
                if (!(ok = mbar_wait(sm.act_ready, (layers_done - 1) & 1, p.err, kErrWaitEpilogue))) break;
                for (int pl = 0; pl < C::kOps; ++pl)
                    for (int c = 0; c < p.nch; ++c)
                        tma_store_2d(pl ? &mOutLo : &mOut,
                                     sm.act[0] + (size_t(pl) * p.nch + c) * p.act_bytes + size_t(p.top) * 128,
                                     c * C::kKc, g * group_rows);
                bulk_commit();
                bulk_wait_read<0>();   // x may be overwritten by the next group's input
                mbar_arrive(sm.out_done);
            }
        }
        if (ok && pend >= 0) {   // the last group's FCs: on the critical path, eight outputs per warp step
            const int octs = head_fc_quad_count<8>(p.head);
            for (int q = e; q < octs; q += kFusedEpiWarps)
                head_fc_quad<8, kFusedFcBoards>(p.head, pend, pend_boards, q, xpol, xval, hid_at, lane);
            fc_finish();
        }
        if (e == 0 && lane == 0) bulk_wait_all();   // every store complete before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols);
    }
}

// ------------------------------------------------------------- board pairs
//
// The split mode at 64 channels with two groups of boards in flight per CTA.
// One group alone runs each layer as its MMAs, then its epilogue (TMEM
// reads, batch norm, the stores): the tensor core idles through the one and
// the epilogue warps through the other. Two groups, each with its own
// activation buffer, its own issuing thread and four epilogue warps, keep the
// tensor core busy with one group's MMAs while the other's epilogue runs,
// and every weight stage feeds both (it is released after both issuers'
// commits). TMEM holds per group one stacked accumulator of 128 columns
// (group g at 128 g), its block input (at 256 + 64 g) and its chunk-0 sums
// (at 384 + 64 g): the two input chunks are two segments in time on the same
// accumulator (the epilogue reads chunk 0's, parks its sums, before chunk
// 1's MMAs start on it), the same MMAs and the same sums, in the same order,
// as the one-group kernel's two stacks, so the outputs are the same bits.
// At every step the epilogue reads both groups' chunk-0 segments before
// either's chunk-1 segment: the issuers share the weight stages (a ring
// shorter than a chunk's taps), so one group's second segment must never
// wait for the other group's output.
//
// Warps: 0 loads (both groups' inputs, then the weight stages both
// consume), 1 and 10 issue group 0's and group 1's MMAs, 2-9 run both
// groups' epilogues, group 0's then group 1's at every step, and the heads.
constexpr int kPairThreads = 352;
constexpr uint32_t kPairTmemCols = 512;

template <int kTps>
struct PairCfg {
    static constexpr int N = 64, kKc = 32, kSteps = 4;
    static constexpr uint32_t kWTile = 64u * 128u;           // one plane of a (chunk, tap) weight tile
    static constexpr uint32_t kTap = 2u * kWTile;            // both planes
    static constexpr uint32_t kStage = uint32_t(kTps) * kTap;
};

// (The batch norm is read through the read-only cache, not staged: its
// 6.6 KB would take the room of the second three-tap weight stage.)
struct PairSmem {
    uint8_t* act[2];   // each group's activations: [plane][chunk] sub-buffers
    uint8_t* ring;
    uint64_t *wfull, *wempty;
    // Two each, one per group (epi: only [0] is used, the eight epilogue
    // warps' barrier for both groups).
    uint64_t *in_full, *seg_full, *seg_empty, *act_ready, *out_done, *epi;
    uint64_t* done;
    uint32_t* tmem_slot;
};

__device__ __forceinline__ PairSmem pair_carve(uint8_t* raw, const FusedArgs& p, uint32_t stage_bytes) {
    PairSmem s;
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    const size_t buf = 2 * size_t(p.nch) * p.act_bytes;
    s.act[0] = base;
    s.act[1] = base + buf;
    s.ring = base + 2 * buf;
    uint64_t* bars = reinterpret_cast<uint64_t*>(s.ring + size_t(p.stages) * stage_bytes);
    s.wfull = bars;
    s.wempty = bars + p.stages;
    uint64_t* g = s.wempty + p.stages;
    s.in_full = g;
    s.seg_full = g + 2;
    s.seg_empty = g + 4;
    s.act_ready = g + 6;
    s.out_done = g + 8;
    s.epi = g + 10;
    s.done = g + 12;
    s.tmem_slot = reinterpret_cast<uint32_t*>(s.done + 1);
    return s;
}

template <int kTps>
__global__ void __launch_bounds__(kPairThreads, 1)
    tower_fused_pair(const __grid_constant__ CUtensorMap mIn, const __grid_constant__ CUtensorMap mInLo,
                     const __grid_constant__ CUtensorMap mStem, const __grid_constant__ CUtensorMap mStemLo,
                     const __grid_constant__ FusedArgs p) {
    using C = PairCfg<kTps>;
    constexpr int N = C::N;
    extern __shared__ uint8_t smem_raw[];
    const PairSmem sm = pair_carve(smem_raw, p, C::kStage);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ngroups = (p.boards + p.group - 1) / p.group, npairs = (ngroups + 1) / 2;
    const int group_rows = p.group * p.S;
    {
        const size_t words = 2 * 2 * size_t(p.nch) * p.act_bytes / 16;
        uint4* w = reinterpret_cast<uint4*>(sm.act[0]);
        for (size_t i = threadIdx.x; i < words; i += blockDim.x) w[i] = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.stages; ++i) {
            mbar_init(&sm.wfull[i], 1);
            mbar_init(&sm.wempty[i], 2);   // both issuers
        }
        for (int g = 0; g < 2; ++g) {
            mbar_init(&sm.in_full[g], 1);
            mbar_init(&sm.seg_full[g], 1);
            mbar_init(&sm.seg_empty[g], kFusedEpiWarps);
            mbar_init(&sm.act_ready[g], kFusedEpiWarps);
            mbar_init(&sm.out_done[g], kFusedEpiWarps);
            mbar_init(&sm.epi[g], kFusedEpiWarps);
        }
        mbar_init(sm.done, 2);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&mIn);
        tma_prefetch_map(&mInLo);
    }
    if (warp == 1) tmem_alloc(sm.tmem_slot, kPairTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *sm.tmem_slot;
    grid_dependency_wait();
    grid_launch_dependents();

    const int first = p.stem_nch > 0 ? 1 : 0, steps = p.layers + first;
    const int in_chunks = first ? p.stem_nch : p.nch;
    const uint32_t in_tx = uint32_t(group_rows) * 128u * 2u * uint32_t(in_chunks);
    if (warp == 0) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            Ring rw;
            uint32_t nw = 0, kin[2] = {0, 0};
            bool ok = true;
            for (int P = blockIdx.x; P < npairs && ok; P += gridDim.x) {
                for (int g = 0; g < 2 && ok; ++g) {
                    const int grp = 2 * P + g;
                    if (grp >= ngroups) continue;
                    // The group's previous pair has been read out of its buffer.
                    if (kin[g] > 0 && !(ok = mbar_wait(&sm.out_done[g], (kin[g] - 1) & 1, p.err, kErrWaitProducer))) break;
                    mbar_arrive_expect_tx(&sm.in_full[g], in_tx);
                    for (int pl = 0; pl < 2; ++pl)
                        for (int c = 0; c < in_chunks; ++c)
                            tma_load_2d(first ? (pl ? &mStemLo : &mStem) : (pl ? &mInLo : &mIn),
                                        sm.act[g] + (size_t(pl) * p.nch + c) * p.act_bytes + size_t(p.top) * 128,
                                        &sm.in_full[g], c * C::kKc, grp * group_rows);
                    ++kin[g];
                }
                for (int st_ = 0; st_ < steps && ok; ++st_) {
                    const bool stem = st_ < first;
                    const FusedLayer& L = stem ? *p.stem : p.layer[st_ - first];
                    // Chunk-major, one issuer's order: a chunk's taps in
                    // stages of kTps (the stem: one tap, one stage per chunk).
                    const int taps = stem ? 1 : 9, per_stage = stem ? 1 : kTps;
                    const int nch = stem ? p.stem_nch : p.nch;
                    for (int c = 0; c < nch && ok; ++c)
                        for (int t0 = 0; t0 < taps && ok; t0 += per_stage) {
                            if (!(ok = mbar_wait(&sm.wempty[rw.idx], rw.phase ^ 1u, p.err, kErrWaitProducer))) break;
                            mbar_arrive_expect_tx(&sm.wfull[rw.idx], uint32_t(per_stage) * C::kTap);
                            for (int j = 0; j < per_stage; ++j) {
                                uint8_t* st = sm.ring + size_t(rw.idx) * C::kStage + size_t(j) * C::kTap;
                                const int x = (c * taps + t0 + j) * C::kKc;
                                tma_load_2d(&L.w, st, &sm.wfull[rw.idx], x, 0);
                                tma_load_2d(&L.w_lo, st + C::kWTile, &sm.wfull[rw.idx], x, 0);
                            }
                            rw.next(p.stages);
                            ++nw;
                        }
                }
            }
            // Every copy issued has landed before the CTA may exit.
            for (uint32_t s = 0; s < uint32_t(p.stages) && s < nw; ++s) {
                const uint32_t uses = (nw - s + p.stages - 1) / p.stages;
                mbar_wait(&sm.wfull[s], (uses - 1) & 1, p.err, kErrWaitDrain);
            }
            for (int g = 0; g < 2; ++g)
                if (kin[g] > 0) mbar_wait(&sm.in_full[g], (kin[g] - 1) & 1, p.err, kErrWaitDrain);
        }
    } else if (warp == 1 || warp == 2 + kFusedEpiWarps) {
        // -------------------------------------------------------- MMA issue
        // Issuer g: its group's MMAs, a segment per input chunk on the
        // group's accumulator. Where its group is absent (an odd number of
        // groups) it walks the ring all the same, releasing each stage.
        const int g = warp == 1 ? 0 : 1;
        if (lane == 0) {
            Ring rw;
            bool ok = true;
            uint32_t segs = 0, steps_done = 0, kin = 0;
            const uint64_t a_desc = sw128_desc(smem_u32(sm.act[g]));
            const uint64_t ring_desc = sw128_desc(smem_u32(sm.ring));
            const uint32_t d = tmem + uint32_t(g) * 128u;
            constexpr uint32_t kStage16 = C::kStage >> 4, kTap16 = C::kTap >> 4;
            constexpr uint32_t kIdescStack = umma_idesc(2 * N, false), kIdesc = umma_idesc(N, false);
            const uint32_t plane16 = (uint32_t(p.nch) * uint32_t(p.act_bytes)) >> 4, chunk16 = uint32_t(p.act_bytes) >> 4;
            const uint32_t centre16 = uint32_t(p.top) * 8u, row16 = uint32_t(p.n + 1) * 8u;
            for (int P = blockIdx.x; P < npairs && ok; P += gridDim.x) {
                const bool mine = 2 * P + g < ngroups;
                for (int st_ = 0; st_ < steps && ok; ++st_) {
                    const bool stem = st_ < first;
                    const int taps = stem ? 1 : 9, per_stage = stem ? 1 : kTps;
                    const int nch = stem ? p.stem_nch : p.nch;
                    if (mine) {
                        // The group's input is loaded, or its previous step
                        // written (and read out of TMEM).
                        ok = st_ == 0 ? mbar_wait(&sm.in_full[g], kin & 1, p.err, kErrWaitMma)
                                      : mbar_wait(&sm.act_ready[g], (steps_done - 1) & 1, p.err, kErrWaitMma);
                        if (!ok) break;
                    }
                    for (int c = 0; c < nch && ok; ++c) {
                        // The accumulator's previous segment has been read.
                        if (mine && !(ok = mbar_wait(&sm.seg_empty[g], (segs & 1) ^ 1, p.err, kErrWaitMma))) break;
                        tc_fence_after();
                        const uint64_t ac = a_desc + uint32_t(c) * chunk16 + centre16;
                        for (int t0 = 0; t0 < taps && ok; t0 += per_stage) {
                            if (!(ok = mbar_wait(&sm.wfull[rw.idx], rw.phase, p.err, kErrWaitMma))) break;
                            if (mine) {
                                tc_fence_after();
                                const uint64_t bs = ring_desc + rw.idx * kStage16;
                                if (stem) {
#pragma unroll
                                    for (int kk = 0; kk < C::kSteps; ++kk) {
                                        umma<false>(d, ac + 2 * kk, bs + 2 * kk, kIdescStack, kk != 0);
                                        umma<false>(d + N, ac + plane16 + 2 * kk, bs + 2 * kk, kIdesc, 1);
                                    }
                                } else {
#pragma unroll
                                    for (int j = 0; j < kTps; ++j) {
                                        const int t = t0 + j;
                                        const uint64_t at = ac + (t / 3 - 1) * int(row16) + (t % 3 - 1) * 8,
                                                       bt = bs + j * kTap16;
#pragma unroll
                                        for (int kk = 0; kk < C::kSteps; ++kk) {
                                            umma<false>(d, at + 2 * kk, bt + 2 * kk, kIdescStack, (t | kk) != 0);
                                            umma<false>(d + N, at + plane16 + 2 * kk, bt + 2 * kk, kIdesc, 1);
                                        }
                                    }
                                }
                                umma_commit(&sm.wempty[rw.idx]);
                            } else {
                                mbar_arrive(&sm.wempty[rw.idx]);
                            }
                            rw.next(p.stages);
                        }
                        if (!ok) break;
                        if (mine) {
                            umma_commit(&sm.seg_full[g]);
                            ++segs;
                        }
                    }
                    if (mine) ++steps_done;
                }
                if (mine) ++kin;
            }
            // Every MMA issued is complete before TMEM is freed (also after an error).
            umma_commit(sm.done);
            mbar_wait(sm.done, 0, p.err, kErrWaitDrain);
        }
    } else if (warp < 2 + kFusedEpiWarps) {
        // ---------------------------------------------------------- epilogue
        // Eight warps for both groups, each step group 0's epilogue then
        // group 1's (so one group's runs while the other's MMAs do): warp w
        // reads TMEM lanes 32 (w % 4) ..., the two warps of a lane quarter
        // split the output columns, as in the one-group kernel.
        const int e = warp - 2, quarter = warp & 3, half = e >> 2;
        const int col0 = half * 32;
        const int row = quarter * 32 + lane;    // row of the tile (and TMEM lane)
        const int brow = p.top + row;           // its row in a group's buffer
        const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16);
        uint32_t segs[2] = {0, 0}, steps_done[2] = {0, 0}, kin = 0, epi_uses = 0;
        bool ok = true;
        auto epi_sync = [&]() -> bool {   // the eight epilogue warps (bounded)
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.epi[0]);
            const bool fine = mbar_wait(&sm.epi[0], epi_uses & 1, p.err, kErrWaitEpilogue);
            ++epi_uses;
            __syncwarp();
            return fine;
        };
        // A pair's FCs run during the next pair's steps, as in the one-group
        // kernel (boards [pend, pend + pend_boards), both groups', in runs of
        // at most kFusedFcBoards).
        int pend = -1, pend_boards = 0, fb = 0;
        const float4* feat4 = reinterpret_cast<const float4*>(p.head.feat);
        const size_t ld4 = size_t(p.head.feat_ld) / 4, val4 = size_t(p.head.feat_val) / 4;
        auto xpol = [&](int gb, int j) { return feat4[size_t(fb + gb) * ld4 + j]; };
        auto xval = [&](int gb, int j) { return feat4[size_t(fb + gb) * ld4 + val4 + j]; };
        auto hid_at = [&](int gb) { return p.head.hid + size_t(fb + gb) * p.head.V; };
        const int fc_quads = head_fc_quad_count<4>(p.head);
        const int warp_quads = (fc_quads + kFusedEpiWarps - 1) / kFusedEpiWarps;
        const int slice = (warp_quads + steps - 2) / (steps - 1);
        auto fc_slice = [&](int i0, int i1) {
            for (int i = i0; i < i1; ++i) {
                const int q = e + i * kFusedEpiWarps;
                if (q >= fc_quads) break;
                for (int b0 = 0; b0 < pend_boards; b0 += kFusedFcBoards) {
                    fb = pend + b0;
                    head_fc_quad<4, kFusedFcBoards, true>(p.head, fb, min(kFusedFcBoards, pend_boards - b0), q, xpol,
                                                          xval, hid_at, lane);
                }
            }
        };
        auto fc_finish = [&]() -> bool {
            if (!epi_sync()) return false;
            fb = pend;
            for (int gb = e; gb < pend_boards; gb += kFusedEpiWarps) head_finish_board(p.head, pend + gb, hid_at(gb), lane);
            pend = -1;
            return true;
        };
        for (int P = blockIdx.x; P < npairs && ok; P += gridDim.x) {
            const int ng = 2 * P + 1 < ngroups ? 2 : 1;   // groups in this pair
            bool valid[2];
            int boards[2];
            for (int g = 0; g < 2; ++g) {
                boards[g] = g < ng ? min(p.group, p.boards - (2 * P + g) * p.group) : 0;
                valid[g] = row < boards[g] * p.S;
                if (valid[g]) {
                    const int r = row % p.S;
                    valid[g] = r >= p.n + 1 && (r % (p.n + 1)) != p.n;
                }
            }
            for (int st_ = 0; st_ < steps && ok; ++st_) {
                const bool stem = st_ < first;
                const int l = stem ? p.layers : st_ - first;   // the batch norm's entry
                const bool skip = !stem && (l & 1) != 0;   // (every step has two segments: nch == stem_nch == 2)
                if (pend >= 0) {
                    if (st_ < steps - 1)
                        fc_slice(st_ * slice, (st_ + 1) * slice);
                    else if (!(ok = fc_finish()))
                        break;
                }
                // Chunk 0's segment of each group first, its sums (hh + mixed)
                // parked in TMEM (at 384 + 64 g): the two issuers share the
                // weight stages, so neither group's second segment may wait
                // for the other group's output.
                for (int g = 0; g < ng && ok; ++g) {
                    const uint8_t* hi = sm.act[g] + size_t(col0 / 32) * p.act_bytes;
                    const uint8_t* lo = sm.act[g] + (size_t(p.nch) + col0 / 32) * p.act_bytes;
                    const uint32_t stack = taddr + uint32_t(g) * 128u + uint32_t(col0);
                    if (!stem && !skip) {
                        // A block's first conv: its input (hi + lo, fp32) into
                        // TMEM (at 256 + 64 g) for the second conv's epilogue.
                        if (st_ == 0 && !(ok = mbar_wait(&sm.in_full[g], kin & 1, p.err, kErrWaitEpilogue))) break;
                        uint32_t r[32];
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const float4 a4 = *reinterpret_cast<const float4*>(hi + swz(brow, u));
                            const float4 l4 = *reinterpret_cast<const float4*>(lo + swz(brow, u));
                            r[4 * u] = __float_as_uint(__fadd_rn(a4.x, l4.x));
                            r[4 * u + 1] = __float_as_uint(__fadd_rn(a4.y, l4.y));
                            r[4 * u + 2] = __float_as_uint(__fadd_rn(a4.z, l4.z));
                            r[4 * u + 3] = __float_as_uint(__fadd_rn(a4.w, l4.w));
                        }
                        tmem_st32(taddr + 256u + uint32_t(g) * 64u + uint32_t(col0), r);
                    }
                    if (!(ok = mbar_wait(&sm.seg_full[g], segs[g] & 1, p.err, kErrWaitEpilogue))) break;
                    tc_fence_after();
                    uint32_t part[32];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint32_t v0[16], w0[16];
                        tmem_ld16(stack + 16u * h, v0);
                        tmem_ld16(stack + N + 16u * h, w0);
                        tmem_wait_ld();
                        tmem_hold(v0);
                        tmem_hold(w0);
#pragma unroll
                        for (int i = 0; i < 16; i += 2) {
                            const float2 pa = fadd2_rn(make_float2(__uint_as_float(v0[i]), __uint_as_float(v0[i + 1])),
                                                       make_float2(__uint_as_float(w0[i]), __uint_as_float(w0[i + 1])));
                            part[16 * h + i] = __float_as_uint(pa.x);
                            part[16 * h + i + 1] = __float_as_uint(pa.y);
                        }
                    }
                    tmem_st32(taddr + 384u + uint32_t(g) * 64u + uint32_t(col0), part);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sm.seg_empty[g]);
                    ++segs[g];
                }
                // Then per group chunk 1's segment added to the parked sums,
                // and the output.
                for (int g = 0; g < ng && ok; ++g) {
                    uint8_t* const buf = sm.act[g];
                    const uint32_t stack = taddr + uint32_t(g) * 128u + uint32_t(col0);
                    uint8_t* hi = buf + size_t(col0 / 32) * p.act_bytes;
                    uint8_t* lo = buf + (size_t(p.nch) + col0 / 32) * p.act_bytes;
                    if (!(ok = mbar_wait(&sm.seg_full[g], segs[g] & 1, p.err, kErrWaitEpilogue))) break;
                    tc_fence_after();
                    float acc[32];
                    {
                        uint32_t pv[32];
                        tmem_ld32(taddr + 384u + uint32_t(g) * 64u + uint32_t(col0), pv);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            uint32_t v0[16], w0[16];
                            tmem_ld16(stack + 16u * h, v0);
                            tmem_ld16(stack + N + 16u * h, w0);
                            tmem_wait_ld();
                            tmem_hold(v0);
                            tmem_hold(w0);
                            if (h == 0) tmem_hold(pv);
#pragma unroll
                            for (int i = 0; i < 16; i += 2) {
                                const int k = 16 * h + i;
                                const float2 pa = fadd2_rn(make_float2(__uint_as_float(v0[i]), __uint_as_float(v0[i + 1])),
                                                           make_float2(__uint_as_float(w0[i]), __uint_as_float(w0[i + 1])));
                                const float2 sa = fadd2_rn(make_float2(__uint_as_float(pv[k]), __uint_as_float(pv[k + 1])), pa);
                                acc[k] = sa.x;
                                acc[k + 1] = sa.y;
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sm.seg_empty[g]);
                    ++segs[g];
                    uint32_t rv[32];
                    if (skip) {
                        tmem_ld32(taddr + 256u + uint32_t(g) * 64u + uint32_t(col0), rv);
                        tmem_wait_ld();
                        tmem_hold(rv);
                    }
                    if (valid[g]) {
                        // The batch norm, the residual, ReLU, the tf32 split, the
                        // stores in place (the reference's separate roundings,
                        // src/cuda/kernels.cu:172-176).
                        // (the weight arena's pieces are 256-byte aligned: 16-byte loads)
                        const FusedLayer& L = stem ? *p.stem : p.layer[l];
                        const float4* sc4 = reinterpret_cast<const float4*>(L.scale + col0);
                        const float4* sh4 = reinterpret_cast<const float4*>(L.shift + col0);
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const float4 a = __ldg(sc4 + u), b = __ldg(sh4 + u);
                            float2 y01 = make_float2(__fadd_rn(__fmul_rn(a.x, acc[4 * u]), b.x),
                                                     __fadd_rn(__fmul_rn(a.y, acc[4 * u + 1]), b.y));
                            float2 y23 = make_float2(__fadd_rn(__fmul_rn(a.z, acc[4 * u + 2]), b.z),
                                                     __fadd_rn(__fmul_rn(a.w, acc[4 * u + 3]), b.w));
                            if (skip) {
                                y01 = fadd2_rn(y01, make_float2(__uint_as_float(rv[4 * u]), __uint_as_float(rv[4 * u + 1])));
                                y23 = fadd2_rn(y23, make_float2(__uint_as_float(rv[4 * u + 2]), __uint_as_float(rv[4 * u + 3])));
                            }
                            y01.x = y01.x > 0.0f ? y01.x : 0.0f;
                            y01.y = y01.y > 0.0f ? y01.y : 0.0f;
                            y23.x = y23.x > 0.0f ? y23.x : 0.0f;
                            y23.y = y23.y > 0.0f ? y23.y : 0.0f;
                            const float4 hv = make_float4(to_tf32(y01.x), to_tf32(y01.y), to_tf32(y23.x), to_tf32(y23.y));
                            const float2 l01 = fsub2_rn(y01, make_float2(hv.x, hv.y));
                            const float2 l23 = fsub2_rn(y23, make_float2(hv.z, hv.w));
                            *reinterpret_cast<float4*>(hi + swz(brow, u)) = hv;
                            *reinterpret_cast<float4*>(lo + swz(brow, u)) = make_float4(l01.x, l01.y, l23.x, l23.y);
                        }
                    }
                    fence_proxy_async_smem();   // the writes, visible to the group's next MMAs
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sm.act_ready[g]);
                    ++steps_done[g];
                }
            }
            if (!ok) break;
            // The pair's heads: each group's 1x1 convolutions once every
            // epilogue warp has written its last layer (the one-group kernel's
            // lane split and tree: the same bits); the FCs wait for the next
            // pair's steps.
            using H = HeadLane<kTF32x3, 16, 1>;
            H hl;
            hl.load(p.head, lane);
            for (int g = 0; g < ng && ok; ++g) {
                if (!(ok = mbar_wait(&sm.act_ready[g], (steps_done[g] - 1) & 1, p.err, kErrWaitEpilogue))) break;
                const int A = p.n * p.n, pts = boards[g] * A, n = p.n, S = p.S, top = p.top;
                const int first_board = (2 * P + g) * p.group;
                const size_t act_bytes = size_t(p.act_bytes), lo_off = size_t(p.nch) * act_bytes;
                const uint8_t* xbuf = sm.act[g];
                auto piece = [=](int pt, int j) {
                    const int b = pt / A, q = pt - b * A, y = q / n, xx = q - y * n;
                    const int pr = top + b * S + (y + 1) * (n + 1) + xx, c = j >> 3, u = j & 7;
                    TrunkPiece<kTF32x3> pc;
                    pc.hi = *reinterpret_cast<const uint4*>(xbuf + size_t(c) * act_bytes + swz(pr, u));
                    pc.lo = *reinterpret_cast<const uint4*>(xbuf + lo_off + size_t(c) * act_bytes + swz(pr, u));
                    return pc;
                };
                auto where = [=](int pt, int* b, int* q) {
                    *b = first_board + pt / A;
                    *q = pt % A;
                };
                for (int base = e * H::kStepRows; base < pts; base += kFusedEpiWarps * H::kStepRows)
                    hl.step(p.head, base, pts, piece, where, lane);
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.out_done[g]);   // the buffer may take the group's next input
            }
            if (!ok || !(ok = epi_sync())) break;   // the features, visible to every epilogue warp
            pend = 2 * P * p.group;
            pend_boards = boards[0] + boards[1];
            ++kin;
        }
        if (ok && pend >= 0) {   // the last pair's FCs: on the critical path, eight outputs per warp step
            const int octs = head_fc_quad_count<8>(p.head);
            for (int q = e; q < octs; q += kFusedEpiWarps)
                for (int b0 = 0; b0 < pend_boards; b0 += kFusedFcBoards) {
                    fb = pend + b0;
                    head_fc_quad<8, kFusedFcBoards>(p.head, fb, min(kFusedFcBoards, pend_boards - b0), q, xpol, xval,
                                                    hid_at, lane);
                }
            fc_finish();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kPairTmemCols);
    }
}

template <int kTps>
cudaError_t launch_pair_tps(const FusedMaps& m, const FusedArgs& a, size_t smem, int sms, cudaStream_t s) {
    if (const cudaError_t e = open_smem<tower_fused_pair<kTps>>(smem); e != cudaSuccess) return e;
    const int groups = (a.boards + a.group - 1) / a.group, pairs = (groups + 1) / 2;
    const int grid = std::max(1, std::min(pairs, sms));
    return launch_pdl(tower_fused_pair<kTps>, dim3(grid), dim3(kPairThreads), smem, s, m.in, m.in_lo, m.stem,
                      m.stem_lo, a);
}

// Shared memory of a pair launch (0 when it does not fit): both groups'
// buffers, then as many weight stages as the room left allows (two at least).
size_t fused_pair_smem(int nch, int act_bytes, int /*layers*/, int* stages, int taps_per_stage) {
    const size_t acts = 2 * 2 * size_t(nch) * act_bytes;
    const size_t stage = size_t(taps_per_stage) * 2 * 64 * 128;
    for (int st = 8; st >= 2; --st) {
        const size_t total = 1024 + acts + st * stage + (2 * st + 13) * 8 + 16;
        if (total <= 227 * 1024) {
            if (stages) *stages = st;
            return total;
        }
    }
    return 0;
}

// The pair kernel where it applies (the split mode at two input chunks,
// heads in the launch) and pays: a pair costs ~1.7 one group's time on an SM
// (measured: both groups' MMAs share the SM's shared-memory operand reads,
// which bound a layer's MMA phase; what overlaps is the epilogue), so pairs
// run only where they save rounds of CTAs: 9x9 at 256 boards (two rounds of
// one group, one of pairs) 184 -> 160 us; at 148 boards 103 against 163 us,
// at 300 and 444 267 against 306 us, at 600 434 against 452 us, at 1024 601
// against 596 us (within the noise; one group). Three taps per stage where
// two such stages fit, else one.
cudaError_t launch_fused_pairs(const FusedMaps& m, FusedArgs a, int sms, cudaStream_t s, bool* launched) {
    *launched = false;
    if (!a.pairs || !a.heads || a.nch != 2) return cudaSuccess;
    const int groups = (a.boards + a.group - 1) / a.group;
    const int rounds = (groups + sms - 1) / sms, pair_rounds = ((groups + 1) / 2 + sms - 1) / sms;
    if (a.pairs == 1 && 10 * rounds <= 18 * pair_rounds) return cudaSuccess;
    for (int tps : {3, 1}) {
        const size_t smem = fused_pair_smem(a.nch, a.act_bytes, a.layers, &a.stages, tps);
        if (smem == 0) continue;
        *launched = true;
        return tps == 3 ? launch_pair_tps<3>(m, a, smem, sms, s) : launch_pair_tps<1>(m, a, smem, sms, s);
    }
    return cudaSuccess;
}

template <int N, bool kBf16, bool kSplit, int kTps>
cudaError_t launch_fused_tps(const FusedMaps& m, const FusedArgs& a, size_t smem, int ctas, int sms, cudaStream_t s) {
    if (const cudaError_t e = open_smem<tower_fused<N, kBf16, kSplit, kTps>>(smem); e != cudaSuccess) return e;
    const int groups = (a.boards + a.group - 1) / a.group;
    const int grid = std::max(1, std::min(groups, sms * ctas));
    return launch_pdl(tower_fused<N, kBf16, kSplit, kTps>, dim3(grid), dim3(kFusedThreads<kSplit>), smem, s, m.in, m.in_lo,
                      m.out, m.out_lo, m.stem, m.stem_lo, a);
}

// The shared-memory plan: two CTAs per SM where the configuration allows
// it, then three taps per ring stage, each with at least two stages.
template <int N, bool kBf16, bool kSplit>
cudaError_t launch_fused_one(const FusedMaps& m, FusedArgs a, int sms, cudaStream_t s) {
    if constexpr (kSplit && N == 64) {
        bool launched = false;
        const cudaError_t e = launch_fused_pairs(m, a, sms, s, &launched);
        if (launched || e != cudaSuccess) return e;
    }
    const int precision = kBf16 ? kBF16 : (kSplit ? kTF32x3 : kTF32);
    for (int ctas = kFusedCtas<kSplit>; ctas >= 1; --ctas)
        for (int tps : {3, 1}) {
            const size_t smem = fused_tower_smem(N, precision, a.nch, a.act_bytes, a.layers, &a.stages, ctas, tps);
            if (smem == 0) continue;
            return tps == 3 ? launch_fused_tps<N, kBf16, kSplit, 3>(m, a, smem, ctas, sms, s)
                            : launch_fused_tps<N, kBf16, kSplit, 1>(m, a, smem, ctas, sms, s);
        }
    return cudaErrorInvalidValue;
}

} // namespace

size_t fused_tower_smem(int n_out, int precision, int nch, int act_bytes, int layers, int* stages, int ctas,
                        int taps_per_stage) {
    const int ops = precision == kTF32x3 ? 2 : 1;
    const size_t acts = size_t(fused_act_bufs(precision == kTF32x3)) * ops * nch * act_bytes;
    const size_t stage = size_t(taps_per_stage) * ops * n_out * 128;
    const size_t bn = size_t(layers + 1) * 2 * n_out * 4;   // the tower's convs and the stem
    // An SM's 228 KB, less 1 KB reserved per CTA, shared by `ctas` CTAs.
    const size_t kMax = ctas > 1 ? (228 * 1024) / size_t(ctas) - 1024 : 227 * 1024;
    for (int st = 8; st >= 2; --st) {
        const size_t total = 1024 + acts + st * stage + bn + (2 * st + 6) * 8 + 16;
        if (total <= kMax) {
            if (stages) *stages = st;
            return total;
        }
    }
    return 0;
}

cudaError_t launch_fused_tower(const FusedMaps& m, const FusedArgs& a, int n_out, int precision, int sms,
                               cudaStream_t s) {
    if (a.boards <= 0 || a.layers <= 0) return cudaSuccess;
    switch (precision) {
        case kBF16:
            return n_out == 32 ? launch_fused_one<32, true, false>(m, a, sms, s)
                               : n_out == 64 ? launch_fused_one<64, true, false>(m, a, sms, s) : cudaErrorInvalidValue;
        case kTF32:
            return n_out == 32 ? launch_fused_one<32, false, false>(m, a, sms, s)
                               : n_out == 64 ? launch_fused_one<64, false, false>(m, a, sms, s) : cudaErrorInvalidValue;
        case kTF32x3:
            return n_out == 32 ? launch_fused_one<32, false, true>(m, a, sms, s)
                               : n_out == 64 ? launch_fused_one<64, false, true>(m, a, sms, s) : cudaErrorInvalidValue;
        default: return cudaErrorInvalidValue;
    }
}

} // namespace azb
