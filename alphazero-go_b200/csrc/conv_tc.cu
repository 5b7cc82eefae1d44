// The fused 3x3 convolution on the tcgen05 tensor cores: an implicit GEMM
// with no im2col buffer.
//
//   D[q][co] = sum over (chunk c, tap t, channel i) of X[q + off(t)][c*KC + i] * W[co][(c*9 + t)*KC + i]
//   out[q][co] = ReLU(scale[co] * D[q][co] + shift[co] (+ skip[q][co]))
//
// q runs over frame rows (kernels.hpp), so a tap is a constant row offset
// off(t) = dy*(n+1) + dx. One CTA owns a 128-row tile of q at a time
// (persistent over tiles). For each 128-byte channel chunk, TMA stages ONE
// "halo" tile of 128 + 2(n+2) rows; the nine taps are nine row-shifted
// views of it, addressed by moving the start of the MMA's shared-memory
// descriptor (the halo is read from L2 once per chunk, not nine times). The
// weights of each (chunk, tap) arrive as an N x 128-byte TMA tile. Both use
// the 128-byte swizzle. The accumulator lives in TMEM, double-buffered, so
// the epilogue of one tile overlaps the MMAs of the next.
//
// Warp roles (320 threads): warp 0 issues TMA, warp 1 issues tcgen05.mma,
// warps 2-9 run the epilogue (TMEM -> registers -> BN, skip, ReLU -> HBM),
// two warps per TMEM lane quarter, each on half of the columns.
//
// Replaces the reference's SIMT gemm_tiled<..., Op::Conv> and
// launchConvBnRelu (src/cuda/kernels.cu:82-180, 215-224): same epilogue
// arithmetic (scale*acc + shift rounded separately, + skip, x > 0 ? x : 0),
// tensor-core accumulation instead of one fmaf chain per output.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <type_traits>

#include "kernels.hpp"
#include "sm100.cuh"

namespace azb {

namespace {

constexpr int kEpiWarps = 8;   // epilogue warps per CTA

template <int N, bool kBf16, bool kSplit, int kTiles = 1>
struct ConvCfg {
    static constexpr int kEsz = kBf16 ? 2 : 4;
    static constexpr int kKc = 128 / kEsz;          // channels per 128-byte chunk
    static constexpr int kKstep = kBf16 ? 16 : 8;   // K of one MMA (32 bytes)
    static constexpr int kSteps = kKc / kKstep;     // MMAs per chunk and tap
    static constexpr int kOps = kSplit ? 2 : 1;     // operand planes per stage
    static constexpr uint32_t kBBytes = uint32_t(N) * 128u;
    // The split mode at N <= 128 stacks the weight tile's two planes into one
    // N' = 2N operand (they are adjacent in shared memory): one MMA computes
    // a_hi.b_hi into columns [0, N) and a_hi.b_lo into [N, 2N), a second adds
    // a_lo.b_hi into [N, 2N); the epilogue adds the halves. Two instructions
    // per K step instead of three, for narrow layers whose MMAs are too
    // short for one thread to issue three back to back; and the large
    // products accumulate alone, in segments (kSeg).
    static constexpr bool kStack = kSplit && N <= 128 && 2 * kTiles * 2 * N <= 512;
    static constexpr int kTileCols = kStack ? 2 * N : N;   // TMEM columns of one tile's accumulator
    // Two accumulators (double buffering) of kTiles tiles each.
    static constexpr int kAccCols = 2 * kTiles * kTileCols;
    static constexpr uint32_t kTmemCols = kAccCols <= 64 ? 64 : (kAccCols <= 128 ? 128 : (kAccCols <= 256 ? 256 : 512));
    static_assert(kAccCols <= 512, "the accumulators fit in TMEM's 512 columns");
    static constexpr uint32_t kIdesc = umma_idesc(N, kBf16);
    // bf16 and plain tf32 store their output (and read their residual input)
    // through shared memory with TMA, in boxes of {32 channels, 32 rows}: one
    // output and one residual box per epilogue warp, 2 KB each (bf16) or 4 KB
    // (fp32). The stacked split mode stores its two planes through one 4 KB
    // box per warp (the residual read directly); the unstacked one stores
    // directly.
    static constexpr bool kEpiTma = !kSplit;
    static constexpr uint32_t kEpiBytes =
        kEpiTma ? uint32_t(kEpiWarps) * (kBf16 ? 4096u : 8192u) : (kStack ? uint32_t(kEpiWarps) * 4096u : 0u);
    static_assert(N % 32 == 0 && N >= 32 && N <= 256, "N is a multiple of 32 in [32, 256]");
};

// The persistent tower's parameters; nothing for the per-layer launches.
struct NoTower {};
template <bool kPersist>
using TowerOf = std::conditional_t<kPersist, TowerArgs, NoTower>;

constexpr int kThreads = 320;   // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
// The two-tile form adds warp 10, which issues the second tile's MMAs: one
// thread issues an MMA about every 61 cycles, no faster than the tensor core
// finishes an M = 128, N = 128 bf16 one (64 cycles), so with one issuing
// thread narrow layers wait on the issue. The two tiles' accumulators are
// disjoint TMEM columns; each thread commits its own MMAs, so the barriers
// they commit to take one arrival per issuing thread.
template <int kTiles>
constexpr int kIssuersOf = kTiles == 2 ? 2 : 1;
template <int kTiles>
constexpr int kThreadsOf = kThreads + 32 * (kIssuersOf<kTiles> - 1);
constexpr int kMaxStages = 8;
constexpr uint32_t kBnBytes = 2 * 256 * 4;   // scale and shift of up to 256 channels

// Shared memory: [halo buffers][weight buffers][barriers][tmem slot].
struct Smem {
    uint8_t* a;
    uint8_t* b;
    uint8_t* epi;   // bf16 epilogue boxes (4 warps x 8 KB), or nothing
    float* bn;      // the folded batch norm: scale[0..N), shift[N..2N)
    uint64_t *a_full, *a_empty, *b_full, *b_empty, *acc_full, *acc_empty, *done;
    uint64_t* skip_full;   // 8 epilogue warps x 2 residual boxes
    uint32_t* tmem_slot;
};

// a_ops halo buffers per A stage (operand planes x tiles), b_ops weight
// buffers per B stage (operand planes).
__device__ __forceinline__ Smem carve(uint8_t* raw, int sa, int sb, int a_ops, int b_ops, int a_bytes,
                                      uint32_t b_bytes, uint32_t epi_bytes) {
    Smem s;
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    s.a = base;
    s.b = base + size_t(sa) * a_ops * a_bytes;
    s.epi = s.b + size_t(sb) * b_ops * b_bytes;
    s.bn = reinterpret_cast<float*>(s.epi + epi_bytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(s.epi + epi_bytes + kBnBytes);
    s.a_full = bars;
    s.a_empty = s.a_full + sa;
    s.b_full = s.a_empty + sa;
    s.b_empty = s.b_full + sb;
    s.acc_full = s.b_empty + sb;
    s.acc_empty = s.acc_full + 2;
    s.done = s.acc_empty + 2;
    s.skip_full = s.done + 1;
    s.tmem_slot = reinterpret_cast<uint32_t*>(s.skip_full + 2 * kEpiWarps);
    return s;
}

__host__ __device__ constexpr size_t smem_total(int sa, int sb, int a_ops, int b_ops, int a_bytes, uint32_t b_bytes,
                                                uint32_t epi_bytes) {
    return 1024 + size_t(sa) * a_ops * a_bytes + size_t(sb) * b_ops * b_bytes + epi_bytes + kBnBytes +
           (2 * sa + 2 * sb + 5 + 2 * kEpiWarps) * 8 + 16;
}

// The nine tap views' start rows inside a halo tile, as descriptor
// increments (16-byte units): halo row n+2 + dy(n+1) + dx is frame row
// q0 + dy(n+1) + dx. A one-tap pass (the stem GEMM) uses the centre view.
__device__ __forceinline__ void tap_offsets(const ConvArgs& p, uint32_t (&off)[9]) {
#pragma unroll
    for (int t = 0; t < 9; ++t) {
        const int tap = p.taps == 9 ? t : 4;
        off[t] = uint32_t(p.n + 2 + (tap / 3 - 1) * (p.n + 1) + (tap % 3 - 1)) * 8u;
    }
}

// One output element of the split mode from its accumulated sum:
// ReLU(scale * acc + shift (+ skip)) with the reference's separate roundings
// (src/cuda/kernels.cu:172-176), the skip given as its two planes.
__device__ __forceinline__ float split_out(float acc, float scale, float shift, bool skip, float s_hi, float s_lo) {
    float y = __fadd_rn(__fmul_rn(scale, acc), shift);
    if (skip) y = __fadd_rn(y, __fadd_rn(s_hi, s_lo));
    return y > 0.0f ? y : 0.0f;
}

// Stores 32 consecutive channels of one row as the tf32 high part (cvt.rna)
// and the exact low remainder.
__device__ __forceinline__ void store_split_planes(float* hi_dst, float* lo_dst, const float (&y)[32]) {
    float4* dst = reinterpret_cast<float4*>(hi_dst);
    float4* dlo = reinterpret_cast<float4*>(lo_dst);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        float4 h, l;
        h.x = to_tf32(y[4 * u]);     l.x = __fsub_rn(y[4 * u], h.x);
        h.y = to_tf32(y[4 * u + 1]); l.y = __fsub_rn(y[4 * u + 1], h.y);
        h.z = to_tf32(y[4 * u + 2]); l.z = __fsub_rn(y[4 * u + 2], h.z);
        h.w = to_tf32(y[4 * u + 3]); l.w = __fsub_rn(y[4 * u + 3], h.w);
        dst[u] = h;
        dlo[u] = l;
    }
}

// The stacked split mode accumulates a tile in segments (tcgen05's fp32
// accumulation rounds toward zero at every MMA, so a long run on one
// accumulator drifts toward zero; short runs summed in round-to-nearest
// keep the sum within a few fp32 roundings). An epilogue thread adds one
// segment's two halves ([0, N) the large products, [N, 2N) the small ones)
// of its row's kMine 32-column chunks from c_begin into its running sums.
// With more than one chunk the halves go 16 columns at a time: the running
// sums of all the chunks stay live, so two 32-column loads beside them
// would not fit in the registers.
template <int N, int kMine>
__device__ __forceinline__ void add_segment(uint32_t taddr, int c_begin, float (&sum)[kMine * 32], bool first) {
    constexpr int kCols = kMine > 1 ? 16 : 32;
#pragma unroll
    for (int cc = 0; cc < kMine; ++cc) {
#pragma unroll
        for (int h = 0; h < 32; h += kCols) {
            uint32_t v[kCols], w[kCols];
            const uint32_t col = uint32_t(c_begin + cc) * 32u + uint32_t(h);
            if constexpr (kCols == 32) {
                tmem_ld32(taddr + col, v);
                tmem_ld32(taddr + uint32_t(N) + col, w);
            } else {
                tmem_ld16(taddr + col, v);
                tmem_ld16(taddr + uint32_t(N) + col, w);
            }
            tmem_wait_ld();
            tmem_hold(v);
            tmem_hold(w);
#pragma unroll
            for (int i = 0; i < kCols; i += 2) {   // paired: half the instructions on this SM's issue slots
                const int k = cc * 32 + h + i;
                const float2 part = fadd2_rn(make_float2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])),
                                             make_float2(__uint_as_float(w[i]), __uint_as_float(w[i + 1])));
                const float2 s2 = first ? part : fadd2_rn(make_float2(sum[k], sum[k + 1]), part);
                sum[k] = s2.x;
                sum[k + 1] = s2.y;
            }
        }
    }
}

// One epilogue thread's accumulator row (TMEM lane of its warp) for a tile in
// the unstacked split mode (one accumulator run per tile), for the 32-column
// chunks [c_begin, c_end). The row's residual (both planes) is requested
// before the TMEM load so the two latencies overlap; the folded batch norm
// comes from shared memory. Padding rows (valid false) read TMEM (the load is
// warp-collective) and store nothing.
template <int N>
__device__ __forceinline__ void store_epilogue_split(const ConvArgs& p, const float* bn, uint32_t taddr, int q,
                                                     bool valid, int c_begin, int c_end) {
#pragma unroll 1
    for (int c0 = c_begin * 32; c0 < c_end * 32; c0 += 32) {
        const size_t off = size_t(q) * p.ld + c0;
        float4 sk[8], sl[8];
        const bool skip = valid && p.skip != nullptr;
        if (skip) {
            const float4* hi = reinterpret_cast<const float4*>(static_cast<const float*>(p.skip) + off);
            const float4* lo = reinterpret_cast<const float4*>(static_cast<const float*>(p.skip_lo) + off);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                sk[u] = hi[u];
                sl[u] = lo[u];
            }
        }
        uint32_t v[32];
        tmem_ld32(taddr + c0, v);
        tmem_wait_ld();
        if (!valid) continue;
        float y[32];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const float* h = &sk[u].x;
            const float* l = &sl[u].x;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = 4 * u + e;
                y[i] = split_out(__uint_as_float(v[i]), bn[c0 + i], bn[N + c0 + i], skip, skip ? h[e] : 0.0f,
                                 skip ? l[e] : 0.0f);
            }
        }
        store_split_planes(static_cast<float*>(p.out) + off, static_cast<float*>(p.out_lo) + off, y);
    }
}

// One epilogue warp's share of a tile (32 rows from row0, all N channels),
// through shared memory: per 32-channel chunk the warp's lanes (one row
// each) write ReLU(scale * acc + shift (+ skip)) into a box of 32 rows x 32
// channels (bf16: 64-byte rows, 2 KB; fp32: 128-byte rows, 4 KB), swizzled
// as TMA's 64-byte / 128-byte swizzle lays it out (16-byte piece u of row r
// at piece u ^ ((r >> 1) & 3), resp. u ^ (r & 7): conflict-free), and one
// lane stores the box with TMA. Padding rows are stored as zeros (they must
// stay zero), rows past the frame are clipped by TMA. The residual input
// arrives the same way, one chunk ahead, in two boxes. Same arithmetic as
// store_epilogue.
// What an epilogue item reads and writes besides its accumulator: the
// folded batch norm, the residual (null: none), the output's boxes (split:
// its high plane) and the residual's boxes (stacked split: the output's low
// plane).
struct ItemIo {
    const float* scale;
    const float* shift;
    const void* res_hi;
    const void* res_lo;
    const CUtensorMap* omap;
    const CUtensorMap* smap;
};

struct EpiWarp {
    uint8_t* obuf;        // 2 output boxes
    uint8_t* sbuf;        // 2 residual boxes
    uint64_t* sbar;       // their 2 barriers
    uint32_t sphase = 0;  // bit i: parity of sbar[i]'s next phase
};

template <bool kBf16>
struct EpiBox {
    static constexpr uint32_t kRowBytes = kBf16 ? 64u : 128u;
    static constexpr uint32_t kBytes = 32u * kRowBytes;
    static constexpr int kBufs = 1;                        // output (and residual) boxes per warp
    static constexpr int kPieces = int(kRowBytes / 16);   // 16-byte pieces per row
    __device__ static uint32_t piece(int row, int u) {     // byte offset of piece u of `row`
        const uint32_t sw = kBf16 ? uint32_t((row >> 1) & 3) : uint32_t(row & 7);
        return uint32_t(row) * kRowBytes + ((uint32_t(u) ^ sw) << 4);
    }
};

// This warp's 32-column chunks [c_begin, c_end) of its 32 rows. With one
// box per role (kBufs 1, as built) the next chunk's residual is requested as
// soon as this chunk's has been read, and the output box is refilled once
// the previous store has read it; with two, one chunk ahead and two behind.
// kOwnShift: the shift is its own array (the persistent tower's layer
// table); otherwise it follows the scale (shared memory, shift at N).
template <int N, bool kBf16, bool kOwnShift = false>
__device__ __forceinline__ void store_epilogue_tma(const ConvArgs& p, const float* scale, const float* shift,
                                                   const void* res, const CUtensorMap* omap, const CUtensorMap* smap,
                                                   uint32_t taddr, int row0, bool valid, int c_begin, int c_end,
                                                   EpiWarp& ew, int lane) {
    using Box = EpiBox<kBf16>;
    constexpr uint32_t kBox = Box::kBytes;
    if (row0 >= p.rows || c_begin >= c_end) return;   // nothing of this warp's to store
    const bool skip = res != nullptr;   // the residual, read through smap
    if (skip && lane == 0) {
        mbar_arrive_expect_tx(&ew.sbar[0], kBox);
        tma_load_2d(smap, ew.sbuf, &ew.sbar[0], c_begin * 32, row0);
    }
#pragma unroll 1
    for (int c = c_begin; c < c_end; ++c) {
        const int cb = Box::kBufs == 2 ? ((c - c_begin) & 1) : 0;
        if (Box::kBufs == 2 && skip && c + 1 < c_end && lane == 0) {   // the other box was last read in chunk c-1
            mbar_arrive_expect_tx(&ew.sbar[cb ^ 1], kBox);
            tma_load_2d(smap, ew.sbuf + (cb ^ 1) * kBox, &ew.sbar[cb ^ 1], (c + 1) * 32, row0);
        }
        uint32_t v[32];
        tmem_ld32(taddr + uint32_t(c) * 32u, v);
        tmem_wait_ld();
        float y[32];
#pragma unroll
        for (int i = 0; i < 32; ++i)
            y[i] = __fadd_rn(__fmul_rn(scale[c * 32 + i], __uint_as_float(v[i])),
                             kOwnShift ? shift[c * 32 + i] : scale[N + c * 32 + i]);
        if (skip) {
            mbar_wait(&ew.sbar[cb], (ew.sphase >> cb) & 1u, p.err, kErrWaitEpilogue);
            ew.sphase ^= 1u << cb;
            const uint8_t* box = ew.sbuf + cb * kBox;
#pragma unroll
            for (int u = 0; u < Box::kPieces; ++u) {
                const uint4 w4 = *reinterpret_cast<const uint4*>(box + Box::piece(lane, u));
                if constexpr (kBf16) {
                    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w4);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __bfloat1622float2(h2[e]);
                        y[u * 8 + 2 * e] = __fadd_rn(y[u * 8 + 2 * e], f.x);
                        y[u * 8 + 2 * e + 1] = __fadd_rn(y[u * 8 + 2 * e + 1], f.y);
                    }
                } else {
                    const float* f = reinterpret_cast<const float*>(&w4);
#pragma unroll
                    for (int e = 0; e < 4; ++e) y[u * 4 + e] = __fadd_rn(y[u * 4 + e], f[e]);
                }
            }
            if (Box::kBufs == 1 && c + 1 < c_end) {   // the box is read: request the next chunk's residual
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive_expect_tx(&ew.sbar[0], kBox);
                    tma_load_2d(smap, ew.sbuf, &ew.sbar[0], (c + 1) * 32, row0);
                }
            }
        }
        uint4 out[Box::kPieces];
#pragma unroll
        for (int u = 0; u < Box::kPieces; ++u) {
            if constexpr (kBf16) {
                __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&out[u]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float a0 = y[u * 8 + 2 * e], a1 = y[u * 8 + 2 * e + 1];
                    h2[e] = valid ? __floats2bfloat162_rn(a0 > 0.0f ? a0 : 0.0f, a1 > 0.0f ? a1 : 0.0f)
                                  : __floats2bfloat162_rn(0.0f, 0.0f);
                }
            } else {
                float* f = reinterpret_cast<float*>(&out[u]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float a = y[u * 4 + e];
                    f[e] = valid && a > 0.0f ? a : 0.0f;
                }
            }
        }
        // The store issued from this box kBufs chunks ago has read it.
        if (lane == 0) {
            if constexpr (Box::kBufs == 2) bulk_wait_read<1>();
            else bulk_wait_read<0>();
        }
        __syncwarp();
        uint8_t* obox = ew.obuf + cb * kBox;
#pragma unroll
        for (int u = 0; u < Box::kPieces; ++u) *reinterpret_cast<uint4*>(obox + Box::piece(lane, u)) = out[u];
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_2d(omap, obox, c * 32, row0);
            bulk_commit();
        }
    }
}

// The stacked split mode's store from the running sums (this thread's row
// q, chunks [c_begin, c_begin + kMine)) through shared memory and TMA: per
// 32-channel chunk the warp writes the high plane into its 4 KB box (32 rows
// x 128 bytes, laid out as the 128-byte swizzle) and stores it with TMA,
// then the low plane the same way once the box has been read. The residual
// is read directly (it was prefetched into L2 at the tile's start). Padding
// rows are stored as zeros (they must stay zero); rows past the frame are
// clipped by TMA.
template <int N, int kMine>
__device__ __forceinline__ void store_split_sums(const ConvArgs& p, const float* scale, const float* shift,
                                                 const void* res_hi, const void* res_lo, float (&sum)[kMine * 32],
                                                 const CUtensorMap* mhi, const CUtensorMap* mlo, uint8_t* box,
                                                 int row0, int q, bool valid, int c_begin, int lane, int col0 = 0) {
    using Box = EpiBox<false>;
    if (row0 >= p.rows) return;   // the warp's rows are all past the frame
    const bool skip = valid && res_hi != nullptr;
#pragma unroll
    for (int cc = 0; cc < kMine; ++cc) {
        const int c0 = (c_begin + cc) * 32;
        const size_t off = size_t(q) * p.ld + c0;
        const float4* hi = reinterpret_cast<const float4*>(static_cast<const float*>(res_hi) + off);
        const float4* lo = reinterpret_cast<const float4*>(static_cast<const float*>(res_lo) + off);
        // The chunk's outputs replace its sums (no second 32-float array live
        // beside the sums and the residual).
        float* y = &sum[cc * 32];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            float4 h4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), l4 = h4;
            if (skip) {
                h4 = hi[u];
                l4 = lo[u];
            }
            const float* h = &h4.x;
            const float* l = &l4.x;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = 4 * u + e;
                y[i] = valid ? split_out(y[i], scale[c0 + i], shift[c0 + i], skip, h[e], l[e]) : 0.0f;
            }
        }
#pragma unroll
        for (int plane = 0; plane < 2; ++plane) {
            float4 out[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                float* f = &out[u].x;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float v = y[4 * u + e], h = to_tf32(v);
                    f[e] = plane == 0 ? h : __fsub_rn(v, h);
                }
            }
            if (lane == 0) bulk_wait_read<0>();   // the box's previous store has read it
            __syncwarp();
#pragma unroll
            for (int u = 0; u < 8; ++u) *reinterpret_cast<float4*>(box + Box::piece(lane, u)) = out[u];
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(plane == 0 ? mhi : mlo, box, col0 + c0, row0);
                bulk_commit();
            }
        }
    }
}

// kSeg: the stacked split mode's accumulation segment in taps (0: one run
// per tile). mOut/mSkip: the epilogue's output and residual boxes; in the
// stacked split mode the high and low output planes.
//
// kWide: the stacked split mode for a layer of 2N output channels, as two
// column halves of N: item it is tile group it / 2 and output channels
// [(it % 2) N, (it % 2 + 1) N). Each item loads its half's weight rows (mW
// and mWlo in boxes of N rows), reads its half of the batch norm (scale and
// shift of all 2N channels in shared memory) and of the residual, and
// stores its half of the output. The two halves of a tile are consecutive
// items, so the second finds the halo in L2. This keeps 256-channel layers
// in the segmented accumulation (each segment's large products on their own
// accumulator, summed in round-to-nearest), which one 256-column
// accumulator per tile cannot hold beside its running sums.
//
// kPersist: the persistent tower (bf16 and tf32; the stacked split mode in
// its segments). Items are (layer, tile group) = (it / ngroups, it %
// ngroups); the producer takes the pass's next item from a global counter
// and hands its index to the MMA and epilogue warps through a shared-memory
// ring. Every item's dependencies have lower indices and were therefore
// taken by CTAs already running, so the tower progresses however many of
// its CTAs are resident (another stream's kernels may hold SMs, a second
// tower among them). The frames come from tf (the six map parameters are
// then unused), the weights and batch norms from tf.tower. With
// tf.stem_first, layer 0 is the stem: one tap (the centre view) over the
// stem's packed operand, tf.stem_nchunks chunks. Each
// epilogue warp adds 1 to its item's counter once its stores have landed;
// an item's halo loads wait until the counters of the previous layer's
// groups g-1, g, g+1 (the rows its halo reads) have reached kEpiWarps.
// Writes need no wait of their own: the buffer an item overwrites was last
// read by items that those same dependencies already include.
template <int N, bool kBf16, bool kSplit, int kTiles, int kSeg, bool kPersist = false, bool kWide = false>
__global__ void __launch_bounds__(kThreadsOf<kTiles>, 1)
    conv3x3_tc(const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mAlo,
               const __grid_constant__ CUtensorMap mW, const __grid_constant__ CUtensorMap mWlo,
               const __grid_constant__ CUtensorMap mOut, const __grid_constant__ CUtensorMap mSkip, const ConvArgs p,
               const __grid_constant__ TowerOf<kPersist> tf) {
    using C = ConvCfg<N, kBf16, kSplit, kTiles>;
    static_assert(!kPersist || (!kSplit && kSeg == 0) || (C::kStack && kSeg != 0 && kTiles == 1),
                  "the persistent tower: bf16 and tf32, or the split mode's segmented single tiles");
    static_assert(!kWide || (C::kStack && kSeg != 0 && kTiles == 1 && !kPersist && 2 * N <= 256),
                  "column halves: the stacked split mode's segmented single tiles, per layer");
    constexpr int kBnCh = kWide ? 2 * N : N;   // batch-norm channels in shared memory (shift at kBnCh)
    extern __shared__ uint8_t smem_raw[];
    const Smem sm = carve(smem_raw, p.sa, p.sb, C::kOps * kTiles, C::kOps, p.a_bytes, C::kBBytes, C::kEpiBytes);
    const int ngroups = (p.ntiles + kTiles - 1) / kTiles;   // a CTA takes kTiles consecutive tiles at a time
    int nitems = ngroups;
    if constexpr (kPersist) nitems = tf.layers * ngroups;
    if constexpr (kWide) nitems = 2 * ngroups;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // The persistent tower's item ring lives where the batch norm would (its
    // batch norms are read from tf.tower): kItemSlots full and empty barriers,
    // then the slots' item indices (-1: no more items).
    constexpr int kItemSlots = 4;
    uint64_t* item_full = reinterpret_cast<uint64_t*>(sm.bn);
    uint64_t* item_empty = item_full + kItemSlots;
    volatile int* item_slot = reinterpret_cast<volatile int*>(item_empty + kItemSlots);
    constexpr int kIssuers = kIssuersOf<kTiles>;   // MMA-issuing threads: warp 1 (and warp 10)

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.sa; ++i) {
            mbar_init(&sm.a_full[i], 1);
            mbar_init(&sm.a_empty[i], kIssuers);
        }
        for (int i = 0; i < p.sb; ++i) {
            mbar_init(&sm.b_full[i], 1);
            mbar_init(&sm.b_empty[i], kIssuers);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.acc_full[i], kIssuers);
            mbar_init(&sm.acc_empty[i], kEpiWarps);   // one arrival per epilogue warp
        }
        mbar_init(sm.done, kIssuers);
        for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&sm.skip_full[i], 1);
        if (kPersist)
            for (int i = 0; i < kItemSlots; ++i) {
                mbar_init(&item_full[i], 1);
                mbar_init(&item_empty[i], kIssuers + kEpiWarps);   // every MMA issuer and epilogue warp reads it
            }
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&mA);
        tma_prefetch_map(&mW);
        if (C::kEpiTma || C::kStack) {
            tma_prefetch_map(&mOut);
            tma_prefetch_map(&mSkip);
        }
        if (kSplit) {
            tma_prefetch_map(&mAlo);
            tma_prefetch_map(&mWlo);
        }
    }
    if (warp == 1) tmem_alloc(sm.tmem_slot, C::kTmemCols);
    if (!kPersist)
        for (int i = threadIdx.x; i < kBnCh; i += kThreadsOf<kTiles>) {
            sm.bn[i] = p.scale[i];
            sm.bn[kBnCh + i] = p.shift[i];
        }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *sm.tmem_slot;
    // Set-up (barriers, TMEM, batch norm, descriptor prefetch) overlapped the
    // previous kernel's tail; its activations are read only from here on.
    grid_dependency_wait();
    grid_launch_dependents();

    if (warp == 0) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            Ring ra, rb;
            uint32_t na = 0, nb = 0;   // loads issued, for the drain below
            const uint32_t a_tx = uint32_t(p.halo_rows) * 128u * C::kOps * kTiles;
            const uint32_t b_tx = C::kBBytes * C::kOps;
            const size_t a_stage = size_t(C::kOps) * kTiles * p.a_bytes;
            bool ok = true;
            Ring ri;
            for (int k = 0; ok; ++k) {
                int it = blockIdx.x + k * int(gridDim.x);
                if constexpr (kPersist) {   // take the pass's next item and hand it on
                    it = int(atomicAdd(tf.flags + size_t(tf.layers) * ngroups, 1u));
                    if (!(ok = mbar_wait(&item_empty[ri.idx], ri.phase ^ 1u, p.err, kErrWaitProducer))) break;
                    item_slot[ri.idx] = it < nitems ? it : -1;
                    mbar_arrive(&item_full[ri.idx]);
                    ri.next(kItemSlots);
                }
                if (it >= nitems) break;
                int g = it, taps = p.taps, nchunks = p.nchunks, wrow = 0;
                if constexpr (kWide) {   // a tile group's column half: its weight rows
                    g = it >> 1;
                    wrow = (it & 1) * N;
                }
                const CUtensorMap* amap = &mA;
                const CUtensorMap* alo = &mAlo;
                const CUtensorMap* wmap = &mW;
                const CUtensorMap* wlo = &mWlo;
                if constexpr (kPersist) {
                    const int layer = it / ngroups;
                    g = it - layer * ngroups;
                    const int conv = layer - tf.stem_first;   // the tower conv; -1: the stem
                    if (conv < 0) {   // the stem: one tap over its packed operand
                        amap = &tf.stem;
                        alo = &tf.stem_lo;
                        taps = 1;
                        nchunks = tf.stem_nchunks;
                    } else {
                        const int in = conv % 3;   // tower conv l reads buffer l mod 3
                        amap = &tf.in[in];
                        alo = &tf.in_lo[in];
                    }
                    const FusedLayer& fl = tf.tower[conv < 0 ? tf.layers - 1 : conv];
                    wmap = &fl.w;
                    wlo = &fl.w_lo;
                    if (layer > 0) {   // the previous layer's groups whose rows this item's halos read
                        const unsigned* prev = tf.flags + size_t(layer - 1) * ngroups;
                        for (int d = g > 0 ? g - 1 : 0; d <= g + 1 && d < ngroups && ok; ++d)
                            ok = flag_wait(prev + d, kEpiWarps + tf.flag_extra, p.err, kErrWaitLayer);
                        if (!ok) break;
                        fence_proxy_async_global();   // the loads below (async proxy) after the acquires
                    }
                }
                for (int c = 0; c < nchunks && ok; ++c) {
                    if (!(ok = mbar_wait(&sm.a_empty[ra.idx], ra.phase ^ 1u, p.err, kErrWaitProducer))) break;
                    mbar_arrive_expect_tx(&sm.a_full[ra.idx], a_tx);
#pragma unroll
                    for (int u = 0; u < kTiles; ++u) {   // each tile's own halo (a tile past the frame reads zeros)
                        const int y0 = (g * kTiles + u) * 128 - (p.n + 2);
                        uint8_t* abuf = sm.a + ra.idx * a_stage + size_t(u) * C::kOps * p.a_bytes;
                        tma_load_2d(amap, abuf, &sm.a_full[ra.idx], c * C::kKc, y0);
                        if (kSplit) tma_load_2d(alo, abuf + p.a_bytes, &sm.a_full[ra.idx], c * C::kKc, y0);
                    }
                    ra.next(p.sa);
                    ++na;
                    for (int t = 0; t < taps; ++t) {
                        if (!(ok = mbar_wait(&sm.b_empty[rb.idx], rb.phase ^ 1u, p.err, kErrWaitProducer))) break;
                        mbar_arrive_expect_tx(&sm.b_full[rb.idx], b_tx);
                        uint8_t* bbuf = sm.b + rb.idx * (C::kOps * C::kBBytes);
                        tma_load_2d(wmap, bbuf, &sm.b_full[rb.idx], (c * taps + t) * C::kKc, wrow);
                        if (kSplit)
                            tma_load_2d(wlo, bbuf + C::kBBytes, &sm.b_full[rb.idx], (c * taps + t) * C::kKc, wrow);
                        rb.next(p.sb);
                        ++nb;
                    }
                }
            }
            // Every copy this thread issued has landed before the CTA may exit:
            // wait (bounded) for each stage's most recent load.
            for (uint32_t s = 0; s < uint32_t(p.sa) && s < na; ++s) {
                const uint32_t uses = (na - s + p.sa - 1) / p.sa;
                mbar_wait(&sm.a_full[s], (uses - 1) & 1, p.err, kErrWaitDrain);
            }
            for (uint32_t s = 0; s < uint32_t(p.sb) && s < nb; ++s) {
                const uint32_t uses = (nb - s + p.sb - 1) / p.sb;
                mbar_wait(&sm.b_full[s], (uses - 1) & 1, p.err, kErrWaitDrain);
            }
        }
    } else if (warp == 1 || warp == kEpiWarps + 2) {
        // --------------------------------------------------------- MMA issue
        // One thread issues every MMA of its tiles, so whatever it computes
        // between two MMAs delays the next: descriptors are built once and
        // advanced by additions, the tap loop is unrolled (its nine row
        // offsets live in registers) and rings advance without divisions.
        // With two issuing threads each walks the same rings and waits,
        // and issues and commits only its own tile's MMAs.
        constexpr int kPer = kTiles / kIssuers;   // tiles this thread issues
        const int first = warp == 1 ? 0 : kPer;   // its first tile in the group
        if (lane == 0) {
            Ring ra, rb;
            uint32_t j = 0;
            bool ok = true;
            const uint32_t a_stage = (uint32_t(C::kOps * kTiles) * uint32_t(p.a_bytes)) >> 4,
                           a_lo = uint32_t(p.a_bytes) >> 4, a_tile = (uint32_t(C::kOps) * uint32_t(p.a_bytes)) >> 4;
            const uint64_t a_desc = sw128_desc(smem_u32(sm.a)) + uint64_t(first) * a_tile,
                           b_desc = sw128_desc(smem_u32(sm.b));
            const uint32_t tmem_mine = tmem + uint32_t(first) * C::kTileCols;
            constexpr uint32_t b_stage = (C::kOps * C::kBBytes) >> 4, b_lo = C::kBBytes >> 4;
            uint32_t toff[9];
            tap_offsets(p, toff);
            if constexpr (kSeg == 0) {
                // One accumulator run per tile (per item: the persistent tower's
                // layers all have this shape).
                Ring ri;
                for (int k = 0; ok; ++k, ++j) {
                    int it = blockIdx.x + k * int(gridDim.x);
                    if constexpr (kPersist) {
                        if (!(ok = mbar_wait(&item_full[ri.idx], ri.phase, p.err, kErrWaitMma))) break;
                        it = item_slot[ri.idx];
                        mbar_arrive(&item_empty[ri.idx]);
                        ri.next(kItemSlots);
                        if (it < 0) break;
                    }
                    if (it >= nitems) break;
                    // The persistent tower's stem item: one tap, the centre view.
                    int taps = p.taps, nchunks = p.nchunks;
                    uint32_t off0 = toff[0];
                    if constexpr (kPersist) {
                        if (it < tf.stem_first * ngroups) {
                            taps = 1;
                            nchunks = tf.stem_nchunks;
                            off0 = toff[4];
                        }
                    }
                    const uint32_t acc = j & 1;
                    if (!(ok = mbar_wait(&sm.acc_empty[acc], ((j >> 1) & 1) ^ 1, p.err, kErrWaitMma))) break;
                    tc_fence_after();
                    const uint32_t d = tmem_mine + acc * (kTiles * C::kTileCols);   // tile u's at + u * kTileCols
                    for (int c = 0; c < nchunks && ok; ++c) {
                        if (!(ok = mbar_wait(&sm.a_full[ra.idx], ra.phase, p.err, kErrWaitMma))) break;
                        const uint64_t ac = a_desc + ra.idx * a_stage;
#pragma unroll
                        for (int t = 0; t < 9; ++t) {
                            if (t >= taps) break;
                            if (!(ok = mbar_wait(&sm.b_full[rb.idx], rb.phase, p.err, kErrWaitMma))) break;
                            tc_fence_after();
                            const uint64_t at = ac + (t == 0 ? off0 : toff[t]), bt = b_desc + rb.idx * b_stage;
#pragma unroll
                            for (int k = 0; k < C::kSteps; ++k) {
#pragma unroll
                                for (int u = 0; u < kPer; ++u) {   // every tile of the group reads this weight tile
                                    const uint32_t du = d + uint32_t(u) * C::kTileCols;
                                    const uint64_t au = at + u * a_tile;
                                    if constexpr (C::kStack) {
                                        // [hi | lo] weight planes as one operand: a_hi.b_hi
                                        // into [0, N), a_hi.b_lo into [N, 2N); a_lo.b_hi into
                                        // [N, 2N) too, so the large products alone
                                        // accumulate in [0, N).
                                        constexpr uint32_t kIdescStack = umma_idesc(2 * N, kBf16);
                                        umma<kBf16>(du, au + 2 * k, bt + 2 * k, kIdescStack, (c | t | k) != 0);
                                        umma<kBf16>(du + N, au + a_lo + 2 * k, bt + 2 * k, C::kIdesc, 1);
                                    } else {
                                        umma<kBf16>(du, au + 2 * k, bt + 2 * k, C::kIdesc, (c | t | k) != 0);
                                        if (kSplit) {
                                            umma<kBf16>(du, au + 2 * k, bt + b_lo + 2 * k, C::kIdesc, 1);
                                            umma<kBf16>(du, au + a_lo + 2 * k, bt + 2 * k, C::kIdesc, 1);
                                        }
                                    }
                                }
                            }
                            umma_commit(&sm.b_empty[rb.idx]);   // frees the weight buffer once read
                            rb.next(p.sb);
                        }
                        if (!ok) break;
                        umma_commit(&sm.a_empty[ra.idx]);       // frees the halo buffer
                        ra.next(p.sa);
                    }
                    if (!ok) break;
                    umma_commit(&sm.acc_full[acc]);             // the tile's accumulator is complete
                }
            } else {
                // The stacked split mode in segments of kSeg taps (a one-tap
                // pass: of one chunk), each on the next accumulator; the
                // epilogue sums them in fp32. Segment bounds fall on unrolled
                // tap positions: a counter and branch per tap in this thread
                // would slow every MMA after it.
                static_assert(C::kStack && 9 % kSeg == 0, "segments: stacked split mode, kSeg divides 9");
                Ring ri;
                for (int k = 0; ok; ++k) {
                    int it = blockIdx.x + k * int(gridDim.x);
                    if constexpr (kPersist) {
                        if (!(ok = mbar_wait(&item_full[ri.idx], ri.phase, p.err, kErrWaitMma))) break;
                        it = item_slot[ri.idx];
                        mbar_arrive(&item_empty[ri.idx]);
                        ri.next(kItemSlots);
                        if (it < 0) break;
                    }
                    if (it >= nitems) break;
                    // The persistent tower's stem item: one tap, the centre view.
                    int taps = p.taps, nchunks = p.nchunks;
                    uint32_t off0 = toff[0];
                    if constexpr (kPersist) {
                        if (it < tf.stem_first * ngroups) {
                            taps = 1;
                            nchunks = tf.stem_nchunks;
                            off0 = toff[4];
                        }
                    }
                    const bool one_tap = taps == 1;
                    uint32_t acc = 0, d = 0;
                    for (int c = 0; c < nchunks && ok; ++c) {
                        if (!(ok = mbar_wait(&sm.a_full[ra.idx], ra.phase, p.err, kErrWaitMma))) break;
                        const uint64_t ac = a_desc + ra.idx * a_stage;
#pragma unroll
                        for (int t = 0; t < 9; ++t) {
                            if (t >= taps) break;
                            if (t % kSeg == 0) {   // open a segment on the next accumulator
                                acc = j & 1;
                                if (!(ok = mbar_wait(&sm.acc_empty[acc], ((j >> 1) & 1) ^ 1, p.err, kErrWaitMma))) break;
                                d = tmem_mine + acc * (kTiles * C::kTileCols);
                            }
                            if (!(ok = mbar_wait(&sm.b_full[rb.idx], rb.phase, p.err, kErrWaitMma))) break;
                            tc_fence_after();
                            const uint64_t at = ac + (t == 0 ? off0 : toff[t]), bt = b_desc + rb.idx * b_stage;
#pragma unroll
                            for (int k = 0; k < C::kSteps; ++k) {
#pragma unroll
                                for (int u = 0; u < kPer; ++u) {
                                    const uint32_t du = d + uint32_t(u) * C::kTileCols;
                                    const uint64_t au = at + u * a_tile;
                                    constexpr uint32_t kIdescStack = umma_idesc(2 * N, kBf16);
                                    umma<kBf16>(du, au + 2 * k, bt + 2 * k, kIdescStack, (t % kSeg) != 0 || k != 0);
                                    umma<kBf16>(du + N, au + a_lo + 2 * k, bt + 2 * k, C::kIdesc, 1);
                                }
                            }
                            umma_commit(&sm.b_empty[rb.idx]);
                            rb.next(p.sb);
                            if (t % kSeg == kSeg - 1) {   // the segment is complete
                                umma_commit(&sm.acc_full[acc]);
                                ++j;
                            }
                        }
                        if (!ok) break;
                        if (one_tap) {   // a one-tap pass closes its segment per chunk
                            umma_commit(&sm.acc_full[acc]);
                            ++j;
                        }
                        umma_commit(&sm.a_empty[ra.idx]);
                        ra.next(p.sa);
                    }
                }
            }
            // All MMAs issued by this thread are complete before teardown.
            umma_commit(sm.done);
            mbar_wait(sm.done, 0, p.err, kErrWaitDrain);
        }
    } else {
        // ----------------------------------------------------------- epilogue
        // Eight warps: warp w reads TMEM lanes 32(w % 4) .. +31 (a warp may
        // read only its own quarter). One tile per group: the two warps on a
        // quarter split the columns (warps 2-5 the first half, 6-9 the
        // rest). Two tiles: warps 2-5 finish tile 0 and warps 6-9 tile 1.
        const int e = warp - 2, quarter = warp & 3;
        constexpr int kChunks = N / 32;
        const int u = kTiles == 2 ? (e >> 2) : 0;
        const int c_begin = kTiles == 2 ? 0 : (kChunks >= 2 ? (e >> 2) * (kChunks / 2) : (e >> 2) * kChunks);
        const int c_end = kTiles == 2 ? kChunks : (kChunks >= 2 ? c_begin + kChunks / 2 : kChunks);
        const int row_in_tile = quarter * 32 + lane;
        const int n1 = p.n + 1;
        EpiWarp ew;
        ew.obuf = sm.epi + e * (C::kEpiBytes / kEpiWarps);
        ew.sbuf = ew.obuf + C::kEpiBytes / kEpiWarps / 2;
        ew.sbar = sm.skip_full + 2 * e;
        uint32_t j = 0;   // accumulator runs consumed (one per tile, or one per segment)
        // Accumulator runs per tile: one, or the split mode's segments (a
        // one-tap pass: one per chunk); the persistent tower's stem items
        // are one-tap.
        auto segs_of = [&](int taps, int nchunks) {
            return kSeg == 0 ? 1 : (taps == 1 ? nchunks : nchunks * (9 / (kSeg > 0 ? kSeg : 1)));
        };
        const int layer_segs = segs_of(p.taps, p.nchunks);
        // An item's ItemIo, derived where it is used rather than held across
        // the segments' accumulation (registers are at the 168 cap).
        auto item_io = [&](int layer, int col0) {
            ItemIo io{sm.bn, sm.bn + N, p.skip, p.skip_lo, &mOut, &mSkip};
            if constexpr (kWide) {   // this item's column half (the residual's rows hold all 2N channels)
                io.scale = sm.bn + col0;
                io.shift = sm.bn + kBnCh + col0;
                if (p.skip) {
                    io.res_hi = static_cast<const float*>(p.skip) + col0;
                    io.res_lo = static_cast<const float*>(p.skip_lo) + col0;
                }
            }
            if constexpr (kPersist) {
                // Tower conv l writes buffer (l+1) mod 3; a block's second conv
                // (l odd) adds its first conv's input, buffer (l-1) mod 3. The
                // stem (l = -1) writes buffer 0 and adds nothing.
                const int conv = layer - tf.stem_first;
                const int out = (conv + 4) % 3, res = (conv + 2) % 3;
                const bool has_res = conv >= 0 && (conv & 1) != 0;
                io.res_hi = has_res ? tf.trunk[res] : nullptr;
                io.res_lo = has_res ? tf.trunk_lo[res] : nullptr;
                io.omap = &tf.out[out];
                io.smap = kSplit ? &tf.out_lo[out] : &tf.out[has_res ? res : out];
                const FusedLayer& fl = tf.tower[conv < 0 ? tf.layers - 1 : conv];
                io.scale = fl.scale;
                io.shift = fl.shift;
            }
            return io;
        };
        Ring ri;
        for (int k = 0;; ++k) {
            int it = blockIdx.x + k * int(gridDim.x);
            if constexpr (kPersist) {
                if (!mbar_wait(&item_full[ri.idx], ri.phase, p.err, kErrWaitEpilogue)) break;
                it = item_slot[ri.idx];
                __syncwarp();
                if (lane == 0) mbar_arrive(&item_empty[ri.idx]);
                ri.next(kItemSlots);
                if (it < 0) break;
            }
            if (it >= nitems) break;
            int g = it, layer = 0, col0 = 0;
            if constexpr (kWide) {   // a tile group's column half
                g = it >> 1;
                col0 = (it & 1) * N;
            }
            if constexpr (kPersist) {
                layer = it / ngroups;
                g = it - layer * ngroups;
                if (layer > 0) {
                    // This warp reads the residual and overwrites rows that
                    // earlier items read: acquire the previous layer's group
                    // (whose own dependencies cover both) here as well.
                    bool ok = true;
                    if (lane == 0) {
                        ok = flag_wait(tf.flags + size_t(layer - 1) * ngroups + g, kEpiWarps + tf.flag_extra, p.err,
                                       kErrWaitLayer);
                        fence_proxy_async_global();
                    }
                    if (!__shfl_sync(0xffffffffu, ok, 0)) break;
                }
            }
            const int tile = g * kTiles + u;
            const int q = tile * 128 + row_in_tile;
            bool valid = q < p.rows;
            if (valid) {
                const int r = q % p.S;
                valid = r >= n1 && (r % n1) != p.n;
            }
            const uint32_t lanes = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(u) * C::kTileCols;
            if constexpr (C::kStack) {
                // The tile's segments, summed in registers; each accumulator
                // is released as soon as it has been read.
                constexpr int kMine = kTiles == 2 ? kChunks : (kChunks >= 2 ? kChunks / 2 : 1);
                const bool mine = c_begin < c_end && tile < p.ntiles;
                float sum[kMine * 32];
                bool ok = true;
                int segs = layer_segs;
                if constexpr (kPersist) {
                    if (layer < tf.stem_first) segs = segs_of(1, tf.stem_nchunks);
                }
                for (int sg = 0; sg < segs; ++sg, ++j) {
                    const uint32_t acc = j & 1;
                    if (sg == segs - 1 && mine && valid) {
                        // The residual reaches L2 while the last segment
                        // accumulates (earlier, a pass whose frames overflow
                        // L2 evicts it again before the store reads it).
                        const ItemIo io = item_io(layer, col0);
                        if (io.res_hi != nullptr) {
                            const size_t off = size_t(q) * p.ld + size_t(c_begin) * 32;
#pragma unroll
                            for (int cc = 0; cc < kMine; ++cc) {
                                prefetch_l2(static_cast<const float*>(io.res_hi) + off + cc * 32);
                                prefetch_l2(static_cast<const float*>(io.res_lo) + off + cc * 32);
                            }
                        }
                    }
                    if (!(ok = mbar_wait(&sm.acc_full[acc], (j >> 1) & 1, p.err, kErrWaitEpilogue))) break;
                    tc_fence_after();
                    if (mine) add_segment<N, kMine>(lanes + acc * (kTiles * C::kTileCols), c_begin, sum, sg == 0);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sm.acc_empty[acc]);
                }
                if (!ok) break;
                if (mine) {
                    const ItemIo io = item_io(layer, col0);
                    store_split_sums<N, kMine>(p, io.scale, io.shift, io.res_hi, io.res_lo, sum, io.omap, io.smap,
                                               ew.obuf, tile * 128 + quarter * 32, q, valid, c_begin, lane, col0);
                }
                if constexpr (kPersist) {
                    if (lane == 0) {   // this warp's part of the item has landed in global memory
                        bulk_wait_all();
                        fence_proxy_async_global();
                        flag_add_release(tf.flags + it, 1u);
                    }
                }
            } else {
                const uint32_t acc = j & 1;
                if (!mbar_wait(&sm.acc_full[acc], (j >> 1) & 1, p.err, kErrWaitEpilogue)) break;
                tc_fence_after();
                const uint32_t taddr = lanes + acc * (kTiles * C::kTileCols);
                const ItemIo io = item_io(layer, 0);
                if constexpr (C::kEpiTma)
                    store_epilogue_tma<N, kBf16, kPersist>(p, io.scale, io.shift, io.res_hi, io.omap, io.smap, taddr,
                                                 tile * 128 + quarter * 32, valid, c_begin, c_end, ew, lane);
                else if (tile < p.ntiles)
                    store_epilogue_split<N>(p, sm.bn, taddr, q, valid, c_begin, c_end);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.acc_empty[acc]);
                ++j;
                if constexpr (kPersist) {
                    if (lane == 0) {   // this warp's part of the item has landed in global memory
                        bulk_wait_all();
                        fence_proxy_async_global();
                        flag_add_release(tf.flags + it, 1u);
                    }
                }
            }
        }
        if ((C::kEpiTma || C::kStack) && lane == 0) bulk_wait_all();   // every output box written before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

// ------------------------------------------------------- the CTA-pair form
//
// The same convolution with M = 256 per MMA: a 2-CTA cluster computes two
// consecutive 128-row tiles at once. Each CTA stages its own tile's halo and
// half of each weight tile (N/2 rows) in its own shared memory; the pair's
// leader (cluster rank 0) issues tcgen05.mma.cta_group::2, which reads both
// CTAs' operands and writes each CTA's 128 accumulator rows into its own TMEM.
// Per SM this halves the weight traffic (TMA writes and MMA operand reads),
// the shared-memory bandwidth the single-CTA form runs out of.
//
// Protocol (all waits bounded):
//  - full barriers live in the leader: its producer arms each with the bytes
//    of BOTH CTAs' loads; both CTAs' TMA loads complete on it;
//  - empty barriers live in each CTA: the leader's MMA thread commits to its
//    own and to the peer's, so each producer reuses its own buffers only when
//    the pair MMAs reading them are done;
//  - acc_full in each CTA (committed by the leader to both), acc_empty in the
//    leader (one arrival per epilogue warp of both CTAs);
//  - TMEM allocated and freed with cta_group::2 by warp 1 of both CTAs; a
//    cluster barrier after set-up and before teardown.
template <int N, bool kBf16, bool kSplit>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    conv3x3_tc_pair(const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mAlo,
                    const __grid_constant__ CUtensorMap mW, const __grid_constant__ CUtensorMap mWlo,
                    const __grid_constant__ CUtensorMap mOut, const __grid_constant__ CUtensorMap mSkip,
                    const ConvArgs p) {
    using C = ConvCfg<N, kBf16, kSplit>;
    constexpr uint32_t kHalfB = uint32_t(N / 2) * 128u;     // this CTA's half of a weight tile
    constexpr uint32_t kIdesc = umma_idesc(N, kBf16, 256);
    extern __shared__ uint8_t smem_raw[];
    const Smem sm = carve(smem_raw, p.sa, p.sb, C::kOps, C::kOps, p.a_bytes, kHalfB, C::kEpiBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.sa; ++i) {
            mbar_init(&sm.a_full[i], 1);
            mbar_init(&sm.a_empty[i], 1);
        }
        for (int i = 0; i < p.sb; ++i) {
            mbar_init(&sm.b_full[i], 1);
            mbar_init(&sm.b_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.acc_full[i], 1);
            mbar_init(&sm.acc_empty[i], 2 * kEpiWarps);   // every epilogue warp of both CTAs
        }
        mbar_init(sm.done, 1);
        for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&sm.skip_full[i], 1);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&mA);
        tma_prefetch_map(&mW);
        if (C::kEpiTma) {
            tma_prefetch_map(&mOut);
            tma_prefetch_map(&mSkip);
        }
        if (kSplit) {
            tma_prefetch_map(&mAlo);
            tma_prefetch_map(&mWlo);
        }
    }
    if (warp == 1) tmem_alloc_pair(sm.tmem_slot, C::kTmemCols);
    for (int i = threadIdx.x; i < N; i += kThreads) {
        sm.bn[i] = p.scale[i];
        sm.bn[N + i] = p.shift[i];
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();   // both CTAs' barriers exist before either addresses the other's
    tc_fence_after();
    const uint32_t tmem = *sm.tmem_slot;
    grid_dependency_wait();   // as in the single-CTA form
    grid_launch_dependents();
    const int npairs = (p.ntiles + 1) / 2;
    const int pair0 = blockIdx.x >> 1, pair_step = gridDim.x >> 1;

    if (warp == 0) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            Ring ra, rb;
            uint32_t na = 0, nb = 0;
            const uint32_t a_tx = uint32_t(p.halo_rows) * 128u * C::kOps * 2u;   // both CTAs
            const uint32_t b_tx = kHalfB * C::kOps * 2u;
            const size_t a_stage = size_t(C::kOps) * p.a_bytes;
            // Both CTAs' copies complete on the leader's full barriers.
            const uint32_t a_full0 = mapa(smem_u32(sm.a_full), 0), b_full0 = mapa(smem_u32(sm.b_full), 0);
            bool ok = true;
            for (int pr = pair0; pr < npairs && ok; pr += pair_step) {
                const int tile = 2 * pr + int(rank);
                const int y0 = tile * 128 - (p.n + 2);
                for (int c = 0; c < p.nchunks && ok; ++c) {
                    if (!(ok = mbar_wait(&sm.a_empty[ra.idx], ra.phase ^ 1u, p.err, kErrWaitProducer))) break;
                    if (leader) mbar_arrive_expect_tx(&sm.a_full[ra.idx], a_tx);
                    const uint32_t full = a_full0 + ra.idx * 8u;
                    uint8_t* abuf = sm.a + ra.idx * a_stage;
                    tma_load_2d_pair(&mA, abuf, full, c * C::kKc, y0);
                    if (kSplit) tma_load_2d_pair(&mAlo, abuf + p.a_bytes, full, c * C::kKc, y0);
                    ra.next(p.sa);
                    ++na;
                    for (int t = 0; t < p.taps; ++t) {
                        if (!(ok = mbar_wait(&sm.b_empty[rb.idx], rb.phase ^ 1u, p.err, kErrWaitProducer))) break;
                        if (leader) mbar_arrive_expect_tx(&sm.b_full[rb.idx], b_tx);
                        const uint32_t bfull = b_full0 + rb.idx * 8u;
                        uint8_t* bbuf = sm.b + rb.idx * (C::kOps * kHalfB);
                        const int x = (c * p.taps + t) * C::kKc, y = int(rank) * (N / 2);
                        tma_load_2d_pair(&mW, bbuf, bfull, x, y);
                        if (kSplit) tma_load_2d_pair(&mWlo, bbuf + kHalfB, bfull, x, y);
                        rb.next(p.sb);
                        ++nb;
                    }
                }
            }
            // The leader's full barriers count both CTAs' copies: once each
            // stage's last phase completed, every copy of the pair has landed.
            if (leader) {
                for (uint32_t s = 0; s < uint32_t(p.sa) && s < na; ++s)
                    mbar_wait(&sm.a_full[s], ((na - s + p.sa - 1) / p.sa - 1) & 1, p.err, kErrWaitDrain);
                for (uint32_t s = 0; s < uint32_t(p.sb) && s < nb; ++s)
                    mbar_wait(&sm.b_full[s], ((nb - s + p.sb - 1) / p.sb - 1) & 1, p.err, kErrWaitDrain);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issue (leader)
        // As in the single-CTA form: descriptors advanced by additions, the
        // tap loop unrolled, and the barrier addresses of both CTAs (for the
        // commits that release each CTA's buffers) computed once.
        if (leader && lane == 0) {
            Ring ra, rb;
            uint32_t j = 0;
            bool ok = true;
            const uint64_t a_desc = sw128_desc(smem_u32(sm.a)), b_desc = sw128_desc(smem_u32(sm.b));
            const uint32_t a_stage = (uint32_t(C::kOps) * uint32_t(p.a_bytes)) >> 4, a_lo = uint32_t(p.a_bytes) >> 4;
            constexpr uint32_t b_stage = (C::kOps * kHalfB) >> 4, b_lo = kHalfB >> 4;
            uint32_t toff[9];
            tap_offsets(p, toff);
            const uint32_t a_empty0 = mapa(smem_u32(sm.a_empty), 0), a_empty1 = mapa(smem_u32(sm.a_empty), 1);
            const uint32_t b_empty0 = mapa(smem_u32(sm.b_empty), 0), b_empty1 = mapa(smem_u32(sm.b_empty), 1);
            const uint32_t acc_full0 = mapa(smem_u32(sm.acc_full), 0), acc_full1 = mapa(smem_u32(sm.acc_full), 1);
            for (int pr = pair0; pr < npairs && ok; pr += pair_step, ++j) {
                const uint32_t acc = j & 1;
                if (!(ok = mbar_wait_cluster(&sm.acc_empty[acc], ((j >> 1) & 1) ^ 1, p.err, kErrWaitMma))) break;
                tc_fence_after();
                const uint32_t d = tmem + acc * N;
                for (int c = 0; c < p.nchunks && ok; ++c) {
                    if (!(ok = mbar_wait(&sm.a_full[ra.idx], ra.phase, p.err, kErrWaitMma))) break;
                    const uint64_t ac = a_desc + ra.idx * a_stage;
#pragma unroll
                    for (int t = 0; t < 9; ++t) {
                        if (t >= p.taps) break;
                        if (!(ok = mbar_wait(&sm.b_full[rb.idx], rb.phase, p.err, kErrWaitMma))) break;
                        tc_fence_after();
                        const uint64_t at = ac + toff[t], bt = b_desc + rb.idx * b_stage;
#pragma unroll
                        for (int k = 0; k < C::kSteps; ++k) {
                            umma_pair<kBf16>(d, at + 2 * k, bt + 2 * k, kIdesc, (c | t | k) != 0);
                            if (kSplit) {
                                umma_pair<kBf16>(d, at + 2 * k, bt + b_lo + 2 * k, kIdesc, 1);
                                umma_pair<kBf16>(d, at + a_lo + 2 * k, bt + 2 * k, kIdesc, 1);
                            }
                        }
                        umma_commit_pair(b_empty0 + rb.idx * 8u);   // each CTA's weight half is free
                        umma_commit_pair(b_empty1 + rb.idx * 8u);
                        rb.next(p.sb);
                    }
                    if (!ok) break;
                    umma_commit_pair(a_empty0 + ra.idx * 8u);
                    umma_commit_pair(a_empty1 + ra.idx * 8u);
                    ra.next(p.sa);
                }
                if (!ok) break;
                umma_commit_pair(acc_full0 + acc * 8u);
                umma_commit_pair(acc_full1 + acc * 8u);
            }
            umma_commit_pair(mapa(smem_u32(sm.done), 0));
            mbar_wait(sm.done, 0, p.err, kErrWaitDrain);
        }
    } else {
        // ------------------------------------------- epilogue (both CTAs)
        // Eight warps per CTA, split as in the single-CTA form.
        const int e = warp - 2, quarter = warp & 3;
        constexpr int kChunks = N / 32;
        const int c_begin = kChunks >= 2 ? (e >> 2) * (kChunks / 2) : (e >> 2) * kChunks;
        const int c_end = kChunks >= 2 ? c_begin + kChunks / 2 : kChunks;
        const int row_in_tile = quarter * 32 + lane;
        const int n1 = p.n + 1;
        const uint32_t leader_empty0 = mapa(smem_u32(&sm.acc_empty[0]), 0), leader_empty1 = leader_empty0 + 8u;
        EpiWarp ew;
        ew.obuf = sm.epi + e * (C::kEpiBytes / kEpiWarps);
        ew.sbuf = ew.obuf + C::kEpiBytes / kEpiWarps / 2;
        ew.sbar = sm.skip_full + 2 * e;
        uint32_t j = 0;
        for (int pr = pair0; pr < npairs; pr += pair_step, ++j) {
            const uint32_t acc = j & 1;
            if (!mbar_wait(&sm.acc_full[acc], (j >> 1) & 1, p.err, kErrWaitEpilogue)) break;
            tc_fence_after();
            const int q = (2 * pr + int(rank)) * 128 + row_in_tile;
            bool valid = q < p.rows;
            if (valid) {
                const int r = q % p.S;
                valid = r >= n1 && (r % n1) != p.n;
            }
            const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16) + acc * N;
            if constexpr (C::kEpiTma)
                store_epilogue_tma<N, kBf16>(p, sm.bn, sm.bn + N, p.skip, &mOut, &mSkip, taddr,
                                             (2 * pr + int(rank)) * 128 + quarter * 32,
                                             valid, c_begin, c_end, ew, lane);
            else
                store_epilogue_split<N>(p, sm.bn, taddr, q, valid, c_begin, c_end);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? leader_empty1 : leader_empty0);
        }
        if (C::kEpiTma && lane == 0) bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();   // no remote arrival or pair MMA is still in flight
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, C::kTmemCols);
    }
}

// ------------------------------------------------------------------- probe

// One CTA, one thread issuing: stage a halo tile and k_chunks weight tiles
// (weight chunk c at K offset c*9*KC, i.e. tap 0 of chunk c), run the MMAs
// on the view starting at row `shift`, and write D raw (fp32 [128][N]).
template <int N, bool kBf16>
__global__ void __launch_bounds__(128, 1)
    umma_probe(const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mW, int halo_rows,
               int a_bytes, int shift, int k_chunks, int base_offset_mode, float* out, int* err) {
    using C = ConvCfg<N, kBf16, false>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a = base;
    uint8_t* b = base + a_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(b + C::kBBytes);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(tslot, C::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (threadIdx.x == 0) {
        for (int c = 0; c < k_chunks; ++c) {
            mbar_arrive_expect_tx(&bars[0], uint32_t(halo_rows) * 128u + C::kBBytes);
            tma_load_2d(&mA, a, &bars[0], c * C::kKc, 0);
            tma_load_2d(&mW, b, &bars[0], c * 9 * C::kKc, 0);
            if (!mbar_wait(&bars[0], c & 1, err, kErrWaitMma)) break;
            tc_fence_after();
            for (int k = 0; k < C::kSteps; ++k) {
                const uint64_t ad = sw128_desc(smem_u32(a) + uint32_t(shift) * 128u + k * 32u, base_offset_mode);
                const uint64_t bd = sw128_desc(smem_u32(b) + k * 32u, base_offset_mode);
                umma<kBf16>(tmem, ad, bd, C::kIdesc, (c | k) != 0);
            }
            umma_commit(&bars[1]);
            if (!mbar_wait(&bars[1], c & 1, err, kErrWaitMma)) break;
        }
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = tmem + (uint32_t(warp * 32) << 16);
    for (int c0 = 0; c0 < N; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(taddr + c0, v);
        tmem_wait_ld();
        for (int i = 0; i < 32; ++i) out[size_t(warp * 32 + lane) * N + c0 + i] = __uint_as_float(v[i]);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

std::atomic<int> g_conv_path{0};   // 0: by width, 1: one tile per CTA, 2: CTA pairs, 3: two tiles per CTA

// Taps per accumulation segment: at 128 channels three (12 MMA K steps of 8
// on the large products' accumulator before the epilogue takes the partial
// sum), at 64 or fewer nine (one chunk): there the epilogue's extra work
// per segment costs as much as the narrow layers' MMAs take, and a chunk's
// 36 K steps already keep the sums within the reference's tolerance against
// double precision.
template <int N>
constexpr int kDefaultSegment = N <= 64 ? 9 : 3;

// The conv forms: one CTA per 128-row tile, one CTA per two tiles sharing
// each weight tile (N <= 128: both accumulators fit in TMEM), or 2-CTA pairs.
enum ConvForm : int { kFormSingle = 1, kFormPair = 2, kFormDual = 3 };

template <int N, bool kBf16, bool kSplit, int kTiles, int kSeg>
cudaError_t launch_single_seg(const ConvMaps& m, ConvArgs a, int sms, cudaStream_t s) {
    using C = ConvCfg<N, kBf16, kSplit, kTiles>;
    conv_smem_bytes(N, kBf16 ? kBF16 : (kSplit ? kTF32x3 : kTF32), a.halo_rows, &a.sa, &a.sb, false, kTiles);
    const size_t smem = smem_total(a.sa, a.sb, C::kOps * kTiles, C::kOps, a.a_bytes, C::kBBytes, C::kEpiBytes);
    if (const cudaError_t e = open_smem<conv3x3_tc<N, kBf16, kSplit, kTiles, kSeg>>(smem); e != cudaSuccess) return e;
    const int groups = (a.ntiles + kTiles - 1) / kTiles;
    const int grid = std::max(1, std::min(groups, sms));
    return launch_pdl(conv3x3_tc<N, kBf16, kSplit, kTiles, kSeg>, dim3(grid), dim3(kThreadsOf<kTiles>), smem, s, m.a,
                      m.a_lo, m.w, m.w_lo, m.out, C::kStack ? m.out_lo : m.skip, a, NoTower{});
}

// A 2N-channel layer in the split mode as two column halves of N (kWide),
// one CTA per item (a tile group's half), in the stacked mode's default
// segments. The weight maps are the pair form's (boxes of N = n_out / 2 rows).
template <int N>
cudaError_t launch_wide(const ConvMaps& m, ConvArgs a, int sms, cudaStream_t s) {
    using C = ConvCfg<N, false, true, 1>;
    constexpr int kSeg = kDefaultSegment<N>;
    conv_smem_bytes(N, kTF32x3, a.halo_rows, &a.sa, &a.sb, false, 1);
    const size_t smem = smem_total(a.sa, a.sb, C::kOps, C::kOps, a.a_bytes, C::kBBytes, C::kEpiBytes);
    if (const cudaError_t e = open_smem<conv3x3_tc<N, false, true, 1, kSeg, false, true>>(smem); e != cudaSuccess)
        return e;
    const int grid = std::max(1, std::min(2 * a.ntiles, sms));
    return launch_pdl(conv3x3_tc<N, false, true, 1, kSeg, false, true>, dim3(grid), dim3(kThreadsOf<1>), smem, s, m.a,
                      m.a_lo, m.w_pair, m.w_lo_pair, m.out, m.out_lo, a, NoTower{});
}

// The stacked split mode runs in segments of kDefaultSegment<N> taps unless
// the test hook asks for one run per tile (a.seg == 0).
template <int N, bool kBf16, bool kSplit, int kTiles>
cudaError_t launch_single(const ConvMaps& m, ConvArgs a, int sms, cudaStream_t s) {
    if constexpr (ConvCfg<N, kBf16, kSplit, kTiles>::kStack) {
        if (a.seg != 0) return launch_single_seg<N, kBf16, kSplit, kTiles, kDefaultSegment<N>>(m, a, sms, s);
    }
    return launch_single_seg<N, kBf16, kSplit, kTiles, 0>(m, a, sms, s);
}

// The persistent tower: bf16 and tf32 take two tiles per item where both
// halos and two weight stages fit (128 channels or fewer), else one; the
// split mode one tile in its default segments. A CTA per SM at most. The six
// per-layer map parameters are unused (valid maps, for the prefetch).
template <int N, bool kBf16, bool kSplit, int kTiles, int kSeg>
cudaError_t launch_persist_tiles(const TowerArgs& f, ConvArgs a, int sms, cudaStream_t s) {
    using C = ConvCfg<N, kBf16, kSplit, kTiles>;
    conv_smem_bytes(N, kBf16 ? kBF16 : (kSplit ? kTF32x3 : kTF32), a.halo_rows, &a.sa, &a.sb, false, kTiles);
    const size_t smem = smem_total(a.sa, a.sb, C::kOps * kTiles, C::kOps, a.a_bytes, C::kBBytes, C::kEpiBytes);
    if (const cudaError_t e = open_smem<conv3x3_tc<N, kBf16, kSplit, kTiles, kSeg, true>>(smem); e != cudaSuccess)
        return e;
    const int groups = (a.ntiles + kTiles - 1) / kTiles;
    const int grid = std::max(1, std::min(groups * f.layers, sms));
    return launch_pdl(conv3x3_tc<N, kBf16, kSplit, kTiles, kSeg, true>, dim3(grid), dim3(kThreadsOf<kTiles>), smem, s,
                      f.in[0], f.in_lo[0], f.in[0], f.in_lo[0], f.out[0], f.out_lo[0], a, f);
}

template <int N, bool kBf16>
cudaError_t launch_persist(const TowerArgs& f, const ConvArgs& a, int sms, cudaStream_t s) {
    if constexpr (N <= 128) {
        if (conv_smem_bytes(N, kBf16 ? kBF16 : kTF32, a.halo_rows, nullptr, nullptr, false, 2) <= 227 * 1024)
            return launch_persist_tiles<N, kBf16, false, 2, 0>(f, a, sms, s);
    }
    return launch_persist_tiles<N, kBf16, false, 1, 0>(f, a, sms, s);
}

template <int N, bool kBf16, bool kSplit>
cudaError_t launch_one(const ConvMaps& m, ConvArgs a, int form, int sms, cudaStream_t s) {
    using C = ConvCfg<N, kBf16, kSplit>;
    if (form == kFormPair) {
        conv_smem_bytes(N, kBf16 ? kBF16 : (kSplit ? kTF32x3 : kTF32), a.halo_rows, &a.sa, &a.sb, true, 1);
        const size_t smem = smem_total(a.sa, a.sb, C::kOps, C::kOps, a.a_bytes, C::kBBytes / 2, C::kEpiBytes);
        if (const cudaError_t e = open_smem<conv3x3_tc_pair<N, kBf16, kSplit>>(smem); e != cudaSuccess) return e;
        const int pairs = (a.ntiles + 1) / 2;
        const int grid = 2 * std::max(1, std::min(pairs, sms / 2));
        return launch_pdl(conv3x3_tc_pair<N, kBf16, kSplit>, dim3(grid), dim3(kThreads), smem, s, m.a, m.a_lo, m.w_pair,
                          m.w_lo_pair, m.out, m.skip, a);
    }
    if constexpr (N <= 128) {
        if (form == kFormDual) return launch_single<N, kBf16, kSplit, 2>(m, a, sms, s);
    }
    return launch_single<N, kBf16, kSplit, 1>(m, a, sms, s);
}

template <bool kBf16, bool kSplit>
cudaError_t dispatch_n(int n_out, const ConvMaps& m, const ConvArgs& a, int form, int sms, cudaStream_t s) {
    switch (n_out) {
        case 32: return launch_one<32, kBf16, kSplit>(m, a, form, sms, s);
        case 64: return launch_one<64, kBf16, kSplit>(m, a, form, sms, s);
        case 128: return launch_one<128, kBf16, kSplit>(m, a, form, sms, s);
        case 256: return launch_one<256, kBf16, kSplit>(m, a, form, sms, s);
        default: return cudaErrorInvalidValue;
    }
}

template <int N, bool kBf16>
cudaError_t probe_one(const ConvMaps& m, int halo_rows, int shift, int k_chunks, int bom, float* out, int* err,
                      cudaStream_t s) {
    using C = ConvCfg<N, kBf16, false>;
    const int a_bytes = (halo_rows * 128 + 1023) / 1024 * 1024;
    const size_t smem = 1024 + size_t(a_bytes) + C::kBBytes + 64;
    cudaError_t e = cudaFuncSetAttribute(umma_probe<N, kBf16>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    umma_probe<N, kBf16><<<1, 128, smem, s>>>(m.a, m.w, halo_rows, a_bytes, shift, k_chunks, bom, out, err);
    return cudaGetLastError();
}

} // namespace

size_t conv_smem_bytes(int n_out, int precision, int halo_rows, int* sa_out, int* sb_out, bool pair, int tiles) {
    const int ops = precision == kTF32x3 ? 2 : 1, a_ops = ops * tiles;
    const int a_bytes = (halo_rows * 128 + 1023) / 1024 * 1024;
    const uint32_t b_bytes = uint32_t(pair ? n_out / 2 : n_out) * 128u;
    // As ConvCfg::kEpiBytes: the stacked split mode (128 channels or fewer,
    // both accumulators of every tile in TMEM) has one 4 KB box per warp.
    const bool stacked = n_out <= 128 && 2 * tiles * 2 * n_out <= 512;
    const uint32_t epi = precision == kTF32x3 ? (stacked ? uint32_t(kEpiWarps) * 4096u : 0u)
                                              : uint32_t(kEpiWarps) * (precision == kBF16 ? 4096u : 8192u);
    constexpr size_t kMax = 227 * 1024;
    int sa = 2, sb = 2;
    for (int cand = kMaxStages; cand >= 2; --cand)
        if (smem_total(2, cand, a_ops, ops, a_bytes, b_bytes, epi) <= kMax) {
            sb = cand;
            break;
        }
    // A third halo stage only if it still leaves four weight buffers.
    if (smem_total(3, std::max(sb - 1, 4), a_ops, ops, a_bytes, b_bytes, epi) <= kMax && sb >= 5) {
        sa = 3;
        while (sb > 2 && smem_total(sa, sb, a_ops, ops, a_bytes, b_bytes, epi) > kMax) --sb;
    }
    if (sa_out) *sa_out = sa;
    if (sb_out) *sb_out = sb;
    return smem_total(sa, sb, a_ops, ops, a_bytes, b_bytes, epi);
}

void set_conv_path(int path) { g_conv_path = path; }

std::atomic<int> g_conv_segment{-1};
void set_conv_segment(int steps) { g_conv_segment = steps; }

std::atomic<int> g_tower_persistent{-1};
void set_tower_persistent(int mode) { g_tower_persistent = mode; }

std::atomic<int> g_tower_starve{0};
void set_tower_starve(int on) { g_tower_starve = on; }
bool tower_starve() { return g_tower_starve.load() != 0; }

bool tower_persistent(int n_out, int precision) {
    const int mode = g_tower_persistent.load();
    if (mode == 0) return false;
    // The split mode: in its default segments, at the widths whose weight
    // planes stack (the 256-channel split layers run per layer).
    if (precision == kTF32x3 && (n_out > 128 || g_conv_segment.load() == 0)) return false;
    if (mode == 1) return true;
    return n_out <= 128;
}

cudaError_t launch_tower_persistent(const TowerArgs& f, const ConvArgs& a, int n_out, int precision, int sms,
                                    cudaStream_t s) {
    if (a.ntiles <= 0 || f.layers <= 0) return cudaSuccess;
    if (f.tower == nullptr || f.flags == nullptr) return cudaErrorNotSupported;
    if (precision == kTF32x3) {
        switch (n_out) {
            case 32: return launch_persist_tiles<32, false, true, 1, kDefaultSegment<32>>(f, a, sms, s);
            case 64: return launch_persist_tiles<64, false, true, 1, kDefaultSegment<64>>(f, a, sms, s);
            case 128: return launch_persist_tiles<128, false, true, 1, kDefaultSegment<128>>(f, a, sms, s);
            default: return cudaErrorNotSupported;
        }
    }
    const bool bf16 = precision == kBF16;
    switch (n_out) {
        case 32: return bf16 ? launch_persist<32, true>(f, a, sms, s) : launch_persist<32, false>(f, a, sms, s);
        case 64: return bf16 ? launch_persist<64, true>(f, a, sms, s) : launch_persist<64, false>(f, a, sms, s);
        case 128: return bf16 ? launch_persist<128, true>(f, a, sms, s) : launch_persist<128, false>(f, a, sms, s);
        case 256: return bf16 ? launch_persist<256, true>(f, a, sms, s) : launch_persist<256, false>(f, a, sms, s);
        default: return cudaErrorNotSupported;
    }
}

// Which form a layer runs: by default the CTA pair for 256 output
// channels, where a weight tile is 32 KB per tap and halving it per SM
// pays (C4 bf16 on B200: 1217 against 1148 TFLOP/s per conv), the two-tile
// form for narrower layers with enough tiles to keep every SM busy (each
// weight tile then feeds two accumulators), and one tile per CTA otherwise.
int conv_form(int ntiles, int n_out, int precision, int halo_rows, int sms) {
    // The two-tile form stages two halos per stage; it must fit with at
    // least two weight stages (the split mode at 128 channels does not).
    // The split mode takes it only where both tiles' stacked accumulators
    // fit in TMEM (64 channels or fewer), so its sums stay segmented.
    const bool dual_fits = n_out <= (precision == kTF32x3 ? 64 : 128) &&
                           conv_smem_bytes(n_out, precision, halo_rows, nullptr, nullptr, false, 2) <= 227 * 1024;
    const int path = g_conv_path.load();
    if (path == kFormSingle) return kFormSingle;
    if (path == kFormPair) return kFormPair;
    if (path == kFormDual) return dual_fits ? kFormDual : kFormSingle;
    if (n_out == 256 && ntiles >= 2) return kFormPair;
    if (dual_fits && ntiles >= 2 * sms) return kFormDual;
    return kFormSingle;
}

cudaError_t launch_conv(const ConvMaps& maps, const ConvArgs& args, int n_out, int precision, int sms, cudaStream_t s) {
    if (args.ntiles <= 0) return cudaSuccess;
    const int form = conv_form(args.ntiles, n_out, precision, args.halo_rows, sms);
    ConvArgs a = args;
    const int segment = g_conv_segment.load();
    a.seg = segment < 0 ? 1 : segment;   // 0: one run per tile; otherwise segments of kDefaultSegment<N> taps
    // The split mode at 256 channels: two segmented column halves of 128
    // (one 256-column accumulator run per tile drifts: tcgen05 accumulates in
    // fp32 rounding toward zero, 864 MMAs per tile, ~4e-4 on the 19x19 20x256
    // network's logits), unless a test hook asks for the pair form or for
    // one run per tile.
    if (precision == kTF32x3 && n_out == 256 && a.seg != 0 && g_conv_path.load() != kFormPair)
        return launch_wide<128>(maps, a, sms, s);
    switch (precision) {
        case kTF32: return dispatch_n<false, false>(n_out, maps, a, form, sms, s);
        case kTF32x3: return dispatch_n<false, true>(n_out, maps, a, form, sms, s);
        case kBF16: return dispatch_n<true, false>(n_out, maps, a, form, sms, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_umma_probe(const ConvMaps& maps, int n_out, int precision, int halo_rows, int shift_rows,
                              int k_chunks, int base_offset_mode, float* d_out, int* err, cudaStream_t s) {
    const bool bf16 = precision == kBF16;
    if (shift_rows < 0 || shift_rows + 128 > halo_rows) return cudaErrorInvalidValue;
    switch (n_out) {
        case 32: return bf16 ? probe_one<32, true>(maps, halo_rows, shift_rows, k_chunks, base_offset_mode, d_out, err, s)
                             : probe_one<32, false>(maps, halo_rows, shift_rows, k_chunks, base_offset_mode, d_out, err, s);
        case 64: return bf16 ? probe_one<64, true>(maps, halo_rows, shift_rows, k_chunks, base_offset_mode, d_out, err, s)
                             : probe_one<64, false>(maps, halo_rows, shift_rows, k_chunks, base_offset_mode, d_out, err, s);
        case 128: return bf16 ? probe_one<128, true>(maps, halo_rows, shift_rows, k_chunks, base_offset_mode, d_out, err, s)
                              : probe_one<128, false>(maps, halo_rows, shift_rows, k_chunks, base_offset_mode, d_out, err, s);
        case 256: return bf16 ? probe_one<256, true>(maps, halo_rows, shift_rows, k_chunks, base_offset_mode, d_out, err, s)
                              : probe_one<256, false>(maps, halo_rows, shift_rows, k_chunks, base_offset_mode, d_out, err, s);
        default: return cudaErrorInvalidValue;
    }
}

} // namespace azb
