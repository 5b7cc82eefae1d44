// The heads' 1x1 convolutions over trunk rows, one warp step at a time:
// shared by the head kernel (stem_heads.cu), which streams the trunk
// through shared memory, and the fused small-board tower (tower_fused.cu),
// which holds it there already. Both run the same lane split and the same
// reduction tree, so a point's head sums are the same bits either way.
#pragma once

#include <cuda_bf16.h>

#include "kernels.hpp"
#include "sm100.cuh"

namespace azb {

// One 16-byte piece of a trunk row (and, split mode, of its low plane) as
// floats: 8 bf16 or 4 fp32 channels; split mode adds hi + lo (one rounding).
template <int kMode>
struct TrunkPiece {
    static constexpr int kWidth = kMode == kBF16 ? 8 : 4;
    uint4 hi, lo;
    __device__ __forceinline__ void values(float* f) const {
        if (kMode == kBF16) {
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&hi);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 t = __bfloat1622float2(h2[e]);
                f[2 * e] = t.x;
                f[2 * e + 1] = t.y;
            }
        } else {
            const float* h = reinterpret_cast<const float*>(&hi);
            const float* l = reinterpret_cast<const float*>(&lo);
#pragma unroll
            for (int e = 0; e < 4; ++e) f[e] = kMode == kTF32x3 ? __fadd_rn(h[e], l[e]) : h[e];
        }
    }
};

// v / n for v >= 0 and n <= 19: below 2^20 with a float reciprocal ((v +
// 0.5)/n stays at least 0.5/n away from the integers, above the float
// error there), else by integer division.
__device__ __forceinline__ int div_small(int v, int n, float inv_n) {
    return v < (1 << 20) ? int((float(v) + 0.5f) * inv_n) : v / n;
}
constexpr int kHcSlots = 4;

// One lane's part of the head convolutions: kLpr lanes share one trunk row
// (kLpr x kNch 16-byte pieces, lane l reading pieces l, l + kLpr, ...),
// each lane summing its channels into 4 slots x 4 heads = 16 partial sums
// with the 1x1 weights of its channels in registers; a reduce-scatter over
// the kLpr lanes (at the step over lane bit b a lane keeps the half of its
// sums that bit selects and adds its partner's copy; once one sum is left, a
// butterfly) leaves each lane its finished sums, which it applies the batch
// norm to and stores: policy and value features (ReLU) into feat, ownership
// (tanh) into ownership_out. Every sum is the same tree of additions whatever
// its slot: outputs do not depend on the batch.
template <int kMode, int kLpr, int kNch>
struct HeadLane {
    static constexpr int W = TrunkPiece<kMode>::kWidth, kC = kNch * W;
    static constexpr int kGroups = 32 / kLpr;                  // rows a warp holds per slot
    static constexpr int kStepRows = kHcSlots * kGroups;       // rows per warp step
    static constexpr int kLog = kLpr == 32 ? 5 : kLpr == 16 ? 4 : 3;
    static constexpr int kScatter = kLog < 4 ? kLog : 4;       // steps that halve the 16 sums
    static constexpr int kBfly = kLog - kScatter;              // butterfly steps after them
    static constexpr int kOwn = (kHcSlots * 4) >> kScatter;    // finished sums per lane
    // The 1x1 weights of this lane's channels, heads paired for the packed
    // fma (each half an IEEE fmaf: the same bits as one head at a time):
    // (policy 0, policy 1), (value, ownership).
    float2 w01[kC], w23[kC];
    float bn_scale[kOwn], bn_shift[kOwn];

    __device__ __forceinline__ void load(const HeadArgs& a, int lane) {
        const int l = lane % kLpr;
#pragma unroll
        for (int j = 0; j < kNch; ++j)
#pragma unroll
            for (int e = 0; e < W; ++e) {
                const int ch = (l + j * kLpr) * W + e, i = j * W + e;
                const bool real = ch < a.F;
                w01[i] = make_float2(real ? __ldg(a.pol_w + ch) : 0.0f, real ? __ldg(a.pol_w + a.F + ch) : 0.0f);
                w23[i] = make_float2(real ? __ldg(a.val_w + ch) : 0.0f, real && a.ownership ? __ldg(a.own_w + ch) : 0.0f);
            }
        // The batch norm of the sums this lane finishes (head k % 4 of its
        // sums k = (l >> kBfly) * kOwn + j), the same for every step.
#pragma unroll
        for (int j = 0; j < kOwn; ++j) {
            const int h = (((l >> kBfly) * kOwn) + j) % 4;
            bn_scale[j] = h == 0 ? __ldg(a.pol_scale) : h == 1 ? __ldg(a.pol_scale + 1) : h == 2 ? __ldg(a.val_scale)
                                                                                       : (a.ownership ? __ldg(a.own_scale) : 0.0f);
            bn_shift[j] = h == 0 ? __ldg(a.pol_shift) : h == 1 ? __ldg(a.pol_shift + 1) : h == 2 ? __ldg(a.val_shift)
                                                                                       : (a.ownership ? __ldg(a.own_shift) : 0.0f);
        }
    }

    // Rows [base, base + kStepRows) of `rows`: piece(row, j) gives a row's
    // 16-byte piece j, where(row, &b, &p) its board and point.
    template <class Piece, class Where>
    __device__ __forceinline__ void step(const HeadArgs& a, int base, int rows, Piece piece, Where where, int lane) const {
        const int l = lane % kLpr, grp = lane / kLpr;
        float acc[kHcSlots * 4];
#pragma unroll
        for (int s = 0; s < kHcSlots; ++s) {
            const int row = base + s * kGroups + grp;
            float2 z01 = make_float2(0.0f, 0.0f), z23 = z01;
            if (row < rows) {
#pragma unroll
                for (int j = 0; j < kNch; ++j) {
                    const TrunkPiece<kMode> pc = piece(row, l + j * kLpr);
                    float f[W];
                    pc.values(f);
#pragma unroll
                    for (int e = 0; e < W; ++e) {
                        const float2 ff = make_float2(f[e], f[e]);
                        z01 = ffma2_rn(w01[j * W + e], ff, z01);
                        z23 = ffma2_rn(w23[j * W + e], ff, z23);
                    }
                }
            }
            acc[s * 4] = z01.x;
            acc[s * 4 + 1] = z01.y;
            acc[s * 4 + 2] = z23.x;
            acc[s * 4 + 3] = z23.y;
        }
        // Reduce-scatter over the high lane bits of the group while there
        // is more than one sum to split, then a butterfly over the rest.
#pragma unroll
        for (int t = 0; t < kLog; ++t) {
            const int off = kLpr >> (t + 1);
            if (t < kScatter) {
                const int half = (kHcSlots * 2) >> t;
                const bool upper = (lane & off) != 0;
#pragma unroll
                for (int k = 0; k < half; ++k) {
                    const float send = upper ? acc[k] : acc[k + half];
                    const float keep = upper ? acc[k + half] : acc[k];
                    acc[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                }
            } else {
                acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], off);
            }
        }
        const bool writer = (l & ((1 << kBfly) - 1)) == 0;
        if (writer) {
            const int A = a.A;
#pragma unroll
            for (int j = 0; j < kOwn; ++j) {
                const int k = (l >> kBfly) * kOwn + j, s = k / 4, h = k % 4;
                const int row = base + s * kGroups + grp;
                if (row >= rows) continue;
                int b, p;
                where(row, &b, &p);
                const float y = __fadd_rn(__fmul_rn(bn_scale[j], acc[j]), bn_shift[j]);
                if (h < 3) {
                    a.feat[size_t(b) * a.feat_ld + (h == 2 ? a.feat_val : h * A) + p] = y > 0.0f ? y : 0.0f;
                } else if (a.ownership && a.ownership_out) {
                    a.ownership_out[size_t(b) * A + p] = tanhf(y);
                }
            }
        }
    }
};

// ------------------------------------------------------------ head FCs
//
// The policy FC (2A -> A+1, + bias) and the value FC1 (A -> V, + bias,
// ReLU) as warp-level dot products, shared by the head tail kernel
// (stem_heads.cu) and the fused small-board tower (tower_fused.cu). One warp
// computes kOuts consecutive outputs [o0, o0 + kOuts) for G <= kBoards
// boards: lane l sums the 16-byte input pieces j = l, l + 32, ... of every
// (output, board) with fmaf over a piece's four values in order (weights
// and inputs zero-padded to whole pieces); the 32 lane partials of every sum
// are then added in one fixed tree, pairs over lane bit 4 first, then bits
// 3, 2, 1, 0: by halving reduce-scatter steps while a lane holds more than
// one sum (at the step over bit b a lane keeps the half of its sums that bit
// selects and adds its partner's copy), by butterfly steps after. The tree
// does not depend on the sum's (output, board) index nor on kOuts x
// kBoards, so a board's outputs are the same bits in any tile, slot or kernel.

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int kOuts, int kBoards>
struct FcWarp {
    static constexpr int kSums = kOuts * kBoards;
    static_assert((kSums & (kSums - 1)) == 0 && kSums >= 2 && kSums <= 1024, "a power of two of sums");
    static constexpr int kLogSums = kSums >= 512 ? 9 : kSums >= 256 ? 8 : kSums >= 128 ? 7 : kSums >= 64 ? 6
                                  : kSums >= 32 ? 5 : kSums >= 16 ? 4 : kSums >= 8 ? 3 : kSums >= 4 ? 2 : 1;
    static constexpr int kHeld = kSums >= 32 ? kSums / 32 : 1;   // sums a lane holds at the end

    // acc[k], k = o * kBoards + g: the dot of output o0 + o's weight row
    // with board g's inputs, x(g, j) the board's input piece j. kTwo: a lane
    // loads its pieces j and j + 32 together (one round trip for both where
    // the inputs are short), adding them in the same order.
    template <bool kTwo = false, class X>
    __device__ __forceinline__ static void dot(const float4* W, int n4, int ncols, int o0, int G, X x,
                                               float (&acc)[kSums], int lane) {
#pragma unroll
        for (int k = 0; k < kSums; ++k) acc[k] = 0.0f;
        constexpr int kPieces = kTwo ? 2 : 1;
        for (int j = lane; j < n4; j += 32 * kPieces) {
            const bool two = kTwo && j + 32 < n4;
            float4 w[kPieces][kOuts];
#pragma unroll
            for (int u = 0; u < kPieces; ++u)
#pragma unroll
                for (int o = 0; o < kOuts; ++o)
                    w[u][o] = o0 + o < ncols && (u == 0 || two) ? __ldg(W + size_t(o0 + o) * n4 + j + 32 * u)
                                                                : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int g = 0; g < kBoards; ++g) {
                if (g >= G) break;
                float4 v[kPieces];
#pragma unroll
                for (int u = 0; u < kPieces; ++u) v[u] = u == 0 || two ? x(g, j + 32 * u) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
                for (int u = 0; u < kPieces; ++u) {
                    if (u > 0 && !two) break;
#pragma unroll
                    for (int o = 0; o < kOuts; ++o) {
                        float& c = acc[o * kBoards + g];
                        c = fmaf(w[u][o].x, v[u].x, c);
                        c = fmaf(w[u][o].y, v[u].y, c);
                        c = fmaf(w[u][o].z, v[u].z, c);
                        c = fmaf(w[u][o].w, v[u].w, c);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < 5; ++t) {
            const int off = 16 >> t;
            if (t < kLogSums) {
                const int half = kSums >> (t + 1);
                const bool upper = (lane & off) != 0;
#pragma unroll
                for (int k = 0; k < half; ++k) {
                    const float send = upper ? acc[k] : acc[k + half];
                    const float keep = upper ? acc[k + half] : acc[k];
                    acc[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                }
            } else {
                acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], off);
            }
        }
    }

    // The index k of the lane's h-th finished sum, or -1 where another lane
    // of a butterfly group reports it.
    __device__ __forceinline__ static int held(int lane, int h) {
        if constexpr (kSums >= 32) {
            return lane * kHeld + h;
        } else {
            const int shift = 5 - kLogSums;
            return (lane & ((1 << shift) - 1)) == 0 ? lane >> shift : -1;
        }
    }
};

// Quads of the FC outputs (kOuts at a time): the policy outputs [0, A+1)
// first, then the value FC1 outputs [0, V).
template <int kOuts>
__device__ __forceinline__ int head_fc_quad_count(const HeadArgs& a) {
    return (a.A + 1 + kOuts - 1) / kOuts + (a.V + kOuts - 1) / kOuts;
}

// One quad q of the FC outputs for the G boards from b0, whose inputs
// x(g, j) are the feature rows: the policy features for policy outputs
// (pieces of 2A values), the value features for value outputs (A values).
// Writes logits and the ReLU of the hidden layer (hid_at(g) gives a board's
// hidden row).
template <int kOuts, int kBoards, bool kTwo = false, class XPol, class XVal, class HidAt>
__device__ __forceinline__ void head_fc_quad(const HeadArgs& a, int b0, int G, int q, XPol xpol, XVal xval,
                                             HidAt hid_at, int lane) {
    using Fc = FcWarp<kOuts, kBoards>;
    const int L = a.A + 1, V = a.V;
    const int pol_quads = (L + kOuts - 1) / kOuts;
    const int n4p = (2 * a.A + 3) / 4, n4v = (a.A + 3) / 4;
    const bool policy = q < pol_quads;
    const int o0 = (policy ? q : q - pol_quads) * kOuts;
    float acc[Fc::kSums];
    if (policy)
        Fc::template dot<kTwo>(reinterpret_cast<const float4*>(a.fc_w), n4p, L, o0, G, xpol, acc, lane);
    else
        Fc::template dot<kTwo>(reinterpret_cast<const float4*>(a.v1_w), n4v, V, o0, G, xval, acc, lane);
#pragma unroll
    for (int h = 0; h < Fc::kHeld; ++h) {
        const int k = Fc::held(lane, h);
        if (k < 0) continue;
        const int o = o0 + k / kBoards, g = k % kBoards;
        if (g >= G || o >= (policy ? L : V)) continue;
        if (policy) {
            a.logits[size_t(b0 + g) * L + o] = __fadd_rn(acc[h], __ldg(a.fc_b + o));
        } else {
            const float y = __fadd_rn(acc[h], __ldg(a.v1_b + o));
            hid_at(g)[o] = y > 0.0f ? y : 0.0f;
        }
    }
}

// One tile's FC outputs: this warp's share of the quads (quad0, quad0 +
// quad_step, ...).
template <int kOuts, int kBoards, class XPol, class XVal, class HidAt>
__device__ __forceinline__ void head_fc_quads(const HeadArgs& a, int b0, int G, int quad0, int quad_step, XPol xpol,
                                              XVal xval, HidAt hid_at, int lane) {
    const int quads = head_fc_quad_count<kOuts>(a);
    for (int q = quad0; q < quads; q += quad_step) head_fc_quad<kOuts, kBoards>(a, b0, G, q, xpol, xval, hid_at, lane);
}

// One warp finishes board b: value = tanh(v2 . hid + b2) and, when asked
// for, the softmax over the A+1 logits. hid and logits may have been written
// by other CTAs: read through L2.
__device__ __forceinline__ void head_finish_board(const HeadArgs& a, int b, const float* hid, int lane) {
    const int L = a.A + 1, V = a.V;
    float acc = 0.0f;
    for (int i = lane; i < V; i += 32) acc = fmaf(__ldg(a.v2_w + i), __ldcg(hid + i), acc);
    acc = warp_sum(acc);
    if (lane == 0) a.values[b] = tanhf(__fadd_rn(acc, __ldg(a.v2_b)));
    if (a.probs) {
        const float* lg = a.logits + size_t(b) * L;
        float m = -INFINITY;
        for (int o = lane; o < L; o += 32) m = fmaxf(m, __ldcg(lg + o));
        m = warp_max(m);
        float s = 0.0f;
        for (int o = lane; o < L; o += 32) s += expf(__ldcg(lg + o) - m);
        s = warp_sum(s);
        const float inv = 1.0f / s;
        for (int o = lane; o < L; o += 32) a.probs[size_t(b) * L + o] = expf(__ldcg(lg + o) - m) * inv;
    }
}

} // namespace azb
