// The heads' 1x1 convolutions over trunk rows, one warp step at a time:
// shared by the head kernel (stem_heads.cu), which streams the trunk
// through shared memory, and the fused small-board tower (tower_fused.cu),
// which holds it there already. Both run the same lane split and the same
// reduction tree, so a point's head sums are the same bits either way.
#pragma once

#include <cuda_bf16.h>

#include "kernels.hpp"

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
    float w[4][kC];
    float bn_scale[kOwn], bn_shift[kOwn];

    __device__ __forceinline__ void load(const HeadArgs& a, int lane) {
        const int l = lane % kLpr;
#pragma unroll
        for (int j = 0; j < kNch; ++j)
#pragma unroll
            for (int e = 0; e < W; ++e) {
                const int ch = (l + j * kLpr) * W + e, i = j * W + e;
                const bool real = ch < a.F;
                w[0][i] = real ? __ldg(a.pol_w + ch) : 0.0f;
                w[1][i] = real ? __ldg(a.pol_w + a.F + ch) : 0.0f;
                w[2][i] = real ? __ldg(a.val_w + ch) : 0.0f;
                w[3][i] = real && a.ownership ? __ldg(a.own_w + ch) : 0.0f;
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
            float z[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (row < rows) {
#pragma unroll
                for (int j = 0; j < kNch; ++j) {
                    const TrunkPiece<kMode> pc = piece(row, l + j * kLpr);
                    float f[W];
                    pc.values(f);
#pragma unroll
                    for (int e = 0; e < W; ++e)
#pragma unroll
                        for (int h = 0; h < 4; ++h) z[h] = fmaf(w[h][j * W + e], f[e], z[h]);
                }
            }
#pragma unroll
            for (int h = 0; h < 4; ++h) acc[s * 4 + h] = z[h];
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

} // namespace azb
