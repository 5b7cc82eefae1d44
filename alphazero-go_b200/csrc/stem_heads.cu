// The stem convolution, the fused heads, and the small kernels the runner's
// checks and test hooks use.
#include <algorithm>

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

// One thread: one pixel, 8 consecutive output channels. Threads of a warp
// share the channel group (weight loads are warp-uniform) and walk
// consecutive pixels of the same plane (input loads coalesce). The sum over
// k = ci*9 + ky*3 + kx runs in the reference's order; in the tf32 modes each
// product and sum is rounded on its own as the naive backend does
// (src/backend.cpp:115-140), so the stem matches it bit for bit.
template <int kMode>
__global__ void __launch_bounds__(256) stem_kernel(const StemArgs a) {
    const int A = a.n * a.n;
    const size_t pixels = size_t(a.B) * A;
    const int groups = a.F / 8;
    const size_t total = pixels * groups;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const int g = static_cast<int>(i / pixels);
        const size_t pix = i % pixels;
        const int b = static_cast<int>(pix / A), p = static_cast<int>(pix % A);
        const int y = p / a.n, x = p % a.n;
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
        const float* in = a.in + size_t(b) * a.P * A;
        const float* w = a.w + size_t(g) * 8 * a.P * 9;
        for (int ci = 0; ci < a.P; ++ci) {
            for (int t = 0; t < 9; ++t) {
                const int sy = y + t / 3 - 1, sx = x + t % 3 - 1;
                const float v = (sy < 0 || sy >= a.n || sx < 0 || sx >= a.n) ? 0.0f : __ldg(in + size_t(ci) * A + sy * a.n + sx);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float wv = __ldg(w + size_t(j) * a.P * 9 + ci * 9 + t);
                    if (kMode == kBF16) acc[j] = fmaf(wv, v, acc[j]);
                    else acc[j] = __fadd_rn(acc[j], __fmul_rn(wv, v));
                }
            }
        }
        const size_t row = size_t(b) * a.S + size_t(y + 1) * (a.n + 1) + x;
        const int c0 = g * 8;
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float yv = __fadd_rn(__fmul_rn(__ldg(a.scale + c0 + j), acc[j]), __ldg(a.shift + c0 + j));
            o[j] = yv > 0.0f ? yv : 0.0f;
        }
        if (kMode == kBF16) {
            uint4 w4;
            __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&w4);
#pragma unroll
            for (int e = 0; e < 4; ++e) h2[e] = __floats2bfloat162_rn(o[2 * e], o[2 * e + 1]);
            *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + row * a.ld + c0) = w4;
        } else if (kMode == kTF32x3) {
            float4* hi = reinterpret_cast<float4*>(static_cast<float*>(a.out) + row * a.ld + c0);
            float4* lo = reinterpret_cast<float4*>(static_cast<float*>(a.out_lo) + row * a.ld + c0);
            float h[8], l[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                h[j] = to_tf32(o[j]);
                l[j] = __fsub_rn(o[j], h[j]);
            }
            hi[0] = make_float4(h[0], h[1], h[2], h[3]);
            hi[1] = make_float4(h[4], h[5], h[6], h[7]);
            lo[0] = make_float4(l[0], l[1], l[2], l[3]);
            lo[1] = make_float4(l[4], l[5], l[6], l[7]);
        } else {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + row * a.ld + c0);
            dst[0] = make_float4(o[0], o[1], o[2], o[3]);
            dst[1] = make_float4(o[4], o[5], o[6], o[7]);
        }
    }
}

// --------------------------------------------------------------- the heads

constexpr int kHeadSamples = 4;    // samples per CTA: the FC weights are read once per group
constexpr int kHeadThreads = 256;
constexpr int kHeadWarps = kHeadThreads / 32;

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

// 8 (bf16) or 4 (fp32) channels of a trunk row as floats; split mode sums hi + lo.
template <int kMode>
struct TrunkVec {
    static constexpr int kWidth = kMode == kBF16 ? 8 : 4;
    __device__ static void load(const HeadArgs& a, size_t off, float* f) {
        if (kMode == kBF16) {
            const uint4 w4 = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.trunk) + off));
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w4);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 t = __bfloat1622float2(h2[e]);
                f[2 * e] = t.x;
                f[2 * e + 1] = t.y;
            }
        } else {
            float4 v = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(a.trunk) + off));
            if (kMode == kTF32x3) {
                const float4 l = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(a.trunk_lo) + off));
                v.x = __fadd_rn(v.x, l.x);
                v.y = __fadd_rn(v.y, l.y);
                v.z = __fadd_rn(v.z, l.z);
                v.w = __fadd_rn(v.w, l.w);
            }
            f[0] = v.x;
            f[1] = v.y;
            f[2] = v.z;
            f[3] = v.w;
        }
    }
};

__device__ __forceinline__ float bn_relu(float z, float scale, float shift) {
    const float y = __fadd_rn(__fmul_rn(scale, z), shift);
    return y > 0.0f ? y : 0.0f;
}

// One CTA: kHeadSamples samples. Phase 1 reads each sample's trunk once
// (a warp per pixel, 16-byte loads across the channels) and produces the
// head convolutions' outputs after batch norm: the policy features in the
// reference's flatten order c*A + p (src/network.cpp:278-285), the value
// features, and the ownership map. Phase 2 runs the FC layers from shared
// memory with each weight row read once per group (a warp per output row,
// coalesced), then tanh for the value and the softmax over A+1 moves.
template <int kMode>
__global__ void __launch_bounds__(kHeadThreads) heads_kernel(const HeadArgs a) {
    extern __shared__ float hs[];
    const int A = a.A, V = a.V, L = A + 1;
    float* pol = hs;                               // [G][2A]
    float* val = pol + kHeadSamples * 2 * A;       // [G][A]
    float* hid = val + kHeadSamples * A;           // [G][V]
    float* lg = hid + kHeadSamples * V;            // [G][A+1]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b0 = blockIdx.x * kHeadSamples;
    const int G = min(kHeadSamples, a.B - b0);
    constexpr int W = TrunkVec<kMode>::kWidth;

    const float ps0 = a.pol_scale[0], ps1 = a.pol_scale[1], ph0 = a.pol_shift[0], ph1 = a.pol_shift[1];
    const float vs = a.val_scale[0], vh = a.val_shift[0];
    const float os = a.ownership ? a.own_scale[0] : 0.0f, oh = a.ownership ? a.own_shift[0] : 0.0f;

    for (int item = warp; item < G * A; item += kHeadWarps) {
        const int g = item / A, p = item % A;
        const int b = b0 + g;
        const size_t row = size_t(b) * a.S + size_t(p / a.n + 1) * (a.n + 1) + p % a.n;
        float z0 = 0.0f, z1 = 0.0f, zv = 0.0f, zo = 0.0f;
        for (int c = lane * W; c < a.F; c += 32 * W) {
            float f[W];
            TrunkVec<kMode>::load(a, row * a.ld + c, f);
#pragma unroll
            for (int e = 0; e < W; ++e) {
                z0 = fmaf(__ldg(a.pol_w + c + e), f[e], z0);
                z1 = fmaf(__ldg(a.pol_w + a.F + c + e), f[e], z1);
                zv = fmaf(__ldg(a.val_w + c + e), f[e], zv);
                if (a.ownership) zo = fmaf(__ldg(a.own_w + c + e), f[e], zo);
            }
        }
        z0 = warp_sum(z0);
        z1 = warp_sum(z1);
        zv = warp_sum(zv);
        if (a.ownership) zo = warp_sum(zo);
        if (lane == 0) {
            pol[g * 2 * A + p] = bn_relu(z0, ps0, ph0);
            pol[g * 2 * A + A + p] = bn_relu(z1, ps1, ph1);
            val[g * A + p] = bn_relu(zv, vs, vh);
            if (a.ownership && a.ownership_out)
                a.ownership_out[size_t(b) * A + p] = tanhf(__fadd_rn(__fmul_rn(os, zo), oh));
        }
    }
    __syncthreads();

    // policy FC: logits[g][o] = sum_i pol[g][i] * fc_w[o][i] + fc_b[o]
    for (int o = warp; o < L; o += kHeadWarps) {
        float acc[kHeadSamples] = {0.0f, 0.0f, 0.0f, 0.0f};
        const float* wr = a.fc_w + size_t(o) * 2 * A;
        for (int i = lane; i < 2 * A; i += 32) {
            const float wv = __ldg(wr + i);
#pragma unroll
            for (int g = 0; g < kHeadSamples; ++g)
                if (g < G) acc[g] = fmaf(wv, pol[g * 2 * A + i], acc[g]);
        }
#pragma unroll
        for (int g = 0; g < kHeadSamples; ++g) acc[g] = warp_sum(acc[g]);
        if (lane == 0) {
            const float bias = __ldg(a.fc_b + o);
            for (int g = 0; g < G; ++g) {
                const float l = __fadd_rn(acc[g], bias);
                lg[g * L + o] = l;
                a.logits[size_t(b0 + g) * L + o] = l;
            }
        }
    }
    // value FC1 + ReLU
    for (int v = warp; v < V; v += kHeadWarps) {
        float acc[kHeadSamples] = {0.0f, 0.0f, 0.0f, 0.0f};
        const float* wr = a.v1_w + size_t(v) * A;
        for (int i = lane; i < A; i += 32) {
            const float wv = __ldg(wr + i);
#pragma unroll
            for (int g = 0; g < kHeadSamples; ++g)
                if (g < G) acc[g] = fmaf(wv, val[g * A + i], acc[g]);
        }
#pragma unroll
        for (int g = 0; g < kHeadSamples; ++g) acc[g] = warp_sum(acc[g]);
        if (lane == 0) {
            const float bias = __ldg(a.v1_b + v);
            for (int g = 0; g < G; ++g) {
                const float h = __fadd_rn(acc[g], bias);
                hid[g * V + v] = h > 0.0f ? h : 0.0f;
            }
        }
    }
    __syncthreads();
    // value FC2 + tanh, and the softmax over the A+1 logits: one warp per sample.
    for (int g = warp; g < G; g += kHeadWarps) {
        float acc = 0.0f;
        for (int i = lane; i < V; i += 32) acc = fmaf(__ldg(a.v2_w + i), hid[g * V + i], acc);
        acc = warp_sum(acc);
        if (lane == 0) a.values[b0 + g] = tanhf(__fadd_rn(acc, __ldg(a.v2_b)));
        if (a.probs) {
            float m = -INFINITY;
            for (int o = lane; o < L; o += 32) m = fmaxf(m, lg[g * L + o]);
            m = warp_max(m);
            float s = 0.0f;
            for (int o = lane; o < L; o += 32) s += expf(lg[g * L + o] - m);
            s = warp_sum(s);
            const float inv = 1.0f / s;
            for (int o = lane; o < L; o += 32) a.probs[size_t(b0 + g) * L + o] = expf(lg[g * L + o] - m) * inv;
        }
    }
}

// ------------------------------------------------------------ small kernels

__global__ void fill_kernel(float* data, size_t n, float value) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
        data[i] = value;
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

cudaError_t launch_stem(const StemArgs& a, int precision, cudaStream_t s) {
    if (a.F % 8 != 0) return cudaErrorInvalidValue;
    const size_t total = size_t(a.B) * a.n * a.n * (a.F / 8);
    if (total == 0) return cudaSuccess;
    const unsigned grid = blocks_for(total, 256);
    switch (precision) {
        case kTF32: stem_kernel<kTF32><<<grid, 256, 0, s>>>(a); break;
        case kTF32x3: stem_kernel<kTF32x3><<<grid, 256, 0, s>>>(a); break;
        case kBF16: stem_kernel<kBF16><<<grid, 256, 0, s>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_heads(const HeadArgs& a, int precision, cudaStream_t s) {
    if (a.B <= 0) return cudaSuccess;
    const int W = precision == kBF16 ? 8 : 4;
    if (a.F % W != 0) return cudaErrorInvalidValue;
    const size_t smem = size_t(kHeadSamples) * (2 * a.A + a.A + a.V + a.A + 1) * sizeof(float);
    const unsigned grid = static_cast<unsigned>((a.B + kHeadSamples - 1) / kHeadSamples);
    switch (precision) {
        case kTF32: heads_kernel<kTF32><<<grid, kHeadThreads, smem, s>>>(a); break;
        case kTF32x3: heads_kernel<kTF32x3><<<grid, kHeadThreads, smem, s>>>(a); break;
        case kBF16: heads_kernel<kBF16><<<grid, kHeadThreads, smem, s>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_fill(float* data, size_t n, float value, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    fill_kernel<<<blocks_for(n, 256), 256, 0, s>>>(data, n, value);
    return cudaGetLastError();
}

cudaError_t fill_attributes(cudaFuncAttributes* attr) { return cudaFuncGetAttributes(attr, fill_kernel); }

cudaError_t launch_spin(unsigned long long ns, cudaStream_t s) {
    if (ns == 0) return cudaSuccess;
    spin_kernel<<<1, 1, 0, s>>>(ns);
    return cudaGetLastError();
}

cudaError_t launch_bounded_wait_probe(int* err, unsigned long long limit_ns, cudaStream_t s) {
    bounded_wait_probe<<<1, 32, 0, s>>>(err, limit_ns);
    return cudaGetLastError();
}

} // namespace azb
