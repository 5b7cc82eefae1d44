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

// The stem's input as a packed GEMM operand: for every board point, the
// 9*P values its 3x3 window reads (tap-major: column t*P + p, t = ky*3 + kx,
// 0 off the board), in the point's frame row. The stem then runs on the
// tensor cores as a one-tap GEMM with K = 9*P (rounded up to whole 128-byte
// chunks), instead of a 3x3 convolution over P channels padded to a chunk.
// Frame padding rows and the columns past 9*P are never written (zero since
// the buffer was allocated).
template <int kMode>
__global__ void __launch_bounds__(256) stem_im2col_kernel(const StemArgs a) {
    const int A = a.n * a.n, K = 9 * a.P;
    const size_t total = size_t(a.B) * A * K;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const size_t pix = i / K;
        const int k = static_cast<int>(i % K);
        const int b = static_cast<int>(pix / A), pt = static_cast<int>(pix % A);
        const int t = k / a.P, pl = k % a.P;
        const int y = pt / a.n + t / 3 - 1, x = pt % a.n + t % 3 - 1;
        const float v = (y < 0 || y >= a.n || x < 0 || x >= a.n)
                            ? 0.0f
                            : __ldg(a.in + (size_t(b) * a.P + pl) * A + y * a.n + x);
        const size_t row = size_t(b) * a.S + size_t(pt / a.n + 1) * (a.n + 1) + pt % a.n;
        const size_t off = row * a.ld + k;
        if (kMode == kBF16) {
            static_cast<__nv_bfloat16*>(a.out)[off] = __float2bfloat16_rn(v);
        } else if (kMode == kTF32x3) {
            const float h = to_tf32(v);
            static_cast<float*>(a.out)[off] = h;
            static_cast<float*>(a.out_lo)[off] = __fsub_rn(v, h);
        } else {
            static_cast<float*>(a.out)[off] = v;
        }
    }
}

// --------------------------------------------------------------- the heads

constexpr int kHeadSamples = 8;    // samples per CTA: each FC weight is read once per group
constexpr int kHeadThreads = 512;
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

size_t head_smem_bytes(int F, int A, int V) {
    return (size_t(4) * F + size_t(kHeadSamples) * (2 * A + A + V + A + 1)) * sizeof(float);
}

// One CTA: kHeadSamples samples.
//  1. Each thread takes whole board points: it reads the point's F trunk
//     channels with 16-byte loads (independent, so many are in flight) and
//     sums the policy, value and ownership 1x1 convolutions in channel
//     order, then applies their batch norms: the policy features land in the
//     reference's flatten order c*A + p (src/network.cpp:278-285).
//  2. Each thread owns one FC output (a policy logit or a value hidden unit)
//     for all the group's samples, summing over the inputs in order; the FC
//     weights are stored input-major, so a warp's loads of one input's
//     weights are one coalesced line.
//  3. One warp per sample: the value FC2 and tanh, and the softmax over
//     the A+1 logits.
// Every output is one thread's fixed-order sum over its own sample's data:
// the results do not depend on the batch or on where a sample sits in it.
template <int kMode>
__global__ void __launch_bounds__(kHeadThreads) heads_kernel(const HeadArgs a) {
    extern __shared__ float hs[];
    const int A = a.A, V = a.V, L = A + 1, F = a.F;
    float* wpol0 = hs;
    float* wpol1 = wpol0 + F;
    float* wval = wpol1 + F;
    float* wown = wval + F;
    float* pol = wown + F;                         // [G][2A]
    float* val = pol + kHeadSamples * 2 * A;       // [G][A]
    float* hid = val + kHeadSamples * A;           // [G][V]
    float* lg = hid + kHeadSamples * V;            // [G][A+1]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b0 = blockIdx.x * kHeadSamples;
    const int G = min(kHeadSamples, a.B - b0);
    constexpr int W = TrunkVec<kMode>::kWidth;

    for (int i = threadIdx.x; i < F; i += kHeadThreads) {
        wpol0[i] = a.pol_w[i];
        wpol1[i] = a.pol_w[F + i];
        wval[i] = a.val_w[i];
        wown[i] = a.ownership ? a.own_w[i] : 0.0f;
    }
    __syncthreads();
    const float ps0 = a.pol_scale[0], ps1 = a.pol_scale[1], ph0 = a.pol_shift[0], ph1 = a.pol_shift[1];
    const float vs = a.val_scale[0], vh = a.val_shift[0];
    const float os = a.ownership ? a.own_scale[0] : 0.0f, oh = a.ownership ? a.own_shift[0] : 0.0f;

    for (int item = threadIdx.x; item < G * A; item += kHeadThreads) {
        const int g = item / A, p = item % A;
        const size_t row = size_t(b0 + g) * a.S + size_t(p / a.n + 1) * (a.n + 1) + p % a.n;
        float z0 = 0.0f, z1 = 0.0f, zv = 0.0f, zo = 0.0f;
#pragma unroll 4
        for (int c = 0; c < F; c += W) {
            float f[W];
            TrunkVec<kMode>::load(a, row * a.ld + c, f);
#pragma unroll
            for (int e = 0; e < W; ++e) {
                z0 = fmaf(wpol0[c + e], f[e], z0);
                z1 = fmaf(wpol1[c + e], f[e], z1);
                zv = fmaf(wval[c + e], f[e], zv);
                zo = fmaf(wown[c + e], f[e], zo);
            }
        }
        pol[g * 2 * A + p] = bn_relu(z0, ps0, ph0);
        pol[g * 2 * A + A + p] = bn_relu(z1, ps1, ph1);
        val[g * A + p] = bn_relu(zv, vs, vh);
        if (a.ownership && a.ownership_out)
            a.ownership_out[size_t(b0 + g) * A + p] = tanhf(__fadd_rn(__fmul_rn(os, zo), oh));
    }
    __syncthreads();

    for (int o = threadIdx.x; o < L + V; o += kHeadThreads) {
        float acc[kHeadSamples];
#pragma unroll
        for (int g = 0; g < kHeadSamples; ++g) acc[g] = 0.0f;
        const bool policy = o < L;
        const int n_in = policy ? 2 * A : A, out = policy ? o : o - L, stride = policy ? L : V;
        const float* wt = policy ? a.fc_wt : a.v1_wt;      // [n_in][stride]
        const float* x = policy ? pol : val;
        const int ld = policy ? 2 * A : A;
#pragma unroll 4
        for (int i = 0; i < n_in; ++i) {
            const float wv = __ldg(wt + size_t(i) * stride + out);
#pragma unroll
            for (int g = 0; g < kHeadSamples; ++g) acc[g] = fmaf(wv, x[g * ld + i], acc[g]);
        }
        if (policy) {
            const float bias = __ldg(a.fc_b + out);
            for (int g = 0; g < G; ++g) {
                const float l = __fadd_rn(acc[g], bias);
                lg[g * L + out] = l;
                a.logits[size_t(b0 + g) * L + out] = l;
            }
        } else {
            const float bias = __ldg(a.v1_b + out);
            for (int g = 0; g < G; ++g) {
                const float h = __fadd_rn(acc[g], bias);
                hid[g * V + out] = h > 0.0f ? h : 0.0f;
            }
        }
    }
    __syncthreads();

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

cudaError_t launch_stem_im2col(const StemArgs& a, int precision, cudaStream_t s) {
    const size_t total = size_t(a.B) * a.n * a.n * 9 * a.P;
    if (total == 0) return cudaSuccess;
    const unsigned grid = blocks_for(total, 256);
    switch (precision) {
        case kTF32: stem_im2col_kernel<kTF32><<<grid, 256, 0, s>>>(a); break;
        case kTF32x3: stem_im2col_kernel<kTF32x3><<<grid, 256, 0, s>>>(a); break;
        case kBF16: stem_im2col_kernel<kBF16><<<grid, 256, 0, s>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_heads(const HeadArgs& a, int precision, cudaStream_t s) {
    if (a.B <= 0) return cudaSuccess;
    const int W = precision == kBF16 ? 8 : 4;
    if (a.F % W != 0) return cudaErrorInvalidValue;
    const size_t smem = head_smem_bytes(a.F, a.A, a.V);
    const unsigned grid = static_cast<unsigned>((a.B + kHeadSamples - 1) / kHeadSamples);
    cudaError_t e = cudaSuccess;
    switch (precision) {
        case kTF32:
            e = cudaFuncSetAttribute(heads_kernel<kTF32>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
            if (e == cudaSuccess) heads_kernel<kTF32><<<grid, kHeadThreads, smem, s>>>(a);
            break;
        case kTF32x3:
            e = cudaFuncSetAttribute(heads_kernel<kTF32x3>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
            if (e == cudaSuccess) heads_kernel<kTF32x3><<<grid, kHeadThreads, smem, s>>>(a);
            break;
        case kBF16:
            e = cudaFuncSetAttribute(heads_kernel<kBF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
            if (e == cudaSuccess) heads_kernel<kBF16><<<grid, kHeadThreads, smem, s>>>(a);
            break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
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
